// attn.cu — gated full-attention core of the verify pass in one kernel: q/k RMSNorm with interleaved mRoPE and the KV
// write (attn_prep, kernels.metal:627-662), split-K causal GQA over the cache (attn_split :713-780) and the log-sum-exp
// merge (attn_combine :783-799), done by the last split CTA of each (row, kv head).
//
// Grid (KV, NSPLIT_ATTN, T), 256 threads (one per head dim). The grid is fixed for graph capture; each CTA derives its
// key range [j0, j1) of [0, off + t] from the device-side KV offset, so one captured graph serves every length. Keys of
// this pass (positions >= off) are prepared by every CTA that needs them, from the projection rows, and written to
// the cache (identical values from every writer); older keys come from the cache.
#include "common.cuh"
#include "kernels.h"

namespace bcu {

constexpr float EPS_A = 1e-6f;

// Score buffer length per query head: the largest key chunk, rounded up to 4 floats so the regions after it in shared
// memory stay 16-byte aligned for the float4 key reads.
__host__ __device__ inline int attn_chunk_max(int ctx) { return (((ctx + NSPLIT_ATTN - 1) / NSPLIT_ATTN) + 3) & ~3; }

__global__ void __launch_bounds__(256) attn_kernel(AttnArgs a) {
    extern __shared__ __align__(16) float sm[];
    __shared__ float buf[256];
    __shared__ int s_last;
    const int kh = blockIdx.x, s = blockIdx.y, t = blockIdx.z;
    const int H = a.H, KV = a.KV, qper = H / KV, aw = H * 256, kvw = KV * 256;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, d = threadIdx.x;
    const int chunk_max = attn_chunk_max(a.ctx);
    float* qs = sm;                            // [qper][256]
    float* sc = qs + qper * 256;               // [qper][chunk_max]
    float* nk = sc + qper * chunk_max;         // [VMAX][256] this pass's keys
    float* nv = nk + VMAX * 256;               // [VMAX][256] this pass's values
    float* ml = nv + VMAX * 256;               // [qper][2]
    const float wq = a.qn[d], wk = a.kn[d];
    pdl_trigger();
    pdl_wait();
    const int off = a.ctl->off;
    const int n = off + t + 1;
    const int chunk = (n + NSPLIT_ATTN - 1) / NSPLIT_ATTN;
    const int j0 = s * chunk, j1 = min(n, j0 + chunk);
    float* pp = a.part + ((size_t)t * H + kh * qper) * NSPLIT_ATTN * 258 + (size_t)s * 258;
    if (n > a.ctx) {
        if (d == 0 && s == 0 && kh == 0) atomicOr(&((Ctl*)a.ctl)->err, ERR_CTX_FULL);
        return;
    }
    if (j0 < j1) {
        // rows to prepare: the qper query heads of row t, then this pass's keys in range (positions >= off);
        // all loaded at once, one block reduction for every row's RMS norm
        const int u0 = max(j0, off) - off, u1 = j1 - off, nkeys = max(u1 - u0, 0);
        const int nrows = qper + nkeys;  // <= 16 + 16
        float x[32], vvals[16];
#pragma unroll
        for (int i = 0; i < 32; i++) {
            x[i] = 0.0f;
            if (i < qper) x[i] = a.qkv[(size_t)t * a.ld + (kh * qper + i) * 512 + d];
            else if (i < nrows) x[i] = a.qkv[(size_t)(u0 + i - qper) * a.ld + 2 * aw + kh * 256 + d];
        }
#pragma unroll
        for (int i = 0; i < 16; i++)
            if (i < nkeys) vvals[i] = a.qkv[(size_t)(u0 + i) * a.ld + 2 * aw + kvw + kh * 256 + d];
        float* rr = buf;  // [8 warps][32 rows]
#pragma unroll
        for (int i = 0; i < 32; i++)
            if (i < nrows) {
                float s2 = warp_sum(x[i] * x[i]);
                if (lane == 0) rr[w * 32 + i] = s2;
            }
        __syncthreads();
        float* xs = nk;  // staging of the normed rows [nrows][256] (nk/nv regions are free until below)
#pragma unroll
        for (int i = 0; i < 32; i++)
            if (i < nrows) {
                float ss = 0.0f;
#pragma unroll
                for (int q = 0; q < 8; q++) ss += rr[q * 32 + i];
                xs[i * 256 + d] = (x[i] * rsqrtf(ss / 256.0f + EPS_A)) * (i < qper ? wq : wk);
            }
        __syncthreads();
        // interleaved mRoPE on the first `rot` dims; text positions: the three position rows are equal
        float y[32];
        const int half = a.rot / 2;
        float invf = d < a.rot ? a.inv_freq[d % half] : 0.0f;
#pragma unroll
        for (int i = 0; i < 32; i++)
            if (i < nrows) {
                float xv = xs[i * 256 + d];
                if (d < a.rot) {
                    int pos = i < qper ? off + t : off + u0 + i - qper;
                    float sn, cs;
                    sincosf((float)pos * invf, &sn, &cs);
                    xv = d < half ? xv * cs - xs[i * 256 + d + half] * sn : xv * cs + xs[i * 256 + d - half] * sn;
                }
                y[i] = xv;
            }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 32; i++) {
            if (i < qper) qs[i * 256 + d] = y[i] * 0.0625f;  // queries scaled by 1/sqrt(256)
            else if (i < nrows) {
                int u = u0 + i - qper;
                nk[u * 256 + d] = y[i];
                a.kc[((size_t)(off + u) * KV + kh) * 256 + d] = y[i];
            }
        }
#pragma unroll
        for (int i = 0; i < 16; i++)
            if (i < nkeys) {
                int u = u0 + i;
                nv[u * 256 + d] = vvals[i];
                a.vc[((size_t)(off + u) * KV + kh) * 256 + d] = vvals[i];
            }
        __syncthreads();
        // scores: warp per key, lanes over dims (8 each); the next key's row is loaded while this one is used
        {
            int j = j0 + w;
            float4 ka = make_float4(0, 0, 0, 0), kb = ka;
            if (j < j1) {
                const float* k = j >= off ? nk + (j - off) * 256 + lane * 8 : a.kc + ((size_t)j * KV + kh) * 256 + lane * 8;
                ka = *(const float4*)k;
                kb = *(const float4*)(k + 4);
            }
            for (; j < j1; j += 8) {
                float4 na = make_float4(0, 0, 0, 0), nb = na;
                int jn = j + 8;
                if (jn < j1) {
                    const float* k = jn >= off ? nk + (jn - off) * 256 + lane * 8 : a.kc + ((size_t)jn * KV + kh) * 256 + lane * 8;
                    na = *(const float4*)k;
                    nb = *(const float4*)(k + 4);
                }
                for (int hq = 0; hq < qper; hq++) {
                    const float* q = qs + hq * 256 + lane * 8;
                    float dd = q[0] * ka.x + q[1] * ka.y + q[2] * ka.z + q[3] * ka.w + q[4] * kb.x + q[5] * kb.y +
                               q[6] * kb.z + q[7] * kb.w;
                    dd = warp_sum(dd);
                    if (lane == 0) sc[hq * chunk_max + (j - j0)] = dd;
                }
                ka = na;
                kb = nb;
            }
        }
        __syncthreads();
        const int cnt = j1 - j0;
        for (int hq = w; hq < qper; hq += 8) {
            float m = -INFINITY;
            for (int i = lane; i < cnt; i += 32) m = fmaxf(m, sc[hq * chunk_max + i]);
            m = warp_max(m);
            float l = 0.0f;
            for (int i = lane; i < cnt; i += 32) {
                float p = expf(sc[hq * chunk_max + i] - m);
                sc[hq * chunk_max + i] = p;
                l += p;
            }
            l = warp_sum(l);
            if (lane == 0) {
                ml[hq * 2] = m;
                ml[hq * 2 + 1] = l;
            }
        }
        __syncthreads();
        // P.V: thread = head dim, keys in order
        float acc[16];
#pragma unroll
        for (int hq = 0; hq < 16; hq++) acc[hq] = 0.0f;
        for (int i0 = 0; i0 < cnt; i0 += 8) {  // 8 value loads in flight, accumulated in key order
            float vv[8];
#pragma unroll
            for (int q = 0; q < 8; q++) {
                int j = j0 + i0 + q;
                vv[q] = i0 + q >= cnt ? 0.0f : (j >= off ? nv[(j - off) * 256 + d] : a.vc[((size_t)j * KV + kh) * 256 + d]);
            }
#pragma unroll
            for (int q = 0; q < 8; q++)
                if (i0 + q < cnt) {
#pragma unroll
                    for (int hq = 0; hq < 16; hq++)
                        if (hq < qper) acc[hq] += sc[hq * chunk_max + i0 + q] * vv[q];
                }
        }
#pragma unroll
        for (int hq = 0; hq < 16; hq++)
            if (hq < qper) {
                float* ph = pp + (size_t)hq * NSPLIT_ATTN * 258;
                if (d == 0) {
                    ph[0] = ml[hq * 2];
                    ph[1] = ml[hq * 2 + 1];
                }
                ph[2 + d] = acc[hq];
            }
    } else if (d < qper) {
        pp[(size_t)d * NSPLIT_ATTN * 258] = -INFINITY;
        pp[(size_t)d * NSPLIT_ATTN * 258 + 1] = 0.0f;
    }
    // the last split CTA of (t, kh) merges (fixed split order)
    __threadfence();
    __syncthreads();
    if (d == 0) s_last = atomicAdd(&a.counters[t * KV + kh], 1u) == NSPLIT_ATTN - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int hq = 0; hq < qper; hq++) {
        const float* p0 = a.part + ((size_t)t * H + kh * qper + hq) * NSPLIT_ATTN * 258;
        float mv[NSPLIT_ATTN], lv[NSPLIT_ATTN], av[NSPLIT_ATTN];
#pragma unroll
        for (int q = 0; q < NSPLIT_ATTN; q++) {
            mv[q] = __ldcg(p0 + q * 258);
            lv[q] = __ldcg(p0 + q * 258 + 1);
            av[q] = __ldcg(p0 + q * 258 + 2 + d);
        }
        float M = -INFINITY;
#pragma unroll
        for (int q = 0; q < NSPLIT_ATTN; q++) M = fmaxf(M, mv[q]);
        float L = 0.0f, acc = 0.0f;
#pragma unroll
        for (int q = 0; q < NSPLIT_ATTN; q++) {
            if (mv[q] == -INFINITY) continue;
            float wgt = expf(mv[q] - M);
            L += lv[q] * wgt;
            acc += av[q] * wgt;
        }
        a.out[(size_t)t * aw + (kh * qper + hq) * 256 + d] = acc / L;
    }
    if (d == 0) a.counters[t * KV + kh] = 0;
}

void launch_attn(const AttnArgs& a, cudaStream_t st) {
    int qper = a.H / a.KV;
    int chunk_max = attn_chunk_max(a.ctx);
    size_t smem = ((size_t)qper * 256 + (size_t)qper * chunk_max + 2 * VMAX * 256 + 2 * qper) * 4;
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        attr = true;
    }
    AttnArgs aa = a;
    void* args[] = {&aa};
    launch_pdl((const void*)attn_kernel, dim3(a.KV, NSPLIT_ATTN, a.T), dim3(256), smem, st, args);
}

}  // namespace bcu
