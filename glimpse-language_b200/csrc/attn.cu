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

// rmsnorm(x) * w then the interleaved mRoPE rotation of the first `rot` dims (text positions: the three position rows
// are equal, so every section uses `pos`). Thread d holds x[d]; buf: 256 floats, red: 32 floats.
__device__ float norm_rope(float x, float w, int pos, const float* inv_freq, int rot, float* buf, float* red) {
    const int d = threadIdx.x;
    float ss = block_sum(x * x, red);
    x = (x * rsqrtf(ss / 256.0f + EPS_A)) * w;
    __syncthreads();
    buf[d] = x;
    __syncthreads();
    if (d < rot) {
        int half = rot / 2, i = d % half;
        float ang = (float)pos * inv_freq[i];
        float sn, cs;
        sincosf(ang, &sn, &cs);
        x = d < half ? x * cs - buf[d + half] * sn : x * cs + buf[d - half] * sn;
    }
    return x;
}

__global__ void __launch_bounds__(256) attn_kernel(AttnArgs a) {
    extern __shared__ float sm[];
    __shared__ float red[32];
    __shared__ float buf[256];
    __shared__ int s_last;
    const int kh = blockIdx.x, s = blockIdx.y, t = blockIdx.z;
    const int H = a.H, KV = a.KV, qper = H / KV, aw = H * 256, kvw = KV * 256;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, d = threadIdx.x;
    const int chunk_max = (a.ctx + NSPLIT_ATTN - 1) / NSPLIT_ATTN;
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
        // queries of the qper heads (scaled by 1/16 = 1/sqrt(256))
        const float* row = a.qkv + (size_t)t * a.ld;
        for (int hq = 0; hq < qper; hq++) {
            float x = row[(kh * qper + hq) * 512 + d];
            qs[hq * 256 + d] = norm_rope(x, wq, off + t, a.inv_freq, a.rot, buf, red) * 0.0625f;
        }
        // this pass's keys in range
        const int u0 = max(j0, off) - off, u1 = j1 - off;
        for (int u = u0; u < u1; u++) {
            const float* r = a.qkv + (size_t)u * a.ld;
            float k = norm_rope(r[2 * aw + kh * 256 + d], wk, off + u, a.inv_freq, a.rot, buf, red);
            float v = r[2 * aw + kvw + kh * 256 + d];
            nk[u * 256 + d] = k;
            nv[u * 256 + d] = v;
            a.kc[((size_t)(off + u) * KV + kh) * 256 + d] = k;
            a.vc[((size_t)(off + u) * KV + kh) * 256 + d] = v;
        }
        __syncthreads();
        // scores: warp per key, lanes over dims (8 each)
        for (int j = j0 + w; j < j1; j += 8) {
            const float* k = j >= off ? nk + (j - off) * 256 + lane * 8 : a.kc + ((size_t)j * KV + kh) * 256 + lane * 8;
            float4 ka = *(const float4*)k, kb = *(const float4*)(k + 4);
            for (int hq = 0; hq < qper; hq++) {
                const float* q = qs + hq * 256 + lane * 8;
                float dd = q[0] * ka.x + q[1] * ka.y + q[2] * ka.z + q[3] * ka.w + q[4] * kb.x + q[5] * kb.y +
                           q[6] * kb.z + q[7] * kb.w;
                dd = warp_sum(dd);
                if (lane == 0) sc[hq * chunk_max + (j - j0)] = dd;
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
        for (int i = 0; i < cnt; i++) {
            int j = j0 + i;
            float v = j >= off ? nv[(j - off) * 256 + d] : a.vc[((size_t)j * KV + kh) * 256 + d];
#pragma unroll
            for (int hq = 0; hq < 16; hq++)
                if (hq < qper) acc[hq] += sc[hq * chunk_max + i] * v;
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
    int chunk_max = (a.ctx + NSPLIT_ATTN - 1) / NSPLIT_ATTN;
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
