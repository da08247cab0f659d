// attn.cu — gated full-attention core of the verify pass in one kernel: q/k RMSNorm with interleaved mRoPE and the KV
// write (attn_prep, kernels.metal:627-662), split-K causal GQA over the cache (attn_split :713-780) and the log-sum-exp
// merge (attn_combine :783-799), done by the last split CTA of each (row, kv head).
//
// Grid (KV, NSPLIT_ATTN, T), 256 threads (one per head dim), two CTAs per SM. The grid is fixed for graph capture;
// each CTA derives its key range [j0, j1) of [0, off + t] from the device-side KV offset, so one captured graph serves
// every length and a row's key partition depends only on its own position (batch invariance). Keys of this pass
// (positions >= off) are normalised and rotated by the CTA whose range holds them, which also writes them to the
// cache; older keys and values stream from the cache through shared memory in double-buffered blocks of KST keys
// (cp.async, every copy of a block in flight at once), and the softmax is accumulated online block by block.
#include "common.cuh"
#include "kernels.h"

namespace bcu {

constexpr float EPS_A = 1e-6f;
constexpr int KST = 16;  // cached keys per staged block

// Shared memory (floats): queries [QP][256], cached K and V blocks [2][KST][256] each, this pass's keys and values
// [VMAX][256] each (also the staging of the normed rows), block scores [QP][KST], block probabilities [KST][QP],
// row sums [8][32] + row scales [32], running max / sum / rescale [3][QP] (+pad), cos/sin table [(1 + VMAX)][rot].
__host__ __device__ inline size_t attn_smem_floats(int qp, int rot) {
    return (size_t)qp * 256 + 4 * KST * 256 + 2 * VMAX * 256 + 2 * (size_t)qp * KST + 288 + 4 * (size_t)qp +
           (size_t)(1 + VMAX) * rot;
}

// QP = query heads per kv head rounded up to a power of two (heads qper..QP-1 are zero padding).
template <int QP>
__global__ void __launch_bounds__(256, 2) attn_kernel(AttnArgs a) {
    extern __shared__ __align__(16) float sm[];
    __shared__ int s_last;
    const int kh = blockIdx.x, s = blockIdx.y, t = blockIdx.z;
    const int H = a.H, KV = a.KV, qper = H / KV, aw = H * 256, kvw = KV * 256;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, d = threadIdx.x;
    const int half = a.rot / 2;
    float* qs = sm;                    // [QP][256]
    float* ks = qs + QP * 256;         // [2][KST][256]
    float* vs = ks + 2 * KST * 256;    // [2][KST][256]
    float* nk = vs + 2 * KST * 256;    // [VMAX][256]
    float* nv = nk + VMAX * 256;       // [VMAX][256]
    float* sc = nv + VMAX * 256;       // [QP][KST] scores of the current block
    float* pj = sc + QP * KST;         // [KST][QP] probabilities of the current block
    float* rr = pj + QP * KST;         // [8][32] row sums of squares, then [32] row scales at rr + 256
    float* stt = rr + 288;             // [QP] running max, [QP] running sum, [QP] rescale of the current block
    float* tab = stt + 4 * QP;         // [1 + VMAX][half] (cos, sin): row 0 the query position, 1 + i new key u0 + i
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
        // cached keys [j0, jc1): blocks of KST, two in flight
        const int jc1 = min(j1, off);
        const int nst = (max(jc1 - j0, 0) + KST - 1) / KST;
        auto issue = [&](int st) {
            const int jb = j0 + st * KST, nr = min(KST, jc1 - jb);
            float* kd = ks + (st & 1) * KST * 256;
            float* vd = vs + (st & 1) * KST * 256;
            for (int i = threadIdx.x; i < nr * 64; i += 256) {
                const int r = i >> 6, c = (i & 63) * 4;
                const size_t src = ((size_t)(jb + r) * KV + kh) * 256 + c;
                cp_async16(kd + r * 256 + c, a.kc + src);
                cp_async16(vd + r * 256 + c, a.vc + src);
            }
            cp_async_commit();
        };
        // rows to prepare: the qper query heads of row t, then this pass's keys in range (positions >= off),
        // all loaded at once, ahead of the cached blocks
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
        if (nst > 0) issue(0);
        if (nst > 1) issue(1);
        for (int e = threadIdx.x; e < (1 + nkeys) * half; e += 256) {
            const int pi = e / half, f = e - pi * half;
            const int pos = pi == 0 ? off + t : off + u0 + pi - 1;
            float sn, cs;
            sincosf((float)pos * a.inv_freq[f], &sn, &cs);
            tab[2 * e] = cs;
            tab[2 * e + 1] = sn;
        }
        // sums of squares of the 32 rows: halving butterfly, lane l ends with its warp's part of row l
        {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; i++) v[i] = x[i] * x[i];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const bool up = (lane & o) != 0;
#pragma unroll
                for (int j = 0; j < o; j++) {
                    const float send = up ? v[j] : v[j + o];
                    const float keep = up ? v[j + o] : v[j];
                    v[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
                }
            }
            rr[w * 32 + lane] = v[0];
        }
        __syncthreads();
        if (d < 32) {
            float ss = 0.0f;
#pragma unroll
            for (int q = 0; q < 8; q++) ss += rr[q * 32 + d];
            rr[256 + d] = rsqrtf(ss / 256.0f + EPS_A);
        }
        __syncthreads();
        float* xs = nk;  // staging of the normed rows [nrows][256] (nk/nv regions are free until below)
#pragma unroll
        for (int i = 0; i < 32; i++)
            if (i < nrows) xs[i * 256 + d] = (x[i] * rr[256 + i]) * (i < qper ? wq : wk);
        __syncthreads();
        // interleaved mRoPE on the first `rot` dims; text positions: the three position rows are equal
        float y[32];
        const int f = d < half ? d : d - half;
#pragma unroll
        for (int i = 0; i < 32; i++)
            if (i < nrows) {
                float xv = xs[i * 256 + d];
                if (d < a.rot) {
                    const int pi = i < qper ? 0 : 1 + (i - qper);
                    const float cs = tab[2 * (pi * half + f)], sn = tab[2 * (pi * half + f) + 1];
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
        for (int h = qper; h < QP; h++) qs[h * 256 + d] = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; i++)
            if (i < nkeys) {
                int u = u0 + i;
                nv[u * 256 + d] = vvals[i];
                a.vc[((size_t)(off + u) * KV + kh) * 256 + d] = vvals[i];
            }
        if (d < QP) {
            stt[d] = -INFINITY;
            stt[QP + d] = 0.0f;
        }

        // blocks of keys in order: the cached blocks, then this pass's keys; online softmax per query head
        float acc[QP];
#pragma unroll
        for (int h = 0; h < QP; h++) acc[h] = 0.0f;
        const int kj = d >> 4, kc = d & 15;  // score mapping: key kj of the block, dims 4 kc + 64 i (i < 4)
        const int nblk = nst + (nkeys > 0 ? 1 : 0);
        for (int st = 0; st < nblk; st++) {
            const bool cached = st < nst;
            const float *kb, *vb;
            int nr;
            if (cached) {
                if (st + 1 < nst) cp_async_wait_group<1>();
                else cp_async_wait_group<0>();
                kb = ks + (st & 1) * KST * 256;
                vb = vs + (st & 1) * KST * 256;
                nr = min(KST, jc1 - (j0 + st * KST));
            } else {
                kb = nk + u0 * 256;
                vb = nv + u0 * 256;
                nr = nkeys;
            }
            __syncthreads();
            // scores: 16 threads per key, each 16 dims for all heads, then a halving butterfly over the 16
            {
                float part[QP];
#pragma unroll
                for (int h = 0; h < QP; h++) part[h] = 0.0f;
                if (kj < nr) {
                    float4 k4[4];
#pragma unroll
                    for (int i = 0; i < 4; i++) k4[i] = *(const float4*)(kb + kj * 256 + 4 * kc + 64 * i);
#pragma unroll
                    for (int h = 0; h < QP; h++) {
                        float a2 = 0.0f;
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            const float4 q4 = *(const float4*)(qs + h * 256 + 4 * kc + 64 * i);
                            a2 += q4.x * k4[i].x + q4.y * k4[i].y + q4.z * k4[i].z + q4.w * k4[i].w;
                        }
                        part[h] = a2;
                    }
                }
                // reduce over the 16 lanes of the key (offsets 8, 4, 2, 1): lane kc ends with head kc * QP / 16
                // (QP >= 16) or, for QP < 16, head (kc >> log2(16 / QP)) summed over the remaining lanes
#pragma unroll
                for (int o = 8, nn = QP; o > 0; o >>= 1) {
                    if (nn > 1) {
                        const bool up = (lane & o) != 0;
                        const int hn = nn / 2;
#pragma unroll
                        for (int j = 0; j < hn; j++) {
                            const float send = up ? part[j] : part[j + hn];
                            const float keep = up ? part[j + hn] : part[j];
                            part[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
                        }
                        nn = hn;
                    } else {
                        part[0] += __shfl_xor_sync(0xffffffffu, part[0], o);
                    }
                }
                // lane bits (from offset 8 down) select the half kept at each halving stage
                int hsel = 0, nn2 = QP;
#pragma unroll
                for (int o = 8; o > 0 && nn2 > 1; o >>= 1) {
                    hsel = hsel * 2 + ((lane & o) ? 1 : 0);
                    nn2 >>= 1;
                }
                const int lanes_per_head = 16 / (QP < 16 ? QP : 16);
                if (kj < nr && (kc % lanes_per_head) == 0 && hsel < QP) sc[hsel * KST + kj] = part[0];
            }
            __syncthreads();
            for (int h = w; h < qper; h += 8) {
                const float sv = lane < nr ? sc[h * KST + lane] : -INFINITY;
                const float mo = stt[h];
                const float mn = fmaxf(mo, warp_max(sv));
                const float p = lane < nr ? expf(sv - mn) : 0.0f;
                const float ps = warp_sum(p);
                if (lane < KST) pj[lane * QP + h] = p;
                if (lane == 0) {
                    const float al = expf(mo - mn);
                    stt[2 * QP + h] = al;
                    stt[QP + h] = stt[QP + h] * al + ps;
                    stt[h] = mn;
                }
            }
            __syncthreads();
            // P.V: thread = head dim, keys in order
            {
                float al[QP];
#pragma unroll
                for (int h = 0; h < QP; h++) al[h] = h < qper ? stt[2 * QP + h] : 0.0f;
#pragma unroll
                for (int h = 0; h < QP; h++) acc[h] *= al[h];
                float vv[KST];
#pragma unroll
                for (int j = 0; j < KST; j++) vv[j] = j < nr ? vb[j * 256 + d] : 0.0f;
#pragma unroll
                for (int j = 0; j < KST; j++)
                    if (j < nr) {
#pragma unroll
                        for (int h4 = 0; h4 < (QP + 3) / 4; h4++) {
                            float4 p4;
                            if (QP >= 4) p4 = *(const float4*)(pj + j * QP + 4 * h4);
                            else p4 = make_float4(pj[j * QP], QP > 1 ? pj[j * QP + 1] : 0.0f, 0.0f, 0.0f);
                            if (4 * h4 + 0 < QP) acc[4 * h4 + 0] += p4.x * vv[j];
                            if (4 * h4 + 1 < QP) acc[4 * h4 + 1] += p4.y * vv[j];
                            if (4 * h4 + 2 < QP) acc[4 * h4 + 2] += p4.z * vv[j];
                            if (4 * h4 + 3 < QP) acc[4 * h4 + 3] += p4.w * vv[j];
                        }
                    }
            }
            __syncthreads();  // the block's buffers are free
            if (cached && st + 2 < nst) issue(st + 2);
        }
#pragma unroll
        for (int h = 0; h < QP; h++)
            if (h < qper) {
                float* ph = pp + (size_t)h * NSPLIT_ATTN * 258;
                if (d == 0) {
                    ph[0] = stt[h];
                    ph[1] = stt[QP + h];
                }
                ph[2 + d] = acc[h];
            }
    } else if (d < qper) {
        pp[(size_t)d * NSPLIT_ATTN * 258] = -INFINITY;
        pp[(size_t)d * NSPLIT_ATTN * 258 + 1] = 0.0f;
    }
    // the last split CTA of (t, kh) merges (fixed split order)
    __syncthreads();
    if (d == 0) {
        unsigned old;
        asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;"
                     : "=r"(old)
                     : "l"(a.counters + t * KV + kh)
                     : "memory");
        s_last = old == NSPLIT_ATTN - 1;
    }
    __syncthreads();
    if (!s_last) return;
    const float* p0 = a.part + ((size_t)t * H + kh * qper) * NSPLIT_ATTN * 258;
    float* mls = qs;  // [qper][NSPLIT][2]
    float av[2][NSPLIT_ATTN], an[2][NSPLIT_ATTN];
    auto load_av = [&](int h0, float (*dst)[NSPLIT_ATTN]) {
#pragma unroll
        for (int hh = 0; hh < 2; hh++)
#pragma unroll
            for (int q = 0; q < NSPLIT_ATTN; q++)
                dst[hh][q] = h0 + hh < qper ? __ldcg(p0 + (size_t)(h0 + hh) * NSPLIT_ATTN * 258 + q * 258 + 2 + d) : 0.0f;
    };
    load_av(0, av);
    for (int e = threadIdx.x; e < qper * NSPLIT_ATTN * 2; e += 256) {
        const int h = e / (2 * NSPLIT_ATTN), r = e - h * 2 * NSPLIT_ATTN;
        mls[e] = __ldcg(p0 + (size_t)h * NSPLIT_ATTN * 258 + (r >> 1) * 258 + (r & 1));
    }
    __syncthreads();
    for (int h0 = 0; h0 < qper; h0 += 2) {
        if (h0 + 2 < qper) load_av(h0 + 2, an);  // the next heads' loads in flight while these are merged
#pragma unroll
        for (int hh = 0; hh < 2; hh++) {
            const int h = h0 + hh;
            if (h >= qper) break;
            const float* m2 = mls + h * NSPLIT_ATTN * 2;
            float M = -INFINITY;
#pragma unroll
            for (int q = 0; q < NSPLIT_ATTN; q++) M = fmaxf(M, m2[2 * q]);
            float L = 0.0f, o = 0.0f;
#pragma unroll
            for (int q = 0; q < NSPLIT_ATTN; q++) {
                if (m2[2 * q] == -INFINITY) continue;
                const float wgt = expf(m2[2 * q] - M);
                L += m2[2 * q + 1] * wgt;
                o += av[hh][q] * wgt;
            }
            a.out[(size_t)t * aw + (kh * qper + h) * 256 + d] = o / L;
        }
#pragma unroll
        for (int hh = 0; hh < 2; hh++)
#pragma unroll
            for (int q = 0; q < NSPLIT_ATTN; q++) av[hh][q] = an[hh][q];
    }
    if (d == 0) a.counters[t * KV + kh] = 0;
}

template <int QP>
static void launch_attn_t(const AttnArgs& a, cudaStream_t st) {
    size_t smem = attn_smem_floats(QP, a.rot) * 4;
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(attn_kernel<QP>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        attr = true;
    }
    AttnArgs aa = a;
    void* args[] = {&aa};
    launch_pdl((const void*)attn_kernel<QP>, dim3(a.KV, NSPLIT_ATTN, a.T), dim3(256), smem, st, args);
}

void launch_attn(const AttnArgs& a, cudaStream_t st) {
    const int qper = a.H / a.KV;
    if (qper <= 1) launch_attn_t<1>(a, st);
    else if (qper <= 2) launch_attn_t<2>(a, st);
    else if (qper <= 4) launch_attn_t<4>(a, st);
    else if (qper <= 8) launch_attn_t<8>(a, st);
    else launch_attn_t<16>(a, st);
}

}  // namespace bcu
