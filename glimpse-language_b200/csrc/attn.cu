// attn.cu — gated full-attention core of the verify pass in two kernels: q/k RMSNorm with interleaved mRoPE and the KV
// write (attn_prep, kernels.metal:627-662) with split-K causal GQA over the cache (attn_split :713-780), then the
// log-sum-exp merge of the splits (attn_combine :783-799) by attn_merge_kernel, one CTA per (row, query head). The
// merge was first done by the last split CTA of each (row, kv head): 13 us of the layer's 32 in the pass graph.
//
// Grid (KV, NSPLIT_ATTN, T), 256 threads, two CTAs per SM. The grid is fixed for graph capture; each CTA derives its
// key range [j0, j1) of [0, off + t] from the device-side KV offset, so one captured graph serves every length and a
// row's key partition depends only on its own position (batch invariance). Keys of this pass (positions >= off) are
// normalised and rotated by every CTA whose range holds them (identical bits; that CTA also writes them to the cache).
// Inside a CTA the range is scored in rounds of up to SUB keys: each warp takes every 8th key (a lane holds 8 of the
// 256 dims of the key and of each query head, so one coalesced 1-KB row read per key), the heads' partial dot
// products are summed across the warp by a halving butterfly, the round's softmax statistics are taken per head,
// and the thread of each head dim accumulates P.V over the round's keys in key order. Three barriers per round;
// one round covers 16 x 512 = 8192 keys of context.
#include "common.cuh"
#include "kernels.h"

namespace bcu {

constexpr float EPS_A = 1e-6f;
constexpr int SUB = 512;  // keys scored per round

// Shared memory (floats): queries [QP][256], this pass's keys and values in range [VMAX][256] each, scores then
// probabilities of a round [SUB][QP], running max / sum / rescale [4][QP], cos/sin table [(1 + VMAX)][rot].
__host__ __device__ inline size_t attn_smem_floats(int qp, int rot) {
    return (size_t)qp * 256 + 2 * VMAX * 256 + (size_t)(SUB > 1024 ? SUB : 1024) * qp + 4 * (size_t)qp +
           (size_t)(1 + VMAX) * rot;
}

// QP = query heads per kv head rounded up to a power of two (heads qper..QP-1 are zero padding).
template <int QP>
__global__ void __launch_bounds__(256, 2) attn_kernel(AttnArgs a) {
    extern __shared__ __align__(16) float sm[];
    constexpr int HG = QP < 8 ? QP : 8;  // heads scored per pass over the keys (their queries live in registers)
    constexpr int LHG = HG >= 8 ? 3 : (HG >= 4 ? 2 : (HG >= 2 ? 1 : 0));
    const int kh = blockIdx.x, s = blockIdx.y, t = blockIdx.z;
    const int H = a.H, KV = a.KV, qper = H / KV, aw = H * 256, kvw = KV * 256;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, d = threadIdx.x;
    const int half = a.rot / 2;
    float* qs = sm;                  // [QP][256]
    float* nk = qs + QP * 256;       // [VMAX][256] keys of this pass in range, index u - u0
    float* nv = nk + VMAX * 256;     // [VMAX][256] their values
    float* pr = nv + VMAX * 256;     // [SUB][QP] scores, then probabilities; at the end the P.V phases [4][QP][256]
    float* stt = pr + (SUB > 1024 ? SUB : 1024) * QP;  // [QP] running max, [QP] running sum, [QP] rescale
    float* tab = stt + 4 * QP;       // [1 + VMAX][half] (cos, sin): row 0 the query position, 1 + i key u0 + i
    pdl_trigger();
    pdl_wait();
    // prefill mode (a.qprep): the queries come prepared and every key of the chunk is already in the cache
    const bool pre = a.qprep != nullptr;
    const int off = pre ? a.off0 : a.ctl->off;
    const int n = off + t + 1;
    const int NS = a.nsplit;
    const int chunk = (n + NS - 1) / NS;
    const int j0 = s * chunk, j1 = min(n, j0 + chunk);
    const int koff = pre ? n : off;  // keys below koff are read from the cache, the others were prepared here
    float* pp = a.part + ((size_t)t * H + kh * qper) * NS * 258 + (size_t)s * 258;
    if (n > a.ctx) {
        if (d == 0 && s == 0 && kh == 0) atomicOr(&((Ctl*)a.ctl)->err, ERR_CTX_FULL);
        return;
    }
    if (j0 < j1) {
        const int u0 = max(j0, koff) - koff, u1 = j1 - koff, nkeys = max(u1 - u0, 0);
        for (int e = threadIdx.x; e < (pre ? 0 : (1 + nkeys) * half); e += 256) {
            const int pi = e / half, f = e - pi * half;
            const int pos = pi == 0 ? off + t : off + u0 + pi - 1;
            float sn, cs;
            sincosf((float)pos * a.inv_freq[f], &sn, &cs);
            tab[2 * e] = cs;
            tab[2 * e + 1] = sn;
        }
        for (int e = threadIdx.x; e < (QP - qper) * 256; e += 256) qs[qper * 256 + e] = 0.0f;
        if (d < QP) {
            stt[d] = -INFINITY;
            stt[QP + d] = 0.0f;
        }
        // values of this pass's keys in range: to shared memory and the cache
        for (int e = threadIdx.x; e < nkeys * 64; e += 256) {
            const int i = e >> 6, c = (e & 63) * 4;
            const float4 v4 = *(const float4*)(a.qkv + (size_t)(u0 + i) * a.ld + 2 * aw + kvw + kh * 256 + c);
            *(float4*)(nv + i * 256 + c) = v4;
            *(float4*)(a.vc + ((size_t)(off + u0 + i) * KV + kh) * 256 + c) = v4;
        }
        __syncthreads();  // the cos/sin table
        // rows to prepare, one warp each: the qper query heads of row t, then this pass's keys in range. A lane holds
        // dims [8 lane, 8 lane + 8): RMSNorm (warp sum of squares), weight, then the rotation of the first `rot`
        // dims against their partner d +- rot/2 read back from the row in shared memory.
        for (int r = w; r < qper + nkeys; r += 8) {
            const bool isq = r < qper;
            if (pre) {  // prepared query rows [T][H][256] (normed, rotated, scaled)
                const float* qsrc = a.qprep + ((size_t)t * H + kh * qper + r) * 256 + lane * 8;
                *(float4*)(qs + r * 256 + lane * 8) = *(const float4*)qsrc;
                *(float4*)(qs + r * 256 + lane * 8 + 4) = *(const float4*)(qsrc + 4);
                continue;
            }
            const float* src = isq ? a.qkv + (size_t)t * a.ld + (kh * qper + r) * 512
                                   : a.qkv + (size_t)(u0 + r - qper) * a.ld + 2 * aw + kh * 256;
            float* dst = isq ? qs + r * 256 : nk + (r - qper) * 256;
            const float* wn = isq ? a.qn : a.kn;
            float x[8];
            *(float4*)&x[0] = *(const float4*)(src + lane * 8);
            *(float4*)&x[4] = *(const float4*)(src + lane * 8 + 4);
            float ss = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; i++) ss += x[i] * x[i];
            const float rs = rsqrtf(warp_sum(ss) / 256.0f + EPS_A);
#pragma unroll
            for (int i = 0; i < 8; i++) x[i] = (x[i] * rs) * wn[lane * 8 + i];
            *(float4*)(dst + lane * 8) = *(const float4*)&x[0];
            *(float4*)(dst + lane * 8 + 4) = *(const float4*)&x[4];
            __syncwarp();
            float y[8];
            const int pi = isq ? 0 : 1 + (r - qper);
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int dd = lane * 8 + i;
                y[i] = x[i];
                if (dd < a.rot) {
                    const int f = dd < half ? dd : dd - half;
                    const float cs = tab[2 * (pi * half + f)], sn = tab[2 * (pi * half + f) + 1];
                    y[i] = dd < half ? x[i] * cs - dst[dd + half] * sn : x[i] * cs + dst[dd - half] * sn;
                }
            }
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 8; i++) y[i] = isq ? y[i] * 0.0625f : y[i];  // queries scaled by 1/sqrt(256)
            *(float4*)(dst + lane * 8) = *(const float4*)&y[0];
            *(float4*)(dst + lane * 8 + 4) = *(const float4*)&y[4];
            if (!isq) {
                float* kd = a.kc + ((size_t)(off + u0 + r - qper) * KV + kh) * 256 + lane * 8;
                *(float4*)kd = *(const float4*)&y[0];
                *(float4*)(kd + 4) = *(const float4*)&y[4];
            }
        }
        __syncthreads();

        float acc[QP][4];
#pragma unroll
        for (int h = 0; h < QP; h++) acc[h][0] = acc[h][1] = acc[h][2] = acc[h][3] = 0.0f;
        const int ph = threadIdx.x >> 6, dc = (threadIdx.x & 63) * 4;
        const int hsel = HG > 1 ? (lane >> (5 - LHG)) & (HG - 1) : 0;
        const bool writer = (lane & ((32 >> LHG) - 1)) == 0;
        for (int jb = j0; jb < j1; jb += SUB) {
            const int nr = min(SUB, j1 - jb);
            // scores of the round: warp w takes keys jb + w, jb + w + 8, ...
#pragma unroll
            for (int hg = 0; hg < QP; hg += HG) {
                // KU keys per warp iteration, their loads issued together; each query head's 8 dims are read from
                // shared memory once per iteration and applied to the KU keys
                constexpr int KU = 4;
                for (int j = w; j < nr; j += 8 * KU) {
                    float k[KU][8];
#pragma unroll
                    for (int u = 0; u < KU; u++) {
                        const int jl = j + 8 * u, jj = jb + jl;
                        if (jl < nr) {
                            const float* kp = jj < koff ? a.kc + ((size_t)jj * KV + kh) * 256 : nk + (jj - koff - u0) * 256;
                            *(float4*)&k[u][0] = *(const float4*)(kp + lane * 8);
                            *(float4*)&k[u][4] = *(const float4*)(kp + lane * 8 + 4);
                        } else {
#pragma unroll
                            for (int i = 0; i < 8; i++) k[u][i] = 0.0f;
                        }
                    }
                    float part[KU][HG];
#pragma unroll
                    for (int h = 0; h < HG; h++) {
                        float qv[8];
                        *(float4*)&qv[0] = *(const float4*)(qs + (hg + h) * 256 + lane * 8);
                        *(float4*)&qv[4] = *(const float4*)(qs + (hg + h) * 256 + lane * 8 + 4);
#pragma unroll
                        for (int u = 0; u < KU; u++) {
                            float a2 = 0.0f;
#pragma unroll
                            for (int i = 0; i < 8; i++) a2 += qv[i] * k[u][i];
                            part[u][h] = a2;
                        }
                    }
#pragma unroll
                    for (int u = 0; u < KU; u++) {
                        const int jl = j + 8 * u;
                        // halving butterfly: lane ends with the warp total of head hsel
#pragma unroll
                        for (int o = 16, nn = HG; o > 0; o >>= 1) {
                            if (nn > 1) {
                                const bool up = (lane & o) != 0;
                                const int hn = nn / 2;
#pragma unroll
                                for (int q = 0; q < hn; q++) {
                                    const float send = up ? part[u][q] : part[u][q + hn];
                                    const float keep = up ? part[u][q + hn] : part[u][q];
                                    part[u][q] = keep + __shfl_xor_sync(0xffffffffu, send, o);
                                }
                                nn = hn;
                            } else {
                                part[u][0] += __shfl_xor_sync(0xffffffffu, part[u][0], o);
                            }
                        }
                        if (writer && jl < nr) pr[jl * QP + hg + hsel] = part[u][0];
                    }
                }
            }
            __syncthreads();
            // softmax statistics of the round per head (warp h), probabilities in place
            for (int h = w; h < qper; h += 8) {
                float mx = -INFINITY;
                for (int j = lane; j < nr; j += 32) mx = fmaxf(mx, pr[j * QP + h]);
                const float mo = stt[h];
                const float mn = fmaxf(mo, warp_max(mx));
                float ps = 0.0f;
                for (int j = lane; j < nr; j += 32) {
                    const float p = expf(pr[j * QP + h] - mn);
                    pr[j * QP + h] = p;
                    ps += p;
                }
                ps = warp_sum(ps);
                if (lane == 0) {
                    const float al = expf(mo - mn);
                    stt[2 * QP + h] = al;
                    stt[QP + h] = stt[QP + h] * al + ps;
                    stt[h] = mn;
                }
            }
            __syncthreads();
            // P.V: thread = (key phase ph = tid / 64, dims 4 (tid % 64) .. + 3); phase ph takes the round's keys
            // ph, ph + 4, ... in order, 4 value rows in flight; the phases are summed in order after the keys
#pragma unroll
            for (int h = 0; h < QP; h++) {
                const float al = h < qper ? stt[2 * QP + h] : 0.0f;
#pragma unroll
                for (int c = 0; c < 4; c++) acc[h][c] *= al;
            }
            for (int j4 = ph; j4 < nr; j4 += 16) {
                float4 vv[4];
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const int jl = j4 + 4 * q, jj = jb + jl;
                    vv[q] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    if (jl < nr)
                        vv[q] = jj < koff ? *(const float4*)(a.vc + ((size_t)jj * KV + kh) * 256 + dc)
                                          : *(const float4*)(nv + (jj - koff - u0) * 256 + dc);
                }
#pragma unroll
                for (int q = 0; q < 4; q++)
                    if (j4 + 4 * q < nr) {
                        const float* pj = pr + (j4 + 4 * q) * QP;
#pragma unroll
                        for (int h = 0; h < QP; h++) {
                            const float pv = pj[h];
                            acc[h][0] += pv * vv[q].x;
                            acc[h][1] += pv * vv[q].y;
                            acc[h][2] += pv * vv[q].z;
                            acc[h][3] += pv * vv[q].w;
                        }
                    }
            }
            __syncthreads();  // the round's scores are consumed
        }
        // the four key phases, summed in phase order (the round buffer is free): [ph][h][256]
        float* ps = pr;
#pragma unroll
        for (int h = 0; h < QP; h++)
            if (h < qper) *(float4*)(ps + ((size_t)ph * QP + h) * 256 + dc) = make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
        __syncthreads();
        for (int h = 0; h < qper; h++) {
            float o = ps[(size_t)h * 256 + d];
#pragma unroll
            for (int q = 1; q < 4; q++) o += ps[((size_t)q * QP + h) * 256 + d];
            float* pq = pp + (size_t)h * NS * 258;
            if (d == 0) {
                pq[0] = stt[h];
                pq[1] = stt[QP + h];
            }
            pq[2 + d] = o;
        }
    } else if (d < qper) {
        pp[(size_t)d * NS * 258] = -INFINITY;
        pp[(size_t)d * NS * 258 + 1] = 0.0f;
    }
}

// The merge of the key splits (attn_combine, kernels.metal:783-799), after the split kernel: one CTA per (row, query
// head), thread = head dim; the splits' running maxima, sums and partial outputs read together, combined in split
// order. Each row's splits and their order depend only on its own position (batch invariance).
__global__ void __launch_bounds__(256) attn_merge_kernel(AttnArgs a) {
    const int t = blockIdx.x, hq = blockIdx.y, d = threadIdx.x;
    const int H = a.H, NS = a.nsplit;
    pdl_trigger();
    pdl_wait();
    const float* p0 = a.part + ((size_t)t * H + hq) * NS * 258;
    float mv[NSPLIT_ATTN], lv[NSPLIT_ATTN], ov[NSPLIT_ATTN];
#pragma unroll
    for (int q = 0; q < NSPLIT_ATTN; q++)
        if (q < NS) {
            mv[q] = __ldcg(p0 + q * 258);
            lv[q] = __ldcg(p0 + q * 258 + 1);
            ov[q] = __ldcg(p0 + q * 258 + 2 + d);
        }
    float M = -INFINITY;
#pragma unroll
    for (int q = 0; q < NSPLIT_ATTN; q++)
        if (q < NS) M = fmaxf(M, mv[q]);
    float L = 0.0f, o = 0.0f;
#pragma unroll
    for (int q = 0; q < NSPLIT_ATTN; q++) {
        if (q >= NS || mv[q] == -INFINITY) continue;
        const float wgt = expf(mv[q] - M);
        L += lv[q] * wgt;
        o += ov[q] * wgt;
    }
    a.out[(size_t)t * H * 256 + hq * 256 + d] = o / L;
}

template <int QP>
static void launch_attn_t(const AttnArgs& a, cudaStream_t st) {
    size_t smem = attn_smem_floats(QP, a.rot) * 4;
    raise_smem_limit((const void*)attn_kernel<QP>, 200 * 1024);
    AttnArgs aa = a;
    void* args[] = {&aa};
    launch_pdl((const void*)attn_kernel<QP>, dim3(a.KV, a.nsplit, a.T), dim3(256), smem, st, args);
    launch_pdl((const void*)attn_merge_kernel, dim3(a.T, a.H), dim3(256), 0, st, args);
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
