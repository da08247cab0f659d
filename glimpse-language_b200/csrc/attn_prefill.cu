// attn_prefill.cu — causal GQA attention of a prefill chunk (attn_split + attn_combine, kernels.metal:713-799, over
// the chunk's rows; the reference runs its prefill attention in 512-key chunks, model.rs:852-855) on the tensor
// cores: one CTA per (kv head, block of RB = 32 / qper rows), i.e. 32 query vectors (the kv head's qper query heads
// of RB rows), over the cached keys in blocks of 64 with an online softmax.
//
// Per key block: S = Q K^T (32 x 64, K = 256) and O += P V (32 x 256, K = 64) as mma.sync tf32 with the three-product
// split (mma_tf32.cuh, fp32-accurate); the causal mask per query vector (key position <= the row's position); the
// running maximum and sum per query vector in fp32 with expf, as the reference's softmax. The keys and values of block
// b + 1 are fetched (cp.async) behind block b's work: K(b + 1) once S(b) is taken, V(b + 1) once O has used V(b).
// Queries come prepared by pf_attn_prep_kernel (normed, rotated, scaled by 1/16); every key of the chunk is in the
// cache before this kernel runs.
#include "common.cuh"
#include "kernels.h"
#include "mma_tf32.cuh"

namespace bcu {

constexpr int AP_M = 32;     // query vectors per CTA
constexpr int AP_KB = 64;    // keys per block
constexpr int AP_QS = 260;   // row stride (floats) of Q and K in shared memory (A / n-major B fragments conflict-free)
constexpr int AP_VS = 264;   // row stride of V (k-major B fragments conflict-free)
constexpr int AP_PS = 68;    // row stride of P

struct ApSmem {
    float q[AP_M][AP_QS];
    float k[AP_KB][AP_QS];
    float v[AP_KB][AP_VS];
    float p[AP_M][AP_PS];
    float mx[AP_M], sum[AP_M], alpha[AP_M];
};

__global__ void __launch_bounds__(256, 1) attn_prefill_kernel(const float* qprep, const float* kc, const float* vc,
                                                              float* out, int T, int H, int KV, int off0) {
    extern __shared__ __align__(16) uint8_t asm_raw[];
    ApSmem& sm = *(ApSmem*)asm_raw;
    const int kh = blockIdx.x, tid = threadIdx.x, lane = tid & 31, w = tid >> 5, g = lane >> 2, qd = lane & 3;
    const int qper = H / KV, RB = AP_M / qper;
    // first row of the block (chunk-relative); the last blocks, with the most keys, are launched first
    const int r0 = (gridDim.y - 1 - blockIdx.y) * RB;
    const int rows = min(RB, T - r0);
    const int last_pos = off0 + r0 + rows - 1;            // the block's largest query position
    const int nkb = last_pos / AP_KB + 1;                 // key blocks covering positions 0 .. last_pos
    // query vector m: row r0 + m / qper, head kh * qper + m % qper
    for (int i = tid; i < AP_M * 64; i += 256) {
        const int m = i >> 6, j = (i & 63) * 4, r = m / qper;
        float4 x = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (r < rows) x = *(const float4*)(qprep + ((size_t)(r0 + r) * H + kh * qper + m % qper) * 256 + j);
        *(float4*)&sm.q[m][j] = x;
    }
    if (tid < AP_M) {
        sm.mx[tid] = -INFINITY;
        sm.sum[tid] = 0.0f;
    }
    auto load_k = [&](int b) {
        for (int i = tid; i < AP_KB * 64; i += 256) {
            const int kk = i >> 6, j = (i & 63) * 4, pos = b * AP_KB + kk;
            if (pos <= last_pos) cp_async16(&sm.k[kk][j], kc + ((size_t)pos * KV + kh) * 256 + j);
            else *(float4*)&sm.k[kk][j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
        cp_async_commit();
    };
    auto load_v = [&](int b) {
        for (int i = tid; i < AP_KB * 64; i += 256) {
            const int kk = i >> 6, j = (i & 63) * 4, pos = b * AP_KB + kk;
            if (pos <= last_pos) cp_async16(&sm.v[kk][j], vc + ((size_t)pos * KV + kh) * 256 + j);
            else *(float4*)&sm.v[kk][j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
        cp_async_commit();
    };
    load_k(0);
    load_v(0);
    const int mt = w & 1;             // query vectors 16 mt .. + 15
    const int ns0 = 2 * (w >> 1);     // S: keys 8 ns0 .. + 15 of the block
    const int nd0 = 8 * (w >> 1);     // O: dims 8 nd0 .. + 63
    float o[8][4];
#pragma unroll
    for (int n = 0; n < 8; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    for (int b = 0; b < nkb; b++) {
        cp_async_wait_group<1>();  // K(b) has landed (V(b) may still be in flight)
        __syncthreads();
        {   // S = Q K^T, masked, into p
            Acc3 s3[2];
            acc3_zero(s3[0]);
            acc3_zero(s3[1]);
#pragma unroll 4
            for (int ks = 0; ks < 32; ks++) {
                Tf32x2 a[4];
                frag_a_rows(&sm.q[0][0], AP_QS, 16 * mt, 8 * ks, a);
#pragma unroll
                for (int n = 0; n < 2; n++) {
                    Tf32x2 bk[2];
                    frag_b_nrows(&sm.k[0][0], AP_QS, 8 * ks, 8 * (ns0 + n), bk);  // (dim, key) = K[key][dim]
                    mma_tf32x3_acc(s3[n], a, bk);
                }
            }
#pragma unroll
            for (int n = 0; n < 2; n++)
#pragma unroll
                for (int hf = 0; hf < 2; hf++) {
                    const int m = 16 * mt + g + 8 * hf, r = m / qper, pos = off0 + r0 + r;
                    const int kl = 8 * (ns0 + n) + 2 * qd, key = b * AP_KB + kl;
                    sm.p[m][kl] = r < rows && key <= pos ? mma3_sum(s3[n], 2 * hf) : -INFINITY;
                    sm.p[m][kl + 1] = r < rows && key + 1 <= pos ? mma3_sum(s3[n], 2 * hf + 1) : -INFINITY;
                }
        }
        __syncthreads();  // the scores; K(b) is free
        if (b + 1 < nkb) load_k(b + 1);
        else cp_async_commit();  // an empty group keeps the wait counts regular
        // online softmax: warp w takes query vectors 4 w .. 4 w + 3, lane keys lane and lane + 32
#pragma unroll
        for (int rr = 0; rr < 4; rr++) {
            const int m = 4 * w + rr;
            const float s0 = sm.p[m][lane], s1 = sm.p[m][lane + 32];
            const float mo = sm.mx[m];
            const float mn = fmaxf(mo, warp_max(fmaxf(s0, s1)));
            const bool none = mn == -INFINITY;  // a padding vector past the chunk's last row
            const float p0 = none ? 0.0f : expf(s0 - mn), p1 = none ? 0.0f : expf(s1 - mn);
            sm.p[m][lane] = p0;
            sm.p[m][lane + 32] = p1;
            const float ps = warp_sum(p0 + p1);
            if (lane == 0) {
                const float al = none ? 1.0f : expf(mo - mn);
                sm.alpha[m] = al;
                sm.sum[m] = sm.sum[m] * al + ps;
                sm.mx[m] = mn;
            }
        }
        cp_async_wait_group<1>();  // V(b) has landed (K(b + 1) may still be in flight)
        __syncthreads();           // probabilities, alpha; V(b)
        {   // O = alpha O + P V
            const float al0 = sm.alpha[16 * mt + g], al1 = sm.alpha[16 * mt + g + 8];
#pragma unroll
            for (int n = 0; n < 8; n++) {
                o[n][0] *= al0;
                o[n][1] *= al0;
                o[n][2] *= al1;
                o[n][3] *= al1;
            }
#pragma unroll 2
            for (int ks = 0; ks < 8; ks++) {
                Tf32x2 a[4];
                frag_a_rows(&sm.p[0][0], AP_PS, 16 * mt, 8 * ks, a);
#pragma unroll
                for (int n = 0; n < 8; n++) {
                    Tf32x2 bv[2];
                    frag_b_krows(&sm.v[0][0], AP_VS, 8 * ks, 8 * (nd0 + n), bv);  // (key, dim) = V[key][dim]
                    mma_tf32x3(o[n], a, bv);
                }
            }
        }
        __syncthreads();  // P and V(b) are free
        if (b + 1 < nkb) load_v(b + 1);
        else cp_async_commit();
    }
    cp_async_wait_all();
    // out[t][head][dim] = O / sum
    const int aw = H * 256;
#pragma unroll
    for (int hf = 0; hf < 2; hf++) {
        const int m = 16 * mt + g + 8 * hf, r = m / qper;
        if (r >= rows) continue;
        const float inv = 1.0f / sm.sum[m];
        float* dst = out + (size_t)(r0 + r) * aw + (kh * qper + m % qper) * 256;
#pragma unroll
        for (int n = 0; n < 8; n++)
            *(float2*)(dst + 8 * (nd0 + n) + 2 * qd) = make_float2(o[n][2 * hf] * inv, o[n][2 * hf + 1] * inv);
    }
}

bool attn_prefill_supported(int H, int KV) {
    const int qper = KV > 0 ? H / KV : 0;
    return qper > 0 && H % KV == 0 && AP_M % qper == 0;
}

void launch_attn_prefill(const float* qprep, const float* kc, const float* vc, float* out, int T, int H, int KV,
                         int off0, cudaStream_t st) {
    const int RB = AP_M / (H / KV);
    raise_smem_limit((const void*)attn_prefill_kernel, (int)sizeof(ApSmem));
    attn_prefill_kernel<<<dim3(KV, (T + RB - 1) / RB), 256, sizeof(ApSmem), st>>>(qprep, kc, vc, out, T, H, KV, off0);
}

}  // namespace bcu
