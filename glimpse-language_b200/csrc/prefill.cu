// prefill.cu — batched prefill of the model (Model::prefill, runtime/mod.rs:341-386): chunks of up to PF_CHUNK
// prompt rows run each linear as one dense contraction on the tcgen05 GEMM (gemm.cu; the reference's prefill qmm,
// kernels.metal:437-500) instead of as 16-row verify passes.
//
// Per chunk of M rows at positions off .. off + M - 1, per layer: the producer kernels below (RMSNorm with the
// residual add of the previous linear folded in, gated RMSNorm, sigmoid gate, SwiGLU; then signs and the
// Walsh-Hadamard transform in fwht512's lane layout) write the rotated fp32 rows the GEMM takes; a GatedDeltaNet layer
// adds the dense a/b rows, the causal conv over [committed conv rows; the chunk] with its per-head norms, the new
// committed conv rows, and the gated delta rule over the M rows (gdn_verify_kernel, n = M); an attention layer adds
// the q/k norm + mRoPE + KV write of the chunk (pf_attn_prep_kernel) and the causal attention of its rows over the
// cache (attn_kernel in its prepared-query mode). The chunk leaves the committed state exactly as M committed rows
// of verify passes would (the conv rows in the double buffer's committed half, no rows to replay).
#include <algorithm>

#include "common.cuh"
#include "gemm_act.cuh"
#include "kernels.h"

namespace bcu {

constexpr float EPS_P = 1e-6f;

__device__ __forceinline__ float sigm_p(float z) { return 1.0f / (1.0f + expf(-z)); }

// Walsh-Hadamard transform of one block of 32 VPL values held by a warp (lane l holds elements l + 32 e): strides 1..16
// across lanes, 32.. inside the lane, ascending (bit-identical to the in-memory radix-2 transform), then x 1/sqrt(HB).
template <int VPL>
__device__ __forceinline__ void fwht_block(float* v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
        const bool up = (lane & m) != 0;
#pragma unroll
        for (int e = 0; e < VPL; e++) {
            const float o = __shfl_xor_sync(0xffffffffu, v[e], m);
            v[e] = up ? __fsub_rn(o, v[e]) : __fadd_rn(v[e], o);
        }
    }
#pragma unroll
    for (int h = 1; h < VPL; h <<= 1)
#pragma unroll
        for (int e = 0; e < VPL; e++)
            if ((e & h) == 0) {
                const float a = v[e], c = v[e + h];
                v[e] = __fadd_rn(a, c);
                v[e + h] = __fsub_rn(a, c);
            }
    const float inv = VPL == 16 ? 0.044194173824159216f : (VPL == 64 ? 0.02209708691207961f : 0.03125f);
#pragma unroll
    for (int e = 0; e < VPL; e++) v[e] = __fmul_rn(v[e], inv);
}

// One row per CTA (one warp per Hadamard block of the row, at most 8): the producer value x_k of the mode, then
// rotate(signs * x) in blocks of HB = 32 VPL (warp w takes blocks w, w + nw, ...), written straight into the GEMM's activation tiles: the rotated row is kept in
// shared memory, its maximum gives the exponent, and the CTA's 8 warps write the tiles with gemm_act_words (the bits
// gemm_prep_kernel would write from the same row in global memory). NORM: x = rmsnorm(h) * w, after h += add (the residual of the
// previous linear, written back). xn (optional, every mode) keeps x unrotated: the GDN a/b rows' input and the
// LoRA input of the linear that follows (lora.rs:1-3: the adapter sees the unrotated input). GATED: per 128-wide head
// (((z * y) * rsqrt(mean(y^2) + eps)) * w) * sigmoid(z), z at src2 (row stride ld2). GATE: attn * sigmoid(gate),
// the gate half of the q projection at src2 (per head 256 q then 256 gate values). SWIGLU: (g * u) * sigmoid(g), g
// and u the two halves of a [2D] row.
template <int VPL>
__global__ void __launch_bounds__(256) pf_rows_kernel(PfRowArgs a) {
    extern __shared__ __align__(16) float s_row[];  // [D] the rotated row
    __shared__ float red[32];
    __shared__ float s_r;
    const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, D = a.D;
    const int nth = blockDim.x, nw = nth >> 5;
    constexpr int HB = VPL * 32;
    float am = 0.0f;  // largest magnitude of this warp's rotated values
    if (a.mode == PF_NORM) {
        float* hr = a.h + (size_t)row * D;
        float ss = 0.0f;
        for (int k = tid; k < D; k += nth) {
            float x = hr[k];
            if (a.add) {
                x = __fadd_rn(x, a.add[(size_t)row * D + k]);
                hr[k] = x;
            }
            ss = __fmaf_rn(x, x, ss);
        }
        const float tot = block_sum(ss, red);
        if (tid == 0) s_r = rsqrtf(tot / (float)D + EPS_P);
        __syncthreads();
    }
    for (int b0 = warp * HB; b0 < D; b0 += nw * HB) {
        float v[VPL];
        if (a.mode == PF_NORM) {
            const float r = s_r;
#pragma unroll
            for (int e = 0; e < VPL; e++) {
                const int k = b0 + lane + 32 * e;
                v[e] = __fmul_rn(__fmul_rn(a.h[(size_t)row * D + k], r), a.w[k]);
                if (a.xn) a.xn[(size_t)row * D + k] = v[e];
            }
        } else if (a.mode == PF_GATED) {
            float y[VPL], z[VPL];
#pragma unroll
            for (int e = 0; e < VPL; e++) {
                const int k = b0 + lane + 32 * e;
                y[e] = a.src[(size_t)row * D + k];
                z[e] = a.src2[(size_t)row * a.ld2 + k];
            }
#pragma unroll
            for (int c = 0; c < VPL / 4; c++) {  // head c of the block: elements e in [4 c, 4 c + 4) of every lane
                float s2 = 0.0f;
#pragma unroll
                for (int e = 4 * c; e < 4 * c + 4; e++) s2 = __fmaf_rn(y[e], y[e], s2);
                const float rh = rsqrtf(warp_sum(s2) / 128.0f + EPS_P);
#pragma unroll
                for (int e = 4 * c; e < 4 * c + 4; e++) {
                    const float wn = a.w[(lane + 32 * e) & 127];
                    v[e] = __fmul_rn(__fmul_rn(__fmul_rn(__fmul_rn(z[e], y[e]), rh), wn), sigm_p(z[e]));
                }
            }
        } else if (a.mode == PF_GATE) {
#pragma unroll
            for (int e = 0; e < VPL; e++) {
                const int k = b0 + lane + 32 * e;
                const float g = a.src2[(size_t)row * a.ld2 + (k >> 8) * 512 + 256 + (k & 255)];
                v[e] = __fmul_rn(a.src[(size_t)row * D + k], sigm_p(g));
            }
        } else {
#pragma unroll
            for (int e = 0; e < VPL; e++) {
                const int k = b0 + lane + 32 * e;
                const float g = a.src[(size_t)row * 2 * D + k], u = a.src[(size_t)row * 2 * D + D + k];
                v[e] = __fmul_rn(__fmul_rn(g, u), sigm_p(g));
            }
        }
        if (a.xn && a.mode != PF_NORM) {
#pragma unroll
            for (int e = 0; e < VPL; e++) a.xn[(size_t)row * D + b0 + lane + 32 * e] = v[e];
        }
        if (a.signs) {
#pragma unroll
            for (int e = 0; e < VPL; e++) v[e] = __fmul_rn(v[e], a.signs[b0 + lane + 32 * e]);
        }
        fwht_block<VPL>(v);
#pragma unroll
        for (int e = 0; e < VPL; e++) {
            s_row[b0 + lane + 32 * e] = v[e];
            am = fmaxf(am, fabsf(v[e]));
        }
    }
    const int E = gemm_act_exponent(block_max(am, red));  // its barriers also publish s_row
    if (tid == 0) a.ex[row] = E;
    gemm_act_words(s_row, row, D, a.G, D / GM_KC, a.nbias, E, 32 * warp, nth, a.bop);
}

void launch_pf_rows(const PfRowArgs& a, int M, int hb, cudaStream_t st) {
    const void* fn = hb == 512 ? (const void*)pf_rows_kernel<16>
                   : hb == 1024 ? (const void*)pf_rows_kernel<32> : (const void*)pf_rows_kernel<64>;
    const size_t smem = (size_t)a.D * 4;
    if (smem > 48 * 1024) raise_smem_limit(fn, 200 * 1024);
    PfRowArgs aa = a;
    void* args[] = {&aa};
    const int nth = 32 * std::min(8, a.D / hb);  // a warp per Hadamard block
    cudaLaunchKernel(fn, dim3(M), dim3(nth), args, smem, st);
}

// Embedding rows of the chunk: the bf16 table's row as is, or the ternary tied table's embed (kernels.metal:230-246,
// the arithmetic of embed_ternary_kernel). One CTA per row.
__global__ void __launch_bounds__(256) pf_embed_kernel(const uint32_t* ids, int V, int d, const uint16_t* bf16,
                                                       const uint32_t* tw, const uint16_t* ts, const uint16_t* tb,
                                                       const float* signs, int group, float* h, int* err) {
    const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint32_t id = ids[row];
    if (id >= (uint32_t)V) {
        if (tid == 0) atomicOr(err, ERR_BAD_TOKEN);
        id = 0;
    }
    if (bf16) {
        for (int k = tid; k < d; k += 256)
            h[(size_t)row * d + k] = __bfloat162float(__ushort_as_bfloat16(bf16[(size_t)id * d + k]));
        return;
    }
    const int kw = d / 16, kg = d / group;
    for (int b0 = warp * 512; b0 < d; b0 += 8 * 512) {
        float v[16];
#pragma unroll
        for (int e = 0; e < 16; e++) {
            const int k = b0 + lane + 32 * e;
            const float c = (float)((tw[(size_t)id * kw + (k >> 4)] >> (2 * (k & 15))) & 3u);
            const float sc = __half2float(__ushort_as_half(ts[(size_t)id * kg + k / group]));
            const float w = tb ? __fadd_rn(__fmul_rn(c, sc), __half2float(__ushort_as_half(tb[(size_t)id * kg + k / group])))
                               : __fmul_rn(c - 1.0f, sc);
            v[e] = __half2float(__float2half_rn(w));
        }
        fwht_block<16>(v);  // the embed's x INV_SQRT512 is the block transform's scale
#pragma unroll
        for (int e = 0; e < 16; e++) {
            const int k = b0 + lane + 32 * e;
            const float sg = signs ? signs[k] : 1.0f;
            h[(size_t)row * d + k] = __half2float(__float2half_rn(__fmul_rn(v[e], sg)));
        }
    }
}

// GDN a/b rows (gdn_ab_row, kernels.metal:265-273): a[t][r] = Wa[r] . xn[t], b[t][r] = Wb[r] . xn[t]. One warp per
// (row, gate row); lane-strided float4 partials, then the warp tree.
__global__ void __launch_bounds__(256) pf_gdn_ab_kernel(const float* wa, const float* wb, const float* xn, float* ga,
                                                        float* gb, int NV, int d, int M) {
    const int t = blockIdx.x, r = blockIdx.y * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (r >= 2 * NV) return;
    const float* wr = r < NV ? wa + (size_t)r * d : wb + (size_t)(r - NV) * d;
    const float* x = xn + (size_t)t * d;
    float acc = 0.0f;
    for (int k = lane * 4; k < d; k += 128) {
        const float4 w4 = *(const float4*)(wr + k), x4 = *(const float4*)(x + k);
        acc += w4.x * x4.x + w4.y * x4.y + w4.z * x4.z + w4.w * x4.w;
    }
    acc = warp_sum(acc);
    if (lane == 0) (r < NV ? ga : gb)[(size_t)t * NV + (r < NV ? r : r - NV)] = acc;
}

// Causal conv (kernel 4) of channel group (128 channels) g at row t over [committed conv rows (3); the chunk's raw
// rows], SiLU, then for q and k heads the per-head RMS norm scaled by 1/128 (q) or 1/sqrt(128) (k) (gdn_conv,
// kernels.metal:515-541). Writes q [M][NK][128], k [M][NK][128], v [M][NV][128].
__global__ void __launch_bounds__(128) pf_gdn_conv_kernel(const float* qkv, int ld, const float* cstate,
                                                          const float* cw, float* q, float* k, float* v, int NK, int NV,
                                                          int C) {
    __shared__ float red[32];
    const int t = blockIdx.x, g = blockIdx.y, c = g * 128 + threadIdx.x;
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int j = t + i;  // row of [state; chunk]
        const float x = j < 3 ? cstate[(size_t)j * C + c] : qkv[(size_t)(j - 3) * ld + c];
        acc = __fmaf_rn(cw[(size_t)c * 4 + i], x, acc);
    }
    float y = acc / (1.0f + expf(-acc));
    if (g < 2 * NK) {
        const float r = rsqrtf(block_sum(y * y, red) / 128.0f + EPS_P);
        y = y * r * (g < NK ? (1.0f / 128.0f) : 0.08838834764831845f);
        float* dst = g < NK ? q : k;
        dst[((size_t)t * NK + (g < NK ? g : g - NK)) * 128 + threadIdx.x] = y;
    } else {
        v[((size_t)t * NV + (g - 2 * NK)) * 128 + threadIdx.x] = y;
    }
}

// New committed conv rows: rows M .. M + 2 of [state; chunk] (conv_state, kernels.metal:544-553). In place.
__global__ void pf_conv_state_kernel(const float* qkv, int ld, float* cstate, int C, int M) {
    const int c = blockIdx.x * 256 + threadIdx.x;
    if (c >= C) return;
    float r[3];
#pragma unroll
    for (int j = 0; j < 3; j++) {
        const int kk = M + j;
        r[j] = kk < 3 ? cstate[(size_t)kk * C + c] : qkv[(size_t)(kk - 3) * ld + c];
    }
#pragma unroll
    for (int j = 0; j < 3; j++) cstate[(size_t)j * C + c] = r[j];
}

// attn_prep (kernels.metal:627-662) for the chunk: row t, head slot hh of (H query heads, KV key heads, KV value
// heads); 256 threads = head dims. Queries: RMSNorm x q_norm, mRoPE, x 1/sqrt(256) into qout [M][H][256]; keys:
// RMSNorm x k_norm, mRoPE, into the cache at position off + t; values: copied into the cache.
__global__ void __launch_bounds__(256) pf_attn_prep_kernel(const float* mix, int ld, const float* qn, const float* kn,
                                                           const float* inv_freq, int rot, int H, int KV, int off,
                                                           float* qout, float* kc, float* vc) {
    __shared__ float red[32];
    __shared__ float buf[256];
    const int t = blockIdx.x, hh = blockIdx.y, d = threadIdx.x;
    const int aw = H * 256, kvw = KV * 256, pos = off + t;
    if (hh >= H + KV) {
        const int kh = hh - H - KV;
        vc[((size_t)pos * KV + kh) * 256 + d] = mix[(size_t)t * ld + 2 * aw + kvw + kh * 256 + d];
        return;
    }
    const bool isq = hh < H;
    const float x = isq ? mix[(size_t)t * ld + hh * 512 + d] : mix[(size_t)t * ld + 2 * aw + (hh - H) * 256 + d];
    const float r = rsqrtf(block_sum(x * x, red) / 256.0f + EPS_P);
    float y = (x * r) * (isq ? qn[d] : kn[d]);
    buf[d] = y;
    __syncthreads();
    const int half = rot / 2;
    if (d < rot) {
        const int f = d < half ? d : d - half;
        float sn, cs;
        sincosf((float)pos * inv_freq[f], &sn, &cs);
        y = d < half ? y * cs - buf[d + half] * sn : y * cs + buf[d - half] * sn;
    }
    if (isq) qout[((size_t)t * H + hh) * 256 + d] = y * 0.0625f;
    else kc[((size_t)pos * KV + (hh - H)) * 256 + d] = y;
}

// LoRA A of a linear over the chunk (norm_rotate's fused A rows, kernels.metal:70-116): u[t][q] = A[q] . xu[t] for
// the R stacked rows of the adapter's group, A fp16 in the device layout [K / HB][R][32 lanes][HB / 32] (element e of
// lane l of block b is input b HB + l + 32 e). One warp per (row, A row): lane l sums its inputs (blocks in order,
// elements in order), then the warp tree.
template <int VPL>
__global__ void __launch_bounds__(256) pf_lora_a_kernel(const uint16_t* A, int R, int K, const float* xu, float* u) {
    const int t = blockIdx.x, q = blockIdx.y * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (q >= R) return;
    constexpr int HB = VPL * 32;
    const float* x = xu + (size_t)t * K;
    float acc = 0.0f;
    for (int b = 0; b < K / HB; b++) {
        const uint4* ap = (const uint4*)(A + (((size_t)b * R + q) * 32 + lane) * VPL);
#pragma unroll
        for (int w8 = 0; w8 < VPL / 8; w8++) {
            const uint4 w = __ldg(ap + w8);
            const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int h = 0; h < 4; h++) {
                const float2 f = __half22float2(*(const __half2*)&ws[h]);
                const int e = 8 * w8 + 2 * h;
                acc = fmaf(f.x, x[b * HB + lane + 32 * e], acc);
                acc = fmaf(f.y, x[b * HB + lane + 32 * (e + 1)], acc);
            }
        }
    }
    acc = warp_sum(acc);
    if (lane == 0) u[(size_t)t * R + q] = acc;
}

// LoRA B (store_post's up projection, kernels.metal:251-262): y[t][o] += B[o] . u[t][member of o], B fp16 [O][r],
// members at rows [0, m1), [m1, m2), [m2, O) with u columns [i r, (i + 1) r). One thread per output.
__global__ void __launch_bounds__(256) pf_lora_b_kernel(const uint16_t* B, int r, int R, int m1, int m2, int O,
                                                        const float* u, float* y) {
    const int t = blockIdx.x, o = blockIdx.y * 256 + threadIdx.x;
    if (o >= O) return;
    const int mem = (o >= m1) + (o >= m2);
    const float* ut = u + (size_t)t * R + mem * r;
    const __half* br = (const __half*)B + (size_t)o * r;
    float a = 0.0f;
    for (int j = 0; j < r; j++) a = fmaf(ut[j], __half2float(br[j]), a);
    y[(size_t)t * O + o] += a;
}

void launch_pf_lora(const uint16_t* A, const uint16_t* B, int R, int r, int m1, int m2, int K, int O, int hb,
                    const float* xu, float* u, float* y, int M, cudaStream_t st) {
    const dim3 ga(M, (R + 7) / 8);
    if (hb == 512) pf_lora_a_kernel<16><<<ga, 256, 0, st>>>(A, R, K, xu, u);
    else pf_lora_a_kernel<32><<<ga, 256, 0, st>>>(A, R, K, xu, u);
    pf_lora_b_kernel<<<dim3(M, (O + 255) / 256), 256, 0, st>>>(B, r, R, m1, m2, O, u, y);
}

void launch_pf_embed(const uint32_t* ids, int M, int V, int d, const uint16_t* bf16, const uint32_t* tw,
                     const uint16_t* ts, const uint16_t* tb, const float* signs, int group, float* h, int* err,
                     cudaStream_t st) {
    pf_embed_kernel<<<M, 256, 0, st>>>(ids, V, d, bf16, tw, ts, tb, signs, group, h, err);
}
void launch_pf_gdn_ab(const float* wa, const float* wb, const float* xn, float* ga, float* gb, int NV, int d, int M,
                      cudaStream_t st) {
    pf_gdn_ab_kernel<<<dim3(M, (2 * NV + 7) / 8), 256, 0, st>>>(wa, wb, xn, ga, gb, NV, d, M);
}
void launch_pf_gdn_conv(const float* qkv, int ld, float* cstate, const float* cw, float* q, float* k, float* v, int NK,
                        int NV, int C, int M, cudaStream_t st) {
    pf_gdn_conv_kernel<<<dim3(M, C / 128), 128, 0, st>>>(qkv, ld, cstate, cw, q, k, v, NK, NV, C);
    pf_conv_state_kernel<<<(C + 255) / 256, 256, 0, st>>>(qkv, ld, cstate, C, M);
}
void launch_pf_attn_prep(const float* mix, int ld, const float* qn, const float* kn, const float* inv_freq, int rot,
                         int H, int KV, int off, int M, float* qout, float* kc, float* vc, cudaStream_t st) {
    pf_attn_prep_kernel<<<dim3(M, H + 2 * KV), 256, 0, st>>>(mix, ld, qn, kn, inv_freq, rot, H, KV, off, qout, kc,
                                                              vc);
}

}  // namespace bcu
