// operand.cuh — the activation operand of the ternary GEMV in tensor-core fragment order, and the device code that
// writes it (used by the GEMV's operand builders in ternary.cu: RMSNorm, gated RMSNorm, SwiGLU and sigmoid-gate
// inputs, then signs, Walsh-Hadamard transform, exponent, fp16 hi/lo split and group sums).
//
// Layout: one region per (block b of HB consecutive inputs, column tile nt of 4 tokens). A region is sb/16 main k16
// steps of B fragments (256 B each: 4 tokens x fp16 hi, lo columns; word (c * 4 + t4) * 2 + which of a step holds
// rows k = 2 t4 + 8 which + {0, 1} of column c), then the block's bias k16 steps (row k = group within the block),
// then the power-of-two exponents of its 4 tokens (16 B). Values are x * 2^E * 4^-j (j = (k % 32) / 8, the decode's
// scale of code pair j) split into hi + lo; the bias step holds the group sums of x * 2^(E - 6).
#pragma once
#include "common.cuh"
#include "kernels.h"

namespace bcu {

constexpr float EPS_OP = 1e-6f;

__device__ __forceinline__ float sigm(float z) { return 1.0f / (1.0f + expf(-z)); }
__device__ __forceinline__ float pow2f(int e) { return __int_as_float((127 + e) << 23); }  // |e| <= 126

__host__ __device__ inline int op_bias_steps(int sb, int group) { return (sb / group + 15) / 16; }
__host__ __device__ inline int op_region_bytes(int sb, int group) { return (sb / 16 + op_bias_steps(sb, group)) * 256 + 16; }

// The part of a Hadamard block that a region holds: elements e in [e_lo, e_hi) of the lane layout below, at
// region-relative k = kr0 + lane + 32 e; sbsz = the region's k extent.
struct OpGeo {
    int sbsz, e_lo, e_hi, kr0;
    bool rotate;  // false: the input is already rotated
};

// Token t's columns of its region when t >= T: zeros (per k16 step the columns col, col + 1 are the 16 words
// [8 col, 8 col + 16)).
__device__ __forceinline__ void zero_token(int t, int sbsz, int group, uint8_t* reg) {
    const int lane = threadIdx.x & 31;
    const int nsteps = sbsz / 16, nbs = op_bias_steps(sbsz, group);
    uint32_t* rw = (uint32_t*)reg;
    const int col = (t & 3) * 2;
    for (int i = lane; i < (nsteps + nbs) * 16; i += 32) rw[(i >> 4) * 64 + col * 8 + (i & 15)] = 0u;
    if (lane == 0) ((int*)(reg + (nsteps + nbs) * 256))[t & 3] = 0;
}

// Writes token t's columns of `reg` from its values v of one Hadamard block (lane l holds element l + 32 e,
// e < VPL = HB / 32, the layout of fwht512, kernels.metal:32-51, so the transform's strides 1..16 run across lanes and
// 32.. inside the lane, in ascending order: bit-identical to an in-memory radix-2 transform). sg: the block's signs
// in the same layout, or null. One warp.
template <int VPL, int GPC>
__device__ void emit_token(const OpGeo& geo, int t, uint8_t* reg, float* v, const float* sg) {
    constexpr int G = 128 / GPC, EPG = G / 32, NGH = VPL * 32 / G;
    const int lane = threadIdx.x & 31;
    const int nsteps = geo.sbsz / 16, nbs = op_bias_steps(geo.sbsz, G);
    const int e_lo = geo.e_lo, e_hi = geo.e_hi, kr0 = geo.kr0;
    uint32_t* rw = (uint32_t*)reg;
    int* r_e = (int*)(reg + (nsteps + nbs) * 256);
    const int col = (t & 3) * 2;  // hi column of the token in its tile; lo = col + 1
    if (sg) {
#pragma unroll
        for (int e = 0; e < VPL; e++) v[e] *= sg[e];
    }
    if (geo.rotate) {
#pragma unroll
        for (int m = 1; m < 32; m <<= 1) {
            const float sgn = (lane & m) ? -1.0f : 1.0f;
#pragma unroll
            for (int e = 0; e < VPL; e++) {
                const float o = __shfl_xor_sync(0xffffffffu, v[e], m);
                v[e] = fmaf(v[e], sgn, o);  // lower lane: v + o, upper lane: o - v
            }
        }
#pragma unroll
        for (int h = 1; h < VPL; h <<= 1)
#pragma unroll
            for (int e = 0; e < VPL; e++)
                if ((e & h) == 0) {
                    const float a = v[e], c = v[e + h];
                    v[e] = a + c;
                    v[e + h] = a - c;
                }
        const float inv = VPL == 16 ? 0.044194173824159216f : (VPL == 64 ? 0.02209708691207961f : 0.03125f);
#pragma unroll
        for (int e = 0; e < VPL; e++) v[e] *= inv;
    }
    float am[VPL];  // |v| over the region's part, reduced as a tree
#pragma unroll
    for (int e = 0; e < VPL; e++) am[e] = (e >= e_lo && e < e_hi) ? fabsf(v[e]) : 0.0f;
#pragma unroll
    for (int h = VPL / 2; h > 0; h >>= 1)
#pragma unroll
        for (int e = 0; e < h; e++) am[e] = fmaxf(am[e], am[e + h]);
    const float amax = warp_max(am[0]);
    int E = 0;
    if (amax > 0.0f && amax < INFINITY) {
        int ex;
        frexpf(amax, &ex);  // amax < 2^ex
        E = min(max(14 - ex, -60), 100);
    }
    if (lane == 0) r_e[t & 3] = E;
    // x * 2^E * 4^-j in fp16 hi + lo, j = (k % 32) / 8 = lane / 8; each lane stores its element's two halves
    {
        const int j = lane >> 3;
        const int t4 = (lane & 7) >> 1, which = (lane & 15) >> 3;
        const int E1 = E - 2 * j;
        const float f = E1 > 60 ? pow2f(60) * pow2f(E1 - 60) : (E1 < -60 ? pow2f(-60) * pow2f(E1 + 60) : pow2f(E1));
        uint16_t* r16 = (uint16_t*)reg;
        const int h_hi = ((col * 4 + t4) * 2 + which) * 2 + (lane & 1), h_lo = h_hi + 16;
        const int step0 = (kr0 >> 4) + (lane >> 4);
#pragma unroll
        for (int e = 0; e < VPL; e++) {
            if (e >= e_lo && e < e_hi) {
                const float a = v[e] * f;
                const __half h = __float2half_rn(a);
                const __half l = __float2half_rn(a - __half2float(h));
                r16[(step0 + 2 * e) * 128 + h_hi] = __half_as_ushort(h);
                r16[(step0 + 2 * e) * 128 + h_lo] = __half_as_ushort(l);
            }
        }
    }
    // group sums of the block's part for the bias steps (x 2^(E-6)); all lanes hold every sum after the reduction
    float gs[NGH];
#pragma unroll
    for (int g = 0; g < NGH; g++) {
        float a = 0.0f;
#pragma unroll
        for (int e = g * EPG; e < (g + 1) * EPG; e++) a += v[e];
        gs[g] = a;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int g = 0; g < NGH; g++) gs[g] += __shfl_xor_sync(0xffffffffu, gs[g], o);
    if (lane < 16) {
        // lane -> column col + lane / 8, word (t4, which) of the bias step: k rows kk0, kk0 + 1
        const int hl = lane >> 3, t4 = (lane >> 1) & 3, wh = lane & 1;
        const int kk0 = wh * 8 + t4 * 2;
        const int g_lo = e_lo / EPG, ngs = (e_hi - e_lo) / EPG;
        const float fb = pow2f(E - 6 > 100 ? 100 : E - 6);
        for (int bs = 0; bs < nbs; bs++) {
            float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
            for (int g = 0; g < NGH; g++) {
                const int gr = g - g_lo;  // block-relative group
                if (gr >= 0 && gr < ngs) {
                    if (gr == bs * 16 + kk0) s0 = gs[g];
                    if (gr == bs * 16 + kk0 + 1) s1 = gs[g];
                }
            }
            const float a0 = s0 * fb, a1 = s1 * fb;
            __half h0 = __float2half_rn(a0), h1 = __float2half_rn(a1);
            if (hl) {
                h0 = __float2half_rn(a0 - __half2float(h0));
                h1 = __float2half_rn(a1 - __half2float(h1));
            }
            rw[(nsteps + bs) * 64 + ((col + hl) * 4 + t4) * 2 + wh] = pack_half2(h0, h1);
        }
    }
}

// Gated RMSNorm of GDN outputs (gated_norm_rotate, kernels.metal:199-226) for one token's block: y values a, gate z
// values b (lane layout above), head-norm weights wn[i] at (lane + 32 i) & 127. A head is 128 = 4 e-values.
template <int VPL>
__device__ __forceinline__ void gated_values(const float* a, const float* b, const float* wn, float* v) {
#pragma unroll
    for (int c = 0; c < VPL / 4; c++) {
        float ss = 0.0f;
#pragma unroll
        for (int e = 4 * c; e < 4 * c + 4; e++) ss += a[e] * a[e];
        const float rh = rsqrtf(warp_sum(ss) / 128.0f + EPS_OP);
#pragma unroll
        for (int e = 4 * c; e < 4 * c + 4; e++) v[e] = (((b[e] * a[e]) * rh) * wn[e & 3]) * sigm(b[e]);
    }
}

// Copies token t's columns of a region built in shared memory (`reg`) to the same region in global memory: per k16
// step the 16 words [8 col, 8 col + 16), then the token's exponent. One warp; 16-byte stores.
__device__ __forceinline__ void store_token_columns(int t, int sbsz, int group, const uint8_t* reg, uint8_t* dst) {
    const int lane = threadIdx.x & 31;
    const int nsteps = sbsz / 16, nbs = op_bias_steps(sbsz, group);
    const int col = (t & 3) * 2;
    for (int i = lane; i < (nsteps + nbs) * 4; i += 32) {
        const int st = i >> 2, q = i & 3;
        const size_t off = (size_t)st * 256 + col * 32 + q * 16;
        *(uint4*)(dst + off) = *(const uint4*)(reg + off);
    }
    if (lane == 0) ((int*)(dst + (nsteps + nbs) * 256))[t & 3] = ((const int*)(reg + (nsteps + nbs) * 256))[t & 3];
}

}  // namespace bcu
