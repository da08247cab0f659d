// act.cuh — block-level producers of the GEMV activation operands: Hadamard rotation of a row held in shared memory
// and its conversion into tensor-core B fragments. One CTA owns one token row; all threads call these.
#pragma once
#include "common.cuh"
#include "kernels.h"

namespace bcu {

// INV_SQRT512 of kernels.metal:8; other blocks 1/sqrt(HB) rounded once from double.
__host__ __device__ inline float hadamard_inv(int HB) {
    return HB == 512 ? 0.044194173824159216f : (HB == 2048 ? 0.02209708691207961f : (HB == 1024 ? 0.03125f : 0.0625f));
}

// In-place x = fwht_blocks(signs * x) * inv(HB) over D values in shared memory (D % HB == 0, HB in {512, 1024,
// 2048}). The 512-point part runs in registers exactly as fwht512 of kernels.metal:32-51 (lane l holds elements
// l + 32e; strides 1..16 across lanes, then 32..256 in the lane), the stages above 512 in shared memory; stage order
// ascending, add/sub only, so the result is bit-identical to an in-memory radix-2 transform.
__device__ inline void block_rotate(float* x, int D, int HB, const float* signs) {
    int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int b0 = w * 512; b0 < D; b0 += nw * 512) {
        float v[16];
#pragma unroll
        for (int e = 0; e < 16; e++) {
            int i = b0 + lane + 32 * e;
            v[e] = signs ? x[i] * signs[i] : x[i];
        }
#pragma unroll
        for (int m = 1; m < 32; m <<= 1) {
            bool up = (lane & m) != 0;
#pragma unroll
            for (int e = 0; e < 16; e++) {
                float o = __shfl_xor_sync(0xffffffffu, v[e], m);
                v[e] = up ? o - v[e] : v[e] + o;
            }
        }
#pragma unroll
        for (int h = 1; h < 16; h <<= 1)
#pragma unroll
            for (int e = 0; e < 16; e++)
                if ((e & h) == 0) {
                    float a = v[e], b = v[e + h];
                    v[e] = a + b;
                    v[e + h] = a - b;
                }
#pragma unroll
        for (int e = 0; e < 16; e++) x[b0 + lane + 32 * e] = v[e];
    }
    __syncthreads();
    for (int h = 512; h < HB; h <<= 1) {
        for (int p = threadIdx.x; p < D / 2; p += blockDim.x) {
            int i = (p / h) * 2 * h + (p % h);
            float a = x[i], b = x[i + h];
            x[i] = a + b;
            x[i + h] = a - b;
        }
        __syncthreads();
    }
    float inv = hadamard_inv(HB);
    for (int i = threadIdx.x; i < D; i += blockDim.x) x[i] *= inv;
    __syncthreads();
}

// Writes token row t (x[0..K) in shared memory; zeros when t >= T) of the ternary GEMV activation operand (layout in
// kernels.h): e_t = 14 - ceil-exponent(max|x|) so every hi part fits fp16, then per k the hi/lo fp16 split of
// x * 2^e_t * 4^-((k%32)/8), placed where mma.m16n8k16 expects B (k = 2t4 + {0,1} (+8), column g).
// Also the group sums of the unscaled x for the bias term. red: >= 32 floats of shared memory.
__device__ inline void write_ternary_act(const float* x, int K, int t, int T, int NT, int group, const TernaryAct& act,
                                         float* red) {
    bool live = t < T;
    float amax = 0.0f;
    if (live)
        for (int i = threadIdx.x; i < K; i += blockDim.x) amax = fmaxf(amax, fabsf(x[i]));
    amax = block_max(amax, red);
    int e = 0;
    if (amax > 0.0f && amax < INFINITY) {
        int E;
        frexpf(amax, &E);  // amax < 2^E
        e = min(max(14 - E, -60), 100);
    }
    int nt = t >> 2, gbase = (t & 3) * 2;
    for (int p = threadIdx.x; p < K / 2; p += blockDim.x) {
        int k = 2 * p;
        uint32_t hi = 0, lo = 0;
        if (live) {
            int j = (k & 31) >> 3;
            float f = ldexpf(1.0f, e - 2 * j);
            float v0 = x[k] * f, v1 = x[k + 1] * f;
            __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
            __half l0 = __float2half_rn(v0 - __half2float(h0)), l1 = __float2half_rn(v1 - __half2float(h1));
            hi = pack_half2(h0, h1);
            lo = pack_half2(l0, l1);
        }
        int s = k >> 4, kk = k & 15, which = kk >> 3, t4 = (kk & 7) >> 1;
        size_t base = ((size_t)s * NT + nt) * 32;
        act.bfrag[(base + gbase * 4 + t4) * 2 + which] = hi;
        act.bfrag[(base + (gbase + 1) * 4 + t4) * 2 + which] = lo;
    }
    int ng = K / group;
    for (int gi = threadIdx.x; gi < ng; gi += blockDim.x) {
        float s = 0.0f;
        if (live)
            for (int i = 0; i < group; i++) s += x[gi * group + i];
        act.xsum[(size_t)t * ng + gi] = s;
    }
    if (threadIdx.x == 0) act.xexp[t] = e;
}

// bf16 operand of the head GEMV: hi = bf16(x), lo = bf16(x - hi) (16 significant bits), same fragment placement.
__device__ inline void write_bf16_act(const float* x, int K, int t, int T, int NT, uint32_t* bfrag) {
    bool live = t < T;
    int nt = t >> 2, gbase = (t & 3) * 2;
    for (int p = threadIdx.x; p < K / 2; p += blockDim.x) {
        int k = 2 * p;
        uint32_t hi = 0, lo = 0;
        if (live) {
            float v0 = x[k], v1 = x[k + 1];
            __nv_bfloat16 h0 = __float2bfloat16_rn(v0), h1 = __float2bfloat16_rn(v1);
            __nv_bfloat16 l0 = __float2bfloat16_rn(v0 - __bfloat162float(h0));
            __nv_bfloat16 l1 = __float2bfloat16_rn(v1 - __bfloat162float(h1));
            hi = pack_bf162(h0, h1);
            lo = pack_bf162(l0, l1);
        }
        int s = k >> 4, kk = k & 15, which = kk >> 3, t4 = (kk & 7) >> 1;
        size_t base = ((size_t)s * NT + nt) * 32;
        bfrag[(base + gbase * 4 + t4) * 2 + which] = hi;
        bfrag[(base + (gbase + 1) * 4 + t4) * 2 + which] = lo;
    }
}

}  // namespace bcu
