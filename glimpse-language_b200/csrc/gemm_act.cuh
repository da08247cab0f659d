// gemm_act.cuh — the prefill GEMM's activation tiles (the B operand of ternary_gemm_kernel), written by
// gemm_prep_kernel (gemm.cu) from fp32 rows, or directly by the prefill producers (pf_rows_kernel, prefill.cu), which
// hold a whole rotated row in shared memory. Both call the functions below, so the tiles are bit-identical.
//
// Layout: per 128-token tile tt and 64-input chunk c a 32-KB block of 256 rows x 64 fp16 with the 128-byte swizzle
// (rows 0..127 the tokens' hi parts, 128..255 their lo parts), main chunks c < nmain = K / 64 then the bias chunks
// (group sums, one input per group). A token's values are x 2^E = hi + lo with E = clamp(14 - frexp exponent of
// max |x|), so every product with a fp16 weight is exact and the sums fp32.
#pragma once
#include "common.cuh"
#include "operand.cuh"  // pow2f

namespace bcu {

constexpr int GM_TOK = 128, GM_KC = 64;                // tile tokens, inputs per chunk
constexpr int GM_B_BYTES = 2 * GM_TOK * GM_KC * 2;     // 32 KB activations (hi and lo) per (tile, chunk)

// Operand tiles in shared memory: K-major with the 128-byte swizzle. A row of a tile is one chunk of 64 fp16 inputs
// (128 bytes); rows are contiguous; 16-byte piece j of row r sits at r * 128 + ((j ^ (r % 8)) * 16), so 8 rows form a
// 1024-byte swizzle atom (tiles start on 1024-byte boundaries).
__host__ __device__ inline int sw128(int r, int j) { return r * 128 + ((j ^ (r & 7)) << 4); }

// Order of the inputs inside a chunk: the weight decode takes two codes of one packed word per LOP3, codes i and i + 8
// (i < 8) of word w (inputs 16 w + i, 16 w + i + 8), so half p of 16-byte piece kk of a chunk row holds input
// 16 (kk / 2) + 4 (kk % 2) + p / 2 + 8 (p % 2). The activations use the same order (any order of the inputs gives
// the same dot products, as long as A and B agree).
__host__ __device__ inline int gemm_k_of(int kk, int p) { return 16 * (kk >> 1) + 4 * (kk & 1) + (p >> 1) + 8 * (p & 1); }

// The token's exponent from the maximum magnitude of its row.
__device__ __forceinline__ int gemm_act_exponent(float am) {
    int E = 0;
    if (am > 0.0f && am < INFINITY) {
        int e2;
        frexpf(am, &e2);
        E = min(max(14 - e2, -60), 100);
    }
    return E;
}

// Token t's tiles from its K values at row (global or shared memory), packed words w0 + lane for w0 = wbeg,
// wbeg + wstride, ... (wbeg and wstride multiples of 32, the same for the warp's lanes): inputs 16 w .. 16 w + 15,
// two 16-byte pieces of the hi and lo rows each, then the group sums x 2^(E - log2 G) (hi + lo) to the bias chunks
// (the G / 16 consecutive lanes of one group summed in a fixed tree).
__device__ __forceinline__ void gemm_act_words(const float* row, int t, int K, int G, int nmain, int nbias, int E,
                                               int wbeg, int wstride, uint8_t* bop) {
    const int lane = threadIdx.x & 31;
    const float f = E > 60 ? pow2f(60) * pow2f(E - 60) : (E < -60 ? pow2f(-60) * pow2f(E + 60) : pow2f(E));
    const int nch = nmain + nbias, tt = t / GM_TOK, tl = t % GM_TOK;
    uint8_t* tile0 = bop + (size_t)tt * nch * GM_B_BYTES;
    const int n_hi = tl, n_lo = GM_TOK + tl;  // rows of the B tile
    const int lg = G == 64 ? 6 : 7, lanes_per_group = G / 16;
    const float fb = pow2f(E - lg > 100 ? 100 : E - lg);
    for (int w0 = wbeg; w0 < K / 16; w0 += wstride) {
        const int w = w0 + lane;  // inputs 16 w .. 16 w + 15
        float gs = 0.0f;
        if (w < K / 16) {
            float v[16];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float4 a = *(const float4*)(row + 16 * w + 4 * i);
                v[4 * i] = a.x;
                v[4 * i + 1] = a.y;
                v[4 * i + 2] = a.z;
                v[4 * i + 3] = a.w;
            }
#pragma unroll
            for (int e = 0; e < 16; e++) gs += v[e];
            uint8_t* chunk = tile0 + (size_t)(w / 4) * GM_B_BYTES;
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int kk = 2 * (w % 4) + h;
                uint16_t hv[8], lv[8];
#pragma unroll
                for (int p = 0; p < 8; p++) {
                    const float s = v[4 * h + (p >> 1) + 8 * (p & 1)] * f;
                    const __half hh = __float2half_rn(s);
                    hv[p] = __half_as_ushort(hh);
                    lv[p] = __half_as_ushort(__float2half_rn(s - __half2float(hh)));
                }
                *(uint4*)(chunk + sw128(n_hi, kk)) = *(const uint4*)hv;
                *(uint4*)(chunk + sw128(n_lo, kk)) = *(const uint4*)lv;
            }
        }
        for (int o = 1; o < lanes_per_group; o <<= 1) gs += __shfl_xor_sync(0xffffffffu, gs, o);
        if (w < K / 16 && (lane % lanes_per_group) == 0) {
            const int g = w / lanes_per_group;
            const float s = gs * fb;
            const __half hh = __float2half_rn(s);
            const __half ll = __float2half_rn(s - __half2float(hh));
            uint8_t* chunk = tile0 + (size_t)(nmain + g / GM_KC) * GM_B_BYTES;
            const int kk = (g % GM_KC) / 8;
            ((__half*)(chunk + sw128(n_hi, kk)))[g % 8] = hh;
            ((__half*)(chunk + sw128(n_lo, kk)))[g % 8] = ll;
        }
    }
}

}  // namespace bcu
