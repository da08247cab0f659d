// mma_tf32.cuh — fp32-accurate warp matrix products on the tensor cores: mma.sync m16n8k8 with tf32 operands, each
// fp32 operand split into hi = tf32(x) and lo = tf32(x - hi) and the product taken as lo.hi + hi.lo + hi.hi (the
// lo.lo term, ~2^-22 relative, is dropped): the error-compensated three-product form of a tf32 contraction. tf32 keeps
// the fp32 exponent, so no range scaling is needed.
//
// Fragments (g = lane / 4, q = lane % 4): A (16 x 8, row-major) a0 = (g, q), a1 = (g + 8, q), a2 = (g, q + 4),
// a3 = (g + 8, q + 4); B (8 x 8, k x n) b0 = (q, g), b1 = (q + 4, g); C (16 x 8) c0 = (g, 2q), c1 = (g, 2q + 1),
// c2 = (g + 8, 2q), c3 = (g + 8, 2q + 1).
#pragma once
#include <stdint.h>

namespace bcu {

__device__ __forceinline__ uint32_t tf32_of(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}

struct Tf32x2 {
    uint32_t hi, lo;
};

__device__ __forceinline__ Tf32x2 tf32_split(float x) {
    Tf32x2 s;
    s.hi = tf32_of(x);
    s.lo = tf32_of(x - __uint_as_float(s.hi));
    return s;
}

__device__ __forceinline__ void mma_tf32(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// c += A B for one 16 x 8 x 8 step from split fragments: small terms first.
__device__ __forceinline__ void mma_tf32x3(float* c, const Tf32x2* a, const Tf32x2* b) {
    mma_tf32(c, a[0].lo, a[1].lo, a[2].lo, a[3].lo, b[0].hi, b[1].hi);
    mma_tf32(c, a[0].hi, a[1].hi, a[2].hi, a[3].hi, b[0].lo, b[1].lo);
    mma_tf32(c, a[0].hi, a[1].hi, a[2].hi, a[3].hi, b[0].hi, b[1].hi);
}

// The same three products into three accumulators (hi.hi, lo.hi, hi.lo), each its own dependency chain; the result
// is (c[1] + c[2]) + c[0] (mma3_sum). For warps that are short of independent work.
struct Acc3 {
    float c[3][4];
};
__device__ __forceinline__ void acc3_zero(Acc3& r) {
#pragma unroll
    for (int j = 0; j < 3; j++) r.c[j][0] = r.c[j][1] = r.c[j][2] = r.c[j][3] = 0.0f;
}
__device__ __forceinline__ void mma_tf32x3_acc(Acc3& r, const Tf32x2* a, const Tf32x2* b) {
    mma_tf32(r.c[1], a[0].lo, a[1].lo, a[2].lo, a[3].lo, b[0].hi, b[1].hi);
    mma_tf32(r.c[2], a[0].hi, a[1].hi, a[2].hi, a[3].hi, b[0].lo, b[1].lo);
    mma_tf32(r.c[0], a[0].hi, a[1].hi, a[2].hi, a[3].hi, b[0].hi, b[1].hi);
}
__device__ __forceinline__ float mma3_sum(const Acc3& r, int e) { return (r.c[1][e] + r.c[2][e]) + r.c[0][e]; }

// A fragment of rows m0.. and columns k0.. of a row-major fp32 matrix in shared memory (row stride ld floats).
__device__ __forceinline__ void frag_a_rows(const float* m, int ld, int m0, int k0, Tf32x2* a) {
    const int g = (threadIdx.x & 31) >> 2, q = threadIdx.x & 3;
    a[0] = tf32_split(m[(m0 + g) * ld + k0 + q]);
    a[1] = tf32_split(m[(m0 + g + 8) * ld + k0 + q]);
    a[2] = tf32_split(m[(m0 + g) * ld + k0 + q + 4]);
    a[3] = tf32_split(m[(m0 + g + 8) * ld + k0 + q + 4]);
}
// A fragment whose element (m, k) is stored at mt[k * ld + m] (the transpose is in memory), scaled by w[k].
__device__ __forceinline__ void frag_a_cols(const float* mt, int ld, int m0, int k0, const float* w, Tf32x2* a) {
    const int g = (threadIdx.x & 31) >> 2, q = threadIdx.x & 3;
    const float w0 = w[k0 + q], w1 = w[k0 + q + 4];
    a[0] = tf32_split(w0 * mt[(k0 + q) * ld + m0 + g]);
    a[1] = tf32_split(w0 * mt[(k0 + q) * ld + m0 + g + 8]);
    a[2] = tf32_split(w1 * mt[(k0 + q + 4) * ld + m0 + g]);
    a[3] = tf32_split(w1 * mt[(k0 + q + 4) * ld + m0 + g + 8]);
}
// B fragment whose element (k, n) is stored at bk[k * ld + n] (k-major rows).
__device__ __forceinline__ void frag_b_krows(const float* bk, int ld, int k0, int n0, Tf32x2* b) {
    const int g = (threadIdx.x & 31) >> 2, q = threadIdx.x & 3;
    b[0] = tf32_split(bk[(k0 + q) * ld + n0 + g]);
    b[1] = tf32_split(bk[(k0 + q + 4) * ld + n0 + g]);
}
// B fragment whose element (k, n) is stored at bn[n * ld + k] (n-major rows, e.g. B = M^T of a row-major M).
__device__ __forceinline__ void frag_b_nrows(const float* bn, int ld, int k0, int n0, Tf32x2* b) {
    const int g = (threadIdx.x & 31) >> 2, q = threadIdx.x & 3;
    b[0] = tf32_split(bn[(n0 + g) * ld + k0 + q]);
    b[1] = tf32_split(bn[(n0 + g) * ld + k0 + q + 4]);
}

}  // namespace bcu
