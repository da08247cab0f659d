// ternary.cu — tensor-core ternary verify GEMV for T <= 16 rows (the reference's qmvxm / qmvx / qmv_cm / qmvr / qmv4,
// kernels.metal:275-404 and 664-709, kernels/qmvx.comp, kernels/qmv_cm.comp), plus the weight repack and the
// standalone rotate-then-linear op of graded config 1.
//
// Why tensor cores at batch 1: a T = 9 verify does 9 multiply-adds per 2-bit weight. At the HBM rate of ~21 T
// weights/s that is ~190 T FMA/s, five times what the CUDA cores can issue, so the products go to mma.m16n8k16 and
// the CUDA cores only decode: per pair of weights one LOP3 ((w & mask) | 0x6400 gives fp16 1024 + c*4^j) and one
// HFMA2 (x s, - 1024 s gives exactly c*s*4^j). The activation operand carries 4^-j and a per-row power-of-two scale
// and is split into fp16 hi + lo columns, so products are exact and the sum is fp32-accurate; the bias term
// sum_g b_g * sum_k x_k is added in fp32 from the producer's group sums. Every output's reduction order is fixed
// and independent of T, so a row's result is bit-identical whether it is verified alone or among 9 rows.
//
// CTA = 128 rows x kslice codes (8 warps = 2 row groups of 64 x 4 k-quarters). One thread streams the CTA's codes
// and scales into shared memory with cp.async.bulk before waiting on the previous kernel (PDL), then the
// activation tile. Split-K partials are summed in a fixed order by the last CTA of each row block.
#include <cstdio>
#include "act.cuh"
#include "common.cuh"
#include "kernels.h"

namespace bcu {

cudaError_t launch_pdl(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t st, void** args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

size_t ternary_codes_bytes(int O, int K) { return (size_t)O * K / 4; }
size_t ternary_scales_bytes(int O, int K, int group) { return (size_t)O * (K / group) * 2; }

// ------------------------------------------------------------------------------------------------ repack
// One thread per output code word.
__global__ void repack_codes_kernel(const uint32_t* __restrict__ w, int O, int K, uint32_t* __restrict__ out) {
    size_t n = (size_t)O * K / 16;
    size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= n) return;
    int q = idx & 3;
    int lane = (idx >> 2) & 31;
    size_t tile = idx >> 7;  // (rb * nkc + kc) * 8 + mt
    int mt = tile & 7;
    size_t rk = tile >> 3;
    int nkc = K / 128;
    int kc = rk % nkc;
    int rb = rk / nkc;
    int g = lane >> 2, t4 = lane & 3;
    uint32_t word = 0;
#pragma unroll
    for (int h = 0; h < 8; h++) {
        int rowhalf = h >> 2, f = (h & 3) >> 1, hs = h & 1;
        int row = rb * 128 + mt * 16 + g + 8 * rowhalf;
#pragma unroll
        for (int e = 0; e < 2; e++) {
            int k = kc * 128 + 32 * q + 16 * f + 8 * hs + 2 * t4 + e;
            uint32_t c = (w[(size_t)row * (K / 16) + k / 16] >> (2 * (k & 15))) & 3u;
            word |= c << (2 * h + 16 * e);
        }
    }
    out[idx] = word;
}

__global__ void repack_scales_kernel(const uint16_t* __restrict__ s, const uint16_t* __restrict__ b, int O, int K,
                                     int group, uint32_t* __restrict__ out, uint16_t* __restrict__ bias) {
    int gpc = 128 / group, ng = K / group;
    size_t n = (size_t)(O / 16) * (K / 128) * gpc * 8;  // entries
    size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx < n) {
        int g = idx & 7;
        size_t r = idx >> 3;
        int gi = r % gpc;
        r /= gpc;
        int mt = r & 7;
        size_t rk = r >> 3;
        int nkc = K / 128;
        int kc = rk % nkc;
        int rb = rk / nkc;
        int row = rb * 128 + mt * 16 + g;
        int grp = kc * gpc + gi;
        out[idx] = (uint32_t)s[(size_t)row * ng + grp] | ((uint32_t)s[(size_t)(row + 8) * ng + grp] << 16);
    }
    size_t nb = (size_t)O * ng;
    for (size_t i = idx; i < nb; i += (size_t)gridDim.x * blockDim.x)
        bias[i] = b ? b[i] : (uint16_t)(s[i] ^ 0x8000u);
}

void repack_ternary(const uint32_t* w_mlx, const uint16_t* s, const uint16_t* b, int O, int K, int group,
                    void* codes, uint32_t* scales, uint16_t* bias, cudaStream_t st) {
    size_t n = (size_t)O * K / 16;
    repack_codes_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(w_mlx, O, K, (uint32_t*)codes);
    size_t ns = (size_t)(O / 16) * (K / 128) * (128 / group) * 8;
    size_t nb = (size_t)O * (K / group);
    size_t nmax = ns > nb ? ns : nb;
    repack_scales_kernel<<<(unsigned)((nmax + 255) / 256), 256, 0, st>>>(s, b, O, K, group, scales, bias);
}

// Split-K plan: the fewest K-slices (multiples of 512 codes, at most 2048 so the CTA's tiles stay under 200 KB of
// shared memory at NT = 4) that give at least one CTA per SM.
void plan_ternary(TernaryMat& m, int num_sms) {
    int rb = m.O / 128;
    int best = 0;
    for (int ns = 1; ns <= m.K / 512; ns++) {
        if (m.K % (ns * 512) != 0) continue;
        if (m.K / ns > 2048) continue;
        best = ns;
        if (rb * ns >= num_sms) break;
    }
    if (best == 0) best = m.K / 512;  // K/ns <= 2048 always holds for ns = K/512
    m.nsplit = best;
    m.kslice = m.K / best;
}

// ------------------------------------------------------------------------------------------------ GEMV
struct GemvParams {
    const uint4* codes;
    const uint32_t* scales;
    const uint16_t* bias;
    const uint32_t* bfrag;
    const float* xsum;
    const int* xexp;
    float* out;
    float* partial;
    unsigned* counters;
    int* err;
    int O, K, group, kslice, nsplit, T, add;
};

template <int NT, int GPC>
__global__ void __launch_bounds__(256) ternary_gemv_kernel(GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* bar = (uint64_t*)smem;
    const int kslice = p.kslice, nkc = kslice / 128;
    uint4* s_codes = (uint4*)(smem + 128);
    uint32_t* s_scales = (uint32_t*)(smem + 128 + (size_t)kslice * 32);
    const size_t scales_bytes = (size_t)nkc * 8 * GPC * 32;
    uint2* s_b = (uint2*)(smem + 128 + (size_t)kslice * 32 + scales_bytes);
    const size_t b_bytes = (size_t)(kslice / 16) * NT * 256;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int rb = blockIdx.x / p.nsplit, ks = blockIdx.x % p.nsplit;
    const int nkc_all = p.K / 128;

    if (tid == 0) {
        mbar_init(bar, 1);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    __syncthreads();
    pdl_trigger();
    if (tid == 0) {
        mbar_expect_tx(bar, (uint32_t)((size_t)kslice * 32 + scales_bytes + b_bytes));
        const uint8_t* gcodes = (const uint8_t*)p.codes + ((size_t)rb * nkc_all + (size_t)ks * nkc) * 8 * 512;
        bulk_g2s(s_codes, gcodes, (uint32_t)(kslice * 32), bar);
        const uint8_t* gsc = (const uint8_t*)p.scales + ((size_t)rb * nkc_all + (size_t)ks * nkc) * 8 * GPC * 32;
        bulk_g2s(s_scales, gsc, (uint32_t)scales_bytes, bar);
    }
    pdl_wait();
    if (tid == 0) {
        const uint8_t* gb = (const uint8_t*)p.bfrag + (size_t)ks * (kslice / 16) * NT * 256;
        bulk_g2s(s_b, gb, (uint32_t)b_bytes, bar);
    }
    bool ok = mbar_wait_bounded(bar, 0);
    if (__syncthreads_or(!ok)) {
        if (tid == 0) atomicOr(p.err, ERR_MBAR_TIMEOUT);
        // the copies may still land; wait (bounded) so none writes to shared memory after exit
        mbar_wait_bounded(bar, 0, 1u << 20);
        return;
    }

    const int rg = warp >> 2, kw = warp & 3;
    const int g = lane >> 2;
    const int nkc_w = nkc / 4;
    float acc[4][NT][4];
#pragma unroll
    for (int m = 0; m < 4; m++)
#pragma unroll
        for (int n = 0; n < NT; n++)
#pragma unroll
            for (int i = 0; i < 4; i++) acc[m][n][i] = 0.0f;

    const uint32_t MAGIC = 0x64006400u, NEG1024 = 0xE400E400u;
    for (int c = 0; c < nkc_w; c++) {
        const int kcl = kw * nkc_w + c;
        uint4 cw[4];
#pragma unroll
        for (int m = 0; m < 4; m++) cw[m] = s_codes[(size_t)(kcl * 8 + rg * 4 + m) * 32 + lane];
#pragma unroll
        for (int gi = 0; gi < GPC; gi++) {
            uint32_t s2lo[4], s2hi[4], n2lo[4], n2hi[4];
#pragma unroll
            for (int m = 0; m < 4; m++) {
                uint32_t u = s_scales[((size_t)(kcl * 8 + rg * 4 + m) * GPC + gi) * 8 + g];
                s2lo[m] = __byte_perm(u, 0, 0x1010);
                s2hi[m] = __byte_perm(u, 0, 0x3232);
                asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(n2lo[m]) : "r"(s2lo[m]), "r"(NEG1024));
                asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(n2hi[m]) : "r"(s2hi[m]), "r"(NEG1024));
            }
            constexpr int SPG = 8 / GPC;  // k16 steps per group
#pragma unroll
            for (int fs = 0; fs < SPG; fs++) {
                const int f = gi * SPG + fs;  // k16 step within the chunk (0..7)
                const int q = f >> 1;
                const bool odd = f & 1;
                uint2 bb[NT];
#pragma unroll
                for (int n = 0; n < NT; n++) bb[n] = s_b[((size_t)(kcl * 8 + f) * NT + n) * 32 + lane];
                const uint32_t mask_a = odd ? 0x00300030u : 0x00030003u;
                const uint32_t mask_b = odd ? 0x00C000C0u : 0x000C000Cu;
#pragma unroll
                for (int m = 0; m < 4; m++) {
                    uint32_t w = q == 0 ? cw[m].x : (q == 1 ? cw[m].y : (q == 2 ? cw[m].z : cw[m].w));
                    uint32_t w8 = w >> 8;
                    uint32_t a0 = hfma2_u32(lop_and_or(w, mask_a, MAGIC), s2lo[m], n2lo[m]);
                    uint32_t a1 = hfma2_u32(lop_and_or(w8, mask_a, MAGIC), s2hi[m], n2hi[m]);
                    uint32_t a2 = hfma2_u32(lop_and_or(w, mask_b, MAGIC), s2lo[m], n2lo[m]);
                    uint32_t a3 = hfma2_u32(lop_and_or(w8, mask_b, MAGIC), s2hi[m], n2hi[m]);
#pragma unroll
                    for (int n = 0; n < NT; n++) mma_f16(acc[m][n], a0, a1, a2, a3, bb[n].x, bb[n].y);
                }
            }
        }
    }

    // in-CTA reduction over the 4 k-quarters, fixed order
    __syncthreads();
    float* red = (float*)(smem + 128);  // [kw 4][rg 2][m 4][NT][2][32]
#pragma unroll
    for (int m = 0; m < 4; m++)
#pragma unroll
        for (int n = 0; n < NT; n++) {
            size_t base = ((((size_t)kw * 2 + rg) * 4 + m) * NT + n) * 2;
            red[(base + 0) * 32 + lane] = acc[m][n][0] + acc[m][n][1];
            red[(base + 1) * 32 + lane] = acc[m][n][2] + acc[m][n][3];
        }
    __syncthreads();
    const int ng_all = p.K / p.group;
    const int ng_slice = kslice / p.group;
    const int entries = 2 * 4 * NT * 2 * 32;
    const size_t quarter = (size_t)2 * 4 * NT * 2 * 32;
    for (int e = tid; e < entries; e += 256) {
        int ln = e & 31;
        int r = e >> 5;
        int which = r & 1;
        r >>= 1;
        int n = r % NT;
        r /= NT;
        int m = r & 3;
        int rgi = r >> 2;
        int token = n * 4 + (ln & 3);
        if (token >= p.T) continue;
        int row = rb * 128 + rgi * 64 + m * 16 + (ln >> 2) + 8 * which;
        float v = red[e] + red[quarter + e] + red[2 * quarter + e] + red[3 * quarter + e];
        v = ldexpf(v, -p.xexp[token]);
        const uint16_t* br = p.bias + (size_t)row * ng_all + ks * ng_slice;
        const float* xs = p.xsum + (size_t)token * ng_all + ks * ng_slice;
        float bt = 0.0f;
        for (int gi = 0; gi < ng_slice; gi++) bt += __half2float(__ushort_as_half(br[gi])) * xs[gi];
        v += bt;
        if (p.nsplit == 1) {
            float* o = p.out + (size_t)token * p.O + row;
            *o = p.add ? *o + v : v;
        } else {
            p.partial[((size_t)ks * p.T + token) * p.O + row] = v;
        }
    }
    if (p.nsplit == 1) return;
    __threadfence();
    __syncthreads();
    __shared__ int s_last;
    if (tid == 0) s_last = atomicAdd(&p.counters[rb], 1u) == (unsigned)(p.nsplit - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int e = tid; e < 128 * p.T; e += 256) {
        int token = e / 128, row = rb * 128 + (e % 128);
        float v = 0.0f;
        for (int s = 0; s < p.nsplit; s++) v += __ldcg(p.partial + ((size_t)s * p.T + token) * p.O + row);
        float* o = p.out + (size_t)token * p.O + row;
        *o = p.add ? *o + v : v;
    }
    if (tid == 0) p.counters[rb] = 0;
}

static size_t gemv_smem(int kslice, int nt, int group) {
    int gpc = 128 / group;
    size_t main = 128 + (size_t)kslice * 32 + (size_t)(kslice / 128) * 8 * gpc * 32 + (size_t)(kslice / 16) * nt * 256;
    size_t red = 128 + (size_t)4 * 2 * 4 * nt * 2 * 32 * 4;
    return main > red ? main : red;
}

template <int NT, int GPC>
static void launch_gemv_t(const GemvParams& p, cudaStream_t st) {
    size_t smem = gemv_smem(p.kslice, NT, p.group);
    auto fn = ternary_gemv_kernel<NT, GPC>;
    static bool attr_done = false;
    if (!attr_done) {
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        attr_done = true;
    }
    GemvParams pp = p;
    void* args[] = {&pp};
    launch_pdl((const void*)fn, dim3((unsigned)((p.O / 128) * p.nsplit)), dim3(256), smem, st, args);
}

void launch_ternary_gemv(const TernaryMat& m, const TernaryAct& a, int T, float* out, int add, float* partial,
                         unsigned* counters, int* err, cudaStream_t st) {
    GemvParams p;
    p.codes = (const uint4*)m.codes;
    p.scales = m.scales;
    p.bias = m.bias;
    p.bfrag = a.bfrag;
    p.xsum = a.xsum;
    p.xexp = a.xexp;
    p.out = out;
    p.partial = partial;
    p.counters = counters;
    p.err = err;
    p.O = m.O;
    p.K = m.K;
    p.group = m.group;
    p.kslice = m.kslice;
    p.nsplit = m.nsplit;
    p.T = T;
    p.add = add;
    int nt = (2 * T + 7) / 8;
    if (m.group == 64) {
        if (nt == 1) launch_gemv_t<1, 2>(p, st);
        else if (nt == 2) launch_gemv_t<2, 2>(p, st);
        else if (nt == 3) launch_gemv_t<3, 2>(p, st);
        else launch_gemv_t<4, 2>(p, st);
    } else {
        if (nt == 1) launch_gemv_t<1, 1>(p, st);
        else if (nt == 2) launch_gemv_t<2, 1>(p, st);
        else if (nt == 3) launch_gemv_t<3, 1>(p, st);
        else launch_gemv_t<4, 1>(p, st);
    }
}

// ------------------------------------------------------------------------------------------------ config 1 producer
// One CTA per padded token row: x (bf16 or fp32) -> rotate -> activation operand.
__global__ void __launch_bounds__(512) rotate_prep_kernel(const uint16_t* x_bf16, const float* x_f32, int T, int K,
                                                          int HB, const float* signs, int group, int NT,
                                                          TernaryAct act, float* xrot) {
    extern __shared__ float xs[];
    __shared__ float red[32];
    int t = blockIdx.x;
    pdl_trigger();
    pdl_wait();
    for (int i = threadIdx.x; i < K; i += blockDim.x) {
        float v = 0.0f;
        if (t < T) v = x_f32 ? x_f32[(size_t)t * K + i] : __bfloat162float(__ushort_as_bfloat16(x_bf16[(size_t)t * K + i]));
        xs[i] = v;
    }
    __syncthreads();
    if (HB > 0) block_rotate(xs, K, HB, signs);
    if (xrot && t < T)
        for (int i = threadIdx.x; i < K; i += blockDim.x) xrot[(size_t)t * K + i] = xs[i];
    write_ternary_act(xs, K, t, T, NT, group, act, red);
}

void launch_rotate_prep(const uint16_t* x_bf16, const float* x_f32, int T, int K, int HB, const float* signs,
                        int group, TernaryAct act, float* xrot, cudaStream_t st) {
    int nt = (2 * T + 7) / 8;
    static bool attr_done = false;
    if (!attr_done) {
        cudaFuncSetAttribute(rotate_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
        attr_done = true;
    }
    void* args[] = {&x_bf16, &x_f32, &T, &K, &HB, &signs, &group, &nt, &act, &xrot};
    launch_pdl((const void*)rotate_prep_kernel, dim3(4 * nt), dim3(512), (size_t)K * 4, st, args);
}

}  // namespace bcu
