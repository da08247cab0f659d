// gemm.cu — ternary GEMM for batched prefill (graded config 5; the reference's prefill matmul qmm,
// kernels.metal:437-500, and its Vulkan coopmat form qmm_cm.comp) on the 5th-generation tensor cores:
// y[M][O] = W . x for M tokens, W the MLX 2-bit pack (w = c s + b per group of G inputs).
//
// Per CTA tile: 256 weight rows (two halves of 128) x 128 tokens, accumulated in tensor memory (TMEM, all 512 columns:
// per half a 256-column accumulator with the tokens' fp16 hi parts in columns 0..127 and lo parts in 128..255, so
// one tcgen05.mma of N = 256 multiplies both by the same weight tile, and the two halves' MMAs share the activation
// tile, halving the activation bytes per flop). K runs in chunks of 64 inputs through a shared-memory pipeline (4
// activation/code stages, 2 decoded-weight buffers) with warp roles:
//   - a loader warp issues 1-D bulk copies (the TMA engine, cp.async.bulk, no tensor map, no multicast) of the chunk's
//     activation tile (32 KB, prepared by gemm_prep_kernel in the MMA's shared-memory layout) and of its packed codes
//     and scales (4.6 KB), completing on the stage's mbarrier;
//   - 8 decoder warps (thread = weight row) turn the codes into fp16 weights c s (one LOP3 per pair of codes gives
//     fp16 1024 + c, one fma with s and -1024 s gives c s, exact for ternary codes) in the K-major layout with the
//     128-byte swizzle;
//   - an MMA warp issues 8 tcgen05.mma.kind::f16 (128 x 256 x 16) per chunk and commits them to the stage's mbarrier,
//     which frees the stage;
//   - 8 epilogue warps read the accumulators (tcgen05.ld) and write y.
// The bias term sum_g b_g sum_{k in g} x_k rides as extra chunks: A = G b (prepared tiles), B = the group sums of the
// token times 2^-log2(G) (prepared with the activations). Activations are fp32 split as x 2^E = hi + lo (fp16 each,
// E per token from its row maximum), so every product is exact and sums are fp32: y = (D_hi + D_lo) 2^-E.
// Every wait is bounded; on a timeout the kernel records ERR_MBAR_TIMEOUT, every role stops, the MMA issuer waits
// (bounded) for its last MMAs, and the tensor memory is freed.

#include "common.cuh"
#include "gemm_act.cuh"
#include "kernels.h"
#include "operand.cuh"  // pow2f

namespace bcu {

// A tile is 256 weight rows (two halves of 128, one MMA each) x 128 tokens; a chunk is 64 inputs.
constexpr int GM_ROWS = 128;  // rows per half (GM_TOK tokens per tile and GM_KC inputs per chunk: gemm_act.cuh)
constexpr int GM_SB = 4;  // activation + code stages (the loader runs up to 3 chunks ahead of the MMAs)
constexpr int GM_SA = 2;  // decoded-weight buffers (the decoders run 1 chunk ahead)
constexpr int GM_A_BYTES = GM_ROWS * GM_KC * 2;           // 16 KB decoded weights per half
constexpr int GM_W_BYTES = GM_ROWS * 16 + GM_ROWS * 2;    // per half: codes [128][4 u32] + scales [128] fp16
// shared memory: B[GM_SB] (32 KB each) | A[GM_SA] (two 16-KB halves each) | W[GM_SB] (two halves of codes + scales)
// | barriers; tiles on 1024-byte boundaries
constexpr int GM_A_OFF = GM_SB * GM_B_BYTES, GM_W_OFF = GM_A_OFF + GM_SA * 2 * GM_A_BYTES;
constexpr int GM_BAR_OFF = GM_W_OFF + GM_SB * 2 * GM_W_BYTES;
constexpr int GM_SMEM = GM_BAR_OFF + 2048;                // + barriers, TMEM address; + 1024 to align the base
static_assert(GM_SMEM <= 227 * 1024, "shared memory of the prefill GEMM");
constexpr uint32_t GM_TMEM_COLS = 256;                    // one accumulator (128 lanes x 256 columns) per half
// kind::f16 instruction descriptor: D f32 (bits 4-5 = 1), A and B f16 (0), both K-major, N = 256 (bits 17-22 =
// N / 8), M = 128 (bits 24-28 = M / 16)
constexpr uint32_t GM_IDESC = (1u << 4) | ((256u / 8) << 17) | ((128u / 16) << 24);

// ----------------------------------------------------------------------------------------------- tcgen05 / TMEM
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// D (TMEM) (+)= A (smem) . B (smem)^T, both K-major; accumulate = 0 overwrites D.
__device__ __forceinline__ void umma_f16(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}
// Arrives on bar once every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// 32 TMEM lanes x 32 consecutive 32-bit columns: thread i of the warp gets lane (lane field of taddr) + i.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr));
}

// Matrix descriptor of a swizzled operand tile (sw128, gemm_act.cuh) for the k16 step at byte offset koff (0, 32, 64,
// 96) of the rows: start address, leading byte offset 16 (unused by swizzled K-major layouts), stride byte offset
// 1024 (8-row groups), version 1 (bit 46), layout SWIZZLE_128B (2 in bits 61-63).
__device__ __forceinline__ uint64_t umma_desc_sw128(const void* tile, uint32_t koff) {
    const uint64_t a = smem_u32(tile) + koff;
    return ((a >> 4) & 0x3FFFull) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// ----------------------------------------------------------------------------------------------- weights
// Row tiles of 256 rows; O is padded to whole tiles with zero weights.
__host__ __device__ inline int gemm_row_tiles(int O) { return (O + 2 * GM_ROWS - 1) / (2 * GM_ROWS); }

// Main chunks: per (row tile rt, chunk c, half h) [128 rows][4 u32 codes of inputs 64 c .. 64 c + 63, MLX order] then
// [128] fp16 scales of the chunk's group; the two halves of a (rt, c) are adjacent. One thread per (rt, c, h, row).
__global__ void gemm_pack_w_kernel(const uint32_t* __restrict__ w, const uint16_t* __restrict__ s, int O, int K, int G,
                                   uint8_t* __restrict__ out) {
    const int nmain = K / GM_KC;
    const size_t n = (size_t)gemm_row_tiles(O) * nmain * 2 * GM_ROWS;
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int r = i % GM_ROWS, h = (i / GM_ROWS) % 2, c = (i / (2 * GM_ROWS)) % nmain;
    const size_t rt = i / ((size_t)2 * GM_ROWS * nmain), row = rt * 2 * GM_ROWS + h * GM_ROWS + r;
    uint8_t* base = out + (((size_t)rt * nmain + c) * 2 + h) * GM_W_BYTES;
    const bool in = row < (size_t)O;
    ((uint4*)base)[r] = in ? *(const uint4*)(w + row * (K / 16) + 4 * c) : make_uint4(0, 0, 0, 0);
    ((uint16_t*)(base + GM_ROWS * 16))[r] = in ? s[row * (K / G) + (GM_KC * c) / G] : (uint16_t)0;
}

// Bias chunks: per (rt, bias chunk cb, half h) the A tile (128 rows of 64 fp16, 128-byte swizzle) of
// G b[row][g], g = 64 cb + k (zero past K / G or O); b = -s for the implicit bias of the reference pack; the two
// halves adjacent. One thread per (rt, cb, h, row, k-chunk).
__global__ void gemm_pack_bias_kernel(const uint16_t* __restrict__ s, const uint16_t* __restrict__ b, int O, int K,
                                      int G, int nbias, uint8_t* __restrict__ out) {
    const size_t n = (size_t)gemm_row_tiles(O) * nbias * 2 * GM_ROWS * 8;
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int kk = i % 8, r = (i / 8) % GM_ROWS, h = (i / (8 * GM_ROWS)) % 2, cb = (i / (16 * GM_ROWS)) % nbias;
    const size_t rt = i / ((size_t)16 * GM_ROWS * nbias), row = rt * 2 * GM_ROWS + h * GM_ROWS + r;
    const int ng = K / G;
    uint16_t v[8];
    for (int e = 0; e < 8; e++) {
        const int g = GM_KC * cb + 8 * kk + e;
        float x = 0.0f;
        if (g < ng && row < (size_t)O) {
            const float bb = b ? __half2float(__ushort_as_half(b[row * ng + g])) : -__half2float(__ushort_as_half(s[row * ng + g]));
            x = bb * (float)G;
        }
        v[e] = __half_as_ushort(__float2half_rn(x));
    }
    uint8_t* tile = out + (((size_t)rt * nbias + cb) * 2 + h) * GM_A_BYTES;
    *(uint4*)(tile + sw128(r, kk)) = *(const uint4*)v;
}

// ----------------------------------------------------------------------------------------------- activations
// One warp per token: the exponent of its row maximum, then its tiles (gemm_act.cuh).
__global__ void gemm_prep_kernel(const float* __restrict__ x, int M, int K, int G, int nmain, int nbias,
                                 uint8_t* __restrict__ bop, int* __restrict__ ex) {
    const int lane = threadIdx.x & 31, t = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (t >= M) return;
    const float* row = x + (size_t)t * K;
    float am = 0.0f;
    for (int k = lane * 4; k < K; k += 128) {
        const float4 v = *(const float4*)(row + k);
        am = fmaxf(am, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
    am = warp_max(am);
    const int E = gemm_act_exponent(am);
    if (lane == 0) ex[t] = E;
    gemm_act_words(row, t, K, G, nmain, nbias, E, 0, 32, bop);
}

// ----------------------------------------------------------------------------------------------- GEMM
struct GemmParams {
    const uint8_t* wt;     // main chunks (gemm_pack_w_kernel)
    const uint8_t* abias;  // bias chunks (gemm_pack_bias_kernel)
    const uint8_t* bop;    // activation chunks (gemm_prep_kernel)
    const int* ex;         // [M] exponents
    float* y;              // [M][O]
    int* err;
    int M, O, nmain, nbias, n_rt, n_tiles;
};

// Warp roles (576 threads): warps 0-7 epilogue (tensor memory -> y; warp w reads half w / 4, lanes 32 (w % 4) ..
// 32 (w % 4) + 31), warps 8-15 decode (thread = weight row of the tile), warp 16 issues the bulk copies, warp 17
// issues the MMAs. Chunk q uses activation/code stage q % GM_SB and decoded-weight buffer q % GM_SA; barriers
// load_full[GM_SB] (copies landed), a_full[GM_SA] (256 decoder arrivals), mma_done[GM_SB] (chunk q's MMAs finished,
// which frees its stage and its weight buffer); the two halves' accumulators fill the
// 512 tensor-memory columns, with acc_full (the tile's MMAs finished) and acc_empty (256 epilogue arrivals).
constexpr int GM_THREADS = 576;

__global__ void __launch_bounds__(GM_THREADS, 1) ternary_gemm_kernel(GemmParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // swizzle atoms need 1024-byte aligned tiles: align the base (the launch adds 1024 bytes of slack)
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint64_t* load_full = (uint64_t*)(smem + GM_BAR_OFF);
    uint64_t* a_full = load_full + GM_SB;
    uint64_t* mma_done = a_full + GM_SA;
    uint64_t* acc_full = mma_done + GM_SB;
    uint64_t* acc_empty = acc_full + 1;
    uint32_t* s_tmem = (uint32_t*)(acc_empty + 1);
    volatile int* s_abort = (volatile int*)(s_tmem + 1);
    const int nch = p.nmain + p.nbias;
    const int my_tiles = p.n_tiles > (int)blockIdx.x ? (p.n_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int total = my_tiles * nch;
    if (tid == 0) {
        for (int i = 0; i < GM_SB; i++) {
            mbar_init(&load_full[i], 1);
            mbar_init(&mma_done[i], 1);
        }
        for (int i = 0; i < GM_SA; i++) mbar_init(&a_full[i], 256);
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, 256);
        *s_abort = 0;
        fence_proxy_async_smem();
    }
    if (warp == 0) {
        tmem_alloc(s_tmem, 2 * GM_TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s_tmem;
    auto fail = [&]() {
        atomicOr(p.err, ERR_MBAR_TIMEOUT);
        *s_abort = 1;
    };
    auto b_of = [&](int q) { return smem + (q % GM_SB) * GM_B_BYTES; };
    auto a_of = [&](int q) { return smem + GM_A_OFF + (q % GM_SA) * 2 * GM_A_BYTES; };
    auto w_of = [&](int q) { return smem + GM_W_OFF + (q % GM_SB) * 2 * GM_W_BYTES; };
    // parity of chunk q's completion of a barrier used once per GM_SB (par) or GM_SA (para) chunks
    auto par = [](int q) { return (uint32_t)((q / GM_SB) & 1); };
    auto para = [](int q) { return (uint32_t)((q / GM_SA) & 1); };

    if (warp == 16) {  // ----------------------------------------------------------------- bulk copies
        if (lane == 0) {
            for (int q = 0; q < total && !*s_abort; q++) {
                const int s = q % GM_SB, c = q % nch, j = q / nch;
                const int tile = blockIdx.x + j * gridDim.x, rt = tile % p.n_rt, tt = tile / p.n_rt;
                // the stage is free once chunk q - GM_SB's MMAs are done; a bias chunk also writes weight buffer
                // q % GM_SA, free once chunk q - GM_SA's MMAs are done
                if ((q >= GM_SB && !mbar_wait_bounded(&mma_done[s], par(q - GM_SB))) ||
                    (c >= p.nmain && q >= GM_SA &&
                     !mbar_wait_bounded(&mma_done[(q - GM_SA) % GM_SB], par(q - GM_SA)))) {
                    fail();
                    break;
                }
                const uint8_t* bsrc = p.bop + ((size_t)tt * nch + c) * GM_B_BYTES;
                if (c < p.nmain) {
                    mbar_expect_tx(&load_full[s], GM_B_BYTES + 2 * GM_W_BYTES);
                    bulk_g2s(b_of(q), bsrc, GM_B_BYTES, &load_full[s]);
                    bulk_g2s(w_of(q), p.wt + ((size_t)rt * p.nmain + c) * 2 * GM_W_BYTES, 2 * GM_W_BYTES, &load_full[s]);
                } else {
                    mbar_expect_tx(&load_full[s], GM_B_BYTES + 2 * GM_A_BYTES);
                    bulk_g2s(b_of(q), bsrc, GM_B_BYTES, &load_full[s]);
                    bulk_g2s(a_of(q), p.abias + ((size_t)rt * p.nbias + (c - p.nmain)) * 2 * GM_A_BYTES, 2 * GM_A_BYTES,
                             &load_full[s]);
                }
            }
        }
        __syncwarp();
    } else if (warp >= 8 && warp < 16) {  // ----------------------------------------------- decode
        const int r = tid - 256, h = r / GM_ROWS, rr = r % GM_ROWS;  // half and row of the tile
        for (int q = 0; q < total && !*s_abort; q++) {
            const int s = q % GM_SB, c = q % nch;
            // weight buffer q % GM_SA is free once chunk q - GM_SA's MMAs are done (waited for bias chunks too, whose
            // buffer the loader fills: so no arrival on a_full can run ahead into the phase of an earlier chunk)
            if (q >= GM_SA && !mbar_wait_bounded(&mma_done[(q - GM_SA) % GM_SB], par(q - GM_SA))) {
                fail();
                break;
            }
            if (c < p.nmain) {
                if (!mbar_wait_bounded(&load_full[s], par(q))) {  // the codes of chunk q have landed
                    fail();
                    break;
                }
                const uint8_t* wh = w_of(q) + h * GM_W_BYTES;
                const uint4 cw = ((const uint4*)wh)[rr];
                const uint16_t sc = ((const uint16_t*)(wh + GM_ROWS * 16))[rr];
                const uint32_t s2 = (uint32_t)sc * 0x10001u;
                uint32_t n2;
                asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(n2) : "r"(s2), "r"(0xE400E400u));  // -1024 s
                const uint32_t words[4] = {cw.x, cw.y, cw.z, cw.w};
                uint8_t* ah = a_of(q) + h * GM_A_BYTES;
#pragma unroll
                for (int wi = 0; wi < 4; wi++) {
                    uint32_t o[8];
#pragma unroll
                    for (int i = 0; i < 8; i++)  // codes i, i + 8: fp16 (1024 + c) pair, then c s (exact for c <= 2)
                        o[i] = hfma2_u32(lop_and_or(words[wi] >> (2 * i), 0x00030003u, 0x64006400u), s2, n2);
                    *(uint4*)(ah + sw128(rr, 2 * wi)) = make_uint4(o[0], o[1], o[2], o[3]);
                    *(uint4*)(ah + sw128(rr, 2 * wi + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
                }
                fence_proxy_async_smem();
            }
            mbar_arrive(&a_full[q % GM_SA]);
        }
    } else if (warp == 17) {  // ---------------------------------------------------------- MMA
        if (lane == 0) {
            for (int q = 0; q < total && !*s_abort; q++) {
                const int s = q % GM_SB, c = q % nch, j = q / nch;
                // the accumulators are free once the epilogue of the previous tile has read them
                if (c == 0 && j >= 1 && !mbar_wait_bounded(acc_empty, (uint32_t)((j - 1) & 1))) {
                    fail();
                    break;
                }
                if (!mbar_wait_bounded(&load_full[s], par(q)) || !mbar_wait_bounded(&a_full[q % GM_SA], para(q))) {
                    fail();
                    break;
                }
                tc_fence_after();
                const uint8_t* bt = b_of(q);
                const uint8_t* at = a_of(q);
#pragma unroll
                for (int ks = 0; ks < 4; ks++) {
                    const uint64_t bd = umma_desc_sw128(bt, 32 * ks);
#pragma unroll
                    for (int h = 0; h < 2; h++)
                        umma_f16(tmem + h * GM_TMEM_COLS, umma_desc_sw128(at + h * GM_A_BYTES, 32 * ks), bd, GM_IDESC,
                                 (c > 0 || ks > 0) ? 1u : 0u);
                }
                umma_commit(&mma_done[s]);
                if (c == nch - 1) umma_commit(acc_full);
            }
        }
        __syncwarp();
    } else {  // ------------------------------------------------------------------ epilogue (warps 0-7)
        const int h = warp >> 2, wq = warp & 3;
        for (int j = 0; j < my_tiles && !*s_abort; j++) {
            const int tile = blockIdx.x + j * gridDim.x, rt = tile % p.n_rt, tt = tile / p.n_rt;
            if (!mbar_wait_bounded(acc_full, (uint32_t)(j & 1))) {
                fail();
                break;
            }
            tc_fence_after();
            const int row = rt * 2 * GM_ROWS + h * GM_ROWS + wq * 32 + lane;
            const uint32_t base = tmem + h * GM_TMEM_COLS + ((uint32_t)(wq * 32) << 16);
#pragma unroll 1
            for (int cb = 0; cb < GM_TOK / 32; cb++) {
                uint32_t hi[32], lo[32];
                tmem_ld32(base + cb * 32, hi);
                tmem_ld32(base + GM_TOK + cb * 32, lo);
                tmem_wait_ld();
                if (row < p.O) {
#pragma unroll
                    for (int i = 0; i < 32; i++) {
                        const int t = tt * GM_TOK + cb * 32 + i;
                        if (t < p.M)
                            p.y[(size_t)t * p.O + row] =
                                (__uint_as_float(hi[i]) + __uint_as_float(lo[i])) * pow2f(-p.ex[t]);
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(acc_empty);
        }
    }
    // drain: the MMA issuer waits (bounded) for its last commit
    if (warp == 17 && lane == 0 && total > 0) mbar_wait_bounded(&mma_done[(total - 1) % GM_SB], par(total - 1), 1u << 20);
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem, 2 * GM_TMEM_COLS);
}

// ----------------------------------------------------------------------------------------------- host
size_t gemm_w_bytes(int O, int K) { return (size_t)gemm_row_tiles(O) * (K / GM_KC) * 2 * GM_W_BYTES; }
int gemm_bias_chunks(int K, int G) { return (K / G + GM_KC - 1) / GM_KC; }
size_t gemm_bias_bytes(int O, int K, int G) {
    return (size_t)gemm_row_tiles(O) * gemm_bias_chunks(K, G) * 2 * GM_A_BYTES;
}
size_t gemm_act_bytes(int M, int K, int G) {
    return (size_t)((M + GM_TOK - 1) / GM_TOK) * (K / GM_KC + gemm_bias_chunks(K, G)) * GM_B_BYTES;
}

void gemm_pack(const uint32_t* w, const uint16_t* s, const uint16_t* b, int O, int K, int G, uint8_t* wt,
               uint8_t* abias, cudaStream_t st) {
    const size_t n1 = (size_t)gemm_row_tiles(O) * (K / GM_KC) * 2 * GM_ROWS;
    gemm_pack_w_kernel<<<(unsigned)((n1 + 255) / 256), 256, 0, st>>>(w, s, O, K, G, wt);
    const int nb = gemm_bias_chunks(K, G);
    const size_t n2 = (size_t)gemm_row_tiles(O) * nb * 2 * GM_ROWS * 8;
    gemm_pack_bias_kernel<<<(unsigned)((n2 + 255) / 256), 256, 0, st>>>(s, b, O, K, G, nb, abias);
}

void gemm_prep_only(const float* x, int M, int K, int G, uint8_t* bop, int* ex, cudaStream_t st) {
    gemm_prep_kernel<<<(unsigned)((M + 7) / 8), 256, 0, st>>>(x, M, K, G, K / GM_KC, gemm_bias_chunks(K, G), bop, ex);
}

cudaError_t gemm_run(const uint8_t* wt, const uint8_t* abias, int O, int K, int G, const float* x, int M, uint8_t* bop,
                     int* ex, float* y, int* err, int num_sms, cudaStream_t st) {
    const int nmain = K / GM_KC, nbias = gemm_bias_chunks(K, G);
    if (x) gemm_prep_kernel<<<(unsigned)((M + 7) / 8), 256, 0, st>>>(x, M, K, G, nmain, nbias, bop, ex);
    GemmParams p;
    p.wt = wt;
    p.abias = abias;
    p.bop = bop;
    p.ex = ex;
    p.y = y;
    p.err = err;
    p.M = M;
    p.O = O;
    p.nmain = nmain;
    p.nbias = nbias;
    p.n_rt = gemm_row_tiles(O);
    p.n_tiles = p.n_rt * ((M + GM_TOK - 1) / GM_TOK);
    raise_smem_limit((const void*)ternary_gemm_kernel, GM_SMEM);
    const int grid = p.n_tiles < num_sms ? p.n_tiles : num_sms;
    ternary_gemm_kernel<<<grid, GM_THREADS, GM_SMEM, st>>>(p);
    return cudaGetLastError();
}

}  // namespace bcu
