// ternary.cu — tensor-core ternary verify GEMV for T <= 16 rows (the reference's qmvxm / qmvx / qmv_cm / qmvr / qmv4,
// kernels.metal:275-404 and 664-709, kernels/qmvx.comp, kernels/qmv_cm.comp, with the rotation kernels of
// kernels.metal:118-226 that feed them).
//
// Why tensor cores at batch 1: a T = 9 verify does 9 multiply-adds per 2-bit weight. At the HBM rate of ~21 T
// weights/s that is ~190 T FMA/s, five times what the CUDA cores can issue, so the products go to mma.m16n8k16 and
// the CUDA cores only decode: per pair of weights one LOP3 ((w & mask) | 0x6400 gives fp16 1024 + c*4^j) and one
// HFMA2 (x s, - 1024 s gives exactly c*s*4^j). The activation operand carries 4^-j and a per-(token, block) power of
// two and is split into fp16 hi + lo columns, so products are exact and sums fp32-accurate. The bias term
// sum_g b_g * sum_k x_k is one more k16 MMA step per warp (A = 64 b, B = group sums / 64). Every output's reduction
// order is fixed and independent of T: a row's result is bit-identical whether it is verified alone or among 16.
//
// CTA = 128 rows x kslice codes (8 warps = 2 row groups of 64 x 4 k-quarters). Before waiting on the previous kernel
// (programmatic dependent launch) one thread streams the CTA's codes and scale/bias tiles into shared memory with
// cp.async.bulk. After the wait the activation operand (operand.cuh) is built once for the whole GEMV by its CTAs
// together (grid_build: one (token, Hadamard block) per warp into a global buffer, a bounded grid-wide wait, then one
// bulk copy per block into each CTA), or, when the grid cannot be resident at once (and for standalone inputs), by
// each CTA for its own K-slice (build_operand). Split-K partials are summed in a fixed order by the last CTA of each
// row block, which applies the residual add, the LoRA up projection and the sums of squares the next norm needs; when
// a row block's splits (at most 8) fit as one thread-block cluster, they sum through the cluster's shared memory
// instead of the global partial buffer.
#include <atomic>
#include <cstdio>
#include <map>
#include <mutex>
#include <set>
#include <tuple>
#include <utility>
#include "common.cuh"
#include "kernels.h"
#include "operand.cuh"

namespace bcu {

constexpr float EPS_T = 1e-6f;
// shared-memory header: mbarriers at 0 (codes) and 8 (operand), exponents [16][4] at 128
constexpr int GEMV_HDR = 384;

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

// launch_pdl with thread-block clusters of `csize` CTAs along x (the grid a multiple of csize).
static cudaError_t launch_pdl_cluster(const void* fn, dim3 grid, int csize, size_t smem, cudaStream_t st,
                                      void** args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = (unsigned)csize;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

size_t ternary_codes_bytes(int O, int K) { return (size_t)O * K / 4; }
size_t ternary_sb_bytes(int O, int K, int group) { return (size_t)O * (K / group) * 4; }

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

// One thread per sb entry: [rb][kc][mt][2][gpc][8].
__global__ void repack_sb_kernel(const uint16_t* __restrict__ s, const uint16_t* __restrict__ b, int O, int K,
                                 int group, uint32_t* __restrict__ out) {
    int gpc = 128 / group, ng = K / group;
    size_t n = (size_t)(O / 16) * (K / 128) * 2 * gpc * 8;
    size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= n) return;
    int g = idx & 7;
    size_t r = idx >> 3;
    int gi = r % gpc;
    r /= gpc;
    int which = r & 1;
    r >>= 1;
    int mt = r & 7;
    size_t rk = r >> 3;
    int nkc = K / 128;
    int kc = rk % nkc;
    int rb = rk / nkc;
    int grp = kc * gpc + gi;
    uint16_t v[2];
    for (int half = 0; half < 2; half++) {
        size_t row = (size_t)rb * 128 + mt * 16 + g + 8 * half;
        uint16_t sv = s[row * ng + grp];
        if (which == 0) {
            v[half] = sv;
        } else {
            __half bb = b ? __ushort_as_half(b[row * ng + grp]) : __hneg(__ushort_as_half(sv));
            v[half] = __half_as_ushort(__float2half_rn(__half2float(bb) * 64.0f));
        }
    }
    out[idx] = (uint32_t)v[0] | ((uint32_t)v[1] << 16);
}

void repack_ternary(const uint32_t* w_mlx, const uint16_t* s, const uint16_t* b, int O, int K, int group,
                    void* codes, uint32_t* sb, cudaStream_t st) {
    size_t n = (size_t)O * K / 16;
    repack_codes_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(w_mlx, O, K, (uint32_t*)codes);
    size_t ns = (size_t)(O / 16) * (K / 128) * 2 * (128 / group) * 8;
    repack_sb_kernel<<<(unsigned)((ns + 255) / 256), 256, 0, st>>>(s, b, O, K, group, sb);
}

// K-slice plan: the longest slice (512, 1024 or 2048 codes; fewest splits) that still puts CTAs on at least ~45% of
// the SMs. Fewer splits save the split-K reduction (a dependent global round trip) and the duplicated operand build;
// one CTA per SM gets the SM's whole issue rate for the decode, so ~70 CTAs of 2048-code slices finish as fast as
// ~140 of 1024. min_kslice: slices never split a Hadamard block (the operand's regions cover whole blocks).
void plan_ternary(TernaryMat& m, int num_sms, int min_kslice) {
    int rb = m.O / 128;
    int best = 0;
    for (int ks : {2048, 1024, 512}) {
        if (m.K % ks || (best && ks < min_kslice)) continue;
        best = ks;
        if (rb * (m.K / ks) * 20 >= num_sms * 9) break;
    }
    m.kslice = best;
    m.nsplit = m.K / best;
}

// ------------------------------------------------------------------------------------------------ GEMV
struct GemvParams {
    const uint8_t* codes;
    const uint32_t* sb;
    ActSrc src;
    GemvOut o;
    AbArgs ab;
    LoraArgs lora;
    int O, K, group, kslice, nsplit, T, n_main, ab_rows;
    int nrb;     // row blocks; CTA = ks * nrb + rb, or rb * nsplit + ks with csplit
    int csplit;  // the K-splits of a row block form one thread-block cluster and sum through its shared memory
};

// Cluster barrier (all threads of every CTA of the cluster): release this CTA's shared-memory writes, acquire the
// others'.
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
// The float at this CTA's shared address `p` in the shared memory of cluster CTA `rank`.
__device__ __forceinline__ float ld_cluster_f32(const float* p, int rank) {
    uint32_t a;
    float v;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(a) : "memory");
    return v;
}

// Per-row scalar of NORM / EMBED: r = rsqrt(mean(h^2) + eps). EMBED also records the id and, in CTA 0, writes the
// row into the residual stream. Fixed-order reductions (lane strides, then the warp tree); loads are issued in
// batches of 8 per lane so the row costs a few memory latencies, not one per element.
__device__ float row_scale(const ActSrc& s, int t, int K, uint32_t* id_out, bool writer) {
    const int lane = threadIdx.x & 31;
    float acc = 0.0f;
    if (s.mode == ACT_NORM) {
        for (int i = lane; i < s.nss; i += 32) acc += s.ss[i * VMAX + t];
    } else if (s.mode == ACT_EMBED) {
        uint32_t id = resolve_id(s.ctl, t);
        if (writer && lane == 0) {
            ((Ctl*)s.ctl)->used[t] = id;
            if (id >= (uint32_t)s.vocab) atomicOr(&((Ctl*)s.ctl)->err, ERR_BAD_TOKEN);
        }
        if (id >= (uint32_t)s.vocab) id = 0;
        *id_out = id;
        const uint16_t* row = s.xb + (size_t)id * K;
        for (int k0 = 0; k0 < K; k0 += 256) {
            float a[8];
#pragma unroll
            for (int i = 0; i < 8; i++) a[i] = __bfloat162float(__ushort_as_bfloat16(row[k0 + i * 32 + lane]));
#pragma unroll
            for (int i = 0; i < 8; i++) {
                acc += a[i] * a[i];
                if (writer) s.h_out[(size_t)t * K + k0 + i * 32 + lane] = a[i];
            }
        }
    } else {
        return 1.0f;
    }
    acc = warp_sum(acc);
    return rsqrtf(acc / (float)K + EPS_T);
}

// Pre-rotation values x_k, k = base + lane + 32 e (e < N), of row t for the modes other than GATED (which needs head
// norms). The mode branch is outside the element loops and every load of the row is issued before the first use.
template <int N>
__device__ __forceinline__ void act_values(const ActSrc& s, int t, int base, int K, float r, uint32_t id, float* v) {
    const int lane = threadIdx.x & 31;
    float a[N], b[N];
    switch (s.mode) {
        case ACT_NORM:
#pragma unroll
            for (int e = 0; e < N; e++) a[e] = s.x[(size_t)t * K + base + lane + 32 * e];
#pragma unroll
            for (int e = 0; e < N; e++) b[e] = s.w[base + lane + 32 * e];
#pragma unroll
            for (int e = 0; e < N; e++) v[e] = (a[e] * r) * b[e];
            break;
        case ACT_EMBED:
#pragma unroll
            for (int e = 0; e < N; e++) a[e] = __bfloat162float(__ushort_as_bfloat16(s.xb[(size_t)id * K + base + lane + 32 * e]));
#pragma unroll
            for (int e = 0; e < N; e++) b[e] = s.w[base + lane + 32 * e];
#pragma unroll
            for (int e = 0; e < N; e++) v[e] = (a[e] * r) * b[e];
            break;
        case ACT_SWIGLU:
#pragma unroll
            for (int e = 0; e < N; e++) a[e] = s.x[(size_t)t * 2 * K + base + lane + 32 * e];
#pragma unroll
            for (int e = 0; e < N; e++) b[e] = s.x[(size_t)t * 2 * K + K + base + lane + 32 * e];
#pragma unroll
            for (int e = 0; e < N; e++) v[e] = (a[e] * b[e]) * sigm(a[e]);
            break;
        case ACT_GATE:
#pragma unroll
            for (int e = 0; e < N; e++) a[e] = s.x[(size_t)t * K + base + lane + 32 * e];
#pragma unroll
            for (int e = 0; e < N; e++) {
                int k = base + lane + 32 * e;
                b[e] = s.x2[(size_t)t * s.ld2 + (k >> 8) * 512 + 256 + (k & 255)];
            }
#pragma unroll
            for (int e = 0; e < N; e++) v[e] = a[e] * sigm(b[e]);
            break;
        default:
            if (s.xb) {
#pragma unroll
                for (int e = 0; e < N; e++)
                    v[e] = __bfloat162float(__ushort_as_bfloat16(s.xb[(size_t)t * K + base + lane + 32 * e]));
            } else {
#pragma unroll
                for (int e = 0; e < N; e++) v[e] = s.x[(size_t)t * K + base + lane + 32 * e];
            }
    }
}


// ------------------------------------------------------------------------------------------------ operand
// Raw source values of one token for elements blk0 + lane + 32 e (every load of the token issued together).
template <int VPL>
struct RawTok {
    float a[VPL], b[VPL];
    float ss;  // NORM: this lane's part of the row's sum of squares (from the per-row-block partials)
};

template <int VPL>
__device__ __forceinline__ void load_raw(const ActSrc& s, int t, int blk0, int K, RawTok<VPL>& R) {
    const int lane = threadIdx.x & 31;
    switch (s.mode) {
        case ACT_NORM:
#pragma unroll
            for (int e = 0; e < VPL; e++) R.a[e] = s.x[(size_t)t * K + blk0 + lane + 32 * e];
            R.ss = 0.0f;
            for (int i = lane; i < s.nss; i += 32) R.ss += s.ss[i * VMAX + t];
            break;
        case ACT_GATED:
#pragma unroll
            for (int e = 0; e < VPL; e++) {
                const int k = blk0 + lane + 32 * e;
                R.a[e] = s.x[(size_t)t * K + k];
                R.b[e] = s.x2[(size_t)t * s.ld2 + s.off2 + k];
            }
            break;
        case ACT_SWIGLU:
#pragma unroll
            for (int e = 0; e < VPL; e++) {
                R.a[e] = s.x[(size_t)t * 2 * K + blk0 + lane + 32 * e];
                R.b[e] = s.x[(size_t)t * 2 * K + K + blk0 + lane + 32 * e];
            }
            break;
        case ACT_GATE:
#pragma unroll
            for (int e = 0; e < VPL; e++) {
                const int k = blk0 + lane + 32 * e;
                R.a[e] = s.x[(size_t)t * K + k];
                R.b[e] = s.x2[(size_t)t * s.ld2 + (k >> 8) * 512 + 256 + (k & 255)];
            }
            break;
        default:
            if (s.xb) {
#pragma unroll
                for (int e = 0; e < VPL; e++)
                    R.a[e] = __bfloat162float(__ushort_as_bfloat16(s.xb[(size_t)t * K + blk0 + lane + 32 * e]));
            } else {
#pragma unroll
                for (int e = 0; e < VPL; e++) R.a[e] = s.x[(size_t)t * K + blk0 + lane + 32 * e];
            }
    }
}

// The producer (RMSNorm, gated RMSNorm, SwiGLU, sigmoid gate; kernels.metal:118-226) applied to raw values; wn: NORM
// weights of the block (VPL) or GATED head-norm weights (4, period 128).
template <int VPL>
__device__ __forceinline__ void transform(const ActSrc& s, int K, const RawTok<VPL>& R, const float* wn, float* v) {
    switch (s.mode) {
        case ACT_NORM: {
            const float r = rsqrtf(warp_sum(R.ss) / (float)K + EPS_T);
#pragma unroll
            for (int e = 0; e < VPL; e++) v[e] = (R.a[e] * r) * wn[e];
            break;
        }
        case ACT_GATED:
            gated_values<VPL>(R.a, R.b, wn, v);
            break;
        case ACT_SWIGLU:
#pragma unroll
            for (int e = 0; e < VPL; e++) v[e] = (R.a[e] * R.b[e]) * sigm(R.a[e]);
            break;
        case ACT_GATE:
#pragma unroll
            for (int e = 0; e < VPL; e++) v[e] = R.a[e] * sigm(R.b[e]);
            break;
        default:
#pragma unroll
            for (int e = 0; e < VPL; e++) v[e] = R.a[e];
    }
}

// One token's HB-point block (HB = 512, 1024 or 2048) built by four warps: warp q of the group holds elements
// e = VQ q + e', e' < VQ = HB / 128, of the one-warp lane layout, i.e. inputs blk0 + (HB / 4) q + lane + 32 e'. The
// radix-2 stages of strides 1..16 run across the lanes and 32..HB/8 inside the lane, the last two (HB/4, HB/2) through
// shared memory (xch: [q][e'][lane]), with the same operations in the same order as the one-warp transform
// (emit_token with HB / 32 values per lane), so the region gets the same bits; the exponent is the maximum over the
// four quarters (s_am: [q]). Writes token t's columns of the HB-input region reg. A quarter of a 512-point block is
// one 128-wide head, so the gated norm's head sums stay inside a warp. Four warps per block shorten the build's chain
// (the producer, the transform and the hi/lo split of a token block) about fourfold against one warp per block.
// Called by every thread of the CTA (it holds block-wide barriers); warps with has = false only pass them. writer:
// this token's builders write the embedding row to the residual stream (EMBED sources).
constexpr int QX_FLOATS = 4 * 16 * 32;  // exchanged values of one group of four warps (2048-point blocks: HB floats)
template <int HB, int GPC>
__device__ void quarter_token(const ActSrc& s, int K, int t, int blk0, bool has, bool writer, uint8_t* reg, float* xch,
                              float* s_am) {
    constexpr int VQ = HB / 128, QW = HB / 4;  // values per lane, inputs per quarter
    constexpr int G = 128 / GPC, EPG = G / 32, NGQ = QW / G;  // groups per quarter
    constexpr float INV = HB == 512 ? 0.044194173824159216f : (HB == 2048 ? 0.02209708691207961f : 0.03125f);
    const int lane = threadIdx.x & 31, q = (threadIdx.x >> 5) & 3;
    const bool rot = s.HB > 0;
    const int base = blk0 + QW * q;
    float v[VQ];
    if (has) {
        float sg[VQ];
        if (s.signs) {
#pragma unroll
            for (int e = 0; e < VQ; e++) sg[e] = s.signs[base + lane + 32 * e];
        }
        if (s.mode == ACT_EMBED) {
            uint32_t id = 0;
            const float r = row_scale(s, t, K, &id, writer && q == 0);  // one writer of the residual row
            act_values<VQ>(s, t, base, K, r, id, v);
        } else {
            float wn[VQ > 4 ? VQ : 4];
            if (s.mode == ACT_NORM) {
#pragma unroll
                for (int e = 0; e < VQ; e++) wn[e] = s.w[base + lane + 32 * e];
            } else if (s.mode == ACT_GATED) {
#pragma unroll
                for (int k = 0; k < 4; k++) wn[k] = s.w[(lane + 32 * k) & 127];
            }
            RawTok<VQ> R;
            load_raw<VQ>(s, t, base, K, R);
            transform<VQ>(s, K, R, wn, v);
        }
        if (s.signs) {
#pragma unroll
            for (int e = 0; e < VQ; e++) v[e] *= sg[e];
        }
        if (rot) {
#pragma unroll
            for (int m = 1; m < 32; m <<= 1) {
                const float sgn = (lane & m) ? -1.0f : 1.0f;
#pragma unroll
                for (int e = 0; e < VQ; e++) {
                    const float o = __shfl_xor_sync(0xffffffffu, v[e], m);
                    v[e] = fmaf(v[e], sgn, o);  // lower lane: v + o, upper lane: o - v
                }
            }
#pragma unroll
            for (int h = 1; h < VQ; h <<= 1)
#pragma unroll
                for (int e = 0; e < VQ; e++)
                    if ((e & h) == 0) {
                        const float a = v[e], c = v[e + h];
                        v[e] = a + c;
                        v[e + h] = a - c;
                    }
#pragma unroll
            for (int e = 0; e < VQ; e++) xch[(q * VQ + e) * 32 + lane] = v[e];
        }
    }
    __syncthreads();
    if (has) {
        if (rot) {  // strides HB/4 (quarters 0|1, 2|3), then HB/2 (0|2, 1|3), then the normalisation
#pragma unroll
            for (int e = 0; e < VQ; e++) {
                const float y0 = xch[e * 32 + lane], y1 = xch[(VQ + e) * 32 + lane];
                const float y2 = xch[(2 * VQ + e) * 32 + lane], y3 = xch[(3 * VQ + e) * 32 + lane];
                const float u0 = y0 + y1, u1 = y0 - y1, u2 = y2 + y3, u3 = y2 - y3;
                const float z = q == 0 ? u0 + u2 : (q == 1 ? u1 + u3 : (q == 2 ? u0 - u2 : u1 - u3));
                v[e] = z * INV;
            }
        }
        float am[VQ];
#pragma unroll
        for (int e = 0; e < VQ; e++) am[e] = fabsf(v[e]);
#pragma unroll
        for (int h = VQ / 2; h > 0; h >>= 1)
#pragma unroll
            for (int e = 0; e < h; e++) am[e] = fmaxf(am[e], am[e + h]);
        const float qmax = warp_max(am[0]);
        if (lane == 0) s_am[q] = qmax;
    }
    __syncthreads();
    int E = 0;
    if (has) {
        const float amax = fmaxf(fmaxf(s_am[0], s_am[1]), fmaxf(s_am[2], s_am[3]));
        if (amax > 0.0f && amax < INFINITY) {
            int ex;
            frexpf(amax, &ex);  // amax < 2^ex
            E = min(max(14 - ex, -60), 100);
        }
        const int nsteps = HB / 16, nbs = op_bias_steps(HB, G);
        const int col = (t & 3) * 2;
        if (lane == 0 && q == 0) ((int*)(reg + (nsteps + nbs) * 256))[t & 3] = E;
        {   // hi + lo of x * 2^E * 4^-j (emit_token's layout): element e' of quarter q is k = QW q + lane + 32 e'
            const int j = lane >> 3;
            const int t4 = (lane & 7) >> 1, which = (lane & 15) >> 3;
            const int E1 = E - 2 * j;
            const float f = E1 > 60 ? pow2f(60) * pow2f(E1 - 60) : (E1 < -60 ? pow2f(-60) * pow2f(E1 + 60) : pow2f(E1));
            uint16_t* r16 = (uint16_t*)reg;
            const int h_hi = ((col * 4 + t4) * 2 + which) * 2 + (lane & 1), h_lo = h_hi + 16;
            const int step0 = (lane >> 4) + (QW / 16) * q;
#pragma unroll
            for (int e = 0; e < VQ; e++) {
                const float a = v[e] * f;
                const __half h = __float2half_rn(a);
                const __half l = __float2half_rn(a - __half2float(h));
                r16[(step0 + 2 * e) * 128 + h_hi] = __half_as_ushort(h);
                r16[(step0 + 2 * e) * 128 + h_lo] = __half_as_ushort(l);
            }
        }
        float gs[NGQ];  // this quarter's group sums
#pragma unroll
        for (int g = 0; g < NGQ; g++) {
            float a = 0.0f;
#pragma unroll
            for (int e = g * EPG; e < (g + 1) * EPG; e++) a += v[e];
            gs[g] = a;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int g = 0; g < NGQ; g++) gs[g] += __shfl_xor_sync(0xffffffffu, gs[g], o);
        // the block's group sums to shared memory (the exchange buffer is free past the barrier above): a bias
        // word pairs groups 2 i, 2 i + 1, which for 128-input groups of a 512-point block lie in two quarters
        if (lane == 0) {
#pragma unroll
            for (int g = 0; g < NGQ; g++) xch[q * NGQ + g] = gs[g];
        }
    }
    __syncthreads();
    if (has && q == 0 && lane < 16) {  // every bias word of the token's columns, as emit_token writes them
        constexpr int NG = HB / G;     // groups in the block; the step's slots past them are zero
        const int nsteps = HB / 16, nbs = op_bias_steps(HB, G);
        const int col = (t & 3) * 2;
        const int hl = lane >> 3, t4 = (lane >> 1) & 3, wh = lane & 1;
        const int kk0 = wh * 8 + t4 * 2;
        const float fb = pow2f(E - 6 > 100 ? 100 : E - 6);
        uint32_t* rw = (uint32_t*)reg;
        for (int bs = 0; bs < nbs; bs++) {
            const int g0 = bs * 16 + kk0;
            const float s0 = g0 < NG ? xch[g0] : 0.0f, s1 = g0 + 1 < NG ? xch[g0 + 1] : 0.0f;
            const float a0 = s0 * fb, a1 = s1 * fb;
            __half h0 = __float2half_rn(a0), h1 = __float2half_rn(a1);
            if (hl) {
                h0 = __float2half_rn(a0 - __half2float(h0));
                h1 = __float2half_rn(a1 - __half2float(h1));
            }
            rw[(nsteps + bs) * 64 + ((col + hl) * 4 + t4) * 2 + wh] = pack_half2(h0, h1);
        }
    }
    __syncthreads();
}

// This CTA's operand for K-slice ks, built by its own warps (sources without a producing kernel: the embedding
// rows of the first layer, standalone inputs): warp w takes block w % nb of the slice and the token slots w / nb,
// w / nb + 8 / nb, ...; the next token's loads are in flight while the current one is built. Regions [nb][NT].
template <int VPL, int GPC>
__device__ void build_operand_warps(const GemvParams& p, int ks, int sbsz, int nb, int NT, uint8_t* s_op, int rsz) {
    constexpr int HBe = VPL * 32, G = 128 / GPC;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const ActSrc& s = p.src;
    const int K = p.K, kslice = p.kslice, T = p.T, ntok = 4 * NT;
    const int k0 = ks * kslice;
    const int b = warp % nb, js = 8 / nb;
    const int blk0 = HBe <= kslice ? k0 + b * HBe : (k0 / HBe) * HBe;
    OpGeo geo;
    geo.sbsz = sbsz;
    geo.e_lo = HBe <= kslice ? 0 : (k0 - blk0) / 32;
    geo.e_hi = HBe <= kslice ? VPL : geo.e_lo + kslice / 32;
    geo.kr0 = HBe <= kslice ? 0 : blk0 - k0;
    geo.rotate = s.HB > 0;
    auto region = [&](int t) { return s_op + (size_t)(b * NT + (t >> 2)) * rsz; };
    float sg[VPL];
    if (s.signs) {
#pragma unroll
        for (int e = 0; e < VPL; e++) sg[e] = s.signs[blk0 + lane + 32 * e];
    }
    if (s.mode == ACT_EMBED) {  // the row scale needs the whole gathered row: one token at a time
        for (int t = warp / nb; t < ntok; t += js) {
            if (t >= T) {
                zero_token(t, sbsz, G, region(t));
                continue;
            }
            float v[VPL];
            uint32_t id = 0;
            const float r = row_scale(s, t, K, &id, blockIdx.x == 0 && b == 0);
            act_values<VPL>(s, t, blk0, K, r, id, v);
            emit_token<VPL, GPC>(geo, t, region(t), v, s.signs ? sg : nullptr);
        }
        return;
    }
    float wn[VPL];
    if (s.mode == ACT_NORM) {
#pragma unroll
        for (int e = 0; e < VPL; e++) wn[e] = s.w[blk0 + lane + 32 * e];
    } else if (s.mode == ACT_GATED) {
#pragma unroll
        for (int i = 0; i < 4; i++) wn[i] = s.w[(lane + 32 * i) & 127];
    }
    RawTok<VPL> cur, nxt;
    int t = warp / nb;
    if (t < T) load_raw<VPL>(s, t, blk0, K, cur);
    for (; t < ntok; t += js) {
        const int tn = t + js;
        if (tn < T) load_raw<VPL>(s, tn, blk0, K, nxt);
        if (t < T) {
            float v[VPL];
            transform<VPL>(s, K, cur, wn, v);
            emit_token<VPL, GPC>(geo, t, region(t), v, s.signs ? sg : nullptr);
        } else {
            zero_token(t, sbsz, G, region(t));
        }
        cur = nxt;
    }
}

// This CTA's operand when its slice is one whole 2048-point block (the host plans slices of whole blocks): warps 0-3
// build the token slots one after another with quarter_token (its exchange after the regions), warp 0 zeroes the
// slots past T.
template <int GPC>
__device__ void build_operand_quarters(const GemvParams& p, int ks, int NT, uint8_t* s_op, int rsz) {
    constexpr int G = 128 / GPC;
    const int warp = threadIdx.x >> 5;
    float* xch = (float*)(s_op + (size_t)NT * rsz);
    float* s_am = xch + QX_FLOATS;
    for (int t = 0; t < 4 * NT; t++) {
        uint8_t* reg = s_op + (size_t)(t >> 2) * rsz;
        if (t >= p.T) {
            if (warp == 0) zero_token(t, 2048, G, reg);
            continue;
        }
        quarter_token<2048, GPC>(p.src, p.K, t, ks * p.kslice, warp < 4, blockIdx.x == 0, reg, xch, s_am);
    }
}

// This CTA's operand for K-slice ks, regions [nb][NT]: build_operand_warps, or four warps per token for 2048-point
// blocks.
template <int VPL, int GPC>
__device__ void build_operand(const GemvParams& p, int ks, int sbsz, int nb, int NT, uint8_t* s_op, int rsz) {
    if constexpr (VPL == 64)
        build_operand_quarters<GPC>(p, ks, NT, s_op, rsz);
    else
        build_operand_warps<VPL, GPC>(p, ks, sbsz, nb, NT, s_op, rsz);
}

// Grid-build tasks (token t, HB-point block b) for groups of four warps: task i = CTA + n_main * grp for warp group
// grp (at most two per CTA), built by quarter_token into the group's scratch region, then stored to the buffer.
// Shared memory: two task regions, then the exchanged values (HB floats) and the quarter maxima of each group.
template <int HB, int GPC>
__device__ void build_quarters(const GemvParams& p, uint8_t* scratch) {
    constexpr int G = 128 / GPC;
    const ActSrc& s = p.src;
    const int warp = threadIdx.x >> 5, grp = warp >> 2, q = warp & 3;
    const int nblk = p.K / HB, ntask = p.T * nblk;
    const int i = blockIdx.x + p.n_main * grp;
    const bool has = i < ntask;
    const int rsz = op_region_bytes(HB, G);
    const int t = has ? i / nblk : 0, b = has ? i % nblk : 0;
    uint8_t* reg = scratch + (size_t)grp * rsz;
    float* xch = (float*)(scratch + 2 * rsz) + grp * HB;
    float* s_am = (float*)(scratch + 2 * rsz) + 2 * HB + grp * 4;
    quarter_token<HB, GPC>(s, p.K, t, b * HB, has, b == 0, reg, xch, s_am);
    if (has && q == 0) store_token_columns(t, HB, G, reg, s.opbuf + ((size_t)b * 4 + (t >> 2)) * rsz);
}

// The whole operand of the GEMV, built once by its CTAs together into the global buffer src.opbuf: task i = (token
// i / nblk, Hadamard block i % nblk of the K inputs) is built by the four warps of group i / n_main of CTA i % n_main
// (quarter_token: load, producer, signs, Walsh-Hadamard, fp16 hi/lo, exponent, group sums) into a scratch region in
// shared memory, whose columns for the token are then stored to the buffer. Then every CTA waits (bounded) until all builder CTAs have counted
// themselves; the grid is resident at once (the host checks), so the wait ends. counters[0] counts builders,
// counters[1] the CTAs past the wait (grid_build_release: the last resets both for the next GEMV). Only thread 0
// waits; the others meet it at the caller's next barrier.
template <int VPL, int GPC>
__device__ void grid_build(const GemvParams& p, uint8_t* scratch, int* s_ok) {
    constexpr int HBe = VPL * 32;
    const ActSrc& s = p.src;
    const int tid = threadIdx.x, c = blockIdx.x;
    const int T = p.T, K = p.K, nblk = K / HBe, ntask = T * nblk;
    const int ncta = p.n_main;
    const int nbuild = ntask < ncta ? ntask : ncta;  // CTAs with at least one task
    build_quarters<HBe, GPC>(p, scratch);
    __syncthreads();  // this CTA's tasks are stored
    if (tid == 0) {
        if (c < nbuild) arrive_release(s.op_counters);
        *s_ok = spin_until_geq(s.op_counters, (unsigned)nbuild);
        if (!*s_ok) atomicOr(p.o.err, ERR_SPIN_TIMEOUT);
    }
}

// After the slice's copies are issued (off the build's critical path): count this CTA past the grid-wide wait; the
// last one resets both counters for the next GEMV. Thread 0.
__device__ __forceinline__ void grid_build_release(const GemvParams& p) {
    unsigned old;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(old) : "l"(p.src.op_counters + 1) : "memory");
    if (old == (unsigned)(p.n_main - 1)) {  // every CTA is past the wait
        p.src.op_counters[0] = 0;
        p.src.op_counters[1] = 0;
    }
}

// LoRA A of a GEMV's input (norm_rotate's fused A rows, kernels.metal:70-116), in a short kernel launched just before
// the GEMV: u partials for every (token t, Hadamard block b) of the input, which the GEMV's output epilogue sums over
// the blocks and multiplies by B. One warp per (t, b, chunk of 8 stacked A rows): the chunk's rows are loaded before
// the dependency wait; after it the warp forms the block's unrotated input values (the producer of the GEMV's source
// mode, without signs or rotation), takes 8 lane-local dot products and sums them across the warp in a fixed order
// (a halving butterfly over offsets 16, 8, 4 leaves lane l with row (l >> 2) & 7, offsets 2 and 1 finish). Stored to
// upart[t][b][row]; nothing depends on T.
template <int VPL>
__global__ void __launch_bounds__(256) lora_a_kernel(GemvParams p) {
    constexpr int HBe = VPL * 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const ActSrc& s = p.src;
    const LoraArgs& L = p.lora;
    const int K = p.K, nblk = K / HBe, nch = L.R / 8;
    const int i = blockIdx.x * 8 + warp;
    pdl_trigger();
    const bool active = i < p.T * nblk * nch;
    const int c = active ? i % nch : 0, b = active ? (i / nch) % nblk : 0, t = active ? i / (nch * nblk) : 0;
    const int blk0 = b * HBe;
    uint4 w[8][VPL / 8];
    float wn[VPL];
    if (active) {
#pragma unroll
        for (int q = 0; q < 8; q++) {
            const uint4* ap = (const uint4*)(L.a + (((size_t)b * L.R + c * 8 + q) * 32 + lane) * VPL);
#pragma unroll
            for (int u = 0; u < VPL / 8; u++) w[q][u] = __ldg(ap + u);
        }
        if (s.mode == ACT_NORM) {
#pragma unroll
            for (int e = 0; e < VPL; e++) wn[e] = s.w[blk0 + lane + 32 * e];
        } else if (s.mode == ACT_GATED) {
#pragma unroll
            for (int q = 0; q < 4; q++) wn[q] = s.w[(lane + 32 * q) & 127];
        }
    }
    pdl_wait();
    if (!active) return;
    float v[VPL];
    if (s.mode == ACT_EMBED) {
        uint32_t id = 0;
        const float r = row_scale(s, t, K, &id, false);
        act_values<VPL>(s, t, blk0, K, r, id, v);
    } else {
        RawTok<VPL> R;
        load_raw<VPL>(s, t, blk0, K, R);
        transform<VPL>(s, K, R, wn, v);
    }
    float acc[8];
#pragma unroll
    for (int q = 0; q < 8; q++) {
        acc[q] = 0.0f;
#pragma unroll
        for (int u = 0; u < VPL / 8; u++) {
            const uint32_t ws[4] = {w[q][u].x, w[q][u].y, w[q][u].z, w[q][u].w};
#pragma unroll
            for (int h = 0; h < 4; h++) {
                const float2 f = __half22float2(*(const __half2*)&ws[h]);
                acc[q] = fmaf(f.x, v[8 * u + 2 * h], acc[q]);
                acc[q] = fmaf(f.y, v[8 * u + 2 * h + 1], acc[q]);
            }
        }
    }
#pragma unroll
    for (int o = 16, n = 4; o >= 4; o >>= 1, n >>= 1) {
        const bool up = (lane & o) != 0;
#pragma unroll
        for (int j = 0; j < n; j++) {
            const float send = up ? acc[j] : acc[j + n];
            const float keep = up ? acc[j + n] : acc[j];
            acc[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
    }
    float a = acc[0];
    a += __shfl_xor_sync(0xffffffffu, a, 2);
    a += __shfl_xor_sync(0xffffffffu, a, 1);
    if ((lane & 3) == 0) L.upart[((size_t)t * nblk + b) * L.R + c * 8 + (lane >> 2)] = a;
}

// GDN a/b gate rows (dense fp32, gdn_ab_row kernels.metal:265-273): rows [r0, r0 + nr) of [Wa; Wb], nr <= AB_ROWS,
// applied to the normed source rows (NORM / EMBED, no rotation). The weight rows, pre-multiplied by the norm weight,
// are staged before the dependency wait; the raw source rows of all tokens are then copied to shared memory with every
// copy in flight at once. Warp w takes the K range w / 8; each lane's AB_ROWS x 16 (row, token) partial sums are
// reduced across the warp by a halving butterfly (each stage keeps half of the slots), then across the warps in a
// fixed order; the per-token norm scale is applied last (the sum is linear in it). Every token's result is computed
// the same way whatever T is. Writes the pending gate inputs of this pass's parity.
constexpr int AB_ROWS = 4;

__device__ void ab_rows(const GemvParams& p, int r0, int nr, uint8_t* smem) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = p.K, NV = p.ab.nv, T = p.T;
    const ActSrc& s = p.src;
    float* s_w = (float*)smem;          // [AB_ROWS][K] weight row x norm weight
    float* xs = s_w + AB_ROWS * K;      // [T][K] source rows
    float* red = xs + (size_t)T * K;    // [8 warps][64 slots]
    float* s_r = red + 8 * 64;          // [16] norm scale per token
    uint32_t* s_id = (uint32_t*)(s_r + 16);
#pragma unroll 4
    for (int i = tid * 4; i < AB_ROWS * K; i += 1024) {
        const int q = i / K, k = i % K, row = r0 + q;
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (q < nr) {
            const float4 w = *(const float4*)(row < NV ? p.ab.wa + (size_t)row * K + k : p.ab.wb + (size_t)(row - NV) * K + k);
            const float4 g = *(const float4*)(s.w + k);
            v = make_float4(w.x * g.x, w.y * g.y, w.z * g.z, w.w * g.w);
        }
        *(float4*)(s_w + i) = v;
    }
    pdl_wait();
    if (s.mode == ACT_NORM) {
        for (int i = tid; i < T * K / 4; i += 256) cp_async16(xs + 4 * i, s.x + 4 * i);
    }
    for (int t = warp; t < T; t += 8) {
        uint32_t id = 0;
        const float r = row_scale(s, t, K, &id, false);
        if (lane == 0) {
            s_r[t] = r;
            s_id[t] = id;
        }
    }
    if (s.mode == ACT_NORM) {
        cp_async_wait_all();
        __syncthreads();
    } else {  // EMBED: bf16 embedding rows of the resolved ids
        __syncthreads();
        for (int i0 = tid; i0 < T * K; i0 += 256 * 8) {
            float a[8];
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int i = i0 + 256 * u;
                a[u] = i < T * K ? __bfloat162float(__ushort_as_bfloat16(s.xb[(size_t)s_id[i / K] * K + i % K])) : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 8; u++)
                if (i0 + 256 * u < T * K) xs[i0 + 256 * u] = a[u];
        }
        __syncthreads();
    }
    // partial sums: slot = row * 16 + token
    float v[64];
#pragma unroll
    for (int i = 0; i < 64; i++) v[i] = 0.0f;
    const int kq = K / 8;
    for (int k = warp * kq + lane; k < (warp + 1) * kq; k += 32) {
        float w[AB_ROWS];
#pragma unroll
        for (int q = 0; q < AB_ROWS; q++) w[q] = s_w[q * K + k];
#pragma unroll
        for (int t = 0; t < 16; t++)
            if (t < T) {
                const float x = xs[t * K + k];
#pragma unroll
                for (int q = 0; q < AB_ROWS; q++) v[q * 16 + t] += w[q] * x;
            }
    }
    // halving butterfly: after offsets 16, 8, 4, 2, 1 lane l holds the warp sums of slots 2 l, 2 l + 1
#pragma unroll
    for (int o = 16, n = 32; o > 0; o >>= 1, n >>= 1) {
        const bool up = (lane & o) != 0;
#pragma unroll
        for (int j = 0; j < n; j++) {
            const float send = up ? v[j] : v[j + n];
            const float keep = up ? v[j + n] : v[j];
            v[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
    }
    red[warp * 64 + 2 * lane] = v[0];
    red[warp * 64 + 2 * lane + 1] = v[1];
    __syncthreads();
    if (tid < 64) {
        const int q = tid >> 4, t = tid & 15;
        if (q < nr && t < T) {
            float a = 0.0f;
#pragma unroll
            for (int w = 0; w < 8; w++) a += red[w * 64 + tid];
            const int par = p.ab.ctl->parity;
            p.ab.pend_ab[((size_t)par * VMAX + t) * 2 * NV + r0 + q] = a * s_r[t];
        }
    }
}

// MINB: 1 for grids that fit the SMs in one wave (up to 255 registers a thread, one CTA per SM: the main loop's
// fragments and accumulators stay in registers; 2.137 -> 1.959 ms per 2B pass), 2 for larger grids (128 registers,
// two CTAs per SM, which the 4B shape's 400-720-CTA GEMVs need: 1294 against 1486 tok/s with one).
template <int NT, int GPC, int VPL, bool LORA, int MINB>
__global__ void __launch_bounds__(256, MINB) ternary_gemv_kernel(GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if ((int)blockIdx.x >= p.n_main) {  // GDN a/b gate rows: the CTAs past the GEMV's own
        pdl_trigger();
        int r0 = ((int)blockIdx.x - p.n_main) * AB_ROWS;
        if (r0 < p.ab_rows) ab_rows(p, r0, min(AB_ROWS, p.ab_rows - r0), smem);
        return;
    }
    constexpr int G = 128 / GPC;
    uint64_t* bar = (uint64_t*)smem;           // codes + scales of this CTA
    uint64_t* bar_op = (uint64_t*)(smem + 8);  // this slice's regions of the grid-built operand
    int* s_e = (int*)(smem + 128);             // [token][block] exponents, kept for the reduction
    const int kslice = p.kslice, nkc = kslice / 128;
    const int sbsz = min(VPL * 32, kslice), nb = kslice / sbsz;
    const int nsteps = sbsz / 16, nbs = op_bias_steps(sbsz, G), rsz = op_region_bytes(sbsz, G);
    const size_t codes_bytes = (size_t)kslice * 32;
    const size_t sb_bytes = (size_t)nkc * 8 * 2 * GPC * 32;
    uint8_t* s_codes = smem + GEMV_HDR;
    uint32_t* s_sb = (uint32_t*)(smem + GEMV_HDR + codes_bytes);
    uint8_t* s_op = smem + GEMV_HDR + codes_bytes + sb_bytes;  // regions [nb][NT]
    const bool prebuilt = p.src.opbuf != nullptr;  // operand built by the whole grid (grid_build)

    const int rb = p.csplit ? blockIdx.x / p.nsplit : blockIdx.x % p.nrb;
    const int ks = p.csplit ? blockIdx.x % p.nsplit : blockIdx.x / p.nrb;  // with csplit: the CTA's cluster rank
    const int nkc_all = p.K / 128;
    if (tid == 0) {
        mbar_init(bar, 1);
        mbar_init(bar_op, 1);
        fence_proxy_async_smem();
    }
    __syncthreads();
    pdl_trigger();
    if (tid == 0) {
        mbar_expect_tx(bar, (uint32_t)(codes_bytes + sb_bytes));
        bulk_g2s(s_codes, p.codes + ((size_t)rb * nkc_all + (size_t)ks * nkc) * 8 * 512, (uint32_t)codes_bytes, bar);
        bulk_g2s(s_sb, (const uint8_t*)p.sb + ((size_t)rb * nkc_all + (size_t)ks * nkc) * 8 * 2 * GPC * 32,
                 (uint32_t)sb_bytes, bar);
    }
    pdl_wait();
    float res[8];  // residual rows of this row block (element e = tid + 256 i of [T][128]), read early
    if (p.o.add) {
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int e = tid + 256 * i;
            res[i] = e < 128 * p.T ? p.o.out[(size_t)(e >> 7) * p.O + rb * 128 + (e & 127)] : 0.0f;
        }
    }
    if (prebuilt) {
        __shared__ int s_ok;
        grid_build<VPL, GPC>(p, s_op, &s_ok);
        if (tid == 0) {  // the slice's regions: nb blocks of NT tiles (the buffer holds 4 tiles per block)
            mbar_expect_tx(bar_op, (uint32_t)(nb * NT * rsz));
            for (int b = 0; b < nb; b++)
                bulk_g2s(s_op + (size_t)b * NT * rsz, p.src.opbuf + ((size_t)(ks * nb + b) * 4) * rsz,
                         (uint32_t)(NT * rsz), bar_op);
            grid_build_release(p);
        }
    }
    if (!prebuilt) build_operand<VPL, GPC>(p, ks, sbsz, nb, NT, s_op, rsz);
    __syncthreads();
    const bool ok = mbar_wait_bounded(bar, 0) && (!prebuilt || mbar_wait_bounded(bar_op, 0));
    if (__syncthreads_or(!ok)) {
        if (tid == 0) atomicOr(p.o.err, ERR_MBAR_TIMEOUT);
        mbar_wait_bounded(bar, 0, 1u << 20);
        if (prebuilt) mbar_wait_bounded(bar_op, 0, 1u << 20);
        if (p.csplit) {  // both cluster barrier phases of the split sum, so that no other rank waits for this one
            cluster_sync_all();
            cluster_arrive();
            cluster_wait();
        }
        return;
    }
    if (tid < p.T * nb) {  // exponents to the header (the regions are overwritten by the reduction)
        const int t = tid / nb, b = tid % nb;
        s_e[t * 4 + b] = ((const int*)(s_op + (size_t)(b * NT + (t >> 2)) * rsz + (nsteps + nbs) * 256))[t & 3];
    }

    const int rg = warp >> 2, kw = warp & 3;
    const int g = lane >> 2, t4 = lane & 3;
    const int nkc_w = nkc / 4;
    const int bw = (kw * (kslice / 4)) / sbsz;  // this warp's block (its k-quarter lies inside one)
    float acc[4][NT][4];
#pragma unroll
    for (int m = 0; m < 4; m++)
#pragma unroll
        for (int n = 0; n < NT; n++)
#pragma unroll
            for (int i = 0; i < 4; i++) acc[m][n][i] = 0.0f;

    const uint32_t MAGIC = 0x64006400u, NEG1024 = 0xE400E400u;
    // B fragments of k16 step (slice-local) st for tile n: region (bw, n), step st - bw * nsteps
    const uint2* s_b2 = (const uint2*)(s_op + (size_t)bw * NT * rsz) - (size_t)bw * nsteps * 32;
    const size_t tile_stride = (size_t)rsz / 8;  // uint2 between tiles
    for (int c = 0; c < nkc_w; c++) {
        const int kcl = kw * nkc_w + c;
        uint4 cw[4];
#pragma unroll
        for (int m = 0; m < 4; m++) cw[m] = ((const uint4*)s_codes)[(size_t)(kcl * 8 + rg * 4 + m) * 32 + lane];
#pragma unroll
        for (int gi = 0; gi < GPC; gi++) {
            uint32_t s2lo[4], s2hi[4], n2lo[4], n2hi[4];
#pragma unroll
            for (int m = 0; m < 4; m++) {
                uint32_t u = s_sb[(((size_t)(kcl * 8 + rg * 4 + m) * 2 + 0) * GPC + gi) * 8 + g];
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
                for (int n = 0; n < NT; n++) bb[n] = s_b2[n * tile_stride + (size_t)(kcl * 8 + f) * 32 + lane];
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
    // bias step: A = 64 b for this warp's groups (columns [o0, o0 + ngw) of its block's bias step bs), B = group
    // sums / 64
    {
        const int ngw = kslice / 4 / G;
        const int gq0 = (kw * (kslice / 4) - bw * sbsz) / G;  // first group of the warp, block-relative
        const int bs = gq0 >> 4, o0 = gq0 & 15;
        const int gbase = bw * sbsz / G + bs * 16;  // slice-local group of column 0
        uint2 bb[NT];
#pragma unroll
        for (int n = 0; n < NT; n++)
            bb[n] = ((const uint2*)(s_op + (size_t)(bw * NT + n) * rsz + (size_t)(nsteps + bs) * 256))[lane];
        const int cols[4] = {2 * t4, 2 * t4 + 1, 2 * t4 + 8, 2 * t4 + 9};
#pragma unroll
        for (int m = 0; m < 4; m++) {
            uint32_t u[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                int c = cols[i];
                u[i] = 0;
                if (c >= o0 && c < o0 + ngw) {
                    int gl = gbase + c;  // slice-local group
                    int kc = gl / GPC, gi = gl % GPC;
                    u[i] = s_sb[(((size_t)(kc * 8 + rg * 4 + m) * 2 + 1) * GPC + gi) * 8 + g];
                }
            }
            uint32_t a0 = __byte_perm(u[0], u[1], 0x5410), a1 = __byte_perm(u[0], u[1], 0x7632);
            uint32_t a2 = __byte_perm(u[2], u[3], 0x5410), a3 = __byte_perm(u[2], u[3], 0x7632);
#pragma unroll
            for (int n = 0; n < NT; n++) mma_f16(acc[m][n], a0, a1, a2, a3, bb[n].x, bb[n].y);
        }
    }
    // in-CTA reduction over the 4 k-quarters, fixed order; partials in units of x (2^-E applied)
    __syncthreads();
    float* red = (float*)(smem + GEMV_HDR);  // [kw 4][rg 2][m 4][NT][2][32]
#pragma unroll
    for (int m = 0; m < 4; m++)
#pragma unroll
        for (int n = 0; n < NT; n++) {
            size_t base = ((((size_t)kw * 2 + rg) * 4 + m) * NT + n) * 2;
            red[(base + 0) * 32 + lane] = acc[m][n][0] + acc[m][n][1];
            red[(base + 1) * 32 + lane] = acc[m][n][2] + acc[m][n][3];
        }
    __syncthreads();
    const int T = p.T, O = p.O;
    const size_t quarter = (size_t)2 * 4 * NT * 2 * 32;
    float* fin = red + 4 * quarter;  // [T][128] final values when this CTA holds the whole K range
    int blk_of_q[4];
#pragma unroll
    for (int q = 0; q < 4; q++) blk_of_q[q] = q * (kslice / 4) / sbsz;
    for (int e = tid; e < (int)quarter; e += 256) {
        int ln = e & 31;
        int r = e >> 5;
        int which = r & 1;
        r >>= 1;
        int n = r % NT;
        r /= NT;
        int m = r & 3;
        int rgi = r >> 2;
        int token = n * 4 + (ln & 3);
        if (token >= T) continue;
        int rloc = rgi * 64 + m * 16 + (ln >> 2) + 8 * which;
        // quarter q of the slice lies in Hadamard block q * kslice / (4 * HB) (its operand's exponent)
        const int* et = s_e + token * 4;
        float v = red[e] * pow2f(-et[blk_of_q[0]]);
        v += red[quarter + e] * pow2f(-et[blk_of_q[1]]);
        v += red[2 * quarter + e] * pow2f(-et[blk_of_q[2]]);
        v += red[3 * quarter + e] * pow2f(-et[blk_of_q[3]]);
        if (p.nsplit == 1 || p.csplit) fin[token * 128 + rloc] = v;
        else p.o.partial[((size_t)ks * T + token) * O + rb * 128 + rloc] = v;
    }
    __shared__ int s_last;
    if (p.csplit) {
        // The K-splits of this row block are the ranks of one cluster, each with its sums in its own shared memory
        // (fin). Rank 0 reads every rank's value of its elements over the cluster's shared memory and sums them in
        // split order (the same sums, in the same order, as the partial-buffer path below, without its global
        // atomic and the L2 round trips of the last CTA's loads); then it releases the other ranks, whose shared
        // memory must stay valid until it has read it.
        cluster_sync_all();
        if (ks != 0) {
            cluster_arrive();
            cluster_wait();
            return;
        }
        constexpr int EPT = VMAX * 128 / 256;
        float v[EPT];
#pragma unroll
        for (int i = 0; i < EPT; i++) {
            const int e = tid + 256 * i;
            float pv[8];
#pragma unroll
            for (int s = 0; s < 8; s++) pv[s] = e < 128 * T && s < p.nsplit ? ld_cluster_f32(fin + e, s) : 0.0f;
            v[i] = 0.0f;
#pragma unroll
            for (int s = 0; s < 8; s++)
                if (s < p.nsplit) v[i] += pv[s];
        }
        cluster_arrive();  // the other ranks' shared memory is read
#pragma unroll
        for (int i = 0; i < EPT; i++)
            if (tid + 256 * i < 128 * T) fin[tid + 256 * i] = v[i];
    } else if (p.nsplit > 1) {
        __syncthreads();  // every partial of this CTA is stored
        if (tid == 0) {
            // release: this CTA's partials before its count; acquire: the other CTAs' partials after theirs
            unsigned old;
            asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(old) : "l"(p.o.counters + rb) : "memory");
            s_last = old == (unsigned)(p.nsplit - 1);
        }
        __syncthreads();
        if (!s_last) return;
        // The other CTAs' partials: a thread's elements e = tid + 256 i (up to 8 of the T x 128 block) and 8 splits
        // at a time have all their loads in flight together (one L2 round trip per 8 splits, not one per element);
        // each element is summed in split order.
        constexpr int EPT = VMAX * 128 / 256;
        float v[EPT];
#pragma unroll
        for (int i = 0; i < EPT; i++) v[i] = 0.0f;
        for (int s0 = 0; s0 < p.nsplit; s0 += 8) {
            float pv[EPT][8];
#pragma unroll
            for (int i = 0; i < EPT; i++) {
                const int e = tid + 256 * i;
                const float* src = p.o.partial + (size_t)(e >> 7) * O + rb * 128 + (e & 127);
#pragma unroll
                for (int s = 0; s < 8; s++)
                    pv[i][s] = e < 128 * T && s0 + s < p.nsplit ? __ldcg(src + (size_t)(s0 + s) * T * O) : 0.0f;
            }
#pragma unroll
            for (int i = 0; i < EPT; i++)
#pragma unroll
                for (int s = 0; s < 8; s++)
                    if (s0 + s < p.nsplit) v[i] += pv[i][s];
        }
#pragma unroll
        for (int i = 0; i < EPT; i++)
            if (tid + 256 * i < 128 * T) fin[tid + 256 * i] = v[i];
        if (tid == 0) p.o.counters[rb] = 0;
    }
    __syncthreads();
    // LoRA: u = A . x of this row block's member (u[t][j] = sum over the Hadamard blocks of lora_a_kernel's partials,
    // in block order; that kernel completed before this one's dependency wait)
    const LoraArgs& L = p.lora;
    const int lr = L.r;
    float* s_u = fin + 128 * T;  // [T][lr]
    const uint16_t* lb = nullptr;
    if (LORA) {
        const int row0 = rb * 128, mem = (row0 >= L.m1) + (row0 >= L.m2), nblk = p.K / (VPL * 32);
        for (int i = tid; i < T * lr; i += 256) {
            const int t = i / lr, j = i % lr;
            const float* src = L.upart + (size_t)t * nblk * L.R + mem * lr + j;
            float a = 0.0f;
            for (int b = 0; b < nblk; b++) a += __ldcg(src + (size_t)b * L.R);
            s_u[i] = a;
        }
        lb = L.b + (size_t)row0 * lr;
        __syncthreads();
    }
    // output (store or residual add, then the LoRA up projection, as store_post kernels.metal:257-262) and the sums
    // of squares of the new rows
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int e = tid + 256 * i;
        if (e < 128 * T) {
            float v = fin[e];
            if (p.o.add) v = res[i] + v;
            if (LORA) {
                const uint4* bp = (const uint4*)(lb + (size_t)(e & 127) * lr);
                const float* ut = s_u + (e >> 7) * lr;
                float a = 0.0f;
                for (int j0 = 0; j0 < lr; j0 += 8) {
                    const uint4 w = __ldg(bp + j0 / 8);
                    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                    for (int h = 0; h < 4; h++) {
                        const float2 f = __half22float2(*(const __half2*)&ws[h]);
                        a = fmaf(ut[j0 + 2 * h], f.x, a);
                        a = fmaf(ut[j0 + 2 * h + 1], f.y, a);
                    }
                }
                v = v + a;
            }
            p.o.out[(size_t)(e >> 7) * O + rb * 128 + (e & 127)] = v;
            fin[e] = v;
        }
    }
    if (p.o.ss_out) {
        __syncthreads();
        for (int token = warp; token < T; token += 8) {
            float a = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                float x = fin[token * 128 + i * 32 + lane];
                a += x * x;
            }
            a = warp_sum(a);
            if (lane == 0) p.o.ss_out[rb * VMAX + token] = a;
        }
    }
}

// tpc: grid-build tasks per CTA (their scratch regions share the operand's space), 0 without a grid build.
static size_t gemv_smem(int kslice, int nt, int group, int T, int K, int ab, int hb, int tpc, int lora_r) {
    int gpc = 128 / group;
    int sbsz = hb < kslice ? hb : kslice;
    size_t ops = (size_t)nt * (kslice / sbsz) * op_region_bytes(sbsz, group);
    if (hb == 2048 && !tpc) ops += (QX_FLOATS + 4) * 4;  // build_operand_quarters' exchange after the regions
    // build_quarters: two task regions, the exchanged values (hb floats per group), the quarter maxima
    const size_t scratch = tpc ? 2 * (size_t)op_region_bytes(hb, group) + (2 * (size_t)hb + 8) * 4 : 0;
    size_t main = GEMV_HDR + (size_t)kslice * 32 + (size_t)(kslice / 128) * 8 * 2 * gpc * 32 + (ops > scratch ? ops : scratch);
    size_t red = GEMV_HDR + (size_t)4 * 2 * 4 * nt * 2 * 32 * 4 + (size_t)T * (128 + lora_r) * 4;
    size_t abs_ = ab ? ((size_t)(AB_ROWS + T) * K + 8 * 64 + 32) * 4 : 0;
    size_t s = main > red ? main : red;
    return s > abs_ ? s : abs_;
}

static int grid_build_tpc(const TernaryMat& m, int T, int hb) {
    const int ntask = T * (m.K / hb), ncta = (m.O / 128) * m.nsplit;
    return (ntask + ncta - 1) / ncta;
}

template <int NT, int GPC, int MINB>
static const void* gemv_fn_vpl(int hb, bool lora) {
    if (lora)  // LoRA variants: 512- and 1024-point blocks (bcu_set_lora checks)
        return hb == 512 ? (const void*)ternary_gemv_kernel<NT, GPC, 16, true, MINB>
                         : (const void*)ternary_gemv_kernel<NT, GPC, 32, true, MINB>;
    if (hb == 512) return (const void*)ternary_gemv_kernel<NT, GPC, 16, false, MINB>;
    if (hb == 1024) return (const void*)ternary_gemv_kernel<NT, GPC, 32, false, MINB>;
    return (const void*)ternary_gemv_kernel<NT, GPC, 64, false, MINB>;
}
template <int NT>
static const void* gemv_fn_gpc(int group, int hb, bool lora, bool wide) {
    if (wide) return group == 64 ? gemv_fn_vpl<NT, 2, 1>(hb, lora) : gemv_fn_vpl<NT, 1, 1>(hb, lora);
    return group == 64 ? gemv_fn_vpl<NT, 2, 2>(hb, lora) : gemv_fn_vpl<NT, 1, 2>(hb, lora);
}
// The kernel for nt column tiles (wide: the one-CTA-per-SM register budget), its shared-memory limit raised on this
// device.
static const void* gemv_fn(int nt, int group, int hb, bool lora, bool wide) {
    const void* fn = nt == 1 ? gemv_fn_gpc<1>(group, hb, lora, wide)
                   : nt == 2 ? gemv_fn_gpc<2>(group, hb, lora, wide)
                   : nt == 3 ? gemv_fn_gpc<3>(group, hb, lora, wide)
                             : gemv_fn_gpc<4>(group, hb, lora, wide);
    raise_smem_limit(fn, 220 * 1024);
    return fn;
}

// SMs of the current device (cached per device).
static int device_sms() {
    static std::mutex mu;
    static int cache[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> g(mu);
    if (dev >= 0 && dev < 64 && !cache[dev]) cudaDeviceGetAttribute(&cache[dev], cudaDevAttrMultiProcessorCount, dev);
    return dev >= 0 && dev < 64 ? cache[dev] : 148;
}

void raise_smem_limit(const void* fn, int bytes) {
    static std::mutex mu;
    static std::set<std::pair<const void*, int>> raised;  // (kernel, device): the attribute is per device
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> g(mu);
    if (raised.insert({fn, dev}).second) cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

int gemv_grid(const TernaryMat& m, int ab_rows) { return (m.O / 128) * m.nsplit + (ab_rows + AB_ROWS - 1) / AB_ROWS; }

// Split sums through cluster shared memory (1, default) or the global partial buffer (0); a test hook compares them.
static std::atomic<int> g_gemv_clusters{1};

// Whether `nclusters` clusters of `csize` CTAs of kernel fn (256 threads, smem bytes of dynamic shared memory) are
// resident on the current device at once, as the grid-built operand's wait needs (a cluster's CTAs share one GPC).
// Cached per (kernel, shared memory, cluster size, clusters, device).
static bool gemv_clusters_fit(const void* fn, size_t smem, int csize, int nclusters) {
    static std::mutex mu;
    static std::map<std::tuple<const void*, size_t, int, int, int>, bool> cache;
    int dev = 0;
    cudaGetDevice(&dev);
    const auto key = std::make_tuple(fn, smem, csize, nclusters, dev);
    {
        std::lock_guard<std::mutex> g(mu);
        auto it = cache.find(key);
        if (it != cache.end()) return it->second;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(csize * nclusters));
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)csize;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    const bool ok = cudaOccupancyMaxActiveClusters(&n, fn, &cfg) == cudaSuccess && n >= nclusters;
    if (!ok) cudaGetLastError();  // a refused query leaves no sticky error behind
    std::lock_guard<std::mutex> g(mu);
    cache[key] = ok;
    return ok;
}

// Whether this GEMV's CTAs can build its operand together (grid_build): every CTA of the grid resident at once
// (they wait for one another) and at most 2 tasks (one per group of four warps) per CTA.
bool gemv_coresident(const TernaryMat& m, int T, int ab_rows, int hb, int num_sms, int lora_r) {
    const int nt = (2 * T + 7) / 8;
    const int tpc = grid_build_tpc(m, T, hb);
    // at most one task per group of four warps; the buffer's regions hold whole blocks
    if (tpc > 2 || hb <= 0 || hb > m.kslice) return false;
    const void* fn = gemv_fn(nt, m.group, hb, lora_r > 0, gemv_grid(m, ab_rows) <= num_sms);
    const size_t smem = gemv_smem(m.kslice, nt, m.group, T, m.K, ab_rows > 0, hb, tpc, lora_r);
    if (smem > 220 * 1024) return false;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, 256, smem) != cudaSuccess) return false;
    return (long)gemv_grid(m, ab_rows) <= (long)per_sm * num_sms;
}

void launch_ternary_gemv(const TernaryMat& m, const ActSrc& src, int T, const GemvOut& o, const AbArgs* ab,
                         cudaStream_t st, const LoraArgs* lora) {
    GemvParams p;
    p.codes = (const uint8_t*)m.codes;
    p.sb = m.sb;
    p.src = src;
    p.o = o;
    p.ab = ab ? *ab : AbArgs();
    p.lora = lora ? *lora : LoraArgs();
    p.O = m.O;
    p.K = m.K;
    p.group = m.group;
    p.kslice = m.kslice;
    p.nsplit = m.nsplit;
    p.T = T;
    p.n_main = (m.O / 128) * m.nsplit;
    p.ab_rows = ab ? 2 * ab->nv : 0;
    p.nrb = m.O / 128;
    int hb = src.HB > 0 ? src.HB : 512;  // unrotated sources use 512-element blocks for their exponents
    int nt = (2 * T + 7) / 8;
    size_t smem = gemv_smem(m.kslice, nt, m.group, T, m.K, p.ab_rows > 0, hb,
                            src.opbuf ? grid_build_tpc(m, T, hb) : 0, p.lora.a ? p.lora.r : 0);
    if (p.lora.a) {  // the LoRA A partials first (lora_a_kernel); hb is 512 or 1024 here (bcu_set_lora checks)
        const int tasks = T * (m.K / hb) * (p.lora.R / 8);
        void* largs[] = {&p};
        launch_pdl(hb == 512 ? (const void*)lora_a_kernel<16> : (const void*)lora_a_kernel<32>,
                   dim3((unsigned)((tasks + 7) / 8)), dim3(256), 0, st, largs);
    }
    const void* fn = gemv_fn(nt, m.group, hb, p.lora.a != nullptr, gemv_grid(m, p.ab_rows) <= device_sms());
    void* args[] = {&p};
    const int n_ab = (p.ab_rows + AB_ROWS - 1) / AB_ROWS;
    // a row block's K-splits as one cluster (at most 8, the portable size) when every cluster is resident at once
    p.csplit = 0;
    if (m.nsplit > 1 && m.nsplit <= 8 && g_gemv_clusters.load(std::memory_order_relaxed)) {
        const int ncl = p.nrb + (n_ab + m.nsplit - 1) / m.nsplit;  // the a/b gate CTAs padded to whole clusters
        if (gemv_clusters_fit(fn, smem, m.nsplit, ncl)) {
            p.csplit = 1;
            launch_pdl_cluster(fn, dim3((unsigned)(ncl * m.nsplit)), m.nsplit, smem, st, args);
            return;
        }
    }
    launch_pdl(fn, dim3((unsigned)(p.n_main + n_ab)), dim3(256), smem, st, args);
}

}  // namespace bcu

// Test hook (not in the ABI header): 0 = split GEMVs sum through the global partial buffer, 1 = through cluster
// shared memory where the clusters fit (the default). Both give the same bits.
extern "C" int bcu_gemv_set_clusters(int on) {
    bcu::g_gemv_clusters.store(on ? 1 : 0);
    return 0;
}

namespace bcu {

}  // namespace bcu
