// kernels.h — host-side launch wrappers of the sm_100a kernels (one translation unit per kernel family).
// Every wrapper enqueues on `stream` with Programmatic Dependent Launch allowed, so consecutive kernels of a pass
// overlap their prologue (weight prefetch) with the previous kernel's tail.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "ctl.h"

namespace bcu {

struct Ctl;

// ------------------------------------------------------------------------------------------------ ternary linear
// Device layout of one packed ternary matrix (O rows x K codes), built by repack_ternary from the MLX pack:
//   codes : [O/128][K/128][8 m-tiles][32 lanes][16 B]; lane (g = l/4, t = l%4) word q holds the 16 codes of rows
//           g and g+8 at k = 32q + {0,8,16,24} + 2t + {0,1}, so one LDS.128 gives a lane its A-fragment codes for
//           8 mma k16-steps; slot h (bits 2h and 16+2h) decodes with a mask at bit 2*(h%4) of w or w >> 8.
//   sb    : [O/128][K/128][8][2][128/group][8 g] u32 = half2(v[row g], v[row g+8]) with v = s (first half) and
//           v = 64 * b (second half; b = the MLX bias, or -s for the reference pack whose weight is s*(code-1))
struct TernaryMat {
    const void* codes = nullptr;
    const uint32_t* sb = nullptr;
    int O = 0, K = 0, group = 64;
    int kslice = 0, nsplit = 1;  // split-K plan: kslice in {512, 1024, 2048}
};

size_t ternary_codes_bytes(int O, int K);
size_t ternary_sb_bytes(int O, int K, int group);
// Converts MLX-packed device arrays (u32 [O][K/16], fp16 [O][K/group] scales, optional biases) into the layout above.
void repack_ternary(const uint32_t* w_mlx, const uint16_t* s, const uint16_t* b, int O, int K, int group,
                    void* codes, uint32_t* sb, cudaStream_t st);
void plan_ternary(TernaryMat& m, int num_sms, int min_kslice = 512);

// Where a GEMV's activation rows come from. Each CTA builds the tensor-core operand of its own K-slice in shared
// memory: the pre-rotation value x_k of the mode, times the input's signs, Walsh-Hadamard transformed in blocks of
// HB, then split into fp16 hi/lo parts (producer steps of the reference: norm_rotate, gated_norm_rotate,
// swiglu_rotate, gate_rotate, kernels.metal:118-226).
enum ActMode : int {
    ACT_NORM = 0,    // x = h * rsqrt(mean(h^2) + eps) * w, mean from the sums of squares `ss` ([nss][VMAX])
    ACT_EMBED = 1,   // as NORM over h = bf16 embedding row of the token (CTA 0 also writes h)
    ACT_GATED = 2,   // GDN output: per 128-wide head (((z * y) * rsqrt(mean(y^2) + eps)) * w) * sigmoid(z)
    ACT_SWIGLU = 3,  // x = (g * u) * sigmoid(g), g and u the two halves of a [T][2K] row
    ACT_GATE = 4,    // attention output: x = attn * sigmoid(gate half of the q projection)
    ACT_EXT = 5      // x given (bf16 or fp32), no normalisation
};

struct ActSrc {
    int mode = ACT_EXT;
    const float* x = nullptr;      // NORM: h [T][K]; GATED: y [T][K]; SWIGLU: [T][2K]; GATE: attn [T][K]; EXT fp32
    const uint16_t* xb = nullptr;  // EMBED: bf16 table [vocab][K]; EXT: bf16 [T][K]
    const float* x2 = nullptr;     // GATED: qkvz rows (z at off2); GATE: q projection rows (ld2)
    int ld2 = 0, off2 = 0;
    const float* w = nullptr;      // NORM/EMBED: [K]; GATED: [128]
    const float* signs = nullptr;  // [K] or null
    const float* ss = nullptr;     // NORM: [nss][VMAX] sums of squares of h by row block
    int nss = 0;
    const Ctl* ctl = nullptr;      // EMBED: token ids
    float* h_out = nullptr;        // EMBED: residual rows (written by CTA 0)
    int HB = 512, vocab = 0;
    // != null: the GEMV's CTAs build the whole operand once, together, in this global buffer ([K / HB blocks]
    // [4 tiles][region]) and then copy their slices from it; op_counters: 2 zeroed words. Needs every CTA of the
    // grid resident at once (gemv_coresident). Null: each CTA builds its own slice's operand.
    uint8_t* opbuf = nullptr;
    unsigned* op_counters = nullptr;
};


struct GemvOut {
    float* out = nullptr;        // [T][O]
    int add = 0;                 // 1: out += W.x (residual)
    float* ss_out = nullptr;     // != null: [O/128][VMAX] sums of squares of the new out rows (next RMSNorm)
    float* partial = nullptr;    // split-K partials [nsplit][T][O]
    unsigned* counters = nullptr;// [O/128], zero between launches
    int* err = nullptr;
};

// The GDN a/b gate projection (gdn_ab, kernels.metal:504-510) rides along the qkvz GEMV as extra CTAs.
struct AbArgs {
    const float* wa = nullptr;   // [NV][d]
    const float* wb = nullptr;
    float* pend_ab = nullptr;    // [2][VMAX][2NV] (written at the pass parity)
    const Ctl* ctl = nullptr;
    int nv = 0;
};

// LoRA of one packed linear (lora.rs:1-5; fused like norm_rotate's A rows and the matmuls' B epilogue,
// kernels.metal:70-116, 251-262): y += B . (A . x) on the linear's unrotated input x. A of the members stacked
// (R = members x r rows), fp16, in the operand builders' lane order [K / HB][R][32 lanes][HB / 32]; B fp16 [O][r]
// (alpha / r and the scale folded in); member i owns rows [m[i], m[i + 1]) of O and u rows [i r, (i + 1) r).
struct LoraArgs {
    const uint16_t* a = nullptr;  // null: no LoRA
    const uint16_t* b = nullptr;
    float* upart = nullptr;       // [VMAX][K / HB][R] partial A . x per (token, Hadamard block)
    int R = 0, r = 0;             // r a multiple of 8 (the adapter's rank, zero-padded)
    int m1 = 0, m2 = 0;           // member starts 1, 2 (O when absent)
};

// y[T][O] (+)= W . rotate(x) (+ LoRA) for T <= 16 rows.
void launch_ternary_gemv(const TernaryMat& m, const ActSrc& src, int T, const GemvOut& o, const AbArgs* ab,
                         cudaStream_t st, const LoraArgs* lora = nullptr);
int gemv_grid(const TernaryMat& m, int ab_rows);
// Whether every CTA of the GEMV fits on the GPU at once (needed when its CTAs build the operand together).
bool gemv_coresident(const TernaryMat& m, int T, int ab_rows, int hb, int num_sms, int lora_r = 0);

// ------------------------------------------------------------------------------------------------ GatedDeltaNet
// One launch per GDN layer: conv (with the deferred conv-state commit) + gated delta rule (with the deferred replay)
// for CTA = (value head, 16 dv rows). Inputs are staged in shared memory, so the sequential rows run without global
// loads on the critical path.
// Raises a kernel's dynamic shared-memory limit on the current device, once per (kernel, device); thread-safe.
void raise_smem_limit(const void* fn, int bytes);

struct GdnArgs {
    const Ctl* ctl;
    const float* qkvz;     // [T][C + gw] GEMV output (qkv first)
    const float* convw;    // [C][4]
    const float* a_log;    // [NV]
    const float* dt_bias;  // [NV]
    float* conv_state;     // [3][C] committed
    float* gdn_state;      // [NV][128][128] committed
    float* pend_qkv;       // [2][VMAX][C] raw qkv rows (conv commit of the next pass)
    float* pend_qkvc;      // [2][VMAX][C] conv outputs (replay)
    float* pend_ab;        // [2][VMAX][2NV] gate inputs (replay; written by the qkvz GEMV)
    float* y;              // [T][NV*128]
    int C, NK, NV, T;
    int prefetch;          // read what the previous pass left before the dependency wait (pass graphs only)
};
void launch_gdn_layer(const GdnArgs& a, cudaStream_t st);

// The prefill chunk's gated delta rule in chunks of 64 rows (gdn_chunk.cu): state advanced by all T rows, outputs of
// every row. ws: gdn_chunk_workspace_bytes(T, NV) of device memory.
size_t gdn_chunk_workspace_bytes(int T, int NV);
void launch_gdn_chunked(const float* q, const float* k, const float* v, const float* a_in, const float* b_in,
                        const float* a_log, const float* dt_bias, float* state, float* y, int T, int NK, int NV,
                        float* ws, cudaStream_t st);

// Standalone verify step with rollback (graded config 2).
void launch_gdn_verify(const float* q, const float* k, const float* v, const float* a_in, const float* b_in,
                       const float* a_log, const float* dt_bias, float* state, float* y, int T, int NK, int NV,
                       int n, cudaStream_t st);

// ------------------------------------------------------------------------------------------------ attention
// Split-K causal GQA over the cache with the q/k prep (RMSNorm + mRoPE) and the KV write fused in; the last split CTA
// of each (row, kv head) merges the partials and writes the attention output rows.
struct AttnArgs {
    const Ctl* ctl;
    const float* qkv;      // [T][ld]: q (with gates, 2*aw), k (kvw), v (kvw)
    const float* qn;       // [256]
    const float* kn;       // [256]
    const float* inv_freq; // [rot/2]
    float* kc;             // [ctx][KV][256]
    float* vc;
    float* part;           // [T][H][NSPLIT][258]: per split the running maximum, sum and partial output
    float* out;            // [T][H*256]
    int H, KV, rot, T, ld, ctx;
    int nsplit = NSPLIT_ATTN;       // key splits per (row, kv head), 1..NSPLIT_ATTN
    // prefill mode: queries prepared by pf_attn_prep ([T][H][256]), every key of rows [0, off0 + T) in the cache,
    // row t at position off0 + t (part [T][H][nsplit][258])
    const float* qprep = nullptr;
    int off0 = 0;
};
// The split kernel, then attn_merge_kernel (two launches).
void launch_attn(const AttnArgs& a, cudaStream_t st);
// Prefill chunk attention on the tensor cores (attn_prefill.cu): queries prepared [T][H][256], every key of positions
// [0, off0 + T) in the cache, out [T][H * 256]; for query heads per kv head dividing 32.
bool attn_prefill_supported(int H, int KV);
void launch_attn_prefill(const float* qprep, const float* kc, const float* vc, float* out, int T, int H, int KV,
                         int off0, cudaStream_t st);

// ------------------------------------------------------------------------------------------------ head + accept
// bf16 tied head in mma fragment order: [V/16][d/16][32 lanes][4] u32.
void repack_head_bf16(const uint16_t* table, int V, int d, uint32_t* out, cudaStream_t st);

struct HeadArgs {
    Ctl* ctl;
    const uint32_t* w;       // repacked head
    const float* h;          // [T][d] residual rows
    const float* ss;         // [nss][VMAX] sums of squares of h by row block
    int nss;
    const float* norm;       // final norm weight [d]
    float* logits;           // [T][V] (written when ctl->in.keep_logits)
    float* pv;               // [grid][T] partial maxima
    int* pi;                 // [grid][T]
    unsigned* counter;       // 1 zeroed uint
    int V, d, T;
    int stages = 0;          // 4-KB table units in flight per warp (set by launch_head)
};
void launch_head(const HeadArgs& a, int NT, int grid, cudaStream_t st);
// Ternary tied table (the reference's format): the head is a ternary GEMV into logits, then this argmax + accept
// kernel (uses ctl, logits, pv, pi, counter, V, T).
void launch_head_argmax(const HeadArgs& a, int grid, cudaStream_t st);

// Embedding rows of the ternary tied table (embed, kernels.metal:230-246) into the residual rows, with their
// row-block sums of squares for the first GEMV's RMSNorm.
struct EmbedArgs {
    Ctl* ctl;
    const uint32_t* w;       // MLX pack [V][d/16]
    const uint16_t* s;       // fp16 scales [V][d/group]
    const uint16_t* b;       // fp16 biases or null (the reference pack: weight = s (code - 1))
    const float* signs;      // [d] or null
    float* h;                // [T][d]
    float* ss;               // [d/128][VMAX]
    int V, d, group, T;
};
void launch_embed_ternary(const EmbedArgs& a, cudaStream_t st);
// Largest hidden size whose head operand fits beside one ring stage (16-row tiles of 4 tokens, 16 rows at T = 16).
constexpr int HEAD_MAX_HIDDEN = 3072;

// Prefill GEMM on tcgen05 (gemm.cu): y[M][O] = W . x for any M. gemm_pack converts the MLX pack (device arrays) once;
// gemm_run prepares the activation tiles (bop: gemm_act_bytes, ex: M ints) and runs the GEMM on the stream.
size_t gemm_w_bytes(int O, int K);
size_t gemm_bias_bytes(int O, int K, int G);
size_t gemm_act_bytes(int M, int K, int G);
void gemm_pack(const uint32_t* w, const uint16_t* s, const uint16_t* b, int O, int K, int G, uint8_t* wt,
               uint8_t* abias, cudaStream_t st);
int gemm_bias_chunks(int K, int G);
void gemm_prep_only(const float* x, int M, int K, int G, uint8_t* bop, int* ex, cudaStream_t st);
// x null: bop and ex already hold the activation tiles (written by the prefill producers).
cudaError_t gemm_run(const uint8_t* wt, const uint8_t* abias, int O, int K, int G, const float* x, int M, uint8_t* bop,
                     int* ex, float* y, int* err, int num_sms, cudaStream_t st);

// ------------------------------------------------------------------------------------------------ batched prefill
// Producer kernels of the prefill chunk (prefill.cu): one row per CTA, x of the mode, signs, Walsh-Hadamard in blocks
// of hb, written as the GEMM's activation tiles.
enum PfMode : int { PF_NORM = 0, PF_GATED = 1, PF_GATE = 2, PF_SWIGLU = 3 };
struct PfRowArgs {
    int mode = PF_NORM, D = 0, ld2 = 0;
    float* h = nullptr;            // NORM: [M][D] residual rows (updated when add != null)
    const float* add = nullptr;    // NORM: [M][D] added to h first, or null
    const float* src = nullptr;    // GATED: y [M][D]; GATE: attn [M][D]; SWIGLU: [M][2D]
    const float* src2 = nullptr;   // GATED: z rows; GATE: q projection rows (row stride ld2)
    const float* w = nullptr;      // NORM: [D]; GATED: [128]
    const float* signs = nullptr;  // [D] or null
    float* xn = nullptr;           // NORM: unrotated normed rows, or null
    uint8_t* bop = nullptr;        // the GEMM's activation tiles (gemm_act_bytes(M, D, G)) and exponents ex [M]
    int* ex = nullptr;
    int G = 0, nbias = 0;          // group size of the GEMM's weights, its bias chunks (gemm_bias_chunks(D, G))
};
void launch_pf_rows(const PfRowArgs& a, int M, int hb, cudaStream_t st);
void launch_pf_embed(const uint32_t* ids, int M, int V, int d, const uint16_t* bf16, const uint32_t* tw,
                     const uint16_t* ts, const uint16_t* tb, const float* signs, int group, float* h, int* err,
                     cudaStream_t st);
void launch_pf_gdn_ab(const float* wa, const float* wb, const float* xn, float* ga, float* gb, int NV, int d, int M,
                      cudaStream_t st);
void launch_pf_gdn_conv(const float* qkv, int ld, float* cstate, const float* cw, float* q, float* k, float* v, int NK,
                        int NV, int C, int M, cudaStream_t st);
// y[M][O] += B (A xu) of one adapted linear (LoRA, the device layout of LoraArgs), u [M][R] scratch.
void launch_pf_lora(const uint16_t* A, const uint16_t* B, int R, int r, int m1, int m2, int K, int O, int hb,
                    const float* xu, float* u, float* y, int M, cudaStream_t st);
void launch_pf_attn_prep(const float* mix, int ld, const float* qn, const float* kn, const float* inv_freq, int rot,
                         int H, int KV, int off, int M, float* qout, float* kc, float* vc, cudaStream_t st);

// Generic launch helper (PDL attribute on).
cudaError_t launch_pdl(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t st, void** args);

}  // namespace bcu
