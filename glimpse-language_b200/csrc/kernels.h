// kernels.h — host-side launch wrappers of the sm_100a kernels (one translation unit per kernel family).
// Every wrapper enqueues on `stream` with Programmatic Dependent Launch allowed, so consecutive kernels of a pass
// overlap their prologue (weight prefetch) with the previous kernel's tail.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace bcu {

struct Ctl;

// ------------------------------------------------------------------------------------------------ ternary linear
// Device layout of one packed ternary matrix (O rows x K codes), built by repack_ternary from the MLX pack:
//   codes  : [O/128][K/128][8 m-tiles][32 lanes][16 B]; lane (g = l/4, t = l%4) word q holds the 16 codes of rows
//            g and g+8 at k = 32q + {0,8,16,24} + 2t + {0,1}, so one LDS.128 gives a lane its A-fragment codes for
//            8 mma k16-steps; slot h (bits 2h and 16+2h) decodes with a mask at bit 2*(h%4) of w or w >> 8.
//   scales : [O/128][K/128][8][128/group][8 g] u32 = half2(s[row g], s[row g+8])
//   bias   : [O][K/group] fp16 = b (MLX affine) or -s (reference pack, weight = s*(code-1))
struct TernaryMat {
    const void* codes = nullptr;
    const uint32_t* scales = nullptr;
    const uint16_t* bias = nullptr;
    int O = 0, K = 0, group = 64;
    int kslice = 0, nsplit = 1;  // split-K plan (kslice multiple of 512)
};

// Activation operand of the ternary GEMV for one pass (written by the producer kernels):
//   bfrag : [K/16][NT][32 lanes][2] u32, column n of n-tile nt = token 4*nt + n/2, n%2 = hi/lo part of
//           fp16(x * 2^e_t * 4^-j(k)), j(k) = (k % 32) / 8
//   xsum  : [T][K/group] fp32 group sums of x (bias term), xexp: [T] e_t
struct TernaryAct {
    uint32_t* bfrag = nullptr;
    float* xsum = nullptr;
    int* xexp = nullptr;
    int K = 0;
};

size_t ternary_codes_bytes(int O, int K);
size_t ternary_scales_bytes(int O, int K, int group);
// Converts MLX-packed device arrays (u32 [O][K/16], fp16 [O][K/group] scales, optional biases) into the layout above.
void repack_ternary(const uint32_t* w_mlx, const uint16_t* s, const uint16_t* b, int O, int K, int group,
                    void* codes, uint32_t* scales, uint16_t* bias, cudaStream_t st);
void plan_ternary(TernaryMat& m, int num_sms);

// y[T][O] (+)= W . x for T <= 4*NT rows. partial: nsplit*T*O floats; counters: O/128 zeroed uints.
void launch_ternary_gemv(const TernaryMat& m, const TernaryAct& a, int T, float* out, int add, float* partial,
                         unsigned* counters, int* err, cudaStream_t st);

// Standalone producer: rotates x (bf16 [T][K], or fp32 when x_f32 != null) with block HB and optional signs and
// writes the activation operand (config 1 path). xrot (optional) receives the rotated fp32 rows.
void launch_rotate_prep(const uint16_t* x_bf16, const float* x_f32, int T, int K, int HB, const float* signs,
                        int group, TernaryAct act, float* xrot, cudaStream_t st);

// ------------------------------------------------------------------------------------------------ producers
// One CTA per (padded) token row. Each writes the ternary activation operand of its row.
struct PrepNormArgs {
    const Ctl* ctl;
    const uint16_t* embed_bf16;  // != null: h[t] = table[ids[t]] first (embedding fused into the first layer)
    float* h;                    // [T][D] residual stream (read; written when embedding)
    const float* w;              // norm weight [D]
    const float* signs;          // [D] or null
    float* xn;                   // [T][D] normed rows (for the GDN a/b gates) or null
    int D, HB, group, T, vocab;
    TernaryAct act;
};
void launch_prep_norm(const PrepNormArgs& a, int NT, cudaStream_t st);

struct PrepSwigluArgs {
    const float* gu;  // [T][2*ff]: gate then up
    const float* signs;
    int ff, HB, group, T;
    TernaryAct act;
};
void launch_prep_swiglu(const PrepSwigluArgs& a, int NT, cudaStream_t st);

struct PrepGatedArgs {
    const float* y;      // [T][gw] GDN outputs
    const float* qkvz;   // [T][C + gw]: z at column C
    const float* w;      // norm weight [128]
    const float* signs;
    int gw, C, HB, group, T;
    TernaryAct act;
};
void launch_prep_gated(const PrepGatedArgs& a, int NT, cudaStream_t st);

struct PrepAttnOutArgs {
    const float* part;   // attention split partials [T][H][NSPLIT][258]
    const float* qkv;    // [T][2*aw + 2*kvw] q projection (gate halves)
    const float* signs;
    int H, HB, group, T, qkv_ld;
    TernaryAct act;
};
void launch_prep_attn_out(const PrepAttnOutArgs& a, int NT, cudaStream_t st);

// Final norm -> bf16 hi/lo operand of the head GEMV: [d/16][NT][32][2] u32.
struct PrepHeadArgs {
    const float* h;
    const float* w;
    uint32_t* bfrag;
    int D, T;
};
void launch_prep_head(const PrepHeadArgs& a, int NT, cudaStream_t st);

// ------------------------------------------------------------------------------------------------ GatedDeltaNet
struct GdnArgs {
    const Ctl* ctl;
    const float* qkvz;     // [T][C + gw] GEMV output (qkv first)
    const float* xn;       // [T][d] normed input (a/b gates)
    const float* wa;       // [NV][d]
    const float* wb;       // [NV][d]
    const float* convw;    // [C][4]
    const float* a_log;    // [NV]
    const float* dt_bias;  // [NV]
    float* conv_state;     // [3][C] committed
    float* gdn_state;      // [NV][128][128] committed
    float* pend_qkv;       // [2][VMAX][C] raw qkv rows (conv commit of the next pass)
    float* pend_qkvc;      // [2][VMAX][C] conv outputs (replay)
    float* pend_ab;        // [2][VMAX][2NV] gate inputs (replay)
    float* y;              // [T][NV*128]
    int d, C, NK, NV, T;
};
void launch_gdn_ab(const GdnArgs& a, cudaStream_t st);
void launch_gdn_conv(const GdnArgs& a, cudaStream_t st);
void launch_gdn_recurrent(const GdnArgs& a, cudaStream_t st);

// Standalone verify step with rollback (graded config 2).
void launch_gdn_verify(const float* q, const float* k, const float* v, const float* a_in, const float* b_in,
                       const float* a_log, const float* dt_bias, float* state, float* y, int T, int NK, int NV,
                       int n, cudaStream_t st);

// ------------------------------------------------------------------------------------------------ attention
struct AttnArgs {
    const Ctl* ctl;
    const float* qkv;      // [T][ld]: q (with gates, 2*aw), k (kvw), v (kvw)
    const float* qn;       // [256]
    const float* kn;       // [256]
    const float* inv_freq; // [rot/2]
    float* q;              // [T][H][256] prepared queries
    float* kc;             // [ctx][KV][256]
    float* vc;
    float* part;           // [T][H][NSPLIT][258]
    int H, KV, rot, T, ld, ctx;
};
void launch_attn_prep(const AttnArgs& a, cudaStream_t st);
void launch_attn_split(const AttnArgs& a, cudaStream_t st);

// ------------------------------------------------------------------------------------------------ head + accept
// bf16 tied head in mma fragment order: [V/16][d/16][32 lanes][4] u32.
void repack_head_bf16(const uint16_t* table, int V, int d, uint32_t* out, cudaStream_t st);

struct HeadArgs {
    Ctl* ctl;
    const uint32_t* w;       // repacked head
    const uint32_t* bfrag;   // [d/16][NT][32][2]
    float* logits;           // [T][V] (written when ctl->keep_logits)
    float* pv;               // [grid][T] partial maxima
    int* pi;                 // [grid][T]
    unsigned* counter;       // 1 zeroed uint
    int V, d, T;
};
void launch_head(const HeadArgs& a, int NT, int grid, cudaStream_t st);

// Embedding gather (bf16 table) for passes whose first layer is attention (no fused prep) — unused otherwise.
void launch_embed(const Ctl* ctl, const uint16_t* table, float* h, int d, int vocab, int T, cudaStream_t st);

// Generic launch helper (PDL attribute on).
cudaError_t launch_pdl(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t st, void** args);

}  // namespace bcu
