// model.h — host-side model object behind the C ABI (include/bonsai_cuda.h).
#pragma once
#include <cuda_runtime.h>

#include <map>
#include <string>
#include <vector>

#include "../../include/bonsai_cuda.h"
#include "ctl.h"
#include "kernels.h"

namespace bcu {

struct DevTensor {
    int dtype = 0;
    std::vector<int64_t> shape;
    void* dev = nullptr;
    size_t bytes = 0;
};

// One packed linear (possibly several reference matrices sharing an input, stacked by rows).
struct Lin {
    TernaryMat m;
    const float* signs = nullptr;
    LoraArgs lora;  // a == null: no adapter on this linear
    // the same matrix in the prefill GEMM's layout (gemm.cu), null when a part is not whole 256-row tiles
    uint8_t* gwt = nullptr;
    uint8_t* gbias = nullptr;
};

// Scratch of the batched prefill, sized for PF_CHUNK rows on first use.
struct Prefill {
    int cap = 0;
    float *h = nullptr, *xn = nullptr, *mix = nullptr, *y = nullptr, *gu = nullptr, *tmp = nullptr;
    float *q = nullptr, *k = nullptr, *v = nullptr, *ga = nullptr, *gb = nullptr, *qbuf = nullptr, *part = nullptr;
    float* lu = nullptr;  // LoRA A products [rows][3 x 256]
    float* gws = nullptr; // chunked gated delta rule workspace (gdn_chunk_workspace_bytes)
    uint8_t* bop = nullptr;
    int* ex = nullptr;
    uint32_t* ids = nullptr;
};

struct Layer {
    bool attn = false;
    const float *in_norm = nullptr, *post_norm = nullptr;
    Lin mix_in;   // GDN: [qkv; z]   attention: [q (with gate); k; v]
    Lin mix_out;  // GDN: out_proj   attention: o_proj
    Lin gu;       // [gate; up]
    Lin down;
    const float *wa = nullptr, *wb = nullptr, *a_log = nullptr, *dt_bias = nullptr, *convw = nullptr, *gnorm = nullptr;
    const float *qn = nullptr, *kn = nullptr;
    int gi = -1, ai = -1;
};

}  // namespace bcu

struct bcu_state {
    int len = 0;
    float *gdn = nullptr, *conv = nullptr, *kc = nullptr, *vc = nullptr;
    size_t gdn_bytes = 0, conv_bytes = 0, kv_bytes = 0;
};

struct bcu_model {
    bcu_config c{};
    int device = 0, num_sms = 148;
    cudaStream_t st = nullptr;
    std::string err;
    std::string launch_err;  // the first kernel launch that failed while capturing a pass
    bool finalized = false;
    volatile int cancel = 0;
    std::map<std::string, bcu::DevTensor> staged;

    // derived sizes
    int C = 0, gw = 0, aw = 0, kvw = 0, n_gdn = 0, n_attn = 0;

    // weights
    void* arena = nullptr;
    size_t arena_bytes = 0, arena_used = 0;
    std::vector<bcu::Layer> layers;
    uint32_t* head_w = nullptr;     // fragment-ordered bf16 table
    uint16_t* embed_rows = nullptr; // row-major bf16 table (gathers)
    // ternary tied table (BCU_HEAD_TERNARY): the head GEMV's matrix (signs: the table's) and the MLX pack for gathers
    bcu::Lin head_lin;
    const uint32_t* emb_w = nullptr;
    const uint16_t *emb_s = nullptr, *emb_b = nullptr;
    const float* final_norm = nullptr;
    float* inv_freq = nullptr;

    // state (fp32, the reference's layouts: gdn [NV][128][128], conv [3][C], K/V [ctx][KV][256] per layer); the conv
    // state is double-buffered by pass parity: [n_gdn][2][3][C], committed rows at parity ^ 1
    float *gdn = nullptr, *conv = nullptr, *kc = nullptr, *vc = nullptr;
    float *pend_qkv = nullptr, *pend_qkvc = nullptr, *pend_ab = nullptr;

    // scratch
    float *h = nullptr, *mix = nullptr, *gubuf = nullptr, *y = nullptr, *apart = nullptr;
    float* ssbuf = nullptr;           // [hidden/128][VMAX] sums of squares of h by row block
    float* logits = nullptr;
    float* partial = nullptr;
    unsigned* counters = nullptr;
    unsigned* head_counter = nullptr;
    bool local_build = false;         // test hook: every GEMV builds its operand per CTA (no grid-wide build)
    uint8_t* opbuf = nullptr;         // a GEMV's rotated operand, built by its CTAs together (grid_build)
    unsigned* op_counters = nullptr;  // 2 words: builder CTAs arrived, CTAs past the grid-wide wait
    size_t opbuf_bytes = 0;
    float* pv = nullptr;
    int* pi = nullptr;
    int head_grid = 0;
    size_t partial_floats = 0;

    bcu::Ctl* ctl = nullptr;       // device
    bcu::CtlIn* h_in = nullptr;    // host copy of the next pass's ctl->in (edited freely; staged by stage_in)
    static constexpr int IN_SLOTS = 64;
    bcu::CtlIn* in_ring = nullptr;  // pinned staging slots: a slot is reused only after its copy has completed
    cudaEvent_t in_ev[IN_SLOTS] = {};
    bool in_used[IN_SLOTS] = {};
    int in_next = 0;
    bcu::Ctl* h_out = nullptr;     // pinned host copy of the control block
    uint32_t* planted_dev = nullptr;
    int planted_cap = 0;

    cudaGraphExec_t graphs[bcu::VMAX + 1] = {};
    int graph_nodes[bcu::VMAX + 1] = {};
    cudaEvent_t ev0 = nullptr, ev1 = nullptr, ev_done = nullptr;
    cudaEvent_t ev_ring[2] = {};  // plain decode: one event per token ring slot
    uint32_t* h_ring = nullptr;   // pinned 2-slot token ring

    // host mirror
    int len = 0;          // committed tokens including the pending commit (= ctl->off)
    int last_t = 0;       // rows of the last pass
    int pending_n = 0;    // rows of the last pass still to be committed on the device

    // LoRA adapter (lora.rs, Text::set_lora model.rs:392-397): one device buffer of every group's A and B, and the
    // partial products of the GEMV that runs
    void* lora_buf = nullptr;
    float* lora_upart = nullptr;
    int lora_rank = 0, lora_linears = 0;
    size_t lora_bytes = 0;  // fp16 A and B of every adapted group, read once per pass

    // batched prefill (prefill.cu) and every other allocation freed with the model
    bcu::Prefill pf;
    bool pf_off = false;  // test hook: prefill with verify passes only
    std::vector<void*> extra_allocs;

    // drafting
    std::vector<uint64_t> keys;   // token_key per vocab id
    std::vector<std::string> vocab_bytes;
    std::vector<uint32_t> fillers;  // draft_source's filler ids (bcu_set_fillers, or derived from the token bytes)
    bool fillers_given = false;
    bcu_encode_fn encode_fn = nullptr;  // normalize_draft's tokenizer (bcu_set_encoder)
    void* encode_user = nullptr;
    bcu_emit_fn emit_fn = nullptr;      // streaming emission (bcu_set_emit)
    void* emit_user = nullptr;
    double cost[9] = {0};         // verify cost per draft count (policy), measured on first use
    bool cost_ready = false;
};

namespace bcu {
// Internal helpers shared by runtime.cu and decode.cpp.
bcu_status run_pass(bcu_model* m, const uint32_t* ids, int T, int commit_all, int feed, bool sync);
bcu_status wait_stream(bcu_model* m, double seconds);
// Copies *m->h_in to ctl->in in stream order through a pinned slot that no later call can overwrite before the copy.
bcu_status stage_in(bcu_model* m);
bcu_status fail(bcu_model* m, bcu_status s, const std::string& msg);
}  // namespace bcu
