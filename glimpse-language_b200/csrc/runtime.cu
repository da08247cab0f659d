// runtime.cu — host runtime behind the C ABI: Model::load / Text::new (runtime/mod.rs:288-324, model.rs:270-368) on a
// B200. Tensors arrive by reference name, are repacked on the device into the tensor-core layouts, and each pass of T
// rows (T = 1 plain step, 2..16 verify, 16-row prefill chunks) is one CUDA graph captured once and replayed; its
// parameters (input ids, KV offset, replay count, parity) live in a device control block, as the Vulkan backend's
// recorded command buffers read per-step parameter slots (gpu_vk.rs:651-666, 778-838).
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <thread>

#include "model.h"
#include "operand.cuh"

using namespace bcu;

namespace bcu {

bcu_status fail(bcu_model* m, bcu_status s, const std::string& msg) {
    if (m) m->err = msg;
    return s;
}

#define CK(call)                                                                                              \
    do {                                                                                                      \
        cudaError_t e_ = (call);                                                                              \
        if (e_ != cudaSuccess)                                                                                \
            return fail(m, e_ == cudaErrorMemoryAllocation ? BCU_ERR_OOM : BCU_ERR_CUDA,                      \
                        std::string(#call) + ": " + cudaGetErrorString(e_));                                  \
    } while (0)

// Polls the model stream with a deadline instead of blocking (every host wait is bounded). The first SPIN_S seconds
// poll without sleeping: a verify pass ends a few ms after it is launched, and a sleep (which the OS may stretch to
// tens of µs) would add its wake-up latency to every decode round; longer waits poll every 20 µs.
bcu_status wait_stream(bcu_model* m, double seconds) {
    constexpr double SPIN_S = 0.01;
    CK(cudaEventRecord(m->ev_done, m->st));
    auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        cudaError_t e = cudaEventQuery(m->ev_done);
        if (e == cudaSuccess) break;
        if (e != cudaErrorNotReady) return fail(m, BCU_ERR_CUDA, std::string("stream: ") + cudaGetErrorString(e));
        double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (el > seconds) return fail(m, BCU_ERR_TIMEOUT, "device work did not finish within the deadline");
        if (el > SPIN_S) std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
    return BCU_OK;
}

bcu_status stage_in(bcu_model* m) {
    int i = m->in_next;
    m->in_next = (i + 1) % bcu_model::IN_SLOTS;
    if (m->in_used[i]) {  // bounded wait for the copy that last used this slot
        auto t0 = std::chrono::steady_clock::now();
        for (;;) {
            cudaError_t e = cudaEventQuery(m->in_ev[i]);
            if (e == cudaSuccess) break;
            if (e != cudaErrorNotReady) return fail(m, BCU_ERR_CUDA, cudaGetErrorString(e));
            if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > 120.0)
                return fail(m, BCU_ERR_TIMEOUT, "input staging slot did not free up");
        }
    }
    m->in_ring[i] = *m->h_in;
    CK(cudaMemcpyAsync(&m->ctl->in, &m->in_ring[i], sizeof(CtlIn), cudaMemcpyHostToDevice, m->st));
    CK(cudaEventRecord(m->in_ev[i], m->st));
    m->in_used[i] = true;
    return BCU_OK;
}

}  // namespace bcu

namespace {

const char* PFX = "language_model.model.";
const double WAIT_S = 120.0;

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

bcu_status check_config(const bcu_config* c, std::string* why) {
    auto bad = [&](const std::string& s) {
        *why = "unsupported config: " + s;
        return BCU_ERR_ARG;
    };
    if (c->n_layers < 1 || c->n_layers > BCU_MAX_LAYERS) return bad("n_layers out of range");
    if (c->head_dim != 256) return bad("head_dim must be 256");
    if (c->lin_k_dim != 128 || c->lin_v_dim != 128) return bad("linear head dims must be 128");
    if (c->conv_kernel != 4) return bad("linear_conv_kernel_dim must be 4");
    if (c->kv_heads < 1 || c->heads % c->kv_heads != 0) return bad("heads not divisible by kv heads");
    if (c->heads / c->kv_heads > 16) return bad("more than 16 q heads per kv head");
    if (c->lin_k_heads < 1 || c->lin_v_heads % c->lin_k_heads != 0) return bad("v heads not divisible by k heads");
    if (c->hidden % 512 || c->intermediate % 512) return bad("hidden/intermediate must be multiples of 512");
    if (c->hidden > HEAD_MAX_HIDDEN) return bad("hidden above 3072 is not supported (the head's operand lives in shared memory)");
    if (c->group_size != 64 && c->group_size != 128) return bad("group_size must be 64 or 128");
    if (c->hadamard != 512 && c->hadamard != 1024 && c->hadamard != 2048) return bad("hadamard block must be 512/1024/2048");
    int C = 2 * c->lin_k_heads * 128 + c->lin_v_heads * 128, gw = c->lin_v_heads * 128, aw = c->heads * 256;
    int kvw = c->kv_heads * 256;
    int dims[] = {c->hidden, c->intermediate, gw, aw};
    for (int d : dims)
        if (d % c->hadamard) return bad("activation widths must be multiples of the hadamard block");
    if (C % 128 || (2 * aw + 2 * kvw) % 128) return bad("projection widths must be multiples of 128");
    if (c->vocab < 16 || c->vocab % 16) return bad("vocab must be a multiple of 16");
    if (c->head_kind != BCU_HEAD_BF16 && c->head_kind != BCU_HEAD_TERNARY) return bad("unknown head kind");
    if (c->head_kind == BCU_HEAD_TERNARY && (c->hadamard != 512 || c->vocab % 128))
        return bad("the ternary tied table needs 512-point rotation blocks and a vocab multiple of 128");
    int half = c->rotary_dims / 2;
    if (c->rotary_dims % 2 || c->rotary_dims > 256 || c->mrope[0] + c->mrope[1] + c->mrope[2] != half)
        return bad("rotary dims / mrope sections");
    if (std::fabs(c->eps - 1e-6) > 1e-12) return bad("rms_norm_eps must be 1e-6");
    if (c->vmax < 1 || c->vmax > VMAX) return bad("vmax must be 1..16");
    if (c->ctx < 16 || c->ctx > 65536) return bad("ctx out of range");
    return BCU_OK;
}

const DevTensor* find(bcu_model* m, const std::string& n) {
    auto it = m->staged.find(n);
    return it == m->staged.end() ? nullptr : &it->second;
}

// Suballocates the weight arena. On overflow it hands out the arena start (no out-of-bounds write) and the caller's
// final size check reports the error.
void* arena_take(bcu_model* m, size_t bytes) {
    if (m->arena_used + align256(bytes) > m->arena_bytes) {
        m->arena_used = m->arena_bytes + 1;
        return m->arena;
    }
    void* p = (char*)m->arena + m->arena_used;
    m->arena_used += align256(bytes);
    return p;
}

// Copies a staged fp32 vector of `n` floats into the arena.
bcu_status arena_f32(bcu_model* m, const std::string& name, size_t n, const float** out) {
    const DevTensor* t = find(m, name);
    if (!t) return fail(m, BCU_ERR_NOT_FOUND, "missing tensor " + name);
    if (t->dtype != BCU_F32 || t->bytes != n * 4)
        return fail(m, BCU_ERR_ARG, "tensor " + name + ": expected fp32 of " + std::to_string(n) + " values");
    void* p = arena_take(m, n * 4);
    CK(cudaMemcpyAsync(p, t->dev, n * 4, cudaMemcpyDeviceToDevice, m->st));
    *out = (const float*)p;
    return BCU_OK;
}

struct Part {
    std::string name;
    int O;
};

// Bytes of one stacked ternary linear in the arena.
size_t lin_bytes(int O, int K, int group) {
    return align256(ternary_codes_bytes(O, K)) + align256(ternary_sb_bytes(O, K, group));
}

// Stacks the parts (rows in order) into one packed linear; the first part's signs rotate the shared input.
bcu_status build_lin(bcu_model* m, const std::vector<Part>& parts, int K, Lin* out) {
    int O = 0;
    for (auto& p : parts) O += p.O;
    int group = m->c.group_size;
    TernaryMat tm;
    tm.O = O;
    tm.K = K;
    tm.group = group;
    uint8_t* codes = (uint8_t*)arena_take(m, ternary_codes_bytes(O, K));
    uint8_t* sb = (uint8_t*)arena_take(m, ternary_sb_bytes(O, K, group));
    tm.codes = codes;
    tm.sb = (const uint32_t*)sb;
    int row = 0;
    for (auto& p : parts) {
        const DevTensor* w = find(m, p.name + ".weight");
        const DevTensor* s = find(m, p.name + ".scales");
        const DevTensor* b = m->c.has_bias ? find(m, p.name + ".biases") : nullptr;
        if (!w || !s || (m->c.has_bias && !b)) return fail(m, BCU_ERR_NOT_FOUND, "missing packed linear " + p.name);
        if (w->dtype != BCU_U32 || w->shape.size() != 2 || w->shape[0] != p.O || w->shape[1] * 16 != K)
            return fail(m, BCU_ERR_ARG, p.name + ".weight: expected u32 [" + std::to_string(p.O) + ", " +
                                            std::to_string(K / 16) + "]");
        size_t ns = (size_t)p.O * (K / group) * 2;
        if (s->dtype != BCU_F16 || s->bytes != ns) return fail(m, BCU_ERR_ARG, p.name + ".scales: wrong shape/dtype");
        if (b && (b->dtype != BCU_F16 || b->bytes != ns)) return fail(m, BCU_ERR_ARG, p.name + ".biases: wrong shape/dtype");
        // row offsets are multiples of 128, so each part lands on whole row blocks of the stacked layout
        repack_ternary((const uint32_t*)w->dev, (const uint16_t*)s->dev, b ? (const uint16_t*)b->dev : nullptr, p.O, K,
                       group, codes + ternary_codes_bytes(row, K), (uint32_t*)(sb + ternary_sb_bytes(row, K, group)),
                       m->st);
        CK(cudaGetLastError());
        row += p.O;
    }
    plan_ternary(tm, m->num_sms, m->c.hadamard);
    out->m = tm;
    // the same matrix in the prefill GEMM's layout (gemm.cu), when every part is whole 256-row tiles
    bool tiles = true;
    for (auto& p : parts) tiles = tiles && p.O % 256 == 0;
    out->gwt = out->gbias = nullptr;
    if (tiles) {
        uint8_t *gw = nullptr, *gb = nullptr;
        if (cudaMalloc(&gw, gemm_w_bytes(O, K)) != cudaSuccess) return fail(m, BCU_ERR_OOM, "prefill GEMM weights");
        m->extra_allocs.push_back(gw);
        if (cudaMalloc(&gb, gemm_bias_bytes(O, K, group)) != cudaSuccess)
            return fail(m, BCU_ERR_OOM, "prefill GEMM weights");
        m->extra_allocs.push_back(gb);
        int r = 0;
        for (auto& p : parts) {
            const DevTensor* w = find(m, p.name + ".weight");
            const DevTensor* s = find(m, p.name + ".scales");
            const DevTensor* b = m->c.has_bias ? find(m, p.name + ".biases") : nullptr;
            gemm_pack((const uint32_t*)w->dev, (const uint16_t*)s->dev, b ? (const uint16_t*)b->dev : nullptr, p.O, K,
                      group, gw + gemm_w_bytes(r, K), gb + gemm_bias_bytes(r, K, group), m->st);
            CK(cudaGetLastError());
            r += p.O;
        }
        out->gwt = gw;
        out->gbias = gb;
    }
    out->signs = nullptr;
    if (m->c.has_signs) {
        const DevTensor* sg = find(m, parts[0].name + ".signs");
        if (!sg || sg->dtype != BCU_F32 || sg->bytes != (size_t)K * 4)
            return fail(m, BCU_ERR_NOT_FOUND, "missing fp32 signs [" + std::to_string(K) + "] of " + parts[0].name);
        void* p = arena_take(m, (size_t)K * 4);
        CK(cudaMemcpyAsync(p, sg->dev, (size_t)K * 4, cudaMemcpyDeviceToDevice, m->st));
        out->signs = (const float*)p;
    }
    return BCU_OK;
}

// Zeroed device allocation. The zeroing is ordered on the model's stream: the stream is non-blocking, so a memset on
// the legacy default stream would not be ordered before the model's own copies into the new buffer.
template <class T>
bcu_status dmalloc(bcu_model* m, T** p, size_t bytes) {
    cudaError_t e = cudaMalloc((void**)p, bytes < 16 ? 16 : bytes);
    if (e != cudaSuccess) return fail(m, BCU_ERR_OOM, "cudaMalloc(" + std::to_string(bytes) + "): " + cudaGetErrorString(e));
    e = cudaMemsetAsync(*p, 0, bytes < 16 ? 16 : bytes, m->st);
    if (e != cudaSuccess) return fail(m, BCU_ERR_CUDA, cudaGetErrorString(e));
    return BCU_OK;
}

#define TRY(x)                          \
    do {                                \
        bcu_status s_ = (x);            \
        if (s_ != BCU_OK) return s_;    \
    } while (0)

// GDN layer kernel arguments (also used with T = 0 by bcu_flush to commit the pending rows).
GdnArgs gdn_args(bcu_model* m, const Layer& L, int T) {
    const bcu_config& c = m->c;
    GdnArgs g{};
    g.ctl = m->ctl;
    g.qkvz = m->mix;
    g.convw = L.convw;
    g.a_log = L.a_log;
    g.dt_bias = L.dt_bias;
    g.conv_state = m->conv + (size_t)L.gi * 2 * 3 * m->C;
    g.gdn_state = m->gdn + (size_t)L.gi * c.lin_v_heads * 128 * 128;
    g.pend_qkv = m->pend_qkv + (size_t)L.gi * 2 * VMAX * m->C;
    g.pend_qkvc = m->pend_qkvc + (size_t)L.gi * 2 * VMAX * m->C;
    g.pend_ab = m->pend_ab + (size_t)L.gi * 2 * VMAX * 2 * c.lin_v_heads;
    g.y = m->y;
    g.C = m->C;
    g.NK = c.lin_k_heads;
    g.NV = c.lin_v_heads;
    g.T = T;
    g.prefetch = T > 0;  // the passes run as graphs, each after the previous one completed; the flush (T = 0) does not
    return g;
}

// The kernels of one pass of T rows, in order (Text::encode_embed + encode_layers + encode_head, model.rs:641-985):
// per layer the mixer's input GEMV (norm + rotation; the GDN a/b gates ride along), the mixer core (GDN conv +
// recurrence, or attention), the mixer's output GEMV (gated norm / gate + rotation, residual add), the MLP gate/up
// GEMV (norm + rotation) and the down GEMV (SwiGLU + rotation, residual add); then the head. Each GEMV's CTAs build
// its rotated operand once, together, in a global buffer and copy their slices from it.
void enqueue_pass(bcu_model* m, int T) {
    const bcu_config& c = m->c;
    const int NT = (2 * T + 7) / 8, d = c.hidden;
    cudaStream_t st = m->st;
    // the GEMV's CTAs build its operand together when they all fit on the GPU at once (grid_build, ternary.cu)
    auto grid_built = [&](ActSrc& src, const Lin& ln, int ab_rows) {
        if (!m->local_build && gemv_coresident(ln.m, T, ab_rows, c.hadamard, m->num_sms, ln.lora.a ? ln.lora.r : 0)) {
            src.opbuf = m->opbuf;
            src.op_counters = m->op_counters;
        }
    };
    auto lora_of = [](const Lin& ln) { return ln.lora.a ? &ln.lora : nullptr; };
    // the first launch that failed (a capture only reports that one did)
    m->launch_err.clear();
    auto note = [&](const char* what, size_t li) {
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess && m->launch_err.empty())
            m->launch_err = std::string(what) + (li != (size_t)-1 ? " of layer " + std::to_string(li) : "") +
                            " (T = " + std::to_string(T) + "): " + cudaGetErrorString(e);
    };
    GemvOut store, resid;
    store.partial = resid.partial = m->partial;
    store.counters = resid.counters = m->counters;
    store.err = resid.err = &m->ctl->err;
    store.out = nullptr;
    resid.out = m->h;
    resid.add = 1;
    resid.ss_out = m->ssbuf;
    const bool ternary_head = c.head_kind == BCU_HEAD_TERNARY;
    if (ternary_head) {  // embed (kernels.metal:230-246) into h and its row-block sums of squares
        EmbedArgs e;
        e.ctl = m->ctl;
        e.w = m->emb_w;
        e.s = m->emb_s;
        e.b = m->emb_b;
        e.signs = m->head_lin.signs;
        e.h = m->h;
        e.ss = m->ssbuf;
        e.V = c.vocab;
        e.d = d;
        e.group = c.group_size;
        e.T = T;
        launch_embed_ternary(e, st);
        note("embedding", (size_t)-1);
    }
    for (size_t li = 0; li < m->layers.size(); li++) {
        const Layer& L = m->layers[li];
        ActSrc in;
        in.mode = li == 0 && !ternary_head ? ACT_EMBED : ACT_NORM;
        in.x = m->h;
        in.xb = m->embed_rows;
        in.w = L.in_norm;
        in.signs = L.mix_in.signs;
        in.ss = m->ssbuf;
        in.nss = d / 128;
        in.ctl = m->ctl;
        in.h_out = m->h;
        in.HB = c.hadamard;
        in.vocab = c.vocab;
        GemvOut mixo = store;
        mixo.out = m->mix;
        ActSrc out;
        out.HB = c.hadamard;
        out.signs = L.mix_out.signs;
        if (!L.attn) {
            AbArgs ab;
            ab.wa = L.wa;
            ab.wb = L.wb;
            ab.pend_ab = m->pend_ab + (size_t)L.gi * 2 * VMAX * 2 * c.lin_v_heads;
            ab.ctl = m->ctl;
            ab.nv = c.lin_v_heads;
            grid_built(in, L.mix_in, 2 * c.lin_v_heads);
            launch_ternary_gemv(L.mix_in.m, in, T, mixo, &ab, st, lora_of(L.mix_in));
            note("mixer input GEMV", li);
            launch_gdn_layer(gdn_args(m, L, T), st);
            note("GDN layer", li);
            out.mode = ACT_GATED;
            out.x = m->y;
            out.x2 = m->mix;
            out.ld2 = m->C + m->gw;
            out.off2 = m->C;
            out.w = L.gnorm;
        } else {
            grid_built(in, L.mix_in, 0);
            launch_ternary_gemv(L.mix_in.m, in, T, mixo, nullptr, st, lora_of(L.mix_in));
            note("mixer input GEMV", li);
            AttnArgs a{};
            a.ctl = m->ctl;
            a.qkv = m->mix;
            a.qn = L.qn;
            a.kn = L.kn;
            a.inv_freq = m->inv_freq;
            a.kc = m->kc + (size_t)L.ai * c.ctx * m->kvw;
            a.vc = m->vc + (size_t)L.ai * c.ctx * m->kvw;
            a.part = m->apart;
            a.out = m->y;
            a.H = c.heads;
            a.KV = c.kv_heads;
            a.rot = c.rotary_dims;
            a.T = T;
            a.ld = 2 * m->aw + 2 * m->kvw;
            a.ctx = c.ctx;
            launch_attn(a, st);
            note("attention", li);
            out.mode = ACT_GATE;
            out.x = m->y;
            out.x2 = m->mix;
            out.ld2 = a.ld;
        }
        grid_built(out, L.mix_out, 0);
        launch_ternary_gemv(L.mix_out.m, out, T, resid, nullptr, st, lora_of(L.mix_out));
        note("mixer output GEMV", li);
        ActSrc post = in;
        post.mode = ACT_NORM;
        post.w = L.post_norm;
        post.signs = L.gu.signs;
        post.opbuf = nullptr;
        post.op_counters = nullptr;
        grid_built(post, L.gu, 0);
        GemvOut guo = store;
        guo.out = m->gubuf;
        launch_ternary_gemv(L.gu.m, post, T, guo, nullptr, st, lora_of(L.gu));
        note("gate/up GEMV", li);
        ActSrc sw;
        sw.mode = ACT_SWIGLU;
        sw.x = m->gubuf;
        sw.signs = L.down.signs;
        sw.HB = c.hadamard;
        grid_built(sw, L.down, 0);
        launch_ternary_gemv(L.down.m, sw, T, resid, nullptr, st, lora_of(L.down));
        note("down GEMV", li);
    }
    if (ternary_head) {  // encode_head_to (model.rs:941-985): norm_rotate with the table's signs, the table, argmax
        ActSrc hs;
        hs.mode = ACT_NORM;
        hs.x = m->h;
        hs.w = m->final_norm;
        hs.signs = m->head_lin.signs;
        hs.ss = m->ssbuf;
        hs.nss = d / 128;
        hs.HB = c.hadamard;
        grid_built(hs, m->head_lin, 0);
        GemvOut ho = store;
        ho.out = m->logits;
        launch_ternary_gemv(m->head_lin.m, hs, T, ho, nullptr, st);
        note("head GEMV", (size_t)-1);
        HeadArgs ha{};
        ha.ctl = m->ctl;
        ha.logits = m->logits;
        ha.pv = m->pv;
        ha.pi = m->pi;
        ha.counter = m->head_counter;
        ha.V = c.vocab;
        ha.d = d;
        ha.T = T;
        launch_head_argmax(ha, m->head_grid, st);
        note("head argmax", (size_t)-1);
        return;
    }
    HeadArgs ha{};
    ha.ctl = m->ctl;
    ha.w = m->head_w;
    ha.h = m->h;
    ha.ss = m->ssbuf;
    ha.nss = d / 128;
    ha.norm = m->final_norm;
    ha.logits = m->logits;
    ha.pv = m->pv;
    ha.pi = m->pi;
    ha.counter = m->head_counter;
    ha.V = c.vocab;
    ha.d = d;
    ha.T = T;
    launch_head(ha, NT, m->head_grid, st);
    note("head", (size_t)-1);
}

bcu_status get_graph(bcu_model* m, int T, cudaGraphExec_t* out) {
    if (m->graphs[T]) {
        *out = m->graphs[T];
        return BCU_OK;
    }
    cudaGraph_t g;
    CK(cudaStreamBeginCapture(m->st, cudaStreamCaptureModeThreadLocal));
    enqueue_pass(m, T);
    cudaError_t e = cudaStreamEndCapture(m->st, &g);
    if (e != cudaSuccess)
        return fail(m, BCU_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(e) +
                                         (m->launch_err.empty() ? "" : "; first failed launch: " + m->launch_err));
    size_t n = 0;
    cudaGraphGetNodes(g, nullptr, &n);
    m->graph_nodes[T] = (int)n;
    e = cudaGraphInstantiate(&m->graphs[T], g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return fail(m, BCU_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
    *out = m->graphs[T];
    return BCU_OK;
}

// A bounded wait that nothing satisfies (bcu_debug_wait_timeout): flag stays 0.
__global__ void wait_timeout_kernel(Ctl* ctl, const unsigned* flag, uint32_t limit) {
    if (!spin_until_geq(flag, 1u, limit)) atomicOr(&ctl->err, ERR_SPIN_TIMEOUT);
}

bcu_status read_ctl(bcu_model* m) {
    CK(cudaMemcpyAsync(m->h_out, m->ctl, sizeof(Ctl), cudaMemcpyDeviceToHost, m->st));
    TRY(wait_stream(m, WAIT_S));
    if (m->h_out->err) {
        int e = m->h_out->err;
        cudaMemsetAsync(&m->ctl->err, 0, 4, m->st);
        if (e & ERR_MBAR_TIMEOUT) return fail(m, BCU_ERR_TIMEOUT, "a kernel gave up waiting for its bulk copies");
        if (e & ERR_SPIN_TIMEOUT) return fail(m, BCU_ERR_TIMEOUT, "a kernel gave up waiting for the other CTAs of its grid");
        if (e & ERR_BAD_TOKEN) return fail(m, BCU_ERR_ARG, "token id out of vocabulary range");
        if (e & ERR_CTX_FULL) return fail(m, BCU_ERR_STATE, "KV context full");
        return fail(m, BCU_ERR_CUDA, "device error " + std::to_string(e));
    }
    return BCU_OK;
}

// Sets the KV offset and the replay count of the control block in stream order (snapshot restore).
__global__ void ctl_set_kernel(Ctl* c, int off, int replay_n) {
    c->off = off;
    c->replay_n = replay_n;
    c->err = 0;
}

// After a commit-only pass: nothing left to replay, next pass at the other parity.
__global__ void ctl_flushed_kernel(Ctl* c) {
    c->replay_n = 0;
    c->parity ^= 1;
}

__global__ void ctl_planted_kernel(Ctl* c, const uint32_t* p, int n) {
    c->planted = p;
    c->planted_n = n;
}

}  // namespace

namespace bcu {

// One pass of T rows: stage the inputs, replay the graph, optionally wait and read the control block back.
bcu_status run_pass(bcu_model* m, const uint32_t* ids, int T, int commit_all, int feed, bool sync) {
    if (!m->finalized) return fail(m, BCU_ERR_STATE, "bcu_finalize has not run");
    if (T < 1 || T > m->c.vmax) return fail(m, BCU_ERR_ARG, "pass rows out of range");
    if (m->len + T > m->c.ctx) return fail(m, BCU_ERR_STATE, "context full");
    cudaGraphExec_t g;
    TRY(get_graph(m, T, &g));
    m->h_in->commit_all = commit_all;
    m->h_in->feed = feed;
    if (ids)
        for (int t = 0; t < T; t++) m->h_in->ids[t] = ids[t];
    TRY(stage_in(m));
    CK(cudaGraphLaunch(g, m->st));
    m->last_t = T;
    if (!sync) return BCU_OK;
    TRY(read_ctl(m));
    m->len = m->h_out->off;
    m->pending_n = m->h_out->replay_n;
    return BCU_OK;
}

}  // namespace bcu

// =============================================================================================== C ABI
extern "C" {

bcu_status bcu_config_check(const bcu_config* cfg, char* err, size_t err_len) {
    std::string why;
    bcu_status s = cfg ? check_config(cfg, &why) : BCU_ERR_ARG;
    if (!cfg) why = "null config";
    if (err && err_len) {
        snprintf(err, err_len, "%s", why.c_str());
    }
    return s;
}

bcu_status bcu_create(const bcu_config* cfg, int device, bcu_model** out) {
    if (!cfg || !out) return BCU_ERR_ARG;
    std::string why;
    if (check_config(cfg, &why) != BCU_OK) return BCU_ERR_ARG;
    bcu_model* m = new bcu_model();
    m->c = *cfg;
    m->device = device;
    *out = m;
    CK(cudaSetDevice(device));
    CK(cudaDeviceGetAttribute(&m->num_sms, cudaDevAttrMultiProcessorCount, device));
    CK(cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking));
    CK(cudaEventCreateWithFlags(&m->ev_done, cudaEventDisableTiming));
    CK(cudaEventCreate(&m->ev0));
    CK(cudaEventCreate(&m->ev1));
    CK(cudaEventCreateWithFlags(&m->ev_ring[0], cudaEventDisableTiming));
    CK(cudaEventCreateWithFlags(&m->ev_ring[1], cudaEventDisableTiming));
    CK(cudaMallocHost(&m->h_ring, 16));
    const bcu_config& c = m->c;
    m->C = 2 * c.lin_k_heads * 128 + c.lin_v_heads * 128;
    m->gw = c.lin_v_heads * 128;
    m->aw = c.heads * 256;
    m->kvw = c.kv_heads * 256;
    for (int i = 0; i < c.n_layers; i++) (c.layer_is_attn[i] ? m->n_attn : m->n_gdn)++;
    return BCU_OK;
}

bcu_status bcu_load_tensor(bcu_model* m, const char* name, int32_t dtype, const int64_t* shape, int32_t ndim,
                           const void* host_data) {
    if (!m || !name || !host_data || ndim < 0 || ndim > 4) return fail(m, BCU_ERR_ARG, "bad tensor arguments");
    if (m->finalized) return fail(m, BCU_ERR_STATE, "tensors must be loaded before bcu_finalize");
    CK(cudaSetDevice(m->device));
    DevTensor t;
    t.dtype = dtype;
    size_t n = 1;
    for (int i = 0; i < ndim; i++) {
        if (shape[i] <= 0) return fail(m, BCU_ERR_ARG, std::string("bad shape of ") + name);
        t.shape.push_back(shape[i]);
        n *= (size_t)shape[i];
    }
    size_t es = (dtype == BCU_U32 || dtype == BCU_F32) ? 4 : 2;
    t.bytes = n * es;
    auto it = m->staged.find(name);
    if (it != m->staged.end()) {
        cudaFree(it->second.dev);
        m->staged.erase(it);
    }
    CK(cudaMalloc(&t.dev, t.bytes));
    // on the model stream (the repack kernels that read it run there) and complete before the caller's buffer is
    // released
    CK(cudaMemcpyAsync(t.dev, host_data, t.bytes, cudaMemcpyHostToDevice, m->st));
    m->staged[name] = t;
    return wait_stream(m, WAIT_S);
}

bcu_status bcu_finalize(bcu_model* m) {
    if (!m) return BCU_ERR_ARG;
    if (m->finalized) return fail(m, BCU_ERR_STATE, "already finalized");
    CK(cudaSetDevice(m->device));
    const bcu_config& c = m->c;
    const int d = c.hidden, ff = c.intermediate, g = c.group_size;
    std::string p = PFX;
    // arena size
    size_t bytes = 0;
    for (int i = 0; i < c.n_layers; i++) {
        if (c.layer_is_attn[i]) {
            bytes += lin_bytes(2 * m->aw + 2 * m->kvw, d, g) + lin_bytes(d, m->aw, g) + 2 * 256 * 4;
        } else {
            bytes += lin_bytes(m->C + m->gw, d, g) + lin_bytes(d, m->gw, g);
            bytes += align256((size_t)2 * c.lin_v_heads * d * 4) * 2 + align256((size_t)m->C * 16) + 4 * 1024;
        }
        bytes += lin_bytes(2 * ff, d, g) + lin_bytes(d, ff, g) + 4 * align256((size_t)std::max(d, ff) * 4) + 8192;
    }
    if (c.head_kind == BCU_HEAD_TERNARY)  // the table in the GEMV layout + its MLX pack for the row gathers + signs
        bytes += lin_bytes(c.vocab, d, g) + align256((size_t)c.vocab * d / 4) +
                 2 * align256((size_t)c.vocab * (d / g) * 2) + align256((size_t)d * 4);
    else
        bytes += align256((size_t)c.vocab * d * 2) * 2;
    bytes += align256((size_t)d * 4) + (4 << 20);
    m->arena_bytes = bytes;
    CK(cudaMalloc(&m->arena, bytes));
    m->arena_used = 0;
    m->layers.resize(c.n_layers);
    int gi = 0, ai = 0;
    for (int i = 0; i < c.n_layers; i++) {
        Layer& L = m->layers[i];
        std::string l = p + "layers." + std::to_string(i) + ".";
        L.attn = c.layer_is_attn[i] != 0;
        TRY(arena_f32(m, l + "input_layernorm.weight", d, &L.in_norm));
        TRY(arena_f32(m, l + "post_attention_layernorm.weight", d, &L.post_norm));
        if (L.attn) {
            std::string a = l + "self_attn.";
            TRY(build_lin(m, {{a + "q_proj", 2 * m->aw}, {a + "k_proj", m->kvw}, {a + "v_proj", m->kvw}}, d, &L.mix_in));
            TRY(build_lin(m, {{a + "o_proj", d}}, m->aw, &L.mix_out));
            TRY(arena_f32(m, a + "q_norm.weight", 256, &L.qn));
            TRY(arena_f32(m, a + "k_norm.weight", 256, &L.kn));
            L.ai = ai++;
        } else {
            std::string a = l + "linear_attn.";
            TRY(build_lin(m, {{a + "in_proj_qkv", m->C}, {a + "in_proj_z", m->gw}}, d, &L.mix_in));
            TRY(build_lin(m, {{a + "out_proj", d}}, m->gw, &L.mix_out));
            TRY(arena_f32(m, a + "in_proj_a.weight", (size_t)c.lin_v_heads * d, &L.wa));
            TRY(arena_f32(m, a + "in_proj_b.weight", (size_t)c.lin_v_heads * d, &L.wb));
            TRY(arena_f32(m, a + "A_log", c.lin_v_heads, &L.a_log));
            TRY(arena_f32(m, a + "dt_bias", c.lin_v_heads, &L.dt_bias));
            TRY(arena_f32(m, a + "conv1d.weight", (size_t)m->C * 4, &L.convw));
            TRY(arena_f32(m, a + "norm.weight", 128, &L.gnorm));
            L.gi = gi++;
        }
        std::string mlp = l + "mlp.";
        TRY(build_lin(m, {{mlp + "gate_proj", ff}, {mlp + "up_proj", ff}}, d, &L.gu));
        TRY(build_lin(m, {{mlp + "down_proj", d}}, ff, &L.down));
    }
    TRY(arena_f32(m, p + "norm.weight", d, &m->final_norm));
    if (c.head_kind == BCU_HEAD_TERNARY) {
        // the reference's tied table (model.rs:356, 962): ternary-packed like the linears, with its own signs
        TRY(build_lin(m, {{p + "embed_tokens", c.vocab}}, d, &m->head_lin));
        const size_t wb = (size_t)c.vocab * d / 4, sb = (size_t)c.vocab * (d / g) * 2;
        const DevTensor* w = find(m, p + "embed_tokens.weight");
        const DevTensor* sc = find(m, p + "embed_tokens.scales");
        const DevTensor* bi = c.has_bias ? find(m, p + "embed_tokens.biases") : nullptr;
        uint32_t* ew = (uint32_t*)arena_take(m, wb);
        uint16_t* es = (uint16_t*)arena_take(m, sb);
        CK(cudaMemcpyAsync(ew, w->dev, wb, cudaMemcpyDeviceToDevice, m->st));
        CK(cudaMemcpyAsync(es, sc->dev, sb, cudaMemcpyDeviceToDevice, m->st));
        m->emb_w = ew;
        m->emb_s = es;
        if (bi) {
            uint16_t* eb = (uint16_t*)arena_take(m, sb);
            CK(cudaMemcpyAsync(eb, bi->dev, sb, cudaMemcpyDeviceToDevice, m->st));
            m->emb_b = eb;
        }
    } else {
        const DevTensor* e = find(m, p + "embed_tokens.weight");
        if (!e || e->dtype != BCU_BF16 || e->bytes != (size_t)c.vocab * d * 2)
            return fail(m, BCU_ERR_NOT_FOUND, "missing bf16 embed_tokens.weight [vocab, hidden]");
        m->embed_rows = (uint16_t*)arena_take(m, (size_t)c.vocab * d * 2);
        CK(cudaMemcpyAsync(m->embed_rows, e->dev, (size_t)c.vocab * d * 2, cudaMemcpyDeviceToDevice, m->st));
        m->head_w = (uint32_t*)arena_take(m, (size_t)c.vocab * d * 2);
        repack_head_bf16((const uint16_t*)e->dev, c.vocab, d, m->head_w, m->st);
        CK(cudaGetLastError());
    }
    {  // model.rs:316-321
        int half = c.rotary_dims / 2;
        std::vector<float> f(half);
        for (int i = 0; i < half; i++) f[i] = 1.0f / std::pow((float)c.rope_theta, (float)(2 * i) / (float)c.rotary_dims);
        m->inv_freq = (float*)arena_take(m, (size_t)half * 4 + 16);
        CK(cudaMemcpyAsync(m->inv_freq, f.data(), (size_t)half * 4, cudaMemcpyHostToDevice, m->st));
    }
    if (m->arena_used > m->arena_bytes) return fail(m, BCU_ERR_STATE, "internal: arena overflow");
    CK(cudaStreamSynchronize(m->st));
    for (auto& kv : m->staged) cudaFree(kv.second.dev);
    m->staged.clear();

    // state and scratch
    const int NV = c.lin_v_heads;
    TRY(dmalloc(m, &m->gdn, (size_t)m->n_gdn * NV * 128 * 128 * 4));
    TRY(dmalloc(m, &m->conv, (size_t)m->n_gdn * 2 * 3 * m->C * 4));
    TRY(dmalloc(m, &m->kc, (size_t)m->n_attn * c.ctx * m->kvw * 4));
    TRY(dmalloc(m, &m->vc, (size_t)m->n_attn * c.ctx * m->kvw * 4));
    TRY(dmalloc(m, &m->pend_qkv, (size_t)m->n_gdn * 2 * VMAX * m->C * 4));
    TRY(dmalloc(m, &m->pend_qkvc, (size_t)m->n_gdn * 2 * VMAX * m->C * 4));
    TRY(dmalloc(m, &m->pend_ab, (size_t)m->n_gdn * 2 * VMAX * 2 * NV * 4));
    int wide = std::max(std::max(d, ff), std::max(m->gw, m->aw));
    int mixw = std::max(m->C + m->gw, 2 * m->aw + 2 * m->kvw);
    TRY(dmalloc(m, &m->h, (size_t)VMAX * d * 4));
    TRY(dmalloc(m, &m->mix, (size_t)VMAX * mixw * 4));
    TRY(dmalloc(m, &m->gubuf, (size_t)VMAX * 2 * ff * 4));
    TRY(dmalloc(m, &m->y, (size_t)VMAX * std::max(m->gw, m->aw) * 4));
    TRY(dmalloc(m, &m->apart, (size_t)VMAX * c.heads * NSPLIT_ATTN * 258 * 4));
    TRY(dmalloc(m, &m->ssbuf, (size_t)(d / 128) * VMAX * 4));
    TRY(dmalloc(m, &m->logits, (size_t)VMAX * c.vocab * 4));
    (void)wide;
    size_t pf = 0;
    int maxrb = 1;
    for (auto& L : m->layers) {
        for (const Lin* ln : {&L.mix_in, &L.mix_out, &L.gu, &L.down}) {
            pf = std::max(pf, (size_t)ln->m.nsplit * VMAX * ln->m.O);
            maxrb = std::max(maxrb, ln->m.O / 128);
        }
    }
    if (c.head_kind == BCU_HEAD_TERNARY) {
        if (m->head_lin.m.nsplit > 1) pf = std::max(pf, (size_t)m->head_lin.m.nsplit * VMAX * m->head_lin.m.O);
        maxrb = std::max(maxrb, m->head_lin.m.O / 128);
    }
    m->partial_floats = pf;
    TRY(dmalloc(m, &m->partial, pf * 4));
    TRY(dmalloc(m, &m->counters, (size_t)maxrb * 4));
    m->head_grid = m->num_sms;  // one CTA per SM (head.cu)
    TRY(dmalloc(m, &m->head_counter, 4));
    {
        // operand buffer: [K / HB blocks][4 tiles][region] for the widest GEMV input
        const int kmax = std::max(std::max(c.hidden, c.intermediate), std::max(m->aw, c.lin_v_heads * 128));
        m->opbuf_bytes = (size_t)(kmax / c.hadamard) * 4 * op_region_bytes(c.hadamard, c.group_size);
        TRY(dmalloc(m, &m->opbuf, m->opbuf_bytes));
        TRY(dmalloc(m, &m->op_counters, 512 * 4));
    }
    TRY(dmalloc(m, &m->pv, (size_t)m->head_grid * VMAX * 4));
    TRY(dmalloc(m, &m->pi, (size_t)m->head_grid * VMAX * 4));
    TRY(dmalloc(m, &m->ctl, sizeof(Ctl)));
    CK(cudaMallocHost(&m->h_in, sizeof(CtlIn)));
    CK(cudaMallocHost(&m->in_ring, sizeof(CtlIn) * bcu_model::IN_SLOTS));
    for (auto& e : m->in_ev) CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    CK(cudaMallocHost(&m->h_out, sizeof(Ctl)));
    memset(m->h_in, 0, sizeof(CtlIn));
    memset(m->h_out, 0, sizeof(Ctl));
    m->finalized = true;
    m->len = 0;
    return BCU_OK;
}

bcu_status bcu_reset(bcu_model* m) {
    if (!m || !m->finalized) return fail(m, BCU_ERR_STATE, "not finalized");
    CK(cudaSetDevice(m->device));
    const int NV = m->c.lin_v_heads;
    CK(cudaMemsetAsync(m->gdn, 0, (size_t)m->n_gdn * NV * 128 * 128 * 4, m->st));
    CK(cudaMemsetAsync(m->conv, 0, (size_t)m->n_gdn * 2 * 3 * m->C * 4, m->st));
    CK(cudaMemsetAsync(m->op_counters, 0, 512 * 4, m->st));
    Ctl z;
    memset(&z, 0, sizeof(z));
    memcpy(m->h_out, &z, sizeof(Ctl));
    CK(cudaMemcpyAsync(m->ctl, m->h_out, sizeof(Ctl), cudaMemcpyHostToDevice, m->st));
    TRY(wait_stream(m, WAIT_S));
    m->len = 0;
    m->pending_n = 0;
    return BCU_OK;
}

const char* bcu_last_error(const bcu_model* m) { return m ? m->err.c_str() : "null model"; }

void bcu_destroy(bcu_model* m) {
    if (!m) return;
    cudaSetDevice(m->device);
    if (m->st) cudaStreamSynchronize(m->st);
    for (auto& g : m->graphs)
        if (g) cudaGraphExecDestroy(g);
    for (auto& kv : m->staged) cudaFree(kv.second.dev);
    void* bufs[] = {m->arena, m->gdn, m->conv, m->kc, m->vc, m->pend_qkv, m->pend_qkvc, m->pend_ab, m->h,
                    m->mix, m->gubuf, m->y, m->apart, m->ssbuf, m->logits,
                    m->partial, m->counters, m->head_counter, m->pv, m->pi, m->ctl, m->planted_dev,
                    m->opbuf, m->op_counters, m->lora_buf, m->lora_upart};
    for (void* b : bufs)
        if (b) cudaFree(b);
    for (void* b : m->extra_allocs) cudaFree(b);
    if (m->h_in) cudaFreeHost(m->h_in);
    if (m->in_ring) cudaFreeHost(m->in_ring);
    for (auto e : m->in_ev)
        if (e) cudaEventDestroy(e);
    if (m->h_out) cudaFreeHost(m->h_out);
    if (m->ev0) cudaEventDestroy(m->ev0);
    if (m->ev1) cudaEventDestroy(m->ev1);
    if (m->ev_done) cudaEventDestroy(m->ev_done);
    for (auto e : m->ev_ring)
        if (e) cudaEventDestroy(e);
    if (m->h_ring) cudaFreeHost(m->h_ring);
    if (m->st) cudaStreamDestroy(m->st);
    delete m;
}

bcu_status bcu_device_name(const bcu_model* m, char* out, size_t out_len) {
    if (!m || !out) return BCU_ERR_ARG;
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, m->device) != cudaSuccess) return BCU_ERR_CUDA;
    snprintf(out, out_len, "%s", p.name);
    return BCU_OK;
}

}  // extern "C"

namespace {

// rows per batched prefill chunk: larger than the reference's TMAX (512, model.rs:9) for fuller GEMM tiles; every
// row's result is independent of the chunking (row-local producers and GEMM, a row's attention splits set by its own
// position, the recurrence sequential)
constexpr int PF_CHUNK = 2048;
constexpr int PF_MIN = 64;     // shorter prompts run as verify passes
constexpr int PF_NSPLIT = 4;   // key splits per (row, kv head) of the chunk's attention

// Whether the batched prefill can run: every linear has its GEMM layout.
bool pf_supported(const bcu_model* m) {
    for (auto& L : m->layers)
        for (const Lin* ln : {&L.mix_in, &L.mix_out, &L.gu, &L.down})
            if (!ln->gwt) return false;
    return true;
}

bcu_status pf_alloc(bcu_model* m) {
    Prefill& p = m->pf;
    if (p.cap) return BCU_OK;
    const bcu_config& c = m->c;
    const size_t P = PF_CHUNK, d = c.hidden, ff = c.intermediate;
    const size_t wide = std::max(std::max(d, ff), (size_t)std::max(m->gw, m->aw));
    const size_t mixw = std::max(m->C + m->gw, 2 * m->aw + 2 * m->kvw);
    const int kmax = (int)std::max(std::max(d, ff), (size_t)std::max(m->gw, m->aw));
    auto get = [&](auto** ptr, size_t bytes) -> bcu_status {
        TRY(dmalloc(m, ptr, bytes));
        m->extra_allocs.push_back((void*)*ptr);
        return BCU_OK;
    };
    TRY(get(&p.h, P * d * 4));
    TRY(get(&p.xn, P * wide * 4));
    TRY(get(&p.lu, P * 3 * 256 * 4));
    TRY(get(&p.gws, gdn_chunk_workspace_bytes((int)P, c.lin_v_heads)));
    TRY(get(&p.mix, P * mixw * 4));
    TRY(get(&p.y, P * std::max(m->gw, m->aw) * 4));
    TRY(get(&p.gu, P * 2 * ff * 4));
    TRY(get(&p.tmp, P * d * 4));
    TRY(get(&p.q, P * c.lin_k_heads * 128 * 4));
    TRY(get(&p.k, P * c.lin_k_heads * 128 * 4));
    TRY(get(&p.v, P * c.lin_v_heads * 128 * 4));
    TRY(get(&p.ga, P * c.lin_v_heads * 4));
    TRY(get(&p.gb, P * c.lin_v_heads * 4));
    TRY(get(&p.qbuf, P * m->aw * 4));
    TRY(get(&p.part, P * c.heads * PF_NSPLIT * 258 * 4));
    TRY(get(&p.bop, gemm_act_bytes((int)P, kmax, c.group_size)));
    TRY(get(&p.ex, P * 4));
    TRY(get(&p.ids, P * 4));
    p.cap = (int)P;
    return BCU_OK;
}

// One linear of the chunk on the tcgen05 GEMM: y[M][O] = W . x (rotated rows), plus its adapter's B (A xu) on the
// unrotated rows xu when one is set.
bcu_status pf_gemm(bcu_model* m, const Lin& ln, const float* x, const float* xu, int M, float* y) {
    CK(gemm_run(ln.gwt, ln.gbias, ln.m.O, ln.m.K, ln.m.group, x, M, m->pf.bop, m->pf.ex, y, &m->ctl->err, m->num_sms,
                m->st));
    if (ln.lora.a) {
        const LoraArgs& L = ln.lora;
        launch_pf_lora(L.a, L.b, L.R, L.r, L.m1, L.m2, ln.m.K, ln.m.O, m->c.hadamard, xu, m->pf.lu, y, M, m->st);
        CK(cudaGetLastError());
    }
    return BCU_OK;
}

// A producer over the chunk's rows straight into the GEMM's activation tiles, then that linear.
bcu_status pf_rows_gemm(bcu_model* m, PfRowArgs r, const Lin& ln, int M, float* y) {
    Prefill& p = m->pf;
    r.bop = p.bop;
    r.ex = p.ex;
    r.G = ln.m.group;
    r.nbias = gemm_bias_chunks(r.D, r.G);
    launch_pf_rows(r, M, m->c.hadamard, m->st);
    return pf_gemm(m, ln, nullptr, p.xn, M, y);
}

// Model::prefill's forward of M rows (ids on the host) at positions off .. off + M - 1 (encode_layers_at,
// model.rs:670-934, without the head): the committed state advances by M rows. par: the control block's parity
// (the committed conv rows live in half par ^ 1 of each layer's double buffer).
bcu_status pf_chunk(bcu_model* m, const uint32_t* ids, int M, int off, int par) {
    const bcu_config& c = m->c;
    Prefill& p = m->pf;
    cudaStream_t st = m->st;
    const int d = c.hidden, ff = c.intermediate, NK = c.lin_k_heads, NV = c.lin_v_heads;
    const int C = m->C, gw = m->gw, aw = m->aw, kvw = m->kvw;
    CK(cudaMemcpyAsync(p.ids, ids, (size_t)M * 4, cudaMemcpyHostToDevice, st));
    const bool tern = c.head_kind == BCU_HEAD_TERNARY;
    launch_pf_embed(p.ids, M, c.vocab, d, tern ? nullptr : m->embed_rows, m->emb_w, m->emb_s, m->emb_b,
                    m->head_lin.signs, c.group_size, p.h, &m->ctl->err, st);
    const float* pending = nullptr;  // the previous residual linear's output, added to h by the next RMSNorm
    for (size_t li = 0; li < m->layers.size(); li++) {
        const Layer& L = m->layers[li];
        const bool last = li + 1 == m->layers.size();
        PfRowArgs in;
        in.mode = PF_NORM;
        in.D = d;
        in.h = p.h;
        in.add = pending;
        in.w = L.in_norm;
        in.signs = L.mix_in.signs;
        in.xn = (!L.attn || L.mix_in.lora.a) ? p.xn : nullptr;  // the GDN a/b rows or the adapter read it
        TRY(pf_rows_gemm(m, in, L.mix_in, M, p.mix));
        PfRowArgs out;
        out.D = L.attn ? aw : gw;
        out.src = p.y;
        out.signs = L.mix_out.signs;
        out.xn = L.mix_out.lora.a ? p.xn : nullptr;  // unrotated rows: only an adapter reads them
        if (!L.attn) {
            launch_pf_gdn_ab(L.wa, L.wb, p.xn, p.ga, p.gb, NV, d, M, st);
            float* cs = m->conv + ((size_t)L.gi * 2 + (par ^ 1)) * 3 * C;  // the committed half
            launch_pf_gdn_conv(p.mix, C + gw, cs, L.convw, p.q, p.k, p.v, NK, NV, C, M, st);
            launch_gdn_chunked(p.q, p.k, p.v, p.ga, p.gb, L.a_log, L.dt_bias,
                               m->gdn + (size_t)L.gi * NV * 128 * 128, p.y, M, NK, NV, p.gws, st);
            out.mode = PF_GATED;
            out.src2 = p.mix + C;
            out.ld2 = C + gw;
            out.w = L.gnorm;
        } else {
            const int ld = 2 * aw + 2 * kvw;
            float* kc = m->kc + (size_t)L.ai * c.ctx * kvw;
            float* vc = m->vc + (size_t)L.ai * c.ctx * kvw;
            launch_pf_attn_prep(p.mix, ld, L.qn, L.kn, m->inv_freq, c.rotary_dims, c.heads, c.kv_heads, off, M, p.qbuf,
                                kc, vc, st);
            AttnArgs a{};
            a.ctl = m->ctl;
            a.qkv = p.mix;
            a.qn = L.qn;
            a.kn = L.kn;
            a.inv_freq = m->inv_freq;
            a.kc = kc;
            a.vc = vc;
            a.part = p.part;
            a.out = p.y;
            a.H = c.heads;
            a.KV = c.kv_heads;
            a.rot = c.rotary_dims;
            a.T = M;
            a.ld = ld;
            a.ctx = c.ctx;
            a.nsplit = PF_NSPLIT;
            a.qprep = p.qbuf;
            a.off0 = off;
            if (!last) {  // the last layer needs only its K/V rows (written by the prep)
                if (attn_prefill_supported(c.heads, c.kv_heads))
                    launch_attn_prefill(p.qbuf, kc, vc, p.y, M, c.heads, c.kv_heads, off, st);
                else
                    launch_attn(a, st);
            }
            out.mode = PF_GATE;
            out.src2 = p.mix;
            out.ld2 = ld;
        }
        CK(cudaGetLastError());
        // the last layer's outputs only feed the residual rows of this chunk, which nothing reads: its state
        // updates above are all the chunk needs from it
        if (last) break;
        TRY(pf_rows_gemm(m, out, L.mix_out, M, p.tmp));
        PfRowArgs post;
        post.mode = PF_NORM;
        post.D = d;
        post.h = p.h;
        post.add = p.tmp;
        post.w = L.post_norm;
        post.signs = L.gu.signs;
        post.xn = L.gu.lora.a ? p.xn : nullptr;
        TRY(pf_rows_gemm(m, post, L.gu, M, p.gu));
        PfRowArgs sw;
        sw.mode = PF_SWIGLU;
        sw.D = ff;
        sw.src = p.gu;
        sw.signs = L.down.signs;
        sw.xn = L.down.lora.a ? p.xn : nullptr;
        TRY(pf_rows_gemm(m, sw, L.down, M, p.tmp));
        pending = p.tmp;
        CK(cudaGetLastError());
    }
    return BCU_OK;
}

}  // namespace

extern "C" {

bcu_status bcu_prefill(bcu_model* m, const uint32_t* ids, int32_t n, uint32_t* next) {
    if (!m || !ids || n < 1) return fail(m, BCU_ERR_ARG, "prefill needs at least one id");
    CK(cudaSetDevice(m->device));
    if (m->len + n > m->c.ctx) return fail(m, BCU_ERR_STATE, "context full");
    // batched: every row but the last through the tcgen05 GEMM in chunks; the last row then runs as a one-row pass,
    // which returns the next token
    if (n - 1 >= PF_MIN && !m->pf_off && pf_supported(m)) {
        TRY(bcu_flush(m));
        TRY(read_ctl(m));
        const int par = m->h_out->parity, off = m->h_out->off;
        TRY(pf_alloc(m));
        for (int i = 0; i < n - 1; i += PF_CHUNK) {
            const int M = std::min(PF_CHUNK, n - 1 - i);
            TRY(pf_chunk(m, ids + i, M, off + i, par));
        }
        TRY(read_ctl(m));  // device errors of the chunks
        ctl_set_kernel<<<1, 1, 0, m->st>>>(m->ctl, off + n - 1, 0);
        CK(cudaGetLastError());
        m->len = off + n - 1;
        m->pending_n = 0;
        TRY(run_pass(m, ids + n - 1, 1, 1, 0, true));
        if (next) *next = m->h_out->bonus;
        return BCU_OK;
    }
    int chunk = m->c.vmax;
    for (int i = 0; i < n; i += chunk) {
        int t = std::min(chunk, n - i);
        bool last = i + t == n;
        TRY(run_pass(m, ids + i, t, 1, 0, last));
        if (!last) m->len += t;  // mirror; the device advanced ctl->off by t
    }
    if (next) *next = m->h_out->bonus;
    return BCU_OK;
}

bcu_status bcu_step(bcu_model* m, uint32_t id, uint32_t* next) {
    if (!m) return BCU_ERR_ARG;
    CK(cudaSetDevice(m->device));
    TRY(run_pass(m, &id, 1, 1, 0, true));
    if (next) *next = m->h_out->bonus;
    return BCU_OK;
}

bcu_status bcu_verify(bcu_model* m, const uint32_t* ids, int32_t t, uint32_t* pred, int32_t* accepted) {
    if (!m || !ids) return fail(m, BCU_ERR_ARG, "null ids");
    CK(cudaSetDevice(m->device));
    TRY(run_pass(m, ids, t, 0, 0, true));
    if (pred)
        for (int i = 0; i < t; i++) pred[i] = m->h_out->pred[i];
    if (accepted) *accepted = m->h_out->accepted;
    return BCU_OK;
}

bcu_status bcu_verify_accept(bcu_model* m, const uint32_t* ids, int32_t t, int32_t* accepted, uint32_t* bonus) {
    if (!m || !ids) return fail(m, BCU_ERR_ARG, "null ids");
    CK(cudaSetDevice(m->device));
    TRY(run_pass(m, ids, t, 0, 0, false));
    // only the accept count and the bonus token come back
    CK(cudaMemcpyAsync(&m->h_out->accepted, &m->ctl->accepted, 8, cudaMemcpyDeviceToHost, m->st));
    TRY(wait_stream(m, WAIT_S));
    int32_t acc = m->h_out->accepted;
    if (acc < 0 || acc >= t) return fail(m, BCU_ERR_CUDA, "device accept count out of range");
    m->len += acc + 1;
    m->pending_n = acc + 1;
    if (accepted) *accepted = acc;
    if (bonus) *bonus = m->h_out->bonus;
    return BCU_OK;
}

bcu_status bcu_accept(bcu_model* m, int32_t t, int32_t n) {
    if (!m) return BCU_ERR_ARG;
    if (t != m->last_t || n < 1 || n > t || m->pending_n < 1) return fail(m, BCU_ERR_ARG, "accept does not match the last verify");
    CK(cudaSetDevice(m->device));
    TRY(read_ctl(m));
    int base = m->h_out->off - m->h_out->replay_n;
    int vals[2] = {base + n, n};  // off, replay_n (adjacent fields)
    static_assert(offsetof(Ctl, replay_n) == offsetof(Ctl, off) + 4, "layout");
    memcpy(&m->h_out->off, vals, 8);
    CK(cudaMemcpyAsync(&m->ctl->off, &m->h_out->off, 8, cudaMemcpyHostToDevice, m->st));
    TRY(wait_stream(m, WAIT_S));
    m->len = base + n;
    m->pending_n = n;
    return BCU_OK;
}

bcu_status bcu_flush(bcu_model* m) {
    if (!m || !m->finalized) return fail(m, BCU_ERR_STATE, "not finalized");
    CK(cudaSetDevice(m->device));
    TRY(read_ctl(m));
    if (m->h_out->replay_n == 0) return BCU_OK;
    // replay-only: the GDN layer kernel with zero new rows commits the pending rows (it writes the conv state at this
    // parity, so the parity flips as after a pass)
    for (auto& L : m->layers)
        if (!L.attn) launch_gdn_layer(gdn_args(m, L, 0), m->st);
    CK(cudaGetLastError());
    ctl_flushed_kernel<<<1, 1, 0, m->st>>>(m->ctl);
    CK(cudaGetLastError());
    TRY(wait_stream(m, WAIT_S));
    m->pending_n = 0;
    return BCU_OK;
}

bcu_status bcu_length(const bcu_model* m, int32_t* len) {
    if (!m || !len) return BCU_ERR_ARG;
    *len = m->len;
    return BCU_OK;
}

bcu_status bcu_set_keep_logits(bcu_model* m, int32_t keep) {
    if (!m || !m->finalized) return fail(m, BCU_ERR_STATE, "not finalized");
    m->h_in->keep_logits = keep ? 1 : 0;
    return BCU_OK;
}

bcu_status bcu_read_logits(bcu_model* m, int32_t row, float* out) {
    if (!m || !out || row < 0 || row >= m->last_t) return fail(m, BCU_ERR_ARG, "row out of range");
    CK(cudaSetDevice(m->device));
    CK(cudaMemcpyAsync(out, m->logits + (size_t)row * m->c.vocab, (size_t)m->c.vocab * 4, cudaMemcpyDeviceToHost, m->st));
    return wait_stream(m, WAIT_S);
}

// ------------------------------------------------------------------------------------------------ snapshots
static void state_sizes(const bcu_model* m, int len, size_t* g, size_t* c, size_t* kv) {
    *g = (size_t)m->n_gdn * m->c.lin_v_heads * 128 * 128 * 4;
    *c = (size_t)m->n_gdn * 3 * m->C * 4;
    *kv = (size_t)m->n_attn * len * m->kvw * 4;
}

bcu_status bcu_state_new(bcu_model* m, int32_t len, bcu_state** out) {
    if (!m || !out || len < 0 || len > m->c.ctx) return fail(m, BCU_ERR_ARG, "bad snapshot length");
    CK(cudaSetDevice(m->device));
    bcu_state* s = new bcu_state();
    s->len = len;
    state_sizes(m, len, &s->gdn_bytes, &s->conv_bytes, &s->kv_bytes);
    bcu_status st;
    if ((st = dmalloc(m, &s->gdn, s->gdn_bytes)) != BCU_OK || (st = dmalloc(m, &s->conv, s->conv_bytes)) != BCU_OK ||
        (st = dmalloc(m, &s->kc, s->kv_bytes)) != BCU_OK || (st = dmalloc(m, &s->vc, s->kv_bytes)) != BCU_OK) {
        bcu_state_free(s);
        return st;
    }
    *out = s;
    return BCU_OK;
}

void bcu_state_free(bcu_state* s) {
    if (!s) return;
    // a restore from this snapshot may still be copying on a model stream (bcu_restore is asynchronous)
    cudaDeviceSynchronize();
    cudaFree(s->gdn);
    cudaFree(s->conv);
    cudaFree(s->kc);
    cudaFree(s->vc);
    delete s;
}

// Text::encode_copy_state (model.rs:1072-1086): GDN and conv state whole, K/V rows [0, len) of every layer.
static bcu_status copy_kv(bcu_model* m, float* dst, int dst_cap, const float* src, int src_cap, int len) {
    if (len == 0) return BCU_OK;
    size_t row = (size_t)m->kvw * 4;
    CK(cudaMemcpy2DAsync(dst, dst_cap * row, src, src_cap * row, len * row, m->n_attn, cudaMemcpyDeviceToDevice, m->st));
    return BCU_OK;
}

bcu_status bcu_snapshot(bcu_model* m, bcu_state** out) {
    if (!m || !out) return BCU_ERR_ARG;
    TRY(bcu_flush(m));
    TRY(read_ctl(m));
    const int par = m->h_out->parity;
    bcu_state* s;
    TRY(bcu_state_new(m, m->len, &s));
    CK(cudaMemcpyAsync(s->gdn, m->gdn, s->gdn_bytes, cudaMemcpyDeviceToDevice, m->st));
    // the committed conv rows of each layer live at parity ^ 1 of its double buffer
    size_t cs = (size_t)3 * m->C * 4;
    if (m->n_gdn)
        CK(cudaMemcpy2DAsync(s->conv, cs, (const char*)m->conv + (par ^ 1) * cs, 2 * cs, cs, m->n_gdn,
                             cudaMemcpyDeviceToDevice, m->st));
    TRY(copy_kv(m, s->kc, s->len, m->kc, m->c.ctx, s->len));
    TRY(copy_kv(m, s->vc, s->len, m->vc, m->c.ctx, s->len));
    TRY(wait_stream(m, WAIT_S));
    *out = s;
    return BCU_OK;
}

bcu_status bcu_restore(bcu_model* m, const bcu_state* s) {
    if (!m || !s || !m->finalized) return fail(m, BCU_ERR_ARG, "bad restore");
    CK(cudaSetDevice(m->device));
    CK(cudaMemcpyAsync(m->gdn, s->gdn, s->gdn_bytes, cudaMemcpyDeviceToDevice, m->st));
    // both halves of each layer's conv double buffer, so whichever parity comes next reads the restored rows
    size_t cs = (size_t)3 * m->C * 4;
    for (int half = 0; half < 2 && m->n_gdn; half++)
        CK(cudaMemcpy2DAsync((char*)m->conv + half * cs, 2 * cs, s->conv, cs, cs, m->n_gdn, cudaMemcpyDeviceToDevice,
                             m->st));
    TRY(copy_kv(m, m->kc, m->c.ctx, s->kc, s->len, s->len));
    TRY(copy_kv(m, m->vc, m->c.ctx, s->vc, s->len, s->len));
    ctl_set_kernel<<<1, 1, 0, m->st>>>(m->ctl, s->len, 0);
    CK(cudaGetLastError());
    m->len = s->len;
    m->pending_n = 0;
    return BCU_OK;
}

bcu_status bcu_state_parts(const bcu_model* m, const bcu_state* s, uint64_t sizes[4], int32_t* len) {
    if (!m || !s || !sizes) return BCU_ERR_ARG;
    sizes[0] = s->gdn_bytes;
    sizes[1] = s->conv_bytes;
    sizes[2] = s->kv_bytes;
    sizes[3] = s->kv_bytes;
    if (len) *len = s->len;
    return BCU_OK;
}

static void* part_ptr(const bcu_state* s, int part, uint64_t* bytes) {
    switch (part) {
        case 0: *bytes = s->gdn_bytes; return s->gdn;
        case 1: *bytes = s->conv_bytes; return s->conv;
        case 2: *bytes = s->kv_bytes; return s->kc;
        case 3: *bytes = s->kv_bytes; return s->vc;
    }
    return nullptr;
}

bcu_status bcu_state_read(const bcu_model* m, const bcu_state* s, int32_t part, void* host, uint64_t bytes) {
    if (!m || !s || !host) return BCU_ERR_ARG;
    uint64_t n;
    void* p = part_ptr(s, part, &n);
    if (!p || bytes != n) return BCU_ERR_ARG;
    if (cudaMemcpyAsync(host, p, n, cudaMemcpyDeviceToHost, m->st) != cudaSuccess) return BCU_ERR_CUDA;
    return cudaStreamSynchronize(m->st) == cudaSuccess ? BCU_OK : BCU_ERR_CUDA;
}

bcu_status bcu_state_write(bcu_model* m, bcu_state* s, int32_t part, const void* host, uint64_t bytes, int32_t len) {
    if (!m || !s || !host || len != s->len) return fail(m, BCU_ERR_ARG, "state part does not match the snapshot");
    uint64_t n;
    void* p = part_ptr(s, part, &n);
    if (!p || bytes != n) return fail(m, BCU_ERR_ARG, "state part size mismatch");
    CK(cudaMemcpyAsync(p, host, n, cudaMemcpyHostToDevice, m->st));
    return wait_stream(m, WAIT_S);
}

// ------------------------------------------------------------------------------------------------ introspection
bcu_status bcu_pass_launches(const bcu_model* m, int32_t t, int32_t* launches) {
    if (!m || !launches || t < 1 || t > VMAX) return BCU_ERR_ARG;
    *launches = m->graph_nodes[t];
    return BCU_OK;
}

bcu_status bcu_pass_bytes(const bcu_model* m, int32_t t, double* bytes) {
    if (!m || !bytes || !m->finalized) return BCU_ERR_ARG;
    const bcu_config& c = m->c;
    double b = 0;
    for (auto& L : m->layers)
        for (const Lin* ln : {&L.mix_in, &L.mix_out, &L.gu, &L.down}) {
            double O = ln->m.O, K = ln->m.K, g = ln->m.group;
            b += O * K / 4 + O * (K / g) * 4;  // codes + fp16 scale and bias per group
        }
    if (c.head_kind == BCU_HEAD_TERNARY)                                          // ternary tied head
        b += (double)c.vocab * c.hidden / 4 + (double)c.vocab * (c.hidden / c.group_size) * 4;
    else
        b += (double)c.vocab * c.hidden * 2;                                      // bf16 head
    b += (double)m->n_gdn * 2 * c.lin_v_heads * c.hidden * 4;                     // dense a/b
    b += (double)m->n_gdn * c.lin_v_heads * 128 * 128 * 4 * 2;                    // GDN state r+w
    b += (double)m->n_gdn * 3 * m->C * 4 * 2;                                     // conv state r+w
    b += (double)m->n_attn * (m->len + t / 2.0) * m->kvw * 4 * 2;                 // fp32 K+V read
    b += (double)m->lora_bytes;                                                   // LoRA A and B (fp16)
    *bytes = b;
    return BCU_OK;
}

bcu_status bcu_set_planted(bcu_model* m, const uint32_t* ids, int32_t n, int32_t base) {
    if (!m || !m->finalized || (!ids && n) || n < 0) return fail(m, BCU_ERR_ARG, "bad planted stream");
    CK(cudaSetDevice(m->device));
    TRY(wait_stream(m, WAIT_S));
    if (n > m->planted_cap) {
        if (m->planted_dev) cudaFree(m->planted_dev);
        m->planted_dev = nullptr;
        TRY(dmalloc(m, &m->planted_dev, (size_t)n * 4));
        m->planted_cap = n;
    }
    if (n) CK(cudaMemcpyAsync(m->planted_dev, ids, (size_t)n * 4, cudaMemcpyHostToDevice, m->st));
    ctl_planted_kernel<<<1, 1, 0, m->st>>>(m->ctl, m->planted_dev, n);
    CK(cudaGetLastError());
    m->h_in->planted_base = base;
    return wait_stream(m, WAIT_S);
}

bcu_status bcu_enqueue_passes(bcu_model* m, int32_t t, int32_t passes, int32_t feed) {
    if (!m || !m->finalized || t < 1 || t > m->c.vmax || passes < 0 || feed < 0 || feed > 2)
        return fail(m, BCU_ERR_ARG, "bad pass request");
    CK(cudaSetDevice(m->device));
    cudaGraphExec_t g;
    TRY(get_graph(m, t, &g));
    m->h_in->commit_all = 0;
    m->h_in->feed = feed;
    TRY(stage_in(m));
    for (int i = 0; i < passes; i++) CK(cudaGraphLaunch(g, m->st));
    m->last_t = t;
    return BCU_OK;
}

bcu_status bcu_sync(bcu_model* m) {
    if (!m || !m->finalized) return fail(m, BCU_ERR_STATE, "not finalized");
    CK(cudaSetDevice(m->device));
    TRY(read_ctl(m));
    m->len = m->h_out->off;
    m->pending_n = m->h_out->replay_n;
    return BCU_OK;
}

bcu_status bcu_stream(bcu_model* m, void** stream) {
    if (!m || !stream) return BCU_ERR_ARG;
    *stream = (void*)m->st;
    return BCU_OK;
}

bcu_status bcu_time_pass(bcu_model* m, int32_t t, int32_t iters, float* ms_per_pass) {
    if (!m || !ms_per_pass || iters < 1 || t < 1 || t > m->c.vmax) return fail(m, BCU_ERR_ARG, "bad timing args");
    CK(cudaSetDevice(m->device));
    if (m->len + t > m->c.ctx) return fail(m, BCU_ERR_STATE, "context full");
    bcu_state* snap;
    TRY(bcu_snapshot(m, &snap));
    cudaGraphExec_t g;
    TRY(get_graph(m, t, &g));
    uint32_t ids[VMAX];
    for (int i = 0; i < t; i++) ids[i] = (uint32_t)(i * 7919 % m->c.vocab);
    for (int i = 0; i < t; i++) m->h_in->ids[i] = ids[i];
    m->h_in->commit_all = 0;
    m->h_in->feed = 0;
    TRY(stage_in(m));
    // each replay verifies on top of the previous one; restore the state every pass so the length stays put
    float total = 0;
    for (int i = 0; i < iters + 1; i++) {
        TRY(bcu_restore(m, snap));
        CK(cudaEventRecord(m->ev0, m->st));
        CK(cudaGraphLaunch(g, m->st));
        CK(cudaEventRecord(m->ev1, m->st));
        TRY(wait_stream(m, WAIT_S));
        float ms;
        CK(cudaEventElapsedTime(&ms, m->ev0, m->ev1));
        if (i > 0) total += ms;
    }
    TRY(bcu_restore(m, snap));
    TRY(wait_stream(m, WAIT_S));
    bcu_state_free(snap);
    *ms_per_pass = total / iters;
    return BCU_OK;
}

// Test hook (not in the ABI header): one thread waits, with the bounded spin the GEMV's grid-wide build uses (a short
// limit here), on a zeroed word that nothing writes; the wait runs out, the kernel records ERR_SPIN_TIMEOUT in the
// control block and returns, and the host reads it as BCU_ERR_TIMEOUT, with the context still usable.
bcu_status bcu_debug_wait_timeout(bcu_model* m) {
    if (!m || !m->finalized) return BCU_ERR_ARG;
    CK(cudaSetDevice(m->device));
    TRY(wait_stream(m, WAIT_S));
    wait_timeout_kernel<<<1, 1, 0, m->st>>>(m->ctl, m->op_counters + 256, 1u << 14);
    CK(cudaGetLastError());
    return read_ctl(m);
}

// Test hook (not in the ABI header): batched != 0 lets bcu_prefill use the tcgen05 GEMM chunks (the default), 0 keeps
// it to verify passes, so tests can compare the two.
bcu_status bcu_set_batched_prefill(bcu_model* m, int32_t batched) {
    if (!m) return BCU_ERR_ARG;
    m->pf_off = batched == 0;
    return BCU_OK;
}

// Test hook (not in the ABI header): local != 0 makes every GEMV build its operand per CTA (build_operand) instead of
// once across the grid, so tests cover both paths; the pass graphs are recaptured.
bcu_status bcu_set_local_build(bcu_model* m, int32_t local) {
    if (!m || !m->finalized) return BCU_ERR_ARG;
    TRY(wait_stream(m, WAIT_S));
    for (int t = 0; t <= VMAX; t++) {
        if (m->graphs[t]) cudaGraphExecDestroy(m->graphs[t]);
        m->graphs[t] = nullptr;
        m->graph_nodes[t] = 0;
    }
    m->local_build = local != 0;
    m->cost_ready = false;
    return BCU_OK;
}

}  // extern "C"
