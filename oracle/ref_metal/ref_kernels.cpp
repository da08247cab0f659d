// ref_kernels.cpp — the reference's own Metal text kernels (src/bonsai/runtime/kernels.metal, compiled here through
// metal_stdlib) behind a C ABI, plus the reference's layer sequence (Text::encode_layers_at, encode_head_to,
// encode_accept; src/bonsai/runtime/model.rs:670-1069) restated on host buffers so a whole pass of the reference
// runs on the CPU. TEST INFRASTRUCTURE ONLY: it pins the oracle (oracle/bonsai_oracle.cpp) to the reference; the
// product never loads it.
//
// Every dispatch below uses the grid and threadgroup size model.rs passes to Cmd::run for that kernel (cited per
// call), and the Metal path of qmm_lora (model.rs:457-526): T = 1 qmv4 (or qmv3 with the GDN a/b rows for a
// single-token decode step), T = 2..3 qmvr, T = 4..16 qmvxm in 8-row slices, T > 16 qmm.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/bonsai_cuda.h"
#include "ref_runtime.h"

#include <metal_stdlib>

namespace ref {
#include REF_KERNELS
}  // namespace ref

using refrt::Ctx;
using refrt::run;

namespace {

const uint ARGMAX_GROUPS = 128;  // model.rs:12
const uint RCHUNK = 2048;        // model.rs:14
const uint VMAX_ = 16;           // model.rs:11

uint2 u2(const uint32_t* a) { return uint2(a[0], a[1]); }

// ------------------------------------------------------------------------------------------------ dispatches
void d_norm_rotate(const float* h, const float* w, const float* signs, float* xn, float* xr, uint D, uint write_xn,
                   uint T) {  // model.rs:690-707
    const metal::half* A = nullptr;
    float* U = xr;
    uint R = 0;
    run(T, (D + RCHUNK - 1) / RCHUNK, 1, 128, 1, 1, [&](const Ctx& c) {
        ref::norm_rotate(h, w, signs, xn, xr, D, write_xn, A, U, R, u2(c.tg), u2(c.ng), c.sid, c.lane);
    });
}

void d_swiglu_rotate(const float* g, const float* u, const float* signs, float* xr, uint D, uint T) {  // :913-928
    const metal::half* A = nullptr;
    float* U = xr;
    uint R = 0;
    run(T, (D + RCHUNK - 1) / RCHUNK, 1, 128, 1, 1, [&](const Ctx& c) {
        ref::swiglu_rotate(g, u, signs, xr, D, A, U, R, u2(c.tg), u2(c.ng), c.sid, c.lane);
    });
}

void d_gate_rotate(const float* attn, const float* qp, const float* signs, float* xr, uint W, uint T) {  // :876-891
    const metal::half* A = nullptr;
    float* U = xr;
    uint R = 0;
    run(T, (W + RCHUNK - 1) / RCHUNK, 1, 128, 1, 1, [&](const Ctx& c) {
        ref::gate_rotate(attn, qp, signs, xr, W, A, U, R, u2(c.tg), u2(c.ng), c.sid, c.lane);
    });
}

void d_gated_norm_rotate(const float* y, const float* zg, const float* w, const float* signs, float* xr, uint W,
                         uint T) {  // :796-812
    const metal::half* A = nullptr;
    float* U = xr;
    uint R = 0;
    run(T, W / RCHUNK, 1, 128, 1, 1, [&](const Ctx& c) {
        ref::gated_norm_rotate(y, zg, w, signs, xr, W, A, U, R, u2(c.tg), u2(c.ng), c.sid, c.lane);
    });
}

void d_embed(const uint32_t* W, const metal::half* S, const float* signs, const int* ids, float* out, uint D,
             uint T) {  // model.rs:613-630
    run(T, (D + RCHUNK - 1) / RCHUNK, 1, 128, 1, 1, [&](const Ctx& c) {
        ref::embed(W, S, signs, ids, out, D, u2(c.tg), u2(c.ng), c.sid, c.lane);
    });
}

// One ternary matrix of the reference pack (g128, implicit bias): codes [O][K/16], fp16 scales [O][K/128].
struct RLin {
    const uint32_t* w = nullptr;
    const metal::half* s = nullptr;
    const float* signs = nullptr;
    uint O = 0, K = 0;
};

// qmm_lora (model.rs:457-526) without LoRA: matrices ls[i] -> ys[i] sharing x, t rows, optional GDN a/b rows for the
// single-token decode step (qmm_multi, :566-611).
struct AbArgs {
    const float *wa, *wb, *xn;
    float* ab;
    uint nv;
};
void d_qmm_lora(const std::vector<RLin>& ls, const std::vector<float*>& ys, const float* x, uint t, bool add,
                const AbArgs* abargs) {
    const metal::half* nb = nullptr;
    const float* nu = nullptr;
    uint lr = 0, UR = 0;
    const RLin& l0 = ls[0];
    const uint K = l0.K;
    auto L = [&](size_t i) -> const RLin& { return ls[std::min(i, ls.size() - 1)]; };
    auto Y = [&](size_t i) { return ys[std::min(i, ys.size() - 1)]; };
    auto o = [&](size_t i) -> uint { return i < ls.size() ? ls[i].O : 0u; };
    uint total = 0;
    for (auto& l : ls) total += l.O;
    if (t == 1 && ls.size() > 1) {  // qmm_multi: qmv3 + the a/b rows (model.rs:566-611)
        const uint O0 = o(0), O1 = o(1);
        uint extra = abargs ? abargs->nv : 0;
        const float* wa = abargs ? abargs->wa : x;
        const float* wb = abargs ? abargs->wb : x;
        const float* xn = abargs ? abargs->xn : x;
        float* ab = abargs ? abargs->ab : ys[0];
        uint NV = abargs ? abargs->nv : 0;
        run(total / 8 + extra, 1, 1, 64, 1, 1, [&](const Ctx& c) {
            ref::qmv3(L(0).w, L(0).s, Y(0), L(1).w, L(1).s, Y(1), L(2).w, L(2).s, Y(2), x, K, O0, O1, nb, nb, nb, nu,
                      lr, wa, wb, xn, ab, NV, total, c.tg[0], c.sid, c.lane);
        });
        return;
    }
    if (t == 1) {  // qmv4 (model.rs:467-484)
        const uint O = l0.O, a = add ? 1u : 0u;
        run(O / 8, 1, 1, 64, 1, 1, [&](const Ctx& c) {
            ref::qmv4(l0.w, l0.s, x, ys[0], K, O, a, nb, nu, lr, c.tg[0], c.sid, c.lane);
        });
        return;
    }
    // Metal: qmvr for T = 2, 3; qmvxm in 8-row slices for 4..16; qmm above (model.rs:486-497, qmm_fused :530-564)
    const uint step = (t == 2 || t == 3) ? t : (t <= 16 ? 8u : t);
    const uint O0 = o(0), O1 = o(1), a = add ? 1u : 0u;
    for (uint c0 = 0; c0 < t; c0 += step) {
        const uint tt = std::min(step, t - c0);
        float* y0 = Y(0) + (size_t)c0 * L(0).O;
        float* y1 = Y(1) + (size_t)c0 * L(1).O;
        float* y2 = Y(2) + (size_t)c0 * L(2).O;
        const float* xc = x + (size_t)c0 * K;
        if (t == 2 || t == 3) {
            run(total / 8, 1, 1, 64 * tt, 1, 1, [&](const Ctx& c) {
                ref::qmvr(L(0).w, L(0).s, y0, L(1).w, L(1).s, y1, L(2).w, L(2).s, y2, xc, K, O0, O1, total, a, tt, nb,
                          nb, nb, nu, lr, UR, c.tg[0], c.sid, c.lane);
            });
        } else if (t <= 16) {
            run(total / 32, 1, 1, 128, 1, 1, [&](const Ctx& c) {
                ref::qmvxm(L(0).w, L(0).s, y0, L(1).w, L(1).s, y1, L(2).w, L(2).s, y2, xc, K, O0, O1, total, a, tt, nb,
                           nb, nb, nu, lr, UR, c.tg[0], c.sid, c.lane);
            });
        } else {
            run(total / 64, (tt + 31) / 32, 1, 64, 1, 1, [&](const Ctx& c) {
                ref::qmm(L(0).w, L(0).s, y0, L(1).w, L(1).s, y1, L(2).w, L(2).s, y2, xc, K, O0, O1, total, a, tt, nb,
                         nb, nb, nu, lr, UR, u2(c.tg), c.tid, c.sid);
            });
        }
    }
}

// ------------------------------------------------------------------------------------------------ the model
struct Tensor {
    std::vector<uint8_t> data;
};

struct RLayer {
    bool attn = false;
    int idx = 0;  // index among the GDN or attention layers
    const float *in_norm = nullptr, *post_norm = nullptr;
    RLin qkv, z, out, q, k, v, o, gate, up, down;
    const float *wa = nullptr, *wb = nullptr, *alog = nullptr, *dtb = nullptr, *convw = nullptr, *gnorm = nullptr;
    const float *qn = nullptr, *kn = nullptr;
};

struct RModel {
    bcu_config c;
    std::map<std::string, Tensor> t;
    std::vector<RLayer> layers;
    RLin embed;
    const float* final_norm = nullptr;
    std::vector<float> inv_freq;
    uint d = 0, ff = 0, V = 0, C = 0, gw = 0, aw = 0, kvw = 0, nk = 0, nv = 0, n_gdn = 0, n_attn = 0, ctx = 0;
    // State (model.rs:175-186, 256-266)
    std::vector<float> gdn, conv, kc, vc;
    uint len = 0;
    // scratch (model.rs:326-360), sized for TMAX = 512 rows
    std::vector<float> h, xn, xr, a1, a2, qkvc, y, ab, kp, vp, qv, logits, pv, apart;
    std::vector<int> ids, pos, pi, out;
    std::vector<float> v_qkv, v_qkvc, v_ab, v_conv, v_gdn;
};

const std::string PFX = "language_model.model.";

template <class T> const T* tp(RModel* m, const std::string& n) {
    auto it = m->t.find(n);
    return it == m->t.end() ? nullptr : (const T*)it->second.data.data();
}

bool rlin(RModel* m, const std::string& n, RLin* l, uint O, uint K) {
    l->w = tp<uint32_t>(m, n + ".weight");
    l->s = tp<metal::half>(m, n + ".scales");
    l->signs = tp<float>(m, n + ".signs");
    l->O = O;
    l->K = K;
    return l->w && l->s && l->signs && m->t[n + ".weight"].data.size() == (size_t)O * K / 4 &&
           m->t[n + ".scales"].data.size() == (size_t)O * (K / 128) * 2;
}

// Text::encode_layers_at (model.rs:670-934) for t rows in h; verify keeps the GDN inputs per layer and writes the
// candidate states to scratch (v_conv, v_gdn), prefill updates the state in place.
void encode_layers(RModel* m, uint t, bool verify) {
    const uint d = m->d, ff = m->ff, C = m->C, gw = m->gw, aw = m->aw, kvw = m->kvw, nk = m->nk, nv = m->nv;
    const uint H = m->c.heads, KV = m->c.kv_heads, ROT = m->c.rotary_dims, s1 = m->c.mrope[1], s2 = m->c.mrope[2];
    const uint off = m->len;
    for (RLayer& l : m->layers) {
        const RLin& first = l.attn ? l.q : l.qkv;
        d_norm_rotate(m->h.data(), l.in_norm, first.signs, m->xn.data(), m->xr.data(), d, l.attn ? 0u : 1u, t);
        if (!l.attn) {
            const size_t gi = l.idx;
            float* qkv_b = verify ? m->v_qkv.data() + gi * VMAX_ * C : m->a1.data();
            float* qkvc_b = verify ? m->v_qkvc.data() + gi * VMAX_ * C : m->qkvc.data();
            float* ab_b = verify ? m->v_ab.data() + gi * VMAX_ * 2 * nv : m->ab.data();
            float* conv_in = m->conv.data() + gi * 3 * C;
            float* gdn_in = m->gdn.data() + gi * (size_t)nv * 128 * 128;
            float* conv_out = verify ? m->v_conv.data() + gi * 3 * C : conv_in;
            float* gdn_out = verify ? m->v_gdn.data() + gi * (size_t)nv * 128 * 128 : gdn_in;
            const bool fused = t == 1 && !verify;  // model.rs:738
            AbArgs aa{l.wa, l.wb, m->xn.data(), ab_b, nv};
            d_qmm_lora({l.qkv, l.z}, {qkv_b, m->a2.data()}, m->xr.data(), t, false, fused ? &aa : nullptr);
            if (!fused) {  // model.rs:743-757
                const uint NV = nv, K = d;
                run(2 * nv / 4, t, 1, 128, 1, 1, [&](const Ctx& c) {
                    ref::gdn_ab(l.wa, l.wb, m->xn.data(), ab_b, NV, K, u2(c.tg), c.sid, c.lane);
                });
            }
            {  // gdn_conv (model.rs:758-771)
                const uint upd = fused ? 1u : 0u, CC = C, NK = nk;
                run(t, C / 128, 1, 128, 1, 1, [&](const Ctx& c) {
                    ref::gdn_conv(qkv_b, conv_in, l.convw, qkvc_b, upd, CC, NK, u2(c.tg), c.tid, c.sid, c.lane);
                });
            }
            if (!fused) {  // conv_state (model.rs:772-779)
                const uint n = t, CC = C;
                run((C + 127) / 128, 1, 1, 128, 1, 1, [&](const Ctx& c) {
                    ref::conv_state(qkv_b, conv_in, conv_out, n, CC, c.gid[0]);
                });
            }
            {  // gdn_recurrent (model.rs:780-795)
                const uint T = t, NK = nk, NV = nv;
                run(nv, 32, 1, 32, 4, 1, [&](const Ctx& c) {
                    ref::gdn_recurrent(qkvc_b, ab_b, l.alog, l.dtb, gdn_in, gdn_out, m->y.data(), T, NK, NV, u2(c.tg),
                                       u2(c.tp));
                });
            }
            d_gated_norm_rotate(m->y.data(), m->a2.data(), l.gnorm, l.out.signs, m->xr.data(), gw, t);
            d_qmm_lora({l.out}, {m->h.data()}, m->xr.data(), t, true, nullptr);
        } else {
            d_qmm_lora({l.q, l.k, l.v}, {m->a1.data(), m->kp.data(), m->vp.data()}, m->xr.data(), t, false, nullptr);
            float* kc = m->kc.data() + (size_t)l.idx * m->ctx * kvw;
            float* vc = m->vc.data() + (size_t)l.idx * m->ctx * kvw;
            {  // attn_prep (model.rs:828-851)
                const uint T = t, OFF = off, HH = H, KK = KV, RR = ROT, S1 = s1, S2 = s2;
                run(t, H + 2 * KV, 1, 256, 1, 1, [&](const Ctx& c) {
                    ref::attn_prep(m->a1.data(), m->kp.data(), m->vp.data(), l.qn, l.kn, m->pos.data(),
                                   m->inv_freq.data(), m->qv.data(), kc, vc, T, OFF, HH, KK, RR, S1, S2, u2(c.tg), c.tid,
                                   c.sid, c.lane);
                });
            }
            // attn_split + attn_combine (model.rs:852-875): 64-key chunks for decode, 512 for larger t
            const uint n = off + t, chunk = t == 1 ? 64u : 512u, ns = (n + chunk - 1) / chunk;
            {
                const uint OFF = off, CH = chunk, NS = ns, HH = H, KK = KV;
                run(KV, ns, t, 256, 1, 1, [&](const Ctx& c) {
                    ref::attn_split(m->qv.data(), kc, vc, m->apart.data(), OFF, CH, NS, HH, KK,
                                    uint3(c.tg[0], c.tg[1], c.tg[2]), c.tid, c.sid, c.lane);
                });
                run(H, t, 1, 256, 1, 1, [&](const Ctx& c) {
                    ref::attn_combine(m->apart.data(), m->y.data(), NS, HH, u2(c.tg), c.tid);
                });
            }
            d_gate_rotate(m->y.data(), m->a1.data(), l.o.signs, m->xr.data(), aw, t);
            d_qmm_lora({l.o}, {m->h.data()}, m->xr.data(), t, true, nullptr);
        }
        d_norm_rotate(m->h.data(), l.post_norm, l.gate.signs, m->xn.data(), m->xr.data(), d, 0u, t);  // :897-911
        d_qmm_lora({l.gate, l.up}, {m->a1.data(), m->a2.data()}, m->xr.data(), t, false, nullptr);
        d_swiglu_rotate(m->a1.data(), m->a2.data(), l.down.signs, m->xr.data(), ff, t);
        d_qmm_lora({l.down}, {m->h.data()}, m->xr.data(), t, true, nullptr);
    }
}

// Text::encode_head_to (model.rs:941-985) for rows [first, first + n).
void encode_head(RModel* m, uint first, uint n) {
    const uint d = m->d, V = m->V;
    d_norm_rotate(m->h.data() + (size_t)first * d, m->final_norm, m->embed.signs, m->xn.data(), m->xr.data(), d, 0u,
                  n);
    d_qmm_lora({m->embed}, {m->logits.data()}, m->xr.data(), n, false, nullptr);
    const uint VV = V;
    run(ARGMAX_GROUPS, n, 1, 256, 1, 1, [&](const Ctx& c) {
        ref::argmax1(m->logits.data(), m->pv.data(), m->pi.data(), VV, u2(c.tg), u2(c.ng), c.tid, c.sid, c.lane);
    });
    const uint G = ARGMAX_GROUPS;
    run(1, 1, 1, n, 1, 1, [&](const Ctx& c) {
        ref::argmax2(m->pv.data(), m->pi.data(), m->out.data(), G, c.gid[0]);
    });
}

}  // namespace

extern "C" {

// ---------------------------------------------------------------------------------------- single kernels
void rk_norm_rotate(const float* h, const float* w, const float* signs, float* xn, float* xr, uint32_t D,
                    uint32_t write_xn, uint32_t T) {
    d_norm_rotate(h, w, signs, xn, xr, D, write_xn, T);
}
void rk_swiglu_rotate(const float* g, const float* u, const float* signs, float* xr, uint32_t D, uint32_t T) {
    d_swiglu_rotate(g, u, signs, xr, D, T);
}
void rk_gate_rotate(const float* attn, const float* qp, const float* signs, float* xr, uint32_t W, uint32_t T) {
    d_gate_rotate(attn, qp, signs, xr, W, T);
}
void rk_gated_norm_rotate(const float* y, const float* zg, const float* w, const float* signs, float* xr, uint32_t W,
                          uint32_t T) {
    d_gated_norm_rotate(y, zg, w, signs, xr, W, T);
}
void rk_embed(const uint32_t* W, const uint16_t* S, const float* signs, const int32_t* ids, float* out, uint32_t D,
              uint32_t T) {
    d_embed(W, (const metal::half*)S, signs, ids, out, D, T);
}
// y[t][O] (+)= x[t][K] W^T through the kernel model.rs picks for t rows (qmv4, qmvr, qmvxm or qmm).
void rk_ternary_matmul(const uint32_t* W, const uint16_t* S, uint32_t O, uint32_t K, const float* x, uint32_t t,
                       float* y, int32_t add) {
    RLin l;
    l.w = W;
    l.s = (const metal::half*)S;
    l.O = O;
    l.K = K;
    d_qmm_lora({l}, {y}, x, t, add != 0, nullptr);
}
// gdn_gates + gdn_recurrent over T rows of qkvc [T][C] and ab [T][2 NV], state in place (sin == sout allowed).
void rk_gdn_recurrent(const float* qkvc, const float* ab, const float* alog, const float* dtb, const float* sin_,
                      float* sout, float* y, uint32_t T, uint32_t NK, uint32_t NV) {
    run(NV, 32, 1, 32, 4, 1, [&](const Ctx& c) {
        ref::gdn_recurrent(qkvc, ab, alog, dtb, sin_, sout, y, T, NK, NV, u2(c.tg), u2(c.tp));
    });
}
void rk_argmax(const float* x, uint32_t V, uint32_t n, int32_t* out) {
    std::vector<float> pv((size_t)n * ARGMAX_GROUPS);
    std::vector<int> pi((size_t)n * ARGMAX_GROUPS);
    const uint G = ARGMAX_GROUPS;
    run(ARGMAX_GROUPS, n, 1, 256, 1, 1, [&](const Ctx& c) {
        ref::argmax1(x, pv.data(), pi.data(), V, u2(c.tg), u2(c.ng), c.tid, c.sid, c.lane);
    });
    run(1, 1, 1, n, 1, 1, [&](const Ctx& c) { ref::argmax2(pv.data(), pi.data(), out, G, c.gid[0]); });
}

// ---------------------------------------------------------------------------------------- the model
void* rk_model_create(const bcu_config* c) {
    RModel* m = new RModel();
    m->c = *c;
    return m;
}

int rk_model_load_tensor(void* mp, const char* name, const void* data, uint64_t bytes) {
    RModel* m = (RModel*)mp;
    Tensor& t = m->t[name];
    t.data.assign((const uint8_t*)data, (const uint8_t*)data + bytes);
    return 0;
}

// Text::new (model.rs:270-368) for the reference pack: resolves the tensors and sizes the state and scratch.
int rk_model_finalize(void* mp) {
    RModel* m = (RModel*)mp;
    const bcu_config& c = m->c;
    if (c.group_size != 128 || c.has_bias || c.hadamard != 512 || !c.has_signs || c.head_kind != BCU_HEAD_TERNARY)
        return -2;
    if (c.heads != 4 * c.kv_heads || c.head_dim != 256) return -2;  // kernels.metal:3-4
    m->d = c.hidden;
    m->ff = c.intermediate;
    m->V = c.vocab;
    m->nk = c.lin_k_heads;
    m->nv = c.lin_v_heads;
    m->C = (2 * m->nk + m->nv) * 128;
    m->gw = m->nv * 128;
    m->aw = c.heads * 256;
    m->kvw = c.kv_heads * 256;
    m->ctx = c.ctx;
    const std::string p = PFX;
    for (int i = 0; i < c.n_layers; i++) {
        RLayer L;
        std::string l = p + "layers." + std::to_string(i) + ".";
        L.attn = c.layer_is_attn[i] != 0;
        L.in_norm = tp<float>(m, l + "input_layernorm.weight");
        L.post_norm = tp<float>(m, l + "post_attention_layernorm.weight");
        bool ok = L.in_norm && L.post_norm;
        if (L.attn) {
            std::string a = l + "self_attn.";
            L.idx = m->n_attn++;
            ok = ok && rlin(m, a + "q_proj", &L.q, 2 * m->aw, m->d) && rlin(m, a + "k_proj", &L.k, m->kvw, m->d) &&
                 rlin(m, a + "v_proj", &L.v, m->kvw, m->d) && rlin(m, a + "o_proj", &L.o, m->d, m->aw);
            L.qn = tp<float>(m, a + "q_norm.weight");
            L.kn = tp<float>(m, a + "k_norm.weight");
            ok = ok && L.qn && L.kn;
        } else {
            std::string a = l + "linear_attn.";
            L.idx = m->n_gdn++;
            ok = ok && rlin(m, a + "in_proj_qkv", &L.qkv, m->C, m->d) && rlin(m, a + "in_proj_z", &L.z, m->gw, m->d) &&
                 rlin(m, a + "out_proj", &L.out, m->d, m->gw);
            L.wa = tp<float>(m, a + "in_proj_a.weight");
            L.wb = tp<float>(m, a + "in_proj_b.weight");
            L.alog = tp<float>(m, a + "A_log");
            L.dtb = tp<float>(m, a + "dt_bias");
            L.convw = tp<float>(m, a + "conv1d.weight");
            L.gnorm = tp<float>(m, a + "norm.weight");
            ok = ok && L.wa && L.wb && L.alog && L.dtb && L.convw && L.gnorm;
        }
        std::string ml = l + "mlp.";
        ok = ok && rlin(m, ml + "gate_proj", &L.gate, m->ff, m->d) && rlin(m, ml + "up_proj", &L.up, m->ff, m->d) &&
             rlin(m, ml + "down_proj", &L.down, m->d, m->ff);
        if (!ok) return -1;
        m->layers.push_back(L);
    }
    m->final_norm = tp<float>(m, p + "norm.weight");
    if (!m->final_norm || !rlin(m, p + "embed_tokens", &m->embed, m->V, m->d)) return -1;
    const uint half_ = c.rotary_dims / 2;
    m->inv_freq.resize(half_);
    for (uint i = 0; i < half_; i++)  // model.rs:317-321
        m->inv_freq[i] = 1.0f / __builtin_powf((float)c.rope_theta, (float)(2 * i) / (float)c.rotary_dims);
    m->gdn.assign((size_t)m->n_gdn * m->nv * 128 * 128, 0.0f);
    m->conv.assign((size_t)m->n_gdn * 3 * m->C, 0.0f);
    m->kc.assign((size_t)m->n_attn * m->ctx * m->kvw, 0.0f);
    m->vc.assign((size_t)m->n_attn * m->ctx * m->kvw, 0.0f);
    const size_t TM = 512, wide = std::max({m->d, m->ff, m->gw, m->aw});
    m->h.assign(TM * m->d, 0.0f);
    m->xn.assign(TM * m->d, 0.0f);
    m->xr.assign(TM * wide, 0.0f);
    m->a1.assign(TM * std::max({m->ff, m->C, 2 * m->aw}), 0.0f);
    m->a2.assign(TM * std::max(m->ff, m->gw), 0.0f);
    m->qkvc.assign(TM * m->C, 0.0f);
    m->y.assign(TM * std::max(m->gw, m->aw), 0.0f);
    m->ab.assign(TM * 2 * m->nv, 0.0f);
    m->kp.assign(TM * m->kvw, 0.0f);
    m->vp.assign(TM * m->kvw, 0.0f);
    m->qv.assign(TM * m->aw, 0.0f);
    m->logits.assign(TM * (size_t)m->V, 0.0f);
    m->pv.assign(TM * ARGMAX_GROUPS, 0.0f);
    m->pi.assign(TM * ARGMAX_GROUPS, 0);
    m->out.assign(TM, 0);
    m->apart.assign(TM * c.heads * 8 * 258, 0.0f);
    m->ids.assign(TM, 0);
    m->pos.assign(3 * TM, 0);
    m->v_qkv.assign((size_t)m->n_gdn * VMAX_ * m->C, 0.0f);
    m->v_qkvc.assign((size_t)m->n_gdn * VMAX_ * m->C, 0.0f);
    m->v_ab.assign((size_t)m->n_gdn * VMAX_ * 2 * m->nv, 0.0f);
    m->v_conv.assign((size_t)m->n_gdn * 3 * m->C, 0.0f);
    m->v_gdn.assign((size_t)m->n_gdn * m->nv * 128 * 128, 0.0f);
    return 0;
}

// One pass of t rows at the current length: embed, layers, head over all t rows (logits [t][V] and argmax [t]).
// verify = 0 is Model::prefill's chunk (the state advances by t, model.rs:341-386, with the head on every row as
// Model::verify computes it); verify = 1 is Model::verify (:407-421): the state waits for rk_model_accept.
int rk_model_pass(void* mp, const uint32_t* ids, uint32_t t, int32_t verify, float* logits, int32_t* pred) {
    RModel* m = (RModel*)mp;
    if (t < 1 || t > 512 || (verify && t > VMAX_) || m->len + t > m->ctx) return -1;
    for (uint i = 0; i < t; i++) {
        m->ids[i] = (int)ids[i];
        for (int r = 0; r < 3; r++) m->pos[r * t + i] = (int)(m->len + i);  // text positions (mod.rs:454)
    }
    d_embed(m->embed.w, m->embed.s, m->embed.signs, m->ids.data(), m->h.data(), m->d, t);
    encode_layers(m, t, verify != 0);
    encode_head(m, 0, t);
    if (logits) std::memcpy(logits, m->logits.data(), (size_t)t * m->V * 4);
    if (pred) std::memcpy(pred, m->out.data(), (size_t)t * 4);
    if (!verify) m->len += t;
    return 0;
}

// Text::encode_accept (model.rs:1025-1069): commits the first n of the last verify pass's t rows.
void rk_model_accept(void* mp, uint32_t t, uint32_t n) {
    RModel* m = (RModel*)mp;
    const uint C = m->C, nk = m->nk, nv = m->nv;
    for (RLayer& l : m->layers) {
        if (l.attn) continue;
        const size_t gi = l.idx, SS = (size_t)nv * 128 * 128;
        float* cb = m->conv.data() + gi * 3 * C;
        float* gdn = m->gdn.data() + gi * SS;
        if (n == t) {
            std::memcpy(cb, m->v_conv.data() + gi * 3 * C, (size_t)3 * C * 4);
            std::memcpy(gdn, m->v_gdn.data() + gi * SS, SS * 4);
        } else {
            const float* qkv = m->v_qkv.data() + gi * VMAX_ * C;
            const uint N = n, CC = C, NK = nk, NV = nv;
            run((C + 127) / 128, 1, 1, 128, 1, 1, [&](const Ctx& c) { ref::conv_state(qkv, cb, cb, N, CC, c.gid[0]); });
            run(nv, 32, 1, 32, 4, 1, [&](const Ctx& c) {
                ref::gdn_recurrent(m->v_qkvc.data() + gi * VMAX_ * C, m->v_ab.data() + gi * VMAX_ * 2 * nv, l.alog,
                                   l.dtb, gdn, gdn, m->y.data(), N, NK, NV, u2(c.tg), u2(c.tp));
            });
        }
    }
    m->len += n;
}

uint32_t rk_model_len(void* mp) { return ((RModel*)mp)->len; }

void rk_model_destroy(void* mp) { delete (RModel*)mp; }

}  // extern "C"
