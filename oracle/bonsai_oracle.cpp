// bonsai_oracle.cpp — CPU ORACLE (test infrastructure only; never linked into, loaded by or called from the product).
//
// Scalar fp32 restatement of the Ternary Bonsai 2 text path of glimpse-language 0.3.0 (a Rust crate whose only
// backends are Metal and Vulkan): the text kernels of src/bonsai/runtime/kernels.metal (the math spec), the layer
// and accept logic of src/bonsai/runtime/model.rs and the host drafting logic of src/bonsai/runtime/mod.rs. Every
// function cites the reference lines it follows. OpenMP parallelises over output rows and heads only; each output is
// computed by one thread in a fixed order, so results do not depend on the thread count.
//
// PINNED TO THE REFERENCE: the reference's own Metal text kernels (kernels.metal) are compiled for the host from
// the reference tree (oracle/Makefile, oracle/ref_metal/: a Metal-language shim and a threadgroup scheduler) and
// run in the reference's layer sequence (model.rs); tests/test_ref_pin.py checks this restatement against them
// kernel by kernel (bit-exact where nothing reduces) and for whole passes of a model in the reference's format.
// The host logic (drafting, policy, the prefix file) is Rust, which cannot be compiled here: it is pinned by
// known-answer checks in tests/ only. The reference's golden vectors (tests/golden/*/*.json) are MLX text outputs
// of the real PrismML weights, which are not available.
//
// Build: oracle/Makefile (g++ -O2 -fopenmp -ffp-contract=off), output under oracle/_build/.

#include <cmath>
#include <cstdint>
#include <cstring>
#include <map>
#include <string>
#include <vector>
#include <algorithm>

#include "../include/bonsai_cuda.h"

namespace {

// ----------------------------------------------------------------------------------------------- number formats
// IEEE binary16 / bfloat16 conversion with round-to-nearest-even: the `half` 2.7.1 crate (lora.rs:62,108) and the
// GPU's float(half) / half(float) in kernels.metal:242,245.

float f16_to_f32(uint16_t h) {
    uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31, m = h & 1023, u;
    if (e == 0) {
        if (m == 0) u = s;
        else {  // subnormal: normalise
            int sh = 0;
            while (!(m & 1024)) { m <<= 1; sh++; }
            m &= 1023;
            u = s | (uint32_t)(113 - sh) << 23 | m << 13;
        }
    } else if (e == 31) u = s | 0x7f800000u | m << 13;
    else u = s | (e + 112) << 23 | m << 13;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

uint16_t f32_to_f16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    uint32_t s = (u >> 16) & 0x8000, e = (u >> 23) & 255, m = u & 0x7fffff;
    if (e == 255) return (uint16_t)(s | 0x7c00 | (m ? 0x200 : 0));
    int ex = (int)e - 127 + 15;
    if (ex >= 31) return (uint16_t)(s | 0x7c00);
    if (ex <= 0) {  // subnormal or zero
        if (ex < -10) return (uint16_t)s;
        m |= 0x800000;
        int shift = 14 - ex;
        uint32_t q = m >> shift, rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1))) q++;
        return (uint16_t)(s | q);
    }
    uint32_t q = (uint32_t)ex << 10 | m >> 13, rem = m & 0x1fff;
    if (rem > 0x1000 || (rem == 0x1000 && (q & 1))) q++;  // may carry into the exponent: still correct
    return (uint16_t)(s | q);
}

float bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

uint16_t f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffff) > 0x7f800000) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7fff + ((u >> 16) & 1);
    return (uint16_t)(u >> 16);
}

const float EPS = 1e-6f;

// ----------------------------------------------------------------------------------------------- rotation
// Unnormalised Walsh-Hadamard transform, radix-2 stages in ascending stride order: kernels.metal:32-51 (fwht512:
// cross-lane strides 1..16 then in-lane 32..256, "the same butterflies in the same stage order as an in-memory
// radix-2 FWHT"). Add/sub only, so the bits do not depend on the machine.
void fwht(float* x, int n) {
    for (int h = 1; h < n; h <<= 1)
        for (int i = 0; i < n; i += 2 * h)
            for (int j = i; j < i + h; j++) {
                float a = x[j], b = x[j + h];
                x[j] = a + b;
                x[j + h] = a - b;
            }
}

// out = fwht_blocks(signs * x) / sqrt(HB): the rotation of norm_rotate / swiglu_rotate / gate_rotate /
// gated_norm_rotate (kernels.metal:142-143,162-163,186-187,224-225): v = a * sign, fwht, v * INV_SQRT(HB).
void rotate(const float* x, const float* signs, int D, int HB, float* out) {
    float inv = HB == 512 ? 0.044194173824159216f : (float)(1.0 / std::sqrt((double)HB));
    std::vector<float> v(HB);
    for (int b0 = 0; b0 < D; b0 += HB) {
        for (int i = 0; i < HB; i++) v[i] = signs ? x[b0 + i] * signs[b0 + i] : x[b0 + i];
        fwht(v.data(), HB);
        for (int i = 0; i < HB; i++) out[b0 + i] = v[i] * inv;
    }
}

// Sum of squares then 1 / sqrt(mean + eps): row_ss + rsqrt (kernels.metal:56-69,132). fp32 sequential sum.
float rms_scale(const float* x, int D) {
    float ss = 0;
    for (int i = 0; i < D; i++) ss += x[i] * x[i];
    return 1.0f / std::sqrt(ss / (float)D + EPS);
}

inline float sigmoidf_(float a) { return 1.0f / (1.0f + std::exp(-a)); }

// norm_rotate (kernels.metal:118-144) on T rows of D: xn = rmsnorm(h) * w; xr = rotate(signs * xn).
void norm_rotate_rows(const float* h, const float* w, const float* signs, int D, int HB, int T, float* xn, float* xr) {
    for (int t = 0; t < T; t++) {
        const float* x = h + (size_t)t * D;
        float r = rms_scale(x, D);
        float* o = xn + (size_t)t * D;
        for (int i = 0; i < D; i++) o[i] = x[i] * r * w[i];
        rotate(o, signs, D, HB, xr + (size_t)t * D);
    }
}

// swiglu_rotate (kernels.metal:147-164): xr = rotate(signs * (g * u) * sigmoid(g)); xu = the unrotated product.
void swiglu_rotate_rows(const float* g, const float* u, const float* signs, int D, int HB, int T, float* xu,
                        float* xr) {
    for (int t = 0; t < T; t++) {
        float* xo = xu + (size_t)t * D;
        for (int e = 0; e < D; e++) {
            float a = g[(size_t)t * D + e];
            xo[e] = (a * u[(size_t)t * D + e]) * (1.0f / (1.0f + std::exp(-a)));
        }
        rotate(xo, signs, D, HB, xr + (size_t)t * D);
    }
}

// gate_rotate (kernels.metal:170-188): x[e] = attn[e] * sigmoid(gate), the gate from the q projection output
// (per head 256 q then 256 gate values); xr = rotate(signs * x).
void gate_rotate_rows(const float* attn, const float* qp, const float* signs, int W, int HB, int T, float* xu,
                      float* xr) {
    for (int t = 0; t < T; t++) {
        float* xo = xu + (size_t)t * W;
        for (int e = 0; e < W; e++) {
            int hd = e >> 8, dd = e & 255;
            float gt = qp[(size_t)t * 2 * W + hd * 512 + 256 + dd];
            xo[e] = attn[(size_t)t * W + e] * sigmoidf_(gt);
        }
        rotate(xo, signs, W, HB, xr + (size_t)t * W);
    }
}

// gated_norm_rotate (kernels.metal:199-226): per 128-wide head, a * y * rmsnorm scale * w * sigmoid(a) with a the
// z projection (the reference's product order); xr = rotate(signs * x).
void gated_norm_rotate_rows(const float* y, const float* z, const float* w, const float* signs, int W, int HB, int T,
                            float* xu, float* xr) {
    for (int t = 0; t < T; t++) {
        float* xo = xu + (size_t)t * W;
        for (int hd = 0; hd < W / 128; hd++) {
            const float* yh = y + (size_t)t * W + hd * 128;
            float r = rms_scale(yh, 128);
            for (int dd = 0; dd < 128; dd++) {
                float a = z[(size_t)t * W + hd * 128 + dd];
                xo[hd * 128 + dd] = (((a * yh[dd]) * r) * w[dd]) * sigmoidf_(a);
            }
        }
        rotate(xo, signs, W, HB, xr + (size_t)t * W);
    }
}

// ----------------------------------------------------------------------------------------------- ternary linear
// y[t][o] = sum over groups of (s * sum(c * x) + b * sum(x)), c the 2-bit code (MLX affine: w = s * c + b); with
// the reference's implicit bias b = -s this is s * (sum(c * x) - sum(x)), the form of qmv_rows
// (kernels.metal:275-313) and qmv.glsl:19-47: per 16-code step d = sum c*x, xs = sum x, acc += s * (d - xs).
// Steps are visited per lane as in qmv_rows (lane l: k0 = 16 l + 512 i), lane partials summed in lane order.
void ternary_linear(const uint32_t* W, const uint16_t* S, const uint16_t* Bi, int O, int K, int group,
                    const float* X, int T, float* Y) {
    int kw = K / 16, kg = K / group;
#pragma omp parallel for schedule(static)
    for (int o = 0; o < O; o++) {
        for (int t = 0; t < T; t++) {
            const float* x = X + (size_t)t * K;
            float lanes[32];
            for (int l = 0; l < 32; l++) {
                float acc = 0;
                for (int k0 = l * 16; k0 < K; k0 += 512) {
                    uint32_t wd = W[(size_t)o * kw + k0 / 16];
                    float d = 0, xs = 0;
                    for (int j = 0; j < 16; j++) {
                        float c = (float)((wd >> (2 * j)) & 3u);
                        d += c * x[k0 + j];
                        xs += x[k0 + j];
                    }
                    float s = f16_to_f32(S[(size_t)o * kg + k0 / group]);
                    if (Bi) acc += s * d + f16_to_f32(Bi[(size_t)o * kg + k0 / group]) * xs;
                    else acc += s * (d - xs);
                }
                lanes[l] = acc;
            }
            float y = 0;
            for (int l = 0; l < 32; l++) y += lanes[l];
            Y[(size_t)t * O + o] = y;
        }
    }
}

// ----------------------------------------------------------------------------------------------- GatedDeltaNet
// gdn_gates (kernels.metal:556-561): g = exp(-exp(A_log) * softplus(a + dt_bias)), beta = sigmoid(b).
void gdn_gates(float a_in, float b_in, float a_log, float dtb, float* g, float* beta) {
    float a = a_in + dtb;
    float sp = std::max(a, 0.0f) + std::log(1.0f + std::exp(-std::fabs(a)));
    *g = std::exp(-std::exp(a_log) * sp);
    *beta = 1.0f / (1.0f + std::exp(-b_in));
}

// One token of the gated delta rule on one dv row (kernels.metal:607-620): S *= g; kv = S.k; delta = (v - kv) beta;
// S += k delta; y = S.q.
inline float gdn_row_step(float* st, const float* q, const float* k, float v, float g, float beta) {
    float kv = 0;
    for (int i = 0; i < 128; i++) { st[i] *= g; kv += st[i] * k[i]; }
    float delta = (v - kv) * beta;
    float o = 0;
    for (int i = 0; i < 128; i++) { st[i] += k[i] * delta; o += st[i] * q[i]; }
    return o;
}

// ----------------------------------------------------------------------------------------------- attention
// attn_prep (kernels.metal:627-662): rmsnorm(x) * w, interleaved mrope on the first ROT dims (sections s1/s2 for
// the h/w position rows, the rest t), cos/sin in double as `precise::` does.
void attn_norm_rope(float* x, const float* w, int pos, const float* inv_freq, int ROT, int s1, int s2) {
    float r = rms_scale(x, 256);
    float buf[256];
    for (int d = 0; d < 256; d++) buf[d] = x[d] * r * w[d];
    int half = ROT / 2;
    for (int d = 0; d < 256; d++) {
        float v = buf[d];
        if (d < ROT) {
            int i = d % half;
            (void)s1; (void)s2;  // text positions: the three position rows are equal, so the section does not matter
            float ang = (float)pos * inv_freq[i];
            float cs = (float)std::cos((double)ang), sn = (float)std::sin((double)ang);
            v = d < half ? buf[d] * cs - buf[d + half] * sn : buf[d] * cs + buf[d - half] * sn;
        }
        x[d] = v;
    }
}

// ----------------------------------------------------------------------------------------------- model
struct Lin {
    const uint32_t* w = nullptr;
    const uint16_t* s = nullptr;
    const uint16_t* b = nullptr;
    const float* signs = nullptr;
    int O = 0, K = 0;
    // LoRA (lora.rs:89-174): A [lr][K] and B [O][lr] as the device holds them (fp16 values; B with alpha / r folded)
    std::vector<float> la, lb;
    int lr = 0;
};

// y[t] += B (A xu[t]) for T rows (lora.rs:1-3: on the linear's unrotated input), sums in index order: u as
// norm_rotate's A rows (kernels.metal:70-116), the up projection as lora_acc (:251-255).
void lora_add(const Lin& l, const float* xu, int T, float* y) {
    if (!l.lr) return;
    std::vector<float> u(l.lr);
    for (int t = 0; t < T; t++) {
        const float* x = xu + (size_t)t * l.K;
        for (int j = 0; j < l.lr; j++) {
            float a = 0;
            for (int k = 0; k < l.K; k++) a += l.la[(size_t)j * l.K + k] * x[k];
            u[j] = a;
        }
        for (int o = 0; o < l.O; o++) {
            float a = 0;
            for (int j = 0; j < l.lr; j++) a += u[j] * l.lb[(size_t)o * l.lr + j];
            y[(size_t)t * l.O + o] += a;
        }
    }
}

struct Layer {
    bool attn = false;
    const float *in_norm = nullptr, *post_norm = nullptr;
    Lin qkv, z, out, q, k, v, o, gate, up, down;
    const float *wa = nullptr, *wb = nullptr, *alog = nullptr, *dtb = nullptr, *convw = nullptr, *gnorm = nullptr;
    const float *qn = nullptr, *kn = nullptr;
    int gi = -1, ai = -1;
};

struct Tensor {
    int dtype;
    std::vector<int64_t> shape;
    std::vector<uint8_t> data;
};

struct Model {
    bcu_config c;
    std::map<std::string, Tensor> t;
    std::vector<Layer> layers;
    Lin head;  // ternary tied head
    const uint16_t* embed_bf16 = nullptr;
    const float* final_norm = nullptr;
    std::vector<float> inv_freq;
    int n_gdn = 0, n_attn = 0, C = 0, gw = 0, aw = 0, kvw = 0;
    // state: State (model.rs:175-186), fp32 like the reference
    std::vector<float> gdn, conv, kc, vc;
    int len = 0;
    // verify candidates: per GDN layer, the state after each row and the raw qkv rows (accept picks one)
    int last_t = 0;
    std::vector<std::vector<float>> cand_gdn;  // [layer][(T+1) * state]
    std::vector<std::vector<float>> cand_qkv;  // [layer][T * C]
    bool pending = false;
};

struct Snap {
    std::vector<float> gdn, conv, kc, vc;
    int len;
};

const char* PFX = "language_model.model.";

const Tensor* find(const Model* m, const std::string& name) {
    auto it = m->t.find(name);
    return it == m->t.end() ? nullptr : &it->second;
}

template <class T>
const T* ptr(const Model* m, const std::string& name) {
    const Tensor* x = find(m, name);
    return x ? (const T*)x->data.data() : nullptr;
}

bool lin(const Model* m, const std::string& name, Lin* l, int O, int K) {
    const Tensor* w = find(m, name + ".weight");
    if (!w || w->shape.size() != 2 || w->shape[0] != O || w->shape[1] * 16 != K) return false;
    l->w = (const uint32_t*)w->data.data();
    l->s = ptr<uint16_t>(m, name + ".scales");
    l->b = m->c.has_bias ? ptr<uint16_t>(m, name + ".biases") : nullptr;
    l->signs = ptr<float>(m, name + ".signs");
    l->O = O;
    l->K = K;
    return l->s && (!m->c.has_bias || l->b);
}

size_t gdn_state_size(const Model* m) { return (size_t)m->c.lin_v_heads * 128 * 128; }
size_t conv_state_size(const Model* m) { return (size_t)3 * m->C; }

// embed (kernels.metal:230-246) for the ternary tied table: (code - 1) * scale rounded to fp16 (or c*s + b), fwht,
// * INV_SQRT * signs, rounded to fp16. bf16 table: the row as is.
// embed (kernels.metal:230-246) of one row of a ternary tied table: (code - 1) * scale (or c * s + b) rounded to
// fp16, fwht, * INV_SQRT * signs, rounded to fp16.
void embed_ternary_row(const uint32_t* W, const uint16_t* S, const uint16_t* Bi, const float* signs, int group, int HB,
                       int d, uint32_t id, float* out) {
    int kg = d / group;
    std::vector<float> v(d);
    for (int k = 0; k < d; k++) {
        uint32_t wd = W[(size_t)id * (d / 16) + k / 16];
        float c = (float)((wd >> (2 * (k & 15))) & 3u);
        float s = f16_to_f32(S[(size_t)id * kg + k / group]);
        float w = Bi ? c * s + f16_to_f32(Bi[(size_t)id * kg + k / group]) : (c - 1.0f) * s;
        v[k] = f16_to_f32(f32_to_f16(w));
    }
    float inv = HB == 512 ? 0.044194173824159216f : (float)(1.0 / std::sqrt((double)HB));
    for (int b0 = 0; b0 < d; b0 += HB) {
        fwht(v.data() + b0, HB);
        for (int i = 0; i < HB; i++) {
            float sg = signs ? signs[b0 + i] : 1.0f;
            out[b0 + i] = f16_to_f32(f32_to_f16(v[b0 + i] * inv * sg));
        }
    }
}

// embed (kernels.metal:230-246) for the ternary tied table; the bf16 table: the row as is.
void embed_row(const Model* m, uint32_t id, float* out) {
    int d = m->c.hidden;
    if (m->c.head_kind == BCU_HEAD_BF16) {
        for (int i = 0; i < d; i++) out[i] = bf16_to_f32(m->embed_bf16[(size_t)id * d + i]);
        return;
    }
    const Lin& e = m->head;
    embed_ternary_row(e.w, e.s, e.b, m->c.has_signs ? e.signs : nullptr, m->c.group_size, m->c.hadamard, d, id, out);
}

// norm_rotate (kernels.metal:118-144): xn = rmsnorm(h) * w; xr = rotate(signs * xn).
void norm_rotate(const Model* m, const float* h, const float* w, const float* signs, int T, float* xn, float* xr) {
    norm_rotate_rows(h, w, m->c.has_signs ? signs : nullptr, m->c.hidden, m->c.hadamard, T, xn, xr);
}

// One forward of T rows from the committed state: Text::encode_layers(verify = true) + encode_head
// (model.rs:670-985). The committed state is read, never written; candidates are kept for accept().
void forward(Model* m, const uint32_t* ids, int T, float* logits, uint32_t* pred) {
    const bcu_config& c = m->c;
    int d = c.hidden, ff = c.intermediate, C = m->C, gw = m->gw, aw = m->aw, kvw = m->kvw;
    int NK = c.lin_k_heads, NV = c.lin_v_heads, H = c.heads, KV = c.kv_heads, HB = c.hadamard;
    int off = m->len;
    std::vector<float> h((size_t)T * d), xn((size_t)T * d), xr((size_t)T * std::max({d, ff, gw, aw}));
    std::vector<float> a1((size_t)T * std::max({ff, C, 2 * aw})), a2((size_t)T * std::max(ff, gw));
    std::vector<float> y((size_t)T * std::max(gw, aw)), tmp((size_t)T * std::max({d, ff, gw, aw}));
    for (int t = 0; t < T; t++) embed_row(m, ids[t], h.data() + (size_t)t * d);
    m->cand_gdn.assign(m->n_gdn, {});
    m->cand_qkv.assign(m->n_gdn, {});
    for (size_t li = 0; li < m->layers.size(); li++) {
        const Layer& L = m->layers[li];
        const Lin& first = L.attn ? L.q : L.qkv;
        norm_rotate(m, h.data(), L.in_norm, first.signs, T, xn.data(), xr.data());
        if (!L.attn) {
            // qkv and z (model.rs:741), a/b gates (gdn_ab, kernels.metal:504-510), conv (gdn_conv :515-541),
            // recurrent (gdn_recurrent :566-622), gated norm + rotate (:199-226), out_proj with add (model.rs:813)
            ternary_linear(L.qkv.w, L.qkv.s, L.qkv.b, C, d, c.group_size, xr.data(), T, a1.data());
            ternary_linear(L.z.w, L.z.s, L.z.b, gw, d, c.group_size, xr.data(), T, a2.data());
            lora_add(L.qkv, xn.data(), T, a1.data());
            lora_add(L.z, xn.data(), T, a2.data());
            std::vector<float> ab((size_t)T * 2 * NV);
            for (int t = 0; t < T; t++)
                for (int r = 0; r < 2 * NV; r++) {
                    const float* wr = r < NV ? L.wa + (size_t)r * d : L.wb + (size_t)(r - NV) * d;
                    float acc = 0;
                    for (int i = 0; i < d; i++) acc += wr[i] * xn[(size_t)t * d + i];
                    ab[(size_t)t * 2 * NV + r] = acc;
                }
            const float* cs = m->conv.data() + (size_t)L.gi * conv_state_size(m);
            std::vector<float> qkvc((size_t)T * C);
            for (int t = 0; t < T; t++)
                for (int grp = 0; grp < C / 128; grp++) {
                    float vals[128];
                    for (int cc = 0; cc < 128; cc++) {
                        int ch = grp * 128 + cc;
                        float acc = 0;
                        for (int i = 0; i < 4; i++) {
                            int j = t + i;
                            float row = j < 3 ? cs[(size_t)j * C + ch] : a1[(size_t)(j - 3) * C + ch];
                            acc += L.convw[(size_t)ch * 4 + i] * row;
                        }
                        vals[cc] = acc / (1.0f + std::exp(-acc));
                    }
                    if (grp < 2 * NK) {
                        float ss = 0;
                        for (int cc = 0; cc < 128; cc++) ss += vals[cc] * vals[cc];
                        float r = 1.0f / std::sqrt(ss / 128.0f + EPS);
                        float sc = grp < NK ? (1.0f / 128.0f) : 0.08838834764831845f;
                        for (int cc = 0; cc < 128; cc++) vals[cc] = vals[cc] * r * sc;
                    }
                    for (int cc = 0; cc < 128; cc++) qkvc[(size_t)t * C + grp * 128 + cc] = vals[cc];
                }
            // candidate states after each row (accept picks row n; encode_accept, model.rs:1025-1069)
            size_t SS = gdn_state_size(m);
            std::vector<float>& cand = m->cand_gdn[L.gi];
            cand.assign((size_t)(T + 1) * SS, 0);
            memcpy(cand.data(), m->gdn.data() + (size_t)L.gi * SS, SS * 4);
            m->cand_qkv[L.gi].assign(a1.begin(), a1.begin() + (size_t)T * C);
            int ratio = NV / NK;
#pragma omp parallel for schedule(static)
            for (int hd = 0; hd < NV; hd++) {
                int hk = hd / ratio;
                float ea_log = L.alog[hd], dtb = L.dtb[hd];
                for (int dv = 0; dv < 128; dv++) {
                    float st[128];
                    memcpy(st, cand.data() + ((size_t)hd * 128 + dv) * 128, 512);
                    for (int t = 0; t < T; t++) {
                        const float* row = qkvc.data() + (size_t)t * C;
                        float g, beta;
                        gdn_gates(ab[(size_t)t * 2 * NV + hd], ab[(size_t)t * 2 * NV + NV + hd], ea_log, dtb, &g, &beta);
                        float o = gdn_row_step(st, row + hk * 128, row + (NK + hk) * 128, row[(2 * NK + hd) * 128 + dv], g, beta);
                        y[(size_t)t * gw + hd * 128 + dv] = o;
                        memcpy(cand.data() + (size_t)(t + 1) * SS + ((size_t)hd * 128 + dv) * 128, st, 512);
                    }
                }
            }
            std::vector<float> xu((size_t)T * gw);
            gated_norm_rotate_rows(y.data(), a2.data(), L.gnorm, c.has_signs ? L.out.signs : nullptr, gw, HB, T,
                                   xu.data(), xr.data());
            ternary_linear(L.out.w, L.out.s, L.out.b, d, gw, c.group_size, xr.data(), T, tmp.data());
            for (size_t i = 0; i < (size_t)T * d; i++) h[i] += tmp[i];
            lora_add(L.out, xu.data(), T, h.data());
        } else {
            // q (with gate) / k / v (model.rs:825), attn_prep (:828-851), split attention + combine
            // (kernels.metal:713-799) as one exact softmax, gate_rotate (:170-188), o_proj with add (model.rs:894)
            std::vector<float> qp((size_t)T * 2 * aw), kp((size_t)T * kvw), vp((size_t)T * kvw);
            ternary_linear(L.q.w, L.q.s, L.q.b, 2 * aw, d, c.group_size, xr.data(), T, qp.data());
            ternary_linear(L.k.w, L.k.s, L.k.b, kvw, d, c.group_size, xr.data(), T, kp.data());
            ternary_linear(L.v.w, L.v.s, L.v.b, kvw, d, c.group_size, xr.data(), T, vp.data());
            lora_add(L.q, xn.data(), T, qp.data());
            lora_add(L.k, xn.data(), T, kp.data());
            lora_add(L.v, xn.data(), T, vp.data());
            float* kc = m->kc.data() + (size_t)L.ai * c.ctx * kvw;
            float* vc = m->vc.data() + (size_t)L.ai * c.ctx * kvw;
            std::vector<float> qr((size_t)T * H * 256);
            for (int t = 0; t < T; t++) {
                int pos = off + t;
                for (int hh = 0; hh < H; hh++) {
                    float* q = qr.data() + ((size_t)t * H + hh) * 256;
                    memcpy(q, qp.data() + (size_t)t * 2 * aw + hh * 512, 1024);
                    attn_norm_rope(q, L.qn, pos, m->inv_freq.data(), c.rotary_dims, c.mrope[1], c.mrope[2]);
                }
                for (int kh = 0; kh < KV; kh++) {
                    float* k = kc + ((size_t)pos * KV + kh) * 256;
                    memcpy(k, kp.data() + (size_t)t * kvw + kh * 256, 1024);
                    attn_norm_rope(k, L.kn, pos, m->inv_freq.data(), c.rotary_dims, c.mrope[1], c.mrope[2]);
                    memcpy(vc + ((size_t)pos * KV + kh) * 256, vp.data() + (size_t)t * kvw + kh * 256, 1024);
                }
            }
            int qper = H / KV;
#pragma omp parallel for schedule(static)
            for (int th = 0; th < T * H; th++) {
                int t = th / H, hh = th % H, kh = hh / qper, n = off + t + 1;
                const float* q = qr.data() + ((size_t)t * H + hh) * 256;
                std::vector<float> sc(n);
                float mx = -INFINITY;
                for (int j = 0; j < n; j++) {
                    const float* k = kc + ((size_t)j * KV + kh) * 256;
                    float s = 0;
                    for (int dd = 0; dd < 256; dd++) s += (q[dd] * 0.0625f) * k[dd];
                    sc[j] = s;
                    mx = std::max(mx, s);
                }
                float l = 0;
                for (int j = 0; j < n; j++) { sc[j] = std::exp(sc[j] - mx); l += sc[j]; }
                float acc[256] = {0};
                for (int j = 0; j < n; j++) {
                    const float* v = vc + ((size_t)j * KV + kh) * 256;
                    for (int dd = 0; dd < 256; dd++) acc[dd] += sc[j] * v[dd];
                }
                for (int dd = 0; dd < 256; dd++) y[(size_t)t * aw + hh * 256 + dd] = acc[dd] / l;
            }
            std::vector<float> xu((size_t)T * aw);
            gate_rotate_rows(y.data(), qp.data(), c.has_signs ? L.o.signs : nullptr, aw, HB, T, xu.data(), xr.data());
            ternary_linear(L.o.w, L.o.s, L.o.b, d, aw, c.group_size, xr.data(), T, tmp.data());
            for (size_t i = 0; i < (size_t)T * d; i++) h[i] += tmp[i];
            lora_add(L.o, xu.data(), T, h.data());
        }
        // MLP (model.rs:897-932): norm_rotate, gate/up, swiglu_rotate (kernels.metal:147-164), down with add
        norm_rotate(m, h.data(), L.post_norm, L.gate.signs, T, xn.data(), xr.data());
        ternary_linear(L.gate.w, L.gate.s, L.gate.b, ff, d, c.group_size, xr.data(), T, a1.data());
        ternary_linear(L.up.w, L.up.s, L.up.b, ff, d, c.group_size, xr.data(), T, a2.data());
        lora_add(L.gate, xn.data(), T, a1.data());
        lora_add(L.up, xn.data(), T, a2.data());
        std::vector<float> xu((size_t)T * ff);
        swiglu_rotate_rows(a1.data(), a2.data(), c.has_signs ? L.down.signs : nullptr, ff, HB, T, xu.data(), xr.data());
        ternary_linear(L.down.w, L.down.s, L.down.b, d, ff, c.group_size, xr.data(), T, tmp.data());
        for (size_t i = 0; i < (size_t)T * d; i++) h[i] += tmp[i];
        lora_add(L.down, xu.data(), T, h.data());
    }
    // head (model.rs:941-985): final norm, tied table, argmax with ties to the lowest index (kernels.metal:802-842)
    int V = c.vocab;
    std::vector<float> lg((size_t)T * V);
    if (c.head_kind == BCU_HEAD_BF16) {
        for (int t = 0; t < T; t++) {
            const float* x = h.data() + (size_t)t * d;
            float r = rms_scale(x, d);
            for (int i = 0; i < d; i++) xn[(size_t)t * d + i] = x[i] * r * m->final_norm[i];
        }
#pragma omp parallel for schedule(static)
        for (int v = 0; v < V; v++)
            for (int t = 0; t < T; t++) {
                const uint16_t* wr = m->embed_bf16 + (size_t)v * d;
                const float* x = xn.data() + (size_t)t * d;
                float acc = 0;
                for (int i = 0; i < d; i++) acc += bf16_to_f32(wr[i]) * x[i];
                lg[(size_t)t * V + v] = acc;
            }
    } else {
        norm_rotate(m, h.data(), m->final_norm, m->head.signs, T, xn.data(), xr.data());
        ternary_linear(m->head.w, m->head.s, m->head.b, V, d, c.group_size, xr.data(), T, lg.data());
    }
    for (int t = 0; t < T; t++) {
        const float* x = lg.data() + (size_t)t * V;
        float bv = -INFINITY;
        int bi = 0;
        for (int v = 0; v < V; v++)
            if (x[v] > bv) { bv = x[v]; bi = v; }
        if (pred) pred[t] = (uint32_t)bi;
    }
    if (logits) memcpy(logits, lg.data(), lg.size() * 4);
    m->last_t = T;
    m->pending = true;
}

// encode_accept (model.rs:1025-1069): conv state = rows n..n+2 of [state; qkv]; GDN state after row n; len += n.
void accept(Model* m, int n) {
    if (!m->pending) return;
    int C = m->C;
    for (int gi = 0; gi < m->n_gdn; gi++) {
        size_t SS = gdn_state_size(m);
        memcpy(m->gdn.data() + (size_t)gi * SS, m->cand_gdn[gi].data() + (size_t)n * SS, SS * 4);
        float* cs = m->conv.data() + (size_t)gi * conv_state_size(m);
        std::vector<float> old(cs, cs + conv_state_size(m));
        const std::vector<float>& q = m->cand_qkv[gi];
        for (int j = 0; j < 3; j++) {
            int k = n + j;
            for (int ch = 0; ch < C; ch++) cs[(size_t)j * C + ch] = k < 3 ? old[(size_t)k * C + ch] : q[(size_t)(k - 3) * C + ch];
        }
    }
    m->len += n;
    m->pending = false;
}

}  // namespace

// =============================================================================================== C ABI (tests only)
extern "C" {

float orc_f16_to_f32(uint16_t h) { return f16_to_f32(h); }
uint16_t orc_f32_to_f16(float f) { return f32_to_f16(f); }
float orc_bf16_to_f32(uint16_t h) { return bf16_to_f32(h); }
uint16_t orc_f32_to_bf16(float f) { return f32_to_bf16(f); }

void orc_fwht(float* x, int n) { fwht(x, n); }

// The rotation producers and the embedding on their own (the pieces forward() runs), for kernel-level checks.
void orc_norm_rotate(const float* h, const float* w, const float* signs, int D, int HB, int T, float* xn, float* xr) {
    norm_rotate_rows(h, w, signs, D, HB, T, xn, xr);
}
void orc_swiglu_rotate(const float* g, const float* u, const float* signs, int D, int HB, int T, float* xr) {
    std::vector<float> xu((size_t)T * D);
    swiglu_rotate_rows(g, u, signs, D, HB, T, xu.data(), xr);
}
void orc_gate_rotate(const float* attn, const float* qp, const float* signs, int W, int HB, int T, float* xr) {
    std::vector<float> xu((size_t)T * W);
    gate_rotate_rows(attn, qp, signs, W, HB, T, xu.data(), xr);
}
void orc_gated_norm_rotate(const float* y, const float* z, const float* w, const float* signs, int W, int HB, int T,
                           float* xr) {
    std::vector<float> xu((size_t)T * W);
    gated_norm_rotate_rows(y, z, w, signs, W, HB, T, xu.data(), xr);
}
void orc_embed_ternary(const uint32_t* W, const uint16_t* S, const uint16_t* B, const float* signs, int group, int HB,
                       int d, const uint32_t* ids, int T, float* out) {
    for (int t = 0; t < T; t++) embed_ternary_row(W, S, B, signs, group, HB, d, ids[t], out + (size_t)t * d);
}
void orc_rotate(const float* x, const float* signs, int D, int HB, float* out) { rotate(x, signs, D, HB, out); }

void orc_ternary_linear(const uint32_t* W, const uint16_t* S, const uint16_t* B, int O, int K, int group,
                        const float* X, int T, float* Y) {
    ternary_linear(W, S, B, O, K, group, X, T, Y);
}

// Graded config 1: Y = W . H(X) with X bf16, H the normalised HB-point transform (optional signs).
void orc_rotate_ternary_linear(const uint32_t* W, const uint16_t* S, const uint16_t* B, int O, int K, int group,
                               const uint16_t* Xbf, int T, int HB, const float* signs, float* Y, float* Xrot) {
    std::vector<float> x((size_t)T * K), xr((size_t)T * K);
    for (size_t i = 0; i < x.size(); i++) x[i] = bf16_to_f32(Xbf[i]);
    for (int t = 0; t < T; t++) rotate(x.data() + (size_t)t * K, signs, K, HB, xr.data() + (size_t)t * K);
    if (Xrot) memcpy(Xrot, xr.data(), xr.size() * 4);
    ternary_linear(W, S, B, O, K, group, xr.data(), T, Y);
}

// Graded config 2: gdn_gates + gdn_recurrent over T rows (kernels.metal:556-622), outputs y for every row and the
// state after the first n rows (rollback, model.rs:1040-1063).
void orc_gdn_verify(const float* q, const float* k, const float* v, const float* a_in, const float* b_in,
                    const float* a_log, const float* dt_bias, float* state, float* y, int T, int NK, int NV, int n) {
    int ratio = NV / NK;
#pragma omp parallel for schedule(static)
    for (int hd = 0; hd < NV; hd++) {
        int hk = hd / ratio;
        for (int dv = 0; dv < 128; dv++) {
            float st[128], keep[128];
            float* S = state + ((size_t)hd * 128 + dv) * 128;
            memcpy(st, S, 512);
            memcpy(keep, S, 512);
            for (int t = 0; t < T; t++) {
                float g, beta;
                gdn_gates(a_in[(size_t)t * NV + hd], b_in[(size_t)t * NV + hd], a_log[hd], dt_bias[hd], &g, &beta);
                y[((size_t)t * NV + hd) * 128 + dv] =
                    gdn_row_step(st, q + ((size_t)t * NK + hk) * 128, k + ((size_t)t * NK + hk) * 128,
                                 v[((size_t)t * NV + hd) * 128 + dv], g, beta);
                if (t + 1 == n) memcpy(keep, st, 512);
            }
            memcpy(S, keep, 512);
        }
    }
}

// Accept length (runtime/mod.rs:867): leading drafts ids[1..t) equal to pred[0..t-1).
int orc_accept_len(const uint32_t* ids, const uint32_t* pred, int t) {
    int m = 0;
    while (m < t - 1 && ids[m + 1] == pred[m]) m++;
    return m;
}

int orc_argmax(const float* x, int n) {
    float bv = -INFINITY;
    int bi = 0;
    for (int i = 0; i < n; i++)
        if (x[i] > bv) { bv = x[i]; bi = i; }
    return bi;
}

void* orc_model_create(const bcu_config* c) {
    Model* m = new Model();
    m->c = *c;
    return m;
}

int orc_model_load_tensor(void* mp, const char* name, int dtype, const int64_t* shape, int ndim, const void* data) {
    Model* m = (Model*)mp;
    Tensor t;
    t.dtype = dtype;
    size_t n = 1;
    for (int i = 0; i < ndim; i++) { t.shape.push_back(shape[i]); n *= (size_t)shape[i]; }
    size_t es = dtype == BCU_U32 || dtype == BCU_F32 ? 4 : 2;
    t.data.assign((const uint8_t*)data, (const uint8_t*)data + n * es);
    m->t[name] = std::move(t);
    return 0;
}

// Text::new (model.rs:270-368): resolve tensors, allocate state. Returns 0 or -1 (missing/mis-shaped tensor).
int orc_model_finalize(void* mp) {
    Model* m = (Model*)mp;
    const bcu_config& c = m->c;
    int d = c.hidden, ff = c.intermediate;
    m->C = 2 * c.lin_k_heads * 128 + c.lin_v_heads * 128;
    m->gw = c.lin_v_heads * 128;
    m->aw = c.heads * 256;
    m->kvw = c.kv_heads * 256;
    m->layers.clear();
    m->n_gdn = m->n_attn = 0;
    std::string p = PFX;
    for (int i = 0; i < c.n_layers; i++) {
        Layer L;
        std::string l = p + "layers." + std::to_string(i) + ".";
        L.attn = c.layer_is_attn[i] != 0;
        L.in_norm = ptr<float>(m, l + "input_layernorm.weight");
        L.post_norm = ptr<float>(m, l + "post_attention_layernorm.weight");
        bool ok = L.in_norm && L.post_norm;
        if (L.attn) {
            ok = ok && lin(m, l + "self_attn.q_proj", &L.q, 2 * m->aw, d) && lin(m, l + "self_attn.k_proj", &L.k, m->kvw, d) &&
                 lin(m, l + "self_attn.v_proj", &L.v, m->kvw, d) && lin(m, l + "self_attn.o_proj", &L.o, d, m->aw);
            L.qn = ptr<float>(m, l + "self_attn.q_norm.weight");
            L.kn = ptr<float>(m, l + "self_attn.k_norm.weight");
            ok = ok && L.qn && L.kn;
            L.ai = m->n_attn++;
        } else {
            std::string a = l + "linear_attn.";
            ok = ok && lin(m, a + "in_proj_qkv", &L.qkv, m->C, d) && lin(m, a + "in_proj_z", &L.z, m->gw, d) &&
                 lin(m, a + "out_proj", &L.out, d, m->gw);
            L.wa = ptr<float>(m, a + "in_proj_a.weight");
            L.wb = ptr<float>(m, a + "in_proj_b.weight");
            L.alog = ptr<float>(m, a + "A_log");
            L.dtb = ptr<float>(m, a + "dt_bias");
            L.convw = ptr<float>(m, a + "conv1d.weight");
            L.gnorm = ptr<float>(m, a + "norm.weight");
            ok = ok && L.wa && L.wb && L.alog && L.dtb && L.convw && L.gnorm;
            L.gi = m->n_gdn++;
        }
        ok = ok && lin(m, l + "mlp.gate_proj", &L.gate, ff, d) && lin(m, l + "mlp.up_proj", &L.up, ff, d) &&
             lin(m, l + "mlp.down_proj", &L.down, d, ff);
        if (!ok) return -1;
        m->layers.push_back(L);
    }
    m->final_norm = ptr<float>(m, p + "norm.weight");
    if (!m->final_norm) return -1;
    if (c.head_kind == BCU_HEAD_BF16) {
        m->embed_bf16 = ptr<uint16_t>(m, p + "embed_tokens.weight");
        if (!m->embed_bf16) return -1;
    } else if (!lin(m, p + "embed_tokens", &m->head, c.vocab, d)) {
        return -1;
    }
    int half = c.rotary_dims / 2;
    m->inv_freq.resize(half);
    for (int i = 0; i < half; i++)  // model.rs:318-320
        m->inv_freq[i] = 1.0f / std::pow((float)c.rope_theta, (float)(2 * i) / (float)c.rotary_dims);
    m->gdn.assign((size_t)m->n_gdn * gdn_state_size(m), 0);
    m->conv.assign((size_t)m->n_gdn * conv_state_size(m), 0);
    m->kc.assign((size_t)m->n_attn * c.ctx * m->kvw, 0);
    m->vc.assign((size_t)m->n_attn * c.ctx * m->kvw, 0);
    m->len = 0;
    m->pending = false;
    return 0;
}

void orc_model_reset(void* mp) {
    Model* m = (Model*)mp;
    std::fill(m->gdn.begin(), m->gdn.end(), 0.0f);
    std::fill(m->conv.begin(), m->conv.end(), 0.0f);
    m->len = 0;
    m->pending = false;
}

// Model::verify (runtime/mod.rs:407-421) without the commit: argmax per row (+ fp32 logits when not NULL). A pending
// accept of the previous pass is applied first (encode_pending, mod.rs:149-153). Returns -1 if the context is full.
int orc_model_forward(void* mp, const uint32_t* ids, int T, float* logits, uint32_t* pred) {
    Model* m = (Model*)mp;
    if (m->len + T > m->c.ctx) return -1;
    forward(m, ids, T, logits, pred);
    return 0;
}

void orc_model_accept(void* mp, int n) { accept((Model*)mp, n); }
int orc_model_len(void* mp) { return ((Model*)mp)->len; }

// Model::prefill / step through forward + accept(all rows).
int orc_model_prefill(void* mp, const uint32_t* ids, int n, int chunk, uint32_t* next) {
    Model* m = (Model*)mp;
    std::vector<uint32_t> pred(chunk);
    for (int i = 0; i < n; i += chunk) {
        int t = std::min(chunk, n - i);
        if (orc_model_forward(m, ids + i, t, nullptr, pred.data())) return -1;
        accept(m, t);
        *next = pred[t - 1];
    }
    return 0;
}

void* orc_model_snapshot(void* mp) {
    Model* m = (Model*)mp;
    Snap* s = new Snap{m->gdn, m->conv, m->kc, m->vc, m->len};
    return s;
}

void orc_model_restore(void* mp, const void* sp) {
    Model* m = (Model*)mp;
    const Snap* s = (const Snap*)sp;
    m->gdn = s->gdn;
    m->conv = s->conv;
    m->kc = s->kc;
    m->vc = s->vc;
    m->len = s->len;
    m->pending = false;
}

void orc_state_free(void* sp) { delete (Snap*)sp; }

// Sets the committed state from the four parts of Text::state_parts (model.rs:1090-1099), the layout the device's
// bcu_state_read/write use: GDN [gdn layer][NV][128][128], conv [gdn layer][3][C], K and V [attn layer][len][KV*256].
// Lets a test start a pass at a long context without prefilling it. Returns -1 when len exceeds the context.
int orc_model_set_state(void* mp, const float* gdn, const float* conv, const float* kc, const float* vc, int len) {
    Model* m = (Model*)mp;
    if (len < 0 || len > m->c.ctx) return -1;
    std::copy(gdn, gdn + m->gdn.size(), m->gdn.begin());
    std::copy(conv, conv + m->conv.size(), m->conv.begin());
    size_t row = (size_t)m->kvw;
    for (int a = 0; a < m->n_attn; a++) {
        std::copy(kc + (size_t)a * len * row, kc + (size_t)(a + 1) * len * row, m->kc.begin() + (size_t)a * m->c.ctx * row);
        std::copy(vc + (size_t)a * len * row, vc + (size_t)(a + 1) * len * row, m->vc.begin() + (size_t)a * m->c.ctx * row);
    }
    m->len = len;
    m->pending = false;
    return 0;
}

// One adapted linear (lora.rs:89-174): A [r][K] rounded to fp16, B [O][r] times fold rounded to fp16. Returns 0, or
// -1 for an unknown layer/module or a shape mismatch. r = 0 removes it.
int orc_model_set_lora(void* mp, int layer, const char* module, const float* a, const float* b, int r, float fold) {
    Model* m = (Model*)mp;
    if (layer < 0 || layer >= (int)m->layers.size()) return -1;
    Layer& L = m->layers[layer];
    const std::string mod(module);
    Lin* l = nullptr;
    if (L.attn) {
        if (mod == "self_attn.q_proj") l = &L.q;
        if (mod == "self_attn.k_proj") l = &L.k;
        if (mod == "self_attn.v_proj") l = &L.v;
        if (mod == "self_attn.o_proj") l = &L.o;
    } else {
        if (mod == "linear_attn.in_proj_qkv") l = &L.qkv;
        if (mod == "linear_attn.in_proj_z") l = &L.z;
        if (mod == "linear_attn.out_proj") l = &L.out;
    }
    if (mod == "mlp.gate_proj") l = &L.gate;
    if (mod == "mlp.up_proj") l = &L.up;
    if (mod == "mlp.down_proj") l = &L.down;
    if (!l) return -1;
    l->lr = r;
    l->la.assign((size_t)r * l->K, 0.0f);
    l->lb.assign((size_t)l->O * r, 0.0f);
    for (size_t i = 0; i < l->la.size(); i++) l->la[i] = f16_to_f32(f32_to_f16(a[i]));
    for (size_t i = 0; i < l->lb.size(); i++) l->lb[i] = f16_to_f32(f32_to_f16(b[i] * fold));
    return 0;
}

// lora_add on its own: y [T][O] += B (A xu) with A [r][K], B [O][r] taken as given (no rounding).
void orc_lora_add(const float* a, const float* b, int r, int O, int K, const float* xu, int T, float* y) {
    Lin l;
    l.O = O;
    l.K = K;
    l.lr = r;
    l.la.assign(a, a + (size_t)r * K);
    l.lb.assign(b, b + (size_t)O * r);
    lora_add(l, xu, T, y);
}

void orc_model_clear_lora(void* mp) {
    for (Layer& L : ((Model*)mp)->layers)
        for (Lin* l : {&L.qkv, &L.z, &L.out, &L.q, &L.k, &L.v, &L.o, &L.gate, &L.up, &L.down}) {
            l->lr = 0;
            l->la.clear();
            l->lb.clear();
        }
}
void orc_model_destroy(void* mp) { delete (Model*)mp; }

// Greedy decoding, one token per step (decode_plain semantics, runtime/mod.rs:901-956): out[0] = first.
int orc_greedy(void* mp, uint32_t first, int max_tokens, const uint32_t* eos, int n_eos, uint32_t* out) {
    Model* m = (Model*)mp;
    int n = 0;
    uint32_t cur = first;
    if (max_tokens <= 0) return 0;
    out[n++] = cur;
    while (n < max_tokens) {
        uint32_t next;
        if (orc_model_forward(m, &cur, 1, nullptr, &next)) break;
        accept(m, 1);
        bool stop = false;
        for (int i = 0; i < n_eos; i++) stop |= next == eos[i];
        if (stop) break;
        out[n++] = next;
        cur = next;
    }
    return n;
}

// ------------------------------------------------------------------------------------ drafting (runtime/mod.rs)
// token_key (mod.rs:73-81): bit 0 = word token, bit 1 = contains a line break; FNV-1a of the lowercase bytes
// without the leading space.
uint64_t orc_token_key(const uint8_t* bytes, int n) {
    uint64_t nl = 0;
    for (int i = 0; i < n; i++)
        if (bytes[i] == '\n') nl = 2;
    const uint8_t* b = bytes;
    int len = n;
    if (len > 0 && b[0] == ' ') { b++; len--; }
    bool all = true;
    for (int i = 0; i < len; i++) {
        uint8_t c = b[i];
        bool punct = (c >= 33 && c <= 47) || (c >= 58 && c <= 64) || (c >= 91 && c <= 96) || (c >= 123 && c <= 126);
        bool ws = c == ' ' || c == '\t' || c == '\n' || c == '\r' || c == 0x0c;
        if (!punct && !ws) { all = false; break; }
    }
    if (all) return nl;
    uint64_t h = 0xcbf29ce484222325ull;
    for (int i = 0; i < len; i++) {
        uint8_t c = b[i];
        if (c >= 'A' && c <= 'Z') c = (uint8_t)(c + 32);
        h = (h ^ c) * 0x100000001b3ull;
    }
    return (h & ~3ull) | 1 | nl;
}

// lookup (mod.rs:87-124) with BACK = 24 (mod.rs:127). src: source ids; keys: per-vocab keys. Writes the draft
// (at most min(draft_max, limit, 15) ids) to out; returns its length, and the source position in *dpos.
int orc_lookup(const uint32_t* src, int n_src, const uint32_t* seq, int n_seq, const uint64_t* keys, int n_keys,
               int ngram_max, int ngram_min, int draft_max, int limit, int cursor, uint32_t* out, int* dpos) {
    const int BACK = 24, VMAX = 16;
    int k = std::min(std::min(draft_max, limit), VMAX - 1);
    *dpos = cursor;
    if (k <= 0) return 0;
    std::vector<std::pair<uint64_t, int>> w;
    for (int i = 0; i < n_src; i++) {
        uint64_t key = (int64_t)src[i] < n_keys ? keys[src[i]] : 0;
        if (key & 1) w.push_back({key, i});
    }
    std::vector<uint64_t> pat;
    int taken = 0;
    for (int i = n_seq - 1; i >= 0 && taken < 4 * ngram_max; i--, taken++) {
        if ((int)pat.size() == ngram_max) break;
        uint64_t key = (int64_t)seq[i] < n_keys ? keys[seq[i]] : 0;
        if (key & 1) pat.push_back(key);
    }
    std::reverse(pat.begin(), pat.end());
    for (int n = std::min(ngram_max, (int)pat.size()); n >= ngram_min && n >= 1; n--) {
        const uint64_t* p = pat.data() + pat.size() - n;
        int hit = -1;
        int lim = (int)w.size() - (n - 1);
        for (int i = 0; i < lim; i++) {
            bool eq = true;
            for (int q = 0; q < n; q++)
                if (w[i + q].first != p[q]) { eq = false; break; }
            if (!eq) continue;
            int j = w[i + n - 1].second + 1;
            if (j < n_src && j + BACK >= cursor && (hit < 0 || j >= cursor)) hit = j;
            if (j >= cursor) break;
        }
        if (hit >= 0) {
            int e = std::min(hit + k, n_src);
            for (int i = hit; i < e; i++) out[i - hit] = src[i];
            *dpos = hit;
            return e - hit;
        }
    }
    return 0;
}

// draft_source (mod.rs:733-768). The vocabulary is one byte string: token i = bytes[offsets[i]..offsets[i+1]).
// Concatenate the user turn's bytes, find the first of SOURCE_TAGS (mod.rs:130) whose opening and then closing tag
// both occur, keep the tokens lying wholly inside (end > lo, start >= lo, end <= hi), drop the filler ids.
int orc_draft_source(const uint32_t* user, int n, const uint8_t* bytes, const uint64_t* offsets, int vocab,
                     const uint32_t* fillers, int n_fillers, uint32_t* out) {
    static const char* tags[2][2] = {{"<transcript>\n", "\n</transcript>"}, {"<text>\n", "\n</text>"}};
    auto tok = [&](uint32_t id) {
        return (int)id < vocab ? std::string((const char*)bytes + offsets[id], offsets[id + 1] - offsets[id]) : std::string();
    };
    std::string text;
    std::vector<size_t> ends;
    for (int i = 0; i < n; i++) {
        text += tok(user[i]);
        ends.push_back(text.size());
    }
    // Rust's find: first window equal to pat at or after `from`
    auto find = [&](const std::string& pat, size_t from, size_t* at) {
        for (size_t i = from; i + pat.size() <= text.size(); i++)
            if (text.compare(i, pat.size(), pat) == 0) { *at = i; return true; }
        return false;
    };
    size_t lo = 0, hi = text.size();
    for (int t = 0; t < 2; t++) {
        size_t a, b;
        if (!find(tags[t][0], 0, &a)) continue;
        a += std::strlen(tags[t][0]);
        if (!find(tags[t][1], a, &b)) continue;
        lo = a;
        hi = b;
        break;
    }
    int m = 0;
    for (int i = 0; i < n; i++) {
        size_t len = tok(user[i]).size();
        if (!(ends[i] > lo && ends[i] - len >= lo && ends[i] <= hi)) continue;
        bool filler = false;
        for (int f = 0; f < n_fillers; f++) filler |= fillers[f] == user[i];
        if (!filler) out[m++] = user[i];
    }
    return m;
}

// normalize_draft (mod.rs:699-729) with the tokenizer as a callback: encode(user, text, n, out, cap) -> count.
typedef int32_t (*orc_encode_fn)(void* user, const uint8_t* text, int32_t n, uint32_t* out, int32_t cap);
int orc_normalize_draft(uint32_t* draft, int n, uint32_t last, const uint8_t* bytes, const uint64_t* offsets, int vocab,
                        orc_encode_fn encode, void* user) {
    static const char* capitalized[18] = {"monday", "tuesday", "wednesday", "thursday", "friday", "saturday",
                                          "sunday", "january", "february", "march", "april", "june", "july",
                                          "august", "september", "october", "november", "december"};
    static const char* contractions[22][2] = {
        {"dont", "don't"}, {"doesnt", "doesn't"}, {"didnt", "didn't"}, {"isnt", "isn't"}, {"wasnt", "wasn't"},
        {"arent", "aren't"}, {"werent", "weren't"}, {"wont", "won't"}, {"cant", "can't"}, {"couldnt", "couldn't"},
        {"wouldnt", "wouldn't"}, {"shouldnt", "shouldn't"}, {"havent", "haven't"}, {"hasnt", "hasn't"},
        {"im", "I'm"}, {"ive", "I've"}, {"youre", "you're"}, {"theyre", "they're"}, {"thats", "that's"},
        {"whats", "what's"}, {"theres", "there's"}, {"lets", "let's"}};
    auto tok = [&](uint32_t id) {
        return (int)id < vocab ? std::string((const char*)bytes + offsets[id], offsets[id + 1] - offsets[id]) : std::string();
    };
    // trim_ascii_end().last() in ".?!"
    auto sentence_end = [](std::string w) {
        while (!w.empty() && (w.back() == ' ' || w.back() == '\t' || w.back() == '\n' || w.back() == '\f' || w.back() == '\r'))
            w.pop_back();
        return !w.empty() && (w.back() == '.' || w.back() == '?' || w.back() == '!');
    };
    const int k = n;
    std::vector<uint32_t> d(draft, draft + n), out;
    bool prev_end = sentence_end(tok(last));
    int i = 0;
    while (i < (int)d.size() && (int)out.size() < k) {
        int j = i + 1;
        for (; j < (int)d.size(); j++) {
            std::string b = tok(d[j]);
            if (b.empty()) continue;
            unsigned char c = (unsigned char)b[0];
            bool alpha = (c >= 'a' && c <= 'z') || (c >= 'A' && c <= 'Z');
            if (!alpha && c != '\'') break;
        }
        std::string w;
        for (int q = i; q < j; q++) w += tok(d[q]);
        std::string v = w;
        bool lower = v.size() > 1 && v[0] == ' ';
        for (size_t q = 1; lower && q < v.size(); q++) lower = v[q] >= 'a' && v[q] <= 'z';
        if (lower) {
            std::string bare = w.substr(1);
            int ci = -1;
            for (int c = 0; c < 22; c++)
                if (bare == contractions[c][0]) { ci = c; break; }
            bool cap = bare == "i" || prev_end;
            for (int c = 0; c < 18; c++) cap = cap || bare == capitalized[c];
            if (ci >= 0) v = std::string(" ") + contractions[ci][1];
            else if (cap) v[1] = (char)(v[1] - 32);
        }
        if (v != w) {
            std::vector<uint32_t> ids(v.size() + 16);
            int c = encode(user, (const uint8_t*)v.data(), (int32_t)v.size(), ids.data(), (int32_t)ids.size());
            out.insert(out.end(), ids.begin(), ids.begin() + c);
        } else {
            out.insert(out.end(), d.begin() + i, d.begin() + j);
        }
        prev_end = sentence_end(w);
        i = j;
    }
    if ((int)out.size() > k) out.resize(k);
    for (size_t q = 0; q < out.size(); q++) draft[q] = out[q];
    return (int)out.size();
}

// Policy::choose (mod.rs:187-202): best k in 1..=min(kmax, limit) by E(k)/cost[k], E(k) = (1 - p^(k+1)) / (1 - p).
int orc_policy_choose(double acc, double rej, const double* cost, int kmax, int limit, double min_gain, double* gain) {
    double p = (acc + 3.4) / (acc + rej + 3.4 + 0.6);
    int bk = 0;
    double bg = 1.0;
    for (int k = 1; k <= std::min(std::min(kmax, 7), limit); k++) {
        double g = (1.0 - std::pow(p, k + 1)) / (1.0 - p) / cost[k];
        if (g > bg && g > min_gain) { bk = k; bg = g; }
    }
    if (gain) *gain = bg;
    return bk;
}

}  // extern "C"
