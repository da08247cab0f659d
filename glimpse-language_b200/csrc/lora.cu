// lora.cu — installs a LoRA adapter (lora.rs:89-174 + Text::set_lora, model.rs:392-397) on the packed linears of a
// finalized model. The GEMV computes it (ternary.cu): its operand builders take the dot products of each token's
// unrotated input block with the stacked A rows (norm_rotate's fused A rows, kernels.metal:70-116), and the CTA that
// writes a row block's outputs adds B . u (store_post, kernels.metal:257-262).
//
// Device layout per adapted group (linears sharing an input, Text::linears order): A fp16 in the builders' lane order
// [K / HB][R = members x r][32 lanes][HB / 32] (element e of lane l of block b is input b HB + l + 32 e), B fp16
// [O of the fused linear][r]; r is the adapter's rank rounded up to a multiple of 8 with zero rows and columns.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "model.h"

using namespace bcu;

namespace {

struct Member {
    const char* name;
    int O, K;
};

// Text::linears (model.rs:372-385) for one layer of this model: the 4 groups and their members (rows of the fused
// linear in member order).
std::vector<std::vector<Member>> groups_of(const bcu_model* m, const Layer& L) {
    const int d = m->c.hidden, ff = m->c.intermediate;
    std::vector<std::vector<Member>> g(4);
    if (L.attn) {
        g[0] = {{"self_attn.q_proj", 2 * m->aw, d}, {"self_attn.k_proj", m->kvw, d}, {"self_attn.v_proj", m->kvw, d}};
        g[1] = {{"self_attn.o_proj", d, m->aw}};
    } else {
        g[0] = {{"linear_attn.in_proj_qkv", m->C, d}, {"linear_attn.in_proj_z", m->gw, d}};
        g[1] = {{"linear_attn.out_proj", d, m->gw}};
    }
    g[2] = {{"mlp.gate_proj", ff, d}, {"mlp.up_proj", ff, d}};
    g[3] = {{"mlp.down_proj", d, ff}};
    return g;
}

Lin* group_lin(Layer& L, int gi) { return gi == 0 ? &L.mix_in : gi == 1 ? &L.mix_out : gi == 2 ? &L.gu : &L.down; }

uint16_t f16(float x) { return __half_as_ushort(__float2half_rn(x)); }

void clear(bcu_model* m) {
    for (auto& L : m->layers)
        for (int gi = 0; gi < 4; gi++) group_lin(L, gi)->lora = LoraArgs();
    if (m->lora_buf) cudaFree(m->lora_buf);
    if (m->lora_upart) cudaFree(m->lora_upart);
    m->lora_buf = nullptr;
    m->lora_upart = nullptr;
    m->lora_rank = m->lora_linears = 0;
    m->lora_bytes = 0;
}

// Pass graphs hold the GEMV parameters by value: drop them (recaptured on next use), and the verify costs measured
// with them.
void drop_graphs(bcu_model* m) {
    for (int t = 0; t <= VMAX; t++) {
        if (m->graphs[t]) cudaGraphExecDestroy(m->graphs[t]);
        m->graphs[t] = nullptr;
        m->graph_nodes[t] = 0;
    }
    m->cost_ready = false;
}

}  // namespace

extern "C" {

bcu_status bcu_set_lora(bcu_model* m, const bcu_lora_linear* lins, int32_t n, float fold) {
    if (!m || !m->finalized || n < 0 || (n && !lins)) return fail(m, BCU_ERR_ARG, "bad LoRA request");
    if (cudaSetDevice(m->device) != cudaSuccess) return fail(m, BCU_ERR_CUDA, "cudaSetDevice");
    const int HB = m->c.hadamard;
    // validate everything before touching the installed adapter
    struct Use {
        const bcu_lora_linear* e = nullptr;
    };
    std::vector<std::vector<std::vector<Use>>> use(m->layers.size());
    for (size_t li = 0; li < m->layers.size(); li++) {
        auto g = groups_of(m, m->layers[li]);
        use[li].resize(4);
        for (int gi = 0; gi < 4; gi++) use[li][gi].resize(g[gi].size());
    }
    int rank = 0;
    for (int i = 0; i < n; i++) {
        const bcu_lora_linear& e = lins[i];
        const std::string key = "layers." + std::to_string(e.layer) + "." + (e.module ? e.module : "");
        if (!e.module || e.layer < 0 || e.layer >= (int)m->layers.size())
            return fail(m, BCU_ERR_ARG, "lora: tensors for unsupported modules, e.g. " + key);
        auto g = groups_of(m, m->layers[e.layer]);
        int gi = -1, mi = -1;
        for (int a = 0; a < 4 && gi < 0; a++)
            for (size_t b = 0; b < g[a].size(); b++)
                if (!strcmp(g[a][b].name, e.module)) {
                    gi = a;
                    mi = (int)b;
                }
        if (gi < 0) return fail(m, BCU_ERR_ARG, "lora: tensors for unsupported modules, e.g. " + key);
        if (use[e.layer][gi][mi].e) return fail(m, BCU_ERR_ARG, "lora: " + key + " given twice");
        if (!e.a || !e.b) return fail(m, BCU_ERR_ARG, "lora: " + key + " needs lora_A and lora_B");
        const Member& mb = g[gi][mi];
        const int64_t r = e.a_shape[0];
        if (r <= 0 || e.a_shape[1] != mb.K || e.b_shape[0] != mb.O || e.b_shape[1] != r)
            return fail(m, BCU_ERR_ARG, "lora: " + key + ": A [" + std::to_string(e.a_shape[0]) + ", " +
                                            std::to_string(e.a_shape[1]) + "] B [" + std::to_string(e.b_shape[0]) +
                                            ", " + std::to_string(e.b_shape[1]) + "], linear is " +
                                            std::to_string(mb.O) + "x" + std::to_string(mb.K));
        if (rank && r != rank) return fail(m, BCU_ERR_ARG, "lora: mixed ranks are not supported");
        if (r > 256) return fail(m, BCU_ERR_ARG, "lora: rank above 256 is not supported");
        rank = (int)r;
        use[e.layer][gi][mi].e = &e;
    }
    if (n && HB > 1024) return fail(m, BCU_ERR_ARG, "lora: needs Hadamard blocks of at most 1024 inputs");
    if (wait_stream(m, 120.0) != BCU_OK) return BCU_ERR_TIMEOUT;
    drop_graphs(m);
    clear(m);
    if (n == 0) return BCU_OK;

    const int rp = (rank + 7) / 8 * 8, VPL = HB / 32;
    // host image of the device buffer: per group A then B, 256-byte aligned offsets
    std::vector<uint16_t> img;
    struct Placed {
        int li, gi;
        size_t a_off, b_off;
        int R, m1, m2;
    };
    std::vector<Placed> placed;
    size_t max_upart = 0;
    auto align = [&]() {
        while (img.size() % 128) img.push_back(0);
    };
    for (size_t li = 0; li < m->layers.size(); li++) {
        auto g = groups_of(m, m->layers[li]);
        for (int gi = 0; gi < 4; gi++) {
            const auto& us = use[li][gi];
            bool any = false;
            for (auto& u : us) any |= u.e != nullptr;
            if (!any) continue;
            const int K = g[gi][0].K, nblk = K / HB, nm = (int)us.size(), R = nm * rp;
            Placed pl{(int)li, gi, 0, 0, R, 0, 0};
            align();
            pl.a_off = img.size();
            img.resize(img.size() + (size_t)nblk * R * 32 * VPL, 0);
            uint16_t* A = img.data() + pl.a_off;
            for (int mi = 0; mi < nm; mi++) {
                const bcu_lora_linear* e = us[mi].e;
                if (!e) continue;
                for (int j = 0; j < rank; j++)
                    for (int k = 0; k < K; k++) {
                        const int b = k / HB, l = k % 32, el = (k % HB) / 32, q = mi * rp + j;
                        A[(((size_t)b * R + q) * 32 + l) * VPL + el] = f16(e->a[(size_t)j * K + k]);
                    }
            }
            align();
            pl.b_off = img.size();
            int Ototal = 0;
            for (auto& mb : g[gi]) Ototal += mb.O;
            img.resize(img.size() + (size_t)Ototal * rp, 0);
            uint16_t* B = img.data() + pl.b_off;
            int row0 = 0;
            int starts[3] = {Ototal, Ototal, Ototal};
            for (int mi = 0; mi < nm; mi++) {
                if (mi > 0 && mi < 3) starts[mi] = row0;
                const bcu_lora_linear* e = us[mi].e;
                const int O = g[gi][mi].O;
                if (e)
                    for (int o = 0; o < O; o++)
                        for (int j = 0; j < rank; j++)
                            B[(size_t)(row0 + o) * rp + j] = f16(e->b[(size_t)o * rank + j] * fold);
                row0 += O;
            }
            pl.m1 = starts[1];
            pl.m2 = starts[2];
            max_upart = std::max(max_upart, (size_t)VMAX * nblk * R);
            placed.push_back(pl);
        }
    }
    void* buf = nullptr;
    float* upart = nullptr;
    if (cudaMalloc(&buf, img.size() * 2) != cudaSuccess || cudaMalloc((void**)&upart, max_upart * 4) != cudaSuccess) {
        if (buf) cudaFree(buf);
        return fail(m, BCU_ERR_OOM, "lora: device allocation failed");
    }
    if (cudaMemcpyAsync(buf, img.data(), img.size() * 2, cudaMemcpyHostToDevice, m->st) != cudaSuccess ||
        cudaMemsetAsync(upart, 0, max_upart * 4, m->st) != cudaSuccess) {
        cudaFree(buf);
        cudaFree(upart);
        return fail(m, BCU_ERR_CUDA, "lora: upload failed");
    }
    bcu_status s = wait_stream(m, 120.0);
    if (s != BCU_OK) {
        cudaFree(buf);
        cudaFree(upart);
        return s;
    }
    m->lora_buf = buf;
    m->lora_upart = upart;
    m->lora_rank = rank;
    m->lora_linears = n;
    m->lora_bytes = img.size() * 2;
    for (const Placed& pl : placed) {
        LoraArgs& la = group_lin(m->layers[pl.li], pl.gi)->lora;
        la.a = (const uint16_t*)buf + pl.a_off;
        la.b = (const uint16_t*)buf + pl.b_off;
        la.upart = upart;
        la.R = pl.R;
        la.r = rp;
        la.m1 = pl.m1;
        la.m2 = pl.m2;
    }
    return BCU_OK;
}

bcu_status bcu_lora_info(const bcu_model* m, int32_t* linears, int32_t* rank) {
    if (!m || !linears || !rank) return BCU_ERR_ARG;
    *linears = m->lora_linears;
    *rank = m->lora_rank;
    return BCU_OK;
}

}  // extern "C"
