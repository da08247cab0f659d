// ref_runtime.cpp — the threadgroup scheduler behind ref_runtime.h and the collectives of metal_stdlib.
// TEST INFRASTRUCTURE ONLY.
#include "ref_runtime.h"

#include <omp.h>
#include <ucontext.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include <metal_stdlib>

namespace {

enum { RUN, SIMD, BAR, DONE };
enum { OP_SUM, OP_MAX, OP_XOR, OP_DOWNF, OP_DOWNI, OP_MMA };

struct Lane {
    ucontext_t ctx;
    int st, op;
    uint32_t v, arg, res;
    float ma[2], mb[2], mc[2], md[2];
};

struct Group {
    std::vector<Lane> lanes;
    std::vector<char*> stacks;
    ucontext_t sched;
    int n = 0, cur = 0;
    refrt::Body body = nullptr;
    void* user = nullptr;
    refrt::Ctx base;
    uint32_t tpg[3];
};

thread_local Group* G = nullptr;
constexpr size_t STACK_BYTES = 128 * 1024;

[[noreturn]] void die(const char* what) {
    std::fprintf(stderr, "ref_runtime: %s\n", what);
    std::abort();
}

void fiber_entry() {
    Group* g = G;
    const int tid = g->cur;
    refrt::Ctx c = g->base;
    c.tid = tid;
    c.tp[0] = tid % g->tpg[0];
    c.tp[1] = (tid / g->tpg[0]) % g->tpg[1];
    c.tp[2] = tid / (g->tpg[0] * g->tpg[1]);
    c.sid = tid / 32;
    c.lane = tid % 32;
    for (int d = 0; d < 3; d++) c.gid[d] = c.tg[d] * g->tpg[d] + c.tp[d];
    g->body(g->user, c);
    g->lanes[tid].st = DONE;  // returns to g->sched through uc_link
}

inline Lane& me() { return G->lanes[G->cur]; }

inline void yield(int st) {
    Lane& L = me();
    L.st = st;
    swapcontext(&L.ctx, &G->sched);
}

inline uint32_t fbits(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    return u;
}
inline float bitsf(uint32_t u) {
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// Resolves the collective that SIMD group `s` is waiting at, if every lane of it has arrived somewhere. Returns
// whether lanes were released.
bool resolve_simd(Group& g, int s) {
    const int l0 = s * 32, l1 = l0 + 32 < g.n ? l0 + 32 : g.n;
    bool part[32] = {false};
    int op = -1;
    for (int l = l0; l < l1; l++) {
        const Lane& L = g.lanes[l];
        if (L.st == RUN) return false;
        if (L.st == SIMD) {
            if (op >= 0 && L.op != op) die("lanes of one SIMD group wait at different collectives");
            op = L.op;
            part[l - l0] = true;
        }
    }
    if (op < 0) return false;
    uint32_t v[32];
    for (int i = 0; i < 32; i++) v[i] = (l0 + i < l1 && part[i]) ? g.lanes[l0 + i].v : 0u;
    auto res = [&](int i, uint32_t r) { g.lanes[l0 + i].res = r; };
    switch (op) {
        case OP_SUM: {  // xor butterfly, inactive lanes contribute 0
            float a[32], b[32];
            for (int i = 0; i < 32; i++) a[i] = bitsf(v[i]);
            for (int m = 16; m >= 1; m >>= 1) {
                for (int i = 0; i < 32; i++) b[i] = a[i] + a[i ^ m];
                std::memcpy(a, b, sizeof a);
            }
            for (int i = 0; i < 32; i++) res(i, fbits(a[i]));
            break;
        }
        case OP_MAX: {
            float m = -INFINITY;
            for (int i = 0; i < 32; i++)
                if (part[i]) m = metal::max(m, bitsf(v[i]));
            for (int i = 0; i < 32; i++) res(i, fbits(m));
            break;
        }
        case OP_XOR:
            for (int i = 0; i < 32; i++)
                if (part[i]) {
                    int j = i ^ (int)(g.lanes[l0 + i].arg & 31u);
                    res(i, part[j] ? v[j] : v[i]);
                }
            break;
        case OP_DOWNF:
        case OP_DOWNI:
            for (int i = 0; i < 32; i++)
                if (part[i]) {
                    int j = i + (int)g.lanes[l0 + i].arg;
                    res(i, (j < 32 && part[j]) ? v[j] : v[i]);
                }
            break;
        case OP_MMA: {
            if (l1 - l0 != 32) die("simdgroup matrix product in a partial SIMD group");
            for (int i = 0; i < 32; i++)
                if (!part[i]) die("simdgroup matrix product with inactive lanes");
            float A[8][8], B[8][8], C[8][8];
            for (int i = 0; i < 32; i++) {
                const Lane& L = g.lanes[l0 + i];
                uint32_t r = metal::sg_row(i), c = metal::sg_col(i);
                for (int e = 0; e < 2; e++) {
                    A[r][c + e] = L.ma[e];
                    B[r][c + e] = L.mb[e];
                    C[r][c + e] = L.mc[e];
                }
            }
            for (int i = 0; i < 32; i++) {
                Lane& L = g.lanes[l0 + i];
                uint32_t r = metal::sg_row(i), c = metal::sg_col(i);
                for (int e = 0; e < 2; e++) {
                    float acc = C[r][c + e];
                    for (int k = 0; k < 8; k++) acc = acc + A[r][k] * B[k][c + e];
                    L.md[e] = acc;
                }
            }
            break;
        }
    }
    for (int l = l0; l < l1; l++)
        if (part[l - l0]) g.lanes[l].st = RUN;
    return true;
}

void run_group(Group& g) {
    for (int t = 0; t < g.n; t++) {
        Lane& L = g.lanes[t];
        getcontext(&L.ctx);
        L.ctx.uc_stack.ss_sp = g.stacks[t];
        L.ctx.uc_stack.ss_size = STACK_BYTES;
        L.ctx.uc_link = &g.sched;
        makecontext(&L.ctx, fiber_entry, 0);
        L.st = RUN;
    }
    for (;;) {
        for (int t = 0; t < g.n; t++) {
            if (g.lanes[t].st != RUN) continue;
            g.cur = t;
            swapcontext(&g.sched, &g.lanes[t].ctx);
        }
        bool progress = false, live = false, all_bar = true;
        for (int s = 0; s * 32 < g.n; s++) progress |= resolve_simd(g, s);
        if (progress) continue;
        for (int t = 0; t < g.n; t++) {
            int st = g.lanes[t].st;
            if (st == DONE) continue;
            live = true;
            if (st != BAR) all_bar = false;
        }
        if (!live) return;
        if (!all_bar) die("threadgroup cannot make progress");
        for (int t = 0; t < g.n; t++)
            if (g.lanes[t].st == BAR) g.lanes[t].st = RUN;
    }
}

}  // namespace

namespace refrt {

void dispatch(const uint32_t grid[3], const uint32_t tpg[3], Body body, void* user) {
    const int n = (int)(tpg[0] * tpg[1] * tpg[2]);
    if (n < 1 || n > 1024) die("threads per threadgroup out of range");
    const long total = (long)grid[0] * grid[1] * grid[2];
#pragma omp parallel
    {
        static thread_local Group group;
        Group& g = group;
        while ((int)g.stacks.size() < n) g.stacks.push_back((char*)std::malloc(STACK_BYTES));
        if ((int)g.lanes.size() < n) g.lanes.resize(n);
        g.n = n;
        g.body = body;
        g.user = user;
        for (int d = 0; d < 3; d++) {
            g.tpg[d] = tpg[d];
            g.base.ng[d] = grid[d];
        }
        G = &g;
#pragma omp for schedule(dynamic, 1)
        for (long i = 0; i < total; i++) {
            g.base.tg[0] = (uint32_t)(i % grid[0]);
            g.base.tg[1] = (uint32_t)((i / grid[0]) % grid[1]);
            g.base.tg[2] = (uint32_t)(i / ((long)grid[0] * grid[1]));
            run_group(g);
        }
        G = nullptr;
    }
}

}  // namespace refrt

namespace metal {

float simd_sum(float v) {
    Lane& L = me();
    L.op = OP_SUM;
    L.v = fbits(v);
    yield(SIMD);
    return bitsf(me().res);
}

float simd_max(float v) {
    Lane& L = me();
    L.op = OP_MAX;
    L.v = fbits(v);
    yield(SIMD);
    return bitsf(me().res);
}

float simd_shuffle_xor(float v, uint mask) {
    Lane& L = me();
    L.op = OP_XOR;
    L.v = fbits(v);
    L.arg = mask;
    yield(SIMD);
    return bitsf(me().res);
}

float simd_shuffle_down(float v, uint delta) {
    Lane& L = me();
    L.op = OP_DOWNF;
    L.v = fbits(v);
    L.arg = delta;
    yield(SIMD);
    return bitsf(me().res);
}

int simd_shuffle_down(int v, uint delta) {
    Lane& L = me();
    L.op = OP_DOWNI;
    L.v = (uint32_t)v;
    L.arg = delta;
    yield(SIMD);
    return (int)me().res;
}

void threadgroup_barrier(mem_flags) { yield(BAR); }

uint simd_lane() { return (uint)(G->cur % 32); }

void simdgroup_mma(const float a[2], const float b[2], const float c[2], float d[2]) {
    Lane& L = me();
    L.op = OP_MMA;
    for (int e = 0; e < 2; e++) {
        L.ma[e] = a[e];
        L.mb[e] = b[e];
        L.mc[e] = c[e];
    }
    yield(SIMD);
    d[0] = me().md[0];
    d[1] = me().md[1];
}

}  // namespace metal
