// gdn_chunk.cu — the gated delta rule of a prefill chunk (gdn_recurrent, kernels.metal:566-622, over the chunk's rows
// in order, as Model::prefill runs it per chunk, runtime/mod.rs:341-386) in chunks of GC = 64 rows: two kernels
// instead of a sequential step per row.
//
// Per value head, with the state S (dv x dk) at the start of a chunk, rows t = 0..63, decays g_t, L_t = sum_{i<=t}
// log g_i and gamma_t = exp(L_t), the step S_t = g_t S_{t-1} + delta_t k_t^T with delta_t = beta_t (v_t - g_t S_{t-1}
// k_t) unrolls to
//   delta_t = beta_t (v_t - gamma_t S k_t - sum_{i<t} exp(L_t - L_i) (k_i . k_t) delta_i)
// i.e. (I + A) Delta = diag(beta) R with A_ti = beta_t exp(L_t - L_i) (k_i . k_t) (i < t) and R_t = v_t - gamma_t S k_t,
// so Delta = X R with X = (I + A)^-1 diag(beta) (lower triangular); the outputs are
//   o_t = gamma_t S q_t + sum_{i<=t} exp(L_t - L_i) (k_i . q_t) delta_i = Z_t + (P Delta)_t
// and the state after the chunk is S' = gamma_63 S + sum_i exp(L_63 - L_i) delta_i k_i^T. The same quantities as
// the per-row recurrence, re-associated; sums run in fp32 in a fixed order, so a row's result does not depend on
// anything but the chunk it lies in.
//
// gdn_chunk_prep_kernel (grid value heads x chunks, all chunks at once): L, X and P of every chunk, from q, k and the
// gate inputs only. gdn_chunk_scan_kernel (grid value heads x 4 blocks of 32 dv rows): the chunks in order, the state
// block in shared memory, each chunk five small products (S k and S q of the 64 rows, X R, P Delta, Delta^T K).
#include "common.cuh"
#include "kernels.h"

namespace bcu {

constexpr int GC = 64;      // rows per chunk
constexpr int GCP = 132;    // padded row stride (floats) of staged q/k rows and of the state block
constexpr int GXP = 68;     // padded row stride of 64 x 64 matrices (16-byte rows, 4-bank shift per row)
constexpr int GVP = 36;     // padded row stride of 64 x 32 blocks
constexpr int GS_ROWS = 32; // dv rows per scan CTA

struct GcPrepSmem {
    float k[GC][GCP];
    float q[GC][GCP];
    float a[GC][GXP];   // A (strictly lower)
    float x[GC][GXP];   // X = (I + A)^-1 diag(beta)
    float lg[GC], L[GC], beta[GC];
    float red[4][GC];
};

struct GcScanSmem {
    float k[GC][GCP];
    float q[GC][GCP];
    float s[GS_ROWS][GCP];  // the state block: dv row r, dk entries
    float v[GC][GVP];       // v rows of the block
    float x[GC][GXP];
    float p[GC][GXP];
    float r[GC][GVP];       // R, then reused
    float d[GC][GVP];       // Delta
    float L[GC], gam[GC], wl[GC];
};

size_t gdn_chunk_workspace_bytes(int T, int NV) {
    const size_t nch = (size_t)(T + GC - 1) / GC;
    return nch * NV * (2 * GC * GC + GC) * sizeof(float);
}

// ---------------------------------------------------------------------------------------------------------- prep
__global__ void __launch_bounds__(256) gdn_chunk_prep_kernel(const float* q, const float* k, const float* a_in,
                                                             const float* b_in, const float* a_log,
                                                             const float* dt_bias, int T, int NK, int NV, float* ws) {
    extern __shared__ __align__(16) uint8_t gsm[];
    GcPrepSmem& sm = *(GcPrepSmem*)gsm;
    const int h = blockIdx.x, c = blockIdx.y, tid = threadIdx.x, lane = tid & 31;
    const int hk = h / (NV / NK), t0 = c * GC, nr = min(GC, T - t0);
    const size_t nch = gridDim.y;
    float* xs = ws + ((size_t)c * NV + h) * GC * GC;
    float* ps = ws + (nch * NV + (size_t)c * NV + h) * GC * GC;
    float* ls = ws + 2 * nch * NV * GC * GC + ((size_t)c * NV + h) * GC;
    for (int i = tid; i < GC * 32; i += 256) {  // q and k rows (zero past the last row)
        const int r = i >> 5, j = (i & 31) * 4;
        float4 kv = make_float4(0.0f, 0.0f, 0.0f, 0.0f), qv = kv;
        if (r < nr) {
            const size_t o = ((size_t)(t0 + r) * NK + hk) * 128 + j;
            kv = *(const float4*)(k + o);
            qv = *(const float4*)(q + o);
        }
        *(float4*)&sm.k[r][j] = kv;
        *(float4*)&sm.q[r][j] = qv;
    }
    if (tid < GC) {  // gates (gdn_gates, kernels.metal:556-561): log decay and beta; rows past the last: 0, 0
        float lgv = 0.0f, bt = 0.0f;
        if (tid < nr) {
            const float x = a_in[(size_t)(t0 + tid) * NV + h] + dt_bias[h];
            const float sp = fmaxf(x, 0.0f) + logf(1.0f + expf(-fabsf(x)));
            lgv = -expf(a_log[h]) * sp;
            bt = 1.0f / (1.0f + expf(-b_in[(size_t)(t0 + tid) * NV + h]));
        }
        sm.lg[tid] = lgv;
        sm.beta[tid] = bt;
    }
    __syncthreads();
    if (tid < 32) {  // inclusive scan of the log decays, two rows per lane
        const float a0 = sm.lg[2 * lane], a1 = sm.lg[2 * lane + 1];
        float s = a0 + a1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float u = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += u;
        }
        float ex = __shfl_up_sync(0xffffffffu, s, 1);
        if (lane == 0) ex = 0.0f;
        const float l0 = ex + a0;
        sm.L[2 * lane] = l0;
        sm.L[2 * lane + 1] = l0 + a1;
        ls[2 * lane] = l0;
        ls[2 * lane + 1] = l0 + a1;
    }
    // K K^T and Q K^T: thread (ti, tj) takes rows t = ti + 16 a and columns i = tj + 16 b (a, b < 4)
    const int ti = tid >> 4, tj = tid & 15;
    float g[4][4], p[4][4];
#pragma unroll
    for (int a = 0; a < 4; a++)
#pragma unroll
        for (int b = 0; b < 4; b++) g[a][b] = p[a][b] = 0.0f;
    for (int d = 0; d < 128; d += 4) {
        float4 kr[4], qr[4], kc[4];
#pragma unroll
        for (int a = 0; a < 4; a++) {
            kr[a] = *(const float4*)&sm.k[ti + 16 * a][d];
            qr[a] = *(const float4*)&sm.q[ti + 16 * a][d];
            kc[a] = *(const float4*)&sm.k[tj + 16 * a][d];
        }
#pragma unroll
        for (int a = 0; a < 4; a++)
#pragma unroll
            for (int b = 0; b < 4; b++) {
                g[a][b] = fmaf(kr[a].x, kc[b].x, g[a][b]);
                g[a][b] = fmaf(kr[a].y, kc[b].y, g[a][b]);
                g[a][b] = fmaf(kr[a].z, kc[b].z, g[a][b]);
                g[a][b] = fmaf(kr[a].w, kc[b].w, g[a][b]);
                p[a][b] = fmaf(qr[a].x, kc[b].x, p[a][b]);
                p[a][b] = fmaf(qr[a].y, kc[b].y, p[a][b]);
                p[a][b] = fmaf(qr[a].z, kc[b].z, p[a][b]);
                p[a][b] = fmaf(qr[a].w, kc[b].w, p[a][b]);
            }
    }
    __syncthreads();  // L
#pragma unroll
    for (int a = 0; a < 4; a++)
#pragma unroll
        for (int b = 0; b < 4; b++) {
            const int t = ti + 16 * a, i = tj + 16 * b;
            const float e = i <= t ? expf(sm.L[t] - sm.L[i]) : 0.0f;
            sm.a[t][i] = i < t ? sm.beta[t] * (g[a][b] * e) : 0.0f;
            ps[t * GC + i] = p[a][b] * e;
        }
    __syncthreads();
    // X = (I + A)^-1 diag(beta) by forward substitution: X_t = beta_t e_t - sum_{i<t} A_ti X_i; thread (part, j)
    // sums i = part, part + 4, ... for column j, the four parts added in order
    {
        const int j = tid & 63, part = tid >> 6;
        for (int t = 0; t < GC; t++) {
            float s = 0.0f;
            for (int i = part; i < t; i += 4) s = fmaf(sm.a[t][i], sm.x[i][j], s);
            sm.red[part][j] = s;
            __syncthreads();
            if (part == 0)
                sm.x[t][j] = (t == j ? sm.beta[t] : 0.0f) - ((sm.red[0][j] + sm.red[1][j]) + (sm.red[2][j] + sm.red[3][j]));
            __syncthreads();
        }
    }
    for (int i = tid; i < GC * GC; i += 256) xs[i] = sm.x[i >> 6][i & 63];
}

// ---------------------------------------------------------------------------------------------------------- scan
__global__ void __launch_bounds__(256, 1) gdn_chunk_scan_kernel(const float* q, const float* k, const float* v,
                                                                const float* ws, float* state, float* y, int T,
                                                                int NK, int NV) {
    extern __shared__ __align__(16) uint8_t gsm[];
    GcScanSmem& sm = *(GcScanSmem*)gsm;
    const int h = blockIdx.x, tid = threadIdx.x;
    const int hk = h / (NV / NK), dvb = blockIdx.y * GS_ROWS;
    const int nch = (T + GC - 1) / GC;
    float* S = state + ((size_t)h * 128 + dvb) * 128;
    // the state block into shared memory
    for (int i = tid; i < GS_ROWS * 32; i += 256) {
        const int r = i >> 5, j = (i & 31) * 4;
        *(float4*)&sm.s[r][j] = *(const float4*)(S + (size_t)r * 128 + j);
    }
    const float4 zero = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    // chunk c's rows into shared memory: q, k (key head hk), v (this block's 32 dv), X, P, L
    auto load_qk = [&](int cc, bool isk) {
        const int t0 = cc * GC, nr = min(GC, T - t0);
        const float* src = isk ? k : q;
        for (int i = tid; i < GC * 32; i += 256) {
            const int r = i >> 5, j = (i & 31) * 4;
            float* dst = isk ? &sm.k[r][j] : &sm.q[r][j];
            if (r < nr) cp_async16(dst, src + ((size_t)(t0 + r) * NK + hk) * 128 + j);
            else *(float4*)dst = zero;
        }
    };
    auto load_v = [&](int cc) {
        const int t0 = cc * GC, nr = min(GC, T - t0);
        for (int i = tid; i < GC * 8; i += 256) {
            const int r = i >> 3, j = (i & 7) * 4;
            if (r < nr) cp_async16(&sm.v[r][j], v + ((size_t)(t0 + r) * NV + h) * 128 + dvb + j);
            else *(float4*)&sm.v[r][j] = zero;
        }
    };
    auto load_mat = [&](int cc, int which) {  // which 0: X, 1: P
        const float* src = ws + ((size_t)which * nch * NV + (size_t)cc * NV + h) * GC * GC;
        float (*dst)[GXP] = which ? sm.p : sm.x;
        for (int i = tid; i < GC * 16; i += 256) {
            const int r = i >> 4, j = (i & 15) * 4;
            cp_async16(&dst[r][j], src + r * GC + j);
        }
    };
    auto load_l = [&](int cc) {
        if (tid < 16) cp_async16(&sm.L[4 * tid], ws + 2 * (size_t)nch * NV * GC * GC + ((size_t)cc * NV + h) * GC + 4 * tid);
    };
    load_qk(0, false);
    load_qk(0, true);
    load_v(0);
    load_mat(0, 0);
    load_mat(0, 1);
    load_l(0);
    cp_async_wait_all();
    __syncthreads();

    // thread tiles: rows t = tg + 16 a (a < 4) x dv = dg + 16 b (b < 2) for steps 1-3; dv row sr, dk = 4 sg + 32 j
    // (j < 4) for the state update
    const int tg = tid >> 4, dg = tid & 15;
    const int sr = tid >> 3, sg = tid & 7;
    for (int c = 0; c < nch; c++) {
        const int t0 = c * GC, nr = min(GC, T - t0);
        if (tid < GC) {
            const float LC = sm.L[GC - 1];
            sm.gam[tid] = expf(sm.L[tid]);
            sm.wl[tid] = expf(LC - sm.L[tid]);
        }
        const float gC = expf(sm.L[GC - 1]);
        __syncthreads();  // gam, wl; L may be refilled
        // ---- step 1: u = S k_t and z = S q_t for the 64 rows; R = v - gamma u, Z = gamma z
        float z[4][2];
        {
            float u[4][2];
#pragma unroll
            for (int a = 0; a < 4; a++)
#pragma unroll
                for (int b = 0; b < 2; b++) u[a][b] = z[a][b] = 0.0f;
            for (int d = 0; d < 128; d += 4) {
                float4 kr[4], qr[4], sv[2];
#pragma unroll
                for (int a = 0; a < 4; a++) {
                    kr[a] = *(const float4*)&sm.k[tg + 16 * a][d];
                    qr[a] = *(const float4*)&sm.q[tg + 16 * a][d];
                }
#pragma unroll
                for (int b = 0; b < 2; b++) sv[b] = *(const float4*)&sm.s[dg + 16 * b][d];
#pragma unroll
                for (int a = 0; a < 4; a++)
#pragma unroll
                    for (int b = 0; b < 2; b++) {
                        u[a][b] = fmaf(kr[a].x, sv[b].x, u[a][b]);
                        u[a][b] = fmaf(kr[a].y, sv[b].y, u[a][b]);
                        u[a][b] = fmaf(kr[a].z, sv[b].z, u[a][b]);
                        u[a][b] = fmaf(kr[a].w, sv[b].w, u[a][b]);
                        z[a][b] = fmaf(qr[a].x, sv[b].x, z[a][b]);
                        z[a][b] = fmaf(qr[a].y, sv[b].y, z[a][b]);
                        z[a][b] = fmaf(qr[a].z, sv[b].z, z[a][b]);
                        z[a][b] = fmaf(qr[a].w, sv[b].w, z[a][b]);
                    }
            }
#pragma unroll
            for (int a = 0; a < 4; a++) {
                const int t = tg + 16 * a;
                const float gm = sm.gam[t];
#pragma unroll
                for (int b = 0; b < 2; b++) {
                    const int dv = dg + 16 * b;
                    sm.r[t][dv] = sm.v[t][dv] - gm * u[a][b];
                    z[a][b] *= gm;
                }
            }
        }
        __syncthreads();  // R; q, v and L are free
        if (c + 1 < nch) {
            load_qk(c + 1, false);
            load_v(c + 1);
            load_l(c + 1);
        }
        // ---- step 2: Delta = X R (X lower triangular: columns past the row are zero)
        {
            float dl[4][2];
#pragma unroll
            for (int a = 0; a < 4; a++) dl[a][0] = dl[a][1] = 0.0f;
            for (int i = 0; i < GC; i += 4) {
                float4 xr[4];
#pragma unroll
                for (int a = 0; a < 4; a++) xr[a] = *(const float4*)&sm.x[tg + 16 * a][i];
                float rv[4][2];
#pragma unroll
                for (int e = 0; e < 4; e++)
#pragma unroll
                    for (int b = 0; b < 2; b++) rv[e][b] = sm.r[i + e][dg + 16 * b];
#pragma unroll
                for (int a = 0; a < 4; a++)
#pragma unroll
                    for (int b = 0; b < 2; b++) {
                        dl[a][b] = fmaf(xr[a].x, rv[0][b], dl[a][b]);
                        dl[a][b] = fmaf(xr[a].y, rv[1][b], dl[a][b]);
                        dl[a][b] = fmaf(xr[a].z, rv[2][b], dl[a][b]);
                        dl[a][b] = fmaf(xr[a].w, rv[3][b], dl[a][b]);
                    }
            }
#pragma unroll
            for (int a = 0; a < 4; a++)
#pragma unroll
                for (int b = 0; b < 2; b++) sm.d[tg + 16 * a][dg + 16 * b] = dl[a][b];
        }
        __syncthreads();  // Delta; X is free
        if (c + 1 < nch) load_mat(c + 1, 0);
        // ---- step 3: outputs o = Z + P Delta
        {
            float o[4][2];
#pragma unroll
            for (int a = 0; a < 4; a++) o[a][0] = o[a][1] = 0.0f;
            for (int i = 0; i < GC; i += 4) {
                float4 pr[4];
#pragma unroll
                for (int a = 0; a < 4; a++) pr[a] = *(const float4*)&sm.p[tg + 16 * a][i];
                float dv4[4][2];
#pragma unroll
                for (int e = 0; e < 4; e++)
#pragma unroll
                    for (int b = 0; b < 2; b++) dv4[e][b] = sm.d[i + e][dg + 16 * b];
#pragma unroll
                for (int a = 0; a < 4; a++)
#pragma unroll
                    for (int b = 0; b < 2; b++) {
                        o[a][b] = fmaf(pr[a].x, dv4[0][b], o[a][b]);
                        o[a][b] = fmaf(pr[a].y, dv4[1][b], o[a][b]);
                        o[a][b] = fmaf(pr[a].z, dv4[2][b], o[a][b]);
                        o[a][b] = fmaf(pr[a].w, dv4[3][b], o[a][b]);
                    }
            }
#pragma unroll
            for (int a = 0; a < 4; a++) {
                const int t = tg + 16 * a;
                if (t < nr)
#pragma unroll
                    for (int b = 0; b < 2; b++)
                        y[((size_t)(t0 + t) * NV + h) * 128 + dvb + dg + 16 * b] = z[a][b] + o[a][b];
            }
        }
        __syncthreads();  // P is free
        if (c + 1 < nch) load_mat(c + 1, 1);
        // ---- step 4: S' = gamma_63 S + sum_i exp(L_63 - L_i) Delta_i k_i^T (this thread: row sr, dk 4 sg + 32 j)
        {
            float acc[4][4];
#pragma unroll
            for (int j = 0; j < 4; j++) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
            for (int i = 0; i < GC; i++) {
                const float dw = sm.wl[i] * sm.d[i][sr];
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const float4 kk = *(const float4*)&sm.k[i][4 * sg + 32 * j];
                    acc[j][0] = fmaf(dw, kk.x, acc[j][0]);
                    acc[j][1] = fmaf(dw, kk.y, acc[j][1]);
                    acc[j][2] = fmaf(dw, kk.z, acc[j][2]);
                    acc[j][3] = fmaf(dw, kk.w, acc[j][3]);
                }
            }
#pragma unroll
            for (int j = 0; j < 4; j++) {
                float4* sp = (float4*)&sm.s[sr][4 * sg + 32 * j];
                const float4 o = *sp;
                *sp = make_float4(fmaf(gC, o.x, acc[j][0]), fmaf(gC, o.y, acc[j][1]), fmaf(gC, o.z, acc[j][2]),
                                  fmaf(gC, o.w, acc[j][3]));
            }
        }
        __syncthreads();  // k is free
        if (c + 1 < nch) load_qk(c + 1, true);
        cp_async_wait_all();
        __syncthreads();
    }
    for (int i = tid; i < GS_ROWS * 32; i += 256) {
        const int r = i >> 5, j = (i & 31) * 4;
        *(float4*)(S + (size_t)r * 128 + j) = *(const float4*)&sm.s[r][j];
    }
}

void launch_gdn_chunked(const float* q, const float* k, const float* v, const float* a_in, const float* b_in,
                        const float* a_log, const float* dt_bias, float* state, float* y, int T, int NK, int NV,
                        float* ws, cudaStream_t st) {
    const int nch = (T + GC - 1) / GC;
    raise_smem_limit((const void*)gdn_chunk_prep_kernel, (int)sizeof(GcPrepSmem));
    raise_smem_limit((const void*)gdn_chunk_scan_kernel, (int)sizeof(GcScanSmem));
    gdn_chunk_prep_kernel<<<dim3(NV, nch), 256, sizeof(GcPrepSmem), st>>>(q, k, a_in, b_in, a_log, dt_bias, T, NK,
                                                                          NV, ws);
    gdn_chunk_scan_kernel<<<dim3(NV, 128 / GS_ROWS), 256, sizeof(GcScanSmem), st>>>(q, k, v, ws, state, y, T, NK, NV);
}

}  // namespace bcu
