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
// gdn_chunk_prep_kernel (grid key heads x chunks, all chunks at once): L, X and P of every chunk for each value head of
// the key head (K K^T and Q K^T shared), from q, k and the gate inputs only; (I + A)^-1 from the inverses of its four
// 16 x 16 diagonal blocks (one warp each, no barrier) and six block steps for the blocks below them. gdn_chunk_scan_kernel (grid value heads x 4 blocks of 32 dv rows): the
// chunks in order, the state block in shared memory, each chunk five small products (S k and S q of the 64 rows,
// X R, P Delta, Delta^T K). Every product runs on the tensor cores as mma.sync tf32 with the three-product split
// (mma_tf32.cuh), fp32-accurate.
#include "common.cuh"
#include "kernels.h"
#include "mma_tf32.cuh"

namespace bcu {

constexpr int GC = 64;      // rows per chunk
constexpr int GCP = 132;    // padded row stride (floats) of staged q/k rows and of the state block
constexpr int GXP = 68;     // padded row stride of 64 x 64 matrices (16-byte rows, 4-bank shift per row)
constexpr int GVP = 40;     // padded row stride of 64 x 32 blocks (conflict-free k-major fragment reads)
constexpr int GS_ROWS = 32; // dv rows per scan CTA

struct GcPrepSmem {
    float k[GC][GCP];
    float q[GC][GCP];
    float a[GC][GXP];   // A (strictly lower)
    float m[GC][GXP];   // (I + A)^-1, built from its 16 x 16 blocks
    float tmp[GC][GXP]; // block products on the way
    float lg[GC], L[GC], beta[GC];
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
    // one CTA per (key head, chunk): K K^T and Q K^T once, then L, A, P and X for each value head of the key head
    const int hk = blockIdx.x, c = blockIdx.y, tid = threadIdx.x, lane = tid & 31;
    const int ratio = NV / NK, t0 = c * GC, nr = min(GC, T - t0);
    const size_t nch = gridDim.y;
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
    // K K^T and Q K^T on the tensor cores: warp w takes rows 16 (w / 2) .. + 15 and columns 32 (w % 2) .. + 31
    const int w = tid >> 5, g = lane >> 2, qd = lane & 3;
    const int mi = w >> 1, nb = 4 * (w & 1);
    float accg[4][4], accp[4][4];
#pragma unroll
    for (int n = 0; n < 4; n++)
#pragma unroll
        for (int e = 0; e < 4; e++) accg[n][e] = accp[n][e] = 0.0f;
    __syncthreads();  // the staged rows
#pragma unroll 2
    for (int ks = 0; ks < 16; ks++) {
        Tf32x2 ak[4], aq[4];
        frag_a_rows(&sm.k[0][0], GCP, 16 * mi, 8 * ks, ak);
        frag_a_rows(&sm.q[0][0], GCP, 16 * mi, 8 * ks, aq);
#pragma unroll
        for (int n = 0; n < 4; n++) {
            Tf32x2 bk[2];
            frag_b_nrows(&sm.k[0][0], GCP, 8 * ks, 8 * (nb + n), bk);  // (dk, i) = k_i[dk]
            mma_tf32x3(accg[n], ak, bk);
            mma_tf32x3(accp[n], aq, bk);
        }
    }
    for (int vv = 0; vv < ratio; vv++) {
        const int h = hk * ratio + vv;
        float* xs = ws + ((size_t)c * NV + h) * GC * GC;
        float* ps = ws + (nch * NV + (size_t)c * NV + h) * GC * GC;
        float* ls = ws + 2 * nch * NV * GC * GC + ((size_t)c * NV + h) * GC;
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
        __syncthreads();  // L
        // A_ti = beta_t exp(L_t - L_i) (k_i . k_t) for i < t; P_ti = exp(L_t - L_i) (q_t . k_i) for i <= t
#pragma unroll
        for (int n = 0; n < 4; n++)
#pragma unroll
            for (int hf = 0; hf < 2; hf++) {
                const int t = 16 * mi + g + 8 * hf, i = 8 * (nb + n) + 2 * qd;
                float av[2], pv[2];
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    const float dcy = i + e <= t ? expf(sm.L[t] - sm.L[i + e]) : 0.0f;
                    av[e] = i + e < t ? sm.beta[t] * (accg[n][2 * hf + e] * dcy) : 0.0f;
                    pv[e] = accp[n][2 * hf + e] * dcy;
                }
                sm.a[t][i] = av[0];
                sm.a[t][i + 1] = av[1];
                *(float2*)&ps[t * GC + i] = make_float2(pv[0], pv[1]);
            }
        __syncthreads();
        // (I + A)^-1 from its 16 x 16 blocks. Diagonal blocks N_b = (I + A_bb)^-1 by forward substitution, one per warp
        // 0..3, lane j < 16 holding column j in registers (no barrier inside): n_t = [t == j] - sum_{i<t} A_ti n_i.
        if (w < 4 && lane < 16) {
            const int b0 = 16 * w, j = lane;
            float nv[16];
#pragma unroll
            for (int t = 0; t < 16; t++) {
                float sacc = 0.0f;
#pragma unroll
                for (int i = 0; i < t; i++) sacc = fmaf(sm.a[b0 + t][b0 + i], nv[i], sacc);
                nv[t] = (t == j ? 1.0f : 0.0f) - sacc;
            }
#pragma unroll
            for (int t = 0; t < 16; t++) sm.m[b0 + t][b0 + j] = nv[t];
        }
        // blocks above the diagonal are zero
        for (int i = tid; i < GC * GC; i += 256) {
            const int r = i >> 6, cc = i & 63;
            if ((cc >> 4) > (r >> 4)) sm.m[r][cc] = 0.0f;
        }
        __syncthreads();
        // the blocks below the diagonal, M_bc = -N_b sum_{c<=k<b} A_bk M_kc, by distance b - c; thread (r, cc) of 16 x 16
        {
            const int r = tid >> 4, cc = tid & 15;
            // out(B) += sign * L(Lb) . R(Rb) for 16 x 16 blocks at block coordinates
            auto prod = [&](float (*L)[GXP], int lb, int lc, float (*R)[GXP], int rb, int rc) {
                float acc = 0.0f;
#pragma unroll
                for (int kk = 0; kk < 16; kk++) acc = fmaf(L[16 * lb + r][16 * lc + kk], R[16 * rb + kk][16 * rc + cc], acc);
                return acc;
            };
            // distance 1: T = A_{c+1,c} N_c, then M_{c+1,c} = -N_{c+1} T
            for (int c2 = 0; c2 < 3; c2++) sm.tmp[16 * (c2 + 1) + r][16 * c2 + cc] = prod(sm.a, c2 + 1, c2, sm.m, c2, c2);
            __syncthreads();
            for (int c2 = 0; c2 < 3; c2++)
                sm.m[16 * (c2 + 1) + r][16 * c2 + cc] = -prod(sm.m, c2 + 1, c2 + 1, sm.tmp, c2 + 1, c2);
            __syncthreads();
            // distance 2: U = A_{c+2,c} N_c + A_{c+2,c+1} M_{c+1,c}, then M_{c+2,c} = -N_{c+2} U
            for (int c2 = 0; c2 < 2; c2++)
                sm.tmp[16 * (c2 + 2) + r][16 * c2 + cc] =
                    prod(sm.a, c2 + 2, c2, sm.m, c2, c2) + prod(sm.a, c2 + 2, c2 + 1, sm.m, c2 + 1, c2);
            __syncthreads();
            for (int c2 = 0; c2 < 2; c2++)
                sm.m[16 * (c2 + 2) + r][16 * c2 + cc] = -prod(sm.m, c2 + 2, c2 + 2, sm.tmp, c2 + 2, c2);
            __syncthreads();
            // distance 3: U = A_30 N_0 + A_31 M_10 + A_32 M_20, then M_30 = -N_3 U
            sm.tmp[48 + r][cc] = (prod(sm.a, 3, 0, sm.m, 0, 0) + prod(sm.a, 3, 1, sm.m, 1, 0)) + prod(sm.a, 3, 2, sm.m, 2, 0);
            __syncthreads();
            sm.m[48 + r][cc] = -prod(sm.m, 3, 3, sm.tmp, 3, 0);
            __syncthreads();
        }
        // X = (I + A)^-1 diag(beta)
        for (int i = tid; i < GC * GC; i += 256) xs[i] = sm.m[i >> 6][i & 63] * sm.beta[i & 63];
        __syncthreads();  // the next value head reuses the shared arrays
    }
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

    // warp tiles (tensor cores, 3 x tf32): steps 1-3 rows 16 mi .. + 15 x dv 16 nh .. + 15 (two 8-wide n tiles);
    // step 4 dv rows 16 m4 .. + 15 x dk 32 n4 .. + 31 (four n tiles)
    const int lane = tid & 31, w = tid >> 5, g = lane >> 2, qd = lane & 3;
    const int mi = w >> 1, nh = 16 * (w & 1);
    const int m4 = w & 1, n4 = 32 * (w >> 1);
    for (int c = 0; c < nch; c++) {
        const int t0 = c * GC, nr = min(GC, T - t0);
        if (tid < GC) {
            const float LC = sm.L[GC - 1];
            sm.gam[tid] = expf(sm.L[tid]);
            sm.wl[tid] = expf(LC - sm.L[tid]);
        }
        const float gC = expf(sm.L[GC - 1]);
        __syncthreads();  // gam, wl; L may be refilled
        // ---- step 1: U = K S^T and Zq = Q S^T for the 64 rows; R = v - gamma U, Z = gamma Zq
        float z[2][4];
        {
            Acc3 u3[2], z3[2];
#pragma unroll
            for (int n = 0; n < 2; n++) {
                acc3_zero(u3[n]);
                acc3_zero(z3[n]);
            }
#pragma unroll 2
            for (int ks = 0; ks < 16; ks++) {
                Tf32x2 ak[4], aq[4];
                frag_a_rows(&sm.k[0][0], GCP, 16 * mi, 8 * ks, ak);
                frag_a_rows(&sm.q[0][0], GCP, 16 * mi, 8 * ks, aq);
#pragma unroll
                for (int n = 0; n < 2; n++) {
                    Tf32x2 bs[2];
                    frag_b_nrows(&sm.s[0][0], GCP, 8 * ks, nh + 8 * n, bs);  // (dk, dv) = S[dv][dk]
                    mma_tf32x3_acc(u3[n], ak, bs);
                    mma_tf32x3_acc(z3[n], aq, bs);
                }
            }
#pragma unroll
            for (int n = 0; n < 2; n++)
#pragma unroll
                for (int hf = 0; hf < 2; hf++) {
                    const int t = 16 * mi + g + 8 * hf, dv = nh + 8 * n + 2 * qd;
                    const float gm = sm.gam[t];
                    const float2 vv = *(const float2*)&sm.v[t][dv];
                    *(float2*)&sm.r[t][dv] =
                        make_float2(vv.x - gm * mma3_sum(u3[n], 2 * hf), vv.y - gm * mma3_sum(u3[n], 2 * hf + 1));
                    z[n][2 * hf] = gm * mma3_sum(z3[n], 2 * hf);
                    z[n][2 * hf + 1] = gm * mma3_sum(z3[n], 2 * hf + 1);
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
            Acc3 dl[2];
#pragma unroll
            for (int n = 0; n < 2; n++) acc3_zero(dl[n]);
#pragma unroll 2
            for (int ks = 0; ks < 8; ks++) {
                Tf32x2 ax[4];
                frag_a_rows(&sm.x[0][0], GXP, 16 * mi, 8 * ks, ax);
#pragma unroll
                for (int n = 0; n < 2; n++) {
                    Tf32x2 br[2];
                    frag_b_krows(&sm.r[0][0], GVP, 8 * ks, nh + 8 * n, br);
                    mma_tf32x3_acc(dl[n], ax, br);
                }
            }
#pragma unroll
            for (int n = 0; n < 2; n++)
#pragma unroll
                for (int hf = 0; hf < 2; hf++) {
                    const int t = 16 * mi + g + 8 * hf, dv = nh + 8 * n + 2 * qd;
                    *(float2*)&sm.d[t][dv] = make_float2(mma3_sum(dl[n], 2 * hf), mma3_sum(dl[n], 2 * hf + 1));
                }
        }
        __syncthreads();  // Delta; X is free
        if (c + 1 < nch) load_mat(c + 1, 0);
        // ---- step 3: outputs o = Z + P Delta
        {
            Acc3 o[2];
#pragma unroll
            for (int n = 0; n < 2; n++) acc3_zero(o[n]);
#pragma unroll 2
            for (int ks = 0; ks < 8; ks++) {
                Tf32x2 ap[4];
                frag_a_rows(&sm.p[0][0], GXP, 16 * mi, 8 * ks, ap);
#pragma unroll
                for (int n = 0; n < 2; n++) {
                    Tf32x2 bd[2];
                    frag_b_krows(&sm.d[0][0], GVP, 8 * ks, nh + 8 * n, bd);
                    mma_tf32x3_acc(o[n], ap, bd);
                }
            }
#pragma unroll
            for (int n = 0; n < 2; n++)
#pragma unroll
                for (int hf = 0; hf < 2; hf++) {
                    const int t = 16 * mi + g + 8 * hf, dv = nh + 8 * n + 2 * qd;
                    if (t < nr)
                        *(float2*)&y[((size_t)(t0 + t) * NV + h) * 128 + dvb + dv] =
                            make_float2(z[n][2 * hf] + mma3_sum(o[n], 2 * hf), z[n][2 * hf + 1] + mma3_sum(o[n], 2 * hf + 1));
                }
        }
        __syncthreads();  // P is free
        if (c + 1 < nch) load_mat(c + 1, 1);
        // ---- step 4: S' = gamma_63 S + (wl . Delta)^T K, accumulated onto gamma_63 S
        {
            Acc3 acc[4];  // hi.hi accumulated onto gamma_63 S
#pragma unroll
            for (int n = 0; n < 4; n++) {
                acc3_zero(acc[n]);
#pragma unroll
                for (int hf = 0; hf < 2; hf++) {
                    const float2 sv = *(const float2*)&sm.s[16 * m4 + g + 8 * hf][n4 + 8 * n + 2 * qd];
                    acc[n].c[0][2 * hf] = gC * sv.x;
                    acc[n].c[0][2 * hf + 1] = gC * sv.y;
                }
            }
#pragma unroll 2
            for (int ks = 0; ks < 8; ks++) {
                Tf32x2 ad[4];
                frag_a_cols(&sm.d[0][0], GVP, 16 * m4, 8 * ks, sm.wl, ad);  // (dv, i) = wl_i Delta[i][dv]
#pragma unroll
                for (int n = 0; n < 4; n++) {
                    Tf32x2 bk[2];
                    frag_b_krows(&sm.k[0][0], GCP, 8 * ks, n4 + 8 * n, bk);  // (i, dk) = k_i[dk]
                    mma_tf32x3_acc(acc[n], ad, bk);
                }
            }
            // each warp reads and writes only its own tile of S here (step 1's reads ended at its barrier)
#pragma unroll
            for (int n = 0; n < 4; n++)
#pragma unroll
                for (int hf = 0; hf < 2; hf++)
                    *(float2*)&sm.s[16 * m4 + g + 8 * hf][n4 + 8 * n + 2 * qd] =
                        make_float2(mma3_sum(acc[n], 2 * hf), mma3_sum(acc[n], 2 * hf + 1));
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
    gdn_chunk_prep_kernel<<<dim3(NK, nch), 256, sizeof(GcPrepSmem), st>>>(q, k, a_in, b_in, a_log, dt_bias, T, NK,
                                                                          NV, ws);
    gdn_chunk_scan_kernel<<<dim3(NV, 128 / GS_ROWS), 256, sizeof(GcScanSmem), st>>>(q, k, v, ws, state, y, T, NK, NV);
}

}  // namespace bcu
