// gdn.cu — GatedDeltaNet layer kernels for the verify pass (gdn_ab, gdn_conv, conv_state, gdn_gates, gdn_recurrent:
// kernels.metal:504-622) with rollback by deferred commit instead of the reference's candidate-state copies and
// re-runs (encode_accept, model.rs:1025-1069).
//
// Deferred commit: a pass never writes its candidate recurrent state. It saves its own conv inputs (raw qkv rows), conv
// outputs and gate inputs in the pending buffer of its parity; the accept step records how many rows n were accepted.
// The next pass first replays those n rows on the committed state (conv shift + n gated-delta steps, in registers),
// writes the committed state once, and only then runs its own rows. State traffic per pass is one read and one write of
// the fp32 state, whatever the accept length, and rollback costs nothing.
#include "common.cuh"
#include "kernels.h"

namespace bcu {

constexpr float EPS_G = 1e-6f;

// gdn_ab (kernels.metal:504-510, gdn_ab_row :265-273): dense fp32 a/b gate rows. One CTA per row (4 warps split K,
// partials summed in warp order), all T tokens at once.
__global__ void __launch_bounds__(128) gdn_ab_kernel(GdnArgs a) {
    __shared__ float part[4][VMAX];
    const int row = blockIdx.x, lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int d = a.d, NV = a.NV, T = a.T;
    const float* wr = row < NV ? a.wa + (size_t)row * d : a.wb + (size_t)(row - NV) * d;
    const int q = d / 4;
    // weights before the dependency wait
    float4 wv[4];
    int nv = 0;
    for (int i = w * q + lane * 4; i < (w + 1) * q && nv < 4; i += 128) wv[nv++] = *(const float4*)(wr + i);
    pdl_trigger();
    pdl_wait();
    const int par = a.ctl->parity;
    float acc[VMAX];
#pragma unroll
    for (int t = 0; t < VMAX; t++) acc[t] = 0.0f;
    int j = 0;
    for (int i = w * q + lane * 4; i < (w + 1) * q; i += 128, j++) {
        float4 ww = j < 4 ? wv[j] : *(const float4*)(wr + i);
#pragma unroll
        for (int t = 0; t < VMAX; t++)
            if (t < T) {
                float4 x = *(const float4*)(a.xn + (size_t)t * d + i);
                acc[t] += ww.x * x.x + ww.y * x.y + ww.z * x.z + ww.w * x.w;
            }
    }
#pragma unroll
    for (int t = 0; t < VMAX; t++)
        if (t < T) {
            float v = warp_sum(acc[t]);
            if (lane == 0) part[w][t] = v;
        }
    __syncthreads();
    if (threadIdx.x < T) {
        int t = threadIdx.x;
        float v = part[0][t] + part[1][t] + part[2][t] + part[3][t];
        a.pend_ab[((size_t)par * VMAX + t) * 2 * NV + row] = v;
    }
}

void launch_gdn_ab(const GdnArgs& a, cudaStream_t st) {
    GdnArgs aa = a;
    void* args[] = {&aa};
    launch_pdl((const void*)gdn_ab_kernel, dim3(2 * a.NV), dim3(128), 0, st, args);
}

// gdn_conv (kernels.metal:515-541) + conv_state (:544-553). CTA = one 128-channel head group, thread = channel.
// First commits the previous pass: the committed conv state becomes rows n..n+2 of [state(3); qkv_prev(n)]. Then the
// causal width-4 conv of this pass's rows over [state; qkv], SiLU, and for q/k groups the per-head RMS norm scaled by
// 1/128 (q) or 1/sqrt(128) (k). Raw rows and outputs go to the pending buffers of this pass's parity.
__global__ void __launch_bounds__(128) gdn_conv_kernel(GdnArgs a) {
    __shared__ float red[32];
    const int grp = blockIdx.x, c = grp * 128 + threadIdx.x, C = a.C, T = a.T;
    float cw[4];
#pragma unroll
    for (int i = 0; i < 4; i++) cw[i] = a.convw[(size_t)c * 4 + i];
    pdl_trigger();
    pdl_wait();
    const int par = a.ctl->parity, prev = par ^ 1, rn = a.ctl->replay_n;
    float st[3];
#pragma unroll
    for (int j = 0; j < 3; j++) st[j] = a.conv_state[(size_t)j * C + c];
    if (rn > 0) {
        const float* pq = a.pend_qkv + (size_t)prev * VMAX * C;
        float ns[3];
#pragma unroll
        for (int j = 0; j < 3; j++) {
            int k = rn + j;
            ns[j] = k < 3 ? st[k] : pq[(size_t)(k - 3) * C + c];
        }
#pragma unroll
        for (int j = 0; j < 3; j++) {
            st[j] = ns[j];
            a.conv_state[(size_t)j * C + c] = ns[j];
        }
    }
    const int ld = C + a.NV * 128;  // qkvz row stride
    float rows[3 + VMAX];
    rows[0] = st[0];
    rows[1] = st[1];
    rows[2] = st[2];
    for (int t = 0; t < T; t++) {
        float v = a.qkvz[(size_t)t * ld + c];
        rows[3 + t] = v;
        a.pend_qkv[((size_t)par * VMAX + t) * C + c] = v;
    }
    const bool qk = grp < 2 * a.NK;
    const float scale = grp < a.NK ? (1.0f / 128.0f) : 0.08838834764831845f;
    for (int t = 0; t < T; t++) {
        float acc = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; i++) acc += cw[i] * rows[t + i];
        float v = acc / (1.0f + expf(-acc));
        if (qk) {
            float ss = block_sum(v * v, red);
            float r = rsqrtf(ss / 128.0f + EPS_G);
            v = v * r * scale;
        }
        a.pend_qkvc[((size_t)par * VMAX + t) * C + c] = v;
    }
}

void launch_gdn_conv(const GdnArgs& a, cudaStream_t st) {
    GdnArgs aa = a;
    void* args[] = {&aa};
    launch_pdl((const void*)gdn_conv_kernel, dim3(a.C / 128), dim3(128), 0, st, args);
}

// gdn_gates (kernels.metal:556-561).
__device__ __forceinline__ void gates(float a_in, float b_in, float ea, float dtb, float& g, float& beta) {
    float x = a_in + dtb;
    float sp = fmaxf(x, 0.0f) + logf(1.0f + expf(-fabsf(x)));
    g = expf(-ea * sp);
    beta = 1.0f / (1.0f + expf(-b_in));
}

// One gated-delta step for the 4 dv rows a warp holds (lane: dk 4*lane..4*lane+3), kernels.metal:607-620:
// S *= g; kv = S.k; delta = (v - kv) beta; S += k delta; y = S.q.
__device__ __forceinline__ void gdn_step4(float4* st, float4 q, float4 k, const float* v, float g, float beta, float* o) {
    float kv[4];
#pragma unroll
    for (int r = 0; r < 4; r++) {
        st[r].x *= g; st[r].y *= g; st[r].z *= g; st[r].w *= g;
        kv[r] = st[r].x * k.x + st[r].y * k.y + st[r].z * k.z + st[r].w * k.w;
    }
#pragma unroll
    for (int r = 0; r < 4; r++) kv[r] = warp_sum(kv[r]);
#pragma unroll
    for (int r = 0; r < 4; r++) {
        float delta = (v[r] - kv[r]) * beta;
        st[r].x += k.x * delta; st[r].y += k.y * delta; st[r].z += k.z * delta; st[r].w += k.w * delta;
        o[r] = st[r].x * q.x + st[r].y * q.y + st[r].z * q.z + st[r].w * q.w;
    }
#pragma unroll
    for (int r = 0; r < 4; r++) o[r] = warp_sum(o[r]);
}

// gdn_recurrent (kernels.metal:566-622) with the deferred replay. Grid (NV, 8): CTA = 16 dv rows of one value head,
// warp = 4 rows, lane = 4 dk entries. V head h reads q/k head h / (NV / NK).
__global__ void __launch_bounds__(128) gdn_recurrent_kernel(GdnArgs a) {
    const int hd = blockIdx.x, lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int NK = a.NK, NV = a.NV, C = a.C;
    const int hk = hd / (NV / NK);
    const int dv0 = blockIdx.y * 16 + w * 4;
    float4 st[4];
    float* S = a.gdn_state + ((size_t)hd * 128 + dv0) * 128 + lane * 4;
    const float ea = expf(a.a_log[hd]), dtb = a.dt_bias[hd];
    pdl_trigger();
    pdl_wait();
#pragma unroll
    for (int r = 0; r < 4; r++) st[r] = *(const float4*)(S + (size_t)r * 128);
    const int par = a.ctl->parity, prev = par ^ 1, rn = a.ctl->replay_n;
    float o[4], vv[4];
    for (int t = 0; t < rn; t++) {
        const float* row = a.pend_qkvc + ((size_t)prev * VMAX + t) * C;
        const float* ab = a.pend_ab + ((size_t)prev * VMAX + t) * 2 * NV;
        float g, beta;
        gates(ab[hd], ab[NV + hd], ea, dtb, g, beta);
        float4 q = *(const float4*)(row + hk * 128 + lane * 4);
        float4 k = *(const float4*)(row + (NK + hk) * 128 + lane * 4);
#pragma unroll
        for (int r = 0; r < 4; r++) vv[r] = row[(2 * NK + hd) * 128 + dv0 + r];
        gdn_step4(st, q, k, vv, g, beta, o);
    }
    if (rn > 0) {
#pragma unroll
        for (int r = 0; r < 4; r++) *(float4*)(S + (size_t)r * 128) = st[r];
    }
    for (int t = 0; t < a.T; t++) {
        const float* row = a.pend_qkvc + ((size_t)par * VMAX + t) * C;
        const float* ab = a.pend_ab + ((size_t)par * VMAX + t) * 2 * NV;
        float g, beta;
        gates(ab[hd], ab[NV + hd], ea, dtb, g, beta);
        float4 q = *(const float4*)(row + hk * 128 + lane * 4);
        float4 k = *(const float4*)(row + (NK + hk) * 128 + lane * 4);
#pragma unroll
        for (int r = 0; r < 4; r++) vv[r] = row[(2 * NK + hd) * 128 + dv0 + r];
        gdn_step4(st, q, k, vv, g, beta, o);
        if (lane < 4) {
            float ov = lane == 0 ? o[0] : (lane == 1 ? o[1] : (lane == 2 ? o[2] : o[3]));
            a.y[(size_t)t * NV * 128 + hd * 128 + dv0 + lane] = ov;
        }
    }
}

void launch_gdn_recurrent(const GdnArgs& a, cudaStream_t st) {
    GdnArgs aa = a;
    void* args[] = {&aa};
    launch_pdl((const void*)gdn_recurrent_kernel, dim3(a.NV, 8), dim3(128), 0, st, args);
}

// Graded config 2: T rows from explicit q/k/v/gate inputs, outputs for every row, and the state written back as it
// was after the first n rows (the checkpoint taken in registers while the rows run).
__global__ void __launch_bounds__(128) gdn_verify_kernel(const float* q, const float* k, const float* v,
                                                         const float* a_in, const float* b_in, const float* a_log,
                                                         const float* dt_bias, float* state, float* y, int T, int NK,
                                                         int NV, int n) {
    const int hd = blockIdx.x, lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int hk = hd / (NV / NK);
    const int dv0 = blockIdx.y * 16 + w * 4;
    float4 st[4], keep[4];
    float* S = state + ((size_t)hd * 128 + dv0) * 128 + lane * 4;
    const float ea = expf(a_log[hd]), dtb = dt_bias[hd];
    pdl_trigger();
    pdl_wait();
#pragma unroll
    for (int r = 0; r < 4; r++) keep[r] = st[r] = *(const float4*)(S + (size_t)r * 128);
    float o[4], vv[4];
    for (int t = 0; t < T; t++) {
        float g, beta;
        gates(a_in[(size_t)t * NV + hd], b_in[(size_t)t * NV + hd], ea, dtb, g, beta);
        float4 qq = *(const float4*)(q + ((size_t)t * NK + hk) * 128 + lane * 4);
        float4 kk = *(const float4*)(k + ((size_t)t * NK + hk) * 128 + lane * 4);
#pragma unroll
        for (int r = 0; r < 4; r++) vv[r] = v[((size_t)t * NV + hd) * 128 + dv0 + r];
        gdn_step4(st, qq, kk, vv, g, beta, o);
        if (lane < 4) {
            float ov = lane == 0 ? o[0] : (lane == 1 ? o[1] : (lane == 2 ? o[2] : o[3]));
            y[((size_t)t * NV + hd) * 128 + dv0 + lane] = ov;
        }
        if (t + 1 == n) {
#pragma unroll
            for (int r = 0; r < 4; r++) keep[r] = st[r];
        }
    }
#pragma unroll
    for (int r = 0; r < 4; r++) *(float4*)(S + (size_t)r * 128) = keep[r];
}

void launch_gdn_verify(const float* q, const float* k, const float* v, const float* a_in, const float* b_in,
                       const float* a_log, const float* dt_bias, float* state, float* y, int T, int NK, int NV,
                       int n, cudaStream_t st) {
    void* args[] = {&q, &k, &v, &a_in, &b_in, &a_log, &dt_bias, &state, &y, &T, &NK, &NV, &n};
    launch_pdl((const void*)gdn_verify_kernel, dim3(NV, 8), dim3(128), 0, st, args);
}

}  // namespace bcu
