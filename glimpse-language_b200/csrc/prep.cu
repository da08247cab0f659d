// prep.cu — producer kernels: the elementwise / normalisation / rotation steps that turn one activation row into the
// tensor-core operand of the next GEMV. One CTA per (padded) token row, 512 threads; the row lives in shared memory.
// They restate norm_rotate, swiglu_rotate, gate_rotate (+ attn_combine), gated_norm_rotate and the head's final norm
// (kernels.metal:118-226, 783-799; model.rs:692-708, 797-812, 872-893, 898-931, 945-961).
#include "act.cuh"
#include "common.cuh"
#include "kernels.h"

namespace bcu {

constexpr float EPS = 1e-6f;

// Token of row t after the feed rule (host ids, previous bonus, or the planted stream).
__device__ inline uint32_t resolve_id(const Ctl* ctl, int t) {
    int feed = ctl->in.feed;
    if (feed == 1 && t == 0) return ctl->bonus;
    if (feed == 2 && ctl->planted) {
        int i = ctl->off - ctl->in.planted_base + t;
        if (i >= 0 && i < ctl->planted_n) return ctl->planted[i];
    }
    return ctl->in.ids[t];
}

// norm_rotate (kernels.metal:118-144) with the bf16 embedding gather fused in front for the first layer.
__global__ void __launch_bounds__(512) prep_norm_kernel(PrepNormArgs a, int NT) {
    const int vocab = a.vocab;
    extern __shared__ float x[];
    __shared__ float red[32];
    const int t = blockIdx.x, D = a.D;
    pdl_trigger();
    pdl_wait();
    if (t < a.T) {
        float* hr = a.h + (size_t)t * D;
        if (a.embed_bf16) {
            uint32_t id = resolve_id(a.ctl, t);
            if (threadIdx.x == 0) {
                ((Ctl*)a.ctl)->used[t] = id;
                if (id >= (uint32_t)vocab) atomicOr(&((Ctl*)a.ctl)->err, ERR_BAD_TOKEN);
            }
            if (id >= (uint32_t)vocab) id = 0;
            const uint16_t* er = a.embed_bf16 + (size_t)id * D;
            for (int i = threadIdx.x; i < D; i += blockDim.x) {
                float v = __bfloat162float(__ushort_as_bfloat16(er[i]));
                x[i] = v;
                hr[i] = v;
            }
        } else {
            for (int i = threadIdx.x; i < D; i += blockDim.x) x[i] = hr[i];
        }
        float ss = 0.0f;
        for (int i = threadIdx.x; i < D; i += blockDim.x) ss += x[i] * x[i];
        ss = block_sum(ss, red);
        float r = rsqrtf(ss / (float)D + EPS);
        for (int i = threadIdx.x; i < D; i += blockDim.x) {
            float v = (x[i] * r) * a.w[i];
            x[i] = v;
            if (a.xn) a.xn[(size_t)t * D + i] = v;
        }
        __syncthreads();
        block_rotate(x, D, a.HB, a.signs);
    }
    write_ternary_act(x, D, t, a.T, NT, a.group, a.act, red);
}

void launch_prep_norm(const PrepNormArgs& a, int NT, cudaStream_t st) {
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(prep_norm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
        attr = true;
    }
    PrepNormArgs aa = a;
    int nt = NT;
    void* args[] = {&aa, &nt};
    launch_pdl((const void*)prep_norm_kernel, dim3(4 * NT), dim3(512), (size_t)a.D * 4, st, args);
}

// swiglu_rotate (kernels.metal:147-164): x = (g * u) * sigmoid(g), then rotate.
__global__ void __launch_bounds__(512) prep_swiglu_kernel(PrepSwigluArgs a, int NT) {
    extern __shared__ float x[];
    __shared__ float red[32];
    const int t = blockIdx.x, ff = a.ff;
    pdl_trigger();
    pdl_wait();
    if (t < a.T) {
        const float* gr = a.gu + (size_t)t * 2 * ff;
        for (int i = threadIdx.x; i < ff; i += blockDim.x) {
            float g = gr[i], u = gr[ff + i];
            x[i] = (g * u) * (1.0f / (1.0f + expf(-g)));
        }
        __syncthreads();
        block_rotate(x, ff, a.HB, a.signs);
    }
    write_ternary_act(x, ff, t, a.T, NT, a.group, a.act, red);
}

void launch_prep_swiglu(const PrepSwigluArgs& a, int NT, cudaStream_t st) {
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(prep_swiglu_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
        attr = true;
    }
    PrepSwigluArgs aa = a;
    int nt = NT;
    void* args[] = {&aa, &nt};
    launch_pdl((const void*)prep_swiglu_kernel, dim3(4 * NT), dim3(512), (size_t)a.ff * 4, st, args);
}

// gated_norm_rotate (kernels.metal:199-226): per 128-wide v head, x = (((z * y) * r) * w) * sigmoid(z) with
// r = rsqrt(mean(y^2) + eps); then rotate.
__global__ void __launch_bounds__(512) prep_gated_kernel(PrepGatedArgs a, int NT) {
    extern __shared__ float x[];
    __shared__ float red[32];
    const int t = blockIdx.x, gw = a.gw;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    pdl_trigger();
    pdl_wait();
    if (t < a.T) {
        const float* y = a.y + (size_t)t * gw;
        const float* z = a.qkvz + (size_t)t * (a.C + gw) + a.C;
        for (int hd = warp; hd < gw / 128; hd += nw) {
            float4 yv = *(const float4*)(y + hd * 128 + lane * 4);
            float ss = warp_sum(yv.x * yv.x + yv.y * yv.y + yv.z * yv.z + yv.w * yv.w);
            float r = rsqrtf(ss / 128.0f + EPS);
            float yy[4] = {yv.x, yv.y, yv.z, yv.w};
#pragma unroll
            for (int i = 0; i < 4; i++) {
                int d = lane * 4 + i;
                float zz = z[hd * 128 + d];
                x[hd * 128 + d] = (((zz * yy[i]) * r) * a.w[d]) * (1.0f / (1.0f + expf(-zz)));
            }
        }
        __syncthreads();
        block_rotate(x, gw, a.HB, a.signs);
    }
    write_ternary_act(x, gw, t, a.T, NT, a.group, a.act, red);
}

void launch_prep_gated(const PrepGatedArgs& a, int NT, cudaStream_t st) {
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(prep_gated_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
        attr = true;
    }
    PrepGatedArgs aa = a;
    int nt = NT;
    void* args[] = {&aa, &nt};
    launch_pdl((const void*)prep_gated_kernel, dim3(4 * NT), dim3(512), (size_t)a.gw * 4, st, args);
}

// attn_combine (kernels.metal:783-799) + gate_rotate (:170-188): log-sum-exp merge of the split partials, times
// sigmoid of the gate half of the q projection, then rotate.
__global__ void __launch_bounds__(512) prep_attn_out_kernel(PrepAttnOutArgs a, int NT) {
    extern __shared__ float x[];
    __shared__ float red[32];
    const int t = blockIdx.x, H = a.H, aw = H * 256;
    pdl_trigger();
    pdl_wait();
    if (t < a.T) {
        for (int e = threadIdx.x; e < aw; e += blockDim.x) {
            int h = e >> 8, d = e & 255;
            const float* p = a.part + ((size_t)t * H + h) * NSPLIT_ATTN * 258;
            float M = -INFINITY;
            for (int s = 0; s < NSPLIT_ATTN; s++) M = fmaxf(M, p[s * 258]);
            float L = 0.0f, acc = 0.0f;
            for (int s = 0; s < NSPLIT_ATTN; s++) {
                float m = p[s * 258];
                if (m == -INFINITY) continue;
                float w = expf(m - M);
                L += p[s * 258 + 1] * w;
                acc += p[s * 258 + 2 + d] * w;
            }
            float gt = a.qkv[(size_t)t * a.qkv_ld + h * 512 + 256 + d];
            x[e] = (acc / L) * (1.0f / (1.0f + expf(-gt)));
        }
        __syncthreads();
        block_rotate(x, aw, a.HB, a.signs);
    }
    write_ternary_act(x, aw, t, a.T, NT, a.group, a.act, red);
}

void launch_prep_attn_out(const PrepAttnOutArgs& a, int NT, cudaStream_t st) {
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(prep_attn_out_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
        attr = true;
    }
    PrepAttnOutArgs aa = a;
    int nt = NT;
    void* args[] = {&aa, &nt};
    launch_pdl((const void*)prep_attn_out_kernel, dim3(4 * NT), dim3(512), (size_t)a.H * 256 * 4, st, args);
}

// Final norm of the head (model.rs:945-961 without the rotation: the bf16 table takes the normed row as is), written as
// the bf16 hi/lo operand of the head GEMV.
__global__ void __launch_bounds__(512) prep_head_kernel(PrepHeadArgs a, int NT) {
    extern __shared__ float x[];
    __shared__ float red[32];
    const int t = blockIdx.x, D = a.D;
    pdl_trigger();
    pdl_wait();
    if (t < a.T) {
        const float* hr = a.h + (size_t)t * D;
        float ss = 0.0f;
        for (int i = threadIdx.x; i < D; i += blockDim.x) {
            float v = hr[i];
            x[i] = v;
            ss += v * v;
        }
        ss = block_sum(ss, red);
        float r = rsqrtf(ss / (float)D + EPS);
        for (int i = threadIdx.x; i < D; i += blockDim.x) x[i] = (x[i] * r) * a.w[i];
        __syncthreads();
    }
    write_bf16_act(x, D, t, a.T, NT, a.bfrag);
}

void launch_prep_head(const PrepHeadArgs& a, int NT, cudaStream_t st) {
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(prep_head_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
        attr = true;
    }
    PrepHeadArgs aa = a;
    int nt = NT;
    void* args[] = {&aa, &nt};
    launch_pdl((const void*)prep_head_kernel, dim3(4 * NT), dim3(512), (size_t)a.D * 4, st, args);
}

// Plain bf16 embedding gather (only needed when a pass does not start with the fused prep_norm).
__global__ void embed_kernel(const Ctl* ctl, const uint16_t* table, float* h, int d, int vocab) {
    int t = blockIdx.x;
    pdl_trigger();
    pdl_wait();
    uint32_t id = resolve_id(ctl, t);
    if (id >= (uint32_t)vocab) id = 0;
    for (int i = threadIdx.x; i < d; i += blockDim.x)
        h[(size_t)t * d + i] = __bfloat162float(__ushort_as_bfloat16(table[(size_t)id * d + i]));
}

void launch_embed(const Ctl* ctl, const uint16_t* table, float* h, int d, int vocab, int T, cudaStream_t st) {
    void* args[] = {&ctl, &table, &h, &d, &vocab};
    launch_pdl((const void*)embed_kernel, dim3(T), dim3(256), 0, st, args);
}

}  // namespace bcu
