// attn.cu — gated full-attention layer kernels: attn_prep (q/k RMSNorm, interleaved mRoPE, KV write;
// kernels.metal:627-662) and split-K causal GQA (attn_split, kernels.metal:713-780). The merge of the partials is fused
// into the next producer (prep_attn_out). The grid is fixed for graph capture; each CTA derives its key range from
// the device-side KV offset, so one captured graph serves every context length.
#include "common.cuh"
#include "kernels.h"

namespace bcu {

constexpr float EPS_A = 1e-6f;

// Grid (T, H + 2 KV), 256 threads (one per head dim): q heads, then k heads, then v heads.
__global__ void __launch_bounds__(256) attn_prep_kernel(AttnArgs a) {
    __shared__ float red[32];
    __shared__ float buf[256];
    const int t = blockIdx.x, hh = blockIdx.y, d = threadIdx.x;
    const int H = a.H, KV = a.KV;
    const float wq = a.qn[d], wk = a.kn[d];
    pdl_trigger();
    pdl_wait();
    const int pos = a.ctl->off + t;
    if (pos >= a.ctx) {
        if (d == 0 && hh == 0) atomicOr(&((Ctl*)a.ctl)->err, ERR_CTX_FULL);
        return;
    }
    const float* row = a.qkv + (size_t)t * a.ld;
    const int aw = H * 256, kvw = KV * 256;
    if (hh >= H + KV) {
        int kh = hh - H - KV;
        a.vc[((size_t)pos * KV + kh) * 256 + d] = row[2 * aw + kvw + kh * 256 + d];
        return;
    }
    const bool isq = hh < H;
    float x = isq ? row[hh * 512 + d] : row[2 * aw + (hh - H) * 256 + d];
    float ss = block_sum(x * x, red);
    float r = rsqrtf(ss / 256.0f + EPS_A);
    x = (x * r) * (isq ? wq : wk);
    buf[d] = x;
    __syncthreads();
    if (d < a.rot) {
        int half = a.rot / 2, i = d % half;
        // text positions: the three mrope position rows are equal, so every section uses `pos`
        float ang = (float)pos * a.inv_freq[i];
        float sn, cs;
        sincosf(ang, &sn, &cs);
        x = d < half ? x * cs - buf[d + half] * sn : x * cs + buf[d - half] * sn;
    }
    if (isq) a.q[((size_t)t * H + hh) * 256 + d] = x;
    else a.kc[((size_t)pos * KV + (hh - H)) * 256 + d] = x;
}

void launch_attn_prep(const AttnArgs& a, cudaStream_t st) {
    AttnArgs aa = a;
    void* args[] = {&aa};
    launch_pdl((const void*)attn_prep_kernel, dim3(a.T, a.H + 2 * a.KV), dim3(256), 0, st, args);
}

// Grid (KV, NSPLIT_ATTN, T), 256 threads. The qper = H / KV query heads of one kv head share each K/V read (the
// reference shares 4, kernels.metal:731-742; the graded 2B shape has 8). Keys [0, off + t] are split into NSPLIT_ATTN
// equal chunks; the CTA writes (max, sum, acc[256]) per query head, like attn_split.
__global__ void __launch_bounds__(256) attn_split_kernel(AttnArgs a) {
    extern __shared__ float sm[];
    const int kh = blockIdx.x, s = blockIdx.y, t = blockIdx.z;
    const int H = a.H, KV = a.KV, qper = H / KV;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, tid = threadIdx.x;
    const int chunk_max = (a.ctx + NSPLIT_ATTN - 1) / NSPLIT_ATTN;
    float* qs = sm;                       // [qper][256]
    float* sc = sm + qper * 256;          // [qper][chunk_max]
    float* ml = sc + qper * chunk_max;    // [qper][2]
    pdl_trigger();
    pdl_wait();
    const int n = a.ctl->off + t + 1;
    const int chunk = (n + NSPLIT_ATTN - 1) / NSPLIT_ATTN;
    const int j0 = s * chunk, j1 = min(n, j0 + chunk);
    float* pp = a.part + ((size_t)t * H + kh * qper) * NSPLIT_ATTN * 258 + (size_t)s * 258;
    if (j0 >= j1) {
        if (tid < qper) {
            pp[(size_t)tid * NSPLIT_ATTN * 258] = -INFINITY;
            pp[(size_t)tid * NSPLIT_ATTN * 258 + 1] = 0.0f;
        }
        return;
    }
    for (int i = tid; i < qper * 256; i += 256) {
        int hq = i >> 8, d = i & 255;
        qs[i] = a.q[((size_t)t * H + kh * qper + hq) * 256 + d] * 0.0625f;
    }
    __syncthreads();
    // scores: warp per key, lanes over dims (8 each)
    for (int j = j0 + w; j < j1; j += 8) {
        const float* k = a.kc + ((size_t)j * KV + kh) * 256 + lane * 8;
        float4 ka = *(const float4*)k, kb = *(const float4*)(k + 4);
        for (int hq = 0; hq < qper; hq++) {
            const float* q = qs + hq * 256 + lane * 8;
            float dd = q[0] * ka.x + q[1] * ka.y + q[2] * ka.z + q[3] * ka.w + q[4] * kb.x + q[5] * kb.y + q[6] * kb.z +
                       q[7] * kb.w;
            dd = warp_sum(dd);
            if (lane == 0) sc[hq * chunk_max + (j - j0)] = dd;
        }
    }
    __syncthreads();
    const int cnt = j1 - j0;
    for (int hq = w; hq < qper; hq += 8) {
        float m = -INFINITY;
        for (int i = lane; i < cnt; i += 32) m = fmaxf(m, sc[hq * chunk_max + i]);
        m = warp_max(m);
        float l = 0.0f;
        for (int i = lane; i < cnt; i += 32) {
            float p = expf(sc[hq * chunk_max + i] - m);
            sc[hq * chunk_max + i] = p;
            l += p;
        }
        l = warp_sum(l);
        if (lane == 0) {
            ml[hq * 2] = m;
            ml[hq * 2 + 1] = l;
        }
    }
    __syncthreads();
    // P.V: thread = head dim, all query heads at once, keys in order
    float acc[16];
#pragma unroll
    for (int hq = 0; hq < 16; hq++) acc[hq] = 0.0f;
    for (int i = 0; i < cnt; i++) {
        float v = a.vc[((size_t)(j0 + i) * KV + kh) * 256 + tid];
#pragma unroll
        for (int hq = 0; hq < 16; hq++)
            if (hq < qper) acc[hq] += sc[hq * chunk_max + i] * v;
    }
#pragma unroll
    for (int hq = 0; hq < 16; hq++)
        if (hq < qper) {
            float* ph = pp + (size_t)hq * NSPLIT_ATTN * 258;
            if (tid == 0) {
                ph[0] = ml[hq * 2];
                ph[1] = ml[hq * 2 + 1];
            }
            ph[2 + tid] = acc[hq];
        }
}

void launch_attn_split(const AttnArgs& a, cudaStream_t st) {
    int qper = a.H / a.KV;
    int chunk_max = (a.ctx + NSPLIT_ATTN - 1) / NSPLIT_ATTN;
    size_t smem = ((size_t)qper * 256 + (size_t)qper * chunk_max + 2 * qper) * 4;
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(attn_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        attr = true;
    }
    AttnArgs aa = a;
    void* args[] = {&aa};
    launch_pdl((const void*)attn_split_kernel, dim3(a.KV, NSPLIT_ATTN, a.T), dim3(256), smem, st, args);
}

}  // namespace bcu
