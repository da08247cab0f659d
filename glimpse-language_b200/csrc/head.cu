// head.cu — tied bf16 lm_head over all T rows with the argmax and the accept length fused in (encode_head_to,
// model.rs:941-985; argmax1/argmax2, kernels.metal:802-842; the accept length of decode_spec, runtime/mod.rs:866-868).
//
// The 248320 x 2048 bf16 table is 62% of a verify pass's bytes, so this kernel is a pure stream: the table is
// stored in mma fragment order (one 16-byte A fragment per lane per 16x16 tile), streamed through shared memory by
// bulk copies, the normed rows are a bf16 hi/lo operand kept in shared memory, and mma.m16n8k16 does the T-row
// products (fp32 accumulate). Logits never go to HBM: every warp keeps
// a running (max, lowest index) per row; CTAs publish partials, and the last CTA to finish merges them in CTA order,
// computes the accept length m on the device and advances the control block (KV offset, replay count, parity), so only
// m and the bonus token need to reach the host.
#include "common.cuh"
#include "kernels.h"

namespace bcu {

__global__ void repack_head_kernel(const uint16_t* __restrict__ table, int V, int d, uint32_t* __restrict__ out) {
    size_t n = (size_t)V * d / 2;  // u32 outputs
    size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= n) return;
    int r = idx & 3;
    int lane = (idx >> 2) & 31;
    size_t tile = idx >> 7;  // mt * (d/16) + ks
    int nks = d / 16;
    int ks = tile % nks;
    size_t mt = tile / nks;
    int g = lane >> 2, t4 = lane & 3;
    size_t row = mt * 16 + g + ((r & 1) ? 8 : 0);
    int k = ks * 16 + 2 * t4 + ((r & 2) ? 8 : 0);
    out[idx] = (uint32_t)table[row * d + k] | ((uint32_t)table[row * d + k + 1] << 16);
}

void repack_head_bf16(const uint16_t* table, int V, int d, uint32_t* out, cudaStream_t st) {
    size_t n = (size_t)V * d / 2;
    repack_head_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(table, V, d, out);
}

// Final norm of row t (model.rs:945-961; the bf16 table takes the normed row as is, no rotation) written as the
// bf16 hi/lo operand of the head GEMV (hi = bf16(x), lo = bf16(x - hi): 16 significant bits) in mma B-fragment order.
template <int NT>
__device__ void head_operand(const HeadArgs& a, int t, uint32_t* s_b) {
    const int lane = threadIdx.x & 31, d = a.d;
    float ss = 0.0f;
    for (int i = lane; i < a.nss; i += 32) ss += a.ss[i * VMAX + t];
    float r = rsqrtf(warp_sum(ss) / (float)d + 1e-6f);
    const int nt = t >> 2, gb = (t & 3) * 2, t4 = (lane & 7) >> 1, which = (lane & 15) >> 3;
#pragma unroll 4
    for (int kb = 0; kb < d; kb += 256) {  // 8 loads per lane and step, four steps' loads in flight together
        float hv[8], wv[8];
#pragma unroll
        for (int i = 0; i < 8; i++) hv[i] = a.h[(size_t)t * d + kb + i * 32 + lane];
#pragma unroll
        for (int i = 0; i < 8; i++) wv[i] = a.norm[kb + i * 32 + lane];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            int k = kb + i * 32 + lane;
            float x0 = (hv[i] * r) * wv[i];
            float x1 = __shfl_down_sync(0xffffffffu, x0, 1);
            if ((lane & 1) == 0) {
                __nv_bfloat16 h0 = __float2bfloat16_rn(x0), h1 = __float2bfloat16_rn(x1);
                __nv_bfloat16 l0 = __float2bfloat16_rn(x0 - __bfloat162float(h0));
                __nv_bfloat16 l1 = __float2bfloat16_rn(x1 - __bfloat162float(h1));
                size_t base = ((size_t)(k >> 4) * NT + nt) * 32;
                s_b[(base + gb * 4 + t4) * 2 + which] = pack_bf162(h0, h1);
                s_b[(base + (gb + 1) * 4 + t4) * 2 + which] = pack_bf162(l0, l1);
            }
        }
    }
}

constexpr int HEAD_KCH = 8;         // k-steps per staged unit: 8 x 512 B = 4 KB per warp
template <int NT>
__host__ __device__ constexpr int head_stages() { return NT >= 4 ? 3 : 4; }  // units in flight per warp (at most)
constexpr size_t HEAD_SMEM_MAX = 225 * 1024;  // the per-block opt-in limit (227 KB) minus the static arrays

// Shared memory: the operand [d/16][NT][32 lanes][2 words], then per warp a ring of head_stages() 4-KB units of the
// table, then their mbarriers.
__host__ __device__ inline size_t head_smem_bytes(int d, int nt, int stages) {
    return (size_t)(d / 16) * nt * 256 + (size_t)8 * stages * 4096 + (size_t)8 * stages * 8;
}

// End of the head (all CTAs): count this CTA's published (max, index) partials; the last CTA to arrive merges them in
// CTA order, computes the predictions, the accept length m on the device (leading drafts equal to the predictions,
// decode_spec's accept, runtime/mod.rs:866-868) and advances the control block (KV offset, replay count, parity).
__device__ void head_finish(const HeadArgs& a, int T) {
    __shared__ int s_last;
    __shared__ uint32_t pred[16];
    const int tid = threadIdx.x;
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(a.counter, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // one warp per row: lane l takes the partials of CTAs l, l + 32, ... with all its loads in flight together, then
    // a butterfly over the lanes. argmax_merge is a total order on (value, index) pairs (NaN never enters), so any
    // merge order gives the same winner.
    const int lane = tid & 31, warp = tid >> 5;
    for (int t = warp; t < T; t += 8) {
        float v = -INFINITY;
        int i = 0x7fffffff;
        for (int c0 = 0; c0 < (int)gridDim.x; c0 += 256) {
            float pv[8];
            int pi[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int c = c0 + lane + 32 * j;
                const bool in = c < (int)gridDim.x;
                pv[j] = in ? __ldcg(a.pv + (size_t)c * T + t) : -INFINITY;
                pi[j] = in ? __ldcg(a.pi + (size_t)c * T + t) : 0x7fffffff;
            }
#pragma unroll
            for (int j = 0; j < 8; j++) argmax_merge(v, i, pv[j], pi[j]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, i, o);
            argmax_merge(v, i, ov, oi);
        }
        if (lane == 0) {
            if (i == 0x7fffffff) i = 0;  // every logit NaN or -inf: index 0, like argmax2's initial value
            pred[t] = (uint32_t)i;
            a.ctl->pred[t] = (uint32_t)i;
        }
    }
    __syncthreads();
    if (tid == 0) {
        Ctl* c = a.ctl;
        int m;
        if (c->in.commit_all) {
            m = T - 1;
        } else {
            m = 0;
            while (m < T - 1 && c->used[m + 1] == pred[m]) m++;
        }
        c->accepted = m;
        c->bonus = pred[m];
        int nrows = c->in.commit_all ? T : m + 1;
        c->replay_n = nrows;
        c->off += nrows;
        c->parity ^= 1;
        *a.counter = 0;
    }
}

// One CTA per SM, 8 warps; warp w streams a contiguous range of 16-row m-tiles (a contiguous byte range of the
// repacked table) through its shared-memory ring with 4-KB bulk copies (cp.async.bulk, no multicast), so each warp
// keeps a.stages x 4 KB of the table in flight while its tensor-core products run (head_stages(), fewer when the
// operand of a wide hidden size leaves less room).
template <int NT>
__global__ void __launch_bounds__(256, 1) head_kernel(HeadArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int S = a.stages;
    uint2* s_b = (uint2*)smem;
    __shared__ float wbv[8][16];
    __shared__ int wbi[8][16];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nks = a.d / 16;
    const int T = a.T;
    const int nmt = a.V / 16;
    const int gw = blockIdx.x * 8 + warp, W = gridDim.x * 8;
    // contiguous m-tile range per warp (rows visited in increasing order)
    const int per = (nmt + W - 1) / W;
    const int mt0 = min(nmt, gw * per), mt1 = min(nmt, mt0 + per);
    const int upm = nks / HEAD_KCH;  // units per m-tile
    const int nunits = (mt1 - mt0) * upm;
    uint8_t* ring = smem + (size_t)nks * NT * 256 + (size_t)warp * S * 4096;
    uint64_t* bars = (uint64_t*)(smem + (size_t)nks * NT * 256 + (size_t)8 * S * 4096) + warp * S;
    const uint8_t* src = (const uint8_t*)a.w + (size_t)mt0 * nks * 512;
    // the table does not depend on the previous kernel: start streaming it before the dependency wait
    if (lane == 0) {
        for (int i = 0; i < S; i++) mbar_init(&bars[i], 1);
        fence_proxy_async_smem();
        for (int u = 0; u < S && u < nunits; u++) {
            mbar_expect_tx(&bars[u], 4096);
            bulk_g2s(ring + u * 4096, src + (size_t)u * 4096, 4096, &bars[u]);
        }
    }
    for (size_t i = tid; i < (size_t)nks * NT * 256 / 16; i += 256) ((uint4*)smem)[i] = make_uint4(0, 0, 0, 0);
    __syncthreads();
    pdl_trigger();
    pdl_wait();
    for (int t = warp; t < T; t += 8) head_operand<NT>(a, t, (uint32_t*)smem);
    __syncthreads();
    const int keep = a.ctl->in.keep_logits;
    const int g = lane >> 2, t4 = lane & 3;
    float bv[NT];
    int bi[NT];
#pragma unroll
    for (int n = 0; n < NT; n++) {
        bv[n] = -INFINITY;
        bi[n] = 0x7fffffff;
    }
    float acc[NT][4];
#pragma unroll
    for (int n = 0; n < NT; n++) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
    int mt = mt0;
    for (int u = 0; u < nunits; u++) {
        const int slot = u % S;
        const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(&bars[slot], (u / S) & 1));
        if (!ok) {  // give up: wait (bounded) for the copies in flight, report, stop streaming
            if (lane == 0) {
                atomicOr(&a.ctl->err, ERR_MBAR_TIMEOUT);
                for (int v = u; v < u + S && v < nunits; v++) mbar_wait_bounded(&bars[v % S], (v / S) & 1, 1u << 20);
            }
            break;
        }
        const uint4* wk = (const uint4*)(ring + slot * 4096) + lane;
        const int kb = (u % upm) * HEAD_KCH;
#pragma unroll
        for (int i = 0; i < HEAD_KCH; i++) {
            const uint4 w = wk[i * 32];
#pragma unroll
            for (int n = 0; n < NT; n++) {
                const uint2 b = s_b[((size_t)(kb + i) * NT + n) * 32 + lane];
                mma_bf16(acc[n], w.x, w.y, w.z, w.w, b.x, b.y);
            }
        }
        __syncwarp();
        if (lane == 0 && u + S < nunits) {  // the slot's data is consumed: refill it with unit u + S
            fence_proxy_async_smem();
            mbar_expect_tx(&bars[slot], 4096);
            bulk_g2s(ring + slot * 4096, src + (size_t)(u + S) * 4096, 4096, &bars[slot]);
        }
        if ((u + 1) % upm == 0) {  // m-tile done: its 16 rows' logits into the running argmax
#pragma unroll
            for (int n = 0; n < NT; n++) {
                int token = n * 4 + t4;
                float v0 = acc[n][0] + acc[n][1], v1 = acc[n][2] + acc[n][3];
                int r0 = mt * 16 + g, r1 = r0 + 8;
                if (keep && token < T) {
                    a.logits[(size_t)token * a.V + r0] = v0;
                    a.logits[(size_t)token * a.V + r1] = v1;
                }
                argmax_merge(bv[n], bi[n], v0, r0);
                argmax_merge(bv[n], bi[n], v1, r1);
                acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
            }
            mt++;
        }
    }
    // lanes with the same t4 hold the same token: merge over g
#pragma unroll
    for (int n = 0; n < NT; n++) {
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
            float ov = __shfl_xor_sync(0xffffffffu, bv[n], o);
            int oi = __shfl_xor_sync(0xffffffffu, bi[n], o);
            argmax_merge(bv[n], bi[n], ov, oi);
        }
        if (g == 0) {
            wbv[warp][n * 4 + t4] = bv[n];
            wbi[warp][n * 4 + t4] = bi[n];
        }
    }
    __syncthreads();
    if (tid < T) {
        float v = -INFINITY;
        int i = 0x7fffffff;
        for (int w = 0; w < 8; w++) argmax_merge(v, i, wbv[w][tid], wbi[w][tid]);
        a.pv[(size_t)blockIdx.x * T + tid] = v;
        a.pi[(size_t)blockIdx.x * T + tid] = i;
    }
    head_finish(a, T);
}

template <int NT>
static void launch_head_t(const HeadArgs& a, int grid, cudaStream_t st) {
    int stages = head_stages<NT>();
    while (stages > 1 && head_smem_bytes(a.d, NT, stages) > HEAD_SMEM_MAX) stages--;
    size_t smem = head_smem_bytes(a.d, NT, stages);
    raise_smem_limit((const void*)head_kernel<NT>, (int)HEAD_SMEM_MAX);
    HeadArgs aa = a;
    aa.stages = stages;
    void* args[] = {&aa};
    launch_pdl((const void*)head_kernel<NT>, dim3(grid), dim3(256), smem, st, args);
}

void launch_head(const HeadArgs& a, int NT, int grid, cudaStream_t st) {
    if (NT == 1) launch_head_t<1>(a, grid, st);
    else if (NT == 2) launch_head_t<2>(a, grid, st);
    else if (NT == 3) launch_head_t<3>(a, grid, st);
    else launch_head_t<4>(a, grid, st);
}

// ------------------------------------------------------------------------------------------------ ternary tied table
// The reference's own embedding and head (model.rs:356, 941-985): a ternary-packed tied table [V][d] with Hadamard
// signs. The head is the ternary GEMV (final norm + rotation by the table's signs, then the table) writing fp32
// logits; head_argmax_kernel then takes the per-row argmax and ends the pass like head_kernel.

// embed (kernels.metal:230-246) of each row of the pass: code -> (c - 1) s (or c s + b) rounded to fp16, the
// 512-point transform in fwht512's lane layout (strides 1..16 across lanes, 32..256 in-lane: bit-identical to the
// in-memory order), x INV_SQRT512 x sign rounded to fp16, written to the residual rows h. Also the row-block sums
// of squares the first GEMV's RMSNorm reads ([d/128][VMAX]: lane l holds elements l + 32 e, so row block e / 4), and
// the ids the pass embedded. One CTA per row, one warp per 512 inputs.
__global__ void __launch_bounds__(256) embed_ternary_kernel(EmbedArgs a) {
    pdl_trigger();
    pdl_wait();  // the ids may be the previous pass's bonus token
    const int t = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int d = a.d, b0 = warp * 512;
    if (b0 >= d) return;
    uint32_t id = resolve_id(a.ctl, t);
    if (warp == 0 && lane == 0) {
        a.ctl->used[t] = id;
        if (id >= (uint32_t)a.V) atomicOr(&a.ctl->err, ERR_BAD_TOKEN);
    }
    if (id >= (uint32_t)a.V) id = 0;
    const int kw = d / 16, kg = d / a.group;
    const uint32_t* wr = a.w + (size_t)id * kw;
    float v[16];
#pragma unroll
    for (int e = 0; e < 16; e++) {
        const int k = b0 + lane + 32 * e;
        const float c = (float)((wr[k >> 4] >> (2 * (k & 15))) & 3u);
        const float sc = __half2float(__ushort_as_half(a.s[(size_t)id * kg + k / a.group]));
        const float w = a.b ? __fadd_rn(__fmul_rn(c, sc), __half2float(__ushort_as_half(a.b[(size_t)id * kg + k / a.group])))
                            : __fmul_rn(c - 1.0f, sc);
        v[e] = __half2float(__float2half_rn(w));
    }
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
        const bool up = (lane & m) != 0;
#pragma unroll
        for (int e = 0; e < 16; e++) {
            const float o = __shfl_xor_sync(0xffffffffu, v[e], m);
            v[e] = up ? __fsub_rn(o, v[e]) : __fadd_rn(v[e], o);
        }
    }
#pragma unroll
    for (int h = 1; h < 16; h <<= 1)
#pragma unroll
        for (int e = 0; e < 16; e++)
            if ((e & h) == 0) {
                const float x = v[e], y = v[e + h];
                v[e] = __fadd_rn(x, y);
                v[e + h] = __fsub_rn(x, y);
            }
    float ss[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int e = 0; e < 16; e++) {
        const int k = b0 + lane + 32 * e;
        const float sg = a.signs ? a.signs[k] : 1.0f;
        const float x = __half2float(__float2half_rn(__fmul_rn(__fmul_rn(v[e], 0.044194173824159216f), sg)));
        a.h[(size_t)t * d + k] = x;
        ss[e >> 2] = __fadd_rn(ss[e >> 2], __fmul_rn(x, x));
    }
#pragma unroll
    for (int r = 0; r < 4; r++) {
        const float tot = warp_sum(ss[r]);
        if (lane == 0) a.ss[(size_t)(b0 / 128 + r) * VMAX + t] = tot;
    }
}

void launch_embed_ternary(const EmbedArgs& a, cudaStream_t st) {
    EmbedArgs aa = a;
    void* args[] = {&aa};
    launch_pdl((const void*)embed_ternary_kernel, dim3(a.T), dim3(32 * (a.d / 512)), 0, st, args);
}

// Argmax over the logits [T][V] the ternary head GEMV wrote (argmax1/argmax2, kernels.metal:802-842): CTA c scans a
// contiguous range of the vocabulary for every row (256 threads strided, then the warp and block merges, lowest index
// on ties), publishes its partials and ends the pass through head_finish.
__global__ void __launch_bounds__(256) head_argmax_kernel(HeadArgs a) {
    pdl_trigger();
    pdl_wait();
    __shared__ float wbv[8][VMAX];
    __shared__ int wbi[8][VMAX];
    const int T = a.T, V = a.V, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int per = (V + gridDim.x - 1) / gridDim.x;
    const int v0 = min(V, (int)blockIdx.x * per), v1 = min(V, v0 + per);
    for (int t = 0; t < T; t++) {
        const float* row = a.logits + (size_t)t * V;
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int i = v0 + tid; i < v1; i += 256) argmax_merge(bv, bi, __ldcg(row + i), i);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            argmax_merge(bv, bi, ov, oi);
        }
        if (lane == 0) {
            wbv[warp][t] = bv;
            wbi[warp][t] = bi;
        }
    }
    __syncthreads();
    if (tid < T) {
        float v = -INFINITY;
        int i = 0x7fffffff;
        for (int w = 0; w < 8; w++) argmax_merge(v, i, wbv[w][tid], wbi[w][tid]);
        a.pv[(size_t)blockIdx.x * T + tid] = v;
        a.pi[(size_t)blockIdx.x * T + tid] = i;
    }
    head_finish(a, T);
}

void launch_head_argmax(const HeadArgs& a, int grid, cudaStream_t st) {
    HeadArgs aa = a;
    void* args[] = {&aa};
    launch_pdl((const void*)head_argmax_kernel, dim3(grid), dim3(256), 0, st, args);
}

}  // namespace bcu
