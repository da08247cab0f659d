// ops.cu — standalone hot ops of the C ABI on caller-owned device buffers: the rotate-then-ternary-linear of graded
// config 1 and the GatedDeltaNet verify step with rollback of graded config 2.
#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/bonsai_cuda.h"
#include "common.cuh"
#include "kernels.h"
#include "operand.cuh"

using namespace bcu;

struct bcu_linear {
    int device = 0, sms = 148;
    TernaryMat m;
    void* codes = nullptr;
    uint32_t* sb = nullptr;
    // per-call scratch, sized for T <= 16
    float* partial = nullptr;
    unsigned* counters = nullptr;
    int* err = nullptr;
    // the rotated operand when the GEMV's CTAs build it together (grid_build): room for the largest block size
    uint8_t* opbuf = nullptr;
    unsigned* op_counters = nullptr;
    bool local_build = false;  // test hook: every CTA builds its own slice
    // prefill GEMM (gemm.cu): packed weights and bias tiles; activation tiles and exponents grown on demand
    uint8_t *gwt = nullptr, *gbias = nullptr, *gbop = nullptr;
    int* gex = nullptr;
    size_t gbop_bytes = 0;
    int gex_n = 0;
};

extern "C" {

bcu_status bcu_linear_prepare(const uint32_t* w_host, const uint16_t* scales_host, const uint16_t* biases_host,
                              int32_t O, int32_t K, int32_t group, int32_t device, bcu_linear** out) {
    if (!w_host || !scales_host || !out || O <= 0 || K <= 0 || O % 128 || K % 512 || (group != 64 && group != 128))
        return BCU_ERR_ARG;
    if (cudaSetDevice(device) != cudaSuccess) return BCU_ERR_CUDA;
    bcu_linear* l = new bcu_linear();
    l->device = device;
    size_t wb = (size_t)O * K / 4, sb = (size_t)O * (K / group) * 2;
    uint32_t* dw = nullptr;
    uint16_t *ds = nullptr, *db = nullptr;
    bool ok = cudaMalloc(&dw, wb) == cudaSuccess && cudaMalloc(&ds, sb) == cudaSuccess &&
              (!biases_host || cudaMalloc(&db, sb) == cudaSuccess) && cudaMalloc(&l->codes, wb) == cudaSuccess &&
              cudaMalloc(&l->sb, ternary_sb_bytes(O, K, group)) == cudaSuccess;
    if (ok) {
        ok = cudaMemcpy(dw, w_host, wb, cudaMemcpyHostToDevice) == cudaSuccess &&
             cudaMemcpy(ds, scales_host, sb, cudaMemcpyHostToDevice) == cudaSuccess &&
             (!biases_host || cudaMemcpy(db, biases_host, sb, cudaMemcpyHostToDevice) == cudaSuccess);
    }
    ok = ok && cudaMalloc(&l->gwt, gemm_w_bytes(O, K)) == cudaSuccess &&
         cudaMalloc(&l->gbias, gemm_bias_bytes(O, K, group)) == cudaSuccess;
    if (ok) {
        repack_ternary(dw, ds, db, O, K, group, l->codes, l->sb, 0);
        gemm_pack(dw, ds, db, O, K, group, l->gwt, l->gbias, 0);
        ok = cudaDeviceSynchronize() == cudaSuccess;
    }
    cudaFree(dw);
    cudaFree(ds);
    cudaFree(db);
    l->m.codes = l->codes;
    l->m.sb = l->sb;
    l->m.O = O;
    l->m.K = K;
    l->m.group = group;
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    l->sms = sms;
    plan_ternary(l->m, sms);
    ok = ok && cudaMalloc(&l->partial, (size_t)l->m.nsplit * VMAX * O * 4) == cudaSuccess &&
         cudaMalloc(&l->counters, (size_t)(O / 128) * 4) == cudaSuccess && cudaMalloc(&l->err, 4) == cudaSuccess &&
         cudaMemset(l->counters, 0, (size_t)(O / 128) * 4) == cudaSuccess && cudaMemset(l->err, 0, 4) == cudaSuccess;
    size_t opb = 0;
    for (int hb : {512, 1024, 2048})
        if (K % hb == 0) opb = std::max(opb, (size_t)(K / hb) * 4 * op_region_bytes(hb, group));
    ok = ok && cudaMalloc(&l->opbuf, opb) == cudaSuccess && cudaMalloc(&l->op_counters, 8) == cudaSuccess &&
         cudaMemset(l->opbuf, 0, opb) == cudaSuccess && cudaMemset(l->op_counters, 0, 8) == cudaSuccess &&
         cudaDeviceSynchronize() == cudaSuccess;  // callers may launch on a non-blocking stream
    if (!ok) {
        bcu_linear_free(l);
        return BCU_ERR_OOM;
    }
    *out = l;
    return BCU_OK;
}

void bcu_linear_free(bcu_linear* l) {
    if (!l) return;
    cudaSetDevice(l->device);
    void* p[] = {l->codes, l->sb,   l->partial, l->counters, l->err,  l->gwt,
                 l->gbias, l->gbop, l->gex,     l->opbuf,    l->op_counters};
    for (void* q : p)
        if (q) cudaFree(q);
    delete l;
}

// The K-slice plan of a call rotating in HB-point blocks: slices of whole blocks (a slice that split a block would
// have every CTA of the block transform all of it, and the grid-built operand holds whole blocks). The plan depends
// on HB only, never on T or on how the operand is built, so a row's result is the same bits at every T.
static TernaryMat rotate_plan(const bcu_linear* l, int HB) {
    TernaryMat mm = l->m;
    if (HB > mm.kslice) plan_ternary(mm, l->sms, HB);
    return mm;
}

static bcu_status linear_run(bcu_linear* l, const uint16_t* xb, const float* xf, int T, int HB, const float* signs,
                             float* y, void* stream) {
    if (!l || (!xb && !xf) || !y || T < 1 || T > VMAX) return BCU_ERR_ARG;
    if (HB && (HB != 512 && HB != 1024 && HB != 2048)) return BCU_ERR_ARG;
    if (HB && l->m.K % HB) return BCU_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    const TernaryMat mm = rotate_plan(l, HB);
    ActSrc src;
    src.mode = ACT_EXT;
    src.x = xf;
    src.xb = xb;
    src.signs = signs;
    src.HB = HB;
    if (HB && !l->local_build && gemv_coresident(mm, T, 0, HB, l->sms, 0)) {  // the CTAs build the operand together
        src.opbuf = l->opbuf;
        src.op_counters = l->op_counters;
    }
    GemvOut o;
    o.out = y;
    o.partial = l->partial;
    o.counters = l->counters;
    o.err = l->err;
    launch_ternary_gemv(mm, src, T, o, nullptr, st);
    if (cudaGetLastError() != cudaSuccess) return BCU_ERR_CUDA;
    return BCU_OK;
}

bcu_status bcu_linear_rotate_forward(bcu_linear* l, const uint16_t* x_bf16_dev, int32_t T, int32_t hadamard,
                                     const float* signs_dev, float* y_dev, void* stream) {
    if (!l) return BCU_ERR_ARG;
    cudaSetDevice(l->device);
    return linear_run(l, x_bf16_dev, nullptr, T, hadamard, signs_dev, y_dev, stream);
}

bcu_status bcu_linear_forward(bcu_linear* l, const float* x_dev, int32_t T, float* y_dev, void* stream) {
    if (!l) return BCU_ERR_ARG;
    cudaSetDevice(l->device);
    return linear_run(l, nullptr, x_dev, T, 0, nullptr, y_dev, stream);
}

bcu_status bcu_linear_gemm(bcu_linear* l, const float* x_dev, int32_t M, float* y_dev, void* stream) {
    if (!l || !x_dev || !y_dev || M < 1) return BCU_ERR_ARG;
    cudaSetDevice(l->device);
    cudaStream_t st = (cudaStream_t)stream;
    const size_t need = gemm_act_bytes(M, l->m.K, l->m.group);
    if (need > l->gbop_bytes || M > l->gex_n) {  // grow the activation tiles (outside any capture)
        if (cudaStreamSynchronize(st) != cudaSuccess) return BCU_ERR_CUDA;
        cudaFree(l->gbop);
        cudaFree(l->gex);
        l->gbop = nullptr;
        l->gex = nullptr;
        l->gbop_bytes = 0;
        l->gex_n = 0;
        if (cudaMalloc(&l->gbop, need) != cudaSuccess || cudaMalloc(&l->gex, (size_t)M * 4) != cudaSuccess)
            return BCU_ERR_OOM;
        l->gbop_bytes = need;
        l->gex_n = M;
    }
    if (gemm_run(l->gwt, l->gbias, l->m.O, l->m.K, l->m.group, x_dev, M, l->gbop, l->gex, y_dev, l->err, l->sms, st) !=
        cudaSuccess)
        return BCU_ERR_CUDA;
    return BCU_OK;
}

// Test hook (not in the ABI header): the GEMM's activation tiles and exponents for x [M][K] (device pointers; bop
// sized by the same rule as bcu_linear_gemm's scratch), so tests can check their layout byte for byte.
bcu_status bcu_gemm_prep_debug(bcu_linear* l, const float* x_dev, int32_t M, void* bop_dev, int32_t* ex_dev) {
    if (!l || !x_dev || !bop_dev || !ex_dev || M < 1) return BCU_ERR_ARG;
    cudaSetDevice(l->device);
    gemm_prep_only(x_dev, M, l->m.K, l->m.group, (uint8_t*)bop_dev, ex_dev, 0);
    return cudaDeviceSynchronize() == cudaSuccess ? BCU_OK : BCU_ERR_CUDA;
}

// Test hook (not in the ABI header): 1 = every CTA builds its own slice of the operand (the path taken when the
// grid cannot hold all CTAs at once), 0 = the default choice.
bcu_status bcu_linear_set_local_build(bcu_linear* l, int32_t on) {
    if (!l) return BCU_ERR_ARG;
    l->local_build = on != 0;
    return BCU_OK;
}

static int* static_error_word(int device);

bcu_status bcu_linear_sync(bcu_linear* l, void* stream) {
    if (!l) return BCU_ERR_ARG;
    cudaSetDevice(l->device);
    if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) return BCU_ERR_CUDA;
    int e = 0;
    if (cudaMemcpy(&e, l->err, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return BCU_ERR_CUDA;
    if (e) cudaMemset(l->err, 0, 4);
    // the error word of bcu_linear_rotate_forward_static (its static array), once that entry has run on this device
    if (int* se = static_error_word(l->device)) {
        int e2 = 0;
        if (cudaMemcpy(&e2, se, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return BCU_ERR_CUDA;
        if (e2) cudaMemset(se, 0, 4);
        e |= e2;
    }
    return e ? BCU_ERR_TIMEOUT : BCU_OK;
}

// ------------------------------------------------------------------------------------------ no-allocation variant
// bcu_linear_rotate_forward with its scratch in a static device array instead of the handle's cudaMalloc'd buffers,
// for callers that may not allocate device memory when they run the layer (a host whose device memory belongs to
// its own pool, or a decode loop that must not stall on the synchronisation a cudaMalloc/cudaFree can cause).
// Layout of the array: split-K partial sums (262144 floats, 1 MiB), then per-row-block counters (1024 words, so
// O <= 131072 rows), then the error word. All calls share it: the counters are cleared on the call's stream before
// its launch (the kernel's last CTA also leaves them at zero); the partial sums are written before they are read.
// The error word starts at zero with the module and is only ever OR-ed by a kernel that gave up a bounded wait, so
// a failure stays recorded across later calls until bcu_linear_sync reads and clears it. Calls that overlap on the
// GPU race on the array. The cached address belongs to the device's current primary context: after a
// cudaDeviceReset the module is loaded again and the address must be looked up again (bcu_static_scratch_forget).
constexpr size_t STATIC_PARTIAL_FLOATS = 262144;
constexpr int STATIC_COUNTERS = 1024;
constexpr size_t STATIC_SCRATCH_BYTES = STATIC_PARTIAL_FLOATS * 4 + STATIC_COUNTERS * 4 + 256;
static __device__ __align__(256) unsigned char g_static_scratch[STATIC_SCRATCH_BYTES];

// Device address of g_static_scratch, looked up once per device with that device current.
static std::mutex g_static_mu;
static void* g_static_ptr[64];

static bcu_status static_scratch(int device, unsigned char** out) {
    if (device < 0 || device >= 64) return BCU_ERR_ARG;
    std::lock_guard<std::mutex> lk(g_static_mu);
    if (!g_static_ptr[device]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess || !p) return BCU_ERR_CUDA;
        g_static_ptr[device] = p;
    }
    *out = (unsigned char*)g_static_ptr[device];
    return BCU_OK;
}

// The static entry's error word on `device`, or null when that entry has not run there yet.
static int* static_error_word(int device) {
    if (device < 0 || device >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(g_static_mu);
    unsigned char* p = (unsigned char*)g_static_ptr[device];
    return p ? (int*)(p + STATIC_PARTIAL_FLOATS * 4 + STATIC_COUNTERS * 4) : nullptr;
}

// Not in the ABI header. Drops the cached address of the static array on `device` (call after a cudaDeviceReset,
// which reloads the module), and test hook: with plant != 0, first records a timeout in that device's error word,
// as a kernel that gave up a wait would, so a test can check that bcu_linear_sync reports it.
bcu_status bcu_static_scratch_debug(int32_t device, int32_t plant) {
    if (plant) {
        int* e = static_error_word(device);
        if (!e) return BCU_ERR_STATE;
        int v = ERR_MBAR_TIMEOUT;
        if (cudaSetDevice(device) != cudaSuccess || cudaMemcpy(e, &v, 4, cudaMemcpyHostToDevice) != cudaSuccess)
            return BCU_ERR_CUDA;
        return BCU_OK;
    }
    if (device < 0 || device >= 64) return BCU_ERR_ARG;
    std::lock_guard<std::mutex> lk(g_static_mu);
    g_static_ptr[device] = nullptr;
    return BCU_OK;
}

bcu_status bcu_linear_rotate_forward_static(bcu_linear* l, const uint16_t* x_bf16_dev, int32_t T, int32_t hadamard,
                                            const float* signs_dev, float* y_dev, void* stream) {
    if (!l || !x_bf16_dev || !y_dev || T < 1 || T > VMAX) return BCU_ERR_ARG;
    if (hadamard && (hadamard != 512 && hadamard != 1024 && hadamard != 2048)) return BCU_ERR_ARG;
    if (hadamard && l->m.K % hadamard) return BCU_ERR_ARG;
    const TernaryMat mm = rotate_plan(l, hadamard);
    const int nrb = mm.O / 128;
    if (nrb > STATIC_COUNTERS) return BCU_ERR_TOO_LARGE;
    if (mm.nsplit > 1 && (size_t)mm.nsplit * T * mm.O > STATIC_PARTIAL_FLOATS) return BCU_ERR_TOO_LARGE;
    if (cudaSetDevice(l->device) != cudaSuccess) return BCU_ERR_CUDA;
    unsigned char* scratch = nullptr;
    bcu_status s = static_scratch(l->device, &scratch);
    if (s != BCU_OK) return s;
    cudaStream_t st = (cudaStream_t)stream;
    unsigned* counters = (unsigned*)(scratch + STATIC_PARTIAL_FLOATS * 4);
    int* err = (int*)(scratch + STATIC_PARTIAL_FLOATS * 4 + STATIC_COUNTERS * 4);
    if (cudaMemsetAsync(counters, 0, (size_t)nrb * 4, st) != cudaSuccess) return BCU_ERR_CUDA;
    ActSrc src;
    src.mode = ACT_EXT;
    src.xb = x_bf16_dev;
    src.signs = signs_dev;
    src.HB = hadamard;
    GemvOut o;
    o.out = y_dev;
    o.partial = (float*)scratch;
    o.counters = counters;
    o.err = err;
    launch_ternary_gemv(mm, src, T, o, nullptr, st);
    return cudaGetLastError() == cudaSuccess ? BCU_OK : BCU_ERR_CUDA;
}

bcu_status bcu_gdn_verify(const float* q, const float* k, const float* v, const float* a_in, const float* b_in,
                          const float* a_log, const float* dt_bias, float* state, float* y, int32_t T, int32_t NK,
                          int32_t NV, int32_t n, void* stream) {
    if (!q || !k || !v || !a_in || !b_in || !a_log || !dt_bias || !state || !y) return BCU_ERR_ARG;
    if (T < 1 || NK < 1 || NV < 1 || NV % NK || n < 0 || n > T) return BCU_ERR_ARG;
    launch_gdn_verify(q, k, v, a_in, b_in, a_log, dt_bias, state, y, T, NK, NV, n, (cudaStream_t)stream);
    return cudaGetLastError() == cudaSuccess ? BCU_OK : BCU_ERR_CUDA;
}

bcu_status bcu_gdn_prefill_workspace(int32_t T, int32_t NV, uint64_t* bytes) {
    if (T < 1 || NV < 1 || !bytes) return BCU_ERR_ARG;
    *bytes = gdn_chunk_workspace_bytes(T, NV);
    return BCU_OK;
}

bcu_status bcu_gdn_prefill(const float* q, const float* k, const float* v, const float* a_in, const float* b_in,
                           const float* a_log, const float* dt_bias, float* state, float* y, int32_t T, int32_t NK,
                           int32_t NV, void* workspace, void* stream) {
    if (!q || !k || !v || !a_in || !b_in || !a_log || !dt_bias || !state || !y || !workspace) return BCU_ERR_ARG;
    if (T < 1 || NK < 1 || NV < 1 || NV % NK) return BCU_ERR_ARG;
    launch_gdn_chunked(q, k, v, a_in, b_in, a_log, dt_bias, state, y, T, NK, NV, (float*)workspace,
                       (cudaStream_t)stream);
    return cudaGetLastError() == cudaSuccess ? BCU_OK : BCU_ERR_CUDA;
}

}  // extern "C"
