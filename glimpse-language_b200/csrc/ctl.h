// ctl.h — the device control block of a model and the constants shared by host and device code.
#pragma once
#include <stdint.h>

namespace bcu {

// Device error codes written to Ctl::err (bitwise OR). A kernel that gives up a bounded wait sets a bit and returns;
// the host maps a non-zero value to BCU_ERR_TIMEOUT / BCU_ERR_CUDA.
enum : int { ERR_MBAR_TIMEOUT = 1, ERR_BAD_TOKEN = 2, ERR_CTX_FULL = 4, ERR_SPIN_TIMEOUT = 8 };

constexpr int VMAX = 16;   // largest pass (rows) the kernels take
constexpr int NSPLIT_ATTN = 16;  // key splits per (kv head, query row) in attention

// Device control block of one model. The host writes `in` (one small copy per pass); the kernels of a pass read it
// and the accept step at the end of the pass writes the rest.
struct CtlIn {
    int commit_all;    // 1: this pass commits every row (prefill, plain step); 0: verify (commits m + 1)
    int feed;          // 0: ids from the host; 1: ids[0] = bonus of the previous pass; 2: all ids from `planted`
    int keep_logits;   // write fp32 logits [T, vocab] (parity tests)
    int planted_base;  // feed 2: ids[t] = planted[off - planted_base + t]
    uint32_t ids[VMAX];  // this pass's input rows (ids[0] = last emitted token, then drafts)
};

struct Ctl {
    CtlIn in;
    int off;          // KV offset of this pass = committed tokens including the pending commit
    int replay_n;     // rows of the previous pass to commit (GDN replay, conv shift) at the start of this pass
    int parity;       // pending-buffer parity of this pass (the previous pass used parity ^ 1)
    int accepted;     // m of the last pass
    uint32_t bonus;   // pred[m] of the last pass
    int err;          // device error bits
    int planted_n;
    int pad0;
    const uint32_t* planted;
    uint32_t used[VMAX];  // ids the pass actually embedded (after feed)
    uint32_t pred[VMAX];  // argmax per row of the last pass
};

}  // namespace bcu
