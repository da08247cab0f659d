// decode.cpp — the decode driver of the Bonsai runtime (runtime/mod.rs:73-209, 699-956) on top of the pass API:
// prompt-lookup drafting, the adaptive speculation policy, the verify/accept loop, and pipelined plain decoding.
// The accept length is computed on the device; a verify round returns 8 bytes (m and the bonus token) to the host.
//
// Left out, because they need the tokenizer (out of scope for a backend): normalize_draft (mod.rs:699-729, re-encodes
// changed words) and the filler / SOURCE_TAGS filtering of draft_source (mod.rs:733-768) — the draft source is the
// user turn as given.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "model.h"

using namespace bcu;

namespace {

const int BACK = 24;          // mod.rs:127
const double KEEP_GAIN = 1.05, ENTER_GAIN = 1.15;  // mod.rs:158-159
const int GIVE_UP_ROUNDS = 6;  // mod.rs:162

// token_key (mod.rs:73-81).
uint64_t token_key(const uint8_t* bytes, size_t n) {
    uint64_t nl = 0;
    for (size_t i = 0; i < n; i++)
        if (bytes[i] == '\n') nl = 2;
    if (n > 0 && bytes[0] == ' ') { bytes++; n--; }
    bool all = true;
    for (size_t i = 0; i < n && all; i++) {
        uint8_t c = bytes[i];
        bool punct = (c >= 33 && c <= 47) || (c >= 58 && c <= 64) || (c >= 91 && c <= 96) || (c >= 123 && c <= 126);
        bool ws = c == ' ' || c == '\t' || c == '\n' || c == '\r' || c == 0x0c;
        all = punct || ws;
    }
    if (all) return nl;
    uint64_t h = 0xcbf29ce484222325ull;
    for (size_t i = 0; i < n; i++) {
        uint8_t c = bytes[i];
        if (c >= 'A' && c <= 'Z') c = (uint8_t)(c + 32);
        h = (h ^ c) * 0x100000001b3ull;
    }
    return (h & ~3ull) | 1 | nl;
}

struct Source {
    std::vector<uint32_t> ids;
    std::vector<std::pair<uint64_t, int>> words;
};

struct Keys {
    const std::vector<uint64_t>* table;
    uint64_t operator()(uint32_t id) const {
        if (table && !table->empty()) return id < table->size() ? (*table)[id] : 0;
        // no vocabulary bytes: every id is its own word
        uint64_t h = (0xcbf29ce484222325ull ^ (uint64_t)id) * 0x100000001b3ull;
        return (h & ~3ull) | 1;
    }
};

Source draft_source(const uint32_t* user, int n, const Keys& keys) {
    Source s;
    s.ids.assign(user, user + n);
    for (int i = 0; i < n; i++) {
        uint64_t k = keys(user[i]);
        if (k & 1) s.words.push_back({k, i});
    }
    return s;
}

// lookup (mod.rs:87-124).
std::vector<uint32_t> lookup(const Source& src, const std::vector<uint32_t>& seq, const Keys& keys, int ngram_max,
                             int ngram_min, int draft_max, int limit, int cursor, int* dpos) {
    int k = std::min(std::min(draft_max, limit), VMAX - 1);
    *dpos = cursor;
    std::vector<uint32_t> out;
    if (k <= 0) return out;
    std::vector<uint64_t> pat;
    int taken = 0;
    for (int i = (int)seq.size() - 1; i >= 0 && taken < 4 * ngram_max; i--, taken++) {
        if ((int)pat.size() == ngram_max) break;
        uint64_t key = keys(seq[i]);
        if (key & 1) pat.push_back(key);
    }
    std::reverse(pat.begin(), pat.end());
    const auto& w = src.words;
    for (int n = std::min(ngram_max, (int)pat.size()); n >= std::max(ngram_min, 1); n--) {
        const uint64_t* p = pat.data() + pat.size() - n;
        int hit = -1;
        int lim = (int)w.size() - (n - 1);
        for (int i = 0; i < lim; i++) {
            bool eq = true;
            for (int q = 0; q < n && eq; q++) eq = w[i + q].first == p[q];
            if (!eq) continue;
            int j = w[i + n - 1].second + 1;
            if (j < (int)src.ids.size() && j + BACK >= cursor && (hit < 0 || j >= cursor)) hit = j;
            if (j >= cursor) break;
        }
        if (hit >= 0) {
            int e = std::min(hit + k, (int)src.ids.size());
            out.assign(src.ids.begin() + hit, src.ids.begin() + e);
            *dpos = hit;
            return out;
        }
    }
    return out;
}

// Policy (mod.rs:168-209).
struct Policy {
    const double* cost;
    int kmax;
    double acc = 0, rej = 0;
    double p() const { return (acc + 3.4) / (acc + rej + 3.4 + 0.6); }
    int choose(int limit, double min_gain) const {
        double pp = p(), best = 1.0;
        int bk = 0;
        for (int k = 1; k <= std::min(kmax, limit); k++) {
            double g = (1.0 - std::pow(pp, k + 1)) / (1.0 - pp) / cost[k];
            if (g > best && g > min_gain) { best = g; bk = k; }
        }
        return bk;
    }
    void update(int k, int m) {
        acc = acc * 0.85 + m;
        rej = rej * 0.85 + (m < k ? 1.0 : 0.0);
    }
};

uint64_t mix64(uint64_t x) {
    x += 0x9e3779b97f4a7c15ull;
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
    return x ^ (x >> 31);
}

// Verify-cost table on this GPU (the role of VERIFY_COST_*, gpu.rs:16-19): time of a pass of k+1 rows over a one-row
// pass, measured once with CUDA events.
bcu_status ensure_cost(bcu_model* m) {
    if (m->cost_ready) return BCU_OK;
    float base = 0;
    for (int k = 0; k <= 8 && k + 1 <= m->c.vmax; k++) {
        float ms;
        bcu_status s = bcu_time_pass(m, k + 1, 3, &ms);
        if (s != BCU_OK) return s;
        if (k == 0) base = ms;
        m->cost[k] = base > 0 ? ms / base : 1.0 + k;
    }
    for (int k = 1; k <= 8; k++)
        if (m->cost[k] <= 0) m->cost[k] = m->cost[k - 1];
    m->cost_ready = true;
    return BCU_OK;
}

bool is_eos(uint32_t id, const uint32_t* eos, int n) {
    for (int i = 0; i < n; i++)
        if (eos[i] == id) return true;
    return false;
}

struct Run {
    bcu_model* m;
    const uint32_t* eos;
    int n_eos;
    int max_tokens;
    uint32_t* out;
    int n = 0;
    bool push(uint32_t id) {  // false: stop (EOS or cap)
        if (is_eos(id, eos, n_eos) || n >= max_tokens) return false;
        out[n++] = id;
        return true;
    }
};

// decode_plain (mod.rs:901-956): one-row passes with the next input taken from the previous pass's bonus on the
// device, two passes in flight. stop(id) is called per emitted token; when it returns true the pass in flight is
// drained, its token emitted and returned through *resume. Returns false on EOS / cap.
template <class Stop>
bcu_status decode_plain(bcu_model* m, uint32_t feed, Run& r, Stop stop, bool* resumed, uint32_t* resume) {
    *resumed = false;
    if (r.n >= r.max_tokens) return BCU_OK;
    bcu_status s;
    uint32_t ids[1] = {feed};
    // Pass k reads its input id from the bonus of pass k-1 on the device (feed = 1), so pass k+1 is enqueued before
    // the host looks at pass k's token; each pass's token is copied to its own pinned ring slot (the 2-slot token ring
    // of model.rs:1000-1022).
    auto enqueue = [&](int k, bool first) -> bcu_status {
        bcu_status e = run_pass(m, first ? ids : nullptr, 1, 1, first ? 0 : 1, false);
        if (e != BCU_OK) return e;
        if (cudaMemcpyAsync(&m->h_ring[k & 1], &m->ctl->bonus, 4, cudaMemcpyDeviceToHost, m->st) != cudaSuccess ||
            cudaEventRecord(m->ev_ring[k & 1], m->st) != cudaSuccess)
            return fail(m, BCU_ERR_CUDA, "ring copy");
        return BCU_OK;
    };
    auto wait_tok = [&](int k, uint32_t* tok) -> bcu_status {
        auto t0 = std::chrono::steady_clock::now();
        for (;;) {
            cudaError_t e = cudaEventQuery(m->ev_ring[k & 1]);
            if (e == cudaSuccess) break;
            if (e != cudaErrorNotReady) return fail(m, BCU_ERR_CUDA, cudaGetErrorString(e));
            if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > 120.0)
                return fail(m, BCU_ERR_TIMEOUT, "plain decode step did not finish");
        }
        *tok = m->h_ring[k & 1];
        m->len += 1;
        return BCU_OK;
    };
    if ((s = enqueue(0, true)) != BCU_OK) return s;
    int k = 0;
    bool inflight_next = false;
    while (true) {
        // keep the next step queued while this one's token is examined
        inflight_next = r.n + 1 < r.max_tokens && !m->cancel && m->len + 2 <= m->c.ctx;
        if (inflight_next && (s = enqueue(k + 1, false)) != BCU_OK) return s;
        uint32_t tok = 0;
        if ((s = wait_tok(k, &tok)) != BCU_OK) return s;
        bool ok = r.push(tok);
        if (!ok || !inflight_next || m->cancel) {
            if (inflight_next) {  // drain the queued step
                uint32_t drop;
                if ((s = wait_tok(k + 1, &drop)) != BCU_OK) return s;
            }
            return m->cancel ? BCU_ERR_CANCELLED : BCU_OK;
        }
        if (stop(tok)) {
            uint32_t nt = 0;
            if ((s = wait_tok(k + 1, &nt)) != BCU_OK) return s;
            if (!r.push(nt)) return BCU_OK;
            *resumed = true;
            *resume = nt;
            return BCU_OK;
        }
        k++;
    }
}

}  // namespace

extern "C" {

bcu_status bcu_set_vocab_bytes(bcu_model* m, const uint8_t* bytes, const uint64_t* offsets, int32_t vocab) {
    if (!m) return BCU_ERR_ARG;
    m->keys.clear();
    if (!bytes || !offsets || vocab <= 0) return BCU_OK;
    m->keys.resize(vocab);
    for (int i = 0; i < vocab; i++) m->keys[i] = token_key(bytes + offsets[i], offsets[i + 1] - offsets[i]);
    return BCU_OK;
}

bcu_status bcu_cancel(bcu_model* m, int32_t flag) {
    if (!m) return BCU_ERR_ARG;
    m->cancel = flag;
    return BCU_OK;
}

// Host-logic exports for tests (no device work).
uint64_t bcu_token_key(const uint8_t* bytes, uint64_t n) { return token_key(bytes, n); }

int32_t bcu_lookup(const uint32_t* src, int32_t n_src, const uint32_t* seq, int32_t n_seq, const uint64_t* keys,
                   int32_t n_keys, int32_t ngram_max, int32_t ngram_min, int32_t draft_max, int32_t limit,
                   int32_t cursor, uint32_t* out, int32_t* dpos) {
    std::vector<uint64_t> table(keys, keys + n_keys);
    Keys k{&table};
    Source s = draft_source(src, n_src, k);
    std::vector<uint32_t> sq(seq, seq + n_seq);
    int dp;
    std::vector<uint32_t> d = lookup(s, sq, k, ngram_max, ngram_min, draft_max, limit, cursor, &dp);
    for (size_t i = 0; i < d.size(); i++) out[i] = d[i];
    *dpos = dp;
    return (int32_t)d.size();
}

int32_t bcu_policy_choose(double acc, double rej, const double* cost, int32_t kmax, int32_t limit, double min_gain) {
    Policy p{cost, std::min(kmax, 7)};
    p.acc = acc;
    p.rej = rej;
    return p.choose(limit, min_gain);
}

bcu_status bcu_decode(bcu_model* m, uint32_t first, const uint32_t* user, int32_t n_user, const bcu_spec* spec,
                      int32_t draft_mode, const uint32_t* planted, int32_t planted_n, uint64_t seed,
                      const uint32_t* eos, int32_t n_eos, int32_t max_tokens, uint32_t* out, int32_t* n_out,
                      bcu_stats* stats) {
    if (!m || !out || !n_out || max_tokens < 0) return BCU_ERR_ARG;
    if (cudaSetDevice(m->device) != cudaSuccess) return BCU_ERR_CUDA;
    auto t0 = std::chrono::steady_clock::now();
    bcu_stats st{};
    Run r{m, eos, n_eos, max_tokens, out};
    *n_out = 0;
    bcu_status s = BCU_OK;
    m->cancel = 0;
    auto finish = [&](bcu_status rs) {
        *n_out = r.n;
        st.gen_tokens = r.n;
        st.decode_s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (stats) *stats = st;
        return rs;
    };
    if (max_tokens == 0 || is_eos(first, eos, n_eos)) return finish(BCU_OK);
    r.push(first);
    bool resumed;
    uint32_t resume;
    if (!spec) {
        s = decode_plain(m, first, r, [](uint32_t) { return false; }, &resumed, &resume);
        return finish(s);
    }
    const bool forced = draft_mode == BCU_DRAFT_PLANTED || draft_mode == BCU_DRAFT_RANDOM;
    int draft_max = std::min(std::max(spec->draft_max, 0), m->c.vmax - 1);
    if (!forced && (s = ensure_cost(m)) != BCU_OK) return finish(s);
    static const double unit[9] = {1, 1, 1, 1, 1, 1, 1, 1, 1};
    Policy pol{forced ? unit : m->cost, std::min(draft_max, 7)};
    Keys keys{&m->keys};
    Source src = draft_source(user, n_user, keys);
    std::vector<uint32_t> seq(user, user + n_user);
    seq.push_back(first);
    int cursor = 0;
    std::pair<int, int> failed = {-1, 0};
    auto nl = [&](uint32_t id) { return (keys(id) & 2) != 0; };
    bool src_nl = false;
    for (uint32_t id : src.ids) src_nl |= nl(id);
    auto brk = [&](uint32_t id) { return nl(id) && !src_nl; };
    auto given_up = [&](std::pair<int, int> f, int j) { return f.first == j && f.second >= 2; };
    double got = 0, spent = 0;
    int rounds = 0;
    while (r.n < max_tokens) {
        if (m->cancel) return finish(BCU_ERR_CANCELLED);
        uint32_t last = seq.back();
        int left = max_tokens - r.n;
        if (!forced && rounds >= GIVE_UP_ROUNDS && got < KEEP_GAIN * spent) {
            s = decode_plain(m, last, r, [](uint32_t) { return false; }, &resumed, &resume);
            return finish(s);
        }
        std::vector<uint32_t> draft;
        int dpos = cursor;
        if (forced) {
            int k = std::min(draft_max, left - 1);
            for (int i = 0; i < k; i++) {
                if (draft_mode == BCU_DRAFT_PLANTED) {
                    int idx = r.n - 1 + i;  // output token r.n + i is planted[r.n - 1 + i]
                    if (!planted || idx >= planted_n) break;
                    draft.push_back(planted[idx]);
                } else {
                    draft.push_back((uint32_t)(mix64(seed ^ ((uint64_t)(r.n + i) << 20)) % (uint64_t)m->c.vocab));
                }
            }
        } else {
            int k = pol.choose(left - 1, KEEP_GAIN);
            draft = lookup(src, seq, keys, spec->ngram_max, spec->ngram_min, k, left - 1, cursor, &dpos);
            if (given_up(failed, dpos) || brk(last)) draft.clear();
        }
        if (draft.empty()) {
            if (forced) {  // nothing to draft (end of the planted stream): one plain step
                uint32_t next;
                if ((s = bcu_step(m, last, &next)) != BCU_OK) return finish(s);
                seq.push_back(next);
                if (!r.push(next)) return finish(BCU_OK);
                continue;
            }
            // plain decoding with shadow rounds (mod.rs:820-860)
            int next_start = (int)seq.size(), sh_pos = 0, sh_src = 0;
            std::vector<uint32_t> sh;
            auto stop = [&](uint32_t id) {
                seq.push_back(id);
                int j = (int)seq.size() - 1;
                if (!sh.empty() && j >= sh_pos) {
                    int i = j - sh_pos;
                    if (seq[j] != sh[i]) {
                        pol.update((int)sh.size(), i);
                        cursor = sh_src + i;
                        sh.clear();
                        next_start = j + 1;
                    } else if (i + 1 == (int)sh.size()) {
                        pol.update((int)sh.size(), (int)sh.size());
                        cursor = sh_src + (int)sh.size();
                        sh.clear();
                        next_start = j + 2;
                    }
                }
                if (sh.empty() && (int)seq.size() >= next_start) {
                    sh = lookup(src, seq, keys, spec->ngram_max, spec->ngram_min, draft_max, 1 << 30, cursor, &sh_src);
                    sh_pos = (int)seq.size();
                    next_start = (int)seq.size() + 1;
                }
                if (pol.choose(draft_max, ENTER_GAIN) > 0 && !brk(id)) {
                    int jj;
                    std::vector<uint32_t> d = lookup(src, seq, keys, spec->ngram_max, spec->ngram_min, draft_max,
                                                     1 << 30, cursor, &jj);
                    return !d.empty() && !given_up(failed, jj);
                }
                return false;
            };
            s = decode_plain(m, last, r, stop, &resumed, &resume);
            if (s != BCU_OK || !resumed) return finish(s);
            seq.push_back(resume);
            st.switches++;
            continue;
        }
        std::vector<uint32_t> ids;
        ids.push_back(last);
        ids.insert(ids.end(), draft.begin(), draft.end());
        int32_t mm;
        uint32_t bonus;
        if ((s = bcu_verify_accept(m, ids.data(), (int)ids.size(), &mm, &bonus)) != BCU_OK) return finish(s);
        int kd = (int)draft.size();
        pol.update(kd, mm);
        cursor = dpos + mm;
        if (mm == 0) failed = failed.first == dpos ? std::make_pair(dpos, failed.second + 1) : std::make_pair(dpos, 1 + (brk(bonus) ? 1 : 0));
        else failed = {-1, 0};
        got = got * 0.85 + (mm + 1);
        spent = spent * 0.85 + (forced ? 1.0 : m->cost[kd]);
        rounds++;
        st.verify_calls++;
        st.drafted += kd;
        st.accepted += mm;
        for (int i = 0; i <= mm; i++) {
            uint32_t id = i < mm ? draft[i] : bonus;
            if (!r.push(id)) return finish(BCU_OK);
            seq.push_back(id);
        }
    }
    return finish(BCU_OK);
}

}  // extern "C"
