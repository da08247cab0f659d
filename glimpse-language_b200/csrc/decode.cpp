// decode.cpp — the decode driver of the Bonsai runtime (runtime/mod.rs:73-209, 699-956) on top of the pass API:
// prompt-lookup drafting, the adaptive speculation policy, the verify/accept loop, and pipelined plain decoding.
// The accept length is computed on the device; a verify round returns 8 bytes (m and the bonus token) to the host.
//
// The tokenizer stays with the caller: draft_source's SOURCE_TAGS block and filler filtering (mod.rs:733-768) work on
// the token bytes given to bcu_set_vocab_bytes (and the filler ids of bcu_set_fillers), and normalize_draft
// (mod.rs:699-729) re-encodes changed words through the caller's bcu_encode_fn. Emitted tokens reach the caller as
// they land through bcu_emit_fn (the `emit` of decode_spec / decode_plain, mod.rs:683, 892, 941).
#include <algorithm>
#include <cctype>
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

// The reference's word tables (runtime/mod.rs:130-146), kept as they are: drafting decisions must match its own.
const char* const SOURCE_TAGS[2][2] = {{"<transcript>\n", "\n</transcript>"}, {"<text>\n", "\n</text>"}};
const char* const CAPITALIZED[18] = {"monday", "tuesday", "wednesday", "thursday", "friday",  "saturday",
                                     "sunday", "january", "february",  "march",    "april",   "june",
                                     "july",   "august",  "september", "october",  "november", "december"};
const char* const CONTRACTIONS[22][2] = {
    {"dont", "don't"},     {"doesnt", "doesn't"},   {"didnt", "didn't"},     {"isnt", "isn't"},
    {"wasnt", "wasn't"},   {"arent", "aren't"},     {"werent", "weren't"},   {"wont", "won't"},
    {"cant", "can't"},     {"couldnt", "couldn't"}, {"wouldnt", "wouldn't"}, {"shouldnt", "shouldn't"},
    {"havent", "haven't"}, {"hasnt", "hasn't"},     {"im", "I'm"},           {"ive", "I've"},
    {"youre", "you're"},   {"theyre", "they're"},   {"thats", "that's"},     {"whats", "what's"},
    {"theres", "there's"}, {"lets", "let's"}};
const char* const FILLERS[12] = {" um", " uh", " Um", " Uh", " umm", " uhm", " erm", " hmm", "um", "uh", "Um", "Uh"};

// The vocabulary as the drafting code sees it: token bytes (bcu_set_vocab_bytes), filler ids, the encoder.
struct Vocab {
    const std::vector<std::string>* bytes = nullptr;
    const std::vector<uint32_t>* fillers = nullptr;
    bcu_encode_fn encode = nullptr;
    void* encode_user = nullptr;
    const std::string& tb(uint32_t id) const {
        static const std::string empty;
        return bytes && id < bytes->size() ? (*bytes)[id] : empty;
    }
};

bool ascii_ws(uint8_t c) { return c == ' ' || c == '\t' || c == '\n' || c == 0x0c || c == '\r'; }

// trim_ascii_end().last() is one of . ? ! (mod.rs:702, 724)
bool ends_sentence(const std::string& w) {
    size_t e = w.size();
    while (e > 0 && ascii_ws((uint8_t)w[e - 1])) e--;
    return e > 0 && (w[e - 1] == '.' || w[e - 1] == '?' || w[e - 1] == '!');
}

// Model::normalize_draft (mod.rs:699-729): per word of the draft (a token, plus the tokens after it that start with
// a letter or an apostrophe or are empty), a lowercase " word" becomes its contraction, or gets a capital when it is
// " i", follows a sentence end or is a CAPITALIZED word; changed words are re-encoded (the caller's encoder; a failed
// encoding keeps the word's tokens), and the draft keeps at most its length. No encoder: the draft is unchanged.
void normalize_draft(const Vocab& vb, std::vector<uint32_t>& draft, uint32_t last) {
    if (!vb.encode || !vb.bytes || vb.bytes->empty()) return;
    const size_t k = draft.size();
    std::vector<uint32_t> out;
    bool prev_end = ends_sentence(vb.tb(last));
    size_t i = 0;
    while (i < draft.size() && out.size() < k) {
        size_t j = i + 1;
        while (j < draft.size()) {
            const std::string& b = vb.tb(draft[j]);
            if (!b.empty() && !(std::isalpha((uint8_t)b[0]) && (uint8_t)b[0] < 128) && b[0] != '\'') break;
            j++;
        }
        std::string w;
        for (size_t q = i; q < j; q++) w += vb.tb(draft[q]);
        std::string v = w;
        bool lower = v.size() > 1 && v[0] == ' ';
        for (size_t q = 1; q < v.size() && lower; q++) lower = v[q] >= 'a' && v[q] <= 'z';
        if (lower) {
            const std::string bare = w.substr(1);
            const char* to = nullptr;
            for (auto& c : CONTRACTIONS)
                if (bare == c[0]) { to = c[1]; break; }
            bool cap = bare == "i" || prev_end;
            for (const char* c : CAPITALIZED) cap = cap || bare == c;
            if (to) v = std::string(" ") + to;
            else if (cap) v[1] = (char)(v[1] - 'a' + 'A');
        }
        bool done = false;
        if (v != w) {
            std::vector<uint32_t> ids(v.size() + 16);
            int32_t n = vb.encode(vb.encode_user, (const uint8_t*)v.data(), (int32_t)v.size(), ids.data(),
                                  (int32_t)ids.size());
            if (n >= 0 && n <= (int32_t)ids.size()) {
                out.insert(out.end(), ids.begin(), ids.begin() + n);
                done = true;
            }
        }
        if (!done) out.insert(out.end(), draft.begin() + i, draft.begin() + j);
        prev_end = ends_sentence(w);
        i = j;
    }
    if (out.size() > k) out.resize(k);
    draft = out;
}

struct Keys {
    const std::vector<uint64_t>* table;
    uint64_t operator()(uint32_t id) const {
        if (table && !table->empty()) return id < table->size() ? (*table)[id] : 0;
        // no vocabulary bytes: every id is its own word
        uint64_t h = (0xcbf29ce484222325ull ^ (uint64_t)id) * 0x100000001b3ull;
        return (h & ~3ull) | 1;
    }
};

// Model::draft_source (mod.rs:733-768): the user tokens inside the first SOURCE_TAGS block of the turn's bytes (all
// of them when there is none, or when no token bytes are known), fillers removed, with the keys of its word tokens.
Source draft_source(const uint32_t* user, int n, const Keys& keys, const Vocab& vb) {
    Source s;
    size_t lo = 0, hi = 0;
    std::vector<size_t> ends(n);
    const bool have = vb.bytes && !vb.bytes->empty();
    if (have) {
        std::string text;
        for (int i = 0; i < n; i++) {
            text += vb.tb(user[i]);
            ends[i] = text.size();
        }
        hi = text.size();
        for (auto& tag : SOURCE_TAGS) {
            size_t a = text.find(tag[0]);
            if (a == std::string::npos) continue;
            a += std::strlen(tag[0]);
            size_t b = text.find(tag[1], a);
            if (b == std::string::npos) continue;
            lo = a;
            hi = b;
            break;
        }
    }
    for (int i = 0; i < n; i++) {
        const uint32_t id = user[i];
        if (have) {
            const size_t len = vb.tb(id).size();
            if (!(ends[i] > lo && ends[i] - len >= lo && ends[i] <= hi)) continue;
        }
        if (vb.fillers && std::find(vb.fillers->begin(), vb.fillers->end(), id) != vb.fillers->end()) continue;
        s.ids.push_back(id);
    }
    for (int i = 0; i < (int)s.ids.size(); i++) {
        uint64_t k = keys(s.ids[i]);
        if (k & 1) s.words.push_back({k, i});
    }
    return s;
}

// The filler ids: the caller's (bcu_set_fillers), else every FILLERS string that is exactly one token's bytes (the
// reference keeps the fillers whose encoding is a single id, mod.rs:750-756).
std::vector<uint32_t> default_fillers(const std::vector<std::string>& bytes) {
    std::vector<uint32_t> f;
    for (const char* w : FILLERS)
        for (size_t id = 0; id < bytes.size(); id++)
            if (bytes[id] == w) {
                f.push_back((uint32_t)id);
                break;
            }
    return f;
}

Vocab vocab_of(bcu_model* m) {
    Vocab v;
    v.bytes = &m->vocab_bytes;
    v.fillers = &m->fillers;
    v.encode = m->encode_fn;
    v.encode_user = m->encode_user;
    return v;
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
    bool push(uint32_t id) {  // false: stop (EOS or cap); an accepted token is emitted as it lands
        if (is_eos(id, eos, n_eos) || n >= max_tokens) return false;
        out[n++] = id;
        if (m->emit_fn) m->emit_fn(m->emit_user, id);
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
    m->vocab_bytes.clear();
    if (!m->fillers_given) m->fillers.clear();
    if (!bytes || !offsets || vocab <= 0) return BCU_OK;
    m->keys.resize(vocab);
    m->vocab_bytes.resize(vocab);
    for (int i = 0; i < vocab; i++) {
        m->keys[i] = token_key(bytes + offsets[i], offsets[i + 1] - offsets[i]);
        m->vocab_bytes[i].assign((const char*)bytes + offsets[i], offsets[i + 1] - offsets[i]);
    }
    if (!m->fillers_given) m->fillers = default_fillers(m->vocab_bytes);
    return BCU_OK;
}

bcu_status bcu_set_fillers(bcu_model* m, const uint32_t* ids, int32_t n) {
    if (!m || n < 0 || (n && !ids)) return BCU_ERR_ARG;
    m->fillers.assign(ids, ids + n);
    m->fillers_given = n > 0;
    if (!n) m->fillers = default_fillers(m->vocab_bytes);
    return BCU_OK;
}

bcu_status bcu_set_encoder(bcu_model* m, bcu_encode_fn fn, void* user) {
    if (!m) return BCU_ERR_ARG;
    m->encode_fn = fn;
    m->encode_user = user;
    return BCU_OK;
}

bcu_status bcu_set_emit(bcu_model* m, bcu_emit_fn fn, void* user) {
    if (!m) return BCU_ERR_ARG;
    m->emit_fn = fn;
    m->emit_user = user;
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
    Source s = draft_source(src, n_src, k, Vocab());
    std::vector<uint32_t> sq(seq, seq + n_seq);
    int dp;
    std::vector<uint32_t> d = lookup(s, sq, k, ngram_max, ngram_min, draft_max, limit, cursor, &dp);
    for (size_t i = 0; i < d.size(); i++) out[i] = d[i];
    *dpos = dp;
    return (int32_t)d.size();
}

// draft_source and normalize_draft on a vocabulary given as one byte string (offsets: vocab + 1 entries), for tests
// of the host logic without a device. fillers: n_fillers ids, or n_fillers < 0 for the default derived from the bytes.
static std::vector<std::string> vocab_strings(const uint8_t* bytes, const uint64_t* offsets, int32_t vocab) {
    std::vector<std::string> v(vocab > 0 ? vocab : 0);
    for (int i = 0; i < vocab; i++) v[i].assign((const char*)bytes + offsets[i], offsets[i + 1] - offsets[i]);
    return v;
}

int32_t bcu_draft_source_host(const uint32_t* user, int32_t n, const uint8_t* bytes, const uint64_t* offsets,
                              int32_t vocab, const uint32_t* fillers, int32_t n_fillers, uint32_t* out) {
    std::vector<std::string> vb = vocab_strings(bytes, offsets, vocab);
    std::vector<uint64_t> keys(vb.size());
    for (size_t i = 0; i < vb.size(); i++) keys[i] = token_key((const uint8_t*)vb[i].data(), vb[i].size());
    std::vector<uint32_t> fl = n_fillers < 0 ? default_fillers(vb) : std::vector<uint32_t>(fillers, fillers + n_fillers);
    Vocab v;
    v.bytes = &vb;
    v.fillers = &fl;
    Keys k{&keys};
    Source s = draft_source(user, n, k, v);
    for (size_t i = 0; i < s.ids.size(); i++) out[i] = s.ids[i];
    return (int32_t)s.ids.size();
}

int32_t bcu_normalize_draft_host(uint32_t* draft, int32_t n, uint32_t last, const uint8_t* bytes,
                                 const uint64_t* offsets, int32_t vocab, bcu_encode_fn fn, void* user) {
    std::vector<std::string> vb = vocab_strings(bytes, offsets, vocab);
    Vocab v;
    v.bytes = &vb;
    v.encode = fn;
    v.encode_user = user;
    std::vector<uint32_t> d(draft, draft + n);
    normalize_draft(v, d, last);
    for (size_t i = 0; i < d.size(); i++) draft[i] = d[i];
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
    const Vocab vb = vocab_of(m);
    Source src = draft_source(user, n_user, keys, vb);
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
        if (!forced) normalize_draft(vb, draft, last);
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
