// prefix.cpp — the saved prefix-cache file (runtime/mod.rs:213-232 and 494-578): its identity, its file name, the
// writer (temporary file then rename, the newest PREFIX_SLOTS files kept) and the reader (exact header match, exact
// size). File layout, all integers little-endian:
//   identity = "BNSPFX01" | u64 words [kernels, adapter, exe size, exe mtime ns, weights size, weights mtime ns,
//              hash(config bytes), n_gdn, n_attn, hidden, kv_width, conv_dim] | device name bytes
//   | ids u32[n] | len u64 (= n) | pos i64 (= len: text only) | state parts gdn, conv, K, V (bcu_state_parts order)
// The file name is "{h:016x}.prefix" with h = hash(hash(FNV, identity), ids bytes).
#include <dirent.h>
#include <errno.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "model.h"

using bcu::fail;

#ifndef BCU_KERNEL_HASH
#error "BCU_KERNEL_HASH (the hash of the CUDA sources and flags) is set by the Makefile"
#endif

namespace {

constexpr int PREFIX_SLOTS = 3;                // runtime/mod.rs:213
constexpr char PREFIX_MAGIC[8] = {'B', 'N', 'S', 'P', 'F', 'X', '0', '1'};  // runtime/mod.rs:215
constexpr uint64_t FNV = 0xcbf29ce484222325ull;  // runtime/mod.rs:216
constexpr uint64_t FNV_PRIME = 0x100000001b3ull;

void put_u64(std::vector<uint8_t>& v, uint64_t x) {
    for (int i = 0; i < 8; i++) v.push_back((uint8_t)(x >> (8 * i)));
}
uint64_t get_u64(const uint8_t* p) {
    uint64_t x = 0;
    for (int i = 7; i >= 0; i--) x = (x << 8) | p[i];
    return x;
}
void put_ids(std::vector<uint8_t>& v, const uint32_t* ids, int n) {
    for (int i = 0; i < n; i++)
        for (int b = 0; b < 4; b++) v.push_back((uint8_t)(ids[i] >> (8 * b)));
}

// std::fs::metadata len + modified() as nanoseconds since the epoch (runtime/mod.rs:495-499).
bool stamp(const char* path, uint64_t w[2]) {
    struct stat sb;
    if (!path || stat(path, &sb) != 0) return false;
    w[0] = (uint64_t)sb.st_size;
    w[1] = (uint64_t)sb.st_mtim.tv_sec * 1000000000ull + (uint64_t)sb.st_mtim.tv_nsec;
    return true;
}

bool read_all(const char* path, std::vector<uint8_t>& out) {
    FILE* f = path ? fopen(path, "rb") : nullptr;
    if (!f) return false;
    out.clear();
    uint8_t buf[1 << 16];
    size_t r;
    while ((r = fread(buf, 1, sizeof buf, f)) > 0) out.insert(out.end(), buf, buf + r);
    bool ok = !ferror(f);
    fclose(f);
    return ok;
}

std::string file_name(const char* dir, const uint8_t* identity, uint64_t idlen, const uint32_t* ids, int n) {
    std::vector<uint8_t> b;
    put_ids(b, ids, n);
    const uint64_t h = bcu_hash_bytes(bcu_hash_bytes(FNV, identity, idlen), b.data(), b.size());
    char name[32];
    snprintf(name, sizeof name, "%016llx", (unsigned long long)h);
    std::string d(dir);
    if (!d.empty() && d.back() != '/') d += '/';
    return d + name;  // + ".prefix" or ".tmp"
}

// std::fs::create_dir_all
bool make_dirs(const std::string& dir) {
    if (dir.empty()) return true;
    std::string cur;
    size_t i = 0;
    while (i <= dir.size()) {
        size_t j = dir.find('/', i);
        if (j == std::string::npos) j = dir.size();
        cur = dir.substr(0, j);
        if (!cur.empty() && mkdir(cur.c_str(), 0777) != 0 && errno != EEXIST) return false;
        i = j + 1;
    }
    struct stat sb;
    return stat(dir.c_str(), &sb) == 0 && S_ISDIR(sb.st_mode);
}

// Writes `data` as {base}.tmp, renames it to {base}.prefix, then keeps the newest PREFIX_SLOTS ".prefix" files of
// `dir` (runtime/mod.rs:562-577). False when the file could not be written (the temporary file is removed).
bool write_and_prune(const std::string& dir, const std::string& base, const std::vector<uint8_t>& data) {
    const std::string tmp = base + ".tmp", path = base + ".prefix";
    bool ok = make_dirs(dir);
    if (ok) {
        FILE* f = fopen(tmp.c_str(), "wb");
        ok = f && fwrite(data.data(), 1, data.size(), f) == data.size();
        if (f && fclose(f) != 0) ok = false;
        if (ok) ok = rename(tmp.c_str(), path.c_str()) == 0;
        if (!ok) unlink(tmp.c_str());
    }
    if (!ok) return false;
    DIR* d = opendir(dir.c_str());
    if (!d) return true;
    struct Entry {
        uint64_t mtime;
        std::string path;
    };
    std::vector<Entry> files;
    std::string pre = dir;
    if (!pre.empty() && pre.back() != '/') pre += '/';
    while (struct dirent* e = readdir(d)) {
        const size_t L = strlen(e->d_name);
        if (L < 7 || strcmp(e->d_name + L - 7, ".prefix") != 0) continue;
        uint64_t w[2];
        const std::string p = pre + e->d_name;
        if (stamp(p.c_str(), w)) files.push_back({w[1], p});
    }
    closedir(d);
    std::stable_sort(files.begin(), files.end(), [](const Entry& a, const Entry& b) { return a.mtime > b.mtime; });
    for (size_t i = PREFIX_SLOTS; i < files.size(); i++) unlink(files[i].path.c_str());
    return true;
}

std::mutex g_saves_mu;
std::vector<std::thread> g_saves;

// Opens {dir}/{name}.prefix and checks identity, ids, len and pos against the caller's; returns the open file
// positioned at the first state part, or null when there is no usable file.
FILE* open_checked(const char* dir, const uint8_t* identity, uint64_t idlen, const uint32_t* ids, int n) {
    const std::string path = file_name(dir, identity, idlen, ids, n) + ".prefix";
    FILE* f = fopen(path.c_str(), "rb");
    if (!f) return nullptr;
    std::vector<uint8_t> want(identity, identity + idlen);
    put_ids(want, ids, n);
    std::vector<uint8_t> head(want.size() + 16);
    if (fread(head.data(), 1, head.size(), f) != head.size() || memcmp(head.data(), want.data(), want.size()) != 0) {
        fclose(f);
        return nullptr;
    }
    const uint64_t len = get_u64(head.data() + want.size());
    const int64_t pos = (int64_t)get_u64(head.data() + want.size() + 8);
    // pos != len only after an image (mrope positions), which a text-only runtime cannot hold
    if (len != (uint64_t)n || pos != (int64_t)n) {
        fclose(f);
        return nullptr;
    }
    return f;
}

}  // namespace

extern "C" {

uint64_t bcu_hash_bytes(uint64_t h, const void* data, uint64_t n) {
    const uint8_t* b = (const uint8_t*)data;
    uint64_t i = 0;
    for (; i + 8 <= n; i += 8) h = (h ^ get_u64(b + i)) * FNV_PRIME;
    for (; i < n; i++) h = (h ^ b[i]) * FNV_PRIME;
    return h ^ n;
}

uint64_t bcu_kernel_hash(void) { return (uint64_t)BCU_KERNEL_HASH; }

bcu_status bcu_prefix_path(const char* dir, const uint8_t* identity, uint64_t identity_len, const uint32_t* ids,
                           int32_t n, char* out, uint64_t out_len) {
    if (!dir || !identity || (!ids && n) || n < 0 || !out) return BCU_ERR_ARG;
    const std::string p = file_name(dir, identity, identity_len, ids, n) + ".prefix";
    if (p.size() + 1 > out_len) return BCU_ERR_TOO_LARGE;
    memcpy(out, p.c_str(), p.size() + 1);
    return BCU_OK;
}

bcu_status bcu_prefix_identity(const bcu_model* m, uint64_t adapter, const char* exe_path, const char* weights_path,
                               const char* config_path, uint8_t* out, uint64_t cap, uint64_t* len) {
    if (!m || !weights_path || !config_path || !len) return BCU_ERR_ARG;
    uint64_t exe[2], wts[2];
    std::vector<uint8_t> cfg;
    if (!stamp(exe_path ? exe_path : "/proc/self/exe", exe) || !stamp(weights_path, wts) ||
        !read_all(config_path, cfg))
        return BCU_ERR_NOT_FOUND;
    char name[256];
    bcu_status s = bcu_device_name(m, name, sizeof name);
    if (s != BCU_OK) return s;
    std::vector<uint8_t> id(PREFIX_MAGIC, PREFIX_MAGIC + 8);
    const uint64_t words[] = {bcu_kernel_hash(), adapter, exe[0], exe[1], wts[0], wts[1],
                              bcu_hash_bytes(FNV, cfg.data(), cfg.size()), (uint64_t)m->n_gdn, (uint64_t)m->n_attn,
                              (uint64_t)m->c.hidden, (uint64_t)m->kvw, (uint64_t)m->C};
    for (uint64_t w : words) put_u64(id, w);
    id.insert(id.end(), name, name + strlen(name));
    *len = id.size();
    if (!out) return BCU_OK;  // size query
    if (cap < id.size()) return BCU_ERR_TOO_LARGE;
    memcpy(out, id.data(), id.size());
    return BCU_OK;
}

bcu_status bcu_prefix_file_write(const char* dir, const uint8_t* identity, uint64_t identity_len, const uint32_t* ids,
                                 int32_t n, const void* const parts[4], const uint64_t sizes[4]) {
    if (!dir || !identity || (!ids && n) || n < 0 || !parts || !sizes) return BCU_ERR_ARG;
    std::vector<uint8_t> data(identity, identity + identity_len);
    put_ids(data, ids, n);
    put_u64(data, (uint64_t)n);
    put_u64(data, (uint64_t)(int64_t)n);
    for (int i = 0; i < 4; i++) {
        if (!parts[i] && sizes[i]) return BCU_ERR_ARG;
        const uint8_t* p = (const uint8_t*)parts[i];
        data.insert(data.end(), p, p + sizes[i]);
    }
    return write_and_prune(dir, file_name(dir, identity, identity_len, ids, n), data) ? BCU_OK : BCU_ERR_IO;
}

bcu_status bcu_prefix_file_read(const char* dir, const uint8_t* identity, uint64_t identity_len, const uint32_t* ids,
                                int32_t n, void* const parts[4], const uint64_t sizes[4], int32_t* found) {
    if (!dir || !identity || (!ids && n) || n < 0 || !parts || !sizes || !found) return BCU_ERR_ARG;
    *found = 0;
    FILE* f = open_checked(dir, identity, identity_len, ids, n);
    if (!f) return BCU_OK;
    bool ok = true;
    for (int i = 0; i < 4 && ok; i++) ok = fread(parts[i], 1, sizes[i], f) == sizes[i];
    uint8_t extra;
    if (ok && fread(&extra, 1, 1, f) != 0) ok = false;  // trailing bytes: not this layout
    fclose(f);
    *found = ok ? 1 : 0;
    return BCU_OK;
}

bcu_status bcu_prefix_save(bcu_model* m, const bcu_state* s, const char* dir, const uint8_t* identity,
                           uint64_t identity_len, const uint32_t* ids, int32_t n, int32_t background) {
    if (!m || !s || !dir || !identity || (!ids && n) || n < 0) return fail(m, BCU_ERR_ARG, "bad prefix save");
    uint64_t sizes[4];
    int32_t len;
    bcu_status st = bcu_state_parts(m, s, sizes, &len);
    if (st != BCU_OK) return st;
    if (len != n) return fail(m, BCU_ERR_ARG, "snapshot length differs from the prefix ids");
    // the device parts are read here, on the caller's thread (runtime/mod.rs:557-560); only the file IO moves
    std::vector<uint8_t> data(identity, identity + identity_len);
    put_ids(data, ids, n);
    put_u64(data, (uint64_t)n);
    put_u64(data, (uint64_t)(int64_t)n);
    for (int i = 0; i < 4; i++) {
        const size_t at = data.size();
        data.resize(at + sizes[i]);
        if (sizes[i] && (st = bcu_state_read(m, s, i, data.data() + at, sizes[i])) != BCU_OK)
            return fail(m, st, "reading a snapshot part failed");
    }
    const std::string d(dir), base = file_name(dir, identity, identity_len, ids, n);
    if (!background) return write_and_prune(d, base, data) ? BCU_OK : fail(m, BCU_ERR_IO, "cannot write " + base);
    std::lock_guard<std::mutex> g(g_saves_mu);
    g_saves.emplace_back([d, base, data = std::move(data)] { write_and_prune(d, base, data); });
    return BCU_OK;
}

bcu_status bcu_prefix_wait_saves(void) {
    std::vector<std::thread> ts;
    {
        std::lock_guard<std::mutex> g(g_saves_mu);
        ts.swap(g_saves);
    }
    for (auto& t : ts) t.join();
    return BCU_OK;
}

bcu_status bcu_prefix_load(bcu_model* m, const char* dir, const uint8_t* identity, uint64_t identity_len,
                           const uint32_t* ids, int32_t n, bcu_state** out) {
    if (!m || !dir || !identity || (!ids && n) || n < 0 || !out) return fail(m, BCU_ERR_ARG, "bad prefix load");
    *out = nullptr;
    if (n > m->c.ctx) return BCU_OK;
    FILE* f = open_checked(dir, identity, identity_len, ids, n);
    if (!f) return BCU_OK;
    bcu_state* s = nullptr;
    bcu_status st = bcu_state_new(m, n, &s);
    if (st != BCU_OK) {
        fclose(f);
        return st;
    }
    uint64_t sizes[4];
    bcu_state_parts(m, s, sizes, nullptr);
    std::vector<uint8_t> part;
    bool ok = true;
    for (int i = 0; i < 4 && ok; i++) {
        part.resize(sizes[i]);
        ok = fread(part.data(), 1, sizes[i], f) == sizes[i];
        if (ok && sizes[i] && (st = bcu_state_write(m, s, i, part.data(), sizes[i], n)) != BCU_OK) {
            fclose(f);
            bcu_state_free(s);
            return st;
        }
    }
    uint8_t extra;
    if (ok && fread(&extra, 1, 1, f) != 0) ok = false;
    fclose(f);
    if (!ok) {
        bcu_state_free(s);
        return BCU_OK;
    }
    *out = s;
    return BCU_OK;
}

}  // extern "C"
