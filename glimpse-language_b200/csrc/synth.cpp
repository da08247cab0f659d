// synth.cpp — seeded synthetic inputs for the graded random-init shapes (no checkpoints are available offline).
// Counter-based: element i of stream (seed, stream) depends only on (seed, stream, i), so tensors can be generated in
// parallel and re-generated identically on any host. Distributions use integer arithmetic plus one fp32 multiply-add:
// "normal" is Irwin-Hall of 12 uniform 16-bit draws (mean 0, variance 1, support +-6), uniform fp32/fp16 take 24
// random bits; fp16/bf16 conversions round to nearest even.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#include "../../include/bonsai_synth.h"

namespace {

inline uint64_t mix64(uint64_t x) {
    x += 0x9e3779b97f4a7c15ull;
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
    return x ^ (x >> 31);
}

inline uint64_t draw(uint64_t seed, uint64_t stream, uint64_t i) {
    return mix64(mix64(seed * 0xd1b54a32d192ed03ull ^ stream) ^ (i * 0x8cb92ba72f3d8dd7ull));
}

inline float unif01(uint64_t u) { return (float)(u >> 40) * (1.0f / 16777216.0f); }

inline float normal(uint64_t seed, uint64_t stream, uint64_t i) {
    int64_t s = 0;
    for (int j = 0; j < 3; j++) {
        uint64_t u = draw(seed, stream, i * 3 + j);
        s += (int64_t)(u & 0xffff) + (int64_t)((u >> 16) & 0xffff) + (int64_t)((u >> 32) & 0xffff) + (int64_t)(u >> 48);
    }
    return (float)(s - 393210) * (1.0f / 65536.0f);
}

uint16_t f32_to_f16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    uint32_t s = (u >> 16) & 0x8000, e = (u >> 23) & 255, m = u & 0x7fffff;
    if (e == 255) return (uint16_t)(s | 0x7c00 | (m ? 0x200 : 0));
    int ex = (int)e - 127 + 15;
    if (ex >= 31) return (uint16_t)(s | 0x7c00);
    if (ex <= 0) {
        if (ex < -10) return (uint16_t)s;
        m |= 0x800000;
        int shift = 14 - ex;
        uint32_t q = m >> shift, rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1))) q++;
        return (uint16_t)(s | q);
    }
    uint32_t q = (uint32_t)ex << 10 | m >> 13, rem = m & 0x1fff;
    if (rem > 0x1000 || (rem == 0x1000 && (q & 1))) q++;
    return (uint16_t)(s | q);
}

uint16_t f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffff) > 0x7f800000) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7fff + ((u >> 16) & 1);
    return (uint16_t)(u >> 16);
}

}  // namespace

extern "C" {

bcu_status bcu_synth_fill(int32_t kind, uint64_t seed, uint64_t stream, double a, double b, void* out, uint64_t n) {
    if (!out && n) return BCU_ERR_ARG;
    const float fa = (float)a, fb = (float)b, w = (float)(b - a);
    switch (kind) {
        case 0: {
            float* o = (float*)out;
#pragma omp parallel for schedule(static)
            for (int64_t i = 0; i < (int64_t)n; i++) o[i] = fa + w * unif01(draw(seed, stream, i));
            return BCU_OK;
        }
        case 1: {
            float* o = (float*)out;
#pragma omp parallel for schedule(static)
            for (int64_t i = 0; i < (int64_t)n; i++) o[i] = fa + fb * normal(seed, stream, i);
            return BCU_OK;
        }
        case 2: {
            uint16_t* o = (uint16_t*)out;
#pragma omp parallel for schedule(static)
            for (int64_t i = 0; i < (int64_t)n; i++) o[i] = f32_to_bf16(fa + fb * normal(seed, stream, i));
            return BCU_OK;
        }
        case 3: {  // ternary codes {0,1,2}, 16 per word, code e at bits 2e
            uint32_t* o = (uint32_t*)out;
#pragma omp parallel for schedule(static)
            for (int64_t i = 0; i < (int64_t)n; i++) {
                uint32_t wd = 0;
                for (int q = 0; q < 4; q++) {
                    uint64_t u = draw(seed, stream, (uint64_t)i * 4 + q);
                    for (int j = 0; j < 4; j++) {
                        uint32_t c = (uint32_t)((((u >> (16 * j)) & 0xffff) * 3) >> 16);
                        wd |= c << (2 * (q * 4 + j));
                    }
                }
                o[i] = wd;
            }
            return BCU_OK;
        }
        case 4:
        case 6: {
            uint16_t* o = (uint16_t*)out;
#pragma omp parallel for schedule(static)
            for (int64_t i = 0; i < (int64_t)n; i++) {
                uint16_t h = f32_to_f16(fa + w * unif01(draw(seed, stream, i)));
                o[i] = kind == 6 ? (uint16_t)(h ^ 0x8000) : h;
            }
            return BCU_OK;
        }
        case 5: {
            float* o = (float*)out;
#pragma omp parallel for schedule(static)
            for (int64_t i = 0; i < (int64_t)n; i++) o[i] = (draw(seed, stream, i) >> 63) ? -1.0f : 1.0f;
            return BCU_OK;
        }
    }
    return BCU_ERR_ARG;
}

bcu_status bcu_synth_zipf(uint64_t seed, double s, int32_t vocab, uint32_t* out, int32_t n) {
    if (!out || vocab < 1 || n < 0) return BCU_ERR_ARG;
    std::vector<double> cdf(vocab);
    double acc = 0;
    for (int k = 0; k < vocab; k++) {
        acc += std::pow((double)(k + 1), -s);
        cdf[k] = acc;
    }
    for (int i = 0; i < n; i++) {
        double u = (double)(draw(seed, 0x21f, i) >> 11) * (1.0 / 9007199254740992.0) * acc;
        int lo = 0, hi = vocab - 1;
        while (lo < hi) {
            int mid = (lo + hi) / 2;
            if (cdf[mid] < u) lo = mid + 1;
            else hi = mid;
        }
        out[i] = (uint32_t)lo;
    }
    return BCU_OK;
}

}  // extern "C"
