/*
 * bonsai_synth.h — seeded synthetic inputs for the graded random-init shapes (libbonsai_synth.so).
 *
 * Not part of the backend: the reference loads real checkpoints, which are not available offline, so the tests and
 * the benchmark generate weights and prompts with these functions. They live in their own host-only library so that
 * the benchmark's reference arm (the CPU oracle) can generate the same bytes without loading the CUDA backend.
 * No counterpart in the reference.
 */
#ifndef BONSAI_SYNTH_H
#define BONSAI_SYNTH_H

#include "bonsai_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Deterministic seeded synthetic tensors (integer-only generators, identical on every host). kind: 0 = uniform
 * [a, b) fp32, 1 = approx-normal (mean a, std b) fp32, 2 = approx-normal bf16, 3 = ternary codes {0,1,2} packed
 * 16 per u32, 4 = uniform fp16 [a, b), 5 = +-1 fp32 signs, 6 = fp16 = -(value of another uniform fp16 stream)
 * (stream/seed as kind 4). n = elements (words for kind 3). */
bcu_status bcu_synth_fill(int32_t kind, uint64_t seed, uint64_t stream, double a, double b, void* out, uint64_t n);
/* Zipf(s) token ids in [0, vocab). */
bcu_status bcu_synth_zipf(uint64_t seed, double s, int32_t vocab, uint32_t* out, int32_t n);

#ifdef __cplusplus
}
#endif

#endif
