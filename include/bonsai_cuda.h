/*
 * bonsai_cuda.h — C ABI of the B200 (sm_100a) backend for the Ternary Bonsai 2 runtime's greedy speculative decode.
 *
 * The reference runtime (glimpse-language 0.3.0, Rust) swaps its GPU backend by module path
 * (src/bonsai/runtime/mod.rs:5-9) and drives it from `Model` (runtime/mod.rs:262-961) through `Text`
 * (runtime/model.rs:224-1100). Its backend surface is name-level (`Cmd::run(name, args, groups, threads)`,
 * runtime/gpu.rs:169-255), which cannot express fused kernels or graph capture, so this ABI sits one level up, at
 * the `Text`/`Model` operations. Each entry point names the reference function it replaces.
 *
 * Conventions
 *  - Plain C types only; every call returns a bcu_status; bcu_last_error() gives the message of the last failure.
 *  - One bcu_model per host thread at a time (the reference serialises the model behind a mutex, handle.rs:96-103).
 *  - Host buffers passed to a call are borrowed for the duration of that call only.
 *  - Every host wait has a deadline (BCU_ERR_TIMEOUT) instead of blocking forever. A wait polls the device without
 *    sleeping for its first 10 ms (a verify pass takes a few ms, and a sleep's wake-up latency would be added to every
 *    decode round), then every 20 us: the calling thread keeps one host core busy while it waits.
 *  - Token ids are uint32 (the reference's u32 ids, runtime/mod.rs:24).
 */
#ifndef BONSAI_CUDA_H
#define BONSAI_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BCU_ABI_VERSION 1
#define BCU_MAX_LAYERS 64

typedef enum {
    BCU_OK = 0,
    BCU_ERR_CUDA = 1,      /* a CUDA call failed (the reference panics in Pending::wait, gpu.rs:330-335) */
    BCU_ERR_ARG = 2,       /* bad argument or unsupported config (Config::check, model.rs:90-129) */
    BCU_ERR_OOM = 3,       /* device allocation failed */
    BCU_ERR_TIMEOUT = 4,   /* a bounded host or device wait ran out */
    BCU_ERR_CANCELLED = 5, /* the cancel flag was raised between steps (ext.rs:21-42) */
    BCU_ERR_STATE = 6,     /* call out of order (e.g. verify before finalize, context full) */
    BCU_ERR_NOT_FOUND = 7, /* unknown or missing tensor name */
    BCU_ERR_TOO_LARGE = 8, /* sizes beyond a fixed capacity (the static scratch of bcu_linear_rotate_forward_static) */
    BCU_ERR_IO = 9         /* a prefix file could not be written (save_prefix drops it silently, mod.rs:562-565) */
} bcu_status;

/* Tensor element types of bcu_load_tensor. */
typedef enum { BCU_U32 = 0, BCU_F16 = 1, BCU_BF16 = 2, BCU_F32 = 3 } bcu_dtype;

/* How the tied embedding / lm_head table is stored. */
typedef enum {
    BCU_HEAD_BF16 = 0,    /* bf16 [vocab, hidden] table, no rotation (the graded synthetic shapes) */
    BCU_HEAD_TERNARY = 1  /* ternary-packed tied table + Hadamard signs, as the reference (model.rs:356, 962) */
} bcu_head_kind;

/*
 * Model sizes. Mirrors `Config` (runtime/model.rs:20-38) plus the packing/rotation parameters the reference fixes
 * in its kernels (kernels.metal:2-4) and the graded synthetic shapes vary.
 */
typedef struct {
    int32_t hidden;          /* hidden_size */
    int32_t intermediate;    /* intermediate_size (SwiGLU) */
    int32_t vocab;           /* vocab_size */
    int32_t n_layers;        /* len(layer_types) */
    uint8_t layer_is_attn[BCU_MAX_LAYERS]; /* 1 = full attention, 0 = GatedDeltaNet */
    int32_t heads;           /* num_attention_heads */
    int32_t kv_heads;        /* num_key_value_heads */
    int32_t head_dim;        /* must be 256 */
    int32_t lin_k_heads;     /* linear_num_key_heads */
    int32_t lin_v_heads;     /* linear_num_value_heads */
    int32_t lin_k_dim;       /* must be 128 */
    int32_t lin_v_dim;       /* must be 128 */
    int32_t conv_kernel;     /* must be 4 */
    double rope_theta;
    int32_t rotary_dims;     /* head_dim * partial_rotary_factor */
    int32_t mrope[3];        /* mrope_section, sums to rotary_dims / 2 */
    double eps;              /* rms_norm_eps, must be 1e-6 */
    int32_t group_size;      /* ternary pack group: 64 or 128 codes per fp16 scale */
    int32_t has_bias;        /* 1: MLX affine fp16 bias per group; 0: implicit bias = -scale (weight = s*(code-1)) */
    int32_t hadamard;        /* Hadamard block of the activation rotation: 512 (reference) or 2048 */
    int32_t has_signs;       /* 1: per-input +-1 signs before the transform (reference); 0: none */
    int32_t head_kind;       /* bcu_head_kind */
    int32_t ctx;             /* KV capacity in positions (reference: CONTEXT=2048, hard cap 4096) */
    int32_t vmax;            /* largest verify chunk, <= 16 (reference VMAX, model.rs:11) */
} bcu_config;

typedef struct bcu_model bcu_model;

/* ------------------------------------------------------------------ lifecycle */

/* Config::check (model.rs:90-129) with the graded shapes' extensions (group 64 + bias, 2048-point rotation, any
 * q-per-kv ratio). Writes a message into err (may be NULL). */
bcu_status bcu_config_check(const bcu_config* cfg, char* err, size_t err_len);

/* Model::load (runtime/mod.rs:288-324) minus file IO: creates device state on `device`. */
bcu_status bcu_create(const bcu_config* cfg, int device, bcu_model** out);

/* Weights::get + lin() (weights.rs:89-97, model.rs:239-248): one named tensor, reference safetensors names
 * ("language_model.model.layers.3.mlp.down_proj.weight", ".scales", ".biases", ".signs", ...). Packed weights are
 * u32 [O, K/16] with code e of a word at bits 2e; scales/biases fp16 [O, K/group]. Copied during the call. */
bcu_status bcu_load_tensor(bcu_model* m, const char* name, int32_t dtype, const int64_t* shape, int32_t ndim,
                           const void* host_data);

/* All tensors present: repack weights into the device layout, build graphs. Text::new (model.rs:270-368). */
bcu_status bcu_finalize(bcu_model* m);

/* Text::reset (model.rs:404-409): empty KV, zero GDN/conv state, no pending accept. */
bcu_status bcu_reset(bcu_model* m);

/* ------------------------------------------------------------------ LoRA adapter (lora.rs, config 4) */

/* One adapted linear of lora::load (lora.rs:89-174) after the safetensors file is read: y = base(x) + (x A^T) B^T on
 * the linear's unrotated input. module is a Text::linears name (model.rs:372-385): "self_attn.q_proj" (q with its
 * gate rows), "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj", "linear_attn.in_proj_qkv",
 * "linear_attn.in_proj_z", "linear_attn.out_proj", "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj". */
typedef struct {
    int32_t layer;
    const char* module;
    const float* a;      /* lora_A [a_shape[0] = r][a_shape[1] = in], rounded to fp16 on load (lora.rs:111-118) */
    const float* b;      /* lora_B [b_shape[0] = out][b_shape[1] = r], times fold, then rounded to fp16 */
    int64_t a_shape[2];
    int64_t b_shape[2];
} bcu_lora_linear;
/* Text::set_lora (model.rs:392-397) with lora::load's grouping: linears that share an input share one stacked A (a
 * member the adapter lacks gets zero A and B rows). n == 0 removes the adapter. fold = alpha / r for PEFT keys
 * (peft_scaling, lora.rs:73-86) times the caller's scale. Errors as lora.rs: unknown module, shape mismatch, mixed
 * ranks; also Hadamard blocks above 1024 inputs. Recaptures the pass graphs and drops the verify-cost table; the
 * caller drops cached prefix states of another adapter (Model::set_lora, mod.rs:328-337). */
bcu_status bcu_set_lora(bcu_model* m, const bcu_lora_linear* lins, int32_t n, float fold);
/* Text::lora_info (model.rs:399-402): adapted linears and rank, 0 and 0 without an adapter. */
bcu_status bcu_lora_info(const bcu_model* m, int32_t* linears, int32_t* rank);

const char* bcu_last_error(const bcu_model* m);
void bcu_destroy(bcu_model* m);

/* Human-readable device name (Gpu::device_name, gpu.rs:91-93). */
bcu_status bcu_device_name(const bcu_model* m, char* out, size_t out_len);

/* ------------------------------------------------------------------ forward passes */

/* Model::prefill (runtime/mod.rs:341-386) for text tokens (positions continue from the current length). Writes the
 * greedy next token. Commits every row. */
bcu_status bcu_prefill(bcu_model* m, const uint32_t* ids, int32_t n, uint32_t* next);

/* Model::step (runtime/mod.rs:389-403): one token; the same kernels as a verify of one row, so plain decoding and
 * speculative decoding produce identical logits row for row. */
bcu_status bcu_step(bcu_model* m, uint32_t id, uint32_t* next);

/* Model::verify (runtime/mod.rs:407-421) + the accept length of decode_spec (runtime/mod.rs:866-868), on the device:
 * ids[0] is the last emitted token, ids[1..t) the drafts. Writes pred[0..t) (argmax per row; may be NULL to skip
 * the copy) and *accepted = m, the number of leading drafts equal to the prediction. The commit of the first m+1
 * rows is deferred into the next pass (defer_accept, runtime/mod.rs:431-434). */
bcu_status bcu_verify(bcu_model* m, const uint32_t* ids, int32_t t, uint32_t* pred, int32_t* accepted);

/* Same as bcu_verify, but only m and pred[m] (the bonus token) come back to the host: 8 bytes per round. */
bcu_status bcu_verify_accept(bcu_model* m, const uint32_t* ids, int32_t t, int32_t* accepted, uint32_t* bonus);

/* Model::accept / defer_accept (runtime/mod.rs:424-442): overrides the pending commit of the last verify of t rows
 * to its first n rows (1 <= n <= t). */
bcu_status bcu_accept(bcu_model* m, int32_t t, int32_t n);

/* Model::flush_accept (runtime/mod.rs:436-442): applies a pending commit now. */
bcu_status bcu_flush(bcu_model* m);

/* Tokens committed to the KV cache (State::len, model.rs:183). */
bcu_status bcu_length(const bcu_model* m, int32_t* len);

/* Debug/parity: copies the fp32 logits of row `row` of the last pass (vocab floats). Only when logits were kept
 * (bcu_set_keep_logits). */
bcu_status bcu_set_keep_logits(bcu_model* m, int32_t keep);
bcu_status bcu_read_logits(bcu_model* m, int32_t row, float* out);

/* ------------------------------------------------------------------ prefix cache (State snapshots) */

/* Snapshot handles: Text::encode_copy_state (model.rs:1072-1086) and State::new sized to the prefix. */
typedef struct bcu_state bcu_state;
bcu_status bcu_snapshot(bcu_model* m, bcu_state** out);            /* copy the live state (compact KV) */
bcu_status bcu_restore(bcu_model* m, const bcu_state* s);          /* copy a snapshot back (start_prefix hit);
                                                                      asynchronous: device copies on the model stream */
void bcu_state_free(bcu_state* s);
/* Text::state_parts (model.rs:1090-1099): byte sizes of [gdn, conv, K, V] and host read/write of them, for the
 * BNSPFX01 prefix files (runtime/mod.rs:494-578). parts[i] may be NULL to query sizes only. */
bcu_status bcu_state_parts(const bcu_model* m, const bcu_state* s, uint64_t sizes[4], int32_t* len);
bcu_status bcu_state_read(const bcu_model* m, const bcu_state* s, int32_t part, void* host, uint64_t bytes);
bcu_status bcu_state_write(bcu_model* m, bcu_state* s, int32_t part, const void* host, uint64_t bytes, int32_t len);
bcu_status bcu_state_new(bcu_model* m, int32_t len, bcu_state** out);

/* ------------------------------------------------------------------ saved prefix files (BNSPFX01) */

/* Layout (runtime/mod.rs:494-578; all integers little-endian): identity | ids u32[n] | len u64 (= n) | pos i64 (= n,
 * text only) | state parts gdn, conv, K, V as bcu_state_parts sizes them. identity = "BNSPFX01" | u64 words [kernel
 * hash, adapter, exe size, exe mtime ns, weights size, weights mtime ns, hash(config bytes), n_gdn, n_attn, hidden,
 * kv_width, conv_dim] | device name bytes. File "{dir}/{h:016x}.prefix", h = hash(hash(FNV, identity), ids bytes). */

/* hash_bytes (runtime/mod.rs:225-235): FNV-1a style over little-endian 8-byte words, then tail bytes, ^ length. */
uint64_t bcu_hash_bytes(uint64_t h, const void* data, uint64_t n);
/* Stands in for hash_bytes(FNV, gpu::KERNEL_BLOB) (runtime/mod.rs:501): the first 64 bits of the SHA-256 of the
 * CUDA sources and nvcc flags this library was built from. */
uint64_t bcu_kernel_hash(void);
/* Model::prefix_identity (runtime/mod.rs:494-510). exe_path NULL = the running executable. BCU_ERR_NOT_FOUND when
 * a file cannot be read (the reference returns None: nothing is saved or loaded). out NULL: *len only. */
bcu_status bcu_prefix_identity(const bcu_model* m, uint64_t adapter, const char* exe_path, const char* weights_path,
                               const char* config_path, uint8_t* out, uint64_t cap, uint64_t* len);
/* Model::prefix_path (runtime/mod.rs:512-515), NUL-terminated into out. */
bcu_status bcu_prefix_path(const char* dir, const uint8_t* identity, uint64_t identity_len, const uint32_t* ids,
                           int32_t n, char* out, uint64_t out_len);
/* Model::save_prefix (runtime/mod.rs:549-578): reads the snapshot's parts to the host on this thread, then writes
 * {h}.tmp, renames it to {h}.prefix and keeps the newest 3 .prefix files of dir (PREFIX_SLOTS, mod.rs:213), on a
 * background thread when background != 0 (failures there are dropped, as in the reference). s's length must be n. */
bcu_status bcu_prefix_save(bcu_model* m, const bcu_state* s, const char* dir, const uint8_t* identity,
                           uint64_t identity_len, const uint32_t* ids, int32_t n, int32_t background);
/* Joins the background writers started by bcu_prefix_save. (No counterpart: the reference detaches them.) */
bcu_status bcu_prefix_wait_saves(void);
/* Model::load_prefix (runtime/mod.rs:517-546): *out = a new snapshot of n tokens when {dir}/{h}.prefix has exactly
 * this identity and these ids, len = n and exactly the parts' bytes; NULL (status BCU_OK) for any other file or none. */
bcu_status bcu_prefix_load(bcu_model* m, const char* dir, const uint8_t* identity, uint64_t identity_len,
                           const uint32_t* ids, int32_t n, bcu_state** out);
/* The file writer and reader alone, on host buffers (no device): the same bytes as bcu_prefix_save / _load. */
bcu_status bcu_prefix_file_write(const char* dir, const uint8_t* identity, uint64_t identity_len, const uint32_t* ids,
                                 int32_t n, const void* const parts[4], const uint64_t sizes[4]);
bcu_status bcu_prefix_file_read(const char* dir, const uint8_t* identity, uint64_t identity_len, const uint32_t* ids,
                                int32_t n, void* const parts[4], const uint64_t sizes[4], int32_t* found);

/* ------------------------------------------------------------------ decode driver (runtime/mod.rs:774-956) */

typedef struct {
    int32_t ngram_max;   /* Spec::ngram_max (3) */
    int32_t ngram_min;   /* Spec::ngram_min (1) */
    int32_t draft_max;   /* Spec::draft_max (7 in the reference; 8 for the graded k=8) */
} bcu_spec;

/* Draft source for benchmarks: the reference has only prompt lookup; the graded configs force planted or random
 * drafts with the adaptive policy bypassed. */
typedef enum { BCU_DRAFT_LOOKUP = 0, BCU_DRAFT_PLANTED = 1, BCU_DRAFT_RANDOM = 2 } bcu_draft_mode;

typedef struct {
    int32_t prompt_tokens, cached_tokens, gen_tokens;
    double prefill_s, ttft_s, decode_s;
    int32_t verify_calls, drafted, accepted, switches;
} bcu_stats;  /* Stats (runtime/mod.rs:246-260) */

/* Per-token matching keys for prompt lookup: token_key (runtime/mod.rs:73-81) of each vocabulary entry's bytes.
 * bytes/offsets describe the vocabulary as one byte string (offsets has vocab+1 entries). Without a table every
 * token counts as a word keyed by its id. */
bcu_status bcu_set_vocab_bytes(bcu_model* m, const uint8_t* bytes, const uint64_t* offsets, int32_t vocab);

/* The filler ids Model::draft_source drops from the draft source (FILLERS, runtime/mod.rs:146, 750-756: the
 * hesitation words " um", " uh", ... whose encoding is one token). n = 0 returns to the default: the ids whose bytes
 * (bcu_set_vocab_bytes) equal a filler string exactly. */
bcu_status bcu_set_fillers(bcu_model* m, const uint32_t* ids, int32_t n);

/* The tokenizer Model::normalize_draft re-encodes changed draft words with (self.tok.encode, runtime/mod.rs:720):
 * encode n bytes of UTF-8 text into at most cap ids and return their count, or -1 (the word keeps its tokens).
 * NULL (the default) leaves drafts as lookup found them. Called on the thread that runs bcu_decode. */
typedef int32_t (*bcu_encode_fn)(void* user, const uint8_t* text, int32_t n, uint32_t* out, int32_t cap);
bcu_status bcu_set_encoder(bcu_model* m, bcu_encode_fn fn, void* user);

/* Streaming emission: fn(user, id) for every token bcu_decode outputs, in order, as it lands (the `emit` of
 * decode_spec / decode_plain, runtime/mod.rs:683, 892, 941; generate_streaming builds text from these ids). EOS is
 * not emitted. NULL (the default) disables. Called on the thread that runs bcu_decode. */
typedef void (*bcu_emit_fn)(void* user, uint32_t id);
bcu_status bcu_set_emit(bcu_model* m, bcu_emit_fn fn, void* user);

/* Model::decode_spec / decode_plain after the prompt has been prefilled: `first` is the token prefill returned,
 * `user` the user-turn ids (draft source: its first SOURCE_TAGS block, fillers removed, runtime/mod.rs:733-768;
 * lookup drafts are normalized when an encoder is set). spec == NULL decodes plainly (pipelined). Writes
 * up to max_tokens ids into out (first included) and returns the count in *n_out. planted/planted_n: the draft
 * stream for BCU_DRAFT_PLANTED (output token i+1 is planted[i]); seed for BCU_DRAFT_RANDOM. eos/n_eos: stop ids
 * (the reference's EOS, runtime/mod.rs:24); n_eos = 0 ignores EOS (ignore_eos). */
bcu_status bcu_decode(bcu_model* m, uint32_t first, const uint32_t* user, int32_t n_user, const bcu_spec* spec,
                      int32_t draft_mode, const uint32_t* planted, int32_t planted_n, uint64_t seed,
                      const uint32_t* eos, int32_t n_eos, int32_t max_tokens, uint32_t* out, int32_t* n_out,
                      bcu_stats* stats);

/* Cancellation between steps (ext.rs:21-42). */
bcu_status bcu_cancel(bcu_model* m, int32_t flag);

/* ------------------------------------------------------------------ standalone hot ops (graded configs 1 and 2) */

/* Config 1: Y[T, O] = W (ternary, MLX pack) . H(X[T, K]) where H is the Hadamard rotation of the model config
 * (block `hadamard`, optional signs, normalised) and X is bf16. All pointers are DEVICE pointers; the packed
 * weights must first be converted with bcu_linear_prepare. Replaces qmvxm/qmvx/qmv_cm (kernels.metal:668-709,
 * kernels/qmvx.comp, kernels/qmv_cm.comp) together with the rotation prologue (norm_rotate, kernels.metal:118-144). */
typedef struct bcu_linear bcu_linear;
bcu_status bcu_linear_prepare(const uint32_t* w_host, const uint16_t* scales_host, const uint16_t* biases_host,
                              int32_t O, int32_t K, int32_t group, int32_t device, bcu_linear** out);
void bcu_linear_free(bcu_linear* l);
bcu_status bcu_linear_rotate_forward(bcu_linear* l, const uint16_t* x_bf16_dev, int32_t T, int32_t hadamard,
                                     const float* signs_dev, float* y_dev, void* stream);
/* Y = W . X for an already rotated fp32 X (device pointers). */
bcu_status bcu_linear_forward(bcu_linear* l, const float* x_dev, int32_t T, float* y_dev, void* stream);
/* Batched prefill matmul (the reference's qmm, kernels.metal:437-500 / qmm_cm.comp; graded config 5): y[M][O] = W x
 * for any M, fp32 x (already rotated) and y on the device, on 5th-generation tensor cores (tcgen05.mma, tensor
 * memory accumulators, bulk-copy staging). Grows its activation scratch on the first call of a larger M (outside any
 * stream capture). Asynchronous: bcu_linear_sync waits and reports a device timeout. */
bcu_status bcu_linear_gemm(bcu_linear* l, const float* x_dev, int32_t M, float* y_dev, void* stream);
/* Waits for `stream` and returns BCU_ERR_TIMEOUT (clearing it) if a kernel of this handle, or a call of
 * bcu_linear_rotate_forward_static on the handle's device (any handle), gave up a bounded wait. */
bcu_status bcu_linear_sync(bcu_linear* l, void* stream);

/* bcu_linear_rotate_forward for callers that may not allocate device memory when they run it: a host that hands
 * all of its device memory to its own pool, or a decode loop that must not stall on the device synchronisation a
 * cudaMalloc/cudaFree can cause. No counterpart in the reference (its backends have no such caller). Same
 * arguments, same result; it allocates nothing: the split-K partial sums, per-row-block counters and error word
 * live in one static device array of 1 MiB + 4 KiB + 256 B in the library, so calls whose splits x T x O exceed
 * 262144 floats or whose O exceeds 131072 rows return BCU_ERR_TOO_LARGE. The first call on a device looks up that
 * array's address (make it before any stream capture). Every call shares the array and clears the counters it
 * needs on `stream` first; calls that overlap on the GPU (other streams, other threads) race on it. A wait that ran
 * out is recorded in the array until bcu_linear_sync (on any handle of the device) reports and clears it. */
bcu_status bcu_linear_rotate_forward_static(bcu_linear* l, const uint16_t* x_bf16_dev, int32_t T, int32_t hadamard,
                                            const float* signs_dev, float* y_dev, void* stream);

/* Config 2: one GatedDeltaNet verify step with rollback. q,k [T, NK, 128] and v [T, NV, 128] fp32 (q, k already
 * normalised as gdn_conv leaves them), a_in/b_in [T, NV] gate logits, A_log/dt_bias [NV], state [NV, 128, 128]
 * fp32 in place: on return it holds the state after the first n rows (0 <= n <= T), y [T, NV, 128] the outputs of
 * all T rows. gdn_gates + gdn_recurrent (kernels.metal:556-622) and the accept/rollback of encode_accept
 * (model.rs:1025-1069). Device pointers. */
bcu_status bcu_gdn_verify(const float* q, const float* k, const float* v, const float* a_in, const float* b_in,
                          const float* a_log, const float* dt_bias, float* state, float* y, int32_t T, int32_t NK,
                          int32_t NV, int32_t n, void* stream);

/* The gated delta rule of a prefill chunk (Model::prefill, runtime/mod.rs:341-386, runs gdn_recurrent,
 * kernels.metal:566-622, over the chunk's rows): the same inputs as bcu_gdn_verify, the state advanced by all T rows
 * (no rollback), y the outputs of every row. Computed in chunks of 64 rows (the per-row recurrence re-associated
 * into products within a chunk; results equal it within fp32 rounding). workspace: device memory of the size
 * bcu_gdn_prefill_workspace returns for (T, NV). Device pointers. */
bcu_status bcu_gdn_prefill_workspace(int32_t T, int32_t NV, uint64_t* bytes);
bcu_status bcu_gdn_prefill(const float* q, const float* k, const float* v, const float* a_in, const float* b_in,
                           const float* a_log, const float* dt_bias, float* state, float* y, int32_t T, int32_t NK,
                           int32_t NV, void* workspace, void* stream);

/* ------------------------------------------------------------------ introspection */

/* Kernel launches in the last pass (graph nodes), for the benchmark's gpu_launches. */
bcu_status bcu_pass_launches(const bcu_model* m, int32_t t, int32_t* launches);
/* Algorithmic bytes of one pass of t rows at the current length (weights + state + KV read). */
bcu_status bcu_pass_bytes(const bcu_model* m, int32_t t, double* bytes);
/* Times `iters` graph replays of a verify pass of t rows with CUDA events on the model's stream (state is saved and
 * restored around it). Writes milliseconds per pass. */
bcu_status bcu_time_pass(bcu_model* m, int32_t t, int32_t iters, float* ms_per_pass);

/* Device-resident draft stream for benchmarks with inputs already in HBM: with feed mode 2 a pass embeds
 * ids[t] = planted[off - base + t] (off = the KV offset of the pass). Copied during the call. */
bcu_status bcu_set_planted(bcu_model* m, const uint32_t* ids, int32_t n, int32_t base);
/* Enqueues `passes` verify passes of t rows without waiting. feed: 1 = row 0 is the previous pass's bonus token and
 * rows 1.. are the host ids of the last call, 2 = all rows from the planted stream. */
bcu_status bcu_enqueue_passes(bcu_model* m, int32_t t, int32_t passes, int32_t feed);
/* Waits (bounded) for everything enqueued on the model's stream and reads the control block back. */
bcu_status bcu_sync(bcu_model* m);
/* The model's CUDA stream (cudaStream_t), for callers that time with their own events. */
bcu_status bcu_stream(bcu_model* m, void** stream);

#ifdef __cplusplus
}
#endif
#endif
