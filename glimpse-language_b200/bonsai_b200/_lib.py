"""ctypes binding of libbonsai_cuda.so (include/bonsai_cuda.h).

The library is the product: there is no Python or CPU fallback. Loading fails loudly when the shared object is
missing; device calls fail with BonsaiError when no GPU is present.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libbonsai_cuda.so")

MAX_LAYERS = 64
VMAX = 16

# bcu_status
OK, ERR_CUDA, ERR_ARG, ERR_OOM, ERR_TIMEOUT, ERR_CANCELLED, ERR_STATE, ERR_NOT_FOUND, ERR_TOO_LARGE, ERR_IO = range(10)
STATUS_NAMES = ["OK", "CUDA", "ARG", "OOM", "TIMEOUT", "CANCELLED", "STATE", "NOT_FOUND", "TOO_LARGE", "IO"]
# bcu_dtype
U32, F16, BF16, F32 = range(4)
# draft modes
DRAFT_LOOKUP, DRAFT_PLANTED, DRAFT_RANDOM = range(3)


# callbacks of bcu_set_encoder / bcu_set_emit
ENCODE_FN = ctypes.CFUNCTYPE(ctypes.c_int32, ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint8), ctypes.c_int32,
                             ctypes.POINTER(ctypes.c_uint32), ctypes.c_int32)
EMIT_FN = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_uint32)


class BcuConfig(ctypes.Structure):
    _fields_ = [
        ("hidden", ctypes.c_int32),
        ("intermediate", ctypes.c_int32),
        ("vocab", ctypes.c_int32),
        ("n_layers", ctypes.c_int32),
        ("layer_is_attn", ctypes.c_uint8 * MAX_LAYERS),
        ("heads", ctypes.c_int32),
        ("kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("lin_k_heads", ctypes.c_int32),
        ("lin_v_heads", ctypes.c_int32),
        ("lin_k_dim", ctypes.c_int32),
        ("lin_v_dim", ctypes.c_int32),
        ("conv_kernel", ctypes.c_int32),
        ("rope_theta", ctypes.c_double),
        ("rotary_dims", ctypes.c_int32),
        ("mrope", ctypes.c_int32 * 3),
        ("eps", ctypes.c_double),
        ("group_size", ctypes.c_int32),
        ("has_bias", ctypes.c_int32),
        ("hadamard", ctypes.c_int32),
        ("has_signs", ctypes.c_int32),
        ("head_kind", ctypes.c_int32),
        ("ctx", ctypes.c_int32),
        ("vmax", ctypes.c_int32),
    ]


class BcuLoraLinear(ctypes.Structure):
    _fields_ = [
        ("layer", ctypes.c_int32),
        ("module", ctypes.c_char_p),
        ("a", ctypes.POINTER(ctypes.c_float)),
        ("b", ctypes.POINTER(ctypes.c_float)),
        ("a_shape", ctypes.c_int64 * 2),
        ("b_shape", ctypes.c_int64 * 2),
    ]


class BcuSpec(ctypes.Structure):
    _fields_ = [("ngram_max", ctypes.c_int32), ("ngram_min", ctypes.c_int32), ("draft_max", ctypes.c_int32)]


class BcuStats(ctypes.Structure):
    _fields_ = [
        ("prompt_tokens", ctypes.c_int32),
        ("cached_tokens", ctypes.c_int32),
        ("gen_tokens", ctypes.c_int32),
        ("prefill_s", ctypes.c_double),
        ("ttft_s", ctypes.c_double),
        ("decode_s", ctypes.c_double),
        ("verify_calls", ctypes.c_int32),
        ("drafted", ctypes.c_int32),
        ("accepted", ctypes.c_int32),
        ("switches", ctypes.c_int32),
    ]


_lib = None

P = ctypes.c_void_p
I32 = ctypes.c_int32
U64 = ctypes.c_uint64
PI32 = ctypes.POINTER(ctypes.c_int32)
PU32 = ctypes.POINTER(ctypes.c_uint32)

# name -> (restype, argtypes)
SIGNATURES = {
    "bcu_config_check": (I32, [ctypes.POINTER(BcuConfig), ctypes.c_char_p, ctypes.c_size_t]),
    "bcu_create": (I32, [ctypes.POINTER(BcuConfig), I32, ctypes.POINTER(P)]),
    "bcu_load_tensor": (I32, [P, ctypes.c_char_p, I32, ctypes.POINTER(ctypes.c_int64), I32, P]),
    "bcu_finalize": (I32, [P]),
    "bcu_reset": (I32, [P]),
    "bcu_last_error": (ctypes.c_char_p, [P]),
    "bcu_destroy": (None, [P]),
    "bcu_device_name": (I32, [P, ctypes.c_char_p, ctypes.c_size_t]),
    "bcu_prefill": (I32, [P, PU32, I32, PU32]),
    "bcu_step": (I32, [P, ctypes.c_uint32, PU32]),
    "bcu_verify": (I32, [P, PU32, I32, PU32, PI32]),
    "bcu_verify_accept": (I32, [P, PU32, I32, PI32, PU32]),
    "bcu_accept": (I32, [P, I32, I32]),
    "bcu_flush": (I32, [P]),
    "bcu_length": (I32, [P, PI32]),
    "bcu_set_keep_logits": (I32, [P, I32]),
    "bcu_read_logits": (I32, [P, I32, P]),
    "bcu_snapshot": (I32, [P, ctypes.POINTER(P)]),
    "bcu_restore": (I32, [P, P]),
    "bcu_state_free": (None, [P]),
    "bcu_state_parts": (I32, [P, P, ctypes.POINTER(U64), PI32]),
    "bcu_state_read": (I32, [P, P, I32, P, U64]),
    "bcu_state_write": (I32, [P, P, I32, P, U64, I32]),
    "bcu_state_new": (I32, [P, I32, ctypes.POINTER(P)]),
    "bcu_set_lora": (I32, [P, ctypes.POINTER(BcuLoraLinear), I32, ctypes.c_float]),
    "bcu_lora_info": (I32, [P, PI32, PI32]),
    "bcu_hash_bytes": (U64, [U64, P, U64]),
    "bcu_kernel_hash": (U64, []),
    "bcu_prefix_identity": (I32, [P, U64, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, P, U64,
                                  ctypes.POINTER(U64)]),
    "bcu_prefix_path": (I32, [ctypes.c_char_p, P, U64, PU32, I32, ctypes.c_char_p, U64]),
    "bcu_prefix_save": (I32, [P, P, ctypes.c_char_p, P, U64, PU32, I32, I32]),
    "bcu_prefix_wait_saves": (I32, []),
    "bcu_prefix_load": (I32, [P, ctypes.c_char_p, P, U64, PU32, I32, ctypes.POINTER(P)]),
    "bcu_prefix_file_write": (I32, [ctypes.c_char_p, P, U64, PU32, I32, ctypes.POINTER(P), ctypes.POINTER(U64)]),
    "bcu_prefix_file_read": (I32, [ctypes.c_char_p, P, U64, PU32, I32, ctypes.POINTER(P), ctypes.POINTER(U64), PI32]),
    "bcu_set_vocab_bytes": (I32, [P, P, ctypes.POINTER(U64), I32]),
    "bcu_decode": (
        I32,
        [P, ctypes.c_uint32, PU32, I32, ctypes.POINTER(BcuSpec), I32, PU32, I32, U64, PU32, I32, I32, PU32, PI32,
         ctypes.POINTER(BcuStats)],
    ),
    "bcu_cancel": (I32, [P, I32]),
    "bcu_set_fillers": (I32, [P, PU32, I32]),
    "bcu_set_encoder": (I32, [P, P, P]),
    "bcu_set_emit": (I32, [P, P, P]),
    "bcu_linear_prepare": (I32, [P, P, P, I32, I32, I32, I32, ctypes.POINTER(P)]),
    "bcu_linear_free": (None, [P]),
    "bcu_linear_rotate_forward": (I32, [P, P, I32, I32, P, P, P]),
    "bcu_linear_forward": (I32, [P, P, I32, P, P]),
    "bcu_linear_gemm": (I32, [P, P, I32, P, P]),
    "bcu_linear_sync": (I32, [P, P]),
    "bcu_linear_rotate_forward_static": (I32, [P, P, I32, I32, P, P, P]),
    "bcu_gdn_verify": (I32, [P, P, P, P, P, P, P, P, P, I32, I32, I32, I32, P]),
    "bcu_gdn_prefill_workspace": (I32, [I32, I32, ctypes.POINTER(U64)]),
    "bcu_gdn_prefill": (I32, [P, P, P, P, P, P, P, P, P, I32, I32, I32, P, P]),
    "bcu_pass_launches": (I32, [P, I32, PI32]),
    "bcu_pass_bytes": (I32, [P, I32, ctypes.POINTER(ctypes.c_double)]),
    "bcu_time_pass": (I32, [P, I32, I32, ctypes.POINTER(ctypes.c_float)]),
    "bcu_set_planted": (I32, [P, PU32, I32, I32]),
    "bcu_enqueue_passes": (I32, [P, I32, I32, I32]),
    "bcu_sync": (I32, [P]),
    "bcu_stream": (I32, [P, ctypes.POINTER(P)]),
    # host-logic exports (not in the ABI header: test hooks of the decode driver and the operand build)
    "bcu_set_local_build": (I32, [P, I32]),
    "bcu_set_batched_prefill": (I32, [P, I32]),
    "bcu_linear_set_local_build": (I32, [P, I32]),
    "bcu_gemv_set_clusters": (I32, [I32]),
    "bcu_static_scratch_debug": (I32, [I32, I32]),
    "bcu_debug_wait_timeout": (I32, [P]),
    "bcu_gemm_prep_debug": (I32, [P, P, I32, P, P]),
    "bcu_token_key": (U64, [P, U64]),
    "bcu_draft_source_host": (I32, [PU32, I32, P, ctypes.POINTER(U64), I32, PU32, I32, PU32]),
    "bcu_normalize_draft_host": (I32, [PU32, I32, ctypes.c_uint32, P, ctypes.POINTER(U64), I32, P, P]),
    "bcu_lookup": (I32, [PU32, I32, PU32, I32, ctypes.POINTER(U64), I32, I32, I32, I32, I32, I32, PU32, PI32]),
    "bcu_policy_choose": (I32, [ctypes.c_double, ctypes.c_double, ctypes.POINTER(ctypes.c_double), I32, I32,
                                ctypes.c_double]),
}


def lib():
    """The loaded library (built in-tree by `make -C glimpse-language_b200`)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build the CUDA backend first (make -C glimpse-language_b200); "
                "there is no fallback path")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib
