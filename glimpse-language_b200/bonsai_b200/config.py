"""Model configurations: the reference's config.json parse (Config::load, runtime/model.rs:41-67; parse_config,
src/bonsai/mod.rs:193-223) and the graded synthetic shapes."""
import json

from . import _lib


def layer_types(n_layers, interval=4):
    """3:1 GatedDeltaNet:full-attention order (`full_attention_interval` 4): every 4th layer is attention."""
    return [(i + 1) % interval == 0 for i in range(n_layers)]


def make_config(hidden, intermediate, vocab, n_layers, heads, kv_heads, lin_k_heads, lin_v_heads, *, group_size=64,
                has_bias=True, hadamard=512, has_signs=True, ctx=2048, vmax=16, rope_theta=1e7, rotary_dims=64,
                mrope=(11, 11, 10), attn_layers=None):
    c = _lib.BcuConfig()
    c.hidden, c.intermediate, c.vocab, c.n_layers = hidden, intermediate, vocab, n_layers
    attn = attn_layers if attn_layers is not None else layer_types(n_layers)
    for i, a in enumerate(attn):
        c.layer_is_attn[i] = 1 if a else 0
    c.heads, c.kv_heads, c.head_dim = heads, kv_heads, 256
    c.lin_k_heads, c.lin_v_heads, c.lin_k_dim, c.lin_v_dim, c.conv_kernel = lin_k_heads, lin_v_heads, 128, 128, 4
    c.rope_theta, c.rotary_dims = rope_theta, rotary_dims
    c.mrope[0], c.mrope[1], c.mrope[2] = mrope
    c.eps = 1e-6
    c.group_size, c.has_bias, c.hadamard, c.has_signs = group_size, int(has_bias), hadamard, int(has_signs)
    c.head_kind = 0
    c.ctx, c.vmax = ctx, vmax
    return c


def bonsai_2b_graded(ctx=2048):
    """Graded config 3: Bonsai-2B shape, 24 layers 3:1, hidden 2048, MLP 6144, 16 q / 2 kv heads (head_dim 256),
    GDN 16 key / 32 value heads, vocab 248320; ternary pack g64 + fp16 bias; activations rotated like the reference
    model (512-point Walsh-Hadamard blocks with per-input signs, kernels.metal:117-144); bf16 tied embedding /
    lm_head."""
    return make_config(2048, 6144, 248320, 24, 16, 2, 16, 32, group_size=64, has_bias=True, hadamard=512,
                       has_signs=True, ctx=ctx)


def bonsai_4b_graded(ctx=4608):
    """Graded config 4 shape: 32 layers 3:1, hidden 2560, MLP 9216, 16 q / 4 kv heads, GDN 16 / 32 heads, 512-point
    rotation blocks with signs."""
    return make_config(2560, 9216, 248320, 32, 16, 4, 16, 32, group_size=64, has_bias=True, hadamard=512,
                       has_signs=True, ctx=ctx)


def tiny(*, group_size=64, has_bias=True, hadamard=512, has_signs=True, n_layers=4, vocab=4096, kv_heads=2, ctx=256,
         hidden=512, intermediate=1024, heads=4, lin_k_heads=2, lin_v_heads=4, head_kind=0):
    """Small shapes for parity tests (every kernel path, seconds on the oracle). head_kind 1: the reference's ternary
    tied embedding / head."""
    c = make_config(hidden, intermediate, vocab, n_layers, heads, kv_heads, lin_k_heads, lin_v_heads,
                    group_size=group_size, has_bias=has_bias, hadamard=hadamard, has_signs=has_signs, ctx=ctx)
    c.head_kind = head_kind
    return c


def parse_config(text):
    """parse_config (src/bonsai/mod.rs:193-223) + Config::load (model.rs:41-67): the text config of a reference
    model directory, mapped to a device config with the reference's own pack (g128, implicit bias, 512-point blocks
    with signs, ternary tied head)."""
    j = json.loads(text)
    t = j.get("text_config")
    if not isinstance(t, dict):
        raise ValueError("config: missing text_config")

    def u(k):
        v = t.get(k)
        if not isinstance(v, int):
            raise ValueError(f"config: missing {k}")
        return v

    r = t.get("rope_parameters") or {}
    head_dim = u("head_dim")
    types = t.get("layer_types")
    if not isinstance(types, list):
        raise ValueError("config: layer_types")
    c = make_config(u("hidden_size"), u("intermediate_size"), u("vocab_size"), len(types),
                    u("num_attention_heads"), u("num_key_value_heads"), u("linear_num_key_heads"),
                    u("linear_num_value_heads"), group_size=128, has_bias=False, hadamard=512, has_signs=True,
                    rope_theta=float(r.get("rope_theta", 1e7)),
                    rotary_dims=int(head_dim * float(r.get("partial_rotary_factor", 0.25))),
                    mrope=tuple(r.get("mrope_section", (11, 11, 10))),
                    attn_layers=[x == "full_attention" for x in types])
    c.head_dim = head_dim
    c.lin_k_dim, c.lin_v_dim = u("linear_key_head_dim"), u("linear_value_head_dim")
    c.conv_kernel = u("linear_conv_kernel_dim")
    c.eps = float(t.get("rms_norm_eps", 0.0))
    c.head_kind = 1
    return c


def check(cfg):
    """bcu_config_check: (ok, message)."""
    buf = __import__("ctypes").create_string_buffer(256)
    s = _lib.lib().bcu_config_check(cfg, buf, 256)
    return s == _lib.OK, buf.value.decode()


def dims(cfg):
    C = 2 * cfg.lin_k_heads * 128 + cfg.lin_v_heads * 128
    return dict(C=C, gw=cfg.lin_v_heads * 128, aw=cfg.heads * 256, kvw=cfg.kv_heads * 256)
