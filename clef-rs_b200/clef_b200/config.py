"""Model geometry shared by the C ABI (struct clef_config in include/clef_b200.h).

Mirrors TextConfig of the reference (crates/core/src/models/qwen.rs:42-58):
the same fields, read from the same Hugging Face `text_config` JSON keys.
"""
import ctypes

MAX_LAYERS = 128


class ClefConfig(ctypes.Structure):
    _fields_ = [
        ("hidden_size", ctypes.c_int32),
        ("intermediate_size", ctypes.c_int32),
        ("num_hidden_layers", ctypes.c_int32),
        ("vocab_size", ctypes.c_int32),
        ("num_attention_heads", ctypes.c_int32),
        ("num_key_value_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("linear_num_key_heads", ctypes.c_int32),
        ("linear_num_value_heads", ctypes.c_int32),
        ("linear_key_head_dim", ctypes.c_int32),
        ("linear_value_head_dim", ctypes.c_int32),
        ("linear_conv_kernel_dim", ctypes.c_int32),
        ("rotary_dim", ctypes.c_int32),
        ("head_outputs", ctypes.c_int32),
        ("rms_norm_eps", ctypes.c_float),
        ("rope_theta", ctypes.c_double),
        ("layer_types", ctypes.c_uint8 * MAX_LAYERS),
    ]

    def is_attention(self, i: int) -> bool:
        return bool(self.layer_types[i])

    def describe(self) -> dict:
        return {name: (list(getattr(self, name))[: self.num_hidden_layers]
                       if name == "layer_types" else getattr(self, name))
                for name, _ in self._fields_}


def from_text_config(c: dict, head_outputs: int = 0) -> ClefConfig:
    """Builds the geometry from a Hugging Face Qwen3.5 `text_config` dict, the
    way Backbone::load reads it (qwen.rs:193-277, :472 for the rotary width)."""
    cfg = ClefConfig()
    for key in ("hidden_size", "intermediate_size", "num_hidden_layers", "vocab_size",
                "num_attention_heads", "num_key_value_heads", "head_dim",
                "linear_num_key_heads", "linear_num_value_heads", "linear_key_head_dim",
                "linear_value_head_dim", "linear_conv_kernel_dim"):
        setattr(cfg, key, int(c[key]))
    rope = c["rope_parameters"]
    cfg.rotary_dim = int(c["head_dim"] * rope["partial_rotary_factor"])
    cfg.rope_theta = float(rope["rope_theta"])
    cfg.rms_norm_eps = float(c["rms_norm_eps"])
    cfg.head_outputs = head_outputs
    for i, t in enumerate(c["layer_types"]):
        cfg.layer_types[i] = 1 if t == "full_attention" else 0
    return cfg


def benchmark_config(layers: int = 32, head_outputs: int = 7) -> ClefConfig:
    """The benchmark geometry: hidden 2560, intermediate 9216, [3 DeltaNet +
    1 attention] blocks, 16 q / 4 kv heads of 256, 16 qk / 32 v linear heads of
    128, conv 4, RoPE 1e7 on 64 of 256 features, eps 1e-6, vocab 248320."""
    cfg = ClefConfig()
    cfg.hidden_size = 2560
    cfg.intermediate_size = 9216
    cfg.num_hidden_layers = layers
    cfg.vocab_size = 248320
    cfg.num_attention_heads = 16
    cfg.num_key_value_heads = 4
    cfg.head_dim = 256
    cfg.linear_num_key_heads = 16
    cfg.linear_num_value_heads = 32
    cfg.linear_key_head_dim = 128
    cfg.linear_value_head_dim = 128
    cfg.linear_conv_kernel_dim = 4
    cfg.rotary_dim = 64
    cfg.head_outputs = head_outputs
    cfg.rms_norm_eps = 1e-6
    cfg.rope_theta = 1e7
    for i in range(layers):
        cfg.layer_types[i] = 1 if i % 4 == 3 else 0
    return cfg


def flash_config(layers: int = 32, head_outputs: int = 7) -> ClefConfig:
    """The released Flash geometry the reference's published numbers are
    quoted on (crates/core/fixtures/release/flash-config.json): hidden 4096,
    intermediate 12288, otherwise as benchmark_config (16/4 x 256 attention,
    16/32 x 128 DeltaNet, RoPE 1e7 on 64 of 256 features, eps 1e-6)."""
    cfg = benchmark_config(layers, head_outputs)
    cfg.hidden_size = 4096
    cfg.intermediate_size = 12288
    return cfg


def layer_prefix(i: int) -> str:
    return f"model.language_model.layers.{i}"


def weight_shapes(cfg: ClefConfig) -> dict:
    """Every tensor the engine expects, with its shape (Backbone::load naming,
    qwen.rs:193-277, FullAttention::load :429-450, Delta::load :528-588)."""
    h = cfg.hidden_size
    key = cfg.linear_num_key_heads * cfg.linear_key_head_dim
    value = cfg.linear_num_value_heads * cfg.linear_value_head_dim
    n = cfg.num_attention_heads * cfg.head_dim
    kv = cfg.num_key_value_heads * cfg.head_dim
    s = {"model.language_model.embed_tokens.weight": (cfg.vocab_size, h),
         "model.language_model.norm.weight": (h,)}
    if cfg.head_outputs:
        s["clef.head.weight"] = (cfg.head_outputs, h)
    for i in range(cfg.num_hidden_layers):
        p = layer_prefix(i)
        s[f"{p}.input_layernorm.weight"] = (h,)
        s[f"{p}.post_attention_layernorm.weight"] = (h,)
        s[f"{p}.mlp.gate_proj.weight"] = (cfg.intermediate_size, h)
        s[f"{p}.mlp.up_proj.weight"] = (cfg.intermediate_size, h)
        s[f"{p}.mlp.down_proj.weight"] = (h, cfg.intermediate_size)
        if cfg.layer_types[i]:
            s[f"{p}.self_attn.q_proj.weight"] = (2 * n, h)
            s[f"{p}.self_attn.k_proj.weight"] = (kv, h)
            s[f"{p}.self_attn.v_proj.weight"] = (kv, h)
            s[f"{p}.self_attn.o_proj.weight"] = (h, n)
            s[f"{p}.self_attn.q_norm.weight"] = (cfg.head_dim,)
            s[f"{p}.self_attn.k_norm.weight"] = (cfg.head_dim,)
        else:
            s[f"{p}.linear_attn.in_proj_qkv.weight"] = (2 * key + value, h)
            s[f"{p}.linear_attn.in_proj_z.weight"] = (value, h)
            s[f"{p}.linear_attn.in_proj_a.weight"] = (cfg.linear_num_value_heads, h)
            s[f"{p}.linear_attn.in_proj_b.weight"] = (cfg.linear_num_value_heads, h)
            s[f"{p}.linear_attn.out_proj.weight"] = (h, value)
            s[f"{p}.linear_attn.conv1d.weight"] = (2 * key + value, 1, cfg.linear_conv_kernel_dim)
            s[f"{p}.linear_attn.dt_bias"] = (cfg.linear_num_value_heads,)
            s[f"{p}.linear_attn.A_log"] = (cfg.linear_num_value_heads,)
            s[f"{p}.linear_attn.norm.weight"] = (cfg.linear_value_head_dim,)
    return s


def linear_flops_per_token(cfg: ClefConfig) -> float:
    """2 x (parameters of every projection): the GEMM FLOPs one token costs."""
    h = cfg.hidden_size
    key = cfg.linear_num_key_heads * cfg.linear_key_head_dim
    value = cfg.linear_num_value_heads * cfg.linear_value_head_dim
    n = cfg.num_attention_heads * cfg.head_dim
    kv = cfg.num_key_value_heads * cfg.head_dim
    lin = 0
    for i in range(cfg.num_hidden_layers):
        lin += 3 * cfg.intermediate_size * h
        if cfg.layer_types[i]:
            lin += (2 * n + 2 * kv) * h + n * h
        else:
            lin += (2 * key + value + value + 2 * cfg.linear_num_value_heads) * h + value * h
    return 2.0 * lin


def flops_per_request(cfg: ClefConfig, tokens: int, prefix: int = 0) -> float:
    """Algorithmic FLOPs of one prefill: 2*params of every linear layer per token
    plus 4*d per (query, key) pair and attention head (QK^T and PV), causal."""
    h = cfg.hidden_size
    key = cfg.linear_num_key_heads * cfg.linear_key_head_dim
    value = cfg.linear_num_value_heads * cfg.linear_value_head_dim
    n = cfg.num_attention_heads * cfg.head_dim
    kv = cfg.num_key_value_heads * cfg.head_dim
    lin = 0
    att_layers = 0
    for i in range(cfg.num_hidden_layers):
        lin += 3 * cfg.intermediate_size * h
        if cfg.layer_types[i]:
            lin += (2 * n + 2 * kv) * h + n * h
            att_layers += 1
        else:
            lin += (2 * key + value + value + 2 * cfg.linear_num_value_heads) * h + value * h
    pairs = tokens * prefix + tokens * (tokens + 1) / 2
    return 2.0 * lin * tokens + att_layers * 4.0 * cfg.num_attention_heads * cfg.head_dim * pairs


def scan_flops_per_token(cfg: ClefConfig, chunk: int = 64) -> float:
    """Chunked-scan FLOPs per token per DeltaNet layer at chunk size C."""
    dk, dv, hv = cfg.linear_key_head_dim, cfg.linear_value_head_dim, cfg.linear_num_value_heads
    c = chunk
    per_chunk = 2 * (2 * c * c * dk) + 2 * (2 * c * c * dk) + 2 * (c * dk * dv) * 3 + 2 * c * c * dv
    return per_chunk * hv / c

