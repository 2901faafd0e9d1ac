"""Seeded random-init weights and architecture presets.

Self-contained (numpy only) so the golden-fixture script can load this file by
path next to the reference package of the same import name.

The weight dicts use HuggingFace key names, the same keys the reference
constructors read: ``GPT2(weights, config)`` (draftkv/gpt2.py:140-165) and
``LlamaLike(weights, config)`` (draftkv/llama.py:115-151).  Every matrix is
N(0, std) from one ``numpy.random.default_rng(seed)`` stream, norm gains are 1
and biases 0, as the benchmark configurations specify.
"""

from __future__ import annotations

import numpy as np

# ---------------------------------------------------------------- presets
# The shapes of the benchmark configurations.  `dtype` is the storage type the
# device path computes in; the numpy oracle is always fed the same values
# widened to fp32.
PRESETS: dict[str, dict] = {
    # distilgpt2 shape: 6L / 768 / 12x64, learned positions (1024), GELU 3072
    "distilgpt2": dict(arch="gpt2", n_layer=6, n_embd=768, n_head=12, n_inner=3072,
                       n_positions=1024, vocab_size=50257, layer_norm_epsilon=1e-5,
                       dtype="f32"),
    # SmolLM2-135M shape: 30L / 576, 9q/3kv x 64, SwiGLU 1536, theta 1e5, tied
    "smollm2-135m": dict(arch="llama", num_hidden_layers=30, hidden_size=576,
                         num_attention_heads=9, num_key_value_heads=3, head_dim=64,
                         intermediate_size=1536, rope_theta=100000.0,
                         vocab_size=49152, rms_norm_eps=1e-5, tie_word_embeddings=True,
                         dtype="bf16"),
    # Llama-3-8B shape: 32L / 4096, 32q/8kv x 128, SwiGLU 14336, theta 5e5
    "llama3-8b": dict(arch="llama", num_hidden_layers=32, hidden_size=4096,
                      num_attention_heads=32, num_key_value_heads=8, head_dim=128,
                      intermediate_size=14336, rope_theta=500000.0,
                      vocab_size=128256, rms_norm_eps=1e-5, tie_word_embeddings=False,
                      dtype="bf16"),
}


def llama_config(n_layers: int, d_model: int, n_heads: int, n_kv_heads: int,
                 d_ff: int, vocab: int, head_dim: int | None = None,
                 theta: float = 10000.0, eps: float = 1e-5, tied: bool = True,
                 dtype: str = "bf16") -> dict:
    return dict(arch="llama", num_hidden_layers=n_layers, hidden_size=d_model,
                num_attention_heads=n_heads, num_key_value_heads=n_kv_heads,
                head_dim=head_dim or d_model // n_heads, intermediate_size=d_ff,
                rope_theta=float(theta), vocab_size=vocab, rms_norm_eps=eps,
                tie_word_embeddings=tied, dtype=dtype)


def gpt2_config(n_layers: int, d_model: int, n_heads: int, vocab: int,
                n_positions: int = 1024, d_ff: int | None = None,
                dtype: str = "f32") -> dict:
    return dict(arch="gpt2", n_layer=n_layers, n_embd=d_model, n_head=n_heads,
                n_inner=d_ff or 4 * d_model, n_positions=n_positions,
                vocab_size=vocab, layer_norm_epsilon=1e-5, dtype=dtype)


# ---------------------------------------------------------------- bf16
def round_bf16(a: np.ndarray) -> np.ndarray:
    """Round fp32 values to the nearest bf16 (ties to even), returned as fp32."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32)
    # NaN payloads must stay NaN
    return np.where(np.isnan(a), a, out).astype(np.float32)


# ---------------------------------------------------------------- factories
def make_weights(cfg: dict, seed: int = 0, std: float = 0.02,
                 attn_gain: float = 1.0, attn_sharpness: float = 1.0) -> dict[str, np.ndarray]:
    """Random-init weights for `cfg` (a preset or a *_config() dict).

    `attn_sharpness` scales the query projection and `attn_gain` the attention
    output projection; small test models use them to get peaked attention and
    logit margins well above the fp32/bf16 tolerances (with plain N(0, 0.02)
    weights every top-2 margin is tiny).  For bf16 configs the values are
    rounded to bf16 so that the device copy and the fp32 oracle copy agree.
    """
    rng = np.random.default_rng(seed)
    f32 = np.float32

    def R(*shape, k=1.0):
        return (rng.standard_normal(shape) * (std * k)).astype(f32)

    w: dict[str, np.ndarray] = {}
    if cfg["arch"] == "gpt2":
        d, L, V, F = cfg["n_embd"], cfg["n_layer"], cfg["vocab_size"], cfg["n_inner"]
        w["wte.weight"] = R(V, d)
        w["wpe.weight"] = R(cfg["n_positions"], d)
        for i in range(L):
            p = f"h.{i}."
            w[p + "ln_1.weight"] = np.ones(d, f32)
            w[p + "ln_1.bias"] = np.zeros(d, f32)
            qkv = R(d, 3 * d)                      # Conv1D layout: [in, out]
            qkv[:, :d] *= attn_sharpness
            w[p + "attn.c_attn.weight"] = qkv
            w[p + "attn.c_attn.bias"] = np.zeros(3 * d, f32)
            w[p + "attn.c_proj.weight"] = R(d, d, k=attn_gain)
            w[p + "attn.c_proj.bias"] = np.zeros(d, f32)
            w[p + "ln_2.weight"] = np.ones(d, f32)
            w[p + "ln_2.bias"] = np.zeros(d, f32)
            w[p + "mlp.c_fc.weight"] = R(d, F)
            w[p + "mlp.c_fc.bias"] = np.zeros(F, f32)
            w[p + "mlp.c_proj.weight"] = R(F, d)
            w[p + "mlp.c_proj.bias"] = np.zeros(d, f32)
        w["ln_f.weight"] = np.ones(d, f32)
        w["ln_f.bias"] = np.zeros(d, f32)
    elif cfg["arch"] == "llama":
        d, L, V = cfg["hidden_size"], cfg["num_hidden_layers"], cfg["vocab_size"]
        H, KV = cfg["num_attention_heads"], cfg["num_key_value_heads"]
        D = cfg.get("head_dim") or d // H
        F = cfg["intermediate_size"]
        w["model.embed_tokens.weight"] = R(V, d)
        w["model.norm.weight"] = np.ones(d, f32)
        for i in range(L):
            p = f"model.layers.{i}."
            w[p + "input_layernorm.weight"] = np.ones(d, f32)
            w[p + "post_attention_layernorm.weight"] = np.ones(d, f32)
            w[p + "self_attn.q_proj.weight"] = R(H * D, d, k=attn_sharpness)
            w[p + "self_attn.k_proj.weight"] = R(KV * D, d)
            w[p + "self_attn.v_proj.weight"] = R(KV * D, d)
            w[p + "self_attn.o_proj.weight"] = R(d, H * D, k=attn_gain)
            w[p + "mlp.gate_proj.weight"] = R(F, d)
            w[p + "mlp.up_proj.weight"] = R(F, d)
            w[p + "mlp.down_proj.weight"] = R(d, F)
        if not cfg.get("tie_word_embeddings", True):
            w["lm_head.weight"] = R(V, d)
    else:
        raise ValueError(f"unknown arch {cfg['arch']!r}")
    if cfg.get("dtype", "f32") == "bf16":
        w = {k: round_bf16(v) for k, v in w.items()}
    return w


def tokens(n: int, vocab: int, seed: int = 1) -> list[int]:
    """Uniform random token ids from `seed` (the benchmark prompts)."""
    return [int(t) for t in np.random.default_rng(seed).integers(0, vocab, n)]
