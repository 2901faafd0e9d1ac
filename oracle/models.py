"""Decoder forward passes over the cache protocol (test infrastructure only).

One class, two architectures, numerics (including numpy's dtype promotions)
as in the reference:

  gpt2   -- draftkv/gpt2.py:120-127 (layer norm, gelu_new) and :182-213
            (learned positions, Conv1D x @ W with bias, MHA, tied head)
  llama  -- draftkv/llama.py:91-108 (rms norm, silu, rotate_half), :164-172
            (fp64 RoPE table, at least 1024 rows) and :175-225 (GQA: the cache
            holds KV heads; attention mass reported per KV head; SwiGLU; tied
            head when lm_head.weight is absent)

Both call cache.append(L, k, v, pos) before attention (a token attends to
itself), read the whole layer back, mask cpos > pos, and report fp32
probabilities through cache.note_attention.
"""

from __future__ import annotations

import numpy as np


def _softmax_last(x):
    z = x - x.max(axis=-1, keepdims=True)
    e = np.exp(z)
    return e / e.sum(axis=-1, keepdims=True)


class OracleModel:
    def __init__(self, weights: dict, config: dict):
        self.w = weights
        self.c = config
        if "n_embd" in config:                       # GPT-2 family
            self.arch = "gpt2"
            self.n_layers = config["n_layer"]
            self.n_heads = config["n_head"]
            self.n_kv_heads = self.n_heads
            self.d_model = config["n_embd"]
            self.eps = config.get("layer_norm_epsilon", 1e-5)
            pre = "transformer." if "transformer.wte.weight" in weights else ""
            self.pre = pre
            self.vocab_size = weights[f"{pre}wte.weight"].shape[0]
        else:
            self.arch = "llama"
            self.n_layers = config["num_hidden_layers"]
            self.n_heads = config["num_attention_heads"]
            self.n_kv_heads = config.get("num_key_value_heads", self.n_heads)
            self.d_model = config["hidden_size"]
            self.eps = config.get("rms_norm_eps", 1e-5)
            self.theta = float(config.get("rope_theta") or 10000.0)
            self.vocab_size = config["vocab_size"]
            self._cos = self._sin = None
        self.d_head = config.get("head_dim") or self.d_model // self.n_heads

    # ----------------------------------------------------------- helpers
    def _ln(self, x, g, b):
        mu = x.mean(-1, keepdims=True)
        var = x.var(-1, keepdims=True)
        return (x - mu) / np.sqrt(var + self.eps) * g + b

    def _rms(self, x, g):
        return x / np.sqrt((x * x).mean(-1, keepdims=True) + self.eps) * g

    def rope(self, pos):
        need = int(pos.max()) + 1
        if self._cos is None or self._cos.shape[0] < need:
            n = max(need, 1024)
            D = self.d_head
            inv = 1.0 / (self.theta ** (np.arange(0, D, 2) / D))
            ang = np.outer(np.arange(n), inv)
            full = np.concatenate([ang, ang], axis=-1)
            self._cos, self._sin = np.cos(full), np.sin(full)
        return self._cos[pos], self._sin[pos]

    @staticmethod
    def _rot(x):
        h = x.shape[-1] // 2
        return np.concatenate([-x[..., h:], x[..., :h]], axis=-1)

    def _attend(self, L, q, k, v, pos, cache, T):
        """Append, read back, causal-mask, softmax; returns (T, H*D)."""
        cache.append(L, k, v, pos)
        ck, cv, cpos = cache.read(L)
        rep = self.n_heads // self.n_kv_heads
        if rep > 1:
            ck = np.repeat(ck, rep, axis=1)
            cv = np.repeat(cv, rep, axis=1)
        s = np.einsum("qhd,khd->qhk", q, ck) / np.sqrt(self.d_head)
        s = np.where((cpos[None, :] > pos[:, None])[:, None, :], -np.inf, s)
        p = _softmax_last(s).astype(np.float32)
        if rep > 1:
            cache.note_attention(L, p.reshape(T, self.n_kv_heads, rep, -1).sum(axis=2))
        else:
            cache.note_attention(L, p)
        return np.einsum("qhk,khd->qhd", p, cv).reshape(T, self.n_heads * self.d_head)

    # ----------------------------------------------------------- forward
    def forward(self, tokens, cache, start_pos):
        tokens = np.asarray(tokens, dtype=np.int64).reshape(-1)
        T = tokens.shape[0]
        pos = np.arange(start_pos, start_pos + T)
        H, KV, D = self.n_heads, self.n_kv_heads, self.d_head
        w = self.w
        if self.arch == "gpt2":
            P = self.pre
            h = w[f"{P}wte.weight"][tokens] + w[f"{P}wpe.weight"][pos]
            for L in range(self.n_layers):
                p = f"{P}h.{L}."
                x = self._ln(h, w[p + "ln_1.weight"], w[p + "ln_1.bias"])
                qkv = x @ w[p + "attn.c_attn.weight"] + w[p + "attn.c_attn.bias"]
                q, k, v = (a.reshape(T, H, D) for a in np.split(qkv, 3, axis=-1))
                a = self._attend(L, q, k, v, pos, cache, T)
                h = h + a @ w[p + "attn.c_proj.weight"] + w[p + "attn.c_proj.bias"]
                x = self._ln(h, w[p + "ln_2.weight"], w[p + "ln_2.bias"])
                u = x @ w[p + "mlp.c_fc.weight"] + w[p + "mlp.c_fc.bias"]
                g = 0.5 * u * (1.0 + np.tanh(0.7978845608028654 * (u + 0.044715 * u ** 3)))
                h = h + g @ w[p + "mlp.c_proj.weight"] + w[p + "mlp.c_proj.bias"]
            h = self._ln(h, w[f"{P}ln_f.weight"], w[f"{P}ln_f.bias"])
            return (h @ w[f"{P}wte.weight"].T).astype(np.float32)

        emb = w["model.embed_tokens.weight"]
        h = emb[tokens].astype(np.float32)
        cos, sin = self.rope(pos)
        cos, sin = cos[:, None, :], sin[:, None, :]
        for L in range(self.n_layers):
            p = f"model.layers.{L}.self_attn."
            m = f"model.layers.{L}.mlp."
            x = self._rms(h, w[f"model.layers.{L}.input_layernorm.weight"])
            q = x @ w[p + "q_proj.weight"].T
            k = x @ w[p + "k_proj.weight"].T
            v = x @ w[p + "v_proj.weight"].T
            if w.get(p + "q_proj.bias") is not None:
                q, k, v = q + w[p + "q_proj.bias"], k + w[p + "k_proj.bias"], v + w[p + "v_proj.bias"]
            q = q.reshape(T, H, D)
            k = k.reshape(T, KV, D)
            v = v.reshape(T, KV, D)
            q = q * cos + self._rot(q) * sin
            k = k * cos + self._rot(k) * sin
            a = self._attend(L, q, k, v, pos, cache, T)
            ob = w.get(p + "o_proj.bias")
            h = h + a @ w[p + "o_proj.weight"].T + (ob if ob is not None else 0.0)
            x = self._rms(h, w[f"model.layers.{L}.post_attention_layernorm.weight"])
            gate = x @ w[m + "gate_proj.weight"].T
            h = h + ((gate / (1.0 + np.exp(-gate))) * (x @ w[m + "up_proj.weight"].T)) @ w[m + "down_proj.weight"].T
        h = self._rms(h, w["model.norm.weight"])
        head = w.get("lm_head.weight", emb)
        return (h @ head.T).astype(np.float32)
