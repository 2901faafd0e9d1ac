"""GPT-2 and Llama/Qwen2 decoders on the device, behind the reference's
model contract  forward(tokens, cache, start_pos) -> logits (T, V).

Constructors take the reference's weight dicts and configs
(draftkv/gpt2.py:130-165 GPT2(weights, config), draftkv/llama.py:112-151
LlamaLike(weights, config)).  At construction the weights are moved to the
device once and re-laid out for the kernels:
  - Llama q/k/v rows concatenated (one QKV GEMM), gate/up interleaved in
    blocks of 64 rows (SwiGLU fused into the GEMM epilogue), every row count
    padded to a multiple of 128, bf16 matrices tiled into mma fragment order;
  - GPT-2 Conv1D matrices ([in, out], x @ W) transposed to [out, in];
  - RoPE cos/sin tables computed in float64 like draftkv/llama.py:164-172.
The forward itself is one native call (dkv_forward) that runs every layer.
"""

from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from .paged import PagedKVCache, dtype_code, torch_dtype

try:
    import torch
except ImportError:  # pragma: no cover
    torch = None


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


class DeviceDecoder:
    """Shared device implementation of both architectures."""

    arch: int = _lib.ARCH_LLAMA

    def __init__(self, weights: dict, config: dict, dtype=None, split_keys: int = 512,
                 max_pos: int | None = None, api_chunk: int = 64, device: str = "cuda") -> None:
        _lib.load()
        self.cfg = config
        self.device = device
        self.split_keys = split_keys
        self.api_chunk = api_chunk
        self.use_graphs = True          # replay repeated forwards as CUDA graphs (forward_raw)
        self._graphs: dict = {}
        self._graph_seen: set = set()
        if dtype is None:
            dtype = config.get("dtype", "f32")
        self.dtype = dtype_code(dtype)
        self.tdt = torch_dtype(self.dtype)
        self._work_cache: dict = {}
        self._parse(config, weights)
        self._build(weights)

    # ------------------------------------------------------------ weights
    def _t(self, a, dtype=None):
        """numpy / torch -> device tensor (model dtype by default)."""
        dt = dtype or self.tdt
        if isinstance(a, torch.Tensor):
            return a.to(self.device, dt).contiguous()
        return torch.from_numpy(np.ascontiguousarray(np.asarray(a, np.float32))).to(self.device, dt)

    def _f32(self, a):
        return None if a is None else self._t(a, torch.float32)

    def _matrix(self, w) -> "torch.Tensor":
        """[M][K] -> kernel layout: rows padded to 128; bf16 tiled."""
        w = self._t(w)
        M, K = w.shape
        Mp = _round_up(M, 128)
        if Mp != M:
            w = torch.cat([w, torch.zeros((Mp - M, K), dtype=w.dtype, device=w.device)], 0)
        if self.dtype == _lib.F32:
            return w.contiguous()
        return _lib.pack_weight(w.contiguous())

    def _pad_bias(self, b, M):
        if b is None:
            return None
        b = self._f32(b)
        Mp = _round_up(M, 128)
        if Mp != b.numel():
            b = torch.cat([b, torch.zeros(Mp - b.numel(), dtype=torch.float32, device=b.device)])
        return b

    def _rope_tables(self, n: int) -> None:
        D = self.d_head
        inv = 1.0 / (self.theta ** (np.arange(0, D, 2) / D))
        ang = np.outer(np.arange(n), inv)
        self.rope_cos = torch.from_numpy(np.cos(ang).astype(np.float32)).to(self.device)
        self.rope_sin = torch.from_numpy(np.sin(ang).astype(np.float32)).to(self.device)
        self.max_pos = n

    # ------------------------------------------------------------ native model
    def _finish_struct(self, tok_emb, pos_emb, head, nf_w, nf_b, layers) -> None:
        self._keep = [tok_emb, pos_emb, head, nf_w, nf_b, layers]
        arr = (_lib.LayerS * self.n_layers)()
        for i, ly in enumerate(layers):
            for name, t in ly.items():
                setattr(arr[i], name, None if t is None else t.data_ptr())
        self._layers_arr = arr
        self._refresh_struct()

    def _refresh_struct(self) -> None:
        tok_emb, pos_emb, head, nf_w, nf_b, _ = self._keep
        cos = getattr(self, "rope_cos", None)
        sin = getattr(self, "rope_sin", None)
        self._s = _lib.ModelS(
            self.arch, self.dtype, self.n_layers, self.d_model, self.n_heads, self.n_kv_heads, self.d_head,
            self.d_ff, self.vocab_size, self.vocab_pad, self.max_pos, float(self.eps),
            tok_emb.data_ptr(), None if pos_emb is None else pos_emb.data_ptr(),
            None if cos is None else cos.data_ptr(), None if sin is None else sin.data_ptr(),
            head.data_ptr(), nf_w.data_ptr(), None if nf_b is None else nf_b.data_ptr(),
            C.cast(self._layers_arr, C.c_void_p), self.split_keys)

    def struct(self) -> "_lib.ModelS":
        return self._s

    @property
    def weight_bytes(self) -> int:
        """Bytes of weights one forward streams (embedding rows are gathered)."""
        tot = 0
        for ly in self._keep[5]:
            for name in ("w_qkv", "w_o", "w_up", "w_down"):
                tot += ly[name].numel() * ly[name].element_size()
        head = self._keep[2]
        return tot + head.numel() * head.element_size()

    # ------------------------------------------------------------ caches
    def new_cache(self, capacity: int = 2048, batch: int = 1):
        from .compress import FullKVCache
        return FullKVCache(self.n_layers, self.n_kv_heads, self.d_head, self.dtype, capacity=capacity, batch=batch)

    def ensure_positions(self, n: int) -> None:
        if self.arch == _lib.ARCH_LLAMA and n > self.max_pos:
            self._rope_tables(max(n, 2 * self.max_pos))
            self._refresh_struct()
        if self.arch == _lib.ARCH_GPT2 and n > self.max_pos:
            raise ValueError(f"position {n - 1} beyond the learned position table ({self.max_pos})")

    def work(self, batch: int, max_T: int, max_ctx: int, comp_cap: int) -> "torch.Tensor":
        key = (batch, max_T, max_ctx, comp_cap)
        w = self._work_cache.get(key)
        if w is None:
            n = _lib.load().dkv_forward_work_bytes(C.byref(self._s), batch, max_T, max_ctx, comp_cap)
            w = torch.zeros(int(n), dtype=torch.uint8, device=self.device)
            self._work_cache[key] = w
        return w

    # ------------------------------------------------------------ forward
    def forward_raw(self, full, comp, tokens_ptr: int, tok_stride: int, pos0: "torch.Tensor", batch: int, T: int,
                    logits: "torch.Tensor", work: "torch.Tensor", max_T: int, max_ctx: int, graph: bool = True) -> None:
        """One native forward for `batch` sequences x T tokens (device pointers);
        `logits` None runs no final norm and head (a prefill chunk).

        With `use_graphs` a forward whose arguments (every address, size and
        the drafter's per-layer configs) have been seen before is replayed as a
        CUDA graph: the second call with given arguments captures it, later
        calls replay it.  The token, position and cache contents are read at
        replay time; only the launch parameters are frozen.  `graph` False
        launches eagerly (prompt chunks: a capture syncs the device and costs
        more than the few launches a replay would save)."""
        step = _lib.StepS(batch, T, tokens_ptr, tok_stride, pos0.data_ptr(), None if logits is None else logits.data_ptr(),
                          work.data_ptr(), work.numel(), max_ctx, max_T)
        fs = None if full is None else full.struct()        # (syncs a changed page table first)
        cs = None if comp is None else comp.struct()

        def run():
            _lib.call("dkv_forward", C.byref(self._s), None if fs is None else C.byref(fs),
                      None if cs is None else C.byref(cs), C.byref(step), _lib.stream_ptr())

        if not (graph and self.use_graphs) or _lib.prof_active:
            run()
            return
        key = (tuple(getattr(step, f) for f, _ in step._fields_),
               None if fs is None else tuple(getattr(fs, f) for f, _ in fs._fields_),
               None if cs is None else (tuple(getattr(cs, f) for f, _ in cs._fields_[:12]), tuple(comp.cfgs)),
               _lib.stream_ptr())
        g = self._graphs.get(key)
        if g is not None:
            g.replay()
            return
        if key not in self._graph_seen:       # first call: eager (sets kernel attributes)
            self._graph_seen.add(key)
            run()
            return
        if len(self._graphs) >= 512:          # stale addresses after reallocations
            self._graphs.clear()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            run()
        self._graphs[key] = g
        g.replay()

    @classmethod
    def from_dir(cls, d, **kw) -> "DeviceDecoder":
        """A model directory (config.json + model.safetensors or shards), as
        the reference's GPT2.from_dir / LlamaLike.from_dir (gpt2.py:167-172,
        llama.py:153-156); weights go straight to the device in their stored
        dtype.  `dtype` overrides the checkpoint's (bf16 for bfloat16 / float16
        checkpoints, f32 otherwise)."""
        from .checkpoint import load_config, load_dir_weights
        cfg = load_config(d)
        if "dtype" in kw:
            cfg["dtype"] = kw.pop("dtype")
        return cls(load_dir_weights(d, device=kw.get("device", "cuda")), cfg, **kw)

    def forward(self, tokens, cache, start_pos: int):
        """Run `tokens` at positions [start_pos, start_pos + T) against `cache`
        (a device FullKVCache / PagedKVCache, or a CompressedKVCache for a
        draft step) and return fp32 logits (T, V) on the device."""
        from .compress import CompressedKVCache, FullKVCache
        toks = np.asarray(tokens, dtype=np.int64).reshape(-1)
        T = int(toks.shape[0])
        self.ensure_positions(start_pos + T)
        logits = torch.empty((T, self.vocab_size), dtype=torch.float32, device=self.device)
        if isinstance(cache, CompressedKVCache):
            if T != 1:
                raise NotImplementedError("draft steps over the compressed cache take one token")
            cache.materialize(self.n_kv_heads, self.d_head, self.dtype)
            cache._grow(cache._hwm_max() + 2)
            tok = torch.tensor(toks, dtype=torch.int32, device=self.device)
            pos0 = torch.tensor([start_pos], dtype=torch.int32, device=self.device)
            w = self.work(1, 1, 16, cache.cap)
            self.forward_raw(None, cache, tok.data_ptr(), 1, pos0, 1, 1, logits, w, 1, 16)
            return logits
        if isinstance(cache, FullKVCache):
            cache.materialize(self.n_kv_heads, self.d_head, self.dtype)
            cache.grow(start_pos + T)
        if not isinstance(cache, PagedKVCache):
            raise TypeError("device models need a device cache (FullKVCache / PagedKVCache / CompressedKVCache)")
        if cache.dtype != self.dtype:
            raise TypeError("cache dtype differs from the model dtype")
        if cache.length != start_pos:
            raise ValueError(f"the device cache appends at its end (length {cache.length}, start_pos {start_pos})")
        cache.ensure(0, start_pos + T)
        tok = torch.tensor(toks, dtype=torch.int32, device=self.device)
        CH = self.api_chunk
        w = self.work(cache.batch, CH, cache.capacity_tokens, 0)
        for c0 in range(0, T, CH):
            c1 = min(T, c0 + CH)
            pos0 = torch.tensor([start_pos + c0] + [0] * (cache.batch - 1), dtype=torch.int32, device=self.device)
            self.forward_raw(cache, None, tok.data_ptr() + 4 * c0, c1 - c0, pos0, 1, c1 - c0, logits[c0:c1], w, CH,
                             cache.capacity_tokens)
            cache.set_length(0, start_pos + c1)
        return logits


class LlamaLike(DeviceDecoder):
    """Llama / Qwen2 decoder (draftkv/llama.py:112-225): RoPE, GQA, RMSNorm,
    SwiGLU, optional q/k/v bias, tied head when lm_head.weight is absent."""

    arch = _lib.ARCH_LLAMA

    def _parse(self, c: dict, w: dict) -> None:
        self.n_layers = c["num_hidden_layers"]
        self.d_model = c["hidden_size"]
        self.n_heads = c["num_attention_heads"]
        self.n_kv_heads = c.get("num_key_value_heads", self.n_heads)
        self.d_head = c.get("head_dim") or self.d_model // self.n_heads
        self.n_rep = self.n_heads // self.n_kv_heads
        self.vocab_size = c["vocab_size"]
        self.eps = c.get("rms_norm_eps", 1e-5)
        self.theta = float(c.get("rope_theta") or 10000.0)
        self.d_ff = c.get("intermediate_size") or w["model.layers.0.mlp.gate_proj.weight"].shape[0]
        if self.d_ff % 64:
            raise ValueError("intermediate_size must be a multiple of 64")

    def _build(self, w: dict) -> None:
        H, KV, D, F = self.n_heads, self.n_kv_heads, self.d_head, self.d_ff
        layers = []
        for i in range(self.n_layers):
            p = f"model.layers.{i}."
            cat = torch.cat if isinstance(w[p + "self_attn.q_proj.weight"], torch.Tensor) else np.concatenate
            qkv = cat([w[p + "self_attn.q_proj.weight"], w[p + "self_attn.k_proj.weight"],
                       w[p + "self_attn.v_proj.weight"]], 0)
            qb = w.get(p + "self_attn.q_proj.bias")
            bqkv = None
            if qb is not None:
                bqkv = self._pad_bias(np.concatenate([np.asarray(qb, np.float32),
                                                      np.asarray(w[p + "self_attn.k_proj.bias"], np.float32),
                                                      np.asarray(w[p + "self_attn.v_proj.bias"], np.float32)]),
                                      (H + 2 * KV) * D)
            gate = self._t(w[p + "mlp.gate_proj.weight"])
            up = self._t(w[p + "mlp.up_proj.weight"])
            gu = torch.stack([gate.view(F // 64, 64, -1), up.view(F // 64, 64, -1)], 1).reshape(2 * F, -1)
            del gate, up
            ob = w.get(p + "self_attn.o_proj.bias")
            layers.append(dict(
                n1_w=self._f32(w[p + "input_layernorm.weight"]), n1_b=None,
                w_qkv=self._matrix(qkv), b_qkv=bqkv,
                w_o=self._matrix(w[p + "self_attn.o_proj.weight"]), b_o=None if ob is None else self._pad_bias(ob, self.d_model),
                n2_w=self._f32(w[p + "post_attention_layernorm.weight"]), n2_b=None,
                w_up=self._matrix(gu), b_up=None,
                w_down=self._matrix(w[p + "mlp.down_proj.weight"]), b_down=None))
            del gu, qkv
        emb = w["model.embed_tokens.weight"]
        head_src = w.get("lm_head.weight")
        tok_emb = self._t(emb)
        head = self._matrix(emb if head_src is None else head_src)
        self.vocab_pad = _round_up(self.vocab_size, 128)     # head rows (padded to whole row tiles)
        self._rope_tables(int(self.cfg.get("max_position_embeddings", 0) or 4096))
        self._finish_struct(tok_emb, None, head, self._f32(w["model.norm.weight"]), None, layers)


class GPT2(DeviceDecoder):
    """GPT-2 (draftkv/gpt2.py:130-213): learned positions, LayerNorm,
    gelu_new, Conv1D x @ W + b, MHA, tied head."""

    arch = _lib.ARCH_GPT2

    def _parse(self, c: dict, w: dict) -> None:
        self.n_layers = c["n_layer"]
        self.n_heads = c["n_head"]
        self.n_kv_heads = self.n_heads
        self.n_rep = 1
        self.d_model = c["n_embd"]
        self.d_head = self.d_model // self.n_heads
        self.vocab_size = c.get("vocab_size", 50257)
        self.eps = c.get("layer_norm_epsilon", 1e-5)
        self.pre = "transformer." if "transformer.wte.weight" in w else ""
        self.d_ff = w[f"{self.pre}h.0.mlp.c_fc.weight"].shape[1]
        self.max_pos = w[f"{self.pre}wpe.weight"].shape[0]

    def _build(self, w: dict) -> None:
        P = self.pre
        layers = []

        def T(a):   # Conv1D [in, out] -> [out, in]
            return a.t() if isinstance(a, torch.Tensor) else np.asarray(a).T

        for i in range(self.n_layers):
            p = f"{P}h.{i}."
            layers.append(dict(
                n1_w=self._f32(w[p + "ln_1.weight"]), n1_b=self._f32(w[p + "ln_1.bias"]),
                w_qkv=self._matrix(T(w[p + "attn.c_attn.weight"])),
                b_qkv=self._pad_bias(w[p + "attn.c_attn.bias"], 3 * self.d_model),
                w_o=self._matrix(T(w[p + "attn.c_proj.weight"])),
                b_o=self._pad_bias(w[p + "attn.c_proj.bias"], self.d_model),
                n2_w=self._f32(w[p + "ln_2.weight"]), n2_b=self._f32(w[p + "ln_2.bias"]),
                w_up=self._matrix(T(w[p + "mlp.c_fc.weight"])),
                b_up=self._pad_bias(w[p + "mlp.c_fc.bias"], self.d_ff),
                w_down=self._matrix(T(w[p + "mlp.c_proj.weight"])),
                b_down=self._pad_bias(w[p + "mlp.c_proj.bias"], self.d_model)))
        wte = w[f"{P}wte.weight"]
        tok_emb = self._t(wte)
        head = self._matrix(wte)
        self.vocab_pad = _round_up(self.vocab_size, 128)     # head rows (padded to whole row tiles)
        pos_emb = self._t(w[f"{P}wpe.weight"])
        self._finish_struct(tok_emb, pos_emb, head, self._f32(w[f"{P}ln_f.weight"]), self._f32(w[f"{P}ln_f.bias"]),
                            layers)


def random_device_weights(cfg: dict, seed: int = 0, std: float = 0.02, device: str = "cuda") -> dict:
    """N(0, std) weights generated on the device from a seeded torch generator,
    norm gains 1, biases 0 (the benchmark's random init for shapes too large
    for numpy).  Keys and shapes follow the reference's checkpoints; dtype is
    the config's (bf16 / f32)."""
    g = torch.Generator(device=device).manual_seed(seed)
    dt = torch.bfloat16 if cfg.get("dtype", "bf16") == "bf16" else torch.float32

    def R(*shape):
        return (torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std).to(dt)

    def ones(n):
        return torch.ones(n, device=device, dtype=torch.float32)

    w = {}
    if cfg["arch"] == "llama":
        d, L, V = cfg["hidden_size"], cfg["num_hidden_layers"], cfg["vocab_size"]
        H, KV = cfg["num_attention_heads"], cfg["num_key_value_heads"]
        D = cfg.get("head_dim") or d // H
        F = cfg["intermediate_size"]
        w["model.embed_tokens.weight"] = R(V, d)
        w["model.norm.weight"] = ones(d)
        for i in range(L):
            p = f"model.layers.{i}."
            w[p + "input_layernorm.weight"] = ones(d)
            w[p + "post_attention_layernorm.weight"] = ones(d)
            w[p + "self_attn.q_proj.weight"] = R(H * D, d)
            w[p + "self_attn.k_proj.weight"] = R(KV * D, d)
            w[p + "self_attn.v_proj.weight"] = R(KV * D, d)
            w[p + "self_attn.o_proj.weight"] = R(d, H * D)
            w[p + "mlp.gate_proj.weight"] = R(F, d)
            w[p + "mlp.up_proj.weight"] = R(F, d)
            w[p + "mlp.down_proj.weight"] = R(d, F)
        if not cfg.get("tie_word_embeddings", True):
            w["lm_head.weight"] = R(V, d)
    else:
        d, L, V, F = cfg["n_embd"], cfg["n_layer"], cfg["vocab_size"], cfg["n_inner"]
        zeros = lambda n: torch.zeros(n, device=device, dtype=torch.float32)  # noqa: E731
        w["wte.weight"] = R(V, d)
        w["wpe.weight"] = R(cfg["n_positions"], d)
        for i in range(L):
            p = f"h.{i}."
            w[p + "ln_1.weight"], w[p + "ln_1.bias"] = ones(d), zeros(d)
            w[p + "attn.c_attn.weight"], w[p + "attn.c_attn.bias"] = R(d, 3 * d), zeros(3 * d)
            w[p + "attn.c_proj.weight"], w[p + "attn.c_proj.bias"] = R(d, d), zeros(d)
            w[p + "ln_2.weight"], w[p + "ln_2.bias"] = ones(d), zeros(d)
            w[p + "mlp.c_fc.weight"], w[p + "mlp.c_fc.bias"] = R(d, F), zeros(F)
            w[p + "mlp.c_proj.weight"], w[p + "mlp.c_proj.bias"] = R(F, d), zeros(d)
        w["ln_f.weight"], w["ln_f.bias"] = ones(d), zeros(d)
    return w


def load_llama(d):
    """(model, tokenizer) for a Llama / Qwen2 checkpoint directory
    (llama.py:228-234); the tokenizer is not part of the device build and is
    returned as None."""
    from pathlib import Path
    if not (Path(d) / "model.safetensors").exists() and not (Path(d) / "model.safetensors.index.json").exists():
        raise FileNotFoundError(f"no checkpoint at {d}")
    return LlamaLike.from_dir(d), None


def from_config(weights: dict, config: dict, **kw) -> DeviceDecoder:
    """GPT2 or LlamaLike by the config's keys."""
    return (GPT2 if "n_embd" in config else LlamaLike)(weights, config, **kw)
