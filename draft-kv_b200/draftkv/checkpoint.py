"""Real checkpoints: safetensors files and HuggingFace-style model directories.

Replaces the reference's loaders, draftkv/gpt2.py:25-46 (load_safetensors)
and :167-172 / draftkv/llama.py:153-156 (from_dir) and :228-234
(load_llama).  The file format: an 8-byte little-endian header length, a
JSON header mapping each tensor name to its dtype, shape and [begin, end)
byte offsets in the data section that follows.

`load_safetensors(path)` returns what the reference returns (numpy fp32
arrays, bf16 widened exactly); `load_safetensors(path, device="cuda")`
returns torch tensors in their stored dtype on the device (a bf16 checkpoint
stays bf16: an 8B model is 16 GB, not 32), reading the file through a
memory map.  A directory holds `model.safetensors` or shards listed in
`model.safetensors.index.json`, and `config.json`.  The tokenizers of the
reference are not part of the decode step and are not provided.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np

_NP = {"F32": np.float32, "F16": np.float16, "BF16": np.uint16, "I64": np.int64, "I32": np.int32,
       "U8": np.uint8, "F64": np.float64}


def _header(path: Path):
    with open(path, "rb") as f:
        n = int.from_bytes(f.read(8), "little")
        header = json.loads(f.read(n))
    return header, 8 + n


def load_safetensors(path, device=None) -> dict:
    """Every tensor of one safetensors file: numpy fp32 (device None, the
    reference's behaviour) or torch tensors of the stored dtype on `device`."""
    path = Path(path)
    header, base = _header(path)
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        dt = _NP.get(meta["dtype"])
        if dt is None:
            raise ValueError(f"{path.name}: tensor {name} has unsupported dtype {meta['dtype']}")
        lo, hi = meta["data_offsets"]
        raw = mm[base + lo: base + hi].view(dt).reshape(meta["shape"])
        if device is None:
            if meta["dtype"] == "BF16":
                out[name] = (raw.astype(np.uint32) << 16).view(np.float32)
            elif np.issubdtype(dt, np.floating):
                out[name] = raw.astype(np.float32)
            else:
                out[name] = np.array(raw)
        else:
            import torch
            t = torch.from_numpy(np.array(raw))
            if meta["dtype"] == "BF16":
                t = t.view(torch.bfloat16)
            out[name] = t.to(device)
    return out


def save_safetensors(tensors: dict, path, metadata: dict | None = None) -> None:
    """Writes numpy arrays (float32 / float16 / int) or torch tensors (any of
    those plus bfloat16) as one safetensors file."""
    path = Path(path)
    header, blobs, off = {}, [], 0
    for name, t in tensors.items():
        if hasattr(t, "detach"):                 # torch tensor
            import torch
            t = t.detach().cpu().contiguous()
            if t.dtype == torch.bfloat16:
                arr, code = t.view(torch.uint16).numpy(), "BF16"
            else:
                arr = t.numpy()
                code = None
        else:
            arr, code = np.ascontiguousarray(t), None
        if code is None:
            code = {np.dtype(np.float32): "F32", np.dtype(np.float16): "F16", np.dtype(np.int64): "I64",
                    np.dtype(np.int32): "I32", np.dtype(np.uint8): "U8", np.dtype(np.float64): "F64"}[arr.dtype]
        b = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": code, "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * (-len(h) % 8)                    # keep the data section 8-byte aligned
    with open(path, "wb") as f:
        f.write(len(h).to_bytes(8, "little"))
        f.write(h)
        for b in blobs:
            f.write(b)


def load_dir_weights(d, device=None) -> dict:
    """The weights of a model directory: model.safetensors, or every shard
    named in model.safetensors.index.json."""
    d = Path(d)
    idx = d / "model.safetensors.index.json"
    if idx.exists():
        shards = sorted(set(json.loads(idx.read_text())["weight_map"].values()))
        out = {}
        for s in shards:
            out.update(load_safetensors(d / s, device))
        return out
    f = d / "model.safetensors"
    if not f.exists():
        raise FileNotFoundError(f"no checkpoint at {d} (model.safetensors or model.safetensors.index.json)")
    return load_safetensors(f, device)


def load_config(d) -> dict:
    """config.json of a model directory, with the device build's `dtype`:
    bf16 for bfloat16 / float16 checkpoints, f32 otherwise (unless given)."""
    cfg = json.loads((Path(d) / "config.json").read_text())
    if "n_embd" in cfg:
        cfg.setdefault("vocab_size", 50257)
    stored = str(cfg.get("dtype") or cfg.get("torch_dtype") or "").lower()
    cfg["dtype"] = "bf16" if stored in ("bf16", "bfloat16", "float16", "fp16") else "f32"
    return cfg
