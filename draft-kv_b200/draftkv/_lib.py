"""ctypes binding of libdraftkv_b200.so (the C ABI in include/draftkv_b200.h).

The library is loaded on first use.  There is no CPU fallback: a missing
library or a machine without a CUDA device raises DraftKVError as soon as a
device operation is requested.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libdraftkv_b200.so"

OK, EINVAL, ECUDA, EUNSUPPORTED, EDEVICE = 0, 1, 2, 3, 4
F32, BF16 = 0, 1
ARCH_LLAMA, ARCH_GPT2 = 0, 1
EPI_STORE, EPI_RESADD, EPI_GELU, EPI_SWIGLU, EPI_QKV = 0, 1, 2, 3, 4

vp = C.c_void_p


class DraftKVError(RuntimeError):
    """A device call failed (bad argument, CUDA error, unsupported shape)."""


class FullCacheS(C.Structure):
    _fields_ = [("k_pool", vp), ("v_pool", vp), ("page_table", vp),
                ("n_pages", C.c_int), ("page_size", C.c_int), ("max_pages", C.c_int), ("dtype", C.c_int)]


class CompCacheS(C.Structure):
    _fields_ = [("k_codes", vp), ("v_codes", vp), ("k_sl", vp), ("v_sl", vp), ("pos", vp),
                ("score", vp), ("mass", vp), ("meta", vp), ("seen", vp), ("tickets", vp),
                ("cap", C.c_int), ("cb_max", C.c_int),
                ("bits", vp), ("keep", vp), ("sink", vp), ("recent", vp)]


class DimsS(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("n_kv", C.c_int), ("d", C.c_int), ("batch", C.c_int)]


class EpilogueS(C.Structure):
    _fields_ = [("kind", C.c_int), ("bias", vp), ("out_f32", vp), ("act", vp),
                ("act_dtype", C.c_int), ("ld_out", C.c_int),
                ("n_heads", C.c_int), ("n_kv", C.c_int), ("d_head", C.c_int), ("tokens_per_seq", C.c_int),
                ("pos0", vp), ("rope_cos", vp), ("rope_sin", vp), ("q_out", vp), ("kv_stage", vp),
                ("full", vp), ("layer", C.c_int), ("n_layers", C.c_int),
                ("norm_in_part", vp), ("norm_n_part", C.c_int), ("norm_ld", C.c_int), ("norm_dm", C.c_int),
                ("norm_eps", C.c_float), ("norm_out_part", vp), ("norm_out_x", vp), ("norm_out_w", vp)]


class LayerS(C.Structure):
    _fields_ = [(n, vp) for n in ("n1_w", "n1_b", "w_qkv", "b_qkv", "w_o", "b_o", "n2_w", "n2_b",
                                   "w_up", "b_up", "w_down", "b_down")]


class ModelS(C.Structure):
    _fields_ = [("arch", C.c_int), ("dtype", C.c_int), ("n_layers", C.c_int), ("d_model", C.c_int),
                ("n_heads", C.c_int), ("n_kv", C.c_int), ("d_head", C.c_int), ("d_ff", C.c_int),
                ("vocab", C.c_int), ("vocab_pad", C.c_int), ("max_pos", C.c_int), ("eps", C.c_float),
                ("tok_emb", vp), ("pos_emb", vp), ("rope_cos", vp), ("rope_sin", vp), ("w_head", vp),
                ("nf_w", vp), ("nf_b", vp), ("layers", vp), ("split_keys", C.c_int)]


class StepS(C.Structure):
    _fields_ = [("batch", C.c_int), ("T", C.c_int), ("tokens", vp), ("tok_stride", C.c_int),
                ("pos0", vp), ("logits", vp), ("work", vp), ("work_bytes", C.c_size_t),
                ("max_ctx", C.c_int), ("max_T", C.c_int)]


_SIGS = {
    "dkv_last_error": (C.c_char_p, []),
    "dkv_version": (C.c_int, []),
    "dkv_device_error": (C.c_int, [C.POINTER(C.c_uint32), vp]),
    "dkv_prof_start": (C.c_int, [C.c_int]),
    "dkv_prof_stop": (C.c_int, []),
    "dkv_prof_summary": (C.c_int, [C.c_int, C.POINTER(C.c_double), C.POINTER(C.c_int64), C.POINTER(C.c_double)]),
    "dkv_quantize": (C.c_int, [vp, C.c_int64, C.c_int, C.c_int, vp, vp, vp, vp, vp]),
    "dkv_quantize_pack": (C.c_int, [vp, C.c_int, C.c_int64, C.c_int, C.c_int, C.c_int, vp, vp, vp]),
    "dkv_full_write": (C.c_int, [C.POINTER(FullCacheS), DimsS, C.c_int, vp, C.c_int, vp, vp, vp]),
    "dkv_full_read": (C.c_int, [C.POINTER(FullCacheS), DimsS, C.c_int, C.c_int, C.c_int, vp, vp]),
    "dkv_comp_append": (C.c_int, [C.POINTER(CompCacheS), C.POINTER(FullCacheS), DimsS, C.c_int, C.c_int,
                                  vp, C.c_int, C.c_int, vp, vp, vp, C.c_int, vp]),
    "dkv_comp_rebuild": (C.c_int, [C.POINTER(CompCacheS), C.POINTER(FullCacheS), DimsS, vp, C.c_int, vp,
                                   C.c_int, vp]),
    "dkv_comp_read": (C.c_int, [C.POINTER(CompCacheS), DimsS, C.c_int, C.c_int, C.c_int, vp, vp, vp, vp,
                                C.POINTER(C.c_int), vp]),
    "dkv_attn_full": (C.c_int, [C.POINTER(FullCacheS), DimsS, C.c_int, C.c_int, C.c_int, vp, vp, vp, C.c_int,
                                C.c_int, vp, C.c_size_t, vp]),
    "dkv_attn_comp": (C.c_int, [C.POINTER(CompCacheS), DimsS, C.c_int, C.c_int, vp, vp, vp, C.c_int, vp,
                                C.c_size_t, vp]),
    "dkv_attn_work_bytes": (C.c_size_t, [DimsS, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]),
    "dkv_pack_weight_bytes": (C.c_size_t, [C.c_int, C.c_int]),
    "dkv_pack_weight": (C.c_int, [vp, C.c_int, C.c_int, vp, vp]),
    "dkv_gemm": (C.c_int, [vp, C.c_int, vp, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(EpilogueS), vp,
                           C.c_size_t, vp]),
    "dkv_gemm_work_bytes": (C.c_size_t, [C.c_int, C.c_int, C.c_int, C.c_int]),
    "dkv_gemm_noalloc": (C.c_int, [vp, C.c_int, vp, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(EpilogueS),
                                   vp]),
    "dkv_embed": (C.c_int, [vp, C.c_int, vp, vp, C.c_int, C.c_int, C.c_int, vp, C.c_int, C.c_int, C.c_int,
                            vp, vp]),
    "dkv_norm": (C.c_int, [vp, C.c_int, C.c_int, C.c_int, vp, vp, C.c_float, vp, C.c_int, vp]),
    "dkv_sample": (C.c_int, [vp, C.c_int, C.c_int, C.c_float, C.c_uint64, vp, vp, C.c_int, vp, C.c_size_t, vp]),
    "dkv_accept": (C.c_int, [vp, vp, C.c_int, C.c_int, C.c_int, C.c_float, C.c_uint64, vp, vp, C.c_int, vp,
                             vp, vp, vp, vp, vp, vp, vp, C.c_size_t, vp]),
    "dkv_sample_work_bytes": (C.c_size_t, [C.c_int, C.c_int]),
    "dkv_forward_work_bytes": (C.c_size_t, [C.POINTER(ModelS), C.c_int, C.c_int, C.c_int, C.c_int]),
    "dkv_forward": (C.c_int, [C.POINTER(ModelS), C.POINTER(FullCacheS), C.POINTER(CompCacheS),
                              C.POINTER(StepS), vp]),
}

_lib: C.CDLL | None = None


def load(require_device: bool = True) -> C.CDLL:
    """The loaded library; raises DraftKVError when it cannot be used."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise DraftKVError(
                f"{LIB_PATH.name} is not built: run `python draft-kv_b200/build.py` "
                "(there is no CPU fallback)")
        lib = C.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    if require_device:
        import torch
        if not torch.cuda.is_available():
            raise DraftKVError("draftkv_b200 needs a CUDA device (B200, sm_100a); none is visible")
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGS)


def check(status: int, what: str = "") -> None:
    if status != OK:
        msg = _lib.dkv_last_error().decode(errors="replace") if _lib else ""
        raise DraftKVError(f"{what or 'draftkv call'} failed (status {status}): {msg}")


# True between dkv_prof_start and dkv_prof_stop issued through call(): the
# engine does not replay CUDA graphs then, so every launch is timed.
prof_active = False


def call(name: str, *args) -> None:
    global prof_active
    lib = load()
    check(getattr(lib, name)(*args), name)
    if name == "dkv_prof_start":
        prof_active = True
    elif name == "dkv_prof_stop":
        prof_active = False


def ptr(t) -> int | None:
    """Device (or host) address of a torch tensor, None for None."""
    return None if t is None else t.data_ptr()


def pack_weight(w):
    """bf16 weight [M][K] (M a multiple of 128) -> its packed tensor-core
    layout (dkv_pack_weight), a flat bf16 device tensor."""
    import torch
    M, K = w.shape
    out = torch.empty(int(load().dkv_pack_weight_bytes(M, K)) // 2, dtype=torch.bfloat16, device=w.device)
    call("dkv_pack_weight", w.data_ptr(), M, K, out.data_ptr(), stream_ptr())
    return out


def stream_ptr() -> int:
    import torch
    return torch.cuda.current_stream().cuda_stream
