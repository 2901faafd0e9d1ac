"""Group-wise asymmetric quantization, restated with its codes exposed.

Follows draftkv/compress.py:21-46.  The reference returns only the
dequantized array; the codes q, the per-group scale and the group minimum lo
exist there as locals (:38-43).  This restatement returns all four so the
device quantizer can be checked code-for-code.

Arithmetic (all fp32, numpy's IEEE ops, no fused multiply-add):
    lo = min(g), hi = max(g)                  per group of 64 (zero padded)
    scale = max((hi - lo) / (2^b - 1), 1e-8)
    q = clip(rint((g - lo) / scale), 0, 2^b - 1)      rint = round half even
    deq = q * scale + lo
"""

from __future__ import annotations

import numpy as np

GROUP = 64


def quant_codes(x: np.ndarray, bits: int, group: int = GROUP):
    """Returns (codes uint8 [rows, n_groups*group], scale f32 [rows, n_groups],
    lo f32 [rows, n_groups], deq f32 x.shape).  bits >= 16: codes/scale/lo are
    None and deq is an fp32 copy (compress.py:28-29)."""
    x = np.asarray(x)
    if bits >= 16:
        return None, None, None, x.astype(np.float32, copy=True)
    d = x.shape[-1]
    n_groups = -(-d // group)
    rows = x.reshape(-1, d).astype(np.float32)
    padded = np.zeros((rows.shape[0], n_groups * group), np.float32)
    padded[:, :d] = rows
    grp = padded.reshape(rows.shape[0], n_groups, group)
    lo = grp.min(axis=2, keepdims=True)
    hi = grp.max(axis=2, keepdims=True)
    top = np.float32((1 << bits) - 1)
    scale = np.maximum((hi - lo) / top, np.float32(1e-8))
    q = np.clip(np.rint((grp - lo) / scale), np.float32(0), top)
    deq = (q * scale + lo).reshape(rows.shape[0], -1)[:, :d].reshape(x.shape)
    return (q.astype(np.uint8).reshape(rows.shape[0], -1), scale[:, :, 0],
            lo[:, :, 0], deq)


def quantize(x: np.ndarray, bits: int, group: int = GROUP) -> np.ndarray:
    """Dequantized round trip, the value compress.quantize returns."""
    return quant_codes(x, bits, group)[3]


# --------------------------------------------------------------------------
# Packed storage layout of the device drafter cache (device build's choice;
# only the byte count d*bits/8 is shared with the reference's accounting,
# draftkv/config.py:39-48).
#
# A K or V vector of d elements (d a multiple of 64) is stored as d*bits/8
# bytes.  Elements are reordered for the tensor-core fragment layout of the
# draft-attention kernel: the vector is cut into 16-wide k-steps, and for
# k-step j and lane quad c (0..3) the four elements
#     16j + 2c, 16j + 2c + 1, 16j + 2c + 8, 16j + 2c + 9
# are consecutive; quad c owns one contiguous quarter of the codes, k-steps in
# order.  Bit layout of each quarter:
#   8 bit: one byte per code
#   4 bit: 8 codes per 32-bit word, code 2i at bits [4i, 4i+4), code 2i+1 at
#          bits [16+4i, 20+4i)  (a shift and a mask give two 16-bit lanes)
#   2 bit: 16 codes per word, code 2i at bits [2i, 2i+2), 2i+1 at [16+2i, 18+2i)
#   3 bit: two planes.  Plane A (all four quarters, d/4 bytes) holds the low
#          2 bits in the 2-bit layout; plane B (d/8 bytes) follows and holds the
#          high bit, 16 codes per 16-bit unit, code 2i at bit i, 2i+1 at bit 8+i.
# --------------------------------------------------------------------------
def fragment_order(d: int) -> np.ndarray:
    """Element index stored at each code position of the packed vector."""
    assert d % 64 == 0, "device drafter layout needs d % 64 == 0"
    order = []
    for c in range(4):
        for j in range(d // 16):
            base = 16 * j + 2 * c
            order += [base, base + 1, base + 8, base + 9]
    return np.asarray(order, np.int64)


def code_bytes(d: int, bits: int) -> int:
    return d * bits // 8


def _pack_lanes(v: np.ndarray, bits: int) -> np.ndarray:
    """v [rows, n] uint codes -> uint8 bytes, 2-lane layout of width `bits`."""
    rows, n = v.shape
    per = 32 // bits
    w = v.astype(np.uint32).reshape(rows, n // per, per)
    out = np.zeros((rows, n // per), np.uint32)
    for i in range(per // 2):
        out |= w[:, :, 2 * i] << np.uint32(bits * i)
        out |= w[:, :, 2 * i + 1] << np.uint32(16 + bits * i)
    return out.view(np.uint8).reshape(rows, -1)


def _unpack_lanes(b: np.ndarray, bits: int, n: int) -> np.ndarray:
    rows = b.shape[0]
    per = 32 // bits
    w = np.ascontiguousarray(b).view(np.uint32).reshape(rows, n // per)
    mask = np.uint32((1 << bits) - 1)
    out = np.zeros((rows, n // per, per), np.uint8)
    for i in range(per // 2):
        out[:, :, 2 * i] = (w >> np.uint32(bits * i)) & mask
        out[:, :, 2 * i + 1] = (w >> np.uint32(16 + bits * i)) & mask
    return out.reshape(rows, n)


def pack_codes(codes: np.ndarray, bits: int, k_order: bool = True) -> np.ndarray:
    """codes [rows, d] in element order -> packed bytes [rows, d*bits/8].
    K vectors use the fragment order, V vectors (k_order=False) element order."""
    rows, d = codes.shape
    s = codes[:, fragment_order(d) if k_order else np.arange(d)].astype(np.uint32)   # storage order
    if bits == 8:
        return s.astype(np.uint8)
    if bits in (2, 4):
        return _pack_lanes(s, bits)
    if bits == 3:
        plane_a = _pack_lanes(s & 3, 2)
        hb = (s >> 2).reshape(rows, d // 16, 16)
        units = np.zeros((rows, d // 16), np.uint16)
        for i in range(8):
            units |= (hb[:, :, 2 * i] << i).astype(np.uint16)
            units |= (hb[:, :, 2 * i + 1] << (8 + i)).astype(np.uint16)
        return np.concatenate([plane_a, units.view(np.uint8).reshape(rows, -1)], axis=1)
    raise ValueError(f"bits={bits}")


def unpack_codes(packed: np.ndarray, bits: int, d: int) -> np.ndarray:
    """Inverse of pack_codes (test helper)."""
    rows = packed.shape[0]
    if bits == 8:
        s = packed.astype(np.uint8)
    elif bits in (2, 4):
        s = _unpack_lanes(packed, bits, d)
    elif bits == 3:
        a = _unpack_lanes(packed[:, : d // 4], 2, d)
        u = np.ascontiguousarray(packed[:, d // 4:]).view(np.uint16).reshape(rows, d // 16)
        hb = np.zeros((rows, d // 16, 16), np.uint8)
        for i in range(8):
            hb[:, :, 2 * i] = (u >> i) & 1
            hb[:, :, 2 * i + 1] = (u >> (8 + i)) & 1
        s = (a | (hb.reshape(rows, d) << 2)).astype(np.uint8)
    else:
        raise ValueError(f"bits={bits}")
    codes = np.zeros((rows, d), np.uint8)
    codes[:, fragment_order(d)] = s
    return codes
