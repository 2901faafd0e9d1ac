"""Drafter-cache compression settings: the arms the controller chooses among.

Same public surface and semantics as the reference's draftkv/config.py:9-119
(CompressionConfig, default_arms, gamma_range, LayerPlan).  A config never
changes emitted tokens -- every drafted token is verified against the full
cache -- it only moves acceptance rate and bytes streamed per draft step.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Iterator, Sequence

_BITS = (2, 3, 4, 8, 16)


@dataclass(frozen=True, order=True)
class CompressionConfig:
    """bits: code width of drafter K/V entries (16 = stored unquantized);
    keep_frac: share of the context the drafter keeps; sink / recent: leading
    and trailing positions that are never evicted.  (config.py:9-52)"""

    bits: int = 16
    keep_frac: float = 1.0
    sink: int = 4
    recent: int = 32

    def __post_init__(self) -> None:
        if self.bits not in _BITS:
            raise ValueError(f"unsupported bits={self.bits}")
        if not (0.0 < self.keep_frac <= 1.0):
            raise ValueError(f"keep_frac must be in (0, 1], got {self.keep_frac}")

    @property
    def lossless(self) -> bool:
        return self.bits == 16 and self.keep_frac >= 1.0

    def bytes_per_entry(self, d_head: int, group: int = 64) -> float:
        """Bytes per (token, head) K or V vector: codes plus an fp16 scale and
        an fp16 zero point per group (config.py:39-48).  This is also the
        device layout's byte count."""
        if self.bits == 16:
            return 2.0 * d_head
        n_groups = max(1, -(-d_head // group))
        return d_head * self.bits / 8.0 + 4.0 * n_groups

    def label(self) -> str:
        tag = "fp16" if self.bits == 16 else f"{self.bits}b"
        return f"{tag}/keep{self.keep_frac:g}"


def default_arms(bits: Sequence[int] = _BITS, keep_fracs: Sequence[float] = (0.25, 0.5, 1.0),
                 sink: int = 4, recent: int = 32) -> list[CompressionConfig]:
    """Cartesian product of bits x keep fractions, sorted (config.py:55-67)."""
    uniq = {(b, k): CompressionConfig(b, k, sink, recent) for b in bits for k in keep_fracs}
    return sorted(uniq.values())


def gamma_range(gamma_max: int = 8) -> Iterator[int]:
    return iter(range(1, gamma_max + 1))


@dataclass(frozen=True)
class LayerPlan:
    """One config per layer (config.py:74-119)."""

    cfgs: tuple[CompressionConfig, ...]

    def __len__(self) -> int:
        return len(self.cfgs)

    def __getitem__(self, i: int) -> CompressionConfig:
        return self.cfgs[i]

    def __iter__(self):
        return iter(self.cfgs)

    def per_layer_bytes(self, ctx: int, n_kv_heads: int, d_head: int) -> float:
        """Exact K+V bytes of the plan, summed layer by layer (config.py:96-106)."""
        tot = 0.0
        for c in self.cfgs:
            kept = min(ctx, max(c.sink + c.recent, int(round(c.keep_frac * ctx))))
            tot += 2.0 * kept * n_kv_heads * c.bytes_per_entry(d_head)
        return tot

    def label(self) -> str:
        labels = [c.label() for c in self.cfgs]
        uniq = sorted(set(labels))
        if len(uniq) == 1:
            return f"plan[{uniq[0]}]"
        return "plan[" + ",".join(f"{u}x{labels.count(u)}" for u in uniq) + "]"

    @classmethod
    def uniform(cls, cfg: CompressionConfig, n_layers: int) -> "LayerPlan":
        return cls((cfg,) * n_layers)


def layer_cfgs(cfg, n_layers: int) -> list[CompressionConfig]:
    """Per-layer configs of a LayerPlan or of one config (engine.py:31-33)."""
    return list(cfg.cfgs) if hasattr(cfg, "cfgs") else [cfg] * n_layers
