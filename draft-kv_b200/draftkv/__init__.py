"""draftkv (B200 build) -- self-speculative decoding with a compressed-KV drafter.

Drop-in for the reference package's decode path (aabhimittal/Draft-KV,
draftkv/__init__.py:8-58): the same names for the engine, the caches, the
compression configs, the controllers and the cost model.  The model forward,
the caches and acceptance run on the GPU through libdraftkv_b200.so (sm_100a);
the controller and the cost model stay on the host.  Importing needs no GPU;
the first device operation raises DraftKVError when the library or the
device is missing (there is no CPU fallback).
"""

from .config import CompressionConfig, LayerPlan, default_arms, gamma_range
from .controller import (DepthThompsonController, FixedPolicy, FlatBandit,
                         OraclePolicy, ThompsonController)
from .throughput import (CostModel, best_gamma, best_gamma_profile, expected_tokens,
                         expected_tokens_profile)
from .paged import BlockPool, BlockPoolExhausted, PagedKVCache, plan_blocks_needed
from .adaptive import AdaptiveLayerController
from .layers import SensitivityProfile, allocate
from ._lib import DraftKVError

_DEVICE_NAMES = {
    "quantize": ".compress", "quantize_codes": ".compress", "FullKVCache": ".compress",
    "CompressedKVCache": ".compress", "DraftKVEngine": ".engine", "GenerationResult": ".engine",
    "RoundLog": ".engine", "GPT2": ".models", "LlamaLike": ".models", "from_config": ".models",
    "load_llama": ".models", "load_safetensors": ".checkpoint", "save_safetensors": ".checkpoint",
}


def __getattr__(name):
    mod = _DEVICE_NAMES.get(name)
    if mod is None:
        raise AttributeError(name)
    import importlib
    return getattr(importlib.import_module(mod, __name__), name)


__all__ = [
    "AdaptiveLayerController", "SensitivityProfile", "allocate",
    "BlockPool", "BlockPoolExhausted", "CompressedKVCache", "CompressionConfig", "CostModel",
    "DepthThompsonController", "DraftKVEngine", "DraftKVError", "FixedPolicy", "FlatBandit",
    "FullKVCache", "GPT2", "GenerationResult", "LayerPlan", "LlamaLike", "OraclePolicy",
    "PagedKVCache", "RoundLog", "ThompsonController", "best_gamma", "best_gamma_profile",
    "default_arms", "expected_tokens", "expected_tokens_profile", "from_config", "gamma_range",
    "plan_blocks_needed", "quantize", "quantize_codes", "load_llama", "load_safetensors", "save_safetensors",
]
__version__ = "0.1.0"
