"""CPU oracle for the self-speculative decode step -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference algorithm (aabhimittal/Draft-KV, a pure
numpy package), written independently and pinned against golden vectors that
were produced by importing the reference itself (tests/golden/make_golden.py,
checked by tests/test_oracle_golden.py).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may
import this package, and only as the checker or the timed CPU baseline.  The
product path (draft-kv_b200/draftkv) never imports it and fails loudly when its
CUDA library is missing.

Modules
  quant   -- group quantization with codes/scale/lo exposed (compress.py:21-46)
  caches  -- full, compressed (sink+recent+H2O eviction) and paged caches
             (compress.py:49-241, paged.py:29-181)
  models  -- GPT-2 and Llama/Qwen2 forward over the cache protocol
             (gpt2.py:182-213, llama.py:175-225)
  engine  -- draft/verify loop, acceptance, baseline decode (engine.py:36-223)
"""

from .quant import quant_codes, quantize, pack_codes, unpack_codes, code_bytes  # noqa: F401
from .caches import OracleFull, OracleComp, OraclePaged, OraclePool  # noqa: F401
from .models import OracleModel  # noqa: F401
from .engine import OracleEngine, probs_of  # noqa: F401
