"""iron_b200: B200 (sm_100a) implementation of IRON's Qwen3 decode hot path.

Operators keep IRON's constructor / arg-spec / callable API (``iron_b200.operators``),
``OperatorSequence`` replays a runlist as a CUDA graph (``iron_b200.sequence``), and
``Qwen3B200`` is the decode runtime (``iron_b200.qwen3``; tensor parallel in
``iron_b200.tp``, batched bf16 Llama decode in ``iron_b200.llama``, GPTQ int8
checkpoints loaded by ``iron_b200.gptq``).  All compute runs in the hand-written
kernels of ``libiron_b200.so`` (C ABI: ``include/iron_b200.h``).
"""

from ._lib import IronError, lib  # noqa: F401
from .base import AIERuntimeArgSpec, Operator, ParamScratchpad  # noqa: F401

__version__ = "0.1.0"
