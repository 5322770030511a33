"""B200-native Needle-3 token loop — Python mirror of rustyneedle's Model/Session API.

The compute path is the in-tree native library (``_native/libneedle_b200.so``,
sm_100a kernels behind the C ABI of ``include/needle_b200.h``). There is no CPU
fallback: when the library is missing, importing the native layer raises.

Reference seams mirrored here (paths inside the rustyneedle workspace):
  Model.open / Model.with_depth      crates/model/src/model.rs:52-66
  Session.feed / push / logits / len crates/model/src/session.rs:44-177
  Session.clone                      the prefix cache (crates/generate/src/generator.rs:36-47)
  Session.step / Batch.step          the greedy loop of generator.rs:99-130 with
                                     argmax_allowed and allowed_statistics (147-194)
"""

from __future__ import annotations

from ._native import (  # noqa: F401
    Batch,
    ContextOverflow,
    CrossMemory,
    DepthError,
    Model,
    ModelConfig,
    NeedleError,
    Session,
    StepStats,
    feed_many,
    library_path,
)
from .grammar import TokenAutomaton, call_automaton, literal_automaton, token_table  # noqa: F401

__all__ = ["Model", "Session", "Batch", "ModelConfig", "StepStats", "NeedleError", "DepthError", "ContextOverflow",
           "feed_many", "library_path", "CrossMemory",
           "TokenAutomaton", "call_automaton", "literal_automaton", "token_table"]
