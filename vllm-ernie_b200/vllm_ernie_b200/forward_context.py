"""Per-step forward context: attention metadata keyed by layer prefix.

When vLLM is importable its own ``get_forward_context`` is used, so the
module reads the scheduler's metadata exactly as the reference does
(``vllm.forward_context.get_forward_context().attn_metadata[prefix]``).
Otherwise (tests, the bench harness) this module-level context stands in.
"""

from __future__ import annotations

import contextlib
from dataclasses import dataclass, field
from typing import Any


@dataclass
class ForwardContext:
    attn_metadata: Any = None
    no_compile_layers: dict = field(default_factory=dict)


_CTX: ForwardContext | None = None


def _vllm_context():
    try:  # pragma: no cover - depends on the serving environment
        from vllm.forward_context import get_forward_context as vget, is_forward_context_available

        if is_forward_context_available():
            return vget()
    except Exception:
        pass
    return None


def get_forward_context() -> ForwardContext:
    if _CTX is not None:
        return _CTX
    ctx = _vllm_context()
    if ctx is not None:
        return ctx
    raise RuntimeError("no forward context is set")


@contextlib.contextmanager
def set_forward_context(attn_metadata: Any):
    global _CTX
    prev = _CTX
    _CTX = ForwardContext(attn_metadata=attn_metadata)
    try:
        yield _CTX
    finally:
        _CTX = prev
