"""Token sampler oracle (CPU, numpy float32).  Test infrastructure only.

Restates ``Sampler.forward`` (``nanovllm/layers/sampler.py:8-12``) and the
draft proposer's per-step sampling (``nanovllm/spec_decode/draft_proposer.py:505-510``),
which compute the same thing, with the exponential draw injected:

* x = logits.float() / T, T broadcast along the request dim (sampler.py:9,
  draft_proposer.py:507: ``temps`` is (B, 1));
* p = softmax(x) (sampler.py:10) -- ``verify.softmax_with_temp``;
* token = argmax(p / max(E, 1e-10)) with E ~ Exp(1) (sampler.py:11,
  draft_proposer.py:508-509), first index on ties (torch.argmax).
"""

from __future__ import annotations

import numpy as np

from .verify import softmax_with_temp


def sample(logits, temperatures=None, *, exponentials) -> np.ndarray:
    """Tokens (B,) int64 for logits (B, V) (any float dtype, converted to float32)."""
    x = np.asarray(logits, dtype=np.float32)
    p = softmax_with_temp(x, temperatures)
    e = np.maximum(np.asarray(exponentials, dtype=np.float32).reshape(x.shape), np.float32(1e-10))
    return (p / e).astype(np.float32).argmax(axis=-1).astype(np.int64)
