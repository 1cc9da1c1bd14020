"""``verify_batch`` rejection-sampling oracle (CPU, numpy float32).  Test infrastructure only.

Restates ``nanovllm/spec_decode/verify.py`` of the reference step by step, with
the two random draws injected instead of drawn inside:

* q = softmax(draft / T) unless the draft is a point mass (:86-89);
  p = softmax(target / T) (:90); T broadcast along the request dim (:178-200).
* candidate j is checked against target row j (:109-111);
  ratio = where(q_tok > 0, min(p_tok / max(q_tok, 1e-10), 1), 0) (:114-118).
* accept_mask = u < ratio with u[b, j] injected (the draw of :120).
* accepted = index of the first rejection, or k if none (:125-129).
* residual row ``a = accepted``: resid = max(p[a] - q_pad[a], 0) with q_pad[k] = 0
  (:141-148); p index clamped to the last target row, q index to k (:143-144);
  fallback to p[a] when the residual sums to 0 (:150-151); normalised with the
  sum clamped at 1e-10 (:152).
* bonus = argmax(resid / max(E, 1e-10)) with E[b, i] injected (the draw of
  :209), first index on ties (torch.argmax).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass
class VerifyResult:
    accepted: np.ndarray      # (B,) int64
    bonus: np.ndarray         # (B,) int64
    n_proposed: np.ndarray    # (B,) int64
    accept_mask: np.ndarray   # (B, k) bool


def softmax_with_temp(logits, temperatures=None) -> np.ndarray:
    """``_softmax_with_temp`` (verify.py:178-200) in float32."""
    x = np.asarray(logits, dtype=np.float32)
    if temperatures is not None:
        t = np.asarray(temperatures, dtype=np.float32)
        if t.ndim == 0:
            x = x / t
        else:
            x = x / t.reshape([t.shape[0]] + [1] * max(0, x.ndim - 1))
    m = x.max(axis=-1, keepdims=True)
    e = np.exp(x - m)
    return (e / e.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)


def verify_batch(draft_probs, target_logits, draft_tokens, temperatures=None,
                 draft_is_point_mass: bool = False, *, uniforms, exponentials) -> VerifyResult:
    draft = np.asarray(draft_probs, dtype=np.float32)
    target = np.asarray(target_logits, dtype=np.float32)
    tok = np.asarray(draft_tokens).astype(np.int64)
    B, k, V = draft.shape
    rows_p = target.shape[1]

    q = draft if draft_is_point_mass else softmax_with_temp(draft, temperatures)
    p = softmax_with_temp(target, temperatures)

    q_tok = np.take_along_axis(q, tok[..., None], axis=2)[..., 0]
    p_tok = np.take_along_axis(p[:, :k, :], tok[..., None], axis=2)[..., 0]
    ratio = np.where(q_tok > 0,
                     np.minimum(p_tok / np.maximum(q_tok, np.float32(1e-10)), np.float32(1.0)),
                     np.float32(0.0)).astype(np.float32)

    u = np.asarray(uniforms, dtype=np.float32).reshape(B, k)
    accept_mask = u < ratio
    rejected = ~accept_mask
    has_reject = rejected.any(axis=1)
    first_reject = rejected.argmax(axis=1)
    accepted = np.where(has_reject, first_reject, k).astype(np.int64)

    p_idx = np.minimum(accepted, rows_p - 1)
    q_idx = np.minimum(accepted, k)
    resid_p = p[np.arange(B), p_idx]                                    # (B, V)
    q_pad = np.concatenate([q, np.zeros_like(q[:, :1, :])], axis=1)
    resid_q = q_pad[np.arange(B), q_idx]
    resid = np.maximum(resid_p - resid_q, np.float32(0.0)).astype(np.float32)
    resid_sum = resid.sum(axis=-1, keepdims=True, dtype=np.float32)
    resid = np.where(resid_sum > 0, resid, resid_p).astype(np.float32)
    z = np.maximum(resid.sum(axis=-1, keepdims=True, dtype=np.float32), np.float32(1e-10))
    probs = (resid / z).astype(np.float32)

    e = np.maximum(np.asarray(exponentials, dtype=np.float32).reshape(B, V), np.float32(1e-10))
    bonus = (probs / e).astype(np.float32).argmax(axis=-1).astype(np.int64)
    return VerifyResult(accepted=accepted, bonus=bonus,
                        n_proposed=np.full((B,), k, dtype=np.int64),
                        accept_mask=accept_mask)


def algorithmic_bytes(B: int, k: int, V: int, target_rows: int | None = None) -> int:
    """One read of every draft and target logit (the sampler's floor)."""
    if target_rows is None:
        target_rows = k + 1
    return B * (k + target_rows) * V * 4
