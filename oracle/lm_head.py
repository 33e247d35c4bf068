"""numpy restatement of the reference's greedy next-token choice.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): the checker for
``pkv_lm_head_argmax`` in ``mini_inference_b200/csrc/lm_head_argmax.cu``.

What it follows in the reference (Ham12-3/mini-inference):

* ``Qwen2ForCausalLM.compute_logits`` (``engine/model.py:321-323``):
  ``F.linear(hidden, weight)`` in the model dtype -- a float32-accumulated dot product
  per (row, vocab entry), rounded once to the model dtype -- then ``.float()``
  (``engine/engine.py:97,106,123``).
* ``Sampler.__call__`` for an all-greedy batch (``engine/sampler.py:27-31``):
  ``logits.argmax(dim=-1)``, the first index among equal maxima (torch's rule; NaN
  counts as the largest).

:func:`greedy_tokens` computes the dot products exactly (float64), rounds them to
float32 and then to the model dtype, and takes the first maximum. A real float32
accumulator (cuBLAS, CPU BLAS, the tensor cores) differs from the exact sum by a few
float32 ulps, which can move a logit that sits on a rounding boundary of the 16-bit
dtype by one of its ulps; :func:`ambiguous_rows` names the rows where that can change
the winner, and the tests accept either candidate there.

Arrays: float16 as numpy float16; bfloat16 as float32 holding the exact bf16 value
(see :mod:`oracle.numerics`).
"""

from __future__ import annotations

import numpy as np

from .numerics import round_to


def exact_logits(hidden: np.ndarray, weight: np.ndarray) -> np.ndarray:
    """``hidden [B, H] . weight [V, H]^T`` in float64 (exact for these inputs up to float64 rounding)."""
    return np.asarray(hidden, np.float64) @ np.asarray(weight, np.float64).T


def rounded_logits(exact: np.ndarray, dtype: str) -> np.ndarray:
    """Model-dtype logits as ``F.linear`` stores them (float32 accumulator, one rounding), as float64."""
    return round_to(np.asarray(exact, np.float32), dtype)


def first_argmax(logits: np.ndarray) -> np.ndarray:
    """torch.argmax(dim=-1): the first maximal index per row; a NaN row entry wins (the first NaN)."""
    logits = np.asarray(logits, np.float64)
    ids = np.argmax(logits, axis=-1)  # numpy also returns the first maximum
    nan = np.isnan(logits)
    has_nan = nan.any(axis=-1)
    ids[has_nan] = np.argmax(nan[has_nan], axis=-1)
    return ids.astype(np.int64)


def greedy_from_exact(exact: np.ndarray, dtype: str) -> tuple[np.ndarray, np.ndarray]:
    """(token ids int64 [B], the largest rounded logit of each row as float64) from exact logits."""
    r = rounded_logits(exact, dtype)
    ids = first_argmax(r)
    return ids, r[np.arange(r.shape[0]), ids]


def greedy_tokens(hidden: np.ndarray, weight: np.ndarray, dtype: str) -> tuple[np.ndarray, np.ndarray]:
    """(token ids int64 [B], the largest rounded logit of each row as float64)."""
    return greedy_from_exact(exact_logits(hidden, weight), dtype)


def ulp(x: np.ndarray, dtype: str) -> np.ndarray:
    """Spacing of the model dtype at |x| (its normal range; subnormal spacing below it)."""
    mant = {"float16": 10, "bfloat16": 7, "float32": 23}[dtype]
    emin = {"float16": -14, "bfloat16": -126, "float32": -126}[dtype]
    e = np.floor(np.log2(np.maximum(np.abs(np.asarray(x, np.float64)), 2.0 ** emin)))
    return 2.0 ** (e - mant)


def acceptable(exact: np.ndarray, dtype: str, got: np.ndarray, slack_ulps: float = 1.0) -> np.ndarray:
    """Per row: is ``got`` a token the reference could return for these logits?

    True when the exact logit of ``got`` is within ``slack_ulps`` model-dtype ulps (at the
    row's maximum) of the row's largest exact logit: any float32-accumulated GEMM rounds
    both to the same or to adjacent 16-bit values, so either may be the first maximum.
    """
    exact = np.asarray(exact, np.float64)
    rows = np.arange(exact.shape[0])
    top = exact.max(axis=-1)
    return exact[rows, got] >= top - slack_ulps * ulp(top, dtype)


def ambiguous_rows(exact: np.ndarray, dtype: str, slack_ulps: float = 1.0) -> np.ndarray:
    """Rows whose runner-up exact logit is within ``slack_ulps`` ulps of the maximum."""
    exact = np.asarray(exact, np.float64)
    part = -np.partition(-exact, 1, axis=-1)
    top, second = part[:, 0], part[:, 1]
    return second >= top - slack_ulps * ulp(top, dtype)
