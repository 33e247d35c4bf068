"""numpy restatement of the reference's rotary position embedding.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): the checker for
``pkv_rope_append`` in ``mini_inference_b200/csrc/rope_append.cu``.

What it follows in the reference (Ham12-3/mini-inference):

* :func:`apply_rope` -- ``apply_rope`` and ``_rotate_half``
  (``engine/model.py:214-224``): ``x * cos + rotate_half(x) * sin`` with
  ``rotate_half(x) = cat(-x[..., d/2:], x[..., :d/2])``, run as the reference runs
  it: eager tensor ops in the storage dtype, each of which computes in float32
  and rounds its result once to the storage dtype. The two products are exact in
  float32 (fp16 and bf16 significands are short enough), the sum is rounded to
  float32 first and then to the storage dtype, exactly as the eager add does.
* :func:`rope_rows` -- the table lookup of ``RotaryEmbedding.forward``
  (``engine/model.py:201-211``): rows of the float32 cos / sin tables, cast to the
  storage dtype. The tables themselves are inputs here; they come from the
  reference's ``_build`` (``engine/model.py:190-199``), run by torch.
* :func:`qkv_split` -- the split and head views of ``Attention.forward``
  (``engine/model.py:236-249``): a ``qkv_proj`` row is ``[q (Hq*d) | k (Hkv*d) | v (Hkv*d)]``.

Arrays hold stored values: float16 as numpy float16, bfloat16 as float32 holding
the exact bf16 value (see :mod:`oracle.numerics`).
"""

from __future__ import annotations

import numpy as np

from .numerics import bf16_bits_to_f32, f32_to_bf16_bits


def _round(x32: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to the storage dtype; returns float32 holding them exactly."""
    if dtype == "float16":
        return np.asarray(x32, np.float32).astype(np.float16).astype(np.float32)
    if dtype == "bfloat16":
        return bf16_bits_to_f32(f32_to_bf16_bits(np.asarray(x32, np.float32)))
    raise ValueError(f"unsupported dtype {dtype}")


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, dtype: str) -> np.ndarray:
    """``x * cos + rotate_half(x) * sin`` over the last axis (engine/model.py:214-224).

    ``cos``/``sin`` broadcast against ``x`` and hold storage-dtype values. Returns
    float32 holding storage-dtype values.
    """
    x32 = np.asarray(x, np.float32)
    c32 = np.asarray(cos, np.float32)
    s32 = np.asarray(sin, np.float32)
    half = x32.shape[-1] // 2
    rot = np.concatenate([-x32[..., half:], x32[..., :half]], axis=-1)
    a = _round(x32 * c32, dtype)  # q * cos
    b = _round(rot * s32, dtype)  # rotate_half(q) * sin
    return _round(a + b, dtype)  # float32 add, then the storage dtype


def rope_rows(cos_table: np.ndarray, sin_table: np.ndarray, positions: np.ndarray,
              dtype: str) -> tuple[np.ndarray, np.ndarray]:
    """Rows ``positions`` of the float32 tables, cast to the storage dtype (engine/model.py:208-210)."""
    pos = np.asarray(positions, np.int64)
    return (_round(np.asarray(cos_table, np.float32)[pos], dtype),
            _round(np.asarray(sin_table, np.float32)[pos], dtype))


def qkv_split(qkv: np.ndarray, hq: int, hkv: int, d: int) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """``[n, (hq + 2 hkv) d]`` rows -> q ``[n, hq, d]``, k ``[n, hkv, d]``, v ``[n, hkv, d]`` (engine/model.py:236-249)."""
    n = qkv.shape[0]
    q = qkv[:, :hq * d].reshape(n, hq, d)
    k = qkv[:, hq * d:(hq + hkv) * d].reshape(n, hkv, d)
    v = qkv[:, (hq + hkv) * d:(hq + 2 * hkv) * d].reshape(n, hkv, d)
    return q, k, v


def rope_append(qkv: np.ndarray, positions: np.ndarray, cos_rows: np.ndarray, sin_rows: np.ndarray,
                hq: int, hkv: int, d: int, dtype: str) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """The qkv-post step: split, rotate q and k by their token's position; v unchanged.

    ``cos_rows``/``sin_rows`` are ``[n, d]`` (one row per token, storage dtype).
    Returns ``(q_rot [n, hq, d], k_rot [n, hkv, d], v [n, hkv, d])`` as float32.
    """
    q, k, v = qkv_split(np.asarray(qkv, np.float32), hq, hkv, d)
    c = np.asarray(cos_rows, np.float32)[:, None, :]
    s = np.asarray(sin_rows, np.float32)[:, None, :]
    return apply_rope(q, c, s, dtype), apply_rope(k, c, s, dtype), v
