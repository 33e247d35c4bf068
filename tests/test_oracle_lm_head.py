"""The greedy LM-head oracle (``oracle/lm_head.py``) against the reference's own outputs.

``tests/golden/lm_head_*.npz`` hold ``Qwen2ForCausalLM.compute_logits(hidden).float()`` and
the greedy ``Sampler``'s tokens, produced by the reference on the CPU
(``tests/golden/make_golden.py --only lm_head``): a tied fp16 embedding and a separate
bf16 ``lm_head``, vocabularies that are not multiples of 64, an exact tie between two
vocabulary entries and a row of NaN logits.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import lm_head
from oracle.numerics import to_compute

CASES = ["fp16_tied", "bf16"]


def _load(golden_dir, name):
    d = np.load(golden_dir / f"lm_head_{name}.npz")
    dtype = str(d["dtype"])
    return dtype, to_compute(d["hidden"], dtype), to_compute(d["weight"], dtype), d["logits"], d["tokens"]


@pytest.mark.parametrize("name", CASES)
def test_oracle_tokens_match_the_reference(golden_dir, name):
    dtype, h, w, ref_logits, ref_tokens = _load(golden_dir, name)
    ids, top = lm_head.greedy_tokens(h, w, dtype)
    exact = lm_head.exact_logits(h, w)
    finite = np.isfinite(exact).all(axis=1)
    two = -np.partition(-np.where(finite[:, None], exact, 0.0), 1, axis=1)[:, :2]
    amb = lm_head.ambiguous_rows(exact, dtype) & finite & (two[:, 0] != two[:, 1])  # exact ties are not ambiguous
    assert amb.shape == (h.shape[0],)
    assert not amb.any(), "these fixtures were drawn without near-ties"
    np.testing.assert_array_equal(ids, ref_tokens)
    # The rounded logits agree with the reference's to within one ulp of the model dtype.
    r = lm_head.rounded_logits(exact, dtype)
    diff = np.abs(r[finite] - ref_logits[finite])
    assert (diff <= lm_head.ulp(ref_logits[finite], dtype)).all()
    np.testing.assert_array_equal(top[finite], ref_logits[finite].max(axis=1))


@pytest.mark.parametrize("name", CASES)
def test_tie_and_nan_rows(golden_dir, name):
    dtype, h, w, ref_logits, ref_tokens = _load(golden_dir, name)
    vocab = w.shape[0]
    assert ref_logits[1, 3] == ref_logits[1, vocab - 2] == ref_logits[1].max()
    assert ref_tokens[1] == 3  # the first of two equal maxima
    assert np.isnan(ref_logits[-1]).all() and ref_tokens[-1] == 0  # NaN wins; the first one
    ids, _ = lm_head.greedy_tokens(h, w, dtype)
    assert ids[1] == 3 and ids[-1] == 0


def test_first_argmax_rules():
    x = np.array([[1.0, 3.0, 3.0, 2.0], [np.nan, 1.0, np.nan, 5.0], [-np.inf, -np.inf, -np.inf, -np.inf]])
    np.testing.assert_array_equal(lm_head.first_argmax(x), [1, 0, 0])


def test_acceptable_and_ambiguous():
    exact = np.array([[1.0, 1.0 + 2.0 ** -12, 0.0], [2.0, 1.0, 0.5]])
    # fp16 ulp at 1.0 is 2^-10: row 0's two leaders are within it, row 1 is clear.
    np.testing.assert_array_equal(lm_head.ambiguous_rows(exact, "float16"), [True, False])
    np.testing.assert_array_equal(lm_head.acceptable(exact, "float16", np.array([0, 0])), [True, True])
    np.testing.assert_array_equal(lm_head.acceptable(exact, "float16", np.array([2, 1])), [False, False])
