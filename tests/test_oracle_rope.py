"""The RoPE oracle and the table builder, pinned to the reference's own outputs.

``tests/golden/rope_*.npz`` hold what the reference's ``RotaryEmbedding`` and
``apply_rope`` (engine/model.py:169-224) produced on seeded q / k at scattered
positions (``tests/golden/make_golden.py``). The comparisons are on bit patterns.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import rope
from oracle.numerics import f32_to_bf16_bits, to_compute

GOLDEN = Path(__file__).parent / "golden"
CASES = ["fp16_h14_d64", "bf16_h28_d128"]


def _bits(x32: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bfloat16":
        return f32_to_bf16_bits(x32)
    return np.asarray(x32, np.float32).astype(np.float16).view(np.uint16)


def _fixture_bits(a: np.ndarray, dtype: str) -> np.ndarray:
    return a.view(np.uint16) if dtype == "bfloat16" else a.astype(np.float16).view(np.uint16)


@pytest.mark.parametrize("name", CASES)
def test_oracle_rotation_matches_the_reference(name):
    z = np.load(GOLDEN / f"rope_{name}.npz")
    dt = str(z["dtype"])
    cos, sin = to_compute(z["cos"], dt)[:, None, :], to_compute(z["sin"], dt)[:, None, :]
    for x, want in (("q", "q_rot"), ("k", "k_rot")):
        got = rope.apply_rope(to_compute(z[x], dt), cos, sin, dt)
        assert np.array_equal(_bits(got, dt), _fixture_bits(z[want], dt)), f"{name}: {x} differs"


@pytest.mark.parametrize("name", CASES)
def test_oracle_table_rows_cast_as_the_reference(name):
    z = np.load(GOLDEN / f"rope_{name}.npz")
    dt = str(z["dtype"])
    cos, sin = rope.rope_rows(z["cos_f32"], z["sin_f32"], np.arange(len(z["positions"])), dt)
    assert np.array_equal(_bits(cos, dt), _fixture_bits(z["cos"], dt))
    assert np.array_equal(_bits(sin, dt), _fixture_bits(z["sin"], dt))


@pytest.mark.parametrize("name", CASES)
def test_table_builder_reproduces_the_reference_tables(name):
    from mini_inference_b200 import ops

    z = np.load(GOLDEN / f"rope_{name}.npz")
    dt = str(z["dtype"])
    d = z["cos"].shape[1]
    pos = torch.from_numpy(z["positions"])
    cos32, sin32 = ops.rope_tables(d, int(z["max_positions"]), float(z["theta"]), torch.float32, "cpu")
    assert torch.equal(cos32[pos], torch.from_numpy(z["cos_f32"]))
    assert torch.equal(sin32[pos], torch.from_numpy(z["sin_f32"]))
    tdtype = getattr(torch, dt)
    cos, sin = ops.rope_tables(d, int(z["max_positions"]), float(z["theta"]), tdtype, "cpu")
    view = torch.int16 if dt == "bfloat16" else torch.float16
    assert torch.equal(cos[pos].view(view), torch.from_numpy(z["cos"]).view(view))
    assert torch.equal(sin[pos].view(view), torch.from_numpy(z["sin"]).view(view))


def test_qkv_split_follows_the_projection_layout():
    hq, hkv, d, n = 4, 2, 8, 3
    qkv = np.arange(n * (hq + 2 * hkv) * d, dtype=np.float32).reshape(n, -1)
    q, k, v = rope.qkv_split(qkv, hq, hkv, d)
    assert q.shape == (n, hq, d) and k.shape == (n, hkv, d) and v.shape == (n, hkv, d)
    assert q[1, 2, 3] == qkv[1, 2 * d + 3]
    assert k[2, 1, 0] == qkv[2, hq * d + d]
    assert v[0, 1, 7] == qkv[0, (hq + hkv) * d + d + 7]
