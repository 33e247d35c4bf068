"""pkv_rope_append (qkv-post: RoPE fused with the KV append) on the GPU, bit-exact.

Checked against the oracle's restatement of the reference's ``apply_rope``
(``oracle/rope.py``, pinned to the reference's outputs in ``tests/golden``) and
against the reference's eager formula run by torch on the same device, on tables
built the way ``RotaryEmbedding._build`` builds them.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import rope
from oracle.numerics import f32_to_bf16_bits

pytestmark = pytest.mark.gpu

SHAPES = [  # (dtype, hq, hkv, d): Qwen2.5-0.5B fp16 and 7B bf16 attention heads
    (torch.float16, 14, 2, 64),
    (torch.bfloat16, 28, 4, 128),
]


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    return torch.device("cuda", 0)


def _bits(t: torch.Tensor) -> torch.Tensor:
    return t.contiguous().view(torch.int16)


def _oracle_bits(x32: np.ndarray, dtype: torch.dtype) -> torch.Tensor:
    if dtype == torch.bfloat16:
        return torch.from_numpy(f32_to_bf16_bits(x32).view(np.int16))
    return torch.from_numpy(np.asarray(x32, np.float32).astype(np.float16).view(np.int16))


def _np(t: torch.Tensor) -> np.ndarray:
    return t.float().cpu().numpy()


def _eager(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """The reference's apply_rope on one tensor (engine/model.py:214-224), eager on the device."""
    x1, x2 = x.chunk(2, dim=-1)
    return x * cos + torch.cat([-x2, x1], dim=-1) * sin


def _case(dev, dtype, hq, hkv, d, n, seed, max_positions=4096, theta=1e6, extra_cols=0):
    from mini_inference_b200 import ops

    g = torch.Generator(device=dev).manual_seed(seed)
    width = (hq + 2 * hkv) * d
    base = (torch.randn(n, width + extra_cols, generator=g, device=dev) * 2).to(dtype)
    qkv = base[:, :width]  # a row stride other than the width when extra_cols > 0
    positions = torch.randint(0, max_positions, (n,), generator=g, device=dev)
    positions[:2] = torch.tensor([0, max_positions - 1], device=dev)
    cos, sin = ops.rope_tables(d, max_positions, theta, dtype, dev)
    return qkv, positions, cos, sin


@pytest.mark.parametrize("dtype,hq,hkv,d", SHAPES)
@pytest.mark.parametrize("extra_cols", [0, 2])  # 16-byte path; 4-byte path (row stride not a multiple of 8)
def test_rotation_is_bit_exact(dev, dtype, hq, hkv, d, extra_cols):
    from mini_inference_b200 import ops

    n = 67
    qkv, positions, cos, sin = _case(dev, dtype, hq, hkv, d, n, seed=1, extra_cols=extra_cols)
    k = torch.zeros(1, 2, hkv, 16, d, dtype=dtype, device=dev)
    pool = ops.make_pool(k, torch.zeros_like(k))
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    q_out, k_out = ops.rope_append(pool, 0, qkv, positions, cos, sin, hq, k_out=True, status=status)
    ops.raise_device_errors(status)
    # Against the oracle.
    c_rows, s_rows = cos[positions], sin[positions]
    q_want, k_want, _ = rope.rope_append(_np(qkv), positions.cpu().numpy(), _np(c_rows), _np(s_rows), hq, hkv, d,
                                         str(dtype).replace("torch.", ""))
    assert torch.equal(_bits(q_out).cpu(), _oracle_bits(q_want, dtype))
    assert torch.equal(_bits(k_out).cpu(), _oracle_bits(k_want, dtype))
    # Against the reference's eager formula on the same device.
    q, kk, _ = qkv.view(n, hq + 2 * hkv, d).split([hq, hkv, hkv], dim=1)
    c, s = c_rows[:, None, :], s_rows[:, None, :]
    assert torch.equal(_bits(q_out), _bits(_eager(q, c, s)))
    assert torch.equal(_bits(k_out), _bits(_eager(kk, c, s)))
    assert torch.equal(k, torch.zeros_like(k))  # no slot_mapping: the pool is untouched


@pytest.mark.parametrize("dtype,hq,hkv,d", SHAPES)
def test_append_writes_rotated_k_and_v_to_their_slots(dev, dtype, hq, hkv, d):
    from mini_inference_b200 import ops

    n, layers, nb = 40, 2, 9
    qkv, positions, cos, sin = _case(dev, dtype, hq, hkv, d, n, seed=2)
    g = torch.Generator(device=dev).manual_seed(3)
    k = torch.randn(layers, nb + 1, hkv, 16, d, generator=g, device=dev).to(dtype)
    v = torch.randn(layers, nb + 1, hkv, 16, d, generator=g, device=dev).to(dtype)
    k0, v0 = k.clone(), v.clone()
    slots = torch.randperm(nb * 16, generator=torch.Generator().manual_seed(4))[:n].to(dev)
    slots[5] = -1  # skipped
    pool = ops.make_pool(k, v)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    q_out, k_out = ops.rope_append(pool, 1, qkv, positions, cos, sin, hq, slot_mapping=slots, status=status)
    ops.raise_device_errors(status)
    assert k_out is None
    q_want, k_want, v_want = rope.rope_append(_np(qkv), positions.cpu().numpy(), _np(cos[positions]),
                                              _np(sin[positions]), hq, hkv, d, str(dtype).replace("torch.", ""))
    assert torch.equal(_bits(q_out).cpu(), _oracle_bits(q_want, dtype))
    for t in range(n):
        s = int(slots[t])
        if s < 0:
            continue
        got_k, got_v = k[1, s // 16, :, s % 16], v[1, s // 16, :, s % 16]
        assert torch.equal(_bits(got_k).cpu(), _oracle_bits(k_want[t], dtype)), t
        assert torch.equal(_bits(got_v).cpu(), _oracle_bits(v_want[t], dtype)), t
    written = torch.zeros(nb + 1, 16, dtype=torch.bool)
    for s in slots.tolist():
        if s >= 0:
            written[s // 16, s % 16] = True
    untouched = ~written.to(dev)
    assert torch.equal(k[0], k0[0]) and torch.equal(v[0], v0[0])  # other layer
    assert torch.equal(k[1].transpose(1, 2)[untouched], k0[1].transpose(1, 2)[untouched])
    assert torch.equal(v[1].transpose(1, 2)[untouched], v0[1].transpose(1, 2)[untouched])


def test_decode_step_through_rope_then_fused_append(dev):
    """qkv-post in k_out mode feeding pkv_decode_attention's fused append = rotate, append, attend."""
    from mini_inference_b200 import ops
    from oracle.paged_kv import decode_attend
    from oracle.numerics import round_to

    dtype, hq, hkv, d, bs = torch.float16, 14, 2, 64, 16
    ctx = [37, 5, 64]
    tables = [[3, 7, 1], [0], [5, 2, 8, 4, 6]]
    B, cols = len(ctx), max(len(t) for t in tables)
    g = torch.Generator(device=dev).manual_seed(5)
    k = torch.randn(1, 10, hkv, bs, d, generator=g, device=dev).to(dtype)
    v = torch.randn(1, 10, hkv, bs, d, generator=g, device=dev).to(dtype)
    k_before, v_before = k.clone(), v.clone()
    qkv = (torch.randn(B, (hq + 2 * hkv) * d, generator=g, device=dev) * 2).to(dtype)
    cos, sin = ops.rope_tables(d, 4096, 1e6, dtype, dev)
    positions = torch.tensor(ctx, dtype=torch.int64, device=dev)
    pool = ops.make_pool(k, v)
    tab = torch.zeros(B, cols, dtype=torch.int32)
    for i, t in enumerate(tables):
        tab[i, :len(t)] = torch.tensor(t)
    tabs = ops.make_tables(tab.to(dev))
    slot = torch.tensor([tables[i][c // bs] * bs + c % bs for i, c in enumerate(ctx)], dtype=torch.int64, device=dev)
    lens = torch.tensor([c + 1 for c in ctx], dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    q_rot, k_rot = ops.rope_append(pool, 0, qkv, positions, cos, sin, hq, k_out=True, status=status)
    v_new = qkv[:, (hq + hkv) * d:].view(B, hkv, d)  # the v columns, strided rows
    ws = torch.zeros(ops.decode_workspace_bytes(B, hkv, cols, bs, d, hq), dtype=torch.uint8, device=dev)
    out = ops.decode_attention(pool, 0, tabs, q_rot, lens, ws, k_new=k_rot, v_new=v_new, slot_mapping=slot,
                               status=status)
    ops.raise_device_errors(status)
    qw, kw, vw = rope.rope_append(_np(qkv), np.array(ctx), _np(cos[positions]), _np(sin[positions]), hq, hkv, d,
                                  "float16")
    k_after, v_after = _np(k_before[0]), _np(v_before[0])  # the oracle appends into these
    want = decode_attend(k_after, v_after, tables, ctx, qw, kw, vw)
    torch.testing.assert_close(out.float().cpu(), torch.from_numpy(round_to(want, "float16")).float(),
                               atol=2e-3, rtol=2e-3)
    assert torch.equal(_bits(k[0]).cpu(), _oracle_bits(k_after, dtype))
    assert torch.equal(_bits(v[0]).cpu(), _oracle_bits(v_after, dtype))


def test_out_of_range_position_is_reported(dev):
    from mini_inference_b200 import PkvError, ops

    dtype, hq, hkv, d = torch.float16, 14, 2, 64
    qkv, positions, cos, sin = _case(dev, dtype, hq, hkv, d, 4, seed=6, max_positions=128)
    positions[2] = 128
    k = torch.zeros(1, 2, hkv, 16, d, dtype=dtype, device=dev)
    pool = ops.make_pool(k, torch.zeros_like(k))
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.rope_append(pool, 0, qkv, positions, cos, sin, hq, k_out=True, status=status)
    with pytest.raises((IndexError, PkvError)):
        ops.raise_device_errors(status)


@pytest.mark.parametrize("dtype,hq,hkv,d", SHAPES)
def test_contexts_attend_qkv_equals_rope_then_attend(dev, dtype, hq, hkv, d):
    """attend_qkv (qkv-post + kernels) = the reference's apply_rope + attend, bit for bit, pools included."""
    from mini_inference_b200 import PagedKVCache, ops

    def cache():
        return PagedKVCache(2, hkv, d, num_blocks=48, block_size=16, max_seqs=4, max_len=512, dtype=dtype, device=dev)

    ca, cb = cache(), cache()
    cos, sin = ops.rope_tables(d, 4096, 1e6, dtype, dev)
    g = torch.Generator(device=dev).manual_seed(9)
    lengths = [40, 23, 7]
    slots_a = [ca.allocate(n + 1) for n in lengths]
    slots_b = [cb.allocate(n + 1) for n in lengths]
    width = (hq + 2 * hkv) * d
    pa = ca.packed_prefill_context(slots_a, lengths)
    pb = cb.packed_prefill_context(slots_b, lengths)
    for layer in range(2):  # prefill
        qkv = (torch.randn(1, sum(lengths), width, generator=g, device=dev) * 2).to(dtype)
        out_a = pa.attend_qkv(layer, qkv, cos, sin, hq)
        q, k, v = qkv.view(1, -1, hq + 2 * hkv, d).transpose(1, 2).split([hq, hkv, hkv], dim=1)
        c, s = cos[pb.positions][None, None], sin[pb.positions][None, None]
        out_b = pb.attend(layer, _eager(q, c, s), _eager(k, c, s), v)
        assert torch.equal(out_a, out_b)
    pa.commit(), pb.commit()
    for step in range(3):  # decode
        for c_, ss in ((ca, slots_a), (cb, slots_b)):
            for s_ in ss:
                assert c_.ensure_capacity(s_, c_.lengths[s_] + 1)
        da, db = ca.decode_context(slots_a), cb.decode_context(slots_b)
        for layer in range(2):
            qkv = (torch.randn(len(lengths), 1, width, generator=g, device=dev) * 2).to(dtype)
            out_a = da.attend_qkv(layer, qkv, cos, sin, hq)
            q, k, v = qkv.view(len(lengths), 1, hq + 2 * hkv, d).transpose(1, 2).split([hq, hkv, hkv], dim=1)
            c, s = cos[db.positions][:, None, None], sin[db.positions][:, None, None]
            out_b = db.attend(layer, _eager(q, c, s), _eager(k, c, s), v)
            assert torch.equal(out_a, out_b), (step, layer)
        da.commit(), db.commit()
    ca.raise_device_errors(), cb.raise_device_errors()
    assert torch.equal(ca.k, cb.k) and torch.equal(ca.v, cb.v)


@pytest.mark.parametrize("dtype,hq,hkv,d", SHAPES)
def test_decode_attention_rope_equals_rope_then_decode(dev, dtype, hq, hkv, d):
    """pkv_decode_attention_rope (rotation inside the decode kernel) = pkv_rope_append then
    pkv_decode_attention, bit for bit: outputs and the appended rows alike, on the config-2
    micro-benchmark's batch (64 sequences of 128..2048 tokens, rows of a wider buffer)."""
    from mini_inference_b200 import ops
    from tests.test_kernels_gpu import micro_bench_case

    batch = 64 if d == 64 else 16
    ctx, tables, k_pool, v_pool, _, _, _ = micro_bench_case(dev, seed=4, batch=batch, dtype=dtype, hq=hq, hkv=hkv, d=d,
                                                            num_blocks=8192 if d == 128 else 16384, layers=1)
    bs = 16
    cols = max(len(t) for t in tables)
    tab = torch.zeros(batch, cols, dtype=torch.int32)
    for i, t in enumerate(tables):
        tab[i, :len(t)] = torch.tensor(t)
    tabs = ops.make_tables(tab.to(dev))
    slot = torch.tensor([tables[i][c // bs] * bs + c % bs for i, c in enumerate(ctx)], dtype=torch.int64, device=dev)
    lens = torch.tensor([c + 1 for c in ctx], dtype=torch.int32, device=dev)
    positions = lens.to(torch.int64) - 1
    g = torch.Generator(device=dev).manual_seed(8)
    width = (hq + 2 * hkv) * d
    qkv = (torch.randn(batch, width + 8, generator=g, device=dev) * 2).to(dtype)[:, :width]
    cos, sin = ops.rope_tables(d, 4096, 1e6, dtype, dev)
    k2, v2 = k_pool.clone(), v_pool.clone()
    pool_a, pool_b = ops.make_pool(k_pool, v_pool), ops.make_pool(k2, v2)
    ws_a = torch.zeros(ops.decode_workspace_bytes(batch, hkv, cols, bs, d, hq), dtype=torch.uint8, device=dev)
    ws_b = torch.zeros_like(ws_a)
    status = torch.zeros(2, dtype=torch.int32, device=dev)
    fused = ops.decode_attention_rope(pool_a, 0, tabs, qkv, cos, sin, lens, ws_a, slot, status=status[0:1])
    q_rot, k_rot = ops.rope_append(pool_b, 0, qkv, positions, cos, sin, hq, k_out=True, status=status[1:2])
    v_new = qkv[:, (hq + hkv) * d:].view(batch, hkv, d)
    split = ops.decode_attention(pool_b, 0, tabs, q_rot, lens, ws_b, k_new=k_rot, v_new=v_new, slot_mapping=slot,
                                 status=status[1:2])
    ops.raise_device_errors(status[0:1])
    ops.raise_device_errors(status[1:2])
    assert torch.equal(_bits(fused), _bits(split))
    assert torch.equal(_bits(k_pool), _bits(k2)) and torch.equal(_bits(v_pool), _bits(v2))


def test_decode_attention_rope_reports_a_position_past_the_tables(dev):
    from mini_inference_b200 import PkvError, ops

    hq, hkv, d, bs = 14, 2, 64, 16
    k = torch.zeros(1, 9, hkv, bs, d, dtype=torch.float16, device=dev)
    pool = ops.make_pool(k, torch.zeros_like(k))
    tab = torch.arange(8, dtype=torch.int32, device=dev).view(1, 8)
    lens = torch.tensor([100], dtype=torch.int32, device=dev)  # position 99, tables of 64 positions
    cos, sin = ops.rope_tables(d, 64, 1e6, torch.float16, dev)
    qkv = torch.randn(1, (hq + 2 * hkv) * d, device=dev).half()
    ws = torch.zeros(ops.decode_workspace_bytes(1, hkv, 8, bs, d, hq), dtype=torch.uint8, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    slot = torch.tensor([6 * bs + 3], dtype=torch.int64, device=dev)
    ops.decode_attention_rope(pool, 0, ops.make_tables(tab), qkv, cos, sin, lens, ws, slot, status=status)
    with pytest.raises((IndexError, PkvError)):
        ops.raise_device_errors(status)
