"""The drop-in cache end to end on a B200: the reference's test scenarios through this package's API.

Mirrors tests/test_kv_cache.py:120-142 and :179-207 of the reference (packed
prefill = each prompt alone; paged decode over scattered blocks = per-sequence
attention), at the micro-benchmark head shape in fp16, checked against the
numpy oracle; plus prefix-cache hits, preemption-style free/reuse, and CUDA
graph capture of the decode step.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.numerics import round_to
from oracle.paged_kv import decode_attend, packed_prefill_attend

pytestmark = pytest.mark.gpu

HQ, HKV, D, BS = 14, 2, 64, 16


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    return torch.device("cuda", 0)


def np64(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def within(got, ref, atol=2e-3):
    return float(np.abs(got - ref).max()) <= atol


def make_cache(dev, num_blocks=64, max_seqs=6, max_len=512, prefix=False, layers=2):
    from mini_inference_b200 import PagedKVCache

    cache = PagedKVCache(num_layers=layers, num_kv_heads=HKV, head_dim=D, num_blocks=num_blocks, block_size=BS,
                         max_seqs=max_seqs, max_len=max_len, dtype=torch.float16, device=dev,
                         enable_prefix_caching=prefix)
    cache.k.normal_()
    cache.v.normal_()  # stale data everywhere: only a sequence's own keys may be read
    return cache


def qkv(n_tok, dev, batch=1, g=None):
    q = torch.randn(batch, HQ, n_tok, D, generator=g).half().to(dev)
    k = torch.randn(batch, HKV, n_tok, D, generator=g).half().to(dev)
    v = torch.randn(batch, HKV, n_tok, D, generator=g).half().to(dev)
    return q, k, v


@torch.inference_mode()
def test_packed_prefill_then_scattered_decode(dev):
    g = torch.Generator().manual_seed(0)
    cache = make_cache(dev)
    lengths = [37, 5, 70, 16]
    slots = [cache.allocate(0) for _ in lengths]
    for grow in range(1, 6):  # interleaved growth scatters the blocks
        for s, n in zip(slots, lengths):
            cache.ensure_capacity(s, min(n + 1, grow * BS))
    tables_before = [cache.block_tables[s] for s in slots]
    kp = np64(cache.k[1]).copy()
    vp = np64(cache.v[1]).copy()
    ctx = cache.packed_prefill_context(slots, lengths)
    assert ctx.positions.cpu().tolist() == [p for n in lengths for p in range(n)]
    total = sum(lengths)
    q, k, v = qkv(total, dev, g=g)
    out = ctx.attend(1, q, k, v)
    ctx.commit()
    cache.raise_device_errors()
    assert [cache.lengths[s] for s in slots] == lengths
    ref = packed_prefill_attend(kp, vp, tables_before, [0] * 4, lengths, np64(q[0]), np64(k[0]), np64(v[0]))
    assert within(np64(out[0]), round_to(ref, "float16"))
    # Cache writes: bit-exact (the oracle wrote the same values into kp).
    assert np.array_equal(np64(cache.k[1]), kp) and np.array_equal(np64(cache.v[1]), vp)

    for s, n in zip(slots, lengths):
        assert cache.ensure_capacity(s, n + 1)
    dq, dk, dv = qkv(1, dev, batch=len(slots), g=g)
    dctx = cache.decode_context(slots)
    assert dctx.positions.cpu().tolist() == lengths
    out = dctx.attend(1, dq, dk, dv)
    dctx.commit()
    cache.raise_device_errors()
    assert [cache.lengths[s] for s in slots] == [n + 1 for n in lengths]
    ref = decode_attend(kp, vp, [cache.block_tables[s] for s in slots], lengths, np64(dq[:, :, 0]),
                        np64(dk[:, :, 0]), np64(dv[:, :, 0]))
    assert within(np64(out[:, :, 0]), round_to(ref, "float16"))
    assert np.array_equal(np64(cache.k[1]), kp)


@torch.inference_mode()
def test_prefix_hit_prefill_reads_shared_blocks(dev):
    g = torch.Generator().manual_seed(1)
    cache = make_cache(dev, prefix=True, layers=1)
    common = list(range(1000, 1040))  # 2 full blocks + 8 tokens
    first = common + [1, 2, 3]
    a = cache.allocate(len(first), token_ids=first)
    kp, vp = np64(cache.k[0]).copy(), np64(cache.v[0]).copy()
    tab_a = cache.block_tables[a]
    q, k, v = qkv(len(first), dev, g=g)
    ctx = cache.packed_prefill_context([a], [len(first)])
    ctx.attend(0, q, k, v)
    ctx.commit()
    packed_prefill_attend(kp, vp, [tab_a], [0], [len(first)], np64(q[0]), np64(k[0]), np64(v[0]))
    cache.register_prefix(a, first)
    prompts = [common + [7] * 9, common + [8] * 30]
    slots = [cache.allocate(len(p), token_ids=p) for p in prompts]
    starts = [cache.lengths[s] for s in slots]
    assert starts == [32, 32] and cache.prefix_hit_tokens == 64
    assert all(cache.block_tables[s][:2] == tab_a[:2] for s in slots)
    new = [len(p) - st for p, st in zip(prompts, starts)]
    tabs = [cache.block_tables[s] for s in slots]
    q, k, v = qkv(sum(new), dev, g=g)
    ctx = cache.packed_prefill_context(slots, new)
    assert ctx.has_prefix
    out = ctx.attend(0, q, k, v)
    ctx.commit()
    cache.raise_device_errors()
    ref = packed_prefill_attend(kp, vp, tabs, starts, new, np64(q[0]), np64(k[0]), np64(v[0]))
    assert within(np64(out[0]), round_to(ref, "float16"))
    assert np.array_equal(np64(cache.k[0]), kp)


@torch.inference_mode()
def test_decode_errors_follow_the_reference(dev):
    cache = make_cache(dev, num_blocks=4, max_len=64)
    s = cache.allocate(16)
    cache.lengths[s] = 16  # its only block is full: the next token has nowhere to go
    with pytest.raises(ValueError, match="no block for its next token"):
        cache.decode_context([s])
    t = cache.allocate(16)
    with pytest.raises(ValueError, match="no room"):
        cache.packed_prefill_context([t], [100])


@torch.inference_mode()
def test_freed_and_reused_slots_never_read_stale_tables(dev):
    """Preemption frees a sequence; its slot and blocks are reused by a shorter one."""
    g = torch.Generator().manual_seed(2)
    cache = make_cache(dev, num_blocks=12, layers=1)
    a = cache.allocate(100)
    q, k, v = qkv(100, dev, g=g)
    c = cache.packed_prefill_context([a], [100])
    c.attend(0, q, k, v)
    c.commit()
    cache.free(a)
    b = cache.allocate(20)
    assert b == a  # the freed slot id comes back first
    kp, vp = np64(cache.k[0]).copy(), np64(cache.v[0]).copy()
    tab = cache.block_tables[b]
    q, k, v = qkv(20, dev, g=g)
    c = cache.packed_prefill_context([b], [20])
    out = c.attend(0, q, k, v)
    c.commit()
    cache.ensure_capacity(b, 21)
    dq, dk, dv = qkv(1, dev, g=g)
    d = cache.decode_context([b])
    dout = d.attend(0, dq, dk, dv)
    cache.raise_device_errors()
    ref = packed_prefill_attend(kp, vp, [tab], [0], [20], np64(q[0]), np64(k[0]), np64(v[0]))
    assert within(np64(out[0]), round_to(ref, "float16"))
    ref = decode_attend(kp, vp, [cache.block_tables[b]], [20], np64(dq[:, :, 0]), np64(dk[:, :, 0]),
                        np64(dv[:, :, 0]))
    assert within(np64(dout[:, :, 0]), round_to(ref, "float16"))


@torch.inference_mode()
def test_decode_step_replays_from_a_cuda_graph(dev):
    """The decode kernel and metadata builder are capturable; a replay with new inputs matches eager."""
    from mini_inference_b200 import ops

    g = torch.Generator().manual_seed(3)
    cache = make_cache(dev, num_blocks=64, layers=1)
    lengths = [30, 64, 5]
    slots = [cache.allocate(n + 1) for n in lengths]
    for s, n in zip(slots, lengths):
        cache.lengths[s] = n
    cache.sync_tables()
    batch = 4  # one padding row
    rows = torch.tensor(slots + [-1], dtype=torch.int32, device=dev)
    lens = torch.tensor(lengths + [0], dtype=torch.int32, device=dev)
    pos = torch.empty(batch, dtype=torch.int64, device=dev)
    sm = torch.empty(batch, dtype=torch.int64, device=dev)
    cl = torch.empty(batch, dtype=torch.int32, device=dev)
    tables = ops.make_tables(cache.tables_dev, rows)
    q = torch.zeros(batch, HQ, D, dtype=torch.float16, device=dev)
    kn = torch.zeros(batch, HKV, D, dtype=torch.float16, device=dev)
    vn = torch.zeros_like(kn)
    out = torch.empty(batch, HQ, D, dtype=torch.float16, device=dev)
    ws = cache.workspace(cache.max_seqs, HQ)

    def step():
        ops.build_decode_metadata(tables, lens, BS, cache.scratch_block, pos, sm, cl, cache.status)
        ops.decode_attention(cache.pool, 0, tables, q, cl, ws, k_new=kn, v_new=vn, slot_mapping=sm, out=out,
                             status=cache.status)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    kp, vp = np64(cache.k[0]).copy(), np64(cache.v[0]).copy()
    q.copy_(torch.randn(batch, HQ, D, generator=g).half())
    kn.copy_(torch.randn(batch, HKV, D, generator=g).half())
    vn.copy_(torch.randn(batch, HKV, D, generator=g).half())
    graph.replay()
    torch.cuda.synchronize()
    cache.raise_device_errors()
    ref = decode_attend(kp, vp, [cache.block_tables[s_] for s_ in slots], lengths, np64(q[:3]), np64(kn[:3]),
                        np64(vn[:3]))
    assert within(np64(out[:3]), round_to(ref, "float16"))
    assert pos.cpu().tolist() == lengths + [0]
