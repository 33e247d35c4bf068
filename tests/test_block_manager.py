"""The C++ block manager against the reference's own traces and the oracle (host only, no GPU).

* every golden allocator trace, replayed call by call: results and the full
  observable state (tables, lengths, free-block order, refcounts, cached
  blocks, prefix_hit_tokens) bit-exact after every call;
* long seeded random traces, native vs the pure-Python oracle;
* the reference's own allocator tests (tests/test_kv_cache.py:163-176,210-243),
  restated on this package's PagedKVCache.
"""

from __future__ import annotations

import json
import random

import pytest
import torch

from mini_inference_b200 import NativeBlockManager, PagedKVCache
from oracle.block_manager import OracleBlockManager
from tests.test_oracle_golden import replay


def test_native_manager_replays_every_reference_trace(golden_dir):
    traces = json.loads((golden_dir / "allocator_traces.json").read_text())
    for t, trace in enumerate(traces):
        cfg = trace["config"]
        m = NativeBlockManager(cfg["num_blocks"], cfg["block_size"], cfg["max_seqs"], cfg["max_len"],
                               cfg["enable_prefix_caching"])
        lengths = _Lengths(m)
        for i, step in enumerate(trace["steps"]):
            got = replay(_Adapter(m, lengths), step["op"])
            assert got == step["result"], (t, i, step["op"])
            assert m.state() == step["state"], (t, i, step["op"])


class _Lengths(dict):
    def __init__(self, m):
        super().__init__()
        self.m = m

    def __setitem__(self, slot, value):
        self.m.set_length(slot, value)


class _Adapter:
    """The trace replayer calls ``manager.lengths[slot] = value``; route it to the native manager."""

    def __init__(self, m, lengths):
        self.m, self.lengths = m, lengths

    def __getattr__(self, name):
        return getattr(self.m, name)


def _random_trace(rng: random.Random, cfg: dict, n_ops: int):
    bs, max_len = cfg["block_size"], cfg["max_len"]
    vocab = rng.choice([3, 20, 1000])  # tiny vocabularies make prefix collisions frequent
    prefixes = [[rng.randrange(vocab) for _ in range(rng.randrange(1, 5 * bs))] for _ in range(4)]
    for _ in range(n_ops):
        r = rng.random()
        if r < 0.3:
            toks = (rng.choice(prefixes) if rng.random() < 0.8 else []) + \
                [rng.randrange(vocab) for _ in range(rng.randrange(0, 2 * bs))]
            toks = toks[:max_len] or [1]
            n = len(toks) if rng.random() < 0.85 else rng.randrange(-1, max_len + 5)
            yield ("allocate", n, toks if rng.random() < 0.9 else None)
        elif r < 0.5:
            yield ("commit", rng.randrange(cfg["max_seqs"]), rng.randrange(0, max_len + 1))
        elif r < 0.7:
            yield ("grow", rng.randrange(cfg["max_seqs"]), rng.randrange(0, max_len + 3))
        elif r < 0.75:
            yield ("can", rng.randrange(-2, max_len + 3))
        else:
            yield ("free", rng.randrange(cfg["max_seqs"]))


def _apply(m, op, tokens_of):
    kind = op[0]
    try:
        if kind == "allocate":
            s = m.allocate(op[1], token_ids=op[2])
            tokens_of[s] = op[2] or []
            return s
        if kind == "commit":
            s, want = op[1], op[2]
            if s not in tokens_of:
                return "skip"
            cap = len(m.block_tables[s]) * m.block_size
            m.lengths[s] = min(want, cap)
            toks = tokens_of[s] + [7] * max(0, min(want, cap) - len(tokens_of[s]))
            return m.register_prefix(s, toks)
        if kind == "grow":
            return m.ensure_capacity(op[1], op[2]) if op[1] in tokens_of else "skip"
        if kind == "can":
            return m.can_allocate(op[1])
        if kind == "free":
            r = m.free(op[1])
            tokens_of.pop(op[1], None)
            return r
    except RuntimeError as e:
        return str(e)
    raise AssertionError(kind)


class _NativeView:
    """Oracle-compatible face of the native manager (lengths / block_tables as dict-likes)."""

    def __init__(self, m: NativeBlockManager):
        self.m = m
        self.block_size = m.block_size
        outer = self

        class L(dict):
            def __setitem__(self, k, v):
                outer.m.set_length(k, v)

        class T:
            def __getitem__(self, k):
                return outer.m.table(k)

        self.lengths = L()
        self.block_tables = T()

    def __getattr__(self, name):
        return getattr(self.m, name)


@pytest.mark.parametrize("seed", range(12))
def test_native_manager_matches_oracle_on_random_traces(seed):
    rng = random.Random(1000 + seed)
    cfg = {"num_blocks": rng.choice([4, 9, 17, 40]), "block_size": rng.choice([1, 2, 4, 16]),
           "max_seqs": rng.choice([1, 3, 6]), "max_len": 0, "enable_prefix_caching": rng.random() < 0.75}
    cfg["max_len"] = rng.choice([4, 8, 24]) * cfg["block_size"]
    oracle = OracleBlockManager(**cfg)
    native = NativeBlockManager(**cfg)
    view = _NativeView(native)
    o_tok: dict = {}
    n_tok: dict = {}
    for i, op in enumerate(_random_trace(rng, cfg, 400)):
        a = _apply(oracle, op, o_tok)
        b = _apply(view, op, n_tok)
        assert a == b, (i, op)
        assert native.state() == oracle.state(), (i, op)


def tiny_paged(num_blocks=12, block_size=4, max_seqs=4, max_len=32, prefix=False) -> PagedKVCache:
    return PagedKVCache(num_layers=1, num_kv_heads=2, head_dim=8, num_blocks=num_blocks, block_size=block_size,
                        max_seqs=max_seqs, max_len=max_len, dtype=torch.float32, device="cpu",
                        enable_prefix_caching=prefix)


def test_paged_block_bookkeeping():
    """tests/test_kv_cache.py:163-176 of the reference, on this package's cache."""
    cache = tiny_paged(num_blocks=6, block_size=4)
    a = cache.allocate(5)
    assert len(cache.block_tables[a]) == 2 and cache.num_free_blocks == 4
    assert cache.ensure_capacity(a, 8) and len(cache.block_tables[a]) == 2
    assert cache.ensure_capacity(a, 9) and len(cache.block_tables[a]) == 3
    b = cache.allocate(12)
    assert cache.num_free_blocks == 0
    assert not cache.can_allocate(1) and not cache.ensure_capacity(b, 13)
    cache.free(a)
    assert cache.num_free_blocks == 3 and cache.can_allocate(12)
    with pytest.raises(RuntimeError):
        cache.free(a)


def test_prefix_blocks_are_shared_refcounted_and_evicted_lru():
    """tests/test_kv_cache.py:210-243 of the reference, on this package's cache."""
    cache = PagedKVCache(num_layers=1, num_kv_heads=1, head_dim=4, num_blocks=16, block_size=4, max_seqs=4,
                         max_len=64, dtype=torch.float32, device="cpu", enable_prefix_caching=True)
    shared = list(range(100, 116))
    a_tokens = shared + [1, 2, 3]
    a = cache.allocate(len(a_tokens), token_ids=a_tokens)
    assert cache.lengths[a] == 0
    cache.lengths[a] = len(a_tokens)
    cache.register_prefix(a, a_tokens)
    b_tokens = shared + [7, 8]
    b = cache.allocate(len(b_tokens), token_ids=b_tokens)
    assert cache.lengths[b] == 16
    assert cache.block_tables[b][:4] == cache.block_tables[a][:4]
    assert cache.block_tables[b][4] != cache.block_tables[a][4]
    c = cache.allocate(16, token_ids=shared)
    assert cache.lengths[c] == 12
    cache.free(a)
    cache.free(b)
    cache.free(c)
    assert cache.num_free_blocks == 16
    d = cache.allocate(18, token_ids=shared + [5, 6])
    assert cache.lengths[d] == 16
    cache.free(d)
    e = cache.allocate(64, token_ids=list(range(64)))
    cache.free(e)
    f = cache.allocate(18, token_ids=shared + [5, 6])
    assert cache.lengths[f] == 0


def test_error_conventions_match_the_reference():
    cache = tiny_paged(num_blocks=2, block_size=4, max_seqs=2, max_len=8)
    with pytest.raises(RuntimeError, match="not enough free KV cache blocks"):
        cache.allocate(100)
    s = cache.allocate(8)
    with pytest.raises(RuntimeError, match="not enough free KV cache blocks"):
        cache.allocate(1)
    cache.free(s)
    with pytest.raises(RuntimeError, match=f"slot {s} freed twice"):
        cache.free(s)
    with pytest.raises(KeyError):
        cache.ensure_capacity(s, 4)
    assert cache.ensure_capacity(s, 9) is False  # past max_len: False before the table lookup, as the reference
    assert cache.can_allocate(8) and not cache.can_allocate(9)


def test_cpu_cache_has_no_attention_path():
    """The attention contexts run on the sm_100a kernels only; a CPU cache refuses them loudly."""
    cache = tiny_paged()
    s = cache.allocate(3)
    with pytest.raises(RuntimeError, match="CUDA"):
        cache.decode_context([s])
    with pytest.raises(RuntimeError, match="CUDA"):
        cache.packed_prefill_context([s], [3])


def test_journal_records_table_edits_for_the_device_mirror():
    m = NativeBlockManager(8, 4, 3, 32, False)
    import numpy as np

    m.set_journal(True)
    a = m.allocate(5)
    m.ensure_capacity(a, 9)
    b = m.allocate(1)
    buf = np.zeros((16, 3), np.int32)
    n, ovf = m.drain_edits(buf)
    assert not ovf
    edits = [tuple(r) for r in buf[:n]]
    ta, tb = m.table(a), m.table(b)
    assert edits == [(a, 0, ta[0]), (a, 1, ta[1]), (a, 2, ta[2]), (b, 0, tb[0])]
    assert m.drain_edits(buf) == (0, False)
    small = np.zeros((1, 3), np.int32)
    assert m.ensure_capacity(a, 16) and m.ensure_capacity(b, 8)  # one new block each
    n, ovf = m.drain_edits(small)
    assert n == 1 and ovf


def test_fork_shares_every_block_and_copy_on_write_unshares_only_what_is_written():
    """No reference counterpart (it never writes a shared block); host-side rules of fork + prepare_write."""
    from mini_inference_b200.cache import NativeBlockManager

    bm = NativeBlockManager(num_blocks=8, block_size=4, max_seqs=4, max_len=32)
    a = bm.allocate(10)  # 3 blocks, the last holding 2 tokens
    bm.set_length(a, 10)
    b = bm.fork(a)
    assert bm.table(b) == bm.table(a) and bm.get_length(b) == 10
    refs = bm.ref_counts()
    assert all(refs[x] == 2 for x in bm.table(a))
    free_before = bm.num_free_blocks
    # Writing tokens 10..13 of b touches blocks 2 and 3 of its table; only block 2 exists and is shared.
    assert bm.ensure_capacity(b, 14)
    pairs = bm.prepare_write(b, 10, 4)
    old_a = bm.table(a)
    assert len(pairs) == 1 and pairs[0][0] == old_a[2] and pairs[0][1] not in old_a
    assert bm.table(b)[:2] == old_a[:2] and bm.table(b)[2] == pairs[0][1]
    assert bm.ref_counts()[old_a[2]] == 1  # now a's alone
    assert bm.num_free_blocks == free_before - 2  # one block for position 12+, one copy
    assert bm.prepare_write(a, 10, 1) == []  # a's block 2 is no longer shared
    bm.free(b)
    assert all(bm.ref_counts()[x] == 1 for x in old_a)
    bm.free(a)
    assert bm.num_free_blocks == 8


def test_copy_on_write_without_room_changes_nothing():
    from mini_inference_b200.cache import NativeBlockManager

    bm = NativeBlockManager(num_blocks=2, block_size=4, max_seqs=3, max_len=16)
    a = bm.allocate(6)  # both blocks
    bm.set_length(a, 6)
    b = bm.fork(a)
    with pytest.raises(RuntimeError, match="not enough free KV cache blocks"):
        bm.prepare_write(b, 6, 1)
    assert bm.table(b) == bm.table(a) and bm.ref_counts() == [2, 2]


def test_fork_needs_the_copy_on_write_cache():
    import torch

    from mini_inference_b200 import PagedKVCache

    cache = PagedKVCache(1, 1, 4, num_blocks=4, block_size=4, max_seqs=2, max_len=16, dtype=torch.float16,
                         device="cpu")
    s = cache.allocate(3)
    with pytest.raises(RuntimeError, match="enable_copy_on_write"):
        cache.fork(s)
    cow = PagedKVCache(1, 1, 4, num_blocks=4, block_size=4, max_seqs=2, max_len=16, dtype=torch.float16,
                       device="cpu", enable_copy_on_write=True)
    s = cow.allocate(3)
    assert cow.block_tables[cow.fork(s)] == cow.block_tables[s]
