"""Copy-on-write of a shared, partially filled block, then attention (needs a B200).

The reference never writes a block that another sequence holds: it shares only full
prefix blocks and always recomputes at least one token (``engine/kv_cache.py:499-501``),
so this has no counterpart there (parity unpinned). The check is the survey's: a sequence
forked from another shares its blocks, the last one only partly filled; both then decode a
token of their own into that block. The first writer gets a private copy (``pkv_bm_prepare_write``
+ ``pkv_copy_blocks``), both attend, and each result must equal attention recomputed from
the sequence's own keys (the prefill rows, then its new row) within the parity bar. The
pool must hold the shared rows in both copies, bit for bit, and each sequence's new row
only in its own.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

L, HQ, HKV, D, BS = 2, 14, 2, 64, 16


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    return torch.device("cuda", 0)


def attention(q, keys, values):
    """float64 GQA attention of one token: q [Hq, d], keys / values [n, Hkv, d] -> [Hq, d]."""
    out = np.empty_like(q)
    for h in range(HQ):
        j = h // (HQ // HKV)
        s = keys[:, j] @ q[h] / np.sqrt(D)
        p = np.exp(s - s.max())
        out[h] = (p / p.sum()) @ values[:, j]
    return out


@pytest.mark.parametrize("graphed", [False, True])
def test_fork_copy_on_write_then_attend_equals_recomputation(dev, graphed):
    from mini_inference_b200 import PagedKVCache
    from oracle.numerics import round_to

    f64 = lambda t: t.detach().float().cpu().numpy().astype(np.float64)  # noqa: E731
    g = torch.Generator().manual_seed(31)
    cache = PagedKVCache(L, HKV, D, num_blocks=32, block_size=BS, max_seqs=4, max_len=256, dtype=torch.float16,
                         device=dev, enable_copy_on_write=True)
    n = 40  # 2 full blocks and 8 tokens of a third
    a = cache.allocate(n)
    pre = [[torch.randn(1, h, n, D, generator=g).half().to(dev) for h in (HQ, HKV, HKV)] for _ in range(L)]
    ctx = cache.packed_prefill_context([a], [n])
    for layer, (q, k, v) in enumerate(pre):
        ctx.attend(layer, q, k, v)
    ctx.commit()
    b = cache.fork(a)
    shared = cache.block_tables[a]
    assert cache.block_tables[b] == shared and cache.lengths[b] == n

    new = [[torch.randn(2, h, 1, D, generator=g).half().to(dev) for h in (HQ, HKV, HKV)] for _ in range(L)]
    if graphed:
        from mini_inference_b200.cuda_graphs import GraphedDecoder

        class Attn:  # a one-op "model": each layer's attention over the step's rows
            cfg = None

            def __call__(self, ids, positions, gctx):
                rows = ids.shape[0]  # the captured bucket's batch
                outs = [gctx.attend(layer, q[:rows], k[:rows], v[:rows])[:, :, 0] for layer, (q, k, v) in enumerate(new)]
                return torch.stack(outs, 1).reshape(rows, 1, -1)

            def compute_logits(self, hidden):
                return hidden.flatten(1)

        dec = GraphedDecoder(Attn(), cache, max_batch=2)
        dec.capture()
        got = dec.decode([a, b], [0, 0]).view(2, L, HQ, D).transpose(0, 1).half()
    else:
        dctx = cache.decode_context([a, b])
        got = torch.stack([dctx.attend(layer, q, k, v)[:, :, 0] for layer, (q, k, v) in enumerate(new)])
        dctx.commit()
    cache.raise_device_errors()
    ta, tb = cache.block_tables[a], cache.block_tables[b]
    assert ta[:2] == shared[:2] and tb[:2] == shared[:2] and ta[2] != tb[2] and shared[2] in (ta[2], tb[2])
    assert cache.lengths[a] == cache.lengths[b] == n + 1

    for layer in range(L):
        kp, vp = cache.k[layer], cache.v[layer]
        k_pre, v_pre = pre[layer][1][0].transpose(0, 1), pre[layer][2][0].transpose(0, 1)  # [n, Hkv, d]
        for row, (slot, table) in enumerate(((a, ta), (b, tb))):
            k_new, v_new = new[layer][1][row, :, 0], new[layer][2][row, :, 0]
            # The pool: the 8 shared rows, then this sequence's own row, in its own copy of block 2.
            blk = kp[table[2]].transpose(0, 1)  # [16, Hkv, d]
            assert torch.equal(blk[:8], k_pre[32:40]) and torch.equal(blk[8], k_new)
            assert torch.equal(vp[table[2]].transpose(0, 1)[8], v_new)
            keys = np.concatenate([f64(k_pre), f64(k_new)[None]])
            values = np.concatenate([f64(v_pre), f64(v_new)[None]])
            want = round_to(attention(f64(new[layer][0][row, :, 0]), keys, values), "float16")
            err = np.abs(f64(got[layer, row]) - want) - 2e-3 * np.abs(want)
            assert err.max() <= 2e-3, (layer, slot, err.max())
