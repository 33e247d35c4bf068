"""GraphedDecoder on the libpkv cache (engine/cuda_graphs.py mirror), against the eager decode step.

A toy stand-in for Qwen2ForCausalLM with the reference model's call shape
(``model(ids, positions, ctx)`` calling ``ctx.attend`` per layer, then
``compute_logits``) drives both paths; the cached K/V are random. The graphed
steps run in a larger batch bucket (padding rows) than the eager ones and
cross block boundaries, so they also check that padding rows touch only the
scratch block and that one graph serves every context length.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

L, HQ, HKV, D, HIDDEN, VOCAB = 2, 14, 2, 64, 128, 97


class ToyModel:
    def __init__(self, dev, seed=0):
        g = torch.Generator(device=dev).manual_seed(seed)

        def w(*shape):
            return (torch.randn(*shape, generator=g, device=dev) * 0.05).half()

        self.embed = w(VOCAB, HIDDEN)
        self.layers = [(w(HIDDEN, HQ * D), w(HIDDEN, HKV * D), w(HIDDEN, HKV * D), w(HQ * D, HIDDEN)) for _ in range(L)]
        self.head = w(HIDDEN, VOCAB)

    def __call__(self, ids, positions, ctx):
        b, t = ids.shape
        x = self.embed[ids]  # [B, T, hidden]
        for layer, (wq, wk, wv, wo) in enumerate(self.layers):
            q = (x @ wq).view(b, t, HQ, D).transpose(1, 2)
            k = (x @ wk).view(b, t, HKV, D).transpose(1, 2)
            v = (x @ wv).view(b, t, HKV, D).transpose(1, 2)
            o = ctx.attend(layer, q, k, v)  # [B, Hq, T, d]
            x = x + o.transpose(1, 2).reshape(b, t, HQ * D) @ wo
        return x

    def compute_logits(self, h):
        return h @ self.head


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    return torch.device("cuda", 0)


def _cache(dev, k0, v0, lengths):
    from mini_inference_b200 import PagedKVCache

    cache = PagedKVCache(L, HKV, D, num_blocks=64, block_size=16, max_seqs=8, max_len=256, dtype=torch.float16,
                         device=dev)
    cache.k.copy_(k0)
    cache.v.copy_(v0)
    slots = []
    for n in lengths:
        s = cache.allocate(n + 1)
        cache.lengths[s] = n
        slots.append(s)
    return cache, slots


def test_graphed_decode_matches_the_eager_step(dev):
    from mini_inference_b200.cuda_graphs import GraphedDecoder

    g = torch.Generator(device=dev).manual_seed(3)
    shape = (L, 65, HKV, 16, D)
    k0 = torch.randn(shape, generator=g, device=dev).half()
    v0 = torch.randn(shape, generator=g, device=dev).half()
    lengths = [13, 47, 31]  # 13 -> 16 and 47 -> 48 cross block boundaries during the steps
    model = ToyModel(dev)
    ca, sa = _cache(dev, k0, v0, lengths)
    cb, sb = _cache(dev, k0, v0, lengths)
    assert sa == sb
    graphed = GraphedDecoder(model, ca, max_batch=4)
    graphed.capture()
    assert sorted(graphed.graphs) == [1, 2, 4]
    tokens = [5, 17, 42]
    for step in range(5):
        for c, slots in ((ca, sa), (cb, sb)):
            for s in slots:
                assert c.ensure_capacity(s, c.lengths[s] + 1)
        got = graphed.decode(sa, tokens)
        assert got is not None and got.shape == (3, VOCAB)
        with torch.inference_mode():
            ctx = cb.decode_context(sb)
            ids = torch.tensor(tokens, device=dev).unsqueeze(1)
            want = model.compute_logits(model(ids, ctx.positions.unsqueeze(1), ctx)[:, -1]).float()
            ctx.commit()
        ca.raise_device_errors()
        cb.raise_device_errors()
        torch.testing.assert_close(got, want, atol=2e-3, rtol=2e-3)
        tokens = [int(t) for t in want.argmax(-1).tolist()]
    assert graphed.replays == 5
    assert [ca.lengths[s] for s in sa] == [n + 5 for n in lengths] == [cb.lengths[s] for s in sb]
    # The pools agree wherever a sequence owns a block (padding rows wrote only the scratch block).
    for s in sa:
        for blk in ca.block_tables[s]:
            torch.testing.assert_close(ca.k[:, blk], cb.k[:, blk], atol=2e-3, rtol=0)
            torch.testing.assert_close(ca.v[:, blk], cb.v[:, blk], atol=2e-3, rtol=0)
    owned = {b for s in sa for b in ca.block_tables[s]}
    untouched = [b for b in range(64) if b not in owned]
    assert torch.equal(ca.k[:, untouched], k0[:, untouched])
    assert graphed.decode(list(range(5)), [0] * 5) is None  # no bucket holds 5 rows
