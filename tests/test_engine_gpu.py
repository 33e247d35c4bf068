"""The whole paged path in an engine loop on the GPU, checked token by token against the oracle.

``LLMEngine.step`` (engine/engine.py:281-312) is driven with every component of this
package in place: the native ``Scheduler`` (continuous batching, prefix-cache admission,
preemption), ``PagedKVCache`` with its packed-prefill and decode contexts (RoPE fused with
the append, ``attend_qkv``), and ``GreedyLMHead`` for the next token, on a small random
transformer with the reference model's call shape (qkv projection with bias, rotary
embedding, paged attention, output projection, residual; tied-style LM head). A small
pool forces preemptions (recomputed by prefill over prompt + outputs) and shared prompt
prefixes give prefix-cache hits.

Every generated token is then checked against a dense float64 recomputation of the same
model over the sequence's tokens (the oracle: ``oracle.rope`` for the rotation, plain
causal attention): at each position the chosen token must be within a small tolerance of
the oracle's best logit, so a wrong block table, a stale or misplaced K/V row, or a wrong
position shows up as a wrong token. The tolerance absorbs fp16 rounding only.
"""

from __future__ import annotations

import random
from dataclasses import dataclass, field
from types import SimpleNamespace

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

L, HQ, HKV, D, H, VOCAB, BS = 2, 14, 2, 64, 128, 97, 16
THETA, MAX_POS = 1e6, 512


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    return torch.device("cuda", 0)


@dataclass
class Sampling:
    max_tokens: int
    ignore_eos: bool = True
    greedy: bool = True


@dataclass(eq=False)
class Seq:
    seq_id: int
    prompt_token_ids: list
    sampling: Sampling
    output_token_ids: list = field(default_factory=list)
    status: object = None
    slot: int | None = None
    finish_reason: object = None
    first_token_time: float | None = None
    finish_time: float | None = None
    num_preemptions: int = 0
    num_cached_tokens: int = 0

    @property
    def prompt_len(self):
        return len(self.prompt_token_ids)

    @property
    def num_tokens(self):
        return len(self.prompt_token_ids) + len(self.output_token_ids)

    @property
    def token_ids(self):
        return self.prompt_token_ids + self.output_token_ids

    @property
    def last_token(self):
        return self.output_token_ids[-1]

    @property
    def is_finished(self):
        from mini_inference_b200.scheduler import SequenceStatus
        return self.status is SequenceStatus.FINISHED


SHAPES = {  # attention heads of the two model families, in their dtypes
    "0.5b_fp16": (HQ, HKV, D, torch.float16),  # Qwen2.5-0.5B: 14 / 2 heads of 64
    "7b_bf16": (28, 4, 128, torch.bfloat16),   # Qwen2.5-7B: 28 / 4 heads of 128
}


class Model:
    """Random weights in the model dtype; the GPU forward uses the package's contexts."""

    def __init__(self, dev, seed=0, shape=SHAPES["0.5b_fp16"]):
        self.hq, self.hkv, self.d, self.dtype = shape
        g = torch.Generator(device="cpu").manual_seed(seed)
        wqkv = (self.hq + 2 * self.hkv) * self.d

        def w(*shape, std):
            return (torch.randn(*shape, generator=g) * std).to(self.dtype).to(dev)

        self.embed = w(VOCAB, H, std=1.0)
        self.layers = [(w(H, wqkv, std=0.08), w(wqkv, std=0.1), w(self.hq * self.d, H, std=0.03 * (64 / self.d) ** 0.5))
                       for _ in range(L)]
        self.lm = w(VOCAB, H, std=0.5)
        from mini_inference_b200 import ops
        self.cos, self.sin = ops.rope_tables(self.d, MAX_POS, THETA, self.dtype, dev)

    def forward(self, ids, ctx):  # ids [B, T] -> hidden [B, T, H]
        b, t = ids.shape
        x = self.embed[ids]
        for layer, (wqkv, bqkv, wo) in enumerate(self.layers):
            qkv = x @ wqkv + bqkv
            o = ctx.attend_qkv(layer, qkv, self.cos, self.sin, self.hq)  # [B, Hq, T, d]
            x = x + o.transpose(1, 2).reshape(b, t, self.hq * self.d) @ wo
        return x


def oracle_logits(model, tokens):
    """Dense float64 forward over one sequence: logits [len(tokens), vocab] (row p predicts token p + 1)."""
    f = lambda t: t.float().cpu().numpy().astype(np.float64)  # noqa: E731
    HQ, HKV, D = model.hq, model.hkv, model.d  # noqa: N806
    cos, sin = f(model.cos), f(model.sin)
    pos = np.arange(len(tokens))
    x = f(model.embed)[tokens]
    scale = 1.0 / np.sqrt(D)
    mask = np.tril(np.ones((len(tokens), len(tokens)), bool))
    for wqkv, bqkv, wo in model.layers:
        qkv = x @ f(wqkv) + f(bqkv)
        q = qkv[:, :HQ * D].reshape(-1, HQ, D)
        k = qkv[:, HQ * D:(HQ + HKV) * D].reshape(-1, HKV, D)
        v = qkv[:, (HQ + HKV) * D:].reshape(-1, HKV, D)
        c, s = cos[pos][:, None, :], sin[pos][:, None, :]

        def rot(a):
            a1, a2 = a[..., :D // 2], a[..., D // 2:]
            return a * c + np.concatenate([-a2, a1], axis=-1) * s

        q, k = rot(q), rot(k)
        out = np.empty_like(q)
        for h in range(HQ):
            kv = h // (HQ // HKV)
            sc = (q[:, h] @ k[:, kv].T) * scale
            sc = np.where(mask, sc, -np.inf)
            p = np.exp(sc - sc.max(axis=1, keepdims=True))
            p /= p.sum(axis=1, keepdims=True)
            out[:, h] = p @ v[:, kv]
        x = x + out.reshape(-1, HQ * D) @ f(wo)
    return x @ f(model.lm).T


def run_engine(dev, model, requests, num_blocks, max_seqs, budget, max_len):
    from mini_inference_b200 import PagedKVCache
    from mini_inference_b200.sampler import GreedyLMHead
    from mini_inference_b200.scheduler import Scheduler, SequenceStatus

    cache = PagedKVCache(L, model.hkv, model.d, num_blocks=num_blocks, block_size=BS, max_seqs=max_seqs,
                         max_len=max_len, dtype=model.dtype, device=dev, enable_prefix_caching=True)
    sched = Scheduler(SimpleNamespace(max_num_seqs=max_seqs, max_num_batched_tokens=budget, max_model_len=max_len,
                                      scheduling="continuous"), cache)
    head = GreedyLMHead(model.lm, max_batch=max_seqs)
    seqs = [Seq(i, list(p), Sampling(m), status=SequenceStatus.WAITING) for i, (p, m) in enumerate(requests)]
    for s in seqs:
        sched.add(s)
    steps = 0
    while sched.has_work():
        steps += 1
        assert steps < 2000, "the engine loop does not finish"
        out = sched.schedule()
        if out.prefills:  # one packed prefill of every admitted request (engine/engine.py:293-304)
            new = [s.token_ids[cache.lengths[s.slot]:] for s in out.prefills]
            ctx = cache.packed_prefill_context([s.slot for s in out.prefills], [len(n) for n in new])
            ids = torch.tensor([[t for n in new for t in n]], device=dev)
            hidden = model.forward(ids, ctx)
            ctx.commit()
            for s in out.prefills:
                cache.register_prefix(s.slot, s.token_ids)
            toks = head.tokens(hidden[0, ctx.last_index].contiguous())
            sched.append_tokens(out.prefills, toks, float(steps))
        if out.decodes:  # engine/engine.py:305-312
            ctx = cache.decode_context([s.slot for s in out.decodes])
            ids = torch.tensor([[s.last_token] for s in out.decodes], device=dev)
            hidden = model.forward(ids, ctx)
            ctx.commit()
            toks = head.tokens(hidden[:, -1].contiguous())
            sched.append_tokens(out.decodes, toks, float(steps))
    cache.raise_device_errors()
    return seqs, sched.num_preemptions, cache.prefix_hit_tokens


@pytest.mark.parametrize("shape", list(SHAPES))
def test_engine_loop_tokens_match_the_dense_oracle(dev, shape):
    rng = random.Random(5)
    prefixes = [[rng.randrange(VOCAB) for _ in range(n)] for n in (40, 23)]
    requests = []
    for i in range(14):
        prompt = (list(rng.choice(prefixes)) if i % 3 else []) + [rng.randrange(VOCAB) for _ in range(rng.randint(1, 30))]
        requests.append((prompt, rng.randint(4, 40)))
    model = Model(dev, shape=SHAPES[shape])
    # 12 blocks of 16 for up to 6 running sequences of up to 110 tokens: preemptions happen.
    seqs, preemptions, hits = run_engine(dev, model, requests, num_blocks=12, max_seqs=6, budget=512, max_len=160)
    assert preemptions > 0 and hits > 0
    checked = 0
    for s in seqs:
        assert len(s.output_token_ids) == s.sampling.max_tokens
        logits = oracle_logits(model, s.token_ids)
        for j, tok in enumerate(s.output_token_ids):
            row = logits[s.prompt_len - 1 + j]
            assert row[tok] >= row.max() - 0.02 * max(1.0, abs(row.max())), (s.seq_id, j, tok, int(row.argmax()))
            checked += 1
    assert checked == sum(m for _, m in requests)


def test_preemption_does_not_change_the_tokens(dev):
    """The reference's own check (tests/test_engine_parity.py:78-89): a pool small enough to
    preempt gives the same outputs as one that never does, up to near-ties of the dense logits."""
    rng = random.Random(9)
    requests = [([rng.randrange(VOCAB) for _ in range(rng.randint(5, 40))], rng.randint(10, 50)) for _ in range(10)]
    model = Model(dev, seed=1)
    small, pre_small, _ = run_engine(dev, model, requests, num_blocks=12, max_seqs=6, budget=512, max_len=128)
    big, pre_big, _ = run_engine(dev, model, requests, num_blocks=200, max_seqs=6, budget=512, max_len=128)
    assert pre_small > 0 and pre_big == 0
    for a, b in zip(small, big):
        if a.output_token_ids == b.output_token_ids:
            continue
        # Where they first differ, both choices must be near-ties of the dense logits.
        j = next(i for i, (x, y) in enumerate(zip(a.output_token_ids, b.output_token_ids)) if x != y)
        row = oracle_logits(model, a.prompt_token_ids + a.output_token_ids[:j])[-1]
        tol = 0.02 * max(1.0, abs(row.max()))
        assert row[a.output_token_ids[j]] >= row.max() - tol and row[b.output_token_ids[j]] >= row.max() - tol


def test_greedy_streams_identical_over_64_tokens(dev):
    """The first 64 greedy tokens of every request equal the dense oracle's own greedy stream
    (float64, recomputed from scratch at every step), all of them: this model's logits are
    spread far wider than float16 rounding, so no near-tie may excuse a difference."""
    rng = random.Random(13)
    prefix = [rng.randrange(VOCAB) for _ in range(33)]
    requests = [((prefix if i % 2 else []) + [rng.randrange(VOCAB) for _ in range(rng.randint(3, 40))], 64)
                for i in range(8)]
    model = Model(dev, seed=2)
    seqs, _, hits = run_engine(dev, model, requests, num_blocks=40, max_seqs=8, budget=1024, max_len=160)
    assert hits > 0
    for s in seqs:
        toks = list(s.prompt_token_ids)
        for j in range(64):
            row = oracle_logits(model, toks)[-1]
            want = int(row.argmax())
            got = s.output_token_ids[j]
            assert got == want, (f"stream {s.seq_id} parts from the oracle at token {j}: {got} vs {want} "
                                 f"(dense logits {row[got]:.5f} vs {row[want]:.5f})")
            toks.append(want)
