"""The reference's serving path restated with PyTorch CPU ops: model, paged contexts, engine step.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``). It is the timed CPU baseline of
the serving benchmark (the reference engine on the host cores) and the checker of the
greedy token streams at small shapes. It replays the reference's own sequence of ATen
calls, so on the same torch build it gives the reference's numbers:

* ``Qwen2ForCausalLM.forward`` / ``compute_logits`` (``engine/model.py:150-323``):
  embedding, per layer ``RMSNorm`` (float32 statistics) -> fused ``qkv_proj`` with bias
  -> split and head views -> RoPE from float32 tables cast per lookup -> ``ctx.attend``
  -> ``o_proj`` -> residual, ``RMSNorm`` -> ``gate_up_proj`` -> SiLU * up ->
  ``down_proj`` -> residual; final norm; LM head (tied or separate);
* ``PackedPrefillContext`` (``engine/kv_cache.py:252-301``): the index_put append of
  the packed tokens, then SDPA (GQA by ``repeat_interleave``) with a causal, a
  block-diagonal or, with prefix hits, a sequence-and-position mask over the keys
  read back from the cache;
* ``PagedDecodeContext`` (``engine/kv_cache.py:592-624``): ``paged_kv_torch``;
* ``LLMEngine.step`` (``engine/engine.py:281-328``) with ``ModelRunner`` and the greedy
  ``Sampler`` (``engine/engine.py:99-123``, ``engine/sampler.py:27-31``) over
  :class:`oracle.scheduler.OracleScheduler` and :class:`oracle.block_manager.OracleBlockManager`.

Weights are passed in as a dict keyed by the reference's parameter names.
"""

from __future__ import annotations

import time
from collections.abc import Sequence

import torch
import torch.nn.functional as F

from .block_manager import OracleBlockManager
from .paged_kv_torch import decode_attend_torch
from .scheduler import OracleSampling, OracleScheduler, OracleSequence


class TorchPagedCache(OracleBlockManager):
    """The reference's paged cache: the allocator plus ``k, v [L, NB+1, Hkv, bs, d]`` on the CPU."""

    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int, num_blocks: int, block_size: int,
                 max_seqs: int, max_len: int, dtype: torch.dtype, enable_prefix_caching: bool = False) -> None:
        super().__init__(num_blocks, block_size, max_seqs, max_len, enable_prefix_caching)
        shape = (num_layers, num_blocks + 1, num_kv_heads, block_size, head_dim)
        self.k = torch.zeros(shape, dtype=dtype)
        self.v = torch.zeros(shape, dtype=dtype)

    def write_index(self, slots, starts, counts) -> tuple[torch.Tensor, torch.Tensor]:
        bs = self.block_size
        blocks, offsets = [], []
        for s, a, n in zip(slots, starts, counts):
            t = self.block_tables[s]
            blocks.extend(t[p // bs] for p in range(a, a + n))
            offsets.extend(p % bs for p in range(a, a + n))
        return torch.tensor(blocks, dtype=torch.int64), torch.tensor(offsets, dtype=torch.int64)


def _sdpa_gqa(q, k, v, mask=None, causal=False):
    groups = q.shape[1] // k.shape[1]
    if groups > 1:
        k = k.repeat_interleave(groups, dim=1)
        v = v.repeat_interleave(groups, dim=1)
    return F.scaled_dot_product_attention(q, k, v, attn_mask=mask, is_causal=causal)


class PrefillContext:
    def __init__(self, cache: TorchPagedCache, slots: Sequence[int], lengths: Sequence[int]) -> None:
        self.cache, self.slots, self.lengths = cache, list(slots), list(lengths)
        self.starts = [cache.lengths[s] for s in self.slots]
        for s, a, n in zip(self.slots, self.starts, self.lengths):
            if not cache.ensure_capacity(s, a + n):
                raise ValueError(f"no room in the KV cache for {a + n} tokens")
        seg = torch.repeat_interleave(torch.arange(len(self.slots)), torch.tensor(self.lengths))
        self.positions = torch.cat([torch.arange(a, a + n) for a, n in zip(self.starts, self.lengths)])
        self.write_at = cache.write_index(self.slots, self.starts, self.lengths)
        self.has_prefix = any(self.starts)
        if self.has_prefix:
            ends = [a + n for a, n in zip(self.starts, self.lengths)]
            self.read_at = cache.write_index(self.slots, [0] * len(self.slots), ends)
            key_seg = torch.repeat_interleave(torch.arange(len(self.slots)), torch.tensor(ends))
            key_pos = torch.cat([torch.arange(e) for e in ends])
            self.mask = (seg[:, None] == key_seg[None, :]) & (key_pos[None, :] <= self.positions[:, None])
        elif len(self.slots) == 1:
            self.mask = None
        else:
            idx = torch.arange(len(seg))
            self.mask = (seg[:, None] == seg[None, :]) & (idx[None, :] <= idx[:, None])
        self.last_index = torch.tensor(self.lengths).cumsum(0) - 1

    def attend(self, layer: int, q, k, v):
        kl, vl = self.cache.k[layer], self.cache.v[layer]
        w0, w2 = self.write_at
        kl[w0, :, w2] = k[0].transpose(0, 1)
        vl[w0, :, w2] = v[0].transpose(0, 1)
        if self.has_prefix:
            r0, r2 = self.read_at
            keys = kl[r0, :, r2].transpose(0, 1).unsqueeze(0)
            values = vl[r0, :, r2].transpose(0, 1).unsqueeze(0)
            return _sdpa_gqa(q, keys, values, mask=self.mask)
        if self.mask is None:
            return _sdpa_gqa(q, k, v, causal=True)
        return _sdpa_gqa(q, k, v, mask=self.mask)

    def commit(self) -> None:
        for s, a, n in zip(self.slots, self.starts, self.lengths):
            self.cache.lengths[s] = a + n


class DecodeContext:
    def __init__(self, cache: TorchPagedCache, slots: Sequence[int]) -> None:
        self.cache, self.slots = cache, list(slots)
        self.pos = [cache.lengths[s] for s in self.slots]
        self.tables = [cache.block_tables[s] for s in self.slots]
        if any(p // cache.block_size >= len(t) for p, t in zip(self.pos, self.tables)):
            raise ValueError("a sequence has no block for its next token (call ensure_capacity first)")
        self.positions = torch.tensor(self.pos)

    def attend(self, layer: int, q, k, v):
        out = decode_attend_torch(self.cache.k[layer], self.cache.v[layer], self.tables, self.pos, q[:, :, 0],
                                  k[:, :, 0], v[:, :, 0])
        return out.unsqueeze(2)

    def commit(self) -> None:
        for s in self.slots:
            self.cache.lengths[s] += 1


class TorchQwen2:
    """``Qwen2ForCausalLM`` as torch CPU ops over a weight dict (the reference's parameter names)."""

    def __init__(self, weights: dict[str, torch.Tensor], num_layers: int, num_heads: int, num_kv_heads: int,
                 head_dim: int, rms_norm_eps: float, rope_theta: float, max_positions: int) -> None:
        self.w = weights
        self.L, self.hq, self.hkv, self.d = num_layers, num_heads, num_kv_heads, head_dim
        self.eps = rms_norm_eps
        self.dtype = weights["embed_tokens.weight"].dtype
        self.lm_head = weights.get("lm_head.weight", weights["embed_tokens.weight"])
        # engine/model.py:190-199: one frequency per pair, the half-table repeated, float32.
        exponents = torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim
        inv_freq = 1.0 / (rope_theta ** exponents)
        freqs = torch.outer(torch.arange(max_positions, dtype=torch.float32), inv_freq)
        angles = torch.cat([freqs, freqs], dim=-1)
        self.cos_t, self.sin_t = angles.cos(), angles.sin()

    def _norm(self, x, w):
        x32 = x.float()
        x32 = x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + self.eps)
        return w * x32.to(x.dtype)

    @staticmethod
    def _rot(x):
        x1, x2 = x.chunk(2, dim=-1)
        return torch.cat([-x2, x1], dim=-1)

    def forward(self, ids: torch.Tensor, positions: torch.Tensor, ctx) -> torch.Tensor:
        w = self.w
        x = F.embedding(ids, w["embed_tokens.weight"])
        cos = self.cos_t[positions].unsqueeze(1).to(x.dtype)
        sin = self.sin_t[positions].unsqueeze(1).to(x.dtype)
        b, t, _ = x.shape
        qs, kvs = self.hq * self.d, self.hkv * self.d
        for i in range(self.L):
            p = f"layers.{i}."
            h = self._norm(x, w[p + "input_norm.weight"])
            q, k, v = F.linear(h, w[p + "attn.qkv_proj.weight"], w.get(p + "attn.qkv_proj.bias")).split(
                [qs, kvs, kvs], dim=-1)
            q = q.view(b, t, self.hq, self.d).transpose(1, 2)
            k = k.view(b, t, self.hkv, self.d).transpose(1, 2)
            v = v.view(b, t, self.hkv, self.d).transpose(1, 2)
            q, k = q * cos + self._rot(q) * sin, k * cos + self._rot(k) * sin
            o = ctx.attend(i, q, k, v)
            x = x + F.linear(o.transpose(1, 2).reshape(b, t, qs), w[p + "attn.o_proj.weight"])
            gate, up = F.linear(self._norm(x, w[p + "post_attn_norm.weight"]), w[p + "mlp.gate_up_proj.weight"]).chunk(
                2, dim=-1)
            x = x + F.linear(F.silu(gate) * up, w[p + "mlp.down_proj.weight"])
        return self._norm(x, w["norm.weight"])

    def logits(self, hidden: torch.Tensor) -> torch.Tensor:
        return F.linear(hidden, self.lm_head).float()


def pack_by_budget(lengths, budget):
    groups, total = [], 0
    for i, n in enumerate(lengths):
        if groups and budget > 0 and total + n <= budget:
            groups[-1].append(i)
            total += n
        else:
            groups.append([i])
            total = n
    return groups


@torch.inference_mode()
def serve(model: TorchQwen2, cache: TorchPagedCache, requests: Sequence[tuple[Sequence[int], int]],
          max_num_seqs: int, max_num_batched_tokens: int, max_model_len: int, record=None) -> list[OracleSequence]:
    """Run greedy requests ``(prompt_ids, max_tokens)`` (EOS ignored) to the end, as ``LLMEngine.step`` loops.

    ``record(seq, logits_row)``, if given, sees every sampled row of float32 logits.
    """
    sched = OracleScheduler(max_num_seqs, max_num_batched_tokens, max_model_len, cache)
    start = time.perf_counter()
    seqs = [OracleSequence(i, list(p), OracleSampling(max_tokens=m, ignore_eos=True), arrival_time=start)
            for i, (p, m) in enumerate(requests)]
    for s in seqs:
        sched.add(s)
    while sched.has_work():
        step = sched.schedule()
        news = {s.seq_id: s.token_ids[cache.lengths[s.slot]:] for s in step.prefills}
        for group in pack_by_budget([len(news[s.seq_id]) for s in step.prefills], max_num_batched_tokens):
            group_seqs = [step.prefills[i] for i in group]
            ctx = PrefillContext(cache, [s.slot for s in group_seqs], [len(news[s.seq_id]) for s in group_seqs])
            ids = torch.tensor([[t for s in group_seqs for t in news[s.seq_id]]])
            hidden = model.forward(ids, ctx.positions.unsqueeze(0), ctx)
            ctx.commit()
            logits = model.logits(hidden[0, ctx.last_index])
            for s in group_seqs:
                cache.register_prefix(s.slot, s.token_ids)
            now = time.perf_counter()
            for s, row in zip(group_seqs, logits):
                if record is not None:
                    record(s, row)
                sched.append_token(s, int(row.argmax()), now)
        if step.decodes:
            ctx = DecodeContext(cache, [s.slot for s in step.decodes])
            ids = torch.tensor([[s.output_token_ids[-1]] for s in step.decodes])
            hidden = model.forward(ids, ctx.positions.unsqueeze(1), ctx)
            ctx.commit()
            logits = model.logits(hidden[:, -1])
            now = time.perf_counter()
            for s, row in zip(step.decodes, logits):
                if record is not None:
                    record(s, row)
                sched.append_token(s, int(row.argmax()), now)
    return seqs


def serve_bookkeeping(cache: OracleBlockManager, requests: Sequence[tuple[Sequence[int], int]], max_num_seqs: int,
                      max_num_batched_tokens: int, max_model_len: int, token: int = 0) -> list[OracleSequence]:
    """The allocator side of :func:`serve` alone, every sampled token being ``token``.

    With EOS ignored and no preemption the scheduler's decisions, the block tables and
    ``prefix_hit_tokens`` do not depend on the tokens (prefix keys come from the prompts),
    so this gives the reference's exact admissions and prefix hits for a workload without
    running a model.
    """
    sched = OracleScheduler(max_num_seqs, max_num_batched_tokens, max_model_len, cache)
    seqs = [OracleSequence(i, list(p), OracleSampling(max_tokens=m, ignore_eos=True)) for i, (p, m) in enumerate(requests)]
    for s in seqs:
        sched.add(s)
    while sched.has_work():
        step = sched.schedule()
        news = {s.seq_id: s.token_ids[cache.lengths[s.slot]:] for s in step.prefills}
        for group in pack_by_budget([len(news[s.seq_id]) for s in step.prefills], max_num_batched_tokens):
            group_seqs = [step.prefills[i] for i in group]
            starts = [cache.lengths[s.slot] for s in group_seqs]
            for s, a in zip(group_seqs, starts):  # PackedPrefillContext: room, then commit
                if not cache.ensure_capacity(s.slot, a + len(news[s.seq_id])):
                    raise ValueError("no room in the KV cache")
            for s, a in zip(group_seqs, starts):
                cache.lengths[s.slot] = a + len(news[s.seq_id])
            for s in group_seqs:
                cache.register_prefix(s.slot, s.token_ids)
            for s in group_seqs:
                sched.append_token(s, token, 0.0)
        for s in step.decodes:  # PagedDecodeContext.commit
            cache.lengths[s.slot] += 1
        for s in step.decodes:
            sched.append_token(s, token, 0.0)
    return seqs
