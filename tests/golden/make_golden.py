"""Generate the golden fixtures in this directory by running the reference's own code.

Usage::

    python tests/golden/make_golden.py --reference <mini-inference checkout>

It imports ``engine.kv_cache`` and ``engine.model`` from a checkout of
Ham12-3/mini-inference (pure Python + PyTorch, run on the CPU) and records:

* ``allocator_traces.json`` -- seeded sequences of allocator calls
  (``allocate`` with and without token ids, ``register_prefix``,
  ``ensure_capacity``, ``free`` including double frees, ``can_allocate``, and
  writes to ``lengths`` as a prefill commit does) with the result of every
  call and the allocator state after it: block tables, lengths, free-block
  order, free slot count, refcounts, cached blocks and ``prefix_hit_tokens``
  (``engine/kv_cache.py:411-560``). The reference's own known-answer test
  ``tests/test_kv_cache.py:210-243`` is one of the traces.
* ``write_index.json`` -- ``PagedKVCache.write_index`` on scattered tables
  (``engine/kv_cache.py:562-573``).
* ``decode_<name>.npz`` -- ``PagedDecodeContext(...).attend`` on seeded pools
  filled through ``packed_prefill_context`` (``engine/kv_cache.py:592-620``):
  the pool before, tables, positions, q, new k/v, the output and the pool after.
* ``prefill_<name>.npz`` -- ``PackedPrefillContext(...).attend`` without a prefix
  (several prompts and one prompt alone) and with prefix-cache hits
  (``engine/kv_cache.py:252-297``).
* ``rope_<name>.npz`` -- ``RotaryEmbedding`` and ``apply_rope``
  (``engine/model.py:169-224``) on seeded q / k at scattered positions: the float32
  table rows, the rows cast to the model dtype, q, k and the rotated q, k.

* ``lm_head_<name>.npz`` -- ``Qwen2ForCausalLM.compute_logits`` and the greedy ``Sampler``
  (``engine/model.py:321-323``, ``engine/sampler.py:27-31``) on seeded hidden rows.
* ``scheduler_traces.json`` -- the reference's ``Scheduler`` over its ``PagedKVCache``
  (``engine/scheduler.py``) on seeded workloads from ``sched_driver.py``: every step's
  prefills, decodes, finishes, queues, preemptions and cache counters.
* ``streams_<name>.npz`` -- greedy token streams of the reference's own model and engine:
  ``Qwen2ForCausalLM`` (``engine/model.py:254-323``) with ``torch.manual_seed(seed)`` and
  ``normal_(0, std)`` over ``named_parameters()`` (std 0.02 at the 0.5B shape), driven as ``LLMEngine.step`` does
  (``ModelRunner.prefill_packed`` / ``decode`` on a ``PagedKVCache``, the ``Scheduler``,
  ``pack_by_budget``, ``register_prefix`` and the greedy ``Sampler``,
  ``engine/engine.py:99-123,281-312``) in float32 on the CPU, for prompts drawn as the task's
  configuration 1 draws them: the generated tokens of every request and, for every sampled
  row, its 32 largest logits (ids and values). ``0p5b`` is configuration 1 itself (the
  Qwen2.5-0.5B shape); ``0p5b_unit_norms`` the same draws with the RMSNorm weights then set
  to 1 (their own initial value), which makes the tokens depend on the context;
  ``0p5b_prefix`` the latter with prefix caching on 12 prompts that share a 96-token prefix
  under a 256-token step budget (it records the cache's ``prefix_hit_tokens`` and each
  request's cached tokens); ``small`` a 2-layer model for the CPU check of the oracle's engine.

The reference does not travel with this repository, so the fixtures are
committed and this script is only rerun by hand.
"""

from __future__ import annotations

import argparse
import json
import random
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _state(cache) -> dict:
    return {
        "block_tables": {str(s): list(t) for s, t in sorted(cache.block_tables.items())},
        "lengths": {str(s): n for s, n in sorted(cache.lengths.items())},
        "free_blocks": list(cache._free_blocks),
        "num_free_slots": cache.num_free_slots,
        "prefix_hit_tokens": cache.prefix_hit_tokens,
        "ref_counts": list(cache._ref_counts),
        "cached_blocks": sorted(cache._block_key),
    }


def _apply(cache, op: dict):
    kind = op["op"]
    try:
        if kind == "allocate":
            return cache.allocate(op["num_tokens"], token_ids=op["token_ids"])
        if kind == "register_prefix":
            return cache.register_prefix(op["slot"], op["token_ids"])
        if kind == "ensure_capacity":
            return cache.ensure_capacity(op["slot"], op["num_tokens"])
        if kind == "free":
            return cache.free(op["slot"])
        if kind == "can_allocate":
            return cache.can_allocate(op["num_tokens"])
        if kind == "set_length":
            cache.lengths[op["slot"]] = op["value"]
            return None
    except RuntimeError as e:
        return {"error": "RuntimeError", "message": str(e)}
    raise ValueError(kind)


def _run_trace(PagedKVCache, config: dict, ops: list[dict]) -> dict:
    cache = PagedKVCache(num_layers=1, num_kv_heads=1, head_dim=4, num_blocks=config["num_blocks"],
                         block_size=config["block_size"], max_seqs=config["max_seqs"], max_len=config["max_len"],
                         dtype=torch.float32, device="cpu",
                         enable_prefix_caching=config["enable_prefix_caching"])
    steps = []
    for op in ops:
        result = _apply(cache, op)
        steps.append({"op": op, "result": result, "state": _state(cache)})
    return {"config": config, "steps": steps}


def _known_answer_ops() -> tuple[dict, list[dict]]:
    """The call sequence of the reference's ``test_prefix_blocks_are_shared_refcounted_and_evicted_lru``."""
    shared = list(range(100, 116))
    a_tokens = shared + [1, 2, 3]
    b_tokens = shared + [7, 8]
    ops = [
        {"op": "allocate", "num_tokens": len(a_tokens), "token_ids": a_tokens},
        {"op": "set_length", "slot": 0, "value": len(a_tokens)},
        {"op": "register_prefix", "slot": 0, "token_ids": a_tokens},
        {"op": "allocate", "num_tokens": len(b_tokens), "token_ids": b_tokens},
        {"op": "allocate", "num_tokens": 16, "token_ids": shared},
        {"op": "free", "slot": 0},
        {"op": "free", "slot": 1},
        {"op": "free", "slot": 2},
        {"op": "allocate", "num_tokens": 18, "token_ids": shared + [5, 6]},
        {"op": "free", "slot": 2},
        {"op": "allocate", "num_tokens": 64, "token_ids": list(range(64))},
        {"op": "free", "slot": 2},
        {"op": "allocate", "num_tokens": 18, "token_ids": shared + [5, 6]},
    ]
    config = {"num_blocks": 16, "block_size": 4, "max_seqs": 4, "max_len": 64, "enable_prefix_caching": True}
    return config, ops


def _bookkeeping_ops() -> tuple[dict, list[dict]]:
    """The call sequence of the reference's ``test_paged_block_bookkeeping``, plus its double free."""
    ops = [
        {"op": "allocate", "num_tokens": 5, "token_ids": None},
        {"op": "ensure_capacity", "slot": 0, "num_tokens": 8},
        {"op": "ensure_capacity", "slot": 0, "num_tokens": 9},
        {"op": "allocate", "num_tokens": 12, "token_ids": None},
        {"op": "can_allocate", "num_tokens": 1},
        {"op": "ensure_capacity", "slot": 1, "num_tokens": 13},
        {"op": "free", "slot": 0},
        {"op": "can_allocate", "num_tokens": 12},
        {"op": "free", "slot": 0},
    ]
    config = {"num_blocks": 6, "block_size": 4, "max_seqs": 4, "max_len": 32, "enable_prefix_caching": False}
    return config, ops


def _random_ops(seed: int, config: dict, n_ops: int) -> list[dict]:
    """A serving-like random workload: shared prompt prefixes, prefill commits, decode growth, frees."""
    rng = random.Random(seed)
    bs, max_len = config["block_size"], config["max_len"]
    prefixes = [[rng.randrange(50) for _ in range(rng.randrange(bs, 4 * bs + 3))] for _ in range(3)]
    live: dict[int, list[int]] = {}  # slot -> token ids (as the test harness believes)
    # Slot ids mirror the reference's rule so the generator can address them.
    stack = list(range(config["max_seqs"] - 1, -1, -1))
    lengths: dict[int, int] = {}
    ops = []
    for _ in range(n_ops):
        r = rng.random()
        if r < 0.35 or not live:
            base = list(rng.choice(prefixes)) if rng.random() < 0.7 else []
            toks = base + [rng.randrange(50) for _ in range(rng.randrange(1, 2 * bs + 2))]
            toks = toks[: max_len]
            ids = toks if rng.random() < 0.9 else None
            n = len(toks) if rng.random() < 0.9 else rng.randrange(0, max_len + 4)
            ops.append({"op": "allocate", "num_tokens": n, "token_ids": ids})
            # The generator cannot know whether it succeeded; it is recorded in the trace.
            # Track optimistically; failed ones are cleaned up by later frees raising errors.
            if stack:
                s = stack[-1]
                live[s] = toks
        elif r < 0.55:
            s = rng.choice(sorted(live))
            n = len(live[s])
            ops.append({"op": "set_length", "slot": s, "value": n})
            ops.append({"op": "register_prefix", "slot": s, "token_ids": live[s]})
            lengths[s] = n
        elif r < 0.75:
            s = rng.choice(sorted(live))
            grow = live[s] + [rng.randrange(50) for _ in range(rng.randrange(1, bs + 2))]
            live[s] = grow[: max_len + 1]
            ops.append({"op": "ensure_capacity", "slot": s, "num_tokens": len(live[s])})
        elif r < 0.8:
            ops.append({"op": "can_allocate", "num_tokens": rng.randrange(0, max_len + 3)})
        else:
            s = rng.choice(sorted(live)) if rng.random() < 0.9 else rng.randrange(config["max_seqs"])
            ops.append({"op": "free", "slot": s})
            live.pop(s, None)
    return ops


def _fix_trace_slots(PagedKVCache, config: dict, ops: list[dict]) -> list[dict]:
    """Drop ops that address slots the reference never handed out (a KeyError is not part of the API)."""
    cache = PagedKVCache(num_layers=1, num_kv_heads=1, head_dim=4, num_blocks=config["num_blocks"],
                         block_size=config["block_size"], max_seqs=config["max_seqs"], max_len=config["max_len"],
                         dtype=torch.float32, device="cpu", enable_prefix_caching=config["enable_prefix_caching"])
    kept = []
    for op in ops:
        if op["op"] in ("register_prefix", "ensure_capacity", "set_length") and op["slot"] not in cache.block_tables:
            continue
        if op["op"] == "set_length":  # a prefill commit never exceeds the blocks it was given
            op = dict(op, value=min(op["value"], len(cache.block_tables[op["slot"]]) * cache.block_size))
        _apply(cache, op)
        kept.append(op)
    return kept


def make_allocator_traces(PagedKVCache) -> None:
    traces = []
    for cfg, ops in (_known_answer_ops(), _bookkeeping_ops()):
        traces.append(_run_trace(PagedKVCache, cfg, ops))
    random_cfgs = [
        {"num_blocks": 24, "block_size": 4, "max_seqs": 6, "max_len": 48, "enable_prefix_caching": True},
        {"num_blocks": 40, "block_size": 16, "max_seqs": 5, "max_len": 160, "enable_prefix_caching": True},
        {"num_blocks": 12, "block_size": 4, "max_seqs": 4, "max_len": 32, "enable_prefix_caching": False},
        {"num_blocks": 9, "block_size": 2, "max_seqs": 8, "max_len": 16, "enable_prefix_caching": True},
    ]
    for seed, cfg in enumerate(random_cfgs):
        ops = _fix_trace_slots(PagedKVCache, cfg, _random_ops(seed, cfg, 160))
        traces.append(_run_trace(PagedKVCache, cfg, ops))
    (HERE / "allocator_traces.json").write_text(json.dumps(traces, separators=(",", ":")))


def make_write_index(PagedKVCache) -> None:
    cache = PagedKVCache(num_layers=1, num_kv_heads=1, head_dim=4, num_blocks=32, block_size=4, max_seqs=4,
                         max_len=64, dtype=torch.float32, device="cpu")
    slots = [cache.allocate(0) for _ in range(3)]
    for grow in range(1, 6):
        for s in slots:
            cache.ensure_capacity(s, grow * 4 + s)
    cases = []
    for starts, counts in (([0, 0, 0], [5, 9, 3]), ([3, 7, 0], [4, 1, 13]), ([19, 0, 4], [1, 20, 0])):
        b, o = cache.write_index(slots, starts, counts)
        cases.append({"slots": slots, "starts": starts, "counts": counts, "blocks": b.tolist(), "offsets": o.tolist()})
    out = {"block_size": 4, "tables": {str(s): cache.block_tables[s] for s in slots}, "cases": cases}
    (HERE / "write_index.json").write_text(json.dumps(out, separators=(",", ":")))


def _written_rows(before: torch.Tensor, after: torch.Tensor) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Rows ``[block, :, offset]`` of one layer that the call changed, and their new contents.

    Storing only these keeps the fixtures small; the full after-state is
    ``before`` with exactly these rows replaced.
    """
    diff = (before != after).any(dim=(1, 3))  # [blocks, block_size]
    blocks, offsets = torch.nonzero(diff, as_tuple=True)
    return blocks.numpy(), offsets.numpy(), _np(after[blocks, :, offsets])


def _np(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:  # numpy has no bfloat16: keep the bit pattern
        return t.view(torch.int16).numpy().copy()
    return t.numpy().copy()


def make_decode_case(PagedKVCache, name: str, dtype, hq: int, hkv: int, d: int, bs: int, num_blocks: int,
                     lengths: list[int], layers: int, layer: int, seed: int) -> None:
    torch.manual_seed(seed)
    cache = PagedKVCache(num_layers=layers, num_kv_heads=hkv, head_dim=d, num_blocks=num_blocks, block_size=bs,
                         max_seqs=len(lengths) + 1, max_len=num_blocks * bs, dtype=dtype, device="cpu")
    # Stale data everywhere: the kernel must never read outside a sequence's table and length.
    cache.k.normal_()
    cache.v.normal_()
    slots = [cache.allocate(0) for _ in lengths]
    # Interleaved growth scatters each sequence's blocks over the pool.
    most = max(lengths) + 1
    for n in range(1, most + bs, bs):
        for s, ln in zip(slots, lengths):
            cache.ensure_capacity(s, min(ln + 1, n))
    with torch.inference_mode():
        for s, ln in zip(slots, lengths):
            if ln == 0:
                continue
            ctx = cache.packed_prefill_context([s], [ln])
            for li in range(layers):
                ctx.attend(li, torch.randn(1, hq, ln, d).to(dtype), torch.randn(1, hkv, ln, d).to(dtype),
                           torch.randn(1, hkv, ln, d).to(dtype))
            ctx.commit()
        k_before, v_before = cache.k.clone(), cache.v.clone()
        batch = len(slots)
        q = torch.randn(batch, hq, 1, d).to(dtype)
        k_new = torch.randn(batch, hkv, 1, d).to(dtype)
        v_new = torch.randn(batch, hkv, 1, d).to(dtype)
        ctx = cache.decode_context(slots)
        positions = ctx.positions.tolist()
        tables = [list(cache.block_tables[s]) for s in slots]
        out = ctx.attend(layer, q, k_new, v_new)
        ctx.commit()
    width = max(len(t) for t in tables)
    tab = np.full((batch, width), -1, np.int64)
    for i, t in enumerate(tables):
        tab[i, : len(t)] = t
    others = [li for li in range(layers) if li != layer]
    assert all(torch.equal(k_before[li], cache.k[li]) and torch.equal(v_before[li], cache.v[li]) for li in others)
    kb, ko, k_rows = _written_rows(k_before[layer], cache.k[layer])
    vb, vo, v_rows = _written_rows(v_before[layer], cache.v[layer])
    np.savez_compressed(
        HERE / f"decode_{name}.npz",
        dtype=np.array(str(dtype).replace("torch.", "")), layer=np.array(layer), block_size=np.array(bs),
        k_before=_np(k_before), v_before=_np(v_before),
        k_written_at=np.stack([kb, ko]), k_written=k_rows, v_written_at=np.stack([vb, vo]), v_written=v_rows,
        tables=tab, table_lens=np.array([len(t) for t in tables]), positions=np.array(positions),
        q=_np(q[:, :, 0]), k_new=_np(k_new[:, :, 0]), v_new=_np(v_new[:, :, 0]), out=_np(out[:, :, 0]),
        slots=np.array(slots),
    )


def make_prefill_case(PagedKVCache, name: str, dtype, hq: int, hkv: int, d: int, bs: int, num_blocks: int,
                      prompt_lens: list[int], prefix_len: int, seed: int) -> None:
    """Packed prefill; with ``prefix_len`` > 0 the first prompt is prefilled alone and registered first."""
    torch.manual_seed(seed)
    g = torch.Generator().manual_seed(seed)
    caching = prefix_len > 0
    cache = PagedKVCache(num_layers=1, num_kv_heads=hkv, head_dim=d, num_blocks=num_blocks, block_size=bs,
                         max_seqs=len(prompt_lens) + 2, max_len=num_blocks * bs, dtype=dtype, device="cpu",
                         enable_prefix_caching=caching)
    cache.k.normal_()
    cache.v.normal_()
    common = torch.randint(0, 1000, (prefix_len,), generator=g).tolist()
    prompts = [common + torch.randint(0, 1000, (n,), generator=g).tolist() for n in prompt_lens]
    with torch.inference_mode():
        if caching:
            first = cache.allocate(len(prompts[0]), token_ids=prompts[0])
            n0 = len(prompts[0])
            ctx = cache.packed_prefill_context([first], [n0])
            ctx.attend(0, torch.randn(1, hq, n0, d).to(dtype), torch.randn(1, hkv, n0, d).to(dtype),
                       torch.randn(1, hkv, n0, d).to(dtype))
            ctx.commit()
            cache.register_prefix(first, prompts[0])
            rest = prompts[1:]
        else:
            rest = prompts
        slots = [cache.allocate(len(p), token_ids=p) for p in rest]
        starts = [cache.lengths[s] for s in slots]
        new = [len(p) - a for p, a in zip(rest, starts)]
        total = sum(new)
        q = torch.randn(1, hq, total, d).to(dtype)
        k = torch.randn(1, hkv, total, d).to(dtype)
        v = torch.randn(1, hkv, total, d).to(dtype)
        k_before, v_before = cache.k.clone(), cache.v.clone()
        ctx = cache.packed_prefill_context(slots, new)
        positions = ctx.positions.tolist()
        last_index = ctx.last_index.tolist()
        tables = [list(cache.block_tables[s]) for s in slots]
        out = ctx.attend(0, q, k, v)
        ctx.commit()
    width = max(len(t) for t in tables)
    tab = np.full((len(slots), width), -1, np.int64)
    for i, t in enumerate(tables):
        tab[i, : len(t)] = t
    kb, ko, k_rows = _written_rows(k_before[0], cache.k[0])
    vb, vo, v_rows = _written_rows(v_before[0], cache.v[0])
    np.savez_compressed(
        HERE / f"prefill_{name}.npz",
        dtype=np.array(str(dtype).replace("torch.", "")), block_size=np.array(bs),
        k_before=_np(k_before[0]), v_before=_np(v_before[0]),
        k_written_at=np.stack([kb, ko]), k_written=k_rows, v_written_at=np.stack([vb, vo]), v_written=v_rows,
        tables=tab, table_lens=np.array([len(t) for t in tables]), starts=np.array(starts), lengths=np.array(new),
        positions=np.array(positions), last_index=np.array(last_index),
        q=_np(q[0]), k=_np(k[0]), v=_np(v[0]), out=_np(out[0]), prefix_hit_tokens=np.array(cache.prefix_hit_tokens),
    )


def make_rope_case(RotaryEmbedding, apply_rope, name: str, dtype, hq: int, hkv: int, d: int, n: int,
                   max_positions: int, theta: float, seed: int) -> None:
    g = torch.Generator().manual_seed(seed)
    rope = RotaryEmbedding(d, max_positions, theta)
    positions = torch.randint(0, max_positions, (1, n), generator=g)
    positions[0, :3] = torch.tensor([0, 1, max_positions - 1])  # both ends of the table
    cos, sin = rope(positions, dtype)  # [1, 1, n, d] in the model dtype
    q = (torch.randn(1, hq, n, d, generator=g) * 2).to(dtype)
    k = (torch.randn(1, hkv, n, d, generator=g) * 2).to(dtype)
    q_rot, k_rot = apply_rope(q, k, cos, sin)
    np.savez_compressed(
        HERE / f"rope_{name}.npz",
        dtype=np.array(str(dtype).replace("torch.", "")), theta=np.array(theta), max_positions=np.array(max_positions),
        positions=positions[0].numpy(), cos_f32=rope._cos[positions[0]].numpy(), sin_f32=rope._sin[positions[0]].numpy(),
        cos=_np(cos[0, 0]), sin=_np(sin[0, 0]), q=_np(q[0].transpose(0, 1)), k=_np(k[0].transpose(0, 1)),
        q_rot=_np(q_rot[0].transpose(0, 1)), k_rot=_np(k_rot[0].transpose(0, 1)),
    )


def make_lm_head_case(engine_model, engine_sampler, name: str, dtype, vocab: int, hidden: int, batch: int,
                      tie: bool, seed: int) -> None:
    """``compute_logits`` + the greedy ``Sampler`` on seeded hidden rows, with an exact tie and a NaN row."""
    torch.manual_seed(seed)
    cfg = engine_model.Qwen2Config(vocab_size=vocab, hidden_size=hidden, intermediate_size=4 * hidden, num_layers=0,
                                   num_heads=2, num_kv_heads=1, head_dim=hidden // 2, rms_norm_eps=1e-6,
                                   rope_theta=1e6, max_position_embeddings=64, tie_word_embeddings=tie,
                                   attention_bias=True)
    model = engine_model.Qwen2ForCausalLM(cfg)
    for _, prm in model.named_parameters():
        prm.data.normal_(0, 0.02)
    model = model.to(dtype)
    weight = model.embed_tokens.weight if model.lm_head is None else model.lm_head.weight
    g = torch.Generator().manual_seed(seed + 1)
    h = torch.randn(batch, hidden, generator=g).to(dtype)
    with torch.no_grad():
        # row 1: vocab entries 3 and vocab - 2 get the same, dominant weight row (an exact tie);
        # the reference returns the first.
        weight[vocab - 2] = weight[3] = (h[1].float() * 0.05).to(dtype)
        h[batch - 1, 5] = float("nan")  # a NaN row: every logit is NaN, argmax returns 0
        logits = model.compute_logits(h).float()
    params = [engine_sampler.SamplingParams() for _ in range(batch)]
    tokens = engine_sampler.Sampler(0, "cpu")(logits, params)
    np.savez_compressed(
        HERE / f"lm_head_{name}.npz", dtype=np.array(str(dtype).replace("torch.", "")),
        hidden=_np(h), weight=_np(weight.detach()), logits=logits.numpy(), tokens=np.array(tokens, np.int64),
    )


# (name, seed, requests, steps, cache blocks, block size, max_seqs, token budget, max_model_len, static,
#  prefix caching, max_tokens range, aborts)
SCHED_CASES = [
    ("continuous_prefix", 21, 40, 160, 40, 8, 8, 192, 160, False, True, (1, 80), 8),
    ("continuous_tight", 22, 30, 280, 20, 4, 6, 96, 72, False, True, (1, 60), 8),  # preemptions, rejections
    ("continuous_plain", 23, 30, 120, 64, 16, 16, 4096, 128, False, False, (1, 40), 6),
    ("static", 24, 30, 220, 30, 8, 6, 64, 160, True, True, (1, 60), 8),
]


def make_scheduler_traces(Scheduler, Sequence, SamplingParams, PagedKVCache) -> None:
    """The reference's Scheduler + PagedKVCache over seeded workloads (``sched_driver``)."""
    from types import SimpleNamespace

    from sched_driver import drive, make_workload

    traces = []
    for name, seed, n_req, steps, blocks, bs, max_seqs, budget, max_len, static, prefix, mt, n_ab in SCHED_CASES:
        workload = make_workload(seed, n_req, steps, max_tokens=mt, n_aborts=n_ab)
        config = SimpleNamespace(max_num_seqs=max_seqs, max_num_batched_tokens=budget, max_model_len=max_len,
                                 scheduling="static" if static else "continuous")
        cache = PagedKVCache(num_layers=1, num_kv_heads=1, head_dim=4, num_blocks=blocks, block_size=bs,
                             max_seqs=max_seqs, max_len=max_len, dtype=torch.float32, device="cpu",
                             enable_prefix_caching=prefix)
        sched = Scheduler(config, cache, eos_token_ids=(0, 1))

        def make_seq(i, prompt, max_tokens, ignore_eos):
            return Sequence(seq_id=i, prompt_token_ids=prompt,
                            sampling=SamplingParams(max_tokens=max_tokens, ignore_eos=ignore_eos), arrival_time=0.0)

        records = drive(sched, make_seq, cache, workload, steps)
        traces.append({"name": name, "config": {"num_blocks": blocks, "block_size": bs, "max_num_seqs": max_seqs,
                                                "max_num_batched_tokens": budget, "max_model_len": max_len,
                                                "static": static, "enable_prefix_caching": prefix,
                                                "eos_token_ids": [0, 1], "steps": steps},
                       "workload": workload, "records": records})
    (HERE / "scheduler_traces.json").write_text(json.dumps(traces))


# Shapes: (layers, hidden, intermediate, vocab, heads, kv heads, head_dim).
_0P5B = (24, 896, 4864, 151936, 14, 2, 64)
STREAM_CASES = {
    # configuration 1: 8 prompts of U{64..256} ids, 64 greedy tokens
    "0p5b": dict(shape=_0P5B, requests=8, lengths=(64, 256), tokens=64, unit_norms=False, std=0.02),
    "0p5b_unit_norms": dict(shape=_0P5B, requests=8, lengths=(64, 256), tokens=64, unit_norms=True, std=0.02),
    # prefix caching: 12 prompts = one shared 96-token prefix + U{8..40} own ids, a 256-token
    # budget so that admissions spread over steps (the first ones miss, later ones hit)
    "0p5b_prefix": dict(shape=_0P5B, requests=12, lengths=(8, 40), tokens=32, unit_norms=True, std=0.02,
                        prefix=96, caching=True, budget=256),
    "small": dict(shape=(2, 256, 512, 1000, 14, 2, 64), requests=4, lengths=(8, 40), tokens=16, unit_norms=True,
                  std=0.1),
}
TOPK = 32


def make_greedy_streams(engine_model, engine_engine, engine_scheduler, engine_sampler, engine_sequence,
                        PagedKVCache, only: str | None = None) -> None:
    """Greedy streams of the reference's model and engine loop (float32, CPU)."""
    from types import SimpleNamespace

    for name, case in STREAM_CASES.items():
        if only and name != only:
            continue
        layers, hidden, inter, vocab, hq, hkv, d = case["shape"]
        n_req, (lo, hi), n_tok = case["requests"], case["lengths"], case["tokens"]
        unit_norms, std, prefix_len = case["unit_norms"], case["std"], case.get("prefix", 0)
        caching, budget = case.get("caching", False), case.get("budget", 4096)
        cfg = engine_model.Qwen2Config(vocab_size=vocab, hidden_size=hidden, intermediate_size=inter,
                                       num_layers=layers, num_heads=hq, num_kv_heads=hkv, head_dim=d,
                                       rms_norm_eps=1e-6, rope_theta=1e6, max_position_embeddings=32768,
                                       tie_word_embeddings=True, attention_bias=True)
        model = engine_model.Qwen2ForCausalLM(cfg)
        torch.manual_seed(0)
        with torch.no_grad():
            for pname, prm in model.named_parameters():
                prm.normal_(0, std)
                if unit_norms and pname.endswith("norm.weight"):
                    prm.fill_(1.0)
        model = model.eval()
        g = torch.Generator().manual_seed(0)
        shared = torch.randint(0, vocab, (prefix_len,), generator=g).tolist()
        lens = torch.randint(lo, hi + 1, (n_req,), generator=g).tolist()
        prompts = [shared + torch.randint(0, vocab, (n,), generator=g).tolist() for n in lens]
        lens = [len(p) for p in prompts]
        max_len = prefix_len + hi + n_tok + 16
        cache = PagedKVCache.for_model(cfg, num_blocks=n_req * (max_len // 16 + 1), block_size=16, max_seqs=n_req,
                                       max_len=max_len, dtype=torch.float32, device="cpu",
                                       enable_prefix_caching=caching)
        runner = engine_engine.ModelRunner(model, cache)
        conf = SimpleNamespace(max_num_seqs=n_req, max_num_batched_tokens=budget, max_model_len=max_len,
                               scheduling="continuous")
        sched = engine_scheduler.Scheduler(conf, cache)
        sampler = engine_sampler.Sampler(0, "cpu")
        seqs = [engine_sequence.Sequence(i, p, engine_sequence.SamplingParams(max_tokens=n_tok, ignore_eos=True), 0.0)
                for i, p in enumerate(prompts)]
        for s in seqs:
            sched.add(s)
        top_ids = np.zeros((n_req, n_tok, TOPK), np.int32)
        top_vals = np.zeros((n_req, n_tok, TOPK), np.float32)

        def record(batch_seqs, logits):
            v, i = logits.topk(TOPK, dim=-1)
            for s, vv, ii in zip(batch_seqs, v, i):
                j = len(s.output_token_ids)
                top_ids[s.seq_id, j], top_vals[s.seq_id, j] = ii.numpy(), vv.numpy()

        with torch.inference_mode():
            while sched.has_work():  # LLMEngine.step (engine/engine.py:281-312)
                batch = sched.schedule()
                new_of = {s.seq_id: s.token_ids[cache.lengths[s.slot]:] for s in batch.prefills}
                for group in engine_engine.pack_by_budget([len(new_of[s.seq_id]) for s in batch.prefills], budget):
                    gs = [batch.prefills[i] for i in group]
                    logits = runner.prefill_packed([s.slot for s in gs], [new_of[s.seq_id] for s in gs])
                    for s in gs:
                        cache.register_prefix(s.slot, s.token_ids)
                    record(gs, logits)
                    for s, t in zip(gs, sampler(logits, [s.sampling for s in gs])):
                        sched.append_token(s, t, 0.0)
                if batch.decodes:
                    logits = runner.decode([s.slot for s in batch.decodes], [s.last_token for s in batch.decodes])
                    record(batch.decodes, logits)
                    for s, t in zip(batch.decodes, sampler(logits, [s.sampling for s in batch.decodes])):
                        sched.append_token(s, t, 0.0)
        flat = [t for p in prompts for t in p]
        np.savez_compressed(
            HERE / f"streams_{name}.npz",
            config=np.array([layers, hidden, inter, vocab, hq, hkv, d], np.int64), unit_norms=np.array(unit_norms),
            std=np.array(std), seed=np.array(0), max_model_len=np.array(max_len),
            prompt_lens=np.array(lens, np.int64), prompt_ids=np.array(flat, np.int64),
            tokens=np.array([s.output_token_ids for s in seqs], np.int64), top_ids=top_ids, top_vals=top_vals,
            threads=np.array(torch.get_num_threads()), prefix_caching=np.array(caching), budget=np.array(budget),
            prefix_hit_tokens=np.array(cache.prefix_hit_tokens),
            cached_tokens=np.array([s.num_cached_tokens for s in seqs], np.int64))
        print(name, "distinct tokens per stream:", [len(set(s.output_token_ids)) for s in seqs],
              "prefix hit tokens:", cache.prefix_hit_tokens)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", required=True, help="path of a Ham12-3/mini-inference checkout")
    ap.add_argument("--only", choices=["rope", "lm_head", "scheduler", "streams"], help="write only these fixtures")
    ap.add_argument("--stream-case", help="with --only streams: just this case")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference).resolve()))
    from engine.kv_cache import PagedKVCache  # noqa: E402  (the reference's own class)
    from engine.model import RotaryEmbedding, apply_rope  # noqa: E402

    torch.set_num_threads(4)
    if args.only == "streams":
        import engine.engine as engine_engine  # noqa: E402
        import engine.model as engine_model  # noqa: E402
        import engine.sampler as engine_sampler  # noqa: E402
        import engine.scheduler as engine_scheduler  # noqa: E402
        import engine.sequence as engine_sequence  # noqa: E402
        make_greedy_streams(engine_model, engine_engine, engine_scheduler, engine_sampler, engine_sequence,
                            PagedKVCache, args.stream_case)
        print("stream fixtures written to", HERE)
        return
    if args.only == "scheduler":
        sys.path.insert(0, str(HERE))
        from engine.scheduler import Scheduler  # noqa: E402
        from engine.sequence import SamplingParams, Sequence  # noqa: E402
        make_scheduler_traces(Scheduler, Sequence, SamplingParams, PagedKVCache)
        print("scheduler traces written to", HERE)
        return
    if args.only == "lm_head":
        import engine.model as engine_model  # noqa: E402
        import engine.sampler as engine_sampler  # noqa: E402  (it imports SamplingParams)
        # Qwen2.5-0.5B style (tied embedding, fp16) and 7B style (separate lm_head, bf16), small sizes;
        # vocabularies that are not multiples of 64.
        make_lm_head_case(engine_model, engine_sampler, "fp16_tied", torch.float16, 1000, 128, 7, True, seed=13)
        make_lm_head_case(engine_model, engine_sampler, "bf16", torch.bfloat16, 777, 192, 5, False, seed=14)
        print("lm_head fixtures written to", HERE)
        return
    # Qwen2.5-0.5B (d 64, theta 1e6) and 7B (d 128) rotary shapes; tokens as rows [n, heads, d].
    make_rope_case(RotaryEmbedding, apply_rope, "fp16_h14_d64", torch.float16, 14, 2, 64, 37, 32768, 1e6, seed=11)
    make_rope_case(RotaryEmbedding, apply_rope, "bf16_h28_d128", torch.bfloat16, 28, 4, 128, 21, 33024, 1e6, seed=12)
    if args.only == "rope":
        print("rope fixtures written to", HERE)
        return
    make_allocator_traces(PagedKVCache)
    make_write_index(PagedKVCache)
    # The reference's own tiny test shapes (tests/test_kv_cache.py:158-160,179-207): 4 / 2 heads, dim 8, blocks of 4.
    make_decode_case(PagedKVCache, "fp32_tiny", torch.float32, 4, 2, 8, 4, 12, [6, 9, 3], layers=1, layer=0, seed=1)
    # Micro-benchmark head shape (Qwen2.5-0.5B): 14 / 2 heads, head_dim 64, blocks of 16.
    make_decode_case(PagedKVCache, "fp16_h14_d64", torch.float16, 14, 2, 64, 16, 16,
                     [70, 16, 47, 3, 31, 0], layers=2, layer=1, seed=2)
    # Qwen2.5-7B head shape: 28 / 4 heads, head_dim 128.
    make_decode_case(PagedKVCache, "bf16_h28_d128", torch.bfloat16, 28, 4, 128, 16, 8,
                     [40, 17, 2], layers=1, layer=0, seed=3)
    make_decode_case(PagedKVCache, "fp16_h28_d128", torch.float16, 28, 4, 128, 16, 9,
                     [33, 15, 48], layers=1, layer=0, seed=4)
    make_prefill_case(PagedKVCache, "fp32_tiny_packed", torch.float32, 4, 2, 8, 4, 12, [5, 3, 7], 0, seed=5)
    make_prefill_case(PagedKVCache, "fp16_single", torch.float16, 14, 2, 64, 16, 5, [50], 0, seed=6)
    make_prefill_case(PagedKVCache, "fp16_packed", torch.float16, 14, 2, 64, 16, 8, [23, 5, 40], 0, seed=10)
    make_prefill_case(PagedKVCache, "fp16_prefix", torch.float16, 14, 2, 64, 16, 12, [9, 20, 1, 16], 40, seed=7)
    make_prefill_case(PagedKVCache, "fp32_tiny_prefix", torch.float32, 4, 2, 8, 4, 24, [3, 10, 7], 9, seed=8)
    make_prefill_case(PagedKVCache, "bf16_prefix_d128", torch.bfloat16, 28, 4, 128, 16, 8, [12, 9], 32, seed=9)
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
