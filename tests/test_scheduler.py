"""The scheduler: the oracle's restatement and the native (C++) one against the reference.

``tests/golden/scheduler_traces.json`` records, step by step, what the reference's
``Scheduler`` over its ``PagedKVCache`` decided on seeded workloads
(``tests/golden/sched_driver.py``): admissions with their slots and prefix-cache hits,
decodes, finishes with their reasons, rejections, aborts, the queues, preemptions and the
cache's free blocks. Both the oracle (``oracle/scheduler.py``) and the native scheduler
(``mini_inference_b200.scheduler`` over ``csrc/scheduler.cpp`` and the C++ block manager)
must reproduce every record exactly; a random differential test then compares the two
on more workloads. Host code only: no GPU.
"""

from __future__ import annotations

import json
import sys
from dataclasses import dataclass, field
from types import SimpleNamespace

import pytest
import torch

from oracle.block_manager import OracleBlockManager
from oracle.scheduler import OracleSampling, OracleScheduler, OracleSequence

from .conftest import GOLDEN

sys.path.insert(0, str(GOLDEN))
from sched_driver import drive, make_workload  # noqa: E402


@dataclass
class Sampling:
    max_tokens: int = 128
    ignore_eos: bool = False


@dataclass(eq=False)
class Seq:
    """The fields and properties of the reference's Sequence (engine/sequence.py:58-100)."""

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
    def is_finished(self):
        from mini_inference_b200.scheduler import SequenceStatus
        return self.status is SequenceStatus.FINISHED


def _traces():
    return json.loads((GOLDEN / "scheduler_traces.json").read_text())


def _run_oracle(cfg, workload):
    cache = OracleBlockManager(cfg["num_blocks"], cfg["block_size"], cfg["max_num_seqs"], cfg["max_model_len"],
                               cfg["enable_prefix_caching"])
    sched = OracleScheduler(cfg["max_num_seqs"], cfg["max_num_batched_tokens"], cfg["max_model_len"], cache,
                            cfg["eos_token_ids"], cfg["static"])
    return drive(sched, lambda i, p, m, ig: OracleSequence(i, p, OracleSampling(m, ig)), cache, workload, cfg["steps"])


def _run_native(cfg, workload):
    from mini_inference_b200 import PagedKVCache
    from mini_inference_b200.scheduler import Scheduler, SequenceStatus

    cache = PagedKVCache(num_layers=1, num_kv_heads=1, head_dim=4, num_blocks=cfg["num_blocks"],
                         block_size=cfg["block_size"], max_seqs=cfg["max_num_seqs"], max_len=cfg["max_model_len"],
                         dtype=torch.float32, device="cpu", enable_prefix_caching=cfg["enable_prefix_caching"])
    config = SimpleNamespace(max_num_seqs=cfg["max_num_seqs"], max_num_batched_tokens=cfg["max_num_batched_tokens"],
                             max_model_len=cfg["max_model_len"],
                             scheduling="static" if cfg["static"] else "continuous")
    sched = Scheduler(config, cache, eos_token_ids=cfg["eos_token_ids"])

    def make(i, p, m, ig):
        return Seq(i, p, Sampling(m, ig), status=SequenceStatus.WAITING)

    return drive(sched, make, cache, workload, cfg["steps"])


@pytest.mark.parametrize("case", [t["name"] for t in _traces()])
def test_oracle_matches_the_reference(case):
    t = next(t for t in _traces() if t["name"] == case)
    assert _run_oracle(t["config"], t["workload"]) == t["records"]


@pytest.mark.parametrize("case", [t["name"] for t in _traces()])
def test_native_scheduler_matches_the_reference(case):
    t = next(t for t in _traces() if t["name"] == case)
    got = _run_native(t["config"], t["workload"])
    for g, want in zip(got, t["records"]):
        assert g == want, f"step {want['step']}"
    assert len(got) == len(t["records"])


def test_traces_exercise_every_rule():
    recs = [r for t in _traces() for r in t["records"]]
    reasons = {f[1] for r in recs for f in r["finished"]}
    assert {"eos", "length", "max_model_len"} <= reasons
    assert {a[1] for r in recs for a in r["aborted"]} >= {"waiting", "running", "finished"}
    assert any(r["rejected"] for r in recs)
    assert max(t["records"][-1]["num_preemptions"] for t in _traces()) > 0
    assert any(p[2] > 0 for r in recs for p in r["prefills"])  # prefix-cache hits at admission


@pytest.mark.parametrize("seed", range(8))
def test_native_matches_oracle_on_random_workloads(seed):
    import random

    rng = random.Random(1000 + seed)
    cfg = {"num_blocks": rng.randint(12, 80), "block_size": rng.choice([4, 8, 16]), "max_num_seqs": rng.randint(2, 12),
           "max_model_len": rng.randint(64, 200), "static": rng.random() < 0.25,
           "enable_prefix_caching": rng.random() < 0.7, "eos_token_ids": [0, 1], "steps": 150}
    cfg["max_num_batched_tokens"] = cfg["max_model_len"] + rng.randint(0, 200)
    workload = make_workload(seed, rng.randint(10, 40), cfg["steps"], max_tokens=(1, 70), n_aborts=6)
    assert _run_native(cfg, workload) == _run_oracle(cfg, workload)


def test_add_rejects_like_the_reference():
    from mini_inference_b200 import PagedKVCache
    from mini_inference_b200.scheduler import Scheduler

    cache = PagedKVCache(1, 1, 4, 16, 4, 4, 32, torch.float32, "cpu")
    sched = Scheduler(SimpleNamespace(max_num_seqs=4, max_num_batched_tokens=64, max_model_len=32,
                                      scheduling="continuous"), cache)
    with pytest.raises(ValueError, match="prompt is empty"):
        sched.add(Seq(0, [], Sampling()))
    with pytest.raises(ValueError, match="max_model_len is 32"):
        sched.add(Seq(1, list(range(32)), Sampling()))
    assert not sched.has_work()


def test_needs_the_native_cache():
    from mini_inference_b200.scheduler import Scheduler

    with pytest.raises(TypeError):
        Scheduler(SimpleNamespace(max_num_seqs=4, max_num_batched_tokens=64, max_model_len=32,
                                  scheduling="continuous"), OracleBlockManager(8, 4, 4, 32))


def _chunked_engine_loop(prompts, budget, max_seqs=4, blocks=64, max_tokens=3, chunked=True):
    """The engine's side of (chunked) prefill on the allocator alone: returns per step
    (prefills as (id, start, count, final), decode ids). Every step also checks the decodes'
    slots and last tokens as the native scheduler reports them for the engine."""
    from mini_inference_b200 import PagedKVCache
    from mini_inference_b200.scheduler import Scheduler, SequenceStatus

    cache = PagedKVCache(num_layers=1, num_kv_heads=1, head_dim=4, num_blocks=blocks, block_size=16,
                         max_seqs=max_seqs, max_len=512, dtype=torch.float32, device="cpu")
    sched = Scheduler(SimpleNamespace(max_num_seqs=max_seqs, max_num_batched_tokens=budget, max_model_len=512,
                                      scheduling="continuous", chunked_prefill=chunked), cache)
    seqs = [Seq(i, list(p), Sampling(max_tokens, True), status=SequenceStatus.WAITING) for i, p in enumerate(prompts)]
    for s in seqs:
        sched.add(s)
    log = []
    while sched.has_work():
        out = sched.schedule()
        assert sched.decode_slots().tolist() == [s.slot for s in out.decodes]
        assert sched.decode_last_tokens().tolist() == [(s.output_token_ids or s.prompt_token_ids)[-1]
                                                       for s in out.decodes]
        step = []
        done = []
        for s, n in zip(out.prefills, out.prefill_tokens):
            a = cache.lengths[s.slot]
            cache.lengths[s.slot] = a + n
            final = a + n == s.num_tokens
            step.append((s.seq_id, a, n, final))
            if final:
                done.append(s)
        tok = 7000 + 10 * len(log)  # a different token per step and sequence
        sched.append_tokens(done, [tok + i for i in range(len(done))], 0.0)
        for s in out.decodes:
            cache.lengths[s.slot] += 1
        sched.append_tokens(out.decodes, [tok + 5 + i for i in range(len(out.decodes))], 0.0)
        log.append((step, [s.seq_id for s in out.decodes]))
        assert len(log) < 100
    return log, seqs


def test_chunked_prefill_splits_prompts_under_the_budget():
    log, seqs = _chunked_engine_loop([list(range(150)), list(range(1000, 1030))], budget=64)
    assert log[0] == ([(0, 0, 64, False)], [])  # the long prompt takes the whole budget
    assert log[1] == ([(0, 64, 64, False)], [])
    assert log[2] == ([(0, 128, 22, True), (1, 0, 30, True)], [])  # its rest, then the next admission
    assert log[3] == ([], [0, 1])  # both decode from here on
    assert all(len(s.output_token_ids) == 3 for s in seqs)


def test_chunked_prefill_runs_decodes_first_and_finishes_a_one_token_tail_by_decode():
    # Budget 33 with one decode running: the new 40-token prompt gets 32, then 8 minus the decode's share.
    log, seqs = _chunked_engine_loop([list(range(20)), list(range(500, 540))], budget=33, max_tokens=4)
    assert log[0][0] == [(0, 0, 20, True), (1, 0, 13, False)]
    assert log[1] == ([(1, 13, 27, True)], [0])
    for step, decodes in log:
        assert sum(n for _, _, n, _ in step) + len(decodes) <= 33
    # A 33-token prompt under a 32-token budget leaves one token, which the next step decodes.
    log, _ = _chunked_engine_loop([list(range(33))], budget=32, max_tokens=2)
    assert log[0] == ([(0, 0, 32, False)], []) and log[1] == ([], [0])


def test_decode_last_tokens_without_chunked_prefill():
    """The slots and last tokens the scheduler reports for a step's decodes (checked every
    step in the loop) with whole-prompt prefills and preemptions in a small pool."""
    prompts = [list(range(k * 100, k * 100 + 20 + 7 * k)) for k in range(6)]
    log, seqs = _chunked_engine_loop(prompts, budget=256, max_seqs=4, blocks=8, max_tokens=12, chunked=False)
    assert any(decodes for _, decodes in log)
    assert all(len(s.output_token_ids) == 12 for s in seqs)
