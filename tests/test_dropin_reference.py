"""The reference's own Scheduler drives this package's cache, step for step (CPU).

The drop-in claim is that the reference's engine runs unchanged on
``mini_inference_b200.PagedKVCache``. Where a checkout of the reference is available (the
``MINI_INFERENCE_REFERENCE`` environment variable, or a ``reference`` directory beside this
repository) its ``engine/scheduler.py`` ``Scheduler`` is run over both caches, the
reference's ``PagedKVCache`` and this package's (allocator on the CPU), on the seeded
workloads of ``tests/golden/scheduler_traces.json``: every step's admissions, slots,
prefix hits, decodes, finishes, queues, preemptions and free blocks must be equal. Without
a checkout the test is skipped (the recorded traces are checked elsewhere).
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest
import torch

from .conftest import GOLDEN, ROOT

sys.path.insert(0, str(GOLDEN))
from sched_driver import drive  # noqa: E402


def _reference_root() -> Path | None:
    env = os.environ.get("MINI_INFERENCE_REFERENCE")
    for cand in ([Path(env)] if env else []) + [ROOT.parent / "reference"]:
        if (cand / "engine" / "scheduler.py").is_file():
            return cand
    return None


@pytest.fixture(scope="module")
def reference():
    root = _reference_root()
    if root is None:
        pytest.skip("no checkout of the reference available")
    sys.path.insert(0, str(root))
    try:
        import engine.kv_cache as kv
        import engine.scheduler as sch
        import engine.sequence as seq
    finally:
        sys.path.remove(str(root))
    return kv, sch, seq


def _cases():
    import json

    return json.loads((GOLDEN / "scheduler_traces.json").read_text())


@pytest.mark.parametrize("case", range(4))
def test_reference_scheduler_on_this_cache_decides_as_on_its_own(reference, case):
    from types import SimpleNamespace

    from mini_inference_b200 import PagedKVCache

    kv, sch, seq = reference
    trace = _cases()[case]
    cfg = trace["config"]
    config = SimpleNamespace(max_num_seqs=cfg["max_num_seqs"], max_num_batched_tokens=cfg["max_num_batched_tokens"],
                             max_model_len=cfg["max_model_len"], scheduling="static" if cfg["static"] else "continuous")

    def run(cache_cls):
        cache = cache_cls(num_layers=1, num_kv_heads=1, head_dim=4, num_blocks=cfg["num_blocks"],
                          block_size=cfg["block_size"], max_seqs=cfg["max_num_seqs"], max_len=cfg["max_model_len"],
                          dtype=torch.float32, device="cpu", enable_prefix_caching=cfg["enable_prefix_caching"])
        scheduler = sch.Scheduler(config, cache, eos_token_ids=cfg["eos_token_ids"])

        def make(i, prompt, max_tokens, ignore_eos):
            return seq.Sequence(seq_id=i, prompt_token_ids=prompt,
                                sampling=seq.SamplingParams(max_tokens=max_tokens, ignore_eos=ignore_eos),
                                arrival_time=0.0)

        return drive(scheduler, make, cache, trace["workload"], cfg["steps"])

    theirs = run(kv.PagedKVCache)
    ours = run(PagedKVCache)
    assert ours == theirs
    assert ours == trace["records"]  # and both are the recorded trace
