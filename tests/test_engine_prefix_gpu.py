"""Configuration 4 end to end: prefix caching at scale (needs a B200).

256 requests share one seeded 1024-token prefix and add U{64..256} tokens of their own;
each generates 128 greedy tokens (``bench.prefix_workload``), served by ``LLMEngine`` with
prefix caching on and the reference's 4096-token step budget. The requests admitted in the
first step miss (their prefix is registered only after their prefill,
``engine/engine.py:297-298``) and later ones hit the 64 prefix blocks. The engine's
``prefix_hit_tokens`` and every request's cached tokens must equal the oracle's replay of the
reference's scheduler and allocator on the same workload exactly.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    return torch.device("cuda", 0)


def test_config4_prefix_hits_equal_the_oracle(dev):
    import bench
    from mini_inference_b200.engine import EngineConfig, LLMEngine, SamplingParams
    from mini_inference_b200.model import Qwen2Config, Qwen2Model, init_random
    from oracle.block_manager import OracleBlockManager
    from oracle.engine_torch import serve_bookkeeping

    cfg = Qwen2Config.qwen2_0_5b()
    requests = bench.prefix_workload(vocab=cfg.vocab_size)
    kv_tokens, max_len, budget, seqs_max = bench.SERVE_KV_TOKENS, bench.SERVE_MAX_LEN, bench.SERVE_BUDGET, 256
    oracle_cache = OracleBlockManager(kv_tokens // 16, 16, seqs_max, max_len, enable_prefix_caching=True)
    want = serve_bookkeeping(oracle_cache, requests, seqs_max, budget, max_len)

    model = Qwen2Model(cfg, init_random(cfg, seed=0, dtype=torch.float16, device=dev, generator_device="cuda"))
    engine = LLMEngine(model, EngineConfig(max_num_seqs=seqs_max, max_model_len=max_len, max_num_batched_tokens=budget,
                                           kv_cache_tokens=kv_tokens, enable_prefix_caching=True))
    got = engine.generate([p for p, _ in requests], [SamplingParams(max_tokens=m, ignore_eos=True) for _, m in requests])
    assert all(len(s.output_token_ids) == m for s, (_, m) in zip(got, requests))
    assert engine.cache.prefix_hit_tokens == oracle_cache.prefix_hit_tokens
    assert [s.num_cached_tokens for s in got] == [s.num_cached_tokens for s in want]
    misses = sum(1 for s in got if s.num_cached_tokens == 0)
    assert 0 < misses < 16 and oracle_cache.prefix_hit_tokens == (len(requests) - misses) * 1024
