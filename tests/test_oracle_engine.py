"""The oracle's serving loop (``oracle/engine_torch.py``) reproduces the reference's own engine.

``tests/golden/streams_small.npz`` holds the greedy streams and top logits of the
reference's ``Qwen2ForCausalLM`` driven through its ``ModelRunner`` / ``Scheduler`` /
``Sampler`` on the CPU (``make_golden.py``). The oracle, fed the same seeded weights and
prompts, must give the same tokens and the same logits: it is the CPU baseline the
serving benchmark is timed against and the checker of the GPU engine's streams.
"""

from __future__ import annotations

import numpy as np
import torch

from oracle.engine_torch import TorchPagedCache, TorchQwen2, serve


def stream_case(golden_dir, name):
    z = np.load(golden_dir / f"streams_{name}.npz")
    layers, hidden, inter, vocab, hq, hkv, d = (int(x) for x in z["config"])
    lens = z["prompt_lens"].tolist()
    flat = z["prompt_ids"].tolist()
    prompts, at = [], 0
    for n in lens:
        prompts.append(flat[at:at + n])
        at += n
    return z, (layers, hidden, inter, vocab, hq, hkv, d), prompts


def seeded_weights(shape, std, unit_norms):
    """The reference model's parameters in order, drawn as the fixture's were (CPU, float32)."""
    from mini_inference_b200.model import Qwen2Config, init_random

    layers, hidden, inter, vocab, hq, hkv, d = shape
    cfg = Qwen2Config(vocab_size=vocab, hidden_size=hidden, intermediate_size=inter, num_layers=layers,
                      num_heads=hq, num_kv_heads=hkv, head_dim=d)
    return cfg, init_random(cfg, seed=0, std=std, dtype=torch.float32, device="cpu", unit_norms=unit_norms)


def test_oracle_engine_reproduces_the_reference_streams(golden_dir):
    z, shape, prompts = stream_case(golden_dir, "small")
    cfg, w = seeded_weights(shape, float(z["std"]), bool(z["unit_norms"]))
    n_tok = z["tokens"].shape[1]
    model = TorchQwen2(w, cfg.num_layers, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, cfg.rms_norm_eps,
                       cfg.rope_theta, cfg.max_position_embeddings)
    max_len = int(z["max_model_len"])
    cache = TorchPagedCache(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, len(prompts) * (max_len // 16 + 1), 16,
                            len(prompts), max_len, torch.float32)
    seen = {}

    def record(seq, row):
        seen[(seq.seq_id, len(seq.output_token_ids))] = row

    seqs = serve(model, cache, [(p, n_tok) for p in prompts], len(prompts), 4096, max_len, record=record)
    assert [s.output_token_ids for s in seqs] == z["tokens"].tolist()
    for b in range(len(prompts)):
        for j in range(n_tok):
            row = seen[(b, j)]
            np.testing.assert_allclose(row[z["top_ids"][b, j]].numpy(), z["top_vals"][b, j], rtol=1e-5, atol=1e-6)


def test_bookkeeping_replay_gives_the_reference_prefix_hits(golden_dir):
    """Scheduling and prefix hits without a model: the reference's recorded hits, request by request."""
    from oracle.block_manager import OracleBlockManager
    from oracle.engine_torch import serve_bookkeeping

    z, _, prompts = stream_case(golden_dir, "0p5b_prefix")
    max_len = int(z["max_model_len"])
    cache = OracleBlockManager(len(prompts) * (max_len // 16 + 1), 16, len(prompts), max_len,
                               enable_prefix_caching=True)
    seqs = serve_bookkeeping(cache, [(p, z["tokens"].shape[1]) for p in prompts], len(prompts), int(z["budget"]),
                             max_len)
    assert cache.prefix_hit_tokens == int(z["prefix_hit_tokens"]) > 0
    assert [s.num_cached_tokens for s in seqs] == z["cached_tokens"].tolist()
