"""Greedy streams of this package's engine against the reference's own model (needs a B200).

``tests/golden/streams_<case>.npz`` records the reference's ``Qwen2ForCausalLM`` at the
Qwen2.5-0.5B shape, seeded as the task's configuration 1 (``manual_seed(0)``, then
``normal_(0, 0.02)`` over ``named_parameters()``), driven through its own ``ModelRunner``,
``Scheduler`` and greedy ``Sampler`` in float32 on the CPU: 8 prompts of 64..256 uniform
token ids, 64 greedy tokens each, and the 32 largest logits of every sampled row.

``0p5b_prefix`` is the same model (RMSNorm weights set to 1) serving 12 prompts that share a
96-token prefix with prefix caching on, under a 256-token step budget: some requests miss
and some hit, and the reference's ``prefix_hit_tokens`` and per-request cached tokens are
recorded; they must be equal here exactly.

Here the same weights (drawn the same way, cast to float16) run through ``LLMEngine``:
the native scheduler, the paged cache with RoPE fused into the append, tcgen05 prefill,
split-K paged decode replayed as CUDA graphs, and the LM head fused with argmax. Every
stream must equal the reference's over all 64 tokens, except where the two parts at a
tie in the sense of the reference's own parity test (``tests/test_model_parity.py:
122-133``): re-running this path on the shared prefix, the gap between the two tokens'
logits must not exceed the largest difference between the two models' logits (here over
the reference's 32 recorded top logits, a lower bound of the full maximum). The gap is
read from the reference's float32 logits: this path's float16 logits are quantised to one
float16 step, which is as large as the closest ties.
That difference itself must stay within float16 rounding of the logits, at the tie and at
the end of every stream, so a broken path cannot pass by making the noise large.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from tests.test_oracle_engine import stream_case

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    return torch.device("cuda", 0)


def last_logits(model, tokens, dev):
    """This path's float32 logits after ``tokens`` (one packed prefill on a fresh cache), as compute_logits().float()."""
    from mini_inference_b200 import PagedKVCache

    cfg = model.cfg
    cache = PagedKVCache(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, num_blocks=len(tokens) // 16 + 2,
                         block_size=16, max_seqs=1, max_len=len(tokens) + 16, dtype=model.dtype, device=dev)
    slot = cache.allocate(len(tokens))
    ctx = cache.packed_prefill_context([slot], [len(tokens)])
    with torch.inference_mode():
        hidden = model(torch.tensor([tokens], device=dev), ctx.positions.unsqueeze(0), ctx)
        out = F.linear(hidden[0, -1], model.lm_head_weight).float().cpu()
    cache.raise_device_errors()
    return out


@pytest.mark.parametrize("case,chunk", [("0p5b", 0), ("0p5b_unit_norms", 0), ("0p5b_prefix", 0),
                                        ("0p5b_unit_norms", 48)])
def test_greedy_streams_equal_the_reference_model(dev, golden_dir, case, chunk):
    """``chunk`` > 0: the same requests with chunked prefill under a budget of that many tokens
    (every prompt is longer), which the reference does not have: same tokens, same tie rule."""
    from mini_inference_b200.engine import EngineConfig, LLMEngine, SamplingParams
    from mini_inference_b200.model import Qwen2Config, Qwen2Model, init_random

    z, (layers, hidden, inter, vocab, hq, hkv, d), prompts = stream_case(golden_dir, case)
    cfg = Qwen2Config(vocab_size=vocab, hidden_size=hidden, intermediate_size=inter, num_layers=layers,
                      num_heads=hq, num_kv_heads=hkv, head_dim=d)
    model = Qwen2Model(cfg, init_random(cfg, seed=0, std=float(z["std"]), dtype=torch.float16, device=dev,
                                        unit_norms=bool(z["unit_norms"])))
    n_tok = z["tokens"].shape[1]
    max_len = int(z["max_model_len"])
    caching = bool(z["prefix_caching"])
    engine = LLMEngine(model, EngineConfig(max_num_seqs=len(prompts), max_model_len=max_len,
                                           max_num_batched_tokens=chunk or int(z["budget"]),
                                           kv_cache_tokens=len(prompts) * (max_len + 16),
                                           enable_prefix_caching=caching, chunked_prefill=chunk > 0))
    seqs = engine.generate(prompts, SamplingParams(max_tokens=n_tok, ignore_eos=True))
    ref = z["tokens"]
    if chunk:
        assert any(st.num_prefill_tokens and st.num_prefill_tokens <= chunk for st in engine.step_stats)
        assert sum(1 for st in engine.step_stats if st.num_prefills) > len(prompts) * 64 // chunk // 2
    else:  # the same admissions, the same prefix hits (exact), whatever the tokens
        assert engine.cache.prefix_hit_tokens == int(z["prefix_hit_tokens"])
        assert [s.num_cached_tokens for s in seqs] == z["cached_tokens"].tolist()

    def noise_at(b, t, ours):
        """max |reference - ours| over the reference's recorded top logits of stream b, step t."""
        ids = torch.from_numpy(z["top_ids"][b, t].astype(np.int64))
        return float((ours[ids] - torch.from_numpy(z["top_vals"][b, t])).abs().max())

    identical, ties = 0, []
    for b, s in enumerate(seqs):
        got = s.output_token_ids
        assert len(got) == n_tok
        t = next((j for j, (x, y) in enumerate(zip(got, ref[b].tolist())) if x != y), None)
        upto = n_tok - 1 if t is None else t
        ours = last_logits(model, prompts[b] + ref[b, :upto].tolist(), dev)
        noise = noise_at(b, upto, ours)
        scale = max(1.0, float(np.abs(z["top_vals"][b, upto]).max()))
        # float16 rounding of logits this size, compounded over the layers: far below any real mismatch.
        assert noise <= 0.03 * scale, f"stream {b}, step {upto}: logits differ by {noise:.4f} from the reference's"
        if t is None:
            identical += 1
            continue
        # The reference's own gap between its token and ours at this step (ours must be among its
        # top logits at all); float16 logits cannot tell tokens apart much closer than this.
        top_ids = z["top_ids"][b, t].tolist()
        assert got[t] in top_ids, f"stream {b}, token {t}: ours={got[t]} is not among the reference's top {len(top_ids)}"
        gap = float(z["top_vals"][b, t][0] - z["top_vals"][b, t][top_ids.index(got[t])])
        assert gap <= noise, (f"stream {b}, token {t}: ours={got[t]} reference={int(ref[b, t])} with a reference logit "
                              f"gap of {gap:.5f}, larger than the models' difference {noise:.5f}: a real mismatch")
        ties.append((b, t, round(gap, 5), round(noise, 5)))
    print(f"\n{case}: {identical}/{len(seqs)} streams identical for {n_tok} tokens; ties: {ties}")
