"""Benchmark of the paged-KV hot path on B200: the paged decode attention micro-benchmark.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P bench.py --gpus N --steps K --warmup W

Workload (configuration 2 of the task, the one the "paged-attn KV GB/s" half of
the metric is quoted on): 64 sequences with context lengths uniform in
128..2048, 14 query / 2 KV heads, head_dim 64, blocks of 16 tokens, fp16,
K/V/Q ~ N(0, 1), block tables = consecutive slices of a seeded permutation of a
16384-block pool, and a one-token KV append per sequence through slot_mapping
in the same call. Data are synthetic (seeded), as the reference's benchmark
has no dataset for this path.

A step is one decode step of that batch through all 24 layers of a
Qwen2.5-0.5B-shaped pool ([24, 16385, 2, 16, 64] for K and for V, 3.2 GB in all,
far above the 126 MB L2, so every layer call reads its KV from HBM): the GPU
metadata builder, then 24 fused append + paged attention calls. ``value`` is
algorithmic KV-path bytes moved per second over the whole job (all ranks);
``e2e`` is the same metric through the C ABI with host buffers (the step's
q / new k / new v and tables copied from pinned host memory, the outputs
copied back, all inside the timed region; the step is one CUDA graph, as the
reference engine runs decode, with the copies chunked to overlap the kernels).

The same line carries the other legs as keys: ``serving`` (config 3: 200 requests
through ``LLMEngine`` at the 0.5B shape, output tok/s, TTFT / TPOT, with a CPU sample of
the reference's loop beside it), ``prefix_serving`` (config 4 with prefix caching and its
``prefix_hit_tokens``), ``long_context`` / ``long_context_step`` (config 5's attention
call and its whole 28-layer 7B-shaped decode step), ``decode_with_rope`` (RoPE fused into
the decode kernel against a separate rotation launch), ``prefill``, ``qkv_post``,
``lm_head`` and ``scheduler``.

Multi-GPU: one process per GPU, each with its own batch and pool (weak scaling,
requests sharded by rank, no collective on the data path); the timed region is
bracketed by barriers and timed on each device with CUDA events, and the job
time is the maximum over ranks. Barriers and the max run on a host ``gloo`` group.

``--impl reference`` times the reference's own algorithm on the host cores:
``oracle/paged_kv_torch.py``, the reference's PyTorch ops for this step
restated on the CPU, on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode tok/s on 200-req mixed workload; paged-attn KV GB/s vs HBM peak"
UNIT = "GB/s"
LAYERS, BATCH, CTX_LO, CTX_HI = 24, 64, 128, 2048
DECODE_KERNELS = 1  # kernels per pkv_decode_attention call
HQ, HKV, D, BS, NUM_BLOCKS = 14, 2, 64, 16, 16384
ELT = 2  # fp16 bytes


def workload(seed: int):
    """Context lengths and block tables of config 2 (seeded per rank)."""
    g = torch.Generator().manual_seed(seed)
    ctx = torch.randint(CTX_LO, CTX_HI + 1, (BATCH,), generator=g).tolist()
    perm = torch.randperm(NUM_BLOCKS, generator=g).tolist()
    tables, at = [], 0
    for c in ctx:
        n = (c + 1 + BS - 1) // BS  # room for the appended token
        tables.append(perm[at:at + n])
        at += n
    return ctx, tables


def prefill_workload(seed: int, n_seq: int = 256):
    """Config 4's prefill: a 1024-token cached prefix plus U{64..256} new tokens per sequence."""
    g = torch.Generator().manual_seed(seed)
    news = torch.randint(64, 257, (n_seq,), generator=g).tolist()
    return [1024] * n_seq, news


def run_prefill(dev, seed: int, layers: int = 2, reps: int = 10) -> dict:
    """Time pkv_prefill_attention (tcgen05) on config 4's prefill over the cached prefix.

    Two layer pools alternate (168 MB of K/V each, above L2). FLOPs count only the causal
    products each query makes with the keys it sees: 4 * Hq * d per (query, key) pair.
    """
    from mini_inference_b200 import ops

    starts, news = prefill_workload(seed)
    ends = [a + n for a, n in zip(starts, news)]
    nblk = [(e + BS - 1) // BS for e in ends]
    nb = sum(nblk) + 1
    g = torch.Generator().manual_seed(seed + 7)
    perm = torch.randperm(nb, generator=g)
    tab = torch.zeros(len(ends), max(nblk), dtype=torch.int32)
    at = 0
    for i, n in enumerate(nblk):
        tab[i, :n] = perm[at:at + n]
        at += n
    gd = torch.Generator(device=dev).manual_seed(seed + 11)
    k = torch.randn(layers, nb + 1, HKV, BS, D, generator=gd, device=dev, dtype=torch.float16)
    v = torch.randn(layers, nb + 1, HKV, BS, D, generator=gd, device=dev, dtype=torch.float16)
    q = torch.randn(layers, sum(news), HQ, D, generator=gd, device=dev, dtype=torch.float16)
    out = torch.empty_like(q[0])
    cu = torch.tensor([0] + torch.tensor(news).cumsum(0).tolist(), dtype=torch.int32, device=dev)
    st = torch.tensor(starts, dtype=torch.int32, device=dev)
    pool, tabs = ops.make_pool(k, v), ops.make_tables(tab.to(dev))
    status = torch.zeros(1, dtype=torch.int32, device=dev)

    def call(layer: int) -> None:
        ops.prefill_attention(pool, layer, tabs, q[layer], cu, st, max(news), out=out, status=status)

    for i in range(3):
        call(i % layers)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(reps):
        call(i % layers)
    e1.record()
    torch.cuda.synchronize()
    ops.raise_device_errors(status)
    ms = e0.elapsed_time(e1) / reps
    pairs = sum(n * a + n * (n + 1) // 2 for a, n in zip(starts, news))
    flops = 4 * HQ * D * pairs
    peaks, kind = measured_peaks()
    tflops = flops / (ms * 1e-3) / 1e12
    return {"workload": "config 4 prefill: 256 sequences x (1024 cached + U{64..256} new) tokens, fp16, "
                        "Hq 14 / Hkv 2 / d 64, one layer call (tcgen05 kernel)",
            "ms_per_call": round(ms, 4), "flops_per_call": flops, "tflops": round(tflops, 1),
            "roofline": {"bound": "tensor", "achieved": round(tflops, 1), "peak": peaks["bf16_tflops"],
                         "unit": "TFLOP/s", "frac": round(tflops / peaks["bf16_tflops"], 4),
                         "peak_kind": f"{kind} dense bf16 GEMM (burst)"}}


def run_long_context(dev, seed: int, reps: int = 10) -> dict:
    """Config 5's attention kernel alone: 7B shapes (Hq 28 / Hkv 4 / d 128, bf16), 64
    sequences with contexts U{8192..32768}, one fused append + decode attention call per
    rep over one ~2.7 GB layer pool (far above L2). Bytes as ``bytes_per_layer_call`` with
    the 7B dims.
    """
    from mini_inference_b200 import ops

    hq, hkv, d, batch = 28, 4, 128, 64
    g = torch.Generator().manual_seed(seed + 5)
    ctx = torch.randint(8192, 32769, (batch,), generator=g).tolist()
    nblk = [(c + 1 + BS - 1) // BS for c in ctx]
    nb = sum(nblk) + 8
    perm = torch.randperm(nb, generator=g)
    tab = torch.zeros(batch, max(nblk), dtype=torch.int32)
    at = 0
    for i, n in enumerate(nblk):
        tab[i, :n] = perm[at:at + n]
        at += n
    gd = torch.Generator(device=dev).manual_seed(seed + 13)
    k = torch.randn(1, nb + 1, hkv, BS, d, generator=gd, device=dev, dtype=torch.bfloat16)
    v = torch.randn(1, nb + 1, hkv, BS, d, generator=gd, device=dev, dtype=torch.bfloat16)
    q = torch.randn(batch, hq, d, generator=gd, device=dev, dtype=torch.bfloat16)
    kn = torch.randn(batch, hkv, d, generator=gd, device=dev, dtype=torch.bfloat16)
    vn = torch.randn(batch, hkv, d, generator=gd, device=dev, dtype=torch.bfloat16)
    out = torch.empty_like(q)
    tab_d = tab.to(dev)
    slot = torch.tensor([int(tab[i, c // BS]) * BS + c % BS for i, c in enumerate(ctx)], dtype=torch.int64, device=dev)
    lens = torch.tensor([c + 1 for c in ctx], dtype=torch.int32, device=dev)
    ws = torch.zeros(ops.decode_workspace_bytes(batch, hkv, max(nblk), BS, d, hq), dtype=torch.uint8, device=dev)
    pool, tabs = ops.make_pool(k, v), ops.make_tables(tab_d)
    status = torch.zeros(1, dtype=torch.int32, device=dev)

    def call() -> None:  # the append rewrites the same row every rep: the keys do not change
        ops.decode_attention(pool, 0, tabs, q, lens, ws, k_new=kn, v_new=vn, slot_mapping=slot, out=out,
                             status=status)

    for _ in range(3):
        call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        call()
    e1.record()
    torch.cuda.synchronize()
    ops.raise_device_errors(status)
    ms = e0.elapsed_time(e1) / reps
    elt = 2
    nbytes = (sum(c + 1 for c in ctx) * hkv * d * elt * 2 + batch * hq * d * elt * 2 + batch * hkv * d * elt * 2
              + sum(nblk) * 4)
    gbs = nbytes / (ms * 1e-3) / 1e9
    peaks, kind = measured_peaks()
    return {"workload": "config 5 attention kernel: 64 sequences, context U{8192..32768}, bf16, Hq 28 / Hkv 4 / "
                        "d 128, one fused append + decode attention call over a 2.7 GB layer pool",
            "ms_per_call": round(ms, 4), "bytes_per_call": nbytes, "gbs": round(gbs, 1),
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(gbs / peaks["hbm_gbs"], 4), "peak_kind": f"{kind} copy bandwidth"}}


def long_context_cpu_sample(seed: int, n_seq: int = 8, reps: int = 5) -> dict:
    """Config 5's layer call on the host cores: the reference's PyTorch ops (``oracle/paged_kv_torch.py``)
    at the 7B dims, bf16, on the first ``n_seq`` sequences of the same seeded contexts (a full
    64-sequence call at these contexts would hold ~2.7 GB of gathered K/V per layer). GB/s of
    the sample's algorithmic bytes; the full call's time at that rate is stated beside it."""
    from oracle.paged_kv_torch import decode_attend_torch

    torch.set_num_threads(os.cpu_count() or 1)
    hq, hkv, d, batch = 28, 4, 128, 64
    g = torch.Generator().manual_seed(seed + 5)
    ctx_all = torch.randint(8192, 32769, (batch,), generator=g).tolist()
    ctx = ctx_all[:n_seq]
    nblk = [(c + 1 + BS - 1) // BS for c in ctx]
    tables, at = [], 0
    for n in nblk:
        tables.append(list(range(at, at + n)))
        at += n
    gc = torch.Generator().manual_seed(seed + 17)
    k = torch.randn(at + 1, hkv, BS, d, generator=gc).bfloat16()
    v = torch.randn(at + 1, hkv, BS, d, generator=gc).bfloat16()
    q = torch.randn(n_seq, hq, d, generator=gc).bfloat16()
    kn = torch.randn(n_seq, hkv, d, generator=gc).bfloat16()
    decode_attend_torch(k, v, tables, ctx, q, kn, kn)  # warm-up
    t0 = time.perf_counter()
    for _ in range(reps):
        decode_attend_torch(k, v, tables, ctx, q, kn, kn)
    dt = (time.perf_counter() - t0) / reps
    elt = 2

    def nbytes(cs: list[int]) -> int:
        return (sum(c + 1 for c in cs) * hkv * d * elt * 2 + len(cs) * (hq + hkv) * d * elt * 2
                + sum((c + 1 + BS - 1) // BS for c in cs) * 4)

    gbs = nbytes(ctx) / dt / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": cpu_threads(), "kind": "port",
            "sample": f"one config-5 layer call over the first {n_seq} of the 64 sequences ({sum(ctx)} cached "
                      f"tokens, bf16, Hq 28 / Hkv 4 / d 128), reference PyTorch ops on the host "
                      f"(oracle/paged_kv_torch.py), {reps} calls; {dt:.3f} s per call, so ~"
                      f"{nbytes(ctx_all) / (gbs * 1e9):.1f} s for the full 64-sequence call at this rate",
            "seconds": round(dt * reps, 2)}


def run_long_step(dev, seed: int, steps: int = 32, warmup: int = 3) -> dict:
    """Config 5's decode step through the whole Qwen2.5-7B-shaped model (bf16, random N(0, 0.02)
    weights drawn on the GPU): 64 sequences with contexts U{8192..32768}, every layer's
    qkv_proj / o_proj / MLP GEMMs and RMSNorms on torch, RoPE + append + paged attention in
    one kernel per layer, the LM head fused with greedy argmax, replayed as one CUDA graph.

    The task builds the contexts by a seeded prefill of uniform token ids (~10^16 FLOP); here
    the pool's K/V are seeded N(0, 1) values written directly, which costs the decode step
    the same bytes. Bytes per step = every weight once (the embedding table only for the
    step's rows) + every context token's K and V in every layer.
    """
    from mini_inference_b200 import PagedKVCache
    from mini_inference_b200.engine import ModelRunner
    from mini_inference_b200.model import Qwen2Config, Qwen2Model, init_random

    cfg = Qwen2Config.qwen2_7b()
    model = Qwen2Model(cfg, init_random(cfg, seed=0, std=0.02, dtype=torch.bfloat16, device=dev,
                                        generator_device="cuda"))
    batch = 64
    g = torch.Generator().manual_seed(seed + 5)
    ctx = torch.randint(8192, 32769, (batch,), generator=g).tolist()
    extra = steps + warmup + 4  # room for the generated tokens
    max_len = max(ctx) + extra + 16
    nblk = sum((c + extra + BS - 1) // BS for c in ctx)
    cache = PagedKVCache(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, num_blocks=nblk + 8, block_size=BS,
                         max_seqs=batch, max_len=max_len, dtype=torch.bfloat16, device=dev)
    gd = torch.Generator(device=dev).manual_seed(seed + 17)
    for layer in range(cfg.num_layers):  # the "prefilled" contexts, layer by layer
        cache.k[layer].normal_(generator=gd)
        cache.v[layer].normal_(generator=gd)
    slots = [cache.allocate(c + extra) for c in ctx]
    for s_, c in zip(slots, ctx):
        cache.lengths[s_] = c
    runner = ModelRunner(model, cache, max_batch=batch)
    runner.enable_cuda_graphs(batch)
    tokens = torch.randint(0, cfg.vocab_size, (batch,), generator=g).tolist()
    for _ in range(warmup):
        tokens = runner.decode_tokens(slots, tokens)
    torch.cuda.synchronize()
    start_ctx = sum(cache.lengths[s_] for s_ in slots)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record()
    for _ in range(steps):
        tokens = runner.decode_tokens(slots, tokens)
    e1.record()
    torch.cuda.synchronize()
    host_s = time.perf_counter() - t0
    cache.raise_device_errors()
    ms = e0.elapsed_time(e1) / steps
    kv_per_token = cfg.num_layers * 2 * cfg.num_kv_heads * cfg.head_dim * 2
    ctx_tokens = sum(start_ctx + batch * (i + 1) for i in range(steps)) / steps  # keys attended per step
    embed_bytes = cfg.vocab_size * cfg.hidden_size * 2
    weight_bytes = model.weight_bytes() - embed_bytes + batch * cfg.hidden_size * 2
    step_bytes = weight_bytes + ctx_tokens * kv_per_token
    gbs = step_bytes / (ms * 1e-3) / 1e9
    peaks, kind = measured_peaks()
    pool_gb = (cache.k.numel() + cache.v.numel()) * 2 / 1e9
    del runner, cache, model
    torch.cuda.empty_cache()
    return {"workload": "config 5 decode step: Qwen2.5-7B shape (28 layers, hidden 3584, 28 / 4 heads of 128, MLP "
                        "18944, vocab 152064), bf16 random-init weights, 64 sequences with contexts U{8192..32768} "
                        "(K/V seeded directly in the pool), greedy",
            "steps": steps, "ms_per_step": round(ms, 3), "tok_s": round(batch / (ms * 1e-3), 1),
            "host_ms_per_step": round(host_s / steps * 1e3, 3),
            "bytes_per_step": int(step_bytes), "weight_bytes": int(weight_bytes),
            "kv_bytes_per_step": int(ctx_tokens * kv_per_token),
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(gbs / peaks["hbm_gbs"], 4), "peak_kind": f"{kind} copy bandwidth"},
            "pool_gb": round(pool_gb, 1)}


def run_qkv_post(dev, seed: int, reps: int = 50) -> dict:
    """``pkv_rope_append`` at 0.5B shapes (Hq 14 / Hkv 2 / d 64, fp16), beside the reference's
    eager path for the same work on the same GPU: the split and head views, ``apply_rope``
    (engine/model.py:214-224) as torch ops, and the index_put append (engine/kv_cache.py:288-289).

    Prefill: a 4096-token pack (``max_num_batched_tokens``) with the append into the pool.
    Decode: 64 tokens, rotated keys handed to the fused decode append (nothing written to the pool).
    """
    from mini_inference_b200 import ops

    hq, hkv, d, dtype = HQ, HKV, D, torch.float16
    width = (hq + 2 * hkv) * d
    cos, sin = ops.rope_tables(d, 32768, 1e6, dtype, dev)
    g = torch.Generator(device=dev).manual_seed(seed + 17)
    peaks, kind = measured_peaks()
    status = torch.zeros(1, dtype=torch.int32, device=dev)

    def timed(fn) -> float:
        """Device time per call: 10 calls recorded as one CUDA graph (the host's ~10 us per
        Python-issued call would otherwise be what is measured), replayed ``reps`` times."""
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                fn()
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(10):
                fn()
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        del graph
        return e0.elapsed_time(e1) / (reps * 10) * 1e3  # us

    def eager_rope(x, c, s):
        x1, x2 = x.chunk(2, dim=-1)
        return x * c + torch.cat([-x2, x1], dim=-1) * s

    result = {}
    for name, n, append in (("prefill_4096", 4096, True), ("decode_64", BATCH, False)):
        qkv = torch.randn(n, width, generator=g, device=dev).to(dtype)
        positions = torch.randint(0, 2048, (n,), generator=g, device=dev)
        nb = n // BS + 2
        k = torch.zeros(1, nb + 1, hkv, BS, d, dtype=dtype, device=dev)
        v = torch.zeros_like(k)
        pool = ops.make_pool(k, v)
        slots = torch.randperm(nb * BS, device=dev)[:n] if append else None
        q_out = torch.empty(n, hq, d, dtype=dtype, device=dev)
        k_out = None if append else torch.empty(n, hkv, d, dtype=dtype, device=dev)

        def ours():
            ops.rope_append(pool, 0, qkv, positions, cos, sin, hq, q_out=q_out, k_out=k_out if k_out is not None else False,
                            slot_mapping=slots, status=status)

        def eager():  # the reference's ops on the same tensors (engine/model.py:201-250, engine/kv_cache.py:288-289)
            q, kk, vv = qkv.view(1, n, hq + 2 * hkv, d).transpose(1, 2).split([hq, hkv, hkv], dim=1)
            c, s = cos[positions][None, None], sin[positions][None, None]
            q_rot, k_rot = eager_rope(q, c, s), eager_rope(kk, c, s)
            if append:
                blocks, offs = slots // BS, slots % BS
                k[0][blocks, :, offs] = k_rot[0].transpose(0, 1)
                v[0][blocks, :, offs] = vv[0].transpose(0, 1)
            return q_rot

        us, us_eager = timed(ours), timed(eager)
        ops.raise_device_errors(status)
        nbytes = n * (width * 2 + hq * d * 2 + (2 if append else 1) * hkv * d * 2 + 2 * d * 2)
        gbs = nbytes / (us * 1e-6) / 1e9
        result[name] = {"tokens": n, "us_per_call": round(us, 2), "bytes_per_call": nbytes, "gbs": round(gbs, 1),
                        "frac_of_hbm": round(gbs / peaks["hbm_gbs"], 4), "reference_eager_torch_us": round(us_eager, 2)}
    result["workload"] = ("pkv_rope_append (RoPE fused with the KV append), 0.5B shapes fp16; the reference's eager "
                          "torch ops for the same work timed beside it on the same GPU; both as CUDA-graph replays "
                          "of 10 calls (device time)")
    result["peak_kind"] = f"{kind} copy bandwidth"
    return result


def run_lm_head(dev, seed: int, reps: int = 20) -> dict:
    """``pkv_lm_head_argmax`` (the LM head fused with greedy selection) at Qwen2.5-0.5B's tied
    151936 x 896 fp16 embedding, beside the reference's path for the same tokens on the same GPU:
    ``compute_logits(hidden).float()`` then ``argmax`` (engine/model.py:321-323, engine/sampler.py:27-31).

    Two weight copies alternate (544 MB, above L2), so every call streams its weight from HBM.
    Batches: 64 (config 2's decode batch) and 256 (``max_num_seqs``).
    """
    from mini_inference_b200 import ops

    vocab, hidden, dtype = 151936, 896, torch.float16
    g = torch.Generator(device=dev).manual_seed(seed + 29)
    weights = [(torch.randn(vocab, hidden, generator=g, device=dev) * 0.02).to(dtype) for _ in range(2)]
    peaks, kind = measured_peaks()
    status = torch.zeros(1, dtype=torch.int32, device=dev)

    def timed(fns) -> float:
        """Device time per call: the calls recorded as one CUDA graph, replayed ``reps`` times."""
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                for fn in fns:
                    fn()
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(5):
                for fn in fns:
                    fn()
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        del graph
        return e0.elapsed_time(e1) / (reps * 5 * len(fns)) * 1e3  # us

    result = {}
    for batch in (BATCH, 256):
        h = torch.randn(batch, hidden, generator=g, device=dev).to(dtype)
        ws = ops.lm_head_argmax_workspace(batch, dev)
        out = torch.empty(batch, dtype=torch.int64, device=dev)
        ref_out = torch.empty(batch, dtype=torch.int64, device=dev)
        ours = [lambda w=w: ops.lm_head_argmax(h, w, ws, out=out, status=status, weight_ready=True) for w in weights]
        ref = [lambda w=w: ref_out.copy_(torch.nn.functional.linear(h, w).float().argmax(dim=-1)) for w in weights]
        us, us_ref = timed(ours), timed(ref)
        ops.raise_device_errors(status)
        same = int((out == ref_out).sum())
        nbytes = vocab * hidden * 2 + batch * hidden * 2 + batch * 8
        gbs = nbytes / (us * 1e-6) / 1e9
        result[f"batch_{batch}"] = {
            "us_per_call": round(us, 2), "bytes_per_call": nbytes, "gbs": round(gbs, 1),
            "frac_of_hbm": round(gbs / peaks["hbm_gbs"], 4), "reference_torch_us": round(us_ref, 2),
            "same_tokens_as_reference": f"{same}/{batch}"}
    result["workload"] = ("pkv_lm_head_argmax at Qwen2.5-0.5B's tied 151936 x 896 fp16 embedding (tcgen05, "
                          "weight streamed once, no logits written); the reference's compute_logits + float + "
                          "argmax by torch (cuBLAS) timed beside it on the same GPU; CUDA-graph replays, two "
                          "alternating weight copies above L2 (device time)")
    result["kernel"] = "pkv lm_head_argmax_kernel<half,1> (batch 64), <half,2> (batch 256)"
    result["peak_kind"] = f"{kind} copy bandwidth"
    return result


def run_scheduler(seed: int, steps: int = 400) -> dict:
    """Host time of one scheduler step at config 3's request mix: 200 requests at t=0, prompts
    round(exp(U(ln 16, ln 1024))) tokens, outputs U{16..512} (ignore_eos), max_num_seqs 256,
    max_num_batched_tokens 4096, max_model_len 2048, blocks of 16 and a pool for every request.

    A step is ``schedule()`` plus the step's ``append_token`` calls (the scheduler's share of
    ``LLMEngine.step``, engine/engine.py:281-312), with the engine's cache commits in between.
    The native scheduler (C++ over the C++ block manager, one call each) is timed beside the
    reference's algorithm in Python over its allocator (``oracle/scheduler.py`` and
    ``oracle/block_manager.py``, the reference's own code path restated: the reference does not
    travel to the GPU box) on the same requests and tokens.
    """
    import random
    from types import SimpleNamespace

    from mini_inference_b200 import PagedKVCache
    from mini_inference_b200.scheduler import Scheduler, SequenceStatus
    from oracle.block_manager import OracleBlockManager
    from oracle.scheduler import OracleSampling, OracleScheduler, OracleSequence

    rng = random.Random(seed + 3)
    reqs = [([rng.randrange(2, 151936) for _ in range(round(math.exp(rng.uniform(math.log(16), math.log(1024)))))],
             rng.randint(16, 512)) for _ in range(200)]
    max_seqs, budget, max_len, bs = 256, 4096, 2048, 16
    blocks = sum(-(-(len(p) + m) // bs) for p, m in reqs)

    class Seq:
        __slots__ = ("seq_id", "prompt_token_ids", "sampling", "output_token_ids", "status", "slot", "finish_reason",
                     "first_token_time", "finish_time", "num_preemptions", "num_cached_tokens")

        def __init__(self, i, prompt, max_tokens):
            self.seq_id, self.prompt_token_ids = i, prompt
            self.sampling = OracleSampling(max_tokens, True)
            self.output_token_ids, self.status, self.slot, self.finish_reason = [], SequenceStatus.WAITING, None, None
            self.first_token_time = self.finish_time = None
            self.num_preemptions = self.num_cached_tokens = 0

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
            return self.status is SequenceStatus.FINISHED

    def run(native: bool) -> tuple[float, float]:
        if native:
            cache = PagedKVCache(1, 1, 4, blocks, bs, max_seqs, max_len, torch.float16, "cpu", True)
            sched = Scheduler(SimpleNamespace(max_num_seqs=max_seqs, max_num_batched_tokens=budget,
                                              max_model_len=max_len, scheduling="continuous"), cache)
            seqs = [Seq(i, list(p), m) for i, (p, m) in enumerate(reqs)]
        else:
            cache = OracleBlockManager(blocks, bs, max_seqs, max_len, True)
            sched = OracleScheduler(max_seqs, budget, max_len, cache)
            seqs = [OracleSequence(i, list(p), OracleSampling(m, True)) for i, (p, m) in enumerate(reqs)]
        for s in seqs:
            sched.add(s)
        total, n, running = 0.0, 0, 0
        for _ in range(steps):
            t0 = time.perf_counter()
            out = sched.schedule()
            t1 = time.perf_counter()
            for s in out.prefills:
                cache.lengths[s.slot] = s.num_tokens
            for s in out.decodes:
                cache.lengths[s.slot] += 1
            step = list(out.prefills) + list(out.decodes)
            toks = [(s.seq_id * 7919 + s.num_tokens) % 151936 for s in step]
            t2 = time.perf_counter()
            if native:
                sched.append_tokens(step, toks, t2)
            else:
                for s, tok in zip(step, toks):
                    sched.append_token(s, tok, t2)
            t3 = time.perf_counter()
            total += (t1 - t0) + (t3 - t2)
            n += 1
            running += len(out.decodes)
        return total / n * 1e6, running / n

    native_us, running = run(True)
    ref_us, _ = run(False)
    return {"us_per_step": round(native_us, 1), "reference_us_per_step": round(ref_us, 1),
            "mean_decodes_per_step": round(running, 1), "steps": steps,
            "workload": "config 3's 200 requests at t=0 (prompts round(exp(U(ln16, ln1024))), outputs U{16..512}), "
                        "max_num_seqs 256, budget 4096, blocks of 16; schedule() + the step's append_token calls, "
                        "host time; reference = the reference's scheduler and allocator algorithm in Python "
                        "(oracle/scheduler.py, oracle/block_manager.py)"}


def bytes_per_layer_call(ctx: list[int]) -> int:
    """Algorithmic bytes of one fused append + decode attention call over the batch.

    K+V read for ctx+1 keys per sequence and KV head, Q read and O write, the
    appended K/V rows written, and the int32 block-table entries read.
    """
    kv = sum(c + 1 for c in ctx) * HKV * D * ELT * 2
    qo = len(ctx) * HQ * D * ELT * 2
    append = len(ctx) * HKV * D * ELT * 2
    table = sum(math.ceil((c + 1) / BS) for c in ctx) * 4
    return kv + qo + append + table


def decode_config(world: int, layers: int) -> dict:
    """The ``config`` of the config-2 line, the same in both arms."""
    ctx, _ = workload(seed=0)
    return {"workload": "config 2: paged decode attention micro-benchmark, fused one-token append",
            "batch_per_gpu": BATCH, "context": f"U{{{CTX_LO}..{CTX_HI}}}", "q_heads": HQ, "kv_heads": HKV,
            "head_dim": D, "block_size": BS, "pool_blocks": NUM_BLOCKS, "layers_per_step": layers,
            "bytes_per_step_per_gpu": bytes_per_layer_call(ctx) * layers, "tokens_per_step_per_gpu": BATCH,
            "l2": f"inputs above L2: {layers} layer pools of 134 MB, each read once per step",
            "parallelism": f"replicas x{world} (requests sharded by rank, no collective)"}


def measured_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def ncu_traffic_per_launch() -> float | None:
    """DRAM bytes per decode launch from the committed ncu summary, if one exists."""
    f = ROOT / "profiles" / "decode_attention_config2.md"
    if not f.exists():
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", f.read_text())
    return float(m.group(1)) if m else None


class ClockSampler:
    """nvidia-smi samples (every 100 ms) of SM clock and throttle reasons while the GPU works."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int) -> None:
        self.index = index
        self.proc = None
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.file, stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict | None:
        if self.proc is None:
            return None
        self.file.flush()
        rows = [r.split(", ") for r in Path(self.file.name).read_text().splitlines() if r.strip()]
        rows = [r for r in rows if len(r) >= 9]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows)}


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        # The replicas share nothing on the data path; the process group only carries the
        # barriers around the timed regions and the max of the ranks' times, on the host (gloo).
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    return rank, world, local


def max_over_ranks(value: float, world: int) -> float:
    """Job time = the slowest rank's device time (a host-side reduction, outside any timed region)."""
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


# ---------------------------------------------------------------------------------------- our arm


def run_ours(args, rank: int, world: int, local: int) -> dict | None:
    from mini_inference_b200 import ops

    LAYERS = args.layers
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    ctx, tables = workload(seed=rank)
    call_bytes = bytes_per_layer_call(ctx)
    step_bytes = call_bytes * LAYERS
    cols = max(len(t) for t in tables)

    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    shape = (LAYERS, NUM_BLOCKS + 1, HKV, BS, D)
    k_pool = torch.randn(shape, generator=g, device=dev, dtype=torch.float16)
    v_pool = torch.randn(shape, generator=g, device=dev, dtype=torch.float16)
    q = torch.randn(LAYERS, BATCH, HQ, D, generator=g, device=dev, dtype=torch.float16)
    kn = torch.randn(LAYERS, BATCH, HKV, D, generator=g, device=dev, dtype=torch.float16)
    vn = torch.randn(LAYERS, BATCH, HKV, D, generator=g, device=dev, dtype=torch.float16)
    out = torch.empty(LAYERS, BATCH, HQ, D, device=dev, dtype=torch.float16)

    # Device table mirror (one row per sequence) + the per-step inputs the builder reads.
    mirror = torch.full((BATCH, cols), -1, dtype=torch.int32)
    for i, t in enumerate(tables):
        mirror[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
    mirror = mirror.to(dev)
    rows = torch.arange(BATCH, dtype=torch.int32, device=dev)
    lengths = torch.tensor(ctx, dtype=torch.int32, device=dev)
    positions = torch.empty(BATCH, dtype=torch.int64, device=dev)
    slot_mapping = torch.empty(BATCH, dtype=torch.int64, device=dev)
    context_lens = torch.empty(BATCH, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    pool = ops.make_pool(k_pool, v_pool)
    tabs = ops.make_tables(mirror, rows)
    ws = torch.zeros(ops.decode_workspace_bytes(BATCH, HKV, cols, BS, D, HQ), dtype=torch.uint8, device=dev)

    def attention_layers(after_builder: bool):
        # Tables and lengths come from the builder at the start of the step, so every layer
        # after the first may start its block lookups before the previous kernel ends.
        for layer in range(LAYERS):
            ops.decode_attention(pool, layer, tabs, q[layer], context_lens, ws, k_new=kn[layer], v_new=vn[layer],
                                 slot_mapping=slot_mapping, out=out[layer], status=status,
                                 inputs_ready=layer > 0 or not after_builder)

    def step():
        ops.build_decode_metadata(tabs, lengths, BS, NUM_BLOCKS, positions, slot_mapping, context_lens, status)
        attention_layers(after_builder=True)

    # Warm-up eagerly (also validates), then capture one step and the attention-only part.
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            step()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    ops.raise_device_errors(status)
    g_step, g_attn = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_step):
        step()
    with torch.cuda.graph(g_attn):
        attention_layers(after_builder=False)
    stream = torch.cuda.current_stream()

    def timed(graph, k: int) -> float:
        for _ in range(args.warmup):
            graph.replay()
        torch.cuda.synchronize()
        barrier(world)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(k):
            graph.replay()
        end.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        return start.elapsed_time(end)

    # The decode step as the model runs it, from each layer's qkv_proj rows: RoPE in its own
    # kernel then the fused append + attention (two launches a layer), or rotated inside the
    # decode kernel (one launch a layer, pkv_decode_attention_rope).
    qkv = torch.randn(LAYERS, BATCH, (HQ + 2 * HKV) * D, generator=g, device=dev, dtype=torch.float16)
    cos, sin = ops.rope_tables(D, CTX_HI + 16, 1e6, torch.float16, dev)
    q_rot = torch.empty(BATCH, HQ, D, device=dev, dtype=torch.float16)
    k_rot = torch.empty(BATCH, HKV, D, device=dev, dtype=torch.float16)

    def rope_split_step():
        ops.build_decode_metadata(tabs, lengths, BS, NUM_BLOCKS, positions, slot_mapping, context_lens, status)
        for layer in range(LAYERS):
            ops.rope_append(pool, layer, qkv[layer], positions, cos, sin, HQ, q_out=q_rot, k_out=k_rot, status=status)
            ops.decode_attention(pool, layer, tabs, q_rot, context_lens, ws, k_new=k_rot,
                                 v_new=qkv[layer][:, (HQ + HKV) * D:].view(BATCH, HKV, D), slot_mapping=slot_mapping,
                                 out=out[layer], status=status, inputs_ready=True)

    def rope_fused_step():
        ops.build_decode_metadata(tabs, lengths, BS, NUM_BLOCKS, positions, slot_mapping, context_lens, status)
        for layer in range(LAYERS):
            ops.decode_attention_rope(pool, layer, tabs, qkv[layer], cos, sin, context_lens, ws, slot_mapping,
                                      out=out[layer], status=status, inputs_ready=layer > 0)

    g_rope = {}
    for name, fn in (("split", rope_split_step), ("fused", rope_fused_step)):
        with torch.cuda.stream(side):
            fn()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        g_rope[name] = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_rope[name]):
            fn()

    with ClockSampler(local) as clocks:
        ms_total = timed(g_step, args.steps)
        ms_attn = timed(g_attn, args.steps)
        rope_steps = max(1, args.steps // 2)
        ms_rope = {name: timed(gr, rope_steps) for name, gr in g_rope.items()}
        if args.profile_case:
            ms_e2e, h2d, d2h, e2e_launches = ms_total, 0, 0, 0
        else:
            ms_e2e, h2d, d2h, e2e_launches = run_e2e(args, dev, pool, tables, ctx, q, kn, vn, world)
    ops.raise_device_errors(status)

    ms_job = max_over_ranks(ms_total, world)
    ms_attn_job = max_over_ranks(ms_attn, world)
    ms_e2e_job = max_over_ranks(ms_e2e, world)
    ms_rope_job = {name: max_over_ranks(v, world) for name, v in ms_rope.items()}
    del g_step, g_attn, g_rope, k_pool, v_pool
    serving = None
    prefix_serving = None
    if not args.profile_case and not args.no_serving and not args.decode_only:  # every rank: configs 3 and 4
        with ClockSampler(local) as serve_clocks:
            serving, model = run_serving(args, rank, world, local)
            prefix_serving = run_prefix_serving(args, rank, world, local, model)
        if serving is not None:
            serving["clocks"] = serve_clocks.summary()
    if rank != 0:
        return None
    peaks, peak_kind = measured_peaks()
    per_launch_ms = ms_attn_job / (args.steps * LAYERS)
    achieved = call_bytes / (per_launch_ms * 1e-3) / 1e9
    traffic = ncu_traffic_per_launch()
    line = {
        "metric": METRIC, "value": round(world * step_bytes * args.steps / (ms_job * 1e-3) / 1e9, 2), "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_job / args.steps, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16", "data": "synthetic (seeded; config 2 shapes and distributions)",
        "config": decode_config(world, LAYERS),
        "decode_steps_per_s": round(world * args.steps / (ms_job * 1e-3), 1),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "peak_kind": f"{peak_kind} copy bandwidth",
                     "traffic": traffic, "algorithmic_bytes_per_launch": call_bytes,
                     "traffic_source": "dram__bytes_read.sum + dram__bytes_write.sum of one ncu capture of this "
                                       "kernel (profiles/decode_attention_config2.md)",
                     "kernel": "pkv decode_kernel<half,64,2,8,256,false> (fused append + paged attention, split items merged)",
                     "launch_us": round(per_launch_ms * 1e3, 3)},
        "e2e": {"value": round(world * step_bytes * args.e2e_steps / (ms_e2e_job * 1e-3) / 1e9, 2), "unit": UNIT,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": round(ms_e2e_job / args.e2e_steps, 4), "steps": args.e2e_steps,
                "path": "C ABI (pkv_decode_attention via ctypes) on pinned host buffers, the step recorded as "
                        "one CUDA graph (as engine/cuda_graphs.py runs decode) with chunked copies overlapping "
                        "the kernels"},
        "decode_with_rope": {
            "workload": "the config-2 step from each layer's qkv_proj rows: metadata, then per layer RoPE + "
                        "append + attention",
            "ms_per_step_rope_then_decode": round(ms_rope_job["split"] / rope_steps, 5),
            "ms_per_step_fused": round(ms_rope_job["fused"] / rope_steps, 5),
            "launches_per_layer": {"rope_then_decode": 2, "fused": 1},
            "kv_gbs_fused": round(world * step_bytes * rope_steps / (ms_rope_job["fused"] * 1e-3) / 1e9, 2),
            "kernel": "pkv_decode_attention_rope (q and the new k rotated in the decode kernel)"},
        "gpu_launches": (args.steps * (1 + LAYERS * DECODE_KERNELS) + args.steps * LAYERS * DECODE_KERNELS + e2e_launches
                         + rope_steps * (1 + 2 * LAYERS) + rope_steps * (1 + LAYERS)),
        "clocks": clocks.summary(),
    }
    if args.profile_case:  # no end-to-end leg in the capture case
        line["e2e"] = None
    elif args.decode_only:
        pass
    else:
        line["prefill"] = run_prefill(dev, seed=rank)
        line["long_context"] = run_long_context(dev, seed=rank)
        if world == 1:
            line["long_context"]["cpu_baseline"] = long_context_cpu_sample(seed=rank)
        if not args.no_long_step:
            line["long_context_step"] = run_long_step(dev, seed=rank)
        line["qkv_post"] = run_qkv_post(dev, seed=rank)
        line["lm_head"] = run_lm_head(dev, seed=rank)
        line["scheduler"] = run_scheduler(seed=rank)
        line["serving"] = serving
        line["prefix_serving"] = prefix_serving
    if world == 1 and not args.profile_case and not args.decode_only:
        line["cpu_baseline"] = cpu_baseline(args)
    return line


def run_e2e(args, dev, pool, tables, ctx, q_dev, kn_dev, vn_dev, world):
    """The same step through the C ABI with host buffers: H2D inputs, 24 calls, D2H outputs.

    As the reference engine runs its decode steps (engine/cuda_graphs.py), the step is a
    CUDA graph, recorded once and replayed per step: the table, slot and length copies,
    then the layers' q / k_new / v_new in chunks of 1, 2, 4, 8, ... layers on a copy
    stream (each layer's call waits only for its chunk, so later chunks land while earlier
    layers compute; the step's inputs sit in one staging buffer, so a chunk is one copy), the
    24 ``pkv_decode_attention`` calls, and the outputs back in chunks that shrink towards the
    last layer on a second copy stream, so only one layer's output is copied after the last
    kernel. Every step copies all its inputs in and all its outputs out inside the timed
    region and ends with the host waiting for its result. (Measured on B200: 0.38 ms per step
    with one copy per chunk and tensor, 0.49 ms with one copy per layer and tensor, 1.6 ms
    issuing the same calls eagerly from Python.)
    """
    from mini_inference_b200 import ops

    LAYERS = args.layers
    cols = max(len(t) for t in tables)
    # One pinned staging buffer per step, as an engine keeps one: the metadata (tables,
    # slots, lengths) and then each layer's q | k_new | v_new back to back, so that a chunk of
    # layers is one contiguous copy (a host-device copy costs ~8-10 us on its own here,
    # measured, whatever its size up to ~150 KB), mirrored by one device buffer.
    def up(n: int) -> int:
        return (n + 255) // 256 * 256

    tab_b, sm_b, cl_b = BATCH * cols * 4, BATCH * 8, BATCH * 4
    q_b, kv_b = BATCH * HQ * D * ELT, BATCH * HKV * D * ELT
    meta = up(tab_b) + up(sm_b) + up(cl_b)
    layer_b = up(q_b + 2 * kv_b)
    buf_h = torch.zeros(meta + LAYERS * layer_b, dtype=torch.uint8).pin_memory()
    buf_d = torch.zeros_like(buf_h, device=dev)

    def views(buf):
        tab = buf[:tab_b].view(torch.int32).view(BATCH, cols)
        sm = buf[up(tab_b):up(tab_b) + sm_b].view(torch.int64)
        cl = buf[up(tab_b) + up(sm_b):up(tab_b) + up(sm_b) + cl_b].view(torch.int32)
        per = []
        for layer in range(LAYERS):
            o = meta + layer * layer_b
            per.append((buf[o:o + q_b].view(torch.float16).view(BATCH, HQ, D),
                        buf[o + q_b:o + q_b + kv_b].view(torch.float16).view(BATCH, HKV, D),
                        buf[o + q_b + kv_b:o + q_b + 2 * kv_b].view(torch.float16).view(BATCH, HKV, D)))
        return tab, sm, cl, per

    tab_h, sm_h, cl_h, per_h = views(buf_h)
    for i, t in enumerate(tables):
        tab_h[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
    sm_h.copy_(torch.tensor([t[c // BS] * BS + c % BS for t, c in zip(tables, ctx)], dtype=torch.int64))
    cl_h.copy_(torch.tensor([c + 1 for c in ctx], dtype=torch.int32))
    for layer, (qh, kh, vh) in enumerate(per_h):
        qh.copy_(q_dev[layer].cpu())
        kh.copy_(kn_dev[layer].cpu())
        vh.copy_(vn_dev[layer].cpu())
    tab_d, sm_d, cl_d, per_d = views(buf_d)
    out_h = torch.empty(LAYERS, BATCH, HQ, D, dtype=torch.float16).pin_memory()
    out_d = torch.empty(LAYERS, BATCH, HQ, D, dtype=torch.float16, device=dev)
    ws = torch.zeros(ops.decode_workspace_bytes(BATCH, HKV, cols, BS, D, HQ), dtype=torch.uint8, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    tabs = ops.make_tables(tab_d)
    h2d = buf_h.numel()
    d2h = out_h.numel() * out_h.element_size()
    h2d_stream, d2h_stream = torch.cuda.Stream(), torch.cuda.Stream()

    h2d_chunks = []  # [first layer, end layer): 1, 2, 4, 8, ... layers
    first, width = 0, 1
    while first < LAYERS:
        h2d_chunks.append((first, min(LAYERS, first + width)))
        first, width = first + width, 2 * width
    d2h_chunks = [(LAYERS - b, LAYERS - a) for (a, b) in reversed(h2d_chunks)]  # the last one is one layer
    d2h_after = {b - 1: (a, b) for (a, b) in d2h_chunks}

    def record_step():
        main = torch.cuda.current_stream()
        h2d_stream.wait_stream(main)
        d2h_stream.wait_stream(main)
        landed = {}
        with torch.cuda.stream(h2d_stream):
            for a, b in h2d_chunks:  # one copy per chunk; the first one carries the metadata too
                lo, hi = (0 if a == 0 else meta + a * layer_b), meta + b * layer_b
                buf_d[lo:hi].copy_(buf_h[lo:hi], non_blocking=True)
                landed[a] = torch.cuda.Event()
                landed[a].record(h2d_stream)
        for layer in range(LAYERS):  # after the first layer the copied tables and lengths are complete
            if layer in landed:
                main.wait_event(landed[layer])
            q_l, kn_l, vn_l = per_d[layer]
            ops.decode_attention(pool, layer, tabs, q_l, cl_d, ws, k_new=kn_l, v_new=vn_l,
                                 slot_mapping=sm_d, out=out_d[layer], status=status, inputs_ready=layer > 0)
            if layer in d2h_after:
                a, b = d2h_after[layer]
                finished = torch.cuda.Event()
                finished.record(main)
                d2h_stream.wait_event(finished)
                with torch.cuda.stream(d2h_stream):
                    out_h[a:b].copy_(out_d[a:b], non_blocking=True)
        main.wait_stream(h2d_stream)
        main.wait_stream(d2h_stream)

    for _ in range(max(3, args.warmup)):  # eager warm-up (kernel attributes, tensor maps)
        record_step()
        torch.cuda.current_stream().synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        record_step()

    def step():
        graph.replay()
        torch.cuda.current_stream().synchronize()  # the caller has its result on the host

    for _ in range(max(3, args.warmup)):
        step()
    barrier(world)
    stream = torch.cuda.current_stream()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.e2e_steps):
        step()
    end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ops.raise_device_errors(status)
    if not torch.equal(out_h[LAYERS - 1], out_d[LAYERS - 1].cpu()):
        raise RuntimeError("e2e: the host copy of the last layer's output differs from the device's")
    del graph
    return start.elapsed_time(end), h2d, d2h, args.e2e_steps * LAYERS * DECODE_KERNELS


# ---------------------------------------------------------------------------------------- serving (config 3)

SERVE_REQUESTS, SERVE_MAX_SEQS, SERVE_MAX_LEN, SERVE_BUDGET = 200, 256, 2048, 4096
SERVE_KV_TOKENS = SERVE_MAX_SEQS * SERVE_MAX_LEN  # 32768 blocks of 16: no sequence is ever preempted


def serving_workload(seed: int = 0, vocab: int = 151936) -> list[tuple[list[int], int]]:
    """Config 3's requests: prompt length round(exp(U(ln 16, ln 1024))), ids U{0..vocab-1}, outputs U{16..512}."""
    g = torch.Generator().manual_seed(seed)
    u = torch.rand(SERVE_REQUESTS, generator=g, dtype=torch.float64)
    lens = torch.round(torch.exp(math.log(16) + u * (math.log(1024) - math.log(16)))).long().tolist()
    outs = torch.randint(16, 513, (SERVE_REQUESTS,), generator=g).tolist()
    return [(torch.randint(0, vocab, (n,), generator=g).tolist(), m) for n, m in zip(lens, outs)]


def serving_config() -> dict:
    return {"workload": "config 3: end-to-end serving, Qwen2.5-0.5B shape, fp16 random-init weights "
                        "(N(0, 0.02), seed 0), 200 requests arriving at t=0, prompts log-uniform 16..1024 "
                        "uniform token ids, outputs U{16..512} with EOS ignored, greedy",
            "max_num_seqs": SERVE_MAX_SEQS, "max_model_len": SERVE_MAX_LEN,
            "max_num_batched_tokens": SERVE_BUDGET, "kv_cache_tokens": SERVE_KV_TOKENS, "block_size": BS,
            "sharding": "request i on rank i mod N (one engine replica and paged pool per GPU)"}


def run_serving(args, rank: int, world: int, local: int) -> dict | None:
    """Config 3 through ``LLMEngine`` on every rank; rank 0 returns the aggregate.

    Each run adds this rank's share of the 200 requests at one common start (after a
    barrier) and steps the engine until all finish. The run's time on a rank is device
    time (CUDA events from the start to the last step's end; every step already waits
    for its tokens); the job's time is the slowest rank's. TTFT and TPOT are the
    reference's host-clock definitions (benchmarks/run_bench.py:201-221) over all 200
    requests, gathered from the ranks.
    """
    from mini_inference_b200.engine import EngineConfig, LLMEngine, SamplingParams
    from mini_inference_b200.model import Qwen2Config, Qwen2Model, init_random

    dev = torch.device("cuda", local)
    cfg = Qwen2Config.qwen2_0_5b()
    model = Qwen2Model(cfg, init_random(cfg, seed=0, std=0.02, dtype=torch.float16, device=dev,
                                        generator_device="cuda"))
    requests = serving_workload(seed=0, vocab=cfg.vocab_size)
    mine = [r for i, r in enumerate(requests) if i % world == rank]
    t0 = time.perf_counter()
    engine = LLMEngine(model, EngineConfig(max_num_seqs=SERVE_MAX_SEQS, max_model_len=SERVE_MAX_LEN,
                                           max_num_batched_tokens=SERVE_BUDGET, kv_cache_tokens=SERVE_KV_TOKENS))
    capture_s = time.perf_counter() - t0
    engine.generate([p for p, _ in requests[:8]], SamplingParams(max_tokens=8, ignore_eos=True))  # warm-up
    stream = torch.cuda.current_stream()
    graphs = engine.runner.graphs
    runs = []
    for run in range(args.serving_warmup + args.serving_runs):
        engine.step_stats.clear()
        graphs.timing = []
        torch.cuda.synchronize()
        barrier(world)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start = time.perf_counter()
        ev0.record(stream)
        ids = [engine.add_request(p, SamplingParams(max_tokens=m, ignore_eos=True), arrival_time=start)
               for p, m in mine]
        while engine.has_unfinished_requests():
            engine.step()
        ev1.record(stream)
        torch.cuda.synchronize()
        seqs = [engine.sequences.pop(i) for i in ids]
        decode_ms = sum(a.elapsed_time(b) for a, b in graphs.timing)
        stats = engine.step_stats
        runs.append({"device_ms": ev0.elapsed_time(ev1), "decode_ms": decode_ms,
                     "records": [(s.arrival_time, s.first_token_time, s.finish_time, len(s.output_token_ids))
                                 for s in seqs],
                     "steps": len(stats), "decode_steps": sum(1 for st in stats if st.num_decodes),
                     "decode_tokens": sum(st.num_decodes for st in stats),
                     "decode_ctx_tokens": sum(st.decode_context_tokens for st in stats),
                     "prefill_tokens": sum(st.num_prefill_tokens for st in stats),
                     "graphed": graphs.replays})
        if args.serving_check:
            engine.check_device_errors()
    engine.check_device_errors()
    timed = runs[args.serving_warmup:]
    # Slowest rank per run; latency records from every rank.
    job_ms = [max_over_ranks(r["device_ms"], world) for r in timed]
    dec_ms = [max_over_ranks(r["decode_ms"], world) for r in timed]
    records = gather_to_rank0([r["records"] for r in timed], world)
    if rank != 0:
        return None, model
    peaks, peak_kind = measured_peaks()
    total_tokens = sum(m for _, m in requests)
    w_bytes = model.weight_bytes()
    kv_per_token = cfg.num_layers * 2 * cfg.num_kv_heads * cfg.head_dim * 2
    r0 = timed[0]
    # Bytes a decode step must move: every weight once (the tied embedding is the LM head),
    # the K/V of every context token in every layer, and the appended rows.
    step_bytes = (r0["decode_steps"] * w_bytes + r0["decode_ctx_tokens"] * kv_per_token)
    lat = []
    for per_rank in records:  # per timed run: [rank][request] -> (arrival, first, finish, tokens)
        flat = [x for rr in per_rank for x in rr]
        ttft = np.array([f - a for a, f, _, _ in flat])
        tpot = np.array([(e - f) / (n - 1) for _, f, e, n in flat if n > 1])
        lat.append((np.percentile(ttft, 50), np.percentile(ttft, 95), np.percentile(tpot, 50),
                    np.percentile(tpot, 95)))
    lat = np.mean(np.array(lat), axis=0)
    # The median run: one run slowed by the shared host (rare, up to ~80% longer, seen with
    # either kernel build) does not move the figure; every run's time is listed beside it.
    ms = statistics.median(job_ms)
    dms = statistics.median(dec_ms)
    r0_dec_ms = statistics.median(r["decode_ms"] for r in timed)
    achieved = step_bytes / (r0_dec_ms * 1e-3) / 1e9
    out = {
        "tok_s": round(total_tokens / (ms * 1e-3), 1), "unit": "output tok/s",
        "decode_tok_s": round(world * r0["decode_tokens"] / (dms * 1e-3), 1),
        "n_gpus": world, "output_tokens": total_tokens, "duration_ms": round(ms, 2),
        "runs": len(timed), "runs_ms": [round(x, 2) for x in job_ms], "warmup_runs": args.serving_warmup,
        "ttft_p50_s": round(float(lat[0]), 4), "ttft_p95_s": round(float(lat[1]), 4),
        "tpot_p50_ms": round(float(lat[2]) * 1e3, 3), "tpot_p95_ms": round(float(lat[3]) * 1e3, 3),
        "rank0": {"requests": len(mine), "steps": r0["steps"], "decode_steps": r0["decode_steps"],
                  "prefill_tokens": r0["prefill_tokens"], "decode_ms": round(r0_dec_ms, 2),
                  "decode_step_ms_avg": round(r0_dec_ms / max(1, r0["decode_steps"]), 4),
                  "graphs_capture_s": round(capture_s, 2)},
        "roofline": {"bound": "hbm", "scope": "rank 0's decode steps (device time, graph replays with their copies)",
                     "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "peak_kind": f"{peak_kind} copy bandwidth",
                     "bytes_per_decode_step_avg": int(step_bytes / max(1, r0["decode_steps"])),
                     "weight_bytes": w_bytes, "kv_bytes_per_context_token": kv_per_token},
        "config": serving_config(),
        "timing": "device time (CUDA events) from the common start to the last step, max over ranks, median "
                  "over the timed runs; TTFT / TPOT from host clocks as benchmarks/run_bench.py:201-221 defines them",
    }
    if world == 1 and not args.profile_case:
        out["cpu_baseline"] = cpu_serving_sample(budget_s=args.serving_cpu_budget)
    return out, model


PREFIX_REQUESTS, PREFIX_LEN, PREFIX_OUT = 256, 1024, 128


def prefix_workload(seed: int = 4, vocab: int = 151936) -> list[tuple[list[int], int]]:
    """Config 4's requests: one seeded 1024-token common prefix + U{64..256} own ids, 128 outputs each."""
    g = torch.Generator().manual_seed(seed)
    shared = torch.randint(0, vocab, (PREFIX_LEN,), generator=g).tolist()
    lens = torch.randint(64, 257, (PREFIX_REQUESTS,), generator=g).tolist()
    return [(shared + torch.randint(0, vocab, (n,), generator=g).tolist(), PREFIX_OUT) for n in lens]


def run_prefix_serving(args, rank: int, world: int, local: int, model=None) -> dict | None:
    """Config 4 through ``LLMEngine`` with prefix caching; rank i mod N serves request i.

    Every run uses a fresh engine (an empty prefix cache), so each run sees the same
    admissions and hits: the requests admitted in the first step miss (their prefix is
    registered only after their prefill, engine/engine.py:297-298) and every later one finds
    the 64 prefix blocks cached.
    """
    from mini_inference_b200.engine import EngineConfig, LLMEngine, SamplingParams
    from mini_inference_b200.model import Qwen2Config, Qwen2Model, init_random

    dev = torch.device("cuda", local)
    cfg = Qwen2Config.qwen2_0_5b()
    if model is None:
        model = Qwen2Model(cfg, init_random(cfg, seed=0, std=0.02, dtype=torch.float16, device=dev,
                                            generator_device="cuda"))
    requests = prefix_workload(vocab=cfg.vocab_size)
    mine = [r for i, r in enumerate(requests) if i % world == rank]
    stream = torch.cuda.current_stream()
    runs = []
    for run in range(1 + args.serving_runs):  # one untimed run first
        engine = LLMEngine(model, EngineConfig(max_num_seqs=SERVE_MAX_SEQS, max_model_len=SERVE_MAX_LEN,
                                               max_num_batched_tokens=SERVE_BUDGET, kv_cache_tokens=SERVE_KV_TOKENS,
                                               enable_prefix_caching=True))
        torch.cuda.synchronize()
        barrier(world)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start = time.perf_counter()
        ev0.record(stream)
        seqs = [engine.sequences[engine.add_request(p, SamplingParams(max_tokens=m, ignore_eos=True),
                                                    arrival_time=start)] for p, m in mine]
        while engine.has_unfinished_requests():
            engine.step()
        ev1.record(stream)
        torch.cuda.synchronize()
        engine.check_device_errors()
        runs.append({"device_ms": ev0.elapsed_time(ev1), "hits": engine.cache.prefix_hit_tokens,
                     "prompt_tokens": sum(len(p) for p, _ in mine),
                     "misses": sum(1 for s in seqs if s.num_cached_tokens == 0),
                     "records": [(s.arrival_time, s.first_token_time, s.finish_time, len(s.output_token_ids))
                                 for s in seqs]})
        del engine
    timed = runs[1:]
    job_ms = [max_over_ranks(r["device_ms"], world) for r in timed]
    hits = [sum_over_ranks(r["hits"], world) for r in timed]
    misses = sum_over_ranks(timed[0]["misses"], world)
    records = gather_to_rank0([r["records"] for r in timed], world)
    if rank != 0:
        return None
    ms = statistics.median(job_ms)  # the median run, as in the config-3 leg
    flat = [x for rr in records[0] for x in rr]
    ttft = np.array([f - a for a, f, _, _ in flat])
    prompt_tokens = sum(len(p) for p, _ in requests)
    return {"workload": "config 4: 256 requests sharing one seeded 1024-token prefix + U{64..256} own tokens, "
                        "128 greedy outputs each, prefix caching on, max_num_batched_tokens 4096",
            "tok_s": round(PREFIX_REQUESTS * PREFIX_OUT / (ms * 1e-3), 1), "unit": "output tok/s", "n_gpus": world,
            "duration_ms": round(ms, 2), "runs": len(timed), "runs_ms": [round(x, 2) for x in job_ms],
            "prefix_hit_tokens": hits[0],
            "prefix_hit_tokens_every_run_equal": len(set(hits)) == 1, "prompt_tokens": prompt_tokens,
            "hit_rate": round(hits[0] / prompt_tokens, 4), "requests_without_hit": misses,
            "ttft_p50_s": round(float(np.percentile(ttft, 50)), 4),
            "ttft_p95_s": round(float(np.percentile(ttft, 95)), 4),
            **({"cpu_baseline": prefix_cpu_sample(budget_s=args.serving_cpu_budget)} if world == 1 else {})}


def prefix_cpu_sample(budget_s: float = 20.0, max_tokens: int = 8) -> dict:
    """Config 4 on the host cores: the reference's engine loop and PyTorch ops in float32
    (``oracle/engine_torch.py``) with prefix caching, on its first requests with outputs capped.

    The first step admits requests up to the 4096-token budget and misses (the prefix is
    registered after its prefill); later admissions hit the 64 prefix blocks, as on the GPU.
    The number of requests is set from a timed probe so the sample fits ``budget_s``.
    """
    from mini_inference_b200.model import Qwen2Config, init_random
    from oracle.engine_torch import TorchPagedCache, TorchQwen2, serve

    torch.set_num_threads(os.cpu_count() or 1)
    cfg = Qwen2Config.qwen2_0_5b()
    w = init_random(cfg, seed=0, std=0.02, dtype=torch.float32, device="cpu")
    model = TorchQwen2(w, cfg.num_layers, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, cfg.rms_norm_eps,
                       cfg.rope_theta, cfg.max_position_embeddings)
    reqs = [(p, min(m, max_tokens)) for p, m in prefix_workload(vocab=cfg.vocab_size)]

    def run(rs):
        cache = TorchPagedCache(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, len(rs) * (SERVE_MAX_LEN // BS), BS,
                                len(rs), SERVE_MAX_LEN, torch.float32, enable_prefix_caching=True)
        t0 = time.perf_counter()
        seqs = serve(model, cache, rs, len(rs), SERVE_BUDGET, SERVE_MAX_LEN)
        return time.perf_counter() - t0, sum(len(s.output_token_ids) for s in seqs), cache.prefix_hit_tokens

    probe_s, _, _ = run(reqs[:1])  # one prefix-length prefill and its decodes
    n = max(1, min(16, int(budget_s / max(probe_s, 1e-3))))
    dt, tokens, hits = run(reqs[:n])
    return {"value": round(tokens / dt, 2), "unit": "output tok/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"config 4's first {n} requests with outputs capped at {max_tokens} tokens, prefix caching on, "
                      f"the reference's engine loop and PyTorch ops in float32 on the host (oracle/engine_torch.py); "
                      f"{tokens} tokens in {dt:.2f} s, {hits} prefix-hit tokens",
            "seconds": round(dt, 2)}


def profile_serving_step(warm_steps: int = 40, steps: int = 5) -> None:
    """Per-kernel device time of config 3's graphed decode step once the batch has formed."""
    from torch.profiler import ProfilerActivity, profile

    from mini_inference_b200.engine import EngineConfig, LLMEngine, SamplingParams
    from mini_inference_b200.model import Qwen2Config, Qwen2Model, init_random

    dev = torch.device("cuda", 0)
    cfg = Qwen2Config.qwen2_0_5b()
    model = Qwen2Model(cfg, init_random(cfg, seed=0, std=0.02, dtype=torch.float16, device=dev,
                                        generator_device="cuda"))
    engine = LLMEngine(model, EngineConfig(max_num_seqs=SERVE_MAX_SEQS, max_model_len=SERVE_MAX_LEN,
                                           max_num_batched_tokens=SERVE_BUDGET, kv_cache_tokens=SERVE_KV_TOKENS))
    for prompt, n in serving_workload(seed=0, vocab=cfg.vocab_size):
        engine.add_request(prompt, SamplingParams(max_tokens=n, ignore_eos=True))
    for _ in range(warm_steps):
        engine.step()
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(steps):
            engine.step()
        torch.cuda.synchronize()
    print(f"{steps} decode steps at {engine.step_stats[-1].num_decodes} sequences")
    print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=20, max_name_column_width=70))


def sum_over_ranks(value: int, world: int) -> int:
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.int64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return int(t.item())


def gather_to_rank0(obj, world: int):
    """Every rank's ``obj`` as a list on rank 0 (gloo, host objects); ``[obj]`` alone at world 1."""
    if world == 1:
        return [[o] for o in obj]
    import torch.distributed as dist

    got = [None] * world
    dist.all_gather_object(got, obj)
    return [[got[r][i] for r in range(world)] for i in range(len(obj))]


def cpu_serving_sample(budget_s: float = 20.0, n_requests: int = 32, max_tokens: int = 32) -> dict:
    """The reference's engine on the host cores (``oracle/engine_torch.py``, float32) on a bounded sample.

    The sample is config 3's first ``n_requests`` requests with their outputs capped at
    ``max_tokens`` (fewer requests if a timed single-request probe says they would not fit
    ``budget_s``), run as the reference's LLMEngine loop; its output tokens per second is
    the number, by the same definition as the GPU leg.
    """
    from mini_inference_b200.model import Qwen2Config, init_random
    from oracle.engine_torch import TorchPagedCache, TorchQwen2, serve

    torch.set_num_threads(os.cpu_count() or 1)
    cfg = Qwen2Config.qwen2_0_5b()
    w = init_random(cfg, seed=0, std=0.02, dtype=torch.float32, device="cpu")
    model = TorchQwen2(w, cfg.num_layers, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, cfg.rms_norm_eps,
                       cfg.rope_theta, cfg.max_position_embeddings)
    reqs = [(p, min(m, max_tokens)) for p, m in serving_workload(seed=0, vocab=cfg.vocab_size)[:n_requests]]

    def run(rs):
        cache = TorchPagedCache(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, len(rs) * (SERVE_MAX_LEN // BS), BS,
                                len(rs), SERVE_MAX_LEN, torch.float32)
        t0 = time.perf_counter()
        seqs = serve(model, cache, rs, len(rs), SERVE_BUDGET, SERVE_MAX_LEN)
        return time.perf_counter() - t0, sum(len(s.output_token_ids) for s in seqs)

    probe_s, _ = run(reqs[:1])
    n = max(1, min(n_requests, int(budget_s / max(probe_s, 1e-3))))
    dt, tokens = run(reqs[:n])
    return {"value": round(tokens / dt, 2), "unit": "output tok/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"config 3's first {n} requests (prompts {[len(p) for p, _ in reqs[:n]]} tokens), outputs "
                      f"capped at {max_tokens} tokens, the reference's engine loop and PyTorch ops in float32 on the "
                      f"host (oracle/engine_torch.py); {tokens} tokens in {dt:.2f} s",
            "seconds": round(dt, 2)}


# ---------------------------------------------------------------------------------------- CPU legs


def cpu_threads() -> int:
    return torch.get_num_threads()


def cpu_sample_run(steps: int, warmup: int, budget_s: float) -> dict:
    """Time the reference's algorithm (PyTorch CPU ops) on a bounded sample of the config-2 layer call.

    Each step is one layer call over the first ``n_seq`` sequences of the batch;
    ``n_seq`` is chosen from a timed full call so that all steps fit ``budget_s``.
    """
    from oracle.paged_kv_torch import decode_attend_torch

    torch.set_num_threads(os.cpu_count() or 1)
    ctx, tables = workload(seed=0)
    g = torch.Generator().manual_seed(99)
    k = torch.randn(NUM_BLOCKS + 1, HKV, BS, D, generator=g).half()
    v = torch.randn(NUM_BLOCKS + 1, HKV, BS, D, generator=g).half()
    q = torch.randn(BATCH, HQ, D, generator=g).half()
    kn = torch.randn(BATCH, HKV, D, generator=g).half()
    t0 = time.perf_counter()
    decode_attend_torch(k, v, tables, ctx, q, kn, kn)
    full = time.perf_counter() - t0
    per_step_budget = budget_s / max(1, steps + warmup)
    n_seq = max(1, min(BATCH, int(BATCH * per_step_budget / max(full, 1e-6))))
    sub_ctx, sub_tab = ctx[:n_seq], tables[:n_seq]
    for _ in range(warmup):
        decode_attend_torch(k, v, sub_tab, sub_ctx, q[:n_seq], kn[:n_seq], kn[:n_seq])
    t0 = time.perf_counter()
    for _ in range(steps):
        decode_attend_torch(k, v, sub_tab, sub_ctx, q[:n_seq], kn[:n_seq], kn[:n_seq])
    dt = time.perf_counter() - t0
    gbs = bytes_per_layer_call(sub_ctx) * steps / dt / 1e9
    return {"value": round(gbs, 3), "unit": UNIT, "cores": cpu_threads(), "kind": "port",
            "sample": f"{steps} layer calls over the first {n_seq} of the 64 config-2 sequences "
                      f"(fp16, {sum(sub_ctx)} cached tokens), reference PyTorch ops on the host "
                      f"(oracle/paged_kv_torch.py); one full 64-sequence call took {full:.3f} s",
            "seconds": round(dt, 2)}


def cpu_baseline(args) -> dict:
    return cpu_sample_run(steps=max(3, min(args.steps, 40)), warmup=1, budget_s=20.0)


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return  # rank 0 alone times the host-core reference
    res = cpu_sample_run(args.steps, args.warmup, budget_s=120.0)
    line = {
        "metric": METRIC, "value": res["value"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded; config 2 shapes and distributions)", "impl": "reference",
        "config": decode_config(world, LAYERS),
        "cpu_baseline": {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": res["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if not args.no_serving:  # config 3 through the reference's engine loop on the host cores
        sample = cpu_serving_sample(budget_s=args.serving_cpu_budget)
        line["serving"] = {"tok_s": sample["value"], "unit": sample["unit"], "cpu_baseline": sample,
                           "config": serving_config()}
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--e2e-steps", type=int, default=200)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--prefill-only", action="store_true",
                    help="only the tcgen05 prefill leg (config 4's prefill), for ncu captures")
    ap.add_argument("--long-only", action="store_true",
                    help="only config 5's attention kernel (7B bf16, contexts 8k..32k), for ncu captures")
    ap.add_argument("--qkv-only", action="store_true",
                    help="only the qkv-post leg (RoPE fused with the KV append), for ncu captures")
    ap.add_argument("--lm-head-only", action="store_true",
                    help="only the greedy LM-head leg (0.5B embedding, batches 64 and 256), for ncu captures")
    ap.add_argument("--serving-runs", type=int, default=3, help="timed runs of configs 3 and 4 (median reported)")
    ap.add_argument("--serving-warmup", type=int, default=1, help="untimed runs of config 3 before them")
    ap.add_argument("--serving-cpu-budget", type=float, default=20.0, help="seconds for the CPU serving sample")
    ap.add_argument("--serving-check", action="store_true", help="check device errors after every serving run")
    ap.add_argument("--no-serving", action="store_true", help="skip the config-3 serving leg")
    ap.add_argument("--no-long-step", action="store_true", help="skip config 5's whole-model decode step")
    ap.add_argument("--long-step-only", action="store_true", help="only config 5's whole-model decode step")
    ap.add_argument("--decode-only", action="store_true",
                    help="only the config-2 decode step and its e2e leg (no other legs, no CPU baseline)")
    ap.add_argument("--serving-only", action="store_true",
                    help="only the config-3 serving leg (under torchrun: every rank its share)")
    ap.add_argument("--profile-case", action="store_true",
                    help="small case for ncu captures: 4 layer pools (536 MB, still above L2), no e2e / CPU legs")
    ap.add_argument("--serving-profile", action="store_true",
                    help="print the kernels of 5 graphed config-3 decode steps (torch profiler device times)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)  # at least 3 untimed warm-up steps
    args.layers = 4 if args.profile_case else LAYERS
    if args.impl == "reference":
        run_reference(args)
        return
    if args.prefill_only or args.long_only or args.lm_head_only or args.qkv_only or args.long_step_only:
        dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        torch.cuda.set_device(dev)
        run = (run_prefill if args.prefill_only else run_long_context if args.long_only
               else run_lm_head if args.lm_head_only else run_long_step if args.long_step_only else run_qkv_post)
        res = run(dev, seed=0) if args.long_step_only else run(dev, seed=0, reps=args.steps)
        print(json.dumps(res), flush=True)
        return
    if args.serving_profile:
        profile_serving_step()
        return
    rank, world, local = dist_setup(args.gpus)
    try:
        if args.serving_only:
            with ClockSampler(local) as serve_clocks:
                line, model = run_serving(args, rank, world, local)
                prefix = run_prefix_serving(args, rank, world, local, model)
            if line is not None:
                line["clocks"] = serve_clocks.summary()
                line["prefix_serving"] = prefix
        else:
            line = run_ours(args, rank, world, local)
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist

            barrier(world)
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
