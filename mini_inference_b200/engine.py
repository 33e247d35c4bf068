"""Continuous-batching serving loop over the paged-KV path: the reference's ``LLMEngine`` step.

``LLMEngine.step`` follows ``engine/engine.py:281-328`` decision for decision: one
scheduler call (the native :class:`~mini_inference_b200.scheduler.Scheduler`, the
reference's admission, token budget, preemption and finish rules), the newly admitted
requests prefilled in packs of at most ``max_num_batched_tokens`` tokens
(``pack_by_budget``, ``engine/engine.py:126-141``) with their prefix registered after
each pack (``engine/engine.py:297-298``), then one batched decode of every running
sequence. What runs underneath is this package: the paged cache and its contexts (RoPE
fused with the KV append, paged prefill on tcgen05, split-K paged decode), the decode step
replayed as one CUDA graph per batch bucket, and the LM head fused with greedy selection,
so no ``[B, vocab]`` logits are written and each step reads back only its token ids.

Only greedy sampling is served (temperature 0, the setting of every configuration this
path is measured on); a request with ``temperature > 0`` is refused when it is added.
Token-id prompts only: the tokenizer is not part of this path.
"""

from __future__ import annotations

import enum
import time
from collections.abc import Callable, Sequence as SequenceOf
from dataclasses import dataclass, field

import numpy as np
import torch

from .cache import PagedKVCache
from .cuda_graphs import GraphedDecoder
from .sampler import GreedyLMHead
from .scheduler import FinishReason, Scheduler, SequenceStatus


@dataclass
class SamplingParams:
    """The reference's ``SamplingParams`` (engine/sequence.py:9-40); only greedy is served here."""

    temperature: float = 0.0
    top_k: int = 0
    top_p: float = 1.0
    max_tokens: int = 128
    ignore_eos: bool = False

    def __post_init__(self) -> None:
        if self.temperature < 0:
            raise ValueError("temperature must be >= 0")
        if self.max_tokens < 1:
            raise ValueError("max_tokens must be at least 1")

    @property
    def greedy(self) -> bool:
        return self.temperature == 0


@dataclass(eq=False)
class Sequence:
    """One request moving through the engine (the fields of engine/sequence.py:58-100)."""

    seq_id: int
    prompt_token_ids: list[int]
    sampling: SamplingParams
    arrival_time: float
    output_token_ids: list[int] = field(default_factory=list)
    status: enum.Enum = SequenceStatus.WAITING
    slot: int | None = None
    finish_reason: FinishReason | None = None
    first_token_time: float | None = None
    finish_time: float | None = None
    num_preemptions: int = 0
    num_cached_tokens: int = 0

    @property
    def prompt_len(self) -> int:
        return len(self.prompt_token_ids)

    @property
    def num_tokens(self) -> int:
        return len(self.prompt_token_ids) + len(self.output_token_ids)

    @property
    def token_ids(self) -> list[int]:
        return self.prompt_token_ids + self.output_token_ids

    @property
    def last_token(self) -> int:
        return self.output_token_ids[-1]

    @property
    def is_finished(self) -> bool:
        return self.status is SequenceStatus.FINISHED


@dataclass
class EngineConfig:
    """The settings of ``engine/config.py:23-109`` that the paged path uses (same names and defaults).

    ``cuda_graph_max_batch`` defaults to ``max_num_seqs`` here: a graph per batch bucket
    serves every context length (the decode kernel reads lengths and tables from device
    memory), so large batches are graphed too.
    """

    max_num_seqs: int = 32
    max_model_len: int = 2048
    max_num_batched_tokens: int = 4096
    scheduling: str = "continuous"
    block_size: int = 16
    enable_prefix_caching: bool = False
    kv_cache_tokens: int | None = None
    batched_prefill: bool = True
    cuda_graphs: bool = True
    cuda_graph_max_batch: int | None = None
    # Prefill long prompts across steps under the token budget (opt-in; the reference has
    # none, README.md:470-473). With it a prompt may be longer than the budget.
    chunked_prefill: bool = False

    def __post_init__(self) -> None:
        if self.max_num_seqs < 1:
            raise ValueError("max_num_seqs must be at least 1")
        if self.max_model_len < 2:
            raise ValueError("max_model_len must be at least 2")
        if self.scheduling not in ("continuous", "static"):
            raise ValueError(f"scheduling must be 'continuous' or 'static', got {self.scheduling!r}")
        if self.kv_cache_tokens is None:
            self.kv_cache_tokens = self.max_num_seqs * self.max_model_len
        if self.kv_cache_tokens < self.max_model_len:
            raise ValueError("kv_cache_tokens must be >= max_model_len")
        if self.max_num_batched_tokens < self.max_model_len and not self.chunked_prefill:
            raise ValueError("max_num_batched_tokens must be >= max_model_len")
        if self.max_num_batched_tokens < 1:
            raise ValueError("max_num_batched_tokens must be at least 1")
        if self.cuda_graph_max_batch is None:
            self.cuda_graph_max_batch = self.max_num_seqs


def pack_by_budget(lengths: SequenceOf[int], budget: int) -> list[list[int]]:
    """Groups of item indices (order kept) whose lengths sum to at most ``budget``; engine/engine.py:126-141."""
    groups: list[list[int]] = []
    total = 0
    for i, n in enumerate(lengths):
        if groups and budget > 0 and total + n <= budget:
            groups[-1].append(i)
            total += n
        else:
            groups.append([i])
            total = n
    return groups


class ModelRunner:
    """One packed prefill or one batched decode per call, returning greedy token ids.

    The reference's ``ModelRunner.prefill_packed`` / ``decode`` (engine/engine.py:99-123)
    followed by the greedy ``Sampler``: the context is built, the model runs, the context
    commits, and the LM head fused with argmax picks each sequence's next token.
    """

    def __init__(self, model, cache: PagedKVCache, max_batch: int) -> None:
        self.model = model
        self.cache = cache
        self.device = cache.device
        self.head = GreedyLMHead(model.lm_head_weight, max_batch=max_batch)
        self.graphs: GraphedDecoder | None = None
        self._ids_host = torch.empty(0, dtype=torch.int64).pin_memory()

    def enable_cuda_graphs(self, max_batch: int) -> None:
        self.graphs = GraphedDecoder(self.model, self.cache, max_batch, head=self.head)
        self.graphs.capture()

    def _ids_to_device(self, ids: list[int]) -> torch.Tensor:
        if self._ids_host.numel() < len(ids):
            self._ids_host = torch.empty(max(len(ids), 2 * self._ids_host.numel()), dtype=torch.int64).pin_memory()
        host = self._ids_host[:len(ids)]
        host.numpy()[:] = ids
        return host.to(self.device, non_blocking=True)

    def _tokens(self, hidden_rows: torch.Tensor) -> list[int]:
        return self.head.tokens(hidden_rows)

    @torch.inference_mode()
    def prefill_tokens(self, slots: SequenceOf[int], prompts: SequenceOf[SequenceOf[int]]) -> list[int]:
        """Prefill several prompts in one pass; the next token of each (engine/engine.py:99-106)."""
        ctx = self.cache.packed_prefill_context(slots, [len(p) for p in prompts])
        ids = self._ids_to_device([t for p in prompts for t in p]).unsqueeze(0)
        hidden = self.model(ids, ctx.positions.unsqueeze(0), ctx)
        ctx.commit()
        return self._tokens(hidden[0, ctx.last_index])

    @torch.inference_mode()
    def decode_tokens(self, slots: SequenceOf[int], last_tokens: SequenceOf[int],
                      while_running: Callable[[], None] | None = None) -> list[int]:
        """One decode step for every sequence; the next token of each (engine/engine.py:108-123).

        ``slots`` may be an int32 numpy array. ``while_running`` is called once the step's
        GPU work is queued and before its tokens are read back, so that host bookkeeping
        overlaps the GPU.
        """
        if self.graphs is not None:
            ids = self.graphs.decode(slots, last_tokens)
            if ids is not None:
                if while_running is not None:
                    while_running()
                return ids.tolist()
        ctx = self.cache.decode_context([int(s) for s in slots])
        ids = self._ids_to_device(list(last_tokens)).unsqueeze(1)
        hidden = self.model(ids, ctx.positions.unsqueeze(1), ctx)
        ctx.commit()
        if while_running is not None:
            while_running()
        return self._tokens(hidden[:, -1])


@dataclass
class StepStats:
    """What one engine step did (engine/engine.py:207-218), plus its decode context size."""

    step: int
    time: float
    num_prefills: int
    num_prefill_tokens: int
    num_decodes: int
    decode_context_tokens: int
    num_finished: int
    num_running: int
    num_waiting: int


class LLMEngine:
    """Continuous batching of greedy requests on the paged-KV path (engine/engine.py:221-364).

    ``model`` is a :class:`~mini_inference_b200.model.Qwen2Model` (or anything with its call
    surface: ``model(ids, positions, ctx)``, ``cfg`` and ``lm_head_weight``) on a CUDA device.
    """

    def __init__(self, model, config: EngineConfig, eos_token_ids: SequenceOf[int] = ()) -> None:
        self.config = config
        self.model = model
        cfg = model.cfg
        self.cache = PagedKVCache(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim,
                                  num_blocks=config.kv_cache_tokens // config.block_size,
                                  block_size=config.block_size, max_seqs=config.max_num_seqs,
                                  max_len=config.max_model_len, dtype=model.dtype, device=model.device,
                                  enable_prefix_caching=config.enable_prefix_caching)
        self.runner = ModelRunner(model, self.cache, max_batch=config.max_num_seqs)
        if config.cuda_graphs:
            self.runner.enable_cuda_graphs(min(config.max_num_seqs, config.cuda_graph_max_batch))
        self.eos_token_ids = list(eos_token_ids)
        self.scheduler = Scheduler(config, self.cache, self.eos_token_ids)
        self.sequences: dict[int, Sequence] = {}
        self.step_stats: list[StepStats] = []
        self._next_id = 0

    def add_request(self, prompt: SequenceOf[int], sampling_params: SamplingParams | None = None,
                    arrival_time: float | None = None) -> int:
        """Queue a request of token ids; returns its id (engine/engine.py:251-272)."""
        if isinstance(prompt, str):
            raise TypeError("this engine takes token ids; the tokenizer is not part of the paged-KV path")
        sp = sampling_params or SamplingParams()
        if not sp.greedy:
            raise NotImplementedError("only greedy requests are served (the LM head is fused with argmax)")
        seq = Sequence(seq_id=self._next_id, prompt_token_ids=list(prompt), sampling=sp,
                       arrival_time=time.perf_counter() if arrival_time is None else arrival_time)
        self.scheduler.add(seq)  # raises if the prompt can never fit
        self.sequences[seq.seq_id] = seq
        self._next_id += 1
        return seq.seq_id

    def has_unfinished_requests(self) -> bool:
        return self.scheduler.has_work()

    def step(self) -> list[tuple[int, int]]:
        """One engine step; returns the ``(request_id, new_token)`` pairs it produced."""
        batch = self.scheduler.schedule()
        new_tokens: list[tuple[int, int]] = []
        budget = self.config.max_num_batched_tokens if self.config.batched_prefill else 0
        # Each prefill processes its next `count` tokens: all it has not cached, unless
        # chunked prefill gave it only part of this step's budget. Only a sequence whose
        # prefill reaches its last token samples one.
        starts = [self.cache.lengths[s.slot] for s in batch.prefills]
        counts = batch.prefill_tokens
        news = [s.token_ids[a:a + n] for s, a, n in zip(batch.prefills, starts, counts)]
        n_prefill_tokens = sum(counts)
        for group in pack_by_budget(counts, budget):
            seqs = [batch.prefills[i] for i in group]
            tokens = self.runner.prefill_tokens([s.slot for s in seqs], [news[i] for i in group])
            for s in seqs:
                self.cache.register_prefix(s.slot, s.token_ids)
            done = [(s, t) for i, s, t in zip(group, seqs, tokens) if starts[i] + counts[i] == s.num_tokens]
            self.scheduler.append_tokens([s for s, _ in done], [t for _, t in done], time.perf_counter())
            new_tokens.extend((s.seq_id, t) for s, t in done)
        ctx_tokens = 0
        n_finished = sum(s.is_finished for s in batch.prefills)
        if batch.decodes:
            context = [0]

            def count_context() -> None:  # step statistics, counted while the GPU decodes
                context[0] = sum(len(s.prompt_token_ids) + len(s.output_token_ids) for s in batch.decodes)

            # The token at each sequence's last position (its last output, or with chunked
            # prefill the last prompt token when the final chunk left exactly that one), as
            # the native scheduler reports it.
            tokens = self.runner.decode_tokens(self.scheduler.decode_slots(), self.scheduler.decode_last_tokens(),
                                               while_running=count_context)
            ctx_tokens = context[0]
            n_finished += self.scheduler.append_tokens(batch.decodes, tokens, time.perf_counter())
            new_tokens.extend(zip((s.seq_id for s in batch.decodes), tokens))
        self.step_stats.append(StepStats(
            step=len(self.step_stats), time=time.perf_counter(), num_prefills=len(batch.prefills),
            num_prefill_tokens=n_prefill_tokens, num_decodes=len(batch.decodes), decode_context_tokens=ctx_tokens,
            num_finished=n_finished,
            num_running=self.scheduler.num_running, num_waiting=self.scheduler.num_waiting))
        return new_tokens

    def abort_request(self, request_id: int) -> None:
        self.scheduler.abort(self.sequences[request_id], time.perf_counter())

    def check_device_errors(self) -> None:
        """Synchronise and raise any error a kernel recorded (bad index, timed-out wait)."""
        self.cache.raise_device_errors()

    def generate(self, prompts: SequenceOf[SequenceOf[int]],
                 sampling_params: SamplingParams | SequenceOf[SamplingParams] | None = None) -> list[Sequence]:
        """Queue every prompt, step until all are done, return the sequences in order."""
        if sampling_params is None or isinstance(sampling_params, SamplingParams):
            sampling_params = [sampling_params or SamplingParams()] * len(prompts)
        ids = [self.add_request(p, sp) for p, sp in zip(prompts, sampling_params)]
        while self.has_unfinished_requests():
            self.step()
        self.check_device_errors()
        return [self.sequences[i] for i in ids]


def summarize(seqs: SequenceOf[Sequence], start: float) -> dict:
    """Throughput and latency as ``benchmarks/run_bench.py:201-221`` defines them.

    TTFT = first token - arrival, TPOT = (finish - first token) / (outputs - 1), and output
    tokens per second over ``max(finish) - start``.
    """
    ttft = np.array([s.first_token_time - s.arrival_time for s in seqs])
    tpot = np.array([(s.finish_time - s.first_token_time) / (len(s.output_token_ids) - 1)
                     for s in seqs if len(s.output_token_ids) > 1])
    duration = max(s.finish_time for s in seqs) - start
    tokens = sum(len(s.output_token_ids) for s in seqs)

    def pct(a: np.ndarray, q: float) -> float:
        return round(float(np.percentile(a, q)), 4) if a.size else 0.0

    return {"num_requests": len(seqs), "output_tokens": tokens, "duration_s": round(duration, 4),
            "output_tokens_per_s": round(tokens / duration, 1), "ttft_p50_s": pct(ttft, 50),
            "ttft_p95_s": pct(ttft, 95), "tpot_p50_ms": round(pct(tpot, 50) * 1000, 3),
            "tpot_p95_ms": round(pct(tpot, 95) * 1000, 3)}
