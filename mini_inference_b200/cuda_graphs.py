"""CUDA-graph decode steps on the libpkv cache: the reference's ``GraphedDecoder`` (engine/cuda_graphs.py).

Same contract as engine/cuda_graphs.py:103-189: :meth:`GraphedDecoder.capture` records
the model's decode step as CUDA graphs once, :meth:`GraphedDecoder.decode` fills static
input buffers and replays one, and returns ``None`` when no captured graph fits (the
caller then runs the eager step). Padding rows of a batch bucket attend to and write
only the scratch block, as in the reference.

What differs is what a graph captures. The reference records one graph per (batch
bucket, KV-length bucket) because its attention gathers a padded copy of every block
table up to the bucket's length (engine/cuda_graphs.py:64-92). Here the decode kernel
reads the device table mirror and each row's length from device memory, so one graph
per batch bucket serves every context length, and a step's only host-to-device traffic
is one pinned copy of its token ids, slot ids and lengths. Inside the graph the
metadata builder derives positions, slot_mapping and context lengths, then every layer
runs the fused append + paged attention kernel.
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np
import torch

from . import ops
from .cache import PagedKVCache


def _batch_buckets(limit: int) -> list[int]:
    """1, 2, 4, 8, then every 16 up to ``limit`` (always including it): engine/cuda_graphs.py:34-43."""
    sizes = [b for b in (1, 2, 4, 8) if b < limit] + list(range(16, limit, 16))
    return sizes + [limit]


class _GraphDecodeContext:
    """The attention context of a captured step: everything comes from the decoder's static buffers."""

    def __init__(self, owner: "GraphedDecoder", batch: int) -> None:
        cache = owner.cache
        self.cache = cache
        self.batch = batch
        dev = cache.device
        self.seq_rows = owner.rows[:batch]
        self.lengths_in = owner.lengths[:batch]
        self.tables = ops.make_tables(cache.tables_dev, self.seq_rows)
        # Written inside the graph on every replay; allocated here so the graph owns them.
        self.positions = torch.empty(batch, dtype=torch.int64, device=dev)
        self.slot_mapping = torch.empty(batch, dtype=torch.int64, device=dev)
        self.context_lens = torch.empty(batch, dtype=torch.int32, device=dev)
        self._attends = 0

    def prepare(self) -> None:
        """Recorded once per step, before the layers: positions, write slots and lengths on the GPU."""
        ops.build_decode_metadata(self.tables, self.lengths_in, self.cache.block_size, self.cache.scratch_block,
                                  self.positions, self.slot_mapping, self.context_lens, self.cache.status)
        self._attends = 0

    def attend(self, layer_idx: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        batch, hq, _, d = q.shape
        ws = self.cache.workspace(self.cache.max_seqs, hq)
        out = torch.empty(batch, 1, hq, d, dtype=q.dtype, device=q.device)
        ops.decode_attention(self.cache.pool, layer_idx, self.tables, q[:, :, 0], self.context_lens, ws,
                             k_new=k[:, :, 0], v_new=v[:, :, 0], slot_mapping=self.slot_mapping,
                             out=out[:, 0], status=self.cache.status, inputs_ready=self._attends > 0)
        self._attends += 1
        return out.transpose(1, 2)

    def attend_qkv(self, layer_idx: int, qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                   num_q_heads: int) -> torch.Tensor:
        """RoPE, append and paged attention in one kernel (as ``PagedDecodeContext.attend_qkv``)."""
        batch = qkv.shape[0]
        rows = qkv.reshape(batch, -1)
        ws = self.cache.workspace(self.cache.max_seqs, num_q_heads)
        out = torch.empty(batch, 1, num_q_heads, self.cache.head_dim, dtype=qkv.dtype, device=qkv.device)
        ops.decode_attention_rope(self.cache.pool, layer_idx, self.tables, rows, cos, sin, self.context_lens, ws,
                                  self.slot_mapping, out=out[:, 0], status=self.cache.status,
                                  inputs_ready=self._attends > 0)
        self._attends += 1
        return out.transpose(1, 2)


class GraphedDecoder:
    """Captures the decode step as CUDA graphs (one per batch bucket) and replays them."""

    def __init__(self, model, cache: PagedKVCache, max_batch: int, head=None) -> None:
        if not isinstance(cache, PagedKVCache) or not cache.on_gpu:
            raise TypeError("GraphedDecoder needs a libpkv PagedKVCache on a CUDA device")
        self.model, self.cache = model, cache
        # With a greedy head (sampler.GreedyLMHead) each graph ends in the fused LM head +
        # argmax and yields token ids instead of float32 logits.
        self.head = head
        self.paged = True
        self.device = cache.device
        self.batch_buckets = _batch_buckets(min(max_batch, cache.max_seqs))
        top = self.batch_buckets[-1]
        self.ids = torch.zeros(top, 1, dtype=torch.long, device=self.device)
        self.rows = torch.full((top,), -1, dtype=torch.int32, device=self.device)  # -1: a padding row
        self.lengths = torch.zeros(top, dtype=torch.int32, device=self.device)
        # batch -> (graph, its logits, its context); the context stays alive with its graph.
        self.graphs: dict[int, tuple[torch.cuda.CUDAGraph, torch.Tensor, _GraphDecodeContext]] = {}
        self._pool = None
        self.replays = 0
        # When a list, every decode() appends a (start, end) pair of CUDA events around its
        # copies and replay, for device-side timing of the steps.
        self.timing: list | None = None

    @torch.inference_mode()
    def capture(self) -> None:
        """Record one graph per batch bucket, largest first so the smaller ones reuse its memory."""
        for batch in reversed(self.batch_buckets):
            self._capture_one(batch)
        torch.cuda.synchronize()

    def _capture_one(self, batch: int) -> None:
        ctx = _GraphDecodeContext(self, batch)

        def step() -> torch.Tensor:
            ctx.prepare()
            hidden = self.model(self.ids[:batch], ctx.positions.unsqueeze(1), ctx)
            if self.head is not None:
                return self.head(hidden[:, -1])
            return self.model.compute_logits(hidden[:, -1]).float()

        self.rows.fill_(-1)  # every row reads and writes the scratch block while recording
        self.lengths.zero_()
        self.cache.sync_tables()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):  # warm-up outside the graph (library and allocator setup)
            for _ in range(2):
                step()
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, pool=self._pool):
            logits = step()
        self._pool = graph.pool()
        self.graphs[batch] = (graph, logits, ctx)

    @torch.inference_mode()
    def decode(self, slots: Sequence[int], last_tokens: Sequence[int]) -> torch.Tensor | None:
        """One decode step through a captured graph: logits ``[len(slots), vocab]``, or None.

        With a greedy head the result is the step's token ids (int64 ``[len(slots)]`` on the
        device, valid until the next replay) instead of logits.
        """
        n = len(slots)
        batch = next((b for b in self.batch_buckets if b >= n), None)
        if batch is None or batch not in self.graphs:
            return None
        graph, logits, _ = self.graphs[batch]
        slots_np = np.asarray(list(slots), dtype=np.int32)
        positions = self.cache._bm.decode_positions(slots_np)  # raises the reference's ValueError
        if self.cache.enable_copy_on_write:
            self.cache.copy_on_write([(s, int(p), 1) for s, p in zip(slots_np.tolist(), positions.tolist())])
        self.cache.sync_tables()
        host = np.zeros((3, batch), dtype=np.int64)
        host[0, :n] = np.asarray(list(last_tokens), dtype=np.int64)
        host[1, :] = -1
        host[1, :n] = slots_np
        host[2, :n] = positions
        if self.timing is not None:
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
        staged = torch.from_numpy(host).pin_memory().to(self.device, non_blocking=True)
        self.ids[:batch, 0].copy_(staged[0])
        self.rows[:batch].copy_(staged[1])
        self.lengths[:batch].copy_(staged[2])
        graph.replay()
        if self.timing is not None:
            end.record()
            self.timing.append((start, end))
        self.replays += 1
        self.cache._bm.commit_decode(slots_np)
        return logits[:n]
