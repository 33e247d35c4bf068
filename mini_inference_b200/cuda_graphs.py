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
        self.ids, self.seq_rows, self.lengths_in = owner.staged_views(batch)
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
        # A step's inputs, read in place by its graph: for a bucket of b rows, b int64 token
        # ids, then b int32 table rows (-1: a padding row) and b int32 lengths, 16 b bytes in
        # all, filled in pinned host memory and sent with one copy per step.
        # The step's table edits (int32 triples) follow the inputs in the same copy.
        self._edit_cap = max(1024, 2 * cache.max_seqs * cache.max_blocks_per_seq)
        nbytes = 16 * top + 12 * self._edit_cap
        self._staged_dev = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        self._staged_host = torch.zeros(nbytes, dtype=torch.uint8).pin_memory()
        self._staged_np = self._staged_host.numpy()
        self._staged_sent = torch.cuda.Event()  # the last copy out of the pinned buffer
        # batch -> (graph, its logits, its context); the context stays alive with its graph.
        self.graphs: dict[int, tuple[torch.cuda.CUDAGraph, torch.Tensor, _GraphDecodeContext]] = {}
        self._pool = None
        self.replays = 0
        # When a list, every decode() appends a (start, end) pair of CUDA events around its
        # copies and replay, for device-side timing of the steps.
        self.timing: list | None = None

    def staged_views(self, batch: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """The device inputs of a ``batch``-row graph: ids ``[batch, 1]`` int64, table rows and lengths int32."""
        buf = self._staged_dev[:16 * batch]
        return (buf[:8 * batch].view(torch.int64).view(batch, 1), buf[8 * batch:12 * batch].view(torch.int32),
                buf[12 * batch:].view(torch.int32))

    def _host_views(self, batch: int) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
        buf = self._staged_np[:16 * batch]
        return buf[:8 * batch].view(np.int64), buf[8 * batch:12 * batch].view(np.int32), buf[12 * batch:].view(np.int32)

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
            hidden = self.model(ctx.ids, ctx.positions.unsqueeze(1), ctx)
            if self.head is not None:
                return self.head(hidden[:, -1])
            return self.model.compute_logits(hidden[:, -1]).float()

        ids, rows, lengths = ctx.ids, ctx.seq_rows, ctx.lengths_in
        ids.zero_()
        rows.fill_(-1)  # every row reads and writes the scratch block while recording
        lengths.zero_()
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
        slots_np = (slots if isinstance(slots, np.ndarray) and slots.dtype == np.int32
                    else np.asarray(list(slots), dtype=np.int32))
        positions = self.cache._bm.decode_positions(slots_np)  # raises the reference's ValueError
        if self.cache.enable_copy_on_write:
            self.cache.copy_on_write([(s, int(p), 1) for s, p in zip(slots_np.tolist(), positions.tolist())])
        # The pinned buffer is rewritten only after the previous step's copy out of it ran
        # (already so when the caller read that step's tokens).
        self._staged_sent.synchronize()
        edits = self._staged_np[16 * batch:16 * batch + 12 * self._edit_cap].view(np.int32).reshape(-1, 3)
        n_edits = self.cache.drain_table_edits(edits)
        h_ids, h_rows, h_len = self._host_views(batch)
        h_ids[:n] = last_tokens
        h_ids[n:] = 0
        h_rows[:n] = slots_np
        h_rows[n:] = -1
        h_len[:n] = positions
        h_len[n:] = 0
        if self.timing is not None:
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
        nbytes = 16 * batch + 12 * n_edits
        self._staged_dev[:nbytes].copy_(self._staged_host[:nbytes], non_blocking=True)
        self._staged_sent.record()
        if n_edits:  # the allocator's new blocks, before the graph reads the tables
            dev_edits = self._staged_dev[16 * batch:nbytes].view(torch.int32).view(n_edits, 3)
            ops.update_tables(self.cache.tables_dev, dev_edits, self.cache.status)
        graph.replay()
        if self.timing is not None:
            end.record()
            self.timing.append((start, end))
        self.replays += 1
        self.cache._bm.commit_decode(slots_np)
        return logits[:n]
