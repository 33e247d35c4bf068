"""Greedy next-token selection fused with the LM head (the reference's sampling seam).

The reference turns the last hidden state of each sequence into float32 logits,
``Qwen2ForCausalLM.compute_logits(hidden).float()`` (``engine/model.py:321-323``,
``engine/engine.py:97-123``), and ``Sampler.__call__`` returns
``logits.argmax(dim=-1).tolist()`` when every request is greedy
(``engine/sampler.py:27-31``). :class:`GreedyLMHead` gives the same token ids from the
hidden states directly, through ``pkv_lm_head_argmax``: the weight is streamed once and
the ``[B, vocab]`` logits are never written. Batches with sampled (non-greedy) requests
need the logits and stay on the reference's ``compute_logits`` + ``Sampler``.
"""

from __future__ import annotations

from collections.abc import Sequence

import torch

from . import ops


class GreedyLMHead:
    """``compute_logits`` + greedy ``Sampler`` as one kernel over ``weight`` ``[vocab, hidden]``.

    ``weight`` is the LM head (the embedding matrix when the embeddings are tied,
    ``engine/model.py:300-323``). One instance per stream: the workspace is reused by
    every call and left zeroed by each. Calls pass ``PKV_LM_WEIGHT_READY``: the weight (a
    model parameter) must not be written by the kernel launched just before a call on the
    same stream.
    """

    KERNEL_ROWS = 256  # rows one pkv_lm_head_argmax call takes; larger batches go in slices

    def __init__(self, weight: torch.Tensor, max_batch: int = 256) -> None:
        if weight.dim() != 2 or not weight.is_cuda:
            raise ValueError("weight must be a [vocab, hidden] CUDA tensor")
        self.weight = weight
        self.max_batch = max_batch
        self.workspace = ops.lm_head_argmax_workspace(min(max_batch, self.KERNEL_ROWS), weight.device)
        self.ids = torch.empty(max_batch, dtype=torch.int64, device=weight.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=weight.device)

    def __call__(self, hidden: torch.Tensor, max_logits: torch.Tensor | None = None) -> torch.Tensor:
        """Token ids (int64 ``[B]``, on the device) of the hidden rows ``[B, hidden]``."""
        n = hidden.shape[0]
        if n > self.max_batch:
            raise ValueError(f"batch {n} exceeds max_batch {self.max_batch}")
        if n <= self.KERNEL_ROWS:
            return ops.lm_head_argmax(hidden, self.weight, self.workspace, out=self.ids, max_logits=max_logits,
                                      status=self.status, weight_ready=True)
        for a in range(0, n, self.KERNEL_ROWS):  # each slice streams the weight once more
            b = min(n, a + self.KERNEL_ROWS)
            ops.lm_head_argmax(hidden[a:b], self.weight, self.workspace, out=self.ids[a:b],
                               max_logits=None if max_logits is None else max_logits[a:b], status=self.status,
                               weight_ready=True)
        return self.ids[:n]

    def tokens(self, hidden: torch.Tensor, params: Sequence | None = None) -> list[int]:
        """``Sampler(...)(compute_logits(hidden).float(), params)`` for an all-greedy batch."""
        if params is not None and not all(p.greedy for p in params):
            raise ValueError("sampled requests need the logits: use compute_logits and the reference Sampler")
        ids = self(hidden).tolist()
        try:
            ops.raise_device_errors(self.status)
        except RuntimeError:
            self.workspace.zero_()  # a call that gave up may have left maxima or its ticket behind
            raise
        return ids
