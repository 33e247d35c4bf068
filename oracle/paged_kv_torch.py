"""The reference's paged decode step restated with PyTorch CPU ops, for the timed CPU baseline.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``). The reference is a
PyTorch program, so its CPU path is a sequence of ATen calls; this module
replays that sequence on the host cores so that ``bench.py --impl reference``
and the ``cpu_baseline`` leg time what the reference itself does, not a
slower numpy transcription. It follows ``PagedDecodeContext``
(``engine/kv_cache.py:592-620``) and ``decode_attention``
(``engine/model.py:126-147``):

1. append: an index_put of each new row at ``(table[p // bs], p % bs)``;
2. gather: every sequence's blocks in table order, padded with block 0 to the
   longest sequence, laid out as ``[B, Hkv, blocks * bs, d]`` (a copy);
3. mask: ``key <= position``;
4. attention: query heads regrouped ``[B, Hq, d] -> [B, Hkv, group, d]`` and one
   scaled-dot-product attention call with the boolean mask.

``tests/test_oracle_golden.py`` pins it to the reference's golden outputs.
"""

from __future__ import annotations

from collections.abc import Sequence

import torch
import torch.nn.functional as F


def decode_attend_torch(k_layer: torch.Tensor, v_layer: torch.Tensor, tables: Sequence[Sequence[int]],
                        positions: Sequence[int], q: torch.Tensor, k_new: torch.Tensor,
                        v_new: torch.Tensor) -> torch.Tensor:
    """One decode step on one layer (mutates the pool); q ``[B, Hq, d]`` -> ``[B, Hq, d]``."""
    bs = k_layer.shape[2]
    batch, hq, d = q.shape
    hkv = k_new.shape[1]
    pos = torch.as_tensor(list(positions), dtype=torch.int64)
    write_blocks = torch.as_tensor([t[p // bs] for t, p in zip(tables, positions)], dtype=torch.int64)
    k_layer[write_blocks, :, pos % bs] = k_new
    v_layer[write_blocks, :, pos % bs] = v_new
    nblk = int(pos.max()) // bs + 1
    padded = torch.as_tensor([list(t[:nblk]) + [0] * (nblk - min(len(t), nblk)) for t in tables], dtype=torch.int64)
    kv_len = nblk * bs
    keys = k_layer[padded].permute(0, 2, 1, 3, 4).reshape(batch, hkv, kv_len, d)
    values = v_layer[padded].permute(0, 2, 1, 3, 4).reshape(batch, hkv, kv_len, d)
    allowed = (torch.arange(kv_len) <= pos[:, None])[:, None, None, :]
    grouped = q.reshape(batch, hkv, hq // hkv, d)
    return F.scaled_dot_product_attention(grouped, keys, values, attn_mask=allowed).reshape(batch, hq, d)
