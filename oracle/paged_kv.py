"""numpy restatement of the reference's paged KV append and paged attention.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): the checker for the
CUDA kernels in ``mini_inference_b200/csrc/`` and the timed CPU restatement
behind ``bench.py --impl reference``.

What each function follows in the reference (Ham12-3/mini-inference):

* :func:`write_index`, :func:`slot_mapping` -- ``PagedKVCache.write_index``,
  ``engine/kv_cache.py:562-573``; the decode write location
  ``(table[p // bs], p % bs)`` of ``engine/kv_cache.py:603-605``.
* :func:`kv_append` -- the index_put scatter ``k_layer[blocks, :, offsets] = k``
  of ``engine/kv_cache.py:613-614`` and ``:288-289``.
* :func:`decode_attend` -- ``PagedDecodeContext.__init__`` / ``.attend``,
  ``engine/kv_cache.py:592-620``: append, gather every sequence's blocks in
  table order padded with block 0 up to the longest sequence, mask
  ``key <= position``, then ``decode_attention`` (``engine/model.py:126-147``):
  query head h reads KV head ``h // group``, scale ``1/sqrt(head_dim)``.
* :func:`packed_prefill_attend` -- ``PackedPrefillContext``,
  ``engine/kv_cache.py:252-297``: write the new tokens' K/V, then each token
  attends to its own sequence's keys ``0..position`` (the block-diagonal
  causal mask without a prefix; keys read back from the cache with one).

Layout (the reference's): one layer of the pool is
``k_layer, v_layer: [num_blocks + 1, num_kv_heads, block_size, head_dim]``.
Arithmetic is done in ``acc`` precision (float64 by default) on the stored
values; callers round to the storage dtype where they compare bit patterns.
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np


def write_index(tables: Sequence[Sequence[int]], starts: Sequence[int], counts: Sequence[int],
                block_size: int) -> tuple[np.ndarray, np.ndarray]:
    """(block, offset) of tokens ``start..start+count-1`` of each sequence, concatenated."""
    blocks, offsets = [], []
    for table, a, n in zip(tables, starts, counts):
        pos = np.arange(a, a + n, dtype=np.int64)
        t = np.asarray(table, dtype=np.int64)
        blocks.append(t[pos // block_size])
        offsets.append(pos % block_size)
    if not blocks:
        return np.zeros(0, np.int64), np.zeros(0, np.int64)
    return np.concatenate(blocks), np.concatenate(offsets)


def slot_mapping(blocks: np.ndarray, offsets: np.ndarray, block_size: int) -> np.ndarray:
    """Flat token slot ``block * block_size + offset`` (the vLLM-style slot_mapping)."""
    return np.asarray(blocks, np.int64) * block_size + np.asarray(offsets, np.int64)


def kv_append(k_layer: np.ndarray, v_layer: np.ndarray, k_rows: np.ndarray, v_rows: np.ndarray,
              blocks: np.ndarray, offsets: np.ndarray) -> None:
    """Scatter rows ``[N, kv_heads, head_dim]`` into ``[blocks, kv_heads, block_size, head_dim]`` in place."""
    for i in range(len(blocks)):
        k_layer[blocks[i], :, offsets[i]] = k_rows[i]
        v_layer[blocks[i], :, offsets[i]] = v_rows[i]


def _softmax_attend(q: np.ndarray, keys: np.ndarray, values: np.ndarray, allowed: np.ndarray,
                    acc) -> np.ndarray:
    """q [..., Tq, d], keys/values [..., Tk, d], allowed [..., Tq, Tk] -> [..., Tq, d]."""
    scale = 1.0 / np.sqrt(q.shape[-1])
    s = np.matmul(q.astype(acc), np.swapaxes(keys.astype(acc), -1, -2)) * acc(scale)
    s = np.where(allowed, s, -np.inf)
    m = np.max(s, axis=-1, keepdims=True)
    p = np.exp(s - m)
    p = np.where(allowed, p, 0)
    return np.matmul(p, values.astype(acc)) / np.sum(p, axis=-1, keepdims=True)


def decode_attend(k_layer: np.ndarray, v_layer: np.ndarray, tables: Sequence[Sequence[int]],
                  positions: Sequence[int], q: np.ndarray, k_new: np.ndarray, v_new: np.ndarray,
                  acc=np.float64) -> np.ndarray:
    """One batched decode step on one layer; mutates the pool (the append) and returns ``[B, Hq, d]``.

    ``positions[b]`` is the number of tokens sequence b already holds, which
    is where its new token goes. q is ``[B, Hq, d]``, k_new / v_new ``[B, Hkv, d]``.
    """
    bs = k_layer.shape[2]
    batch, hq, d = q.shape
    hkv = k_new.shape[1]
    pos = np.asarray(positions, np.int64)
    if any(p // bs >= len(t) for p, t in zip(pos, tables)):
        raise ValueError("a sequence has no block for its next token (call ensure_capacity first)")
    wb = np.array([t[p // bs] for t, p in zip(tables, pos)], np.int64)
    kv_append(k_layer, v_layer, k_new, v_new, wb, pos % bs)
    nblk = int(pos.max()) // bs + 1
    padded = np.array([list(t[:nblk]) + [0] * (nblk - len(t[:nblk])) for t in tables], np.int64)
    kv_len = nblk * bs
    # [B, nblk, Hkv, bs, d] -> [B, Hkv, nblk * bs, d]
    keys = k_layer[padded].transpose(0, 2, 1, 3, 4).reshape(batch, hkv, kv_len, d)
    values = v_layer[padded].transpose(0, 2, 1, 3, 4).reshape(batch, hkv, kv_len, d)
    group = hq // hkv
    qg = q.reshape(batch, hkv, group, d)  # query head h -> (h // group, h % group)
    allowed = (np.arange(kv_len)[None, :] <= pos[:, None])[:, None, None, :]
    out = _softmax_attend(qg, keys, values, allowed, acc)
    return out.reshape(batch, hq, d)


def packed_prefill_attend(k_layer: np.ndarray, v_layer: np.ndarray, tables: Sequence[Sequence[int]],
                          starts: Sequence[int], lengths: Sequence[int], q: np.ndarray, k: np.ndarray,
                          v: np.ndarray, acc=np.float64) -> np.ndarray:
    """Packed prefill of several sequences on one layer; mutates the pool and returns ``[Hq, N, d]``.

    q is ``[Hq, N, d]`` and k / v ``[Hkv, N, d]`` for the N packed new tokens
    (sequence after sequence). Sequence i already holds ``starts[i]`` tokens
    (a prefix-cache hit when > 0) and adds ``lengths[i]``.
    """
    bs = k_layer.shape[2]
    hq, n_tok, d = q.shape
    hkv = k.shape[0]
    group = hq // hkv
    blocks, offsets = write_index(tables, starts, lengths, bs)
    kv_append(k_layer, v_layer, np.swapaxes(k, 0, 1), np.swapaxes(v, 0, 1), blocks, offsets)
    out = np.zeros((hq, n_tok, d), dtype=acc)
    at = 0
    for table, a, n in zip(tables, starts, lengths):
        if n == 0:  # no query: nothing to attend (the reference packs only sequences with tokens)
            continue
        end = a + n
        rb, ro = write_index([table], [0], [end], bs)
        keys = k_layer[rb, :, ro].transpose(1, 0, 2)  # [Hkv, end, d]
        values = v_layer[rb, :, ro].transpose(1, 0, 2)
        qpos = np.arange(a, end)
        allowed = np.arange(end)[None, :] <= qpos[:, None]  # [n, end]
        for h in range(hq):
            j = h // group
            out[h, at:at + n] = _softmax_attend(q[h, at:at + n], keys[j], values[j], allowed, acc)
        at += n
    return out


def block_copy(k_pool: np.ndarray, v_pool: np.ndarray, src: Sequence[int], dst: Sequence[int]) -> None:
    """Copy whole blocks ``src[i] -> dst[i]`` in every layer of ``[L, blocks, Hkv, bs, d]`` pools.

    The reference has no copy-on-write (it never writes a shared block); this is
    the plain definition the CoW kernel is checked against.
    """
    for s, t in zip(src, dst):
        k_pool[:, t] = k_pool[:, s]
        v_pool[:, t] = v_pool[:, s]


def decode_metadata(tables: Sequence[Sequence[int]], lengths: Sequence[int], block_size: int,
                    width: int, pad_block: int) -> dict[str, np.ndarray]:
    """What a decode step derives from block tables and lengths (``engine/kv_cache.py:597-609``).

    Returns positions, the write slot of each new token (slot_mapping), the
    context length after the append, and the tables padded to ``width``
    columns with ``pad_block``.
    """
    pos = np.asarray(lengths, np.int64)
    wb = np.array([t[p // block_size] for t, p in zip(tables, pos)], np.int64)
    padded = np.full((len(tables), width), pad_block, np.int64)
    for i, t in enumerate(tables):
        m = min(len(t), width)
        padded[i, :m] = t[:m]
    return {
        "positions": pos,
        "slot_mapping": wb * block_size + pos % block_size,
        "context_lens": pos + 1,
        "block_tables": padded,
    }
