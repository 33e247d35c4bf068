"""Drop-in paged KV cache for mini-inference, backed by libpkv (C++ allocator + sm_100a kernels).

Mirrors the reference's ``engine/kv_cache.py`` interface for the paged path:

* :class:`PagedKVCache` -- same constructor, ``for_model``, allocator methods
  (``allocate``, ``ensure_capacity``, ``free``, ``register_prefix``,
  ``can_allocate``, ``blocks_for``), properties (``num_free_slots``,
  ``num_free_blocks``) and public attributes (``k``, ``v``, ``lengths``,
  ``block_tables``, ``block_size``, ``max_len``, ``num_blocks``,
  ``scratch_block``, ``prefix_hit_tokens``, ``enable_prefix_caching``) as
  ``engine/kv_cache.py:377-579``. Errors are the reference's: ``RuntimeError``
  when the pool is out of blocks (``:520``) or a slot is freed twice (``:556``),
  ``ValueError`` when a sequence has no block for its next token (``:600``) or a
  packed prefill has no room (``:259``), ``KeyError`` for an unknown slot.
* :class:`PagedDecodeContext` / :class:`PackedPrefillContext` -- the
  ``AttentionContext`` objects ``Attention.forward`` calls
  (``engine/model.py:89-98,250``) with ``attend(layer_idx, q, k, v)`` and
  ``commit()``, plus ``positions`` / ``last_index`` as the runner reads them
  (``engine/engine.py:102-106,119-123``).

The block bookkeeping runs in C++ (``csrc/block_manager.cpp``) with the
reference's exact decisions. Block tables are also kept on the GPU as a
mirror indexed by slot, updated from a journal of the allocator's edits, so a
step sends only its slot ids and positions to the device. Attention and the
KV append are sm_100a kernels; there is no CPU path: a cache on a CPU device
supports the allocator only, and its contexts raise.
"""

from __future__ import annotations

import ctypes
from collections.abc import Iterator, Mapping, MutableMapping, Sequence

import numpy as np
import torch

from . import ops
from ._lib import (PKV_ERR_DOUBLE_FREE, PKV_ERR_NO_BLOCKS, PKV_ERR_OUT_OF_RANGE, PKV_ERR_UNKNOWN_SLOT, PkvError,
                   check, lib)


class NativeBlockManager:
    """Thin owner of a ``pkv_block_manager`` (engine/kv_cache.py:411-560 in C++)."""

    def __init__(self, num_blocks: int, block_size: int, max_seqs: int, max_len: int,
                 enable_prefix_caching: bool = False) -> None:
        h = ctypes.c_void_p()
        check(lib.pkv_bm_create(num_blocks, block_size, max_seqs, max_len, int(enable_prefix_caching),
                                ctypes.byref(h)), "block manager")
        self._h = h
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.max_seqs = max_seqs
        self.max_len = max_len
        self._i32 = ctypes.c_int32()
        self._i64 = ctypes.c_int64()

    def __del__(self) -> None:
        h = getattr(self, "_h", None)
        if h is not None and h.value and lib is not None:  # lib is gone at interpreter exit
            lib.pkv_bm_destroy(h)
            self._h = None

    @staticmethod
    def _ids(token_ids: Sequence[int] | None) -> tuple[np.ndarray | None, int]:
        if token_ids is None:
            return None, 0
        arr = np.ascontiguousarray(np.asarray(token_ids, dtype=np.int64).reshape(-1))
        return arr, arr.size

    # ------------------------------------------------------------ allocator
    def can_allocate(self, num_tokens: int) -> bool:
        check(lib.pkv_bm_can_allocate(self._h, num_tokens, ctypes.byref(self._i32)), "can_allocate")
        return bool(self._i32.value)

    def allocate(self, num_tokens: int = 0, token_ids: Sequence[int] | None = None) -> int:
        arr, n = self._ids(token_ids)
        st = lib.pkv_bm_allocate(self._h, num_tokens, arr.ctypes.data if arr is not None and n else None, n,
                                 ctypes.byref(self._i32))
        if st == PKV_ERR_NO_BLOCKS:
            raise RuntimeError("not enough free KV cache blocks")
        check(st, "allocate")
        return self._i32.value

    def register_prefix(self, slot: int, token_ids: Sequence[int]) -> None:
        arr, n = self._ids(token_ids)
        st = lib.pkv_bm_register_prefix(self._h, slot, arr.ctypes.data if n else None, n)
        if st == PKV_ERR_UNKNOWN_SLOT:
            raise KeyError(slot)
        if st == PKV_ERR_OUT_OF_RANGE:
            raise IndexError("list index out of range")
        check(st, "register_prefix")

    def ensure_capacity(self, slot: int, num_tokens: int) -> bool:
        st = lib.pkv_bm_ensure_capacity(self._h, slot, num_tokens, ctypes.byref(self._i32))
        if st == PKV_ERR_UNKNOWN_SLOT:
            raise KeyError(slot)
        check(st, "ensure_capacity")
        return bool(self._i32.value)

    def free(self, slot: int) -> None:
        st = lib.pkv_bm_free(self._h, slot)
        if st == PKV_ERR_DOUBLE_FREE:
            raise RuntimeError(f"slot {slot} freed twice")
        check(st, "free")

    # ------------------------------------------------------------ state
    def get_length(self, slot: int) -> int:
        st = lib.pkv_bm_get_length(self._h, slot, ctypes.byref(self._i64))
        if st == PKV_ERR_UNKNOWN_SLOT:
            raise KeyError(slot)
        check(st, "lengths")
        return self._i64.value

    def set_length(self, slot: int, value: int) -> None:
        st = lib.pkv_bm_set_length(self._h, slot, int(value))
        if st == PKV_ERR_UNKNOWN_SLOT:
            raise KeyError(slot)
        check(st, "lengths")

    def table(self, slot: int) -> list[int]:
        cap = self.blocks_for(self.max_len) + 2
        buf = (ctypes.c_int32 * cap)()
        st = lib.pkv_bm_get_table(self._h, slot, buf, cap, ctypes.byref(self._i32))
        if st == PKV_ERR_UNKNOWN_SLOT:
            raise KeyError(slot)
        check(st, "block_tables")
        n = self._i32.value
        if n > cap:
            buf = (ctypes.c_int32 * n)()
            check(lib.pkv_bm_get_table(self._h, slot, buf, n, ctypes.byref(self._i32)), "block_tables")
        return list(buf[:n])

    def live_slots(self) -> list[int]:
        buf = (ctypes.c_int32 * max(self.max_seqs, 1))()
        check(lib.pkv_bm_live_slots(self._h, buf, self.max_seqs, ctypes.byref(self._i32)), "live slots")
        return list(buf[: self._i32.value])

    def decode_positions(self, slots: np.ndarray) -> np.ndarray:
        out = np.empty(len(slots), np.int32)
        st = lib.pkv_bm_decode_positions(self._h, slots.ctypes.data, len(slots), out.ctypes.data)
        if st == PKV_ERR_OUT_OF_RANGE:
            raise ValueError("a sequence has no block for its next token (call ensure_capacity first)")
        if st == PKV_ERR_UNKNOWN_SLOT:
            raise KeyError("slot without a block table")
        check(st, "decode positions")
        return out

    def fork(self, slot: int) -> int:
        st = lib.pkv_bm_fork(self._h, slot, ctypes.byref(self._i32))
        if st == PKV_ERR_UNKNOWN_SLOT:
            raise KeyError(slot)
        if st == PKV_ERR_NO_BLOCKS:
            raise RuntimeError("no free slot to fork into")
        check(st, "fork")
        return self._i32.value

    def prepare_write(self, slot: int, first_pos: int, n_tokens: int) -> list[tuple[int, int]]:
        """(old, fresh) block pairs to copy before tokens first_pos.. of slot are written (shared blocks only)."""
        cap = self.blocks_for(n_tokens) + 1
        buf = (ctypes.c_int32 * (2 * cap))()
        st = lib.pkv_bm_prepare_write(self._h, slot, first_pos, n_tokens, buf, cap, ctypes.byref(self._i32))
        if st == PKV_ERR_NO_BLOCKS:
            raise RuntimeError("not enough free KV cache blocks")
        if st == PKV_ERR_UNKNOWN_SLOT:
            raise KeyError(slot)
        check(st, "prepare_write")
        return [(buf[2 * i], buf[2 * i + 1]) for i in range(self._i32.value)]

    def commit_decode(self, slots: np.ndarray) -> None:
        check(lib.pkv_bm_commit_decode(self._h, slots.ctypes.data, len(slots)), "commit")

    @property
    def num_free_blocks(self) -> int:
        check(lib.pkv_bm_num_free_blocks(self._h, ctypes.byref(self._i32)), "num_free_blocks")
        return self._i32.value

    @property
    def num_free_slots(self) -> int:
        check(lib.pkv_bm_num_free_slots(self._h, ctypes.byref(self._i32)), "num_free_slots")
        return self._i32.value

    @property
    def prefix_hit_tokens(self) -> int:
        check(lib.pkv_bm_prefix_hit_tokens(self._h, ctypes.byref(self._i64)), "prefix_hit_tokens")
        return self._i64.value

    def free_block_order(self) -> list[int]:
        buf = (ctypes.c_int32 * max(self.num_blocks, 1))()
        check(lib.pkv_bm_free_order(self._h, buf, self.num_blocks, ctypes.byref(self._i32)), "free order")
        return list(buf[: self._i32.value])

    def ref_counts(self) -> list[int]:
        buf = (ctypes.c_int32 * max(self.num_blocks, 1))()
        check(lib.pkv_bm_ref_counts(self._h, buf, self.num_blocks), "ref counts")
        return list(buf[: self.num_blocks])

    def cached_blocks(self) -> list[int]:
        buf = (ctypes.c_int32 * max(self.num_blocks, 1))()
        check(lib.pkv_bm_cached_blocks(self._h, buf, self.num_blocks, ctypes.byref(self._i32)), "cached blocks")
        return list(buf[: self._i32.value])

    def blocks_for(self, num_tokens: int) -> int:
        return -(-num_tokens // self.block_size)

    def set_journal(self, on: bool) -> None:
        check(lib.pkv_bm_set_journal(self._h, int(on)), "journal")

    def drain_edits(self, buf: np.ndarray) -> tuple[int, bool]:
        """Copy pending (slot, column, block) edits into ``buf`` ([cap, 3] int32); returns (count, overflowed)."""
        ovf = ctypes.c_int32()
        check(lib.pkv_bm_drain_table_edits(self._h, buf.ctypes.data, buf.shape[0], ctypes.byref(self._i32),
                                           ctypes.byref(ovf)), "drain table edits")
        return self._i32.value, bool(ovf.value)

    def state(self) -> dict:
        """Everything a caller can observe, in the same form as the oracle's ``state()``."""
        slots = self.live_slots()
        return {
            "block_tables": {str(s): self.table(s) for s in slots},
            "lengths": {str(s): self.get_length(s) for s in slots},
            "free_blocks": self.free_block_order(),
            "num_free_slots": self.num_free_slots,
            "prefix_hit_tokens": self.prefix_hit_tokens,
            "ref_counts": self.ref_counts(),
            "cached_blocks": self.cached_blocks(),
        }


class _LengthsView(MutableMapping):
    """``cache.lengths``: slot -> tokens stored, read and written through to the native manager."""

    def __init__(self, bm: NativeBlockManager) -> None:
        self._bm = bm

    def __getitem__(self, slot: int) -> int:
        return self._bm.get_length(slot)

    def __setitem__(self, slot: int, value: int) -> None:
        self._bm.set_length(slot, value)

    def __delitem__(self, slot: int) -> None:
        raise TypeError("lengths entries are removed by free()")

    def __iter__(self) -> Iterator[int]:
        return iter(self._bm.live_slots())

    def __len__(self) -> int:
        return len(self._bm.live_slots())

    def __contains__(self, slot: object) -> bool:
        return isinstance(slot, int) and slot in self._bm.live_slots()


class _TablesView(Mapping):
    """``cache.block_tables``: slot -> list of block ids (a fresh list per access)."""

    def __init__(self, bm: NativeBlockManager) -> None:
        self._bm = bm

    def __getitem__(self, slot: int) -> list[int]:
        return self._bm.table(slot)

    def __iter__(self) -> Iterator[int]:
        return iter(self._bm.live_slots())

    def __len__(self) -> int:
        return len(self._bm.live_slots())

    def __contains__(self, slot: object) -> bool:
        return isinstance(slot, int) and slot in self._bm.live_slots()


class PagedKVCache:
    """A KV cache of fixed-size blocks, the reference's ``PagedKVCache`` on libpkv.

    Memory layout is the reference's: ``k, v: [num_layers, num_blocks + 1,
    num_kv_heads, block_size, head_dim]``, block ``num_blocks`` being the scratch
    block that CUDA-graph padding rows write to.
    """

    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int, num_blocks: int, block_size: int,
                 max_seqs: int, max_len: int, dtype: torch.dtype, device: torch.device | str,
                 enable_prefix_caching: bool = False, enable_copy_on_write: bool = False) -> None:
        shape = (num_layers, num_blocks + 1, num_kv_heads, block_size, head_dim)
        self.k = torch.zeros(shape, dtype=dtype, device=device)
        self.v = torch.zeros(shape, dtype=dtype, device=device)
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.num_blocks = num_blocks
        self.scratch_block = num_blocks
        self.block_size = block_size
        self.max_seqs = max_seqs
        self.max_len = max_len
        self.enable_prefix_caching = enable_prefix_caching
        # Copy-on-write of shared partially filled blocks (fork). Off by default: the
        # reference never writes a shared block, and with it off every allocator decision
        # is the reference's.
        self.enable_copy_on_write = enable_copy_on_write
        self._bm = NativeBlockManager(num_blocks, block_size, max_seqs, max_len, enable_prefix_caching)
        self.lengths = _LengthsView(self._bm)
        self.block_tables = _TablesView(self._bm)
        self.device = self.k.device
        self.on_gpu = self.k.is_cuda
        if self.on_gpu:
            self.max_blocks_per_seq = max(1, self._bm.blocks_for(max_len))
            # Device mirror of the block tables, one row per slot, plus the status word
            # the kernels write index errors to.
            self.tables_dev = torch.full((max_seqs, self.max_blocks_per_seq), -1, dtype=torch.int32,
                                         device=self.device)
            self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
            self.pool = ops.make_pool(self.k, self.v)
            # The allocator's table edits are drained straight into pinned memory and sent
            # with one copy per sync; the buffer is refilled only after that copy ran.
            cap = max(1024, 2 * num_blocks)
            self._edits_host = torch.zeros((cap, 3), dtype=torch.int32).pin_memory()
            self._edits = self._edits_host.numpy()
            self._edits_dev = torch.empty((cap, 3), dtype=torch.int32, device=self.device)
            self._edits_sent = torch.cuda.Event()
            self._bm.set_journal(True)
            self._workspaces: dict[tuple[int, int], torch.Tensor] = {}

    @classmethod
    def for_model(cls, cfg, num_blocks: int, block_size: int, max_seqs: int, max_len: int, dtype: torch.dtype,
                  device: torch.device | str, enable_prefix_caching: bool = False) -> "PagedKVCache":
        return cls(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, num_blocks, block_size, max_seqs, max_len,
                   dtype, device, enable_prefix_caching)

    # ------------------------------------------------------------ allocator API (engine/kv_cache.py:455-560)
    @property
    def num_free_slots(self) -> int:
        return self._bm.num_free_slots

    @property
    def num_free_blocks(self) -> int:
        return self._bm.num_free_blocks

    @property
    def prefix_hit_tokens(self) -> int:
        return self._bm.prefix_hit_tokens

    def blocks_for(self, num_tokens: int) -> int:
        return -(-num_tokens // self.block_size)

    def can_allocate(self, num_tokens: int) -> bool:
        return self._bm.can_allocate(num_tokens)

    def allocate(self, num_tokens: int = 0, token_ids: Sequence[int] | None = None) -> int:
        return self._bm.allocate(num_tokens, token_ids)

    def register_prefix(self, slot: int, token_ids: Sequence[int]) -> None:
        self._bm.register_prefix(slot, token_ids)

    def ensure_capacity(self, slot: int, num_tokens: int) -> bool:
        return self._bm.ensure_capacity(slot, num_tokens)

    def free(self, slot: int) -> None:
        self._bm.free(slot)

    def fork(self, slot: int) -> int:
        """A new sequence sharing all of ``slot``'s blocks and length (copy-on-write on its first write).

        No counterpart in the reference. Needs ``enable_copy_on_write``: whichever of the two
        sequences first writes into a block they share (the partially filled last block, on
        the next token) gets a private copy of it, made on the device before the write.
        """
        if not self.enable_copy_on_write:
            raise RuntimeError("fork needs a cache built with enable_copy_on_write=True")
        return self._bm.fork(slot)

    def copy_on_write(self, writes: Sequence[tuple[int, int, int]]) -> int:
        """Give every (slot, first position, tokens) about to be written its own copy of any shared block.

        Launches one ``pkv_copy_blocks`` (every layer, K and V) for all the copies, on the
        current stream, ahead of the writes; the table mirror is updated by the next
        :meth:`sync_tables`. Returns the number of blocks copied.
        """
        if not self.enable_copy_on_write:
            return 0
        pairs = [pr for slot, a, n in writes for pr in self._bm.prepare_write(slot, a, n)]
        if pairs and self.on_gpu:
            dev = torch.from_numpy(np.asarray(pairs, np.int32).T.copy()).pin_memory().to(self.device, non_blocking=True)
            ops.copy_blocks(self.pool, dev[0], dev[1], self.status)
        return len(pairs)

    def write_index(self, slots: Sequence[int], starts: Sequence[int], counts: Sequence[int]
                    ) -> tuple[torch.Tensor, torch.Tensor]:
        """Where tokens ``start..start+count-1`` of each sequence live: ``(block, offset)`` (engine/kv_cache.py:562-573)."""
        bs = self.block_size
        blocks, offsets = [], []
        for slot, a, n in zip(slots, starts, counts):
            table = self._bm.table(slot)
            pos = range(a, a + n)
            blocks.extend(table[p // bs] for p in pos)
            offsets.extend(p % bs for p in pos)
        return (torch.tensor(blocks, dtype=torch.int64, device=self.device),
                torch.tensor(offsets, dtype=torch.int64, device=self.device))

    # ------------------------------------------------------------ device mirror
    def sync_tables(self) -> None:
        """Push the allocator's table edits since the last sync to the device mirror."""
        if not self.on_gpu:
            return
        self._edits_sent.synchronize()
        n, overflow = self._bm.drain_edits(self._edits)
        if overflow:
            self._rebuild_mirror()
            return
        if n:
            upd = self._edits_dev[:n]
            upd.copy_(self._edits_host[:n], non_blocking=True)
            self._edits_sent.record()
            ops.update_tables(self.tables_dev, upd, self.status)

    def drain_table_edits(self, buf: np.ndarray) -> int:
        """Move the allocator's pending table edits into ``buf`` (int32 ``[cap, 3]``); returns how many.

        The caller applies them to ``tables_dev`` (``ops.update_tables``) before its next
        kernel reads the tables. If more were pending than ``buf`` holds, the device mirror
        is rebuilt from the allocator here instead and 0 is returned.
        """
        n, overflow = self._bm.drain_edits(buf)
        if overflow:
            self._rebuild_mirror()
            return 0
        return n

    def _rebuild_mirror(self) -> None:
        rows = torch.full((self.max_seqs, self.max_blocks_per_seq), -1, dtype=torch.int32)
        for s in self._bm.live_slots():
            t = self._bm.table(s)
            rows[s, : len(t)] = torch.tensor(t, dtype=torch.int32)
        self.tables_dev.copy_(rows.pin_memory(), non_blocking=True)

    def workspace(self, batch: int, num_q_heads: int) -> torch.Tensor:
        """Split-K workspace for decode batches up to ``batch`` rows (zeroed once, reused)."""
        key = (batch, num_q_heads)
        ws = self._workspaces.get(key)
        if ws is None:
            nbytes = ops.decode_workspace_bytes(batch, self.num_kv_heads, self.max_blocks_per_seq, self.block_size,
                                                self.head_dim, num_q_heads)
            ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=self.device)
            self._workspaces[key] = ws
        return ws

    def raise_device_errors(self) -> None:
        """Synchronise and raise any error a kernel recorded for this cache.

        After an error the decode workspaces' ticket counters are zeroed before the
        exception propagates: a call that gave up part-way must not leave a ticket that
        makes a later call merge the wrong chunks.
        """
        if not self.on_gpu:
            return
        try:
            ops.raise_device_errors(self.status)
        except (RuntimeError, IndexError):
            for ws in self._workspaces.values():
                ops.decode_reset_workspace(ws)
            raise

    # ------------------------------------------------------------ contexts
    def _require_gpu(self) -> None:
        if not self.on_gpu:
            raise RuntimeError("PagedKVCache attention runs on the sm_100a kernels only: put the cache on a CUDA device")

    def packed_prefill_context(self, slots: Sequence[int], lengths: Sequence[int]) -> "PackedPrefillContext":
        return PackedPrefillContext(self, slots, lengths)

    def decode_context(self, slots: Sequence[int]) -> "PagedDecodeContext":
        return PagedDecodeContext(self, slots)


class PagedDecodeContext:
    """A batched decode step on the paged cache (engine/kv_cache.py:582-624).

    ``positions`` (int64 [B], on the device) is where each new token goes and
    what RoPE uses. ``attend`` runs the fused append + split-K paged attention
    kernel; nothing is gathered or padded.
    """

    def __init__(self, cache: PagedKVCache, slots: Sequence[int]) -> None:
        cache._require_gpu()
        self.cache = cache
        self.slots = list(slots)
        self._slots_np = np.asarray(self.slots, dtype=np.int32)
        pos = cache._bm.decode_positions(self._slots_np)  # raises the reference's ValueError
        if cache.enable_copy_on_write:
            cache.copy_on_write([(s, int(p), 1) for s, p in zip(self.slots, pos)])
        cache.sync_tables()
        batch = len(self.slots)
        dev = cache.device
        staged = torch.from_numpy(np.stack([self._slots_np, pos])).pin_memory().to(dev, non_blocking=True)
        self.seq_rows = staged[0]
        self.lengths_in = staged[1]
        self.positions = torch.empty(batch, dtype=torch.int64, device=dev)
        self.slot_mapping = torch.empty(batch, dtype=torch.int64, device=dev)
        self.context_lens = torch.empty(batch, dtype=torch.int32, device=dev)
        self.tables = ops.make_tables(cache.tables_dev, self.seq_rows)
        ops.build_decode_metadata(self.tables, self.lengths_in, cache.block_size, cache.scratch_block,
                                  self.positions, self.slot_mapping, self.context_lens, cache.status)
        self._attends = 0

    @property
    def write_blocks(self) -> torch.Tensor:
        return self.slot_mapping // self.cache.block_size

    @property
    def write_offsets(self) -> torch.Tensor:
        return self.slot_mapping % self.cache.block_size

    def attend(self, layer_idx: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        """q ``[B, Hq, 1, d]``, k / v ``[B, Hkv, 1, d]`` -> ``[B, Hq, 1, d]``."""
        batch, hq, _, d = q.shape
        if q.dtype != self.cache.k.dtype:
            raise TypeError(f"q is {q.dtype} but the cache holds {self.cache.k.dtype}")
        ws = self.cache.workspace(self.cache.max_seqs, hq)
        out = torch.empty(batch, 1, hq, d, dtype=q.dtype, device=q.device)
        # The metadata was built when this context was made; once one attend of this step has
        # run, it is complete before whatever kernel precedes the next one, so the kernel may
        # start its block lookups early (PKV_DECODE_INPUTS_READY).
        ops.decode_attention(self.cache.pool, layer_idx, self.tables, q[:, :, 0], self.context_lens, ws,
                             k_new=k[:, :, 0], v_new=v[:, :, 0], slot_mapping=self.slot_mapping,
                             out=out[:, 0], status=self.cache.status, inputs_ready=self._attends > 0)
        self._attends += 1
        return out.transpose(1, 2)

    def attend_qkv(self, layer_idx: int, qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                   num_q_heads: int) -> torch.Tensor:
        """The ``qkv_proj`` output ``[B, 1, (Hq + 2 Hkv) d]`` -> ``[B, Hq, 1, d]``, RoPE included.

        Replaces the split, head views and ``apply_rope`` of Attention.forward
        (engine/model.py:241-250) plus :meth:`attend` with one kernel
        (``pkv_decode_attention_rope``): q and k are rotated (bit-identical to the
        reference's) on the full ``cos`` / ``sin`` tables of ``ops.rope_tables`` while the
        step's append and paged attention run.
        """
        batch = qkv.shape[0]
        rows = qkv.reshape(batch, -1)
        ws = self.cache.workspace(self.cache.max_seqs, num_q_heads)
        out = torch.empty(batch, 1, num_q_heads, self.cache.head_dim, dtype=qkv.dtype, device=qkv.device)
        ops.decode_attention_rope(self.cache.pool, layer_idx, self.tables, rows, cos, sin, self.context_lens, ws,
                                  self.slot_mapping, out=out[:, 0], status=self.cache.status,
                                  inputs_ready=self._attends > 0)
        self._attends += 1
        return out.transpose(1, 2)

    def commit(self) -> None:
        self.cache._bm.commit_decode(self._slots_np)


class PackedPrefillContext:
    """Prefill of several prompts packed end to end, prefix hits included (engine/kv_cache.py:218-301).

    Each new token's K/V is appended through a slot_mapping built on the GPU,
    then the varlen paged attention kernel reads each sequence's keys
    ``0..position`` in place.
    """

    def __init__(self, cache: PagedKVCache, slots: Sequence[int], lengths: Sequence[int]) -> None:
        cache._require_gpu()
        self.cache = cache
        self.slots = list(slots)
        self.lengths = list(lengths)
        self.starts = [cache.lengths[s] for s in self.slots]
        for s, start, n in zip(self.slots, self.starts, self.lengths):
            if not cache.ensure_capacity(s, start + n):
                raise ValueError(f"no room in the KV cache for {start + n} tokens")
        cache.copy_on_write(list(zip(self.slots, self.starts, self.lengths)))
        cache.sync_tables()
        dev = cache.device
        cu = np.zeros(len(self.slots) + 1, np.int32)
        np.cumsum(self.lengths, out=cu[1:])
        self.total = int(cu[-1])
        self.max_new = max(self.lengths) if self.lengths else 0
        host = np.concatenate([np.asarray(self.slots, np.int32), np.asarray(self.starts, np.int32), cu])
        staged = torch.from_numpy(host).pin_memory().to(dev, non_blocking=True)
        b = len(self.slots)
        self.seq_rows, self.starts_dev, self.cu_seqlens = staged[:b], staged[b:2 * b], staged[2 * b:]
        self.tables = ops.make_tables(cache.tables_dev, self.seq_rows)
        self.positions = torch.empty(self.total, dtype=torch.int64, device=dev)
        self.slot_mapping = torch.empty(self.total, dtype=torch.int64, device=dev)
        ops.build_prefill_metadata(self.tables, self.cu_seqlens, self.starts_dev, cache.block_size, self.total,
                                   self.positions, self.slot_mapping, cache.status)
        self.has_prefix = any(self.starts)
        self.last_index = self.cu_seqlens[1:].to(torch.int64) - 1

    def attend(self, layer_idx: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        """q ``[1, Hq, N, d]``, k / v ``[1, Hkv, N, d]`` -> ``[1, Hq, N, d]``."""
        _, hq, n, d = q.shape
        if q.dtype != self.cache.k.dtype:
            raise TypeError(f"q is {q.dtype} but the cache holds {self.cache.k.dtype}")
        ops.kv_append(self.cache.pool, layer_idx, k[0].transpose(0, 1), v[0].transpose(0, 1), self.slot_mapping,
                      self.cache.status)
        out = torch.empty(n, hq, d, dtype=q.dtype, device=q.device)
        ops.prefill_attention(self.cache.pool, layer_idx, self.tables, q[0].transpose(0, 1), self.cu_seqlens,
                              self.starts_dev, self.max_new, out=out, status=self.cache.status)
        return out.unsqueeze(0).transpose(1, 2)

    def attend_qkv(self, layer_idx: int, qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                   num_q_heads: int) -> torch.Tensor:
        """The ``qkv_proj`` output ``[1, N, (Hq + 2 Hkv) d]`` -> ``[1, Hq, N, d]``, RoPE included.

        ``pkv_rope_append`` rotates q and k (bit-identical to the reference's
        ``apply_rope``, engine/model.py:214-224) and writes the rotated keys and the
        values to their slots in one pass, replacing :meth:`attend`'s separate append;
        then the varlen paged kernel reads every sequence's keys in place.
        """
        rows = qkv.reshape(-1, qkv.shape[-1])
        d = self.cache.head_dim
        q_rot, _ = ops.rope_append(self.cache.pool, layer_idx, rows, self.positions, cos, sin, num_q_heads,
                                   slot_mapping=self.slot_mapping, status=self.cache.status)
        out = torch.empty(rows.shape[0], num_q_heads, d, dtype=qkv.dtype, device=qkv.device)
        ops.prefill_attention(self.cache.pool, layer_idx, self.tables, q_rot, self.cu_seqlens, self.starts_dev,
                              self.max_new, out=out, status=self.cache.status)
        return out.unsqueeze(0).transpose(1, 2)

    def commit(self) -> None:
        for slot, start, n in zip(self.slots, self.starts, self.lengths):
            self.cache.lengths[slot] = start + n
