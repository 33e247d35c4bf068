"""Pure-Python restatement of the reference's paged block allocator and prefix cache.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): the checker for the
native block manager in ``mini_inference_b200/csrc/block_manager.cpp``.

Restates ``PagedKVCache``'s host bookkeeping in ``engine/kv_cache.py``:

* ``blocks_for`` / ``can_allocate`` -- ``engine/kv_cache.py:459-464``
* free pool order, ``_new_block`` / ``_share`` / ``_release`` -- ``:468-488``
* prefix keys and matching, ``_chain_keys`` / ``_match_prefix`` -- ``:490-508``
* ``allocate`` -- ``:512-529``; ``register_prefix`` -- ``:531-540``
* ``ensure_capacity`` -- ``:542-551``; ``free`` -- ``:553-560``
* slot ids handed out lowest first, freed ids reused last-in first-out -- ``:431,560``

Differences in form, not in result:

* The free pool is an explicit doubly linked list over block ids instead of an
  ordered dict. The order rules are the reference's: take from the head
  (least recently freed), a released block whose key is cached goes to the
  tail, a released block without a key goes to the head, and sharing a free
  cached block unlinks it from wherever it sits.
* A block's content key nests the parent key itself, ``(parent key, its
  tokens)``, where the reference nests ``hash(parent key)``. The two agree
  except when CPython's 64-bit tuple hash collides, and that hash is not
  reproducible across processes anyway (``hash(None)`` is address-based on
  CPython 3.12). Matching is therefore the same decision on every input.
"""

from __future__ import annotations

from collections.abc import Sequence


class _FreeList:
    """Doubly linked list of block ids with O(1) push/pop at both ends and unlink."""

    def __init__(self, n: int) -> None:
        self.prev: dict[int, int] = {}
        self.next: dict[int, int] = {}
        self.head = -1
        self.tail = -1
        self.size = 0
        for b in range(n):
            self.push_back(b)

    def __contains__(self, b: int) -> bool:
        return b in self.prev

    def push_back(self, b: int) -> None:
        self.prev[b], self.next[b] = self.tail, -1
        if self.tail >= 0:
            self.next[self.tail] = b
        else:
            self.head = b
        self.tail = b
        self.size += 1

    def push_front(self, b: int) -> None:
        self.prev[b], self.next[b] = -1, self.head
        if self.head >= 0:
            self.prev[self.head] = b
        else:
            self.tail = b
        self.head = b
        self.size += 1

    def unlink(self, b: int) -> None:
        p, n = self.prev.pop(b), self.next.pop(b)
        if p >= 0:
            self.next[p] = n
        else:
            self.head = n
        if n >= 0:
            self.prev[n] = p
        else:
            self.tail = p
        self.size -= 1

    def pop_front(self) -> int:
        b = self.head
        if b < 0:
            raise RuntimeError("free block pool is empty")
        self.unlink(b)
        return b

    def order(self) -> list[int]:
        out, b = [], self.head
        while b >= 0:
            out.append(b)
            b = self.next[b]
        return out


class OracleBlockManager:
    """Host-side state of a paged KV cache: slots, block tables, refcounts, prefix keys."""

    def __init__(self, num_blocks: int, block_size: int, max_seqs: int, max_len: int,
                 enable_prefix_caching: bool = False) -> None:
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.max_seqs = max_seqs
        self.max_len = max_len
        self.scratch_block = num_blocks
        self.enable_prefix_caching = enable_prefix_caching
        self.lengths: dict[int, int] = {}
        self.block_tables: dict[int, list[int]] = {}
        # Slot ids form a stack: 0 on top at the start, and a freed id goes back on top.
        self._slot_stack = [max_seqs - 1 - i for i in range(max_seqs)]
        self._pool = _FreeList(num_blocks)
        self._refs = [0] * num_blocks
        self._key_of: dict[int, tuple] = {}  # block -> content key
        self._block_of: dict[tuple, int] = {}  # content key -> block
        self.prefix_hit_tokens = 0

    # ---------------------------------------------------------------- queries
    @property
    def num_free_slots(self) -> int:
        return len(self._slot_stack)

    @property
    def num_free_blocks(self) -> int:
        return self._pool.size

    def free_block_order(self) -> list[int]:
        return self._pool.order()

    def ref_counts(self) -> list[int]:
        return list(self._refs)

    def blocks_for(self, num_tokens: int) -> int:
        bs = self.block_size
        return (num_tokens + bs - 1) // bs

    def can_allocate(self, num_tokens: int) -> bool:
        return (len(self._slot_stack) > 0 and num_tokens <= self.max_len
                and self.blocks_for(num_tokens) <= self._pool.size)

    # ---------------------------------------------------------------- blocks
    def _take_fresh(self) -> int:
        b = self._pool.pop_front()
        key = self._key_of.pop(b, None)
        if key is not None:
            del self._block_of[key]
        self._refs[b] = 1
        return b

    def _add_ref(self, b: int) -> None:
        if self._refs[b] == 0:
            self._pool.unlink(b)
        self._refs[b] += 1

    def _drop_ref(self, b: int) -> None:
        self._refs[b] -= 1
        if self._refs[b] == 0:
            if b in self._key_of:
                self._pool.push_back(b)
            else:
                self._pool.push_front(b)

    def _prefix_keys(self, token_ids: Sequence[int], count: int):
        """Keys of the first ``count`` blocks: key_i = (key_{i-1}, tokens of block i), key_{-1} = None."""
        bs = self.block_size
        key = None
        for i in range(count):
            key = (key, tuple(token_ids[i * bs : (i + 1) * bs]))
            yield key

    def _matched_blocks(self, token_ids: Sequence[int]) -> list[int]:
        usable = (len(token_ids) - 1) // self.block_size  # at least one token is always recomputed
        found = []
        for key in self._prefix_keys(token_ids, max(usable, 0)):
            b = self._block_of.get(key)
            if b is None:
                break
            found.append(b)
        return found

    # ---------------------------------------------------------------- sequences
    def allocate(self, num_tokens: int = 0, token_ids: Sequence[int] | None = None) -> int:
        if not self.can_allocate(num_tokens):
            raise RuntimeError("not enough free KV cache blocks")
        shared = self._matched_blocks(token_ids) if (self.enable_prefix_caching and token_ids) else []
        for b in shared:
            self._add_ref(b)
        slot = self._slot_stack.pop()
        fresh = [self._take_fresh() for _ in range(max(0, self.blocks_for(num_tokens) - len(shared)))]
        self.block_tables[slot] = shared + fresh
        self.lengths[slot] = len(shared) * self.block_size
        self.prefix_hit_tokens += self.lengths[slot]
        return slot

    def register_prefix(self, slot: int, token_ids: Sequence[int]) -> None:
        if not self.enable_prefix_caching:
            return
        table = self.block_tables[slot]
        full = self.lengths[slot] // self.block_size
        for i, key in enumerate(self._prefix_keys(token_ids, full)):
            if key not in self._block_of and table[i] not in self._key_of:
                self._block_of[key] = table[i]
                self._key_of[table[i]] = key

    def ensure_capacity(self, slot: int, num_tokens: int) -> bool:
        if num_tokens > self.max_len:
            return False
        table = self.block_tables[slot]
        missing = self.blocks_for(num_tokens) - len(table)
        if missing > self._pool.size:
            return False
        for _ in range(missing):
            table.append(self._take_fresh())
        return True

    def free(self, slot: int) -> None:
        if slot not in self.block_tables:
            raise RuntimeError(f"slot {slot} freed twice")
        table = self.block_tables.pop(slot)
        for b in table[::-1]:
            self._drop_ref(b)
        del self.lengths[slot]
        self._slot_stack.append(slot)

    # ---------------------------------------------------------------- snapshots
    def state(self) -> dict:
        """Everything a caller can observe, in a JSON-friendly form."""
        return {
            "block_tables": {str(s): list(t) for s, t in sorted(self.block_tables.items())},
            "lengths": {str(s): n for s, n in sorted(self.lengths.items())},
            "free_blocks": self.free_block_order(),
            "num_free_slots": self.num_free_slots,
            "prefix_hit_tokens": self.prefix_hit_tokens,
            "ref_counts": self.ref_counts(),
            "cached_blocks": sorted(self._key_of),
        }
