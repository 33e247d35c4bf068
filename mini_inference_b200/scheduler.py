"""The reference's continuous-batching scheduler with its decisions made in C++.

``Scheduler`` has the API and behaviour of ``engine/scheduler.py``'s ``Scheduler``
(``add``, ``has_work``, ``schedule``, ``append_token``, ``abort``, ``waiting``,
``running``, ``num_preemptions``) and works on the engine's ``Sequence`` objects, but the
step's decisions -- making room for every running sequence's next token (with preemption),
the FIFO admission under ``max_num_seqs``, the token budget and the cache, and the finish
rules -- run in ``pkv_sched_*`` (``csrc/scheduler.cpp``) directly against the native block
manager of a libpkv :class:`~mini_inference_b200.cache.PagedKVCache`: one call per step
instead of one Python -> allocator round trip per running sequence. This module then
writes the results back into the ``Sequence`` objects (slot, status, cached tokens,
preemption counts, outputs, finish reason and times), as the reference does.
"""

from __future__ import annotations

import ctypes
import enum
from collections import deque
from collections.abc import Iterable, Sequence as SequenceOf
from dataclasses import dataclass, field

import numpy as np

from ._lib import (PKV_ERR_EMPTY_PROMPT, PKV_ERR_PROMPT_TOO_LONG, PKV_SEQ_FINISHED, PKV_SEQ_RUNNING, PkvError,
                   PkvSchedStep, lib)


class SequenceStatus(enum.Enum):
    """Same values as the reference's ``SequenceStatus`` (engine/sequence.py:45-48)."""

    WAITING = "waiting"
    RUNNING = "running"
    FINISHED = "finished"


class FinishReason(str, enum.Enum):
    """Same values as the reference's ``FinishReason`` (engine/sequence.py:51-55)."""

    EOS = "eos"
    LENGTH = "length"
    MAX_MODEL_LEN = "max_model_len"
    ABORT = "abort"


@dataclass
class SchedulerOutput:
    """What to run in one engine step (engine/scheduler.py:30-39)."""

    prefills: list = field(default_factory=list)
    decodes: list = field(default_factory=list)
    # Tokens each prefill processes this step, parallel to ``prefills``: all the sequence's
    # uncached tokens, or with chunked prefill the part the step's budget allows.
    prefill_tokens: list = field(default_factory=list)

    @property
    def is_empty(self) -> bool:
        return not self.prefills and not self.decodes


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise PkvError(rc, what)


class Scheduler:
    """``engine/scheduler.py``'s ``Scheduler`` over a libpkv ``PagedKVCache``.

    ``statuses`` and ``reasons`` are the enum types written into the sequences: pass the
    reference's ``SequenceStatus`` and ``FinishReason`` when driving the reference engine's
    ``Sequence`` objects (whose ``is_finished`` compares against its own enum); the
    defaults are this module's copies with the same values.
    """

    def __init__(self, config, cache, eos_token_ids: Iterable[int] = (), statuses=SequenceStatus,
                 reasons=FinishReason) -> None:
        bm = getattr(cache, "_bm", None)
        if bm is None:
            raise TypeError("the native scheduler needs a mini_inference_b200 PagedKVCache (its block manager is C++)")
        self.config = config
        self.cache = cache
        self.eos_token_ids = set(eos_token_ids)
        self._status = statuses
        self._reason = {1: reasons.EOS, 2: reasons.LENGTH, 3: reasons.MAX_MODEL_LEN, 4: reasons.ABORT}
        eos = np.array(sorted(self.eos_token_ids), dtype=np.int64)
        h = ctypes.c_void_p()
        _check(lib.pkv_sched_create(bm._h, config.max_num_seqs, config.max_num_batched_tokens, config.max_model_len,
                                    int(config.scheduling == "static"), eos.ctypes.data if eos.size else None,
                                    int(eos.size), ctypes.byref(h)), "scheduler")
        self._h = h
        self._bm = bm  # the scheduler holds a pointer to it: keep it alive as long
        cap = max(1, config.max_num_seqs)
        self._cap = cap
        self._pre_ids = np.zeros(cap, np.int64)
        self._pre_slots = np.zeros(cap, np.int32)
        self._pre_cached = np.zeros(cap, np.int64)
        self._dec_ids = np.zeros(cap, np.int64)
        self._dec_slots = np.zeros(cap, np.int32)
        self._preempted = np.zeros(cap, np.int64)
        self._pre_new = np.zeros(cap, np.int64)
        self._dec_last = np.zeros(cap, np.int64)
        self._step = PkvSchedStep(cap, self._pre_ids.ctypes.data, self._pre_slots.ctypes.data,
                                  self._pre_cached.ctypes.data, self._dec_ids.ctypes.data,
                                  self._dec_slots.ctypes.data, self._preempted.ctypes.data, 0, 0, 0,
                                  self._pre_new.ctypes.data, self._dec_last.ctypes.data)
        self.chunked_prefill = bool(getattr(config, "chunked_prefill", False))
        if self.chunked_prefill:
            _check(lib.pkv_sched_set_chunked_prefill(self._h, 1), "chunked prefill")
        self._seqs: dict[int, object] = {}  # unfinished sequences by id
        self._i32a, self._i32b, self._i64 = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int64()

    def __del__(self) -> None:
        h = getattr(self, "_h", None)
        if h is not None and h.value and lib is not None:  # lib is gone at interpreter exit
            lib.pkv_sched_destroy(h)
            self._h = None

    # ------------------------------------------------------------ queues (engine/scheduler.py:52-53)
    def _queues(self) -> tuple[list[int], list[int]]:
        _check(lib.pkv_sched_counts(self._h, ctypes.byref(self._i32a), ctypes.byref(self._i32b),
                                    ctypes.byref(self._i64)), "scheduler counts")
        n_wait, n_run = self._i32a.value, self._i32b.value
        cap = max(n_wait, n_run, 1)
        w, r = np.zeros(cap, np.int64), np.zeros(cap, np.int64)
        _check(lib.pkv_sched_queues(self._h, w.ctypes.data, r.ctypes.data, cap), "scheduler queues")
        return w[:n_wait].tolist(), r[:n_run].tolist()

    @property
    def waiting(self) -> deque:
        return deque(self._seqs[i] for i in self._queues()[0])

    @property
    def running(self) -> list:
        return [self._seqs[i] for i in self._queues()[1]]

    @property
    def num_waiting(self) -> int:
        """``len(self.waiting)`` without building the queue."""
        _check(lib.pkv_sched_counts(self._h, ctypes.byref(self._i32a), ctypes.byref(self._i32b),
                                    ctypes.byref(self._i64)), "scheduler counts")
        return self._i32a.value

    @property
    def num_running(self) -> int:
        """``len(self.running)`` without building the list."""
        _check(lib.pkv_sched_counts(self._h, ctypes.byref(self._i32a), ctypes.byref(self._i32b),
                                    ctypes.byref(self._i64)), "scheduler counts")
        return self._i32b.value

    @property
    def num_preemptions(self) -> int:
        _check(lib.pkv_sched_counts(self._h, ctypes.byref(self._i32a), ctypes.byref(self._i32b),
                                    ctypes.byref(self._i64)), "scheduler counts")
        return self._i64.value

    # ------------------------------------------------------------ engine/scheduler.py:55-111
    def add(self, seq) -> None:
        """Queue a new request, rejecting ones that can never fit."""
        ids = np.asarray(seq.prompt_token_ids, dtype=np.int64)
        rc = lib.pkv_sched_add(self._h, seq.seq_id, ids.ctypes.data if ids.size else None, int(ids.size),
                               seq.sampling.max_tokens, int(seq.sampling.ignore_eos))
        if rc == PKV_ERR_EMPTY_PROMPT:
            raise ValueError("prompt is empty")
        if rc == PKV_ERR_PROMPT_TOO_LONG:
            raise ValueError(f"prompt has {seq.prompt_len} tokens but max_model_len is {self.config.max_model_len}; "
                             "it would leave no room to generate")
        _check(rc, "scheduler add")
        self._seqs[seq.seq_id] = seq

    def has_work(self) -> bool:
        _check(lib.pkv_sched_counts(self._h, ctypes.byref(self._i32a), ctypes.byref(self._i32b),
                                    ctypes.byref(self._i64)), "scheduler counts")
        return self._i32a.value > 0 or self._i32b.value > 0

    def schedule(self) -> SchedulerOutput:
        """Choose this step's prefills and decodes."""
        st = self._step
        _check(lib.pkv_sched_schedule(self._h, ctypes.byref(st)), "scheduler step")
        waiting = self._status.WAITING
        for i in self._preempted[:st.n_preempted].tolist():
            seq = self._seqs[i]
            seq.slot = None
            seq.status = waiting
            seq.num_preemptions += 1
        out = SchedulerOutput(decodes=[self._seqs[i] for i in self._dec_ids[:st.n_decodes].tolist()])
        running = self._status.RUNNING
        out.prefill_tokens = self._pre_new[:st.n_prefills].tolist()
        for i, slot, cached in zip(self._pre_ids[:st.n_prefills].tolist(), self._pre_slots[:st.n_prefills].tolist(),
                                   self._pre_cached[:st.n_prefills].tolist()):
            seq = self._seqs[i]
            if seq.status is not running:  # admitted now (a chunked prefill already running keeps its own)
                seq.slot = slot
                seq.num_cached_tokens = cached
                seq.status = running
            out.prefills.append(seq)
        return out

    def decode_slots(self) -> np.ndarray:
        """Slots of the last ``schedule()``'s decodes, in ``decodes`` order (int32; a view that
        the next ``schedule()`` overwrites)."""
        return self._dec_slots[:self._step.n_decodes]

    def decode_last_tokens(self) -> np.ndarray:
        """The token each of the last ``schedule()``'s decodes feeds the model: its last output,
        or its last prompt token after a chunked prefill that left only that one (int64, in
        ``decodes`` order; a view that the next ``schedule()`` overwrites)."""
        return self._dec_last[:self._step.n_decodes]

    # ------------------------------------------------------------ engine/scheduler.py:143-169
    def append_token(self, seq, token: int, now: float) -> None:
        """Record a newly sampled token and finish the sequence if it is done."""
        self.append_tokens([seq], [token], now)

    def append_tokens(self, seqs: SequenceOf, tokens: SequenceOf[int], now: float) -> int:
        """``append_token`` for a whole step's sequences in one call (same order, same effects).

        Returns how many of them finished.
        """
        n = len(seqs)
        if n == 0:
            return 0
        ids = np.fromiter((s.seq_id for s in seqs), dtype=np.int64, count=n)
        toks = np.asarray(tokens, dtype=np.int64)
        reasons = np.zeros(n, np.int32)
        _check(lib.pkv_sched_append_tokens(self._h, ids.ctypes.data, toks.ctypes.data, n, reasons.ctypes.data),
               "scheduler append")
        finished = self._status.FINISHED
        n_done = 0
        for seq, token, why in zip(seqs, toks.tolist(), reasons.tolist()):
            seq.output_token_ids.append(token)
            if seq.first_token_time is None:
                seq.first_token_time = now
            if why:
                seq.status = finished
                seq.finish_reason = self._reason[why]
                seq.finish_time = now
                seq.slot = None
                del self._seqs[seq.seq_id]
                n_done += 1
        return n_done

    def abort(self, seq, now: float) -> None:
        """Cancel a request wherever it is: drop it from the queue, or finish it and free its slot."""
        if seq.is_finished:
            return
        _check(lib.pkv_sched_abort(self._h, seq.seq_id, ctypes.byref(self._i32a)), "scheduler abort")
        if self._i32a.value == PKV_SEQ_FINISHED:
            return
        seq.status = self._status.FINISHED
        seq.finish_reason = self._reason[4]
        seq.finish_time = now
        if self._i32a.value == PKV_SEQ_RUNNING:
            seq.slot = None
        self._seqs.pop(seq.seq_id, None)
