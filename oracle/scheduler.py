"""Pure-Python restatement of the reference's continuous-batching scheduler.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): the checker for the native
scheduler in ``mini_inference_b200/csrc/scheduler.cpp``, and the CPU baseline it is timed
against.

Restates ``Scheduler`` in ``engine/scheduler.py`` over :class:`oracle.block_manager.OracleBlockManager`
(or any object with the reference cache's ``can_allocate`` / ``allocate`` /
``ensure_capacity`` / ``free`` / ``lengths``):

* ``add`` -- ``engine/scheduler.py:55-64``: an empty prompt, or one of ``max_model_len``
  tokens or more, is refused with ``ValueError``;
* ``schedule`` -- ``:68-111``: make room for every running sequence's next token, then
  admit from the front of the queue while ``max_num_seqs``, the token budget
  (``max_num_batched_tokens`` minus one per decode; strict FIFO) and the cache allow; a
  static batch admits only when nothing runs and ignores the budget;
* ``_make_room_for_decodes`` / ``_preempt`` -- ``:113-141``: oldest first, preempting the
  newest running sequence until the block fits, preempted sequences to the queue's front;
* ``append_token`` / ``abort`` / ``_finish`` -- ``:143-169``: EOS (unless ``ignore_eos``),
  then ``max_tokens``, then ``max_model_len``; finishing frees the slot at once.

Sequences are :class:`OracleSequence` records with the reference ``Sequence``'s fields
(``engine/sequence.py:58-100``); statuses and finish reasons are the reference's string
values.
"""

from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field

WAITING, RUNNING, FINISHED = "waiting", "running", "finished"
EOS, LENGTH, MAX_MODEL_LEN, ABORT = "eos", "length", "max_model_len", "abort"


@dataclass
class OracleSampling:
    max_tokens: int = 128
    ignore_eos: bool = False


@dataclass
class OracleSequence:
    seq_id: int
    prompt_token_ids: list[int]
    sampling: OracleSampling
    arrival_time: float = 0.0
    output_token_ids: list[int] = field(default_factory=list)
    status: str = WAITING
    slot: int | None = None
    finish_reason: str | None = None
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
    def is_finished(self) -> bool:
        return self.status == FINISHED


@dataclass
class OracleStep:
    prefills: list = field(default_factory=list)
    decodes: list = field(default_factory=list)


class OracleScheduler:
    def __init__(self, max_num_seqs: int, max_num_batched_tokens: int, max_model_len: int, cache,
                 eos_token_ids=(), static: bool = False) -> None:
        self.max_num_seqs = max_num_seqs
        self.max_num_batched_tokens = max_num_batched_tokens
        self.max_model_len = max_model_len
        self.static = static
        self.cache = cache
        self.eos_token_ids = set(eos_token_ids)
        self.waiting: deque = deque()
        self.running: list = []
        self.num_preemptions = 0

    def add(self, seq) -> None:
        if seq.prompt_len == 0:
            raise ValueError("prompt is empty")
        if seq.prompt_len >= self.max_model_len:
            raise ValueError(f"prompt has {seq.prompt_len} tokens but max_model_len is {self.max_model_len}; "
                             "it would leave no room to generate")
        self.waiting.append(seq)

    def has_work(self) -> bool:
        return bool(self.waiting or self.running)

    def schedule(self) -> OracleStep:
        self._make_room_for_decodes()
        out = OracleStep(decodes=list(self.running))
        if self.static and self.running:
            return out
        budget = self.max_num_batched_tokens - len(out.decodes)
        while self.waiting and len(self.running) < self.max_num_seqs:
            seq = self.waiting[0]
            n = seq.num_tokens
            if n > budget and not self.static:
                break
            if not self.cache.can_allocate(n + 1):
                break
            self.waiting.popleft()
            seq.slot = self.cache.allocate(n, token_ids=seq.token_ids)
            seq.num_cached_tokens = self.cache.lengths[seq.slot]
            seq.status = RUNNING
            self.running.append(seq)
            out.prefills.append(seq)
            budget -= n - seq.num_cached_tokens
        return out

    def _make_room_for_decodes(self) -> None:
        for seq in list(self.running):
            if seq not in self.running:
                continue
            while not self.cache.ensure_capacity(seq.slot, seq.num_tokens):
                victim = self.running[-1]
                self._preempt(victim)
                if victim is seq:
                    break

    def _preempt(self, seq) -> None:
        self.running.remove(seq)
        self.cache.free(seq.slot)
        seq.slot = None
        seq.status = WAITING
        seq.num_preemptions += 1
        self.waiting.appendleft(seq)
        self.num_preemptions += 1

    def append_token(self, seq, token: int, now: float) -> None:
        seq.output_token_ids.append(token)
        if seq.first_token_time is None:
            seq.first_token_time = now
        reason = None
        if token in self.eos_token_ids and not seq.sampling.ignore_eos:
            reason = EOS
        elif len(seq.output_token_ids) >= seq.sampling.max_tokens:
            reason = LENGTH
        elif seq.num_tokens >= self.max_model_len:
            reason = MAX_MODEL_LEN
        if reason is not None:
            self._finish(seq, reason, now)

    def abort(self, seq, now: float) -> None:
        if seq.is_finished:
            return
        if seq in self.waiting:
            self.waiting.remove(seq)
            seq.status = FINISHED
            seq.finish_reason = ABORT
            seq.finish_time = now
        else:
            self._finish(seq, ABORT, now)

    def _finish(self, seq, reason: str, now: float) -> None:
        seq.status = FINISHED
        seq.finish_reason = reason
        seq.finish_time = now
        self.running.remove(seq)
        self.cache.free(seq.slot)
        seq.slot = None
