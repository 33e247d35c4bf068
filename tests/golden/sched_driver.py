"""Seeded scheduler workloads and the step loop that records a scheduler's decisions.

Shared by ``make_golden.py`` (which runs it on the reference's ``Scheduler`` and
``PagedKVCache``) and the tests (which run it on ``oracle/scheduler.py`` and on the native
scheduler), so all three see the same requests, tokens and aborts. The step loop is
``LLMEngine.step`` (``engine/engine.py:281-312``) with the model and sampler replaced by a
deterministic token rule: after ``schedule()`` the prefills' tokens are committed to the
cache (``lengths[slot] = num_tokens``, then ``register_prefix``) and every decode adds one
token, exactly the cache effects of the engine's packed-prefill and decode contexts.
"""

from __future__ import annotations

import random


def make_workload(seed: int, n_requests: int, steps: int, vocab: int = 50, n_prefixes: int = 3,
                  prefix_len: tuple[int, int] = (20, 48), suffix_len: tuple[int, int] = (1, 40),
                  max_tokens: tuple[int, int] = (1, 40), n_aborts: int = 4) -> dict:
    """Requests with shared prompt prefixes (prefix-cache hits), arrival steps and aborts."""
    rng = random.Random(seed)
    prefixes = [[rng.randrange(2, vocab) for _ in range(rng.randint(*prefix_len))] for _ in range(n_prefixes)]
    requests = []
    for i in range(n_requests):
        prompt = list(rng.choice(prefixes)) if rng.random() < 0.7 else []
        prompt += [rng.randrange(2, vocab) for _ in range(rng.randint(*suffix_len))]
        requests.append({"id": i, "arrival": rng.randrange(0, max(1, steps // 3)), "prompt": prompt,
                         "max_tokens": rng.randint(*max_tokens), "ignore_eos": rng.random() < 0.3})
    aborts = [{"step": rng.randrange(1, steps), "id": rng.randrange(n_requests)} for _ in range(n_aborts)]
    return {"seed": seed, "vocab": vocab, "requests": requests, "aborts": aborts}


def next_token(seq_id: int, num_tokens: int, vocab: int) -> int:
    """The 'sampled' token: a fixed function of the request and its length (0 and 1 are EOS)."""
    return (seq_id * 7919 + num_tokens * 104729 + (seq_id * num_tokens) % 13) % vocab


def _reason(r) -> str | None:
    return None if r is None else getattr(r, "value", r)


def drive(scheduler, make_sequence, cache, workload: dict, steps: int) -> list[dict]:
    """Run ``steps`` engine steps; one record per step of everything the scheduler decided."""
    vocab = workload["vocab"]
    seqs = {}
    arrivals: dict[int, list[dict]] = {}
    for r in workload["requests"]:
        arrivals.setdefault(r["arrival"], []).append(r)
    aborts: dict[int, list[int]] = {}
    for a in workload["aborts"]:
        aborts.setdefault(a["step"], []).append(a["id"])
    records = []
    for step in range(steps):
        rejected, aborted = [], []
        for r in arrivals.get(step, []):
            seq = make_sequence(r["id"], list(r["prompt"]), r["max_tokens"], r["ignore_eos"])
            try:
                scheduler.add(seq)
            except ValueError as e:  # an empty prompt, or one that leaves no room to generate
                rejected.append([r["id"], str(e)])
                continue
            seqs[r["id"]] = seq
        for sid in aborts.get(step, []):
            if sid in seqs:
                was = seqs[sid].status
                scheduler.abort(seqs[sid], float(step))
                aborted.append([sid, _reason(was), _reason(seqs[sid].finish_reason)])
        out = scheduler.schedule()
        prefills = [[s.seq_id, s.slot, s.num_cached_tokens] for s in out.prefills]
        decodes = [[s.seq_id, s.slot] for s in out.decodes]
        for s in out.prefills:  # the packed-prefill context's commit, then the engine's register_prefix
            cache.lengths[s.slot] = s.num_tokens
            cache.register_prefix(s.slot, s.token_ids)
        for s in out.decodes:  # the decode context's commit
            cache.lengths[s.slot] += 1
        finished = []
        for s in list(out.prefills) + list(out.decodes):
            scheduler.append_token(s, next_token(s.seq_id, s.num_tokens, vocab), float(step))
            if s.is_finished:
                finished.append([s.seq_id, _reason(s.finish_reason)])
        records.append({
            "step": step,
            "rejected": rejected,
            "aborted": aborted,
            "prefills": prefills,
            "decodes": decodes,
            "finished": finished,
            "waiting": [s.seq_id for s in scheduler.waiting],
            "running": [[s.seq_id, s.slot] for s in scheduler.running],
            "num_preemptions": scheduler.num_preemptions,
            "num_free_blocks": cache.num_free_blocks,
            "prefix_hit_tokens": cache.prefix_hit_tokens,
        })
    return records
