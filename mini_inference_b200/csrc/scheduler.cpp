// Continuous-batching scheduler over the native block manager: the decisions of the
// reference's Scheduler (engine/scheduler.py:42-169), made in one call per step instead of
// one Python -> allocator round trip per running sequence.
//
// It keeps the reference's two collections: `waiting`, a FIFO of requests without a cache
// slot (preempted ones go back to its front), and `running`, the requests that own a slot,
// oldest admission first. Every step it first makes room for each running sequence's next
// token (preempting the newest on exhaustion), then admits from the front of the queue while
// max_num_seqs, the token budget and the cache allow. Requests are identified by the
// caller's sequence id; the scheduler keeps each one's tokens (prompt, then outputs) for
// the prefix lookup of its (re)admission and the finish rules of append_token.
#include <algorithm>
#include <deque>
#include <new>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "../../include/pkv.h"

namespace {

struct Request {
  std::vector<int64_t> tokens;  // prompt followed by outputs
  int64_t prompt_len = 0;
  int32_t max_tokens = 0;
  bool ignore_eos = false;
  int32_t slot = -1;
  int32_t status = PKV_SEQ_WAITING;
  int32_t num_preemptions = 0;
  int64_t num_cached_tokens = 0;
  int64_t num_outputs() const { return static_cast<int64_t>(tokens.size()) - prompt_len; }
};

}  // namespace

struct pkv_scheduler {
  pkv_block_manager* bm = nullptr;
  int32_t max_num_seqs = 0;
  int64_t max_num_batched_tokens = 0;
  int64_t max_model_len = 0;
  bool static_batching = false;
  bool chunked_prefill = false;  // split prompts across steps under the token budget (opt-in)
  std::unordered_set<int64_t> eos;
  std::unordered_map<int64_t, Request> reqs;  // unfinished requests
  std::deque<int64_t> waiting;
  std::vector<int64_t> running;
  int64_t num_preemptions = 0;

  Request& req(int64_t id) { return reqs.find(id)->second; }

  void remove_running(int64_t id) { running.erase(std::find(running.begin(), running.end(), id)); }

  int preempt(int64_t id, std::vector<int64_t>& log) {  // engine/scheduler.py:134-141
    Request& r = req(id);
    remove_running(id);
    const int rc = pkv_bm_free(bm, r.slot);
    if (rc != PKV_OK) return rc;
    r.slot = -1;
    r.status = PKV_SEQ_WAITING;
    r.num_preemptions += 1;
    waiting.push_front(id);
    num_preemptions += 1;
    log.push_back(id);
    return PKV_OK;
  }

  int make_room_for_decodes(std::vector<int64_t>& preempted) {  // engine/scheduler.py:113-132
    const std::vector<int64_t> snapshot = running;  // oldest first
    for (int64_t id : snapshot) {
      if (std::find(running.begin(), running.end(), id) == running.end()) continue;  // preempted in this loop
      Request& r = req(id);
      for (;;) {
        int32_t ok = 0;
        const int rc = pkv_bm_ensure_capacity(bm, r.slot, static_cast<int64_t>(r.tokens.size()), &ok);
        if (rc != PKV_OK) return rc;
        if (ok) break;
        const int64_t victim = running.back();
        const int prc = preempt(victim, preempted);
        if (prc != PKV_OK) return prc;
        if (victim == id) break;
      }
    }
    return PKV_OK;
  }

  int finish(int64_t id) {  // engine/scheduler.py:161-169: leave running, free the slot at once
    Request& r = req(id);
    remove_running(id);
    const int rc = pkv_bm_free(bm, r.slot);
    reqs.erase(id);
    return rc;
  }
};

extern "C" {

int pkv_sched_create(pkv_block_manager* bm, int32_t max_num_seqs, int64_t max_num_batched_tokens,
                     int64_t max_model_len, int32_t static_batching, const int64_t* eos_token_ids, int32_t n_eos,
                     pkv_scheduler** out) {
  if (!bm || !out || max_num_seqs < 0 || n_eos < 0 || (n_eos > 0 && !eos_token_ids)) return PKV_ERR_INVALID_ARGUMENT;
  pkv_scheduler* s = new (std::nothrow) pkv_scheduler();
  if (!s) return PKV_ERR_INVALID_ARGUMENT;
  s->bm = bm;
  s->max_num_seqs = max_num_seqs;
  s->max_num_batched_tokens = max_num_batched_tokens;
  s->max_model_len = max_model_len;
  s->static_batching = static_batching != 0;
  for (int32_t i = 0; i < n_eos; ++i) s->eos.insert(eos_token_ids[i]);
  *out = s;
  return PKV_OK;
}

void pkv_sched_destroy(pkv_scheduler* s) { delete s; }

int pkv_sched_add(pkv_scheduler* s, int64_t seq_id, const int64_t* prompt_ids, int64_t n, int32_t max_tokens,
                  int32_t ignore_eos) {
  if (!s || n < 0 || (n > 0 && !prompt_ids)) return PKV_ERR_INVALID_ARGUMENT;
  if (n == 0) return PKV_ERR_EMPTY_PROMPT;                          // engine/scheduler.py:57-58
  if (n >= s->max_model_len) return PKV_ERR_PROMPT_TOO_LONG;        // :59-63
  if (s->reqs.count(seq_id)) return PKV_ERR_INVALID_ARGUMENT;        // ids are unique
  Request r;
  r.tokens.assign(prompt_ids, prompt_ids + n);
  r.prompt_len = n;
  r.max_tokens = max_tokens;
  r.ignore_eos = ignore_eos != 0;
  s->reqs.emplace(seq_id, std::move(r));
  s->waiting.push_back(seq_id);
  return PKV_OK;
}

namespace {

// Chunked prefill (opt-in; the reference has none, README.md:470-473). A running sequence
// whose cache holds all its tokens but the last sampled one decodes; one that holds fewer
// is still prefilling and continues with as many of its remaining tokens as the budget
// leaves. Each step: decodes first (one token each), then the running prefills oldest
// first, then admissions from the front of the queue while the budget lasts, each taking
// what is left of it (at least one token). Preemption and the cache checks are the
// reference's (whole-sequence allocation at admission).
int schedule_chunked(pkv_scheduler* s, pkv_sched_step* out) {
  std::vector<int64_t> preempted;
  int rc = s->make_room_for_decodes(preempted);
  if (rc != PKV_OK) return rc;
  const int32_t cap = out->capacity;
  if (static_cast<int64_t>(preempted.size()) > cap) return PKV_ERR_WORKSPACE;
  for (int64_t id : preempted) out->preempted_ids[out->n_preempted++] = id;
  auto emit_prefill = [&](int64_t id, const Request& r, int64_t cached, int64_t n_new) {
    if (out->n_prefills >= cap) return PKV_ERR_WORKSPACE;
    out->prefill_slots[out->n_prefills] = r.slot;
    out->prefill_cached_tokens[out->n_prefills] = cached;
    if (out->prefill_new_tokens) out->prefill_new_tokens[out->n_prefills] = n_new;
    out->prefill_ids[out->n_prefills++] = id;
    return PKV_OK;
  };
  int64_t budget = s->max_num_batched_tokens;
  std::vector<std::pair<int64_t, int64_t>> partial;  // (id, tokens still to prefill)
  for (int64_t id : s->running) {
    const Request& r = s->req(id);
    int64_t held = 0;
    rc = pkv_bm_get_length(s->bm, r.slot, &held);
    if (rc != PKV_OK) return rc;
    const int64_t remaining = static_cast<int64_t>(r.tokens.size()) - held;
    if (remaining > 1) { partial.emplace_back(id, remaining); continue; }
    if (out->n_decodes >= cap) return PKV_ERR_WORKSPACE;
    if (out->decode_last_tokens) out->decode_last_tokens[out->n_decodes] = r.tokens.back();
    out->decode_slots[out->n_decodes] = r.slot;
    out->decode_ids[out->n_decodes++] = id;
    budget -= 1;
  }
  for (const auto& [id, remaining] : partial) {
    const int64_t chunk = std::min(remaining, budget);
    if (chunk <= 0) break;
    int64_t held = 0;
    pkv_bm_get_length(s->bm, s->req(id).slot, &held);
    if ((rc = emit_prefill(id, s->req(id), held, chunk)) != PKV_OK) return rc;
    budget -= chunk;
  }
  if (s->static_batching && !s->running.empty()) return PKV_OK;
  while (budget > 0 && !s->waiting.empty() && static_cast<int32_t>(s->running.size()) < s->max_num_seqs) {
    const int64_t id = s->waiting.front();
    Request& r = s->req(id);
    const int64_t num_tokens = static_cast<int64_t>(r.tokens.size());
    int32_t fits = 0;
    rc = pkv_bm_can_allocate(s->bm, num_tokens + 1, &fits);
    if (rc != PKV_OK) return rc;
    if (!fits) break;
    if (out->n_prefills >= cap) return PKV_ERR_WORKSPACE;
    s->waiting.pop_front();
    int32_t slot = -1;
    rc = pkv_bm_allocate(s->bm, num_tokens, r.tokens.data(), num_tokens, &slot);
    if (rc != PKV_OK) return rc;
    int64_t cached = 0;
    pkv_bm_get_length(s->bm, slot, &cached);
    r.slot = slot;
    r.num_cached_tokens = cached;
    r.status = PKV_SEQ_RUNNING;
    s->running.push_back(id);
    const int64_t chunk = std::min(num_tokens - cached, budget);
    if ((rc = emit_prefill(id, r, cached, chunk)) != PKV_OK) return rc;
    budget -= chunk;
  }
  return PKV_OK;
}

}  // namespace

int pkv_sched_set_chunked_prefill(pkv_scheduler* s, int32_t enable) {
  if (!s) return PKV_ERR_INVALID_ARGUMENT;
  s->chunked_prefill = enable != 0;
  return PKV_OK;
}

int pkv_sched_schedule(pkv_scheduler* s, pkv_sched_step* out) {  // engine/scheduler.py:68-111
  if (!s || !out) return PKV_ERR_INVALID_ARGUMENT;
  out->n_prefills = out->n_decodes = out->n_preempted = 0;
  if (s->chunked_prefill) return schedule_chunked(s, out);
  std::vector<int64_t> preempted;
  int rc = s->make_room_for_decodes(preempted);
  if (rc != PKV_OK) return rc;
  const int32_t cap = out->capacity;
  if (static_cast<int64_t>(preempted.size()) > cap) return PKV_ERR_WORKSPACE;
  for (int64_t id : preempted) out->preempted_ids[out->n_preempted++] = id;
  for (int64_t id : s->running) {
    if (out->n_decodes >= cap) return PKV_ERR_WORKSPACE;
    const Request& r = s->req(id);
    if (out->decode_last_tokens) out->decode_last_tokens[out->n_decodes] = r.tokens.back();
    out->decode_slots[out->n_decodes] = r.slot;
    out->decode_ids[out->n_decodes++] = id;
  }
  if (s->static_batching && !s->running.empty()) return PKV_OK;  // nobody joins a running static batch
  int64_t budget = s->max_num_batched_tokens - out->n_decodes;
  while (!s->waiting.empty() && static_cast<int32_t>(s->running.size()) < s->max_num_seqs) {
    const int64_t id = s->waiting.front();
    Request& r = s->req(id);
    const int64_t num_tokens = static_cast<int64_t>(r.tokens.size());  // a preempted request recomputes its outputs too
    if (num_tokens > budget && !s->static_batching) break;              // strict FIFO
    int32_t fits = 0;
    rc = pkv_bm_can_allocate(s->bm, num_tokens + 1, &fits);  // the prompt and its first decoded token
    if (rc != PKV_OK) return rc;
    if (!fits) break;
    if (out->n_prefills >= cap) return PKV_ERR_WORKSPACE;
    s->waiting.pop_front();
    int32_t slot = -1;
    rc = pkv_bm_allocate(s->bm, num_tokens, r.tokens.data(), num_tokens, &slot);
    if (rc != PKV_OK) return rc;
    int64_t cached = 0;
    pkv_bm_get_length(s->bm, slot, &cached);  // a prefix-cache hit leaves lengths[slot] > 0
    r.slot = slot;
    r.num_cached_tokens = cached;
    r.status = PKV_SEQ_RUNNING;
    s->running.push_back(id);
    out->prefill_slots[out->n_prefills] = slot;
    out->prefill_cached_tokens[out->n_prefills] = cached;
    if (out->prefill_new_tokens) out->prefill_new_tokens[out->n_prefills] = num_tokens - cached;
    out->prefill_ids[out->n_prefills++] = id;
    budget -= num_tokens - cached;
  }
  return PKV_OK;
}

int pkv_sched_append_tokens(pkv_scheduler* s, const int64_t* seq_ids, const int64_t* tokens, int32_t n,
                            int32_t* finish_reasons) {  // engine/scheduler.py:143-159, per token in order
  if (!s || n < 0 || (n > 0 && (!seq_ids || !tokens || !finish_reasons))) return PKV_ERR_INVALID_ARGUMENT;
  for (int32_t i = 0; i < n; ++i) {
    auto it = s->reqs.find(seq_ids[i]);
    if (it == s->reqs.end() || it->second.status != PKV_SEQ_RUNNING) return PKV_ERR_UNKNOWN_SLOT;
    Request& r = it->second;
    r.tokens.push_back(tokens[i]);
    int32_t reason = PKV_FINISH_NONE;
    if (s->eos.count(tokens[i]) && !r.ignore_eos) {
      reason = PKV_FINISH_EOS;
    } else if (r.num_outputs() >= r.max_tokens) {
      reason = PKV_FINISH_LENGTH;
    } else if (static_cast<int64_t>(r.tokens.size()) >= s->max_model_len) {
      reason = PKV_FINISH_MAX_MODEL_LEN;
    }
    finish_reasons[i] = reason;
    if (reason != PKV_FINISH_NONE) {
      const int rc = s->finish(seq_ids[i]);
      if (rc != PKV_OK) return rc;
    }
  }
  return PKV_OK;
}

int pkv_sched_abort(pkv_scheduler* s, int64_t seq_id, int32_t* where) {  // engine/scheduler.py:150-159
  if (!s || !where) return PKV_ERR_INVALID_ARGUMENT;
  *where = PKV_SEQ_FINISHED;
  auto it = s->reqs.find(seq_id);
  if (it == s->reqs.end()) return PKV_OK;  // finished (or never added): nothing to do
  if (it->second.status == PKV_SEQ_WAITING) {
    s->waiting.erase(std::find(s->waiting.begin(), s->waiting.end(), seq_id));
    s->reqs.erase(it);
    *where = PKV_SEQ_WAITING;
    return PKV_OK;
  }
  *where = PKV_SEQ_RUNNING;
  return s->finish(seq_id);
}

int pkv_sched_counts(const pkv_scheduler* s, int32_t* n_waiting, int32_t* n_running, int64_t* num_preemptions) {
  if (!s || !n_waiting || !n_running || !num_preemptions) return PKV_ERR_INVALID_ARGUMENT;
  *n_waiting = static_cast<int32_t>(s->waiting.size());
  *n_running = static_cast<int32_t>(s->running.size());
  *num_preemptions = s->num_preemptions;
  return PKV_OK;
}

int pkv_sched_queues(const pkv_scheduler* s, int64_t* waiting, int64_t* running, int32_t cap) {
  if (!s || (cap > 0 && (!waiting || !running))) return PKV_ERR_INVALID_ARGUMENT;
  if (static_cast<int64_t>(s->waiting.size()) > cap || static_cast<int64_t>(s->running.size()) > cap)
    return PKV_ERR_WORKSPACE;
  std::copy(s->waiting.begin(), s->waiting.end(), waiting);
  std::copy(s->running.begin(), s->running.end(), running);
  return PKV_OK;
}

}  // extern "C"
