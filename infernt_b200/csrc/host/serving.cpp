// serving.cpp — continuous batching over a paged batched engine.
//
// The reference serves one sequence per engine: InferenceEngine::generate
// (src/engine.cpp:106-170) feeds the prompt one token per forward, then
// decodes until max_new_tokens, with one KVCache [N_kv, max_seq, D] per layer
// (include/kv_cache.h:7-15).  Paged KV and continuous batching are listed as
// future work in its README; this file adds them on top of the batched
// engine (batch_engine.cpp).
//
// Scheduler (host only): `slots` sequence slots, a pool of pages of
// page_size positions (a free list), requests queued first-come
// first-served.  Each plan():
//   1. running requests, oldest admission first, get a page for the
//      position they decode next; with the pool empty the most recently
//      admitted running request is preempted (pages freed, back to the head
//      of the queue with its generated tokens kept: it is prefilled again
//      over prompt + generated, i.e. recomputation);
//   2. the queue's head is admitted while a slot is free and the pool holds
//      pages for its known tokens and the next position (no request jumps
//      the queue, so the oldest always progresses: a request that fits the
//      pool alone always finishes);
//   3. the step's work: a prefill per admitted request, and one batched
//      decode position per running request.
// commit() appends the step's tokens; a request finishes after
// max_new_tokens tokens or at its eos token, and frees its slot and pages.
//
// Server: plan -> page tables into the engine (infernt_batch_engine_set_
// pages) -> each prefill (infernt_batch_engine_prefill) -> one batched step
// of every slot (empty slots at position -1) -> commit.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdint>
#include <deque>
#include <memory>
#include <new>
#include <unordered_map>
#include <vector>

#include "../../../include/infernt_capi.h"
#include "../internal.h"

namespace {

using infernt::fail;

struct Request {
    int64_t id = 0;
    std::vector<int> tokens;  // prompt, then the generated tokens
    int prompt_len = 0;
    int max_new = 0;
    int eos = -1;
    int state = INFERNT_REQUEST_WAITING;
    int slot = -1;
    int fed = 0;              // positions [0, fed) hold cache rows
    std::vector<int> pages;   // pages of positions [0, pages.size() x page_size)
    long long admitted = -1;  // admission counter (preemption takes the largest)
    int preemptions = 0;
    bool prefill = false;     // admitted by the current plan

    int generated() const { return (int)tokens.size() - prompt_len; }
};

}  // namespace

struct infernt_scheduler {
    int slots = 0, page_size = 0, num_pages = 0, max_seq = 0, max_pages = 0;
    int64_t next_id = 1;
    long long admissions = 0;
    std::unordered_map<int64_t, std::unique_ptr<Request>> reqs;
    std::deque<Request*> queue;
    std::vector<Request*> slot_req;  // [slots]
    std::vector<int> free_pages;     // a stack: the last freed page is reused first
    bool planned = false;            // a plan awaits its commit
    // the current plan's arrays
    std::vector<int> pf_slot, pf_off, pf_len, pf_tokens;
    std::vector<int> tokens, positions, changed, table, n_pages;
    std::vector<char> slot_changed;
    int n_decode = 0, n_preempted = 0;
    long long steps = 0, preemptions = 0, prefill_tokens = 0, decode_tokens = 0;
    int finished = 0;
};

namespace {

int pages_for(const infernt_scheduler* s, int positions) { return (positions + s->page_size - 1) / s->page_size; }

void mark(infernt_scheduler* s, int slot) {
    if (!s->slot_changed[slot]) {
        s->slot_changed[slot] = 1;
        s->changed.push_back(slot);
    }
}

// Frees r's slot and pages.
void vacate(infernt_scheduler* s, Request* r) {
    for (auto it = r->pages.rbegin(); it != r->pages.rend(); ++it) s->free_pages.push_back(*it);
    r->pages.clear();
    if (r->slot >= 0) {
        s->slot_req[r->slot] = nullptr;
        mark(s, r->slot);
    }
    r->slot = -1;
    r->fed = 0;
    r->prefill = false;
}

void preempt(infernt_scheduler* s, Request* r) {
    vacate(s, r);
    r->state = INFERNT_REQUEST_WAITING;
    r->admitted = -1;
    r->preemptions += 1;
    s->preemptions += 1;
    s->n_preempted += 1;
    s->queue.push_front(r);
}

void finish(infernt_scheduler* s, Request* r, int state) {
    vacate(s, r);
    r->state = state;
    s->finished += state == INFERNT_REQUEST_FINISHED;
}

// The running request admitted last (the preemption victim), or null.
Request* youngest(infernt_scheduler* s) {
    Request* v = nullptr;
    for (Request* r : s->slot_req)
        if (r && (!v || r->admitted > v->admitted)) v = r;
    return v;
}

int take_page(infernt_scheduler* s) {
    const int p = s->free_pages.back();
    s->free_pages.pop_back();
    return p;
}

int plan(infernt_scheduler* s, infernt_sched_plan* out) {
    INFERNT_REQUIRE(!s->planned, "scheduler_plan: the previous plan has not been committed");
    s->n_preempted = 0;
    // 1. pages for the running requests' next positions, oldest first
    std::vector<Request*> running;
    for (Request* r : s->slot_req)
        if (r) running.push_back(r);
    std::sort(running.begin(), running.end(), [](const Request* a, const Request* b) { return a->admitted < b->admitted; });
    for (Request* r : running) {
        if (r->state != INFERNT_REQUEST_RUNNING) continue;  // preempted by an older request in this loop
        const int need = r->fed / s->page_size + 1;
        while ((int)r->pages.size() < need) {
            if (s->free_pages.empty()) {
                Request* v = youngest(s);
                preempt(s, v);
                if (v == r) break;
                continue;
            }
            r->pages.push_back(take_page(s));
            mark(s, r->slot);
        }
    }
    // 2. admissions, first come first served
    while (!s->queue.empty()) {
        Request* r = s->queue.front();
        int slot = -1;
        for (int i = 0; i < s->slots && slot < 0; ++i)
            if (!s->slot_req[i]) slot = i;
        const int need = (int)r->tokens.size() / s->page_size + 1;
        if (slot < 0 || need > (int)s->free_pages.size()) break;
        s->queue.pop_front();
        r->slot = slot;
        r->state = INFERNT_REQUEST_RUNNING;
        r->admitted = s->admissions++;
        r->prefill = true;
        r->fed = 0;
        for (int i = 0; i < need; ++i) r->pages.push_back(take_page(s));
        s->slot_req[slot] = r;
        mark(s, slot);
    }
    // 3. the step's work
    s->pf_slot.clear();
    s->pf_off.clear();
    s->pf_len.clear();
    s->pf_tokens.clear();
    s->n_decode = 0;
    for (int i = 0; i < s->slots; ++i) {
        Request* r = s->slot_req[i];
        s->tokens[i] = 0;
        s->positions[i] = -1;
        if (!r) continue;
        if (r->prefill) {
            s->pf_slot.push_back(i);
            s->pf_off.push_back((int)s->pf_tokens.size());
            s->pf_len.push_back((int)r->tokens.size());
            s->pf_tokens.insert(s->pf_tokens.end(), r->tokens.begin(), r->tokens.end());
        } else {
            s->tokens[i] = r->tokens[r->fed];
            s->positions[i] = r->fed;
            s->n_decode += 1;
        }
    }
    for (int i : s->changed) {
        Request* r = s->slot_req[i];
        int* row = s->table.data() + (size_t)i * s->max_pages;
        const int n = r ? (int)r->pages.size() : 0;
        for (int j = 0; j < s->max_pages; ++j) row[j] = j < n ? r->pages[j] : -1;
        s->n_pages[i] = n;
    }
    out->n_prefill = (int)s->pf_slot.size();
    out->prefill_slot = s->pf_slot.data();
    out->prefill_offset = s->pf_off.data();
    out->prefill_len = s->pf_len.data();
    out->prefill_tokens = s->pf_tokens.data();
    out->n_decode = s->n_decode;
    out->tokens = s->tokens.data();
    out->positions = s->positions.data();
    out->n_changed = (int)s->changed.size();
    out->changed_slot = s->changed.data();
    out->pages = s->table.data();
    out->n_pages = s->n_pages.data();
    out->max_pages = s->max_pages;
    out->n_preempted = s->n_preempted;
    s->planned = true;
    return INFERNT_OK;
}

void append(infernt_scheduler* s, Request* r, int token) {
    r->tokens.push_back(token);
    if (r->generated() >= r->max_new || (r->eos >= 0 && token == r->eos)) finish(s, r, INFERNT_REQUEST_FINISHED);
}

int commit(infernt_scheduler* s, const int* prefill_next, const int* decode_next) {
    INFERNT_REQUIRE(s->planned, "scheduler_commit: no plan to commit");
    INFERNT_REQUIRE(s->pf_slot.empty() || prefill_next, "scheduler_commit: %d prefills need their tokens",
                    (int)s->pf_slot.size());
    INFERNT_REQUIRE(!s->n_decode || decode_next, "scheduler_commit: %d decoding slots need their tokens", s->n_decode);
    for (size_t k = 0; k < s->pf_slot.size(); ++k)
        INFERNT_REQUIRE(prefill_next[k] >= 0, "scheduler_commit: token %d after prefill %zu", prefill_next[k], k);
    for (int i = 0; i < s->slots; ++i)
        INFERNT_REQUIRE(s->positions[i] < 0 || decode_next[i] >= 0, "scheduler_commit: token %d of slot %d",
                        decode_next[i], i);
    // the page tables the plan reported are now the engine's
    for (int i : s->changed) s->slot_changed[i] = 0;
    s->changed.clear();
    for (size_t k = 0; k < s->pf_slot.size(); ++k) {
        Request* r = s->slot_req[s->pf_slot[k]];
        r->prefill = false;
        r->fed = (int)r->tokens.size();
        s->prefill_tokens += r->fed;
        append(s, r, prefill_next[k]);
    }
    for (int i = 0; i < s->slots; ++i) {
        if (s->positions[i] < 0) continue;
        Request* r = s->slot_req[i];
        r->fed += 1;
        s->decode_tokens += 1;
        append(s, r, decode_next[i]);
    }
    s->steps += 1;
    s->planned = false;
    return INFERNT_OK;
}

}  // namespace

extern "C" {

int infernt_scheduler_create(int slots, int page_size, int num_pages, int max_seq_len, infernt_scheduler** out) {
    INFERNT_REQUIRE(out, "scheduler_create: null argument");
    *out = nullptr;
    INFERNT_REQUIRE(slots >= 1 && slots <= 4096 && page_size >= 1 && num_pages >= 1 && max_seq_len >= 2,
                    "scheduler_create: %d slots, %d pages of %d positions, max_seq_len %d", slots, num_pages,
                    page_size, max_seq_len);
    infernt_scheduler* s = new (std::nothrow) infernt_scheduler();
    INFERNT_REQUIRE(s, "scheduler_create: host allocation failed");
    s->slots = slots;
    s->page_size = page_size;
    s->num_pages = num_pages;
    s->max_seq = max_seq_len;
    s->max_pages = pages_for(s, max_seq_len);
    s->slot_req.assign(slots, nullptr);
    for (int p = num_pages - 1; p >= 0; --p) s->free_pages.push_back(p);  // page 0 is taken first
    s->tokens.assign(slots, 0);
    s->positions.assign(slots, -1);
    s->table.assign((size_t)slots * s->max_pages, -1);
    s->n_pages.assign(slots, 0);
    s->slot_changed.assign(slots, 0);
    *out = s;
    return INFERNT_OK;
}

int infernt_scheduler_destroy(infernt_scheduler* s) {
    delete s;
    return INFERNT_OK;
}

int infernt_scheduler_submit(infernt_scheduler* s, const int* prompt, int n, int max_new_tokens, int eos,
                             int64_t* id) {
    INFERNT_REQUIRE(s && prompt && id, "scheduler_submit: null argument");
    INFERNT_REQUIRE(n >= 1 && max_new_tokens >= 1 && (long long)n + max_new_tokens <= s->max_seq,
                    "scheduler_submit: %d prompt tokens + %d new pass max_seq_len %d", n, max_new_tokens, s->max_seq);
    // the most a request holds: pages through position n + max_new - 1
    const int most = (n + max_new_tokens - 1) / s->page_size + 1;
    INFERNT_REQUIRE(most <= s->num_pages, "scheduler_submit: the request needs %d pages; the pool has %d", most,
                    s->num_pages);
    for (int i = 0; i < n; ++i) INFERNT_REQUIRE(prompt[i] >= 0, "scheduler_submit: token %d at %d", prompt[i], i);
    std::unique_ptr<Request> r(new (std::nothrow) Request());
    INFERNT_REQUIRE(r, "scheduler_submit: host allocation failed");
    r->id = s->next_id++;
    r->tokens.assign(prompt, prompt + n);
    r->prompt_len = n;
    r->max_new = max_new_tokens;
    r->eos = eos;
    s->queue.push_back(r.get());
    *id = r->id;
    s->reqs.emplace(r->id, std::move(r));
    return INFERNT_OK;
}

int infernt_scheduler_cancel(infernt_scheduler* s, int64_t id) {
    INFERNT_REQUIRE(s, "scheduler_cancel: null scheduler");
    INFERNT_REQUIRE(!s->planned, "scheduler_cancel: a plan awaits its commit");
    auto it = s->reqs.find(id);
    INFERNT_REQUIRE(it != s->reqs.end(), "scheduler_cancel: no request %lld", (long long)id);
    Request* r = it->second.get();
    if (r->state == INFERNT_REQUEST_WAITING)
        s->queue.erase(std::find(s->queue.begin(), s->queue.end(), r));
    if (r->state == INFERNT_REQUEST_WAITING || r->state == INFERNT_REQUEST_RUNNING) {
        vacate(s, r);
        r->state = INFERNT_REQUEST_CANCELLED;
    }
    return INFERNT_OK;
}

int infernt_scheduler_plan(infernt_scheduler* s, infernt_sched_plan* out) {
    INFERNT_REQUIRE(s && out, "scheduler_plan: null argument");
    return plan(s, out);
}

int infernt_scheduler_commit(infernt_scheduler* s, const int* prefill_next, const int* decode_next) {
    INFERNT_REQUIRE(s, "scheduler_commit: null scheduler");
    return commit(s, prefill_next, decode_next);
}

int infernt_scheduler_result(infernt_scheduler* s, int64_t id, int* tokens, int cap, int* n, int* state,
                             int* preemptions) {
    INFERNT_REQUIRE(s && n && state && cap >= 0 && (cap == 0 || tokens), "scheduler_result: bad arguments");
    auto it = s->reqs.find(id);
    INFERNT_REQUIRE(it != s->reqs.end(), "scheduler_result: no request %lld", (long long)id);
    const Request* r = it->second.get();
    *n = r->generated();
    *state = r->state;
    if (preemptions) *preemptions = r->preemptions;
    const int k = std::min(cap, *n);
    std::copy(r->tokens.begin() + r->prompt_len, r->tokens.begin() + r->prompt_len + k, tokens);
    return INFERNT_OK;
}

int infernt_scheduler_release(infernt_scheduler* s, int64_t id) {
    INFERNT_REQUIRE(s, "scheduler_release: null scheduler");
    auto it = s->reqs.find(id);
    INFERNT_REQUIRE(it != s->reqs.end(), "scheduler_release: no request %lld", (long long)id);
    INFERNT_REQUIRE(it->second->state == INFERNT_REQUEST_FINISHED || it->second->state == INFERNT_REQUEST_CANCELLED,
                    "scheduler_release: request %lld is still queued or running", (long long)id);
    s->reqs.erase(it);
    return INFERNT_OK;
}

int infernt_scheduler_stats(infernt_scheduler* s, infernt_sched_stats* out) {
    INFERNT_REQUIRE(s && out, "scheduler_stats: null argument");
    out->waiting = (int)s->queue.size();
    out->running = 0;
    for (Request* r : s->slot_req) out->running += r != nullptr;
    out->finished = s->finished;
    out->free_pages = (int)s->free_pages.size();
    out->steps = s->steps;
    out->preemptions = s->preemptions;
    out->prefill_tokens = s->prefill_tokens;
    out->decode_tokens = s->decode_tokens;
    return INFERNT_OK;
}

}  // extern "C"

struct infernt_server {
    infernt_batch_engine* engine = nullptr;
    infernt_scheduler* sched = nullptr;
    int slots = 0, vocab = 0;
    bool salted = false;
    std::vector<int> next, pf_next;
    std::vector<uint64_t> salts;

    ~infernt_server() {
        if (engine) infernt_batch_engine_destroy(engine);
        if (sched) infernt_scheduler_destroy(sched);
    }
};

namespace {

int server_step(infernt_server* v, int* n_finished) {
    infernt_sched_stats before{};
    infernt_scheduler_stats(v->sched, &before);
    infernt_sched_plan p{};
    if (int s = infernt_scheduler_plan(v->sched, &p)) return s;
    bool salts_changed = false;
    for (int k = 0; k < p.n_changed; ++k) {
        const int slot = p.changed_slot[k];
        if (int s = infernt_batch_engine_set_pages(v->engine, slot, p.pages + (size_t)slot * p.max_pages,
                                                   p.n_pages[slot]))
            return s;
        // the slot's request id keys its temperature draws
        const Request* r = v->sched->slot_req[slot];
        const uint64_t salt = r ? (uint64_t)r->id : 0;
        if (v->salts[slot] != salt) {
            v->salts[slot] = salt;
            salts_changed = true;
        }
    }
    if (v->salted && salts_changed)
        if (int s = infernt_batch_engine_set_salts(v->engine, v->salts.data())) return s;
    v->pf_next.assign(p.n_prefill, 0);
    for (int k = 0; k < p.n_prefill; ++k)
        if (int s = infernt_batch_engine_prefill(v->engine, p.prefill_slot[k], p.prefill_tokens + p.prefill_offset[k],
                                                 p.prefill_len[k], 0, 0, &v->pf_next[k], nullptr, nullptr))
            return s;
    if (p.n_decode)
        if (int s = infernt_batch_engine_step(v->engine, p.tokens, p.positions, v->next.data())) return s;
    if (int s = infernt_scheduler_commit(v->sched, v->pf_next.data(), v->next.data())) return s;
    if (n_finished) {
        infernt_sched_stats after{};
        infernt_scheduler_stats(v->sched, &after);
        *n_finished = after.finished - before.finished;
    }
    return INFERNT_OK;
}

}  // namespace

extern "C" {

int infernt_server_create_seeded(const infernt_llama_config* cfg, int slots, int page_size, int num_pages,
                                 uint64_t seed, float std_dev, infernt_server** out) {
    INFERNT_REQUIRE(cfg && out, "server_create: null argument");
    *out = nullptr;
    std::unique_ptr<infernt_server> v(new (std::nothrow) infernt_server());
    INFERNT_REQUIRE(v, "server_create: host allocation failed");
    if (int s = infernt_scheduler_create(slots, page_size, num_pages, cfg->max_seq_len, &v->sched)) return s;
    if (int s = infernt_batch_engine_create_paged(cfg, slots, page_size, num_pages, seed, std_dev, 0, &v->engine))
        return s;
    v->slots = slots;
    v->vocab = cfg->vocab_size;
    v->next.assign(slots, 0);
    v->salts.assign(slots, 0);
    *out = v.release();
    return INFERNT_OK;
}

int infernt_server_destroy(infernt_server* srv) {
    delete srv;
    return INFERNT_OK;
}

int infernt_server_submit(infernt_server* srv, const int* prompt, int n, int max_new_tokens, int eos, int64_t* id) {
    INFERNT_REQUIRE(srv && prompt, "server_submit: null argument");
    for (int i = 0; i < n; ++i)
        INFERNT_REQUIRE(prompt[i] >= 0 && prompt[i] < srv->vocab, "server_submit: token %d at %d outside [0, %d)",
                        prompt[i], i, srv->vocab);
    return infernt_scheduler_submit(srv->sched, prompt, n, max_new_tokens, eos, id);
}

int infernt_server_step(infernt_server* srv, int* n_finished) {
    INFERNT_REQUIRE(srv, "server_step: null server");
    if (int s = server_step(srv, n_finished)) {
        // the step did not complete: its plan is dropped with its requests'
        // state as the plan left it (the server is not usable after an error)
        return s;
    }
    return INFERNT_OK;
}

int infernt_server_run(infernt_server* srv, double* ms) {
    INFERNT_REQUIRE(srv, "server_run: null server");
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        infernt_sched_stats st{};
        infernt_scheduler_stats(srv->sched, &st);
        if (st.waiting == 0 && st.running == 0) break;
        if (int s = server_step(srv, nullptr)) return s;
    }
    if (ms) *ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    return INFERNT_OK;
}

int infernt_server_result(infernt_server* srv, int64_t id, int* tokens, int cap, int* n, int* state,
                          int* preemptions) {
    INFERNT_REQUIRE(srv, "server_result: null server");
    return infernt_scheduler_result(srv->sched, id, tokens, cap, n, state, preemptions);
}

int infernt_server_stats(infernt_server* srv, infernt_sched_stats* out) {
    INFERNT_REQUIRE(srv, "server_stats: null server");
    return infernt_scheduler_stats(srv->sched, out);
}

int infernt_server_set_sampling(infernt_server* srv, float temperature, uint64_t seed) {
    INFERNT_REQUIRE(srv, "server_set_sampling: null server");
    if (int s = infernt_batch_engine_set_sampling(srv->engine, temperature, seed)) return s;
    srv->salted = true;
    for (int i = 0; i < srv->slots; ++i) {
        const Request* r = srv->sched->slot_req[i];
        srv->salts[i] = r ? (uint64_t)r->id : 0;
    }
    return infernt_batch_engine_set_salts(srv->engine, srv->salts.data());
}

int infernt_server_engine(infernt_server* srv, infernt_batch_engine** out) {
    INFERNT_REQUIRE(srv && out, "server_engine: null argument");
    *out = srv->engine;
    return INFERNT_OK;
}

}  // extern "C"
