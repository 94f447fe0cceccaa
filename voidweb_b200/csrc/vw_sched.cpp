// vw_sched.cpp -- the continuous-batching scheduler wired to the paged KV
// bookkeeping (host side, C++17).
//
// Reference: scheduler/scheduler.bm:186-293 (Scheduler: a FCFS waiting queue,
// a running set, a prefill-token budget per step, chunked prefill of at most
// 2048 prompt tokens, one decode token per running sequence, commit_step /
// drain_finished) and engine/engine.bm:127-146 (Engine::step: schedule, forward,
// sample, commit).  The reference never connects it to the KV cache: request
// block tables stay empty, the block manager and the radix tree are never
// called, and a request whose prompt needs a second chunk is never scheduled
// again (promotion only takes from the waiting queue).  This scheduler keeps
// the reference's batching rules and adds the bookkeeping:
//  * block tables: every scheduled sequence's table covers the positions it
//    writes this step, allocated from the block manager (engine/kv_cache.bm:
//    69-91) before the step;
//  * prefix reuse: full 16-token pages are indexed by the block manager's
//    chained prefix hash (kv_cache.bm:127-164, rolling_hash), which is
//    page-aligned by construction; an admitted request starts from the longest
//    indexed chain of its prompt (at least one token is always computed), its
//    table shares those pages (incref) and its prefill starts after them.
//    The radix tree (radix_cache.bm) is not used as the page map: its lookup
//    returns every block of a partially matched edge and its splits leave
//    blocks that do not start at a page boundary, so the i-th block on a
//    matched path need not hold the path's page i;
//  * the index holds one reference per page it keeps; when the pool runs out,
//    the least recently used pages only the index holds are released;
//  * copy-on-write: a step that writes into a page with ref_count > 1 gets a
//    private copy first (vw_bm_cow) and the (src, dst) pair is returned for
//    vw_block_copy to run before the step;
//  * preemption: when a decode cannot get a page even after eviction, the most
//    recently admitted running request is preempted (its pages released, its
//    tokens kept) and re-prefilled later from the waiting queue's front;
//  * chunk continuation: a request with prompt tokens left is scheduled again.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <deque>
#include <list>
#include <unordered_map>
#include <vector>

#include "../../include/voidweb_kv.h"

namespace {

constexpr uint32_t kPage = 16;

struct Req {
    uint64_t id = 0;
    std::vector<uint32_t> tokens;    // prompt, then the sampled tokens
    uint32_t prompt_len = 0;
    uint32_t max_new = 0;
    int64_t stop = -1;
    uint32_t cached = 0;             // tokens whose K/V rows are in the pages
    uint32_t outputs = 0;
    std::vector<uint32_t> table;     // physical block ids, page p -> table[p]
    uint64_t admitted = 0;           // admission order (preemption picks the youngest)
    // this step
    uint32_t n = 0;
    bool samples = false;
    bool in_step = false;
};

// The tokens to cache before the next sample: the whole prompt for a fresh
// request; after a preemption, every token but the last sampled one.
uint32_t prefill_end(const Req& r) {
    return r.outputs == 0 ? r.prompt_len : (uint32_t)r.tokens.size() - 1;
}

}  // namespace

struct vw_sched {
    vw_sched_config cfg{};
    vw_block_manager* bm = nullptr;
    uint64_t next_id = 1, admit_clock = 0, preemptions = 0;
    std::deque<Req*> waiting;
    std::vector<Req*> running;                       // admission order
    std::unordered_map<uint64_t, Req*> by_id;
    std::deque<Req*> finished;
    // prefix index: chained page hash -> block, LRU order (front = oldest)
    struct Entry {
        uint32_t block;
        std::list<uint64_t>::iterator pos;
    };
    std::unordered_map<uint64_t, Entry> index;
    std::list<uint64_t> lru;
    // the last schedule's arrays
    std::vector<vw_sched_seq> seqs;
    std::vector<uint32_t> tokens, tables, copies;
    std::vector<Req*> step;

    ~vw_sched() {
        for (auto& kv : by_id) delete kv.second;
        for (Req* r : finished) delete r;
    }

    void touch(std::unordered_map<uint64_t, Entry>::iterator it) {
        lru.erase(it->second.pos);
        lru.push_back(it->first);
        it->second.pos = std::prev(lru.end());
    }

    // Release up to `need` pages that only the index holds, oldest first.
    uint32_t evict(uint32_t need) {
        uint32_t freed = 0;
        for (auto it = lru.begin(); it != lru.end() && freed < need;) {
            auto e = index.find(*it);
            if (vw_bm_ref_count(bm, e->second.block) == 1) {
                vw_bm_decref(bm, e->second.block);
                index.erase(e);
                it = lru.erase(it);
                ++freed;
            } else {
                ++it;
            }
        }
        return freed;
    }

    bool alloc_one(uint32_t* id) {
        if (vw_bm_alloc(bm, id) == VW_OK) return true;
        if (evict(1) == 1 && vw_bm_alloc(bm, id) == VW_OK) return true;
        return false;
    }

    void release(Req* r) {
        vw_bm_free_seq(bm, r->table.data(), (uint32_t)r->table.size());
        r->table.clear();
    }

    // Pages for positions [0, upto) and a private copy of the first page this
    // step writes (position r->cached) when it is shared.
    bool ensure_pages(Req* r, uint32_t upto) {
        const uint32_t need = (upto + kPage - 1) / kPage;
        const uint32_t first = r->cached / kPage;
        if (first < r->table.size() && vw_bm_ref_count(bm, r->table[first]) > 1) {
            uint32_t pair[2], copied = 0;
            if (vw_bm_cow(bm, r->table.data(), first, pair, &copied) != VW_OK) {
                if (evict(1) != 1 || vw_bm_cow(bm, r->table.data(), first, pair, &copied) != VW_OK)
                    return false;
            }
            if (copied) { copies.push_back(pair[0]); copies.push_back(pair[1]); }
        }
        while (r->table.size() < need) {
            uint32_t id;
            if (!alloc_one(&id)) return false;
            r->table.push_back(id);
        }
        return true;
    }

    // Longest indexed chain of full pages among the first `limit` tokens.
    void reuse_prefix(Req* r, uint32_t limit) {
        uint64_t h = 0;
        for (uint32_t p = 0; (p + 1) * kPage <= limit; ++p) {
            h = vw_rolling_hash(h, r->tokens.data() + p * kPage, kPage);
            auto it = index.find(h);
            if (it == index.end()) break;
            vw_bm_incref(bm, it->second.block);
            touch(it);
            r->table.push_back(it->second.block);
            r->cached = (p + 1) * kPage;
        }
    }

    // Index the pages that became full with this step's tokens.
    void register_pages(Req* r, uint32_t before, uint32_t after) {
        if (!cfg.prefix_cache) return;
        uint64_t h = 0;
        for (uint32_t p = 0; (p + 1) * kPage <= after; ++p) {
            h = vw_rolling_hash(h, r->tokens.data() + p * kPage, kPage);
            if ((p + 1) * kPage <= before) continue;
            if (index.count(h)) {
                touch(index.find(h));
                continue;
            }
            vw_bm_incref(bm, r->table[p]);
            lru.push_back(h);
            index[h] = Entry{r->table[p], std::prev(lru.end())};
        }
    }

    void preempt(Req* r) {
        release(r);
        r->cached = 0;
        running.erase(std::find(running.begin(), running.end(), r));
        waiting.push_front(r);
        ++preemptions;
    }
};

extern "C" {

int32_t vw_sched_create(const vw_sched_config* cfg, vw_block_manager* bm, vw_sched** out) {
    if (!cfg || !bm || !out) return VW_ERR_INVALID_ARG;
    if (cfg->reserved || cfg->max_batch_tokens == 0 || cfg->max_running_seqs == 0 ||
        cfg->max_chunk == 0 || cfg->max_seq_len == 0)
        return VW_ERR_INVALID_ARG;
    vw_sched* s = new vw_sched();
    s->cfg = *cfg;
    s->bm = bm;
    *out = s;
    return VW_OK;
}

int32_t vw_sched_destroy(vw_sched* s) {
    if (!s) return VW_OK;
    for (auto& kv : s->by_id) s->release(kv.second);
    for (auto& e : s->index) vw_bm_decref(s->bm, e.second.block);
    delete s;
    return VW_OK;
}

int32_t vw_sched_add_request(vw_sched* s, const uint32_t* prompt, uint32_t n, uint32_t max_new_tokens,
                             int64_t stop_token, uint64_t* id_out) {
    if (!s || !prompt || n == 0 || !id_out || max_new_tokens == 0) return VW_ERR_INVALID_ARG;
    if ((uint64_t)n + max_new_tokens > s->cfg.max_seq_len) return VW_ERR_INVALID_ARG;
    Req* r = new Req();
    r->id = s->next_id++;
    r->tokens.assign(prompt, prompt + n);
    r->prompt_len = n;
    r->max_new = max_new_tokens;
    r->stop = stop_token;
    s->waiting.push_back(r);
    s->by_id[r->id] = r;
    *id_out = r->id;
    return VW_OK;
}

int32_t vw_sched_schedule(vw_sched* s, vw_sched_batch* out) {
    if (!s || !out) return VW_ERR_INVALID_ARG;
    for (Req* r : s->step) { r->in_step = false; r->n = 0; r->samples = false; }
    s->step.clear();
    s->copies.clear();
    std::vector<Req*> decodes, prefills;
    // 1. decodes get their pages first: a running sequence whose prompt is cached
    for (size_t i = 0; i < s->running.size(); ++i) {
        Req* r = s->running[i];
        if (r->cached < prefill_end(*r) || r->outputs == 0) continue;
        while (!s->ensure_pages(r, r->cached + 1)) {
            // preempt the youngest other running request; if none, this one waits
            Req* victim = nullptr;
            for (Req* o : s->running)
                if (o != r && !o->in_step && (!victim || o->admitted > victim->admitted)) victim = o;
            if (!victim) { s->preempt(r); r = nullptr; break; }
            const size_t vpos = std::find(s->running.begin(), s->running.end(), victim) - s->running.begin();
            s->preempt(victim);
            if (vpos < i) --i;
        }
        if (!r) { --i; continue; }
        r->n = 1;
        r->samples = true;
        r->in_step = true;
        decodes.push_back(r);
    }
    // 2. prompt chunks of running requests (scheduler.bm:251-256 budget and chunk
    //    rules), then admissions from the waiting queue (scheduler.bm:248-275)
    uint32_t budget = s->cfg.max_batch_tokens;
    auto plan_prefill = [&](Req* r) -> bool {
        const uint32_t end = prefill_end(*r);
        const uint32_t n = std::min(std::min(end - r->cached, budget), s->cfg.max_chunk);
        if (n == 0 || !s->ensure_pages(r, r->cached + n)) return false;
        r->n = n;
        r->samples = r->outputs == 0 && r->cached + n == end;
        r->in_step = true;
        budget -= n;
        prefills.push_back(r);
        return true;
    };
    for (Req* r : s->running)
        if (!r->in_step && r->cached < prefill_end(*r) && budget > 0) plan_prefill(r);
    while (!s->waiting.empty() && s->running.size() < s->cfg.max_running_seqs && budget > 0) {
        Req* r = s->waiting.front();
        if (s->cfg.prefix_cache && r->cached == 0) s->reuse_prefix(r, prefill_end(*r) - 1);
        if (!plan_prefill(r)) {
            s->release(r);             // keep nothing from a failed admission
            r->cached = 0;
            break;
        }
        s->waiting.pop_front();
        r->admitted = ++s->admit_clock;
        s->running.push_back(r);
    }
    // 3. the batch: prefill chunks first, then decodes (scheduler.bm:134-170)
    s->seqs.clear();
    s->tokens.clear();
    s->step = prefills;
    s->step.insert(s->step.end(), decodes.begin(), decodes.end());
    uint32_t stride = 1;
    for (Req* r : s->step) stride = std::max(stride, (uint32_t)r->table.size());
    s->tables.assign(s->step.size() * stride, 0);
    for (size_t k = 0; k < s->step.size(); ++k) {
        Req* r = s->step[k];
        vw_sched_seq q{};
        q.seq_id = r->id;
        q.is_prefill = k < prefills.size() ? 1u : 0u;
        q.num_tokens = r->n;
        q.ctx_start = r->cached;
        q.samples = r->samples ? 1u : 0u;
        q.token_offset = (uint32_t)s->tokens.size();
        s->tokens.insert(s->tokens.end(), r->tokens.begin() + r->cached, r->tokens.begin() + r->cached + r->n);
        std::copy(r->table.begin(), r->table.end(), s->tables.begin() + k * stride);
        s->seqs.push_back(q);
    }
    out->num_seqs = (uint32_t)s->seqs.size();
    out->table_stride = stride;
    out->seqs = s->seqs.data();
    out->tokens = s->tokens.data();
    out->block_tables = s->tables.data();
    out->num_copies = (uint32_t)(s->copies.size() / 2);
    out->copies = s->copies.data();
    return VW_OK;
}

int32_t vw_sched_commit(vw_sched* s, const uint64_t* ids, const uint32_t* tokens, uint32_t n) {
    if (!s || (n && (!ids || !tokens))) return VW_ERR_INVALID_ARG;
    // every scheduled sequence's tokens are now cached
    for (Req* r : s->step) {
        const uint32_t before = r->cached;
        r->cached += r->n;
        s->register_pages(r, before, r->cached);
    }
    int32_t rc = VW_OK;
    for (uint32_t i = 0; i < n; ++i) {
        auto it = s->by_id.find(ids[i]);
        if (it == s->by_id.end() || !it->second->in_step || !it->second->samples) {
            rc = VW_ERR_INVALID_ARG;           // not a sampling sequence of this step
            continue;
        }
        Req* r = it->second;
        r->tokens.push_back(tokens[i]);
        r->outputs += 1;
        r->samples = false;
        if (r->outputs >= r->max_new || (r->stop >= 0 && (int64_t)tokens[i] == r->stop)) {
            s->release(r);
            s->running.erase(std::find(s->running.begin(), s->running.end(), r));
            s->by_id.erase(it);
            s->finished.push_back(r);
        }
    }
    for (Req* r : s->step) { r->in_step = false; r->n = 0; r->samples = false; }
    s->step.clear();
    return rc;
}

int32_t vw_sched_take_finished(vw_sched* s, uint64_t* id, uint32_t* out_tokens, uint32_t cap,
                               uint32_t* num_out) {
    if (!s || !id || !num_out) return VW_ERR_INVALID_ARG;
    if (s->finished.empty()) return VW_ERR_INVALID_ARG;
    Req* r = s->finished.front();
    *id = r->id;
    *num_out = r->outputs;
    for (uint32_t i = 0; i < r->outputs && i < cap && out_tokens; ++i)
        out_tokens[i] = r->tokens[r->prompt_len + i];
    s->finished.pop_front();
    delete r;
    return VW_OK;
}

int32_t vw_sched_stats(const vw_sched* s, vw_sched_stat* st) {
    if (!s || !st) return VW_ERR_INVALID_ARG;
    st->waiting = (uint32_t)s->waiting.size();
    st->running = (uint32_t)s->running.size();
    st->finished = (uint32_t)s->finished.size();
    st->cached_pages = (uint32_t)s->index.size();
    uint32_t refs = 0;
    for (const Req* r : s->running) refs += (uint32_t)r->table.size();
    for (const Req* r : s->waiting) refs += (uint32_t)r->table.size();
    st->table_refs = refs;
    st->free_blocks = vw_bm_free_count(s->bm);
    st->preemptions = (uint32_t)s->preemptions;
    st->reserved = 0;
    return VW_OK;
}

}  // extern "C"
