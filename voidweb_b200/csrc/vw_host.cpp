// vw_host.cpp -- host-side block bookkeeping behind the C ABI: the paged-KV
// block manager (engine/kv_cache.bm:29-164) and the radix prefix tree
// (radix_cache/radix_cache.bm:27-285), in C++17.
//
// Observable behaviour follows the reference (allocation order, ref counts,
// prefix-hash chains, radix lookup/insert/split rules).  The data structures
// are this library's own:
//  * per-block state lives in dense arrays indexed by block id instead of a
//    HashMap<BlockId, KvPage> (ids are < max_blocks by construction), so
//    alloc / incref / decref are O(1) without hashing;
//  * radix nodes live in an index-addressed arena with small sorted child
//    vectors, and the evictable leaves (no children, blocks held, ref_count 0)
//    are kept in an ordered set keyed by last access, so an LRU eviction is
//    O(log n) instead of the reference's full-tree DFS per evicted leaf
//    (radix_cache.bm:256-274).
// Deliberate divergences from the reference, shared with the CPU oracle:
// timestamps come from a logical clock (radix_cache.bm:41,46-48 use wall-clock
// microseconds); the evicted leaf is found by edge, not token by token
// (radix_cache.bm:278-281 fails for edges longer than one token), its ids are
// returned to the caller and the emptied leaf is removed; lock/unlock maintain
// the ref_count the reference declares (radix_cache.bm:32) but never updates.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <set>
#include <unordered_map>
#include <vector>

#include "../../include/voidweb_kv.h"
#include "vw_fault.h"

struct vw_block_manager {
    uint32_t block_size = 16, max_blocks = 0, used = 0;
    std::vector<uint32_t> free_blocks;          // pop from the back (kv_cache.bm:70)
    std::vector<uint32_t> ref;                  // 0 = not allocated
    std::vector<uint64_t> token_hash;
    std::unordered_map<uint64_t, std::vector<uint32_t>> prefix;   // kv_cache.bm:37
};

extern "C" {

uint64_t vw_rolling_hash(uint64_t prev, const uint32_t* tokens, uint32_t n) {
    // kv_cache.bm:157-164: wrapping polynomial hash with Knuth's constant
    const uint64_t P = 0x9e3779b97f4a7c15ull;
    uint64_t h = prev + (uint64_t)n * P;
    for (uint32_t i = 0; i < n; ++i) h = h * P + tokens[i];
    return h;
}

int32_t vw_bm_create(uint32_t block_size, uint32_t max_blocks, vw_block_manager** out) {
    if (!out || block_size == 0) return VW_ERR_INVALID_ARG;
    vw_block_manager* bm = new vw_block_manager();
    bm->block_size = block_size;
    bm->max_blocks = max_blocks;
    bm->free_blocks.resize(max_blocks);
    for (uint32_t i = 0; i < max_blocks; ++i) bm->free_blocks[i] = i;   // kv_cache.bm:48
    bm->ref.assign(max_blocks, 0);
    bm->token_hash.assign(max_blocks, 0);
    *out = bm;
    return VW_OK;
}

int32_t vw_bm_destroy(vw_block_manager* bm) {
    delete bm;
    return VW_OK;
}

uint32_t vw_bm_capacity(const vw_block_manager* bm) {
    return (uint32_t)bm->free_blocks.size() + bm->used;
}

uint32_t vw_bm_free_count(const vw_block_manager* bm) { return (uint32_t)bm->free_blocks.size(); }

}  // extern "C"

namespace {
// kv_cache.bm:69-78 (the caller checked that a block is free)
uint32_t bm_pop(vw_block_manager* bm) {
    const uint32_t id = bm->free_blocks.back();
    bm->free_blocks.pop_back();
    bm->ref[id] = 1;
    bm->token_hash[id] = 0;
    bm->used += 1;
    return id;
}
}  // namespace

extern "C" {

int32_t vw_bm_alloc(vw_block_manager* bm, uint32_t* out) {
    if (vw::fault_take(vw::kCanOom, nullptr) != VW_OK) return VW_ERR_OOM;   // vw_fault_inject
    if (bm->free_blocks.empty()) return VW_ERR_OOM;
    *out = bm_pop(bm);
    return VW_OK;
}

int32_t vw_bm_alloc_seq(vw_block_manager* bm, uint32_t n, uint32_t* out) {
    if (vw::fault_take(vw::kCanOom, nullptr) != VW_OK) return VW_ERR_OOM;   // vw_fault_inject
    if (bm->free_blocks.size() < n) return VW_ERR_OOM;               // kv_cache.bm:82-85
    for (uint32_t i = 0; i < n; ++i) out[i] = bm_pop(bm);
    return VW_OK;
}

void vw_bm_incref(vw_block_manager* bm, uint32_t id) {
    if (id < bm->max_blocks && bm->ref[id] > 0) bm->ref[id] += 1;
}

void vw_bm_decref(vw_block_manager* bm, uint32_t id) {
    if (id >= bm->max_blocks || bm->ref[id] == 0) return;
    if (--bm->ref[id] == 0) {
        bm->used -= 1;
        bm->free_blocks.push_back(id);                                // kv_cache.bm:109-112
    }
}

void vw_bm_free_seq(vw_block_manager* bm, const uint32_t* table, uint32_t n) {
    for (uint32_t i = 0; i < n; ++i) vw_bm_decref(bm, table[i]);
}

uint32_t vw_bm_ref_count(const vw_block_manager* bm, uint32_t id) {
    return id < bm->max_blocks ? bm->ref[id] : 0;
}

uint32_t vw_bm_prefix_lookup(const vw_block_manager* bm, const uint32_t* tokens, uint32_t n,
                             uint32_t* out, uint32_t cap) {
    uint32_t count = 0;
    uint64_t hash = 0;
    for (uint32_t off = 0; off < n; off += bm->block_size) {
        const uint32_t len = std::min(bm->block_size, n - off);
        hash = vw_rolling_hash(hash, tokens + off, len);
        auto it = bm->prefix.find(hash);
        if (it == bm->prefix.end()) break;                            // kv_cache.bm:134
        for (uint32_t id : it->second) {
            if (count < cap) out[count] = id;
            ++count;
        }
    }
    return count;
}

void vw_bm_register_prefix_block(vw_block_manager* bm, uint32_t id, uint64_t token_hash) {
    if (id < bm->max_blocks && bm->ref[id] > 0) bm->token_hash[id] = token_hash;
    bm->prefix[token_hash].push_back(id);                             // duplicates accumulate
    vw_bm_incref(bm, id);
}

uint32_t vw_bm_free_list(const vw_block_manager* bm, uint32_t* out, uint32_t cap) {
    const uint32_t n = (uint32_t)bm->free_blocks.size();
    std::memcpy(out, bm->free_blocks.data(), sizeof(uint32_t) * std::min(n, cap));
    return n;
}

int32_t vw_bm_cow(vw_block_manager* bm, uint32_t* table, uint32_t index, uint32_t* pair_out,
                  uint32_t* copied) {
    *copied = 0;
    const uint32_t id = table[index];
    if (id >= bm->max_blocks || bm->ref[id] <= 1) return VW_OK;
    uint32_t fresh;
    if (vw_bm_alloc(bm, &fresh) != VW_OK) return VW_ERR_OOM;
    vw_bm_decref(bm, id);
    table[index] = fresh;
    pair_out[0] = id;
    pair_out[1] = fresh;
    *copied = 1;
    return VW_OK;
}

uint32_t vw_bm_compact(vw_block_manager* bm, uint32_t* pairs_out, uint32_t cap) {
    const uint32_t target = bm->used;
    std::vector<uint32_t> holes, movers;
    for (uint32_t i = 0; i < target; ++i)
        if (bm->ref[i] == 0) holes.push_back(i);
    for (uint32_t i = target; i < bm->max_blocks; ++i)
        if (bm->ref[i] > 0) movers.push_back(i);
    std::unordered_map<uint32_t, uint32_t> remap;
    const uint32_t n = (uint32_t)movers.size();   // == holes.size()
    for (uint32_t k = 0; k < n; ++k) {
        const uint32_t s = movers[k], d = holes[k];
        bm->ref[d] = bm->ref[s];
        bm->token_hash[d] = bm->token_hash[s];
        bm->ref[s] = 0;
        bm->token_hash[s] = 0;
        remap[s] = d;
        if (k < cap) { pairs_out[2 * k] = s; pairs_out[2 * k + 1] = d; }
    }
    for (auto& kv : bm->prefix)
        for (auto& id : kv.second) {
            auto it = remap.find(id);
            if (it != remap.end()) id = it->second;
        }
    // free ids are now exactly [target, max_blocks); keep the lowest on top of
    // the stack so the pool stays compact as it refills
    bm->free_blocks.clear();
    for (uint32_t i = bm->max_blocks; i > target; --i) bm->free_blocks.push_back(i - 1);
    return n;
}

}  // extern "C"

// ----------------------------------------------------------------- radix tree

namespace {

struct RNode {
    std::vector<uint32_t> edge, blocks;
    std::vector<std::pair<uint32_t, int32_t>> children;   // (first token, node), sorted
    int32_t parent = -1;
    uint64_t last = 0;
    uint32_t ref = 0;
    bool in_set = false;
    bool live = false;
};

}  // namespace

struct vw_radix {
    std::vector<RNode> nodes;
    std::vector<int32_t> spare;
    uint32_t block_size = 16, max_blocks = 0;
    uint64_t clock = 0, total = 0;
    std::set<std::pair<uint64_t, int32_t>> evictable;   // (last access, node)

    int32_t new_node() {
        int32_t i;
        if (!spare.empty()) { i = spare.back(); spare.pop_back(); nodes[i] = RNode(); }
        else { i = (int32_t)nodes.size(); nodes.emplace_back(); }
        nodes[i].live = true;
        return i;
    }
    bool can_evict(int32_t i) const {
        const RNode& n = nodes[i];
        return i != 0 && n.children.empty() && !n.blocks.empty() && n.ref == 0;
    }
    void refresh(int32_t i) {
        RNode& n = nodes[i];
        const bool e = can_evict(i);
        if (n.in_set && !e) { evictable.erase({n.last, i}); n.in_set = false; }
        else if (!n.in_set && e) { evictable.insert({n.last, i}); n.in_set = true; }
    }
    void touch(int32_t i) {
        RNode& n = nodes[i];
        const uint64_t now = ++clock;
        if (n.in_set && can_evict(i)) {
            // re-key the set's node in place (no allocation): the newest access
            // goes last
            auto nh = evictable.extract({n.last, i});
            nh.value() = {now, i};
            evictable.insert(evictable.end(), std::move(nh));
            n.last = now;
            return;
        }
        if (n.in_set) { evictable.erase({n.last, i}); n.in_set = false; }
        n.last = now;
        refresh(i);
    }
    int32_t child(int32_t i, uint32_t tok) const {
        const auto& c = nodes[i].children;
        auto it = std::lower_bound(c.begin(), c.end(), std::make_pair(tok, INT32_MIN));
        return (it != c.end() && it->first == tok) ? it->second : -1;
    }
    void set_child(int32_t i, uint32_t tok, int32_t node) {
        auto& c = nodes[i].children;
        auto it = std::lower_bound(c.begin(), c.end(), std::make_pair(tok, INT32_MIN));
        if (it != c.end() && it->first == tok) it->second = node;
        else c.insert(it, {tok, node});
        nodes[node].parent = i;
    }
    void drop_child(int32_t i, uint32_t tok) {
        auto& c = nodes[i].children;
        auto it = std::lower_bound(c.begin(), c.end(), std::make_pair(tok, INT32_MIN));
        if (it != c.end() && it->first == tok) c.erase(it);
    }
    static uint32_t common(const std::vector<uint32_t>& e, const uint32_t* t, uint32_t n) {
        uint32_t k = 0;
        while (k < e.size() && k < n && e[k] == t[k]) ++k;
        return k;
    }
    uint32_t evict_one(std::vector<uint32_t>* freed) {
        if (evictable.empty()) return 0;
        const int32_t i = evictable.begin()->second;
        evictable.erase(evictable.begin());
        RNode& n = nodes[i];
        n.in_set = false;
        const uint32_t k = (uint32_t)n.blocks.size();
        if (freed) freed->insert(freed->end(), n.blocks.begin(), n.blocks.end());
        total -= k;
        const int32_t par = n.parent;
        drop_child(par, n.edge[0]);
        n.live = false;
        n.blocks.clear();
        n.edge.clear();
        spare.push_back(i);
        refresh(par);
        return k;
    }
};

extern "C" {

int32_t vw_radix_create(uint32_t block_size, uint32_t max_blocks, vw_radix** out) {
    if (!out || block_size == 0) return VW_ERR_INVALID_ARG;
    vw_radix* r = new vw_radix();
    r->block_size = block_size;
    r->max_blocks = max_blocks;
    r->new_node();               // root = 0
    r->touch(0);
    *out = r;
    return VW_OK;
}

int32_t vw_radix_destroy(vw_radix* r) {
    delete r;
    return VW_OK;
}

uint32_t vw_radix_lookup(vw_radix* r, const uint32_t* tokens, uint32_t n, uint32_t* matched_len,
                         uint32_t* out, uint32_t cap) {
    // radix_cache.bm:77-108
    int32_t node = 0;
    uint32_t pos = 0, count = 0, matched = 0;
    for (;;) {
        r->touch(node);
        if (pos >= n) break;
        const int32_t c = r->child(node, tokens[pos]);
        if (c < 0) break;
        const uint32_t ml = vw_radix::common(r->nodes[c].edge, tokens + pos, n - pos);
        if (ml == 0) break;
        matched += ml;
        for (uint32_t id : r->nodes[c].blocks) {
            if (count < cap) out[count] = id;
            ++count;
        }
        r->touch(c);
        if (ml < r->nodes[c].edge.size()) break;
        pos += ml;
        node = c;
    }
    *matched_len = matched;
    return count;
}

uint32_t vw_radix_insert(vw_radix* r, const uint32_t* tokens, uint32_t n, const uint32_t* blocks,
                         uint32_t nb, uint32_t* freed_out, uint32_t cap) {
    // radix_cache.bm:111-179
    const uint32_t bs = r->block_size;
    int32_t node = 0;
    uint32_t pos = 0, blk = 0;
    while (pos < n && blk < nb) {
        const uint32_t first = tokens[pos];
        const int32_t c = r->child(node, first);
        if (c >= 0) {
            const uint32_t ml = vw_radix::common(r->nodes[c].edge, tokens + pos, n - pos);
            if (ml == r->nodes[c].edge.size()) {                     // :127-134
                r->touch(c);
                pos += ml;
                blk += (ml + bs - 1) / bs;
                node = c;
                continue;
            }
            // :136-167 split; the suffix keeps the old blocks, children, time, refs
            const int32_t sfx = r->new_node();
            RNode& C = r->nodes[c];
            RNode& S = r->nodes[sfx];
            S.edge.assign(C.edge.begin() + ml, C.edge.end());
            S.blocks = std::move(C.blocks);
            S.children = std::move(C.children);
            S.last = C.last;
            S.ref = C.ref;
            for (auto& ch : S.children) r->nodes[ch.second].parent = sfx;
            const uint32_t take = (ml + bs - 1) / bs;
            C.blocks.clear();
            for (uint32_t k = blk; k < nb && k < blk + take; ++k) C.blocks.push_back(blocks[k]);
            C.edge.resize(ml);
            C.children.clear();
            if (C.in_set) { r->evictable.erase({C.last, c}); C.in_set = false; }
            r->total += C.blocks.size();      // suffix keeps the old count; prefix adds new
            r->set_child(c, S.edge[0], sfx);
            r->refresh(sfx);
            r->touch(c);
            pos += ml;
            blk += take;
            node = c;
            continue;
        }
        // :170-177 new leaf holding one block
        const uint32_t chunk = std::min(bs, n - pos);
        const int32_t leaf = r->new_node();
        RNode& Lf = r->nodes[leaf];
        Lf.edge.assign(tokens + pos, tokens + pos + chunk);
        Lf.blocks.push_back(blocks[blk]);
        r->total += 1;
        r->set_child(node, first, leaf);
        r->refresh(node);
        r->touch(leaf);
        pos += chunk;
        blk += 1;
        node = leaf;
    }
    std::vector<uint32_t> freed;
    if (r->total > r->max_blocks) r->evict_one(&freed);               // :225-227
    for (uint32_t i = 0; i < freed.size() && i < cap; ++i) freed_out[i] = freed[i];
    return (uint32_t)freed.size();
}

uint32_t vw_radix_evict_lru(vw_radix* r, uint32_t target, uint32_t* freed_out, uint32_t cap) {
    // radix_cache.bm:231-240
    std::vector<uint32_t> freed;
    uint32_t total = 0;
    while (total < target) {
        const uint32_t e = r->evict_one(&freed);
        if (e == 0) break;
        total += e;
    }
    for (uint32_t i = 0; i < freed.size() && i < cap; ++i) freed_out[i] = freed[i];
    return total;
}

uint32_t vw_radix_total_blocks(const vw_radix* r) { return (uint32_t)r->total; }

static void radix_lock(vw_radix* r, const uint32_t* tokens, uint32_t n, int delta) {
    int32_t node = 0;
    uint32_t pos = 0;
    while (pos < n) {
        const int32_t c = r->child(node, tokens[pos]);
        if (c < 0) break;
        const uint32_t ml = vw_radix::common(r->nodes[c].edge, tokens + pos, n - pos);
        if (ml == 0) break;
        RNode& C = r->nodes[c];
        if (delta > 0) C.ref += 1; else if (C.ref > 0) C.ref -= 1;
        r->refresh(c);
        if (ml < C.edge.size()) break;
        pos += ml;
        node = c;
    }
}

void vw_radix_lock(vw_radix* r, const uint32_t* tokens, uint32_t n) { radix_lock(r, tokens, n, +1); }
void vw_radix_unlock(vw_radix* r, const uint32_t* tokens, uint32_t n) { radix_lock(r, tokens, n, -1); }

void vw_radix_remap(vw_radix* r, const uint32_t* pairs, uint32_t num_pairs) {
    std::unordered_map<uint32_t, uint32_t> m;
    for (uint32_t i = 0; i < num_pairs; ++i) m[pairs[2 * i]] = pairs[2 * i + 1];
    for (auto& nd : r->nodes) {
        if (!nd.live) continue;
        for (auto& id : nd.blocks) {
            auto it = m.find(id);
            if (it != m.end()) id = it->second;
        }
    }
}

}  // extern "C"
