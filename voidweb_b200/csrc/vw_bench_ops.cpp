// vw_bench_ops.cpp -- ns/op of the library's host block bookkeeping (the block
// manager of engine/kv_cache.bm and the radix tree of radix_cache/radix_cache.bm
// as vw_bm_* / vw_radix_* implement them), on the operations the reference's
// published micro-benchmark table lists (BENCHMARKS.md:118-135): one alloc, a
// 16-block alloc_seq and free_seq, a 16-block prefix lookup, a 256-token radix
// insert, a full-hit and a cold-miss radix lookup, one LRU eviction, and a
// 16-token rolling hash.  One thread; prints one JSON object.
//
//   vw_bench_ops [iterations]
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "../../include/voidweb_kv.h"

namespace {

using clk = std::chrono::steady_clock;

double ns_since(clk::time_point a, double n) {
    return std::chrono::duration<double, std::nano>(clk::now() - a).count() / n;
}

}  // namespace

int main(int argc, char** argv) {
    const uint32_t iters = argc > 1 ? (uint32_t)std::strtoul(argv[1], nullptr, 10) : 200000u;
    volatile uint64_t sink = 0;
    vw_block_manager* bm = nullptr;
    if (vw_bm_create(16, 1u << 16, &bm) != VW_OK) return 1;

    // one alloc and one free per round; the pair's time halved
    uint32_t id = 0;
    auto t0 = clk::now();
    for (uint32_t i = 0; i < iters; ++i) {
        vw_bm_alloc(bm, &id);
        vw_bm_decref(bm, id);
    }
    const double alloc_ns = ns_since(t0, iters) / 2.0;

    uint32_t ids[16];
    double a_ns = 0, f_ns = 0;
    for (uint32_t i = 0; i < iters; ++i) {
        auto a = clk::now();
        vw_bm_alloc_seq(bm, 16, ids);
        auto b = clk::now();
        vw_bm_free_seq(bm, ids, 16);
        auto c = clk::now();
        a_ns += std::chrono::duration<double, std::nano>(b - a).count();
        f_ns += std::chrono::duration<double, std::nano>(c - b).count();
    }

    // a registered 16-block prefix chain, looked up whole
    std::vector<uint32_t> toks(256);
    for (uint32_t i = 0; i < 256; ++i) toks[i] = (i * 2654435761u) % 151000u;
    uint64_t h = 0;
    for (uint32_t c = 0; c < 16; ++c) {
        vw_bm_alloc(bm, &id);
        h = vw_rolling_hash(h, &toks[c * 16], 16);
        vw_bm_register_prefix_block(bm, id, h);
    }
    uint32_t outids[64];
    t0 = clk::now();
    for (uint32_t i = 0; i < iters; ++i) sink += vw_bm_prefix_lookup(bm, toks.data(), 256, outids, 64);
    const double lookup_ns = ns_since(t0, iters);
    vw_bm_destroy(bm);

    // radix tree: 64 finished 256-token sequences sharing a 128-token prefix,
    // rebuilt every round so that the tree's size stays bounded
    std::vector<uint32_t> seq(toks), blocks(16);
    uint32_t freed[16], ml = 0, miss = 151001u;
    const uint32_t rounds = iters / 64 < 200 ? (iters / 64 ? iters / 64 : 1) : 200;
    double ins_ns = 0, hit_ns = 0, miss_ns = 0, ev_ns = 0;
    uint64_t ins_n = 0, hit_n = 0, miss_n = 0, ev_n = 0;
    for (uint32_t r = 0; r < rounds; ++r) {
        vw_radix* rx = nullptr;
        if (vw_radix_create(16, 1u << 30, &rx) != VW_OK) return 1;
        for (uint32_t i = 0; i < 64; ++i) {
            for (uint32_t k = 128; k < 256; ++k) seq[k] = (toks[k] + i * 7919u + k) % 151000u;
            for (uint32_t k = 0; k < 16; ++k) blocks[k] = i * 16 + k;
            auto a = clk::now();
            vw_radix_insert(rx, seq.data(), 256, blocks.data(), 16, freed, 16);
            ins_ns += std::chrono::duration<double, std::nano>(clk::now() - a).count();
            ++ins_n;
        }
        auto a = clk::now();
        for (uint32_t i = 0; i < 64; ++i) sink += vw_radix_lookup(rx, seq.data(), 256, &ml, outids, 64);
        hit_ns += std::chrono::duration<double, std::nano>(clk::now() - a).count();
        hit_n += 64;
        a = clk::now();
        for (uint32_t i = 0; i < 64; ++i) sink += vw_radix_lookup(rx, &miss, 1, &ml, outids, 64);
        miss_ns += std::chrono::duration<double, std::nano>(clk::now() - a).count();
        miss_n += 64;
        a = clk::now();
        for (uint32_t i = 0; i < 32; ++i) sink += vw_radix_evict_lru(rx, 1, freed, 16);
        ev_ns += std::chrono::duration<double, std::nano>(clk::now() - a).count();
        ev_n += 32;
        vw_radix_destroy(rx);
    }
    t0 = clk::now();
    for (uint32_t i = 0; i < iters; ++i) sink += vw_rolling_hash(i, toks.data(), 16);
    const double hash_ns = ns_since(t0, iters);
    std::printf(
        "{\"alloc\": %.1f, \"alloc_seq_16\": %.1f, \"free_seq_16\": %.1f, \"prefix_lookup_16\": %.1f, "
        "\"radix_insert_256\": %.1f, \"radix_lookup_hit\": %.1f, \"radix_lookup_miss\": %.1f, "
        "\"radix_evict_lru_1\": %.1f, \"rolling_hash_16\": %.1f}\n",
        alloc_ns, a_ns / iters, f_ns / iters, lookup_ns, ins_ns / ins_n, hit_ns / hit_n, miss_ns / miss_n,
        ev_ns / ev_n, hash_ns);
    return sink == 0xFFFFFFFFFFFFFFFFull ? 2 : 0;
}
