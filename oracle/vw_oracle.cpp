// vw_oracle.cpp -- CPU ORACLE for the paged KV-cache hot path.
//
// TEST INFRASTRUCTURE ONLY.  This file is the checker: only tests/, the
// smoke() entry of __graft_entry__.py and the cpu_baseline / reference arm of
// bench.py may load it.  The product (voidweb_b200/) never links or calls it.
//
// PARITY UNPINNED: the reference (VOIDWEB, written in the BlackMagic language)
// cannot be compiled in this environment (no `bmc` compiler) and ships no
// tests, golden vectors or fixtures.  This oracle is therefore a restatement
// of the reference source, function by function, with each function citing
// the reference file:line it follows.  It is cross-checked against a second,
// independent pure-Python transliteration (tests/golden/make_golden.py) whose
// outputs are committed as fixtures under tests/golden/.
//
// Reference citations are relative to the reference project root.
//
// Pool layout shared by oracle and product (the reference stores one head as
// kv_cache[TOTAL_BLOCKS][2][BLOCK_SIZE][HEAD_DIM], flash_attention.bm:116; the
// multi-layer, multi-head generalisation keeps that per-head [2][16][D] page
// and stacks heads, blocks and layers outside it):
//   data  [L][NB][Hkv][2][16][D]   element = f16 / bf16 (2 B) or E4M3 code (1 B)
//   scale [L][NB][Hkv][2][16]      f32, only for the FP8 pool
// Index 0 of the "2" axis is K, index 1 is V (flash_attention.bm:146,155).

#include <cmath>
#include <cstdint>
#include <cstring>
#include <cstdlib>
#include <algorithm>
#include <limits>
#include <map>
#include <memory>
#include <unordered_map>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

extern "C" {

// ---------------------------------------------------------------------------
// Scalar codecs
// ---------------------------------------------------------------------------

static inline uint32_t f2u(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }

// utils/simd.bm:149-151  bf16_to_f32: widen by shifting into the high half.
float vwo_bf16_to_f32(uint16_t x) { return u2f((uint32_t)x << 16); }

// utils/simd.bm:153-158  f32_to_bf16: round to nearest, ties to even, on the
// raw bits: (bits + 0x7FFF + ((bits >> 16) & 1)) >> 16.  No NaN special case
// (the reference has none); inputs here are finite.
uint16_t vwo_f32_to_bf16(float x) {
    uint32_t bits = f2u(x);
    uint32_t round = (bits >> 16) & 1u;
    return (uint16_t)((bits + 0x7FFFu + round) >> 16);
}

// IEEE binary16 conversions.  The reference casts with `as f16`
// (flash_attention.bm:53,104,146,161), i.e. IEEE round-to-nearest-even.
float vwo_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    if (exp == 0) {
        // zero or subnormal: man * 2^-24
        float v = std::ldexp((float)man, -24);
        return sign ? -v : v;
    }
    if (exp == 31) return u2f(sign | 0x7F800000u | (man << 13));
    return u2f(sign | ((exp + 112u) << 23) | (man << 13));
}

uint16_t vwo_f32_to_f16(float f) {
    uint32_t x = f2u(f);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax > 0x7F800000u) return sign | 0x7E00u;              // NaN
    if (ax >= 0x477FF000u) return sign | 0x7C00u;             // >= 65520 rounds to inf
    if (ax >= 0x38800000u) {                                  // normal binary16 range
        uint32_t r = ax - 0x38000000u;                        // rebias 127 -> 15
        r = (r + 0xFFFu + ((r >> 13) & 1u)) >> 13;
        return sign | (uint16_t)r;
    }
    // subnormal binary16 (or zero): round(|f| * 2^24) half-to-even
    float v = std::fabs(f) * 16777216.0f;                     // exact (power of two)
    float fl = std::floor(v);
    float rem = v - fl;
    uint32_t n = (uint32_t)fl;
    if (rem > 0.5f || (rem == 0.5f && (n & 1u))) n += 1;
    return sign | (uint16_t)n;                                // n == 1024 -> min normal
}

// kernels/norm/rms_norm.bm:98-113  f32_to_fp8_e4m3 ("reference codec"):
// clamp to +-448, then take sign, rebias the exponent by -127+7 and TRUNCATE
// the mantissa to its top 3 bits.  exp <= 0 flushes to 0x00 (sign lost);
// exp >= 15 saturates to sign|0x7F.
uint8_t vwo_fp8_encode_ref(float x) {
    const float FP8_MAX = 448.0f;
    float clamped = x < -FP8_MAX ? -FP8_MAX : (x > FP8_MAX ? FP8_MAX : x);
    uint32_t bits = f2u(clamped);
    uint8_t sign = (uint8_t)(bits >> 31);
    int32_t exp = (int32_t)((bits >> 23) & 0xFFu) - 127 + 7;
    uint8_t mant = (uint8_t)((bits >> 20) & 0x7u);
    if (exp <= 0) return 0u;
    if (exp >= 15) return (uint8_t)((sign << 7) | (0xF << 3) | 0x7);
    return (uint8_t)((sign << 7) | ((uint8_t)exp << 3) | mant);
}

// kernels/gemm/gemm_fp8.bm:110-116  fp8_to_f32: 0 -> 0, otherwise
// sign * (1 + m/8) * 2^(e-7).  No subnormals; 0x7F decodes to 480.
float vwo_fp8_decode_ref(uint8_t x) {
    if (x == 0) return 0.0f;
    float sign = (x >> 7) ? -1.0f : 1.0f;
    int32_t exp = (int32_t)((x >> 3) & 0xF) - 7;
    float mant = 1.0f + (float)(x & 0x7) / 8.0f;
    return sign * mant * std::ldexp(1.0f, exp);
}

// Optional non-default mode (no counterpart in the reference): OCP E4M3FN with
// round-to-nearest-even and saturation to +-448 (what `cvt.rn.satfinite` does).
uint8_t vwo_fp8_encode_ocp(float x) {
    uint32_t bits = f2u(x);
    uint8_t sign = (uint8_t)((bits >> 31) << 7);
    float a = std::fabs(x);
    if (std::isnan(x)) return 0x7F;
    if (a >= 464.0f) return sign | 0x7E;                      // saturate (448 + half ulp rounds up to 480 -> clamp)
    // value grid: normals e=1..15 (m 0..7) except 0x7F; subnormals m*2^-9
    if (a < std::ldexp(1.0f, -6)) {                           // subnormal range
        float v = a * 512.0f;                                 // units of 2^-9
        float fl = std::floor(v);
        float rem = v - fl;
        uint32_t n = (uint32_t)fl;
        if (rem > 0.5f || (rem == 0.5f && (n & 1u))) n += 1;
        return sign | (uint8_t)n;                             // n == 8 -> 0x08 = 2^-6
    }
    int e; float fr = std::frexp(a, &e);                      // a = fr * 2^e, fr in [0.5,1)
    int E = e - 1;                                            // a = (2fr) * 2^E
    float m = (2.0f * fr - 1.0f) * 8.0f;                      // in [0, 8)
    float fl = std::floor(m);
    float rem = m - fl;
    uint32_t n = (uint32_t)fl;
    if (rem > 0.5f || (rem == 0.5f && (n & 1u))) n += 1;
    if (n == 8) { n = 0; E += 1; }
    int ef = E + 7;
    if (ef > 15 || (ef == 15 && n == 7)) return sign | 0x7E;
    return sign | (uint8_t)((ef << 3) | n);
}

float vwo_fp8_decode_ocp(uint8_t x) {
    float sign = (x >> 7) ? -1.0f : 1.0f;
    uint32_t e = (x >> 3) & 0xF, m = x & 7;
    if (e == 15 && m == 7) return std::numeric_limits<float>::quiet_NaN();
    if (e == 0) return sign * std::ldexp((float)m, -9);
    return sign * (1.0f + (float)m / 8.0f) * std::ldexp(1.0f, (int)e - 7);
}

// Per-token-per-head quantisation (no reference counterpart; the north star
// defines it): amax over the row, scale = amax / 448 as one IEEE f32 division
// (amax == 0 -> scale = 1), code = encode(x / scale) with IEEE division.
void vwo_fp8_quant_row(const float* x, int n, int mode, uint8_t* codes, float* scale_out) {
    float amax = 0.0f;
    for (int i = 0; i < n; ++i) amax = std::max(amax, std::fabs(x[i]));
    float scale = amax == 0.0f ? 1.0f : amax / 448.0f;
    for (int i = 0; i < n; ++i) {
        float v = x[i] / scale;
        codes[i] = mode == 0 ? vwo_fp8_encode_ref(v) : vwo_fp8_encode_ocp(v);
    }
    *scale_out = scale;
}

float vwo_fp8_decode(uint8_t c, int mode) {
    return mode == 0 ? vwo_fp8_decode_ref(c) : vwo_fp8_decode_ocp(c);
}

// ---------------------------------------------------------------------------
// Pool geometry and byte-level ops (append / COW copy / move / gather)
// ---------------------------------------------------------------------------

enum { VWO_F16 = 0, VWO_BF16 = 1, VWO_FP8 = 2 };

typedef struct {
    uint32_t num_layers, num_kv_heads, head_dim, num_blocks;
    uint32_t kv_dtype;   // VWO_F16 / VWO_BF16 / VWO_FP8
    uint32_t io_dtype;   // VWO_F16 / VWO_BF16 (q, new rows, outputs)
    uint32_t fp8_mode;   // 0 = reference codec, 1 = OCP RNE satfinite
} vwo_geom;

static inline size_t elem_bytes(uint32_t dt) { return dt == VWO_FP8 ? 1 : 2; }

static inline size_t row_index(const vwo_geom* g, uint32_t l, uint32_t blk, uint32_t kv,
                               uint32_t h, uint32_t t) {
    return ((((size_t)l * g->num_blocks + blk) * g->num_kv_heads + h) * 2 + kv) * 16 + t;
}

static inline float io_to_f32(const void* p, size_t i, uint32_t io) {
    uint16_t v = ((const uint16_t*)p)[i];
    return io == VWO_BF16 ? vwo_bf16_to_f32(v) : vwo_f16_to_f32(v);
}

static inline uint16_t f32_to_io(float f, uint32_t io) {
    return io == VWO_BF16 ? vwo_f32_to_bf16(f) : vwo_f32_to_f16(f);
}

// Value of element d of row `row` (K or V) as the attention math sees it.
static inline float kv_value(const vwo_geom* g, const void* data, const float* scales,
                             size_t row, uint32_t d) {
    size_t i = row * g->head_dim + d;
    if (g->kv_dtype == VWO_FP8)
        return vwo_fp8_decode(((const uint8_t*)data)[i], (int)g->fp8_mode) * scales[row];
    return io_to_f32(data, i, g->kv_dtype);
}

// Reshape-and-cache.  The reference has no append kernel; its paging rule
// (flash_attention.bm:132-140: token p of a sequence lives in logical block
// p/16 at slot p%16) gives slot = block_table[p/16]*16 + p%16.  Each token's
// K and V rows for every KV head are bit-copied into that slot (or quantised
// per token per head for the FP8 pool).  A negative slot skips the token.
// k_new / v_new: [n][Hkv][D] in io dtype.
void vwo_kv_append(const vwo_geom* g, void* data, float* scales, uint32_t layer,
                   const void* k_new, const void* v_new, const int64_t* slots, uint32_t n) {
    const uint32_t H = g->num_kv_heads, D = g->head_dim;
    std::vector<float> row(D);
    for (uint32_t i = 0; i < n; ++i) {
        int64_t slot = slots[i];
        if (slot < 0) continue;
        uint32_t blk = (uint32_t)(slot / 16), t = (uint32_t)(slot % 16);
        for (uint32_t kv = 0; kv < 2; ++kv) {
            const void* src = kv == 0 ? k_new : v_new;
            for (uint32_t h = 0; h < H; ++h) {
                size_t r = row_index(g, layer, blk, kv, h, t);
                size_t s0 = ((size_t)i * H + h) * D;
                if (g->kv_dtype == VWO_FP8) {
                    for (uint32_t d = 0; d < D; ++d) row[d] = io_to_f32(src, s0 + d, g->io_dtype);
                    vwo_fp8_quant_row(row.data(), (int)D, (int)g->fp8_mode,
                                      (uint8_t*)data + r * D, &scales[r]);
                } else {
                    std::memcpy((uint16_t*)data + r * D, (const uint16_t*)src + s0, D * 2);
                }
            }
        }
    }
}

// Copy-on-write block copy / compaction move (no reference counterpart; the
// decision point is the ref-count in engine/kv_cache.bm:94-113).  For each
// (src, dst) pair, every layer's K and V rows of every head (and the FP8
// scales) of block src are copied to block dst.  Reads see the pool as it was
// before the call (pairs are applied from a snapshot).
void vwo_block_copy(const vwo_geom* g, void* data, float* scales, const uint32_t* pairs,
                    uint32_t n) {
    const size_t eb = elem_bytes(g->kv_dtype);
    const size_t per_layer_block = (size_t)2 * g->num_kv_heads * 16 * g->head_dim * eb;
    const size_t per_layer_scales = (size_t)2 * g->num_kv_heads * 16;
    std::vector<uint8_t> snap(per_layer_block * (size_t)n);
    std::vector<float> snaps(per_layer_scales * (size_t)n);
    for (uint32_t l = 0; l < g->num_layers; ++l) {
        for (uint32_t i = 0; i < n; ++i) {
            size_t off = ((size_t)l * g->num_blocks + pairs[2 * i]) * per_layer_block;
            std::memcpy(&snap[i * per_layer_block], (uint8_t*)data + off, per_layer_block);
            if (g->kv_dtype == VWO_FP8) {
                size_t so = ((size_t)l * g->num_blocks + pairs[2 * i]) * per_layer_scales;
                std::memcpy(&snaps[i * per_layer_scales], scales + so, per_layer_scales * 4);
            }
        }
        for (uint32_t i = 0; i < n; ++i) {
            size_t off = ((size_t)l * g->num_blocks + pairs[2 * i + 1]) * per_layer_block;
            std::memcpy((uint8_t*)data + off, &snap[i * per_layer_block], per_layer_block);
            if (g->kv_dtype == VWO_FP8) {
                size_t so = ((size_t)l * g->num_blocks + pairs[2 * i + 1]) * per_layer_scales;
                std::memcpy(scales + so, &snaps[i * per_layer_scales], per_layer_scales * 4);
            }
        }
    }
}

// Block-table gather of one sequence for one layer: contiguous raw rows
// out_k/out_v [Hkv][seq_len][D] (pool element type) and, for FP8, their
// scales out_ks/out_vs [Hkv][seq_len].  Follows the paging walk of
// flash_attention.bm:132-140.
void vwo_kv_gather(const vwo_geom* g, const void* data, const float* scales, uint32_t layer,
                   const uint32_t* block_table, uint32_t seq_len, void* out_k, void* out_v,
                   float* out_ks, float* out_vs) {
    const size_t eb = elem_bytes(g->kv_dtype);
    const uint32_t H = g->num_kv_heads, D = g->head_dim;
    for (uint32_t p = 0; p < seq_len; ++p) {
        uint32_t blk = block_table[p / 16], t = p % 16;
        for (uint32_t h = 0; h < H; ++h) {
            size_t rk = row_index(g, layer, blk, 0, h, t), rv = row_index(g, layer, blk, 1, h, t);
            size_t o = (size_t)h * seq_len + p;
            std::memcpy((uint8_t*)out_k + o * D * eb, (const uint8_t*)data + rk * D * eb, D * eb);
            std::memcpy((uint8_t*)out_v + o * D * eb, (const uint8_t*)data + rv * D * eb, D * eb);
            if (g->kv_dtype == VWO_FP8) { out_ks[o] = scales[rk]; out_vs[o] = scales[rv]; }
        }
    }
}

// ---------------------------------------------------------------------------
// Paged decode attention
// ---------------------------------------------------------------------------

// kernels/attention/flash_attention.bm:113-162 (paged_attention_decode),
// generalised to GQA: query head hq reads KV head hq / (Hq/Hkv).  Exact
// reference order in f32: per token, dot = sum_dd q*k accumulated in order
// (:144-147), s = dot*scale (:148), online softmax m/alpha/acc/l (:151-157),
// o = acc/l cast to the io type (:161).  q / out: [B][Hq][D] io dtype;
// block_tables: [B][bt_stride] u32.  Returns nonzero if any seq_len is 0
// (the reference would produce 0/0 = NaN there; this build rejects it).
int vwo_paged_decode_f32(const vwo_geom* g, const void* data, const float* scales,
                         uint32_t layer, const void* q, uint32_t Hq, const uint32_t* bt,
                         uint32_t bt_stride, const uint32_t* seq_lens, uint32_t B, float scale,
                         void* out, int nthreads) {
    const uint32_t H = g->num_kv_heads, D = g->head_dim, G = Hq / H;
    for (uint32_t b = 0; b < B; ++b) if (seq_lens[b] == 0) return 1;
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1)
#endif
    for (int64_t job = 0; job < (int64_t)B * Hq; ++job) {
        uint32_t b = (uint32_t)(job / Hq), hq = (uint32_t)(job % Hq), h = hq / G;
        std::vector<float> qf(D), acc(D, 0.0f), kr(D), vr(D);
        for (uint32_t d = 0; d < D; ++d) qf[d] = io_to_f32(q, ((size_t)b * Hq + hq) * D + d, g->io_dtype);
        float m = -std::numeric_limits<float>::infinity(), l = 0.0f;
        uint32_t seq_len = seq_lens[b];
        uint32_t num_blocks = (seq_len + 15) / 16;
        for (uint32_t blk = 0; blk < num_blocks; ++blk) {
            uint32_t phys = bt[(size_t)b * bt_stride + blk];
            uint32_t tokens = blk == num_blocks - 1 ? seq_len - blk * 16 : 16;
            for (uint32_t t = 0; t < tokens; ++t) {
                size_t rk = row_index(g, layer, phys, 0, h, t), rv = row_index(g, layer, phys, 1, h, t);
                float dot = 0.0f;
                for (uint32_t dd = 0; dd < D; ++dd) dot += qf[dd] * kv_value(g, data, scales, rk, dd);
                float s = dot * scale;
                float m_new = std::max(m, s);
                float exp_s = std::exp(s - m_new);
                float alpha = std::exp(m - m_new);
                for (uint32_t d = 0; d < D; ++d)
                    acc[d] = alpha * acc[d] + exp_s * kv_value(g, data, scales, rv, d);
                l = alpha * l + exp_s;
                m = m_new;
            }
        }
        uint16_t* o = (uint16_t*)out + ((size_t)b * Hq + hq) * D;
        for (uint32_t d = 0; d < D; ++d) o[d] = f32_to_io(acc[d] / l, g->io_dtype);
    }
    return 0;
}

// Same attention in fp64 with a two-pass softmax: the high-precision
// reference that tolerance checks compare against.  out: [B][Hq][D] f64.
int vwo_paged_decode_f64(const vwo_geom* g, const void* data, const float* scales,
                         uint32_t layer, const void* q, uint32_t Hq, const uint32_t* bt,
                         uint32_t bt_stride, const uint32_t* seq_lens, uint32_t B, double scale,
                         double* out, int nthreads) {
    const uint32_t H = g->num_kv_heads, D = g->head_dim, G = Hq / H;
    for (uint32_t b = 0; b < B; ++b) if (seq_lens[b] == 0) return 1;
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1)
#endif
    for (int64_t job = 0; job < (int64_t)B * Hq; ++job) {
        uint32_t b = (uint32_t)(job / Hq), hq = (uint32_t)(job % Hq), h = hq / G;
        uint32_t seq_len = seq_lens[b];
        std::vector<double> qf(D), s(seq_len), acc(D, 0.0);
        for (uint32_t d = 0; d < D; ++d) qf[d] = io_to_f32(q, ((size_t)b * Hq + hq) * D + d, g->io_dtype);
        double mx = -std::numeric_limits<double>::infinity();
        for (uint32_t p = 0; p < seq_len; ++p) {
            uint32_t phys = bt[(size_t)b * bt_stride + p / 16];
            size_t rk = row_index(g, layer, phys, 0, h, p % 16);
            double dot = 0.0;
            for (uint32_t d = 0; d < D; ++d) dot += qf[d] * (double)kv_value(g, data, scales, rk, d);
            s[p] = dot * scale;
            mx = std::max(mx, s[p]);
        }
        double den = 0.0;
        for (uint32_t p = 0; p < seq_len; ++p) {
            uint32_t phys = bt[(size_t)b * bt_stride + p / 16];
            size_t rv = row_index(g, layer, phys, 1, h, p % 16);
            double w = std::exp(s[p] - mx);
            den += w;
            for (uint32_t d = 0; d < D; ++d) acc[d] += w * (double)kv_value(g, data, scales, rv, d);
        }
        double* o = out + ((size_t)b * Hq + hq) * D;
        for (uint32_t d = 0; d < D; ++d) o[d] = acc[d] / den;
    }
    return 0;
}

// ---------------------------------------------------------------------------
// Paged prefill attention
// ---------------------------------------------------------------------------

// kernels/attention/flash_attention.bm:31-106 (flash_attention_fwd) over the
// pool: query token i of sequence b (rows cu_q[b] .. cu_q[b+1]-1 of q) sits
// at position p = ctx_start[b] + i - cu_q[b] and attends, with `causal`, to
// keys 0 .. p, else to all ctx_start[b] + n_b keys (the reference's seq_kv,
// no mask).  f32 in the reference's order: keys in tiles of BLOCK_KV = 64
// (:56-58), dot = sum_d q*k in order (:66-68), s = dot*scale (:69), per tile
// the online update of :80-96.  One change: the running maximum is
// max(m_i, tile max), where :80-81 take the tile max alone; the two agree
// after the final division unless a later tile's maximum is far below an
// earlier one (then the reference's alpha = exp(m_i - m_new) > 1 overflows),
// and with a causal mask a tile can hold no key of a row at all, which the
// reference's rule turns into 0/0.  q / out: [T][Hq][D] io dtype.  Returns
// nonzero for a chunk past its block table row.
int vwo_paged_prefill_f32(const vwo_geom* g, const void* data, const float* scales,
                          uint32_t layer, const void* q, uint32_t Hq, const int32_t* cu_q,
                          const int32_t* ctx_start, const uint32_t* bt, uint32_t bt_stride,
                          uint32_t B, int causal, float scale, void* out, int nthreads) {
    const uint32_t H = g->num_kv_heads, D = g->head_dim, G = Hq / H;
    for (uint32_t b = 0; b < B; ++b)
        if (ctx_start[b] < 0 || cu_q[b + 1] < cu_q[b] ||
            (int64_t)ctx_start[b] + cu_q[b + 1] - cu_q[b] > (int64_t)bt_stride * 16)
            return 1;
    const int64_t T = cu_q[B];
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1)
#endif
    for (int64_t job = 0; job < T * (int64_t)Hq; ++job) {
        const int64_t i = job / Hq;
        const uint32_t hq = (uint32_t)(job % Hq), h = hq / G;
        uint32_t b = 0;
        while (b + 1 < B && cu_q[b + 1] <= i) ++b;
        const int64_t p = ctx_start[b] + (i - cu_q[b]);
        const int64_t total = ctx_start[b] + (cu_q[b + 1] - cu_q[b]);
        const int64_t kend = causal ? p + 1 : total;
        std::vector<float> qf(D), acc(D, 0.0f), st(64);
        for (uint32_t d = 0; d < D; ++d) qf[d] = io_to_f32(q, ((size_t)i * Hq + hq) * D + d, g->io_dtype);
        float m = -std::numeric_limits<float>::infinity(), l = 0.0f;
        for (int64_t k0 = 0; k0 < kend; k0 += 64) {
            float tmax = -std::numeric_limits<float>::infinity();
            for (int64_t kv = 0; kv < 64; ++kv) {
                const int64_t key = k0 + kv;
                if (key >= kend) { st[kv] = -std::numeric_limits<float>::infinity(); continue; }
                const uint32_t phys = bt[(size_t)b * bt_stride + key / 16];
                const size_t rk = row_index(g, layer, phys, 0, h, (uint32_t)(key % 16));
                float dot = 0.0f;
                for (uint32_t d = 0; d < D; ++d) dot += qf[d] * kv_value(g, data, scales, rk, d);
                st[kv] = dot * scale;
                tmax = std::max(tmax, st[kv]);
            }
            const float m_new = std::max(m, tmax);
            float exp_sum = 0.0f;
            for (int64_t kv = 0; kv < 64; ++kv) exp_sum += std::exp(st[kv] - m_new);
            const float alpha = std::exp(m - m_new);
            for (uint32_t d = 0; d < D; ++d) {
                float a = 0.0f;
                for (int64_t kv = 0; kv < 64; ++kv) {
                    const int64_t key = k0 + kv;
                    if (key >= kend) continue;
                    const uint32_t phys = bt[(size_t)b * bt_stride + key / 16];
                    const size_t rv = row_index(g, layer, phys, 1, h, (uint32_t)(key % 16));
                    a += std::exp(st[kv] - m_new) * kv_value(g, data, scales, rv, d);
                }
                acc[d] = acc[d] * alpha + a;
            }
            l = alpha * l + exp_sum;
            m = m_new;
        }
        uint16_t* o = (uint16_t*)out + ((size_t)i * Hq + hq) * D;
        for (uint32_t d = 0; d < D; ++d) o[d] = f32_to_io(acc[d] / l, g->io_dtype);
    }
    return 0;
}

// Same attention in fp64 with a two-pass softmax (the tolerance reference).
// out: [T][Hq][D] f64.
int vwo_paged_prefill_f64(const vwo_geom* g, const void* data, const float* scales,
                          uint32_t layer, const void* q, uint32_t Hq, const int32_t* cu_q,
                          const int32_t* ctx_start, const uint32_t* bt, uint32_t bt_stride,
                          uint32_t B, int causal, double scale, double* out, int nthreads) {
    const uint32_t H = g->num_kv_heads, D = g->head_dim, G = Hq / H;
    for (uint32_t b = 0; b < B; ++b)
        if (ctx_start[b] < 0 || cu_q[b + 1] < cu_q[b] ||
            (int64_t)ctx_start[b] + cu_q[b + 1] - cu_q[b] > (int64_t)bt_stride * 16)
            return 1;
    const int64_t T = cu_q[B];
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1)
#endif
    for (int64_t job = 0; job < T * (int64_t)Hq; ++job) {
        const int64_t i = job / Hq;
        const uint32_t hq = (uint32_t)(job % Hq), h = hq / G;
        uint32_t b = 0;
        while (b + 1 < B && cu_q[b + 1] <= i) ++b;
        const int64_t p = ctx_start[b] + (i - cu_q[b]);
        const int64_t total = ctx_start[b] + (cu_q[b + 1] - cu_q[b]);
        const int64_t kend = causal ? p + 1 : total;
        std::vector<double> qf(D), sc((size_t)kend), acc(D, 0.0);
        for (uint32_t d = 0; d < D; ++d) qf[d] = io_to_f32(q, ((size_t)i * Hq + hq) * D + d, g->io_dtype);
        double mx = -std::numeric_limits<double>::infinity();
        for (int64_t key = 0; key < kend; ++key) {
            const uint32_t phys = bt[(size_t)b * bt_stride + key / 16];
            const size_t rk = row_index(g, layer, phys, 0, h, (uint32_t)(key % 16));
            double dot = 0.0;
            for (uint32_t d = 0; d < D; ++d) dot += qf[d] * (double)kv_value(g, data, scales, rk, d);
            sc[key] = dot * scale;
            mx = std::max(mx, sc[key]);
        }
        double den = 0.0;
        for (int64_t key = 0; key < kend; ++key) {
            const uint32_t phys = bt[(size_t)b * bt_stride + key / 16];
            const size_t rv = row_index(g, layer, phys, 1, h, (uint32_t)(key % 16));
            const double w = std::exp(sc[key] - mx);
            den += w;
            for (uint32_t d = 0; d < D; ++d) acc[d] += w * (double)kv_value(g, data, scales, rv, d);
        }
        double* o = out + ((size_t)i * Hq + hq) * D;
        for (uint32_t d = 0; d < D; ++d) o[d] = acc[d] / den;
    }
    return 0;
}

// ---------------------------------------------------------------------------
// FP8 weight path (kernels/norm/rms_norm.bm:62-94, kernels/gemm/gemm_fp8.bm:31-107)
// ---------------------------------------------------------------------------

// rms_norm_fp8_out (rms_norm.bm:62-94) for `rows` rows of `hidden` f16 values:
// one warp per row in the reference, so the sum of squares is restated in
// its order -- lane l sums x[l], x[l+32], ... in f32 (:73-77), then the
// butterfly shuffles add the partner lane's sum at distances 16, 8, 4, 2, 1
// (:79-83; every lane ends with the same value) -- then
// inv_rms = 1 / sqrt(sum / hidden + eps) (:85) and each element
// ((x * inv_rms) * w) * scale (:90, left to right) goes through the reference
// encoder (:98-113).  x, weight: f16 bits; out: E4M3 codes.
void vwo_rms_norm_fp8_out(const uint16_t* x, const uint16_t* weight, uint32_t rows,
                          uint32_t hidden, float scale, float eps, uint8_t* out) {
    for (uint32_t r = 0; r < rows; ++r) {
        const uint16_t* xr = x + (size_t)r * hidden;
        float part[32];
        for (uint32_t l = 0; l < 32; ++l) {
            float acc = 0.0f;
            for (uint32_t d = l; d < hidden; d += 32) {
                const float v = vwo_f16_to_f32(xr[d]);
                acc += v * v;
            }
            part[l] = acc;
        }
        for (uint32_t off = 16; off >= 1; off >>= 1) {
            float nxt[32];
            for (uint32_t l = 0; l < 32; ++l) nxt[l] = part[l] + part[l ^ off];
            std::memcpy(part, nxt, sizeof part);
        }
        const float inv_rms = 1.0f / std::sqrt(part[0] / (float)hidden + eps);
        for (uint32_t d = 0; d < hidden; ++d) {
            const float v = vwo_f16_to_f32(xr[d]), w = vwo_f16_to_f32(weight[d]);
            const float normed = v * inv_rms * w * scale;
            out[(size_t)r * hidden + d] = vwo_fp8_encode_ref(normed);
        }
    }
}

// gemm_fp8 (gemm_fp8.bm:31-107) in f64: C[m][n] = (a_scale * b_scale) *
// sum_k dec(A[m][k]) dec(B[k][n]) + bias[n], dec = the reference decoder
// (:110-116), A [M][K] and B [K][N] E4M3 codes row-major, bias and the result
// C f64 [M][N] (the tolerance reference; the reference rounds C to bf16).
void vwo_gemm_fp8_f64(const uint8_t* a, const uint8_t* b, const uint16_t* bias_bf16, uint32_t M,
                      uint32_t N, uint32_t K, float a_scale, float b_scale, double* c, int nthreads) {
    float dec[256];
    for (int i = 0; i < 256; ++i) dec[i] = vwo_fp8_decode_ref((uint8_t)i);
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(static)
#endif
    for (int64_t m = 0; m < (int64_t)M; ++m) {
        std::vector<double> acc(N, 0.0);
        for (uint32_t k = 0; k < K; ++k) {
            const double av = dec[a[(size_t)m * K + k]];
            if (av == 0.0) continue;
            const uint8_t* brow = b + (size_t)k * N;
            for (uint32_t n = 0; n < N; ++n) acc[n] += av * dec[brow[n]];
        }
        const double sc = (double)(a_scale * b_scale);
        for (uint32_t n = 0; n < N; ++n)
            c[(size_t)m * N + n] = acc[n] * sc + (bias_bf16 ? (double)vwo_bf16_to_f32(bias_bf16[n]) : 0.0);
    }
}

// ---------------------------------------------------------------------------
// BlockManager  (engine/kv_cache.bm:29-164)
// ---------------------------------------------------------------------------

struct OPage { uint32_t block_id; uint16_t used_slots; uint32_t ref_count; uint64_t token_hash; };

struct OBlockManager {
    uint32_t block_size;
    std::vector<uint32_t> free_blocks;                       // kv_cache.bm:35
    std::unordered_map<uint32_t, OPage> used_blocks;         // kv_cache.bm:36
    std::unordered_map<uint64_t, std::vector<uint32_t>> prefix_cache;  // kv_cache.bm:37
};

// kv_cache.bm:157-164 rolling_hash: h = prev + len*P, then h = h*P + t
// (wrapping u64), P = 0x9e3779b97f4a7c15.
// Rotary position embedding in place on x [n][H][D] (io dtype bits), token i at
// position pos[i]: kernels/rope/rope.bm:22-52.  For each pair (d, d + D/2):
// freq = 1 / theta^(2d / D), angle = freq * pos, (x_r, x_i) ->
// (x_r cos - x_i sin, x_r sin + x_i cos) in f32 (no contraction: this file is
// built with -ffp-contract=off), stored back rounded to the io type (:48-49).
void vwo_rope_apply(void* x, uint32_t n, uint32_t H, uint32_t D, const uint32_t* pos,
                    float theta, uint32_t io) {
    const uint32_t half = D / 2;
    for (uint32_t i = 0; i < n; ++i)
        for (uint32_t h = 0; h < H; ++h)
            for (uint32_t d = 0; d < half; ++d) {
                const float freq = 1.0f / std::pow(theta, 2.0f * (float)d / (float)D);
                const float angle = freq * (float)pos[i];
                const float s = std::sin(angle), c = std::cos(angle);
                const size_t base = ((size_t)i * H + h) * D;
                const float xr = io_to_f32(x, base + d, io), xi = io_to_f32(x, base + d + half, io);
                static_cast<uint16_t*>(x)[base + d] = f32_to_io(xr * c - xi * s, io);
                static_cast<uint16_t*>(x)[base + d + half] = f32_to_io(xr * s + xi * c, io);
            }
}

uint64_t vwo_rolling_hash(uint64_t prev, const uint32_t* tokens, uint32_t n) {
    const uint64_t P = 0x9e3779b97f4a7c15ull;
    uint64_t h = prev + (uint64_t)n * P;
    for (uint32_t i = 0; i < n; ++i) h = h * P + (uint64_t)tokens[i];
    return h;
}

// kv_cache.bm:41-58: free list is 0..max_blocks in ascending order.
void* vwo_bm_new(uint32_t block_size, uint32_t max_blocks) {
    OBlockManager* bm = new OBlockManager();
    bm->block_size = block_size;
    bm->free_blocks.resize(max_blocks);
    for (uint32_t i = 0; i < max_blocks; ++i) bm->free_blocks[i] = i;
    return bm;
}
void vwo_bm_delete(void* p) { delete (OBlockManager*)p; }
uint32_t vwo_bm_capacity(void* p) {                            // kv_cache.bm:60-62
    OBlockManager* bm = (OBlockManager*)p;
    return (uint32_t)(bm->free_blocks.size() + bm->used_blocks.size());
}
uint32_t vwo_bm_free_count(void* p) { return (uint32_t)((OBlockManager*)p)->free_blocks.size(); }

// kv_cache.bm:69-78: pop from the END of the free list (LIFO), ref_count 1.
int64_t vwo_bm_alloc(void* p) {
    OBlockManager* bm = (OBlockManager*)p;
    if (bm->free_blocks.empty()) return -1;
    uint32_t id = bm->free_blocks.back();
    bm->free_blocks.pop_back();
    bm->used_blocks[id] = OPage{id, 0, 1, 0};
    return id;
}

// kv_cache.bm:81-91: all-or-nothing OOM check, then n single allocs.
int32_t vwo_bm_alloc_seq(void* p, uint32_t n, uint32_t* out) {
    OBlockManager* bm = (OBlockManager*)p;
    if (bm->free_blocks.size() < n) return 1;
    for (uint32_t i = 0; i < n; ++i) out[i] = (uint32_t)vwo_bm_alloc(p);
    return 0;
}

// kv_cache.bm:94-98: unknown ids are ignored.
void vwo_bm_incref(void* p, uint32_t id) {
    OBlockManager* bm = (OBlockManager*)p;
    auto it = bm->used_blocks.find(id);
    if (it != bm->used_blocks.end()) it->second.ref_count += 1;
}

// kv_cache.bm:101-113: saturating decrement; at 0 the block is removed from
// the used map and pushed on the END of the free list.
void vwo_bm_decref(void* p, uint32_t id) {
    OBlockManager* bm = (OBlockManager*)p;
    auto it = bm->used_blocks.find(id);
    if (it == bm->used_blocks.end()) return;
    if (it->second.ref_count > 0) it->second.ref_count -= 1;
    if (it->second.ref_count == 0) {
        bm->used_blocks.erase(it);
        bm->free_blocks.push_back(id);
    }
}

// kv_cache.bm:116-120
void vwo_bm_free_seq(void* p, const uint32_t* table, uint32_t n) {
    for (uint32_t i = 0; i < n; ++i) vwo_bm_decref(p, table[i]);
}

// Ref count of a block (0 when the block is free).
uint32_t vwo_bm_ref_count(void* p, uint32_t id) {
    OBlockManager* bm = (OBlockManager*)p;
    auto it = bm->used_blocks.find(id);
    return it == bm->used_blocks.end() ? 0 : it->second.ref_count;
}

// kv_cache.bm:127-138: hash chunk by chunk (the last chunk may be partial),
// append every cached id list, stop at the first miss.  Returns the number of
// ids (written up to cap).
uint32_t vwo_bm_prefix_lookup(void* p, const uint32_t* tokens, uint32_t n, uint32_t* out,
                              uint32_t cap) {
    OBlockManager* bm = (OBlockManager*)p;
    uint32_t count = 0;
    uint64_t hash = 0;
    for (uint32_t off = 0; off < n; off += bm->block_size) {
        uint32_t len = std::min(bm->block_size, n - off);
        hash = vwo_rolling_hash(hash, tokens + off, len);
        auto it = bm->prefix_cache.find(hash);
        if (it == bm->prefix_cache.end()) break;
        for (uint32_t id : it->second) { if (count < cap) out[count] = id; ++count; }
    }
    return count;
}

// kv_cache.bm:142-151: record the hash on the page (if used), append the id
// to the hash's list (duplicates accumulate), then incref.
void vwo_bm_register_prefix_block(void* p, uint32_t id, uint64_t token_hash) {
    OBlockManager* bm = (OBlockManager*)p;
    auto it = bm->used_blocks.find(id);
    if (it != bm->used_blocks.end()) it->second.token_hash = token_hash;
    bm->prefix_cache[token_hash].push_back(id);
    vwo_bm_incref(p, id);
}

// Free list snapshot (order matters: the next alloc pops the last entry).
uint32_t vwo_bm_free_list(void* p, uint32_t* out, uint32_t cap) {
    OBlockManager* bm = (OBlockManager*)p;
    uint32_t n = (uint32_t)bm->free_blocks.size();
    for (uint32_t i = 0; i < n && i < cap; ++i) out[i] = bm->free_blocks[i];
    return n;
}

// ---------------------------------------------------------------------------
// Radix prefix tree  (radix_cache/radix_cache.bm:27-285)
//
// Deliberate, documented divergences (the reference's eviction cannot work):
//  * timestamps come from a logical clock incremented on every touch, not
//    wall-clock microseconds (radix_cache.bm:41,46-48), so runs are
//    deterministic and no two touches tie;
//  * children are kept in an ordered map (first-token order) instead of a
//    HashMap; with unique timestamps the LRU choice does not depend on it;
//  * clear_leaf_at walks the path edge by edge (the reference walks it token
//    by token against first-token keys, radix_cache.bm:278-281, which fails
//    for any edge longer than one token), returns the freed ids, and removes
//    the emptied leaf from its parent so the parent can become evictable;
//  * lock/unlock add and drop one reference on every node of a matched path
//    (ref_count is never incremented in the reference).
// ---------------------------------------------------------------------------

struct ONode {
    std::vector<uint32_t> edge, blocks;
    std::map<uint32_t, std::unique_ptr<ONode>> children;
    uint64_t last_access = 0;
    uint32_t ref_count = 0;
};

struct ORadix {
    ONode root;
    uint32_t block_size, max_blocks;
    uint64_t clock = 0;
    void touch(ONode* n) { n->last_access = ++clock; }
};

void* vwo_radix_new(uint32_t block_size, uint32_t max_blocks) {
    ORadix* r = new ORadix();
    r->block_size = block_size;
    r->max_blocks = max_blocks;
    r->touch(&r->root);
    return r;
}
void vwo_radix_delete(void* p) { delete (ORadix*)p; }

static uint32_t common_len(const std::vector<uint32_t>& edge, const uint32_t* rem, uint32_t n) {
    uint32_t k = 0;
    while (k < edge.size() && k < n && edge[k] == rem[k]) ++k;
    return k;
}

// radix_cache.bm:77-108 RadixTree::lookup.  Note the reference appends all of
// a child's blocks even on a partial edge match (:97-101).
uint32_t vwo_radix_lookup(void* p, const uint32_t* tokens, uint32_t n, uint32_t* matched_len,
                          uint32_t* out, uint32_t cap) {
    ORadix* r = (ORadix*)p;
    ONode* node = &r->root;
    uint32_t pos = 0, count = 0, matched = 0;
    for (;;) {
        r->touch(node);
        if (pos >= n) break;
        auto it = node->children.find(tokens[pos]);
        if (it == node->children.end()) break;
        ONode* child = it->second.get();
        uint32_t ml = common_len(child->edge, tokens + pos, n - pos);
        if (ml == 0) break;
        matched += ml;
        for (uint32_t id : child->blocks) { if (count < cap) out[count] = id; ++count; }
        r->touch(child);
        if (ml < child->edge.size()) break;
        pos += ml;
        node = child;
    }
    *matched_len = matched;
    return count;
}

static uint32_t count_blocks(const ONode* n) {                 // radix_cache.bm:186-192
    uint32_t c = (uint32_t)n->blocks.size();
    for (auto& kv : n->children) c += count_blocks(kv.second.get());
    return c;
}
uint32_t vwo_radix_total_blocks(void* p) { return count_blocks(&((ORadix*)p)->root); }

// radix_cache.bm:256-274 find_oldest_leaf (DFS; strict '<' on last_access).
static void find_oldest(const ONode* node, std::vector<uint32_t>& path, uint64_t* oldest,
                        std::vector<uint32_t>* oldest_path) {
    if (node->children.empty() && !node->blocks.empty() && node->ref_count == 0) {
        if (node->last_access < *oldest) { *oldest = node->last_access; *oldest_path = path; }
        return;
    }
    for (auto& kv : node->children) {
        const ONode* c = kv.second.get();
        size_t mark = path.size();
        path.insert(path.end(), c->edge.begin(), c->edge.end());
        find_oldest(c, path, oldest, oldest_path);
        path.resize(mark);
    }
}

// radix_cache.bm:246-254 evict_one + :276-285 clear_leaf_at (edge walk fix).
static uint32_t evict_one(ORadix* r, std::vector<uint32_t>* freed) {
    uint64_t oldest = std::numeric_limits<uint64_t>::max();
    std::vector<uint32_t> path, opath;
    find_oldest(&r->root, path, &oldest, &opath);
    if (opath.empty()) return 0;
    ONode* parent = nullptr;
    ONode* node = &r->root;
    size_t pos = 0;
    while (pos < opath.size()) {
        auto it = node->children.find(opath[pos]);
        if (it == node->children.end()) return 0;
        parent = node;
        node = it->second.get();
        pos += node->edge.size();
    }
    uint32_t n = (uint32_t)node->blocks.size();
    if (freed) freed->insert(freed->end(), node->blocks.begin(), node->blocks.end());
    node->blocks.clear();
    if (parent && node->children.empty()) parent->children.erase(node->edge[0]);
    return n;
}

// radix_cache.bm:111-179 RadixTree::insert, then :225-227 (evict one LRU leaf
// when over budget).  Ids freed by that eviction are written to freed_out.
uint32_t vwo_radix_insert(void* p, const uint32_t* tokens, uint32_t n, const uint32_t* blocks,
                          uint32_t nb, uint32_t* freed_out, uint32_t cap) {
    ORadix* r = (ORadix*)p;
    const uint32_t bs = r->block_size;
    ONode* node = &r->root;
    uint32_t pos = 0, blk = 0;
    while (pos < n && blk < nb) {
        const uint32_t* rem = tokens + pos;
        uint32_t rem_n = n - pos;
        uint32_t first = rem[0];
        auto it = node->children.find(first);
        if (it != node->children.end()) {
            ONode* child = it->second.get();
            std::vector<uint32_t> edge = child->edge;
            uint32_t ml = common_len(edge, rem, rem_n);
            if (ml == edge.size()) {                          // :127-134 full edge match
                r->touch(child);
                pos += ml;
                blk += (ml + bs - 1) / bs;
                node = child;
                continue;
            }
            // :136-167 split: suffix keeps old blocks/children/time/refs;
            // the prefix node takes the INSERTING sequence's blocks.
            std::unique_ptr<ONode> suffix(new ONode());
            suffix->edge.assign(edge.begin() + ml, edge.end());
            suffix->blocks = child->blocks;
            suffix->children = std::move(child->children);
            suffix->last_access = child->last_access;
            suffix->ref_count = child->ref_count;
            uint32_t old_first = suffix->edge[0];
            std::vector<uint32_t> split_blocks;
            uint32_t take = (ml + bs - 1) / bs;
            for (uint32_t k = blk; k < nb && k < blk + take; ++k) split_blocks.push_back(blocks[k]);
            child->edge.assign(edge.begin(), edge.begin() + ml);
            child->blocks = split_blocks;
            child->children.clear();
            child->children[old_first] = std::move(suffix);
            r->touch(child);
            pos += ml;
            blk += take;
            node = child;
            continue;
        }
        // :170-177 new leaf of at most one block's worth of tokens
        uint32_t chunk = std::min(bs, rem_n);
        std::unique_ptr<ONode> leaf(new ONode());
        leaf->edge.assign(rem, rem + chunk);
        leaf->blocks.push_back(blocks[blk]);
        r->touch(leaf.get());
        ONode* lp = leaf.get();
        node->children[first] = std::move(leaf);
        pos += chunk;
        blk += 1;
        node = lp;
    }
    std::vector<uint32_t> freed;
    if (count_blocks(&r->root) > r->max_blocks) evict_one(r, &freed);
    for (uint32_t i = 0; i < freed.size() && i < cap; ++i) freed_out[i] = freed[i];
    return (uint32_t)freed.size();
}

// radix_cache.bm:231-240 evict_lru: evict leaves until target ids are freed
// or nothing is evictable.  Freed ids go to freed_out (up to cap); returns
// the number freed.
uint32_t vwo_radix_evict_lru(void* p, uint32_t target, uint32_t* freed_out, uint32_t cap) {
    ORadix* r = (ORadix*)p;
    std::vector<uint32_t> freed;
    uint32_t total = 0;
    while (total < target) {
        uint32_t e = evict_one(r, &freed);
        if (e == 0) break;
        total += e;
    }
    for (uint32_t i = 0; i < freed.size() && i < cap; ++i) freed_out[i] = freed[i];
    return total;
}

// Lock / unlock every node on the longest matched path (adds the ref_count
// bookkeeping the reference declares but never maintains, radix_cache.bm:32).
static void lock_path(ORadix* r, const uint32_t* tokens, uint32_t n, int delta) {
    ONode* node = &r->root;
    uint32_t pos = 0;
    while (pos < n) {
        auto it = node->children.find(tokens[pos]);
        if (it == node->children.end()) break;
        ONode* c = it->second.get();
        uint32_t ml = common_len(c->edge, tokens + pos, n - pos);
        if (ml == 0) break;
        if (delta > 0) c->ref_count += 1; else if (c->ref_count > 0) c->ref_count -= 1;
        if (ml < c->edge.size()) break;
        pos += ml;
        node = c;
    }
}
void vwo_radix_lock(void* p, const uint32_t* tokens, uint32_t n) { lock_path((ORadix*)p, tokens, n, +1); }
void vwo_radix_unlock(void* p, const uint32_t* tokens, uint32_t n) { lock_path((ORadix*)p, tokens, n, -1); }

}  // extern "C"

// ---------------------------------------------------------------------------
// CPU baseline timing of the reference's block bookkeeping (the operations
// the reference's benchmark table lists: BENCHMARKS.md:118-135), single
// thread, ns per operation.  out[0..8] = alloc single, alloc_seq(16),
// free_seq(16), prefix_lookup(16-block chain), radix insert(256 tokens),
// radix lookup full hit, radix lookup cold miss, radix evict_lru(1 leaf),
// rolling_hash(16 tokens).
// ---------------------------------------------------------------------------
#include <chrono>
extern "C" void vwo_bench_block_ops(uint32_t iters, double* out) {
    using clk = std::chrono::steady_clock;
    auto ns = [](clk::time_point a, clk::time_point b, double n) {
        return std::chrono::duration<double, std::nano>(b - a).count() / n;
    };
    volatile uint64_t sink = 0;
    void* bm = vwo_bm_new(16, 1u << 16);
    auto t0 = clk::now();
    for (uint32_t i = 0; i < iters; ++i) { int64_t id = vwo_bm_alloc(bm); vwo_bm_decref(bm, (uint32_t)id); }
    out[0] = ns(t0, clk::now(), iters) / 2.0;           // one alloc (+ one free, halved)
    uint32_t ids[16];
    double a_ns = 0, f_ns = 0;
    for (uint32_t i = 0; i < iters; ++i) {
        auto a = clk::now(); vwo_bm_alloc_seq(bm, 16, ids); auto b = clk::now();
        vwo_bm_free_seq(bm, ids, 16); auto c = clk::now();
        a_ns += std::chrono::duration<double, std::nano>(b - a).count();
        f_ns += std::chrono::duration<double, std::nano>(c - b).count();
    }
    out[1] = a_ns / iters; out[2] = f_ns / iters;
    std::vector<uint32_t> toks(256);
    for (uint32_t i = 0; i < 256; ++i) toks[i] = (i * 2654435761u) % 151000u;
    uint64_t h = 0;
    for (uint32_t c = 0; c < 16; ++c) {
        int64_t id = vwo_bm_alloc(bm);
        h = vwo_rolling_hash(h, &toks[c * 16], 16);
        vwo_bm_register_prefix_block(bm, (uint32_t)id, h);
    }
    uint32_t outids[64];
    t0 = clk::now();
    for (uint32_t i = 0; i < iters; ++i) sink += vwo_bm_prefix_lookup(bm, toks.data(), 256, outids, 64);
    out[3] = ns(t0, clk::now(), iters);
    vwo_bm_delete(bm);
    // radix: a cache of 64 finished 256-token sequences sharing a 128-token
    // prefix, rebuilt every round so the tree size stays bounded (the
    // reference's insert recounts the whole tree, radix_cache.bm:225)
    std::vector<uint32_t> seq(toks), blocks(16);
    uint32_t freed[16], ml = 0;
    const uint32_t rounds = iters / 64 < 200 ? (iters / 64 ? iters / 64 : 1) : 200;
    double ins_ns = 0, hit_ns = 0, miss_ns = 0, ev_ns = 0;
    uint64_t ins_n = 0, hit_n = 0, miss_n = 0, ev_n = 0;
    uint32_t miss = 151001u;
    for (uint32_t r = 0; r < rounds; ++r) {
        void* rx = vwo_radix_new(16, 1u << 30);
        for (uint32_t i = 0; i < 64; ++i) {
            for (uint32_t k = 128; k < 256; ++k) seq[k] = (toks[k] + i * 7919u + k) % 151000u;
            for (uint32_t k = 0; k < 16; ++k) blocks[k] = i * 16 + k;
            auto a = clk::now();
            vwo_radix_insert(rx, seq.data(), 256, blocks.data(), 16, freed, 16);
            ins_ns += std::chrono::duration<double, std::nano>(clk::now() - a).count();
            ++ins_n;
        }
        auto a = clk::now();
        for (uint32_t i = 0; i < 64; ++i) sink += vwo_radix_lookup(rx, seq.data(), 256, &ml, outids, 64);
        hit_ns += std::chrono::duration<double, std::nano>(clk::now() - a).count(); hit_n += 64;
        a = clk::now();
        for (uint32_t i = 0; i < 64; ++i) sink += vwo_radix_lookup(rx, &miss, 1, &ml, outids, 64);
        miss_ns += std::chrono::duration<double, std::nano>(clk::now() - a).count(); miss_n += 64;
        a = clk::now();
        for (uint32_t i = 0; i < 32; ++i) sink += vwo_radix_evict_lru(rx, 1, freed, 16);
        ev_ns += std::chrono::duration<double, std::nano>(clk::now() - a).count(); ev_n += 32;
        vwo_radix_delete(rx);
    }
    out[4] = ins_ns / ins_n; out[5] = hit_ns / hit_n; out[6] = miss_ns / miss_n; out[7] = ev_ns / ev_n;
    t0 = clk::now();
    uint64_t hh = 0;
    for (uint32_t i = 0; i < iters; ++i) hh = vwo_rolling_hash(hh, &toks[(i & 7) * 16], 16);
    out[8] = ns(t0, clk::now(), iters);
    sink += hh;
}
