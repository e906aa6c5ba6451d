// mrl_oracle.cpp — TEST INFRASTRUCTURE ONLY (the checker, never the product).
//
// CPU restatement of the reference crate `mrl_index` v0.3.5 PaxBlock64 scan path. Each function
// cites the reference file:line it follows (paths relative to the reference project root). Built
// with -ffp-contract=off and without fast-math so every f32 operation rounds exactly where the
// Rust code rounds (Rust never contracts a*b+c).
//
// Parity status: partially pinned — see mrl_oracle.h. The restatement is checked against the
// known-answer values of the reference's own tests; no golden scan outputs exist upstream and the
// Rust binary cannot be built here.
//
// Third-party arithmetic restated here (not vendored in the reference, pinned in its Cargo.lock):
//   * half 2.7.1     — f32 <-> binary16, IEEE round-to-nearest-even (used by VectorMeta).
//   * crc32fast 1.5.3 — CRC-32/ISO-HDLC (reflected 0xEDB88320, init/xorout 0xFFFFFFFF).
//   * rayon 1.12.0   — scheduling only; restated as an ordered chunk map with std::thread.

#include "mrl_oracle.h"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <functional>
#include <thread>
#include <vector>

namespace {

constexpr int VPB = 64;          // src/block.rs:9
constexpr int BLOCK = 4096;      // src/block.rs:10
constexpr int PREFIX = 64;       // src/block.rs:11
constexpr int RABITQ = 128;      // src/block.rs:12
constexpr int TAIL_START = 192;  // src/block.rs:15
constexpr int FOLD = 64;         // src/block.rs:17
constexpr int FOLD_BLOCKS = 9;   // src/block.rs:19

// Byte offsets of PaxBlock64 fields (src/block.rs:31-144, pinned by
// tests/test_challenger_architecture.rs:286-311).
constexpr int OFF_MIN_TS = 0, OFF_MAX_TS = 4, OFF_SRC = 8, OFF_TOMB = 16, OFF_CRC = 24;
constexpr int OFF_META = 64, OFF_S0 = 512, OFF_S1 = 1024, OFF_S2 = 2048, OFF_S3 = 2560,
              OFF_S4 = 3072, OFF_S5 = 3584;

inline uint32_t rd32(const uint8_t* p) { uint32_t v; std::memcpy(&v, p, 4); return v; }
inline uint64_t rd64(const uint8_t* p) { uint64_t v; std::memcpy(&v, p, 8); return v; }
inline void wr32(uint8_t* p, uint32_t v) { std::memcpy(p, &v, 4); }
inline void wr64(uint8_t* p, uint64_t v) { std::memcpy(p, &v, 8); }
inline uint16_t rd16(const uint8_t* p) { uint16_t v; std::memcpy(&v, p, 2); return v; }
inline void wr16(uint8_t* p, uint16_t v) { std::memcpy(p, &v, 2); }

inline uint64_t plane_word(const uint8_t* blk, int off, int d) { return rd64(blk + off + 8 * d); }

// ---------------------------------------------------------------------------------------------
// binary16 conversion (half 2.7.1 semantics: IEEE 754 round-to-nearest-even).
uint16_t f32_to_f16(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ex = (x >> 23) & 0xFFu;
    uint32_t man = x & 0x7FFFFFu;
    if (ex == 0xFFu) {  // inf / nan
        return (uint16_t)(sign | 0x7C00u | (man ? (0x200u | (man >> 13)) : 0u));
    }
    int e = (int)ex - 127 + 15;  // rebias
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);  // overflow -> inf
    if (e <= 0) {
        // subnormal half (or zero): value = man_full * 2^(ex-150); half unit = 2^-24
        if (e < -10) return (uint16_t)sign;  // below half of the smallest subnormal
        const uint32_t full = man | 0x800000u;
        const int shift = 14 - e;  // 14..24
        uint32_t q = full >> shift;
        const uint32_t rem = full & ((1u << shift) - 1u);
        const uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (q & 1u))) q += 1;
        return (uint16_t)(sign | q);
    }
    uint32_t q = ((uint32_t)e << 10) | (man >> 13);
    const uint32_t rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q += 1;  // carry may roll into inf: correct
    return (uint16_t)(sign | q);
}

float f16_to_f32(uint16_t h) {
    const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    const uint32_t ex = (h >> 10) & 0x1Fu;
    const uint32_t man = h & 0x3FFu;
    uint32_t bits;
    if (ex == 0) {
        if (man == 0) {
            bits = sign;
        } else {  // subnormal: normalise
            int e = -1;
            uint32_t m = man;
            do { m <<= 1; ++e; } while (!(m & 0x400u));
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((m & 0x3FFu) << 13);
        }
    } else if (ex == 0x1F) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((ex - 15 + 127) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

// ---------------------------------------------------------------------------------------------
// CRC-32 (crc32fast::hash, used by PaxBlock64::recompute_crc, src/block.rs:186-197).
struct CrcTable {
    uint32_t t[256];
    CrcTable() {
        for (uint32_t i = 0; i < 256; ++i) {
            uint32_t c = i;
            for (int k = 0; k < 8; ++k) c = (c & 1u) ? (0xEDB88320u ^ (c >> 1)) : (c >> 1);
            t[i] = c;
        }
    }
};
const CrcTable kCrc;

uint32_t crc32(const uint8_t* p, size_t n) {
    uint32_t c = 0xFFFFFFFFu;
    for (size_t i = 0; i < n; ++i) c = kCrc.t[(c ^ p[i]) & 0xFFu] ^ (c >> 8);
    return c ^ 0xFFFFFFFFu;
}

// ---------------------------------------------------------------------------------------------
// Rotations (src/rotate.rs).

// fwht_inplace, src/rotate.rs:13-33: butterflies with h = 1, 2, 4, ... then scale by 1/sqrt(n).
void fwht(float* a, int n) {
    for (int h = 1; h < n; h *= 2) {
        for (int i = 0; i < n; i += 2 * h) {
            for (int j = i; j < i + h; ++j) {
                const float x = a[j];
                const float y = a[j + h];
                a[j] = x + y;
                a[j + h] = x - y;
            }
        }
    }
    const float scale = 1.0f / std::sqrt((float)n);
    for (int i = 0; i < n; ++i) a[i] *= scale;
}

// SplitMix-style sign hash shared by tail_rademacher (src/rotate.rs:53-67) and
// rademacher_diag (src/eden.rs:75-88).
inline float sign_hash(uint64_t a, uint64_t i) {
    uint64_t x = (a * 0x9E3779B97F4A7C15ULL + i) * 0xBF58476D1CE4E5B9ULL;
    x ^= x >> 30;
    x *= 0x94D049BB133111EBULL;
    x ^= x >> 27;
    return (x & 1u) == 0 ? 1.0f : -1.0f;
}

constexpr float kPiF = 3.14159265358979323846f;  // std::f32::consts::PI

// rabitq_bit_scale, src/rotate.rs:46-49
float rabitq_bit_scale() { return std::sqrt(2.0f / kPiF) / std::sqrt((float)RABITQ); }
// tail_fold_bit_scale, src/rotate.rs:124-126
float tail_fold_bit_scale() { return std::sqrt(2.0f / kPiF) / std::sqrt((float)FOLD); }

// fold_tail, src/rotate.rs:73-93
void fold_tail(const float* vec, int len, float* u) {
    for (int d = 0; d < FOLD; ++d) u[d] = 0.0f;
    if (len <= TAIL_START) return;
    const int available = len - TAIL_START;
    const int nb = std::min(available / PREFIX, FOLD_BLOCKS);
    for (int b = 0; b < nb; ++b) {
        const int base = TAIL_START + b * PREFIX;
        for (int d = 0; d < FOLD; ++d) u[d] += sign_hash((uint64_t)b, (uint64_t)d) * vec[base + d];
    }
}

// rotate_tail_fold, src/rotate.rs:96-100
void rotate_tail_fold(const float* vec, int len, float* out) {
    fold_tail(vec, len, out);
    fwht(out, FOLD);
}

// ---------------------------------------------------------------------------------------------
// EDEN (src/eden.rs).

// Lloyd-Max N(0,1) centroids, src/eden.rs:15-44 (restated constants; pinned by the reference's
// table test src/eden.rs:374-381).
const float kB1[2] = {-0.79788456f, 0.79788456f};
const float kB2[4] = {-1.51041761f, -0.45278003f, 0.45278003f, 1.51041761f};
const float kB3[8] = {-2.15194570f, -1.34390928f, -0.75600528f, -0.24509418f,
                      0.24509418f,  0.75600528f,  1.34390928f,  2.15194570f};
const float kB4[16] = {-2.73258958f, -2.06901724f, -1.61804640f, -1.25623121f,
                       -0.94234046f, -0.65675912f, -0.38804830f, -0.12839503f,
                       0.12839503f,  0.38804830f,  0.65675912f,  0.94234046f,
                       1.25623121f,  1.61804640f,  2.06901724f,  2.73258958f};

const float* lloyd(int bits) {
    switch (bits) {
        case 1: return kB1;
        case 2: return kB2;
        case 3: return kB3;
        case 4: return kB4;
        default: return nullptr;
    }
}

// nearest_centroid, src/eden.rs:57-71: binary search; exact hit returns its index; otherwise the
// closer neighbour, ties to the lower index.
int nearest_centroid(const float* cb, int n, float z) {
    int lo = 0, hi = n;  // first index with cb[i] >= z
    while (lo < hi) {
        const int mid = (lo + hi) / 2;
        if (cb[mid] < z) lo = mid + 1; else hi = mid;
    }
    if (lo < n && cb[lo] == z) return lo;
    if (lo == 0) return 0;
    if (lo >= n) return n - 1;
    return (std::fabs(z - cb[lo - 1]) <= std::fabs(cb[lo] - z)) ? lo - 1 : lo;
}

// structured_hadamard_inplace, src/eden.rs:91-98
void structured_hadamard(float* v, int d, uint64_t seed) {
    for (int i = 0; i < d; ++i) v[i] *= sign_hash(seed, (uint64_t)i);
    fwht(v, d);
}

// encode_slice, src/eden.rs:225-269
void eden_encode_slice(const float* mean, int d, uint64_t seed, int bits, const float* x,
                       uint8_t* levels, float* centered_norm_out, float* scale_s_out) {
    const float* cb = lloyd(bits);
    const int ncb = 1 << bits;
    const float sqrt_d = std::sqrt((float)d);
    const float inv_sqrt_d = 1.0f / sqrt_d;
    float c[128];
    float norm_sq = 0.0f;
    for (int i = 0; i < d; ++i) {
        const float v = x[i] - mean[i];
        c[i] = v;
        norm_sq += v * v;
    }
    const float centered_norm = std::fmax(std::sqrt(norm_sq), 1e-12f);
    const float inv_norm = 1.0f / centered_norm;
    for (int i = 0; i < d; ++i) c[i] *= inv_norm;
    structured_hadamard(c, d, seed);
    float ip = 0.0f;
    for (int i = 0; i < d; ++i) {
        const int level = nearest_centroid(cb, ncb, c[i] * sqrt_d);
        levels[i] = (uint8_t)level;
        const float cw = cb[level] * inv_sqrt_d;
        ip += c[i] * cw;
    }
    *centered_norm_out = centered_norm;
    *scale_s_out = (std::fabs(ip) > 1e-12f) ? 1.0f / ip : 0.0f;
}

// ---------------------------------------------------------------------------------------------
// Encode (src/quantize.rs).

struct VecCode {
    uint16_t scale, offset, tail;
    uint8_t flags;
    uint8_t bits4[64];
    uint8_t rabitq[128];
    uint8_t fold[64];
};

// VectorMeta::pack_rho_flags, src/block.rs:102-108
uint8_t pack_rho_flags(float high, float rest) {
    if (rest <= 1e-12f) return 0;
    const float r = std::min(std::max(high / rest, 0.0f), 1.0f);
    const float q = std::min(std::max(std::round(r * 255.0f), 0.0f), 255.0f);
    return (uint8_t)q;
}

// residual_norms, src/quantize.rs:184-203
void residual_norms(const float* v, int dims, float* rest, uint8_t* flags) {
    float mid_sq = 0.0f;
    for (int i = PREFIX; i < PREFIX + RABITQ; ++i) mid_sq += v[i] * v[i];
    float high_sq = 0.0f;
    for (int i = TAIL_START; i < dims; ++i) high_sq += v[i] * v[i];
    *rest = std::sqrt(mid_sq + high_sq);
    const float high = std::sqrt(high_sq);
    *flags = pack_rho_flags(high, *rest);
}

// mid_and_fold_bits, src/quantize.rs:205-218
void mid_and_fold_bits(const float* v, int dims, uint8_t* rabitq, uint8_t* fold) {
    float rot[RABITQ];
    std::memcpy(rot, v + PREFIX, sizeof(rot));
    fwht(rot, RABITQ);
    for (int i = 0; i < RABITQ; ++i) rabitq[i] = rot[i] >= 0.0f ? 1 : 0;
    float f[FOLD];
    rotate_tail_fold(v, dims, f);
    for (int i = 0; i < FOLD; ++i) fold[i] = f[i] >= 0.0f ? 1 : 0;
}

// quantize_vector, src/quantize.rs:220-246 (min-max 4-bit prefix)
void quantize_vector(const float* v, int dims, VecCode* out) {
    float mn = INFINITY, mx = -INFINITY;
    for (int i = 0; i < PREFIX; ++i) { mn = std::fmin(mn, v[i]); mx = std::fmax(mx, v[i]); }
    const float range = std::fmax(mx - mn, 1e-8f);
    const float scale = range / 15.0f;
    const float offset = mn;
    for (int i = 0; i < PREFIX; ++i) {
        const float q = std::min(std::max(std::round((v[i] - offset) / scale), 0.0f), 15.0f);
        out->bits4[i] = (uint8_t)q;
    }
    mid_and_fold_bits(v, dims, out->rabitq, out->fold);
    float rest;
    residual_norms(v, dims, &rest, &out->flags);
    out->scale = f32_to_f16(scale);
    out->offset = f32_to_f16(offset);
    out->tail = f32_to_f16(rest);
}

// quantize_vector_eden_dual, src/quantize.rs:265-295
void quantize_vector_eden_dual(const float* mean, uint64_t seed, const float* mid_mean,
                               uint64_t mid_seed, const float* v, int dims, VecCode* out) {
    float cn, ss;
    eden_encode_slice(mean, PREFIX, seed, 4, v, out->bits4, &cn, &ss);
    float mid_alpha = 0.0f;
    uint8_t rabitq_signs[RABITQ];
    mid_and_fold_bits(v, dims, rabitq_signs, out->fold);  // fold bits are used either way
    if (mid_mean) {  // EDEN b=1 levels replace the RaBitQ signs in stratum 1
        float mcn, mss;
        eden_encode_slice(mid_mean, RABITQ, mid_seed, 1, v + PREFIX, out->rabitq, &mcn, &mss);
        mid_alpha = mcn * mss;
    } else {
        std::memcpy(out->rabitq, rabitq_signs, RABITQ);
    }
    float rest;
    residual_norms(v, dims, &rest, &out->flags);
    out->scale = f32_to_f16(cn * ss);  // EdenCode::alpha, src/eden.rs:219-221
    out->offset = f32_to_f16(mid_alpha);
    out->tail = f32_to_f16(rest);
}

// encode_block_with_fits, src/quantize.rs:36-96 (+ write_*_plane :297-333, recompute_crc
// src/block.rs:186-190)
int encode_block(const float* vecs, int n, int dims, const uint32_t* ts, const uint32_t* src,
                 int prefix_codec, const float* eden_mean, uint64_t eden_seed,
                 const float* mid_mean, uint64_t mid_seed, uint8_t* out) {
    if (n < 1 || n > VPB || dims < PREFIX + RABITQ) return -1;
    if (prefix_codec == 1 && !eden_mean) return -2;
    if (mid_mean && prefix_codec != 1) return -3;
    std::memset(out, 0, BLOCK);
    uint32_t min_ts = 0xFFFFFFFFu, max_ts = 0, mask = 0;
    for (int i = 0; i < n; ++i) {
        const float* v = vecs + (size_t)i * dims;
        min_ts = std::min(min_ts, ts[i]);
        max_ts = std::max(max_ts, ts[i]);
        mask |= src[i];
        VecCode c;
        if (prefix_codec == 1) quantize_vector_eden_dual(eden_mean, eden_seed, mid_mean, mid_seed, v, dims, &c);
        else quantize_vector(v, dims, &c);
        uint8_t* m = out + OFF_META + 7 * i;
        wr16(m, c.scale);
        wr16(m + 2, c.offset);
        wr16(m + 4, c.tail);
        m[6] = c.flags;
        const uint64_t bit = 1ULL << i;
        for (int d = 0; d < PREFIX; ++d) {
            const uint8_t q = c.bits4[d];
            if (q & 8) wr64(out + OFF_S0 + 8 * d, rd64(out + OFF_S0 + 8 * d) | bit);
            if (q & 4) wr64(out + OFF_S2 + 8 * d, rd64(out + OFF_S2 + 8 * d) | bit);
            if (q & 2) wr64(out + OFF_S3 + 8 * d, rd64(out + OFF_S3 + 8 * d) | bit);
            if (q & 1) wr64(out + OFF_S5 + 8 * d, rd64(out + OFF_S5 + 8 * d) | bit);
        }
        for (int d = 0; d < RABITQ; ++d)
            if (c.rabitq[d]) wr64(out + OFF_S1 + 8 * d, rd64(out + OFF_S1 + 8 * d) | bit);
        for (int d = 0; d < FOLD; ++d)
            if (c.fold[d]) wr64(out + OFF_S4 + 8 * d, rd64(out + OFF_S4 + 8 * d) | bit);
    }
    uint64_t tomb = 0;
    for (int i = n; i < VPB; ++i) tomb |= 1ULL << i;  // unused slots: zero meta, tombstoned
    wr32(out + OFF_MIN_TS, min_ts);
    wr32(out + OFF_MAX_TS, max_ts);
    wr32(out + OFF_SRC, mask);
    wr64(out + OFF_TOMB, tomb);
    wr32(out + OFF_CRC, 0);
    wr32(out + OFF_CRC, crc32(out, BLOCK));
    return 0;
}

// ---------------------------------------------------------------------------------------------
// Meta decode (src/block.rs:60-99).
struct Meta {
    float scale, offset, tail, mid_norm, high_norm;
};

inline Meta decode_meta(const uint8_t* blk, int v) {
    const uint8_t* m = blk + OFF_META + 7 * v;
    Meta o;
    o.scale = f16_to_f32(rd16(m));
    o.offset = f16_to_f32(rd16(m + 2));
    o.tail = f16_to_f32(rd16(m + 4));
    const float rho = (float)m[6] / 255.0f;                   // rho_ratio, :74-76
    const float t = std::fmax(o.tail, 0.0f);
    const float r = std::min(std::max(rho, 0.0f), 1.0f);
    o.mid_norm = std::sqrt(std::fmax(1.0f - r * r, 0.0f)) * t;  // mid_norm_f32, :80-84
    o.high_norm = rho * t;                                     // high_tail_norm_f32, :88-90
    return o;
}

// ---------------------------------------------------------------------------------------------
// Scan (src/scan.rs).

struct Hit {
    uint64_t id;  // VectorId::as_u64 = block << 16 | slot (src/block.rs:213-215)
    float score;
};

// Shortlist, src/scan.rs:310-399
struct Shortlist {
    size_t cap;
    std::vector<Hit> heap;
    size_t min_idx = 0;
    float min_score = INFINITY;
    float floor_tau = -INFINITY;
    explicit Shortlist(size_t c, float floor = -INFINITY) : cap(std::max<size_t>(c, 1)), floor_tau(floor) {
        heap.reserve(cap);
    }
    float threshold() const { return heap.size() < cap ? floor_tau : std::fmax(min_score, floor_tau); }
    void push(const Hit& h) {
        if (h.score < floor_tau) return;
        if (heap.size() < cap) {
            const size_t idx = heap.size();
            if (h.score < min_score) { min_score = h.score; min_idx = idx; }
            heap.push_back(h);
            return;
        }
        if (h.score > min_score) {
            heap[min_idx] = h;
            recompute_min();
        }
    }
    void recompute_min() {
        size_t mi = 0;
        float ms = INFINITY;
        for (size_t i = 0; i < heap.size(); ++i)
            if (heap[i].score < ms) { ms = heap[i].score; mi = i; }
        min_idx = mi;
        min_score = ms;
    }
    void merge(const Shortlist& o) { for (const Hit& h : o.heap) push(h); }
    std::vector<Hit> into_sorted() {
        std::stable_sort(heap.begin(), heap.end(), [](const Hit& a, const Hit& b) { return a.score > b.score; });
        return heap;
    }
};

struct State {
    float scores[VPB];
    uint64_t survivors;
    float mid_n[VPB];
    float high_n[VPB];
    uint64_t active;
};

struct Ctx {
    const uint8_t* blk;
    const ora_query_plan* plan;
    ora_scan_cfg scan;
    float tau;
    float alpha;
};

inline int ctz64(uint64_t x) { return __builtin_ctzll(x); }

// stage_prefix_ip_and_cs_split, src/scan.rs:453-517
void stage_prefix(const Ctx& c, State& s) {
    const bool eden = c.plan->prefix_codec == 1;
    float acc[VPB];
    for (int v = 0; v < VPB; ++v) acc[v] = 0.0f;
    for (int d = 0; d < PREFIX; ++d) {
        const float weight = eden ? c.plan->eden_q_rot[d] * c.plan->eden_inv_sqrt_d : c.plan->prefix[d];
        if (weight == 0.0f) continue;
        const uint64_t b0 = plane_word(c.blk, OFF_S5, d), b1 = plane_word(c.blk, OFF_S3, d);
        const uint64_t b2 = plane_word(c.blk, OFF_S2, d), b3 = plane_word(c.blk, OFF_S0, d);
        for (int v = 0; v < VPB; ++v) {  // same per-vector accumulation order as the SWAR loop
            const int level = (int)(((b0 >> v) & 1) | (((b1 >> v) & 1) << 1) | (((b2 >> v) & 1) << 2) |
                                    (((b3 >> v) & 1) << 3));
            if (eden) acc[v] += c.plan->eden_codebook[level] * weight;
            else acc[v] += (float)level * weight;
        }
    }
    uint64_t surv = 0;
    for (int v = 0; v < VPB; ++v) {
        const uint64_t bit = 1ULL << v;
        if (!(s.active & bit)) continue;
        const Meta m = decode_meta(c.blk, v);
        s.mid_n[v] = std::fmax(m.mid_norm, 1e-6f);
        s.high_n[v] = std::fmax(m.high_norm, 0.0f);
        const float prefix_ip = eden ? c.plan->eden_mean_ip + m.scale * acc[v]
                                     : acc[v] * m.scale + m.offset * c.plan->prefix_sum;
        s.scores[v] = prefix_ip;
        const float ub = prefix_ip + c.alpha * (c.plan->q_mid_norm * s.mid_n[v] +
                                                c.plan->q_tail_norm * s.high_n[v]);
        if (ub >= c.tau) surv |= bit;
    }
    s.survivors = surv;
}

// stage_rabitq_ip, src/scan.rs:520-569
void stage_rabitq(const Ctx& c, State& s) {
    if (c.plan->mid_codec == 1) {
        float base = 0.0f;
        float deltas[RABITQ];
        const float c0 = c.plan->eden_mid_codebook[0], c1 = c.plan->eden_mid_codebook[1];
        const float inv = c.plan->eden_mid_inv_sqrt_d;
        for (int d = 0; d < RABITQ; ++d) {
            const float q = c.plan->eden_mid_q_rot[d] * inv;
            base += c0 * q;
            deltas[d] = (c1 - c0) * q;
        }
        float cw[VPB];
        for (int v = 0; v < VPB; ++v) cw[v] = base;
        for (int d = 0; d < RABITQ; ++d) {
            uint64_t bits = plane_word(c.blk, OFF_S1, d) & s.survivors;
            while (bits) { const int v = ctz64(bits); cw[v] += deltas[d]; bits &= bits - 1; }
        }
        uint64_t sb = s.survivors;
        while (sb) {
            const int v = ctz64(sb);
            const float mid_alpha = decode_meta(c.blk, v).offset;
            s.scores[v] += c.plan->eden_mid_mean_ip + mid_alpha * cw[v];
            sb &= sb - 1;
        }
        return;
    }
    float s1[VPB];
    for (int v = 0; v < VPB; ++v) s1[v] = c.plan->rabitq_base;
    for (int d = 0; d < RABITQ; ++d) {
        uint64_t bits = plane_word(c.blk, OFF_S1, d) & s.survivors;
        const float w = c.plan->rabitq_weights2[d];
        while (bits) { const int v = ctz64(bits); s1[v] += w; bits &= bits - 1; }
    }
    uint64_t sb = s.survivors;
    while (sb) { const int v = ctz64(sb); s.scores[v] += s1[v] * s.mid_n[v]; sb &= sb - 1; }
}

// stage_cs_tail, src/scan.rs:572-584
void stage_cs_tail(const Ctx& c, State& s) {
    uint64_t s2 = 0, cb = s.survivors;
    while (cb) {
        const int v = ctz64(cb);
        const float ub = s.scores[v] + c.alpha * c.plan->q_after_s1 * s.high_n[v];
        if (ub >= c.tau) s2 |= 1ULL << v;
        cb &= cb - 1;
    }
    s.survivors = s2;
}

// stage_s4_abs_budget, src/scan.rs:587-607
void stage_s4_budget(const Ctx& c, State& s) {
    if (c.scan.strata_depth != 2) return;
    if (!(c.plan->has_tail_fold && c.plan->s4_abs_budget > 0.0f)) return;
    const float w = c.scan.stratum4_weight;
    uint64_t s3 = 0, b = s.survivors;
    while (b) {
        const int v = ctz64(b);
        const float ub = s.scores[v] + c.alpha * std::fmax(s.high_n[v], 1e-6f) * w * c.plan->s4_abs_budget;
        if (ub >= c.tau) s3 |= 1ULL << v;
        b &= b - 1;
    }
    s.survivors = s3;
}

// stage_tail_fold_ip, src/scan.rs:610-634
void stage_tail_fold(const Ctx& c, State& s) {
    if (c.scan.strata_depth != 2) return;
    if (!c.plan->has_tail_fold) return;
    const float w = c.scan.stratum4_weight;
    float s4[VPB];
    for (int v = 0; v < VPB; ++v) s4[v] = c.plan->tail_fold_base;
    for (int d = 0; d < FOLD; ++d) {
        uint64_t bits = plane_word(c.blk, OFF_S4, d) & s.survivors;
        const float wd = c.plan->tail_fold_weights2[d];
        while (bits) { const int v = ctz64(bits); s4[v] += wd; bits &= bits - 1; }
    }
    uint64_t sb = s.survivors;
    while (sb) {
        const int v = ctz64(sb);
        s.scores[v] += s4[v] * std::fmax(s.high_n[v], 1e-6f) * w;
        sb &= sb - 1;
    }
}

// run_default_scan_kernel, src/scan.rs:654-691
void run_default(const Ctx& c, State& s, ora_scan_stats* st) {
    stage_prefix(c, s);
    if (st) st->after_prefix += __builtin_popcountll(s.survivors);
    if (!s.survivors) return;
    if (c.scan.strata_depth >= 1) {
        stage_rabitq(c, s);
        stage_cs_tail(c, s);
    }
    if (st) st->after_s1 += __builtin_popcountll(s.survivors);
    if (!s.survivors) return;
    if (c.scan.strata_depth == 2) {
        stage_s4_budget(c, s);
        if (st) st->after_s4_budget += __builtin_popcountll(s.survivors);
        if (!s.survivors) return;
        stage_tail_fold(c, s);
    } else if (st) {
        st->after_s4_budget += __builtin_popcountll(s.survivors);
    }
}

void finish_push(uint32_t block_idx, uint64_t surv, const float* scores, Shortlist& sl) {
    while (surv) {
        const int v = ctz64(surv);
        sl.push(Hit{((uint64_t)block_idx << 16) | (uint64_t)v, scores[v]});
        surv &= surv - 1;
    }
}

struct TimeRange {
    bool has_lo, has_hi;
    uint32_t lo, hi;
};

inline bool temporal_skip(const uint8_t* blk, const ora_scan_cfg& cfg, const TimeRange& tr) {
    if (!cfg.temporal_filter_enable) return false;
    if (tr.has_lo && rd32(blk + OFF_MAX_TS) < tr.lo) return true;
    if (tr.has_hi && rd32(blk + OFF_MIN_TS) > tr.hi) return true;
    return false;
}

// scan_block_stats, src/scan.rs:709-799. When `tau_override` is non-null the block is scored with
// that threshold instead of the shortlist's (used for full scores with tau = -inf).
void scan_block(const uint8_t* blk, uint32_t block_idx, const ora_query_plan* plan,
                const ora_scan_cfg& cfg, Shortlist* sl, const TimeRange& tr, ora_scan_stats* st,
                const float* tau_override, float* scores_out, uint64_t* surv_out) {
    if (surv_out) *surv_out = 0;
    if (temporal_skip(blk, cfg, tr)) return;
    const float tau = tau_override ? *tau_override : sl->threshold();
    const float alpha = cfg.cs_tolerance;
    const uint64_t active = ~rd64(blk + OFF_TOMB);
    if (active == 0) return;
    if (st) { st->blocks += 1; st->active_vecs += __builtin_popcountll(active); }
    State s;
    for (int v = 0; v < VPB; ++v) { s.scores[v] = 0.0f; s.mid_n[v] = 0.0f; s.high_n[v] = 0.0f; }
    s.survivors = 0;
    s.active = active;
    Ctx c{blk, plan, cfg, tau, alpha};
    if (cfg.strata_depth == 0) {  // L0Only, src/scan.rs:753-790
        float code_dot[VPB];
        for (int v = 0; v < VPB; ++v) code_dot[v] = 0.0f;
        for (int d = 0; d < PREFIX; ++d) {  // accum_plane, src/scan.rs:403-413
            const float w = plan->bit_weights[d][3];
            if (w == 0.0f) continue;
            uint64_t bits = plane_word(blk, OFF_S0, d) & active;
            while (bits) { const int v = ctz64(bits); code_dot[v] += w; bits &= bits - 1; }
        }
        uint64_t surv = 0;
        for (int v = 0; v < VPB; ++v) {
            const uint64_t bit = 1ULL << v;
            if (!(active & bit)) continue;
            const Meta m = decode_meta(blk, v);
            const float prefix_ip = code_dot[v] * m.scale + m.offset * plan->prefix_sum;
            s.scores[v] = prefix_ip;
            const float x_rest = std::fmax(m.tail, 0.0f);
            const float ub = prefix_ip + alpha * plan->q_after_prefix * x_rest;
            if (ub >= tau) surv |= bit;
        }
        if (surv) {
            if (st) {
                const uint64_t n = __builtin_popcountll(surv);
                st->after_prefix += n; st->after_s1 += n; st->after_s4_budget += n; st->pushed += n;
            }
            if (sl) finish_push(block_idx, surv, s.scores, *sl);
        }
        if (scores_out) std::memcpy(scores_out, s.scores, sizeof(s.scores));
        if (surv_out) *surv_out = surv;
        return;
    }
    run_default(c, s, st);
    if (s.survivors) {
        if (st) st->pushed += __builtin_popcountll(s.survivors);
        if (sl) finish_push(block_idx, s.survivors, s.scores, *sl);
    }
    if (scores_out) std::memcpy(scores_out, s.scores, sizeof(s.scores));
    if (surv_out) *surv_out = s.survivors;
}

void parallel_chunks(size_t n_tasks, int threads, const std::function<void(size_t)>& fn) {
    if (threads <= 1 || n_tasks <= 1) {
        for (size_t i = 0; i < n_tasks; ++i) fn(i);
        return;
    }
    std::atomic<size_t> next{0};
    std::vector<std::thread> pool;
    const int nt = (int)std::min<size_t>((size_t)threads, n_tasks);
    for (int t = 0; t < nt; ++t)
        pool.emplace_back([&] {
            for (size_t i = next.fetch_add(1); i < n_tasks; i = next.fetch_add(1)) fn(i);
        });
    for (auto& th : pool) th.join();
}

// scan_blocks_stats, src/scan.rs:813-886
std::vector<Hit> scan_blocks(const uint8_t* blocks, uint64_t n, const ora_query_plan* plan,
                             const ora_scan_cfg& cfg, const TimeRange& tr, int threads,
                             ora_scan_stats* st) {
    Shortlist sl(cfg.shortlist_cand);
    if (n == 0) return {};
    const uint64_t PAR_THRESHOLD = 64;
    if (cfg.numa_sharding && n >= PAR_THRESHOLD && !st) {
        const uint64_t warm = std::min<uint64_t>(std::min<uint64_t>(cfg.shortlist_cand / VPB + 1, 32), n);
        for (uint64_t i = 0; i < warm; ++i)
            scan_block(blocks + i * BLOCK, (uint32_t)i, plan, cfg, &sl, tr, nullptr, nullptr, nullptr, nullptr);
        const uint64_t rest = n - warm;
        const uint64_t shards = std::max<uint64_t>((uint64_t)std::max(threads, 1) * 2, 8);
        const uint64_t chunk = std::max<uint64_t>((rest + shards - 1) / shards, 16);
        const float floor_tau = sl.threshold();
        const uint64_t n_chunks = (rest + chunk - 1) / chunk;
        std::vector<Shortlist> partials(n_chunks, Shortlist(cfg.shortlist_cand, floor_tau));
        parallel_chunks(n_chunks, threads, [&](size_t ci) {
            const uint64_t b0 = warm + ci * chunk;
            const uint64_t b1 = std::min<uint64_t>(b0 + chunk, n);
            for (uint64_t b = b0; b < b1; ++b)
                scan_block(blocks + b * BLOCK, (uint32_t)b, plan, cfg, &partials[ci], tr, nullptr,
                           nullptr, nullptr, nullptr);
        });
        for (const Shortlist& p : partials) sl.merge(p);
        return sl.into_sorted();
    }
    for (uint64_t i = 0; i < n; ++i)
        scan_block(blocks + i * BLOCK, (uint32_t)i, plan, cfg, &sl, tr, st, nullptr, nullptr, nullptr);
    return sl.into_sorted();
}

// ---------------------------------------------------------------------------------------------
// Fixed-point formulation (the product's fast mode restated). Per-dimension stage values are
// exact double products of f32 plan quantities, scaled by 2^shift and rounded to nearest-even;
// stage sums are exact int32 sums of table entries.

int stage_shift(double maxabs, int count) {
    if (!(maxabs > 0.0)) return 0;
    int k = 0;
    std::frexp(maxabs * (double)count, &k);
    return 30 - k;
}

inline int32_t fix(double v, int shift) { return (int32_t)std::nearbyint(std::ldexp(v, shift)); }
inline float unfix(int64_t i, int shift) { return (float)std::ldexp((double)i, -shift); }

void build_windows(const double* val1, const double* val0, int ndim, int shift, int32_t (*lut)[32]) {
    const int nwin = (ndim + 4) / 5;
    for (int g = 0; g < nwin; ++g) {
        const int w = std::min(5, ndim - 5 * g);
        for (int m = 0; m < 32; ++m) {
            int32_t s = 0;
            if (m < (1 << w)) {
                for (int i = 0; i < w; ++i) {
                    const int d = 5 * g + i;
                    s += fix(((m >> i) & 1) ? val1[d] : val0[d], shift);
                }
            }
            lut[g][m] = s;
        }
    }
}

void fixed_plan_build(const ora_query_plan* p, const ora_scan_cfg* cfg, ora_fixed_plan* o) {
    std::memset(o, 0, sizeof(*o));
    // prefix
    double val[PREFIX][16];
    double mx = 0.0;
    for (int d = 0; d < PREFIX; ++d) {
        for (int l = 0; l < 16; ++l) {
            double v;
            if (cfg->strata_depth == 0) {
                v = (l & 8) ? (double)p->bit_weights[d][3] : 0.0;
            } else if (p->prefix_codec == 1) {
                const float w = p->eden_q_rot[d] * p->eden_inv_sqrt_d;
                v = (double)p->eden_codebook[l] * (double)w;
            } else {
                v = (double)l * (double)p->prefix[d];
            }
            val[d][l] = v;
            mx = std::max(mx, std::fabs(v));
        }
    }
    o->prefix_shift = stage_shift(mx, PREFIX);
    for (int d = 0; d < PREFIX; ++d)
        for (int l = 0; l < 16; ++l) o->prefix_lut[d][l] = fix(val[d][l], o->prefix_shift);
    // mid band
    double v1[RABITQ], v0[RABITQ];
    mx = 0.0;
    for (int d = 0; d < RABITQ; ++d) {
        if (p->mid_codec == 1) {
            const float q = p->eden_mid_q_rot[d] * p->eden_mid_inv_sqrt_d;
            v1[d] = (double)p->eden_mid_codebook[1] * (double)q;
            v0[d] = (double)p->eden_mid_codebook[0] * (double)q;
        } else {
            const double pos = 0.5 * (double)p->rabitq_weights2[d];
            v1[d] = pos;
            v0[d] = -pos;
        }
        mx = std::max(mx, std::max(std::fabs(v1[d]), std::fabs(v0[d])));
    }
    o->s1_shift = stage_shift(mx, RABITQ);
    build_windows(v1, v0, RABITQ, o->s1_shift, o->s1_lut);
    // folded tail
    double t1[FOLD], t0[FOLD];
    mx = 0.0;
    for (int d = 0; d < FOLD; ++d) {
        const double pos = 0.5 * (double)p->tail_fold_weights2[d];
        t1[d] = pos;
        t0[d] = -pos;
        mx = std::max(mx, std::fabs(pos));
    }
    o->s4_shift = stage_shift(mx, FOLD);
    build_windows(t1, t0, FOLD, o->s4_shift, o->s4_lut);
}

}  // namespace

// =============================================================================================
// C ABI
extern "C" {

uint16_t ora_f32_to_f16(float x) { return f32_to_f16(x); }
float ora_f16_to_f32(uint16_t h) { return f16_to_f32(h); }
uint32_t ora_crc32(const uint8_t* data, size_t n) { return crc32(data, n); }
void ora_fwht(float* a, int n) { fwht(a, n); }
void ora_rotate_mid_band(const float* mid, float* out) {
    std::memcpy(out, mid, RABITQ * sizeof(float));
    fwht(out, RABITQ);
}
void ora_rotate_tail_fold(const float* vec, int dims, float* out) { rotate_tail_fold(vec, dims, out); }
float ora_tail_rademacher(uint64_t b, uint64_t d) { return sign_hash(b, d); }
float ora_rademacher_diag(uint64_t seed, uint64_t i) { return sign_hash(seed, i); }
float ora_rabitq_bit_scale(void) { return rabitq_bit_scale(); }
float ora_tail_fold_bit_scale(void) { return tail_fold_bit_scale(); }
void ora_lloyd_max(int bits, float* out) {
    const float* cb = lloyd(bits);
    if (cb) std::memcpy(out, cb, sizeof(float) * (1u << bits));
}
int ora_nearest_centroid(const float* cb, int n, float z) { return nearest_centroid(cb, n, z); }

// EdenFit::fit_band, src/eden.rs:130-161 (f32 sequential sum over rows, then * (1/n))
void ora_eden_fit_band(const float* rows, uint64_t n, int dims, int start, int width, float* mean) {
    for (int d = 0; d < width; ++d) mean[d] = 0.0f;
    for (uint64_t r = 0; r < n; ++r)
        for (int d = 0; d < width; ++d) mean[d] += rows[r * (uint64_t)dims + start + d];
    const float inv = 1.0f / (float)n;
    for (int d = 0; d < width; ++d) mean[d] *= inv;
}
void ora_eden_fit_prefix(const float* rows, uint64_t n, int dims, float* mean) {
    ora_eden_fit_band(rows, n, dims, 0, PREFIX, mean);
}
void ora_eden_encode_slice(const float* mean, int d, uint64_t seed, int bits, const float* x,
                           uint8_t* levels, float* cn, float* ss) {
    eden_encode_slice(mean, d, seed, bits, x, levels, cn, ss);
}

int ora_encode_block(const float* vecs, int n, int dims, const uint32_t* ts, const uint32_t* src,
                     int prefix_codec, const float* eden_mean, uint64_t eden_seed,
                     const float* mid_mean, uint64_t mid_seed, uint8_t* out) {
    return encode_block(vecs, n, dims, ts, src, prefix_codec, eden_mean, eden_seed, mid_mean, mid_seed, out);
}

// encode_f32_corpus_par, src/encoder.rs:195-219
int ora_encode_corpus(const float* rows, uint64_t n, int dims, uint32_t src, int prefix_codec,
                      const float* eden_mean, uint64_t eden_seed, const float* mid_mean,
                      uint64_t mid_seed, int threads, uint8_t* out) {
    const uint64_t nb = (n + VPB - 1) / VPB;
    std::atomic<int> err{0};
    parallel_chunks(nb, threads, [&](size_t b) {
        const uint64_t s = b * VPB, e = std::min<uint64_t>(s + VPB, n);
        uint32_t ts[VPB], sr[VPB];
        for (uint64_t j = s; j < e; ++j) { ts[j - s] = (uint32_t)j; sr[j - s] = src; }
        const int rc = encode_block(rows + s * (uint64_t)dims, (int)(e - s), dims, ts, sr, prefix_codec,
                                    eden_mean, eden_seed, mid_mean, mid_seed, out + b * BLOCK);
        if (rc) err = rc;
    });
    return err.load();
}

// PaxBlock64::verify_crc, src/block.rs:192-197
int ora_verify_crc(const uint8_t* blk) {
    uint8_t copy[BLOCK];
    std::memcpy(copy, blk, BLOCK);
    const uint32_t expected = rd32(copy + OFF_CRC);
    wr32(copy + OFF_CRC, 0);
    return crc32(copy, BLOCK) == expected ? 1 : 0;
}

// QueryPlan::from_query_codec, src/scan.rs:105-266 (+ rotate_query src/eden.rs:275-281)
int ora_plan_build(const float* q, int dims, int prefix_codec, int mid_codec, const float* eden_mean,
                   uint64_t eden_seed, const float* mid_mean, uint64_t mid_seed, ora_query_plan* o) {
    if (dims < PREFIX + RABITQ) return -1;
    if (prefix_codec == 1 && !eden_mean) return -2;
    if (mid_codec == 1 && !mid_mean) return -3;
    std::memset(o, 0, sizeof(*o));
    o->dims = (uint32_t)dims;
    o->prefix_codec = (uint32_t)prefix_codec;
    o->mid_codec = (uint32_t)mid_codec;
    for (int d = 0; d < PREFIX; ++d) o->prefix[d] = q[d];
    float l1 = 0.0f, sum = 0.0f;
    for (int d = 0; d < PREFIX; ++d) {
        const float qd = o->prefix[d];
        l1 += std::fabs(qd);
        sum += qd;
        o->bit_weights[d][0] = qd * 1.0f;
        o->bit_weights[d][1] = qd * 2.0f;
        o->bit_weights[d][2] = qd * 4.0f;
        o->bit_weights[d][3] = qd * 8.0f;
    }
    o->prefix_l1 = l1;
    o->prefix_sum = sum;
    o->eden_inv_sqrt_d = 1.0f / std::sqrt((float)PREFIX);
    if (prefix_codec == 1) {
        float rot[PREFIX];
        std::memcpy(rot, q, sizeof(rot));
        structured_hadamard(rot, PREFIX, eden_seed);
        std::memcpy(o->eden_q_rot, rot, sizeof(rot));
        float ip = 0.0f;
        for (int d = 0; d < PREFIX; ++d) ip += q[d] * eden_mean[d];
        o->eden_mean_ip = ip;
        o->eden_inv_sqrt_d = 1.0f / std::sqrt((float)PREFIX);
        std::memcpy(o->eden_codebook, kB4, sizeof(kB4));
    }
    o->eden_mid_inv_sqrt_d = 1.0f / std::sqrt((float)RABITQ);
    if (mid_codec == 1) {
        float rot[RABITQ];
        std::memcpy(rot, q + PREFIX, sizeof(rot));
        structured_hadamard(rot, RABITQ, mid_seed);
        std::memcpy(o->eden_mid_q_rot, rot, sizeof(rot));
        float ip = 0.0f;
        for (int d = 0; d < RABITQ; ++d) ip += q[PREFIX + d] * mid_mean[d];
        o->eden_mid_mean_ip = ip;
        o->eden_mid_inv_sqrt_d = 1.0f / std::sqrt((float)RABITQ);
        o->eden_mid_codebook[0] = kB1[0];
        o->eden_mid_codebook[1] = kB1[1];
    }
    std::memcpy(o->rabitq_q, q + PREFIX, RABITQ * sizeof(float));
    fwht(o->rabitq_q, RABITQ);
    o->rabitq_scale = rabitq_bit_scale();
    float base = 0.0f;
    for (int d = 0; d < RABITQ; ++d) {
        const float pos = o->rabitq_q[d] * o->rabitq_scale;
        base -= pos;
        o->rabitq_weights2[d] = 2.0f * pos;
    }
    o->rabitq_base = base;
    for (int g = 0; g < RABITQ / 4; ++g) {
        const float p0 = o->rabitq_q[4 * g] * o->rabitq_scale;
        const float p1 = o->rabitq_q[4 * g + 1] * o->rabitq_scale;
        const float p2 = o->rabitq_q[4 * g + 2] * o->rabitq_scale;
        const float p3 = o->rabitq_q[4 * g + 3] * o->rabitq_scale;
        for (int m = 0; m < 16; ++m) {
            const float s0 = (m & 1) ? p0 : -p0, s1 = (m & 2) ? p1 : -p1;
            const float s2 = (m & 4) ? p2 : -p2, s3 = (m & 8) ? p3 : -p3;
            o->rabitq_lut[g][m] = s0 + s1 + s2 + s3;
        }
    }
    float tail_sq = 0.0f;
    for (int d = TAIL_START; d < dims; ++d) tail_sq += q[d] * q[d];
    o->q_tail_norm = std::sqrt(tail_sq);
    float mid_sq = 0.0f;
    for (int i = 0; i < RABITQ; ++i) mid_sq += q[PREFIX + i] * q[PREFIX + i];
    o->q_mid_norm = std::sqrt(mid_sq);
    o->q_after_prefix = std::sqrt(mid_sq + tail_sq);
    o->has_tail_fold = dims > TAIL_START ? 1u : 0u;
    if (o->has_tail_fold) rotate_tail_fold(q, dims, o->tail_fold_q);
    const float ts = tail_fold_bit_scale();
    float tbase = 0.0f, budget = 0.0f;
    if (o->has_tail_fold) {
        for (int d = 0; d < FOLD; ++d) {
            const float pos = o->tail_fold_q[d] * ts;
            tbase -= pos;
            o->tail_fold_weights2[d] = 2.0f * pos;
            budget += std::fabs(pos);
        }
    }
    o->tail_fold_base = tbase;
    o->s4_abs_budget = budget;
    o->q_after_s1 = o->q_tail_norm;
    return 0;
}

int ora_scan_blocks(const uint8_t* blocks, uint64_t n, const ora_query_plan* plan, const ora_scan_cfg* cfg,
                    int has_lo, uint32_t lo, int has_hi, uint32_t hi, int threads, ora_scan_stats* st,
                    uint64_t* ids, float* scores) {
    const TimeRange tr{has_lo != 0, has_hi != 0, lo, hi};
    std::vector<Hit> hits = scan_blocks(blocks, n, plan, *cfg, tr, threads, st);
    for (size_t i = 0; i < hits.size(); ++i) { ids[i] = hits[i].id; scores[i] = hits[i].score; }
    return (int)hits.size();
}

void ora_full_scores(const uint8_t* blocks, uint64_t n, const ora_query_plan* plan, const ora_scan_cfg* cfg,
                     int has_lo, uint32_t lo, int has_hi, uint32_t hi, float* out, uint8_t* act) {
    const TimeRange tr{has_lo != 0, has_hi != 0, lo, hi};
    const float ninf = -INFINITY;
    for (uint64_t b = 0; b < n; ++b) {
        const uint8_t* blk = blocks + b * BLOCK;
        float sc[VPB];
        uint64_t surv = 0;
        for (int v = 0; v < VPB; ++v) sc[v] = 0.0f;
        scan_block(blk, (uint32_t)b, plan, *cfg, nullptr, tr, nullptr, &ninf, sc, &surv);
        for (int v = 0; v < VPB; ++v) {
            out[b * VPB + v] = sc[v];
            act[b * VPB + v] = (uint8_t)((surv >> v) & 1u);
        }
    }
}

void ora_block_stages(const uint8_t* blk, const ora_query_plan* plan, const ora_scan_cfg* cfg, float tau,
                      uint64_t* masks, float* scores) {
    State s;
    for (int v = 0; v < VPB; ++v) { s.scores[v] = 0.0f; s.mid_n[v] = 0.0f; s.high_n[v] = 0.0f; }
    s.active = ~rd64(blk + OFF_TOMB);
    s.survivors = 0;
    Ctx c{blk, plan, *cfg, tau, cfg->cs_tolerance};
    stage_prefix(c, s);
    masks[0] = s.survivors;
    stage_rabitq(c, s);
    stage_cs_tail(c, s);
    masks[1] = s.survivors;
    stage_s4_budget(c, s);
    masks[2] = s.survivors;
    stage_tail_fold(c, s);
    masks[3] = s.survivors;
    std::memcpy(scores, s.scores, sizeof(s.scores));
}

void ora_fixed_plan_build(const ora_query_plan* plan, const ora_scan_cfg* cfg, ora_fixed_plan* out) {
    fixed_plan_build(plan, cfg, out);
}

void ora_fixed_scores(const uint8_t* blocks, uint64_t n, const ora_query_plan* p, const ora_fixed_plan* fp,
                      const ora_scan_cfg* cfg, int has_lo, uint32_t lo, int has_hi, uint32_t hi,
                      int32_t* partials, float* out, uint8_t* act) {
    const TimeRange tr{has_lo != 0, has_hi != 0, lo, hi};
    for (uint64_t b = 0; b < n; ++b) {
        const uint8_t* blk = blocks + b * BLOCK;
        const bool skip = temporal_skip(blk, *cfg, tr);
        const uint64_t active = skip ? 0 : ~rd64(blk + OFF_TOMB);
        for (int v = 0; v < VPB; ++v) {
            const uint64_t idx = b * VPB + v;
            int32_t* pp = partials + idx * 3;
            pp[0] = pp[1] = pp[2] = 0;
            out[idx] = 0.0f;
            act[idx] = (uint8_t)((active >> v) & 1u);
            if (!act[idx]) continue;
            int32_t P = 0, S1 = 0, S4 = 0;
            for (int d = 0; d < PREFIX; ++d) {
                const uint64_t b0 = plane_word(blk, OFF_S5, d), b1 = plane_word(blk, OFF_S3, d);
                const uint64_t b2 = plane_word(blk, OFF_S2, d), b3 = plane_word(blk, OFF_S0, d);
                const int level = (int)(((b0 >> v) & 1) | (((b1 >> v) & 1) << 1) | (((b2 >> v) & 1) << 2) |
                                        (((b3 >> v) & 1) << 3));
                P += fp->prefix_lut[d][level];
            }
            for (int g = 0; g < 26; ++g) {
                int m = 0;
                for (int i = 0; i < 5 && 5 * g + i < RABITQ; ++i)
                    m |= (int)((plane_word(blk, OFF_S1, 5 * g + i) >> v) & 1) << i;
                S1 += fp->s1_lut[g][m];
            }
            for (int g = 0; g < 13; ++g) {
                int m = 0;
                for (int i = 0; i < 5 && 5 * g + i < FOLD; ++i)
                    m |= (int)((plane_word(blk, OFF_S4, 5 * g + i) >> v) & 1) << i;
                S4 += fp->s4_lut[g][m];
            }
            pp[0] = P; pp[1] = S1; pp[2] = S4;
            const Meta m = decode_meta(blk, v);
            const float mid_n = std::fmax(m.mid_norm, 1e-6f);
            const float high_n = std::fmax(m.high_norm, 0.0f);
            const float code_dot = unfix(P, fp->prefix_shift);
            float score;
            if (cfg->strata_depth == 0) {
                score = code_dot * m.scale + m.offset * p->prefix_sum;
            } else {
                score = (p->prefix_codec == 1) ? p->eden_mean_ip + m.scale * code_dot
                                               : code_dot * m.scale + m.offset * p->prefix_sum;
                if (p->mid_codec == 1) {
                    const float cw = unfix(S1, fp->s1_shift);
                    score += p->eden_mid_mean_ip + m.offset * cw;
                } else {
                    const float s1 = unfix(S1, fp->s1_shift);
                    score += s1 * mid_n;
                }
                if (cfg->strata_depth == 2 && p->has_tail_fold) {
                    const float s4 = unfix(S4, fp->s4_shift);
                    score += s4 * std::fmax(high_n, 1e-6f) * cfg->stratum4_weight;
                }
            }
            out[idx] = score;
        }
    }
}

void ora_device_layout(const uint8_t* blk, uint8_t* out, uint32_t* ts2) {
    std::memset(out, 0, BLOCK);
    const uint64_t tomb = rd64(blk + OFF_TOMB);
    for (int v = 0; v < VPB; ++v) {
        uint32_t w[16] = {0};
        for (int d = 0; d < PREFIX; ++d) {
            const uint32_t lv = (uint32_t)(((plane_word(blk, OFF_S5, d) >> v) & 1) |
                                           (((plane_word(blk, OFF_S3, d) >> v) & 1) << 1) |
                                           (((plane_word(blk, OFF_S2, d) >> v) & 1) << 2) |
                                           (((plane_word(blk, OFF_S0, d) >> v) & 1) << 3));
            w[d / 8] |= lv << (4 * (d % 8));
        }
        for (int d = 0; d < RABITQ; ++d)
            w[8 + d / 32] |= (uint32_t)((plane_word(blk, OFF_S1, d) >> v) & 1) << (d % 32);
        for (int d = 0; d < FOLD; ++d)
            w[12 + d / 32] |= (uint32_t)((plane_word(blk, OFF_S4, d) >> v) & 1) << (d % 32);
        const uint8_t* m = blk + OFF_META + 7 * v;
        w[14] = (uint32_t)rd16(m) | ((uint32_t)rd16(m + 2) << 16);
        w[15] = (uint32_t)rd16(m + 4) | ((uint32_t)m[6] << 16) | ((uint32_t)((tomb >> v) & 1) << 24);
        for (int c = 0; c < 4; ++c)
            std::memcpy(out + c * 1024 + v * 16, &w[4 * c], 16);
    }
    ts2[0] = rd32(blk + OFF_MIN_TS);
    ts2[1] = rd32(blk + OFF_MAX_TS);
}

// ---- seeded synthetic generator (same integer recipe in the product's GPU generator) ----
static inline uint64_t splitmix64(uint64_t x) {  // SplitMix64 output function (Steele et al. 2014)
    x += 0x9E3779B97F4A7C15ULL;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ULL;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBULL;
    return x ^ (x >> 31);
}
// Irwin-Hall(12) - 6 from twelve 16-bit uniforms (midpoint lattice); exact in f32.
static inline float ih_gauss(uint64_t seed, uint64_t idx) {
    int64_t s = 0;
    for (uint64_t j = 0; j < 3; ++j) {
        const uint64_t h = splitmix64(seed * 0xD1B54A32D192ED03ULL + idx * 3 + j);
        s += (int64_t)(h & 0xFFFF) + (int64_t)((h >> 16) & 0xFFFF) + (int64_t)((h >> 32) & 0xFFFF) +
             (int64_t)(h >> 48);
    }
    const int32_t num = (int32_t)(2 * s + 12 - 786432);
    return (float)num * (1.0f / 131072.0f);
}
static void synth_row(uint64_t seed, uint64_t row, int dims, float* x) {
    float ss = 0.0f;
    for (int d = 0; d < dims; ++d) {
        const float sigma = 1.0f / std::sqrt((float)(d + 1));
        x[d] = ih_gauss(seed, row * (uint64_t)dims + (uint64_t)d) * sigma;
    }
    for (int d = 0; d < dims; ++d) ss += x[d] * x[d];
    const float nrm = std::fmax(std::sqrt(ss), 1e-12f);
    for (int d = 0; d < dims; ++d) x[d] = x[d] / nrm;
}

void ora_synth_docs(uint64_t seed, uint64_t row0, uint64_t n, int dims, int threads, float* out) {
    const uint64_t chunk = 4096;
    const uint64_t nc = (n + chunk - 1) / chunk;
    parallel_chunks(nc, threads, [&](size_t c) {
        const uint64_t s = c * chunk, e = std::min<uint64_t>(s + chunk, n);
        for (uint64_t r = s; r < e; ++r) synth_row(seed, row0 + r, dims, out + r * (uint64_t)dims);
    });
}

void ora_synth_queries(uint64_t doc_seed, uint64_t n_docs, uint64_t q_seed, uint64_t n_q, int dims,
                       float sigma, float* out, uint64_t* pick) {
    std::vector<float> x((size_t)dims);
    const uint64_t noise_seed = splitmix64(q_seed ^ 0x6E6F697365ULL);
    for (uint64_t i = 0; i < n_q; ++i) {
        const uint64_t p = splitmix64(q_seed * 0x9E3779B97F4A7C15ULL + i) % n_docs;
        if (pick) pick[i] = p;
        synth_row(doc_seed, p, dims, x.data());
        float* q = out + i * (uint64_t)dims;
        float ss = 0.0f;
        for (int d = 0; d < dims; ++d) q[d] = x[d] + sigma * ih_gauss(noise_seed, i * (uint64_t)dims + (uint64_t)d);
        for (int d = 0; d < dims; ++d) ss += q[d] * q[d];
        const float nrm = std::fmax(std::sqrt(ss), 1e-12f);
        for (int d = 0; d < dims; ++d) q[d] = q[d] / nrm;
    }
}

int ora_topk_by_key(const float* scores, const uint8_t* active, uint64_t n, uint32_t k, uint64_t* ids,
                    float* out) {
    std::vector<uint64_t> idx;
    for (uint64_t i = 0; i < n; ++i) if (active[i]) idx.push_back(i);
    const size_t kk = std::min<size_t>(k, idx.size());
    std::partial_sort(idx.begin(), idx.begin() + kk, idx.end(), [&](uint64_t a, uint64_t b) {
        if (scores[a] != scores[b]) return scores[a] > scores[b];
        return a < b;
    });
    for (size_t i = 0; i < kk; ++i) {
        ids[i] = ((idx[i] / VPB) << 16) | (idx[i] % VPB);
        out[i] = scores[idx[i]];
    }
    return (int)kk;
}

// ---- exact inner products on the query path -------------------------------------------------
// dot / dot_768 (src/embed.rs:115-152).
float ora_dot(const float* a, const float* b, uint64_t n) {
    if (n == 768) {
        float acc[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
        for (uint64_t i = 0; i < 768; i += 8)
            for (int j = 0; j < 8; ++j) acc[j] = acc[j] + a[i + j] * b[i + j];
        float r = acc[0];
        for (int j = 1; j < 8; ++j) r = r + acc[j];
        return r;
    }
    float s = -0.0f;
    for (uint64_t i = 0; i < n; ++i) s = s + a[i] * b[i];
    return s;
}

// RingBuffer::search_exact (src/ring.rs:109-119): scored.sort_by(desc) is stable.
uint32_t ora_ring_search(const float* pending, uint64_t n, int dims, const float* q, uint32_t k, uint32_t* out_pos,
                         float* out_scores) {
    std::vector<std::pair<float, uint32_t>> sc(n);
    for (uint64_t i = 0; i < n; ++i) sc[i] = {ora_dot(pending + i * (uint64_t)dims, q, (uint64_t)dims), (uint32_t)i};
    std::stable_sort(sc.begin(), sc.end(), [](const auto& x, const auto& y) { return x.first > y.first; });
    const uint32_t m = (uint32_t)std::min<uint64_t>(k, n);
    for (uint32_t i = 0; i < m; ++i) { out_pos[i] = sc[i].second; out_scores[i] = sc[i].first; }
    return m;
}

// QueryPipeline::rerank_exact_rows (src/pipeline.rs:157-169): dot(query, row), stable sort desc.
void ora_rerank_rows(const float* rows, int dims, const float* q, const uint64_t* cand, uint64_t n_cand,
                     uint64_t* out_rows, float* out_scores) {
    std::vector<std::pair<float, uint64_t>> sc(n_cand);
    for (uint64_t i = 0; i < n_cand; ++i) sc[i] = {ora_dot(q, rows + cand[i] * (uint64_t)dims, (uint64_t)dims), cand[i]};
    std::stable_sort(sc.begin(), sc.end(), [](const auto& x, const auto& y) { return x.first > y.first; });
    for (uint64_t i = 0; i < n_cand; ++i) { out_rows[i] = sc[i].second; out_scores[i] = sc[i].first; }
}

}  // extern "C"
