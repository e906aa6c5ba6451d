// scan_common.cuh — slot decode and scoring helpers shared by the single-query scan (scan.cu)
// and the batched scan (bscan.cu): fast-mode integer stage sums over shared-memory tables, the
// VectorMeta decode, the f32 score formulas of the reference, page loads, and warp sorting
// networks over 64-bit selection keys.
#pragma once
#include "mrl_internal.cuh"

namespace mrl {
namespace {

typedef unsigned long long u64;
constexpr unsigned kFull = 0xffffffffu;

struct Scalars {
    float eden_mean_ip, prefix_sum, mid_mean_ip, w_s4, mid_base, tail_base;
    double un_prefix, un_s1, un_s4, un_l0;
    float unf_prefix, unf_s1, unf_s4, unf_l0;  // 2^-shift as f32 when every product stays normal
    uint32_t eden, mid_b1, has_tail, depth, f32_unscale;
    int32_t one;  // runtime 1: integer accumulations written as v * one + acc issue on the FMA pipe
};

__device__ __forceinline__ int lds_byte(const int* tab, uint32_t byte_off) {
    return *reinterpret_cast<const int*>(reinterpret_cast<const char*>(tab) + byte_off);
}

// v * 2^-shift rounded to f32. With |v| < 2^31 and -96 <= shift <= 126 every nonzero product
// is a normal f32, so rounding v first and scaling by the exact power of two equals rounding the
// exact product (the double-precision path, used otherwise).
__device__ __forceinline__ float unfix(int32_t v, double unscale, float unscale_f, bool use_f) {
    if (use_f) return __fmul_rn(__int2float_rn(v), unscale_f);
    return __double2float_rn(__dmul_rn((double)v, unscale));
}

// Sum of 64 per-dimension table entries, tab[d*16 + level_d]. The accumulations are written as
// v * one + acc (one == 1 at run time) so they issue on the FMA pipe, leaving the ALU pipe to the
// byte extraction.
__device__ __forceinline__ int32_t prefix_fixed(const uint4& c0, const uint4& c1, const int* tab, int32_t one) {
    const uint32_t w[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    int32_t acc0 = 0, acc1 = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t e = (w[j] << 2) & 0x3C3C3C3Cu;  // levels of dims 8j, 8j+2, 8j+4, 8j+6 (x4)
        const uint32_t o = (w[j] >> 2) & 0x3C3C3C3Cu;  // levels of dims 8j+1, +3, +5, +7 (x4)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            acc0 = lds_byte(tab, (8 * j + 2 * k) * 64 + __byte_perm(e, 0, 0x4440 + k)) * one + acc0;
            acc1 = lds_byte(tab, (8 * j + 2 * k + 1) * 64 + __byte_perm(o, 0, 0x4440 + k)) * one + acc1;
        }
    }
    return acc0 + acc1;
}

// Sum over 5-bit windows of an `NBITS`-bit little-endian bit string held in `words`.
template <int NBITS>
__device__ __forceinline__ int32_t window_fixed(const uint32_t* words, const int* tab, int32_t one) {
    constexpr int kWords = NBITS / 32;
    constexpr int kWin = (NBITS + 4) / 5;
    int32_t acc0 = 0, acc1 = 0;
#pragma unroll
    for (int g = 0; g < kWin; ++g) {
        const int start = 5 * g, q = start >> 5, r = start & 31;
        uint32_t idx4;
        if (r < 2) {
            idx4 = (words[q] << (2 - r)) & 0x7Cu;
        } else if (r + 5 > 32 && q + 1 < kWords) {
            idx4 = __funnelshift_r(words[q], words[q + 1], r - 2) & 0x7Cu;
        } else {
            idx4 = (words[q] >> (r - 2)) & 0x7Cu;
        }
        const int v = lds_byte(tab, g * 128 + idx4);
        if (g & 1) acc1 = v * one + acc1; else acc0 = v * one + acc0;
    }
    return acc0 + acc1;
}

__device__ __forceinline__ uint32_t level_of(const uint4& c0, const uint4& c1, int d) {
    const uint32_t w[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    return (w[d >> 3] >> (4 * (d & 7))) & 15u;
}

struct Partials {
    int32_t p, s1, s4;
};

// VectorMeta decode (src/block.rs:60-90) with the scan's clamps (src/scan.rs:495-496); the
// rho = flags/255 and sqrt(max(1 - rho^2, 0)) factors come from a 256-entry table computed with
// the same correctly rounded f32 operations.
__device__ __forceinline__ SlotMeta slot_meta_tab(uint32_t w2, uint32_t w3, const float2* rho_tab) {
    SlotMeta m;
    m.scale = __half2float(__ushort_as_half((unsigned short)(w2 & 0xFFFFu)));
    m.offset = __half2float(__ushort_as_half((unsigned short)(w2 >> 16)));
    const float t = fmaxf(__half2float(__ushort_as_half((unsigned short)(w3 & 0xFFFFu))), 0.0f);
    const float2 rs = rho_tab[(w3 >> 16) & 0xFFu];
    m.tomb = (w3 >> 24) != 0u;
    m.mid_n = fmaxf(__fmul_rn(rs.y, t), 1e-6f);
    m.high_n = fmaxf(__fmul_rn(rs.x, t), 0.0f);
    return m;
}

// Fast-mode score from the three integer stage sums (depth L1 or full; src/scan.rs:499-505,
// 546-547, 566, 631).
__device__ __forceinline__ float fast_score(const SlotMeta& m, int32_t P, int32_t s1, int32_t s4, const Scalars& S) {
    const float cd = unfix(P, S.un_prefix, S.unf_prefix, S.f32_unscale);
    float sc = S.eden ? __fadd_rn(S.eden_mean_ip, __fmul_rn(m.scale, cd))
                      : __fadd_rn(__fmul_rn(cd, m.scale), __fmul_rn(m.offset, S.prefix_sum));
    if (S.depth >= MRL_DEPTH_L1) {
        const float v = unfix(s1, S.un_s1, S.unf_s1, S.f32_unscale);
        if (S.mid_b1) sc = __fadd_rn(sc, __fadd_rn(S.mid_mean_ip, __fmul_rn(m.offset, v)));
        else sc = __fadd_rn(sc, __fmul_rn(v, m.mid_n));
    }
    if (S.depth == MRL_DEPTH_FULL && S.has_tail) {
        const float v = unfix(s4, S.un_s4, S.unf_s4, S.f32_unscale);
        sc = __fadd_rn(sc, __fmul_rn(__fmul_rn(v, fmaxf(m.high_n, 1e-6f)), S.w_s4));
    }
    return sc;
}

struct Slot4 {
    uint4 c0, c1, c2, c3;
};

__device__ __forceinline__ void load_slot(const uint4* __restrict__ pages, uint32_t b, int v, Slot4& s) {
    const uint4* p = pages + (size_t)b * 256 + v;
    s.c0 = __ldg(p);
    s.c1 = __ldg(p + 64);
    s.c2 = __ldg(p + 128);
    s.c3 = __ldg(p + 192);
}

__device__ __forceinline__ bool block_live(const ScanLaunch& p, uint32_t b) {
    if (!p.use_time) return true;
    const uint2 t = __ldg(p.block_ts + b);  // [min_ts, max_ts], src/scan.rs:719-730
    if (p.has_lo && t.y < p.lo) return false;
    if (p.has_hi && t.x > p.hi) return false;
    return true;
}

// ---- warp sorting networks over 64-bit keys (lane i holds rank i, descending) ----
__device__ __forceinline__ u64 umax64(u64 a, u64 b) { return a > b ? a : b; }
__device__ __forceinline__ u64 umin64(u64 a, u64 b) { return a < b ? a : b; }

__device__ __forceinline__ u64 warp_sort32(u64 x, int lane) {
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            const u64 y = __shfl_xor_sync(kFull, x, j);
            const bool keep_max = ((lane & j) == 0) == ((lane & k) == 0);
            x = keep_max ? umax64(x, y) : umin64(x, y);
        }
    }
    return x;
}

// Top 32 of two descending lists, descending.
__device__ __forceinline__ u64 warp_merge32(u64 L, u64 S, int lane) {
    u64 x = umax64(L, __shfl_sync(kFull, S, 31 - lane));
#pragma unroll
    for (int j = 16; j > 0; j >>= 1) {
        const u64 y = __shfl_xor_sync(kFull, x, j);
        x = ((lane & j) == 0) ? umax64(x, y) : umin64(x, y);
    }
    return x;
}

// Scalars of one plan: its stage scalars, 2^-shift both as f64 and (when every product stays a
// normal f32) as f32, codec flags, and the scan's w_s4 and depth.
__device__ __forceinline__ void fill_scalars(const DevPlan* __restrict__ P, float w_s4, uint32_t depth, int32_t one,
                                             Scalars& S) {
    S.eden_mean_ip = P->qp.eden_mean_ip;
    S.prefix_sum = P->qp.prefix_sum;
    S.mid_mean_ip = P->qp.eden_mid_mean_ip;
    S.w_s4 = w_s4;
    S.mid_base = P->mid_base;
    S.tail_base = P->tail_base;
    S.un_prefix = P->unscale_prefix;
    S.un_s1 = P->unscale_s1;
    S.un_s4 = P->unscale_s4;
    S.un_l0 = P->unscale_l0;
    const int sh[4] = {P->shift_prefix, P->shift_s1, P->shift_s4, P->shift_l0};
    bool ok = true;
    for (int i = 0; i < 4; ++i) ok = ok && sh[i] >= -96 && sh[i] <= 126;
    S.f32_unscale = ok ? 1u : 0u;
    S.unf_prefix = ok ? __double2float_rn(P->unscale_prefix) : 0.0f;
    S.unf_s1 = ok ? __double2float_rn(P->unscale_s1) : 0.0f;
    S.unf_s4 = ok ? __double2float_rn(P->unscale_s4) : 0.0f;
    S.unf_l0 = ok ? __double2float_rn(P->unscale_l0) : 0.0f;
    S.eden = P->qp.prefix_codec == MRL_PREFIX_EDEN;
    S.mid_b1 = P->qp.mid_codec == MRL_MID_EDEN_B1;
    S.has_tail = P->qp.has_tail_fold;
    S.depth = depth;
    S.one = one;
}

// rho_ratio = flags / 255 and sqrt(max(1 - r^2, 0)) (src/block.rs:74-84) for every flags byte.
__device__ __forceinline__ void fill_rho_tab(float2* rho_tab, int tid, int nthr) {
    for (int i = tid; i < 256; i += nthr) {
        const float rho = __fdiv_rn((float)i, 255.0f);
        const float r = fminf(fmaxf(rho, 0.0f), 1.0f);
        rho_tab[i] = make_float2(rho, __fsqrt_rn(fmaxf(__fsub_rn(1.0f, __fmul_rn(r, r)), 0.0f)));
    }
}

}  // namespace
}  // namespace mrl
