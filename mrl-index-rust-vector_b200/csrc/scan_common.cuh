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


// Shared-memory table layout of the single-query scan (ints in fast mode, floats in exact mode).
constexpr int kTabInts = kPrefix * 16 + kS1Windows * 32 + kS4Windows * 32 + kPrefix * 16;  // 3296
constexpr int kTabS1 = kPrefix * 16;
constexpr int kTabS4 = kTabS1 + kS1Windows * 32;
constexpr int kTabL0 = kTabS4 + kS4Windows * 32;
// exact-mode layout inside the same table space (floats)
constexpr int kTabMidW = kPrefix * 16;
constexpr int kTabTailW = kTabMidW + kRabitq;
constexpr int kTabBw3 = kTabTailW + kFold;

// Full score of one slot; returns false for tombstoned slots.
template <int MODE>
__device__ __forceinline__ bool slot_score(const uint4& c0, const uint4& c1, const uint4& c2,
                                           const uint4& c3, const int* tab, const float2* rho_tab,
                                           const Scalars& S, float& score, Partials* parts) {
    const SlotMeta m = slot_meta_tab(c3.z, c3.w, rho_tab);
    if (m.tomb) return false;
    if (MODE == MRL_MODE_FAST) {
        const uint32_t s1w[4] = {c2.x, c2.y, c2.z, c2.w};
        const uint32_t s4w[2] = {c3.x, c3.y};
        if (S.depth == MRL_DEPTH_L0) {  // src/scan.rs:753-771
            const int32_t P = prefix_fixed(c0, c1, tab + kTabL0, S.one);
            const float cd = unfix(P, S.un_l0, S.unf_l0, S.f32_unscale);
            score = __fadd_rn(__fmul_rn(cd, m.scale), __fmul_rn(m.offset, S.prefix_sum));
            if (parts) {
                parts->p = P;
                parts->s1 = window_fixed<128>(s1w, tab + kTabS1, S.one);
                parts->s4 = window_fixed<64>(s4w, tab + kTabS4, S.one);
            }
            return true;
        }
        const int32_t P = prefix_fixed(c0, c1, tab, S.one);
        int32_t s1 = 0, s4 = 0;
        if (S.depth >= MRL_DEPTH_L1 || parts) s1 = window_fixed<128>(s1w, tab + kTabS1, S.one);
        if ((S.depth == MRL_DEPTH_FULL && S.has_tail) || parts) s4 = window_fixed<64>(s4w, tab + kTabS4, S.one);
        if (parts) { parts->p = P; parts->s1 = s1; parts->s4 = s4; }
        score = fast_score(m, P, s1, s4, S);
        return true;
    } else {
        const float* ft = reinterpret_cast<const float*>(tab);
        if (S.depth == MRL_DEPTH_L0) {
            float acc = 0.0f;
#pragma unroll
            for (int d = 0; d < kPrefix; ++d)
                if (level_of(c0, c1, d) & 8u) acc = __fadd_rn(acc, ft[kTabBw3 + d]);
            score = __fadd_rn(__fmul_rn(acc, m.scale), __fmul_rn(m.offset, S.prefix_sum));
            return true;
        }
        float acc = 0.0f;  // src/scan.rs:456-487, per-slot sequential order over d
        {
            const uint32_t w[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
            for (int d = 0; d < kPrefix; ++d) {
                const uint32_t sh = 4 * (d & 7);
                const uint32_t idx4 = sh >= 2 ? ((w[d >> 3] >> (sh - 2)) & 0x3Cu) : ((w[d >> 3] << 2) & 0x3Cu);
                acc = __fadd_rn(acc, *reinterpret_cast<const float*>(reinterpret_cast<const char*>(ft) + d * 64 + idx4));
            }
        }
        float sc = S.eden ? __fadd_rn(S.eden_mean_ip, __fmul_rn(m.scale, acc))
                          : __fadd_rn(__fmul_rn(acc, m.scale), __fmul_rn(m.offset, S.prefix_sum));
        if (S.depth >= MRL_DEPTH_L1) {  // src/scan.rs:520-569
            const uint32_t s1w[4] = {c2.x, c2.y, c2.z, c2.w};
            float s = S.mid_base;
            const float4* mw = reinterpret_cast<const float4*>(ft + kTabMidW);
#pragma unroll
            for (int g = 0; g < kRabitq / 4; ++g) {
                const float4 w4 = mw[g];
                const uint32_t bits = s1w[g >> 3] >> (4 * (g & 7));
                if (bits & 1u) s = __fadd_rn(s, w4.x);
                if (bits & 2u) s = __fadd_rn(s, w4.y);
                if (bits & 4u) s = __fadd_rn(s, w4.z);
                if (bits & 8u) s = __fadd_rn(s, w4.w);
            }
            if (S.mid_b1) sc = __fadd_rn(sc, __fadd_rn(S.mid_mean_ip, __fmul_rn(m.offset, s)));
            else sc = __fadd_rn(sc, __fmul_rn(s, m.mid_n));
        }
        if (S.depth == MRL_DEPTH_FULL && S.has_tail) {  // src/scan.rs:610-634
            const uint32_t s4w[2] = {c3.x, c3.y};
            float t = S.tail_base;
            const float4* tw = reinterpret_cast<const float4*>(ft + kTabTailW);
#pragma unroll
            for (int g = 0; g < kFold / 4; ++g) {
                const float4 w4 = tw[g];
                const uint32_t bits = s4w[g >> 3] >> (4 * (g & 7));
                if (bits & 1u) t = __fadd_rn(t, w4.x);
                if (bits & 2u) t = __fadd_rn(t, w4.y);
                if (bits & 4u) t = __fadd_rn(t, w4.z);
                if (bits & 8u) t = __fadd_rn(t, w4.w);
            }
            sc = __fadd_rn(sc, __fmul_rn(__fmul_rn(t, fmaxf(m.high_n, 1e-6f)), S.w_s4));
        }
        score = sc;
        return true;
    }
}

// Upper bound on |fast-mode score - exact-mode score| for every slot whose meta factors lie within
// mm = {max |scale|, max |offset|, max mid_n, max max(high_n, 1e-6)} (a segment's maxima). Both
// modes approximate the same real-valued stage sums of the same f32 table values:
//   * the exact mode's sequential f32 sum of n terms is within gamma_{n-1} * sum |terms| of the
//     real sum (recursive summation; Higham, Accuracy and Stability of Numerical Algorithms,
//     2nd ed., 4.2), plus one product rounding per term where the terms are products; the mid band
//     and tail sums start from an f32 base that is itself a 128- or 64-term sum;
//   * the fast mode's integer sum of n entries rint(v * 2^shift) is within n/2 units of 2^-shift of
//     the real sum, plus the rounding of its conversion to f32;
// and each mode's score formula (src/scan.rs:499-505, 546-547, 566, 631) rounds at most 8 times,
// each time by at most u = 2^-24 of a value no larger than the sum of all term magnitudes. The
// coefficients below round those counts up, and the total is doubled for slack. Not finite (+inf)
// when the segment holds non-finite factors.
__device__ __forceinline__ float fast_error_bound(const DevPlan& P, float4 mm, float w_s4, uint32_t depth) {
    const double u = 0x1p-24;
    const double sc = mm.x, of = mm.y, mid = mm.z, hp = mm.w, w = fabs((double)w_s4);
    const bool eden = P.qp.prefix_codec == MRL_PREFIX_EDEN, b1 = P.qp.mid_codec == MRL_MID_EDEN_B1;
    double dev, mag;
    if (depth == MRL_DEPTH_L0) {  // code_dot * scale + offset * prefix_sum (src/scan.rs:753-771)
        const double dp = 72.0 * u * P.err_0 + 40.0 * P.unscale_l0;
        dev = sc * dp;
        mag = sc * (P.err_0 + dp) + of * fabs((double)P.qp.prefix_sum);
    } else {
        const double dp = 72.0 * u * P.err_p + 40.0 * P.unscale_prefix;
        dev = sc * dp;
        mag = (eden ? fabs((double)P.qp.eden_mean_ip) : of * fabs((double)P.qp.prefix_sum)) + sc * (P.err_p + dp);
        const double d1 = 530.0 * u * P.err_1 + 70.0 * P.unscale_s1, f1 = b1 ? of : mid;
        dev += f1 * d1;
        mag += f1 * (P.err_1 + d1) + (b1 ? fabs((double)P.qp.eden_mid_mean_ip) : 0.0);
        if (depth == MRL_DEPTH_FULL && P.qp.has_tail_fold) {
            const double d4 = 270.0 * u * P.err_4 + 40.0 * P.unscale_s4;
            dev += hp * w * d4;
            mag += hp * w * (P.err_4 + d4);
        }
    }
    const double e = 2.0 * (dev + 16.0 * u * mag) + 1e-35;
    return e < 3.0e38 ? __double2float_ru(e) : __int_as_float(0x7F800000);
}

}  // namespace
}  // namespace mrl
