// plan_build.cuh — the query-side plan build (QueryPlan::from_query_codec, src/scan.rs:105-266) as
// a device function run by a whole CTA (at least 256 threads), shared by the standalone plan kernel
// (plan.cu) and the scan kernel's fused plan prologue (scan.cu).
//
// The Rademacher signs are computed while the query loads are in flight; eight warps then build
// independent parts of the plan (prefix, mid band, folded tail, long reductions, the raw-query
// sums), and every thread of the CTA fills the tables. FWHTs run on warp shuffles (each butterfly
// output depends only on its two inputs, so the values equal the sequential loop's); each
// sequential reduction runs on one lane in the reference's order over addends the warp formed in
// parallel; every f32 operation is an explicit round-to-nearest intrinsic (the library is compiled
// with -fmad=false), so the plan is bit-identical to the reference arithmetic. The build also makes
// the two scoring-table sets the scan uses, written either into the plan or straight into a scan's
// shared-memory tables:
//   * fast mode: per-stage int32 tables whose exact integer sums replace the f32 loops; entries
//     are rint(v * 2^shift) of exact products v of two f32 values (computed in integer
//     arithmetic, fix_prod), with shift chosen so that every stage sum stays below 2^30 in
//     magnitude;
//   * exact mode: the f32 products / addends of the reference loops.
#pragma once

#include "mrl_internal.cuh"

namespace mrl {
namespace planb {

__device__ __forceinline__ float f_add(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float f_sub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float f_mul(float a, float b) { return __fmul_rn(a, b); }

// Correctly rounded f32 values of the reference's constant expressions: 1/sqrt(64), 1/sqrt(128),
// 2/pi (pi rounded to f32 first), sqrt(2/pi)/sqrt(128) (src/rotate.rs:46-49) and sqrt(2/pi)/8
// (src/rotate.rs:124-126), each operation rounded to nearest as the reference's f32 arithmetic
// does. IEEE division and square root are correctly rounded, so these equal what __fdiv_rn and
// __fsqrt_rn compute from the same operands.
constexpr float kInvSqrt64 = 0x1p-3f;
constexpr float kInvSqrt128 = 0x1.6a09e6p-4f;
constexpr float kRabitqScale = 0x1.20dd74p-4f;
constexpr float kTailScale = 0x1.988452p-4f;

// One fwht_inplace (src/rotate.rs:13-33) over n = 32*R values held by one warp, element
// lane + 32*r in v[r]. Stage h pairs elements j and j+h (bit h of j clear) into (x+y, x-y): for
// h < 32 the partner sits in lane ^ h of the same register, for h >= 32 in register r ^ (h/32) of
// the same lane. Each output is computed from the same two operands as the sequential loop, so
// the values are identical. The final scale is 1/sqrt(n) rounded to f32.
template <int R>
__device__ __forceinline__ void fwht_warp(float (&v)[R], int lane) {
    static_assert(R == 2 || R == 4, "64 or 128 values");
#pragma unroll
    for (int h = 1; h < 32; h <<= 1) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const float o = __shfl_xor_sync(0xffffffffu, v[r], h);
            v[r] = (lane & h) ? f_sub(o, v[r]) : f_add(v[r], o);
        }
    }
#pragma unroll
    for (int hr = 1; hr < R; hr <<= 1) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
            if (!(r & hr)) {
                const float x = v[r], y = v[r + hr];
                v[r] = f_add(x, y);
                v[r + hr] = f_sub(x, y);
            }
        }
    }
    const float scale = R == 2 ? kInvSqrt64 : kInvSqrt128;
#pragma unroll
    for (int r = 0; r < R; ++r) v[r] = f_mul(v[r], scale);
}

__device__ __forceinline__ int stage_shift(double maxabs, int count) {
    if (!(maxabs > 0.0)) return 0;
    int k = 0;
    frexp(maxabs * (double)count, &k);
    return 30 - k;
}
// 2^e as a double (exact for the shifts a plan uses; ldexp outside the normal range)
__device__ __forceinline__ double pow2(int e) {
    return e >= -1022 && e <= 1023 ? __longlong_as_double((long long)(1023 + e) << 52) : ldexp(1.0, e);
}
// rint(a * b * 2^sh), nearest-even, for finite f32 a and b: the exact product of the two 24-bit
// significands (at most 48 bits), scaled by a power of two and rounded once, all in integer
// arithmetic. It equals __double2int_rn((double)a * (double)b * 2^sh) (the double product is exact)
// whenever the result fits in int32, which the stage shifts guarantee; double-precision
// arithmetic is slow on this part and sits on every scan's critical path here.
__device__ __forceinline__ int32_t fix_prod(float a, float b, int sh) {
    const uint32_t ua = __float_as_uint(a), ub = __float_as_uint(b);
    const uint32_t xa = (ua >> 23) & 0xFFu, xb = (ub >> 23) & 0xFFu;
    const uint64_t ma = (ua & 0x7FFFFFu) | (xa ? 0x800000u : 0u);
    const uint64_t mb = (ub & 0x7FFFFFu) | (xb ? 0x800000u : 0u);
    const uint64_t prod = ma * mb;
    const int e = (int)(xa ? xa : 1u) + (int)(xb ? xb : 1u) - 300 + sh;  // |a * b * 2^sh| = prod * 2^e
    uint64_t q;
    if (e >= 0) {
        q = e < 31 ? prod << e : 0ull;  // e >= 31 only for prod == 0 when the result fits
    } else if (e <= -64) {
        q = 0ull;  // prod < 2^48 < 2^(-e-1): below one half
    } else {
        const int n = -e;
        q = prod >> n;
        const uint64_t rem = prod - (q << n), half = 1ull << (n - 1);
        q += (rem > half || (rem == half && (q & 1ull))) ? 1ull : 0ull;
    }
    const int32_t v = (int32_t)q;
    return ((ua ^ ub) & 0x80000000u) ? -v : v;
}

// Largest |x| over the warp, as a double, as fmax over the lanes would give it (NaN lanes ignored;
// 0 if every lane is NaN or zero): nonnegative floats order like their bit patterns. fmaxf also
// ignores a NaN operand, so per-lane maxima taken with it keep that rule.
__device__ __forceinline__ double warp_max_abs(float x) {
    const float a = fabsf(x);
    const unsigned b = a == a ? __float_as_uint(a) : 0u;
    return (double)__uint_as_float(__reduce_max_sync(0xffffffffu, b));
}
__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
// One reference-order sequential f32 sum per lane: acc = ((0 + row[0]) + row[1]) + ... A lane
// that subtracts holds the negated terms (x - y and x + (-y) round identically).
__device__ __forceinline__ float lane_chain(const float* row, int len) {
    float acc = 0.0f;
#pragma unroll 8
    for (int d = 0; d < len; ++d) acc = f_add(acc, row[d]);
    return acc;
}
// A double sum of nonnegative terms rounded up to f32 with room for the double roundings: the
// error-bound magnitudes stored in the plan (err_p, err_1, err_4, err_0).
__device__ __forceinline__ float bound_up(double v) { return __double2float_ru(v * (1.0 + 0x1p-40)); }

// Entry (g, m) of a fast-mode window table of one 1-bit stage (lut_s1 / lut_s4): the exact integer
// sum over the window's dims i of fix(bit i of m ? val1 : val0). `fx` holds the fixed values per
// dim interleaved (fx[2 i] for bit 0, fx[2 i + 1] for bit 1).
template <int DIMS>
__device__ __forceinline__ int32_t window_entry(const int32_t* fx, int g, int m) {
    const int w = min(5, DIMS - 5 * g);
    if (m >= (1 << w)) return 0;
    int32_t sum = 0;
#pragma unroll
    for (int i = 0; i < 5; ++i)
        if (i < w) sum += fx[2 * (5 * g + i) + ((m >> i) & 1)];
    return sum;
}

// Entry m of the 4-dim window table g of a 1-bit stage (lut4_s1 / lut4_s4): the same exact sum
// over 4 dims instead of 5, so the batched scan's stage sums are the same integers.
__device__ __forceinline__ int32_t window4_entry(const int32_t* fx, int g, int m) {
    int32_t sum = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) sum += fx[2 * (4 * g + i) + ((m >> i) & 1)];
    return sum;
}

// What a plan build writes: kNeedAll = every field of DevPlan (the stored plan); a scan that only
// needs its own mode's tables asks for kNeedFast (+ kNeedL0 at depth L0Only) or kNeedExact. The
// scalars and shifts are always written to the plan; the tables go where PlanDest points.
constexpr uint32_t kNeedFast = 1u, kNeedExact = 2u, kNeedL0 = 4u, kNeedBatch = 8u, kNeedAll = 0xFu;

// Where the build writes its scoring tables: the plan's own arrays (plan_dest), or a scan's
// shared-memory tables directly. bw3 (bit_weights[d][3], contiguous) is null for the plan, whose
// bit_weights hold all four columns.
struct PlanDest {
    int32_t* lut_prefix;
    int32_t* lut_s1;
    int32_t* lut_s4;
    int32_t* lut_l0;
    float* fp_prefix;
    float* mid_w;
    float* tail_w;
    float* bw3;
};
__device__ __forceinline__ PlanDest plan_dest(DevPlan* P) {
    return PlanDest{P->lut_prefix, P->lut_s1, P->lut_s4, P->lut_l0, P->fp_prefix, P->mid_w, P->tail_w, nullptr};
}

constexpr int kSigns = kPrefix + kRabitq + kFoldBlocks * kPrefix;  // 768
// rows of PlanShared::terms: the addends of the reference-order sequential sums
enum { kRowL1, kRowSum, kRowIp, kRowMs, kRowMip, kRowBase, kRowB1, kRowTb, kRowBud, kRows };

// Shared scratch of one plan build (besides the dims-float query copy).
struct PlanShared {
    float mean[kPrefix + kRabitq];
    float rot[kPrefix];
    int32_t fx[2 * (kRabitq + kFold)];  // fixed 1-bit stage values, see window_entry
    float scal[16];
    float cb[16];
    float w[kPrefix];  // EDEN prefix weight per dim: rot[d] / sqrt(64)
    int32_t psh[2];    // shift of the prefix and L0 tables
    // Rademacher signs: EDEN prefix rotation (64), EdenB1 mid-band rotation (128), tail fold
    // blocks (9 x 64)
    float sg[kSigns];
    float terms[kRows][kRabitq];
};

// Sign t of PlanShared::sg: rademacher_diag (src/eden.rs:75-88) of the prefix and mid band, and
// tail_rademacher (src/rotate.rs:53-67) of fold block b, dim d.
__device__ __forceinline__ float plan_sign(int t, uint64_t eden_seed, uint64_t mid_seed) {
    if (t < kPrefix) return sign_hash(eden_seed, (uint64_t)t);
    if (t < kPrefix + kRabitq) return sign_hash(mid_seed, (uint64_t)(t - kPrefix));
    const int f = t - kPrefix - kRabitq;
    return sign_hash((uint64_t)(f / kPrefix), (uint64_t)(f % kPrefix));
}

// The build's inputs into shared memory: the query, the codec centres, the b=4 codebook, and the
// Rademacher signs (computed while the loads are in flight). Every thread of the CTA calls it;
// build_plan synchronises before reading them.
template <bool kParamQuery = false>
__device__ __forceinline__ void plan_inputs(const float* __restrict__ q, uint32_t dims, const float* __restrict__ eden_mean,
                                            const float* __restrict__ mid_mean, uint64_t eden_seed, uint64_t mid_seed,
                                            float* s_q, PlanShared& sh) {
    const int tid = threadIdx.x, nthr = blockDim.x;
    // the loads are issued before the work and stores that consume them, so their latencies overlap
    float m = 0.0f, c = 0.0f;
    if (tid < kPrefix + kRabitq) {  // either centre array may be NULL
        const float* src = tid < kPrefix ? eden_mean : mid_mean;
        m = src ? __ldg(src + (tid < kPrefix ? tid : tid - kPrefix)) : 0.0f;
    }
    if (tid < 16) c = g_lloyd_b4[tid];
    if (kParamQuery) {
        // the query sits in the kernel's parameter bank (16-byte aligned), where lanes that read
        // different addresses are served one address at a time: each warp reads whole 16-byte
        // chunks at one address per instruction, and one lane stores them
        const int lane = tid & 31, warp = tid >> 5, nw = nthr >> 5;
        const uint32_t n4 = dims / 4u;
        const float4* q4 = reinterpret_cast<const float4*>(q);
        float4* s4 = reinterpret_cast<float4*>(s_q);
        for (uint32_t j = warp; j < n4; j += 4u * nw) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (j + u * nw < n4) v[u] = q4[j + u * nw];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (lane == 0 && j + u * nw < n4) s4[j + u * nw] = v[u];
        }
        for (uint32_t i = 4u * n4 + warp; i < dims; i += nw) {
            const float v = q[i];
            if (lane == 0) s_q[i] = v;
        }
        for (int t = tid; t < kSigns; t += nthr) sh.sg[t] = plan_sign(t, eden_seed, mid_seed);
    } else {
        const uint32_t i0 = tid, i1 = tid + nthr;
        const float v0 = i0 < dims ? q[i0] : 0.0f;  // plain loads: q may be global or kernel-parameter memory
        const float v1 = i1 < dims ? q[i1] : 0.0f;
        for (int t = tid; t < kSigns; t += nthr) sh.sg[t] = plan_sign(t, eden_seed, mid_seed);
        if (i0 < dims) s_q[i0] = v0;
        if (i1 < dims) s_q[i1] = v1;
        for (uint32_t i = tid + 2u * nthr; i < dims; i += nthr) s_q[i] = q[i];
    }
    if (tid < kPrefix + kRabitq) sh.mean[tid] = m;
    if (tid < 16) sh.cb[tid] = c;
}

// The mid band's two rotations (src/rotate.rs:36-42 and, for EdenB1, src/scan.rs:159-174) by one
// warp: rq = FWHT128 of the raw mid band, mq = FWHT128 of its Rademacher-signed copy (EdenB1 only).
__device__ __forceinline__ void mid_rotations(const float* s_q, const PlanShared& sh, bool mid_b1, int lane,
                                              float (&rq)[4], float (&mq)[4]) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int i = lane + 32 * r;
        rq[r] = s_q[kPrefix + i];
        mq[r] = f_mul(s_q[kPrefix + i], sh.sg[kPrefix + i]);
    }
    fwht_warp<4>(rq, lane);
    if (mid_b1) fwht_warp<4>(mq, lane);
}

// fold_tail (src/rotate.rs:73-93) then FWHT64 (rotate_tail_fold) by one warp.
__device__ __forceinline__ void tail_rotation(const float* s_q, const PlanShared& sh, uint32_t dims, bool has_tail,
                                              int lane, float (&u)[2]) {
    u[0] = 0.0f;
    u[1] = 0.0f;
    if (has_tail) {
        const int nb = min((int)((dims - kTailStart) / kPrefix), kFoldBlocks);
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int d = lane + 32 * r;
            for (int b = 0; b < nb; ++b)
                u[r] = f_add(u[r], f_mul(sh.sg[kPrefix + kRabitq + b * kPrefix + d], s_q[kTailStart + b * kPrefix + d]));
        }
    }
    fwht_warp<2>(u, lane);
}

// Phase A, threads 0..255 in eight warp roles (independent until phase B). The longest
// sequential sums (128 terms) set its length, so each runs on a warp of its own, and the warps
// that need a rotation's values for other work recompute the rotation instead of waiting for it:
//   warp 0: prefix — EDEN query rotation, bit weights, prefix weights and the prefix shift;
//   warp 1: mid band — the rabitq_base and EdenB1 base sums;
//   warp 6: mid band — mid_w, the S1 shift and fixed values, the stored plan's mid-band fields;
//   warp 2: folded tail — the tail_fold_base and s4_abs_budget sums;
//   warp 7: folded tail — tail_w, the S4 shift and fixed values, the stored plan's tail fields;
//   warp 3: q_tail_sq (the longest sequential sum) and rabitq_lut, for a full plan only;
//   warp 4: the prefix sums of the raw query (prefix_l1, prefix_sum, eden_mean_ip) and the L0 shift;
//   warp 5: the mid-band sums of the raw query (q_mid_sq, eden_mid_mean_ip);
//   warps 8 and up, when `rho_tab` is given: the scan's rho table (fill_rho_tab).
// Each sequential sum keeps the reference's order: the warp first forms its addends in parallel,
// then one lane per sum adds them in sequence (lane_chain).
// Phase B, every thread of the CTA: the tables `need` asks for, written through `dst`.
// Every thread of the CTA (at least 256, and more than 256 to fill `rho_tab`) must call it, after
// plan_inputs; P may be global or shared memory, s_q holds the dims floats plan_inputs loaded.
__device__ __forceinline__ void build_plan(uint32_t dims, uint32_t prefix_codec, uint32_t mid_codec, DevPlan* P,
                                           float* s_q, PlanShared& sh, uint32_t need, const PlanDest& dst,
                                           float2* rho_tab = nullptr) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nthr = blockDim.x;
    const bool full = need == kNeedAll;
    mrl_query_plan* qp = &P->qp;
    float* s_mean = sh.mean;
    float* s_rot = sh.rot;
    int32_t* s_fx = sh.fx;
    float* s_scal = sh.scal;
    float* s_cb = sh.cb;
    const bool eden = prefix_codec == MRL_PREFIX_EDEN;
    const bool mid_b1 = mid_codec == MRL_MID_EDEN_B1;
    const bool has_tail = dims > (uint32_t)kTailStart;

    __syncthreads();  // plan_inputs done

    if (warp == 0) {
        // ---- prefix copy + bit weights (src/scan.rs:126-140), EDEN rotate_query (src/eden.rs:275-281)
        float v[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int d = lane + 32 * r;
            const float qd = s_q[d];
            if (full) {
                qp->prefix[d] = qd;
                qp->bit_weights[d][0] = f_mul(qd, 1.0f);
                qp->bit_weights[d][1] = f_mul(qd, 2.0f);
                qp->bit_weights[d][2] = f_mul(qd, 4.0f);
                qp->bit_weights[d][3] = f_mul(qd, 8.0f);
            }
            if (dst.bw3) dst.bw3[d] = f_mul(qd, 8.0f);
            v[r] = f_mul(qd, sh.sg[d]);
        }
        fwht_warp<2>(v, lane);
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            s_rot[lane + 32 * r] = v[r];
            if (full) qp->eden_q_rot[lane + 32 * r] = eden ? v[r] : 0.0f;
        }
        if (full && lane < 16) qp->eden_codebook[lane] = eden ? s_cb[lane] : 0.0f;
        // Prefix weights and shift. An entry is (double)cb[l] * w_d (EDEN) or (double)l * q_d
        // (MinMax), both exact products, so the largest |entry| of dim d is max|cb| * |w_d| or
        // 15 * |q_d|, and the largest over the dims is max|cb| * max|w| or 15 * max|q|.
        const double cbmax = warp_max_abs(lane < 16 ? s_cb[lane] : 0.0f);
        double ea = 0.0;
        float wq[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int d = lane + 32 * r;
            const float w = eden ? f_mul(v[r], kInvSqrt64) : 0.0f;
            sh.w[d] = w;
            wq[r] = eden ? w : s_q[d];
            ea += eden ? cbmax * fabs((double)w) : 15.0 * fabs((double)s_q[d]);
        }
        const double mxa = warp_max_abs(fmaxf(fabsf(wq[0]), fabsf(wq[1])));
        const int sh_p = stage_shift(eden ? cbmax * mxa : 15.0 * mxa, kPrefix);
        ea = warp_sum(ea);
        if (lane == 0) {
            P->err_p = bound_up(ea);
            P->shift_prefix = sh_p;
            P->unscale_prefix = pow2(-sh_p);
            sh.psh[0] = sh_p;
        }
    } else if (warp == 1) {
        // ---- mid band: the addends of rabitq_base (src/scan.rs:180-186, subtracted) and of the
        // EdenB1 base (src/scan.rs:523-532), then the two sums in reference order (lanes 0 and 1)
        float rq[4], mq[4];
        mid_rotations(s_q, sh, mid_b1, lane, rq, mq);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int i = lane + 32 * r;
            sh.terms[kRowBase][i] = -f_mul(rq[r], kRabitqScale);
            sh.terms[kRowB1][i] = f_mul(-kLloydB1Hi, f_mul(mq[r], kInvSqrt128));
        }
        __syncwarp();
        if (lane < 2) {
            const float acc = lane_chain(sh.terms[kRowBase + lane], kRabitq);
            if (lane == 0) s_scal[6] = acc;
            else s_scal[9] = mid_b1 ? acc : 0.0f;
        }
    } else if (warp == 6) {
        // ---- mid band: mid_w, the S1 shift and fixed values, the stored plan's fields
        float rq[4], mq[4];
        mid_rotations(s_q, sh, mid_b1, lane, rq, mq);
        float v1f[4];
        double ea = 0.0;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int i = lane + 32 * r;
            const float pos = f_mul(rq[r], kRabitqScale);
            if (full) {
                qp->rabitq_q[i] = rq[r];
                qp->eden_mid_q_rot[i] = mid_b1 ? mq[r] : 0.0f;
                qp->rabitq_weights2[i] = f_mul(2.0f, pos);
            }
            const float qd = f_mul(mq[r], kInvSqrt128);
            dst.mid_w[i] = mid_b1 ? f_mul(f_sub(kLloydB1Hi, -kLloydB1Hi), qd) : f_mul(2.0f, pos);
            // fixed S1 value of bit 1 (bit 0: its negation): kLloydB1Hi * qd (exact double
            // product) for EdenB1, pos for RaBitQ
            v1f[r] = mid_b1 ? qd : pos;
            const double v1 = mid_b1 ? (double)kLloydB1Hi * (double)qd : (double)pos;
            ea += fabs(v1);
        }
        const double mv = warp_max_abs(fmaxf(fmaxf(fabsf(v1f[0]), fabsf(v1f[1])), fmaxf(fabsf(v1f[2]), fabsf(v1f[3]))));
        const int sh_1 = stage_shift(mid_b1 ? (double)kLloydB1Hi * mv : mv, kRabitq);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int i = lane + 32 * r;
            const int32_t f = fix_prod(mid_b1 ? kLloydB1Hi : v1f[r], mid_b1 ? v1f[r] : 1.0f, sh_1);
            s_fx[2 * i] = -f;
            s_fx[2 * i + 1] = f;
        }
        ea = warp_sum(ea);
        if (lane == 0) {
            P->err_1 = bound_up(ea);
            P->shift_s1 = sh_1;
            P->unscale_s1 = pow2(-sh_1);
        }
    } else if (warp == 2) {
        // ---- folded tail: the addends of tail_fold_base (subtracted) and s4_abs_budget
        // (src/scan.rs:222-233), then the two sums in reference order (lanes 0 and 1)
        float u[2];
        tail_rotation(s_q, sh, dims, has_tail, lane, u);
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int d = lane + 32 * r;
            const float pos = has_tail ? f_mul(u[r], kTailScale) : 0.0f;
            sh.terms[kRowTb][d] = -pos;
            sh.terms[kRowBud][d] = fabsf(pos);
        }
        __syncwarp();
        if (lane < 2) {
            const float acc = has_tail ? lane_chain(sh.terms[kRowTb + lane], kFold) : 0.0f;
            s_scal[7 + lane] = acc;
        }
    } else if (warp == 7) {
        // ---- folded tail: tail_w, the S4 shift and fixed values, the stored plan's fields
        float u[2];
        tail_rotation(s_q, sh, dims, has_tail, lane, u);
        float pf[2];
        double ea = 0.0;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int d = lane + 32 * r;
            const float pos = has_tail ? f_mul(u[r], kTailScale) : 0.0f;
            if (full) {
                qp->tail_fold_q[d] = has_tail ? u[r] : 0.0f;
                qp->tail_fold_weights2[d] = has_tail ? f_mul(2.0f, pos) : 0.0f;
            }
            dst.tail_w[d] = has_tail ? f_mul(2.0f, pos) : 0.0f;
            pf[r] = pos;
            ea += fabs((double)pos);
        }
        const int sh_4 = stage_shift(warp_max_abs(fmaxf(fabsf(pf[0]), fabsf(pf[1]))), kFold);
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int d = lane + 32 * r;
            const int32_t f = fix_prod(pf[r], 1.0f, sh_4);
            s_fx[2 * (kRabitq + d)] = -f;
            s_fx[2 * (kRabitq + d) + 1] = f;
        }
        ea = warp_sum(ea);
        if (lane == 0) {
            P->err_4 = bound_up(ea);
            P->shift_s4 = sh_4;
            P->unscale_s4 = pow2(-sh_4);
        }
    } else if (warp == 3) {
        // q_tail_sq (src/scan.rs:203-207): the longest sequential sum; only the stored plan's
        // norms use it (no scan score does), so a scan's own table build skips it
        if (lane == 0) {
            float ts = 0.0f;
            if (full) {
#pragma unroll 8
                for (uint32_t d = kTailStart; d < dims; ++d) ts = f_add(ts, f_mul(s_q[d], s_q[d]));
            }
            s_scal[2] = ts;
        }
        if (full) {
            // rabitq_lut (src/scan.rs:188-201): computed by the reference, unused by its stages; it
            // needs the rotated mid band, so this warp rotates it again (cheaper than a barrier)
            float rq[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) rq[r] = s_q[kPrefix + lane + 32 * r];
            fwht_warp<4>(rq, lane);
            // lane holds rotated dims lane + 32 r; group g = dims 4g..4g+3 lives in lanes 4(g%8)..+3
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const int gl = (lane >> 2);  // group within this register's 32 dims
                const float base_v = f_mul(rq[r], kRabitqScale);
                float p[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) p[j] = __shfl_sync(0xffffffffu, base_v, (gl << 2) + j);
                const int g = r * 8 + gl;
                // this lane writes entries m = 4 (lane & 3) .. +3 of group g
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int m = (lane & 3) * 4 + j;
                    const float a0 = (m & 1) ? p[0] : -p[0], a1 = (m & 2) ? p[1] : -p[1];
                    const float a2 = (m & 4) ? p[2] : -p[2], a3 = (m & 8) ? p[3] : -p[3];
                    qp->rabitq_lut[g][m] = f_add(f_add(f_add(a0, a1), a2), a3);
                }
            }
        }
    } else if (warp == 4) {
        // prefix_l1, prefix_sum, eden_mean_ip (src/scan.rs:126-151) in reference order, lanes 0-2
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int d = lane + 32 * r;
            const float qd = s_q[d];
            sh.terms[kRowL1][d] = fabsf(qd);
            sh.terms[kRowSum][d] = qd;
            sh.terms[kRowIp][d] = f_mul(qd, s_mean[d]);
        }
        __syncwarp();
        if (lane < 3) {
            const float acc = lane_chain(sh.terms[kRowL1 + lane], kPrefix);
            if (lane == 0) s_scal[0] = acc;
            else if (lane == 1) s_scal[1] = acc;
            else s_scal[4] = eden ? acc : 0.0f;
        }
        // L0Only shift (accum_plane, src/scan.rs:753-762): entries bit 3 of the level times
        // f32(q_d * 8)
        float e0[2];
        double ea0 = 0.0;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            e0[r] = f_mul(s_q[lane + 32 * r], 8.0f);
            ea0 += fabs((double)e0[r]);
        }
        const int sh_0 = stage_shift(warp_max_abs(fmaxf(fabsf(e0[0]), fabsf(e0[1]))), kPrefix);
        ea0 = warp_sum(ea0);
        if (lane == 0) {
            P->err_0 = bound_up(ea0);
            P->shift_l0 = sh_0;
            P->unscale_l0 = pow2(-sh_0);
            sh.psh[1] = sh_0;
        }
    } else if (warp == 5) {
        // q_mid_sq (src/scan.rs:209-213) and eden_mid_mean_ip (src/scan.rs:167-169), lanes 0-1
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int i = lane + 32 * r;
            const float qd = s_q[kPrefix + i];
            sh.terms[kRowMs][i] = f_mul(qd, qd);
            sh.terms[kRowMip][i] = f_mul(qd, s_mean[kPrefix + i]);
        }
        __syncwarp();
        if (lane < 2) {
            const float acc = lane_chain(sh.terms[kRowMs + lane], kRabitq);
            if (lane == 0) s_scal[3] = acc;
            else s_scal[5] = mid_b1 ? acc : 0.0f;
        }
    } else if (rho_tab) {
        fill_rho_tab(rho_tab, tid - 256, nthr - 256);
    }
    __syncthreads();

    // ---- phase B: tables, one entry per item (prefix entry e = 16 d + l)
    if (need & kNeedFast) {
        const int sp = sh.psh[0];
        for (int t = tid; t < kPrefix * 16; t += nthr) {
            const int d = t >> 4, l = t & 15;
            dst.lut_prefix[t] = eden ? fix_prod(s_cb[l], sh.w[d], sp) : fix_prod((float)l, s_q[d], sp);
        }
        for (int t = tid; t < kS1Windows * 32; t += nthr) dst.lut_s1[t] = window_entry<kRabitq>(s_fx, t >> 5, t & 31);
        for (int t = tid; t < kS4Windows * 32; t += nthr)
            dst.lut_s4[t] = window_entry<kFold>(s_fx + 2 * kRabitq, t >> 5, t & 31);
    }
    if (need & kNeedBatch) {
        for (int t = tid; t < (kRabitq / 4) * 16; t += nthr) P->lut4_s1[t] = window4_entry(s_fx, t >> 4, t & 15);
        for (int t = tid; t < (kFold / 4) * 16; t += nthr)
            P->lut4_s4[t] = window4_entry(s_fx + 2 * kRabitq, t >> 4, t & 15);
    }
    if (need & kNeedL0) {  // bit 3 of the level times bit_weights[d][3] (accum_plane, src/scan.rs:753-762)
        const int s0 = sh.psh[1];
        for (int t = tid; t < kPrefix * 16; t += nthr) {
            const int d = t >> 4, l = t & 15;
            dst.lut_l0[t] = (l & 8) ? fix_prod(f_mul(s_q[d], 8.0f), 1.0f, s0) : 0;
        }
    }
    if (need & kNeedExact) {  // f32 products of the reference's prefix loop (src/scan.rs:456-487)
        for (int t = tid; t < kPrefix * 16; t += nthr) {
            const int d = t >> 4, l = t & 15;
            dst.fp_prefix[t] = eden ? f_mul(s_cb[l], sh.w[d]) : f_mul((float)l, s_q[d]);
        }
    }
    if (tid == 0) {
        qp->dims = dims;
        qp->prefix_codec = prefix_codec;
        qp->mid_codec = mid_codec;
        qp->has_tail_fold = has_tail ? 1u : 0u;
        qp->rabitq_scale = kRabitqScale;
        qp->rabitq_base = s_scal[6];
        qp->tail_fold_base = s_scal[7];
        qp->s4_abs_budget = s_scal[8];
        qp->prefix_l1 = s_scal[0];
        qp->prefix_sum = s_scal[1];
        qp->eden_mean_ip = s_scal[4];
        qp->eden_inv_sqrt_d = kInvSqrt64;
        qp->eden_mid_mean_ip = s_scal[5];
        qp->eden_mid_inv_sqrt_d = kInvSqrt128;
        qp->eden_mid_codebook[0] = mid_b1 ? -kLloydB1Hi : 0.0f;
        qp->eden_mid_codebook[1] = mid_b1 ? kLloydB1Hi : 0.0f;
        if (full) {
            qp->q_tail_norm = __fsqrt_rn(s_scal[2]);
            qp->q_mid_norm = __fsqrt_rn(s_scal[3]);
            qp->q_after_prefix = __fsqrt_rn(f_add(s_scal[3], s_scal[2]));
            qp->q_after_s1 = qp->q_tail_norm;
        }
        P->mid_base = mid_b1 ? s_scal[9] : s_scal[6];
        P->tail_base = s_scal[7];
        P->pad2 = 0.0f;
        P->pad3 = 0.0f;
    }
}

}  // namespace planb
}  // namespace mrl
