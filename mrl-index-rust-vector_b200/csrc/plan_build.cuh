// plan_build.cuh — the query-side plan build (QueryPlan::from_query_codec, src/scan.rs:105-266) as
// a device function run by a whole CTA (at least 128 threads), shared by the standalone plan kernel
// (plan.cu) and the scan kernel's fused plan prologue (scan.cu).
//
// Four warps build independent parts of the plan (prefix, mid band, folded tail, long reductions),
// then every thread of the CTA fills the tables. FWHTs run on warp shuffles (each
// butterfly output depends only on its two inputs, so the values equal the sequential loop's),
// sequential reductions run on one lane in the reference's order, and every f32 operation is an
// explicit round-to-nearest intrinsic (the library is compiled with -fmad=false) so the plan is
// bit-identical to the reference arithmetic. The build also makes the two scoring-table sets the
// scan uses:
//   * fast mode: per-stage int32 tables whose exact integer sums replace the f32 loops; entries
//     are rint(v * 2^shift) of exact double products, with shift chosen so that every stage sum
//     stays below 2^30 in magnitude;
//   * exact mode: the f32 products / addends of the reference loops.
#pragma once

#include "mrl_internal.cuh"

namespace mrl {
namespace planb {

constexpr int kPlanThreads = 128;

__device__ __forceinline__ float f_add(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float f_sub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float f_mul(float a, float b) { return __fmul_rn(a, b); }

// One fwht_inplace (src/rotate.rs:13-33) over n = 32*R values held by one warp, element
// lane + 32*r in v[r]. Stage h pairs elements j and j+h (bit h of j clear) into (x+y, x-y): for
// h < 32 the partner sits in lane ^ h of the same register, for h >= 32 in register r ^ (h/32) of
// the same lane. Each output is computed from the same two operands as the sequential loop, so
// the values are identical.
template <int R>
__device__ __forceinline__ void fwht_warp(float (&v)[R], int lane) {
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
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)(32 * R)));
#pragma unroll
    for (int r = 0; r < R; ++r) v[r] = f_mul(v[r], scale);
}

__device__ __forceinline__ int stage_shift(double maxabs, int count) {
    if (!(maxabs > 0.0)) return 0;
    int k = 0;
    frexp(maxabs * (double)count, &k);
    return 30 - k;
}
// rint(v * 2^shift): `pow2` = 2^shift exactly, so the product is exact and the conversion rounds
// to nearest-even once.
__device__ __forceinline__ int32_t fix(double v, double pow2) { return __double2int_rn(__dmul_rn(v, pow2)); }

__device__ __forceinline__ double warp_max(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
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
    for (int i = 0; i < w; ++i) sum += fx[2 * (5 * g + i) + ((m >> i) & 1)];
    return sum;
}

// Entry m of the 4-dim window table g of a 1-bit stage (lut4_s1 / lut4_s4): the same exact sum
// over 4 dims instead of 5, so the batched scan's stage sums are the same integers.
__device__ __forceinline__ int32_t window4_entry(const int32_t* fx, int g, int m) {
    int32_t sum = 0;
    for (int i = 0; i < 4; ++i) sum += fx[2 * (4 * g + i) + ((m >> i) & 1)];
    return sum;
}

// What a plan build writes: kNeedAll = every field of DevPlan (the stored plan); a scan that only
// needs its own mode's tables asks for kNeedFast (+ kNeedL0 at depth L0Only) or kNeedExact. The
// scalars, shifts, bit weights, mid_w and tail_w are always written.
constexpr uint32_t kNeedFast = 1u, kNeedExact = 2u, kNeedL0 = 4u, kNeedBatch = 8u, kNeedAll = 0xFu;

// Shared scratch of one plan build (besides the dims-float query copy).
struct PlanShared {
    float mean[kPrefix + kRabitq];
    float rot[kPrefix];
    float rq[kRabitq];
    float mq[kRabitq];
    float tf[kFold];
    int32_t fx[2 * (kRabitq + kFold)];  // fixed 1-bit stage values, see build_window_table
    float scal[16];
    float cb[16];
    float w[kPrefix];  // EDEN prefix weight per dim: rot[d] / sqrt(64)
    double pw[2];      // 2^shift of the prefix and L0 tables
};

// The build's inputs into shared memory: the query, the codec centres, the b=4 codebook. Every
// thread of the CTA calls it; build_plan synchronises before reading them.
__device__ __forceinline__ void plan_inputs(const float* __restrict__ q, uint32_t dims, const float* __restrict__ eden_mean,
                                            const float* __restrict__ mid_mean, float* s_q, PlanShared& sh) {
    const int tid = threadIdx.x, nthr = blockDim.x;
    // the loads are issued before the stores that consume them, so their latencies overlap
    float m = 0.0f, c = 0.0f;
    if (tid < kPrefix + kRabitq) {  // either centre array may be NULL
        const float* src = tid < kPrefix ? eden_mean : mid_mean;
        m = src ? __ldg(src + (tid < kPrefix ? tid : tid - kPrefix)) : 0.0f;
    }
    if (tid < 16) c = g_lloyd_b4[tid];
    for (uint32_t i0 = tid; i0 < dims; i0 += 2u * nthr) {
        const uint32_t i1 = i0 + nthr;
        const float v0 = __ldg(q + i0);
        const float v1 = i1 < dims ? __ldg(q + i1) : 0.0f;
        s_q[i0] = v0;
        if (i1 < dims) s_q[i1] = v1;
    }
    if (tid < kPrefix + kRabitq) sh.mean[tid] = m;
    if (tid < 16) sh.cb[tid] = c;
}

// Phase A, threads 0..127 in four warp roles (the plan branches are independent until the final
// scalars):
//   warp 0: prefix — EDEN query rotation, prefix scalars, prefix weights and the prefix/L0 shifts;
//   warp 1: mid band — RaBitQ and EdenB1 rotations, their scalars, mid_w, the S1 shift and fixed
//           values;
//   warp 2: folded tail — fold, rotation, tail scalars, tail_w, the S4 shift and fixed values;
//   warp 3: q_tail_sq (the longest sequential sum) and, for a full plan, rabitq_lut.
// Phase B, every thread of the CTA: the 1024-entry tables `need` asks for and the window tables.
// Every thread of the CTA (at least 128) must call it, after plan_inputs; P may be global or shared
// memory, s_q holds the dims floats plan_inputs loaded.
__device__ __forceinline__ void build_plan(uint32_t dims, uint32_t prefix_codec, uint32_t mid_codec,
                                           uint64_t eden_seed, uint64_t mid_seed, DevPlan* P, float* s_q,
                                           PlanShared& sh, uint32_t need) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nthr = blockDim.x;
    const bool full = need == kNeedAll;
    mrl_query_plan* qp = &P->qp;
    float* s_mean = sh.mean;
    float* s_rot = sh.rot;
    float* s_rq = sh.rq;
    float* s_mq = sh.mq;
    float* s_tf = sh.tf;
    int32_t* s_fx = sh.fx;
    float* s_scal = sh.scal;
    float* s_cb = sh.cb;
    const bool eden = prefix_codec == MRL_PREFIX_EDEN;
    const bool mid_b1 = mid_codec == MRL_MID_EDEN_B1;
    const bool has_tail = dims > (uint32_t)kTailStart;

    __syncthreads();  // plan_inputs done

    const float inv_sqrt_64 = __fdiv_rn(1.0f, __fsqrt_rn(64.0f));
    const float inv_sqrt_128 = __fdiv_rn(1.0f, __fsqrt_rn(128.0f));
    const float two_over_pi = __fdiv_rn(2.0f, 3.14159265358979323846f);
    const float rabitq_scale = __fdiv_rn(__fsqrt_rn(two_over_pi), __fsqrt_rn(128.0f));  // src/rotate.rs:46-49
    const float tail_scale = __fdiv_rn(__fsqrt_rn(two_over_pi), __fsqrt_rn(64.0f));     // src/rotate.rs:124-126

    if (warp == 0) {
        // ---- prefix copy + bit weights (src/scan.rs:126-140), EDEN rotate_query (src/eden.rs:275-281)
        float v[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int d = lane + 32 * r;
            const float qd = s_q[d];
            if (full) qp->prefix[d] = qd;
            qp->bit_weights[d][0] = f_mul(qd, 1.0f);
            qp->bit_weights[d][1] = f_mul(qd, 2.0f);
            qp->bit_weights[d][2] = f_mul(qd, 4.0f);
            qp->bit_weights[d][3] = f_mul(qd, 8.0f);
            v[r] = f_mul(qd, sign_hash(eden_seed, (uint64_t)d));
        }
        fwht_warp<2>(v, lane);
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            s_rot[lane + 32 * r] = v[r];
            if (full) qp->eden_q_rot[lane + 32 * r] = eden ? v[r] : 0.0f;
        }
        if (full && lane < 16) qp->eden_codebook[lane] = eden ? s_cb[lane] : 0.0f;
        __syncwarp();
        // prefix_l1, prefix_sum, eden_mean_ip: sequential in the reference's order (src/scan.rs:126-151)
        if (lane == 0) {
            float l1 = 0.0f, sum = 0.0f, ip = 0.0f;
#pragma unroll 8
            for (int d = 0; d < kPrefix; ++d) {
                const float qd = s_q[d];
                l1 = f_add(l1, fabsf(qd));
                sum = f_add(sum, qd);
                ip = f_add(ip, f_mul(qd, s_mean[d]));
            }
            if (!eden) ip = 0.0f;
            s_scal[0] = l1;
            s_scal[1] = sum;
            s_scal[4] = ip;
        }
        // Prefix weights and shifts. An entry is (double)cb[l] * w_d (EDEN) or (double)l * q_d
        // (MinMax), both exact products, so the largest |entry| of dim d is max|cb| * |w_d| or
        // 15 * |q_d|.
        double cbmax = 0.0;
#pragma unroll
        for (int l = 0; l < 16; ++l) cbmax = fmax(cbmax, fabs((double)s_cb[l]));
        double mx = 0.0, mx0 = 0.0, ea = 0.0, ea0 = 0.0;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int d = lane + 32 * r;
            const float w = eden ? f_mul(s_rot[d], inv_sqrt_64) : 0.0f;
            sh.w[d] = w;
            const double e = eden ? cbmax * fabs((double)w) : 15.0 * fabs((double)s_q[d]);
            const double e0 = fabs((double)f_mul(s_q[d], 8.0f));
            mx = fmax(mx, e);
            mx0 = fmax(mx0, e0);
            ea += e;
            ea0 += e0;
        }
        const int sh_p = stage_shift(warp_max(mx), kPrefix);
        const int sh_0 = stage_shift(warp_max(mx0), kPrefix);  // L0Only (accum_plane, src/scan.rs:753-762)
        ea = warp_sum(ea);
        ea0 = warp_sum(ea0);
        if (lane == 0) {
            P->err_p = bound_up(ea);
            P->err_0 = bound_up(ea0);
            P->shift_prefix = sh_p;
            P->shift_l0 = sh_0;
            P->unscale_prefix = ldexp(1.0, -sh_p);
            P->unscale_l0 = ldexp(1.0, -sh_0);
            sh.pw[0] = ldexp(1.0, sh_p);
            sh.pw[1] = ldexp(1.0, sh_0);
        }
    } else if (warp == 1) {
        // ---- mid band: rotate_mid_band (src/rotate.rs:36-42) and the EdenB1 rotation (src/scan.rs:159-174)
        float rq[4], mq[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int i = lane + 32 * r;
            rq[r] = s_q[kPrefix + i];
            mq[r] = f_mul(s_q[kPrefix + i], sign_hash(mid_seed, (uint64_t)i));
        }
        fwht_warp<4>(rq, lane);
        if (mid_b1) fwht_warp<4>(mq, lane);
        double mx = 0.0;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int i = lane + 32 * r;
            s_rq[i] = rq[r];
            s_mq[i] = mq[r];
            const float pos = f_mul(rq[r], rabitq_scale);
            if (full) {
                qp->rabitq_q[i] = rq[r];
                qp->eden_mid_q_rot[i] = mid_b1 ? mq[r] : 0.0f;
                qp->rabitq_weights2[i] = f_mul(2.0f, pos);
            }
            double v1;
            if (mid_b1) {
                const float qd = f_mul(mq[r], inv_sqrt_128);
                P->mid_w[i] = f_mul(f_sub(kLloydB1Hi, -kLloydB1Hi), qd);
                v1 = (double)kLloydB1Hi * (double)qd;
            } else {
                P->mid_w[i] = f_mul(2.0f, pos);
                v1 = (double)pos;
            }
            mx = fmax(mx, fabs(v1));
        }
        __syncwarp();
        // q_mid_sq, rabitq_base, eden_mid_mean_ip, EdenB1 base: sequential in reference order
        // (src/scan.rs:209-213, 180-186, 167-169, 523-532)
        if (lane == 0) {
            float ms = 0.0f, base = 0.0f, mip = 0.0f, b1 = 0.0f;
            if (mid_b1) {
#pragma unroll 8
                for (int d = 0; d < kRabitq; ++d) {
                    const float qd = s_q[kPrefix + d];
                    ms = f_add(ms, f_mul(qd, qd));
                    base = f_sub(base, f_mul(s_rq[d], rabitq_scale));
                    mip = f_add(mip, f_mul(qd, s_mean[kPrefix + d]));
                    b1 = f_add(b1, f_mul(-kLloydB1Hi, f_mul(s_mq[d], inv_sqrt_128)));
                }
            } else {
#pragma unroll 8
                for (int d = 0; d < kRabitq; ++d) {
                    const float qd = s_q[kPrefix + d];
                    ms = f_add(ms, f_mul(qd, qd));
                    base = f_sub(base, f_mul(s_rq[d], rabitq_scale));
                }
            }
            s_scal[3] = ms;
            s_scal[5] = mip;
            s_scal[6] = base;
            s_scal[9] = b1;
        }
        // fixed S1 values per dim for the window table
        const int sh_1 = stage_shift(warp_max(mx), kRabitq);
        const double pw_1 = ldexp(1.0, sh_1);
        double ea = 0.0;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int i = lane + 32 * r;
            double v1;
            if (mid_b1) v1 = (double)kLloydB1Hi * (double)f_mul(s_mq[i], inv_sqrt_128);
            else v1 = (double)f_mul(s_rq[i], rabitq_scale);
            s_fx[2 * i] = fix(-v1, pw_1);
            s_fx[2 * i + 1] = fix(v1, pw_1);
            ea += fabs(v1);
        }
        ea = warp_sum(ea);
        if (lane == 0) {
            P->err_1 = bound_up(ea);
            P->shift_s1 = sh_1;
            P->unscale_s1 = ldexp(1.0, -sh_1);
        }
    } else if (warp == 2) {
        // ---- folded tail: fold_tail (src/rotate.rs:73-93) then FWHT64 (rotate_tail_fold)
        float u[2] = {0.0f, 0.0f};
        if (has_tail) {
            const int nb = min((int)((dims - kTailStart) / kPrefix), kFoldBlocks);
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const int d = lane + 32 * r;
                for (int b = 0; b < nb; ++b)
                    u[r] = f_add(u[r], f_mul(sign_hash((uint64_t)b, (uint64_t)d), s_q[kTailStart + b * kPrefix + d]));
            }
        }
        fwht_warp<2>(u, lane);
        double mx = 0.0;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int d = lane + 32 * r;
            s_tf[d] = u[r];
            const float pos = has_tail ? f_mul(u[r], tail_scale) : 0.0f;
            if (full) {
                qp->tail_fold_q[d] = has_tail ? u[r] : 0.0f;
                qp->tail_fold_weights2[d] = has_tail ? f_mul(2.0f, pos) : 0.0f;
            }
            P->tail_w[d] = has_tail ? f_mul(2.0f, pos) : 0.0f;
            mx = fmax(mx, fabs((double)pos));
        }
        __syncwarp();
        // tail_fold_base / s4_abs_budget (src/scan.rs:222-233): sequential in reference order
        if (lane == 0) {
            float tb = 0.0f, bud = 0.0f;
            if (has_tail) {
#pragma unroll 8
                for (int d = 0; d < kFold; ++d) {
                    const float pos = f_mul(s_tf[d], tail_scale);
                    tb = f_sub(tb, pos);
                    bud = f_add(bud, fabsf(pos));
                }
            }
            s_scal[7] = tb;
            s_scal[8] = bud;
        }
        // fixed S4 values per dim for the window table
        const int sh_4 = stage_shift(warp_max(mx), kFold);
        const double pw_4 = ldexp(1.0, sh_4);
        double ea = 0.0;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int d = lane + 32 * r;
            const double pos = has_tail ? (double)f_mul(s_tf[d], tail_scale) : 0.0;
            s_fx[2 * (kRabitq + d)] = fix(-pos, pw_4);
            s_fx[2 * (kRabitq + d) + 1] = fix(pos, pw_4);
            ea += fabs(pos);
        }
        ea = warp_sum(ea);
        if (lane == 0) {
            P->err_4 = bound_up(ea);
            P->shift_s4 = sh_4;
            P->unscale_s4 = ldexp(1.0, -sh_4);
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
                const float base_v = f_mul(rq[r], rabitq_scale);
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
    }
    __syncthreads();

    // ---- phase B: tables, four consecutive levels of one dim per item (entry e = 16 d + l)
    if (need & kNeedFast) {
        const double pw_p = sh.pw[0];
        for (int t = tid; t < kPrefix * 4; t += nthr) {
            const int d = t >> 2, l0 = (t & 3) * 4;
            const float w = sh.w[d];
            int4 o;
            int* oi = &o.x;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int l = l0 + j;
                oi[j] = fix(eden ? (double)s_cb[l] * (double)w : (double)l * (double)s_q[d], pw_p);
            }
            reinterpret_cast<int4*>(P->lut_prefix)[t] = o;
        }
        for (int t = tid; t < kS1Windows * 32; t += nthr) P->lut_s1[t] = window_entry<kRabitq>(s_fx, t >> 5, t & 31);
        for (int t = tid; t < kS4Windows * 32; t += nthr)
            P->lut_s4[t] = window_entry<kFold>(s_fx + 2 * kRabitq, t >> 5, t & 31);
    }
    if (need & kNeedBatch) {
        for (int t = tid; t < (kRabitq / 4) * 16; t += nthr) P->lut4_s1[t] = window4_entry(s_fx, t >> 4, t & 15);
        for (int t = tid; t < (kFold / 4) * 16; t += nthr)
            P->lut4_s4[t] = window4_entry(s_fx + 2 * kRabitq, t >> 4, t & 15);
    }
    if (need & kNeedL0) {  // bit 3 of the level times bit_weights[d][3] (accum_plane, src/scan.rs:753-762)
        const double pw_0 = sh.pw[1];
        for (int t = tid; t < kPrefix * 4; t += nthr) {
            const int d = t >> 2, l0 = (t & 3) * 4;
            const int32_t f = fix((double)f_mul(s_q[d], 8.0f), pw_0);
            int4 o;
            o.x = ((l0 + 0) & 8) ? f : 0;
            o.y = ((l0 + 1) & 8) ? f : 0;
            o.z = ((l0 + 2) & 8) ? f : 0;
            o.w = ((l0 + 3) & 8) ? f : 0;
            reinterpret_cast<int4*>(P->lut_l0)[t] = o;
        }
    }
    if (need & kNeedExact) {  // f32 products of the reference's prefix loop (src/scan.rs:456-487)
        for (int t = tid; t < kPrefix * 4; t += nthr) {
            const int d = t >> 2, l0 = (t & 3) * 4;
            const float w = sh.w[d];
            float4 o;
            float* of = &o.x;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int l = l0 + j;
                of[j] = eden ? f_mul(s_cb[l], w) : f_mul((float)l, s_q[d]);
            }
            reinterpret_cast<float4*>(P->fp_prefix)[t] = o;
        }
    }
    if (tid == 0) {
        qp->dims = dims;
        qp->prefix_codec = prefix_codec;
        qp->mid_codec = mid_codec;
        qp->has_tail_fold = has_tail ? 1u : 0u;
        qp->rabitq_scale = rabitq_scale;
        qp->rabitq_base = s_scal[6];
        qp->tail_fold_base = s_scal[7];
        qp->q_tail_norm = __fsqrt_rn(s_scal[2]);
        qp->q_mid_norm = __fsqrt_rn(s_scal[3]);
        qp->q_after_prefix = __fsqrt_rn(f_add(s_scal[3], s_scal[2]));
        qp->q_after_s1 = qp->q_tail_norm;
        qp->s4_abs_budget = s_scal[8];
        qp->prefix_l1 = s_scal[0];
        qp->prefix_sum = s_scal[1];
        qp->eden_mean_ip = s_scal[4];
        qp->eden_inv_sqrt_d = inv_sqrt_64;
        qp->eden_mid_mean_ip = s_scal[5];
        qp->eden_mid_inv_sqrt_d = inv_sqrt_128;
        qp->eden_mid_codebook[0] = mid_b1 ? -kLloydB1Hi : 0.0f;
        qp->eden_mid_codebook[1] = mid_b1 ? kLloydB1Hi : 0.0f;
        P->mid_base = mid_b1 ? s_scal[9] : s_scal[6];
        P->tail_base = s_scal[7];
        P->pad2 = 0.0f;
        P->pad3 = 0.0f;
    }
}

}  // namespace planb
}  // namespace mrl
