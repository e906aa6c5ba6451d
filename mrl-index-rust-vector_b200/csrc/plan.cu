// plan.cu — query-side plan build on the device (QueryPlan::from_query_codec, src/scan.rs:105-266).
//
// One CTA of 128 threads per query. Butterflies of every FWHT stage run in parallel (each output
// depends only on its two inputs, so the values equal the sequential loop's), sequential
// reductions run on one thread in the reference's order, and every f32 operation is an explicit
// round-to-nearest intrinsic (the file is also compiled with -fmad=false) so the plan is
// bit-identical to the reference arithmetic. The kernel also builds the two scoring-table sets
// the scan uses:
//   * fast mode: per-stage int32 tables whose exact integer sums replace the f32 loops; entries
//     are rint(v * 2^shift) of exact double products, with shift chosen so that every stage sum
//     stays below 2^30 in magnitude;
//   * exact mode: the f32 products / addends of the reference loops.
#include "mrl_internal.cuh"

namespace mrl {
namespace {

constexpr int kThreads = 128;

__device__ __forceinline__ float f_add(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float f_sub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float f_mul(float a, float b) { return __fmul_rn(a, b); }

// fwht_inplace (src/rotate.rs:13-33) over smem, n in {64, 128}; all threads of the CTA call it.
__device__ void fwht_smem(float* a, int n) {
    for (int h = 1; h < n; h *= 2) {
        for (int t = threadIdx.x; t < n / 2; t += blockDim.x) {
            const int blk = t / h, off = t % h;
            const int j = blk * 2 * h + off;
            const float x = a[j], y = a[j + h];
            a[j] = f_add(x, y);
            a[j + h] = f_sub(x, y);
        }
        __syncthreads();
    }
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)n));
    for (int t = threadIdx.x; t < n; t += blockDim.x) a[t] = f_mul(a[t], scale);
    __syncthreads();
}

__device__ int stage_shift(double maxabs, int count) {
    if (!(maxabs > 0.0)) return 0;
    int k = 0;
    frexp(maxabs * (double)count, &k);
    return 30 - k;
}
// rint(v * 2^shift): `pow2` = 2^shift exactly, so the product is exact and the conversion rounds
// to nearest-even once.
__device__ __forceinline__ int32_t fix(double v, double pow2) { return __double2int_rn(__dmul_rn(v, pow2)); }

// Block-wide max of non-negative doubles.
__device__ double block_max(double v, double* red) {
    for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    double m = 0.0;
    for (int w = 0; w < kThreads / 32; ++w) m = fmax(m, red[w]);
    __syncthreads();
    return m;
}


__global__ void __launch_bounds__(kThreads)
plan_kernel(const float* __restrict__ queries, uint32_t dims, uint32_t prefix_codec,
            uint32_t mid_codec, const float* __restrict__ eden_mean, uint64_t eden_seed,
            const float* __restrict__ mid_mean, uint64_t mid_seed, DevPlan* __restrict__ plans) {
    extern __shared__ float s_q[];  // dims floats
    __shared__ float s_rot[kPrefix];
    __shared__ float s_rq[kRabitq];
    __shared__ float s_mq[kRabitq];
    __shared__ float s_tf[kFold];
    __shared__ double s_val1[kRabitq];
    __shared__ double s_val0[kRabitq];
    __shared__ double s_red[kThreads / 32];
    __shared__ float s_scal[16];
    __shared__ float s_cb[16];

    const int tid = threadIdx.x;
    const float* q = queries + (size_t)blockIdx.x * dims;
    DevPlan* P = plans + blockIdx.x;
    mrl_query_plan* qp = &P->qp;

    for (uint32_t i = tid; i < dims; i += kThreads) s_q[i] = q[i];
    if (tid < 16) s_cb[tid] = g_lloyd_b4[tid];
    __syncthreads();

    // ---- prefix copy + bit weights (src/scan.rs:126-140)
    if (tid < kPrefix) {
        const float qd = s_q[tid];
        qp->prefix[tid] = qd;
        qp->bit_weights[tid][0] = f_mul(qd, 1.0f);
        qp->bit_weights[tid][1] = f_mul(qd, 2.0f);
        qp->bit_weights[tid][2] = f_mul(qd, 4.0f);
        qp->bit_weights[tid][3] = f_mul(qd, 8.0f);
    }
    // ---- sequential reductions on dedicated threads (reference order)
    if (tid == 0) {
        float l1 = 0.0f, sum = 0.0f;
        for (int d = 0; d < kPrefix; ++d) { l1 = f_add(l1, fabsf(s_q[d])); sum = f_add(sum, s_q[d]); }
        s_scal[0] = l1;
        s_scal[1] = sum;
    } else if (tid == 32) {
        float ts = 0.0f;  // q_tail_sq, src/scan.rs:203-207
        for (uint32_t d = kTailStart; d < dims; ++d) ts = f_add(ts, f_mul(s_q[d], s_q[d]));
        s_scal[2] = ts;
    } else if (tid == 64) {
        float ms = 0.0f;  // q_mid_sq, src/scan.rs:209-213
        for (int i = 0; i < kRabitq; ++i) ms = f_add(ms, f_mul(s_q[kPrefix + i], s_q[kPrefix + i]));
        s_scal[3] = ms;
    } else if (tid == 96) {
        float ip = 0.0f, mip = 0.0f;  // eden_mean_ip / eden_mid_mean_ip (src/scan.rs:149-151,167-169)
        if (prefix_codec == MRL_PREFIX_EDEN)
            for (int d = 0; d < kPrefix; ++d) ip = f_add(ip, f_mul(s_q[d], eden_mean[d]));
        if (mid_codec == MRL_MID_EDEN_B1)
            for (int d = 0; d < kRabitq; ++d) mip = f_add(mip, f_mul(s_q[kPrefix + d], mid_mean[d]));
        s_scal[4] = ip;
        s_scal[5] = mip;
    }
    // ---- rotations: EDEN prefix (rotate_query, src/eden.rs:275-281), mid band (src/rotate.rs:36-42),
    //      EDEN mid, folded tail (fold_tail, src/rotate.rs:73-93)
    if (tid < kPrefix) s_rot[tid] = f_mul(s_q[tid], sign_hash(eden_seed, (uint64_t)tid));
    if (tid < kRabitq) {
        s_rq[tid] = s_q[kPrefix + tid];
        s_mq[tid] = f_mul(s_q[kPrefix + tid], sign_hash(mid_seed, (uint64_t)tid));
    }
    const bool has_tail = dims > (uint32_t)kTailStart;
    if (tid < kFold) {
        float u = 0.0f;
        if (has_tail) {
            const int nb = min((int)((dims - kTailStart) / kPrefix), kFoldBlocks);
            for (int b = 0; b < nb; ++b)
                u = f_add(u, f_mul(sign_hash((uint64_t)b, (uint64_t)tid), s_q[kTailStart + b * kPrefix + tid]));
        }
        s_tf[tid] = u;
    }
    __syncthreads();
    fwht_smem(s_rot, kPrefix);
    fwht_smem(s_rq, kRabitq);
    fwht_smem(s_mq, kRabitq);
    fwht_smem(s_tf, kFold);

    const float inv_sqrt_64 = __fdiv_rn(1.0f, __fsqrt_rn(64.0f));
    const float inv_sqrt_128 = __fdiv_rn(1.0f, __fsqrt_rn(128.0f));
    const float two_over_pi = __fdiv_rn(2.0f, 3.14159265358979323846f);
    const float rabitq_scale = __fdiv_rn(__fsqrt_rn(two_over_pi), __fsqrt_rn(128.0f));  // src/rotate.rs:46-49
    const float tail_scale = __fdiv_rn(__fsqrt_rn(two_over_pi), __fsqrt_rn(64.0f));     // src/rotate.rs:124-126

    if (tid < kPrefix) {
        qp->eden_q_rot[tid] = prefix_codec == MRL_PREFIX_EDEN ? s_rot[tid] : 0.0f;
        qp->tail_fold_q[tid] = has_tail ? s_tf[tid] : 0.0f;
    }
    if (tid < kRabitq) {
        qp->rabitq_q[tid] = s_rq[tid];
        qp->eden_mid_q_rot[tid] = mid_codec == MRL_MID_EDEN_B1 ? s_mq[tid] : 0.0f;
        qp->rabitq_weights2[tid] = f_mul(2.0f, f_mul(s_rq[tid], rabitq_scale));
    }
    if (tid < kFold) {
        const float pos = has_tail ? f_mul(s_tf[tid], tail_scale) : 0.0f;
        qp->tail_fold_weights2[tid] = has_tail ? f_mul(2.0f, pos) : 0.0f;
    }
    // rabitq_lut (src/scan.rs:188-201): computed by the reference, unused by its stages.
    for (int e = tid; e < 32 * 16; e += kThreads) {
        const int g = e >> 4, m = e & 15;
        const float p0 = f_mul(s_rq[4 * g], rabitq_scale), p1 = f_mul(s_rq[4 * g + 1], rabitq_scale);
        const float p2 = f_mul(s_rq[4 * g + 2], rabitq_scale), p3 = f_mul(s_rq[4 * g + 3], rabitq_scale);
        const float a0 = (m & 1) ? p0 : -p0, a1 = (m & 2) ? p1 : -p1;
        const float a2 = (m & 4) ? p2 : -p2, a3 = (m & 8) ? p3 : -p3;
        qp->rabitq_lut[g][m] = f_add(f_add(f_add(a0, a1), a2), a3);
    }
    if (tid == 0) {  // rabitq_base (src/scan.rs:180-186)
        float base = 0.0f;
        for (int d = 0; d < kRabitq; ++d) base = f_sub(base, f_mul(s_rq[d], rabitq_scale));
        s_scal[6] = base;
    } else if (tid == 32) {  // tail_fold_base / s4_abs_budget (src/scan.rs:222-233)
        float tb = 0.0f, bud = 0.0f;
        if (has_tail) {
            for (int d = 0; d < kFold; ++d) {
                const float pos = f_mul(s_tf[d], tail_scale);
                tb = f_sub(tb, pos);
                bud = f_add(bud, fabsf(pos));
            }
        }
        s_scal[7] = tb;
        s_scal[8] = bud;
    } else if (tid == 64) {  // EdenB1 all-zero-bits baseline (src/scan.rs:523-532)
        float base = 0.0f;
        if (mid_codec == MRL_MID_EDEN_B1) {
            for (int d = 0; d < kRabitq; ++d) base = f_add(base, f_mul(-kLloydB1Hi, f_mul(s_mq[d], inv_sqrt_128)));
        }
        s_scal[9] = base;
    }
    __syncthreads();
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
        qp->eden_mid_codebook[0] = mid_codec == MRL_MID_EDEN_B1 ? -kLloydB1Hi : 0.0f;
        qp->eden_mid_codebook[1] = mid_codec == MRL_MID_EDEN_B1 ? kLloydB1Hi : 0.0f;
        P->mid_base = mid_codec == MRL_MID_EDEN_B1 ? s_scal[9] : s_scal[6];
        P->tail_base = s_scal[7];
    }
    if (tid < 16) qp->eden_codebook[tid] = prefix_codec == MRL_PREFIX_EDEN ? s_cb[tid] : 0.0f;

    // ---- exact-mode tables
    for (int e = tid; e < kPrefix * 16; e += kThreads) {
        const int d = e >> 4, l = e & 15;
        float v;
        if (prefix_codec == MRL_PREFIX_EDEN) v = f_mul(s_cb[l], f_mul(s_rot[d], inv_sqrt_64));
        else v = f_mul((float)l, s_q[d]);
        P->fp_prefix[e] = v;
    }
    if (tid < kRabitq) {
        if (mid_codec == MRL_MID_EDEN_B1) {
            const float qd = f_mul(s_mq[tid], inv_sqrt_128);
            P->mid_w[tid] = f_mul(f_sub(kLloydB1Hi, -kLloydB1Hi), qd);
        } else {
            P->mid_w[tid] = f_mul(2.0f, f_mul(s_rq[tid], rabitq_scale));
        }
    }
    if (tid < kFold) P->tail_w[tid] = has_tail ? f_mul(2.0f, f_mul(s_tf[tid], tail_scale)) : 0.0f;

    // ---- fast-mode tables
    // prefix: value of dim d at level l (EDEN: codebook * weight, MinMax: level * q_d)
    double mx = 0.0;
    for (int e = tid; e < kPrefix * 16; e += kThreads) {
        const int d = e >> 4, l = e & 15;
        double v;
        if (prefix_codec == MRL_PREFIX_EDEN) v = (double)s_cb[l] * (double)f_mul(s_rot[d], inv_sqrt_64);
        else v = (double)l * (double)s_q[d];
        mx = fmax(mx, fabs(v));
    }
    const int sh_p = stage_shift(block_max(mx, s_red), kPrefix);
    const double pw_p = ldexp(1.0, sh_p);
    for (int e = tid; e < kPrefix * 16; e += kThreads) {
        const int d = e >> 4, l = e & 15;
        double v;
        if (prefix_codec == MRL_PREFIX_EDEN) v = (double)s_cb[l] * (double)f_mul(s_rot[d], inv_sqrt_64);
        else v = (double)l * (double)s_q[d];
        P->lut_prefix[e] = fix(v, pw_p);
    }
    // L0Only: bit 3 of the level times bit_weights[d][3] (accum_plane, src/scan.rs:753-762)
    mx = 0.0;
    if (tid < kPrefix) mx = fabs((double)f_mul(s_q[tid], 8.0f));
    const int sh_0 = stage_shift(block_max(mx, s_red), kPrefix);
    const double pw_0 = ldexp(1.0, sh_0);
    for (int e = tid; e < kPrefix * 16; e += kThreads) {
        const int d = e >> 4, l = e & 15;
        P->lut_l0[e] = (l & 8) ? fix((double)f_mul(s_q[d], 8.0f), pw_0) : 0;
    }
    // mid band: value of dim d for bit 1 / bit 0
    if (tid < kRabitq) {
        if (mid_codec == MRL_MID_EDEN_B1) {
            const double qd = (double)f_mul(s_mq[tid], inv_sqrt_128);
            s_val1[tid] = (double)kLloydB1Hi * qd;
            s_val0[tid] = -(double)kLloydB1Hi * qd;
        } else {
            const double pos = (double)f_mul(s_rq[tid], rabitq_scale);
            s_val1[tid] = pos;
            s_val0[tid] = -pos;
        }
    }
    __syncthreads();
    mx = 0.0;
    if (tid < kRabitq) mx = fmax(fabs(s_val1[tid]), fabs(s_val0[tid]));
    const int sh_1 = stage_shift(block_max(mx, s_red), kRabitq);
    const double pw_1 = ldexp(1.0, sh_1);
    for (int e = tid; e < kS1Windows * 32; e += kThreads) {
        const int g = e >> 5, m = e & 31;
        const int w = min(5, kRabitq - 5 * g);
        int32_t s = 0;
        if (m < (1 << w))
            for (int i = 0; i < w; ++i) s += fix(((m >> i) & 1) ? s_val1[5 * g + i] : s_val0[5 * g + i], pw_1);
        P->lut_s1[e] = s;
    }
    __syncthreads();
    // folded tail
    if (tid < kFold) {
        const double pos = has_tail ? (double)f_mul(s_tf[tid], tail_scale) : 0.0;
        s_val1[tid] = pos;
        s_val0[tid] = -pos;
    }
    __syncthreads();
    mx = 0.0;
    if (tid < kFold) mx = fabs(s_val1[tid]);
    const int sh_4 = stage_shift(block_max(mx, s_red), kFold);
    const double pw_4 = ldexp(1.0, sh_4);
    for (int e = tid; e < kS4Windows * 32; e += kThreads) {
        const int g = e >> 5, m = e & 31;
        const int w = min(5, kFold - 5 * g);
        int32_t s = 0;
        if (m < (1 << w))
            for (int i = 0; i < w; ++i) s += fix(((m >> i) & 1) ? s_val1[5 * g + i] : s_val0[5 * g + i], pw_4);
        P->lut_s4[e] = s;
    }
    if (tid == 0) {
        P->shift_prefix = sh_p;
        P->shift_s1 = sh_1;
        P->shift_s4 = sh_4;
        P->shift_l0 = sh_0;
        P->unscale_prefix = ldexp(1.0, -sh_p);
        P->unscale_s1 = ldexp(1.0, -sh_1);
        P->unscale_s4 = ldexp(1.0, -sh_4);
        P->unscale_l0 = ldexp(1.0, -sh_0);
        P->pad2 = 0.0f;
        P->pad3 = 0.0f;
    }
}

}  // namespace

int launch_plan_build(const float* d_queries, uint32_t n_q, uint32_t dims, uint32_t prefix_codec,
                      uint32_t mid_codec, const float* d_eden_mean, uint64_t eden_seed,
                      const float* d_mid_mean, uint64_t mid_seed, DevPlan* d_plans,
                      cudaStream_t stream) {
    if (n_q == 0) return 0;
    const size_t smem = (size_t)dims * sizeof(float);
    if (smem > 48 * 1024) {
        if (cudaFuncSetAttribute(plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem) != cudaSuccess)
            return -1;
    }
    plan_kernel<<<n_q, kThreads, smem, stream>>>(d_queries, dims, prefix_codec, mid_codec, d_eden_mean,
                                                 eden_seed, d_mid_mean, mid_seed, d_plans);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace mrl
