// plan.cu — the standalone plan kernel (QueryPlan::from_query_codec, src/scan.rs:105-266): one CTA
// of 512 threads per query runs build_plan (plan_build.cuh) into the plan array in global memory.
#include "plan_build.cuh"

namespace mrl {
namespace {

constexpr int kPlanKernelThreads = 512;  // six warps build the plan's branches, all fill its tables

__global__ void __launch_bounds__(kPlanKernelThreads)
plan_kernel(const float* __restrict__ queries, uint32_t dims, uint32_t prefix_codec,
            uint32_t mid_codec, const float* __restrict__ eden_mean, uint64_t eden_seed,
            const float* __restrict__ mid_mean, uint64_t mid_seed, DevPlan* __restrict__ plans) {
    extern __shared__ float s_q[];  // dims floats
    __shared__ planb::PlanShared sh;
    planb::plan_inputs(queries + (size_t)blockIdx.x * dims, dims, eden_mean, mid_mean, eden_seed, mid_seed, s_q, sh);
    planb::build_plan(dims, prefix_codec, mid_codec, plans + blockIdx.x, s_q, sh, planb::kNeedAll,
                      planb::plan_dest(plans + blockIdx.x));
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
    plan_kernel<<<n_q, kPlanKernelThreads, smem, stream>>>(d_queries, dims, prefix_codec, mid_codec, d_eden_mean,
                                                 eden_seed, d_mid_mean, mid_seed, d_plans);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace mrl
