// merge.cu — the exchange step of the sharded scan as a standalone kernel: n exchange records
// (one per rank, gathered into one device buffer by any collective) merged into the global top-k
// by xch::merge_records (exchange.cuh). One CTA; no scratch, no atomics on the data path.
#include "exchange.cuh"

namespace mrl {
namespace {

constexpr int kMergeThreads = 1024;

__global__ void __launch_bounds__(kMergeThreads)
merge_topk_kernel(const unsigned char* __restrict__ lists, uint32_t n_lists, uint32_t stride, uint32_t k,
                  uint64_t* __restrict__ out_ids, float* __restrict__ out_scores, uint32_t* __restrict__ out_count) {
    xch::merge_records<true>(lists, n_lists, stride, k, out_ids, out_scores, out_count);
}

}  // namespace

int launch_merge_topk(const void* d_lists, uint32_t n_lists, uint32_t stride, uint32_t k, uint64_t* d_out_ids,
                      float* d_out_scores, uint32_t* d_out_count, cudaStream_t stream) {
    merge_topk_kernel<<<1, kMergeThreads, 0, stream>>>(static_cast<const unsigned char*>(d_lists), n_lists, stride,
                                                       k, d_out_ids, d_out_scores, d_out_count);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace mrl
