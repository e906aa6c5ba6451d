// merge.cu — the exchange step of the sharded scan as a standalone kernel: n exchange records
// (one per rank, gathered into one device buffer by any collective) merged into the global top-k
// by xch::merge_records (exchange.cuh). One CTA per query; no scratch, no atomics on the data
// path.
#include "exchange.cuh"

namespace mrl {
namespace {

constexpr int kMergeThreads = 1024;

__global__ void __launch_bounds__(kMergeThreads)
merge_topk_kernel(const unsigned char* __restrict__ lists, uint32_t n_lists, uint32_t stride, uint32_t k,
                  uint64_t* __restrict__ out_ids, float* __restrict__ out_scores, uint32_t* __restrict__ out_count) {
    xch::merge_records<true>(lists, n_lists, stride, k, out_ids, out_scores, out_count);
}

// One CTA per query: the n_lists records of query q sit n_q records apart (rank-major, as an
// all-gather of every rank's n_q records lays them out).
__global__ void __launch_bounds__(512)
merge_topk_batch_kernel(const unsigned char* __restrict__ lists, uint32_t n_lists, uint32_t n_q, uint32_t stride,
                        uint32_t k, uint64_t* __restrict__ out_ids, float* __restrict__ out_scores,
                        uint32_t* __restrict__ out_counts) {
    const uint32_t q = blockIdx.x;
    const size_t rb = MRL_MERGE_RECORD_BYTES(stride);
    xch::merge_records<true>(lists + (size_t)q * rb, (size_t)n_q * rb, n_lists, stride, k, out_ids + (size_t)q * k,
                             out_scores + (size_t)q * k, out_counts + q);
}

// Record q (stride k) from row q of the batched scan's outputs.
__global__ void __launch_bounds__(256)
pack_records_kernel(const uint64_t* __restrict__ ids, const float* __restrict__ scores,
                    const uint32_t* __restrict__ counts, uint32_t k, unsigned char* __restrict__ records) {
    const uint32_t q = blockIdx.x;
    unsigned char* r = records + (size_t)q * MRL_MERGE_RECORD_BYTES(k);
    for (uint32_t i = threadIdx.x; i < k; i += blockDim.x) {
        reinterpret_cast<uint64_t*>(r)[i] = ids[(size_t)q * k + i];
        reinterpret_cast<float*>(r + (size_t)k * 8)[i] = scores[(size_t)q * k + i];
    }
    if (threadIdx.x == 0) *reinterpret_cast<uint32_t*>(r + (size_t)k * 12) = counts[q];
}

}  // namespace

int launch_pack_records(const uint64_t* d_ids, const float* d_scores, const uint32_t* d_counts, uint32_t n_q,
                        uint32_t k, void* d_records, cudaStream_t stream) {
    if (n_q == 0) return 0;
    pack_records_kernel<<<n_q, 256, 0, stream>>>(d_ids, d_scores, d_counts, k, static_cast<unsigned char*>(d_records));
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int launch_merge_topk_batch(const void* d_lists, uint32_t n_lists, uint32_t n_q, uint32_t stride, uint32_t k,
                            uint64_t* d_out_ids, float* d_out_scores, uint32_t* d_out_counts, cudaStream_t stream) {
    if (n_q == 0) return 0;
    merge_topk_batch_kernel<<<n_q, 512, 0, stream>>>(static_cast<const unsigned char*>(d_lists), n_lists, n_q, stride,
                                                     k, d_out_ids, d_out_scores, d_out_counts);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int launch_merge_topk(const void* d_lists, uint32_t n_lists, uint32_t stride, uint32_t k, uint64_t* d_out_ids,
                      float* d_out_scores, uint32_t* d_out_count, cudaStream_t stream) {
    merge_topk_kernel<<<1, kMergeThreads, 0, stream>>>(static_cast<const unsigned char*>(d_lists), n_lists, stride,
                                                       k, d_out_ids, d_out_scores, d_out_count);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace mrl
