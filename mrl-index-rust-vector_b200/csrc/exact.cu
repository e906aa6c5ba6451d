// exact.cu — exact f32 inner products on the query path (sm_100a):
//   * the ring buffer's brute-force search over pending (unflushed) vectors,
//     RingBuffer::search_exact (src/ring.rs:109-119), merged into the scan's shortlist by the engine
//     (src/engine.rs:584-594) under the sentinel block id u32::MAX;
//   * the exact rerank of candidate rows, QueryPipeline::rerank_exact_rows (src/pipeline.rs:157-169).
// Both use the reference's `dot` (src/embed.rs:115-152) with its summation order: at 768 dims
// `dot_768` (eight accumulators acc_j += a[i+j]*b[i+j] over i = 0, 8, .., then acc0 + acc1 + .. +
// acc7 left to right), otherwise one sequential sum of products starting from -0.0. Products and sums round to
// nearest (the library is compiled with -fmad=false), so every score is bit-identical to the
// reference. Results are ordered by score descending and, for equal scores, by input position
// (the reference's stable sort).
#include "mrl_internal.cuh"

namespace mrl {
namespace {

constexpr int kDotThreads = 256;     // 8 warps, one row per warp
constexpr int kSortThreads = 1024;
constexpr uint32_t kMaxSort = 4096;

// dot(q, row) of the reference, computed by one warp (the value is valid in lane 0).
__device__ __forceinline__ float ref_dot(const float* __restrict__ q, const float* __restrict__ row, uint32_t dims,
                                         int lane) {
    float r = 0.0f;
    if (dims == 768) {
        float acc = 0.0f;  // lane j < 8 owns acc_j
        if (lane < 8)
            for (uint32_t i = 0; i < 768; i += 8) acc = __fadd_rn(acc, __fmul_rn(row[i + lane], q[i + lane]));
        float a[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) a[j] = __shfl_sync(0xffffffffu, acc, j);
        r = a[0];
#pragma unroll
        for (int j = 1; j < 8; ++j) r = __fadd_rn(r, a[j]);
    } else if (lane == 0) {
        r = -0.0f;  // the neutral element of Rust's f32 Sum
        for (uint32_t i = 0; i < dims; ++i) r = __fadd_rn(r, __fmul_rn(q[i], row[i]));
    }
    return r;
}

// scores[i] = dot(q, rows[sel ? sel[i] : i]); one warp per candidate.
__global__ void __launch_bounds__(kDotThreads)
dots_kernel(const float* __restrict__ q, const float* __restrict__ rows, uint64_t n_rows, uint32_t dims,
            const uint64_t* __restrict__ sel, uint32_t n, float* __restrict__ scores, uint32_t* __restrict__ bad) {
    const int lane = threadIdx.x & 31;
    const uint32_t i = blockIdx.x * (kDotThreads / 32) + (threadIdx.x >> 5);
    if (i >= n) return;
    const uint64_t r = sel ? sel[i] : i;
    if (r >= n_rows) {  // candidate row out of range: reported, scored 0
        if (lane == 0) { atomicExch(bad, 1u); scores[i] = 0.0f; }
        return;
    }
    const float s = ref_dot(q, rows + r * dims, dims, lane);
    if (lane == 0) scores[i] = s;
}

// Sorts (score desc, position asc) and writes the first `keep` entries: ids from `ids_in`
// (position -> id), or `id_base | position` when ids_in is NULL. One CTA, bitonic over <= 4096 keys.
__global__ void __launch_bounds__(kSortThreads)
rank_kernel(const float* __restrict__ scores, uint32_t n, const uint64_t* __restrict__ ids_in, uint64_t id_base,
            uint32_t keep, uint64_t* __restrict__ out_ids, float* __restrict__ out_scores, uint32_t* out_count) {
    __shared__ unsigned long long s_key[kMaxSort];
    uint32_t p2 = 1;
    while (p2 < n) p2 <<= 1;
    for (uint32_t i = threadIdx.x; i < p2; i += blockDim.x)
        s_key[i] = i < n ? make_key(scores[i], i) : 0ull;  // key: score word << 32 | ~position
    __syncthreads();
    for (uint32_t kk = 2; kk <= p2; kk <<= 1) {
        for (uint32_t j = kk >> 1; j > 0; j >>= 1) {
            for (uint32_t i = threadIdx.x; i < p2; i += blockDim.x) {
                const uint32_t ixj = i ^ j;
                if (ixj > i) {
                    const unsigned long long a = s_key[i], b = s_key[ixj];
                    const bool desc = (i & kk) == 0;
                    if (desc ? (a < b) : (a > b)) { s_key[i] = b; s_key[ixj] = a; }
                }
            }
            __syncthreads();
        }
    }
    const uint32_t m = min(keep, n);
    for (uint32_t i = threadIdx.x; i < m; i += blockDim.x) {
        const unsigned long long key = s_key[i];
        const uint32_t pos = key_ordinal(key);
        out_ids[i] = ids_in ? ids_in[pos] : (id_base | pos);
        out_scores[i] = scores[pos];  // the score itself (keeps -0.0)
    }
    if (threadIdx.x == 0 && out_count) *out_count = m;
}

// RingBuffer::search_exact for a batch: CTA q scores query q against the n pending rows (one warp
// per row, the reference's dot), sorts (score desc, position asc) and writes its top k as record q
// (stride k) with the ring sentinel ids VectorId(u32::MAX, position).
constexpr int kRingThreads = 256;
constexpr uint32_t kRingMaxRows = 1024;
__global__ void __launch_bounds__(kRingThreads)
ring_batch_kernel(const float* __restrict__ queries, uint32_t dims, const float* __restrict__ rows, uint32_t n,
                  uint32_t slot_base, uint32_t k, unsigned char* __restrict__ records) {
    __shared__ float s_sc[kRingMaxRows];
    __shared__ unsigned long long s_key[kRingMaxRows];
    const uint32_t q = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const float* qv = queries + (size_t)q * dims;
    for (uint32_t r = warp; r < n; r += kRingThreads / 32) {
        const float sc = ref_dot(qv, rows + (size_t)r * dims, dims, lane);
        if (lane == 0) s_sc[r] = sc;
    }
    __syncthreads();
    uint32_t p2 = 1;
    while (p2 < n) p2 <<= 1;
    for (uint32_t i = threadIdx.x; i < p2; i += kRingThreads) s_key[i] = i < n ? make_key(s_sc[i], i) : 0ull;
    __syncthreads();
    for (uint32_t kk = 2; kk <= p2; kk <<= 1) {
        for (uint32_t j = kk >> 1; j > 0; j >>= 1) {
            for (uint32_t i = threadIdx.x; i < p2; i += kRingThreads) {
                const uint32_t ixj = i ^ j;
                if (ixj > i) {
                    const unsigned long long a = s_key[i], b = s_key[ixj];
                    const bool desc = (i & kk) == 0;
                    if (desc ? (a < b) : (a > b)) { s_key[i] = b; s_key[ixj] = a; }
                }
            }
            __syncthreads();
        }
    }
    unsigned char* rec = records + (size_t)q * MRL_MERGE_RECORD_BYTES(k);
    const uint32_t m = min(k, n);
    for (uint32_t i = threadIdx.x; i < m; i += kRingThreads) {
        const uint32_t pos = key_ordinal(s_key[i]);
        reinterpret_cast<uint64_t*>(rec)[i] = ((uint64_t)0xFFFFFFFFu << 16) | (slot_base + pos);
        reinterpret_cast<float*>(rec + (size_t)k * 8)[i] = s_sc[pos];  // the score itself (keeps -0.0)
    }
    if (threadIdx.x == 0) *reinterpret_cast<uint32_t*>(rec + (size_t)k * 12) = m;
}

}  // namespace

int launch_ring_search_batch(const float* d_queries, uint32_t n_q, uint32_t dims, const float* d_rows, uint32_t n,
                             uint32_t slot_base, uint32_t k, void* d_records, cudaStream_t stream) {
    if (n_q == 0) return 0;
    if (n > kRingMaxRows) return -1;
    ring_batch_kernel<<<n_q, kRingThreads, 0, stream>>>(d_queries, dims, d_rows, n, slot_base, k,
                                                        static_cast<unsigned char*>(d_records));
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int launch_exact_dots(const float* d_query, const float* d_rows, uint64_t n_rows, uint32_t dims, const uint64_t* d_sel,
                      uint32_t n, float* d_scores, uint32_t* d_bad, cudaStream_t stream) {
    if (n == 0) return 0;
    const uint32_t grid = (n + kDotThreads / 32 - 1) / (kDotThreads / 32);
    dots_kernel<<<grid, kDotThreads, 0, stream>>>(d_query, d_rows, n_rows, dims, d_sel, n, d_scores, d_bad);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int launch_exact_rank(const float* d_scores, uint32_t n, const uint64_t* d_ids, uint64_t id_base, uint32_t keep,
                      uint64_t* d_out_ids, float* d_out_scores, uint32_t* d_out_count, cudaStream_t stream) {
    if (n > kMaxSort) return -1;
    rank_kernel<<<1, kSortThreads, 0, stream>>>(d_scores, n, d_ids, id_base, keep, d_out_ids, d_out_scores,
                                                d_out_count);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace mrl
