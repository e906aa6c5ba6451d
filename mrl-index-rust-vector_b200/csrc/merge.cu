// merge.cu — the exchange step of the sharded scan on sm_100a: the per-shard top-k lists of all
// ranks, gathered into one device buffer, merged into the global top-k.
//
// Replaces the merge of per-shard shortlists at the end of scan_blocks_stats
// (src/scan.rs:866-870: Shortlist::merge of every partial, then into_sorted) at GPU granularity.
// Order: score descending, then id (VectorId::as_u64) ascending. Shards carry distinct
// block_id_base values, so ids are unique and the order is total; at exactly tied scores the lower
// (block, slot) wins, as in the serial reference scan.
//
// Input: n_lists exchange records of `record_bytes` each (MRL_MERGE_RECORD_BYTES(stride)): stride
// u64 ids, then stride f32 scores, then the u32 count of valid entries, padded to 16 bytes. A
// record is exactly what mrl_scan_device writes when its id / score / count pointers point into it,
// so one all-gather of records is the whole collective.
//
// One CTA: entry x of list i gets rank = (its position in list i) + (the entries of every other
// list that order before it, found by binary search: each list is sorted by the same order), and
// is written to out[rank] when rank < k. No scratch and no atomics on the data path.
#include "mrl_internal.cuh"

namespace mrl {
namespace {

constexpr int kMergeThreads = 1024;

__device__ __forceinline__ bool before(float sa, uint64_t ia, float sb, uint64_t ib) {
    return sa > sb || (sa == sb && ia < ib);
}

struct Record {
    const uint64_t* ids;
    const float* scores;
    uint32_t count;
};

__device__ __forceinline__ Record record(const unsigned char* lists, size_t record_bytes, uint32_t stride, uint32_t i) {
    const unsigned char* r = lists + (size_t)i * record_bytes;
    Record out;
    out.ids = reinterpret_cast<const uint64_t*>(r);
    out.scores = reinterpret_cast<const float*>(r + (size_t)stride * 8);
    out.count = min(__ldg(reinterpret_cast<const uint32_t*>(r + (size_t)stride * 12)), stride);
    return out;
}

__global__ void __launch_bounds__(kMergeThreads)
merge_topk_kernel(const unsigned char* __restrict__ lists, size_t record_bytes, uint32_t n_lists, uint32_t stride,
                  uint32_t k, uint64_t* __restrict__ out_ids, float* __restrict__ out_scores,
                  uint32_t* __restrict__ out_count) {
    const uint32_t total = n_lists * stride;
    for (uint32_t e = threadIdx.x; e < total; e += blockDim.x) {
        const uint32_t i = e / stride, pos = e % stride;
        const Record ri = record(lists, record_bytes, stride, i);
        if (pos >= ri.count || pos >= k) continue;  // a list position >= k can never rank below k
        const float sx = __ldg(ri.scores + pos);
        const uint64_t ix = __ldg(ri.ids + pos);
        uint32_t rank = pos;
        for (uint32_t j = 0; j < n_lists && rank < k; ++j) {
            if (j == i) continue;
            const Record rj = record(lists, record_bytes, stride, j);
            const uint32_t cj = rj.count;
            const float* sj = rj.scores;
            const uint64_t* ij = rj.ids;
            uint32_t lo = 0, hi = min(cj, k);  // only the first k of a list can precede a top-k entry
            while (lo < hi) {
                const uint32_t mid = (lo + hi) >> 1;
                if (before(__ldg(sj + mid), __ldg(ij + mid), sx, ix)) lo = mid + 1; else hi = mid;
            }
            rank += lo;
        }
        if (rank < k) {
            out_ids[rank] = ix;
            out_scores[rank] = sx;
        }
    }
    if (threadIdx.x == 0) {
        uint32_t n = 0;
        for (uint32_t i = 0; i < n_lists; ++i) n += record(lists, record_bytes, stride, i).count;
        *out_count = min(n, k);
    }
}

}  // namespace

int launch_merge_topk(const void* d_lists, uint32_t n_lists, uint32_t stride, uint32_t k, uint64_t* d_out_ids,
                      float* d_out_scores, uint32_t* d_out_count, cudaStream_t stream) {
    merge_topk_kernel<<<1, kMergeThreads, 0, stream>>>(static_cast<const unsigned char*>(d_lists),
                                                       MRL_MERGE_RECORD_BYTES(stride), n_lists, stride, k, d_out_ids,
                                                       d_out_scores, d_out_count);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace mrl
