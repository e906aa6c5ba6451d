// exchange.cuh — the merge of per-rank top-k records, shared by the standalone merge kernel
// (merge.cu) and the scan kernel's NVLink exchange tail (scan.cu).
//
// A record holds one rank's top list: `stride` u64 ids, then `stride` f32 scores, then the u32
// count of valid entries, padded to MRL_MERGE_RECORD_BYTES(stride) bytes. The merge replaces the
// merge of per-shard shortlists at the end of scan_blocks_stats (src/scan.rs:866-870) at GPU
// granularity. Order: score descending, then id (VectorId::as_u64) ascending; shards carry
// distinct block_id_base values, so ids are unique and the order is total.
#pragma once

#include "mrl_internal.cuh"

namespace mrl {
namespace xch {

__device__ __forceinline__ bool before(float sa, uint64_t ia, float sb, uint64_t ib) {
    return sa > sb || (sa == sb && ia < ib);
}

struct Record {
    const uint64_t* ids;
    const float* scores;
    uint32_t count;
};

// Loads of record data: through L2 only for records in global memory (they may have been written
// by another GPU since this SM last read them), plain loads for copies in shared memory.
template <bool kGlobal, class T>
__device__ __forceinline__ T rd(const T* p) {
    if (kGlobal) return __ldcg(p);
    return *p;
}

template <bool kGlobal>
__device__ __forceinline__ Record record(const unsigned char* lists, size_t record_bytes, uint32_t stride, uint32_t i) {
    const unsigned char* r = lists + (size_t)i * record_bytes;
    Record out;
    out.ids = reinterpret_cast<const uint64_t*>(r);
    out.scores = reinterpret_cast<const float*>(r + (size_t)stride * 8);
    out.count = min(rd<kGlobal>(reinterpret_cast<const uint32_t*>(r + (size_t)stride * 12)), stride);
    return out;
}

// Every thread of the CTA calls it; kGlobal: the records are in global memory (else shared). Entry
// x of record i gets rank = (its position in record i) +
// (the entries of every other record that order before it, by binary search: each record is
// sorted by the same order) and is written to out[rank] when rank < k.
// `list_bytes`: distance between consecutive records (MRL_MERGE_RECORD_BYTES(stride) when they are
// contiguous).
template <bool kGlobal>
__device__ __forceinline__ void merge_records(const unsigned char* lists, size_t list_bytes, uint32_t n_lists,
                                              uint32_t stride, uint32_t k, uint64_t* out_ids, float* out_scores,
                                              uint32_t* out_count) {
    const size_t rb = list_bytes;
    const uint32_t total = n_lists * stride;
    for (uint32_t e = threadIdx.x; e < total; e += blockDim.x) {
        const uint32_t i = e / stride, pos = e % stride;
        const Record ri = record<kGlobal>(lists, rb, stride, i);
        if (pos >= ri.count || pos >= k) continue;  // a list position >= k can never rank below k
        const float sx = rd<kGlobal>(ri.scores + pos);
        const uint64_t ix = rd<kGlobal>(ri.ids + pos);
        uint32_t rank = pos;
        for (uint32_t j = 0; j < n_lists && rank < k; ++j) {
            if (j == i) continue;
            const Record rj = record<kGlobal>(lists, rb, stride, j);
            uint32_t lo = 0, hi = min(rj.count, k);  // only the first k of a list can precede a top-k entry
            while (lo < hi) {
                const uint32_t mid = (lo + hi) >> 1;
                if (before(rd<kGlobal>(rj.scores + mid), rd<kGlobal>(rj.ids + mid), sx, ix)) lo = mid + 1; else hi = mid;
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
        for (uint32_t i = 0; i < n_lists; ++i) n += record<kGlobal>(lists, rb, stride, i).count;
        *out_count = min(n, k);
    }
}

template <bool kGlobal>
__device__ __forceinline__ void merge_records(const unsigned char* lists, uint32_t n_lists, uint32_t stride,
                                              uint32_t k, uint64_t* out_ids, float* out_scores,
                                              uint32_t* out_count) {
    merge_records<kGlobal>(lists, MRL_MERGE_RECORD_BYTES(stride), n_lists, stride, k, out_ids, out_scores, out_count);
}

// Number of the first n entries of a sorted record part (ids, scores) that order before (sx, ix).
__device__ __forceinline__ uint32_t count_before(const uint64_t* ids, const float* scores, uint32_t n, float sx,
                                                 uint64_t ix) {
    uint32_t lo = 0, hi = n;
    while (lo < hi) {
        const uint32_t mid = (lo + hi) >> 1;
        if (before(scores[mid], ids[mid], sx, ix)) lo = mid + 1; else hi = mid;
    }
    return lo;
}

// The same merge for records in shared memory (the scan kernel's NVLink exchange tail), as a tree
// of pairwise merges: at each level every entry of a pair's two sorted records is placed by one
// binary search in the partner record, the merged top-k becomes a record of the next level, and
// the last level writes the outputs. Levels alternate between `recs` (n_lists records) and `tmp`
// (room for ceil(n_lists / 2) records). Every thread of the CTA calls it.
__device__ __forceinline__ void merge_records_tree(unsigned char* recs, unsigned char* tmp, uint32_t n_lists,
                                                   uint32_t stride, uint32_t k, uint64_t* out_ids,
                                                   float* out_scores, uint32_t* out_count) {
    const size_t rb = MRL_MERGE_RECORD_BYTES(stride);
    k = min(k, stride);
    unsigned char* src = recs;
    unsigned char* dst = tmp;
    uint32_t n = n_lists;
    for (;;) {
        const bool last = n <= 2;
        const uint32_t m = (n + 1) >> 1;
        const uint32_t total = 2 * m * k;  // entry e: pair e / (2k), side (e / k) & 1, index e % k
        for (uint32_t e = threadIdx.x; e < total; e += blockDim.x) {
            const uint32_t pr = e / (2 * k), side = (e / k) & 1u, idx = e % k;
            const uint32_t li = 2 * pr + side, qi = 2 * pr + (side ^ 1u);
            if (li >= n) continue;
            const Record L = record<false>(src, rb, stride, li);
            if (idx >= L.count) continue;
            const float sx = L.scores[idx];
            const uint64_t ix = L.ids[idx];
            uint32_t r = idx;
            if (qi < n) {
                const Record Q = record<false>(src, rb, stride, qi);
                r += count_before(Q.ids, Q.scores, min(Q.count, k), sx, ix);
            }
            if (r < k) {
                if (last) {
                    out_ids[r] = ix;
                    out_scores[r] = sx;
                } else {
                    unsigned char* d = dst + (size_t)pr * rb;
                    reinterpret_cast<uint64_t*>(d)[r] = ix;
                    reinterpret_cast<float*>(d + (size_t)stride * 8)[r] = sx;
                }
            }
        }
        if (threadIdx.x < m) {  // merged counts
            const uint32_t a = record<false>(src, rb, stride, 2 * threadIdx.x).count;
            const uint32_t b = 2 * threadIdx.x + 1 < n ? record<false>(src, rb, stride, 2 * threadIdx.x + 1).count : 0u;
            const uint32_t c = min(min(a, k) + min(b, k), k);
            if (last) *out_count = c;
            else *reinterpret_cast<uint32_t*>(dst + (size_t)threadIdx.x * rb + (size_t)stride * 12) = c;
        }
        __syncthreads();
        if (last) return;
        unsigned char* t = src;
        src = dst;
        dst = t;
        n = m;
    }
}

}  // namespace xch
}  // namespace mrl
