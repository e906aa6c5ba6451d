// bscan.cu — batched fast-mode scan for sm_100a: a tile of query plans scored against every page
// a CTA loads.
//
// The same scan as scan.cu's MRL_MODE_FAST (scan_blocks, src/scan.rs:802-886, for many plans),
// restructured for throughput when many queries share one pass over the segment:
//
//   * Work split: one CTA per SM, each owning a contiguous range of pages (sizes differ by <= 1).
//     A CTA walks its range once per tile of kTile queries; the pages come from L2 after the first
//     tile (a 1M-vector segment is 64 MB, L2 is 126 MB).
//   * Scoring: one thread per slot (two slots per lane and page). All three stages are sums of
//     16-entry tables indexed by nibbles of the slot's 64 bytes: the 4-bit prefix levels (64
//     dims), and the mid-band and folded-tail bits in 4-dim windows (32 + 16 windows, the plan's
//     lut4_s1 / lut4_s4). The tables of two queries are interleaved (int2 per entry), so one
//     64-bit shared load returns both queries' entries and a dim's table is exactly one 128-byte
//     row of banks: no bank conflict for any index pattern. The stage sums are the same integers as
//     the single-query kernel's (integer sums regrouped), and the f32 score formulas are the same
//     functions, so every score is bit-identical to mrl_scan_device's fast mode.
//   * Selection: per (warp, query) a sorted top-32 in registers, filtered against max(own 32nd
//     key, the CTA's bound for that query), candidates queued in shared memory and merged 32 at a
//     time (as in scan.cu). At the end of a tile the 16 warp lists of every query are tree-merged
//     (all queries at once) into the CTA's exact top-32, written to global scratch.
//   * bselect_kernel (one CTA per query): radix select of the k-th key over the G lists, then a
//     bitonic sort of the top k. The union of CTA lists holds the exact top-k unless a CTA's full
//     list ends inside it; such a query is reported (status bit 3) and the host entry reruns it
//     through the single-query kernel, so host-facing results are exact for every input.
#include "scan_common.cuh"
#include "umma.cuh"

namespace mrl {
namespace {

constexpr int kBWarps = 16;
constexpr int kBThreads = kBWarps * 32;
constexpr int kTile = 8;           // queries per tile (even)
constexpr int kPairs = kTile / 2;
constexpr int kBQueue = 64;        // queued candidates per (warp, query): one offer adds <= 64
constexpr int kNibPrefix = kPrefix;          // 64 nibble tables
constexpr int kNibS1 = kRabitq / 4;          // 32
constexpr int kNibS4 = kFold / 4;            // 16
constexpr int kNibTabs = kNibPrefix + kNibS1 + kNibS4;  // 112 tables of 16 entries per query
constexpr int kSelThreads = 1024;
constexpr int kSelBins = 2048;
constexpr uint32_t kStatusUncertified = 8u;

// Per (warp, query) selection state, all in shared memory: the sorted top-32 (wlist), the
// warp's bound (high word of its 32nd key, 0 until full) and the queue fill.
struct BWarpState {
    uint32_t tau;
    int qn;
};

struct BShared {
    int2 tab[kPairs][kNibTabs * 16];   // 57,344 B: entry (t, l) of queries (2i, 2i+1)
    Scalars S[kTile];
    float2 rho[256];
    u64 tau[kTile];                    // CTA bound per query (high word used)
    BWarpState wst[kBWarps][kTile];
    u64 queue[kBWarps][kTile][kBQueue];  // 64 KB
    u64 wlist[kTile][kBWarps][32];       // 32 KB: each warp's top-32 per query, then the merge
};

__device__ __forceinline__ int2 lds64(const int2* tab, uint32_t byte_off) {
    return *reinterpret_cast<const int2*>(reinterpret_cast<const char*>(tab) + byte_off);
}

// Sums, for two queries, of the nibble tables t0 .. t0 + 8*NW - 1 indexed by the nibbles of
// `w` (nibble n of word j feeds table t0 + 8 j + n).
template <int NW>
__device__ __forceinline__ void nib_sum2(const uint32_t* w, const int2* tab, int32_t one, int32_t& a, int32_t& b) {
    int32_t a0 = 0, a1 = 0, b0 = 0, b1 = 0;
#pragma unroll
    for (int j = 0; j < NW; ++j) {
        const uint32_t e = (w[j] << 3) & 0x78787878u;  // low nibbles x 8: tables 8j, 8j+2, 8j+4, 8j+6
        const uint32_t o = (w[j] >> 1) & 0x78787878u;  // high nibbles x 8: tables 8j+1, +3, +5, +7
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int2 x = lds64(tab, (8 * j + 2 * k) * 128 + __byte_perm(e, 0, 0x4440 + k));
            const int2 y = lds64(tab, (8 * j + 2 * k + 1) * 128 + __byte_perm(o, 0, 0x4440 + k));
            a0 = x.x * one + a0;  // one == 1: the accumulations issue on the FMA pipe, the
            b0 = x.y * one + b0;  // nibble extraction on the ALU pipe
            a1 = y.x * one + a1;
            b1 = y.y * one + b1;
        }
    }
    a = a0 + a1;
    b = b0 + b1;
}

__device__ __forceinline__ void bsel_flush(u64* wl, u64* q, int lane, u64* cta_tau, BWarpState* st) {
    __syncwarp();
    const int qn = st->qn;
    u64 list = wl[lane];
    for (int base = 0; base < qn; base += 32) {
        u64 x = (base + lane < qn) ? q[base + lane] : 0ull;
        x = warp_sort32(x, lane);
        list = warp_merge32(list, x, lane);
    }
    const u64 t = __shfl_sync(kFull, list, 31);
    wl[lane] = list;
    __syncwarp();
    if (lane == 0) {
        st->qn = 0;
        st->tau = (uint32_t)(t >> 32);
        if (t) atomicMax(cta_tau, t);
    }
    __syncwarp();
}

__device__ __forceinline__ void bsel_offer(u64* wl, u64* q, int lane, u64* cta_tau, BWarpState* st, u64 k0,
                                           u64 k1) {
    const uint32_t tc = (uint32_t)(*reinterpret_cast<volatile u64*>(cta_tau) >> 32);
    const uint32_t tau = max(max(st->tau, tc), 1u);
    const bool p0 = (uint32_t)(k0 >> 32) >= tau, p1 = (uint32_t)(k1 >> 32) >= tau;
    const unsigned m0 = __ballot_sync(kFull, p0), m1 = __ballot_sync(kFull, p1);
    if ((m0 | m1) == 0u) return;
    const int nn = __popc(m0) + __popc(m1);
    if (st->qn + nn > kBQueue) bsel_flush(wl, q, lane, cta_tau, st);
    const int qn = st->qn;
    const unsigned lt = (1u << lane) - 1u;
    if (p0) q[qn + __popc(m0 & lt)] = k0;
    if (p1) q[qn + __popc(m0) + __popc(m1 & lt)] = k1;
    __syncwarp();
    if (lane == 0) st->qn = qn + nn;
    __syncwarp();
    if (qn + nn >= 32) bsel_flush(wl, q, lane, cta_tau, st);
}

// Integer stage sums of one slot for the query pair whose interleaved tables start at `tab`
// (index h = query 2i + h).
__device__ __forceinline__ void pair_sums(const Slot4& s, const int2* tab, uint32_t depth, int32_t one,
                                          int32_t (&P)[2], int32_t (&S1)[2], int32_t (&S4)[2]) {
    uint32_t pw[8] = {s.c0.x, s.c0.y, s.c0.z, s.c0.w, s.c1.x, s.c1.y, s.c1.z, s.c1.w};
    uint32_t s1w[4] = {s.c2.x, s.c2.y, s.c2.z, s.c2.w};
    uint32_t s4w[2] = {s.c3.x, s.c3.y};
    // The words are the same for every query pair of a page; opaque copies keep the compiler from
    // hoisting all 112 table offsets out of the pair loop (which would spill).
#pragma unroll
    for (int i = 0; i < 8; ++i) asm volatile("" : "+r"(pw[i]));
#pragma unroll
    for (int i = 0; i < 4; ++i) asm volatile("" : "+r"(s1w[i]));
    asm volatile("" : "+r"(s4w[0]), "+r"(s4w[1]));
    S1[0] = S1[1] = S4[0] = S4[1] = 0;
    nib_sum2<8>(pw, tab, one, P[0], P[1]);
    if (depth >= MRL_DEPTH_L1) nib_sum2<4>(s1w, tab + kNibPrefix * 16, one, S1[0], S1[1]);
    if (depth == MRL_DEPTH_FULL) nib_sum2<2>(s4w, tab + (kNibPrefix + kNibS1) * 16, one, S4[0], S4[1]);
}

struct BatchLaunch {
    const uint4* pages;
    const uint2* block_ts;
    uint32_t n_blocks;
    const DevPlan* plans;  // n_q plans
    uint32_t n_q;
    float w_s4;
    uint32_t depth;
    uint32_t use_time, has_lo, lo, has_hi, hi;
    u64* lists;            // [n_q][G][32] keys: each CTA's exact top-32 per query
};

__device__ __forceinline__ bool page_live(const BatchLaunch& p, uint32_t b) {
    if (!p.use_time) return true;
    const uint2 t = __ldg(p.block_ts + b);  // [min_ts, max_ts], src/scan.rs:719-730
    if (p.has_lo && t.y < p.lo) return false;
    if (p.has_hi && t.x > p.hi) return false;
    return true;
}

__global__ void __launch_bounds__(kBThreads, 1) bscan_kernel(const BatchLaunch p) {
    extern __shared__ __align__(16) unsigned char b_dyn[];
    BShared& sh = *reinterpret_cast<BShared*>(b_dyn);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t G = gridDim.x;
    const uint32_t lo_b = (uint32_t)(((uint64_t)p.n_blocks * blockIdx.x) / G);
    const uint32_t hi_b = (uint32_t)(((uint64_t)p.n_blocks * (blockIdx.x + 1)) / G);
    fill_rho_tab(sh.rho, tid, kBThreads);
    const int32_t one = (int32_t)(p.n_q != 0u);  // 1 at run time, opaque to the compiler

    for (uint32_t q0 = 0; q0 < p.n_q; q0 += kTile) {
        const uint32_t nq = min((uint32_t)kTile, p.n_q - q0);
        __syncthreads();  // the previous tile's lists are written out
        // tables of this tile: entry (t, l) of query 2i in .x, of query 2i+1 in .y (a missing
        // query of an odd last tile reads as zeros and is never offered)
#pragma unroll 4
        for (int i = tid; i < kPairs * kNibTabs * 16; i += kBThreads) {
            const int pr = i / (kNibTabs * 16), e = i % (kNibTabs * 16);
            int2 v = make_int2(0, 0);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t qi = 2 * pr + h;
                if (qi >= nq) continue;
                const DevPlan* P = p.plans + q0 + qi;
                int32_t x;
                if (e < kNibPrefix * 16) x = P->lut_prefix[e];
                else if (e < (kNibPrefix + kNibS1) * 16) x = P->lut4_s1[e - kNibPrefix * 16];
                else x = P->lut4_s4[e - (kNibPrefix + kNibS1) * 16];
                if (h) v.y = x; else v.x = x;
            }
            sh.tab[pr][e] = v;
        }
        if (tid < kTile) {
            if ((uint32_t)tid < nq) fill_scalars(p.plans + q0 + tid, p.w_s4, p.depth, one, sh.S[tid]);
            sh.tau[tid] = 0ull;
        }
        if (tid < kBWarps * kTile) sh.wst[tid / kTile][tid % kTile] = BWarpState{0u, 0};
        for (int i = tid; i < kTile * kBWarps * 32; i += kBThreads) (&sh.wlist[0][0][0])[i] = 0ull;
        __syncthreads();

        for (uint32_t b = lo_b + warp; b < hi_b; b += kBWarps) {
            if (!page_live(p, b)) continue;  // warp-uniform
            Slot4 s0, s1;
            load_slot(p.pages, b, lane, s0);
            load_slot(p.pages, b, lane + 32, s1);
            const SlotMeta m0 = slot_meta_tab(s0.c3.z, s0.c3.w, sh.rho);
            const SlotMeta m1 = slot_meta_tab(s1.c3.z, s1.c3.w, sh.rho);
            const uint32_t o0 = b * 64 + lane, o1 = o0 + 32;
#pragma unroll 1
            for (int pr = 0; pr < kPairs; ++pr) {
                if ((uint32_t)(2 * pr) >= nq) break;  // warp-uniform
                int32_t P0[2], A0[2], B0[2], P1[2], A1[2], B1[2];
                pair_sums(s0, sh.tab[pr], p.depth, one, P0, A0, B0);
                pair_sums(s1, sh.tab[pr], p.depth, one, P1, A1, B1);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int q = 2 * pr + h;
                    if ((uint32_t)q < nq) {  // warp-uniform
                        const Scalars& S = sh.S[q];
                        const u64 k0 = m0.tomb ? 0ull : make_key(fast_score(m0, P0[h], A0[h], B0[h], S), o0);
                        const u64 k1 = m1.tomb ? 0ull : make_key(fast_score(m1, P1[h], A1[h], B1[h], S), o1);
                        bsel_offer(sh.wlist[q][warp], sh.queue[warp][q], lane, &sh.tau[q], &sh.wst[warp][q], k0, k1);
                    }
                }
            }
        }
        for (int q = 0; q < kTile; ++q)
            if (sh.wst[warp][q].qn) bsel_flush(sh.wlist[q][warp], sh.queue[warp][q], lane, &sh.tau[q], &sh.wst[warp][q]);
        __syncthreads();
        u64* lists = &sh.wlist[0][0][0];  // [kTile][kBWarps][32]
        for (int half = kBWarps / 2; half >= 1; half >>= 1) {
            for (int m = warp; m < kTile * half; m += kBWarps) {
                const int q = m / half, i = m % half;
                u64* a = lists + (q * kBWarps + i) * 32;
                const u64 r = warp_merge32(a[lane], lists[(q * kBWarps + i + half) * 32 + lane], lane);
                __syncwarp();
                a[lane] = r;
            }
            __syncthreads();
        }
        for (int i = tid; i < (int)nq * 32; i += kBThreads) {
            const int q = i >> 5;
            p.lists[((size_t)(q0 + q) * G + blockIdx.x) * 32 + (i & 31)] = lists[(q * kBWarps) * 32 + (i & 31)];
        }
    }
}

// ---- per-query selection over the CTA lists ----

struct SelectLaunch {
    const u64* lists;  // [n_q][G][32]
    const uint32_t* err;  // scan error word (bit 1: a bounded wait ran out), ORed into every status
    uint32_t G, n_q, k, block_id_base;
    // exact finishing: the pages (candidates are rescored in the reference's f32 order), the plans,
    // the segment's meta maxima (fast/exact score bound), and the scan's w_s4 and depth
    const uint4* pages;
    const DevPlan* plans;
    const float* metamax;
    float w_s4;
    uint32_t depth;
    uint32_t cap;  // candidate capacity (power of two >= k)
    uint64_t* out_ids;
    float* out_scores;
    uint32_t* out_counts;
    uint32_t* out_status;
};

__device__ __forceinline__ u64 probe_atleast_b(float s) { return (make_key(s, 0u) & 0xFFFFFFFF00000000ull) - 1ull; }

__global__ void __launch_bounds__(kSelThreads) bselect_kernel(const SelectLaunch p) {
    extern __shared__ __align__(16) unsigned char s_dyn[];
    const uint32_t q = blockIdx.x;
    const uint32_t n = p.G * 32;
    u64* keys = reinterpret_cast<u64*>(s_dyn);                  // n
    unsigned* hist = reinterpret_cast<unsigned*>(keys + n);     // kSelBins
    u64* top = reinterpret_cast<u64*>(hist + kSelBins);         // P2 (power of two >= k)
    __shared__ u64 s_prefix, s_mask;
    __shared__ unsigned s_rem, s_done, s_valid, s_cnt, s_flag, s_bin, s_above;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const u64* src = p.lists + (size_t)q * n;
    for (uint32_t i = tid; i < n; i += kSelThreads) keys[i] = src[i];
    if (tid == 0) { s_valid = 0; s_cnt = 0; s_flag = 0; s_prefix = 0; s_mask = 0; s_rem = p.k; s_done = 0; }
    __syncthreads();
    {
        unsigned v = 0;
        for (uint32_t i = tid; i < n; i += kSelThreads) v += keys[i] != 0ull;
        v = __reduce_add_sync(kFull, v);
        if (lane == 0 && v) atomicAdd(&s_valid, v);
    }
    __syncthreads();
    const uint32_t k = p.k;
    // threshold T: the keys >= T are exactly the top min(k, valid) keys (keys are unique)
    u64 T = 1ull;
    if (s_valid > k) {
        // 11-bit digits from the top (bits 53-63, 42-52, 31-41, 20-30, 9-19), then bits 0-8
        for (int d = 0; d < 6 && !s_done; ++d) {
            const int shift = d < 5 ? 53 - 11 * d : 0;
            const int bits = d < 5 ? 11 : 9;
            const u64 dmask = (((u64)1 << bits) - 1) << shift;
            for (int i = tid; i < kSelBins; i += kSelThreads) hist[i] = 0u;
            __syncthreads();
            const u64 pre = s_prefix, msk = s_mask;
            for (uint32_t i = tid; i < n; i += kSelThreads) {
                const u64 x = keys[i];
                if (x != 0ull && (x & msk) == pre) atomicAdd(&hist[(x & dmask) >> shift], 1u);
            }
            __syncthreads();
            if (warp == 0) {  // find the bin holding the s_rem-th key from the top
                unsigned part = 0;
                for (int j = 0; j < kSelBins / 32; ++j) part += hist[kSelBins - 1 - (lane * (kSelBins / 32) + j)];
                unsigned incl = part;  // inclusive prefix over lanes (lane 0 = highest bins)
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const unsigned y = __shfl_up_sync(kFull, incl, o);
                    if (lane >= o) incl += y;
                }
                const unsigned rem = s_rem;
                const unsigned excl = incl - part;
                if (excl < rem && rem <= incl) {
                    unsigned acc = excl;
                    for (int j = 0; j < kSelBins / 32; ++j) {
                        const int bin = kSelBins - 1 - (lane * (kSelBins / 32) + j);
                        const unsigned h = hist[bin];
                        if (acc + h >= rem) { s_bin = (unsigned)bin; s_above = acc; break; }
                        acc += h;
                    }
                }
            }
            __syncthreads();
            if (tid == 0) {
                const unsigned bin = s_bin;
                s_rem -= s_above;
                s_prefix |= (u64)bin << shift;
                s_mask |= dmask;
                if (hist[bin] == s_rem) s_done = 1;
            }
            __syncthreads();
        }
        T = s_prefix;
    }
    // Exact finishing. Every fast score is within E of the slot's exact score, so the exact top k
    // lies among the keys whose fast score is >= F_k - 2E (F_k: the k-th fast score), provided no
    // CTA list dropped such a key: a full list is safe when its last fast score + 4E < F_k. Those
    // candidates are rescored in the reference's f32 order and sorted by exact key.
    __shared__ __align__(16) float s_xt[kTabBw3 + kPrefix];
    __shared__ float2 s_rho[256];
    __shared__ float s_E;
    const DevPlan* P = p.plans + q;
    for (int i = tid; i < kPrefix * 16; i += kSelThreads) s_xt[i] = P->fp_prefix[i];
    for (int i = tid; i < kRabitq; i += kSelThreads) s_xt[kTabMidW + i] = P->mid_w[i];
    for (int i = tid; i < kFold; i += kSelThreads) s_xt[kTabTailW + i] = P->tail_w[i];
    for (int i = tid; i < kPrefix; i += kSelThreads) s_xt[kTabBw3 + i] = P->qp.bit_weights[i][3];
    fill_rho_tab(s_rho, tid, kSelThreads);
    if (tid == 0) s_E = fast_error_bound(*P, __ldg(reinterpret_cast<const float4*>(p.metamax)), p.w_s4, p.depth);
    const uint32_t cap = p.cap;
    for (uint32_t i = tid; i < cap; i += kSelThreads) top[i] = 0ull;
    __syncthreads();
    const float E = s_E;
    const bool all = s_valid <= k;
    const float fk = all ? 0.0f : key_score(T);
    const u64 lo = all ? 0ull : probe_atleast_b(__fsub_rd(fk, 2.0f * E));
    for (uint32_t i = tid; i < n; i += kSelThreads) {
        const u64 x = keys[i];
        if (x != 0ull && x > lo) {
            const unsigned at = atomicAdd(&s_cnt, 1u);
            if (at < cap) top[at] = x;
            else atomicOr(&s_flag, 1u);  // more candidates than room: rerun on the single-query kernel
        }
        // a full CTA list may have dropped a slot that belongs to the exact top k
        if ((i & 31u) == 31u && x != 0ull && (all || __fadd_ru(key_score(x), 4.0f * E) >= fk)) atomicOr(&s_flag, 1u);
    }
    __syncthreads();
    {
        Scalars S;
        fill_scalars(P, p.w_s4, p.depth, 1, S);
        const uint32_t nc = min(s_cnt, cap);
        for (uint32_t i = tid; i < nc; i += kSelThreads) {
            const uint32_t ord = key_ordinal(top[i]);
            Slot4 sl;
            load_slot(p.pages, ord >> 6, (int)(ord & 63u), sl);
            float sc = 0.0f;
            slot_score<MRL_MODE_EXACT>(sl.c0, sl.c1, sl.c2, sl.c3, reinterpret_cast<const int*>(s_xt), s_rho, S, sc,
                                       nullptr);
            top[i] = make_key(sc, ord);
        }
    }
    __syncthreads();
    for (uint32_t kk = 2; kk <= cap; kk <<= 1) {
        for (uint32_t j = kk >> 1; j > 0; j >>= 1) {
            for (uint32_t i = tid; i < cap; i += kSelThreads) {
                const uint32_t ixj = i ^ j;
                if (ixj > i) {
                    const u64 a = top[i], b = top[ixj];
                    const bool desc = (i & kk) == 0;
                    if (desc ? (a < b) : (a > b)) { top[i] = b; top[ixj] = a; }
                }
            }
            __syncthreads();
        }
    }
    const uint32_t m = min(s_valid, k);
    for (uint32_t i = tid; i < m; i += kSelThreads) {
        const u64 key = top[i];
        const uint32_t ord = key_ordinal(key);
        p.out_ids[(size_t)q * k + i] = ((uint64_t)(p.block_id_base + (ord >> 6)) << 16) | (uint64_t)(ord & 63u);
        p.out_scores[(size_t)q * k + i] = key_score(key);
    }
    if (tid == 0) {
        p.out_counts[q] = m;
        if (p.out_status) p.out_status[q] = (s_flag ? kStatusUncertified : 0u) | (p.err ? *p.err : 0u);
    }
}

// ---- tensor-core engine (tcgen05, kind::i8) ----
//
// The three stage sums of a slot for a query are dot products of 8-bit vectors:
//   prefix  = sum over (d, l) of [level_d == l] * T[d][l]     (one-hot of the 64 levels, K = 1024)
//   mid     = C1 + sum over d of bit_d * (fx1_d - fx0_d)        (the 128 mid-band bits, K = 128)
//   tail    = C4 + sum over d of bit_d * (fx1_d - fx0_d)        (the 64 folded-tail bits, K = 64)
// with the plan's int32 table entries split into four balanced base-256 digits in [-128, 127]
// (T = t0 + 2^8 t1 + 2^16 t2 + 2^24 t3). One int8 GEMM per stage, A = the slots' 0/1 bytes
// (128 slots x 1216 bytes, in tensor memory), B = the digits of 16 queries (64 rows x 1216 bytes,
// shared memory), D = 64 int32 columns per stage in tensor memory; each digit column sums at most
// 128 products of magnitude <= 128, and the stage sum is sum_j 2^(8j) D_j evaluated mod 2^32,
// which is exact because the true sum fits in int32. So the stage sums are the same integers as
// the table sums of the CUDA-core engine and of the single-query kernel.
constexpr int kTQ = 16;                 // queries per tensor tile
constexpr int kTG = 2;                  // query tiles per walk over the pages: one A build serves both
constexpr int kTN = 4 * kTQ;            // B rows: 4 digits per query
constexpr int kKAll = kPrefix * 16 + kRabitq + kFold;   // 1216 bytes of A per slot
constexpr int kACols = kKAll / 4;       // 304 tensor-memory columns hold a slot's A row
constexpr int kColP = kACols, kColS1 = kColP + kTN, kColS4 = kColS1 + kTN;  // 304, 368, 432
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kBTileBytes = (uint32_t)kTN * kKAll;  // 77,824: 76 K-blocks of 8 row groups x 128 B
constexpr uint32_t kKBlockBytes = (kTN / 8) * 128;        // 1,024: LBO (next 16 K bytes)
constexpr uint32_t kWaitPolls = 1u << 20;

// Byte offset of B element (row n, k) in the no-swizzle K-major core-matrix layout.
__host__ __device__ __forceinline__ uint32_t b_offset(int n, int k) {
    return (uint32_t)((k >> 4) * (kTN / 8) + (n >> 3)) * 128u + (uint32_t)(n & 7) * 16u + (uint32_t)(k & 15);
}

// B tiles and the constant terms of every query: digit j of entry k of query q at row 4 (q % 16) + j
// of tile q / 16.
__global__ void __launch_bounds__(256) tprep_kernel(const DevPlan* __restrict__ plans, uint32_t n_q,
                                                    uint8_t* __restrict__ tiles, int32_t* __restrict__ consts) {
    const uint32_t q = blockIdx.x;
    const DevPlan* P = plans + q;
    uint8_t* tile = tiles + (size_t)(q / kTQ) * kBTileBytes;
    const int r0 = 4 * (int)(q % kTQ);
    for (int k = threadIdx.x; k < kKAll; k += blockDim.x) {
        int32_t T;
        if (k < kPrefix * 16) {
            T = P->lut_prefix[k];
        } else if (k < kPrefix * 16 + kRabitq) {
            const int d = k - kPrefix * 16, g = d >> 2;
            T = P->lut4_s1[g * 16 + (1 << (d & 3))] - P->lut4_s1[g * 16];
        } else {
            const int d = k - kPrefix * 16 - kRabitq, g = d >> 2;
            T = P->lut4_s4[g * 16 + (1 << (d & 3))] - P->lut4_s4[g * 16];
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int32_t t = (int32_t)(int8_t)(T & 0xFF);  // balanced digit in [-128, 127]
            tile[b_offset(r0 + j, k)] = (uint8_t)t;
            T = (T - t) >> 8;
        }
    }
    if (threadIdx.x == 0) {
        int32_t c1 = 0, c4 = 0;
        for (int g = 0; g < kRabitq / 4; ++g) c1 += P->lut4_s1[g * 16];
        for (int g = 0; g < kFold / 4; ++g) c4 += P->lut4_s4[g * 16];
        consts[2 * q] = c1;
        consts[2 * q + 1] = c4;
    }
}

// The per-query constants of the f32 score path (fast_score with f32 unscaling), packed for
// three 16-byte shared loads; flags: bit 0 EdenProd prefix, 1 EdenB1 mid, 2 depth >= L1, 3 depth
// full with a tail fold, 4 f32 unscaling (else the query takes fast_score on its Scalars).
struct __align__(16) QConst {
    float eden_mean_ip, prefix_sum, mid_mean_ip, w_s4;
    float unf_p, unf_s1, unf_s4;
    uint32_t flags;
    int32_t c1, c4, pad0, pad1;
};

// fast_score (scan_common.cuh) on a QConst: the same operations in the same order.
__device__ __forceinline__ float qscore(const SlotMeta& m, int32_t P, int32_t s1, int32_t s4, const QConst& c) {
    const float cd = __fmul_rn(__int2float_rn(P), c.unf_p);
    float sc = (c.flags & 1u) ? __fadd_rn(c.eden_mean_ip, __fmul_rn(m.scale, cd))
                              : __fadd_rn(__fmul_rn(cd, m.scale), __fmul_rn(m.offset, c.prefix_sum));
    if (c.flags & 4u) {
        const float v = __fmul_rn(__int2float_rn(s1), c.unf_s1);
        if (c.flags & 2u) sc = __fadd_rn(sc, __fadd_rn(c.mid_mean_ip, __fmul_rn(m.offset, v)));
        else sc = __fadd_rn(sc, __fmul_rn(v, m.mid_n));
    }
    if (c.flags & 8u) {
        const float v = __fmul_rn(__int2float_rn(s4), c.unf_s4);
        sc = __fadd_rn(sc, __fmul_rn(__fmul_rn(v, fmaxf(m.high_n, 1e-6f)), c.w_s4));
    }
    return sc;
}

struct TShared {
    uint8_t B[kTG][kBTileBytes];         // offset 0 (1 KB aligned); tile t at t x 77,824 (76 KB)
    Scalars S[kTG * kTQ];
    QConst qc[kTG * kTQ];
    float2 rho[256];
    u64 tau[kTG * kTQ];
    BWarpState wst[kTG][kBWarps][4];
    u64 wlist[kTG][kBWarps][4][32];      // [tile][warp][query of its group][32]
    u64 queue[kTG][kBWarps][4][32];
    uint32_t pub[kTG * kTQ][16];         // per query: 8th/16th/24th/32nd key words of each lane quarter
    uint64_t bar;
    uint32_t taddr;
};

struct TensorLaunch {
    BatchLaunch b;
    const uint8_t* tiles;
    const int32_t* consts;
    uint32_t* err;
};

// The tensor engine's flush: bsel_flush, and the list also publishes the high words of its 8th,
// 16th, 24th and 32nd keys in its query's row `pub` (4 lane quarters x 4 words; 0 = no such key).
// A published word w_i of a list certifies 8 (i + 1) keys of that list with high word >= w_i, so
// the CTA holds >= 32 keys with high word >= v whenever at least four of the row's 16 words are
// >= v; the CTA bound rises to the largest such v (a key below it is not among the CTA's top 32).
// Words of other lists are read as they are: a list's i-th key only rises, so an older word still
// certifies its count.
__device__ __forceinline__ void tsel_flush(u64* wl, u64* q, int lane, u64* cta_tau, BWarpState* st, uint32_t* pub,
                                           int qw) {
    __syncwarp();
    const int qn = st->qn;
    u64 list = wl[lane];
    for (int base = 0; base < qn; base += 32) {
        u64 x = (base + lane < qn) ? q[base + lane] : 0ull;
        x = warp_sort32(x, lane);
        list = warp_merge32(list, x, lane);
    }
    const u64 t = __shfl_sync(kFull, list, 31);
    wl[lane] = list;
    volatile uint32_t* vp = pub;
    if ((lane & 7) == 7) vp[4 * qw + (lane >> 3)] = (uint32_t)(list >> 32);
    __syncwarp();
    uint32_t best = 0u;
    if (lane < 16) {
        const uint32_t v = vp[lane];
        if (v) {
            int c = 0;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const uint32_t w = vp[i];
                c += (w != 0u && w >= v) ? 1 : 0;
            }
            if (c >= 4) best = v;
        }
    }
    best = __reduce_max_sync(kFull, best);
    if (lane == 0) {
        st->qn = 0;
        st->tau = (uint32_t)(t >> 32);
        if (best) atomicMax(cta_tau, (u64)best << 32);
    }
    __syncwarp();
}

__device__ __forceinline__ void tsel_offer1(u64* wl, u64* q, int lane, u64* cta_tau, BWarpState* st, uint32_t* pub,
                                            int qw, u64 k0) {
    const uint32_t tc_ = (uint32_t)(*reinterpret_cast<volatile u64*>(cta_tau) >> 32);
    const uint32_t tau = max(max(st->tau, tc_), 1u);
    const bool p0 = (uint32_t)(k0 >> 32) >= tau;
    const unsigned m0 = __ballot_sync(kFull, p0);
    if (m0 == 0u) return;
    const int nn = __popc(m0);
    if (st->qn + nn > 32) tsel_flush(wl, q, lane, cta_tau, st, pub, qw);
    const int qn = st->qn;
    if (p0) q[qn + __popc(m0 & ((1u << lane) - 1u))] = k0;
    __syncwarp();
    if (lane == 0) st->qn = qn + nn;
    __syncwarp();
    if (qn + nn >= 32) tsel_flush(wl, q, lane, cta_tau, st, pub, qw);
}

// 1 << s, or 0 when s >= 32 (PTX shl.b32 clamps the shift amount to 32).
__device__ __forceinline__ uint32_t shl_clamp(uint32_t a, uint32_t s) {
    uint32_t d;
    asm("shl.b32 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(s));
    return d;
}
// One-hot bytes of the four 4-bit levels in nibbles 0..3 of `w`, 4 columns each: level l sets
// byte l & 3 of column l >> 2, i.e. column c = 1 << (8 l - 32 c), zero when that shift is outside
// 0..31 (a negative one wraps to a large unsigned shift). ALU only; a shared-memory pattern table
// costs bank conflicts under the data-dependent indices.
__device__ __forceinline__ void onehot4(uint32_t w, uint32_t (&r)[16]) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t s8 = i == 0 ? (w << 3) & 0x78u : (w >> (4 * i - 3)) & 0x78u;  // 8 x level i
#pragma unroll
        for (int c = 0; c < 4; ++c) r[4 * i + c] = shl_clamp(1u, s8 - 32u * (uint32_t)c);
    }
}
// 0/1 bytes of the 16 nibbles' bits of two words (64 bits) into 16 columns.
__device__ __forceinline__ void bits16(uint32_t w0, uint32_t w1, uint32_t (&r)[16]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        r[i] = (((w0 >> (4 * i)) & 15u) * 0x00204081u) & 0x01010101u;
        r[8 + i] = (((w1 >> (4 * i)) & 15u) * 0x00204081u) & 0x01010101u;
    }
}

__device__ __forceinline__ int32_t digits4(const uint32_t* d) {
    return (int32_t)(d[0] + (d[1] << 8) + (d[2] << 16) + (d[3] << 24));
}

// The 38 MMAs of one slot tile against one query tile's B digits (at b_smem), then the commit.
// Fully unrolled: consecutive K steps are 2 KB apart in B, i.e. +128 in the descriptor's
// start-address field (address >> 4; B ends below 256 KB, so the field never carries).
__device__ __forceinline__ void tile_mmas(uint32_t tbase, uint32_t b_smem, uint32_t idesc, uint64_t* bar) {
    const uint64_t d0 = tc::sdesc_kmajor(b_smem, kKBlockBytes, 128u);
    constexpr uint64_t kStep = (2u * kKBlockBytes) >> 4;
#pragma unroll
    for (int k = 0; k < kPrefix * 16 / 32; ++k)
        tc::mma_i8_ts(tbase + kColP, tbase + 8u * k, d0 + kStep * k, idesc, k > 0);
#pragma unroll
    for (int k = 0; k < kRabitq / 32; ++k)
        tc::mma_i8_ts(tbase + kColS1, tbase + 256u + 8u * k, d0 + kStep * (32 + k), idesc, k > 0);
#pragma unroll
    for (int k = 0; k < kFold / 32; ++k)
        tc::mma_i8_ts(tbase + kColS4, tbase + 288u + 8u * k, d0 + kStep * (36 + k), idesc, k > 0);
    tc::mma_commit(bar);
}

// Scores of this thread's slot for queries 4 g4 .. 4 g4 + 3 of query tile tt (stage sums as
// digit columns dp, d1, d4), then offered to the tile's selection. The four scores are made
// unrolled (the digit columns stay in registers); the offers run in a rolled loop, so the
// selection code (the flush's sort and merge) exists once per call site: with one copy per query
// the kernel's code overflowed the instruction cache (about 4% of a batch's time).
__device__ __forceinline__ void tile_epilogue(TShared& sh, int tt, uint32_t nq, int g4, int warp, int lane,
                                             const SlotMeta& m, bool live, uint32_t gid, const uint32_t (&dp)[16],
                                             const uint32_t (&d1)[16], const uint32_t (&d4)[16]) {
    u64 key[4];  // a query past the tile's last is scored on a stale constant row, never offered
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int qi = tt * kTQ + min(4 * g4 + j, kTQ - 1);
        const QConst c = sh.qc[qi];
        const int32_t P = digits4(dp + 4 * j);
        const int32_t A1 = c.c1 + digits4(d1 + 4 * j);
        const int32_t A4 = c.c4 + digits4(d4 + 4 * j);
        const float sc = (c.flags & 16u) ? qscore(m, P, A1, A4, c) : fast_score(m, P, A1, A4, sh.S[qi]);
        key[j] = (!live || m.tomb) ? 0ull : make_key(sc, gid);
    }
    const int nj = min(4, max(0, (int)nq - 4 * g4));  // warp-uniform: this group's queries in the tile
#pragma unroll 1
    for (int j = 0; j < nj; ++j) {
        const int qi = tt * kTQ + 4 * g4 + j;
        const u64 k0 = j == 0 ? key[0] : (j == 1 ? key[1] : (j == 2 ? key[2] : key[3]));
        tsel_offer1(sh.wlist[tt][warp][j], sh.queue[tt][warp][j], lane, &sh.tau[qi], &sh.wst[tt][warp][j],
                    sh.pub[qi], warp & 3, k0);
    }
}

__global__ void __launch_bounds__(kBThreads, 1) tscan_kernel(const TensorLaunch t) {
    extern __shared__ __align__(1024) unsigned char t_dyn[];
    TShared& sh = *reinterpret_cast<TShared*>(t_dyn);
    const BatchLaunch& p = t.b;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int qw = warp & 3, g4 = warp >> 2;  // lane quarter (slots) and column / query group
    const uint32_t G = gridDim.x;
    const uint32_t lo_b = (uint32_t)(((uint64_t)p.n_blocks * blockIdx.x) / G);
    const uint32_t hi_b = (uint32_t)(((uint64_t)p.n_blocks * (blockIdx.x + 1)) / G);
    if (warp == 0) {
        tc::tmem_alloc(&sh.taddr, kTmemCols);
        tc::tmem_relinquish();
    }
    if (tid == 0) {
        tc::mbar_init(&sh.bar, 1);
        tc::fence_mbar_init();
    }
    fill_rho_tab(sh.rho, tid, kBThreads);
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tbase = sh.taddr;
    const uint32_t my_lane = (uint32_t)(32 * qw) << 16;  // this warp's tensor-memory lane quarter
    const uint32_t idesc = tc::idesc_i8(128, kTN);
    const uint32_t b_smem = tc::smem_u32(&sh.B[0][0]);
    uint32_t phase = 0;
    bool failed = false;

    for (uint32_t q0 = 0; q0 < p.n_q && !failed; q0 += kTG * kTQ) {
        const uint32_t nqg = min((uint32_t)(kTG * kTQ), p.n_q - q0);  // queries of this group
        const int nt = (int)((nqg + kTQ - 1) / kTQ);                    // its query tiles (1 or 2)
        const uint32_t nq0 = min((uint32_t)kTQ, nqg), nq1 = nqg - nq0;
        __syncthreads();
        {  // the group's B digits, scalars, constants; selection state reset
            const uint4* src = reinterpret_cast<const uint4*>(t.tiles + (size_t)(q0 / kTQ) * kBTileBytes);
            uint4* dst = reinterpret_cast<uint4*>(&sh.B[0][0]);
            const uint32_t n16 = (uint32_t)nt * (kBTileBytes / 16);
            for (uint32_t i = tid; i < n16; i += kBThreads) dst[i] = __ldg(src + i);
        }
        if (tid < kTG * kTQ) {
            if ((uint32_t)tid < nqg) {
                fill_scalars(p.plans + q0 + tid, p.w_s4, p.depth, 1, sh.S[tid]);
                const Scalars& S = sh.S[tid];
                QConst c;
                c.eden_mean_ip = S.eden_mean_ip;
                c.prefix_sum = S.prefix_sum;
                c.mid_mean_ip = S.mid_mean_ip;
                c.w_s4 = S.w_s4;
                c.unf_p = S.unf_prefix;
                c.unf_s1 = S.unf_s1;
                c.unf_s4 = S.unf_s4;
                c.flags = (S.eden ? 1u : 0u) | (S.mid_b1 ? 2u : 0u) | (S.depth >= MRL_DEPTH_L1 ? 4u : 0u) |
                          (S.depth == MRL_DEPTH_FULL && S.has_tail ? 8u : 0u) | (S.f32_unscale ? 16u : 0u);
                c.c1 = t.consts[2 * (q0 + tid)];
                c.c4 = t.consts[2 * (q0 + tid) + 1];
                c.pad0 = c.pad1 = 0;
                sh.qc[tid] = c;
            }
            sh.tau[tid] = 0ull;
        }
        if (tid < kTG * kBWarps * 4) (&sh.wst[0][0][0])[tid] = BWarpState{0u, 0};
        for (int i = tid; i < kTG * kBWarps * 4 * 32; i += kBThreads) (&sh.wlist[0][0][0][0])[i] = 0ull;
        for (int i = tid; i < kTG * kTQ * 16; i += kBThreads) (&sh.pub[0][0])[i] = 0u;
        tc::fence_proxy_async_smem();  // generic-proxy writes of B -> tensor-core reads
        tc::fence_before();
        __syncthreads();
        tc::fence_after();

        // this thread's slot row of each tile: lane quarter qw; slot data one tile ahead
        const int r = 32 * qw + lane;
        const int v = r & 63;
        Slot4 nxt;
        nxt.c0 = nxt.c1 = nxt.c2 = nxt.c3 = make_uint4(0u, 0u, 0u, 0u);
        if (lo_b + (uint32_t)(r >> 6) < hi_b && page_live(p, lo_b + (uint32_t)(r >> 6)))
            load_slot(p.pages, lo_b + (uint32_t)(r >> 6), v, nxt);
        for (uint32_t pg = lo_b; pg < hi_b; pg += 2) {
            // ---- A: this thread's slot row, this warp's column share (g4)
            const uint32_t b = pg + (uint32_t)(r >> 6);
            const bool live = b < hi_b && page_live(p, b);  // warp-uniform
            const Slot4 s = nxt;
            {
                const uint32_t bn = b + 2;
                nxt.c0 = nxt.c1 = nxt.c2 = nxt.c3 = make_uint4(0u, 0u, 0u, 0u);
                if (bn < hi_b && page_live(p, bn)) load_slot(p.pages, bn, v, nxt);
            }
            const SlotMeta m = slot_meta_tab(s.c3.z, s.c3.w, sh.rho);
            {
                // levels of dims 16 g4 .. 16 g4 + 15: words 2 g4 and 2 g4 + 1 of the prefix
                const uint32_t wa = g4 < 2 ? (g4 == 0 ? s.c0.x : s.c0.z) : (g4 == 2 ? s.c1.x : s.c1.z);
                const uint32_t wb = g4 < 2 ? (g4 == 0 ? s.c0.y : s.c0.w) : (g4 == 2 ? s.c1.y : s.c1.w);
                uint32_t rr[16];
#pragma unroll
                for (int c = 0; c < 4; ++c) {  // dims 16 g4 + 4c .. + 3
                    const uint32_t w = (c < 2 ? wa : wb) >> (16 * (c & 1));
                    onehot4(w, rr);
                    TC_ST16(tbase + my_lane + (uint32_t)(64 * g4 + 16 * c), rr);
                }
                if (g4 == 0) { bits16(s.c2.x, s.c2.y, rr); TC_ST16(tbase + my_lane + 256u, rr); }
                if (g4 == 1) { bits16(s.c2.z, s.c2.w, rr); TC_ST16(tbase + my_lane + 272u, rr); }
                if (g4 == 2) { bits16(s.c3.x, s.c3.y, rr); TC_ST16(tbase + my_lane + 288u, rr); }
            }
            tc::wait_st();
            tc::fence_before();
            __syncthreads();
            if (tid == 0) {
                tc::fence_after();
                tile_mmas(tbase, b_smem, idesc, &sh.bar);
            }
            // one thread polls the mbarrier; the others sleep in the CTA barrier (no issue slots
            // or shared-memory polls taken from the MMA issue)
            bool ok = tid != 0 || tc::mbar_wait(&sh.bar, phase, kWaitPolls);
            phase ^= 1u;
            if (__syncthreads_or(!ok)) {
                failed = true;
                break;
            }
            tc::fence_after();
            // ---- epilogue: this thread's slot; tile 1's MMAs run while tile 0's scores are made
            uint32_t dp[16], d1[16], d4[16];
            TC_LD16(dp, tbase + my_lane + (uint32_t)(kColP + 16 * g4));
            TC_LD16(d1, tbase + my_lane + (uint32_t)(kColS1 + 16 * g4));
            TC_LD16(d4, tbase + my_lane + (uint32_t)(kColS4 + 16 * g4));
            tc::wait_ld();
            if (nt > 1) {
                tc::fence_before();
                __syncthreads();  // every thread has read D: tile 1's MMAs may overwrite it
                if (tid == 0) {
                    tc::fence_after();
                    tile_mmas(tbase, b_smem + kBTileBytes, idesc, &sh.bar);
                }
            }
            const uint32_t gid = b * 64 + v;
            tile_epilogue(sh, 0, nq0, g4, warp, lane, m, live, gid, dp, d1, d4);
            if (nt > 1) {
                ok = tid != 0 || tc::mbar_wait(&sh.bar, phase, kWaitPolls);
                phase ^= 1u;
                if (__syncthreads_or(!ok)) {
                    failed = true;
                    break;
                }
                tc::fence_after();
                TC_LD16(dp, tbase + my_lane + (uint32_t)(kColP + 16 * g4));
                TC_LD16(d1, tbase + my_lane + (uint32_t)(kColS1 + 16 * g4));
                TC_LD16(d4, tbase + my_lane + (uint32_t)(kColS4 + 16 * g4));
                tc::wait_ld();
                tile_epilogue(sh, 1, nq1, g4, warp, lane, m, live, gid, dp, d1, d4);
            }
            tc::fence_before();
            __syncthreads();  // tensor memory (A and D) free for the next slot tile
        }
        if (failed) break;
#pragma unroll 1
        for (int tt = 0; tt < nt; ++tt)
#pragma unroll 1
            for (int j = 0; j < 4; ++j)
                if (sh.wst[tt][warp][j].qn)
                    tsel_flush(sh.wlist[tt][warp][j], sh.queue[tt][warp][j], lane, &sh.tau[tt * kTQ + 4 * g4 + j],
                               &sh.wst[tt][warp][j], sh.pub[tt * kTQ + 4 * g4 + j], qw);
        __syncthreads();
        for (int tt = 0; tt < nt; ++tt) {
            if ((uint32_t)warp < (tt == 0 ? nq0 : nq1)) {  // warp w merges query w: the 4 lane quarters' lists
                const int g = warp >> 2, j = warp & 3;
                const u64 a = warp_merge32(sh.wlist[tt][4 * g + 0][j][lane], sh.wlist[tt][4 * g + 1][j][lane], lane);
                const u64 c = warp_merge32(sh.wlist[tt][4 * g + 2][j][lane], sh.wlist[tt][4 * g + 3][j][lane], lane);
                p.lists[((size_t)(q0 + tt * kTQ + warp) * G + blockIdx.x) * 32 + lane] = warp_merge32(a, c, lane);
            }
        }
    }
    if (failed) {
        if (tid == 0) atomicOr(t.err, 2u);
        tc::mbar_wait(&sh.bar, phase ^ 1u, kWaitPolls);  // the MMAs in flight, bounded
    }
    tc::fence_before();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tbase, kTmemCols);
}

}  // namespace

size_t batch_scratch_bytes(uint32_t ctas, uint32_t n_q) {
    const size_t lists = (size_t)n_q * ctas * 32 * sizeof(u64);
    const size_t tiles = (size_t)((n_q + kTQ - 1) / kTQ) * kBTileBytes;
    return lists + tiles + (size_t)n_q * 2 * sizeof(int32_t) + 256;
}

int launch_scan_batch(const uint4* pages, const uint2* block_ts, uint32_t n_blocks, uint32_t block_id_base,
                      const float* metamax, const DevPlan* plans, uint32_t n_q, uint32_t k, float w_s4, uint32_t depth, uint32_t use_time,
                      uint32_t has_lo, uint32_t lo, uint32_t has_hi, uint32_t hi, uint32_t ctas, uint32_t engine,
                      void* scratch, uint64_t* out_ids, float* out_scores, uint32_t* out_counts, uint32_t* out_status,
                      cudaStream_t stream) {
    if (n_q == 0) return 0;
    if (k < 1 || k > 4096 || depth == MRL_DEPTH_L0 || ctas < 1) return -1;
    BatchLaunch b{};
    b.pages = pages;
    b.block_ts = block_ts;
    b.n_blocks = n_blocks;
    b.plans = plans;
    b.n_q = n_q;
    b.w_s4 = w_s4;
    b.depth = depth;
    b.use_time = use_time;
    b.has_lo = has_lo;
    b.lo = lo;
    b.has_hi = has_hi;
    b.hi = hi;
    // scratch: lists [n_q][ctas][32] keys | B digit tiles | per-query constants | error word
    unsigned char* base = static_cast<unsigned char*>(scratch);
    const size_t lists_bytes = (size_t)n_q * ctas * 32 * sizeof(u64);
    const size_t tiles_bytes = (size_t)((n_q + kTQ - 1) / kTQ) * kBTileBytes;
    b.lists = reinterpret_cast<u64*>(base);
    uint8_t* tiles = base + ((lists_bytes + 255) & ~(size_t)255);
    int32_t* consts = reinterpret_cast<int32_t*>(tiles + tiles_bytes);
    uint32_t* err = reinterpret_cast<uint32_t*>(consts + 2 * (size_t)n_q);
    if (engine == MRL_BATCH_TENSOR) {
        static_assert(sizeof(TShared) <= 227 * 1024, "tensor batched scan shared memory");
        // at least 120 KB, so that one CTA (and its 512 tensor-memory columns) occupies each SM
        const size_t smem = sizeof(TShared) > 120 * 1024 ? sizeof(TShared) : 120 * 1024;
        if (cudaFuncSetAttribute(tscan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return -1;
        if (cudaMemsetAsync(tiles, 0, tiles_bytes, stream) != cudaSuccess) return -1;
        if (cudaMemsetAsync(err, 0, sizeof(uint32_t), stream) != cudaSuccess) return -1;
        tprep_kernel<<<n_q, 256, 0, stream>>>(plans, n_q, tiles, consts);
        if (cudaGetLastError() != cudaSuccess) return -1;
        TensorLaunch t{b, tiles, consts, err};
        tscan_kernel<<<ctas, kBThreads, smem, stream>>>(t);
    } else {
        static_assert(sizeof(BShared) <= 227 * 1024, "batched scan shared memory");
        const size_t smem = sizeof(BShared);
        if (cudaFuncSetAttribute(bscan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return -1;
        if (cudaMemsetAsync(err, 0, sizeof(uint32_t), stream) != cudaSuccess) return -1;
        bscan_kernel<<<ctas, kBThreads, smem, stream>>>(b);
    }
    if (cudaGetLastError() != cudaSuccess) return -1;
    // candidate room: k plus the near-ties of the k-th score, as a power of two
    uint32_t P2 = 1;
    while (P2 < k + 64) P2 <<= 1;
    const size_t ssmem = (size_t)ctas * 32 * sizeof(u64) + kSelBins * sizeof(unsigned) + (size_t)P2 * sizeof(u64);
    if (ssmem > 227 * 1024) return -1;
    if (cudaFuncSetAttribute(bselect_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ssmem) != cudaSuccess)
        return -1;
    SelectLaunch s{};
    s.lists = b.lists;
    s.err = err;
    s.G = ctas;
    s.n_q = n_q;
    s.k = k;
    s.block_id_base = block_id_base;
    s.pages = pages;
    s.plans = plans;
    s.metamax = metamax;
    s.w_s4 = w_s4;
    s.depth = depth;
    s.cap = P2;
    s.out_ids = out_ids;
    s.out_scores = out_scores;
    s.out_counts = out_counts;
    s.out_status = out_status;
    bselect_kernel<<<n_q, kSelThreads, ssmem, stream>>>(s);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace mrl
