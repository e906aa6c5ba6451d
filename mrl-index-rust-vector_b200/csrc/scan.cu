// scan.cu — fused single-query PaxBlock64 scan + top-k for sm_100a.
//
// Replaces scan_blocks / scan_block / Shortlist (src/scan.rs:310-886). One launch scores every
// live slot of a segment for one plan and leaves the top-k (by score, ties to the lower slot
// ordinal) in the output buffers.
//
// Work split: one 512-thread CTA per SM. The first 7/8 of the pages are split into one contiguous
// range per CTA, whose warps take pages from a shared-memory counter; the last 1/8 is handed out one
// page at a time from a global counter to CTAs that have finished their range. Each warp scores two
// slots per lane, reading each slot's 64 bytes of the vector-major page layout with four coalesced
// 16-byte loads, and loads the next page while it scores the current one.
//
// Scoring (one thread per slot):
//   * MRL_MODE_FAST — every stage inner product is an exact int32 sum of table entries held in
//     shared memory: 64 per-dimension 16-entry prefix tables indexed by the slot's 4-bit level, and
//     5-bit-window tables over the 128 mid-band and 64 folded-tail bits. Tables have <= 32 entries,
//     so a warp-uniform table index never causes a shared-memory bank conflict. Each fast score is
//     within a proven bound E of the slot's exact score; the fast scores only choose candidates,
//     which are rescored in the reference's f32 order before the final ranking, so the results
//     are the exact mode's.
//   * MRL_MODE_EXACT — the reference's f32 loops in the reference order (sequential adds of
//     rounded products), giving bit-identical scores.
// Both compute the full score of every live slot (no stage pruning). Under the reference's
// exactness condition (cs_tolerance >= 1 and w_s4*sqrt(2/pi)*sqrt(B) <= cs_tolerance, true for
// the defaults) every stage bound of src/scan.rs:453-607 is >= the full score, so the reference's
// final shortlist is exactly the top-k by full score; computing all scores reproduces it without
// the order-dependent threshold. Configurations outside that condition are refused by the host.
//
// Selection: each warp keeps a sorted top-32 of its keys in registers (one key per lane) and
// filters new keys against max(its own list_len-th key, a CTA-wide bound in shared memory);
// survivors go through a per-warp shared-memory queue and are merged 32 at a time with warp
// bitonic networks. Each CTA tree-merges its warps' lists, rescores them exactly (fast mode) and
// publishes its top-`list_len` with a ready flag. The first CTA to publish is the finisher: it loads
// every CTA's list as that list's flag appears (overlapping the other CTAs' scoring), checks that
// the union of the lists holds the top-k, locates the k-th key in a histogram of score words,
// gathers the keys within 2E of it and ranks them by exact key. The other CTAs exit at once. If a
// CTA's full list may have dropped a top-k member, the finisher rescans that CTA's pages (owner[])
// and reselects by radix select + bitonic sort, so the result is exact for every input (status
// bit 0 reports it).
//
// Overlapping queries: every CTA lets the next launch on the stream start (programmatic dependent
// launch) at its own start, so the next query's CTAs take each SM as soon as this query's CTA there
// has published. The context's scratch comes in two parities used by alternate launches; a launch
// touches its parity only once the launch two back has released it (a done word the last CTA to
// exit stores after zeroing the control words), and its finisher writes the outputs only after the
// previous launch has completed (griddepcontrol.wait).
#include <algorithm>
#include <atomic>
#include <cstring>

#include "exchange.cuh"
#include "plan_build.cuh"
#include "scan_common.cuh"

namespace mrl {
namespace {

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kQueue = 64;
template <int MODE>
__device__ __forceinline__ u64 slot_key(const Slot4& s, uint32_t ordinal, const int* tab, const float2* rho_tab,
                                        const Scalars& S) {
    float sc;
    if (!slot_score<MODE>(s.c0, s.c1, s.c2, s.c3, tab, rho_tab, S, sc, nullptr)) return 0ull;
    return make_key(sc, ordinal);
}

struct WarpSel {
    u64 list;       // this lane's rank in the warp's top-32
    uint32_t tau;   // high word of list[list_len-1] (0 until the list holds list_len keys)
    int qn;         // queued candidates
};

__device__ __forceinline__ void warp_flush(WarpSel& ws, u64* q, int lane, uint32_t list_len, u64* cta_tau) {
    __syncwarp();
    for (int base = 0; base < ws.qn; base += 32) {
        u64 x = (base + lane < ws.qn) ? q[base + lane] : 0ull;
        x = warp_sort32(x, lane);
        ws.list = warp_merge32(ws.list, x, lane);
    }
    ws.qn = 0;
    const u64 t = __shfl_sync(kFull, ws.list, list_len - 1);
    ws.tau = (uint32_t)(t >> 32);
    if (lane == 0 && t) atomicMax(cta_tau, t);
    __syncwarp();
}

// Offer two keys per lane. A key survives when its score word is >= the score word of the
// current bound (the warp's list_len-th key or the CTA bound): a conservative test, exact ties are
// settled by the 64-bit merges. Active keys always have a nonzero score word.
__device__ __forceinline__ void warp_offer(WarpSel& ws, u64* q, int lane, uint32_t list_len, u64* cta_tau,
                                           u64 k0, u64 k1) {
    const uint32_t tc = (uint32_t)(*reinterpret_cast<volatile u64*>(cta_tau) >> 32);
    const uint32_t tau = max(max(ws.tau, tc), 1u);
    const bool p0 = (uint32_t)(k0 >> 32) >= tau, p1 = (uint32_t)(k1 >> 32) >= tau;
    const unsigned m0 = __ballot_sync(kFull, p0), m1 = __ballot_sync(kFull, p1);
    if ((m0 | m1) == 0u) return;
    const int nn = __popc(m0) + __popc(m1);
    if (ws.qn + nn > kQueue) warp_flush(ws, q, lane, list_len, cta_tau);
    const unsigned lt = (1u << lane) - 1u;
    if (p0) q[ws.qn + __popc(m0 & lt)] = k0;
    if (p1) q[ws.qn + __popc(m0) + __popc(m1 & lt)] = k1;
    ws.qn += nn;
    if (ws.qn >= 32) warp_flush(ws, q, lane, list_len, cta_tau);
}

// ---- final selection helpers (last CTA) ----
constexpr int kBins = 2048;  // 11-bit radix digits

__device__ __forceinline__ void hist_add(unsigned* hist, bool valid, unsigned bin, int lane) {
    const unsigned act = __ballot_sync(kFull, valid);
    if (valid) {
        const unsigned peers = __match_any_sync(act, bin);
        if (lane == __ffs(peers) - 1) atomicAdd(&hist[bin], (unsigned)__popc(peers));
    }
}

struct SelState {
    u64 prefix, mask;
    unsigned rem;
    unsigned done;
    unsigned bin, before;
    unsigned warp_sum[kWarps];
};

template <int MODE>
struct Finisher {
    const ScanLaunch& p;
    const int* tab;         // the scan's tables (this mode's)
    const int* xtab;        // exact-mode tables (== tab in MRL_MODE_EXACT)
    const float2* rho_tab;
    const Scalars& S;
    const u64* cand;        // G * 32 scan keys, the first list_len of each CTA are live
    const u64* xcand;       // the same entries' exact keys (== cand in MRL_MODE_EXACT)
    const unsigned* flags;  // flagged CTA ids
    unsigned nflag;
    unsigned G;
    unsigned list_len;

    // Visit every candidate of the (virtual) set by its exact key: the CTA lists in shared memory
    // plus, for flagged CTAs, a rescan of the pages they scored keeping the slots whose scan key is
    // below their list minimum (the ones the list dropped). fn(valid, exact_key, lane) is called
    // warp-uniformly.
    template <class Fn>
    __device__ __forceinline__ void visit(Fn fn) const {
        const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
        const unsigned nu = G * list_len;
        for (unsigned base = 0; base < nu; base += kThreads) {
            const unsigned i = base + tid;
            const unsigned at = (i / list_len) * 32 + (i % list_len);
            const u64 x = i < nu ? cand[at] : 0ull;
            fn(x != 0ull, x != 0ull ? xcand[at] : 0ull, lane);
        }
        for (unsigned f = 0; f < nflag; ++f) {
            const unsigned c = flags[f];
            const u64 minc = cand[c * 32 + list_len - 1];
            for (uint32_t b = warp; b < p.n_blocks; b += kWarps) {
                if (__ldcg(p.owner + b) != (uint8_t)c) continue;  // warp-uniform
                u64 k0 = 0, k1 = 0, x0 = 0, x1 = 0;
                if (block_live(p, b)) {
                    Slot4 s0, s1;
                    load_slot(p.pages, b, lane, s0);
                    load_slot(p.pages, b, lane + 32, s1);
                    k0 = slot_key<MODE>(s0, b * 64 + lane, tab, rho_tab, S);
                    k1 = slot_key<MODE>(s1, b * 64 + lane + 32, tab, rho_tab, S);
                    x0 = MODE == MRL_MODE_FAST ? slot_key<MRL_MODE_EXACT>(s0, b * 64 + lane, xtab, rho_tab, S) : k0;
                    x1 = MODE == MRL_MODE_FAST ? slot_key<MRL_MODE_EXACT>(s1, b * 64 + lane + 32, xtab, rho_tab, S) : k1;
                }
                fn(k0 != 0ull && k0 < minc, x0, lane);
                fn(k1 != 0ull && k1 < minc, x1, lane);
            }
        }
    }
};

// Exact k-th largest key of the candidate set: radix select, 11-bit digits from the top with an
// early exit once the current digit's bin holds exactly the keys still to be selected. Returns T
// such that the keys >= T are exactly the top min(k, count) keys.
template <int MODE>
__device__ __forceinline__ u64 select_threshold(const Finisher<MODE>& F, unsigned k, unsigned* hist, SelState* st) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) { st->prefix = 0; st->mask = 0; st->rem = k; st->done = 0; }
    if (tid == 0) hist[0] = 0;
    __syncthreads();
    F.visit([&](bool valid, u64, int ln) { hist_add(hist, valid, 0u, ln); });
    __syncthreads();
    const unsigned total = hist[0];
    __syncthreads();
    if (total <= k) return 1ull;
    const int shifts[6] = {53, 42, 32, 21, 10, 0};
    const int widths[6] = {11, 11, 10, 11, 11, 10};
    for (int pass = 0; pass < 6; ++pass) {
        const int shift = shifts[pass];
        const unsigned nb = 1u << widths[pass];
        for (unsigned i = tid; i < (unsigned)kBins; i += kThreads) hist[i] = 0;
        __syncthreads();
        const u64 prefix = st->prefix, mask = st->mask;
        F.visit([&](bool valid, u64 x, int ln) {
            const bool in = valid && ((x & mask) == prefix);
            hist_add(hist, in, (unsigned)((x >> shift) & (nb - 1)), ln);
        });
        __syncthreads();
        unsigned c[4], lsum = 0;  // descending scan: thread t owns bins nb-1-4t .. nb-4-4t
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int bin = (int)nb - 1 - 4 * tid - j;
            c[j] = bin >= 0 ? hist[bin] : 0u;
            lsum += c[j];
        }
        unsigned incl = lsum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned y = __shfl_up_sync(kFull, incl, o);
            if (lane >= o) incl += y;
        }
        if (lane == 31) st->warp_sum[warp] = incl;
        __syncthreads();
        unsigned wbase = 0;
        for (int w = 0; w < warp; ++w) wbase += st->warp_sum[w];
        unsigned cum = wbase + incl - lsum;
        const unsigned rem = st->rem;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (cum < rem && rem <= cum + c[j]) { st->bin = (unsigned)((int)nb - 1 - 4 * tid - j); st->before = cum; }
            cum += c[j];
        }
        __syncthreads();
        if (tid == 0) {
            const unsigned bin = st->bin;
            st->prefix |= (u64)bin << shift;
            st->mask |= (u64)(nb - 1) << shift;
            st->rem -= st->before;
            if (hist[bin] == st->rem) st->done = 1;
        }
        __syncthreads();
        if (st->done) break;
    }
    return st->prefix;
}

// Rare path, one CTA: some CTA lists (`flags`, `nflag` of them) ended inside the top-k, so they may
// have dropped members. Reselect over the union of lists plus those CTAs' rescanned keys and write
// the whole output.
template <int MODE>
__device__ __forceinline__ void reselect(const ScanLaunch& p, const int* tab, const int* xtab, const float2* rho_tab, const Scalars& S,
                         u64* cand, u64* xcand, u64* gath, unsigned* hist, const unsigned* flags, unsigned nflag,
                         SelState* st, unsigned* s_misc) {
    const int tid = threadIdx.x;
    const unsigned G = gridDim.x;
    for (unsigned i = tid; i < G * 32; i += kThreads) {
        cand[i] = __ldcg(p.cta_keys + i);
        if (MODE == MRL_MODE_FAST) xcand[i] = __ldcg(p.cta_xkeys + i);
    }
    if (tid == 0) s_misc[1] = 0;
    __syncthreads();
    Finisher<MODE> F{p, tab, xtab, rho_tab, S, cand, MODE == MRL_MODE_FAST ? xcand : cand, flags, nflag, G, p.list_len};
    const u64 tau = select_threshold<MODE>(F, p.k, hist, st);
    F.visit([&](bool valid, u64 x, int ln) {
        const bool in = valid && x >= tau;
        const unsigned m = __ballot_sync(kFull, in);
        unsigned base = 0;
        if (ln == 0 && m) base = atomicAdd(&s_misc[1], (unsigned)__popc(m));
        base = __shfl_sync(kFull, base, 0);
        if (in) gath[base + __popc(m & ((1u << ln) - 1u))] = x;
    });
    __syncthreads();
    const unsigned ng = min(s_misc[1], p.k);
    unsigned P2 = 1;
    while (P2 < ng) P2 <<= 1;
    for (unsigned i = ng + tid; i < P2; i += kThreads) gath[i] = 0ull;
    __syncthreads();
    for (unsigned kk = 2; kk <= P2; kk <<= 1) {
        for (unsigned j = kk >> 1; j > 0; j >>= 1) {
            for (unsigned i = tid; i < P2; i += kThreads) {
                const unsigned ixj = i ^ j;
                if (ixj > i) {
                    const u64 a = gath[i], b = gath[ixj];
                    const bool desc = (i & kk) == 0;
                    if (desc ? (a < b) : (a > b)) { gath[i] = b; gath[ixj] = a; }
                }
            }
            __syncthreads();
        }
    }
    for (unsigned i = tid; i < ng; i += kThreads) {
        const u64 key = gath[i];
        const uint32_t ord = key_ordinal(key);
        p.out_ids[i] = ((uint64_t)(p.block_id_base + (ord >> 6)) << 16) | (uint64_t)(ord & 63u);
        p.out_scores[i] = key_score(key);
    }
    if (tid == 0) *p.out_count = ng;
}

// The scan's shared-memory tables from a plan (ints in fast mode, floats in exact mode).
__device__ __forceinline__ void copy_tables(const DevPlan* __restrict__ P, int mode, int* tab, const ScanLaunch& p) {
    const int tid = threadIdx.x;
    if (mode == MRL_MODE_FAST) {
        for (int i = tid; i < kPrefix * 16; i += kThreads) tab[i] = P->lut_prefix[i];
        for (int i = tid; i < kS1Windows * 32; i += kThreads) tab[kTabS1 + i] = P->lut_s1[i];
        for (int i = tid; i < kS4Windows * 32; i += kThreads) tab[kTabS4 + i] = P->lut_s4[i];
        if (p.depth == MRL_DEPTH_L0)
            for (int i = tid; i < kPrefix * 16; i += kThreads) tab[kTabL0 + i] = P->lut_l0[i];
    } else {
        float* ft = reinterpret_cast<float*>(tab);
        for (int i = tid; i < kPrefix * 16; i += kThreads) ft[i] = P->fp_prefix[i];
        for (int i = tid; i < kRabitq; i += kThreads) ft[kTabMidW + i] = P->mid_w[i];
        for (int i = tid; i < kFold; i += kThreads) ft[kTabTailW + i] = P->tail_w[i];
        for (int i = tid; i < kPrefix; i += kThreads) ft[kTabBw3 + i] = P->qp.bit_weights[i][3];
    }
}

__device__ __forceinline__ void load_tables(const DevPlan* __restrict__ P, int mode, int* tab, float2* rho_tab,
                                            Scalars& S, const ScanLaunch& p) {
    copy_tables(P, mode, tab, p);
    fill_rho_tab(rho_tab, threadIdx.x, kThreads);
    fill_scalars(P, p.w_s4, p.depth, (int32_t)(p.list_len != 0u), S);  // one: 1 for every launch, opaque to the compiler
}

// Fast mode's copy of the exact-mode tables (same layout as load_tables' exact branch), read only
// by the exact rescoring of list entries.
__device__ __forceinline__ void load_exact_tables(const DevPlan* __restrict__ P, float* ft) {
    const int tid = threadIdx.x;
    for (int i = tid; i < kPrefix * 16; i += kThreads) ft[i] = P->fp_prefix[i];
    for (int i = tid; i < kRabitq; i += kThreads) ft[kTabMidW + i] = P->mid_w[i];
    for (int i = tid; i < kFold; i += kThreads) ft[kTabTailW + i] = P->tail_w[i];
    for (int i = tid; i < kPrefix; i += kThreads) ft[kTabBw3 + i] = P->qp.bit_weights[i][3];
}

// Number of keys greater than x in lst[0..n), 1 <= n <= 32, sorted descending (keys unique, empty
// slots 0 at the end): a branch-free binary lift of six fixed steps (clamped loads, selects), so
// independent calls overlap.
__device__ __forceinline__ unsigned count_greater(const u64* lst, unsigned n, u64 x) {
    unsigned lo = 0;
#pragma unroll
    for (int s = 5; s >= 0; --s) {
        const unsigned t = lo + (1u << s);
        const u64 v = lst[min(t, n) - 1];
        lo = (t <= n && v > x) ? t : lo;
    }
    return lo;
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Last step of the NVLink exchange, by the finisher once this rank's record is complete in
// xch_stage: wait until the previous launch on the stream has completed (its finisher may still be
// merging from this parity's area two launches back, or writing the same outputs), copy the record
// into this rank's slot of every rank's area (peer stores over NVLink for the others), raise this
// rank's flag in the other areas (release, system scope), wait (bounded, ~2-3 s) for every other
// rank's flag of this epoch in this rank's own area, copy all records of this area into shared
// memory (`smem`, at least xch_world records; local loads only) and merge them into the outputs.
// Only this step is ordered after the previous launch; the load and ranking of this rank's lists
// before it overlap the previous query's exchange. Status bit 2 reports a timeout.
__device__ void xch_publish_and_merge(const ScanLaunch& p, unsigned char* smem, int* s_ok, unsigned status) {
    const int tid = threadIdx.x;
    const size_t rb = MRL_MERGE_RECORD_BYTES(p.k), words = rb / 16;
    const unsigned nw = (unsigned)words;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    __syncthreads();
    {
        // this rank's record (staged) into its slot in every rank's area: posted stores, all
        // threads, so the copies to all peers are in flight at once
        const uint4* src = reinterpret_cast<const uint4*>(p.xch_stage);
        const unsigned total = p.xch_world * nw;
        for (unsigned i = tid; i < total; i += kThreads)
            reinterpret_cast<uint4*>(p.xch_rec[i / nw])[i % nw] = __ldcg(src + i % nw);
    }
    __syncthreads();
    if (tid < 32) {
        // warp 0: lane w raises this rank's flag in rank w's area; lane s polls rank s's flag in
        // this area, so all waits overlap and every poll is a local load
        const bool peer = (unsigned)tid < p.xch_world && (unsigned)tid != p.xch_rank;
        if (peer) {
            __threadfence_system();
            st_release_sys(p.xch_flag[tid], p.xch_epoch);
        }
        bool arrived = !peer;
        unsigned it = 0;
        while (!__all_sync(kFull, arrived)) {
            if (!arrived) arrived = ld_acquire_sys(p.xch_flag_in + tid) == p.xch_epoch;
            if (++it > (1u << 22)) break;  // ~2-3 s
            if (it > 256) __nanosleep(128);
        }
        const bool ok = __all_sync(kFull, arrived);
        if (tid == 0) *s_ok = ok ? 1 : 0;
    }
    __syncthreads();
    if (!*s_ok) {
        if (tid == 0 && p.out_status) *p.out_status = status | 4u;  // a rank's record never arrived
        return;
    }
    {
        // every rank's record (this area's receive slots) into shared memory, four loads in flight per
        // thread before their stores
        const unsigned total = p.xch_world * nw;
        const uint4* src = reinterpret_cast<const uint4*>(p.xch_recv);
        for (unsigned i0 = tid; i0 < total; i0 += 4u * kThreads) {
            uint4 x[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const unsigned i = i0 + (unsigned)j * kThreads;
                if (i < total) x[j] = __ldcg(src + i);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const unsigned i = i0 + (unsigned)j * kThreads;
                if (i < total) reinterpret_cast<uint4*>(smem)[i] = x[j];
            }
        }
    }
    __syncthreads();
    if (p.xch_tree)
        xch::merge_records_tree(smem, smem + (size_t)p.xch_world * rb, p.xch_world, p.k, p.k, p.out_ids, p.out_scores,
                                p.out_count);
    else
        xch::merge_records<false>(smem, p.xch_world, p.k, p.k, p.out_ids, p.out_scores, p.out_count);
    if (tid == 0 && p.out_status) *p.out_status = status;
}


// Shared-memory layout of the fused plan build, aliasing the selection buffers (unused until the
// scoring loop): the plan, the query copy, the build's scratch.
__host__ __device__ constexpr size_t align16(size_t x) { return (x + 15) & ~(size_t)15; }
__host__ __device__ inline size_t fused_plan_bytes(uint32_t dims) {
    return align16(sizeof(DevPlan)) + align16((size_t)dims * sizeof(float)) + align16(sizeof(planb::PlanShared));
}

// Score-word probe for count_greater: the keys above probe_above(s) are those with a score > s.
__device__ __forceinline__ u64 probe_above(float s) { return make_key(s, 0u) | 0xFFFFFFFFull; }

// Order-preserving word of a score (the high word of its selection key): scores at least s are
// the keys whose high word is at least score_word(s).
__device__ __forceinline__ unsigned score_word(float s) { return (unsigned)(make_key(s, 0u) >> 32); }

// Bin of a score word among kBins equal bins over [lo, lo + kBins / scale): monotone in w.
__device__ __forceinline__ unsigned bin_of(unsigned w, unsigned lo, float scale) {
    return min((unsigned)kBins - 1u, (unsigned)__fmul_rz(__uint2float_rz(w - lo), scale));
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_gpu(unsigned* p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Summary of the CTA lists gathered by the finisher.
struct ListSums {
    unsigned total;  // keys in the union
    unsigned lo, hi; // lowest and highest score word
    u64 xm;          // largest last key of a full list (0: no list is full)
};

// The finisher (the first CTA to publish) loads every CTA's list into shared memory (rows LP keys
// apart) as each list's ready flag appears, so the loads overlap the other CTAs' scoring: thread c
// waits for CTA c's flag and loads its list, all lists in parallel. Every wait is bounded (about
// 1 s); returns false if a list never arrived.
template <bool kFast>
__device__ __forceinline__ bool finisher_load(const ScanLaunch& p, u64* cand, u64* xcand, unsigned LP, unsigned G,
                                              ListSums& out) {
    __shared__ unsigned s_lo[kWarps], s_hi[kWarps], s_n[kWarps], s_ok[kWarps];
    __shared__ u64 s_xm[kWarps];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const unsigned L = p.list_len;
    unsigned lo = 0xFFFFFFFFu, hi = 0u, cnt = 0u;
    u64 xm = 0ull;
    bool ok = true;
    for (unsigned c = tid; c < G; c += kThreads) {
        const unsigned* ready = p.ctl + kCtlReady + c;
        unsigned it = 0;
        while (ld_acquire_gpu(ready) == 0u) {
            if (++it > (1u << 20)) { ok = false; break; }
            if (it > 8) __nanosleep(64);
        }
        if (!ok) break;
        const uint4* src = reinterpret_cast<const uint4*>(p.cta_keys + c * 32);
        const uint4* xsrc = reinterpret_cast<const uint4*>(p.cta_xkeys + c * 32);
        const unsigned nv = (L + 1u) / 2u;  // 16-byte pairs of entries (the row holds 32 entries)
        for (unsigned h = 0; h < nv; h += 4u) {  // four 16-byte loads (8 keys) of each array in flight
            uint4 v[4], xv[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (h + j < nv) {
                    v[j] = __ldcg(src + h + j);
                    if (kFast) xv[j] = __ldcg(xsrc + h + j);
                }
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const unsigned e = 2u * (h + j);  // entry index of the pair's first key
                if (e < L) {
                    const u64 x0 = ((u64)v[j].y << 32) | v[j].x, x1 = ((u64)v[j].w << 32) | v[j].z;
                    cand[c * LP + e] = x0;
                    if (kFast) xcand[c * LP + e] = ((u64)xv[j].y << 32) | xv[j].x;
                    if (x0) { lo = min(lo, (unsigned)(x0 >> 32)); hi = max(hi, (unsigned)(x0 >> 32)); ++cnt; }
                    if (e == L - 1u) xm = x0 > xm ? x0 : xm;  // the list's last key
                    if (e + 1u < L) {
                        cand[c * LP + e + 1] = x1;
                        if (kFast) xcand[c * LP + e + 1] = ((u64)xv[j].w << 32) | xv[j].z;
                        if (x1) { lo = min(lo, (unsigned)(x1 >> 32)); hi = max(hi, (unsigned)(x1 >> 32)); ++cnt; }
                        if (e + 1u == L - 1u) xm = x1 > xm ? x1 : xm;
                    }
                }
            }
        }
    }
    lo = __reduce_min_sync(kFull, lo);
    hi = __reduce_max_sync(kFull, hi);
    cnt = __reduce_add_sync(kFull, cnt);
    const bool wok = __all_sync(kFull, ok);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const u64 y = __shfl_xor_sync(kFull, xm, o);
        xm = y > xm ? y : xm;
    }
    if (lane == 0) {
        s_lo[warp] = lo;
        s_hi[warp] = hi;
        s_n[warp] = cnt;
        s_xm[warp] = xm;
        s_ok[warp] = wok ? 1u : 0u;
    }
    __syncthreads();
    out.total = 0;
    out.lo = 0xFFFFFFFFu;
    out.hi = 0u;
    out.xm = 0ull;
    bool all = true;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
        out.total += s_n[w];
        out.lo = min(out.lo, s_lo[w]);
        out.hi = max(out.hi, s_hi[w]);
        out.xm = s_xm[w] > out.xm ? s_xm[w] : out.xm;
        all = all && s_ok[w] != 0u;
    }
    return all;
}

// The finisher's ranking, every list in shared memory. The lists' union holds the top k unless a
// full list dropped a member: a list may have dropped one only if it is full and the slots it
// dropped could still rank below k. Exact mode: its last key ranks below k. Fast mode: a dropped
// slot's exact score is at most last + E and a top-k slot's exact score is at least F_k - E, so
// the lists are safe when at least k keys score above F(x_max) + 4E, x_max being the largest last
// key of a full list (ranks fall as keys grow, so it decides for all lists). In that (clean) case
// the keys whose fast score is at least F_k - 2E (F_k: the k-th largest fast score of the union)
// hold the top k by exact key, and they all score above x_max. The CTA locates F_k's bin in a
// histogram of the score words above x_max, gathers the exact keys of the keys whose score raised
// by 2E reaches that bin, and ranks each gathered key by counting the larger ones; the first k go to
// the outputs in rank order. Exact mode (E = 0, exact keys = scan keys) takes the same path. Returns
// false, having written no output, when the union may miss a top-k member or more than `cap` keys
// pass the gather; the caller then reselects.
template <bool kFast>
__device__ __forceinline__ bool finish_rank(const ScanLaunch& p, uint64_t* out_ids, float* out_scores,
                                            uint32_t* out_count, const u64* cand, const u64* xcand, unsigned LP,
                                            unsigned G, float E, const ListSums& ls, unsigned* hist, u64* gath,
                                            unsigned cap, unsigned* s_misc) {
    __shared__ unsigned s_a[kWarps], s_n[kWarps];
    __shared__ unsigned s_b;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const unsigned L = p.list_len, k = p.k, n = G * L, lsh = (unsigned)(__ffs((int)L) - 1);
    const unsigned total = ls.total;
    if (total == 0u) {  // nothing live
        if (tid == 0) *out_count = 0u;
        return true;
    }
    const u64 xm = ls.xm;
    const u64 probe = kFast ? probe_above(__fadd_ru(key_score(xm), 4.0f * E)) : xm;
    const unsigned base = xm ? (unsigned)(xm >> 32) : ls.lo;  // the histogram covers [base, hi]
    const float scale = __fdiv_rz((float)kBins, __fadd_ru(__uint2float_ru(ls.hi - base), 1.0f));
    for (unsigned i = tid; i < (unsigned)kBins; i += kThreads) hist[i] = 0u;
    if (tid == 0) s_misc[1] = 0u;
    __syncthreads();
    // the clean test and the histogram, one pass (four keys in flight per thread)
    unsigned above = 0;
    for (unsigned b0 = tid; b0 < n; b0 += 4u * kThreads) {
        u64 x[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const unsigned i = b0 + (unsigned)j * kThreads;
            x[j] = i < n ? cand[(i >> lsh) * LP + (i & (L - 1))] : 0ull;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const unsigned w = (unsigned)(x[j] >> 32);
            above += x[j] > probe ? 1u : 0u;
            if (x[j] != 0ull && w >= base && total > k) atomicAdd(&hist[bin_of(w, base, scale)], 1u);
        }
    }
    above = __reduce_add_sync(kFull, above);
    if (lane == 0) s_a[warp] = above;
    __syncthreads();
    above = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) above += s_a[w];
    if (xm != 0ull && above < k) return false;  // block-uniform
    unsigned bstar = 0;
    if (total > k) {
        // bin of the k-th largest key: descending scan, thread t owns bins kBins-1-4t .. kBins-4-4t
        unsigned c[4], lsum = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            c[j] = hist[kBins - 1 - 4 * tid - j];
            lsum += c[j];
        }
        unsigned incl = lsum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned y = __shfl_up_sync(kFull, incl, o);
            if (lane >= o) incl += y;
        }
        if (lane == 31) s_n[warp] = incl;
        __syncthreads();
        unsigned cum = incl - lsum;
        for (int w = 0; w < warp; ++w) cum += s_n[w];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (cum < k && k <= cum + c[j]) s_b = (unsigned)(kBins - 1 - 4 * tid - j);
            cum += c[j];
        }
        __syncthreads();
        bstar = s_b;
    }
    for (unsigned b0 = tid; b0 < n; b0 += 4u * kThreads) {  // four keys in flight per thread
        u64 x[4];
        unsigned at[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const unsigned i = b0 + (unsigned)j * kThreads;
            at[j] = (i >> lsh) * LP + (i & (L - 1));
            x[j] = i < n ? cand[at[j]] : 0ull;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            bool in = x[j] != 0ull;
            if (in && total > k) {
                const unsigned w2 = kFast ? score_word(__fadd_ru(key_score(x[j]), 2.0f * E)) : (unsigned)(x[j] >> 32);
                in = w2 >= base && bin_of(w2, base, scale) >= bstar;
            }
            if (in) {
                const unsigned pos = atomicAdd(&s_misc[1], 1u);
                if (pos < cap) gath[pos] = kFast ? xcand[at[j]] : x[j];
            }
        }
    }
    __syncthreads();
    const unsigned mc = s_misc[1];
    if (mc > cap) return false;  // block-uniform
    if (tid == 0) gath[mc] = 0ull;  // pad to an even count for the pair loads (gath holds cap + 2)
    __syncthreads();
    const ulonglong2* g2 = reinterpret_cast<const ulonglong2*>(gath);
    const unsigned np = (mc + 1u) / 2u;
    for (unsigned i = tid; i < mc; i += kThreads) {
        const u64 x = gath[i];
        unsigned r[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        unsigned j = 0;
        for (; j + 4u <= np; j += 4u) {  // every thread reads the same entries: broadcasts
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const ulonglong2 y = g2[j + q];
                r[2 * q] += y.x > x ? 1u : 0u;
                r[2 * q + 1] += y.y > x ? 1u : 0u;
            }
        }
        for (; j < np; ++j) {
            const ulonglong2 y = g2[j];
            r[0] += y.x > x ? 1u : 0u;
            r[1] += y.y > x ? 1u : 0u;
        }
        const unsigned rk = r[0] + r[1] + r[2] + r[3] + r[4] + r[5] + r[6] + r[7];
        if (rk < k) {
            const uint32_t ord = key_ordinal(x);
            out_ids[rk] = ((uint64_t)(p.block_id_base + (ord >> 6)) << 16) | (uint64_t)(ord & 63u);
            out_scores[rk] = key_score(x);
        }
    }
    if (tid == 0) *out_count = min(total, k);
    return true;
}

// The finisher's last act when the caller waits on a completion word (p.out_flag, typically in
// pinned host memory): every thread's output stores, then the word, at system scope.
__device__ __forceinline__ void signal_done(const ScanLaunch& p) {
    if (!p.out_flag) return;
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p.out_flag), "r"(p.out_flag_val) : "memory");
}

// Returns false only when the launch left without touching its scratch (the scratch stayed busy).
// `query` (fused launches): the query's dims floats, in global or kernel-parameter memory.
template <int MODE, bool FUSED, bool QPARAM = false>
__device__ __forceinline__ bool scan_body(const ScanLaunch& p, const float* query) {
    constexpr bool kFast = MODE == MRL_MODE_FAST;
    __shared__ __align__(16) int s_tab[kTabInts];
    // fast mode: the exact-mode tables too, for the exact rescoring of the CTA's list
    __shared__ __align__(16) float s_xtab[kFast ? kTabBw3 + kPrefix : 1];
    __shared__ float2 s_rho[256];
    __shared__ u64 s_cta_tau;
    __shared__ unsigned s_seed_min, s_seed_cnt;
    __shared__ unsigned s_next;  // the CTA's next page of its range
    __shared__ unsigned s_nflag;
    __shared__ unsigned s_last;
    __shared__ int s_ok;
    __shared__ SelState s_sel;
    __shared__ unsigned s_misc[4];
    __shared__ float s_E;
    extern __shared__ __align__(16) unsigned char s_dyn[];
    u64* s_queue = reinterpret_cast<u64*>(s_dyn);  // kWarps * kQueue
    u64* s_lists = s_queue + kWarps * kQueue;       // kWarps * 32
    u64* s_cand = s_lists + kWarps * 32;            // G * 33: scan keys of every CTA list
    const unsigned G = gridDim.x;
    u64* s_xcand = s_cand + G * 33;                 // G * 33: their exact keys (fast mode)
    u64* s_gath = s_xcand + (kFast ? G * 33 : 0);   // 2 * pow2 >= k
    unsigned P2 = 1;
    while (P2 < p.k) P2 <<= 1;
    const unsigned gath_cap = 2u * P2;
    unsigned* s_hist = reinterpret_cast<unsigned*>(s_gath + gath_cap + 2);  // kBins
    unsigned* s_flags = s_hist + kBins;                          // G

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // The plan of an unfused launch may come from the launch before (a fused scan's stored plan),
    // which may still be finishing under programmatic dependent launch: wait for it first.
    if (!FUSED) asm volatile("griddepcontrol.wait;" ::: "memory");
    // Programmatic dependent launch: the next launch on the stream may start now; its CTAs take the
    // SMs this launch's CTAs leave as they publish. It touches its scratch (the other parity) only
    // once the launch that used that scratch before has released it (p.done), and its outputs only
    // after this launch has completed (griddepcontrol.wait in its finisher).
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const unsigned L = p.list_len;
    unsigned* counter = p.ctl;
    const int* xtab = kFast ? reinterpret_cast<const int*>(s_xtab) : s_tab;

    // fused plan build: its inputs first, so they are not queued behind the page loads
    DevPlan* ps = reinterpret_cast<DevPlan*>(s_dyn);
    float* s_qb = reinterpret_cast<float*>(s_dyn + align16(sizeof(DevPlan)));
    planb::PlanShared* s_pb =
        reinterpret_cast<planb::PlanShared*>(s_dyn + align16(sizeof(DevPlan)) + align16((size_t)p.dims * sizeof(float)));
    if (FUSED) planb::plan_inputs<QPARAM>(query, p.dims, p.eden_mean, p.mid_mean, p.eden_seed, p.mid_seed, s_qb, *s_pb);
    float4 mm = make_float4(0.f, 0.f, 0.f, 0.f);
    if (kFast) mm = __ldg(reinterpret_cast<const float4*>(p.metamax));

    // Page schedule: the first 7/8 of the pages are split into one contiguous range per CTA, whose
    // warps take pages from a shared-memory counter (the first two per warp static); the last 1/8
    // is a pool handed out one page at a time from the global counter to CTAs that have finished
    // their range, which evens out the finishing times. Global atomics are thus rare, and one
    // page's grab is issued a page ahead so its latency overlaps the scoring.
    const uint32_t n_pool = p.n_blocks / 8u, n_static = p.n_blocks - n_pool;
    const uint32_t lo_c = (uint32_t)(((uint64_t)n_static * blockIdx.x) / G);
    const uint32_t hi_c = (uint32_t)(((uint64_t)n_static * (blockIdx.x + 1)) / G);
    auto grab = [&](uint32_t g) -> uint32_t {  // lane 0: a page from the range, else from the pool
        if (g < hi_c) return g;
        return n_static + atomicAdd(counter, 1u);
    };
    // The warps' first two pages come from the CTA's own range when it has them (no scratch is
    // touched before the scratch wait below), else from the pool after that wait.
    const uint32_t none = 0xFFFFFFFFu;
    uint32_t b = lo_c + (uint32_t)warp < hi_c ? lo_c + (uint32_t)warp : none;
    uint32_t bn = lo_c + (uint32_t)(kWarps + warp) < hi_c ? lo_c + (uint32_t)(kWarps + warp) : none;
    // first page in flight before the tables are read
    Slot4 a0, a1;
    if (b != none) { load_slot(p.pages, b, lane, a0); load_slot(p.pages, b, lane + 32, a1); }

    Scalars S;
    if (tid == 0) {
        s_cta_tau = 0ull; s_seed_min = 0xFFFFFFFFu; s_seed_cnt = 0u; s_nflag = 0u;
        s_next = lo_c + 2u * kWarps;
    }
    const DevPlan* plan = p.plan;
    bool built = false;  // the tables are in shared memory already
    if (FUSED) {
        // QueryPipeline::build_plan fused into the scan (src/pipeline.rs:63-74): every CTA builds the
        // plan in shared memory while its first pages are in flight; no CTA waits on another.
        // CTA 0 stores the complete plan; the others build only what this mode scans with (fast
        // mode also needs the exact-mode prefix products for the rescoring of its list), writing
        // the tables straight into the scan's shared-memory tables
        const bool full = blockIdx.x == 0 && p.plan_out;
        const uint32_t need = full ? planb::kNeedAll
                                   : (kFast ? planb::kNeedFast | planb::kNeedExact | (p.depth == MRL_DEPTH_L0 ? planb::kNeedL0 : 0u)
                                            : planb::kNeedExact);
        float* xt = kFast ? s_xtab : reinterpret_cast<float*>(s_tab);
        const planb::PlanDest dst =
            full ? planb::plan_dest(ps)
                 : planb::PlanDest{s_tab, s_tab + kTabS1, s_tab + kTabS4, s_tab + kTabL0, xt, xt + kTabMidW, xt + kTabTailW,
                                   xt + kTabBw3};
        planb::build_plan(p.dims, p.prefix_codec, p.mid_codec, ps, s_qb, *s_pb, need, dst, s_rho);
        __syncthreads();
        if (full) {  // keep the plan for mrl_plan_read and later scans
            const uint4* src = reinterpret_cast<const uint4*>(ps);
            uint4* out = reinterpret_cast<uint4*>(p.plan_out);
            for (unsigned i = tid; i < sizeof(DevPlan) / 16; i += kThreads) out[i] = src[i];
        }
        plan = ps;
        built = !full;
    }
    if (!built) {
        copy_tables(plan, MODE, s_tab, p);
        if constexpr (kFast) load_exact_tables(plan, s_xtab);
    }
    if (!FUSED) fill_rho_tab(s_rho, tid, kThreads);  // the fused build fills it with otherwise idle warps
    fill_scalars(plan, p.w_s4, p.depth, (int32_t)(p.list_len != 0u), S);  // one: 1 for every launch, opaque to the compiler
    // bound on |fast score - exact score| of every slot of this segment (0 in exact mode), by one
    // thread (double-precision arithmetic)
    if (kFast && tid == 0) s_E = fast_error_bound(*plan, mm, p.w_s4, p.depth);
    // This launch's scratch (page counter, lists, ready flags, owner) is free once the launch that
    // used it before has released it (*done == done_prev); normally it has long before. Bounded
    // (about 1 s).
    if (p.done && tid == 0) {
        unsigned it = 0;
        int ok = 1;
        while (ld_acquire_gpu(p.done) != p.done_prev) {
            if (++it > (1u << 20)) { ok = 0; break; }
            if (it > 8) __nanosleep(128);
        }
        s_ok = ok;
    }
    __syncthreads();
    if (p.done && !s_ok) {
        if (tid == 0 && p.out_status) *p.out_status = 8u;  // the scratch stayed busy: no result
        return false;
    }
    const float E = kFast ? s_E : 0.0f;
    {
        const bool b_static = b != none;  // warp-uniform
        if (lane == 0) {  // pool pages for warps whose range had none left
            if (b == none) b = n_static + atomicAdd(counter, 1u);
            if (bn == none) bn = n_static + atomicAdd(counter, 1u);
        }
        b = __shfl_sync(kFull, b, 0);
        bn = __shfl_sync(kFull, bn, 0);
        if (!b_static && b < p.n_blocks) { load_slot(p.pages, b, lane, a0); load_slot(p.pages, b, lane + 32, a1); }
    }

    WarpSel ws{0ull, 0u, 0};
    u64* q = s_queue + warp * kQueue;
    bool first = true;
    while (b < p.n_blocks) {
        Slot4 n0, n1;
        if (bn < p.n_blocks) { load_slot(p.pages, bn, lane, n0); load_slot(p.pages, bn, lane + 32, n1); }
        const bool more = bn < p.n_blocks;  // warp-uniform
        uint32_t grabbed = 0;
        if (more && lane == 0) grabbed = grab(atomicAdd(&s_next, 1u));
        u64 k0 = 0ull, k1 = 0ull;
        if (block_live(p, b)) {
            k0 = slot_key<MODE>(a0, b * 64 + lane, s_tab, s_rho, S);
            k1 = slot_key<MODE>(a1, b * 64 + lane + 32, s_tab, s_rho, S);
        }
        if (lane == 0) p.owner[b] = (uint8_t)blockIdx.x;
        if (first) {
            // Seed the CTA bound: each warp's best first-page key certifies one distinct key, so
            // once all warps report, the smallest of their score words bounds the CTA's
            // list_len-th key from below (list_len <= kWarps).
            first = false;
            const unsigned wmax = __reduce_max_sync(kFull, max((unsigned)(k0 >> 32), (unsigned)(k1 >> 32)));
            if (lane == 0 && L <= (uint32_t)kWarps) {
                atomicMin(&s_seed_min, wmax);
                __threadfence_block();
                if (atomicAdd(&s_seed_cnt, 1u) == (unsigned)kWarps - 1u) {
                    const unsigned m = atomicMin(&s_seed_min, 0xFFFFFFFFu);
                    if (m) atomicMax(&s_cta_tau, (u64)m << 32);
                }
            }
        }
        warp_offer(ws, q, lane, L, &s_cta_tau, k0, k1);
        const uint32_t bnn = more ? __shfl_sync(kFull, grabbed, 0) : bn;
        b = bn;
        bn = bnn;
        a0 = n0;
        a1 = n1;
    }
    if (ws.qn) warp_flush(ws, q, lane, L, &s_cta_tau);

    // CTA top-list_len from the warps' lists: pairwise tree merge
    s_lists[warp * 32 + lane] = ws.list;
    __syncthreads();
    for (int half = kWarps / 2; half >= 1; half >>= 1) {
        if (warp < half) {
            const u64 m = warp_merge32(s_lists[warp * 32 + lane], s_lists[(warp + half) * 32 + lane], lane);
            __syncwarp();
            s_lists[warp * 32 + lane] = m;
        }
        __syncthreads();
    }
    if (warp == 0) {
        // publish the CTA's list; fast mode also rescores each entry in the reference's exact f32
        // order (src/scan.rs:453-634) and publishes that key beside it
        const u64 fk = (uint32_t)lane < L ? s_lists[lane] : 0ull;
        u64 xk = fk;
        if (kFast && fk != 0ull) {
            const uint32_t ord = key_ordinal(fk);
            Slot4 sl;
            load_slot(p.pages, ord >> 6, (int)(ord & 63u), sl);
            xk = slot_key<MRL_MODE_EXACT>(sl, ord, xtab, s_rho, S);
        }
        p.cta_keys[blockIdx.x * 32 + lane] = fk;
        if (kFast) p.cta_xkeys[blockIdx.x * 32 + lane] = xk;
        __threadfence();
        __syncwarp();
        if (lane == 0) st_release_gpu(p.ctl + kCtlReady + blockIdx.x, 1u);  // this CTA's list is out
    }
    // Publish ticket (control word 1): the first CTA to publish its list (ticket 0) finishes the
    // query; the others leave, and their SMs take the next launch's CTAs.
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(p.ctl + 1, 1u) == 0u ? 1u : 0u;
    __syncthreads();
    if (!s_last) return true;
    // Wait until the previous launch on the stream has completed: its finisher may still be writing
    // its query's result into the same outputs. With the exchange, this rank's ranking goes to its
    // own staged record first and the wait comes before the exchange (xch_publish_and_merge).
    if (!p.xch_world) asm volatile("griddepcontrol.wait;" ::: "memory");
    const unsigned LP = L | 1u;
    ListSums ls;
    if (!finisher_load<kFast>(p, s_cand, s_xcand, LP, G, ls)) {
        asm volatile("griddepcontrol.wait;" ::: "memory");  // (a no-op when it has returned before)
        if (tid == 0 && p.out_status) *p.out_status = 2u;  // a CTA's list never arrived: no result
        signal_done(p);
        return true;
    }

    // outputs: the caller's, or this rank's staged record of the NVLink exchange
    uint64_t* o_ids = p.out_ids;
    float* o_scores = p.out_scores;
    uint32_t* o_count = p.out_count;
    if (p.xch_world) {
        unsigned char* rec = p.xch_stage;
        o_ids = reinterpret_cast<uint64_t*>(rec);
        o_scores = reinterpret_cast<float*>(rec + (size_t)p.k * 8);
        o_count = reinterpret_cast<uint32_t*>(rec + (size_t)p.k * 12);
    }
    if (finish_rank<kFast>(p, o_ids, o_scores, o_count, s_cand, kFast ? s_xcand : s_cand, LP, G, E, ls, s_hist, s_gath,
                           gath_cap, s_misc)) {
        if (p.xch_world) {
            __threadfence();  // the record (stored by every thread) before its copies to the peers
            xch_publish_and_merge(p, s_dyn, &s_ok, 0u);
            signal_done(p);
        } else {
            if (tid == 0 && p.out_status) *p.out_status = 0u;
            signal_done(p);
        }
        return true;
    }
    // Rare path: find the flagged lists (full, and dropped slots could rank below k), reselect by
    // exact key over the lists plus those CTAs' rescanned pages, and write the whole output.
    for (unsigned c = warp; c < G; c += kWarps) {
        const u64 lc = s_cand[c * LP + L - 1];
        if (lc == 0ull) continue;  // warp-uniform: list not full
        const u64 pr = kFast ? probe_above(__fadd_ru(key_score(lc), 4.0f * E)) : lc;
        unsigned r = 0;
        for (unsigned j = lane; j < G; j += 32) r += count_greater(s_cand + j * LP, L, pr);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) r += __shfl_xor_sync(kFull, r, o);
        if (lane == 0 && r < p.k) s_flags[atomicAdd(&s_nflag, 1u)] = c;
    }
    __syncthreads();
    ScanLaunch own = p;
    own.out_ids = o_ids;
    own.out_scores = o_scores;
    own.out_count = o_count;
    reselect<MODE>(own, s_tab, xtab, s_rho, S, s_cand, s_xcand, s_gath, s_hist, s_flags, s_nflag, &s_sel, s_misc);
    if (p.xch_world) {
        __threadfence();
        xch_publish_and_merge(p, s_dyn, &s_ok, 1u);
        signal_done(p);
        return true;
    }
    if (tid == 0 && p.out_status) *p.out_status = 1u;
    signal_done(p);
    return true;
}

// Exit ticket (control word 7): the last CTA to leave zeroes this launch's control words and
// ready flags, so the launch that next uses this scratch starts clean whichever path this one
// took, a wait that ran out included. The ticket is an acquire-release add: every CTA's uses of
// the words come before its ticket, and the last holder sees them all before it stores the zeros,
// which the next launch on this scratch sees at the kernel boundary.
__device__ __forceinline__ void scan_exit(const ScanLaunch& p);

template <int MODE, bool FUSED>
__global__ void __launch_bounds__(kThreads, 1) scan_kernel(const ScanLaunch p) {
    if (!scan_body<MODE, FUSED>(p, p.query)) return;  // the scratch stayed busy: leave it untouched
    scan_exit(p);
}

// The fused scan of one query passed in the launch's parameters (host queries: no copy precedes
// the launch, so consecutive launches on a stream still overlap).
struct __align__(16) QueryParam {
    float q[kInlineQueryMax];
};
template <int MODE>
__global__ void __launch_bounds__(kThreads, 1) scan_kernel_q(const ScanLaunch p, const __grid_constant__ QueryParam qp) {
    if (!scan_body<MODE, true, true>(p, qp.q)) return;
    scan_exit(p);
}

__device__ __forceinline__ void scan_exit(const ScanLaunch& p) {
    __shared__ unsigned s_exit;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned before;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(before) : "l"(p.ctl + 7) : "memory");
        s_exit = before == gridDim.x - 1 ? 1u : 0u;
    }
    __syncthreads();
    if (s_exit) {
        for (unsigned i = threadIdx.x; i < (unsigned)kCtlWords; i += blockDim.x) p.ctl[i] = 0u;
        __syncthreads();
        if (threadIdx.x == 0 && p.done) {  // the scratch is free for the launch after next
            __threadfence();
            st_release_gpu(p.done, p.seq);
        }
    }
}

// ---- ScanStats (src/scan.rs:269-302, 654-799) ----------------------------------------------------
// The reference counts, per block scanned, its active vectors and the survivors of each stage,
// every stage pruning against the shortlist threshold tau at block entry with its Cauchy-Schwarz
// bounds scaled by cs_tolerance. Its serial scan raises tau block by block, so its counts depend on
// the scan order. The device counts every block against one tau: the shortlist's final threshold
// (src/scan.rs:396-399: the k-th score once the list is full, else the floor, -inf), which is the
// threshold every block would see if the scan were fully warmed. The stage values and the bounds
// are the reference's f32 expressions in its order (exact-mode tables), so the counts are exact.
struct StatsTotals {
    unsigned long long blocks, active_vecs, after_prefix, after_s1, after_s4_budget, pushed;
};

// Survivor bits of one slot after the prefix (bit 0), mid-band + CS-tail (bit 1) and S4 budget
// (bit 2) stages; 0 when tombstoned. `act` receives whether the slot is active.
__device__ __forceinline__ uint32_t stats_slot(const Slot4& sl, const float* ft, const float2* rho_tab,
                                               const Scalars& S, const DevPlan& P, float alpha, float tau,
                                               bool& act) {
    const SlotMeta m = slot_meta_tab(sl.c3.z, sl.c3.w, rho_tab);
    act = !m.tomb;
    if (m.tomb) return 0u;
    const uint32_t w[8] = {sl.c0.x, sl.c0.y, sl.c0.z, sl.c0.w, sl.c1.x, sl.c1.y, sl.c1.z, sl.c1.w};
    if (S.depth == MRL_DEPTH_L0) {  // src/scan.rs:753-790
        float acc = 0.0f;
#pragma unroll
        for (int d = 0; d < kPrefix; ++d)
            if ((w[d >> 3] >> (4 * (d & 7))) & 8u) acc = __fadd_rn(acc, ft[kTabBw3 + d]);
        const float ip = __fadd_rn(__fmul_rn(acc, m.scale), __fmul_rn(m.offset, S.prefix_sum));
        const float x_rest = fmaxf(__half2float(__ushort_as_half((unsigned short)(sl.c3.w & 0xFFFFu))), 0.0f);
        const float ub = __fadd_rn(ip, __fmul_rn(__fmul_rn(alpha, P.qp.q_after_prefix), x_rest));
        return ub >= tau ? 7u : 0u;
    }
    float acc = 0.0f;  // src/scan.rs:456-505
#pragma unroll
    for (int d = 0; d < kPrefix; ++d) acc = __fadd_rn(acc, ft[d * 16 + ((w[d >> 3] >> (4 * (d & 7))) & 15u)]);
    float sc = S.eden ? __fadd_rn(S.eden_mean_ip, __fmul_rn(m.scale, acc))
                      : __fadd_rn(__fmul_rn(acc, m.scale), __fmul_rn(m.offset, S.prefix_sum));
    const float ub0 = __fadd_rn(sc, __fmul_rn(alpha, __fadd_rn(__fmul_rn(P.qp.q_mid_norm, m.mid_n),
                                                            __fmul_rn(P.qp.q_tail_norm, m.high_n))));  // :508-514
    uint32_t bits = ub0 >= tau ? 1u : 0u;
    if (!bits) return 0u;
    if (S.depth >= MRL_DEPTH_L1) {  // src/scan.rs:520-584
        const uint32_t b1[4] = {sl.c2.x, sl.c2.y, sl.c2.z, sl.c2.w};
        float v = S.mid_base;
#pragma unroll
        for (int d = 0; d < kRabitq; ++d)
            if ((b1[d >> 5] >> (d & 31)) & 1u) v = __fadd_rn(v, ft[kTabMidW + d]);
        if (S.mid_b1) sc = __fadd_rn(sc, __fadd_rn(S.mid_mean_ip, __fmul_rn(m.offset, v)));
        else sc = __fadd_rn(sc, __fmul_rn(v, m.mid_n));
        const float ub1 = __fadd_rn(sc, __fmul_rn(__fmul_rn(alpha, P.qp.q_after_s1), m.high_n));
        if (!(ub1 >= tau)) return bits;
    }
    bits |= 2u;
    if (S.depth == MRL_DEPTH_FULL && P.qp.has_tail_fold && P.qp.s4_abs_budget > 0.0f) {  // :587-607
        const float ub2 = __fadd_rn(sc, __fmul_rn(__fmul_rn(__fmul_rn(alpha, fmaxf(m.high_n, 1e-6f)), S.w_s4),
                                                  P.qp.s4_abs_budget));
        if (!(ub2 >= tau)) return bits;
    }
    return bits | 4u;
}

// One warp per page (two slots per lane); tau from the scan's own results: the k-th score when it
// returned k hits, else -inf.
__global__ void __launch_bounds__(kThreads) stats_kernel(const ScanLaunch p, float alpha, const uint32_t* count,
                                                         const float* scores, StatsTotals* tot) {
    __shared__ __align__(16) float s_ft[kTabBw3 + kPrefix];
    __shared__ float2 s_rho[256];
    __shared__ unsigned long long s_tot[6];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const DevPlan& P = *p.plan;
    load_exact_tables(p.plan, s_ft);
    fill_rho_tab(s_rho, tid, kThreads);
    Scalars S;
    fill_scalars(p.plan, p.w_s4, p.depth, 1, S);
    if (tid < 6) s_tot[tid] = 0ull;
    __syncthreads();
    const uint32_t n = *count;
    const float tau = n >= p.k && n > 0 ? scores[p.k - 1] : -INFINITY;
    unsigned long long c[6] = {0, 0, 0, 0, 0, 0};
    for (uint32_t b = blockIdx.x * kWarps + warp; b < p.n_blocks; b += gridDim.x * kWarps) {
        if (!block_live(p, b)) continue;  // warp-uniform
        Slot4 s0, s1;
        load_slot(p.pages, b, lane, s0);
        load_slot(p.pages, b, lane + 32, s1);
        bool a0, a1;
        const uint32_t m0 = stats_slot(s0, s_ft, s_rho, S, P, alpha, tau, a0);
        const uint32_t m1 = stats_slot(s1, s_ft, s_rho, S, P, alpha, tau, a1);
        const unsigned act = __popc(__ballot_sync(kFull, a0)) + __popc(__ballot_sync(kFull, a1));
        if (act == 0u) continue;
        c[0] += 1;
        c[1] += act;
        c[2] += __popc(__ballot_sync(kFull, m0 & 1u)) + __popc(__ballot_sync(kFull, m1 & 1u));
        c[3] += __popc(__ballot_sync(kFull, m0 & 2u)) + __popc(__ballot_sync(kFull, m1 & 2u));
        c[4] += __popc(__ballot_sync(kFull, m0 & 4u)) + __popc(__ballot_sync(kFull, m1 & 4u));
    }
    c[5] = c[4];  // the tail-fold stage adds to scores but prunes nothing: its survivors are pushed
    if (lane == 0)
        for (int i = 0; i < 6; ++i)
            if (c[i]) atomicAdd(&s_tot[i], c[i]);
    __syncthreads();
    if (tid < 6 && s_tot[tid]) atomicAdd(reinterpret_cast<unsigned long long*>(tot) + tid, s_tot[tid]);
}

template <int MODE>
__global__ void __launch_bounds__(kThreads) debug_scores_kernel(const ScanLaunch p, float* out,
                                                                uint8_t* active, int32_t* parts) {
    __shared__ __align__(16) int s_tab[kTabInts];
    __shared__ float2 s_rho[256];
    Scalars S;
    load_tables(p.plan, MODE, s_tab, s_rho, S, p);
    __syncthreads();
    const uint32_t total = p.n_blocks * 64u;
    for (uint32_t i = blockIdx.x * kThreads + threadIdx.x; i < total; i += gridDim.x * kThreads) {
        const uint32_t b = i >> 6, v = i & 63u;
        Slot4 s;
        load_slot(p.pages, b, (int)v, s);
        float sc = 0.0f;
        Partials pr{0, 0, 0};
        bool ok = block_live(p, b) &&
                  slot_score<MODE>(s.c0, s.c1, s.c2, s.c3, s_tab, s_rho, S, sc, MODE == MRL_MODE_FAST ? &pr : nullptr);
        out[i] = ok ? sc : 0.0f;
        active[i] = ok ? 1 : 0;
        if (parts) {
            parts[3 * (size_t)i] = ok ? pr.p : 0;
            parts[3 * (size_t)i + 1] = ok ? pr.s1 : 0;
            parts[3 * (size_t)i + 2] = ok ? pr.s4 : 0;
        }
    }
}

__global__ void score_bound_kernel(const DevPlan* __restrict__ plan, const float* __restrict__ metamax, float w_s4,
                                   uint32_t depth, float* out) {
    if (threadIdx.x == 0)
        *out = fast_error_bound(*plan, *reinterpret_cast<const float4*>(metamax), w_s4, depth);
}

}  // namespace

int launch_score_bound(const ScanLaunch& p, float* d_out, cudaStream_t stream) {
    score_bound_kernel<<<1, 32, 0, stream>>>(p.plan, p.metamax, p.w_s4, p.depth, d_out);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int scan_ctas(int device_sms) { return device_sms; }

// Shared memory of the exchange merge: the world's records, plus room for the merge tree's first
// level (ceil(world / 2) records) when that stays within kXchTreeBytes; else the records alone and
// the one-level merge.
constexpr size_t kXchTreeBytes = 200 * 1024;
bool xch_use_tree(uint32_t world, uint32_t k) {
    return (size_t)(world + (world + 1) / 2) * MRL_MERGE_RECORD_BYTES(k) <= kXchTreeBytes;
}
size_t xch_merge_bytes(uint32_t world, uint32_t k) {
    return (size_t)(xch_use_tree(world, k) ? world + (world + 1) / 2 : world) * MRL_MERGE_RECORD_BYTES(k);
}

size_t scan_smem_bytes(uint32_t ctas, uint32_t k, uint32_t fused_dims, uint32_t xch_world, uint32_t mode) {
    size_t p2 = 1;
    while (p2 < k) p2 <<= 1;
    const size_t lists = (size_t)ctas * 33 * (mode == MRL_MODE_FAST ? 2 : 1);  // scan keys (+ exact keys)
    size_t bytes = sizeof(u64) * (kWarps * kQueue + kWarps * 32 + lists + 2 * p2 + 2) + sizeof(unsigned) * (kBins + ctas);
    if (fused_dims) bytes = std::max(bytes, fused_plan_bytes(fused_dims));
    if (xch_world) bytes = std::max(bytes, xch_merge_bytes(xch_world, k));  // records to merge
    return bytes;
}

// One CTA per SM. With `pdl` the launch may begin while the previous kernel on the stream finishes
// (programmatic dependent launch; the kernel waits for it before touching what they share). With
// `h_query` (host memory, p.dims <= kInlineQueryMax floats) the fused scan takes the query in its
// launch parameters.
int launch_scan(const ScanLaunch& p, uint32_t ctas, cudaStream_t stream, bool pdl, const float* h_query) {
    const bool fused = p.query != nullptr || h_query != nullptr;
    if (h_query && p.dims > kInlineQueryMax) return -1;
    const size_t smem = scan_smem_bytes(ctas, p.k, fused ? p.dims : 0u, p.xch_world, p.mode);
    const bool fast = p.mode == MRL_MODE_FAST;
    const void* fn = h_query ? (fast ? (const void*)scan_kernel_q<MRL_MODE_FAST> : (const void*)scan_kernel_q<MRL_MODE_EXACT>)
                   : fast ? (fused ? (const void*)scan_kernel<MRL_MODE_FAST, true> : (const void*)scan_kernel<MRL_MODE_FAST, false>)
                          : (fused ? (const void*)scan_kernel<MRL_MODE_EXACT, true> : (const void*)scan_kernel<MRL_MODE_EXACT, false>);
    // the attribute is per function and device: set it only when a launch needs more than before
    static std::atomic<size_t> set_bytes[64][6];
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return -1;
    std::atomic<size_t>& cur = set_bytes[device & 63][h_query ? 4 + (fast ? 0 : 1) : (fast ? 0 : 2) + (fused ? 1 : 0)];
    if (smem > cur.load(std::memory_order_relaxed)) {
        if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return -1;
        cur.store(smem, std::memory_order_relaxed);
    }
    ScanLaunch arg = p;
    arg.xch_tree = p.xch_world && xch_use_tree(p.xch_world, p.k) ? 1u : 0u;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ctas);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (h_query) {
        QueryParam qp;
        std::memcpy(qp.q, h_query, sizeof(float) * p.dims);
        void* args[] = {&arg, &qp};
        return cudaLaunchKernelExC(&cfg, fn, args) == cudaSuccess ? 0 : -1;
    }
    void* args[] = {&arg};
    if (cudaLaunchKernelExC(&cfg, fn, args) != cudaSuccess) return -1;
    return 0;
}

int launch_scan_stats(const ScanLaunch& p, float cs_tolerance, const uint32_t* d_count, const float* d_scores,
                      unsigned long long* d_totals, cudaStream_t stream) {
    if (cudaMemsetAsync(d_totals, 0, sizeof(StatsTotals), stream) != cudaSuccess) return -1;
    const uint32_t grid = (uint32_t)std::max<uint64_t>(1, std::min<uint64_t>(((uint64_t)p.n_blocks + kWarps - 1) / kWarps,
                                                                            148u * 4u));
    stats_kernel<<<grid, kThreads, 0, stream>>>(p, cs_tolerance, d_count, d_scores,
                                                reinterpret_cast<StatsTotals*>(d_totals));
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int launch_debug_scores(const ScanLaunch& p, float* d_scores, uint8_t* d_active, int32_t* d_partials,
                        cudaStream_t stream) {
    const uint32_t total = p.n_blocks * 64u;
    const uint32_t grid = total ? (total + kThreads - 1) / kThreads : 1;
    if (p.mode == MRL_MODE_FAST)
        debug_scores_kernel<MRL_MODE_FAST><<<grid, kThreads, 0, stream>>>(p, d_scores, d_active, d_partials);
    else
        debug_scores_kernel<MRL_MODE_EXACT><<<grid, kThreads, 0, stream>>>(p, d_scores, d_active, d_partials);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace mrl
