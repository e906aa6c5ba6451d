// mrl_internal.cuh — shared device structures and helpers of libmrl_b200 (sm_100a).
//
// HBM scan layout ("vector-major pages"): each 4096-byte PaxBlock64 page (src/block.rs:130-144)
// is transcoded once at upload into four 1 KiB chunk planes; chunk c of slot v lives at byte
// c*1024 + v*16 of the page, so a warp reading 32 consecutive slots of one chunk issues 32
// contiguous 16-byte loads (512 B). Per slot (64 bytes, the same information as the page):
//   chunk 0: 4-bit prefix levels of dims 0..31  (word j, nibble i = level of dim 8j+i)
//   chunk 1: 4-bit prefix levels of dims 32..63
//   chunk 2: the 128 stratum-1 bits (word j bit i = dim 32j+i)
//   chunk 3: word 0/1 = the 64 stratum-4 bits; word 2 = f16 scale | f16 offset << 16;
//            word 3 = f16 tail_norm | rho flags << 16 | tombstone << 24
// Level bit order follows write_4bit_planes (src/quantize.rs:297-315): bit3 = stratum0,
// bit2 = stratum2, bit1 = stratum3, bit0 = stratum5. Block header timestamps go to a separate
// uint2 array [min_ts, max_ts] per page.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../../include/mrl_cuda.h"

namespace mrl {

constexpr int kVPB = 64;
constexpr int kBlockBytes = 4096;
constexpr int kPrefix = 64;
constexpr int kRabitq = 128;
constexpr int kTailStart = 192;
constexpr int kFold = 64;
constexpr int kFoldBlocks = 9;
constexpr int kS1Windows = 26;  // 5-dim windows over 128 mid-band bits (last one 3 dims)
constexpr int kS4Windows = 13;  // 5-dim windows over 64 folded-tail bits (last one 4 dims)

// PaxBlock64 field offsets (src/block.rs:31-144).
constexpr int kOffMinTs = 0, kOffMaxTs = 4, kOffSrc = 8, kOffTomb = 16, kOffCrc = 24;
constexpr int kOffMeta = 64, kOffS0 = 512, kOffS1 = 1024, kOffS2 = 2048, kOffS3 = 2560,
              kOffS4 = 3072, kOffS5 = 3584;

// Device-resident query plan: the reference QueryPlan plus the per-mode scoring tables.
struct DevPlan {
    mrl_query_plan qp;
    // fast mode: exact int32 stage sums of 2^shift-scaled table entries
    int32_t lut_prefix[kPrefix * 16];
    int32_t lut_s1[kS1Windows * 32];
    int32_t lut_s4[kS4Windows * 32];
    int32_t lut_l0[kPrefix * 16];  // L0Only: stratum-0 bit of each level times bit_weights[d][3]
    // the same stage sums over 4-dim windows (16 entries each), for the batched scan
    int32_t lut4_s1[(kRabitq / 4) * 16];
    int32_t lut4_s4[(kFold / 4) * 16];
    int32_t shift_prefix, shift_s1, shift_s4, shift_l0;
    double unscale_prefix, unscale_s1, unscale_s4, unscale_l0;  // 2^-shift
    // exact mode: f32 products and addends in reference order
    float fp_prefix[kPrefix * 16];
    float mid_w[kRabitq];   // Rabitq: rabitq_weights2; EdenB1: (c1 - c0) * q
    float tail_w[kFold];    // tail_fold_weights2
    float mid_base, tail_base;
    // upper bounds of sum over dims of max |entry| per stage (prefix, mid band, folded tail,
    // L0Only), rounded up: the magnitudes the fast/exact score difference bound scales with
    float err_p, err_1, err_4, err_0, pad2, pad3;
};
static_assert(sizeof(mrl_query_plan) % 16 == 0, "plan alignment");
static_assert(sizeof(DevPlan) % 16 == 0, "plan alignment");

// ---------------------------------------------------------------------------------------------
// Hashes shared with the reference: tail_rademacher (src/rotate.rs:53-67) and rademacher_diag
// (src/eden.rs:75-88) use the same SplitMix-style sign mix.
__host__ __device__ __forceinline__ float sign_hash(uint64_t a, uint64_t i) {
    uint64_t x = (a * 0x9E3779B97F4A7C15ULL + i) * 0xBF58476D1CE4E5B9ULL;
    x ^= x >> 30;
    x *= 0x94D049BB133111EBULL;
    x ^= x >> 27;
    return (x & 1u) == 0 ? 1.0f : -1.0f;
}

// SplitMix64 output function (Steele, Lea & Flood 2014), for the seeded synthetic inputs.
__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ULL;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ULL;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBULL;
    return x ^ (x >> 31);
}

// Irwin-Hall(12) - 6 from twelve 16-bit midpoint-lattice uniforms: variance 1, exact in f32, and
// free of transcendental functions so host and device produce identical values.
__host__ __device__ __forceinline__ float ih_gauss(uint64_t seed, uint64_t idx) {
    int64_t s = 0;
    for (uint64_t j = 0; j < 3; ++j) {
        const uint64_t h = splitmix64(seed * 0xD1B54A32D192ED03ULL + idx * 3 + j);
        s += (int64_t)(h & 0xFFFF) + (int64_t)((h >> 16) & 0xFFFF) + (int64_t)((h >> 32) & 0xFFFF) +
             (int64_t)(h >> 48);
    }
    const int32_t num = (int32_t)(2 * s + 12 - 786432);
    return (float)num * (1.0f / 131072.0f);
}

// Lloyd-Max N(0,1) centroids (src/eden.rs:15-44), b = 4. Device code copies them into shared
// memory once per CTA (a runtime-indexed local array would live on the stack).
__device__ const float g_lloyd_b4[16] = {-2.73258958f, -2.06901724f, -1.61804640f, -1.25623121f,
                                         -0.94234046f, -0.65675912f, -0.38804830f, -0.12839503f,
                                         0.12839503f,  0.38804830f,  0.65675912f,  0.94234046f,
                                         1.25623121f,  1.61804640f,  2.06901724f,  2.73258958f};
constexpr float kLloydB1Hi = 0.79788456f;

// Total order used by every selection stage: larger key = better hit. High word: the f32 score
// mapped to an order-preserving unsigned (zero canonicalised to +0); low word: the complement of
// the slot ordinal, so equal scores rank the lower (block, slot) first. Key 0 = no hit.
__device__ __forceinline__ unsigned long long make_key(float score, uint32_t ordinal) {
    uint32_t u = __float_as_uint(score);
    if (score == 0.0f) u = 0u;
    const uint32_t o = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)o << 32) | (unsigned long long)(0xFFFFFFFFu - ordinal);
}
__device__ __forceinline__ float key_score(unsigned long long k) {
    const uint32_t o = (uint32_t)(k >> 32);
    const uint32_t u = (o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o;
    return __uint_as_float(u);
}
__device__ __forceinline__ uint32_t key_ordinal(unsigned long long k) {
    return 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull);
}

// Per-slot rest statistics (VectorMeta::{mid_norm_f32, high_tail_norm_f32}, src/block.rs:60-90)
// with the scan's clamps (src/scan.rs:495-496).
struct SlotMeta {
    float scale, offset, mid_n, high_n;
    bool tomb;
};
__device__ __forceinline__ SlotMeta decode_slot_meta(uint32_t w2, uint32_t w3) {
    SlotMeta m;
    m.scale = __half2float(__ushort_as_half((unsigned short)(w2 & 0xFFFFu)));
    m.offset = __half2float(__ushort_as_half((unsigned short)(w2 >> 16)));
    const float tail = __half2float(__ushort_as_half((unsigned short)(w3 & 0xFFFFu)));
    const uint32_t flags = (w3 >> 16) & 0xFFu;
    m.tomb = ((w3 >> 24) & 1u) != 0;
    const float rho = __fdiv_rn((float)flags, 255.0f);
    const float t = fmaxf(tail, 0.0f);
    const float r = fminf(fmaxf(rho, 0.0f), 1.0f);
    const float mid = __fmul_rn(__fsqrt_rn(fmaxf(__fsub_rn(1.0f, __fmul_rn(r, r)), 0.0f)), t);
    const float high = __fmul_rn(rho, t);
    m.mid_n = fmaxf(mid, 1e-6f);
    m.high_n = fmaxf(high, 0.0f);
    return m;
}

// rho_ratio = flags / 255 and sqrt(max(1 - r^2, 0)) (src/block.rs:74-84) for every flags byte,
// filled by threads tid = 0 .. nthr-1.
__device__ __forceinline__ void fill_rho_tab(float2* rho_tab, int tid, int nthr) {
    for (int i = tid; i < 256; i += nthr) {
        const float rho = __fdiv_rn((float)i, 255.0f);
        const float r = fminf(fmaxf(rho, 0.0f), 1.0f);
        rho_tab[i] = make_float2(rho, __fsqrt_rn(fmaxf(__fsub_rn(1.0f, __fmul_rn(r, r)), 0.0f)));
    }
}

}  // namespace mrl

// Host-side launchers implemented in the .cu files, used by the C ABI layer.
namespace mrl {
struct Segment;
int launch_plan_build(const float* d_queries, uint32_t n_q, uint32_t dims, uint32_t prefix_codec,
                      uint32_t mid_codec, const float* d_eden_mean, uint64_t eden_seed,
                      const float* d_mid_mean, uint64_t mid_seed, DevPlan* d_plans,
                      cudaStream_t stream);
int launch_transcode(const uint8_t* d_pax, uint64_t n_blocks, uint4* d_pages, uint2* d_ts,
                     cudaStream_t stream);
// Merge into d_metamax[0..3] the maxima over pages [0, n_blocks) of the per-slot factors that scale
// the stage sums in a score: |scale|, |offset|, mid_n, max(high_n, 1e-6) (NaN counts as +inf).
int launch_metamax(const uint4* d_pages, uint64_t n_blocks, float* d_metamax, cudaStream_t stream);
int launch_encode(const float* d_rows, uint64_t n, uint32_t dims, const uint32_t* d_ts,
                  const uint32_t* d_src, uint32_t src_const, uint32_t prefix_codec,
                  const float* d_eden_mean, uint64_t eden_seed, const float* d_mid_mean,
                  uint64_t mid_seed, uint8_t* d_pax, uint4* d_pages, uint2* d_block_ts,
                  cudaStream_t stream);
int launch_eden_fit(const float* d_rows, uint64_t n, uint32_t dims, uint32_t start,
                    uint32_t width, float* d_mean, cudaStream_t stream);
int launch_synth_docs(uint64_t seed, uint64_t row0, uint64_t n, uint32_t dims, float* d_out,
                      cudaStream_t stream);
int launch_synth_queries(uint64_t doc_seed, uint64_t n_docs, uint64_t q_seed, uint64_t n_q,
                         uint32_t dims, float sigma, float* d_out, uint64_t* d_pick,
                         cudaStream_t stream);

constexpr int kMaxRanks = 8;  // NVLink exchange: ranks of one node

struct ScanLaunch {
    const uint4* pages;
    const uint2* block_ts;
    uint32_t n_blocks;
    uint32_t block_id_base;
    const DevPlan* plan;
    uint32_t k;
    uint32_t list_len;
    float w_s4;
    uint32_t depth;
    uint32_t mode;
    uint32_t use_time;  // temporal filter active for this call
    uint32_t has_lo, lo, has_hi, hi;
    // scratch (owned by the context, one set per launch parity: consecutive launches on a stream
    // may overlap; zero-initialised once, left zeroed by every launch)
    unsigned long long* cta_keys;  // ctas * 32: each CTA's exact top-list_len keys (scan order)
    unsigned long long* cta_xkeys; // ctas * 32: fast mode, the same entries' exact-mode keys
    unsigned int* ctl;             // kCtlWords: [0] page counter, [1] publish ticket, [7] exit ticket,
                                   // [kCtlReady + c] CTA c's list is published; the last CTA to
                                   // exit zeroes them all
    // completion word (nullptr: none): the finisher stores out_flag_val there, system scope, after
    // every output (for a host that waits on pinned, device-mapped outputs)
    unsigned int* out_flag;
    uint32_t out_flag_val;
    unsigned int* done;            // launch sequence number of the last launch to release this
                                   // scratch (nullptr: scratch of one launch at a time, no check)
    uint32_t seq;                  // this launch's sequence number on the context
    uint32_t done_prev;            // *done must hold this (the previous user's seq) before the
                                   // launch touches the scratch
    const float* metamax;          // the segment's 4 meta-factor maxima (launch_metamax)
    uint8_t* owner;                // n_blocks: CTA that scored each page
    uint64_t* out_ids;
    float* out_scores;
    uint32_t* out_count;
    uint32_t* out_status;
    // fused plan build (query != nullptr): every CTA builds the plan of `query` in shared memory
    // before scanning, and CTA 0 also stores it to plan_out
    const float* query;
    uint32_t dims, prefix_codec, mid_codec;
    const float* eden_mean;
    const float* mid_mean;
    uint64_t eden_seed, mid_seed;
    DevPlan* plan_out;
    // NVLink exchange (xch_world > 0), by pushes: every rank's area holds, per buffer parity
    // (xch_epoch & 1), one receive record and one flag word per sending rank. The finisher ranks
    // this rank's top-k into xch_stage (a record of this launch's scratch set, so it needs no
    // ordering against the previous launch), then, once the previous launch has completed, copies
    // it into its record slot in every rank's area (peer stores over NVLink for the others), raises
    // this rank's flag in every other area (release, system scope), waits (bounded) for the other
    // ranks' flags in its own area, and merges the records there, all in local memory, into out_*
    // (the global top-k)
    uint32_t xch_world, xch_rank, xch_epoch;
    uint32_t xch_tree;  // set by launch_scan: merge as a pairwise tree (room for its buffers)
    unsigned char* xch_rec[kMaxRanks];   // this rank's record slot in rank w's area (this parity)
    unsigned int* xch_flag[kMaxRanks];   // this rank's flag word in rank w's area (this parity)
    const unsigned char* xch_recv;       // this parity's receive records in this rank's area, by sender
    const unsigned int* xch_flag_in;     // this parity's flag words in this rank's area, by sender
    unsigned char* xch_stage;            // this rank's record of this launch, before its copies
};
int scan_ctas(int device_sms);
size_t scan_smem_bytes(uint32_t ctas, uint32_t k, uint32_t fused_dims, uint32_t xch_world, uint32_t mode);
// Longest query a launch can carry in its parameters (launch_scan's h_query).
constexpr uint32_t kInlineQueryMax = 1024;
int launch_scan(const ScanLaunch& p, uint32_t ctas, cudaStream_t stream, bool pdl, const float* h_query = nullptr);
int launch_exact_dots(const float* d_query, const float* d_rows, uint64_t n_rows, uint32_t dims, const uint64_t* d_sel,
                      uint32_t n, float* d_scores, uint32_t* d_bad, cudaStream_t stream);
int launch_ring_search_batch(const float* d_queries, uint32_t n_q, uint32_t dims, const float* d_rows, uint32_t n,
                             uint32_t slot_base, uint32_t k, void* d_records, cudaStream_t stream);
int launch_exact_rank(const float* d_scores, uint32_t n, const uint64_t* d_ids, uint64_t id_base, uint32_t keep,
                      uint64_t* d_out_ids, float* d_out_scores, uint32_t* d_out_count, cudaStream_t stream);
int launch_merge_topk(const void* d_lists, uint32_t n_lists, uint32_t stride, uint32_t k, uint64_t* d_out_ids,
                      float* d_out_scores, uint32_t* d_out_count, cudaStream_t stream);
int launch_pack_records(const uint64_t* d_ids, const float* d_scores, const uint32_t* d_counts, uint32_t n_q,
                        uint32_t k, void* d_records, cudaStream_t stream);
int launch_merge_topk_batch(const void* d_lists, uint32_t n_lists, uint32_t n_q, uint32_t stride, uint32_t k,
                            uint64_t* d_out_ids, float* d_out_scores, uint32_t* d_out_counts, cudaStream_t stream);
// Scan control words per launch: [0] page counter, [1] publish ticket, [7] exit ticket, then from
// kCtlReady one ready flag per CTA (at most kMaxScanCtas CTAs).
constexpr int kMaxScanCtas = 256;
constexpr int kCtlReady = 8;
constexpr int kCtlWords = kCtlReady + kMaxScanCtas;
// batched fast-mode scan (bscan.cu): per-(query, CTA) top-32 lists in `scratch`
// (batch_scratch_bytes), then one selection CTA per query
size_t batch_scratch_bytes(uint32_t ctas, uint32_t n_q);
int launch_scan_batch(const uint4* pages, const uint2* block_ts, uint32_t n_blocks, uint32_t block_id_base,
                      const float* metamax, const DevPlan* plans, uint32_t n_q, uint32_t k, float w_s4, uint32_t depth, uint32_t use_time,
                      uint32_t has_lo, uint32_t lo, uint32_t has_hi, uint32_t hi, uint32_t ctas, uint32_t engine,
                      void* scratch, uint64_t* out_ids, float* out_scores, uint32_t* out_counts, uint32_t* out_status,
                      cudaStream_t stream);
// The fast/exact score difference bound the scan uses for plan p.plan over the segment whose maxima
// are p.metamax (one float to d_out).
int launch_score_bound(const ScanLaunch& p, float* d_out, cudaStream_t stream);
// ScanStats counters (6 u64: blocks, active vectors, survivors after prefix / S1 / S4 budget,
// pushed) of plan p.plan over the segment, every block pruned against the final shortlist
// threshold of a scan whose count and scores (device, shortlist k = p.k) are given.
int launch_scan_stats(const ScanLaunch& p, float cs_tolerance, const uint32_t* d_count, const float* d_scores,
                      unsigned long long* d_totals, cudaStream_t stream);
int launch_debug_scores(const ScanLaunch& p, float* d_scores, uint8_t* d_active,
                        int32_t* d_partials, cudaStream_t stream);
}  // namespace mrl
