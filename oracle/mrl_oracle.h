/*
 * mrl_oracle.h — TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the reference crate `mrl_index` (v0.3.5) PaxBlock64 scan path, used as the
 * checker for the CUDA product library. Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline / reference arm may load this library. The product path never calls it.
 *
 * Parity status: PARTIALLY PINNED. The reference is Rust and no Rust toolchain exists in this
 * image, so the reference binary cannot be run. The restatement is pinned against every
 * known-answer value the reference's own tests hold for this path (Lloyd-Max tables, PaxBlock64
 * field offsets, ballot word order, FWHT norm preservation, the fold operator) plus the
 * standard CRC-32 check value and IEEE binary16 round-to-nearest-even; the reference ships no
 * golden scan scores or id lists, so end-to-end scan parity with the Rust binary is unpinned.
 *
 * All functions are plain C ABI over caller-owned buffers.
 */
#ifndef MRL_ORACLE_H
#define MRL_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Mirror of `QueryPlan` (src/scan.rs:19-71) field by field, plus the three enum/bool fields. */
typedef struct ora_query_plan {
    uint32_t dims;
    uint32_t prefix_codec; /* 0 = MinMax4, 1 = EdenProd (src/config.rs:8-16) */
    uint32_t mid_codec;    /* 0 = Rabitq, 1 = EdenB1 (src/config.rs:19-28) */
    uint32_t has_tail_fold;
    float prefix[64];
    float bit_weights[64][4];
    float rabitq_q[128];
    float rabitq_scale;
    float rabitq_weights2[128];
    float rabitq_base;
    float rabitq_lut[32][16];
    float tail_fold_q[64];
    float tail_fold_weights2[64];
    float tail_fold_base;
    float q_tail_norm;
    float q_mid_norm;
    float q_after_prefix;
    float q_after_s1;
    float s4_abs_budget;
    float prefix_l1;
    float prefix_sum;
    float eden_q_rot[64];
    float eden_mean_ip;
    float eden_inv_sqrt_d;
    float eden_codebook[16];
    float eden_mid_q_rot[128];
    float eden_mid_mean_ip;
    float eden_mid_inv_sqrt_d;
    float eden_mid_codebook[2];
} ora_query_plan;

/* Mirror of `ScanConfig` (src/config.rs:79-88). */
typedef struct ora_scan_cfg {
    uint32_t shortlist_cand;
    float cs_tolerance;
    float stratum4_weight;
    uint32_t strata_depth; /* 0 = L0Only, 1 = L1Rabitq, 2 = Full64b */
    uint32_t temporal_filter_enable;
    uint32_t numa_sharding;
} ora_scan_cfg;

/* Mirror of `ScanStats` (src/scan.rs:269-278). */
typedef struct ora_scan_stats {
    uint64_t blocks, active_vecs, after_prefix, after_s1, after_s4_budget, pushed;
} ora_scan_stats;

/* Fixed-point restatement used by the product's fast mode: every stage's inner product is an
 * exact int32 sum of table entries; tables are built from the f32 plan in double precision. */
typedef struct ora_fixed_plan {
    int32_t prefix_lut[64][16]; /* value of dim d at 4-bit level l, scaled by 2^prefix_shift */
    int32_t s1_lut[26][32];     /* 5-dim windows over the 128 mid-band bits (last window 3 dims) */
    int32_t s4_lut[13][32];     /* 5-dim windows over the 64 folded-tail bits (last window 4 dims) */
    int32_t prefix_shift, s1_shift, s4_shift, pad;
} ora_fixed_plan;

/* ---- scalar building blocks ---- */
uint16_t ora_f32_to_f16(float x);
float ora_f16_to_f32(uint16_t h);
uint32_t ora_crc32(const uint8_t* data, size_t n);
void ora_fwht(float* a, int n);
void ora_rotate_mid_band(const float* mid128, float* out128);
void ora_rotate_tail_fold(const float* vec, int dims, float* out64);
float ora_tail_rademacher(uint64_t block, uint64_t dim);
float ora_rademacher_diag(uint64_t seed, uint64_t i);
float ora_rabitq_bit_scale(void);
float ora_tail_fold_bit_scale(void);
void ora_lloyd_max(int bits, float* out /* 2^bits */);
int ora_nearest_centroid(const float* codebook, int n, float z);

/* ---- EDEN (src/eden.rs) ---- */
void ora_eden_fit_prefix(const float* rows, uint64_t n_rows, int dims, float* mean_out64);
void ora_eden_fit_band(const float* rows, uint64_t n_rows, int dims, int start, int width,
                       float* mean_out);
/* returns levels[64 or 128], centered_norm, scale_s */
void ora_eden_encode_slice(const float* mean, int d, uint64_t seed, int bits, const float* x,
                           uint8_t* levels, float* centered_norm, float* scale_s);

/* ---- encode (src/quantize.rs) ---- */
/* prefix_codec: 0 MinMax4, 1 EdenProd. mid_mean may be NULL (Rabitq mid). */
int ora_encode_block(const float* vecs, int n, int dims, const uint32_t* ts, const uint32_t* src,
                     int prefix_codec, const float* eden_mean, uint64_t eden_seed,
                     const float* mid_mean, uint64_t mid_seed, uint8_t* out4096);
/* encode_f32_corpus_par: timestamps = row index, sources = `src` for every row. */
int ora_encode_corpus(const float* rows, uint64_t n, int dims, uint32_t src, int prefix_codec,
                      const float* eden_mean, uint64_t eden_seed, const float* mid_mean,
                      uint64_t mid_seed, int threads, uint8_t* out_blocks);
int ora_verify_crc(const uint8_t* block4096);

/* ---- plan (src/scan.rs:105-266) ---- */
int ora_plan_build(const float* q, int dims, int prefix_codec, int mid_codec,
                   const float* eden_mean, uint64_t eden_seed, const float* mid_mean,
                   uint64_t mid_seed, ora_query_plan* out);

/* ---- scan (src/scan.rs:450-886) ---- */
/* Full reference semantics (warm-up, sharding, pruning). threads = Rayon thread count.
 * Returns number of hits written (<= shortlist_cand). has_lo/has_hi emulate Option<u32>. */
int ora_scan_blocks(const uint8_t* blocks, uint64_t n_blocks, const ora_query_plan* plan,
                    const ora_scan_cfg* cfg, int has_lo, uint32_t lo, int has_hi, uint32_t hi,
                    int threads, ora_scan_stats* stats, uint64_t* out_ids, float* out_scores);
/* Per-vector full score (all stages, no pruning, reference f32 arithmetic).
 * out_scores[b*64+v]; out_active[b*64+v] = 1 when the slot is live and the block passes the
 * temporal filter. */
void ora_full_scores(const uint8_t* blocks, uint64_t n_blocks, const ora_query_plan* plan,
                     const ora_scan_cfg* cfg, int has_lo, uint32_t lo, int has_hi, uint32_t hi,
                     float* out_scores, uint8_t* out_active);
/* Individual stages on one block for the narrowing property test (src/scan.rs:925-957).
 * Writes survivor masks after each stage and the scores after the last stage. */
void ora_block_stages(const uint8_t* block, const ora_query_plan* plan, const ora_scan_cfg* cfg,
                      float tau, uint64_t* masks4, float* scores64);

/* ---- fixed-point formulation ---- */
void ora_fixed_plan_build(const ora_query_plan* plan, const ora_scan_cfg* cfg,
                          ora_fixed_plan* out);
/* partials[(b*64+v)*3 + {0,1,2}] = {prefix, mid, tail} int32 sums; scores as assembled in f32 */
void ora_fixed_scores(const uint8_t* blocks, uint64_t n_blocks, const ora_query_plan* plan,
                      const ora_fixed_plan* fp, const ora_scan_cfg* cfg, int has_lo, uint32_t lo,
                      int has_hi, uint32_t hi, int32_t* partials, float* out_scores,
                      uint8_t* out_active);

/* ---- device layout (scan-side transcode of a PaxBlock64 page) ---- */
void ora_device_layout(const uint8_t* block4096, uint8_t* out4096, uint32_t* out_ts2);

/* ---- seeded synthetic inputs ---- */
/* docs: x_d = z_d / sqrt(d+1), z ~ Irwin-Hall(12)-6 (variance 1), then L2-normalised. */
void ora_synth_docs(uint64_t seed, uint64_t row0, uint64_t n, int dims, int threads, float* out);
/* queries: q = doc[pick] + sigma * z, renormalised; pick = hash(seed_pick, i) mod n_docs */
void ora_synth_queries(uint64_t doc_seed, uint64_t n_docs, uint64_t q_seed, uint64_t n_q, int dims,
                       float sigma, float* out, uint64_t* out_pick);

/* ---- exact top-k by (score desc, ordinal asc) over ora_full_scores output ---- */
int ora_topk_by_key(const float* scores, const uint8_t* active, uint64_t n, uint32_t k,
                    uint64_t* out_ids, float* out_scores);

/* ---- exact inner products on the query path ---- */
/* dot / dot_768 (src/embed.rs:115-152): at n == 768 eight accumulators over i = 0, 8, .. summed
 * acc0 + .. + acc7 left to right; otherwise a sequential sum of products starting from -0.0
 * (Iterator::sum for f32 in current Rust; only the sign of an all -0.0 sum depends on it). */
float ora_dot(const float* a, const float* b, uint64_t n);
/* RingBuffer::search_exact (src/ring.rs:109-119): dots of the query against n pending rows,
 * stable sort by score descending, first k; returns the count, positions in out_pos. */
uint32_t ora_ring_search(const float* pending, uint64_t n, int dims, const float* q, uint32_t k,
                         uint32_t* out_pos, float* out_scores);
/* QueryPipeline::rerank_exact_rows (src/pipeline.rs:157-169): dots against rows[cand[i]], stable
 * sort by score descending. */
void ora_rerank_rows(const float* rows, int dims, const float* q, const uint64_t* cand, uint64_t n_cand,
                     uint64_t* out_rows, float* out_scores);

#ifdef __cplusplus
}
#endif
#endif
