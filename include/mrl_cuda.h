/*
 * mrl_cuda.h — C ABI of the B200 (sm_100a) PaxBlock64 scan library (libmrl_b200.so).
 *
 * Drop-in boundary for the reference crate `mrl_index` v0.3.5 scan path. Each entry point names
 * the reference interface it replaces (file:line relative to the reference project root). Plain
 * pointers and sizes only; every function returns an int status (0 = OK, negative = error) and
 * never aborts or throws across the boundary; `mrl_last_error` explains the last failure.
 * Buffers are caller-owned unless a function says otherwise. A context drives one CUDA device
 * and one stream; it is not thread-safe (callers serialise, as the reference's IndexEngine
 * already does with its Mutex, src/engine.rs:564-581).
 *
 * Units: a block is one 4096-byte PaxBlock64 page (src/block.rs:130-144); a vector id is
 * VectorId::as_u64 = block << 16 | slot (src/block.rs:213-215).
 */
#ifndef MRL_CUDA_H
#define MRL_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MRL_OK 0
#define MRL_ERR_INVALID (-1) /* bad argument or contract violation (the reference panics) */
#define MRL_ERR_CUDA (-2)    /* CUDA runtime failure or no usable sm_100 device */
#define MRL_ERR_NOMEM (-3)   /* device allocation failed */

#define MRL_PREFIX_MINMAX4 0u /* PrefixCodec::MinMax4, src/config.rs:12 */
#define MRL_PREFIX_EDEN 1u    /* PrefixCodec::EdenProd, src/config.rs:15 */
#define MRL_MID_RABITQ 0u     /* MidCodec::Rabitq, src/config.rs:24 */
#define MRL_MID_EDEN_B1 1u    /* MidCodec::EdenB1, src/config.rs:27 */
#define MRL_DEPTH_L0 0u       /* StrataDepth::L0Only, src/config.rs:38 */
#define MRL_DEPTH_L1 1u       /* StrataDepth::L1Rabitq, src/config.rs:40 */
#define MRL_DEPTH_FULL 2u     /* StrataDepth::Full64b, src/config.rs:46 */
#define MRL_MODE_FAST 0u      /* fixed-point int32 stage sums choose candidates; results rescored exactly */
#define MRL_MODE_EXACT 1u     /* f32 sequential sums, bit-identical to the reference arithmetic */

typedef struct mrl_ctx mrl_ctx;
typedef struct mrl_seg mrl_seg;
typedef struct mrl_plans mrl_plans;

/* Field-for-field C mirror of `QueryPlan` (src/scan.rs:19-71). */
typedef struct mrl_query_plan {
    uint32_t dims;
    uint32_t prefix_codec;
    uint32_t mid_codec;
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
} mrl_query_plan;

/* Codec + fitted EDEN centres a plan is built against: `EdenFit` (src/eden.rs:104-113) as
 * persisted in eden_prefix.json. Host pointers. */
typedef struct mrl_codec_desc {
    uint32_t prefix_codec;
    uint32_t mid_codec;
    const float* eden_mean; /* [64]; required when prefix_codec == MRL_PREFIX_EDEN */
    uint64_t eden_seed;
    const float* mid_mean;  /* [128]; required when mid_codec == MRL_MID_EDEN_B1 */
    uint64_t mid_seed;
} mrl_codec_desc;

/* `ScanConfig` (src/config.rs:79-88) plus the device scoring mode. numa_sharding is a CPU
 * scheduling knob and is ignored on the device. Every scan returns the top shortlist_cand hits by
 * full score. That is the reference's own result whenever its pruning bounds (src/scan.rs:508-514,
 * 572-584, 587-607) are never below a full score: cs_tolerance >= 0 at L0Only, >= sqrt(2/pi) from
 * L1Rabitq on, and with the folded tail (Full64b, dims > 192) also cs_tolerance >= 1 and
 * |stratum4_weight| * sqrt(2/pi) * sqrt(B) <= cs_tolerance, B = min((dims - 192) / 64, 9). The
 * defaults (1.0, 0.20) qualify. Outside that region the reference's result depends on the order it
 * scans blocks in, and scans fail with MRL_ERR_INVALID naming the violated condition. */
typedef struct mrl_scan_cfg {
    uint32_t shortlist_cand;
    float cs_tolerance;
    float stratum4_weight;
    uint32_t strata_depth;
    uint32_t temporal_filter_enable;
    uint32_t numa_sharding;
    uint32_t mode;
} mrl_scan_cfg;

/* ---- context ---------------------------------------------------------------------------- */
/* Create a context on CUDA device `device` (needs compute capability 10.x). */
int mrl_ctx_create(int device, mrl_ctx** out);
void mrl_ctx_destroy(mrl_ctx* ctx);
const char* mrl_last_error(const mrl_ctx* ctx);
/* The CUDA stream the context launches on (cudaStream_t as void*). */
void* mrl_ctx_stream(mrl_ctx* ctx);
/* Use `stream` (cudaStream_t as void*; NULL = the context's own stream) for later launches. */
int mrl_ctx_set_stream(mrl_ctx* ctx, void* stream);

/* ---- segments: SegmentReader::open + as_slice (src/segment.rs:88-193) ------------------- */
/* Upload `n_blocks` PaxBlock64 pages from host memory into HBM. Pages are transcoded on the
 * device into the scan layout. `block_id_base` is added to the block index of every hit. */
int mrl_segment_upload(mrl_ctx* ctx, const uint8_t* blocks, uint64_t n_blocks,
                       uint32_t block_id_base, mrl_seg** out);
/* SegmentReader::open (src/segment.rs:88-162) into HBM: read a segment file (concatenated
 * 4096-byte pages, e.g. segments/000001.pax) through pinned, double-buffered staging, so file
 * reads overlap the copies and the transcode. A size that is not a multiple of 4096 fails with
 * "corrupt segment size N (not multiple of 4096)" (SegmentError::CorruptSize). Synchronous. */
int mrl_segment_load(mrl_ctx* ctx, const char* path, uint32_t block_id_base, mrl_seg** out);
/* SegmentReader::append_live (src/segment.rs:217-232): append one page. */
int mrl_segment_append(mrl_ctx* ctx, mrl_seg* seg, const uint8_t* block4096);
/* The same for n_blocks pages already in device memory (e.g. written by mrl_encode_device), on
 * the context stream: live ingest without a host round trip. */
int mrl_segment_append_device(mrl_ctx* ctx, mrl_seg* seg, const uint8_t* d_blocks, uint64_t n_blocks);
int mrl_segment_free(mrl_ctx* ctx, mrl_seg* seg);
uint64_t mrl_segment_blocks(const mrl_seg* seg);
/* Device pointer of the scan-layout pages (n_blocks * 4096 bytes) and block time ranges. */
int mrl_segment_device_ptrs(const mrl_seg* seg, void** pages, void** block_ts);
/* Copy the scan-layout pages and [min_ts, max_ts] pairs back to host memory (parity tests). */
int mrl_segment_read_layout(mrl_ctx* ctx, const mrl_seg* seg, uint8_t* out_pages,
                            uint32_t* out_ts);

/* ---- plans: QueryPlan::from_query_codec (src/scan.rs:105-266) --------------------------- */
/* Build `n_q` plans from host queries (row-major n_q x dims f32) on the device. */
int mrl_plan_build(mrl_ctx* ctx, const float* queries, uint32_t n_q, uint32_t dims,
                   const mrl_codec_desc* codec, mrl_plans** out);
/* Allocate plan storage for `n_q` queries of `dims` without building. */
int mrl_plans_alloc(mrl_ctx* ctx, uint32_t n_q, uint32_t dims, mrl_plans** out);
/* Build plans from device-resident queries into preallocated storage, on the context stream. */
int mrl_plan_build_device(mrl_ctx* ctx, const float* d_queries, uint32_t n_q, uint32_t dims,
                          const mrl_codec_desc* codec, mrl_plans* plans);
/* Rebuild plans [0, n_q) of existing storage from host queries, asynchronously on the context
 * stream and without allocating (the per-query host path of QueryPipeline::build_plan,
 * src/pipeline.rs:63-74). The host buffers may be reused once the call returns. */
int mrl_plan_rebuild(mrl_ctx* ctx, const float* queries, uint32_t n_q, uint32_t dims,
                     const mrl_codec_desc* codec, mrl_plans* plans);
int mrl_plans_free(mrl_ctx* ctx, mrl_plans* plans);
/* Read plan `i`'s reference fields back to the host (parity tests / debugging). */
int mrl_plan_read(mrl_ctx* ctx, const mrl_plans* plans, uint32_t i, mrl_query_plan* out);

/* ---- scan: scan_blocks / scan_blocks_stats (src/scan.rs:802-886) ------------------------ */
/* Scan every plan against the segment. time_lo / time_hi are Option<u32> (NULL = None).
 * Writes, per query q, up to k = cfg->shortlist_cand hits sorted by score descending into
 * out_ids[q*k ..] and out_scores[q*k ..], and the hit count into out_counts[q]. Host
 * buffers; synchronous. */
int mrl_scan(mrl_ctx* ctx, const mrl_seg* seg, const mrl_plans* plans, const mrl_scan_cfg* cfg,
             const uint32_t* time_lo, const uint32_t* time_hi, uint64_t* out_ids,
             float* out_scores, uint32_t* out_counts);
/* Same scan for plans [q0, q0+n_q) writing device buffers, asynchronously on the context
 * stream (no host synchronisation). out_status[q] (device, may be NULL) receives the selection
 * status word: bit 0 = the exact re-selection path ran, bit 1 = a CTA's list did not reach the
 * finishing CTA within about 1 s (no result), bit 3 = the context's scratch stayed busy for about
 * 1 s (the launch two before on the stream never released it; no result). */
int mrl_scan_device(mrl_ctx* ctx, const mrl_seg* seg, const mrl_plans* plans, uint32_t q0,
                    uint32_t n_q, const mrl_scan_cfg* cfg, const uint32_t* time_lo,
                    const uint32_t* time_hi, uint64_t* d_out_ids, float* d_out_scores,
                    uint32_t* d_out_counts, uint32_t* d_out_status);
/* scan_blocks for many plans in one pass over the pages (batched throughput): same arguments
 * and outputs as mrl_scan_device, two launches for all n_q plans. In MRL_MODE_FAST at depth L1 or
 * full, every result is bit-identical to mrl_scan_device's except for a query whose status has
 * MRL_STATUS_UNCERTIFIED set: there, one SM's share of the segment held more than 32 of that
 * query's top k, and the query must be rerun with mrl_scan_device (mrl_scan does this itself; it
 * uses this path from 8 plans on). Other modes and depths run mrl_scan_device. Scratch: n_q x SMs
 * x 256 bytes, grown on demand. */
#define MRL_STATUS_UNCERTIFIED 8u
/* Engines of the batched scan (mrl_set_batch_engine): the 5th-generation tensor cores (tcgen05
 * kind::i8 GEMMs of the slots' one-hot levels and bits against the plans' 8-bit table digits, the
 * default), or CUDA-core shared-memory table sums. Both give the same integers and scores. */
#define MRL_BATCH_TENSOR 0u
#define MRL_BATCH_CUDA_CORE 1u
int mrl_set_batch_engine(mrl_ctx* ctx, uint32_t engine);
int mrl_scan_batch_device(mrl_ctx* ctx, const mrl_seg* seg, const mrl_plans* plans, uint32_t q0,
                          uint32_t n_q, const mrl_scan_cfg* cfg, const uint32_t* time_lo,
                          const uint32_t* time_hi, uint64_t* d_out_ids, float* d_out_scores,
                          uint32_t* d_out_counts, uint32_t* d_out_status);
/* No counterpart in the reference (its scan allocates its shortlist on the Rust heap per call).
 * Same arguments, results and errors as mrl_scan_device, but the scan scratch comes from a static
 * per-device region inside the library instead of the context, so a successful call allocates no
 * device or host memory: for callers that must not allocate while answering a query. Limits, set
 * by that region's fixed size (1,180,928 bytes): seg must hold at most MRL_STATIC_MAX_BLOCKS pages
 * and the device at most MRL_STATIC_MAX_CTAS SMs, else MRL_ERR_INVALID with a message naming the
 * limit. The first call on a device looks the region up (and may load the module), so make it
 * before any stream capture begins. The looked-up address is kept for the life of the process and
 * is valid only while the device's primary context lives: after cudaDeviceReset (or anything else
 * that destroys the primary context) do not call this function again in the same process. The
 * region is shared by every context on a device: calls in
 * flight at the same time on one device (other streams, contexts or threads) race on it, while
 * calls ordered on one stream do not. Each call zeroes the region's control words on the context
 * stream before its first launch. out_status bit 1 = a CTA's list did not reach the finishing CTA
 * within about 1 s (no result). */
#define MRL_STATIC_MAX_BLOCKS 1048576u
#define MRL_STATIC_MAX_CTAS 256u
int mrl_scan_device_static(mrl_ctx* ctx, const mrl_seg* seg, const mrl_plans* plans, uint32_t q0,
                           uint32_t n_q, const mrl_scan_cfg* cfg, const uint32_t* time_lo,
                           const uint32_t* time_hi, uint64_t* d_out_ids, float* d_out_scores,
                           uint32_t* d_out_counts, uint32_t* d_out_status);
/* `ScanStats` (src/scan.rs:269-302): blocks scanned, their active vectors, and the survivors of the
 * prefix bound, of the mid-band + CS-tail bound, of the S4 budget bound, and the pushed ones. */
typedef struct mrl_scan_stats {
    uint64_t blocks;
    uint64_t active_vecs;
    uint64_t after_prefix;
    uint64_t after_s1;
    uint64_t after_s4_budget;
    uint64_t pushed;
} mrl_scan_stats;
/* scan_blocks_stats (src/scan.rs:813-886) for plan q: the results of mrl_scan (host buffers:
 * shortlist_cand ids and scores, the hit count) and, when `stats` is non-NULL, the prune counters
 * of src/scan.rs:654-799. The reference evaluates each block's bounds against its shortlist
 * threshold at block entry, which rises as its serial scan proceeds, so its counts depend on the
 * block order. Here every block is evaluated against the final threshold (the k-th score when the
 * scan returned k hits, else -inf): the counts the reference reports once its shortlist is warm,
 * exact for that threshold (the reference's f32 stage and bound expressions, in its order).
 * Counting costs one more pass over the segment. Synchronous. */
int mrl_scan_blocks_stats(mrl_ctx* ctx, const mrl_seg* seg, const mrl_plans* plans, uint32_t q,
                   const mrl_scan_cfg* cfg, const uint32_t* time_lo, const uint32_t* time_hi,
                   uint64_t* out_ids, float* out_scores, uint32_t* out_count, mrl_scan_stats* stats);
/* ---- fused plan + scan: QueryPipeline::build_plan + scan_segments_into (src/pipeline.rs:63-133) -- */
/* Build the plans of n_q device queries (row-major n_q x dims f32) into `plans` [0, n_q) and scan
 * the segment with each, in one launch per query: every CTA builds the query's plan in shared
 * memory while its first pages load, so no separate plan launch precedes the scan. Results and
 * status as mrl_scan_device; asynchronous on the context stream. */
int mrl_query_scan_device(mrl_ctx* ctx, const mrl_seg* seg, const float* d_queries, uint32_t n_q,
                          uint32_t dims, const mrl_codec_desc* codec, mrl_plans* plans,
                          const mrl_scan_cfg* cfg, const uint32_t* time_lo,
                          const uint32_t* time_hi, uint64_t* d_out_ids, float* d_out_scores,
                          uint32_t* d_out_counts, uint32_t* d_out_status);
/* The same from host queries to host results (synchronous). Each query (dims <= 1024) travels in
 * its scan launch's parameters, and the scan stores its top-k straight into a pinned,
 * device-mapped result slot of the context (mrl_query_submit / mrl_query_collect below), so the
 * call issues no separate copy in either direction; up to MRL_MAX_INFLIGHT of its queries are in
 * flight at once. Larger dims or an empty segment go through a pinned staging buffer instead (one
 * host-to-device copy). Fails with MRL_ERR_INVALID while submitted queries are uncollected. */
int mrl_query_scan(mrl_ctx* ctx, const mrl_seg* seg, const float* queries, uint32_t n_q, uint32_t dims,
                   const mrl_codec_desc* codec, mrl_plans* plans, const mrl_scan_cfg* cfg,
                   const uint32_t* time_lo, const uint32_t* time_hi, uint64_t* out_ids,
                   float* out_scores, uint32_t* out_counts);
/* ---- pipelined host queries (no counterpart in the reference, whose scan is a blocking call) --- */
/* mrl_query_submit launches the fused plan + scan of one host query (dims <= 1024 floats, carried in
 * the launch's parameters; non-finite values refused) and returns without waiting; the scan stores
 * the query's top-k, count and status in the context's result slot `slot` (pinned, device-mapped
 * host memory) and then that slot's completion word. mrl_query_collect waits for the slot's word
 * (spinning on host memory; about 10 s at most), then copies the `count` hits into out_ids /
 * out_scores (room for shortlist_cand each) and frees the slot. Queries on different slots may be in
 * flight together: consecutive scan launches on the context's stream overlap, so a caller that keeps
 * two or more submitted reaches the device's throughput from host memory. Results and errors are
 * those of mrl_query_scan; a slot must be collected before it is submitted again, and a larger
 * shortlist_cand than before needs every slot collected. The plan is not stored. */
#define MRL_MAX_INFLIGHT 8
int mrl_query_submit(mrl_ctx* ctx, const mrl_seg* seg, const float* query, uint32_t dims,
                     const mrl_codec_desc* codec, const mrl_scan_cfg* cfg, const uint32_t* time_lo,
                     const uint32_t* time_hi, uint32_t slot);
int mrl_query_collect(mrl_ctx* ctx, uint32_t slot, uint64_t* out_ids, float* out_scores,
                      uint32_t* out_count);
/* ---- NVLink exchange: the sharded scan's merge inside the scan launch --------------------- */
/* One exchange per rank (one process per GPU of a node, up to 8). Each rank's scan leaves its
 * top-k record (layout below) in its own exchange area and raises a flag there; the last CTA to
 * finish waits (bounded, about 2-3 s) until every other rank's flag for the same query is up,
 * reads their records over NVLink (peer loads) and merges them, so every rank ends with the
 * global top-k from one launch, with no collective library call on the query path. Replaces the
 * merge of per-shard shortlists in scan_blocks_stats (src/scan.rs:866-870) across GPUs. Set-up:
 * mrl_exchange_create on every rank (it fills `ipc_handle`, 64 bytes, when world > 1),
 * all-gather the handles (ordered by rank) by any means, then mrl_exchange_open. Every rank must
 * then call mrl_query_scan_exchange for the same sequence of queries. Records are double-buffered
 * by query parity, so no rank overwrites a record another rank may still read. world x
 * MRL_MERGE_RECORD_BYTES(k) must not exceed 200 KiB (k <= 2048 at world 8). Destroy only after all
 * ranks stopped scanning (a barrier). */
typedef struct mrl_exchange mrl_exchange;
int mrl_exchange_create(mrl_ctx* ctx, uint32_t world, uint32_t rank, uint32_t k, void* ipc_handle,
                        mrl_exchange** out);
int mrl_exchange_open(mrl_ctx* ctx, mrl_exchange* ex, const void* ipc_handles);
int mrl_exchange_destroy(mrl_ctx* ctx, mrl_exchange* ex);
/* Fused plan + scan of one device query (as mrl_query_scan_device with n_q = 1) whose outputs are
 * the GLOBAL top-k over all ranks' segments. cfg->shortlist_cand must equal the exchange's k.
 * out_status: bit 0 = re-selection ran, bit 1 = a CTA's list did not reach the finishing CTA in
 * time, bit 2 = a rank's record did not arrive in time, bit 3 = the scratch stayed busy (bits 1-3:
 * no result). */
int mrl_query_scan_exchange(mrl_ctx* ctx, const mrl_seg* seg, const float* d_query, uint32_t dims,
                            const mrl_codec_desc* codec, mrl_plans* plans, const mrl_scan_cfg* cfg,
                            const uint32_t* time_lo, const uint32_t* time_hi, mrl_exchange* ex,
                            uint64_t* d_out_ids, float* d_out_scores, uint32_t* d_out_count,
                            uint32_t* d_out_status);
/* mrl_query_submit over the exchange: the host query's fused plan + scan + merge, whose result slot
 * (collected with mrl_query_collect) receives the GLOBAL top-k over all ranks' segments. Every rank
 * must submit the same sequence of queries; consecutive submits overlap on the device as with
 * mrl_query_submit, and a rank ranks its own lists while the previous query's exchange runs.
 * mrl_query_collect fails when a rank's record did not arrive in time (status bit 2). */
int mrl_query_submit_exchange(mrl_ctx* ctx, const mrl_seg* seg, const float* query, uint32_t dims,
                              const mrl_codec_desc* codec, const mrl_scan_cfg* cfg, const uint32_t* time_lo,
                              const uint32_t* time_hi, mrl_exchange* ex, uint32_t slot);
/* ---- exact inner products: dot (src/embed.rs:115-152), bit-identical ------------------------ */
/* RingBuffer::search_exact (src/ring.rs:109-119): exact dots of the query against n_pending
 * unflushed vectors (device rows, n_pending x dims f32), top k written as one exchange record
 * (layout below, stride k) with ids VectorId(u32::MAX, i).as_u64(), the engine's ring sentinel
 * (src/engine.rs:584-594). mrl_merge_topk of the scan's record and this one gives the engine's
 * merged shortlist. Asynchronous on the context stream. n_pending <= 4096. */
int mrl_ring_search(mrl_ctx* ctx, const float* d_query, const float* d_pending, uint32_t n_pending,
                    uint32_t dims, uint32_t k, void* d_record);
/* QueryPipeline::rerank_exact_rows (src/pipeline.rs:157-169): exact dots of the query against
 * the candidate rows (row ids into d_rows, n_rows x dims f32), all candidates returned sorted by
 * score descending (equal scores keep candidate order). n_cand <= 4096. Synchronous (an out of
 * range row id fails with MRL_ERR_INVALID). */
int mrl_rerank_exact(mrl_ctx* ctx, const float* d_query, const float* d_rows, uint64_t n_rows,
                     uint32_t dims, const uint64_t* d_cand, uint32_t n_cand, uint64_t* d_out_rows,
                     float* d_out_scores);
/* RingBuffer (src/ring.rs:49-119): its pending embeddings mirrored in HBM, rows in push order.
 * The host keeps the rest of each PendingVector (passage id, timestamp, text). capacity is raised
 * to 64 (RingBuffer::new) and may not exceed 4096; mrl_ring_push fails when the ring is full
 * (RingBuffer::push flushes at 64, so an engine never fills it). mrl_ring_push copies one host row
 * (dims f32) on the context stream; mrl_ring_drain drops the first n rows (flush_block's
 * drain(..take)), keeping the order of the rest. */
typedef struct mrl_ring mrl_ring;
int mrl_ring_create(mrl_ctx* ctx, uint32_t dims, uint32_t capacity, mrl_ring** out);
int mrl_ring_push(mrl_ctx* ctx, mrl_ring* ring, const float* row);
int mrl_ring_drain(mrl_ctx* ctx, mrl_ring* ring, uint32_t n);
/* mrl_ring_push for n rows already in device memory (n x dims f32), on the context stream. */
int mrl_ring_push_device(mrl_ctx* ctx, mrl_ring* ring, const float* d_rows, uint32_t n);
/* search_exact for a batch: n_q device queries (n_q x dims f32) against the ring's pending rows
 * (NULL or empty: no hits), record q (stride k, the mrl_merge_topk layout) holding query q's top k
 * with the ring sentinel ids VectorId(u32::MAX, slot_base + position); the same scores and order
 * as mrl_ring_search. slot_base = 0 is the reference's sentinel; a sharded caller passes
 * rank x 4096 so the ring hits of different ranks stay distinct after the records are merged
 * across ranks (slot_base + pending rows must stay <= 65536). At most 1024 pending rows. With the
 * batch's scan records (mrl_pack_records) laid out before them, mrl_merge_topk_batch with
 * n_lists = 2 gives every query the engine's merged shortlist. */
int mrl_ring_search_batch(mrl_ctx* ctx, const float* d_queries, uint32_t n_q, uint32_t dims,
                          const mrl_ring* ring, uint32_t slot_base, uint32_t k, void* d_records);
uint32_t mrl_ring_len(const mrl_ring* ring);
int mrl_ring_rows(const mrl_ring* ring, const float** d_rows);
int mrl_ring_destroy(mrl_ctx* ctx, mrl_ring* ring);
/* The scan half of IndexEngine::query_filtered (src/engine.rs:564-594) for one device query:
 * fused plan + scan of `seg`, then the exact search of the ring's pending rows (NULL or empty:
 * none), merged into one shortlist of at most cfg->shortlist_cand hits, ordered by score
 * descending then id ascending (ring hits carry VectorId(u32::MAX, i), so a scanned hit keeps its
 * place against an equal ring score, as Shortlist::push keeps the incumbent). Three launches
 * when the ring holds rows, one otherwise; asynchronous on the context stream. */
int mrl_engine_scan(mrl_ctx* ctx, const mrl_seg* seg, const float* d_query, uint32_t dims,
                    const mrl_codec_desc* codec, mrl_plans* plans, const mrl_scan_cfg* cfg,
                    const uint32_t* time_lo, const uint32_t* time_hi, const mrl_ring* ring,
                    uint64_t* d_out_ids, float* d_out_scores, uint32_t* d_out_count,
                    uint32_t* d_out_status);
/* Exchange step of the sharded scan. An exchange record holds one rank's top list: `stride` u64
 * ids, then `stride` f32 scores, then the u32 count of valid entries, padded to
 * MRL_MERGE_RECORD_BYTES(stride) bytes (a multiple of 16). mrl_scan_device fills one when its
 * d_out_ids / d_out_scores / d_out_counts point at the record's three parts (k == stride). Each
 * rank all-gathers the records (one collective), then mrl_merge_topk merges the n_lists records at
 * d_lists (device, contiguous) into the global top-k, ordered by score descending then id
 * ascending, on the context stream. Replaces the merge of per-shard shortlists in
 * scan_blocks_stats (src/scan.rs:866-870) across GPUs. n_lists in [1, 1024], stride and k in
 * [1, 4096]; d_lists 16-byte aligned. */
#define MRL_MERGE_RECORD_BYTES(stride) ((((size_t)(stride)) * 12u + 4u + 15u) & ~(size_t)15u)
int mrl_merge_topk(mrl_ctx* ctx, const void* d_lists, uint32_t n_lists, uint32_t stride, uint32_t k,
                   uint64_t* d_out_ids, float* d_out_scores, uint32_t* d_out_count);
/* The exchange step for a batch (each rank scans its pages for n_q queries with
 * mrl_scan_batch_device). mrl_pack_records writes the batch's outputs (n_q rows of k ids / scores,
 * n_q counts) as n_q records of stride k. After an all-gather of every rank's records (rank-major:
 * record q of list r at (r * n_q + q) * MRL_MERGE_RECORD_BYTES(stride)), mrl_merge_topk_batch
 * merges each query's n_lists records into its global top-k (rows of k in the outputs, counts),
 * one CTA per query, in the same order as mrl_merge_topk. Device buffers, context stream. */
int mrl_pack_records(mrl_ctx* ctx, const uint64_t* d_ids, const float* d_scores, const uint32_t* d_counts,
                     uint32_t n_q, uint32_t k, void* d_records);
int mrl_merge_topk_batch(mrl_ctx* ctx, const void* d_lists, uint32_t n_lists, uint32_t n_q, uint32_t stride,
                         uint32_t k, uint64_t* d_out_ids, float* d_out_scores, uint32_t* d_out_counts);
/* Per-vector scores of plan `q` for every slot (n_blocks*64, host), and for MRL_MODE_FAST the
 * three int32 stage sums per slot (prefix, mid band, folded tail; may be NULL). Inactive slots
 * (tombstoned or temporally filtered) get score 0 and active 0. */
int mrl_debug_vector_scores(mrl_ctx* ctx, const mrl_seg* seg, const mrl_plans* plans, uint32_t q,
                            const mrl_scan_cfg* cfg, const uint32_t* time_lo,
                            const uint32_t* time_hi, float* out_scores, uint8_t* out_active,
                            int32_t* out_partials);

/* The bound E the fast mode's final ranking uses for plan q over seg: every slot's fast-mode score
 * (the fixed-point stage sums) is within E of its exact-mode score (the reference's f32 loops).
 * Derived from the plan's per-stage magnitudes and the segment's maxima of |scale|, |offset|, mid_n
 * and max(high_n, 1e-6), which every call that adds pages keeps current. Synchronous. */
int mrl_debug_score_bound(mrl_ctx* ctx, const mrl_seg* seg, const mrl_plans* plans, uint32_t q,
                          const mrl_scan_cfg* cfg, float* out_bound);
/* The context's scan control words into out[128]: 8 per scratch set (page counter, publish ticket,
 * five unused words, exit ticket). Consecutive scan launches use the sixteen sets in turn; every
 * launch leaves its set's words at zero, whichever path it took. Synchronous. */
int mrl_debug_control_words(mrl_ctx* ctx, uint32_t* out);

/* ---- encode: encode_block_with_fits (src/quantize.rs:36-96) ----------------------------- */
/* Encode host rows (n x dims f32, rows 64*b .. 64*b+63 form block b) into PaxBlock64 pages.
 * ts / src give each row's timestamp and source mask (NULL: ts = row index, src = DOC). */
int mrl_encode_blocks(mrl_ctx* ctx, const float* rows, uint64_t n, uint32_t dims,
                      const uint32_t* ts, const uint32_t* src, const mrl_codec_desc* codec,
                      uint8_t* out_pages);
/* Device-resident variant: rows, pages (NULL allowed) are device pointers; when `seg_out` is
 * non-NULL a segment is also created directly in the scan layout. ts = row index. */
int mrl_encode_device(mrl_ctx* ctx, const float* d_rows, uint64_t n, uint32_t dims, uint32_t src,
                      const mrl_codec_desc* codec, uint8_t* d_pages, uint32_t block_id_base,
                      mrl_seg** seg_out);
/* EdenFit::fit_prefix / fit_band (src/eden.rs:116-161) over device rows; mean to host. */
int mrl_eden_fit_device(mrl_ctx* ctx, const float* d_rows, uint64_t n, uint32_t dims,
                        uint32_t start, uint32_t width, float* mean_out);

/* ---- seeded synthetic inputs (benchmarks; same integer recipe as the test oracle) -------- */
/* Docs: x_d = z_d / sqrt(d+1) with z ~ Irwin-Hall(12) - 6, L2-normalised. Device output. */
int mrl_synth_docs_device(mrl_ctx* ctx, uint64_t seed, uint64_t row0, uint64_t n, uint32_t dims,
                          float* d_out);
/* Queries: a seeded doc plus sigma * z per dim, L2-normalised. Device output. */
int mrl_synth_queries_device(mrl_ctx* ctx, uint64_t doc_seed, uint64_t n_docs, uint64_t q_seed,
                             uint64_t n_q, uint32_t dims, float sigma, float* d_out,
                             uint64_t* d_pick);

/* ---- introspection --------------------------------------------------------------------- */
/* Number of CTAs the scan kernel launches on this device and the per-CTA candidate list
 * length used for shortlist k. */
int mrl_scan_geometry(mrl_ctx* ctx, uint32_t k, uint32_t* ctas, uint32_t* list_len);
/* Override the per-CTA candidate list length: 0 = automatic, else a power of two <= 32. Smaller
 * values exercise the exact re-selection path in tests. */
int mrl_set_list_len(mrl_ctx* ctx, uint32_t list_len);
/* CTAs of each single-query scan launch (mrl_scan, mrl_query_scan*, mrl_query_submit, the
 * exchange): 0 (the default) = one per SM, the lowest latency for one query at a time; fewer
 * spread each CTA's fixed costs (its plan build and its list) over more pages, and consecutive
 * queries then run side by side on the free SMs, which raises the throughput of a stream of
 * queries at the cost of each query's latency. At most the device's SM count. No counterpart in the
 * reference. */
int mrl_set_scan_ctas(mrl_ctx* ctx, uint32_t ctas);

#ifdef __cplusplus
}
#endif
#endif /* MRL_CUDA_H */
