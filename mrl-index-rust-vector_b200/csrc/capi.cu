// capi.cu — the C ABI of libmrl_b200 (include/mrl_cuda.h): contexts, device segments, plans,
// scans and encodes. Host-side C++; every entry point catches its own failures and reports them
// through a status code plus mrl_last_error, never by aborting.
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "mrl_internal.cuh"

// Scan scratch for mrl_scan_device_static, placed in the module's own global memory so that entry
// point allocates nothing. Layout (bytes): control words and per-CTA ready flags [0, 1280), per-CTA
// key lists [1280, 1280 + 256*32*8), their exact-mode keys (the next 256*32*8), one owner byte per
// page after that. Sized for grids of at most MRL_STATIC_MAX_CTAS CTAs and segments of at most
// MRL_STATIC_MAX_BLOCKS pages: 1,180,928 bytes per device in all.
namespace {
constexpr size_t kStaticCtlOff = 0;
constexpr size_t kStaticKeysOff = 1280;
constexpr size_t kStaticListBytes = (size_t)MRL_STATIC_MAX_CTAS * 32 * sizeof(unsigned long long);
constexpr size_t kStaticXKeysOff = kStaticKeysOff + kStaticListBytes;
constexpr size_t kStaticOwnerOff = kStaticXKeysOff + kStaticListBytes;
constexpr size_t kStaticBytes = kStaticOwnerOff + (size_t)MRL_STATIC_MAX_BLOCKS;
static_assert(kStaticBytes == 1180928, "static scratch size is documented in the header");
static_assert(mrl::kCtlWords * sizeof(unsigned) <= kStaticKeysOff - kStaticCtlOff, "control words overflow");
static_assert(MRL_STATIC_MAX_CTAS <= 256 && MRL_STATIC_MAX_CTAS <= mrl::kMaxScanCtas, "owner bytes hold CTA indices < 256");
}  // namespace
static __device__ __align__(256) unsigned char g_static_scan_scratch[kStaticBytes];

namespace {
// Scratch sets of the single-query scans (consecutive launches may be in flight together).
constexpr uint32_t kScratchSets = 16;
// Initial done words of the scratch sets: launch s < kScratchSets waits for s - kScratchSets.
const unsigned int kDoneInit[kScratchSets] = {
    0xFFFFFFF0u, 0xFFFFFFF1u, 0xFFFFFFF2u, 0xFFFFFFF3u, 0xFFFFFFF4u, 0xFFFFFFF5u, 0xFFFFFFF6u, 0xFFFFFFF7u,
    0xFFFFFFF8u, 0xFFFFFFF9u, 0xFFFFFFFAu, 0xFFFFFFFBu, 0xFFFFFFFCu, 0xFFFFFFFDu, 0xFFFFFFFEu, 0xFFFFFFFFu};
}  // namespace

struct mrl_ctx {
    int device = 0;
    int sms = 0;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    std::string err;
    // scan scratch, kScratchSets sets used by consecutive scan launches in turn: launches on the
    // stream may overlap (programmatic dependent launch), and a launch touches its set only once the
    // launch that used it before has released it. Per set: per-CTA lists, control words, per-page
    // owner (grow-only; each set owns an equal share of `owner`).
    unsigned long long* cta_keys = nullptr;  // per set 2 * sms * 32: scan keys, then their exact keys
    unsigned int* ctl = nullptr;             // per set mrl::kCtlWords
    uint8_t* owner = nullptr;
    size_t owner_bytes = 0;
    uint32_t scan_seq = 0;      // launches so far; launch s uses scratch set s % kScratchSets
    uint32_t scan_ctas = 0;     // CTAs per single-query scan launch (0: one per SM)
    unsigned int* done = nullptr;  // per set: sequence number of the last launch that released it
    uint32_t list_len_override = 0;
    // grow-only scratch for host-facing calls: inputs (queries, rows, means) and outputs
    void* tmp = nullptr;
    size_t tmp_bytes = 0;
    void* tmp_out = nullptr;
    size_t tmp_out_bytes = 0;
    // device copy of the last codec centres uploaded (64 prefix + 128 mid floats) and its host
    // twin, so repeated plan builds against one EdenFit issue no host->device copy
    float* d_means = nullptr;
    float h_means[192];
    bool means_valid = false;
    // grow-only scratch of the exact paths (scores, flag)
    void* xbuf = nullptr;
    size_t xbuf_bytes = 0;
    // two merge records (scan, ring) of mrl_engine_scan
    void* ebuf = nullptr;
    size_t ebuf_bytes = 0;
    // per-(query, CTA) top lists and tensor-core operand tiles of the batched scan
    void* bbuf = nullptr;
    size_t bbuf_bytes = 0;
    uint32_t batch_engine = MRL_BATCH_TENSOR;
    // pinned host staging of mrl_query_scan, mapped into the device's address space: the query is
    // copied to the device from here, and the scan kernel stores its results straight into it
    // (no device-to-host copies on the query path)
    void* h_io = nullptr;
    void* h_io_dev = nullptr;
    size_t h_io_bytes = 0;
    // pipelined host queries (mrl_query_submit / mrl_query_collect): MRL_MAX_INFLIGHT result slots
    // in pinned, device-mapped memory, laid out for shortlists up to slot_k; the scan stores each
    // query's top-k there and then the slot's completion word, on which the host waits
    unsigned char* h_slots = nullptr;
    unsigned char* d_slots = nullptr;
    size_t slot_stride = 0;
    uint32_t slot_k = 0;
    uint32_t slot_seq[MRL_MAX_INFLIGHT] = {};
    bool slot_busy[MRL_MAX_INFLIGHT] = {};
};

// RingBuffer's pending embeddings (src/ring.rs:49-119) mirrored in HBM: `len` rows of `dims` f32
// in push order.
struct mrl_ring {
    float* rows = nullptr;
    uint32_t dims = 0, capacity = 0, len = 0;
};

struct mrl_seg {
    uint4* pages = nullptr;
    uint2* ts = nullptr;
    uint64_t n_blocks = 0;
    uint64_t cap_blocks = 0;
    uint32_t block_id_base = 0;
    // device: maxima of the slots' score factors (mrl::launch_metamax), kept current by every call
    // that adds pages; fast-mode scans derive their fast/exact score bound from them
    float* metamax = nullptr;
};

struct mrl_plans {
    mrl::DevPlan* d = nullptr;
    uint32_t n_q = 0;
    uint32_t dims = 0;
};

// NVLink exchange: this rank's area on this GPU (for both buffer parities, one receive record per
// sending rank, then one flag word per parity and sender) and the mapped areas of the other ranks
// of the node, into which this rank pushes its record and raises its flags.
struct mrl_exchange {
    int device = 0;
    uint32_t world = 0, rank = 0, k = 0;
    size_t rb = 0;                               // bytes per record
    unsigned char* local = nullptr;              // this rank's area (cudaMalloc)
    unsigned char* area[mrl::kMaxRanks] = {};    // every rank's area (area[rank] == local)
    unsigned char* stage = nullptr;              // kScratchSets staged records, one per scratch set
    uint32_t epoch = 0;
    bool opened = false;
    size_t flags_off() const { return 2 * (size_t)world * rb; }
    size_t bytes() const { return flags_off() + ((2 * (size_t)world * sizeof(unsigned) + 15) & ~(size_t)15); }
};

namespace {

int fail(mrl_ctx* ctx, int code, const std::string& msg) {
    if (ctx) ctx->err = msg;
    return code;
}

int cuda_fail(mrl_ctx* ctx, cudaError_t e, const char* what) {
    return fail(ctx, MRL_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

#define MRL_CUDA_TRY(ctx, expr)                                   \
    do {                                                          \
        cudaError_t _e = (expr);                                  \
        if (_e != cudaSuccess) return cuda_fail((ctx), _e, #expr); \
    } while (0)

int set_device(mrl_ctx* ctx) {
    const cudaError_t e = cudaSetDevice(ctx->device);
    return e == cudaSuccess ? MRL_OK : cuda_fail(ctx, e, "cudaSetDevice");
}

// Device address of g_static_scan_scratch on ctx's device (which must be current), looked up on
// the first call per device and cached. The lookup may load this module onto the device, so the
// first mrl_scan_device_static call on a device should come before any stream capture begins.
constexpr int kStaticMaxDevices = 64;
unsigned char* g_static_base[kStaticMaxDevices] = {};
std::mutex g_static_mu;

int static_scratch(mrl_ctx* ctx, unsigned char** out) {
    if (ctx->device >= kStaticMaxDevices) return fail(ctx, MRL_ERR_INVALID, "device ordinal >= 64");
    std::lock_guard<std::mutex> lock(g_static_mu);
    if (!g_static_base[ctx->device]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scan_scratch);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaGetSymbolAddress(g_static_scan_scratch)");
        g_static_base[ctx->device] = static_cast<unsigned char*>(p);
    }
    *out = g_static_base[ctx->device];
    return MRL_OK;
}

int ensure_buf(mrl_ctx* ctx, void** buf, size_t* have, size_t bytes) {
    if (*have >= bytes) return MRL_OK;
    if (*buf) cudaFree(*buf);  // synchronises the device: no launch still reads the old buffer
    *buf = nullptr;
    *have = 0;
    const cudaError_t e = cudaMalloc(buf, bytes);
    if (e != cudaSuccess) return fail(ctx, MRL_ERR_NOMEM, std::string("cudaMalloc scratch: ") + cudaGetErrorString(e));
    *have = bytes;
    return MRL_OK;
}
int ensure_tmp(mrl_ctx* ctx, size_t bytes) { return ensure_buf(ctx, &ctx->tmp, &ctx->tmp_bytes, bytes); }
int ensure_host_io(mrl_ctx* ctx, size_t bytes) {
    if (ctx->h_io_bytes >= bytes) return MRL_OK;
    bytes = (bytes + 65535) & ~(size_t)65535;
    if (ctx->h_io) {
        cudaStreamSynchronize(ctx->stream);  // no launch still writes the old staging
        cudaFreeHost(ctx->h_io);
    }
    ctx->h_io = ctx->h_io_dev = nullptr;
    ctx->h_io_bytes = 0;
    cudaError_t e = cudaHostAlloc(&ctx->h_io, bytes, cudaHostAllocMapped | cudaHostAllocPortable);
    if (e != cudaSuccess) {
        ctx->h_io = nullptr;
        return fail(ctx, MRL_ERR_NOMEM, std::string("cudaHostAlloc staging: ") + cudaGetErrorString(e));
    }
    e = cudaHostGetDevicePointer(&ctx->h_io_dev, ctx->h_io, 0);
    if (e != cudaSuccess) {
        cudaFreeHost(ctx->h_io);
        ctx->h_io = ctx->h_io_dev = nullptr;
        return cuda_fail(ctx, e, "cudaHostGetDevicePointer");
    }
    ctx->h_io_bytes = bytes;
    return MRL_OK;
}
int ensure_out(mrl_ctx* ctx, size_t bytes) { return ensure_buf(ctx, &ctx->tmp_out, &ctx->tmp_out_bytes, bytes); }

// mrl_scan switches to the batched scan from this many plans on (fast mode, depth L1 or full)
constexpr uint32_t kBatchMinQueries = 8;

uint32_t auto_list_len(uint32_t k, uint32_t ctas) {
    // Expected top-k members per CTA is k/ctas; keep 2.5x that plus 8, as a power of two in
    // [16, 32]. Larger concentrations are caught by the final selection's verification.
    const double want = 2.5 * (double)k / (double)ctas + 8.0;
    uint32_t l = 16;
    while (l < want && l < 32) l <<= 1;
    return l;
}

// The reference prunes with Cauchy-Schwarz bounds scaled by cs_tolerance (alpha) against the
// shortlist's running threshold (src/scan.rs:508-514, 572-584, 587-607, 766-767). Where every bound
// is >= the full score, a pruned vector could not have entered the shortlist anyway, so the
// reference's result is the top-k by full score whatever order the blocks are scanned in. That is
// what this library computes. It holds when
//   * L0Only: alpha >= 0 (the bound adds alpha * |q_after_prefix| * |x_rest| to the pushed score);
//   * L1Rabitq and deeper: alpha >= sqrt(2/pi), since |s1| <= sqrt(2/pi) |q_mid| (src/rotate.rs:46-49);
//   * Full64b with a folded tail: also alpha >= 1 (the S4 budget bound is alpha * |s4|max) and
//     |stratum4_weight| * sqrt(2/pi) * sqrt(B) <= alpha, B = min((dims - 192) / 64, 9) folded
//     blocks, since |s4| <= sqrt(2/pi) sqrt(B) |q_tail| (src/rotate.rs:73-93, 120-126).
// Outside that region the reference's result depends on the order the blocks are scanned in (its
// serial scan and its Rayon shards already disagree), which no parallel scan can reproduce, so the
// configuration is refused. `dims` = 0: the call does not select a shortlist (no check).
int check_cfg(mrl_ctx* ctx, const mrl_scan_cfg* cfg, uint32_t dims) {
    if (!cfg) return fail(ctx, MRL_ERR_INVALID, "cfg is NULL");
    if (cfg->shortlist_cand < 1 || cfg->shortlist_cand > 4096)
        return fail(ctx, MRL_ERR_INVALID, "shortlist_cand must be in [1, 4096]");
    if (cfg->strata_depth > MRL_DEPTH_FULL) return fail(ctx, MRL_ERR_INVALID, "strata_depth must be 0, 1 or 2");
    if (cfg->mode > MRL_MODE_EXACT) return fail(ctx, MRL_ERR_INVALID, "mode must be MRL_MODE_FAST or MRL_MODE_EXACT");
    if (!std::isfinite(cfg->stratum4_weight) || !std::isfinite(cfg->cs_tolerance))
        return fail(ctx, MRL_ERR_INVALID, "stratum4_weight and cs_tolerance must be finite");
    if (dims == 0) return MRL_OK;
    const double alpha = cfg->cs_tolerance, sqrt_2_pi = std::sqrt(2.0 / 3.14159265358979323846);
    const uint32_t B = dims > 192u ? std::min<uint32_t>((dims - 192u) / 64u, 9u) : 0u;
    const bool tail = cfg->strata_depth == MRL_DEPTH_FULL && dims > 192u;
    std::string why;
    if (alpha < 0.0) why = "cs_tolerance < 0";
    else if (cfg->strata_depth >= MRL_DEPTH_L1 && alpha < sqrt_2_pi) why = "cs_tolerance < sqrt(2/pi)";
    else if (tail && alpha < 1.0) why = "cs_tolerance < 1 with the folded-tail stage (S4 budget bound)";
    else if (tail && std::fabs((double)cfg->stratum4_weight) * sqrt_2_pi * std::sqrt((double)B) > alpha)
        why = "stratum4_weight * sqrt(2/pi) * sqrt(" + std::to_string(B) + " folded blocks) > cs_tolerance";
    if (!why.empty())
        return fail(ctx, MRL_ERR_INVALID,
                    why + ": the reference's pruning bounds are then lossy and its result depends on the block "
                          "scan order; only order-independent configurations are supported");
    return MRL_OK;
}

// CTAs of a single-query scan launch.
uint32_t scan_grid(const mrl_ctx* ctx) { return ctx->scan_ctas ? ctx->scan_ctas : (uint32_t)ctx->sms; }

mrl::ScanLaunch make_launch(mrl_ctx* ctx, const mrl_seg* seg, const mrl_plans* plans, uint32_t q,
                            const mrl_scan_cfg* cfg, const uint32_t* lo, const uint32_t* hi) {
    mrl::ScanLaunch p{};
    p.pages = seg->pages;
    p.block_ts = seg->ts;
    p.n_blocks = (uint32_t)seg->n_blocks;
    p.block_id_base = seg->block_id_base;
    p.plan = plans ? plans->d + q : nullptr;
    p.k = cfg->shortlist_cand;
    p.list_len = ctx->list_len_override ? ctx->list_len_override : auto_list_len(p.k, scan_grid(ctx));
    p.w_s4 = cfg->stratum4_weight;
    p.depth = cfg->strata_depth;
    p.mode = cfg->mode;
    p.use_time = cfg->temporal_filter_enable && (lo || hi) ? 1u : 0u;
    p.has_lo = lo ? 1u : 0u;
    p.lo = lo ? *lo : 0u;
    p.has_hi = hi ? 1u : 0u;
    p.hi = hi ? *hi : 0u;
    p.metamax = seg->metamax;
    return p;
}

// Grows the per-page owner scratch to kScratchSets sets of n_blocks bytes each.
int ensure_owner(mrl_ctx* ctx, uint64_t n_blocks) {
    return ensure_buf(ctx, (void**)&ctx->owner, &ctx->owner_bytes, kScratchSets * (n_blocks ? n_blocks : 1));
}

// The context scratch of the next scan launch: the sets are used in turn. Launch s waits until
// launch s - kScratchSets (the previous user of its set) has released it; a set's done word starts
// at the sequence number such a launch before the first would have had. launched() advances the
// sequence once the launch has been issued.
void take_scratch(mrl_ctx* ctx, mrl::ScanLaunch& p) {
    const size_t set = ctx->scan_seq % kScratchSets;
    p.cta_keys = ctx->cta_keys + set * 2 * 32 * (size_t)ctx->sms;
    p.cta_xkeys = p.cta_keys + 32 * (size_t)ctx->sms;
    p.ctl = ctx->ctl + set * mrl::kCtlWords;
    p.owner = ctx->owner + set * (ctx->owner_bytes / kScratchSets);
    p.done = ctx->done + set;
    p.seq = ctx->scan_seq;
    p.done_prev = ctx->scan_seq - kScratchSets;
}
void launched(mrl_ctx* ctx) { ++ctx->scan_seq; }

int check_codec(mrl_ctx* ctx, const mrl_codec_desc* codec) {
    if (!codec) return fail(ctx, MRL_ERR_INVALID, "codec is NULL");
    if (codec->prefix_codec > MRL_PREFIX_EDEN || codec->mid_codec > MRL_MID_EDEN_B1)
        return fail(ctx, MRL_ERR_INVALID, "unknown codec");
    if (codec->prefix_codec == MRL_PREFIX_EDEN && !codec->eden_mean)
        return fail(ctx, MRL_ERR_INVALID, "EdenProd requires EdenFit (eden_mean)");  // src/scan.rs:116
    if (codec->mid_codec == MRL_MID_EDEN_B1 && !codec->mid_mean)
        return fail(ctx, MRL_ERR_INVALID, "EdenB1 mid requires EdenFit (mid_mean)");   // src/scan.rs:121
    return MRL_OK;
}

// Makes ctx->d_means hold the codec's centres (64 prefix + 128 mid floats); copies only when they
// differ from the last upload. Returns the device pointer through `out`.
int upload_means(mrl_ctx* ctx, const mrl_codec_desc* codec, float** out) {
    float h[192];
    for (int i = 0; i < 192; ++i) h[i] = 0.0f;
    if (codec->eden_mean) std::memcpy(h, codec->eden_mean, 64 * sizeof(float));
    if (codec->mid_mean) std::memcpy(h + 64, codec->mid_mean, 128 * sizeof(float));
    if (!ctx->means_valid || std::memcmp(h, ctx->h_means, sizeof(h)) != 0) {
        std::memcpy(ctx->h_means, h, sizeof(h));
        MRL_CUDA_TRY(ctx, cudaMemcpyAsync(ctx->d_means, ctx->h_means, sizeof(h), cudaMemcpyHostToDevice, ctx->stream));
        MRL_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));  // h_means may change on the next call
        ctx->means_valid = true;
    }
    *out = ctx->d_means;
    return MRL_OK;
}

// A new empty segment with its meta maxima zeroed (synchronous), or an error.
int seg_new(mrl_ctx* ctx, uint32_t block_id_base, mrl_seg** out) {
    *out = nullptr;
    mrl_seg* s = new mrl_seg();
    s->block_id_base = block_id_base;
    if (cudaMalloc(&s->metamax, 4 * sizeof(float)) != cudaSuccess) {
        delete s;
        return fail(ctx, MRL_ERR_NOMEM, "cudaMalloc segment maxima");
    }
    const cudaError_t e = cudaMemset(s->metamax, 0, 4 * sizeof(float));
    if (e != cudaSuccess) {
        cudaFree(s->metamax);
        delete s;
        return cuda_fail(ctx, e, "cudaMemset segment maxima");
    }
    *out = s;
    return MRL_OK;
}

// Fold pages [b0, b0 + nb) of s into its meta maxima (on the context stream).
int seg_note_pages(mrl_ctx* ctx, mrl_seg* s, uint64_t b0, uint64_t nb) {
    if (mrl::launch_metamax(s->pages + b0 * 256, nb, s->metamax, ctx->stream))
        return cuda_fail(ctx, cudaGetLastError(), "segment maxima launch");
    return MRL_OK;
}

int seg_reserve(mrl_ctx* ctx, mrl_seg* s, uint64_t blocks) {
    if (blocks <= s->cap_blocks) return MRL_OK;
    uint64_t cap = s->cap_blocks ? s->cap_blocks : 64;
    while (cap < blocks) cap *= 2;
    uint4* np = nullptr;
    uint2* nt = nullptr;
    if (cudaMalloc(&np, cap * (uint64_t)mrl::kBlockBytes) != cudaSuccess) return fail(ctx, MRL_ERR_NOMEM, "cudaMalloc pages");
    if (cudaMalloc(&nt, cap * sizeof(uint2)) != cudaSuccess) {
        cudaFree(np);
        return fail(ctx, MRL_ERR_NOMEM, "cudaMalloc block_ts");
    }
    if (s->n_blocks) {
        MRL_CUDA_TRY(ctx, cudaMemcpyAsync(np, s->pages, s->n_blocks * (uint64_t)mrl::kBlockBytes, cudaMemcpyDeviceToDevice, ctx->stream));
        MRL_CUDA_TRY(ctx, cudaMemcpyAsync(nt, s->ts, s->n_blocks * sizeof(uint2), cudaMemcpyDeviceToDevice, ctx->stream));
        MRL_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    }
    cudaFree(s->pages);
    cudaFree(s->ts);
    s->pages = np;
    s->ts = nt;
    s->cap_blocks = cap;
    return MRL_OK;
}

}  // namespace

extern "C" {

int mrl_ctx_create(int device, mrl_ctx** out) {
    if (!out) return MRL_ERR_INVALID;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return MRL_ERR_CUDA;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return MRL_ERR_CUDA;
    if (prop.major != 10) return MRL_ERR_CUDA;  // built for sm_100a only
    mrl_ctx* ctx = new mrl_ctx();
    ctx->device = device;
    ctx->sms = prop.multiProcessorCount;
    if (ctx->sms > mrl::kMaxScanCtas) {  // one scan CTA per SM, each with a ready flag
        delete ctx;
        return MRL_ERR_INVALID;
    }
    if (cudaSetDevice(device) != cudaSuccess || cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking) != cudaSuccess) {
        delete ctx;
        return MRL_ERR_CUDA;
    }
    ctx->stream = ctx->own_stream;
    if (cudaMalloc(&ctx->cta_keys, sizeof(unsigned long long) * kScratchSets * 2 * 32 * (size_t)ctx->sms) != cudaSuccess ||
        cudaMalloc(&ctx->ctl, sizeof(unsigned int) * kScratchSets * mrl::kCtlWords) != cudaSuccess ||
        cudaMalloc(&ctx->done, sizeof(unsigned int) * kScratchSets) != cudaSuccess ||
        cudaMalloc(&ctx->d_means, 192 * sizeof(float)) != cudaSuccess ||
        cudaMemset(ctx->ctl, 0, sizeof(unsigned int) * kScratchSets * mrl::kCtlWords) != cudaSuccess ||
        cudaMemcpy(ctx->done, kDoneInit, sizeof(kDoneInit), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess) {
        mrl_ctx_destroy(ctx);
        return MRL_ERR_NOMEM;
    }
    *out = ctx;
    return MRL_OK;
}

void mrl_ctx_destroy(mrl_ctx* ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    cudaFree(ctx->cta_keys);
    cudaFree(ctx->ctl);
    cudaFree(ctx->done);
    cudaFree(ctx->owner);
    cudaFree(ctx->tmp);
    cudaFree(ctx->tmp_out);
    cudaFree(ctx->d_means);
    cudaFree(ctx->xbuf);
    cudaFree(ctx->ebuf);
    cudaFree(ctx->bbuf);
    if (ctx->h_io) cudaFreeHost(ctx->h_io);
    if (ctx->h_slots) cudaFreeHost(ctx->h_slots);
    if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
    delete ctx;
}

const char* mrl_last_error(const mrl_ctx* ctx) { return ctx ? ctx->err.c_str() : "no context"; }

void* mrl_ctx_stream(mrl_ctx* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

int mrl_ctx_set_stream(mrl_ctx* ctx, void* stream) {
    if (!ctx) return MRL_ERR_INVALID;
    ctx->stream = stream ? (cudaStream_t)stream : ctx->own_stream;
    return MRL_OK;
}

int mrl_segment_upload(mrl_ctx* ctx, const uint8_t* blocks, uint64_t n_blocks, uint32_t block_id_base, mrl_seg** out) {
    if (!ctx || !out) return MRL_ERR_INVALID;
    *out = nullptr;
    if (n_blocks && !blocks) return fail(ctx, MRL_ERR_INVALID, "blocks is NULL");
    if (n_blocks >= (1ull << 26)) return fail(ctx, MRL_ERR_INVALID, "segment larger than 2^26 pages");
    if ((uint64_t)block_id_base + n_blocks > (1ull << 32)) return fail(ctx, MRL_ERR_INVALID, "block ids overflow u32");
    if (int rc = set_device(ctx)) return rc;
    mrl_seg* s = nullptr;
    if (int rc = seg_new(ctx, block_id_base, &s)) return rc;
    if (int rc = seg_reserve(ctx, s, n_blocks ? n_blocks : 1)) { mrl_segment_free(ctx, s); return rc; }
    const uint64_t chunk = 16384;  // pages per staging copy (64 MiB)
    if (n_blocks) {
        if (int rc = ensure_tmp(ctx, std::min<uint64_t>(n_blocks, chunk) * mrl::kBlockBytes)) { mrl_segment_free(ctx, s); return rc; }
        for (uint64_t b0 = 0; b0 < n_blocks; b0 += chunk) {
            const uint64_t nb = std::min<uint64_t>(chunk, n_blocks - b0);
            cudaError_t e = cudaMemcpyAsync(ctx->tmp, blocks + b0 * mrl::kBlockBytes, nb * mrl::kBlockBytes,
                                            cudaMemcpyHostToDevice, ctx->stream);
            if (e != cudaSuccess) { mrl_segment_free(ctx, s); return cuda_fail(ctx, e, "upload copy"); }
            if (mrl::launch_transcode((const uint8_t*)ctx->tmp, nb, s->pages + b0 * 256, s->ts + b0, ctx->stream)) {
                mrl_segment_free(ctx, s);
                return cuda_fail(ctx, cudaGetLastError(), "transcode launch");
            }
        }
        if (int rc = seg_note_pages(ctx, s, 0, n_blocks)) { mrl_segment_free(ctx, s); return rc; }
    }
    const cudaError_t e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) { mrl_segment_free(ctx, s); return cuda_fail(ctx, e, "segment upload"); }
    s->n_blocks = n_blocks;
    *out = s;
    return MRL_OK;
}

int mrl_segment_load(mrl_ctx* ctx, const char* path, uint32_t block_id_base, mrl_seg** out) {
    if (!ctx || !path || !out) return MRL_ERR_INVALID;
    *out = nullptr;
    FILE* f = std::fopen(path, "rb");
    if (!f) return fail(ctx, MRL_ERR_INVALID, std::string("io: cannot open ") + path);
    std::fseek(f, 0, SEEK_END);
    const long long size = std::ftell(f);
    std::fseek(f, 0, SEEK_SET);
    if (size < 0) { std::fclose(f); return fail(ctx, MRL_ERR_INVALID, std::string("io: cannot size ") + path); }
    if (size % mrl::kBlockBytes) {  // SegmentError::CorruptSize (src/segment.rs:17)
        std::fclose(f);
        return fail(ctx, MRL_ERR_INVALID, "corrupt segment size " + std::to_string(size) + " (not multiple of 4096)");
    }
    const uint64_t n_blocks = (uint64_t)size / mrl::kBlockBytes;
    if (n_blocks >= (1ull << 26)) { std::fclose(f); return fail(ctx, MRL_ERR_INVALID, "segment larger than 2^26 pages"); }
    if ((uint64_t)block_id_base + n_blocks > (1ull << 32)) { std::fclose(f); return fail(ctx, MRL_ERR_INVALID, "block ids overflow u32"); }
    if (int rc = set_device(ctx)) { std::fclose(f); return rc; }
    mrl_seg* s = nullptr;
    if (int rc = seg_new(ctx, block_id_base, &s)) { std::fclose(f); return rc; }
    if (int rc = seg_reserve(ctx, s, n_blocks ? n_blocks : 1)) { std::fclose(f); mrl_segment_free(ctx, s); return rc; }
    // Two pinned host buffers and two device staging buffers: the file read of chunk c+1 overlaps
    // the copy and transcode of chunk c.
    const uint64_t chunk = 16384;  // pages (64 MiB)
    const size_t cb = (size_t)std::min<uint64_t>(n_blocks ? n_blocks : 1, chunk) * mrl::kBlockBytes;
    uint8_t* host[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    int rc = ensure_tmp(ctx, 2 * cb);
    for (int i = 0; i < 2 && rc == MRL_OK; ++i) {
        if (cudaHostAlloc((void**)&host[i], cb, cudaHostAllocDefault) != cudaSuccess) rc = fail(ctx, MRL_ERR_NOMEM, "cudaHostAlloc staging");
        else if (cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming) != cudaSuccess) rc = fail(ctx, MRL_ERR_CUDA, "event");
    }
    for (uint64_t b0 = 0, c = 0; rc == MRL_OK && b0 < n_blocks; b0 += chunk, ++c) {
        const int i = (int)(c & 1);
        const uint64_t nb = std::min<uint64_t>(chunk, n_blocks - b0);
        if (c >= 2 && cudaEventSynchronize(done[i]) != cudaSuccess) { rc = fail(ctx, MRL_ERR_CUDA, "staging wait"); break; }
        if (std::fread(host[i], mrl::kBlockBytes, nb, f) != nb) { rc = fail(ctx, MRL_ERR_INVALID, std::string("io: short read ") + path); break; }
        uint8_t* dst = static_cast<uint8_t*>(ctx->tmp) + (size_t)i * cb;
        cudaError_t e = cudaMemcpyAsync(dst, host[i], nb * mrl::kBlockBytes, cudaMemcpyHostToDevice, ctx->stream);
        if (e != cudaSuccess) { rc = cuda_fail(ctx, e, "segment upload copy"); break; }
        if (mrl::launch_transcode(dst, nb, s->pages + b0 * 256, s->ts + b0, ctx->stream)) {
            rc = cuda_fail(ctx, cudaGetLastError(), "transcode launch");
            break;
        }
        if (cudaEventRecord(done[i], ctx->stream) != cudaSuccess) { rc = fail(ctx, MRL_ERR_CUDA, "event record"); break; }
    }
    std::fclose(f);
    if (rc == MRL_OK) rc = seg_note_pages(ctx, s, 0, n_blocks);
    const cudaError_t se = cudaStreamSynchronize(ctx->stream);
    if (rc == MRL_OK && se != cudaSuccess) rc = cuda_fail(ctx, se, "segment load");
    for (int i = 0; i < 2; ++i) {
        if (host[i]) cudaFreeHost(host[i]);
        if (done[i]) cudaEventDestroy(done[i]);
    }
    if (rc != MRL_OK) { mrl_segment_free(ctx, s); return rc; }
    s->n_blocks = n_blocks;
    *out = s;
    return MRL_OK;
}

int mrl_segment_append(mrl_ctx* ctx, mrl_seg* seg, const uint8_t* block4096) {
    if (!ctx || !seg || !block4096) return MRL_ERR_INVALID;
    if (seg->n_blocks + 1 >= (1ull << 26)) return fail(ctx, MRL_ERR_INVALID, "segment larger than 2^26 pages");
    if (int rc = set_device(ctx)) return rc;
    if (int rc = seg_reserve(ctx, seg, seg->n_blocks + 1)) return rc;
    if (int rc = ensure_tmp(ctx, mrl::kBlockBytes)) return rc;
    MRL_CUDA_TRY(ctx, cudaMemcpyAsync(ctx->tmp, block4096, mrl::kBlockBytes, cudaMemcpyHostToDevice, ctx->stream));
    if (mrl::launch_transcode((const uint8_t*)ctx->tmp, 1, seg->pages + seg->n_blocks * 256, seg->ts + seg->n_blocks, ctx->stream))
        return cuda_fail(ctx, cudaGetLastError(), "transcode launch");
    if (int rc = seg_note_pages(ctx, seg, seg->n_blocks, 1)) return rc;
    MRL_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    seg->n_blocks += 1;
    return MRL_OK;
}

int mrl_segment_append_device(mrl_ctx* ctx, mrl_seg* seg, const uint8_t* d_blocks, uint64_t n_blocks) {
    if (!ctx || !seg || (n_blocks && !d_blocks)) return MRL_ERR_INVALID;
    if (seg->n_blocks + n_blocks >= (1ull << 26)) return fail(ctx, MRL_ERR_INVALID, "segment larger than 2^26 pages");
    if (n_blocks == 0) return MRL_OK;
    if (int rc = set_device(ctx)) return rc;
    if (int rc = seg_reserve(ctx, seg, seg->n_blocks + n_blocks)) return rc;
    if (mrl::launch_transcode(d_blocks, n_blocks, seg->pages + seg->n_blocks * 256, seg->ts + seg->n_blocks, ctx->stream))
        return cuda_fail(ctx, cudaGetLastError(), "transcode launch");
    if (int rc = seg_note_pages(ctx, seg, seg->n_blocks, n_blocks)) return rc;
    seg->n_blocks += n_blocks;
    return MRL_OK;
}

int mrl_segment_free(mrl_ctx* ctx, mrl_seg* seg) {
    if (!seg) return MRL_OK;
    if (ctx) cudaSetDevice(ctx->device);
    cudaFree(seg->pages);
    cudaFree(seg->ts);
    cudaFree(seg->metamax);
    delete seg;
    return MRL_OK;
}

uint64_t mrl_segment_blocks(const mrl_seg* seg) { return seg ? seg->n_blocks : 0; }

int mrl_segment_device_ptrs(const mrl_seg* seg, void** pages, void** block_ts) {
    if (!seg) return MRL_ERR_INVALID;
    if (pages) *pages = seg->pages;
    if (block_ts) *block_ts = seg->ts;
    return MRL_OK;
}

int mrl_segment_read_layout(mrl_ctx* ctx, const mrl_seg* seg, uint8_t* out_pages, uint32_t* out_ts) {
    if (!ctx || !seg) return MRL_ERR_INVALID;
    if (int rc = set_device(ctx)) return rc;
    if (out_pages && seg->n_blocks)
        MRL_CUDA_TRY(ctx, cudaMemcpyAsync(out_pages, seg->pages, seg->n_blocks * mrl::kBlockBytes, cudaMemcpyDeviceToHost, ctx->stream));
    if (out_ts && seg->n_blocks)
        MRL_CUDA_TRY(ctx, cudaMemcpyAsync(out_ts, seg->ts, seg->n_blocks * sizeof(uint2), cudaMemcpyDeviceToHost, ctx->stream));
    MRL_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    return MRL_OK;
}

int mrl_plans_alloc(mrl_ctx* ctx, uint32_t n_q, uint32_t dims, mrl_plans** out) {
    if (!ctx || !out) return MRL_ERR_INVALID;
    *out = nullptr;
    if (dims < 192) return fail(ctx, MRL_ERR_INVALID, "dims must be >= 192 (src/scan.rs:114)");
    if (dims > 16384) return fail(ctx, MRL_ERR_INVALID, "dims must be <= 16384");
    if (int rc = set_device(ctx)) return rc;
    mrl_plans* p = new mrl_plans();
    p->n_q = n_q;
    p->dims = dims;
    if (n_q && cudaMalloc(&p->d, sizeof(mrl::DevPlan) * (size_t)n_q) != cudaSuccess) {
        delete p;
        return fail(ctx, MRL_ERR_NOMEM, "cudaMalloc plans");
    }
    *out = p;
    return MRL_OK;
}

int mrl_plan_build_device(mrl_ctx* ctx, const float* d_queries, uint32_t n_q, uint32_t dims,
                          const mrl_codec_desc* codec, mrl_plans* plans) {
    if (!ctx || !plans) return MRL_ERR_INVALID;
    if (int rc = check_codec(ctx, codec)) return rc;
    if (n_q > plans->n_q || dims != plans->dims) return fail(ctx, MRL_ERR_INVALID, "plan storage too small or dims mismatch");
    if (n_q == 0) return MRL_OK;
    if (int rc = set_device(ctx)) return rc;
    float* d_means = nullptr;
    if (int rc = upload_means(ctx, codec, &d_means)) return rc;
    if (mrl::launch_plan_build(d_queries, n_q, dims, codec->prefix_codec, codec->mid_codec, d_means, codec->eden_seed,
                               codec->mid_codec == MRL_MID_EDEN_B1 ? d_means + 64 : nullptr, codec->mid_seed,
                               plans->d, ctx->stream))
        return cuda_fail(ctx, cudaGetLastError(), "plan launch");
    return MRL_OK;
}

int mrl_plan_build(mrl_ctx* ctx, const float* queries, uint32_t n_q, uint32_t dims, const mrl_codec_desc* codec,
                   mrl_plans** out) {
    if (!ctx || !out) return MRL_ERR_INVALID;
    *out = nullptr;
    if (n_q && !queries) return fail(ctx, MRL_ERR_INVALID, "queries is NULL");
    if (int rc = check_codec(ctx, codec)) return rc;
    for (uint64_t i = 0; i < (uint64_t)n_q * dims; ++i)
        if (!std::isfinite(queries[i])) return fail(ctx, MRL_ERR_INVALID, "query contains a non-finite value");
    mrl_plans* p = nullptr;
    if (int rc = mrl_plans_alloc(ctx, n_q, dims, &p)) return rc;
    const size_t qbytes = (size_t)n_q * dims * sizeof(float);
    if (int rc = ensure_tmp(ctx, qbytes)) { mrl_plans_free(ctx, p); return rc; }
    float* d_means = nullptr;
    float* d_q = (float*)ctx->tmp;
    if (qbytes) {
        cudaError_t e = cudaMemcpyAsync(d_q, queries, qbytes, cudaMemcpyHostToDevice, ctx->stream);
        if (e != cudaSuccess) { mrl_plans_free(ctx, p); return cuda_fail(ctx, e, "query copy"); }
    }
    if (int rc = upload_means(ctx, codec, &d_means)) { mrl_plans_free(ctx, p); return rc; }
    if (n_q && mrl::launch_plan_build(d_q, n_q, dims, codec->prefix_codec, codec->mid_codec, d_means, codec->eden_seed,
                                      codec->mid_codec == MRL_MID_EDEN_B1 ? d_means + 64 : nullptr, codec->mid_seed, p->d,
                                      ctx->stream)) {
        mrl_plans_free(ctx, p);
        return cuda_fail(ctx, cudaGetLastError(), "plan launch");
    }
    const cudaError_t e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) { mrl_plans_free(ctx, p); return cuda_fail(ctx, e, "plan build"); }
    *out = p;
    return MRL_OK;
}

int mrl_plan_rebuild(mrl_ctx* ctx, const float* queries, uint32_t n_q, uint32_t dims, const mrl_codec_desc* codec,
                     mrl_plans* plans) {
    if (!ctx || !plans) return MRL_ERR_INVALID;
    if (n_q && !queries) return fail(ctx, MRL_ERR_INVALID, "queries is NULL");
    if (int rc = check_codec(ctx, codec)) return rc;
    if (n_q > plans->n_q || dims != plans->dims) return fail(ctx, MRL_ERR_INVALID, "plan storage too small or dims mismatch");
    for (uint64_t i = 0; i < (uint64_t)n_q * dims; ++i)
        if (!std::isfinite(queries[i])) return fail(ctx, MRL_ERR_INVALID, "query contains a non-finite value");
    if (n_q == 0) return MRL_OK;
    if (int rc = set_device(ctx)) return rc;
    const size_t qbytes = (size_t)n_q * dims * sizeof(float);
    if (int rc = ensure_tmp(ctx, qbytes)) return rc;
    float* d_means = nullptr;
    float* d_q = (float*)ctx->tmp;
    MRL_CUDA_TRY(ctx, cudaMemcpyAsync(d_q, queries, qbytes, cudaMemcpyHostToDevice, ctx->stream));
    if (int rc = upload_means(ctx, codec, &d_means)) return rc;
    if (mrl::launch_plan_build(d_q, n_q, dims, codec->prefix_codec, codec->mid_codec, d_means, codec->eden_seed,
                               codec->mid_codec == MRL_MID_EDEN_B1 ? d_means + 64 : nullptr, codec->mid_seed, plans->d,
                               ctx->stream))
        return cuda_fail(ctx, cudaGetLastError(), "plan launch");
    return MRL_OK;
}

int mrl_plans_free(mrl_ctx* ctx, mrl_plans* plans) {
    if (!plans) return MRL_OK;
    if (ctx) cudaSetDevice(ctx->device);
    cudaFree(plans->d);
    delete plans;
    return MRL_OK;
}

int mrl_plan_read(mrl_ctx* ctx, const mrl_plans* plans, uint32_t i, mrl_query_plan* out) {
    if (!ctx || !plans || !out) return MRL_ERR_INVALID;
    if (i >= plans->n_q) return fail(ctx, MRL_ERR_INVALID, "plan index out of range");
    if (int rc = set_device(ctx)) return rc;
    MRL_CUDA_TRY(ctx, cudaMemcpyAsync(out, &plans->d[i].qp, sizeof(mrl_query_plan), cudaMemcpyDeviceToHost, ctx->stream));
    MRL_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    return MRL_OK;
}

int mrl_scan_device(mrl_ctx* ctx, const mrl_seg* seg, const mrl_plans* plans, uint32_t q0, uint32_t n_q,
                    const mrl_scan_cfg* cfg, const uint32_t* time_lo, const uint32_t* time_hi, uint64_t* d_out_ids,
                    float* d_out_scores, uint32_t* d_out_counts, uint32_t* d_out_status) {
    if (!ctx || !seg || !plans) return MRL_ERR_INVALID;
    if (int rc = check_cfg(ctx, cfg, plans->dims)) return rc;
    if ((uint64_t)q0 + n_q > plans->n_q) return fail(ctx, MRL_ERR_INVALID, "plan range out of bounds");
    if (n_q && (!d_out_ids || !d_out_scores || !d_out_counts)) return fail(ctx, MRL_ERR_INVALID, "output is NULL");
    if (int rc = set_device(ctx)) return rc;
    if (int rc = ensure_owner(ctx, seg->n_blocks)) return rc;
    const uint32_t k = cfg->shortlist_cand;
    for (uint32_t i = 0; i < n_q; ++i) {
        mrl::ScanLaunch p = make_launch(ctx, seg, plans, q0 + i, cfg, time_lo, time_hi);
        p.out_ids = d_out_ids + (size_t)i * k;
        p.out_scores = d_out_scores + (size_t)i * k;
        p.out_count = d_out_counts + i;
        p.out_status = d_out_status ? d_out_status + i : nullptr;
        if (seg->n_blocks == 0) {
            MRL_CUDA_TRY(ctx, cudaMemsetAsync(p.out_count, 0, sizeof(uint32_t), ctx->stream));
            if (p.out_status) MRL_CUDA_TRY(ctx, cudaMemsetAsync(p.out_status, 0, sizeof(uint32_t), ctx->stream));
            continue;
        }
        take_scratch(ctx, p);
        if (mrl::launch_scan(p, scan_grid(ctx), ctx->stream, true)) return cuda_fail(ctx, cudaGetLastError(), "scan launch");
        launched(ctx);
    }
    return MRL_OK;
}

int mrl_scan_batch_device(mrl_ctx* ctx, const mrl_seg* seg, const mrl_plans* plans, uint32_t q0, uint32_t n_q,
                          const mrl_scan_cfg* cfg, const uint32_t* time_lo, const uint32_t* time_hi,
                          uint64_t* d_out_ids, float* d_out_scores, uint32_t* d_out_counts, uint32_t* d_out_status) {
    if (!ctx || !seg || !plans) return MRL_ERR_INVALID;
    if (int rc = check_cfg(ctx, cfg, plans->dims)) return rc;
    if ((uint64_t)q0 + n_q > plans->n_q) return fail(ctx, MRL_ERR_INVALID, "plan range out of bounds");
    if (n_q && (!d_out_ids || !d_out_scores || !d_out_counts)) return fail(ctx, MRL_ERR_INVALID, "output is NULL");
    if (n_q == 0) return MRL_OK;
    if (cfg->mode != MRL_MODE_FAST || cfg->strata_depth == MRL_DEPTH_L0 || seg->n_blocks == 0)
        return mrl_scan_device(ctx, seg, plans, q0, n_q, cfg, time_lo, time_hi, d_out_ids, d_out_scores, d_out_counts,
                               d_out_status);
    if (int rc = set_device(ctx)) return rc;
    const uint32_t ctas = (uint32_t)ctx->sms;
    if (int rc = ensure_buf(ctx, &ctx->bbuf, &ctx->bbuf_bytes, mrl::batch_scratch_bytes(ctas, n_q))) return rc;
    const bool use_time = cfg->temporal_filter_enable && (time_lo || time_hi);
    if (mrl::launch_scan_batch(seg->pages, seg->ts, (uint32_t)seg->n_blocks, seg->block_id_base, seg->metamax,
                               plans->d + q0, n_q,
                               cfg->shortlist_cand, cfg->stratum4_weight, cfg->strata_depth, use_time ? 1u : 0u,
                               time_lo ? 1u : 0u, time_lo ? *time_lo : 0u, time_hi ? 1u : 0u, time_hi ? *time_hi : 0u,
                               ctas, ctx->batch_engine, ctx->bbuf, d_out_ids, d_out_scores, d_out_counts, d_out_status,
                               ctx->stream))
        return cuda_fail(ctx, cudaGetLastError(), "batched scan launch");
    return MRL_OK;
}

// mrl_scan_device with the scan scratch taken from g_static_scan_scratch instead of the context's
// buffers: on success it allocates no device or host memory. It is for callers that must not
// allocate while answering a query, such as a serving process that reserved its device memory at
// start-up, where a cudaMalloc could stall other streams or fail under memory pressure mid-request.
// Of the scratch, only the control words must be zero when a launch starts; every completed scan
// leaves them zero, and each call also zeroes them (one memset on the context stream) so a call
// after a wait that ran out starts clean. Lists, flags and owner bytes are written before they
// are read. The scratch is one per device per process, so two calls in flight on the same device
// at once (different streams, contexts or threads) race on it; calls ordered on one stream do not.
int mrl_scan_device_static(mrl_ctx* ctx, const mrl_seg* seg, const mrl_plans* plans, uint32_t q0, uint32_t n_q,
                           const mrl_scan_cfg* cfg, const uint32_t* time_lo, const uint32_t* time_hi,
                           uint64_t* d_out_ids, float* d_out_scores, uint32_t* d_out_counts,
                           uint32_t* d_out_status) {
    if (!ctx || !seg || !plans) return MRL_ERR_INVALID;
    if (int rc = check_cfg(ctx, cfg, plans->dims)) return rc;
    if ((uint64_t)q0 + n_q > plans->n_q) return fail(ctx, MRL_ERR_INVALID, "plan range out of bounds");
    if (n_q && (!d_out_ids || !d_out_scores || !d_out_counts)) return fail(ctx, MRL_ERR_INVALID, "output is NULL");
    if (seg->n_blocks > MRL_STATIC_MAX_BLOCKS)
        return fail(ctx, MRL_ERR_INVALID,
                    "segment has " + std::to_string(seg->n_blocks) +
                        " pages; mrl_scan_device_static's static scratch holds at most " +
                        std::to_string(MRL_STATIC_MAX_BLOCKS) + " (use mrl_scan_device)");
    if ((uint32_t)ctx->sms > MRL_STATIC_MAX_CTAS)
        return fail(ctx, MRL_ERR_INVALID,
                    "device has " + std::to_string(ctx->sms) + " SMs; mrl_scan_device_static's static scratch holds at most " +
                        std::to_string(MRL_STATIC_MAX_CTAS) + " CTA lists (use mrl_scan_device)");
    if (int rc = set_device(ctx)) return rc;
    unsigned char* base = nullptr;
    if (int rc = static_scratch(ctx, &base)) return rc;
    MRL_CUDA_TRY(ctx, cudaMemsetAsync(base + kStaticCtlOff, 0, sizeof(unsigned) * mrl::kCtlWords, ctx->stream));
    const uint32_t k = cfg->shortlist_cand;
    for (uint32_t i = 0; i < n_q; ++i) {
        mrl::ScanLaunch p = make_launch(ctx, seg, plans, q0 + i, cfg, time_lo, time_hi);
        p.cta_keys = reinterpret_cast<unsigned long long*>(base + kStaticKeysOff);
        p.cta_xkeys = reinterpret_cast<unsigned long long*>(base + kStaticXKeysOff);
        p.ctl = reinterpret_cast<unsigned int*>(base + kStaticCtlOff);
        p.owner = base + kStaticOwnerOff;
        p.out_ids = d_out_ids + (size_t)i * k;
        p.out_scores = d_out_scores + (size_t)i * k;
        p.out_count = d_out_counts + i;
        p.out_status = d_out_status ? d_out_status + i : nullptr;
        if (seg->n_blocks == 0) {
            MRL_CUDA_TRY(ctx, cudaMemsetAsync(p.out_count, 0, sizeof(uint32_t), ctx->stream));
            if (p.out_status) MRL_CUDA_TRY(ctx, cudaMemsetAsync(p.out_status, 0, sizeof(uint32_t), ctx->stream));
            continue;
        }
        // an ordinary launch (no programmatic dependent launch): every call shares the one region
        if (mrl::launch_scan(p, scan_grid(ctx), ctx->stream, false)) return cuda_fail(ctx, cudaGetLastError(), "scan launch");
    }
    return MRL_OK;
}

int mrl_scan_blocks_stats(mrl_ctx* ctx, const mrl_seg* seg, const mrl_plans* plans, uint32_t q, const mrl_scan_cfg* cfg,
                   const uint32_t* time_lo, const uint32_t* time_hi, uint64_t* out_ids, float* out_scores,
                   uint32_t* out_count, mrl_scan_stats* stats) {
    if (!ctx || !seg || !plans || !out_ids || !out_scores || !out_count) return MRL_ERR_INVALID;
    if (int rc = check_cfg(ctx, cfg, plans->dims)) return rc;
    if (q >= plans->n_q) return fail(ctx, MRL_ERR_INVALID, "plan index out of range");
    if (int rc = set_device(ctx)) return rc;
    const uint32_t k = cfg->shortlist_cand;
    const size_t ids_b = (size_t)k * sizeof(uint64_t), sc_off = (ids_b + 255) & ~(size_t)255;
    const size_t cnt_off = (sc_off + (size_t)k * sizeof(float) + 255) & ~(size_t)255, tot_off = cnt_off + 256;
    if (int rc = ensure_out(ctx, tot_off + sizeof(mrl_scan_stats))) return rc;
    unsigned char* base = static_cast<unsigned char*>(ctx->tmp_out);
    uint64_t* d_ids = reinterpret_cast<uint64_t*>(base);
    float* d_sc = reinterpret_cast<float*>(base + sc_off);
    uint32_t* d_cnt = reinterpret_cast<uint32_t*>(base + cnt_off);
    unsigned long long* d_tot = reinterpret_cast<unsigned long long*>(base + tot_off);
    if (int rc = mrl_scan_device(ctx, seg, plans, q, 1, cfg, time_lo, time_hi, d_ids, d_sc, d_cnt, nullptr)) return rc;
    if (stats) {
        if (seg->n_blocks) {
            if (mrl::launch_scan_stats(make_launch(ctx, seg, plans, q, cfg, time_lo, time_hi), cfg->cs_tolerance, d_cnt,
                                       d_sc, d_tot, ctx->stream))
                return cuda_fail(ctx, cudaGetLastError(), "stats launch");
            MRL_CUDA_TRY(ctx, cudaMemcpyAsync(stats, d_tot, sizeof(mrl_scan_stats), cudaMemcpyDeviceToHost, ctx->stream));
        } else {
            std::memset(stats, 0, sizeof(mrl_scan_stats));
        }
    }
    MRL_CUDA_TRY(ctx, cudaMemcpyAsync(out_count, d_cnt, sizeof(uint32_t), cudaMemcpyDeviceToHost, ctx->stream));
    MRL_CUDA_TRY(ctx, cudaMemcpyAsync(out_ids, d_ids, ids_b, cudaMemcpyDeviceToHost, ctx->stream));
    MRL_CUDA_TRY(ctx, cudaMemcpyAsync(out_scores, d_sc, (size_t)k * sizeof(float), cudaMemcpyDeviceToHost, ctx->stream));
    MRL_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    return MRL_OK;
}

int mrl_query_scan_device(mrl_ctx* ctx, const mrl_seg* seg, const float* d_queries, uint32_t n_q, uint32_t dims,
                          const mrl_codec_desc* codec, mrl_plans* plans, const mrl_scan_cfg* cfg,
                          const uint32_t* time_lo, const uint32_t* time_hi, uint64_t* d_out_ids, float* d_out_scores,
                          uint32_t* d_out_counts, uint32_t* d_out_status) {
    if (!ctx || !seg || !plans) return MRL_ERR_INVALID;
    if (int rc = check_cfg(ctx, cfg, dims)) return rc;
    if (int rc = check_codec(ctx, codec)) return rc;
    if (n_q > plans->n_q || dims != plans->dims) return fail(ctx, MRL_ERR_INVALID, "plan storage too small or dims mismatch");
    if (n_q && (!d_queries || !d_out_ids || !d_out_scores || !d_out_counts)) return fail(ctx, MRL_ERR_INVALID, "buffer is NULL");
    if (n_q == 0) return MRL_OK;
    if (int rc = set_device(ctx)) return rc;
    if (int rc = ensure_owner(ctx, seg->n_blocks)) return rc;
    float* d_means = nullptr;
    if (int rc = upload_means(ctx, codec, &d_means)) return rc;
    const float* d_mid = codec->mid_codec == MRL_MID_EDEN_B1 ? d_means + 64 : nullptr;
    const uint32_t k = cfg->shortlist_cand;
    for (uint32_t i = 0; i < n_q; ++i) {
        mrl::ScanLaunch p = make_launch(ctx, seg, plans, i, cfg, time_lo, time_hi);
        p.out_ids = d_out_ids + (size_t)i * k;
        p.out_scores = d_out_scores + (size_t)i * k;
        p.out_count = d_out_counts + i;
        p.out_status = d_out_status ? d_out_status + i : nullptr;
        if (seg->n_blocks == 0) {  // nothing to scan: build the plan alone
            if (mrl::launch_plan_build(d_queries + (size_t)i * dims, 1, dims, codec->prefix_codec, codec->mid_codec,
                                       d_means, codec->eden_seed, d_mid, codec->mid_seed, plans->d + i, ctx->stream))
                return cuda_fail(ctx, cudaGetLastError(), "plan launch");
            MRL_CUDA_TRY(ctx, cudaMemsetAsync(p.out_count, 0, sizeof(uint32_t), ctx->stream));
            if (p.out_status) MRL_CUDA_TRY(ctx, cudaMemsetAsync(p.out_status, 0, sizeof(uint32_t), ctx->stream));
            continue;
        }
        p.query = d_queries + (size_t)i * dims;
        p.dims = dims;
        p.prefix_codec = codec->prefix_codec;
        p.mid_codec = codec->mid_codec;
        p.eden_mean = d_means;
        p.eden_seed = codec->eden_seed;
        p.mid_mean = d_mid;
        p.mid_seed = codec->mid_seed;
        p.plan_out = plans->d + i;
        take_scratch(ctx, p);
        if (mrl::launch_scan(p, scan_grid(ctx), ctx->stream, true)) return cuda_fail(ctx, cudaGetLastError(), "scan launch");
        launched(ctx);
    }
    return MRL_OK;
}

// mrl_query_scan for queries a launch cannot carry (dims > kInlineQueryMax) or an empty segment:
// the queries go to the device from the context's pinned staging, and the results come back into it.
static int query_scan_staged(mrl_ctx* ctx, const mrl_seg* seg, const float* queries, uint32_t n_q, uint32_t dims,
                             const mrl_codec_desc* codec, mrl_plans* plans, const mrl_scan_cfg* cfg,
                             const uint32_t* time_lo, const uint32_t* time_hi, uint64_t* out_ids, float* out_scores,
                             uint32_t* out_counts) {
    const size_t qbytes = (size_t)n_q * dims * sizeof(float);
    const size_t nk = (size_t)n_q * cfg->shortlist_cand;
    const size_t o_off = (qbytes + 255) & ~(size_t)255;
    const size_t obytes = nk * (sizeof(uint64_t) + sizeof(float)) + 2 * sizeof(uint32_t) * n_q;
    if (int rc = ensure_host_io(ctx, o_off + obytes)) return rc;
    if (int rc = ensure_tmp(ctx, qbytes)) return rc;
    float* h_q = static_cast<float*>(ctx->h_io);
    for (uint64_t i = 0; i < (uint64_t)n_q * dims; ++i) {
        const float v = queries[i];
        if (!std::isfinite(v)) return fail(ctx, MRL_ERR_INVALID, "query contains a non-finite value");
        h_q[i] = v;
    }
    // results: in the mapped staging when there are pages to scan (the scan stores them there);
    // an empty segment clears the counts with device memsets, so its results go to device scratch
    const bool mapped = seg->n_blocks > 0;
    if (!mapped)
        if (int rc = ensure_out(ctx, obytes + 64)) return rc;
    unsigned char* h_out = static_cast<unsigned char*>(ctx->h_io) + o_off;
    unsigned char* d_out = mapped ? static_cast<unsigned char*>(ctx->h_io_dev) + o_off
                                  : static_cast<unsigned char*>(ctx->tmp_out);
    float* d_q = (float*)ctx->tmp;
    uint64_t* d_ids = reinterpret_cast<uint64_t*>(d_out);
    float* d_sc = reinterpret_cast<float*>(d_out + nk * sizeof(uint64_t));
    uint32_t* d_cnt = reinterpret_cast<uint32_t*>(d_out + nk * (sizeof(uint64_t) + sizeof(float)));
    uint32_t* d_st = d_cnt + n_q;
    MRL_CUDA_TRY(ctx, cudaMemcpyAsync(d_q, h_q, qbytes, cudaMemcpyHostToDevice, ctx->stream));
    if (int rc = mrl_query_scan_device(ctx, seg, d_q, n_q, dims, codec, plans, cfg, time_lo, time_hi, d_ids, d_sc, d_cnt,
                                       d_st))
        return rc;
    if (!mapped)
        MRL_CUDA_TRY(ctx, cudaMemcpyAsync(h_out, d_out, obytes, cudaMemcpyDeviceToHost, ctx->stream));
    MRL_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    const uint32_t* cs = reinterpret_cast<const uint32_t*>(h_out + nk * (sizeof(uint64_t) + sizeof(float)));
    for (uint32_t q = 0; q < n_q; ++q)
        if (cs[n_q + q] & 10u) return fail(ctx, MRL_ERR_CUDA, "scan: a bounded wait ran out (status bits 1/3)");
    std::memcpy(out_ids, h_out, nk * sizeof(uint64_t));
    std::memcpy(out_scores, h_out + nk * sizeof(uint64_t), nk * sizeof(float));
    std::memcpy(out_counts, cs, n_q * sizeof(uint32_t));
    return MRL_OK;
}

namespace {

// Result slot layout (bytes) for shortlists up to k: ids k*8 | scores k*4 | count | status |
// completion word.
size_t slot_stride_for(uint32_t k) { return ((size_t)k * 12 + 12 + 255) & ~(size_t)255; }

int ensure_slots(mrl_ctx* ctx, uint32_t k) {
    if (ctx->slot_k >= k && ctx->h_slots) return MRL_OK;
    for (int s = 0; s < MRL_MAX_INFLIGHT; ++s)
        if (ctx->slot_busy[s]) return fail(ctx, MRL_ERR_INVALID, "a larger shortlist_cand needs every query slot collected first");
    if (ctx->h_slots) cudaFreeHost(ctx->h_slots);
    ctx->h_slots = ctx->d_slots = nullptr;
    ctx->slot_k = 0;
    const size_t stride = slot_stride_for(k);
    void* h = nullptr;
    cudaError_t e = cudaHostAlloc(&h, stride * MRL_MAX_INFLIGHT, cudaHostAllocMapped | cudaHostAllocPortable);
    if (e != cudaSuccess) return fail(ctx, MRL_ERR_NOMEM, std::string("cudaHostAlloc query slots: ") + cudaGetErrorString(e));
    void* d = nullptr;
    e = cudaHostGetDevicePointer(&d, h, 0);
    if (e != cudaSuccess) {
        cudaFreeHost(h);
        return cuda_fail(ctx, e, "cudaHostGetDevicePointer query slots");
    }
    std::memset(h, 0, stride * MRL_MAX_INFLIGHT);
    ctx->h_slots = static_cast<unsigned char*>(h);
    ctx->d_slots = static_cast<unsigned char*>(d);
    ctx->slot_stride = stride;
    ctx->slot_k = k;
    for (int s = 0; s < MRL_MAX_INFLIGHT; ++s) ctx->slot_seq[s] = 0;
    return MRL_OK;
}

// The exchange's checks for a scan of cfg on ctx (mrl_query_scan_exchange, mrl_query_submit_exchange).
int check_exchange(mrl_ctx* ctx, const mrl_exchange* ex, const mrl_scan_cfg* cfg) {
    if (!ex->opened) return fail(ctx, MRL_ERR_INVALID, "exchange not opened");
    if (ex->device != ctx->device) return fail(ctx, MRL_ERR_INVALID, "exchange belongs to another device");
    if (cfg->shortlist_cand != ex->k) return fail(ctx, MRL_ERR_INVALID, "shortlist_cand differs from the exchange's k");
    if ((size_t)ex->world * ex->rb > 200 * 1024)
        return fail(ctx, MRL_ERR_INVALID, "k x world too large to merge in shared memory; use mrl_merge_topk");
    return MRL_OK;
}

// The exchange fields of the next scan launch on ctx: the next epoch's buffer parity, this rank's
// record and flag slots in every area, and the staged record of the launch's scratch set (free once
// the set's previous user has completed, which the launch waits for before its scoring loop).
// Call right before take_scratch.
void set_exchange(mrl_ctx* ctx, mrl_exchange* ex, mrl::ScanLaunch& p) {
    const uint32_t epoch = ++ex->epoch;
    const size_t parity = epoch & 1u;
    p.xch_world = ex->world;
    p.xch_rank = ex->rank;
    p.xch_epoch = epoch;
    for (uint32_t w = 0; w < ex->world; ++w) {
        p.xch_rec[w] = ex->area[w] + (parity * ex->world + ex->rank) * ex->rb;
        p.xch_flag[w] = reinterpret_cast<unsigned*>(ex->area[w] + ex->flags_off()) + parity * ex->world + ex->rank;
    }
    p.xch_recv = ex->local + parity * ex->world * ex->rb;
    p.xch_flag_in = reinterpret_cast<const unsigned*>(ex->local + ex->flags_off()) + parity * ex->world;
    p.xch_stage = ex->stage + (ctx->scan_seq % kScratchSets) * ex->rb;
}

// Submits one host query into `slot`; plan_out (device, may be NULL) receives its plan. With `ex`
// the slot receives the global top-k over every rank of the exchange.
int query_submit(mrl_ctx* ctx, const mrl_seg* seg, const float* query, uint32_t dims, const mrl_codec_desc* codec,
                 mrl::DevPlan* plan_out, const mrl_scan_cfg* cfg, const uint32_t* time_lo, const uint32_t* time_hi,
                 uint32_t slot, mrl_exchange* ex = nullptr) {
    if (!ctx || !seg || !query) return MRL_ERR_INVALID;
    if (int rc = check_cfg(ctx, cfg, dims)) return rc;
    if (int rc = check_codec(ctx, codec)) return rc;
    if (ex)
        if (int rc = check_exchange(ctx, ex, cfg)) return rc;
    if (slot >= MRL_MAX_INFLIGHT) return fail(ctx, MRL_ERR_INVALID, "slot >= MRL_MAX_INFLIGHT");
    if (ctx->slot_busy[slot]) return fail(ctx, MRL_ERR_INVALID, "slot still holds a query that was not collected");
    if (dims > mrl::kInlineQueryMax) return fail(ctx, MRL_ERR_INVALID, "dims > 1024: use mrl_query_scan_device");
    for (uint32_t i = 0; i < dims; ++i)
        if (!std::isfinite(query[i])) return fail(ctx, MRL_ERR_INVALID, "query contains a non-finite value");
    if (int rc = set_device(ctx)) return rc;
    if (int rc = ensure_slots(ctx, cfg->shortlist_cand)) return rc;
    const size_t kk = ctx->slot_k;  // the slots' layout
    unsigned char* h = ctx->h_slots + slot * ctx->slot_stride;
    unsigned char* d = ctx->d_slots + slot * ctx->slot_stride;
    const uint32_t expect = ++ctx->slot_seq[slot];
    if (seg->n_blocks == 0 && !ex) {  // nothing to scan (an exchange rank still takes part)
        volatile uint32_t* cs = reinterpret_cast<volatile uint32_t*>(h + kk * 12);
        cs[0] = 0u;
        cs[1] = 0u;
        cs[2] = expect;
        ctx->slot_busy[slot] = true;
        return MRL_OK;
    }
    if (int rc = ensure_owner(ctx, seg->n_blocks)) return rc;
    float* d_means = nullptr;
    if (int rc = upload_means(ctx, codec, &d_means)) return rc;
    mrl::ScanLaunch p = make_launch(ctx, seg, nullptr, 0, cfg, time_lo, time_hi);
    p.out_ids = reinterpret_cast<uint64_t*>(d);
    p.out_scores = reinterpret_cast<float*>(d + kk * 8);
    p.out_count = reinterpret_cast<uint32_t*>(d + kk * 12);
    p.out_status = p.out_count + 1;
    p.out_flag = p.out_count + 2;
    p.out_flag_val = expect;
    p.dims = dims;
    p.prefix_codec = codec->prefix_codec;
    p.mid_codec = codec->mid_codec;
    p.eden_mean = d_means;
    p.eden_seed = codec->eden_seed;
    p.mid_mean = codec->mid_codec == MRL_MID_EDEN_B1 ? d_means + 64 : nullptr;
    p.mid_seed = codec->mid_seed;
    p.plan_out = plan_out;
    if (ex) set_exchange(ctx, ex, p);
    take_scratch(ctx, p);
    if (mrl::launch_scan(p, scan_grid(ctx), ctx->stream, true, query)) return cuda_fail(ctx, cudaGetLastError(), "scan launch");
    launched(ctx);
    ctx->slot_busy[slot] = true;
    return MRL_OK;
}

// Waits (spinning on the slot's completion word, at most about 10 s) for the query in `slot`.
int query_collect(mrl_ctx* ctx, uint32_t slot, uint64_t* out_ids, float* out_scores, uint32_t* out_count) {
    if (!ctx) return MRL_ERR_INVALID;
    if (slot >= MRL_MAX_INFLIGHT || !ctx->slot_busy[slot]) return fail(ctx, MRL_ERR_INVALID, "slot holds no query");
    const size_t kk = ctx->slot_k;
    const unsigned char* h = ctx->h_slots + slot * ctx->slot_stride;
    const volatile uint32_t* cs = reinterpret_cast<const volatile uint32_t*>(h + kk * 12);
    const uint32_t expect = ctx->slot_seq[slot];
    const auto t0 = std::chrono::steady_clock::now();
    for (uint64_t it = 1; cs[2] != expect; ++it) {
        if ((it & 4095u) == 0u) {
            const cudaError_t e = cudaStreamQuery(ctx->stream);
            if (e != cudaSuccess && e != cudaErrorNotReady) {
                ctx->slot_busy[slot] = false;
                return cuda_fail(ctx, e, "scan (query slot)");
            }
            if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(10)) {
                ctx->slot_busy[slot] = false;
                return fail(ctx, MRL_ERR_CUDA, "query slot: no result within 10 s");
            }
        }
    }
    std::atomic_thread_fence(std::memory_order_acquire);
    ctx->slot_busy[slot] = false;
    const uint32_t n = cs[0], st = cs[1];
    if (st & 2u) return fail(ctx, MRL_ERR_CUDA, "scan: a CTA's list never arrived (waited about 1 s)");
    if (st & 4u) return fail(ctx, MRL_ERR_CUDA, "exchange: a rank's record never arrived (waited about 2-3 s)");
    if (st & 8u) return fail(ctx, MRL_ERR_CUDA, "scan: the context's scratch stayed busy (waited about 1 s)");
    if (out_count) *out_count = n;
    if (out_ids) std::memcpy(out_ids, h, (size_t)n * sizeof(uint64_t));
    if (out_scores) std::memcpy(out_scores, h + kk * 8, (size_t)n * sizeof(float));
    return MRL_OK;
}

}  // namespace

int mrl_query_submit(mrl_ctx* ctx, const mrl_seg* seg, const float* query, uint32_t dims, const mrl_codec_desc* codec,
                     const mrl_scan_cfg* cfg, const uint32_t* time_lo, const uint32_t* time_hi, uint32_t slot) {
    return query_submit(ctx, seg, query, dims, codec, nullptr, cfg, time_lo, time_hi, slot);
}

int mrl_query_collect(mrl_ctx* ctx, uint32_t slot, uint64_t* out_ids, float* out_scores, uint32_t* out_count) {
    return query_collect(ctx, slot, out_ids, out_scores, out_count);
}

int mrl_query_submit_exchange(mrl_ctx* ctx, const mrl_seg* seg, const float* query, uint32_t dims,
                              const mrl_codec_desc* codec, const mrl_scan_cfg* cfg, const uint32_t* time_lo,
                              const uint32_t* time_hi, mrl_exchange* ex, uint32_t slot) {
    if (!ex) return MRL_ERR_INVALID;
    return query_submit(ctx, seg, query, dims, codec, nullptr, cfg, time_lo, time_hi, slot, ex);
}

int mrl_query_scan(mrl_ctx* ctx, const mrl_seg* seg, const float* queries, uint32_t n_q, uint32_t dims,
                   const mrl_codec_desc* codec, mrl_plans* plans, const mrl_scan_cfg* cfg, const uint32_t* time_lo,
                   const uint32_t* time_hi, uint64_t* out_ids, float* out_scores, uint32_t* out_counts) {
    if (!ctx || !seg || !plans) return MRL_ERR_INVALID;
    if (int rc = check_cfg(ctx, cfg, dims)) return rc;
    if (n_q == 0) return MRL_OK;
    if (!queries || !out_ids || !out_scores || !out_counts) return fail(ctx, MRL_ERR_INVALID, "buffer is NULL");
    if (n_q > plans->n_q || dims != plans->dims) return fail(ctx, MRL_ERR_INVALID, "plan storage too small or dims mismatch");
    for (int s = 0; s < MRL_MAX_INFLIGHT; ++s)
        if (ctx->slot_busy[s]) return fail(ctx, MRL_ERR_INVALID, "mrl_query_scan while submitted queries are uncollected");
    if (dims > mrl::kInlineQueryMax || seg->n_blocks == 0)
        return query_scan_staged(ctx, seg, queries, n_q, dims, codec, plans, cfg, time_lo, time_hi, out_ids, out_scores,
                                 out_counts);
    // every query's scan is launched with the query in its parameters; up to MRL_MAX_INFLIGHT are
    // in flight, and each result is collected from its slot in order
    const size_t k = cfg->shortlist_cand;
    int rc = MRL_OK;
    uint32_t next = 0;  // next query to collect
    for (uint32_t i = 0; i < n_q && rc == MRL_OK; ++i) {
        const uint32_t slot = i % MRL_MAX_INFLIGHT;
        if (i >= MRL_MAX_INFLIGHT) {
            rc = query_collect(ctx, slot, out_ids + next * k, out_scores + next * k, out_counts + next);
            ++next;
            if (rc) break;
        }
        rc = query_submit(ctx, seg, queries + (size_t)i * dims, dims, codec, plans->d + i, cfg, time_lo, time_hi, slot);
    }
    for (; next < n_q; ++next) {  // drain (also after a failure, so no slot stays busy)
        const uint32_t slot = next % MRL_MAX_INFLIGHT;
        if (!ctx->slot_busy[slot]) continue;
        const int r = query_collect(ctx, slot, out_ids + next * k, out_scores + next * k, out_counts + next);
        if (rc == MRL_OK) rc = r;
    }
    return rc;
}

int mrl_exchange_create(mrl_ctx* ctx, uint32_t world, uint32_t rank, uint32_t k, void* ipc_handle,
                        mrl_exchange** out) {
    if (!ctx || !out) return MRL_ERR_INVALID;
    *out = nullptr;
    if (world < 1 || world > (uint32_t)mrl::kMaxRanks) return fail(ctx, MRL_ERR_INVALID, "world must be in [1, 8]");
    if (rank >= world) return fail(ctx, MRL_ERR_INVALID, "rank must be < world");
    if (k < 1 || k > 4096) return fail(ctx, MRL_ERR_INVALID, "k must be in [1, 4096]");
    if (world > 1 && !ipc_handle) return fail(ctx, MRL_ERR_INVALID, "ipc_handle is NULL");
    if (int rc = set_device(ctx)) return rc;
    mrl_exchange* ex = new mrl_exchange();
    ex->device = ctx->device;
    ex->world = world;
    ex->rank = rank;
    ex->k = k;
    ex->rb = MRL_MERGE_RECORD_BYTES(k);
    if (cudaMalloc(&ex->local, ex->bytes()) != cudaSuccess) {
        delete ex;
        return fail(ctx, MRL_ERR_NOMEM, "cudaMalloc exchange area");
    }
    if (cudaMalloc(&ex->stage, kScratchSets * ex->rb) != cudaSuccess) {
        cudaFree(ex->local);
        delete ex;
        return fail(ctx, MRL_ERR_NOMEM, "cudaMalloc exchange staging records");
    }
    const cudaError_t e = cudaMemset(ex->local, 0, ex->bytes());
    if (e != cudaSuccess) {
        cudaFree(ex->stage);
        cudaFree(ex->local);
        delete ex;
        return cuda_fail(ctx, e, "exchange area memset");
    }
    ex->area[rank] = ex->local;
    if (world > 1) {
        cudaIpcMemHandle_t h;
        const cudaError_t he = cudaIpcGetMemHandle(&h, ex->local);
        if (he != cudaSuccess) {
            cudaFree(ex->stage);
            cudaFree(ex->local);
            delete ex;
            return cuda_fail(ctx, he, "cudaIpcGetMemHandle");
        }
        std::memcpy(ipc_handle, &h, sizeof(h));
    } else {
        ex->opened = true;
    }
    *out = ex;
    return MRL_OK;
}

int mrl_exchange_open(mrl_ctx* ctx, mrl_exchange* ex, const void* ipc_handles) {
    if (!ctx || !ex) return MRL_ERR_INVALID;
    if (ex->opened) return MRL_OK;
    if (!ipc_handles) return fail(ctx, MRL_ERR_INVALID, "ipc_handles is NULL");
    if (int rc = set_device(ctx)) return rc;
    for (uint32_t r = 0; r < ex->world; ++r) {
        if (r == ex->rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const unsigned char*>(ipc_handles) + (size_t)r * sizeof(h), sizeof(h));
        void* ptr = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (uint32_t q = 0; q < r; ++q)
                if (q != ex->rank && ex->area[q]) { cudaIpcCloseMemHandle(ex->area[q]); ex->area[q] = nullptr; }
            return cuda_fail(ctx, e, "cudaIpcOpenMemHandle (peer exchange area)");
        }
        ex->area[r] = static_cast<unsigned char*>(ptr);
    }
    ex->opened = true;
    return MRL_OK;
}

int mrl_exchange_destroy(mrl_ctx* ctx, mrl_exchange* ex) {
    if (!ex) return MRL_OK;
    cudaSetDevice(ex->device);
    cudaDeviceSynchronize();
    for (uint32_t r = 0; r < ex->world; ++r)
        if (r != ex->rank && ex->area[r]) cudaIpcCloseMemHandle(ex->area[r]);
    cudaFree(ex->stage);
    cudaFree(ex->local);
    delete ex;
    (void)ctx;
    return MRL_OK;
}

int mrl_query_scan_exchange(mrl_ctx* ctx, const mrl_seg* seg, const float* d_query, uint32_t dims,
                            const mrl_codec_desc* codec, mrl_plans* plans, const mrl_scan_cfg* cfg,
                            const uint32_t* time_lo, const uint32_t* time_hi, mrl_exchange* ex, uint64_t* d_out_ids,
                            float* d_out_scores, uint32_t* d_out_count, uint32_t* d_out_status) {
    if (!ctx || !seg || !plans || !ex) return MRL_ERR_INVALID;
    if (int rc = check_cfg(ctx, cfg, dims)) return rc;
    if (int rc = check_codec(ctx, codec)) return rc;
    if (int rc = check_exchange(ctx, ex, cfg)) return rc;
    if (plans->n_q < 1 || dims != plans->dims) return fail(ctx, MRL_ERR_INVALID, "plan storage too small or dims mismatch");
    if (!d_query || !d_out_ids || !d_out_scores || !d_out_count) return fail(ctx, MRL_ERR_INVALID, "buffer is NULL");
    if (int rc = set_device(ctx)) return rc;
    if (int rc = ensure_owner(ctx, seg->n_blocks)) return rc;
    float* d_means = nullptr;
    if (int rc = upload_means(ctx, codec, &d_means)) return rc;
    mrl::ScanLaunch p = make_launch(ctx, seg, plans, 0, cfg, time_lo, time_hi);
    p.out_ids = d_out_ids;
    p.out_scores = d_out_scores;
    p.out_count = d_out_count;
    p.out_status = d_out_status;
    p.query = d_query;
    p.dims = dims;
    p.prefix_codec = codec->prefix_codec;
    p.mid_codec = codec->mid_codec;
    p.eden_mean = d_means;
    p.eden_seed = codec->eden_seed;
    p.mid_mean = codec->mid_codec == MRL_MID_EDEN_B1 ? d_means + 64 : nullptr;
    p.mid_seed = codec->mid_seed;
    p.plan_out = plans->d;
    set_exchange(ctx, ex, p);
    take_scratch(ctx, p);
    if (mrl::launch_scan(p, scan_grid(ctx), ctx->stream, true)) return cuda_fail(ctx, cudaGetLastError(), "scan launch");
    launched(ctx);
    return MRL_OK;
}

int mrl_ring_search(mrl_ctx* ctx, const float* d_query, const float* d_pending, uint32_t n_pending, uint32_t dims,
                    uint32_t k, void* d_record) {
    if (!ctx) return MRL_ERR_INVALID;
    if (k < 1 || k > 4096) return fail(ctx, MRL_ERR_INVALID, "k must be in [1, 4096]");
    if (n_pending > 4096) return fail(ctx, MRL_ERR_INVALID, "at most 4096 pending vectors");
    if (dims < 1 || dims > 16384) return fail(ctx, MRL_ERR_INVALID, "dims must be in [1, 16384]");
    if (!d_record || (n_pending && (!d_query || !d_pending))) return fail(ctx, MRL_ERR_INVALID, "buffer is NULL");
    if (reinterpret_cast<uintptr_t>(d_record) % 16) return fail(ctx, MRL_ERR_INVALID, "d_record must be 16-byte aligned");
    if (int rc = set_device(ctx)) return rc;
    if (int rc = ensure_buf(ctx, &ctx->xbuf, &ctx->xbuf_bytes, sizeof(float) * (n_pending + 4) + 16)) return rc;
    float* d_scores = static_cast<float*>(ctx->xbuf);
    uint32_t* d_bad = reinterpret_cast<uint32_t*>(d_scores + n_pending + 1);
    unsigned char* rec = static_cast<unsigned char*>(d_record);
    if (mrl::launch_exact_dots(d_query, d_pending, n_pending, dims, nullptr, n_pending, d_scores, d_bad, ctx->stream) ||
        mrl::launch_exact_rank(d_scores, n_pending, nullptr, (uint64_t)0xFFFFFFFFu << 16, k,
                               reinterpret_cast<uint64_t*>(rec), reinterpret_cast<float*>(rec + (size_t)k * 8),
                               reinterpret_cast<uint32_t*>(rec + (size_t)k * 12), ctx->stream))
        return cuda_fail(ctx, cudaGetLastError(), "ring search launch");
    return MRL_OK;
}

int mrl_rerank_exact(mrl_ctx* ctx, const float* d_query, const float* d_rows, uint64_t n_rows, uint32_t dims,
                     const uint64_t* d_cand, uint32_t n_cand, uint64_t* d_out_rows, float* d_out_scores) {
    if (!ctx) return MRL_ERR_INVALID;
    if (n_cand > 4096) return fail(ctx, MRL_ERR_INVALID, "at most 4096 candidates");
    if (dims < 1 || dims > 16384) return fail(ctx, MRL_ERR_INVALID, "dims must be in [1, 16384]");
    if (n_cand == 0) return MRL_OK;
    if (!d_query || !d_rows || !d_cand || !d_out_rows || !d_out_scores) return fail(ctx, MRL_ERR_INVALID, "buffer is NULL");
    if (int rc = set_device(ctx)) return rc;
    if (int rc = ensure_buf(ctx, &ctx->xbuf, &ctx->xbuf_bytes, sizeof(float) * (n_cand + 4) + 16)) return rc;
    float* d_scores = static_cast<float*>(ctx->xbuf);
    uint32_t* d_bad = reinterpret_cast<uint32_t*>(d_scores + n_cand + 1);
    MRL_CUDA_TRY(ctx, cudaMemsetAsync(d_bad, 0, sizeof(uint32_t), ctx->stream));
    if (mrl::launch_exact_dots(d_query, d_rows, n_rows, dims, d_cand, n_cand, d_scores, d_bad, ctx->stream) ||
        mrl::launch_exact_rank(d_scores, n_cand, d_cand, 0, n_cand, d_out_rows, d_out_scores, nullptr, ctx->stream))
        return cuda_fail(ctx, cudaGetLastError(), "rerank launch");
    uint32_t bad = 0;
    MRL_CUDA_TRY(ctx, cudaMemcpyAsync(&bad, d_bad, sizeof(bad), cudaMemcpyDeviceToHost, ctx->stream));
    MRL_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    if (bad) return fail(ctx, MRL_ERR_INVALID, "candidate row id out of range");
    return MRL_OK;
}

int mrl_ring_create(mrl_ctx* ctx, uint32_t dims, uint32_t capacity, mrl_ring** out) {
    if (!ctx || !out) return MRL_ERR_INVALID;
    *out = nullptr;
    if (dims < 1 || dims > 16384) return fail(ctx, MRL_ERR_INVALID, "dims must be in [1, 16384]");
    capacity = std::max<uint32_t>(capacity, 64);  // RingBuffer::new: capacity.max(VECTORS_PER_BLOCK)
    if (capacity > 4096) return fail(ctx, MRL_ERR_INVALID, "ring capacity must be <= 4096");
    if (int rc = set_device(ctx)) return rc;
    mrl_ring* r = new mrl_ring();
    r->dims = dims;
    r->capacity = capacity;
    const cudaError_t e = cudaMalloc(&r->rows, (size_t)capacity * dims * sizeof(float));
    if (e != cudaSuccess) { delete r; return fail(ctx, MRL_ERR_NOMEM, "cudaMalloc ring rows"); }
    *out = r;
    return MRL_OK;
}

int mrl_ring_push(mrl_ctx* ctx, mrl_ring* ring, const float* row) {
    if (!ctx || !ring || !row) return MRL_ERR_INVALID;
    if (ring->len >= ring->capacity) return fail(ctx, MRL_ERR_INVALID, "ring is full (flush a block first)");
    if (int rc = set_device(ctx)) return rc;
    MRL_CUDA_TRY(ctx, cudaMemcpyAsync(ring->rows + (size_t)ring->len * ring->dims, row, ring->dims * sizeof(float),
                                      cudaMemcpyHostToDevice, ctx->stream));
    ring->len += 1;
    return MRL_OK;
}

int mrl_ring_push_device(mrl_ctx* ctx, mrl_ring* ring, const float* d_rows, uint32_t n) {
    if (!ctx || !ring || (n && !d_rows)) return MRL_ERR_INVALID;
    if ((uint64_t)ring->len + n > ring->capacity) return fail(ctx, MRL_ERR_INVALID, "ring is full (flush a block first)");
    if (n == 0) return MRL_OK;
    if (int rc = set_device(ctx)) return rc;
    MRL_CUDA_TRY(ctx, cudaMemcpyAsync(ring->rows + (size_t)ring->len * ring->dims, d_rows,
                                      (size_t)n * ring->dims * sizeof(float), cudaMemcpyDeviceToDevice, ctx->stream));
    ring->len += n;
    return MRL_OK;
}

int mrl_ring_search_batch(mrl_ctx* ctx, const float* d_queries, uint32_t n_q, uint32_t dims, const mrl_ring* ring,
                          uint32_t slot_base, uint32_t k, void* d_records) {
    if (!ctx) return MRL_ERR_INVALID;
    if (k < 1 || k > 4096) return fail(ctx, MRL_ERR_INVALID, "k must be in [1, 4096]");
    if (ring && ring->dims != dims) return fail(ctx, MRL_ERR_INVALID, "ring dims differ from the queries'");
    const uint32_t n = ring ? ring->len : 0;
    if (n > 1024) return fail(ctx, MRL_ERR_INVALID, "at most 1024 pending rows for a batched ring search");
    if ((uint64_t)slot_base + n > 65536u) return fail(ctx, MRL_ERR_INVALID, "slot_base + pending rows exceeds 65536");
    if (n_q && (!d_queries || !d_records)) return fail(ctx, MRL_ERR_INVALID, "buffer is NULL");
    if (reinterpret_cast<uintptr_t>(d_records) % 16) return fail(ctx, MRL_ERR_INVALID, "d_records must be 16-byte aligned");
    if (int rc = set_device(ctx)) return rc;
    if (mrl::launch_ring_search_batch(d_queries, n_q, dims, ring ? ring->rows : nullptr, n, slot_base, k, d_records,
                                      ctx->stream))
        return cuda_fail(ctx, cudaGetLastError(), "batched ring search launch");
    return MRL_OK;
}

int mrl_ring_drain(mrl_ctx* ctx, mrl_ring* ring, uint32_t n) {
    if (!ctx || !ring) return MRL_ERR_INVALID;
    n = std::min(n, ring->len);
    const uint32_t rest = ring->len - n;
    if (n && rest) {  // keep the order: rows [n, len) move to the front through the staging buffer
        if (int rc = set_device(ctx)) return rc;
        const size_t bytes = (size_t)rest * ring->dims * sizeof(float);
        if (int rc = ensure_tmp(ctx, bytes)) return rc;
        MRL_CUDA_TRY(ctx, cudaMemcpyAsync(ctx->tmp, ring->rows + (size_t)n * ring->dims, bytes,
                                          cudaMemcpyDeviceToDevice, ctx->stream));
        MRL_CUDA_TRY(ctx, cudaMemcpyAsync(ring->rows, ctx->tmp, bytes, cudaMemcpyDeviceToDevice, ctx->stream));
    }
    ring->len = rest;
    return MRL_OK;
}

uint32_t mrl_ring_len(const mrl_ring* ring) { return ring ? ring->len : 0; }

int mrl_ring_rows(const mrl_ring* ring, const float** d_rows) {
    if (!ring || !d_rows) return MRL_ERR_INVALID;
    *d_rows = ring->rows;
    return MRL_OK;
}

int mrl_ring_destroy(mrl_ctx* ctx, mrl_ring* ring) {
    if (!ring) return MRL_OK;
    if (ctx) cudaSetDevice(ctx->device);
    cudaFree(ring->rows);
    delete ring;
    return MRL_OK;
}

int mrl_engine_scan(mrl_ctx* ctx, const mrl_seg* seg, const float* d_query, uint32_t dims,
                    const mrl_codec_desc* codec, mrl_plans* plans, const mrl_scan_cfg* cfg, const uint32_t* time_lo,
                    const uint32_t* time_hi, const mrl_ring* ring, uint64_t* d_out_ids, float* d_out_scores,
                    uint32_t* d_out_count, uint32_t* d_out_status) {
    if (!ctx || !seg || !plans) return MRL_ERR_INVALID;
    if (int rc = check_cfg(ctx, cfg, dims)) return rc;
    if (ring && ring->dims != dims) return fail(ctx, MRL_ERR_INVALID, "ring dims differ from the query's");
    if (!ring || ring->len == 0)  // nothing pending: the scan's list is the shortlist
        return mrl_query_scan_device(ctx, seg, d_query, 1, dims, codec, plans, cfg, time_lo, time_hi, d_out_ids,
                                     d_out_scores, d_out_count, d_out_status);
    if (!d_out_ids || !d_out_scores || !d_out_count) return fail(ctx, MRL_ERR_INVALID, "buffer is NULL");
    const uint32_t k = cfg->shortlist_cand;
    const size_t rb = MRL_MERGE_RECORD_BYTES(k);
    if (int rc = set_device(ctx)) return rc;
    if (int rc = ensure_buf(ctx, &ctx->ebuf, &ctx->ebuf_bytes, 2 * rb)) return rc;
    unsigned char* rec = static_cast<unsigned char*>(ctx->ebuf);
    if (int rc = mrl_query_scan_device(ctx, seg, d_query, 1, dims, codec, plans, cfg, time_lo, time_hi,
                                       reinterpret_cast<uint64_t*>(rec), reinterpret_cast<float*>(rec + (size_t)k * 8),
                                       reinterpret_cast<uint32_t*>(rec + (size_t)k * 12), d_out_status))
        return rc;
    if (int rc = mrl_ring_search(ctx, d_query, ring->rows, ring->len, dims, k, rec + rb)) return rc;
    return mrl_merge_topk(ctx, rec, 2, k, k, d_out_ids, d_out_scores, d_out_count);
}

int mrl_merge_topk(mrl_ctx* ctx, const void* d_lists, uint32_t n_lists, uint32_t stride, uint32_t k,
                   uint64_t* d_out_ids, float* d_out_scores, uint32_t* d_out_count) {
    if (!ctx) return MRL_ERR_INVALID;
    if (n_lists < 1 || n_lists > 1024) return fail(ctx, MRL_ERR_INVALID, "n_lists must be in [1, 1024]");
    if (stride < 1 || stride > 4096 || k < 1 || k > 4096) return fail(ctx, MRL_ERR_INVALID, "stride and k must be in [1, 4096]");
    if (!d_lists || !d_out_ids || !d_out_scores || !d_out_count) return fail(ctx, MRL_ERR_INVALID, "buffer is NULL");
    if (reinterpret_cast<uintptr_t>(d_lists) % 16) return fail(ctx, MRL_ERR_INVALID, "d_lists must be 16-byte aligned");
    if (int rc = set_device(ctx)) return rc;
    if (mrl::launch_merge_topk(d_lists, n_lists, stride, k, d_out_ids, d_out_scores, d_out_count, ctx->stream))
        return cuda_fail(ctx, cudaGetLastError(), "merge launch");
    return MRL_OK;
}

int mrl_pack_records(mrl_ctx* ctx, const uint64_t* d_ids, const float* d_scores, const uint32_t* d_counts, uint32_t n_q,
                     uint32_t k, void* d_records) {
    if (!ctx) return MRL_ERR_INVALID;
    if (k < 1 || k > 4096) return fail(ctx, MRL_ERR_INVALID, "k must be in [1, 4096]");
    if (n_q && (!d_ids || !d_scores || !d_counts || !d_records)) return fail(ctx, MRL_ERR_INVALID, "buffer is NULL");
    if (reinterpret_cast<uintptr_t>(d_records) % 16) return fail(ctx, MRL_ERR_INVALID, "d_records must be 16-byte aligned");
    if (int rc = set_device(ctx)) return rc;
    if (mrl::launch_pack_records(d_ids, d_scores, d_counts, n_q, k, d_records, ctx->stream))
        return cuda_fail(ctx, cudaGetLastError(), "pack launch");
    return MRL_OK;
}

int mrl_merge_topk_batch(mrl_ctx* ctx, const void* d_lists, uint32_t n_lists, uint32_t n_q, uint32_t stride, uint32_t k,
                         uint64_t* d_out_ids, float* d_out_scores, uint32_t* d_out_counts) {
    if (!ctx) return MRL_ERR_INVALID;
    if (n_lists < 1 || n_lists > 1024) return fail(ctx, MRL_ERR_INVALID, "n_lists must be in [1, 1024]");
    if (stride < 1 || stride > 4096 || k < 1 || k > 4096) return fail(ctx, MRL_ERR_INVALID, "stride and k must be in [1, 4096]");
    if (n_q && (!d_lists || !d_out_ids || !d_out_scores || !d_out_counts)) return fail(ctx, MRL_ERR_INVALID, "buffer is NULL");
    if (reinterpret_cast<uintptr_t>(d_lists) % 16) return fail(ctx, MRL_ERR_INVALID, "d_lists must be 16-byte aligned");
    if (int rc = set_device(ctx)) return rc;
    if (mrl::launch_merge_topk_batch(d_lists, n_lists, n_q, stride, k, d_out_ids, d_out_scores, d_out_counts, ctx->stream))
        return cuda_fail(ctx, cudaGetLastError(), "batched merge launch");
    return MRL_OK;
}

int mrl_scan(mrl_ctx* ctx, const mrl_seg* seg, const mrl_plans* plans, const mrl_scan_cfg* cfg, const uint32_t* time_lo,
             const uint32_t* time_hi, uint64_t* out_ids, float* out_scores, uint32_t* out_counts) {
    if (!ctx || !seg || !plans) return MRL_ERR_INVALID;
    if (int rc = check_cfg(ctx, cfg, plans->dims)) return rc;
    const uint32_t n_q = plans->n_q, k = cfg->shortlist_cand;
    if (n_q == 0) return MRL_OK;
    if (!out_ids || !out_scores || !out_counts) return fail(ctx, MRL_ERR_INVALID, "output is NULL");
    if (int rc = set_device(ctx)) return rc;
    const size_t nk = (size_t)n_q * k;
    if (int rc = ensure_out(ctx, nk * (sizeof(uint64_t) + sizeof(float)) + 2 * sizeof(uint32_t) * n_q + 64)) return rc;
    uint64_t* d_ids = (uint64_t*)ctx->tmp_out;
    float* d_sc = (float*)(d_ids + nk);
    uint32_t* d_cnt = (uint32_t*)(d_sc + nk);
    uint32_t* d_st = d_cnt + n_q;
    // many plans in fast mode: the batched scan, with the rare uncertified query rerun alone
    const bool batch = n_q >= kBatchMinQueries && cfg->mode == MRL_MODE_FAST && cfg->strata_depth != MRL_DEPTH_L0;
    if (batch) {
        if (int rc = mrl_scan_batch_device(ctx, seg, plans, 0, n_q, cfg, time_lo, time_hi, d_ids, d_sc, d_cnt, d_st))
            return rc;
        std::vector<uint32_t> st(n_q);
        MRL_CUDA_TRY(ctx, cudaMemcpyAsync(st.data(), d_st, n_q * sizeof(uint32_t), cudaMemcpyDeviceToHost, ctx->stream));
        MRL_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
        for (uint32_t q = 0; q < n_q; ++q)
            if (st[q] & 2u) return fail(ctx, MRL_ERR_CUDA, "batched scan: a bounded tensor-core wait ran out");
        for (uint32_t q = 0; q < n_q; ++q)
            if (st[q] & MRL_STATUS_UNCERTIFIED)
                if (int rc = mrl_scan_device(ctx, seg, plans, q, 1, cfg, time_lo, time_hi, d_ids + (size_t)q * k,
                                             d_sc + (size_t)q * k, d_cnt + q, d_st + q))
                    return rc;
    } else if (int rc = mrl_scan_device(ctx, seg, plans, 0, n_q, cfg, time_lo, time_hi, d_ids, d_sc, d_cnt, d_st)) {
        return rc;
    }
    MRL_CUDA_TRY(ctx, cudaMemcpyAsync(out_ids, d_ids, nk * sizeof(uint64_t), cudaMemcpyDeviceToHost, ctx->stream));
    MRL_CUDA_TRY(ctx, cudaMemcpyAsync(out_scores, d_sc, nk * sizeof(float), cudaMemcpyDeviceToHost, ctx->stream));
    MRL_CUDA_TRY(ctx, cudaMemcpyAsync(out_counts, d_cnt, n_q * sizeof(uint32_t), cudaMemcpyDeviceToHost, ctx->stream));
    std::vector<uint32_t> st(n_q);
    MRL_CUDA_TRY(ctx, cudaMemcpyAsync(st.data(), d_st, n_q * sizeof(uint32_t), cudaMemcpyDeviceToHost, ctx->stream));
    MRL_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    for (uint32_t q = 0; q < n_q; ++q)
        if (st[q] & 10u) return fail(ctx, MRL_ERR_CUDA, "scan: a bounded wait ran out (status bits 1/3)");
    return MRL_OK;
}

int mrl_debug_vector_scores(mrl_ctx* ctx, const mrl_seg* seg, const mrl_plans* plans, uint32_t q, const mrl_scan_cfg* cfg,
                            const uint32_t* time_lo, const uint32_t* time_hi, float* out_scores, uint8_t* out_active,
                            int32_t* out_partials) {
    if (!ctx || !seg || !plans || !out_scores || !out_active) return MRL_ERR_INVALID;
    if (int rc = check_cfg(ctx, cfg, 0)) return rc;
    if (q >= plans->n_q) return fail(ctx, MRL_ERR_INVALID, "plan index out of range");
    if (int rc = set_device(ctx)) return rc;
    const size_t n = (size_t)seg->n_blocks * 64;
    if (n == 0) return MRL_OK;
    if (int rc = ensure_out(ctx, n * (sizeof(float) + 1 + 3 * sizeof(int32_t)) + 64)) return rc;
    float* d_sc = (float*)ctx->tmp_out;
    int32_t* d_parts = (int32_t*)(d_sc + n);
    uint8_t* d_act = (uint8_t*)(d_parts + 3 * n);
    mrl::ScanLaunch p = make_launch(ctx, seg, plans, q, cfg, time_lo, time_hi);
    if (mrl::launch_debug_scores(p, d_sc, d_act, d_parts, ctx->stream)) return cuda_fail(ctx, cudaGetLastError(), "debug launch");
    MRL_CUDA_TRY(ctx, cudaMemcpyAsync(out_scores, d_sc, n * sizeof(float), cudaMemcpyDeviceToHost, ctx->stream));
    MRL_CUDA_TRY(ctx, cudaMemcpyAsync(out_active, d_act, n, cudaMemcpyDeviceToHost, ctx->stream));
    if (out_partials)
        MRL_CUDA_TRY(ctx, cudaMemcpyAsync(out_partials, d_parts, 3 * n * sizeof(int32_t), cudaMemcpyDeviceToHost, ctx->stream));
    MRL_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    return MRL_OK;
}

int mrl_debug_score_bound(mrl_ctx* ctx, const mrl_seg* seg, const mrl_plans* plans, uint32_t q,
                          const mrl_scan_cfg* cfg, float* out_bound) {
    if (!ctx || !seg || !plans || !out_bound) return MRL_ERR_INVALID;
    if (int rc = check_cfg(ctx, cfg, 0)) return rc;
    if (q >= plans->n_q) return fail(ctx, MRL_ERR_INVALID, "plan index out of range");
    if (int rc = set_device(ctx)) return rc;
    if (int rc = ensure_out(ctx, 64)) return rc;
    const mrl::ScanLaunch p = make_launch(ctx, seg, plans, q, cfg, nullptr, nullptr);
    if (mrl::launch_score_bound(p, (float*)ctx->tmp_out, ctx->stream)) return cuda_fail(ctx, cudaGetLastError(), "bound launch");
    MRL_CUDA_TRY(ctx, cudaMemcpyAsync(out_bound, ctx->tmp_out, sizeof(float), cudaMemcpyDeviceToHost, ctx->stream));
    MRL_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    return MRL_OK;
}

int mrl_debug_control_words(mrl_ctx* ctx, uint32_t* out) {
    if (!ctx || !out) return MRL_ERR_INVALID;
    if (int rc = set_device(ctx)) return rc;
    for (uint32_t set = 0; set < kScratchSets; ++set)  // the 8 control words of each scratch set
        MRL_CUDA_TRY(ctx, cudaMemcpyAsync(out + 8 * set, ctx->ctl + set * mrl::kCtlWords, 8 * sizeof(unsigned),
                                          cudaMemcpyDeviceToHost, ctx->stream));
    MRL_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    return MRL_OK;
}

int mrl_encode_device(mrl_ctx* ctx, const float* d_rows, uint64_t n, uint32_t dims, uint32_t src,
                      const mrl_codec_desc* codec, uint8_t* d_pages, uint32_t block_id_base, mrl_seg** seg_out) {
    if (!ctx) return MRL_ERR_INVALID;
    if (seg_out) *seg_out = nullptr;
    if (int rc = check_codec(ctx, codec)) return rc;
    if (dims < 192) return fail(ctx, MRL_ERR_INVALID, "dims must be >= 192 (src/quantize.rs:47)");
    if (codec->mid_codec == MRL_MID_EDEN_B1 && codec->prefix_codec != MRL_PREFIX_EDEN)
        return fail(ctx, MRL_ERR_INVALID, "eden_mid requires eden prefix fit (src/quantize.rs:52-54)");
    const uint64_t nb = (n + 63) / 64;
    if (nb >= (1ull << 26)) return fail(ctx, MRL_ERR_INVALID, "segment larger than 2^26 pages");
    if (int rc = set_device(ctx)) return rc;
    float* d_means = nullptr;
    if (int rc = upload_means(ctx, codec, &d_means)) return rc;
    mrl_seg* s = nullptr;
    if (seg_out) {
        if (int rc = seg_new(ctx, block_id_base, &s)) return rc;
        if (int rc = seg_reserve(ctx, s, nb ? nb : 1)) { mrl_segment_free(ctx, s); return rc; }
    }
    if (mrl::launch_encode(d_rows, n, dims, nullptr, nullptr, src, codec->prefix_codec, d_means, codec->eden_seed,
                           codec->mid_codec == MRL_MID_EDEN_B1 ? d_means + 64 : nullptr, codec->mid_seed, d_pages,
                           s ? s->pages : nullptr, s ? s->ts : nullptr, ctx->stream)) {
        mrl_segment_free(ctx, s);
        return cuda_fail(ctx, cudaGetLastError(), "encode launch");
    }
    if (s)
        if (int rc = seg_note_pages(ctx, s, 0, nb)) { mrl_segment_free(ctx, s); return rc; }
    const cudaError_t e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) { mrl_segment_free(ctx, s); return cuda_fail(ctx, e, "encode"); }
    if (s) { s->n_blocks = nb; *seg_out = s; }
    return MRL_OK;
}

int mrl_encode_blocks(mrl_ctx* ctx, const float* rows, uint64_t n, uint32_t dims, const uint32_t* ts,
                      const uint32_t* src, const mrl_codec_desc* codec, uint8_t* out_pages) {
    if (!ctx || (n && (!rows || !out_pages))) return MRL_ERR_INVALID;
    if (int rc = check_codec(ctx, codec)) return rc;
    if (dims < 192) return fail(ctx, MRL_ERR_INVALID, "dims must be >= 192 (src/quantize.rs:47)");
    if (codec->mid_codec == MRL_MID_EDEN_B1 && codec->prefix_codec != MRL_PREFIX_EDEN)
        return fail(ctx, MRL_ERR_INVALID, "eden_mid requires eden prefix fit (src/quantize.rs:52-54)");
    if (n == 0) return MRL_OK;
    for (uint64_t i = 0; i < n * dims; ++i)
        if (!std::isfinite(rows[i])) return fail(ctx, MRL_ERR_INVALID, "rows contain a non-finite value");
    if (int rc = set_device(ctx)) return rc;
    const uint64_t nb = (n + 63) / 64;
    const size_t rbytes = n * dims * sizeof(float), pbytes = nb * mrl::kBlockBytes, abytes = n * sizeof(uint32_t);
    if (int rc = ensure_tmp(ctx, rbytes + pbytes + 2 * abytes + 64)) return rc;
    float* d_means = nullptr;
    float* d_rows = (float*)ctx->tmp;
    uint8_t* d_pax = (uint8_t*)(d_rows + n * dims);
    uint32_t* d_ts = (uint32_t*)(d_pax + pbytes);
    uint32_t* d_src = d_ts + n;
    MRL_CUDA_TRY(ctx, cudaMemcpyAsync(d_rows, rows, rbytes, cudaMemcpyHostToDevice, ctx->stream));
    if (ts) MRL_CUDA_TRY(ctx, cudaMemcpyAsync(d_ts, ts, abytes, cudaMemcpyHostToDevice, ctx->stream));
    if (src) MRL_CUDA_TRY(ctx, cudaMemcpyAsync(d_src, src, abytes, cudaMemcpyHostToDevice, ctx->stream));
    if (int rc = upload_means(ctx, codec, &d_means)) return rc;
    if (mrl::launch_encode(d_rows, n, dims, ts ? d_ts : nullptr, src ? d_src : nullptr, 8u /* source::DOC */,
                           codec->prefix_codec, d_means, codec->eden_seed,
                           codec->mid_codec == MRL_MID_EDEN_B1 ? d_means + 64 : nullptr, codec->mid_seed, d_pax, nullptr,
                           nullptr, ctx->stream))
        return cuda_fail(ctx, cudaGetLastError(), "encode launch");
    MRL_CUDA_TRY(ctx, cudaMemcpyAsync(out_pages, d_pax, pbytes, cudaMemcpyDeviceToHost, ctx->stream));
    MRL_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    return MRL_OK;
}

int mrl_eden_fit_device(mrl_ctx* ctx, const float* d_rows, uint64_t n, uint32_t dims, uint32_t start, uint32_t width,
                        float* mean_out) {
    if (!ctx || !d_rows || !mean_out) return MRL_ERR_INVALID;
    if (n == 0) return fail(ctx, MRL_ERR_INVALID, "empty corpus for EdenFit (src/eden.rs:149)");
    if (start + width > dims || width == 0 || (width & (width - 1)))
        return fail(ctx, MRL_ERR_INVALID, "EDEN slice must be a power of two inside the row (src/eden.rs:138)");
    if (int rc = set_device(ctx)) return rc;
    if (int rc = ensure_tmp(ctx, width * sizeof(float))) return rc;
    if (mrl::launch_eden_fit(d_rows, n, dims, start, width, (float*)ctx->tmp, ctx->stream))
        return cuda_fail(ctx, cudaGetLastError(), "eden fit launch");
    MRL_CUDA_TRY(ctx, cudaMemcpyAsync(mean_out, ctx->tmp, width * sizeof(float), cudaMemcpyDeviceToHost, ctx->stream));
    MRL_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    return MRL_OK;
}

int mrl_synth_docs_device(mrl_ctx* ctx, uint64_t seed, uint64_t row0, uint64_t n, uint32_t dims, float* d_out) {
    if (!ctx || (n && !d_out) || dims == 0) return MRL_ERR_INVALID;
    if (int rc = set_device(ctx)) return rc;
    if (mrl::launch_synth_docs(seed, row0, n, dims, d_out, ctx->stream)) return cuda_fail(ctx, cudaGetLastError(), "synth launch");
    MRL_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    return MRL_OK;
}

int mrl_synth_queries_device(mrl_ctx* ctx, uint64_t doc_seed, uint64_t n_docs, uint64_t q_seed, uint64_t n_q,
                             uint32_t dims, float sigma, float* d_out, uint64_t* d_pick) {
    if (!ctx || (n_q && !d_out) || n_docs == 0 || dims == 0) return MRL_ERR_INVALID;
    if (int rc = set_device(ctx)) return rc;
    if (mrl::launch_synth_queries(doc_seed, n_docs, q_seed, n_q, dims, sigma, d_out, d_pick, ctx->stream))
        return cuda_fail(ctx, cudaGetLastError(), "synth launch");
    MRL_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    return MRL_OK;
}

int mrl_scan_geometry(mrl_ctx* ctx, uint32_t k, uint32_t* ctas, uint32_t* list_len) {
    if (!ctx) return MRL_ERR_INVALID;
    if (ctas) *ctas = scan_grid(ctx);
    if (list_len) *list_len = ctx->list_len_override ? ctx->list_len_override : auto_list_len(k, scan_grid(ctx));
    return MRL_OK;
}

int mrl_set_scan_ctas(mrl_ctx* ctx, uint32_t ctas) {
    if (!ctx) return MRL_ERR_INVALID;
    if (ctas > (uint32_t)ctx->sms)
        return fail(ctx, MRL_ERR_INVALID, "ctas must be 0 (one per SM) or at most the device's " + std::to_string(ctx->sms) + " SMs");
    ctx->scan_ctas = ctas;
    return MRL_OK;
}

int mrl_set_batch_engine(mrl_ctx* ctx, uint32_t engine) {
    if (!ctx) return MRL_ERR_INVALID;
    if (engine > MRL_BATCH_CUDA_CORE) return fail(ctx, MRL_ERR_INVALID, "engine must be MRL_BATCH_TENSOR or MRL_BATCH_CUDA_CORE");
    ctx->batch_engine = engine;
    return MRL_OK;
}

int mrl_set_list_len(mrl_ctx* ctx, uint32_t list_len) {
    if (!ctx) return MRL_ERR_INVALID;
    if (list_len > 32 || (list_len & (list_len - 1)))
        return fail(ctx, MRL_ERR_INVALID, "list_len must be 0 (auto) or a power of two <= 32");
    ctx->list_len_override = list_len;
    return MRL_OK;
}

}  // extern "C"
