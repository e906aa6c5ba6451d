// encode.cu — page transcode, block encode, EDEN fit and seeded synthetic inputs on sm_100a.
//
// * transcode: PaxBlock64 pages (src/block.rs:130-144) -> the vector-major scan layout
//   (see mrl_internal.cuh), one 64-thread CTA per page staged through shared memory.
// * encode: encode_block_with_fits (src/quantize.rs:36-96) for up to 64 rows per page, one
//   64-thread CTA per page (thread t encodes slot t in the reference's f32 order), bit planes
//   assembled with warp ballots (word d of a plane = ballot of warp 0 | ballot of warp 1 << 32,
//   the little-endian layout the reference pins in tests/test_challenger_architecture.rs:27-187),
//   header + tombstones + CRC-32 (crc32fast::hash over the page with the CRC field zeroed,
//   src/block.rs:186-190). Writes the PaxBlock64 page and/or the scan-layout page.
// * eden fit: EdenFit::fit_band (src/eden.rs:130-161), one thread per coordinate summing the
//   rows in order.
// * synthetic docs / queries: the integer recipe documented in mrl_cuda.h.
#include <algorithm>

#include "mrl_internal.cuh"

namespace mrl {
namespace {

__device__ __forceinline__ float f_add(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float f_sub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float f_mul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float f_div(float a, float b) { return __fdiv_rn(a, b); }

__device__ __forceinline__ uint64_t plane64(const uint64_t* blk, int off, int d) { return blk[(off >> 3) + d]; }

__global__ void __launch_bounds__(64) transcode_kernel(const uint8_t* __restrict__ pax, uint4* __restrict__ pages,
                                                       uint2* __restrict__ ts) {
    __shared__ __align__(16) uint64_t s_blk[512];
    const uint64_t b = blockIdx.x;
    const uint4* src = reinterpret_cast<const uint4*>(pax + b * kBlockBytes);
    for (int i = threadIdx.x; i < 256; i += 64) reinterpret_cast<uint4*>(s_blk)[i] = src[i];
    __syncthreads();
    const int v = threadIdx.x;
    uint32_t w[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) w[i] = 0;
    for (int d = 0; d < kPrefix; ++d) {
        const uint32_t lv = (uint32_t)((plane64(s_blk, kOffS5, d) >> v) & 1u) |
                            ((uint32_t)((plane64(s_blk, kOffS3, d) >> v) & 1u) << 1) |
                            ((uint32_t)((plane64(s_blk, kOffS2, d) >> v) & 1u) << 2) |
                            ((uint32_t)((plane64(s_blk, kOffS0, d) >> v) & 1u) << 3);
        w[d >> 3] |= lv << (4 * (d & 7));
    }
    for (int d = 0; d < kRabitq; ++d) w[8 + (d >> 5)] |= (uint32_t)((plane64(s_blk, kOffS1, d) >> v) & 1u) << (d & 31);
    for (int d = 0; d < kFold; ++d) w[12 + (d >> 5)] |= (uint32_t)((plane64(s_blk, kOffS4, d) >> v) & 1u) << (d & 31);
    const uint8_t* bytes = reinterpret_cast<const uint8_t*>(s_blk);
    const uint8_t* m = bytes + kOffMeta + 7 * v;
    const uint64_t tomb = s_blk[kOffTomb >> 3];
    w[14] = (uint32_t)m[0] | ((uint32_t)m[1] << 8) | ((uint32_t)m[2] << 16) | ((uint32_t)m[3] << 24);
    w[15] = (uint32_t)m[4] | ((uint32_t)m[5] << 8) | ((uint32_t)m[6] << 16) | ((uint32_t)((tomb >> v) & 1u) << 24);
    uint4* dst = pages + b * 256 + v;
#pragma unroll
    for (int c = 0; c < 4; ++c) dst[64 * c] = make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
    if (v == 0) {
        const uint32_t* h = reinterpret_cast<const uint32_t*>(s_blk);
        ts[b] = make_uint2(h[kOffMinTs / 4], h[kOffMaxTs / 4]);
    }
}

// ---- encode ----

// nearest_centroid, src/eden.rs:57-71
__device__ __forceinline__ int nearest_centroid(const float* cb, int n, float z) {
    int lo = 0, hi = n;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (cb[mid] < z) lo = mid + 1; else hi = mid;
    }
    if (lo < n && cb[lo] == z) return lo;
    if (lo == 0) return 0;
    if (lo >= n) return n - 1;
    return (fabsf(f_sub(z, cb[lo - 1])) <= fabsf(f_sub(cb[lo], z))) ? lo - 1 : lo;
}

// In-thread FWHT (src/rotate.rs:13-33) over a per-thread strided smem vector a[i*stride].
__device__ void fwht_strided(float* a, int n, int stride) {
    for (int h = 1; h < n; h *= 2)
        for (int i = 0; i < n; i += 2 * h)
            for (int j = i; j < i + h; ++j) {
                const float x = a[j * stride], y = a[(j + h) * stride];
                a[j * stride] = f_add(x, y);
                a[(j + h) * stride] = f_sub(x, y);
            }
    const float scale = f_div(1.0f, __fsqrt_rn((float)n));
    for (int i = 0; i < n; ++i) a[i * stride] = f_mul(a[i * stride], scale);
}

// encode_slice (src/eden.rs:225-269) of x[0..d) (strided smem scratch `c`), bits 4 or 1.
__device__ void eden_slice(const float* mean, const float* diag, int d, int bits, const float* x,
                           float* c, int stride, uint8_t* levels, float* alpha) {
    float cbuf[16];
    const int ncb = 1 << bits;
    if (bits == 4) {
        for (int i = 0; i < 16; ++i) cbuf[i] = g_lloyd_b4[i];
    } else {
        cbuf[0] = -kLloydB1Hi;
        cbuf[1] = kLloydB1Hi;
    }
    const float sqrt_d = __fsqrt_rn((float)d);
    const float inv_sqrt_d = f_div(1.0f, sqrt_d);
    float ns = 0.0f;
    for (int i = 0; i < d; ++i) {
        const float v = f_sub(x[i], mean[i]);
        c[i * stride] = v;
        ns = f_add(ns, f_mul(v, v));
    }
    const float cn = fmaxf(__fsqrt_rn(ns), 1e-12f);
    const float inv = f_div(1.0f, cn);
    for (int i = 0; i < d; ++i) c[i * stride] = f_mul(f_mul(c[i * stride], inv), diag[i]);
    fwht_strided(c, d, stride);
    float ip = 0.0f;
    for (int i = 0; i < d; ++i) {
        const float ci = c[i * stride];
        const int lv = nearest_centroid(cbuf, ncb, f_mul(ci, sqrt_d));
        levels[i] = (uint8_t)lv;
        ip = f_add(ip, f_mul(ci, f_mul(cbuf[lv], inv_sqrt_d)));
    }
    const float ss = fabsf(ip) > 1e-12f ? f_div(1.0f, ip) : 0.0f;
    *alpha = f_mul(cn, ss);  // EdenCode::alpha, src/eden.rs:219-221
}

__device__ uint32_t crc32_bytes(const uint8_t* p, int n, const uint32_t* tab) {
    uint32_t c = 0xFFFFFFFFu;
    for (int i = 0; i < n; ++i) c = tab[(c ^ p[i]) & 0xFFu] ^ (c >> 8);
    return c ^ 0xFFFFFFFFu;
}

constexpr int kEncThreads = 64;

__global__ void __launch_bounds__(kEncThreads)
encode_kernel(const float* __restrict__ rows, uint64_t n, uint32_t dims, const uint32_t* __restrict__ ts_in,
              const uint32_t* __restrict__ src_in, uint32_t src_const, uint32_t prefix_codec,
              const float* __restrict__ eden_mean, uint64_t eden_seed, const float* __restrict__ mid_mean,
              uint64_t mid_seed, uint8_t* __restrict__ pax_out, uint4* __restrict__ pages, uint2* __restrict__ block_ts) {
    __shared__ __align__(16) uint64_t s_page[512];
    __shared__ float s_scratch[128 * kEncThreads];
    __shared__ uint32_t s_crc[256];
    __shared__ float s_diag[64];
    __shared__ float s_mdiag[128];
    __shared__ float s_fold_sign[kFoldBlocks * kFold];
    __shared__ float s_mean[64];
    __shared__ float s_mmean[128];
    __shared__ uint32_t s_red[4];

    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const uint64_t blk = blockIdx.x;
    const uint64_t row = blk * 64 + t;
    const bool valid = row < n;

    for (int i = t; i < 512; i += kEncThreads) s_page[i] = 0ull;
    for (int i = t; i < 256; i += kEncThreads) {
        uint32_t c = (uint32_t)i;
        for (int k = 0; k < 8; ++k) c = (c & 1u) ? (0xEDB88320u ^ (c >> 1)) : (c >> 1);
        s_crc[i] = c;
    }
    if (t < 64) {
        s_diag[t] = sign_hash(eden_seed, (uint64_t)t);
        s_mean[t] = (prefix_codec == MRL_PREFIX_EDEN) ? eden_mean[t] : 0.0f;
    }
    for (int i = t; i < 128; i += kEncThreads) {
        s_mdiag[i] = sign_hash(mid_seed, (uint64_t)i);
        s_mmean[i] = mid_mean ? mid_mean[i] : 0.0f;
    }
    for (int i = t; i < kFoldBlocks * kFold; i += kEncThreads)
        s_fold_sign[i] = sign_hash((uint64_t)(i / kFold), (uint64_t)(i % kFold));
    if (t == 0) { s_red[0] = 0xFFFFFFFFu; s_red[1] = 0u; s_red[2] = 0u; }
    __syncthreads();

    float* c = s_scratch + t;  // strided per-thread scratch: c[i * kEncThreads]
    const float* x = rows + (valid ? row : 0) * (uint64_t)dims;
    uint8_t lv4[64];
    uint8_t mid_bits[128];
    uint8_t fold_bits[64];
    uint16_t h_scale = 0, h_offset = 0, h_tail = 0;
    uint8_t flags = 0;
    if (valid) {
        float scale, offset = 0.0f;
        if (prefix_codec == MRL_PREFIX_EDEN) {
            float xs[64];
            for (int i = 0; i < 64; ++i) xs[i] = x[i];
            eden_slice(s_mean, s_diag, 64, 4, xs, c, kEncThreads, lv4, &scale);
        } else {  // quantize_vector, src/quantize.rs:220-246
            float mn = INFINITY, mx = -INFINITY;
            for (int i = 0; i < 64; ++i) { mn = fminf(mn, x[i]); mx = fmaxf(mx, x[i]); }
            const float range = fmaxf(f_sub(mx, mn), 1e-8f);
            scale = f_div(range, 15.0f);
            offset = mn;
            for (int i = 0; i < 64; ++i)
                lv4[i] = (uint8_t)fminf(fmaxf(roundf(f_div(f_sub(x[i], offset), scale)), 0.0f), 15.0f);
        }
        float mid_alpha = 0.0f;
        // mid band: RaBitQ signs of FWHT128 (src/quantize.rs:205-211) or EDEN b=1 levels
        if (mid_mean) {
            float xs[128];
            for (int i = 0; i < 128; ++i) xs[i] = x[64 + i];
            eden_slice(s_mmean, s_mdiag, 128, 1, xs, c, kEncThreads, mid_bits, &mid_alpha);
        } else {
            for (int i = 0; i < 128; ++i) c[i * kEncThreads] = x[64 + i];
            fwht_strided(c, 128, kEncThreads);
            for (int i = 0; i < 128; ++i) mid_bits[i] = c[i * kEncThreads] >= 0.0f ? 1 : 0;
        }
        // folded tail (fold_tail + FWHT64, src/rotate.rs:73-100)
        for (int d = 0; d < 64; ++d) c[d * kEncThreads] = 0.0f;
        if (dims > (uint32_t)kTailStart) {
            const int nb = min((int)((dims - kTailStart) / kPrefix), kFoldBlocks);
            for (int b = 0; b < nb; ++b)
                for (int d = 0; d < 64; ++d)
                    c[d * kEncThreads] = f_add(c[d * kEncThreads], f_mul(s_fold_sign[b * kFold + d], x[kTailStart + b * 64 + d]));
        }
        fwht_strided(c, 64, kEncThreads);
        for (int d = 0; d < 64; ++d) fold_bits[d] = c[d * kEncThreads] >= 0.0f ? 1 : 0;
        // residual norms (src/quantize.rs:184-203) and rho flags (src/block.rs:102-108)
        float mid_sq = 0.0f, high_sq = 0.0f;
        for (int i = 64; i < 192; ++i) mid_sq = f_add(mid_sq, f_mul(x[i], x[i]));
        for (uint32_t i = kTailStart; i < dims; ++i) high_sq = f_add(high_sq, f_mul(x[i], x[i]));
        const float rest = __fsqrt_rn(f_add(mid_sq, high_sq));
        const float high = __fsqrt_rn(high_sq);
        if (rest <= 1e-12f) {
            flags = 0;
        } else {
            const float r = fminf(fmaxf(f_div(high, rest), 0.0f), 1.0f);
            flags = (uint8_t)fminf(fmaxf(roundf(f_mul(r, 255.0f)), 0.0f), 255.0f);
        }
        h_scale = __half_as_ushort(__float2half_rn(scale));
        h_offset = __half_as_ushort(__float2half_rn(prefix_codec == MRL_PREFIX_EDEN ? mid_alpha : offset));
        h_tail = __half_as_ushort(__float2half_rn(rest));
        const uint32_t tsv = ts_in ? ts_in[row] : (uint32_t)row;
        const uint32_t srcv = src_in ? src_in[row] : src_const;
        atomicMin(&s_red[0], tsv);
        atomicMax(&s_red[1], tsv);
        atomicOr(&s_red[2], srcv);
    } else {
        for (int i = 0; i < 64; ++i) { lv4[i] = 0; fold_bits[i] = 0; }
        for (int i = 0; i < 128; ++i) mid_bits[i] = 0;
    }
    // planes via ballots: warp w owns 32-bit half w of every 64-bit plane word
    uint32_t* page32 = reinterpret_cast<uint32_t*>(s_page);
    for (int d = 0; d < 64; ++d) {
        const uint32_t q = lv4[d];
        const uint32_t b3 = __ballot_sync(0xffffffffu, (q & 8u) != 0);
        const uint32_t b2 = __ballot_sync(0xffffffffu, (q & 4u) != 0);
        const uint32_t b1 = __ballot_sync(0xffffffffu, (q & 2u) != 0);
        const uint32_t b0 = __ballot_sync(0xffffffffu, (q & 1u) != 0);
        const uint32_t bf = __ballot_sync(0xffffffffu, fold_bits[d] != 0);
        if (lane == 0) {
            page32[(kOffS0 + 8 * d) / 4 + warp] = b3;
            page32[(kOffS2 + 8 * d) / 4 + warp] = b2;
            page32[(kOffS3 + 8 * d) / 4 + warp] = b1;
            page32[(kOffS5 + 8 * d) / 4 + warp] = b0;
            page32[(kOffS4 + 8 * d) / 4 + warp] = bf;
        }
    }
    for (int d = 0; d < 128; ++d) {
        const uint32_t bm = __ballot_sync(0xffffffffu, mid_bits[d] != 0);
        if (lane == 0) page32[(kOffS1 + 8 * d) / 4 + warp] = bm;
    }
    __syncthreads();
    uint8_t* page8 = reinterpret_cast<uint8_t*>(s_page);
    {
        uint8_t* m = page8 + kOffMeta + 7 * t;
        m[0] = (uint8_t)h_scale; m[1] = (uint8_t)(h_scale >> 8);
        m[2] = (uint8_t)h_offset; m[3] = (uint8_t)(h_offset >> 8);
        m[4] = (uint8_t)h_tail; m[5] = (uint8_t)(h_tail >> 8);
        m[6] = flags;
    }
    __syncthreads();
    if (t == 0) {
        const uint64_t n_in = min((uint64_t)64, n - blk * 64);
        uint64_t tomb = 0;
        for (uint64_t i = n_in; i < 64; ++i) tomb |= 1ull << i;
        page32[kOffMinTs / 4] = s_red[0];
        page32[kOffMaxTs / 4] = s_red[1];
        page32[kOffSrc / 4] = s_red[2];
        s_page[kOffTomb / 8] = tomb;
        page32[kOffCrc / 4] = 0u;
        page32[kOffCrc / 4] = crc32_bytes(page8, kBlockBytes, s_crc);
        if (block_ts) block_ts[blk] = make_uint2(s_red[0], s_red[1]);
    }
    __syncthreads();
    if (pax_out) {
        uint4* dst = reinterpret_cast<uint4*>(pax_out + blk * kBlockBytes);
        for (int i = t; i < 256; i += kEncThreads) dst[i] = reinterpret_cast<const uint4*>(s_page)[i];
    }
    if (pages) {
        uint32_t w[16];
        for (int i = 0; i < 16; ++i) w[i] = 0;
        for (int d = 0; d < 64; ++d) w[d >> 3] |= (uint32_t)lv4[d] << (4 * (d & 7));
        for (int d = 0; d < 128; ++d) w[8 + (d >> 5)] |= (uint32_t)mid_bits[d] << (d & 31);
        for (int d = 0; d < 64; ++d) w[12 + (d >> 5)] |= (uint32_t)fold_bits[d] << (d & 31);
        const uint64_t tomb = s_page[kOffTomb / 8];
        w[14] = (uint32_t)h_scale | ((uint32_t)h_offset << 16);
        w[15] = (uint32_t)h_tail | ((uint32_t)flags << 16) | ((uint32_t)((tomb >> t) & 1u) << 24);
        uint4* dst = pages + blk * 256 + t;
        for (int ch = 0; ch < 4; ++ch) dst[64 * ch] = make_uint4(w[4 * ch], w[4 * ch + 1], w[4 * ch + 2], w[4 * ch + 3]);
    }
}

// EdenFit::fit_band, src/eden.rs:130-161: mean[d] = (sum over rows in order) * (1 / n)
__global__ void eden_fit_kernel(const float* __restrict__ rows, uint64_t n, uint32_t dims, uint32_t start,
                                uint32_t width, float* __restrict__ mean) {
    const uint32_t d = blockIdx.x * blockDim.x + threadIdx.x;
    if (d >= width) return;
    const float* col = rows + start + d;
    float s = 0.0f;
    uint64_t r = 0;
    for (; r + 8 <= n; r += 8) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = __ldg(col + (r + j) * (uint64_t)dims);
#pragma unroll
        for (int j = 0; j < 8; ++j) s = f_add(s, v[j]);
    }
    for (; r < n; ++r) s = f_add(s, __ldg(col + r * (uint64_t)dims));
    const float inv = f_div(1.0f, __ull2float_rn(n));
    mean[d] = f_mul(s, inv);
}

__device__ void synth_row_dev(uint64_t seed, uint64_t row, uint32_t dims, float* out) {
    float ss = 0.0f;
    for (uint32_t d = 0; d < dims; ++d) {
        const float sigma = f_div(1.0f, __fsqrt_rn((float)(d + 1)));
        const float v = f_mul(ih_gauss(seed, row * (uint64_t)dims + d), sigma);
        ss = f_add(ss, f_mul(v, v));
    }
    const float nrm = fmaxf(__fsqrt_rn(ss), 1e-12f);
    for (uint32_t d = 0; d < dims; ++d) {
        const float sigma = f_div(1.0f, __fsqrt_rn((float)(d + 1)));
        const float v = f_mul(ih_gauss(seed, row * (uint64_t)dims + d), sigma);
        out[d] = f_div(v, nrm);
    }
}

__global__ void synth_docs_kernel(uint64_t seed, uint64_t row0, uint64_t n, uint32_t dims, float* __restrict__ out) {
    const uint64_t r = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
    if (r >= n) return;
    synth_row_dev(seed, row0 + r, dims, out + r * (uint64_t)dims);
}

__global__ void synth_queries_kernel(uint64_t doc_seed, uint64_t n_docs, uint64_t q_seed, uint64_t n_q, uint32_t dims,
                                     float sigma, float* __restrict__ out, uint64_t* __restrict__ pick) {
    const uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
    if (i >= n_q) return;
    const uint64_t noise_seed = splitmix64(q_seed ^ 0x6E6F697365ULL);
    const uint64_t pk = splitmix64(q_seed * 0x9E3779B97F4A7C15ULL + i) % n_docs;
    if (pick) pick[i] = pk;
    float* q = out + i * (uint64_t)dims;
    synth_row_dev(doc_seed, pk, dims, q);  // doc row first, then add noise in place
    float ss = 0.0f;
    for (uint32_t d = 0; d < dims; ++d) {
        const float v = f_add(q[d], f_mul(sigma, ih_gauss(noise_seed, i * (uint64_t)dims + d)));
        q[d] = v;
        ss = f_add(ss, f_mul(v, v));
    }
    const float nrm = fmaxf(__fsqrt_rn(ss), 1e-12f);
    for (uint32_t d = 0; d < dims; ++d) q[d] = f_div(q[d], nrm);
}

// Maxima of the per-slot score factors (|scale|, |offset|, mid_n, max(high_n, 1e-6)) over a run of
// scan-layout pages, merged into m[0..3] with atomic max on the float bit patterns (valid for
// nonnegative floats; NaN is mapped to +inf first so it cannot hide behind a smaller value).
// Tombstoned slots are included: a superset only loosens the bound the scans derive from it.
__device__ __forceinline__ unsigned max_word(float v) {
    return v == v ? __float_as_uint(v) : 0x7F800000u;
}

__global__ void __launch_bounds__(256) metamax_kernel(const uint4* __restrict__ pages, uint64_t n_slots,
                                                      float* __restrict__ m) {
    unsigned a = 0u, b = 0u, c = 0u, d = 0u;
    for (uint64_t i = blockIdx.x * 256ull + threadIdx.x; i < n_slots; i += (uint64_t)gridDim.x * 256ull) {
        const uint4 w = __ldg(pages + (i >> 6) * 256 + 192 + (i & 63));  // chunk 3: meta words
        const SlotMeta sm = decode_slot_meta(w.z, w.w);
        a = max(a, max_word(fabsf(sm.scale)));
        b = max(b, max_word(fabsf(sm.offset)));
        c = max(c, max_word(sm.mid_n));
        d = max(d, max_word(fmaxf(sm.high_n, 1e-6f)));
    }
    a = __reduce_max_sync(0xffffffffu, a);
    b = __reduce_max_sync(0xffffffffu, b);
    c = __reduce_max_sync(0xffffffffu, c);
    d = __reduce_max_sync(0xffffffffu, d);
    if ((threadIdx.x & 31) == 0) {
        unsigned* mu = reinterpret_cast<unsigned*>(m);
        atomicMax(mu + 0, a);
        atomicMax(mu + 1, b);
        atomicMax(mu + 2, c);
        atomicMax(mu + 3, d);
    }
}

}  // namespace

int launch_metamax(const uint4* d_pages, uint64_t n_blocks, float* d_metamax, cudaStream_t stream) {
    if (n_blocks == 0) return 0;
    const uint64_t slots = n_blocks * 64;
    const unsigned grid = (unsigned)std::min<uint64_t>((slots + 255) / 256, 148ull * 8);
    metamax_kernel<<<grid, 256, 0, stream>>>(d_pages, slots, d_metamax);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int launch_transcode(const uint8_t* d_pax, uint64_t n_blocks, uint4* d_pages, uint2* d_ts, cudaStream_t stream) {
    if (n_blocks == 0) return 0;
    transcode_kernel<<<(unsigned)n_blocks, 64, 0, stream>>>(d_pax, d_pages, d_ts);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int launch_encode(const float* d_rows, uint64_t n, uint32_t dims, const uint32_t* d_ts, const uint32_t* d_src,
                  uint32_t src_const, uint32_t prefix_codec, const float* d_eden_mean, uint64_t eden_seed,
                  const float* d_mid_mean, uint64_t mid_seed, uint8_t* d_pax, uint4* d_pages, uint2* d_block_ts,
                  cudaStream_t stream) {
    if (n == 0) return 0;
    const uint64_t nb = (n + 63) / 64;
    encode_kernel<<<(unsigned)nb, kEncThreads, 0, stream>>>(d_rows, n, dims, d_ts, d_src, src_const, prefix_codec,
                                                           d_eden_mean, eden_seed, d_mid_mean, mid_seed, d_pax,
                                                           d_pages, d_block_ts);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int launch_eden_fit(const float* d_rows, uint64_t n, uint32_t dims, uint32_t start, uint32_t width, float* d_mean,
                    cudaStream_t stream) {
    eden_fit_kernel<<<(width + 63) / 64, 64, 0, stream>>>(d_rows, n, dims, start, width, d_mean);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int launch_synth_docs(uint64_t seed, uint64_t row0, uint64_t n, uint32_t dims, float* d_out, cudaStream_t stream) {
    if (n == 0) return 0;
    synth_docs_kernel<<<(unsigned)((n + 127) / 128), 128, 0, stream>>>(seed, row0, n, dims, d_out);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int launch_synth_queries(uint64_t doc_seed, uint64_t n_docs, uint64_t q_seed, uint64_t n_q, uint32_t dims,
                         float sigma, float* d_out, uint64_t* d_pick, cudaStream_t stream) {
    if (n_q == 0) return 0;
    synth_queries_kernel<<<(unsigned)((n_q + 127) / 128), 128, 0, stream>>>(doc_seed, n_docs, q_seed, n_q, dims,
                                                                           sigma, d_out, d_pick);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace mrl
