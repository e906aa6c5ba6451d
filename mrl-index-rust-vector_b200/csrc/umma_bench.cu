// umma_bench.cu — throughput of back-to-back tcgen05.mma kind::i8 (M = 128, K = 32) for several N,
// with A in tensor memory (TS) or shared memory (SS), one CTA per SM: the rates the batched tensor
// scan is planned against. Build: make umma_bench; run: _build/umma_bench (needs an sm_100 GPU).
#include <cstdio>
#include <vector>
#include "umma.cuh"

template <int N, bool TS>
__global__ void __launch_bounds__(128) k_bench(int iters, unsigned long long* cyc, uint32_t* err) {
    extern __shared__ __align__(1024) uint8_t sm[];
    uint8_t* sB = sm;              // N x 32 bytes
    uint8_t* sA = sm + 256 * 32;   // 128 x 32
    __shared__ uint32_t s_taddr;
    __shared__ __align__(8) uint64_t bar;
    const int tid = threadIdx.x, warp = tid >> 5;
    if (warp == 0) { tc::tmem_alloc(&s_taddr, 512); tc::tmem_relinquish(); }
    if (tid == 0) { tc::mbar_init(&bar, 1); tc::fence_mbar_init(); }
    for (int i = tid; i < 256 * 32 + 128 * 32; i += 128) sm[i] = (uint8_t)(i * 7);
    tc::fence_proxy_async_smem();
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tbase = s_taddr;
    if (tid == 0) {
        const uint32_t idesc = tc::idesc_i8(128, N);
        const uint64_t bd = tc::sdesc_kmajor(tc::smem_u32(sB), (N / 8) * 128, 128);
        const uint64_t ad = tc::sdesc_kmajor(tc::smem_u32(sA), 16 * 128, 128);
        const unsigned long long t0 = clock64();
        for (int i = 0; i < iters; ++i) {
            if (TS) tc::mma_i8_ts(tbase + 256, tbase, bd, idesc, i > 0);
            else tc::mma_i8_ss(tbase + 256, ad, bd, idesc, i > 0);
        }
        tc::mma_commit(&bar);
        const bool ok = tc::mbar_wait(&bar, 0, 1u << 24);
        const unsigned long long t1 = clock64();
        cyc[blockIdx.x] = t1 - t0;
        if (!ok) atomicOr(err, 1u);
    } else {
        // the other threads wait for the same completion
        tc::mbar_wait(&bar, 0, 1u << 24);
    }
    tc::fence_before();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tbase, 512);
}

template <int N, bool TS>
void run(int ctas) {
    unsigned long long* dc; uint32_t* de;
    cudaMalloc(&dc, ctas * 8); cudaMalloc(&de, 4); cudaMemset(de, 0, 4);
    cudaFuncSetAttribute(k_bench<N, TS>, cudaFuncAttributeMaxDynamicSharedMemorySize, 130 * 1024);
    const int iters = 4096;
    k_bench<N, TS><<<ctas, 128, 130 * 1024>>>(16, dc, de);  // warm-up
    cudaEvent_t e0, e1; cudaEventCreate(&e0); cudaEventCreate(&e1);
    cudaEventRecord(e0);
    k_bench<N, TS><<<ctas, 128, 130 * 1024>>>(iters, dc, de);
    cudaEventRecord(e1);
    cudaError_t e = cudaDeviceSynchronize();
    float ms = 0; cudaEventElapsedTime(&ms, e0, e1);
    std::vector<unsigned long long> c(ctas); uint32_t err;
    cudaMemcpy(c.data(), dc, ctas * 8, cudaMemcpyDeviceToHost); cudaMemcpy(&err, de, 4, cudaMemcpyDeviceToHost);
    double macs = (double)ctas * iters * 128.0 * N * 32.0;
    printf("N=%3d %s ctas=%3d: %s err=%u cycles/MMA %.1f, %.3f ms, %.0f TOPS (int8 ops = 2*MAC)\n", N, TS ? "TS" : "SS", ctas,
           cudaGetErrorString(e), err, (double)c[0] / iters, ms, 2.0 * macs / (ms * 1e-3) / 1e12);
    cudaFree(dc); cudaFree(de);
}

int main() {
    int sms = 0; cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
    run<64, true>(1); run<64, false>(1); run<128, true>(1); run<256, true>(1); run<256, false>(1);
    run<64, true>(sms); run<128, true>(sms); run<256, true>(sms); run<256, false>(sms);
    return 0;
}
