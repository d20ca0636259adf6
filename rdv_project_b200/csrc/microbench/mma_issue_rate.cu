// Measurement tool (not part of librdvb.so): tcgen05.mma issue rate on
// B200 for the shapes the fused-MLP kernels issue (M = 128, K = 16 per
// instruction, float16 operands, fp32 accumulation), one CTA per SM.
//
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 \
//        -o mma_issue_rate rdv_project_b200/csrc/microbench/mma_issue_rate.cu && ./mma_issue_rate
//
// Part 1: one issuing thread, N in {16, 32, 64, 128, 256}, A from shared
// memory (SS) or TMEM (TS), K steps per commit + mbarrier wait, 1..4
// accumulators round-robin. Part 2: 1..6 issuing threads (one per warp),
// each its own accumulator and barrier, 1/4/8 MMAs per commit + wait -- the
// per-layer pattern of the MLP kernel's slots. Operands are zero; every
// wait is bounded (ptx.cuh), and a timed-out thread drains its MMAs before
// TMEM is released.
#include <cstdio>
#include <cuda_runtime.h>

#include "../ptx.cuh"
using namespace rdvb;

__device__ unsigned long long g_cycles[148];
__device__ unsigned g_fail;

// Shared set-up: zeroed operand tiles, one barrier per issuer, all of TMEM.
struct Setup {
    uint32_t base, tm;
};
__device__ __forceinline__ Setup setup(uint8_t* smem_raw, uint32_t bytes, uint64_t* bars, int n_bars,
                                       uint32_t* tmem_slot, uint32_t* abort_word) {
    const uint32_t raw = smem_addr(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    for (uint32_t i = threadIdx.x; i < bytes / 16; i += blockDim.x) st_shared_v4(base + i * 16, 0, 0, 0, 0);
    fence_proxy_async_smem();
    if (threadIdx.x == 0) {
        for (int i = 0; i < n_bars; ++i) mbar_init(smem_addr(&bars[i]), 1);
        *abort_word = 0;
        fence_mbarrier_init();
    }
    if (threadIdx.x < 32) {
        tmem_alloc(smem_addr(tmem_slot), 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    return {base, *tmem_slot};
}

__device__ __forceinline__ void teardown(uint32_t tm) {
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x < 32) {
        tc_fence_after();
        tmem_dealloc(tm, 512);
    }
}

// Part 1: one issuing thread.
template <int N, int TS, int NACC, int KS>
__global__ void __launch_bounds__(128, 1) one_issuer(int iters) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint32_t tmem_slot, abort_word;
    __shared__ __align__(8) uint64_t bars[1];
    const Setup su = setup(smem_raw, 16384 + N * 128, bars, 1, &tmem_slot, &abort_word);
    if (threadIdx.x == 0) {
        const uint32_t idesc = umma_idesc_f16(N, 0);
        const uint64_t adesc = umma_desc_sw128(su.base);
        const uint64_t bdesc = umma_desc_sw128(su.base + 16384);
        const uint32_t a_tm = su.tm + 256;  // A (TS): columns 256..287
        const uint32_t bar = smem_addr(&bars[0]);
        const long long t0 = clock64();
        uint32_t ph = 0;
        bool ok = true;
        for (int it = 0; it < iters && ok; ++it) {
            for (int j = 0; j < KS; ++j) {
                const uint32_t d = su.tm + static_cast<uint32_t>((it * KS + j) % NACC) * (N > 64 ? N : 64);
                if (TS) umma_f16_ts(d, a_tm + (j & 3) * 8u, bdesc + (j & 3) * 2, idesc, 1u);
                else umma_f16(d, adesc + (j & 3) * 2, bdesc + (j & 3) * 2, idesc, 1u);
            }
            umma_commit(bar);
            ok = mbar_wait(bar, ph, &abort_word, &g_fail, 1u);
            ph ^= 1u;
        }
        if (!ok) {
            umma_commit(bar);
            drain_wait(bar, ph);
        }
        g_cycles[blockIdx.x] = static_cast<unsigned long long>(clock64() - t0);
    }
    teardown(su.tm);
}

// Part 2: ISS issuing threads, lane 0 of each warp.
template <int N, int ISS, int KS>
__global__ void __launch_bounds__(ISS * 32, 1) many_issuers(int iters) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint32_t tmem_slot, abort_word;
    __shared__ __align__(8) uint64_t bars[8];
    const Setup su = setup(smem_raw, N * 128, bars, 8, &tmem_slot, &abort_word);
    const int w = threadIdx.x >> 5;
    const long long t0 = clock64();
    if ((threadIdx.x & 31) == 0) {
        const uint32_t idesc = umma_idesc_f16(N, 0);
        const uint64_t bdesc = umma_desc_sw128(su.base);
        const uint32_t d = su.tm + w * 64;  // accumulators at columns 0, 64, ... (N <= 64)
        const uint32_t a_tm = su.tm + 384;  // shared A (TS)
        const uint32_t bar = smem_addr(&bars[w]);
        uint32_t ph = 0;
        bool ok = true;
        for (int it = 0; it < iters && ok; ++it) {
            for (int j = 0; j < KS; ++j) umma_f16_ts(d, a_tm + (j & 3) * 8u, bdesc + (j & 3) * 2, idesc, j > 0);
            umma_commit(bar);
            ok = mbar_wait(bar, ph, &abort_word, &g_fail, 1u);
            ph ^= 1u;
        }
        if (!ok) {
            umma_commit(bar);
            drain_wait(bar, ph);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) g_cycles[blockIdx.x] = static_cast<unsigned long long>(clock64() - t0);
    teardown(su.tm);
}

static double mean_cycles() {
    unsigned long long c[148];
    cudaMemcpyFromSymbol(c, g_cycles, sizeof(c));
    double avg = 0;
    for (int i = 0; i < 148; ++i) avg += static_cast<double>(c[i]);
    return avg / 148;
}

static bool report(const char* name, double mmas, double macs_per_mma, double per_round_div) {
    const cudaError_t e = cudaDeviceSynchronize();
    unsigned fail = 0;
    cudaMemcpyFromSymbol(&fail, g_fail, sizeof(fail));
    const double avg = mean_cycles();
    printf("%-30s err=%d timeouts=%u cycles/MMA=%7.1f MAC/clk/SM=%6.0f (%.2f of 4096) cycles/round=%7.1f\n", name,
           static_cast<int>(e), fail, avg / mmas, macs_per_mma * mmas / avg, macs_per_mma * mmas / avg / 4096.0,
           avg / per_round_div);
    return e == cudaSuccess && fail == 0;
}

template <int N, int TS, int NACC, int KS>
static bool part1(const char* name, int iters) {
    auto k = one_issuer<N, TS, NACC, KS>;
    const int smem = 16384 + N * 128 + 2048;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    k<<<148, 128, smem>>>(iters);
    return report(name, static_cast<double>(iters) * KS, 128.0 * N * 16, iters);
}

template <int N, int ISS, int KS>
static bool part2(const char* name, int iters) {
    auto k = many_issuers<N, ISS, KS>;
    const int smem = N * 128 + 2048;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    k<<<148, ISS * 32, smem>>>(iters);
    return report(name, static_cast<double>(iters) * KS * ISS, 128.0 * N * 16, iters);
}

int main() {
    bool ok = true;
    ok &= part1<64, 1, 1, 4>("N64 TS 1 acc, 4 per commit", 2000);
    ok &= part1<64, 1, 1, 16>("N64 TS 1 acc, 16 per commit", 500);
    ok &= part1<64, 1, 4, 16>("N64 TS 4 acc, 16 per commit", 500);
    ok &= part1<64, 0, 1, 16>("N64 SS 1 acc, 16 per commit", 500);
    ok &= part1<16, 1, 1, 16>("N16 TS 1 acc, 16 per commit", 500);
    ok &= part1<32, 1, 1, 16>("N32 TS 1 acc, 16 per commit", 500);
    ok &= part1<128, 1, 1, 16>("N128 TS 1 acc, 16 per commit", 500);
    ok &= part1<128, 0, 1, 16>("N128 SS 1 acc, 16 per commit", 500);
    ok &= part1<256, 1, 1, 16>("N256 TS 1 acc, 16 per commit", 500);
    ok &= part1<256, 0, 1, 16>("N256 SS 1 acc, 16 per commit", 500);
    ok &= part2<64, 1, 4>("N64 1 issuer, 4 per commit", 4000);
    ok &= part2<64, 2, 4>("N64 2 issuers, 4 per commit", 4000);
    ok &= part2<64, 4, 4>("N64 4 issuers, 4 per commit", 4000);
    ok &= part2<64, 5, 4>("N64 5 issuers, 4 per commit", 4000);
    ok &= part2<64, 6, 4>("N64 6 issuers, 4 per commit", 4000);
    ok &= part2<64, 1, 1>("N64 1 issuer, 1 per commit", 4000);
    ok &= part2<64, 4, 1>("N64 4 issuers, 1 per commit", 4000);
    ok &= part2<16, 4, 4>("N16 4 issuers, 4 per commit", 4000);
    ok &= part2<64, 4, 8>("N64 4 issuers, 8 per commit", 2000);
    ok &= part2<64, 6, 8>("N64 6 issuers, 8 per commit", 2000);
    return ok ? 0 : 1;
}
