// Direct 'same' stride-1 KHxKW convolution as an implicit GEMM on tcgen05:
// the reference's tensor-core convolution operators (Conv2DTensorOpFast /
// Simple / Simple3x3 / Window3x3, rdv/domain/nn.py:608-999) with float16 or
// bfloat16 operands and fp32 accumulation.
//
// For a block of 128 consecutive output pixels (rows of the flattened
// [N*H*W, COUT] output), D[128 x COUT] = sum over taps (kh, kw) of
// A_tap[128 x CIN] * W_tap[CIN x COUT], where A_tap holds each pixel's
// input at (oh + kh - KH/2, ow + kw - KW/2) (zero outside the image).
//
// Design (one persistent CTA per SM, 16 warps):
//   * every tap's weights stay resident in shared memory (K-major,
//     128-byte swizzle, one COUT x 128-byte block per tap), loaded once by
//     one bulk copy;
//   * warps 0-10 stage the A tile of each (block, tap) into a ring of 4
//     shared-memory tiles (fp32 or fp16 input -> f16/bf16), waiting until
//     the GEMM that last read the tile released it;
//   * warp 15 issues, per tap, CIN/16 MMAs (M = 128, N = COUT) into the
//     block's TMEM accumulator once the tap's tile is written; the first
//     tap's MMAs and the others are separate code paths, so every MMA's
//     accumulate flag is a compile-time constant;
//   * accumulators are double buffered across blocks; warps 11-14 (one per
//     TMEM lane quadrant) add the bias to each finished block and store it
//     while the next block's GEMMs run, then free the half for block b + 2.
// Every wait is bounded (ptx.cuh) and reports through the status word.
#pragma once
#include <cuda.h>  // CUtensorMap (the type only; the map is encoded on the host)
#include "ptx.cuh"

namespace rdvb {
namespace convtc {

constexpr int kTileM = 128;
constexpr int kXWarps = 11;                       // staging warps 0-10
constexpr int kXThreads = kXWarps * 32;
constexpr int kEpiWarp0 = 11;                     // epilogue warps 11-14, one per TMEM lane quadrant
constexpr int kIssueWarp = 15;
constexpr int kThreads = 16 * 32;
constexpr int kRing = 4;                          // A tiles in flight
constexpr uint32_t kATileBytes = kTileM * 128;    // 128 rows x 64 16-bit K elements
constexpr int kMaxCin = 64;
constexpr int kMaxCout = 256;                     // two accumulators of COUT columns in 512
constexpr int kMaxTaps = 25;
constexpr uint32_t kTmemCols = 512;
constexpr int kMaxItems = 3;                      // (pixel, 8-channel) items per staging thread: 128 * 8 / 352

struct Params {
    const void* x;            // [N*H*W, CIN] float32 or float16
    float* y;                 // [N*H*W, COUT] float32
    const uint8_t* wpack;     // per tap: COUT rows x 128 bytes, K-major SW128
    const float* bias;        // [COUT] or null
    long long n_pix;
    int h, w, cin, cout, kh, kw, taps;
    int x_f16, bf16;
    int n_blocks;
    uint32_t w_bytes;         // taps * COUT * 128
    uint32_t off_a, off_bar;
    uint32_t idesc;
};

enum : int {
    kBarWFull = 0,
    kBarAFull = 1,              // + ring slot: A tile written (one arrival per staging warp)
    kBarAEmpty = 1 + kRing,     // + ring slot: the GEMMs reading it are done (commit)
    kBarDFull = 1 + 2 * kRing,  // + half: a block's accumulator is final (commit)
    kBarDEmpty = 3 + 2 * kRing, // + half: the epilogue read it (one arrival per epilogue warp)
    kBarDrain = 5 + 2 * kRing,
    kNumBars = 6 + 2 * kRing,
};
constexpr uint32_t kBarBlockBytes = kNumBars * 8 + 16;

__device__ __forceinline__ uint32_t pack2(float a, float b, int bf16) {
    return bf16 ? pack_bf16x2(a, b) : pack_f16x2(a, b);
}

// The KS MMAs (K = 16 each) of one tap; FIRST: the block's first tap, whose
// first MMA overwrites the accumulator.
template <int KS, bool FIRST>
__device__ __forceinline__ void issue_tap_ks(uint32_t d, uint64_t a_desc, uint64_t b_desc, uint32_t idesc) {
#pragma unroll
    for (int k = 0; k < KS; ++k)
        umma_f16(d, a_desc + 2u * k, b_desc + 2u * k, idesc, (FIRST && k == 0) ? 0u : 1u);
}

template <bool FIRST>
__device__ __forceinline__ void issue_tap(int ksteps, uint32_t d, uint64_t a_desc, uint64_t b_desc, uint32_t idesc) {
    switch (ksteps) {
        case 1: issue_tap_ks<1, FIRST>(d, a_desc, b_desc, idesc); break;
        case 2: issue_tap_ks<2, FIRST>(d, a_desc, b_desc, idesc); break;
        case 3: issue_tap_ks<3, FIRST>(d, a_desc, b_desc, idesc); break;
        default: issue_tap_ks<4, FIRST>(d, a_desc, b_desc, idesc); break;
    }
}

__global__ void __launch_bounds__(kThreads, 1) conv_tc_kernel(const __grid_constant__ Params p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_addr(smem_raw);
    const uint32_t base = (raw_addr + 1023u) & ~1023u;
    uint8_t* const base_ptr = smem_raw + (base - raw_addr);
    const uint32_t w_base = base;
    const uint32_t a_base = base + p.off_a;
    const uint32_t bar_base = base + p.off_bar;
    auto bar = [&](int i) -> uint32_t { return bar_base + 8u * static_cast<uint32_t>(i); };
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base_ptr + p.off_bar + kNumBars * 8);
    volatile uint32_t* abort = reinterpret_cast<volatile uint32_t*>(base_ptr + p.off_bar + kNumBars * 8 + 4);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        mbar_init(bar(kBarWFull), 1);
        for (int s = 0; s < kRing; ++s) {
            mbar_init(bar(kBarAFull + s), kXWarps);
            mbar_init(bar(kBarAEmpty + s), 1);
        }
        mbar_init(bar(kBarDFull), 1);
        mbar_init(bar(kBarDFull + 1), 1);
        mbar_init(bar(kBarDEmpty), 4);
        mbar_init(bar(kBarDEmpty + 1), 4);
        mbar_init(bar(kBarDrain), 1);
        *abort = 0u;
        fence_mbarrier_init();
    }
    if (warp == 0) {
        tmem_alloc(smem_addr(tmem_slot), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int n_mine = blockIdx.x < p.n_blocks ? (p.n_blocks - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const int taps = p.taps;
    const uint32_t d_cols = static_cast<uint32_t>(p.cout);
    bool ok = true;

    if (warp == kIssueWarp) {
        // --------------------------------------------------- MMA issuer
        if (lane == 0) {
            mbar_arrive_expect_tx(bar(kBarWFull), p.w_bytes);
            bulk_g2s(w_base, p.wpack, p.w_bytes, bar(kBarWFull));
            ok = mbar_wait(bar(kBarWFull), 0u, abort, &g_status, kStatusTimeoutWFull);
            const uint64_t w_desc0 = umma_desc_sw128(w_base);
            const uint64_t a_desc0 = umma_desc_sw128(a_base);
            const uint64_t tap_step = static_cast<uint64_t>(p.cout) * 8u;  // one tap block, 16-byte units
            const int ksteps = p.cin >> 4;
            bool issued = false;
            for (int bl = 0; ok && bl < n_mine; ++bl) {
                const uint32_t d = tmem_base + (bl & 1) * d_cols;
                // the accumulator half was read out by the epilogue of block bl - 2
                if (bl >= 2 && !mbar_wait(bar(kBarDEmpty + (bl & 1)), ((bl >> 1) - 1) & 1, abort, &g_status,
                                          kStatusTimeoutOther)) {
                    ok = false;
                    break;
                }
                for (int t = 0; t < taps; ++t) {
                    const int g = bl * taps + t;
                    const int s = g % kRing;
                    if (!mbar_wait(bar(kBarAFull + s), (g / kRing) & 1, abort, &g_status, kStatusTimeoutAFull)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t a_desc = a_desc0 + static_cast<uint64_t>(s) * (kATileBytes >> 4);
                    const uint64_t b_desc = w_desc0 + static_cast<uint64_t>(t) * tap_step;
                    if (t == 0) issue_tap<true>(ksteps, d, a_desc, b_desc, p.idesc);
                    else issue_tap<false>(ksteps, d, a_desc, b_desc, p.idesc);
                    issued = true;
                    umma_commit(bar(kBarAEmpty + s));  // the tile may be rewritten
                    if (t == taps - 1) umma_commit(bar(kBarDFull + (bl & 1)));
                }
            }
            if (!ok) *abort = 1u;
            if (issued) {
                // every issued MMA completes before TMEM is released
                umma_commit(bar(kBarDrain));
                const uint64_t t0 = global_timer_ns();
                while (!mbar_try_wait_sleep(bar(kBarDrain), 0u, 500000u))
                    if (global_timer_ns() - t0 > RDVB_WAIT_LIMIT_NS) {
                        atomicOr(&g_status, kStatusTimeoutDrain);
                        break;
                    }
            }
        }
    } else if (warp >= kEpiWarp0) {
        // -------------------------------------------------------- epilogue
        // Warp (11 + q) % 4 = its TMEM lane quadrant: every 16-column chunk
        // of its 32 pixels, + bias, to the output; then the half is free.
        const int quad = warp & 3;
        const int n_chunks = p.cout >> 4;
        for (int bl = 0; ok && bl < n_mine; ++bl) {
            const uint32_t half = bl & 1;
            if (!mbar_wait_warp(bar(kBarDFull + half), (bl >> 1) & 1, abort, &g_status, kStatusTimeoutAccFull)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const long long pix = (static_cast<long long>(blockIdx.x) + static_cast<long long>(bl) * gridDim.x) *
                                      kTileM + quad * 32 + lane;
            const bool valid = pix < p.n_pix;
            for (int c = 0; c < n_chunks; ++c) {
                uint32_t r[16];
                tmem_ld16(tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + half * d_cols + 16u * c, r);
                tmem_wait_ld(r);
                if (valid) {
                    float o[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i)
                        o[i] = __uint_as_float(r[i]) + (p.bias ? __ldg(p.bias + 16 * c + i) : 0.0f);
                    float4* dst = reinterpret_cast<float4*>(p.y + pix * p.cout + 16 * c);
                    dst[0] = make_float4(o[0], o[1], o[2], o[3]);
                    dst[1] = make_float4(o[4], o[5], o[6], o[7]);
                    dst[2] = make_float4(o[8], o[9], o[10], o[11]);
                    dst[3] = make_float4(o[12], o[13], o[14], o[15]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kBarDEmpty + half));
        }
        if (!ok) *abort = 1u;
    } else {
        // ------------------------------------------------------- staging
        const int xt = threadIdx.x;  // 0 .. kXThreads - 1
        const int cch = p.cin >> 3;  // 8-channel chunks per pixel
        const int items = kTileM * cch;
        const long long row_stride = static_cast<long long>(p.w) * p.cin;
        // per item, fixed over the taps: the input element offset of the
        // pixel's own position and channel chunk, its row / column, and the
        // item's offset inside an A tile
        long long item_e[kMaxItems];
        int pix_oh[kMaxItems], pix_ow[kMaxItems];
        uint32_t item_soff[kMaxItems];
        bool pix_ok[kMaxItems];

        for (int bl = 0; ok && bl < n_mine; ++bl) {
            const long long blk = static_cast<long long>(blockIdx.x) + static_cast<long long>(bl) * gridDim.x;
            // this thread's pixels of the block (fixed over the taps)
#pragma unroll
            for (int i = 0; i < kMaxItems; ++i) {
                const int item = xt + i * kXThreads;
                pix_ok[i] = false;
                pix_oh[i] = pix_ow[i] = 0;
                item_e[i] = 0;
                item_soff[i] = 0;
                if (item < items) {
                    const int r = item / cch, c = item - (item / cch) * cch;
                    item_soff[i] = sw128_offset(static_cast<uint32_t>(r), static_cast<uint32_t>(c * 8), kTileM);
                    const long long pix = blk * kTileM + r;
                    if (pix < p.n_pix) {
                        pix_ok[i] = true;
                        pix_ow[i] = static_cast<int>(pix % p.w);
                        const long long rest = pix / p.w;
                        pix_oh[i] = static_cast<int>(rest % p.h);
                        item_e[i] = pix * p.cin + c * 8;  // NHWC: the pixel's own element offset
                    }
                }
            }
            int dh = -(p.kh / 2), dw = -(p.kw / 2);  // tap offsets, row-major over (kh, kw)
            for (int t = 0; ok && t < taps; ++t) {
                const int g = bl * taps + t;
                const int s = g % kRing;
                if (!mbar_wait_warp(bar(kBarAEmpty + s), ((g / kRing) & 1) ^ 1, abort, &g_status,
                                    kStatusTimeoutXEmpty)) {
                    ok = false;
                    break;
                }
                const long long shift = dh * row_stride + static_cast<long long>(dw) * p.cin;
                const uint32_t a_tile = a_base + static_cast<uint32_t>(s) * kATileBytes;
#pragma unroll
                for (int i = 0; i < kMaxItems; ++i) {
                    const int item = xt + i * kXThreads;
                    if (item >= items) break;
                    uint32_t q0 = 0u, q1 = 0u, q2 = 0u, q3 = 0u;
                    const int ih = pix_oh[i] + dh, iw = pix_ow[i] + dw;
                    if (pix_ok[i] && ih >= 0 && ih < p.h && iw >= 0 && iw < p.w) {
                        const long long e = item_e[i] + shift;
                        if (p.x_f16) {
                            const uint4 v = __ldg(reinterpret_cast<const uint4*>(static_cast<const __half*>(p.x) + e));
                            if (p.bf16) {
                                const __half2* h2 = reinterpret_cast<const __half2*>(&v);
                                const float2 f0 = __half22float2(h2[0]), f1 = __half22float2(h2[1]);
                                const float2 f2 = __half22float2(h2[2]), f3 = __half22float2(h2[3]);
                                q0 = pack2(f0.x, f0.y, 1); q1 = pack2(f1.x, f1.y, 1);
                                q2 = pack2(f2.x, f2.y, 1); q3 = pack2(f3.x, f3.y, 1);
                            } else {
                                q0 = v.x; q1 = v.y; q2 = v.z; q3 = v.w;
                            }
                        } else {
                            const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(p.x) + e);
                            const float4 a = __ldg(src), b = __ldg(src + 1);
                            q0 = pack2(a.x, a.y, p.bf16); q1 = pack2(a.z, a.w, p.bf16);
                            q2 = pack2(b.x, b.y, p.bf16); q3 = pack2(b.z, b.w, p.bf16);
                        }
                    }
                    st_shared_v4(a_tile + item_soff[i], q0, q1, q2, q3);
                }
                if (++dw > p.kw - 1 - p.kw / 2) {
                    dw = -(p.kw / 2);
                    ++dh;
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(kBarAFull + s));
            }
        }
        if (!ok) *abort = 1u;
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

// ---------------------------------------------------------------------------
// TMA-fed variant for float16 input with 64 channels and float16 operands
// (the input needs no conversion, so the copy engine stages it directly):
// a block is an 8-row x 16-column rectangle of output pixels of one image,
// and tap (dh, dw)'s A tile is the input box {64 channels, 16 columns, 8
// rows, 1 image} at (0, w0 + dw, h0 + dh, n), loaded by one thread with the
// 128-byte swizzle the MMA reads; the copy zero-fills the box where it
// leaves the image, which is the convolution's 'same' padding.
// Two independent streams, even and odd blocks, each with its producer, its
// half of the tile ring and its MMA issuer (one thread's waits, issues and
// commits per tap bound a single stream), sharing the weights and the
// epilogue; stream i accumulates into TMEM half i. Every ring barrier has
// one producer and one consumer, so parity waits stay within one phase.
//   warps 0, 7: producers of streams 0 and 1 (warp 0 also loads the weights)
//   warps 1, 6: MMA issuers of streams 0 and 1 (warp 1 allocates TMEM)
//   warps 2-5: epilogue, one per TMEM lane quadrant, blocks in order: + bias,
//           store the block's in-image pixels; then frees the accumulator half.
constexpr int kTmaThreads = 8 * 32;
constexpr int kTmaMaxRing = 10;           // both streams' tiles
constexpr int kBoxW = 16, kBoxH = 8;

struct TmaParams {
    CUtensorMap tmap;         // x [N, H, W, 64] float16: dims {64, W, H, N}, box {64, 16, 8, 1}, SWIZZLE_128B
    float* y;                 // [N*H*W, COUT] float32
    const uint8_t* wpack;     // per tap: COUT rows x 128 bytes, K-major SW128
    const float* bias;        // [COUT] or null
    int n, h, w, cout, kh, kw, taps;
    int blocks_w, blocks_h, n_blocks;
    int ring;                 // A tiles per stream (1..5); stream i uses slots [i * ring, (i + 1) * ring)
    uint32_t w_bytes, off_a, off_bar, off_bias, idesc;
};

enum : int {
    kTBarWFull = 0,
    kTBarFull = 1,                            // + ring slot: the box landed (TMA tx)
    kTBarEmpty = 1 + kTmaMaxRing,             // + ring slot: the GEMMs reading it are done (commit)
    kTBarDFull = 1 + 2 * kTmaMaxRing,         // + half
    kTBarDEmpty = 3 + 2 * kTmaMaxRing,        // + half (one arrival per epilogue warp)
    kTBarDrain = 5 + 2 * kTmaMaxRing,         // + issuer
    kTNumBars = 7 + 2 * kTmaMaxRing,
};
constexpr uint32_t kTBarBlockBytes = kTNumBars * 8 + 16;

__device__ __forceinline__ void tma_block_origin(const TmaParams& p, int blk, int& img, int& h0, int& w0) {
    const int per_img = p.blocks_w * p.blocks_h;
    img = blk / per_img;
    const int rem = blk - img * per_img;
    const int hb = rem / p.blocks_w;
    h0 = hb * kBoxH;
    w0 = (rem - hb * p.blocks_w) * kBoxW;
}

__global__ void __launch_bounds__(kTmaThreads, 1) conv_tc_tma_kernel(const __grid_constant__ TmaParams p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_addr(smem_raw);
    const uint32_t base = (raw_addr + 1023u) & ~1023u;
    uint8_t* const base_ptr = smem_raw + (base - raw_addr);
    const uint32_t w_base = base;
    const uint32_t a_base = base + p.off_a;
    const uint32_t bar_base = base + p.off_bar;
    auto bar = [&](int i) -> uint32_t { return bar_base + 8u * static_cast<uint32_t>(i); };
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base_ptr + p.off_bar + kTNumBars * 8);
    volatile uint32_t* abort = reinterpret_cast<volatile uint32_t*>(base_ptr + p.off_bar + kTNumBars * 8 + 4);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int R = p.ring;

    if (threadIdx.x == 0) {
        mbar_init(bar(kTBarWFull), 1);
        for (int s = 0; s < kTmaMaxRing; ++s) {
            mbar_init(bar(kTBarFull + s), 1);
            mbar_init(bar(kTBarEmpty + s), 1);
        }
        for (int h = 0; h < 2; ++h) {
            mbar_init(bar(kTBarDFull + h), 1);
            mbar_init(bar(kTBarDEmpty + h), 4);
        }
        mbar_init(bar(kTBarDrain), 1);
        mbar_init(bar(kTBarDrain + 1), 1);
        *abort = 0u;
        fence_mbarrier_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_addr(tmem_slot), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int n_mine = blockIdx.x < p.n_blocks ? (p.n_blocks - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const int taps = p.taps;
    const uint32_t d_cols = static_cast<uint32_t>(p.cout);
    bool ok = true;

    if (warp == 0 || warp == 7) {
        // ----------------------------------------------------- producers
        const int mi = warp == 0 ? 0 : 1;  // blocks mi, mi + 2, ...
        if (lane == 0) {
            if (mi == 0) {
                mbar_arrive_expect_tx(bar(kTBarWFull), p.w_bytes);
                bulk_g2s(w_base, p.wpack, p.w_bytes, bar(kTBarWFull));
            }
            int g = 0;  // this stream's load count
            for (int bl = mi; ok && bl < n_mine; bl += 2) {
                int img, h0, w0;
                tma_block_origin(p, static_cast<int>(blockIdx.x) + bl * static_cast<int>(gridDim.x), img, h0, w0);
                int dh = -(p.kh / 2), dw = -(p.kw / 2);
                for (int t = 0; t < taps; ++t, ++g) {
                    const int s = mi * R + g % R;
                    if (!mbar_wait(bar(kTBarEmpty + s), ((g / R) & 1) ^ 1, abort, &g_status, kStatusTimeoutXEmpty)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(bar(kTBarFull + s), kATileBytes);
                    tma_load_4d(a_base + static_cast<uint32_t>(s) * kATileBytes, &p.tmap, 0, w0 + dw, h0 + dh, img,
                                bar(kTBarFull + s));
                    if (++dw > p.kw - 1 - p.kw / 2) {
                        dw = -(p.kw / 2);
                        ++dh;
                    }
                }
            }
            if (!ok) *abort = 1u;
            // every copy this thread started lands before the CTA exits
            for (int k = (g > R ? g - R : 0); k < g; ++k) drain_wait(bar(kTBarFull + mi * R + k % R), (k / R) & 1);
            if (mi == 0) drain_wait(bar(kTBarWFull), 0u);
        }
    } else if (warp == 1 || warp == 6) {
        // -------------------------------------------------- MMA issuers
        const int mi = warp == 1 ? 0 : 1;  // blocks mi, mi + 2, ... into accumulator half mi
        if (lane == 0) {
            ok = mbar_wait(bar(kTBarWFull), 0u, abort, &g_status, kStatusTimeoutWFull);
            const uint64_t w_desc0 = umma_desc_sw128(w_base);
            const uint64_t a_desc0 = umma_desc_sw128(a_base);
            const uint64_t tap_step = static_cast<uint64_t>(p.cout) * 8u;  // one tap block, 16-byte units
            bool issued = false;
            for (int bl = mi; ok && bl < n_mine; bl += 2) {
                const uint32_t d = tmem_base + (bl & 1) * d_cols;
                if (bl >= 2 && !mbar_wait(bar(kTBarDEmpty + (bl & 1)), ((bl >> 1) - 1) & 1, abort, &g_status,
                                          kStatusTimeoutOther)) {
                    ok = false;
                    break;
                }
                int g = (bl >> 1) * taps;  // the stream's load index of this block's first tap
                for (int t = 0; t < taps; ++t, ++g) {
                    const int s = mi * R + g % R;
                    if (!mbar_wait(bar(kTBarFull + s), (g / R) & 1, abort, &g_status, kStatusTimeoutAFull)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t a_desc = a_desc0 + static_cast<uint64_t>(s) * (kATileBytes >> 4);
                    const uint64_t b_desc = w_desc0 + static_cast<uint64_t>(t) * tap_step;
                    if (t == 0) issue_tap_ks<4, true>(d, a_desc, b_desc, p.idesc);
                    else issue_tap_ks<4, false>(d, a_desc, b_desc, p.idesc);
                    issued = true;
                    umma_commit(bar(kTBarEmpty + s));  // the tile may be reloaded
                    if (t == taps - 1) umma_commit(bar(kTBarDFull + (bl & 1)));
                }
            }
            if (!ok) *abort = 1u;
            if (issued) {
                umma_commit(bar(kTBarDrain + mi));
                drain_wait(bar(kTBarDrain + mi), 0u);
            }
        }
    } else {
        // ------------------------------------------------------- epilogue
        const int quad = warp & 3;
        const int r = quad * 32 + lane;  // TMEM lane = pixel (r / 16, r % 16) of the block
        const int n_chunks = p.cout >> 4;
        // the bias once into shared memory (zeros without one)
        float* bias_s = reinterpret_cast<float*>(base_ptr + p.off_bias);
        for (int i = threadIdx.x - 64; i < p.cout; i += 128) bias_s[i] = p.bias ? __ldg(p.bias + i) : 0.0f;
        asm volatile("bar.sync 1, 128;" ::: "memory");  // the 4 epilogue warps
        for (int bl = 0; ok && bl < n_mine; ++bl) {
            const uint32_t half = bl & 1;
            if (!mbar_wait_warp(bar(kTBarDFull + half), (bl >> 1) & 1, abort, &g_status, kStatusTimeoutAccFull)) {
                ok = false;
                break;
            }
            tc_fence_after();
            int img, h0, w0;
            tma_block_origin(p, static_cast<int>(blockIdx.x) + bl * static_cast<int>(gridDim.x), img, h0, w0);
            const int oh = h0 + r / kBoxW, ow = w0 + r % kBoxW;
            const bool valid = oh < p.h && ow < p.w;
            float* yrow = p.y + ((static_cast<long long>(img) * p.h + oh) * p.w + ow) * p.cout;
            const uint32_t t0 = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + half * d_cols;
            // up to 4 chunks (64 columns) per TMEM round trip
            for (int c0 = 0; c0 < n_chunks; c0 += 4) {
                uint32_t v[4][16];
                tmem_ld16(t0 + 16u * c0, v[0]);
                if (c0 + 1 < n_chunks) tmem_ld16(t0 + 16u * (c0 + 1), v[1]);
                if (c0 + 2 < n_chunks) tmem_ld16(t0 + 16u * (c0 + 2), v[2]);
                if (c0 + 3 < n_chunks) tmem_ld16(t0 + 16u * (c0 + 3), v[3]);
                tmem_wait_ld(v[0]);
                reg_barrier(v[1]);
                reg_barrier(v[2]);
                reg_barrier(v[3]);
                if (valid) {
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const int c = c0 + k;
                        if (c >= n_chunks) break;
                        const float4* b4 = reinterpret_cast<const float4*>(bias_s + 16 * c);
                        float4* dst = reinterpret_cast<float4*>(yrow + 16 * c);
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const float4 b = b4[q];
                            dst[q] = make_float4(__uint_as_float(v[k][4 * q]) + b.x, __uint_as_float(v[k][4 * q + 1]) + b.y,
                                                 __uint_as_float(v[k][4 * q + 2]) + b.z,
                                                 __uint_as_float(v[k][4 * q + 3]) + b.w);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kTBarDEmpty + half));
        }
        if (!ok) *abort = 1u;
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

// Weights [KH, KW, CIN, COUT] fp32 -> per tap a COUT x 128-byte K-major
// SW128 block of float16 / bfloat16 (K = CIN <= 64; unused K columns zero).
__global__ void conv_tc_pack_kernel(const float* __restrict__ w, int taps, int cin, int cout, int bf16,
                                    uint8_t* __restrict__ wpack) {
    const long long total = static_cast<long long>(taps) * cout * 64;
    for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int t = static_cast<int>(idx / (cout * 64));
        const int rem = static_cast<int>(idx - static_cast<long long>(t) * cout * 64);
        const int co = rem / 64, ci = rem - co * 64;
        const float v = ci < cin ? w[(static_cast<long long>(t) * cin + ci) * cout + co] : 0.0f;
        uint16_t bits;
        if (bf16) {
            const __nv_bfloat16 b = __float2bfloat16_rn(v);
            bits = *reinterpret_cast<const uint16_t*>(&b);
        } else {
            const __half hv = __float2half_rn(v);
            bits = *reinterpret_cast<const uint16_t*>(&hv);
        }
        *reinterpret_cast<uint16_t*>(wpack + static_cast<size_t>(t) * cout * 128 +
                                     sw128_offset(static_cast<uint32_t>(co), static_cast<uint32_t>(ci),
                                                  static_cast<uint32_t>(cout))) = bits;
    }
}

}  // namespace convtc
}  // namespace rdvb
