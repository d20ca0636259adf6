// Fused small-MLP forward on the 5th-generation tensor cores (tcgen05).
//
// Replaces the reference's cooperative-matrix Map chain
// (rdv/shaders/maps/linear_fast.h:39-109 composed by
// rdv/shaders/maps/composite.h:8-12 and driven one row per thread by
// rdv/shaders/maps/map_evaluator.h:1-5). Same arithmetic contract: inputs and
// weights staged as float16 (or bfloat16), products accumulated in fp32,
// fp32 bias added after, ReLU in fp32 (applied before the next layer's
// float16 staging), fp32 output.
//
// Design (one persistent CTA per SM, 320 threads):
//   warps 0-7  epilogue: stage the input tile (fp32 -> f16, SW128 layout),
//              then per layer read the TMEM accumulator (tcgen05.ld), add
//              bias, ReLU + convert to f16 and write the next layer's A tile
//              back into shared memory; the last layer writes fp32 rows.
//   warp 8     producer: 1-D bulk (TMA) copies of input tiles and of the
//              pre-swizzled weight blocks (resident, or streamed per layer
//              through a ring when they do not fit).
//   warp 9     MMA issuer: allocates TMEM, one thread issues
//              tcgen05.mma (M=128, N=layer width, K=16 steps) per layer and
//              commits completion to mbarriers.
// Two 128-row tiles ("slots") are in flight so one slot's epilogue overlaps
// the other slot's MMAs. No activation ever leaves the SM between layers.
#pragma once
#include "ptx.cuh"

namespace rdvb {
namespace mlp_tc {

constexpr int kMaxLayers = 16;
constexpr int kTileM = 128;
constexpr int kSlots = 2;
constexpr int kEpiWarps = 8;
constexpr int kEpiThreads = kEpiWarps * 32;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kThreads = 320;
constexpr uint32_t kAtomBytes = kTileM * 128;      // one 64-wide K atom of a 128-row tile
constexpr int kMaxKAtoms = 2;                       // layer width <= 128
constexpr uint32_t kABytes = kAtomBytes * kMaxKAtoms;
constexpr int kMaxWStages = 4;
constexpr uint32_t kMaxWidth = 128;

struct Layer {
    uint32_t k_pad;   // input width rounded up to 16
    uint32_t n_pad;   // output width rounded up to 16
    uint32_t w_off;   // byte offset of the packed block in the weight pack
    uint32_t w_bytes; // n_pad * katoms * 128
    uint32_t b_off;   // float offset in the bias pack
    uint32_t idesc;
    uint32_t relu;
};

struct Params {
    const void* x;
    float* y;
    const uint8_t* wpack;
    const float* bpack;
    long long n_rows;
    int n_tiles;
    int in_dim;
    int out_dim;
    int x_dtype;  // 0 f32, 1 f16, 2 bf16
    int relu_in;
    int bf16;     // operand type: 0 f16, 1 bf16
    int n_layers;
    int resident;
    int w_stages;
    uint32_t w_slot_bytes;
    uint32_t w_total_bytes;
    uint32_t bias_floats;
    uint32_t x_stage_bytes;
    uint32_t off_w, off_x, off_bias, off_bar;
    uint32_t tmem_cols;
    int y_vec4;
    Layer layer[kMaxLayers];
};

// Barrier slots in the barrier block.
enum : int {
    kBarXFull = 0,
    kBarXEmpty = kBarXFull + kSlots,
    kBarAFull = kBarXEmpty + kSlots,
    kBarAccFull = kBarAFull + kSlots,
    kBarWFull = kBarAccFull + kSlots,
    kBarWEmpty = kBarWFull + kMaxWStages,
    kBarDrain = kBarWEmpty + kMaxWStages,
    kNumBars = kBarDrain + 1,
};
constexpr uint32_t kBarBlockBytes = kNumBars * 8 + 16;  // + tmem base + abort word

__device__ __forceinline__ float load_x_elem(const uint8_t* xs, int dtype, uint32_t idx) {
    if (dtype == 0) return reinterpret_cast<const float*>(xs)[idx];
    if (dtype == 1) return __half2float(reinterpret_cast<const __half*>(xs)[idx]);
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(xs)[idx]);
}

__device__ __forceinline__ uint32_t pack2(float a, float b, int bf16, int relu) {
    if (bf16) return relu ? pack_bf16x2_relu(a, b) : pack_bf16x2(a, b);
    return relu ? pack_f16x2_relu(a, b) : pack_f16x2(a, b);
}

// Drain wait used on the abort path: ignores the abort flag, keeps its own
// time limit.
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity, uint32_t* status) {
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_timer_ns() - t0 > RDVB_WAIT_LIMIT_NS) {
            atomicOr(status, kStatusTimeoutDrain);
            return;
        }
    }
}

__global__ void __launch_bounds__(kThreads, 1) mlp_tc_kernel(const __grid_constant__ Params p) {
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment for the SW128 atoms.
    const uint32_t raw_addr = smem_addr(smem_raw);
    const uint32_t base = (raw_addr + 1023u) & ~1023u;
    uint8_t* const base_ptr = smem_raw + (base - raw_addr);

    const uint32_t a_base = base;                      // kSlots * kABytes
    const uint32_t w_base = base + p.off_w;
    const uint32_t x_base = base + p.off_x;
    const float* bias_s = reinterpret_cast<const float*>(base_ptr + p.off_bias);
    float* bias_w = reinterpret_cast<float*>(base_ptr + p.off_bias);
    const uint32_t bar_base = base + p.off_bar;
    auto bar = [&](int i) -> uint32_t { return bar_base + 8u * static_cast<uint32_t>(i); };
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base_ptr + p.off_bar + kNumBars * 8);
    volatile uint32_t* abort = reinterpret_cast<volatile uint32_t*>(base_ptr + p.off_bar + kNumBars * 8 + 4);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kSlots; ++s) {
            mbar_init(bar(kBarXFull + s), 1);
            mbar_init(bar(kBarXEmpty + s), kEpiWarps);
            mbar_init(bar(kBarAFull + s), kEpiWarps);
            mbar_init(bar(kBarAccFull + s), 1);
        }
        for (int q = 0; q < kMaxWStages; ++q) {
            mbar_init(bar(kBarWFull + q), 1);
            mbar_init(bar(kBarWEmpty + q), 1);
        }
        mbar_init(bar(kBarDrain), 1);
        *abort = 0u;
        fence_mbarrier_init();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(smem_addr(tmem_slot), p.tmem_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int n_layers = p.n_layers;
    const int G = gridDim.x;

    if (warp == kProducerWarp) {
        if (lane == 0) {
            uint32_t xu[kSlots] = {0, 0};
            uint32_t wcount = 0;
            const int esize = p.x_dtype == 0 ? 4 : 2;
            bool ok = true;
            if (p.resident) {
                mbar_arrive_expect_tx(bar(kBarWFull), p.w_total_bytes);
                for (int l = 0; l < n_layers; ++l)
                    bulk_g2s(w_base + p.layer[l].w_off, p.wpack + p.layer[l].w_off, p.layer[l].w_bytes,
                             bar(kBarWFull));
            }
            for (int r = 0; ok; ++r) {
                const int tile0 = (r * G + blockIdx.x) * kSlots;
                if (tile0 >= p.n_tiles) break;
                for (int s = 0; s < kSlots && ok; ++s) {
                    const int t = tile0 + s;
                    if (t >= p.n_tiles) break;
                    if (!mbar_wait(bar(kBarXEmpty + s), (xu[s] & 1u) ^ 1u, abort, &g_status, kStatusTimeoutXEmpty)) {
                        ok = false;
                        break;
                    }
                    long long row0 = static_cast<long long>(t) * kTileM;
                    long long rows = p.n_rows - row0;
                    if (rows > kTileM) rows = kTileM;
                    const uint32_t bytes = static_cast<uint32_t>(rows) * p.in_dim * esize;
                    mbar_arrive_expect_tx(bar(kBarXFull + s), bytes);
                    bulk_g2s(x_base + s * p.x_stage_bytes,
                             static_cast<const uint8_t*>(p.x) + row0 * p.in_dim * esize, bytes, bar(kBarXFull + s));
                    ++xu[s];
                }
                if (!p.resident) {
                    for (int l = 0; l < n_layers && ok; ++l) {
                        const uint32_t q = wcount % p.w_stages;
                        const uint32_t ph = (wcount / p.w_stages) & 1u;
                        if (!mbar_wait(bar(kBarWEmpty + q), ph ^ 1u, abort, &g_status, kStatusTimeoutWEmpty)) {
                            ok = false;
                            break;
                        }
                        mbar_arrive_expect_tx(bar(kBarWFull + q), p.layer[l].w_bytes);
                        bulk_g2s(w_base + q * p.w_slot_bytes, p.wpack + p.layer[l].w_off, p.layer[l].w_bytes,
                                 bar(kBarWFull + q));
                        ++wcount;
                    }
                }
            }
            if (!ok) {
                // Let every copy this thread started land before the CTA exits.
                for (int s = 0; s < kSlots; ++s)
                    if (xu[s]) drain_wait(bar(kBarXFull + s), (xu[s] - 1u) & 1u, &g_status);
                if (p.resident) {
                    drain_wait(bar(kBarWFull), 0u, &g_status);
                } else {
                    for (uint32_t c = (wcount > (uint32_t)p.w_stages ? wcount - p.w_stages : 0u); c < wcount; ++c)
                        drain_wait(bar(kBarWFull + c % p.w_stages), (c / p.w_stages) & 1u, &g_status);
                }
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            uint32_t au[kSlots] = {0, 0};
            uint32_t wcount = 0;
            bool ok = true;
            bool issued = false;
            if (p.resident) ok = mbar_wait(bar(kBarWFull), 0u, abort, &g_status, kStatusTimeoutWFull);
            for (int r = 0; ok; ++r) {
                const int tile0 = (r * G + blockIdx.x) * kSlots;
                if (tile0 >= p.n_tiles) break;
                const int nslots = min(kSlots, p.n_tiles - tile0);
                for (int l = 0; l < n_layers && ok; ++l) {
                    const Layer& L = p.layer[l];
                    uint32_t wb;
                    uint32_t q = 0;
                    if (p.resident) {
                        wb = w_base + L.w_off;
                    } else {
                        q = wcount % p.w_stages;
                        if (!mbar_wait(bar(kBarWFull + q), (wcount / p.w_stages) & 1u, abort, &g_status,
                                       kStatusTimeoutWFull)) {
                            ok = false;
                            break;
                        }
                        wb = w_base + q * p.w_slot_bytes;
                    }
                    for (int s = 0; s < nslots; ++s) {
                        if (!mbar_wait(bar(kBarAFull + s), au[s] & 1u, abort, &g_status, kStatusTimeoutAFull)) {
                            ok = false;
                            break;
                        }
                        ++au[s];
                        tc_fence_after();
                        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(s) * kMaxWidth;
                        const uint32_t a_tile = a_base + static_cast<uint32_t>(s) * kABytes;
                        const uint32_t ksteps = L.k_pad >> 4;
                        for (uint32_t j = 0; j < ksteps; ++j) {
                            const uint32_t koff = (j >> 2) * kAtomBytes + (j & 3u) * 32u;
                            const uint32_t kboff = (j >> 2) * (L.n_pad * 128u) + (j & 3u) * 32u;
                            umma_f16(d_tmem, umma_desc_sw128(a_tile + koff), umma_desc_sw128(wb + kboff), L.idesc,
                                     j > 0 ? 1u : 0u);
                        }
                        umma_commit(bar(kBarAccFull + s));
                        issued = true;
                    }
                    if (!ok) break;
                    if (!p.resident) {
                        umma_commit(bar(kBarWEmpty + q));
                        ++wcount;
                    }
                }
            }
            if (!ok && issued) {
                umma_commit(bar(kBarDrain));
                drain_wait(bar(kBarDrain), 0u, &g_status);
            }
        }
    } else {
        // ------------------------------------------------------ epilogue
        const int et = threadIdx.x;  // 0..255
        for (uint32_t i = et; i < p.bias_floats; i += kEpiThreads) bias_w[i] = p.bpack[i];
        named_bar_sync(1, kEpiThreads);

        const int quad = warp & 3;
        const int grp = warp >> 2;
        const int row = quad * 32 + lane;
        const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
        uint32_t xf[kSlots] = {0, 0};
        uint32_t ac[kSlots] = {0, 0};
        const int esize = p.x_dtype == 0 ? 4 : 2;
        const uint32_t kch0 = p.layer[0].k_pad >> 3;
        bool ok = true;

        for (int r = 0; ok; ++r) {
            const int tile0 = (r * G + blockIdx.x) * kSlots;
            if (tile0 >= p.n_tiles) break;
            const int nslots = min(kSlots, p.n_tiles - tile0);

            // Stage the input tiles: [rows, in_dim] (x dtype) -> A[s] f16/bf16.
            for (int s = 0; s < nslots; ++s) {
                if (!mbar_wait(bar(kBarXFull + s), xf[s] & 1u, abort, &g_status, kStatusTimeoutXFull)) {
                    ok = false;
                    break;
                }
                ++xf[s];
                const long long row0 = static_cast<long long>(tile0 + s) * kTileM;
                long long rv = p.n_rows - row0;
                const int rows_valid = rv > kTileM ? kTileM : static_cast<int>(rv);
                const uint8_t* xs = base_ptr + p.off_x + s * p.x_stage_bytes;
                const uint32_t a_tile = a_base + static_cast<uint32_t>(s) * kABytes;
                for (uint32_t idx = et; idx < kTileM * kch0; idx += kEpiThreads) {
                    const uint32_t ri = idx / kch0;
                    const uint32_t c = idx - ri * kch0;
                    float v[8];
                    if (p.x_dtype == 0 && (p.in_dim & 7) == 0 && ri < (uint32_t)rows_valid &&
                        c * 8 + 8 <= (uint32_t)p.in_dim) {
                        const float4* src = reinterpret_cast<const float4*>(xs + (ri * p.in_dim + c * 8) * 4);
                        const float4 u0 = src[0], u1 = src[1];
                        v[0] = u0.x; v[1] = u0.y; v[2] = u0.z; v[3] = u0.w;
                        v[4] = u1.x; v[5] = u1.y; v[6] = u1.z; v[7] = u1.w;
                    } else {
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            const uint32_t k = c * 8 + e;
                            v[e] = (ri < (uint32_t)rows_valid && k < (uint32_t)p.in_dim)
                                       ? load_x_elem(xs, p.x_dtype, ri * p.in_dim + k)
                                       : 0.0f;
                        }
                    }
                    const uint32_t w0 = pack2(v[0], v[1], p.bf16, p.relu_in);
                    const uint32_t w1 = pack2(v[2], v[3], p.bf16, p.relu_in);
                    const uint32_t w2 = pack2(v[4], v[5], p.bf16, p.relu_in);
                    const uint32_t w3 = pack2(v[6], v[7], p.bf16, p.relu_in);
                    st_shared_v4(a_tile + sw128_offset(ri, c * 8, kTileM), w0, w1, w2, w3);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(bar(kBarXEmpty + s));
                    mbar_arrive(bar(kBarAFull + s));
                }
                (void)esize;
            }
            if (!ok) break;

            for (int l = 0; l < n_layers && ok; ++l) {
                const Layer& L = p.layer[l];
                const bool last = (l == n_layers - 1);
                const uint32_t nch = L.n_pad >> 4;
                for (int s = 0; s < nslots; ++s) {
                    if (!mbar_wait(bar(kBarAccFull + s), ac[s] & 1u, abort, &g_status, kStatusTimeoutAccFull)) {
                        ok = false;
                        break;
                    }
                    ++ac[s];
                    tc_fence_after();
                    const uint32_t t_col = tmem_base + lane_off + static_cast<uint32_t>(s) * kMaxWidth;
                    uint32_t v[4][16];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint32_t c = grp + 2 * j;
                        if (c < nch) tmem_ld16(t_col + c * 16, v[j]);
                    }
                    tmem_wait_ld();
                    if (!last) {
                        const uint32_t a_tile = a_base + static_cast<uint32_t>(s) * kABytes;
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const uint32_t c = grp + 2 * j;
                            if (c < nch) {
                                const float* bb = bias_s + L.b_off + c * 16;
                                uint32_t pk[8];
#pragma unroll
                                for (int i = 0; i < 16; i += 2) {
                                    float a0 = __uint_as_float(v[j][i]);
                                    float a1 = __uint_as_float(v[j][i + 1]);
                                    add_f32x2(a0, a1, bb[i], bb[i + 1]);
                                    pk[i >> 1] = pack2(a0, a1, p.bf16, L.relu);
                                }
                                // columns c*16 .. c*16+15 of this layer = K chunks 2c, 2c+1 of the next
                                st_shared_v4(a_tile + sw128_offset(row, c * 16, kTileM), pk[0], pk[1], pk[2], pk[3]);
                                st_shared_v4(a_tile + sw128_offset(row, c * 16 + 8, kTileM), pk[4], pk[5], pk[6],
                                             pk[7]);
                            }
                        }
                        fence_proxy_async_smem();
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(bar(kBarAFull + s));
                    } else {
                        const long long grow = static_cast<long long>(tile0 + s) * kTileM + row;
                        if (grow < p.n_rows) {
                            float* yrow = p.y + grow * p.out_dim;
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                const uint32_t c = grp + 2 * j;
                                if (c < nch) {
                                    const float* bb = bias_s + L.b_off + c * 16;
                                    float o[16];
#pragma unroll
                                    for (int i = 0; i < 16; i += 2) {
                                        float a0 = __uint_as_float(v[j][i]);
                                        float a1 = __uint_as_float(v[j][i + 1]);
                                        add_f32x2(a0, a1, bb[i], bb[i + 1]);
                                        if (L.relu) {
                                            a0 = fmaxf(a0, 0.0f);
                                            a1 = fmaxf(a1, 0.0f);
                                        }
                                        o[i] = a0;
                                        o[i + 1] = a1;
                                    }
                                    const int col0 = c * 16;
                                    if (p.y_vec4 && col0 + 16 <= p.out_dim) {
                                        float4* dst = reinterpret_cast<float4*>(yrow + col0);
                                        dst[0] = make_float4(o[0], o[1], o[2], o[3]);
                                        dst[1] = make_float4(o[4], o[5], o[6], o[7]);
                                        dst[2] = make_float4(o[8], o[9], o[10], o[11]);
                                        dst[3] = make_float4(o[12], o[13], o[14], o[15]);
                                    } else {
#pragma unroll
                                        for (int i = 0; i < 16; ++i)
                                            if (col0 + i < p.out_dim) yrow[col0 + i] = o[i];
                                    }
                                }
                            }
                        }
                        tc_fence_before();
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem_base, p.tmem_cols);
    }
}

// Packs fp32 [N, K] row-major weights (PyTorch nn.Linear layout) of every
// layer into the K-major SW128 image the kernel copies straight into shared
// memory (zero padding to n_pad x katoms*64), and the biases into one fp32
// array padded to n_pad per layer.
struct PackLayer {
    const float* W;
    const float* b;
    uint32_t K, N, n_pad, katoms, w_off, b_off;
};
struct PackParams {
    PackLayer layer[kMaxLayers];
    int n_layers;
    int bf16;
    uint8_t* wpack;
    float* bpack;
    uint32_t total_chunks;  // sum over layers of n_pad * katoms * 8
};

__global__ void mlp_pack_kernel(const __grid_constant__ PackParams p) {
    for (uint32_t g = blockIdx.x * blockDim.x + threadIdx.x; g < p.total_chunks; g += gridDim.x * blockDim.x) {
        uint32_t rem = g;
        int l = 0;
        for (; l < p.n_layers; ++l) {
            const uint32_t nc = p.layer[l].n_pad * p.layer[l].katoms * 8;
            if (rem < nc) break;
            rem -= nc;
        }
        const PackLayer& L = p.layer[l];
        const uint32_t chunks_per_row = L.katoms * 8;
        const uint32_t n = rem / chunks_per_row;
        const uint32_t kc = rem - n * chunks_per_row;
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
            const uint32_t k0 = kc * 8 + e;
            const float v0 = (n < L.N && k0 < L.K) ? L.W[static_cast<size_t>(n) * L.K + k0] : 0.0f;
            const float v1 = (n < L.N && k0 + 1 < L.K) ? L.W[static_cast<size_t>(n) * L.K + k0 + 1] : 0.0f;
            w[e >> 1] = p.bf16 ? pack_bf16x2(v0, v1) : pack_f16x2(v0, v1);
        }
        uint4* dst = reinterpret_cast<uint4*>(p.wpack + L.w_off + sw128_offset(n, kc * 8, L.n_pad));
        *dst = make_uint4(w[0], w[1], w[2], w[3]);
        if (kc == 0) p.bpack[L.b_off + n] = (n < L.N) ? L.b[n] : 0.0f;
    }
}

}  // namespace mlp_tc
}  // namespace rdvb
