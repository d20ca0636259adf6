// Fused small-MLP forward on the 5th-generation tensor cores (tcgen05).
//
// Replaces the reference's cooperative-matrix Map chain
// (rdv/shaders/maps/linear_fast.h:39-109 composed by
// rdv/shaders/maps/composite.h:8-12 and driven one row per thread by
// rdv/shaders/maps/map_evaluator.h:1-5). Arithmetic contract: inputs and
// weights staged as float16 (or bfloat16), products accumulated in fp32, the
// fp32 bias added to the fp32 accumulator (the reference's order: products
// first, then + b), ReLU applied before the next layer's float16 staging,
// fp32 output. The epilogue does the bias add (TMEM load -> + b -> ReLU +
// convert -> TMEM store): the single MMA-issuing thread is the kernel's
// serial resource, so it issues only the K steps.
//
// Design (one persistent CTA per SM, 20 warps):
//   warps 0-15 epilogue. Warp w owns TMEM lane quadrant (w % 4) -- rows
//              32*(w%4) .. +31 of every tile. Warp group g = w / 4 owns slot
//              g % SLOTS and, of that slot's 16-column chunks, every
//              (4/SLOTS)-th one starting at g / SLOTS: the slots' epilogues
//              run concurrently, each warp waiting only on its own slot. Per
//              layer it reads its accumulator chunks (tcgen05.ld), applies
//              ReLU while converting to f16/bf16 (cvt.rn.relu) and writes them
//              back into TMEM (tcgen05.st) as the next layer's A operand, so
//              hidden activations never touch shared memory; the last layer
//              writes fp32 rows to global memory (or, in ray mode, composites
//              the ray's samples into one RGBA pixel).
//   warp 16    producer: 1-D bulk (TMA) copies of input tiles and of the
//              pre-swizzled weight blocks (resident, or streamed per layer
//              through a ring), issued from one event loop.
//   warps 17, 19 (+ 20, 21)  MMA issuers (with 4 slots and resident
//              weights one per slot, else even / odd slots; warp 17
//              allocates TMEM): one thread each issues tcgen05.mma
//              (M=128, N=layer width, K=16 steps) per layer -- A from shared
//              memory for the first layer, from TMEM after -- and commits
//              completion to mbarriers.
//   warp 18    input staging: converts each input tile (x dtype ->
//              f16/bf16, zero-padded to 16) into the first layer's A tile in
//              shared memory (K-major, 128B swizzle).
// SLOTS independent 128-row tiles are in flight per CTA (one TMEM
// accumulator and one TMEM activation tile each), so the epilogue of one
// tile overlaps the MMAs of the others. Shared memory only feeds the weights
// and the first layer's A, well inside its bandwidth.
#pragma once
#include "ptx.cuh"

namespace rdvb {
namespace mlp_tc {

constexpr int kMaxLayers = 16;
constexpr int kTileM = 128;
constexpr int kMaxSlots = 4;
constexpr int kEpiWarps = 16;
constexpr int kProducerWarp = 16;
constexpr int kMmaWarp = 17;        // issues the MMAs of the even slots; allocates TMEM
constexpr int kMmaWarp2 = 19;       // issues the MMAs of the odd slots
constexpr int kMaxIssuers = 4;      // with 4: warps 17, 19, 20, 21, one slot each
// Issuer number of an MMA-issuing warp (-1 for other warps).
__host__ __device__ constexpr int issuer_index(int warp) {
    return warp == kMmaWarp ? 0 : (warp == kMmaWarp2 ? 1 : (warp >= 20 ? warp - 18 : -1));
}
// CTA size for ISSUERS MMA-issuing warps: 16 epilogue + producer + MMA +
// staging (+ the other issuers). Streamed-weight chains run 19 warps, which
// leaves their register-heavy epilogue the larger budget.
__host__ __device__ constexpr int cta_threads(int issuers) { return (18 + issuers) * 32; }
constexpr int kStageWarp = 18;
constexpr uint32_t kAtomBytes = kTileM * 128;      // one 64-wide K atom of a 128-row tile
constexpr int kMaxWStages = 4;
constexpr uint32_t kMaxWidth = 128;
constexpr uint32_t kTmemCols = 512;

struct Layer {
    uint32_t k_pad;    // input width rounded up to 16
    uint32_t n_pad;    // output width rounded up to 16
    uint32_t w_off;    // byte offset of the layer block in the weight pack
    uint32_t w_bytes;  // layer block: SW128 weights, 1 KB multiple
    uint32_t b_idx;    // first element of the layer's fp32 bias in the bias block
    uint32_t idesc;
    uint32_t relu;
};

// Transmittance march (RaymarchingTransmittance): a ray's entry point and
// object-space direction, its step count (the reference's d > 0 loop, at
// most 4096) and the index of its first 128-step chunk in the chunk list.
struct MarchRay {
    float x[3];
    float w[3];
    int n_steps;
    int base;
};

// Kernel modes (template argument RAY): rows of x, volume render, transmittance march.
constexpr int kModeRows = 0;
constexpr int kModeRender = 1;
constexpr int kModeMarch = 2;

// Volume ray-march modes. Render (march = 0): one 128-row tile is one ray's
// 128 samples, composited into an RGBA pixel. Transmittance (march = 1):
// one tile is 128 consecutive steps of one ray; the tile's result is the sum
// of its steps' extinction * scale * step and the largest prefix of that sum.
struct RayParams {
    const int* hit_list;   // render: pixel index (within the band) of every ray that hits the box;
                           // march: ray index of every chunk
    const int* n_hits;     // number of entries of hit_list (device)
    int march;
    const MarchRay* rec;   // march: per-ray records
    float2* chunk_out;     // march: (sum, largest prefix) per chunk
    float step, scale;     // march: step size, density scale
    float* rgba;           // [band rows * width, 4]
    float org[3];          // camera origin
    float xa[3], ya[3], za[3];  // camera basis (cameras.h: xaxis, yaxis, zaxis)
    float aspect, sz;      // sx = p.x * aspect; sz = 1 / tan(fov / 2)
    int width, height, row_begin;
};

struct Params {
    const void* x;
    float* y;
    const uint8_t* wpack;
    long long n_rows;
    int n_tiles;
    int in_dim;
    int out_dim;
    int x_dtype;  // 0 f32, 1 f16, 2 bf16
    int relu_in;
    int n_layers;
    int resident;
    int w_stages;
    uint32_t w_slot_bytes;
    uint32_t w_total_bytes;
    uint32_t x_stage_bytes;
    uint32_t off_w, off_x, off_bias, off_bar;
    uint32_t bias_bytes;   // fp32 biases of every layer (n_pad each), 16-byte multiple
    uint32_t bias_gofs;    // their byte offset in the weight pack
    uint32_t a0_bytes;     // shared-memory A tile of layer 0, per slot
    uint32_t acc_stride;   // TMEM columns of one slot's fp32 accumulator
    uint32_t act_base;     // first TMEM column of the activation regions
    uint32_t act_stride;   // TMEM columns of one slot's 16-bit activation tile
    int y_vec4;
    uint32_t off_ray;      // ray mode: compositing scratch (4 column groups x 4 quadrants x 4 floats)
    Layer layer[kMaxLayers];
    RayParams ray;
};

// Barrier slots in the barrier block.
enum : int {
    kBarXFull = 0,                             // input tile landed in staging (TMA tx)
    kBarXEmpty = kBarXFull + kMaxSlots,        // staging buffer consumed
    kBarA0Full = kBarXEmpty + kMaxSlots,       // layer-0 A tile written
    kBarA0Empty = kBarA0Full + kMaxSlots,      // layer-0 MMAs done reading it
    kBarAFull = kBarA0Empty + kMaxSlots,       // epilogue done with a layer of the slot
    kBarAccFull = kBarAFull + kMaxSlots,       // accumulator ready
    kBarWFull = kBarAccFull + kMaxSlots,
    kBarWEmpty = kBarWFull + kMaxWStages,
    kBarDrain = kBarWEmpty + kMaxWStages,      // + issuer
    kBarComp = kBarDrain + kMaxIssuers,        // ray mode: per slot, 4 quadrant partials written
    kBarBias = kBarComp + 4,                   // fp32 biases landed (TMA tx)
    kNumBars = kBarBias + 1,
};
constexpr uint32_t kRayScratchBytes = 4 * 4 * 4 * 4;
constexpr uint32_t kBarBlockBytes = kNumBars * 8 + 16;  // + tmem base + abort word

__device__ __forceinline__ float load_x_elem(const uint8_t* xs, int dtype, uint32_t idx) {
    if (dtype == 0) return reinterpret_cast<const float*>(xs)[idx];
    if (dtype == 1) return __half2float(reinterpret_cast<const __half*>(xs)[idx]);
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(xs)[idx]);
}

template <int BF16, bool RELU>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
    if (BF16) return RELU ? pack_bf16x2_relu(a, b) : pack_bf16x2(a, b);
    return RELU ? pack_f16x2_relu(a, b) : pack_f16x2(a, b);
}

template <int BF16>
__device__ __forceinline__ uint32_t pack2_rt(float a, float b, int relu) {
    return relu ? pack2<BF16, true>(a, b) : pack2<BF16, false>(a, b);
}

// Tile index of (round r, slot s) for this CTA, or -1 past the end.
template <int SLOTS>
__device__ __forceinline__ int tile_of(int r, int s, int n_tiles) {
    const int t = (r * static_cast<int>(gridDim.x) + static_cast<int>(blockIdx.x)) * SLOTS + s;
    return t < n_tiles ? t : -1;
}

// Exactly KS K-step MMAs of one layer for one slot: A from the slot's
// shared-memory tile (SS) or from its TMEM activations (TS). The MMAs are
// straight-line code selected by a switch on the layer's K steps: in a fixed
// 8-step unrolled loop, a step skipped by its runtime condition measured
// about as expensive for the issuing thread as an issued MMA (~140 cycles),
// up to ~500 cycles per layer of a narrow chain.
template <int KS>
__device__ __forceinline__ void issue_ks(bool ts, uint32_t d, uint64_t a0_desc, uint32_t a_tm,
                                         const uint64_t (&b)[8], uint32_t idesc) {
    if (ts) {
#pragma unroll
        for (int j = 0; j < KS; ++j) umma_f16_ts(d, a_tm + j * 8u, b[j], idesc, j > 0 ? 1u : 0u);
    } else {
#pragma unroll
        for (int j = 0; j < KS; ++j)
            umma_f16(d, a0_desc + (j >> 2) * (kAtomBytes >> 4) + (j & 3) * 2, b[j], idesc, j > 0 ? 1u : 0u);
    }
}

__device__ __forceinline__ void issue_layer(uint32_t ksteps, bool ts, uint32_t d, uint64_t a0_desc, uint32_t a_tm,
                                            const uint64_t (&b)[8], uint32_t idesc) {
    switch (ksteps) {
        case 1: issue_ks<1>(ts, d, a0_desc, a_tm, b, idesc); break;
        case 2: issue_ks<2>(ts, d, a0_desc, a_tm, b, idesc); break;
        case 3: issue_ks<3>(ts, d, a0_desc, a_tm, b, idesc); break;
        case 4: issue_ks<4>(ts, d, a0_desc, a_tm, b, idesc); break;
        case 5: issue_ks<5>(ts, d, a0_desc, a_tm, b, idesc); break;
        case 6: issue_ks<6>(ts, d, a0_desc, a_tm, b, idesc); break;
        case 7: issue_ks<7>(ts, d, a0_desc, a_tm, b, idesc); break;
        default: issue_ks<8>(ts, d, a0_desc, a_tm, b, idesc); break;
    }
}

// + fp32 bias of the chunk's 16 columns (shared memory, broadcast to all
// lanes), in place on the raw accumulator words.
__device__ __forceinline__ void add_bias16(uint32_t (&v)[16], const float* b) {
    const float4* b4 = reinterpret_cast<const float4*>(b);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float4 bb = b4[q];
        float x0 = __uint_as_float(v[4 * q]), x1 = __uint_as_float(v[4 * q + 1]);
        float x2 = __uint_as_float(v[4 * q + 2]), x3 = __uint_as_float(v[4 * q + 3]);
        add_f32x2(x0, x1, bb.x, bb.y);
        add_f32x2(x2, x3, bb.z, bb.w);
        v[4 * q] = __float_as_uint(x0);
        v[4 * q + 1] = __float_as_uint(x1);
        v[4 * q + 2] = __float_as_uint(x2);
        v[4 * q + 3] = __float_as_uint(x3);
    }
}

// One warp's share of a 16-column accumulator chunk -> packed 16-bit
// activations (8 TMEM columns).
template <int BF16, bool RELU>
__device__ __forceinline__ void convert_chunk(const uint32_t (&v)[16], uint32_t (&pk)[8]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) pk[i] = pack2<BF16, RELU>(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
}

// Pinhole ray of pixel `pix` of the band (cameras.h:1-20: pixel centre,
// p in [-1, 1], w = normalize(xaxis * p.x * aspect + yaxis * p.y + zaxis *
// sz)) and its [-1, 1]^3 slab interval (math_library.h:48-57), entry clamped
// to 0 (raymarching_transmittance.h:11-19). Returns false on a miss.
__device__ __forceinline__ bool ray_setup(const RayParams& rp, int pix, float (&o)[3], float (&w)[3], float& t0,
                                          float& t1) {
    const int py = rp.row_begin + pix / rp.width, px = pix - (pix / rp.width) * rp.width;
    const float fx = (static_cast<float>(px) + 0.5f) / static_cast<float>(rp.width) * 2.0f - 1.0f;
    const float fy = (static_cast<float>(py) + 0.5f) / static_cast<float>(rp.height) * 2.0f - 1.0f;
    const float sx = fx * rp.aspect, sy = fy;
    float d[3];
#pragma unroll
    for (int c = 0; c < 3; ++c) d[c] = rp.xa[c] * sx + rp.ya[c] * sy + rp.za[c] * rp.sz;
    const float inv_len = 1.0f / sqrtf(d[0] * d[0] + d[1] * d[1] + d[2] * d[2]);
    float tmin = -INFINITY, tmax = INFINITY;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        o[c] = rp.org[c];
        w[c] = d[c] * inv_len;
        const float inv = 1.0f / w[c];
        const float xc = -o[c] * inv, sc = fabsf(inv);
        tmin = fmaxf(tmin, xc - sc);
        tmax = fminf(tmax, xc + sc);
    }
    t0 = fmaxf(tmin, 0.0f);
    t1 = tmax;
    return !(tmax <= 0.0f || tmin > tmax);
}

__device__ __forceinline__ float softplus_f(float v) { return fmaxf(v, 0.0f) + log1pf(expf(-fabsf(v))); }
__device__ __forceinline__ float sigmoid_f(float v) { return 1.0f / (1.0f + expf(-v)); }

template <int SLOTS, int BF16, int RAY, int ISSUERS>
__global__ void __launch_bounds__(cta_threads(ISSUERS), 1) mlp_tc_kernel(const __grid_constant__ Params p) {
    static_assert(SLOTS == 2 || SLOTS == 4, "the epilogue splits 4 warp groups evenly over the slots");
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment for the SW128 atoms.
    const uint32_t raw_addr = smem_addr(smem_raw);
    const uint32_t base = (raw_addr + 1023u) & ~1023u;
    uint8_t* const base_ptr = smem_raw + (base - raw_addr);

    const uint32_t a_base = base;  // SLOTS * a0_bytes (layer-0 A tiles)
    const uint32_t w_base = base + p.off_w;
    const uint32_t x_base = base + p.off_x;
    const uint32_t bar_base = base + p.off_bar;
    auto bar = [&](int i) -> uint32_t { return bar_base + 8u * static_cast<uint32_t>(i); };
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base_ptr + p.off_bar + kNumBars * 8);
    volatile uint32_t* abort = reinterpret_cast<volatile uint32_t*>(base_ptr + p.off_bar + kNumBars * 8 + 4);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kMaxSlots; ++s) {
            mbar_init(bar(kBarXFull + s), 1);
            mbar_init(bar(kBarXEmpty + s), 1);
            mbar_init(bar(kBarA0Full + s), 1);
            mbar_init(bar(kBarA0Empty + s), 1);
            mbar_init(bar(kBarAFull + s), kEpiWarps / SLOTS);  // the warps owning the slot
            mbar_init(bar(kBarAccFull + s), 1);
        }
        for (int q = 0; q < kMaxWStages; ++q) {
            mbar_init(bar(kBarWFull + q), 1);
            mbar_init(bar(kBarWEmpty + q), 1);  // streamed weights: a single issuer
        }
        for (int i = 0; i < kMaxIssuers; ++i) mbar_init(bar(kBarDrain + i), 1);
        for (int g = 0; g < 4; ++g) mbar_init(bar(kBarComp + g), 4);
        mbar_init(bar(kBarBias), 1);
        *abort = 0u;
        fence_mbarrier_init();
    }
    // Layer-0 A tiles start zeroed: chunks past the input width stay zero.
    for (uint32_t i = threadIdx.x; i < SLOTS * p.a0_bytes / 16; i += cta_threads(ISSUERS)) st_shared_v4(a_base + i * 16, 0u, 0u, 0u, 0u);
    fence_proxy_async_smem();
    if (warp == kMmaWarp) {
        tmem_alloc(smem_addr(tmem_slot), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int n_layers = p.n_layers;
    const int esize = p.x_dtype == 0 ? 4 : 2;
    // ray mode: the hit list's length is produced on the device
    const int n_tiles = RAY ? *p.ray.n_hits : p.n_tiles;

    if (warp == kProducerWarp) {
        if (lane == 0) {
            // Two independent copy streams, issued by one thread in an event
            // loop so neither blocks the other: input tiles (x_empty[s]
            // gates each slot's staging buffer) and weight blocks (w_empty
            // gates each ring slot). Both follow the consumers' order.
            uint32_t xph = 0u, xused = 0u;  // per-slot parity of the next load / slot used
            uint32_t wcount = 0, q = 0, wph = 0;
            bool ok = true;
            int xr = 0, xs = 0;  // next input tile to load: (round, slot)
            int wr = 0, wl = 0;  // next weight block: (round, layer)
            const bool no_tiles = tile_of<SLOTS>(0, 0, n_tiles) < 0;
            bool x_done = RAY || no_tiles;  // ray mode: samples are generated, not loaded
            bool w_done = p.resident || no_tiles;
            // fp32 biases of every layer, read by the epilogue
            mbar_arrive_expect_tx(bar(kBarBias), p.bias_bytes);
            bulk_g2s(base + p.off_bias, p.wpack + p.bias_gofs, p.bias_bytes, bar(kBarBias));
            if (p.resident) {
                mbar_arrive_expect_tx(bar(kBarWFull), p.w_total_bytes);
                for (int l = 0; l < n_layers; ++l)
                    bulk_g2s(w_base + p.layer[l].w_off, p.wpack + p.layer[l].w_off, p.layer[l].w_bytes,
                             bar(kBarWFull));
            }
            uint64_t t_last = global_timer_ns();
            while (!(x_done && w_done)) {
                bool progressed = false;
                if (!x_done && mbar_test_wait(bar(kBarXEmpty + xs), ((xph >> xs) & 1u) ^ 1u)) {
                    const int t = tile_of<SLOTS>(xr, xs, n_tiles);
                    const long long row0 = static_cast<long long>(t) * kTileM;
                    long long rows = p.n_rows - row0;
                    if (rows > kTileM) rows = kTileM;
                    const uint32_t bytes = static_cast<uint32_t>(rows) * p.in_dim * esize;
                    mbar_arrive_expect_tx(bar(kBarXFull + xs), bytes);
                    bulk_g2s(x_base + xs * p.x_stage_bytes,
                             static_cast<const uint8_t*>(p.x) + row0 * p.in_dim * esize, bytes, bar(kBarXFull + xs));
                    xph ^= 1u << xs;
                    xused |= 1u << xs;
                    if (++xs == SLOTS) {
                        xs = 0;
                        ++xr;
                    }
                    x_done = tile_of<SLOTS>(xr, xs, n_tiles) < 0;
                    progressed = true;
                }
                if (!w_done && mbar_test_wait(bar(kBarWEmpty + q), wph ^ 1u)) {
                    mbar_arrive_expect_tx(bar(kBarWFull + q), p.layer[wl].w_bytes);
                    bulk_g2s(w_base + q * p.w_slot_bytes, p.wpack + p.layer[wl].w_off, p.layer[wl].w_bytes,
                             bar(kBarWFull + q));
                    ++wcount;
                    if (++q == static_cast<uint32_t>(p.w_stages)) {
                        q = 0;
                        wph ^= 1u;
                    }
                    if (++wl == n_layers) {
                        wl = 0;
                        ++wr;
                    }
                    w_done = tile_of<SLOTS>(wr, 0, n_tiles) < 0;
                    progressed = true;
                }
                if (progressed) {
                    t_last = global_timer_ns();
                } else if (*abort) {
                    ok = false;
                    break;
                } else if (global_timer_ns() - t_last > RDVB_WAIT_LIMIT_NS) {
                    *abort = 1u;
                    atomicOr(&g_status, x_done ? kStatusTimeoutWEmpty : kStatusTimeoutXEmpty);
                    ok = false;
                    break;
                } else {
                    __nanosleep(128);  // leave the scheduler to the compute warps
                }
            }
            if (!ok) {
                // Let every copy this thread started land before the CTA exits.
                for (int s = 0; s < SLOTS; ++s)
                    if ((xused >> s) & 1u) drain_wait(bar(kBarXFull + s), ((xph >> s) & 1u) ^ 1u);
                if (p.resident) {
                    drain_wait(bar(kBarWFull), 0u);
                } else {
                    for (uint32_t c = (wcount > (uint32_t)p.w_stages ? wcount - p.w_stages : 0u); c < wcount; ++c)
                        drain_wait(bar(kBarWFull + c % p.w_stages), (c / p.w_stages) & 1u);
                }
            }
            // the bias copy is waited for by the epilogue only when the CTA has tiles
            drain_wait(bar(kBarBias), 0u);
        }
    } else if (warp == kStageWarp) {
        // ---------------------------------------------- input staging
        uint32_t xfph = 0u, a0eph = 0u;
        const uint32_t kch0 = p.layer[0].k_pad >> 3;
        // only chunks holding input columns are rewritten; the rest stay zero
        const uint32_t kch_in = (static_cast<uint32_t>(p.in_dim) + 7u) >> 3;
        const bool vec = p.x_dtype == 0 && (p.in_dim & 7) == 0;
        bool ok = true;
        (void)kch0;
        for (int r = 0; ok && tile_of<SLOTS>(r, 0, n_tiles) >= 0; ++r) {
            for (int s = 0; s < SLOTS; ++s) {
                const int t = tile_of<SLOTS>(r, s, n_tiles);
                if (t < 0) break;
                if constexpr (RAY) {
                    // sample i of the ray at t_i = t0 + (i + 1/2) * dt, dt = (t1 - t0) / 128,
                    // as float16/bfloat16 (x, y, z, 0...) in the layer-0 A tile
                    const bool good = mbar_wait(bar(kBarA0Empty + s), ((a0eph >> s) & 1u) ^ 1u, abort, &g_status,
                                                kStatusTimeoutOther);
                    if (!__all_sync(0xffffffffu, good)) {
                        ok = false;
                        break;
                    }
                    a0eph ^= 1u << s;
                    if constexpr (RAY == kModeMarch) {
                        // step k = 128 c + i of the ray at x_e + (k * step) * w
                        const int ray = __ldg(p.ray.hit_list + t);
                        const MarchRay& mr = p.ray.rec[ray];
                        const int c = t - __ldg(&mr.base);
                        const float xe0 = __ldg(&mr.x[0]), xe1 = __ldg(&mr.x[1]), xe2 = __ldg(&mr.x[2]);
                        const float w0 = __ldg(&mr.w[0]), w1 = __ldg(&mr.w[1]), w2 = __ldg(&mr.w[2]);
                        const uint32_t a_tile = a_base + static_cast<uint32_t>(s) * p.a0_bytes;
#pragma unroll
                        for (int k = 0; k < kTileM / 32; ++k) {
                            const uint32_t ri = static_cast<uint32_t>(k * 32 + lane);
                            const float tk = __fmul_rn(static_cast<float>(c * kTileM + static_cast<int>(ri)), p.ray.step);
                            st_shared_v4(a_tile + sw128_offset(ri, 0, kTileM),
                                         pack2_rt<BF16>(__fadd_rn(xe0, __fmul_rn(tk, w0)), __fadd_rn(xe1, __fmul_rn(tk, w1)),
                                                        p.relu_in),
                                         pack2_rt<BF16>(__fadd_rn(xe2, __fmul_rn(tk, w2)), 0.0f, p.relu_in), 0u, 0u);
                        }
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(bar(kBarA0Full + s));
                        continue;
                    }
                    float o[3], w[3], t0, t1;
                    ray_setup(p.ray, __ldg(p.ray.hit_list + t), o, w, t0, t1);
                    const float dt = (t1 - t0) / static_cast<float>(kTileM);
                    const uint32_t a_tile = a_base + static_cast<uint32_t>(s) * p.a0_bytes;
#pragma unroll
                    for (int k = 0; k < kTileM / 32; ++k) {
                        const uint32_t ri = static_cast<uint32_t>(k * 32 + lane);
                        const float ts = t0 + (static_cast<float>(ri) + 0.5f) * dt;
                        st_shared_v4(a_tile + sw128_offset(ri, 0, kTileM), pack2_rt<BF16>(o[0] + ts * w[0], o[1] + ts * w[1], 0),
                                     pack2_rt<BF16>(o[2] + ts * w[2], 0.0f, 0), 0u, 0u);
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(bar(kBarA0Full + s));
                    continue;
                }
                bool good = mbar_wait(bar(kBarXFull + s), (xfph >> s) & 1u, abort, &g_status, kStatusTimeoutXFull) &&
                            mbar_wait(bar(kBarA0Empty + s), ((a0eph >> s) & 1u) ^ 1u, abort, &g_status,
                                      kStatusTimeoutOther);
                // every lane leaves together, so the warp-wide steps below
                // never run diverged
                if (!__all_sync(0xffffffffu, good)) {
                    ok = false;
                    break;
                }
                xfph ^= 1u << s;
                a0eph ^= 1u << s;
                const long long row0 = static_cast<long long>(t) * kTileM;
                const long long rv = p.n_rows - row0;
                const uint32_t rows_valid = rv > kTileM ? static_cast<uint32_t>(kTileM) : static_cast<uint32_t>(rv);
                const uint8_t* xs = base_ptr + p.off_x + s * p.x_stage_bytes;
                const uint32_t a_tile = a_base + static_cast<uint32_t>(s) * p.a0_bytes;
                for (uint32_t idx = lane; idx < kTileM * kch_in; idx += 32) {
                    const uint32_t ri = idx / kch_in;
                    const uint32_t c = idx - ri * kch_in;
                    float v[8];
                    if (vec && ri < rows_valid) {
                        const float4* src = reinterpret_cast<const float4*>(xs + (ri * p.in_dim + c * 8) * 4);
                        const float4 u0 = src[0], u1 = src[1];
                        v[0] = u0.x; v[1] = u0.y; v[2] = u0.z; v[3] = u0.w;
                        v[4] = u1.x; v[5] = u1.y; v[6] = u1.z; v[7] = u1.w;
                    } else {
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            const uint32_t k = c * 8 + e;
                            v[e] = (ri < rows_valid && k < static_cast<uint32_t>(p.in_dim))
                                       ? load_x_elem(xs, p.x_dtype, ri * p.in_dim + k)
                                       : 0.0f;
                        }
                    }
                    st_shared_v4(a_tile + sw128_offset(ri, c * 8, kTileM), pack2_rt<BF16>(v[0], v[1], p.relu_in),
                                 pack2_rt<BF16>(v[2], v[3], p.relu_in), pack2_rt<BF16>(v[4], v[5], p.relu_in),
                                 pack2_rt<BF16>(v[6], v[7], p.relu_in));
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(bar(kBarXEmpty + s));
                    mbar_arrive(bar(kBarA0Full + s));
                }
            }
        }
    } else if (warp == kMmaWarp || (ISSUERS > 1 && warp == kMmaWarp2) || (ISSUERS > 2 && warp >= 20)) {
        // With resident weights the slots are independent and the issuing
        // threads split them (slot s goes to issuer s % ISSUERS): a
        // slot-layer's wait, K-step MMAs and commit are a few hundred cycles
        // of one thread's time, and an issuer walking its slots in order
        // waits on a slot that is behind while another is ready. Measured on
        // width-64 chains: 2 issuers -> 4 (one per slot) takes config 5 from
        // 6.3 to 5.5 ms. Streamed weights keep one issuer, whose in-order
        // walk over the slots releases each ring block.
        const int mi = issuer_index(warp);
        constexpr int n_iss = ISSUERS;  // the host launches 2 or 4 only with resident weights
        if (lane == 0) {
            uint32_t aph = 0u, a0ph = 0u;  // per-slot parities of the next a_full / a0_full phase
            uint32_t q = 0, wph = 0;       // weight ring slot and its phase
            bool ok = true;
            bool issued = false;
            const uint64_t w_desc_sw = umma_desc_sw128(w_base);     // + (byte offset >> 4)
            if (p.resident) ok = mbar_wait(bar(kBarWFull), 0u, abort, &g_status, kStatusTimeoutWFull);
            // Per-slot operand addresses, fixed for the whole kernel.
            uint32_t d_tm[SLOTS], a_tm[SLOTS];
            uint64_t a0_desc[SLOTS];
#pragma unroll
            for (int s = 0; s < SLOTS; ++s) {
                d_tm[s] = tmem_base + static_cast<uint32_t>(s) * p.acc_stride;
                a_tm[s] = tmem_base + p.act_base + static_cast<uint32_t>(s) * p.act_stride;
                a0_desc[s] = umma_desc_sw128(a_base + static_cast<uint32_t>(s) * p.a0_bytes);
            }
            for (int r = 0; ok && tile_of<SLOTS>(r, 0, n_tiles) >= 0; ++r) {
                for (int l = 0; l < n_layers && ok; ++l) {
                    const uint32_t ksteps = p.layer[l].k_pad >> 4;
                    const uint32_t n8 = p.layer[l].n_pad * 8u;  // one K atom of B, in 16-byte units
                    const uint32_t idesc = p.layer[l].idesc;
                    uint32_t blk;  // byte offset of this layer's block from w_base
                    if (p.resident) {
                        blk = p.layer[l].w_off;
                    } else {
                        if (!mbar_wait(bar(kBarWFull + q), wph, abort, &g_status, kStatusTimeoutWFull)) {
                            ok = false;
                            break;
                        }
                        blk = q * p.w_slot_bytes;
                    }
                    // B descriptors of this layer's K steps, shared by every slot
                    const uint64_t b0 = w_desc_sw + (blk >> 4);
                    uint64_t b_desc[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) b_desc[j] = b0 + (j >> 2) * n8 + (j & 3) * 2;
#pragma unroll
                    for (int s = 0; s < SLOTS; ++s) {
                        if (s % n_iss != mi) continue;
                        if (tile_of<SLOTS>(r, s, n_tiles) < 0) break;
                        if (l == 0) {
                            if (!mbar_wait(bar(kBarA0Full + s), (a0ph >> s) & 1u, abort, &g_status,
                                           kStatusTimeoutXFull)) {
                                ok = false;
                                break;
                            }
                            a0ph ^= 1u << s;
                        }
                        // previous layer's activations written (or, at layer 0,
                        // the previous round's last accumulator read)
                        if (l > 0 || r > 0) {
                            if (!mbar_wait(bar(kBarAFull + s), (aph >> s) & 1u, abort, &g_status,
                                           kStatusTimeoutAFull)) {
                                ok = false;
                                break;
                            }
                            aph ^= 1u << s;
                        }
                        tc_fence_after();
                        // input layer: A from the staged shared-memory tile; hidden
                        // layers: A = previous activations, resident in TMEM.
                        // Resident-weight chains (two issuers, mostly narrow
                        // layers) issue exactly ksteps MMAs; the streamed-weight
                        // kernel keeps the fixed 8-step loop, which measured
                        // faster for its 8-step layers.
                        if constexpr (ISSUERS >= 2) {
                            issue_layer(ksteps, l > 0, d_tm[s], a0_desc[s], a_tm[s], b_desc, idesc);
                        } else if (l == 0) {
#pragma unroll
                            for (int j = 0; j < 8; ++j)
                                if (j < static_cast<int>(ksteps))
                                    umma_f16(d_tm[s], a0_desc[s] + (j >> 2) * (kAtomBytes >> 4) + (j & 3) * 2,
                                             b_desc[j], idesc, j > 0 ? 1u : 0u);
                        } else {
#pragma unroll
                            for (int j = 0; j < 8; ++j)
                                if (j < static_cast<int>(ksteps))
                                    umma_f16_ts(d_tm[s], a_tm[s] + j * 8u, b_desc[j], idesc, j > 0 ? 1u : 0u);
                        }
                        if (l == 0) umma_commit(bar(kBarA0Empty + s));
                        umma_commit(bar(kBarAccFull + s));
                        issued = true;
                    }
                    if (!ok) break;
                    if (!p.resident) {
                        umma_commit(bar(kBarWEmpty + q));
                        if (++q == static_cast<uint32_t>(p.w_stages)) {
                            q = 0;
                            wph ^= 1u;
                        }
                    }
                }
            }
            if (!ok && issued) {
                umma_commit(bar(kBarDrain + mi));
                drain_wait(bar(kBarDrain + mi), 0u);
            }
        }
    } else {
        // ------------------------------------------------------ epilogue
        const int quad = warp & 3;
        const int grp = warp >> 2;
        const int row = quad * 32 + lane;
        const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
        // Warp group grp owns slot grp % SLOTS and, of that slot's 16-column
        // chunks, every kGroupsPerSlot-th one starting at grp / SLOTS, so the
        // slots' epilogues run concurrently and a warp only ever waits on its
        // own slot's accumulator.
        constexpr int kGroupsPerSlot = 4 / SLOTS;
        const int s = grp % SLOTS;
        const uint32_t sub = static_cast<uint32_t>(grp / SLOTS);
        const uint32_t t_col = tmem_base + lane_off + static_cast<uint32_t>(s) * p.acc_stride;
        const uint32_t t_act = tmem_base + lane_off + p.act_base + static_cast<uint32_t>(s) * p.act_stride;
        uint32_t acph = 0u;     // parity of the slot's next acc_full phase
        uint32_t comp_ph = 0u;  // ray mode: parity of the slot's next compositing phase
        bool ok = true;
        const float* bias_smem = reinterpret_cast<const float*>(base_ptr + p.off_bias);
        if (tile_of<SLOTS>(0, s, n_tiles) >= 0) {
            const bool got = mbar_wait(bar(kBarBias), 0u, abort, &g_status, kStatusTimeoutWFull);
            ok = __all_sync(0xffffffffu, got);
        }

        for (int r = 0; ok; ++r) {
            const int t = tile_of<SLOTS>(r, s, n_tiles);
            if (t < 0) break;
            for (int l = 0; l < n_layers && ok; ++l) {
                const bool last = (l == n_layers - 1);
                const uint32_t nch = p.layer[l].n_pad >> 4;
                const bool relu = p.layer[l].relu != 0;
                const float* bias_l = bias_smem + p.layer[l].b_idx;
                const bool good = mbar_wait(bar(kBarAccFull + s), acph, abort, &g_status, kStatusTimeoutAccFull);
                // tcgen05.ld/st below are warp-collective: leave together
                if (!__all_sync(0xffffffffu, good)) {
                    ok = false;
                    break;
                }
                acph ^= 1u;
                tc_fence_after();
                if (!last) {
                    // two chunks per round trip: columns c*16..c*16+15 of this
                    // layer are K elements c*16.. of the next, 8 packed columns
                    for (uint32_t c = sub; c < nch; c += 2 * kGroupsPerSlot) {
                        const uint32_t c2 = c + kGroupsPerSlot;
                        uint32_t v0[16], v1[16];
                        tmem_ld16(t_col + c * 16, v0);
                        if (c2 < nch) tmem_ld16(t_col + c2 * 16, v1);
                        tmem_wait_ld(v0);
                        reg_barrier(v1);
                        add_bias16(v0, bias_l + c * 16);
                        if (c2 < nch) add_bias16(v1, bias_l + c2 * 16);
                        uint32_t pk[8];
                        if (relu) convert_chunk<BF16, true>(v0, pk);
                        else convert_chunk<BF16, false>(v0, pk);
                        tmem_st8(t_act + c * 8, pk);
                        if (c2 < nch) {
                            if (relu) convert_chunk<BF16, true>(v1, pk);
                            else convert_chunk<BF16, false>(v1, pk);
                            tmem_st8(t_act + c2 * 8, pk);
                        }
                    }
                    tmem_wait_st();
                } else if constexpr (RAY) {
                    if constexpr (RAY == kModeMarch) {
                        if (sub == 0) {
                            // transmittance: tau_i = extinction_i * scale * step for
                            // the chunk's valid steps (0 past the ray's end); each
                            // quadrant scans its 32 steps, quadrant 0 chains the 4
                            // (sum, largest prefix) partials in step order
                            uint32_t v0[16];
                            tmem_ld16(t_col, v0);
                            tmem_wait_ld(v0);
                            add_bias16(v0, bias_l);
                            const int ray = __ldg(p.ray.hit_list + t);
                            const MarchRay& mr = p.ray.rec[ray];
                            const int c = t - __ldg(&mr.base);
                            float e = __uint_as_float(v0[0]);
                            if (relu) e = fmaxf(e, 0.0f);
                            const bool valid = c * kTileM + row < __ldg(&mr.n_steps);
                            const float tau = valid ? __fmul_rn(__fmul_rn(e, p.ray.scale), p.ray.step) : 0.0f;
                            float incl = tau;
    #pragma unroll
                            for (int d = 1; d < 32; d <<= 1) {
                                const float nb = __shfl_up_sync(0xffffffffu, incl, d);
                                if (lane >= d) incl += nb;
                            }
                            float pmax = valid ? incl : -INFINITY;
    #pragma unroll
                            for (int d = 16; d > 0; d >>= 1) pmax = fmaxf(pmax, __shfl_xor_sync(0xffffffffu, pmax, d));
                            const float sum_q = __shfl_sync(0xffffffffu, incl, 31);
                            float* scr = reinterpret_cast<float*>(base_ptr + p.off_ray) + s * 16;
                            if (lane == 0) {
                                scr[quad * 4 + 0] = sum_q;
                                scr[quad * 4 + 1] = pmax;
                                mbar_arrive(bar(kBarComp + s));
                            }
                            if (quad == 0) {
                                bool got = true;
                                if (lane == 0) {
                                    got = mbar_wait(bar(kBarComp + s), comp_ph, abort, &g_status, kStatusTimeoutOther);
                                    if (got) {
                                        float sum = 0.0f, best = -INFINITY;
    #pragma unroll
                                        for (int q = 0; q < 4; ++q) {
                                            best = fmaxf(best, sum + scr[q * 4 + 1]);
                                            sum += scr[q * 4 + 0];
                                        }
                                        p.ray.chunk_out[t] = make_float2(sum, best);
                                    }
                                }
                                comp_ph ^= 1u;
                                if (!__shfl_sync(0xffffffffu, got ? 1 : 0, 0)) ok = false;
                            }
                        }
                    } else if (sub == 0) {
                        // render: front-to-back emission-absorption
                        // compositing of the ray's 128 samples (rows = samples
                        // in order): the warps owning columns 0..15 (sigma, r,
                        // g, b) each scan their quadrant's 32 samples with
                        // shuffles; quadrant 0 chains the 4 partials.
                        uint32_t v0[16];
                        tmem_ld16(t_col, v0);
                        tmem_wait_ld(v0);
                        add_bias16(v0, bias_l);
                        const int pix = __ldg(p.ray.hit_list + t);
                        float o[3], w[3], t0, t1;
                        ray_setup(p.ray, pix, o, w, t0, t1);
                        const float dt = (t1 - t0) / static_cast<float>(kTileM);
                        const float tau = softplus_f(__uint_as_float(v0[0])) * dt;
                        const float alpha = -expm1f(-tau);
                        float incl = tau;
#pragma unroll
                        for (int d = 1; d < 32; d <<= 1) {
                            const float nb = __shfl_up_sync(0xffffffffu, incl, d);
                            if (lane >= d) incl += nb;
                        }
                        float excl = __shfl_up_sync(0xffffffffu, incl, 1);
                        if (lane == 0) excl = 0.0f;
                        const float wgt = expf(-excl) * alpha;  // T_i * alpha_i within the quadrant
                        float cr = wgt * sigmoid_f(__uint_as_float(v0[1]));
                        float cg = wgt * sigmoid_f(__uint_as_float(v0[2]));
                        float cb = wgt * sigmoid_f(__uint_as_float(v0[3]));
#pragma unroll
                        for (int d = 16; d > 0; d >>= 1) {
                            cr += __shfl_xor_sync(0xffffffffu, cr, d);
                            cg += __shfl_xor_sync(0xffffffffu, cg, d);
                            cb += __shfl_xor_sync(0xffffffffu, cb, d);
                        }
                        const float tau_q = __shfl_sync(0xffffffffu, incl, 31);
                        float* scr = reinterpret_cast<float*>(base_ptr + p.off_ray) + s * 16;
                        if (lane == 0) {
                            scr[quad * 4 + 0] = cr;
                            scr[quad * 4 + 1] = cg;
                            scr[quad * 4 + 2] = cb;
                            scr[quad * 4 + 3] = tau_q;
                            mbar_arrive(bar(kBarComp + s));
                        }
                        if (quad == 0) {
                            // the 4 partials of this ray, chained front to back
                            bool got = true;
                            if (lane == 0) {
                                got = mbar_wait(bar(kBarComp + s), comp_ph, abort, &g_status, kStatusTimeoutOther);
                                if (got) {
                                    float rr = 0.0f, gg = 0.0f, bb = 0.0f, tsum = 0.0f;
#pragma unroll
                                    for (int q = 0; q < 4; ++q) {
                                        const float tr = expf(-tsum);
                                        rr += tr * scr[q * 4 + 0];
                                        gg += tr * scr[q * 4 + 1];
                                        bb += tr * scr[q * 4 + 2];
                                        tsum += scr[q * 4 + 3];
                                    }
                                    reinterpret_cast<float4*>(p.ray.rgba)[pix] = make_float4(rr, gg, bb, -expm1f(-tsum));
                                }
                            }
                            comp_ph ^= 1u;
                            if (!__shfl_sync(0xffffffffu, got ? 1 : 0, 0)) ok = false;
                        }
                    }
                } else {
                    const long long grow = static_cast<long long>(t) * kTileM + row;
                    float* yrow = p.y + grow * p.out_dim;
                    for (uint32_t c = sub; c < nch; c += kGroupsPerSlot) {
                        uint32_t v0[16];
                        tmem_ld16(t_col + c * 16, v0);
                        tmem_wait_ld(v0);
                        add_bias16(v0, bias_l + c * 16);
                        if (grow < p.n_rows) {
                            float o[16];
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                const float a = __uint_as_float(v0[i]);
                                o[i] = relu ? fmaxf(a, 0.0f) : a;
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
                // activations written (or, after the last layer, the
                // accumulator read): the slot's next MMA may proceed
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(kBarAFull + s));
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

// Packs fp32 [N, K] row-major weights (PyTorch nn.Linear layout) and fp32
// biases of every layer into the image the kernel copies straight into
// shared memory: per layer the K-major SW128 weight block (zero padded to
// n_pad x katoms*64, float16 or bfloat16), then one block holding every
// layer's fp32 bias zero padded to n_pad.
struct PackLayer {
    const float* W;
    const float* b;
    uint32_t K, N, n_pad, katoms, w_off, b_idx;
};
struct PackParams {
    PackLayer layer[kMaxLayers];
    int n_layers;
    int bf16;
    uint8_t* wpack;
    uint32_t bias_gofs;     // byte offset of the bias block
    uint32_t w_chunks;      // 16-byte weight chunks of all layers
    uint32_t total_chunks;  // + 4-float bias chunks
};

__global__ void mlp_pack_kernel(const __grid_constant__ PackParams p) {
    for (uint32_t g = blockIdx.x * blockDim.x + threadIdx.x; g < p.total_chunks; g += gridDim.x * blockDim.x) {
        if (g >= p.w_chunks) {
            // bias chunk: 4 consecutive entries of the padded bias block
            const uint32_t e0 = (g - p.w_chunks) * 4;
            float v[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t e = e0 + k;
                int l = 0;
                while (l + 1 < p.n_layers && e >= p.layer[l + 1].b_idx) ++l;
                const uint32_t n = e - p.layer[l].b_idx;
                v[k] = (n < p.layer[l].N) ? p.layer[l].b[n] : 0.0f;
            }
            *reinterpret_cast<float4*>(p.wpack + p.bias_gofs + e0 * 4) = make_float4(v[0], v[1], v[2], v[3]);
            continue;
        }
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
        *reinterpret_cast<uint4*>(p.wpack + L.w_off + sw128_offset(n, kc * 8, L.n_pad)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

}  // namespace mlp_tc
}  // namespace rdvb
