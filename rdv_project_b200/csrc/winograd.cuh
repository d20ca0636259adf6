// Winograd F(2x2, 3x3) convolution (stride 1, zero padding 1) with the
// input transform, the per-position GEMMs and the output transform fused in
// one kernel, plus the filter transform and a direct convolution.
//
// Replaces Conv2DTensorOpWinograd3x3 (rdv/domain/nn.py:1002-1087,
// rdv/shaders/tensors/conv2d_tensor_op_winograd3x3.h:95-178) and extends it
// to batched NHWC tensors and to 64 channels. Same arithmetic contract: the
// input transform V = B^T d B in fp32 (same operation order as
// _winograd_fwd, :59-78), V staged float16; the filter transform U = G g G^T
// in fp32, staged float16 (nn.py:525-538); products of float16 operands
// accumulated in fp32 on the tensor core; bias added in fp32 (:164-174).
//
// The inverse transform Y_ij = sum_uv A^T[i][u] A^T[j][v] M_uv (coefficients
// 0/+1/-1) runs on the tensor core as well: each output position (i, j) of
// the 2x2 tile has its own TMEM accumulator, and every nonzero term adds
// +-V_uv * U_uv to it (the sign is the MMA's negate-B bit), 36 position-GEMMs
// per block of tiles instead of 16 plus a CUDA-core inverse. The tensor
// core has the headroom; the CUDA cores, whose registers would otherwise hold
// the 2x2 x COUT partial outputs of every tile, are left free to transform
// and prefetch the input.
//
// Design (one persistent CTA per SM, 16 warps):
//   * U for all 16 positions stays resident in shared memory (K-major,
//     128-byte swizzle), loaded once by one bulk copy.
//   * A CTA walks blocks of 120 Winograd tiles (raster order over
//     (image, tile row, tile column)), each block as 4 "rows" u of the 4x4
//     transform domain. Warps 0-14 (480 threads, two (tile, 8-channel)
//     items each) load a row's input (16 x 16-byte loads in flight), form
//     the first (row) pass of B^T d B, then for v = 0..3 wait until the
//     GEMMs of the previous row released V tile v, write V_uv (float16) and
//     arrive. Warp 15 only issues: once all 15 warps wrote V tile v it issues
//     position (u, v)'s GEMMs (M = 128; V rows 120-127 are not used), so the
//     transform of row r + 1 overlaps the GEMMs of row r, position by position.
//   * TMEM: the 4 accumulators (i, j) of a block, COUT columns each, double
//     buffered across blocks (512 columns). After a block's last GEMM, warp w
//     of 0-14 reads lane quadrant w%4 x channels 16*(w/4)..+15 (warp 3 also
//     channels 48-63 of quadrant 3), adds the bias and stores, while the
//     next block's GEMMs run.
// HBM traffic is the input read (halo re-reads hit L1/L2) plus the output
// write, the operator's roofline.
#pragma once
#include <cuda.h>  // CUtensorMap (the type only; the map is encoded on the host)
#include "ptx.cuh"

namespace rdvb {
namespace wino {

constexpr int kTileM = 128;         // GEMM M: rows of a V tile and TMEM lanes
constexpr int kBlockTiles = 120;    // Winograd tiles per block (V rows 120-127 are unused)
constexpr int kXWarps = 15;         // transform + epilogue warps: 480 threads x 2 items = 120 tiles x 8 chunks
constexpr int kXThreads = kXWarps * 32;
constexpr int kIssueWarp = 15;      // the MMA-issuing warp
constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxChannels = 64;    // CIN, COUT: multiples of 16, at most 64
constexpr uint32_t kATileBytes = kTileM * 128;  // one position's V tile (128-byte rows)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kDCols = 4 * kMaxChannels;   // one block's 4 output accumulators

struct Params {
    const void* x;          // [N, H, W, CIN] NHWC, float32 or float16
    void* y;                // [N, H, W, COUT] NHWC, float32 or float16
    const uint8_t* u_pack;  // 16 blocks of (COUT rows x 128 B), K-major SW128
    const float* bias;      // [COUT] or null
    int h, w, cin, cout;
    int y_f16;
    int tiles_w, tiles_per_img;
    int n_tiles;
    int n_blocks;
    uint32_t u_bytes;       // 16 * cout * 128
    uint32_t off_a, off_bar;
    uint32_t idesc;         // M = 128, N = COUT, f16 x f16 -> f32
};

enum : int {
    kBarUFull = 0,
    kBarAFull = 1,       // + v: V tile v written (16 warp arrivals)
    kBarAEmpty = 5,      // + v: the GEMMs reading V tile v are done (commit)
    kBarDFull = 9,       // + half: a block's accumulators are final (commit)
    kBarDrain = 11,
    kNumBars = 12,
};
constexpr uint32_t kBarBlockBytes = kNumBars * 8 + 16;
constexpr uint32_t kNegateB = 1u << 14;  // instruction-descriptor bit: negate the B operand

// A^T of F(2, 3) = [[1, 1, 1, 0], [0, 1, -1, -1]] (the reference's
// _winograd_inv, :80-93).
__host__ __device__ constexpr int at_coef(int i, int u) {
    return i == 0 ? (u < 3 ? 1 : 0) : (u == 0 ? 0 : (u == 1 ? 1 : -1));
}

// One transform item: a Winograd tile of the current block and an 8-channel
// chunk of its input.
struct Item {
    long long e0;      // element offset of patch (row 0, col 0), channel chunk start
    uint32_t rmask;    // bit k: patch row k inside the image (0 if no item)
    uint32_t cmask;    // bit c: patch column c inside the image
    uint32_t soff;     // byte offset of (tile row, chunk) inside a V tile
};

// Item `idx` (tile row idx / (CIN/8) of block `blk`, chunk idx % (CIN/8)).
// Returns false when the block has no such item. Tiles past the end get an
// all-invalid patch, so their V rows are written as zeros.
__device__ __forceinline__ bool make_item(const Params& p, int blk, int idx, Item& it) {
    const int cch = p.cin >> 3;
    it.rmask = 0;
    it.cmask = 0;
    it.e0 = 0;
    it.soff = 0;
    if (idx >= kBlockTiles * cch) return false;
    const int tr = idx / cch, ck = idx - tr * cch;
    it.soff = sw128_offset(static_cast<uint32_t>(tr), static_cast<uint32_t>(ck * 8), kTileM);
    const int t = blk * kBlockTiles + tr;
    if (t < p.n_tiles) {
        const int img = t / p.tiles_per_img;
        const int rem = t - img * p.tiles_per_img;
        const int ty = rem / p.tiles_w, tx = rem - ty * p.tiles_w;
        const int gh0 = 2 * ty - 1, gw0 = 2 * tx - 1;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            if (gh0 + k >= 0 && gh0 + k < p.h) it.rmask |= 1u << k;
            if (gw0 + k >= 0 && gw0 + k < p.w) it.cmask |= 1u << k;
        }
        it.e0 = ((static_cast<long long>(img) * p.h + gh0) * p.w + gw0) * p.cin + ck * 8;
    }
    return true;
}

__device__ __forceinline__ void h8_to_f32(const uint4& q, float (&v)[8]) {
    const __half2* h2 = reinterpret_cast<const __half2*>(&q);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(h2[e]);
        v[2 * e] = f.x;
        v[2 * e + 1] = f.y;
    }
}

// Row pairs and signs of B^T (the reference's _winograd_fwd, :59-78): the
// first pass of domain row u is m = d_k0 + t_u * d_k1 (one rounding, so
// fma(t, b, a) is the reference's a - b / a + b exactly), times s_u:
//   u = 0: d0 - d2      u = 1: d1 + d2      u = 2: d2 - d1 = -(d1 - d2)
//   u = 3: d1 - d3.
// The same holds for the second pass over columns v. The factor s = -1 of
// u = 2 and v = 2 is not applied to V (float16 rounding is symmetric, so
// -fp16(x) == fp16(-x)); it flips the sign of the position's GEMMs instead.
__host__ __device__ constexpr int bt_k0(int u) { return u == 0 ? 0 : 1; }
__host__ __device__ constexpr int bt_k1(int u) { return u == 0 ? 2 : (u == 3 ? 3 : 2); }
__host__ __device__ constexpr float bt_t(int u) { return u == 1 ? 1.0f : -1.0f; }
__host__ __device__ constexpr int bt_s(int u) { return u == 2 ? -1 : 1; }

// m for both items of the thread (domain row u): all 16 loads of a float16
// input are issued before the first use.
template <bool X16>
__device__ __forceinline__ void first_pass(const Params& p, const Item (&it)[2], long long row_stride, int u,
                                           float (&m)[2][4][8]) {
    const int k0 = bt_k0(u), k1 = bt_k1(u);
    const float t = bt_t(u);
    const long long o0 = k0 * row_stride, o1 = k1 * row_stride;
    if constexpr (X16) {
        const __half* x = static_cast<const __half*>(p.x);
        uint4 ra[2][4], rb[2][4];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const bool v0 = (it[i].rmask >> k0) & 1u, v1 = (it[i].rmask >> k1) & 1u;
#pragma unroll
            for (int col = 0; col < 4; ++col) {
                const bool vc = (it[i].cmask >> col) & 1u;
                const long long ec = it[i].e0 + static_cast<long long>(col) * p.cin;
                ra[i][col] = (vc && v0) ? __ldg(reinterpret_cast<const uint4*>(x + ec + o0)) : make_uint4(0u, 0u, 0u, 0u);
                rb[i][col] = (vc && v1) ? __ldg(reinterpret_cast<const uint4*>(x + ec + o1)) : make_uint4(0u, 0u, 0u, 0u);
            }
        }
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
            for (int col = 0; col < 4; ++col) {
                float a[8], b[8];
                h8_to_f32(ra[i][col], a);
                h8_to_f32(rb[i][col], b);
#pragma unroll
                for (int e = 0; e < 8; ++e) m[i][col][e] = fmaf(t, b[e], a[e]);
            }
    } else {
        const float* x = static_cast<const float*>(p.x);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const bool v0 = (it[i].rmask >> k0) & 1u, v1 = (it[i].rmask >> k1) & 1u;
#pragma unroll
            for (int col = 0; col < 4; ++col) {
                const bool vc = (it[i].cmask >> col) & 1u;
                const long long ec = it[i].e0 + static_cast<long long>(col) * p.cin;
                const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
                const float4* pa = reinterpret_cast<const float4*>(x + ec + o0);
                const float4* pb = reinterpret_cast<const float4*>(x + ec + o1);
                const float4 a0 = (vc && v0) ? __ldg(pa) : z, a1 = (vc && v0) ? __ldg(pa + 1) : z;
                const float4 b0 = (vc && v1) ? __ldg(pb) : z, b1 = (vc && v1) ? __ldg(pb + 1) : z;
                const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
                for (int e = 0; e < 8; ++e) m[i][col][e] = fmaf(t, b[e], a[e]);
            }
        }
    }
}

// Second (column) pass for domain column V of one item (without the factor
// s_V), float16, into V tile V.
template <int V>
__device__ __forceinline__ void store_v(const float (&m)[4][8], uint32_t dst) {
    constexpr int c0 = bt_k0(V), c1 = bt_k1(V);
    constexpr float t = bt_t(V);
    uint32_t pk[4];
#pragma unroll
    for (int e = 0; e < 8; e += 2)
        pk[e >> 1] = pack_f16x2(fmaf(t, m[c1][e], m[c0][e]), fmaf(t, m[c1][e + 1], m[c0][e + 1]));
    st_shared_v4(dst, pk[0], pk[1], pk[2], pk[3]);
}

// The GEMMs of domain position (u, v): for every output position (i, j)
// with a nonzero coefficient c = A^T[i][u] * A^T[j][v], D_ij += c * s_u * s_v
// * V'_uv * U_uv (V' as stored). The first contribution to D_ij in a block
// comes from (u, v) = (i, j) (A^T[1][0] = 0) and overwrites it.
// Fully unrolled, every descriptor in its own register: an MMA's operand
// registers are read after issue, so recomputing one in a loop would stall
// the issuing thread until the previous MMA has consumed it.
__device__ __forceinline__ void issue_position(int u, int v, uint32_t d_base, uint64_t ad, uint64_t bd,
                                               uint32_t idesc, uint32_t ksteps) {
    const int s = bt_s(u) * bt_s(v);
    uint64_t a[4], b[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        a[k] = ad + 2 * k;
        b[k] = bd + 2 * k;
    }
    const uint32_t id_neg = idesc | kNegateB;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int i = q >> 1, j = q & 1;
        const int c = at_coef(i, u) * at_coef(j, v) * s;
        if (c == 0) continue;
        const uint32_t acc0 = (u == i && v == j) ? 0u : 1u;
        const uint32_t d = d_base + static_cast<uint32_t>(q * kMaxChannels);
        const uint32_t id = c > 0 ? idesc : id_neg;
#pragma unroll
        for (int k = 0; k < 4; ++k)
            if (k < static_cast<int>(ksteps)) umma_f16(d, a[k], b[k], id, k == 0 ? acc0 : 1u);
    }
}

// D_ij + bias of this lane's tile (channels 16*grp..+15) to the output.
// The TMEM loads are warp-collective: every lane runs them, only lanes with
// a valid tile store.
__device__ __forceinline__ void store_block(const Params& p, int t, bool valid, int grp, uint32_t td) {
    const int tt = valid ? t : 0;
    const int img = tt / p.tiles_per_img;
    const int rem = tt - img * p.tiles_per_img;
    const int ty = rem / p.tiles_w, tx = rem - ty * p.tiles_w;
    float b[16];
#pragma unroll
    for (int c = 0; c < 16; ++c) b[c] = p.bias ? __ldg(p.bias + 16 * grp + c) : 0.0f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint32_t r[16];
        tmem_ld16(td + static_cast<uint32_t>(q * kMaxChannels), r);
        tmem_wait_ld(r);
        const int oh = 2 * ty + (q >> 1), ow = 2 * tx + (q & 1);
        if (!valid || oh >= p.h || ow >= p.w) continue;  // past the end; odd h or w
        const long long o = ((static_cast<long long>(img) * p.h + oh) * p.w + ow) * p.cout + 16 * grp;
        float y[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) y[c] = __uint_as_float(r[c]) + b[c];
        if (!p.y_f16) {
            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.y) + o);
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4)
                dst[c4] = make_float4(y[4 * c4], y[4 * c4 + 1], y[4 * c4 + 2], y[4 * c4 + 3]);
        } else {
            uint32_t pk[8];
#pragma unroll
            for (int c = 0; c < 16; c += 2) pk[c >> 1] = pack_f16x2(y[c], y[c + 1]);
            uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(p.y) + o);
            dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
    }
}

struct RowCtx {
    const Params* p;
    Item it[2];
    bool has[2];
    long long row_stride;
    uint32_t a_base, bar_base;
    int r, u, lane;
    volatile uint32_t* abort;
    __device__ __forceinline__ uint32_t bar(int i) const { return bar_base + 8u * static_cast<uint32_t>(i); }
};

// Domain column V of the current row: wait until the GEMMs of the previous
// row released V tile V, write it (float16), signal the issuing warp.
template <int V>
__device__ __forceinline__ bool do_position(const RowCtx& c, const float (&m)[2][4][8]) {
    if (!mbar_wait_warp(c.bar(kBarAEmpty + V), (c.r & 1) ^ 1, c.abort, &g_status, kStatusTimeoutXEmpty))
        return false;
    if (c.has[0]) store_v<V>(m[0], c.a_base + V * kATileBytes + c.it[0].soff);
    if (c.has[1]) store_v<V>(m[1], c.a_base + V * kATileBytes + c.it[1].soff);
    fence_proxy_async_smem();
    __syncwarp();
    if (c.lane == 0) mbar_arrive(c.bar(kBarAFull + V));
    return true;
}

template <bool X16>
__device__ __forceinline__ bool do_row(const RowCtx& c) {
    float m[2][4][8];
    first_pass<X16>(*c.p, c.it, c.row_stride, c.u, m);
    return do_position<0>(c, m) && do_position<1>(c, m) && do_position<2>(c, m) && do_position<3>(c, m);
}

template <bool X16>
__global__ void __launch_bounds__(kThreads, 1) winograd_f23_kernel(const __grid_constant__ Params p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_addr(smem_raw);
    const uint32_t base = (raw_addr + 1023u) & ~1023u;
    uint8_t* const base_ptr = smem_raw + (base - raw_addr);
    const uint32_t u_base = base;  // U at offset 0
    RowCtx c;
    c.p = &p;
    c.a_base = base + p.off_a;
    c.bar_base = base + p.off_bar;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base_ptr + p.off_bar + kNumBars * 8);
    c.abort = reinterpret_cast<volatile uint32_t*>(base_ptr + p.off_bar + kNumBars * 8 + 4);

    const int warp = threadIdx.x >> 5;
    c.lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        mbar_init(c.bar(kBarUFull), 1);
        for (int v = 0; v < 4; ++v) {
            mbar_init(c.bar(kBarAFull + v), kXWarps);
            mbar_init(c.bar(kBarAEmpty + v), 1);
        }
        mbar_init(c.bar(kBarDFull), 1);
        mbar_init(c.bar(kBarDFull + 1), 1);
        mbar_init(c.bar(kBarDrain), 1);
        *c.abort = 0u;
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
    // blocks blockIdx.x, blockIdx.x + gridDim.x, ...; 4 domain rows each
    const int n_mine = blockIdx.x < p.n_blocks ? (p.n_blocks - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const int rows = 4 * n_mine;
    bool ok = true;

    if (warp == kIssueWarp) {
        // ----------------------------------------------------- MMA issuer
        if (c.lane == 0) {
            mbar_arrive_expect_tx(c.bar(kBarUFull), p.u_bytes);
            bulk_g2s(u_base, p.u_pack, p.u_bytes, c.bar(kBarUFull));
            ok = mbar_wait(c.bar(kBarUFull), 0u, c.abort, &g_status, kStatusTimeoutWFull);
            const uint64_t u_desc0 = umma_desc_sw128(u_base);
            const uint64_t u_pos = static_cast<uint64_t>(p.cout) * 8u;  // one position of U, 16-byte units
            const uint32_t ksteps = static_cast<uint32_t>(p.cin) >> 4;
            uint64_t a_desc[4];
#pragma unroll
            for (int v = 0; v < 4; ++v) a_desc[v] = umma_desc_sw128(c.a_base + v * kATileBytes);
            // The row loop is unrolled: every MMA's accumulate flag, sign and
            // operand offsets are compile-time constants. (With the row index
            // u a loop variable, some builds of this loop lost MMAs, or
            // accumulated into stale TMEM, depending only on how the
            // surrounding code was laid out; every build with constant
            // per-MMA flags gave exact results.)
            for (int bl = 0; ok && bl < n_mine; ++bl) {
                const uint32_t d_base = tmem_base + (bl & 1) * kDCols;
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int r = bl * 4 + u;
                    if (!ok) break;
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        if (!mbar_wait(c.bar(kBarAFull + v), r & 1, c.abort, &g_status, kStatusTimeoutAFull)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        issue_position(u, v, d_base, a_desc[v], u_desc0 + static_cast<uint64_t>(u * 4 + v) * u_pos,
                                       p.idesc, ksteps);
                        umma_commit(c.bar(kBarAEmpty + v));  // V tile v may be rewritten
                        if (u == 3 && v == 3) umma_commit(c.bar(kBarDFull + (bl & 1)));
                    }
                }
            }
            if (!ok) *c.abort = 1u;
            // every issued MMA completes before TMEM is released
            umma_commit(c.bar(kBarDrain));
            const uint64_t t0 = global_timer_ns();
            while (!mbar_try_wait_sleep(c.bar(kBarDrain), 0u, 500000u))
                if (global_timer_ns() - t0 > RDVB_WAIT_LIMIT_NS) {
                    atomicOr(&g_status, kStatusTimeoutDrain);
                    break;
                }
        }
    } else {
        // ------------------------------------------- transform + epilogue
        // Epilogue share: (lane quadrant, 16-channel group) pairs w and, for
        // warp 3, pair 15 (quadrant 3, channels 48-63).
        const int quad = warp & 3;
        const long long blk_tiles = kBlockTiles;
        c.row_stride = static_cast<long long>(p.w) * p.cin;
        auto epilogue = [&](int bl) -> bool {
            const uint32_t half = bl & 1;
            if (!mbar_wait_warp(c.bar(kBarDFull + half), (bl >> 1) & 1, c.abort, &g_status, kStatusTimeoutAccFull))
                return false;
            tc_fence_after();
            const int row = quad * 32 + c.lane;
            const int t = static_cast<int>((blockIdx.x + static_cast<long long>(bl) * gridDim.x) * blk_tiles) + row;
            const bool valid = row < kBlockTiles && t < p.n_tiles;
            for (int pr = warp; pr < 16; pr += 12) {  // warp 3: pairs 3 and 15
                const int grp = pr >> 2;
                if (16 * grp < p.cout)
                    store_block(p, t, valid, grp,
                                tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + 16u * grp + half * kDCols);
                if (warp != 3) break;
            }
            tc_fence_before();
            return true;
        };
        const int xt = threadIdx.x;  // 0 .. 479
        for (int r = 0; ok && r < rows; ++r) {
            const int u = r & 3;
            const int bl = r >> 2;
            c.r = r;
            c.u = u;
            if (u == 0) {
                const int blk = blockIdx.x + bl * gridDim.x;
                c.has[0] = make_item(p, blk, xt, c.it[0]);
                c.has[1] = make_item(p, blk, xt + kXThreads, c.it[1]);
            }
            ok = do_row<X16>(c);
            // the previous block's outputs, while this block's GEMMs run
            if (ok && u == 0 && bl > 0) ok = epilogue(bl - 1);
        }
        if (ok && rows > 0) ok = epilogue(n_mine - 1);
        if (!ok) *c.abort = 1u;
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

// ---------------------------------------------------------------------------
// TMA-fed variant (float16 input with 64 channels). A block is a rectangle
// of 8 x 15 Winograd tiles (16 x 30 output pixels) of one image; its whole
// input halo -- 18 rows x 32 columns x 64 channels, the top/left padding
// row and column included -- is ONE tensor-map copy into shared memory
// (72 KB), zero-filled where it leaves the image, so the transform needs no
// masks and reads its patches from shared memory instead of waiting on
// global loads. U is streamed per domain position from L2 through a ring of
// 4 blocks (one position of U is COUT x 128 B), which leaves room for the
// input box beside the 4 V tiles. The MMA-issuing thread also issues the
// copies: the next block's box as soon as every transform warp has written
// V(3, 0) of this block (after its last read of the box), and U of
// position P + 3 after position P's MMAs (into the slot of P - 1, whose
// MMAs have completed). Four epilogue warps (16-19, one per TMEM lane
// quadrant) add the bias and store each finished block while the transform
// warps go on with the next one (the output stores, issued by the transform
// warps, were the longest part of a block), then free the accumulator half
// for block b + 2. Issue order, accumulate flags and signs and the V tiles
// are those of winograd_f23_kernel.
constexpr int kTBlockTR = 8, kTBlockTC = 15;    // tiles per block: rows x columns (120)
constexpr int kTBoxW = 2 * kTBlockTC + 2;       // 32 input columns
constexpr int kTBoxH = 2 * kTBlockTR + 2;       // 18 input rows
constexpr uint32_t kTBoxBytes = 64u * 2u * kTBoxW * kTBoxH;  // 73,728
constexpr int kURing = 4;
constexpr int kTEpiWarp0 = 16;                 // epilogue warps 16-19
constexpr int kTWThreads = 20 * 32;

struct TmaParams {
    CUtensorMap tmap;       // x [N, H, W, 64] float16: dims {64, W, H, N}, box {64, 32, 18, 1}, no swizzle
    void* y;                // [N, H, W, COUT] float32 or float16
    const uint8_t* u_pack;  // 16 blocks of (COUT rows x 128 B), K-major SW128
    const float* bias;      // [COUT] or null
    int h, w, cout, y_f16;
    int tiles_h, tiles_w, blocks_h, blocks_w, n_blocks;
    uint32_t u_pos_bytes;   // COUT * 128: one position of U
    uint32_t off_v, off_u, off_bar;
    uint32_t idesc;
};

enum : int {
    kTBarXFull = 0,                 // the block's input box landed (TMA tx)
    kTBarAFull = 1,                 // + v: V tile v written (15 warp arrivals)
    kTBarAEmpty = 5,                // + v: the GEMMs reading V tile v are done (commit)
    kTBarUFull = 9,                 // + ring slot: U block landed (tx)
    kTBarUEmpty = 9 + kURing,       // + ring slot: the GEMMs reading it are done (commit)
    kTBarDFull = 9 + 2 * kURing,    // + half
    kTBarDrain = 11 + 2 * kURing,
    kTBarDEmpty = 12 + 2 * kURing,  // + half: the epilogue read it (4 warp arrivals)
    kTNumBars = 14 + 2 * kURing,
};
constexpr uint32_t kTBarBlockBytes = kTNumBars * 8 + 16;

__device__ __forceinline__ void tma_wino_block(const TmaParams& p, int blk, int& img, int& by, int& bx) {
    const int per_img = p.blocks_h * p.blocks_w;
    img = blk / per_img;
    const int rem = blk - img * per_img;
    by = rem / p.blocks_w;
    bx = rem - by * p.blocks_w;
}

// First pass of domain row u for both items of the thread, from the box:
// m = d_k0 + t_u * d_k1 per patch column (rows k0(u), k1(u) of the patch).
__device__ __forceinline__ void first_pass_smem(uint32_t box, const uint32_t (&poff)[2], int u,
                                                float (&m)[2][4][8]) {
    const int k0 = bt_k0(u), k1 = bt_k1(u);
    const float t = bt_t(u);
    const uint32_t o0 = static_cast<uint32_t>(k0 * kTBoxW * 128), o1 = static_cast<uint32_t>(k1 * kTBoxW * 128);
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int col = 0; col < 4; ++col) {
            uint4 qa, qb;
            asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(qa.x), "=r"(qa.y), "=r"(qa.z), "=r"(qa.w)
                         : "r"(box + poff[i] + o0 + col * 128u));
            asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(qb.x), "=r"(qb.y), "=r"(qb.z), "=r"(qb.w)
                         : "r"(box + poff[i] + o1 + col * 128u));
            float a[8], b[8];
            h8_to_f32(qa, a);
            h8_to_f32(qb, b);
#pragma unroll
            for (int e = 0; e < 8; ++e) m[i][col][e] = fmaf(t, b[e], a[e]);
        }
}

// D_ij + bias of this lane's tile (block row `row` < 120) for 16 channels
// of group grp: the 4 output positions of the 2x2 tile.
__device__ __forceinline__ void store_block_tma(const TmaParams& p, int img, int by, int bx, int row, int grp,
                                                uint32_t td) {
    const bool in_block = row < kTBlockTR * kTBlockTC;
    const int ty = by * kTBlockTR + (in_block ? row / kTBlockTC : 0);
    const int tx = bx * kTBlockTC + (in_block ? row % kTBlockTC : 0);
    float b[16];
#pragma unroll
    for (int c = 0; c < 16; ++c) b[c] = p.bias ? __ldg(p.bias + 16 * grp + c) : 0.0f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint32_t r[16];
        tmem_ld16(td + static_cast<uint32_t>(q * kMaxChannels), r);
        tmem_wait_ld(r);
        const int oh = 2 * ty + (q >> 1), ow = 2 * tx + (q & 1);
        if (!in_block || oh >= p.h || ow >= p.w) continue;
        const long long o = ((static_cast<long long>(img) * p.h + oh) * p.w + ow) * p.cout + 16 * grp;
        float y[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) y[c] = __uint_as_float(r[c]) + b[c];
        if (!p.y_f16) {
            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.y) + o);
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4)
                dst[c4] = make_float4(y[4 * c4], y[4 * c4 + 1], y[4 * c4 + 2], y[4 * c4 + 3]);
        } else {
            uint32_t pk[8];
#pragma unroll
            for (int c = 0; c < 16; c += 2) pk[c >> 1] = pack_f16x2(y[c], y[c + 1]);
            uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(p.y) + o);
            dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
    }
}

__global__ void __launch_bounds__(kTWThreads, 1) winograd_f23_tma_kernel(const __grid_constant__ TmaParams p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_addr(smem_raw);
    const uint32_t base = (raw_addr + 1023u) & ~1023u;
    uint8_t* const base_ptr = smem_raw + (base - raw_addr);
    const uint32_t box = base;  // the input box at offset 0
    const uint32_t v_base = base + p.off_v;
    const uint32_t u_base = base + p.off_u;
    const uint32_t bar_base = base + p.off_bar;
    auto bar = [&](int i) -> uint32_t { return bar_base + 8u * static_cast<uint32_t>(i); };
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base_ptr + p.off_bar + kTNumBars * 8);
    volatile uint32_t* abort = reinterpret_cast<volatile uint32_t*>(base_ptr + p.off_bar + kTNumBars * 8 + 4);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        mbar_init(bar(kTBarXFull), 1);
        for (int v = 0; v < 4; ++v) {
            mbar_init(bar(kTBarAFull + v), kXWarps);
            mbar_init(bar(kTBarAEmpty + v), 1);
        }
        for (int q = 0; q < kURing; ++q) {
            mbar_init(bar(kTBarUFull + q), 1);
            mbar_init(bar(kTBarUEmpty + q), 1);
        }
        mbar_init(bar(kTBarDFull), 1);
        mbar_init(bar(kTBarDFull + 1), 1);
        mbar_init(bar(kTBarDEmpty), 4);
        mbar_init(bar(kTBarDEmpty + 1), 4);
        mbar_init(bar(kTBarDrain), 1);
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
    bool ok = true;

    if (warp == kIssueWarp) {
        // ------------------------------------ MMA issuer and copy producer
        if (lane == 0) {
            const int n_pos = 16 * n_mine;
            int x_issued = 0, u_issued = 0;  // copies started (input boxes, U blocks)
            auto load_box = [&](int bl) {
                int img, by, bx;
                tma_wino_block(p, static_cast<int>(blockIdx.x) + bl * static_cast<int>(gridDim.x), img, by, bx);
                mbar_arrive_expect_tx(bar(kTBarXFull), kTBoxBytes);
                tma_load_4d(box, &p.tmap, 0, 2 * kTBlockTC * bx - 1, 2 * kTBlockTR * by - 1, img, bar(kTBarXFull));
                ++x_issued;
            };
            auto load_u = [&](int pos) {
                const int q = pos % kURing;
                mbar_arrive_expect_tx(bar(kTBarUFull + q), p.u_pos_bytes);
                bulk_g2s(u_base + static_cast<uint32_t>(q) * p.u_pos_bytes, p.u_pack + (pos % 16) * p.u_pos_bytes,
                         p.u_pos_bytes, bar(kTBarUFull + q));
                ++u_issued;
            };
            if (n_mine > 0) load_box(0);
            for (int pos = 0; pos < 3 && pos < n_pos; ++pos) load_u(pos);
            const uint64_t v_desc0 = umma_desc_sw128(v_base);
            const uint64_t u_desc0 = umma_desc_sw128(u_base);
            const uint64_t u_step = static_cast<uint64_t>(p.u_pos_bytes >> 4);
            const uint32_t ksteps = 4;  // CIN = 64
            uint64_t a_desc[4];
#pragma unroll
            for (int v = 0; v < 4; ++v) a_desc[v] = v_desc0 + static_cast<uint64_t>(v) * (kATileBytes >> 4);
            // Unrolled over the domain rows, like winograd_f23_kernel: every
            // MMA's accumulate flag and sign is a compile-time constant.
            for (int bl = 0; ok && bl < n_mine; ++bl) {
                const uint32_t d_base = tmem_base + (bl & 1) * kDCols;
                // the accumulator half was read out by the epilogue of block bl - 2
                if (bl >= 2 && !mbar_wait(bar(kTBarDEmpty + (bl & 1)), ((bl >> 1) - 1) & 1, abort, &g_status,
                                          kStatusTimeoutOther)) {
                    ok = false;
                    break;
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int r = bl * 4 + u;
                    if (!ok) break;
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        const int pos = r * 4 + v;
                        if (!mbar_wait(bar(kTBarAFull + v), r & 1, abort, &g_status, kStatusTimeoutAFull)) {
                            ok = false;
                            break;
                        }
                        // every transform warp has written V(3, 0): none reads the box again
                        if (u == 3 && v == 0 && bl + 1 < n_mine) load_box(bl + 1);
                        const int q = pos % kURing;
                        if (!mbar_wait(bar(kTBarUFull + q), (pos / kURing) & 1, abort, &g_status,
                                       kStatusTimeoutWFull)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        issue_position(u, v, d_base, a_desc[v], u_desc0 + static_cast<uint64_t>(q) * u_step, p.idesc,
                                       ksteps);
                        umma_commit(bar(kTBarAEmpty + v));  // V tile v may be rewritten
                        umma_commit(bar(kTBarUEmpty + q));  // U slot q may be reloaded
                        if (u == 3 && v == 3) umma_commit(bar(kTBarDFull + (bl & 1)));
                        // U of position pos + 3 into the slot of pos - 1 once its GEMMs are done
                        if (pos + 3 < n_pos) {
                            if (pos >= 1 && !mbar_wait(bar(kTBarUEmpty + (pos - 1) % kURing), ((pos - 1) / kURing) & 1,
                                                       abort, &g_status, kStatusTimeoutOther)) {
                                ok = false;
                                break;
                            }
                            load_u(pos + 3);
                        }
                    }
                }
            }
            if (!ok) *abort = 1u;
            // every issued MMA completes before TMEM is released, every copy
            // lands before the CTA exits
            umma_commit(bar(kTBarDrain));
            drain_wait(bar(kTBarDrain), 0u);
            if (x_issued > 0) drain_wait(bar(kTBarXFull), (x_issued - 1) & 1);
            for (int k = (u_issued > kURing ? u_issued - kURing : 0); k < u_issued; ++k)
                drain_wait(bar(kTBarUFull + k % kURing), (k / kURing) & 1);
        }
    } else if (warp >= kTEpiWarp0) {
        // -------------------------------------------------------- epilogue
        // Warp (16 + q) owns TMEM lane quadrant q: tiles 32 q .. 32 q + 31 of
        // the block, every 16-channel group; then frees the half.
        const int quad = warp & 3;
        const int row = quad * 32 + lane;
        for (int bl = 0; ok && bl < n_mine; ++bl) {
            const uint32_t half = bl & 1;
            if (!mbar_wait_warp(bar(kTBarDFull + half), (bl >> 1) & 1, abort, &g_status, kStatusTimeoutAccFull)) {
                ok = false;
                break;
            }
            tc_fence_after();
            int img, by, bx;
            tma_wino_block(p, static_cast<int>(blockIdx.x) + bl * static_cast<int>(gridDim.x), img, by, bx);
            for (int grp = 0; 16 * grp < p.cout; ++grp)
                store_block_tma(p, img, by, bx, row, grp,
                                tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + 16u * grp + half * kDCols);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kTBarDEmpty + half));
        }
        if (!ok) *abort = 1u;
    } else {
        // -------------------------------------------------------- transform
        // this thread's two (tile, 8-channel chunk) items: byte offset of the
        // patch's (row 0, col 0) in the box, and of the tile row in a V tile
        const int xt = threadIdx.x;  // 0 .. 479
        uint32_t poff[2], soff[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int idx = xt + i * kXThreads;
            const int tr = idx >> 3, ck = idx & 7;  // block tile 0..119, channel chunk
            const int trow = tr / kTBlockTC, tcol = tr - trow * kTBlockTC;
            poff[i] = static_cast<uint32_t>(((2 * trow) * kTBoxW + 2 * tcol) * 128 + ck * 16);
            soff[i] = sw128_offset(static_cast<uint32_t>(tr), static_cast<uint32_t>(ck * 8), kTileM);
        }
        RowCtx c;
        c.p = nullptr;
        c.has[0] = c.has[1] = true;
        c.it[0].soff = soff[0];
        c.it[1].soff = soff[1];
        c.a_base = v_base;
        c.bar_base = bar_base;
        c.abort = abort;
        c.lane = lane;
        for (int bl = 0; ok && bl < n_mine; ++bl) {
            // the block's input box
            if (!mbar_wait_warp(bar(kTBarXFull), bl & 1, abort, &g_status, kStatusTimeoutXFull)) {
                ok = false;
                break;
            }
            for (int u = 0; ok && u < 4; ++u) {
                c.r = bl * 4 + u;
                c.u = u;
                float m[2][4][8];
                first_pass_smem(box, poff, u, m);
                ok = do_position<0>(c, m) && do_position<1>(c, m) && do_position<2>(c, m) && do_position<3>(c, m);
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

// U = G g G^T per (cin, cout) filter in fp32 -- G g first, then (G g) G^T,
// each a left-to-right sum of exact products (G holds 0, 1/2 and 1), as the
// reference's torch expression computes it (nn.py:533-538) -- staged float16.
// Written as the reference's flat [16][CIN][COUT] array (u_plain, optional)
// and as 16 K-major SW128 operand blocks of COUT rows (u_pack, optional).
__global__ void winograd_f23_filter_kernel(const float* __restrict__ w33io, int cin, int cout,
                                           __half* __restrict__ u_plain, uint8_t* __restrict__ u_pack) {
    const int total = cin * cout;
    for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += gridDim.x * blockDim.x) {
        const int ci = idx / cout, co = idx - ci * cout;
        float g[3][3];
#pragma unroll
        for (int kh = 0; kh < 3; ++kh)
#pragma unroll
            for (int kw = 0; kw < 3; ++kw) g[kh][kw] = w33io[((kh * 3 + kw) * cin + ci) * cout + co];
        constexpr float G[4][3] = {{1.0f, 0.0f, 0.0f}, {0.5f, 0.5f, 0.5f}, {0.5f, -0.5f, 0.5f}, {0.0f, 0.0f, 1.0f}};
        float t[4][3];
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int c = 0; c < 3; ++c)
                t[a][c] = __fadd_rn(__fadd_rn(__fmul_rn(G[a][0], g[0][c]), __fmul_rn(G[a][1], g[1][c])),
                                    __fmul_rn(G[a][2], g[2][c]));
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const float uv = __fadd_rn(__fadd_rn(__fmul_rn(t[a][0], G[b][0]), __fmul_rn(t[a][1], G[b][1])),
                                           __fmul_rn(t[a][2], G[b][2]));
                const int pos = a * 4 + b;
                const __half hv = __float2half_rn(uv);
                if (u_plain) u_plain[(static_cast<size_t>(pos) * cin + ci) * cout + co] = hv;
                if (u_pack)
                    *reinterpret_cast<__half*>(u_pack + static_cast<size_t>(pos) * cout * 128 +
                                               sw128_offset(co, ci, cout)) = hv;
            }
    }
}

// Operand staging of the direct convolution: 0 exact fp32, 1 float16,
// 2 bfloat16 (round to nearest even, value kept in fp32).
template <int MATH>
__device__ __forceinline__ float conv_stage(float v) {
    if constexpr (MATH == 1) return __half2float(__float2half_rn(v));
    if constexpr (MATH == 2) return __bfloat162float(__float2bfloat16_rn(v));
    return v;
}

// 'Same' (zero padding KH/2, KW/2), stride-1 direct convolution: acc over
// (kh, kw, cin) in that order, one fused multiply-add per tap, fp32
// accumulation. MATH 0 is Conv2DTensorOp's exact fp32 arithmetic (acc =
// bias first, rdv/shaders/tensors/conv2d_tensor_op.h:21-87); MATH 1 / 2
// round x and w to float16 / bfloat16 first (products exact in fp32), the
// reference's tensor-core conv ops: bias seeding the accumulator
// (BIAS_FIRST: Conv2DTensorOpSimple, Simple3x3, Window3x3 --
// conv2d_tensor_op_simple.h:108-117, conv2d_tensor_op_simple3x3.h:98-102,
// conv2d_tensor_op_window3x3.h:160-165) or added after the sum
// (Conv2DTensorOpFast, conv2d_tensor_op_fast.h:100-104).
// One thread per (pixel, 8 output channels). x float32 or float16.
template <bool X16, int MATH, bool BIAS_FIRST>
__global__ void conv2d_direct_kernel(const void* __restrict__ x, const float* __restrict__ wt,
                                     const float* __restrict__ bias, float* __restrict__ y, int n, int h, int w,
                                     int cin, int cout, int kh_n, int kw_n) {
    const int chunks = cout >> 3;
    const long long total = static_cast<long long>(n) * h * w * chunks;
    for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long pix = idx / chunks;
        const int c0 = static_cast<int>(idx - pix * chunks) * 8;
        const int ow = static_cast<int>(pix % w);
        const long long t = pix / w;
        const int oh = static_cast<int>(t % h);
        const long long img = t / h;
        float acc[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[c] = (bias && BIAS_FIRST) ? bias[c0 + c] : 0.0f;
        for (int kh = 0; kh < kh_n; ++kh) {
            const int ih = oh + kh - kh_n / 2;
            if (ih < 0 || ih >= h) continue;
            for (int kw = 0; kw < kw_n; ++kw) {
                const int iw = ow + kw - kw_n / 2;
                if (iw < 0 || iw >= w) continue;
                const long long xin = ((img * h + ih) * w + iw) * cin;
                const float* wk = wt + static_cast<long long>(kh * kw_n + kw) * cin * cout + c0;
                for (int k = 0; k < cin; ++k) {
                    const float xv = conv_stage<MATH>(X16 ? __half2float(static_cast<const __half*>(x)[xin + k])
                                                          : static_cast<const float*>(x)[xin + k]);
                    const float4 wa = __ldg(reinterpret_cast<const float4*>(wk + static_cast<long long>(k) * cout));
                    const float4 wb =
                        __ldg(reinterpret_cast<const float4*>(wk + static_cast<long long>(k) * cout + 4));
                    acc[0] = fmaf(xv, conv_stage<MATH>(wa.x), acc[0]);
                    acc[1] = fmaf(xv, conv_stage<MATH>(wa.y), acc[1]);
                    acc[2] = fmaf(xv, conv_stage<MATH>(wa.z), acc[2]);
                    acc[3] = fmaf(xv, conv_stage<MATH>(wa.w), acc[3]);
                    acc[4] = fmaf(xv, conv_stage<MATH>(wb.x), acc[4]);
                    acc[5] = fmaf(xv, conv_stage<MATH>(wb.y), acc[5]);
                    acc[6] = fmaf(xv, conv_stage<MATH>(wb.z), acc[6]);
                    acc[7] = fmaf(xv, conv_stage<MATH>(wb.w), acc[7]);
                }
            }
        }
        if (bias && !BIAS_FIRST) {
#pragma unroll
            for (int c = 0; c < 8; ++c) acc[c] += bias[c0 + c];
        }
        float4* dst = reinterpret_cast<float4*>(y + pix * cout + c0);
        dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
}

}  // namespace wino
}  // namespace rdvb
