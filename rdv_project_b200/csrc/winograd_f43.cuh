// Winograd F(4x4, 3x3) convolution on CUDA cores (a B200 extension; the
// reference operator Conv2DTensorOpWinograd3x3, rdv/domain/nn.py:1002-1087,
// is F(2x2, 3x3) only).
//
// Transform matrices: the Toom-Cook construction for F(4, 3) on the points
// {0, 1, -1, 2, -1/2, inf} (Lavin & Gray, arXiv:1509.09308, section 4). With
// float16 staging of U and V this point set keeps the error about 3x below
// the textbook {0, 1, -1, 2, -2, inf} (Barabasz et al., arXiv:1803.10986).
// A^T and B^T are exact in fp32; G is rounded to fp32.
//
// Precision recipe, as for F(2x2): U = G g G^T in fp32, stored float16;
// V = B^T d B in fp32, staged float16; the 36 per-position CIN reductions in
// fp32; Y = A^T M A in fp32, plus bias.
//
// Data layout: x NHWC [n, h, w, cin] fp32 or fp16; U [36][cin][cout] fp16
// (the packed operand is this plain array); y NHWC [n, h, w, cout] fp32 or
// fp16. Tile (ty, tx) of image b covers outputs rows 4 ty .. 4 ty + 3,
// columns 4 tx .. 4 tx + 3 and reads input rows 4 ty - 1 .. 4 ty + 4 (zero
// outside the image); partial tiles at the bottom/right edges store only
// their in-image outputs.
//
// winograd_f43_kernel: persistent CTAs of 256 threads walk blocks of 8
// tiles, three phases per block separated by block barriers:
//   1. items (tile, ci): the 6x6 patch is loaded (consecutive threads read
//      consecutive channels) and transformed; V is written float16 to shared
//      memory as [36][cin][8 tiles], so one 16-byte load gives a (position,
//      channel)'s V for all 8 tiles;
//   2. items (position q, output-channel pair): 8 tiles x 2 channels of fp32
//      accumulators over ascending ci -- per ci one 16-byte V load and two
//      float16 U loads (coalesced over output channels, from L2) feed 16
//      FMAs; M written to shared memory as [36][8 tiles][cout] fp32;
//   3. items (tile, co): the 36 M values, the inverse transform, bias and the
//      store (coalesced over co).
// Shared memory: 576 cin + 1152 cout bytes (221,184 at 128/128 channels).
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

namespace rdvb {
namespace wino43 {

constexpr int kA = 6;             // transform size m + r - 1
constexpr int kM = 4;             // output tile size
constexpr int kPos = kA * kA;     // 36 transform positions
constexpr int kBlockTiles = 8;    // tiles per block of a CTA (one 16-byte V load)
constexpr int kThreads = 256;
constexpr int kMaxChannels = 128;

__device__ constexpr float kBT[kA][kA] = {
    {1.0f, 1.5f, -2.0f, -1.5f, 1.0f, 0.0f},  {0.0f, -1.0f, -2.5f, -0.5f, 1.0f, 0.0f},
    {0.0f, 1.0f, 0.5f, -2.5f, 1.0f, 0.0f},   {0.0f, -0.5f, -1.0f, 0.5f, 1.0f, 0.0f},
    {0.0f, 2.0f, -1.0f, -2.0f, 1.0f, 0.0f},  {0.0f, 1.0f, 1.5f, -2.0f, -1.5f, 1.0f}};
__device__ constexpr float kAT[kM][kA] = {{1.0f, 1.0f, 1.0f, 1.0f, 1.0f, 0.0f},
                                          {0.0f, 1.0f, -1.0f, 2.0f, -0.5f, 0.0f},
                                          {0.0f, 1.0f, 1.0f, 4.0f, 0.25f, 0.0f},
                                          {0.0f, 1.0f, -1.0f, 8.0f, -0.125f, 1.0f}};
// G[j] = (f_j^0, f_j^1, f_j^2) / prod_{l != j} (f_j - f_l); last row the point at infinity
__device__ constexpr float kG[kA][3] = {{1.0f, 0.0f, 0.0f},
                                        {-1.0f / 3.0f, -1.0f / 3.0f, -1.0f / 3.0f},
                                        {1.0f / 3.0f, -1.0f / 3.0f, 1.0f / 3.0f},
                                        {1.0f / 15.0f, 2.0f / 15.0f, 4.0f / 15.0f},
                                        {-16.0f / 15.0f, 8.0f / 15.0f, -4.0f / 15.0f},
                                        {0.0f, 0.0f, 1.0f}};

// U[i][j][ci][co] = (G g G^T)[i][j], g[r][c] = w[r][c][ci][co]; one thread per
// (ci, co), fp32 arithmetic in the order (G g) G^T, float16 result.
__global__ void winograd_f43_filter_kernel(const float* __restrict__ w, int cin, int cout, __half* __restrict__ u) {
    const long long total = static_cast<long long>(cin) * cout;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        float g[3][3];
#pragma unroll
        for (int r = 0; r < 3; ++r)
#pragma unroll
            for (int c = 0; c < 3; ++c) g[r][c] = w[(r * 3 + c) * total + i];
        float t[kA][3];
#pragma unroll
        for (int a = 0; a < kA; ++a)
#pragma unroll
            for (int c = 0; c < 3; ++c)
                t[a][c] = __fadd_rn(__fadd_rn(__fmul_rn(kG[a][0], g[0][c]), __fmul_rn(kG[a][1], g[1][c])),
                                    __fmul_rn(kG[a][2], g[2][c]));
#pragma unroll
        for (int a = 0; a < kA; ++a)
#pragma unroll
            for (int b = 0; b < kA; ++b) {
                const float v = __fadd_rn(__fadd_rn(__fmul_rn(t[a][0], kG[b][0]), __fmul_rn(t[a][1], kG[b][1])),
                                          __fmul_rn(t[a][2], kG[b][2]));
                u[(a * kA + b) * total + i] = __float2half_rn(v);
            }
    }
}

struct Params {
    const void* x;      // [n, h, w, cin]
    void* y;            // [n, h, w, cout]
    const __half* u;    // [36][cin][cout]
    const float* bias;  // [cout] or null
    int h, w, cin, cout;
    int y_f16;
    int tiles_w, tiles_per_img;
    long long n_tiles;
};

template <bool XF16>
__device__ __forceinline__ float load_x(const void* x, long long i) {
    if constexpr (XF16) return __half2float(static_cast<const __half*>(x)[i]);
    else return static_cast<const float*>(x)[i];
}

// Shared-memory bytes of winograd_f43_kernel for (cin, cout).
inline size_t smem_bytes(int cin, int cout) {
    return static_cast<size_t>(kPos) * kBlockTiles * (static_cast<size_t>(cin) * sizeof(__half) +
                                                      static_cast<size_t>(cout) * sizeof(float));
}

template <bool XF16>
__global__ void __launch_bounds__(kThreads) winograd_f43_kernel(const __grid_constant__ Params p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int cin = p.cin, cout = p.cout;
    __half* vsm = reinterpret_cast<__half*>(smem_raw);  // [36][cin][kBlockTiles]
    float* msm = reinterpret_cast<float*>(smem_raw + static_cast<size_t>(kPos) * cin * kBlockTiles * sizeof(__half));
    const int n_pairs = (cout + 1) / 2;
    for (long long t0 = static_cast<long long>(blockIdx.x) * kBlockTiles; t0 < p.n_tiles;
         t0 += static_cast<long long>(gridDim.x) * kBlockTiles) {
        // Phase 1: V = B^T d B of (tile, ci), staged float16.
        for (int it = threadIdx.x; it < kBlockTiles * cin; it += kThreads) {
            const int tl = it / cin, ci = it - tl * cin;
            const long long tile = t0 + tl;
            float d[kA][kA];
            if (tile < p.n_tiles) {
                const long long img = tile / p.tiles_per_img;
                const int rem = static_cast<int>(tile - img * p.tiles_per_img);
                const int ty = rem / p.tiles_w, tx = rem - ty * p.tiles_w;
#pragma unroll
                for (int r = 0; r < kA; ++r) {
                    const int iy = ty * kM - 1 + r;
#pragma unroll
                    for (int c = 0; c < kA; ++c) {
                        const int ix = tx * kM - 1 + c;
                        d[r][c] = (iy >= 0 && iy < p.h && ix >= 0 && ix < p.w)
                                      ? load_x<XF16>(p.x, ((img * p.h + iy) * p.w + ix) * cin + ci)
                                      : 0.0f;
                    }
                }
            } else {
#pragma unroll
                for (int r = 0; r < kA; ++r)
#pragma unroll
                    for (int c = 0; c < kA; ++c) d[r][c] = 0.0f;
            }
            float t[kA][kA];  // B^T d
#pragma unroll
            for (int a = 0; a < kA; ++a)
#pragma unroll
                for (int c = 0; c < kA; ++c) {
                    float s = 0.0f;
#pragma unroll
                    for (int r = 0; r < kA; ++r)
                        if (kBT[a][r] != 0.0f) s = fmaf(kBT[a][r], d[r][c], s);
                    t[a][c] = s;
                }
            __half* vt = vsm + static_cast<size_t>(ci) * kBlockTiles + tl;
#pragma unroll
            for (int a = 0; a < kA; ++a)
#pragma unroll
                for (int b = 0; b < kA; ++b) {
                    float s = 0.0f;
#pragma unroll
                    for (int c = 0; c < kA; ++c)
                        if (kBT[b][c] != 0.0f) s = fmaf(t[a][c], kBT[b][c], s);
                    vt[static_cast<size_t>(a * kA + b) * cin * kBlockTiles] = __float2half_rn(s);
                }
        }
        __syncthreads();
        // Phase 2: M[q][tile][co] = sum over ascending ci of V * U.
        for (int it = threadIdx.x; it < kPos * n_pairs; it += kThreads) {
            const int q = it / n_pairs, co = 2 * (it - q * n_pairs);
            const bool two = co + 1 < cout;
            float acc[kBlockTiles][2];
#pragma unroll
            for (int t = 0; t < kBlockTiles; ++t) acc[t][0] = acc[t][1] = 0.0f;
            const uint4* vq = reinterpret_cast<const uint4*>(vsm + static_cast<size_t>(q) * cin * kBlockTiles);
            const __half* uq = p.u + static_cast<size_t>(q) * cin * cout + co;
            for (int ci = 0; ci < cin; ++ci) {
                const uint4 vv = vq[ci];
                const float u0 = __half2float(uq[static_cast<size_t>(ci) * cout]);
                const float u1 = two ? __half2float(uq[static_cast<size_t>(ci) * cout + 1]) : 0.0f;
                const __half2* vh = reinterpret_cast<const __half2*>(&vv);
#pragma unroll
                for (int t2 = 0; t2 < kBlockTiles / 2; ++t2) {
                    const float2 f = __half22float2(vh[t2]);
                    acc[2 * t2][0] = fmaf(f.x, u0, acc[2 * t2][0]);
                    acc[2 * t2][1] = fmaf(f.x, u1, acc[2 * t2][1]);
                    acc[2 * t2 + 1][0] = fmaf(f.y, u0, acc[2 * t2 + 1][0]);
                    acc[2 * t2 + 1][1] = fmaf(f.y, u1, acc[2 * t2 + 1][1]);
                }
            }
            float* mq = msm + static_cast<size_t>(q) * kBlockTiles * cout + co;
#pragma unroll
            for (int t = 0; t < kBlockTiles; ++t) {
                mq[static_cast<size_t>(t) * cout] = acc[t][0];
                if (two) mq[static_cast<size_t>(t) * cout + 1] = acc[t][1];
            }
        }
        __syncthreads();
        // Phase 3: Y = A^T M A + bias for (tile, co).
        for (int it = threadIdx.x; it < kBlockTiles * cout; it += kThreads) {
            const int tl = it / cout, co = it - tl * cout;
            const long long tile = t0 + tl;
            if (tile >= p.n_tiles) continue;
            float m[kPos];
#pragma unroll
            for (int q = 0; q < kPos; ++q) m[q] = msm[(static_cast<size_t>(q) * kBlockTiles + tl) * cout + co];
            float s[kM][kA];  // A^T M
#pragma unroll
            for (int i = 0; i < kM; ++i)
#pragma unroll
                for (int b = 0; b < kA; ++b) {
                    float acc = 0.0f;
#pragma unroll
                    for (int a = 0; a < kA; ++a)
                        if (kAT[i][a] != 0.0f) acc = fmaf(kAT[i][a], m[a * kA + b], acc);
                    s[i][b] = acc;
                }
            const float bv = p.bias ? p.bias[co] : 0.0f;
            const long long img = tile / p.tiles_per_img;
            const int rem = static_cast<int>(tile - img * p.tiles_per_img);
            const int ty = rem / p.tiles_w, tx = rem - ty * p.tiles_w;
#pragma unroll
            for (int i = 0; i < kM; ++i) {
                const int oy = ty * kM + i;
                if (oy >= p.h) continue;
#pragma unroll
                for (int j = 0; j < kM; ++j) {
                    const int ox = tx * kM + j;
                    if (ox >= p.w) continue;
                    float acc = 0.0f;
#pragma unroll
                    for (int b = 0; b < kA; ++b)
                        if (kAT[j][b] != 0.0f) acc = fmaf(s[i][b], kAT[j][b], acc);
                    const float v = acc + bv;
                    const long long o = ((img * p.h + oy) * p.w + ox) * cout + co;
                    if (p.y_f16) static_cast<__half*>(p.y)[o] = __float2half_rn(v);
                    else static_cast<float*>(p.y)[o] = v;
                }
            }
        }
        __syncthreads();
    }
}

}  // namespace wino43
}  // namespace rdvb
