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
// Precision: every operand stays fp32 -- U = G g G^T, V = B^T d B, the 36
// per-position CIN reductions and Y = A^T M A + bias. The float16 staging of
// U and V that F(2x2) uses is not accurate enough here: the larger entries
// of the 6x6 transforms amplify its rounding to about 1.3e-2 of the output
// at 64 channels (elementwise against the float64 direct convolution),
// above the 1e-2 float16 tolerance; fp32 operands give about 1e-6.
//
// Data layout: x NHWC [n, h, w, cin] fp32 or fp16; U [36][cin][cout] fp32
// (the packed operand is this plain array); y NHWC [n, h, w, cout] fp32 or
// fp16. Tile (ty, tx) of image b covers outputs rows 4 ty .. 4 ty + 3,
// columns 4 tx .. 4 tx + 3 and reads input rows 4 ty - 1 .. 4 ty + 4 (zero
// outside the image); partial tiles at the bottom/right edges store only
// their in-image outputs.
//
// winograd_f43_kernel<XF16, BT>: persistent CTAs of 512 threads walk blocks
// of BT tiles (8, or 4 when the channels need more shared memory), three
// phases per block separated by block barriers:
//   1. items (tile, ci): the 6x6 patch is loaded (consecutive threads read
//      consecutive channels) and transformed; V is written to shared memory
//      as [36][cin][BT tiles], so 16-byte loads give a (position, channel)'s
//      V for all BT tiles;
//   2. items (position q, output-channel pair): BT tiles x 2 channels of
//      fp32 accumulators over ascending ci -- per ci BT/4 16-byte V loads
//      and two U loads (coalesced over output channels, from L2) feed 2 BT
//      FMAs; M written to shared memory as [36][BT tiles][cout];
//   3. items (tile, co): the 36 M values, the inverse transform, bias and the
//      store (coalesced over co).
// Shared memory: 144 BT (cin + cout) bytes (147,456 at 64/64 channels with
// BT = 8, at 128/128 with BT = 4).
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

namespace rdvb {
namespace wino43 {

constexpr int kA = 6;             // transform size m + r - 1
constexpr int kM = 4;             // output tile size
constexpr int kPos = kA * kA;     // 36 transform positions
constexpr int kThreads = 512;
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
// (ci, co), fp32 arithmetic in the order (G g) G^T.
__global__ void winograd_f43_filter_kernel(const float* __restrict__ w, int cin, int cout, float* __restrict__ u) {
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
                u[(a * kA + b) * total + i] = v;
            }
    }
}

struct Params {
    const void* x;      // [n, h, w, cin]
    void* y;            // [n, h, w, cout]
    const float* u;     // [36][cin][cout]
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

// Shared-memory bytes of winograd_f43_kernel for (cin, cout) and BT tiles per block.
inline size_t smem_bytes(int cin, int cout, int bt) {
    return static_cast<size_t>(kPos) * bt * (static_cast<size_t>(cin) + cout) * sizeof(float);
}

template <bool XF16, int BT>
__global__ void __launch_bounds__(kThreads, 1) winograd_f43_kernel(const __grid_constant__ Params p) {
    static_assert(BT % 4 == 0, "V is read in 16-byte groups of 4 tiles");
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int cin = p.cin, cout = p.cout;
    float* vsm = reinterpret_cast<float*>(smem_raw);  // [36][cin][BT]
    float* msm = vsm + static_cast<size_t>(kPos) * cin * BT;  // [36][BT][cout]
    const int n_pairs = (cout + 1) / 2;
    for (long long t0 = static_cast<long long>(blockIdx.x) * BT; t0 < p.n_tiles;
         t0 += static_cast<long long>(gridDim.x) * BT) {
        // Phase 1: V = B^T d B of (tile, ci).
        for (int it = threadIdx.x; it < BT * cin; it += kThreads) {
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
            float* vt = vsm + static_cast<size_t>(ci) * BT + tl;
#pragma unroll
            for (int a = 0; a < kA; ++a)
#pragma unroll
                for (int b = 0; b < kA; ++b) {
                    float s = 0.0f;
#pragma unroll
                    for (int c = 0; c < kA; ++c)
                        if (kBT[b][c] != 0.0f) s = fmaf(t[a][c], kBT[b][c], s);
                    vt[static_cast<size_t>(a * kA + b) * cin * BT] = s;
                }
        }
        __syncthreads();
        // Phase 2: M[q][tile][co] = sum over ascending ci of V * U.
        for (int it = threadIdx.x; it < kPos * n_pairs; it += kThreads) {
            const int q = it / n_pairs, co = 2 * (it - q * n_pairs);
            const bool two = co + 1 < cout;
            float acc[BT][2];
#pragma unroll
            for (int t = 0; t < BT; ++t) acc[t][0] = acc[t][1] = 0.0f;
            const float4* vq = reinterpret_cast<const float4*>(vsm + static_cast<size_t>(q) * cin * BT);
            const float* uq = p.u + static_cast<size_t>(q) * cin * cout + co;
            for (int ci = 0; ci < cin; ++ci) {
                float4 vv[BT / 4];
#pragma unroll
                for (int g = 0; g < BT / 4; ++g) vv[g] = vq[ci * (BT / 4) + g];
                const float u0 = __ldg(uq + static_cast<size_t>(ci) * cout);
                const float u1 = two ? __ldg(uq + static_cast<size_t>(ci) * cout + 1) : 0.0f;
#pragma unroll
                for (int g = 0; g < BT / 4; ++g) {
                    const float f[4] = {vv[g].x, vv[g].y, vv[g].z, vv[g].w};
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        acc[4 * g + k][0] = fmaf(f[k], u0, acc[4 * g + k][0]);
                        acc[4 * g + k][1] = fmaf(f[k], u1, acc[4 * g + k][1]);
                    }
                }
            }
            float* mq = msm + static_cast<size_t>(q) * BT * cout + co;
#pragma unroll
            for (int t = 0; t < BT; ++t) {
                mq[static_cast<size_t>(t) * cout] = acc[t][0];
                if (two) mq[static_cast<size_t>(t) * cout + 1] = acc[t][1];
            }
        }
        __syncthreads();
        // Phase 3: Y = A^T M A + bias for (tile, co).
        for (int it = threadIdx.x; it < BT * cout; it += kThreads) {
            const int tl = it / cout, co = it - tl * cout;
            const long long tile = t0 + tl;
            if (tile >= p.n_tiles) continue;
            float m[kPos];
#pragma unroll
            for (int q = 0; q < kPos; ++q) m[q] = msm[(static_cast<size_t>(q) * BT + tl) * cout + co];
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
