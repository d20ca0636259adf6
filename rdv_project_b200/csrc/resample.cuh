// Resampling and concatenation tensor ops over flattened [H*W, C] fp32
// tensors (C a multiple of 8). Pure data movement: every thread moves
// 8 channels (two 16-byte loads / stores), grid-stride over the output.
//   downsample2x  out[oh, ow] = ((x[2oh, 2ow] + x[2oh, 2ow+1]) + x[2oh+1, 2ow])
//                               + x[2oh+1, 2ow+1], times 0.25 -- the
//                 reference's summation order
//                 (rdv/shaders/tensors/downsample2x_tensor_op.h:1-45)
//   upsample2x    out[oh, ow] = x[oh / 2, ow / 2]
//                 (rdv/shaders/tensors/upsample2x_tensor_op.h:1-33)
//   concat        out[r] = x1[r] | x2[r] along channels
//                 (rdv/shaders/tensors/concat_tensor_op.h:1-35)
#pragma once
#include <cuda_runtime.h>

namespace rdvb {
namespace resample {

__device__ __forceinline__ void ld8(const float* p, float4& a, float4& b) {
    a = __ldg(reinterpret_cast<const float4*>(p));
    b = __ldg(reinterpret_cast<const float4*>(p) + 1);
}
__device__ __forceinline__ void st8(float* p, const float4& a, const float4& b) {
    reinterpret_cast<float4*>(p)[0] = a;
    reinterpret_cast<float4*>(p)[1] = b;
}
__device__ __forceinline__ float4 add4(const float4& a, const float4& b) {
    return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}
__device__ __forceinline__ float4 mul4(const float4& a, float s) { return make_float4(a.x * s, a.y * s, a.z * s, a.w * s); }

// x [h, w, c] -> y [h/2, w/2, c] (h, w even)
__global__ void downsample2x_kernel(const float* __restrict__ x, float* __restrict__ y, int h, int w, int c) {
    const int wo = w >> 1, ho = h >> 1, cb = c >> 3;
    const long long total = static_cast<long long>(ho) * wo * cb;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long orow = i / cb;
        const int c0 = static_cast<int>(i - orow * cb) * 8;
        const int oh = static_cast<int>(orow / wo), ow = static_cast<int>(orow - static_cast<long long>(oh) * wo);
        const long long r00 = (static_cast<long long>(2 * oh) * w + 2 * ow) * c + c0;
        const long long r10 = r00 + static_cast<long long>(w) * c;
        float4 a0, a1, b0, b1, c0v, c1v, d0, d1;
        ld8(x + r00, a0, a1);
        ld8(x + r00 + c, b0, b1);
        ld8(x + r10, c0v, c1v);
        ld8(x + r10 + c, d0, d1);
        st8(y + orow * c + c0, mul4(add4(add4(add4(a0, b0), c0v), d0), 0.25f),
            mul4(add4(add4(add4(a1, b1), c1v), d1), 0.25f));
    }
}

// x [h, w, c] -> y [2h, 2w, c]
__global__ void upsample2x_kernel(const float* __restrict__ x, float* __restrict__ y, int h, int w, int c) {
    const int wo = w * 2, cb = c >> 3;
    const long long total = static_cast<long long>(2 * h) * wo * cb;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long orow = i / cb;
        const int c0 = static_cast<int>(i - orow * cb) * 8;
        const int oh = static_cast<int>(orow / wo), ow = static_cast<int>(orow - static_cast<long long>(oh) * wo);
        float4 a, b;
        ld8(x + (static_cast<long long>(oh >> 1) * w + (ow >> 1)) * c + c0, a, b);
        st8(y + orow * c + c0, a, b);
    }
}

// x1 [rows, c1], x2 [rows, c2] -> y [rows, c1 + c2]
__global__ void concat_kernel(const float* __restrict__ x1, const float* __restrict__ x2, float* __restrict__ y,
                              long long rows, int c1, int c2) {
    const int co = c1 + c2, cb = co >> 3;
    const long long total = rows * cb;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long r = i / cb;
        const int cc = static_cast<int>(i - r * cb) * 8;
        float4 a, b;
        if (cc < c1) ld8(x1 + r * c1 + cc, a, b);
        else ld8(x2 + r * c2 + (cc - c1), a, b);
        st8(y + r * co + cc, a, b);
    }
}

}  // namespace resample
}  // namespace rdvb
