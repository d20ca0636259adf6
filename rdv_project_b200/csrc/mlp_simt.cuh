// MLP chain on the CUDA cores, one row per thread.
//
// Serves the chains the tensor-core kernel does not take:
//  * exact fp32 Linear layers (rdv/shaders/maps/linear.h:28-31):
//    acc = b[o]; acc += x[k] * W[o, k] for k ascending -- the same summation
//    order as the reference (each step an FFMA);
//  * LinearFast layers in a chain that mixes precisions, with float16 /
//    bfloat16 staging of x and W emulated on the CUDA cores, accumulation
//    from 0 and bias added after (linear_fast.h:61-98);
//  * the trailing partial 32-row workgroup of a LinearFast chain, which the
//    reference evaluates in exact fp32 (linear_fast.h:102-108).
// Weights are staged through shared memory 32 outputs at a time
// ([k][32] so a k step is 8 broadcast 16-byte loads); activations live in
// shared memory transposed ([feature][row]) so every access is
// bank-conflict free.
#pragma once
#include "ptx.cuh"

namespace rdvb {
namespace mlp_simt {

constexpr int kMaxLayers = 16;
constexpr int kRows = 64;   // rows (threads) per block
constexpr int kOch = 32;    // outputs per weight chunk
constexpr int kMaxWidth = 256;

struct Layer {
    const float* W;  // [N, K]
    const float* b;  // [N]
    int K, N;
    int math;        // 0 f32 exact, 1 f16 staging, 2 bf16 staging
    int relu;
};

struct Params {
    const void* x;
    int x_dtype;
    float* y;
    long long row_begin, row_end;
    int n_layers;
    int relu_in;
    int maxw;
    Layer layer[kMaxLayers];
};

__device__ __forceinline__ float stage_val(float v, int math) {
    if (math == 1) return __half2float(__float2half_rn(v));
    if (math == 2) return __bfloat162float(__float2bfloat16_rn(v));
    return v;
}

__global__ void __launch_bounds__(kRows) mlp_simt_kernel(const __grid_constant__ Params p) {
    extern __shared__ float sm[];
    float* act0 = sm;
    float* act1 = act0 + p.maxw * kRows;
    float* wch = act1 + p.maxw * kRows;  // [maxw][kOch]
    const int t = threadIdx.x;
    const long long row = p.row_begin + static_cast<long long>(blockIdx.x) * kRows + t;
    const bool valid = row < p.row_end;

    const int in0 = p.layer[0].K;
    for (int k = 0; k < in0; ++k) {
        float v = 0.0f;
        if (valid) {
            const long long i = row * in0 + k;
            if (p.x_dtype == 0) v = static_cast<const float*>(p.x)[i];
            else if (p.x_dtype == 1) v = __half2float(static_cast<const __half*>(p.x)[i]);
            else v = __bfloat162float(static_cast<const __nv_bfloat16*>(p.x)[i]);
            if (p.relu_in) v = fmaxf(v, 0.0f);
        }
        act0[k * kRows + t] = v;
    }

    float* ain = act0;
    float* aout = act1;
    for (int l = 0; l < p.n_layers; ++l) {
        const Layer L = p.layer[l];
        if (L.math != 0)
            for (int k = 0; k < L.K; ++k) ain[k * kRows + t] = stage_val(ain[k * kRows + t], L.math);
        for (int o0 = 0; o0 < L.N; o0 += kOch) {
            __syncthreads();
            for (int i = t; i < L.K * kOch; i += kRows) {
                const int k = i / kOch;
                const int j = i - k * kOch;
                const int o = o0 + j;
                float w = (o < L.N) ? L.W[static_cast<size_t>(o) * L.K + k] : 0.0f;
                wch[i] = stage_val(w, L.math);
            }
            __syncthreads();
            float acc[kOch];
#pragma unroll
            for (int j = 0; j < kOch; ++j)
                acc[j] = (L.math == 0 && o0 + j < L.N) ? L.b[o0 + j] : 0.0f;
            for (int k = 0; k < L.K; ++k) {
                const float a = ain[k * kRows + t];
                const float4* wr = reinterpret_cast<const float4*>(wch + k * kOch);
#pragma unroll
                for (int j4 = 0; j4 < kOch / 4; ++j4) {
                    const float4 w = wr[j4];
                    acc[4 * j4 + 0] = fmaf(a, w.x, acc[4 * j4 + 0]);
                    acc[4 * j4 + 1] = fmaf(a, w.y, acc[4 * j4 + 1]);
                    acc[4 * j4 + 2] = fmaf(a, w.z, acc[4 * j4 + 2]);
                    acc[4 * j4 + 3] = fmaf(a, w.w, acc[4 * j4 + 3]);
                }
            }
#pragma unroll
            for (int j = 0; j < kOch; ++j) {
                const int o = o0 + j;
                if (o < L.N) {
                    float v = acc[j];
                    if (L.math != 0) v += L.b[o];
                    if (L.relu) v = fmaxf(v, 0.0f);
                    aout[o * kRows + t] = v;
                }
            }
        }
        float* tmp = ain;
        ain = aout;
        aout = tmp;
    }
    if (valid) {
        const int outd = p.layer[p.n_layers - 1].N;
        float* yr = p.y + row * outd;
        for (int o = 0; o < outd; ++o) yr[o] = ain[o * kRows + t];
    }
}

// y = max(x, 0) over n floats (ReLUTensorOp, rdv/shaders/tensors/relu_tensor_op.h:3-22).
__global__ void relu_kernel(const float* __restrict__ x, float* __restrict__ y, long long n) {
    const long long n4 = n >> 2;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4; i += stride) {
        float4 v = reinterpret_cast<const float4*>(x)[i];
        v.x = fmaxf(v.x, 0.0f);
        v.y = fmaxf(v.y, 0.0f);
        v.z = fmaxf(v.z, 0.0f);
        v.w = fmaxf(v.w, 0.0f);
        reinterpret_cast<float4*>(y)[i] = v;
    }
    for (long long i = (n4 << 2) + blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n; i += stride)
        y[i] = fmaxf(x[i], 0.0f);
}

}  // namespace mlp_simt
}  // namespace rdvb
