// TensorSampler (rdv/maths/__init__.py:2050-2083,
// rdv/shaders/samplers/tensor_sampler.h): multilinear or nearest lookup of a
// dense fp32 tensor t [D0, ..., D(IN-1), OUT] at points x in [-1, 1]^IN.
// Dimension i of t is addressed by coordinate x[IN-1-i] (the last
// coordinate runs along the first dimension, as torch's grid_sample).
//   index_f = (x * (D - a) + D) * 0.5 - 0.5   (a = 1 when aligned: -1/+1 at
//             the first/last cell centres; a = 0: at the outer edges)
//   lo = floor(index_f), hi = lo + 1, alpha = index_f - lo
//   linear:  corner weights (1 - alpha, alpha) per dimension, the innermost
//            pair blended as mix(left, right, alpha) = left (1 - alpha) +
//            right alpha, times the product of the outer weights, added in
//            the reference's corner order; a corner outside the tensor
//            contributes 0 unless clamp (then its index is clamped)
//   nearest: lo + (alpha >= 0.5); outside -> 0 unless clamp.
// One thread per (point, channel); every product and sum is rounded
// separately, in the reference's order.
#pragma once
#include <cuda_runtime.h>

namespace rdvb {
namespace sampler {

struct Params {
    const float* t;
    const float* x;   // [n, IN]
    float* y;         // [n, OUT]
    long long n;
    int out;
    int dim[3];
    int clamp, aligned, linear;
};

__device__ __forceinline__ float mixf(float a, float b, float t) {
    return __fadd_rn(__fmul_rn(a, __fsub_rn(1.0f, t)), __fmul_rn(b, t));
}

// dst += rest * blend of the pair (left, right) at offset `off` and `off + d`
// along the innermost dimension, with the inside flags of both corners.
__device__ __forceinline__ float blend_pair(const float* __restrict__ t, long long off, long long d, bool left_in,
                                            bool right_in, float xw, float rest, float dst) {
    if (!left_in && !right_in) return dst;
    const float l = __ldg(t + off), r = __ldg(t + off + d);
    if (left_in && right_in) return __fadd_rn(dst, __fmul_rn(rest, mixf(l, r, xw)));
    if (left_in) return __fadd_rn(dst, __fmul_rn(__fmul_rn(rest, __fsub_rn(1.0f, xw)), l));
    return __fadd_rn(dst, __fmul_rn(__fmul_rn(rest, xw), r));
}

__device__ __forceinline__ void coord(float xc, int dim, float ac, bool border, int& lo, int& clo, int& chi,
                                      float& alpha, bool& lo_in, bool& hi_in) {
    const float g = static_cast<float>(dim);
    const float index_f = __fsub_rn(__fmul_rn(__fadd_rn(__fmul_rn(xc, __fsub_rn(g, ac)), g), 0.5f), 0.5f);
    lo = static_cast<int>(floorf(index_f));
    const int hi = lo + 1;
    alpha = __fsub_rn(index_f, static_cast<float>(lo));
    lo_in = border || (lo >= 0 && lo < dim);
    hi_in = border || (hi >= 0 && hi < dim);
    clo = min(max(lo, 0), dim - 1);
    chi = min(max(hi, 0), dim - 1);
}

// Channel k of a 2-D lookup into t [dim0, dim1, out] at (x0, x1) (x1 runs
// along dim0), with the kernel's arithmetic: the IN = 2 case of
// tensor_sampler_kernel, and the environment lookup of an equirectangular
// image (XRProject >> TensorSampler) in the PBVR kernel.
__device__ __forceinline__ float sample2(const float* __restrict__ t, int dim0, int dim1, int out, int k, float x0,
                                         float x1, bool border, bool aligned, bool linear) {
    const float ac = aligned ? 1.0f : 0.0f;
    int lo[2], clo[2], chi[2];
    float alpha[2];
    bool lo_in[2], hi_in[2];
    coord(x1, dim0, ac, border, lo[0], clo[0], chi[0], alpha[0], lo_in[0], hi_in[0]);
    coord(x0, dim1, ac, border, lo[1], clo[1], chi[1], alpha[1], lo_in[1], hi_in[1]);
    const long long st0 = static_cast<long long>(out) * dim1, st1 = out;
    if (!linear) {
        bool inside = true;
        long long off = k;
        const int dims[2] = {dim0, dim1};
        const long long st[2] = {st0, st1};
#pragma unroll
        for (int d = 0; d < 2; ++d) {
            int id = lo[d] + (alpha[d] >= 0.5f ? 1 : 0);
            inside = inside && id >= 0 && id < dims[d];
            id = min(max(id, 0), dims[d] - 1);
            off += id * st[d];
        }
        return (border || inside) ? __ldg(t + off) : 0.0f;
    }
    const long long dl = static_cast<long long>(chi[1] - clo[1]) * st1;
    const long long base = clo[0] * st0 + clo[1] * st1 + k;
    const long long d0 = static_cast<long long>(chi[0] - clo[0]) * st0;
    float v = 0.0f;
    v = blend_pair(t, base, dl, lo_in[0] && lo_in[1], lo_in[0] && hi_in[1], alpha[1], __fsub_rn(1.0f, alpha[0]), v);
    v = blend_pair(t, base + d0, dl, hi_in[0] && lo_in[1], hi_in[0] && hi_in[1], alpha[1], alpha[0], v);
    return v;
}

// Channel k of the TensorSampler at the point x (x[0] the first
// coordinate, addressing the last dimension), t [dim[0], ..., dim[IN-1], out].
template <int IN>
__device__ __forceinline__ float tensor_sample(const float* __restrict__ t, const int* dim, int out, int k,
                                               const float* x, bool border, bool aligned, bool linear) {
    if constexpr (IN == 2) {
        return sample2(t, dim[0], dim[1], out, k, x[0], x[1], border, aligned, linear);
    } else {
    const float ac = aligned ? 1.0f : 0.0f;
    int lo[IN], clo[IN], chi[IN];
    float alpha[IN];
    bool lo_in[IN], hi_in[IN];
#pragma unroll
    for (int d = 0; d < IN; ++d)
        coord(x[IN - 1 - d], dim[d], ac, border, lo[d], clo[d], chi[d], alpha[d], lo_in[d], hi_in[d]);
    // element strides of the spatial dimensions
    long long st[IN];
    st[IN - 1] = out;
#pragma unroll
    for (int d = IN - 2; d >= 0; --d) st[d] = st[d + 1] * dim[d + 1];
    float v = 0.0f;
    if (!linear) {
        bool inside = true;
        long long off = k;
#pragma unroll
        for (int d = 0; d < IN; ++d) {
            int id = lo[d] + (alpha[d] >= 0.5f ? 1 : 0);
            inside = inside && id >= 0 && id < dim[d];
            id = min(max(id, 0), dim[d] - 1);
            off += id * st[d];
        }
        return (border || inside) ? __ldg(t + off) : 0.0f;
    }
    const int L = IN - 1;  // innermost (fastest) dimension
    const long long dl = static_cast<long long>(chi[L] - clo[L]) * st[L];
    if constexpr (IN == 1) {
        v = blend_pair(t, clo[0] * st[0] + k, dl, lo_in[0], hi_in[0], alpha[0], 1.0f, v);
    } else {
        long long ptr = clo[0] * st[0] + clo[1] * st[1] + clo[2] * st[2] + k;
        const long long d0 = static_cast<long long>(chi[0] - clo[0]) * st[0];
        const long long d1 = static_cast<long long>(chi[1] - clo[1]) * st[1];
        const float a0 = alpha[0], a1 = alpha[1];
        v = blend_pair(t, ptr, dl, lo_in[0] && lo_in[1] && lo_in[2], lo_in[0] && lo_in[1] && hi_in[2], alpha[2],
                       __fmul_rn(__fsub_rn(1.0f, a0), __fsub_rn(1.0f, a1)), v);
        ptr += d1;
        v = blend_pair(t, ptr, dl, lo_in[0] && hi_in[1] && lo_in[2], lo_in[0] && hi_in[1] && hi_in[2], alpha[2],
                       __fmul_rn(__fsub_rn(1.0f, a0), a1), v);
        ptr += d0;
        v = blend_pair(t, ptr, dl, hi_in[0] && hi_in[1] && lo_in[2], hi_in[0] && hi_in[1] && hi_in[2], alpha[2],
                       __fmul_rn(a0, a1), v);
        ptr -= d1;
        v = blend_pair(t, ptr, dl, hi_in[0] && lo_in[1] && lo_in[2], hi_in[0] && lo_in[1] && hi_in[2], alpha[2],
                       __fmul_rn(a0, __fsub_rn(1.0f, a1)), v);
    }
    return v;
    }
}

template <int IN>
__global__ void tensor_sampler_kernel(const __grid_constant__ Params p) {
    const long long total = p.n * p.out;
    const bool border = p.clamp != 0;
    for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long i = idx / p.out;
        const int k = static_cast<int>(idx - i * p.out);
        float x[IN];
#pragma unroll
        for (int d = 0; d < IN; ++d) x[d] = __ldg(p.x + i * IN + d);
        p.y[idx] = tensor_sample<IN>(p.t, p.dim, p.out, k, x, border, p.aligned != 0, p.linear != 0);
    }
}

// GridSampler (rdv/maths/__init__.py:2018-2047, rdv/shaders/samplers/
// grid_sampler.h) over a dense grid (a TensorGrid, grids/tensor_grid.h:
// row-major [D0, ..., D(IN-1), OUT]). Its arithmetic differs from the
// TensorSampler's: per dimension i (coordinate x[IN-1-i])
//   t = x * 0.5 + 0.5
//   pos = aligned ? t * (D - 1) : t * D - 0.5
//   voxel = floor(pos), alpha = pos - voxel
// linear: the 2^IN corners in the order of their bit masks (bit i: +1 along
// dimension i), each weighted by the product, over i ascending and starting
// from 1, of alpha_i or 1 - alpha_i, accumulated as out += w * value; a
// corner outside the grid is skipped unless clamp (then clamped).
// nearest: voxel + (alpha >= 0.5), skipped outside unless clamp.
struct GridParams {
    const float* t;
    const float* x;   // [n, IN]
    float* y;         // [n, OUT]
    long long n;
    int out;
    int dim[4];
    int clamp, aligned, linear;
};

// Channel k of the GridSampler at the point x (x[0] the first coordinate,
// addressing the last dimension), t [dim[0], ..., dim[IN-1], out].
template <int IN>
__device__ __forceinline__ float grid_sample(const float* __restrict__ t, const int* dim, int out, int k,
                                             const float* x, bool clamp, bool aligned, bool linear) {
    int voxel[IN];
    float alpha[IN];
#pragma unroll
    for (int d = 0; d < IN; ++d) {
        const float tc = __fadd_rn(__fmul_rn(x[IN - 1 - d], 0.5f), 0.5f);
        const float pos = aligned ? __fmul_rn(tc, static_cast<float>(dim[d] - 1))
                                  : __fsub_rn(__fmul_rn(tc, static_cast<float>(dim[d])), 0.5f);
        const float fv = floorf(pos);
        voxel[d] = static_cast<int>(fv);
        alpha[d] = __fsub_rn(pos, fv);
    }
    float v = 0.0f;
    if (!linear) {
        bool inside = true;
        long long off = 0;
#pragma unroll
        for (int d = 0; d < IN; ++d) {
            int c = voxel[d] + (alpha[d] >= 0.5f ? 1 : 0);
            if (clamp) c = min(max(c, 0), dim[d] - 1);
            inside = inside && c >= 0 && c < dim[d];
            off = off * dim[d] + c;
        }
        return (clamp || inside) ? __ldg(t + off * out + k) : 0.0f;
    }
#pragma unroll
    for (int bits = 0; bits < (1 << IN); ++bits) {
        bool inside = true;
        long long off = 0;
        float w = 1.0f;
#pragma unroll
        for (int d = 0; d < IN; ++d) {
            const int up = (bits >> d) & 1;
            int c = voxel[d] + up;
            if (clamp) c = min(max(c, 0), dim[d] - 1);
            inside = inside && c >= 0 && c < dim[d];
            off = off * dim[d] + c;
            w = __fmul_rn(w, up ? alpha[d] : __fsub_rn(1.0f, alpha[d]));
        }
        if (!clamp && !inside) continue;
        v = __fadd_rn(v, __fmul_rn(w, __ldg(t + off * out + k)));
    }
    return v;
}

// Four consecutive channels k0..k0+3 of a 3-D sampler at x in one pass
// (16-byte loads: out % 4 == 0 and t 16-byte aligned), each channel with
// exactly the arithmetic of tensor_sample<3> / grid_sample<3> (used by
// sampler3_vec4_kernel below).
__device__ __forceinline__ float4 f4_fma_lerp(float4 l, float4 r, float xw) {
    const float omx = __fsub_rn(1.0f, xw);
    return make_float4(__fadd_rn(__fmul_rn(l.x, omx), __fmul_rn(r.x, xw)),
                       __fadd_rn(__fmul_rn(l.y, omx), __fmul_rn(r.y, xw)),
                       __fadd_rn(__fmul_rn(l.z, omx), __fmul_rn(r.z, xw)),
                       __fadd_rn(__fmul_rn(l.w, omx), __fmul_rn(r.w, xw)));
}
__device__ __forceinline__ float4 f4_add_scaled(float4 d, float s, float4 v) {
    return make_float4(__fadd_rn(d.x, __fmul_rn(s, v.x)), __fadd_rn(d.y, __fmul_rn(s, v.y)),
                       __fadd_rn(d.z, __fmul_rn(s, v.z)), __fadd_rn(d.w, __fmul_rn(s, v.w)));
}
// blend of a loaded pair for 4 channels: dst + rest mix(l, r, xw), or a
// single side, or nothing (blend_pair's cases)
__device__ __forceinline__ float4 blend_loaded4(float4 l, float4 r, bool left_in, bool right_in, float xw, float rest,
                                                float4 dst) {
    if (left_in && right_in) return f4_add_scaled(dst, rest, f4_fma_lerp(l, r, xw));
    if (left_in) return f4_add_scaled(dst, __fmul_rn(rest, __fsub_rn(1.0f, xw)), l);
    if (right_in) return f4_add_scaled(dst, __fmul_rn(rest, xw), r);
    return dst;
}

// The 8 corner loads are issued before any blending (they are independent;
// the clamped corner indices are always inside the tensor, and a corner
// that does not count is loaded and then skipped).
__device__ __forceinline__ float4 tensor_sample3_4(const float* __restrict__ t, const int* dim, int out, int k0,
                                                   const float* x, bool border, bool aligned, bool linear) {
    const float ac = aligned ? 1.0f : 0.0f;
    int lo[3], clo[3], chi[3];
    float alpha[3];
    bool lo_in[3], hi_in[3];
#pragma unroll
    for (int d = 0; d < 3; ++d) coord(x[2 - d], dim[d], ac, border, lo[d], clo[d], chi[d], alpha[d], lo_in[d], hi_in[d]);
    const long long st2 = out, st1 = st2 * dim[2], st0 = st1 * dim[1];
    float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (!linear) {
        bool inside = true;
        long long off = k0;
        const long long st[3] = {st0, st1, st2};
#pragma unroll
        for (int d = 0; d < 3; ++d) {
            int id = lo[d] + (alpha[d] >= 0.5f ? 1 : 0);
            inside = inside && id >= 0 && id < dim[d];
            id = min(max(id, 0), dim[d] - 1);
            off += id * st[d];
        }
        return (border || inside) ? __ldg(reinterpret_cast<const float4*>(t + off)) : v;
    }
    const long long dl = static_cast<long long>(chi[2] - clo[2]) * st2;
    const long long p00 = clo[0] * st0 + clo[1] * st1 + clo[2] * st2 + k0;
    const long long d0 = static_cast<long long>(chi[0] - clo[0]) * st0;
    const long long d1 = static_cast<long long>(chi[1] - clo[1]) * st1;
    // the pairs in the reference's order: (lo, lo), (lo, hi), (hi, hi), (hi, lo) of dims 0 and 1
    const long long base[4] = {p00, p00 + d1, p00 + d1 + d0, p00 + d0};
    float4 l[4], r[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        l[q] = __ldg(reinterpret_cast<const float4*>(t + base[q]));
        r[q] = __ldg(reinterpret_cast<const float4*>(t + base[q] + dl));
    }
    const float a0 = alpha[0], a1 = alpha[1];
    v = blend_loaded4(l[0], r[0], lo_in[0] && lo_in[1] && lo_in[2], lo_in[0] && lo_in[1] && hi_in[2], alpha[2],
                      __fmul_rn(__fsub_rn(1.0f, a0), __fsub_rn(1.0f, a1)), v);
    v = blend_loaded4(l[1], r[1], lo_in[0] && hi_in[1] && lo_in[2], lo_in[0] && hi_in[1] && hi_in[2], alpha[2],
                      __fmul_rn(__fsub_rn(1.0f, a0), a1), v);
    v = blend_loaded4(l[2], r[2], hi_in[0] && hi_in[1] && lo_in[2], hi_in[0] && hi_in[1] && hi_in[2], alpha[2],
                      __fmul_rn(a0, a1), v);
    v = blend_loaded4(l[3], r[3], hi_in[0] && lo_in[1] && lo_in[2], hi_in[0] && lo_in[1] && hi_in[2], alpha[2],
                      __fmul_rn(a0, __fsub_rn(1.0f, a1)), v);
    return v;
}

__device__ __forceinline__ float4 grid_sample3_4(const float* __restrict__ t, const int* dim, int out, int k0,
                                                 const float* x, bool clamp, bool aligned, bool linear) {
    int voxel[3];
    float alpha[3];
#pragma unroll
    for (int d = 0; d < 3; ++d) {
        const float tc = __fadd_rn(__fmul_rn(x[2 - d], 0.5f), 0.5f);
        const float pos = aligned ? __fmul_rn(tc, static_cast<float>(dim[d] - 1))
                                  : __fsub_rn(__fmul_rn(tc, static_cast<float>(dim[d])), 0.5f);
        const float fv = floorf(pos);
        voxel[d] = static_cast<int>(fv);
        alpha[d] = __fsub_rn(pos, fv);
    }
    float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (!linear) {
        bool inside = true;
        long long off = 0;
#pragma unroll
        for (int d = 0; d < 3; ++d) {
            int c = voxel[d] + (alpha[d] >= 0.5f ? 1 : 0);
            if (clamp) c = min(max(c, 0), dim[d] - 1);
            inside = inside && c >= 0 && c < dim[d];
            off = off * dim[d] + c;
        }
        return (clamp || inside) ? __ldg(reinterpret_cast<const float4*>(t + off * out + k0)) : v;
    }
    float4 val[8];
    bool use[8];
#pragma unroll
    for (int bits = 0; bits < 8; ++bits) {
        bool inside = true;
        long long off = 0;
#pragma unroll
        for (int d = 0; d < 3; ++d) {
            const int c = voxel[d] + ((bits >> d) & 1);
            inside = inside && c >= 0 && c < dim[d];
            off = off * dim[d] + min(max(c, 0), dim[d] - 1);  // clamped: a valid address either way
        }
        use[bits] = clamp || inside;
        val[bits] = __ldg(reinterpret_cast<const float4*>(t + off * out + k0));
    }
#pragma unroll
    for (int bits = 0; bits < 8; ++bits) {
        float w = 1.0f;
#pragma unroll
        for (int d = 0; d < 3; ++d) w = __fmul_rn(w, ((bits >> d) & 1) ? alpha[d] : __fsub_rn(1.0f, alpha[d]));
        if (use[bits]) v = f4_add_scaled(v, w, val[bits]);
    }
    return v;
}

// 3-D samplers with out % 4 == 0 (16-byte aligned tensor and output): one
// thread per (point, 4 channels), the corner indices and weights computed
// once per 4 channels and 16-byte gathers -- the same per-channel
// arithmetic as the kernels above (tensor_sample3_4 / grid_sample3_4).
template <bool GRID>
__global__ void sampler3_vec4_kernel(const __grid_constant__ GridParams p) {
    const int quads = p.out >> 2;
    const long long total = p.n * quads;
    for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long i = idx / quads;
        const int k0 = static_cast<int>(idx - i * quads) * 4;
        const float x[3] = {__ldg(p.x + i * 3), __ldg(p.x + i * 3 + 1), __ldg(p.x + i * 3 + 2)};
        const float4 v = GRID ? grid_sample3_4(p.t, p.dim, p.out, k0, x, p.clamp != 0, p.aligned != 0, p.linear != 0)
                              : tensor_sample3_4(p.t, p.dim, p.out, k0, x, p.clamp != 0, p.aligned != 0,
                                                 p.linear != 0);
        *reinterpret_cast<float4*>(p.y + i * p.out + k0) = v;
    }
}

template <int IN>
__global__ void grid_sampler_kernel(const __grid_constant__ GridParams p) {
    const long long total = p.n * p.out;
    for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long i = idx / p.out;
        const int k = static_cast<int>(idx - i * p.out);
        float x[IN];
#pragma unroll
        for (int d = 0; d < IN; ++d) x[d] = __ldg(p.x + i * IN + d);
        p.y[idx] = grid_sample<IN>(p.t, p.dim, p.out, k, x, p.clamp != 0, p.aligned != 0, p.linear != 0);
    }
}

}  // namespace sampler
}  // namespace rdvb
