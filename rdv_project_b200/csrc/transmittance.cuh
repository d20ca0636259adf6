// RaymarchingTransmittance: fixed-step absorption march with an MLP
// extinction, one persistent thread per ray.
//
// Per ray (x, w) -- rdv/shaders/volumes/raymarching_transmittance.h:1-21:
//   x <- L (x - O), w <- L w   (L = inverse of the node transform's 3x3
//                               part, O its translation; L is formed on the
//                               host)
//   slab test against [-1, 1]^3 (rdv/shaders/libraries/math_library.h:48-57);
//   a ray with tMax <= 0 or tMin > tMax returns 1;
//   tMin <- max(0, tMin), x <- x + w tMin, d <- tMax - tMin, then
//   rdv/shaders/volumes/raymarching_transmittance_trait.h:1-14:
//     tau = 0; while d > 0 (at most 4096 steps):
//       tau += extinction(x) * scale * step; tau > 16 -> return 0;
//       d -= step; x += step * w
//     return exp(-tau)
// The march arithmetic is written with explicit round-to-nearest products
// and sums (no contraction into FMAs), so the step count, the positions and
// the early exit follow the reference's fp32 operations one for one.
//
// The extinction is a chain of Linear (exact fp32: acc = b, acc += x W in
// ascending k, rdv/shaders/maps/linear.h:28-31) or LinearFast layers
// (float16 / bfloat16 staged operands, fp32 accumulation, bias after,
// rdv/shaders/maps/linear_fast.h:61-98) with optional ReLUs, 3 inputs and 1
// output. All layers' weights are staged once per CTA into shared memory as
// [K][chunk] blocks (one broadcast 16-byte load feeds 4 FMAs); activations
// live in shared memory transposed ([feature][thread]), conflict free.
//
// Rays are handed out by one global counter: a thread whose ray finished
// takes the next one, so the lanes of a warp stay busy although rays march
// different numbers of steps.
#pragma once
#include "mlp_tc.cuh"
#include "rng.cuh"
#include "sampler.cuh"

namespace rdvb {
namespace trm {

constexpr int kThreads = 128;    // rays in flight per CTA (transmittance_kernel)
constexpr int kRtWideThreads = 384;  // ratiotracking_kernel when the chain is at most 64 wide
constexpr int kMaxLayers = 8;
constexpr int kMaxWidth = 128;
constexpr int kSafety = 4096;    // raymarching_transmittance_trait.h:4

struct Layer {
    const float* W;  // [N, K] fp32 (the caller's layout)
    const float* b;  // [N] fp32
    int K, N;
    int chunk;     // 4 or 32 outputs per weight block
    int w_off;     // float offset of this layer's blocks in the shared weight image
    int b_off;     // float offset of its bias
    int math;      // 0 f32 exact, 1 f16 staging, 2 bf16 staging
    int relu;
};

struct Params {
    const float* rays;      // [n_rays, 6] (x, w)
    float* out;             // [n_rays]
    long long n_rays;
    int* counter;                   // next ray index (0 at launch)
    unsigned long long* evaluations; // extinction evaluations of the launch (0 at launch)
    float L[9];             // row-major 3x3: x_obj[i] = sum_j L[3 i + j] (x - O)[j]
    float O[3];
    float step, scale;
    int n_layers;
    int input_relu;
    int maxw;               // widest activation (>= 3)
    int w_floats;           // floats of the shared weight image (weight blocks, then biases)
    Layer layer[kMaxLayers];
    // input encoding (a sampler of a dense 3-D grid in front of the chain)
    int enc;                // 0 none, 1 TensorSampler, 2 GridSampler
    const float* enc_t;     // [D, H, W, F] fp32
    int enc_dim[3];         // D, H, W
    int enc_out;            // F (the chain's input width, or 1 without layers)
    int enc_clamp, enc_aligned, enc_linear;
    // ratiotracking_kernel / pbvr_kernel only
    const float* maj;       // majorant voxels [D, H, W] (z, y, x), [D, H, W, 2] for a sphere field
    int mdim[3];            // W, H, D: cells along x, y, z
    float mvs[3];           // voxel sizes 2 / mdim (fp32 division, as the reference's vec3(2.0) / dim)
    int field;              // 0 VoxelMajorantField, 1 SphereMajorantField
    unsigned seeds[4];      // the dispatch's generator seeds
    int draws_before;       // draws of each ray's generator already used upstream (a jittered camera: 2)
    // chain_rows_kernel only
    const void* x;          // [rows, IN] float32 / float16 / bfloat16
    int x_dtype;            // 0 f32, 1 f16, 2 bf16
    float* y;               // [rows, OUT]
    long long row_begin, row_end;
};

__device__ __forceinline__ float stage_val(float v, int math) {
    if (math == 1) return __half2float(__float2half_rn(v));
    if (math == 2) return __bfloat162float(__float2bfloat16_rn(v));
    return v;
}

// One chunk of CH outputs of layer L for this thread: acc over ascending k.
template <int CH, int T = kThreads>
__device__ __forceinline__ void chunk_eval(const Layer& L, const float* __restrict__ wsm, const float* __restrict__ bsm,
                                           const float* ain, int o0, float (&acc)[CH]) {
#pragma unroll
    for (int j = 0; j < CH; ++j) acc[j] = (L.math == 0 && o0 + j < L.N) ? bsm[L.b_off + o0 + j] : 0.0f;
    const float* wb = wsm + L.w_off + o0 * L.K;  // block of outputs o0..o0+CH-1: [K][CH]
    for (int k = 0; k < L.K; ++k) {
        const float a = ain[k * T];
        const float4* wr = reinterpret_cast<const float4*>(wb + k * CH);
        float4 wk[CH / 4];  // the step's operands first, then its FMAs
#pragma unroll
        for (int j4 = 0; j4 < CH / 4; ++j4) wk[j4] = wr[j4];
#pragma unroll
        for (int j4 = 0; j4 < CH / 4; ++j4) {
            acc[4 * j4 + 0] = fmaf(a, wk[j4].x, acc[4 * j4 + 0]);
            acc[4 * j4 + 1] = fmaf(a, wk[j4].y, acc[4 * j4 + 1]);
            acc[4 * j4 + 2] = fmaf(a, wk[j4].z, acc[4 * j4 + 2]);
            acc[4 * j4 + 3] = fmaf(a, wk[j4].w, acc[4 * j4 + 3]);
        }
    }
}

// Finishes a chunk: bias after (staged layers), ReLU, staging for the next
// layer's operands; writes outputs o0.. into aout (the thread's column).
template <int CH, int T = kThreads>
__device__ __forceinline__ void chunk_store(const Layer& L, const float* __restrict__ bsm, int next_math, int o0,
                                            const float (&acc)[CH], float* aout) {
#pragma unroll
    for (int j = 0; j < CH; ++j) {
        const int o = o0 + j;
        if (o < L.N) {
            float v = acc[j];
            if (L.math != 0) v += bsm[L.b_off + o];
            if (L.relu) v = fmaxf(v, 0.0f);
            aout[o * T] = stage_val(v, next_math);
        }
    }
}

// The chain on this thread's activation column act0 (the input, already
// staged for layer 0); returns the column holding the last layer's outputs.
// T: threads of the CTA, the stride of the [feature][thread] columns.
template <int T = kThreads>
__device__ __forceinline__ const float* eval_chain(const Params& p, const float* __restrict__ wsm,
                                                   const float* __restrict__ bsm, float* act0, float* act1) {
    float* ain = act0;
    float* aout = act1;
    for (int l = 0; l < p.n_layers; ++l) {
        const Layer L = p.layer[l];
        const int next_math = l + 1 < p.n_layers ? p.layer[l + 1].math : 0;
        if (L.chunk == 4) {
            for (int o0 = 0; o0 < L.N; o0 += 4) {
                float acc[4];
                chunk_eval<4, T>(L, wsm, bsm, ain, o0, acc);
                chunk_store<4, T>(L, bsm, next_math, o0, acc, aout);
            }
        } else {
            for (int o0 = 0; o0 < L.N; o0 += 32) {
                float acc[32];
                chunk_eval<32, T>(L, wsm, bsm, ain, o0, acc);
                chunk_store<32, T>(L, bsm, next_math, o0, acc, aout);
            }
        }
        float* t = ain;
        ain = aout;
        aout = t;
    }
    return ain;
}

// extinction(x) for this thread: the chain on the 3-vector x, or on the
// F features the input encoding samples at x (the sampler's own arithmetic,
// sampler.cuh); an encoding without layers is the extinction itself. ENC =
// false compiles the kernel without the encoding's sampler code (for
// launches whose Params have none: a smaller instruction footprint).
template <int T = kThreads, bool ENC = true>
__device__ __forceinline__ float extinction(const Params& p, const float* __restrict__ wsm,
                                            const float* __restrict__ bsm, float* act0, float* act1,
                                            const float (&x)[3]) {
    const int m0 = p.n_layers > 0 ? p.layer[0].math : 0;
    if (ENC && p.enc) {
        for (int k = 0; k < p.enc_out; ++k) {
            float v = p.enc == 1 ? sampler::tensor_sample<3>(p.enc_t, p.enc_dim, p.enc_out, k, x, p.enc_clamp != 0,
                                                              p.enc_aligned != 0, p.enc_linear != 0)
                                 : sampler::grid_sample<3>(p.enc_t, p.enc_dim, p.enc_out, k, x, p.enc_clamp != 0,
                                                            p.enc_aligned != 0, p.enc_linear != 0);
            if (p.input_relu) v = fmaxf(v, 0.0f);
            act0[k * T] = stage_val(v, m0);
        }
    } else {
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            float v = x[k];
            if (p.input_relu) v = fmaxf(v, 0.0f);
            act0[k * T] = stage_val(v, m0);
        }
    }
    return eval_chain<T>(p, wsm, bsm, act0, act1)[0];
}

// raymarching_transmittance.h:4-19 for one ray r = (x, w): object space,
// slab test, entry clamp. Returns false on a miss; else the entry point x,
// the object-space direction w and d = tMax - tMin.
__device__ __forceinline__ bool march_entry(const float* __restrict__ r, const float (&L)[9], const float (&O)[3],
                                            float (&x)[3], float (&w)[3], float& d) {
    float xr[3], wr[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        xr[k] = __fsub_rn(r[k], O[k]);
        wr[k] = r[3 + k];
    }
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        x[i] = __fadd_rn(__fadd_rn(__fmul_rn(L[3 * i], xr[0]), __fmul_rn(L[3 * i + 1], xr[1])),
                         __fmul_rn(L[3 * i + 2], xr[2]));
        w[i] = __fadd_rn(__fadd_rn(__fmul_rn(L[3 * i], wr[0]), __fmul_rn(L[3 * i + 1], wr[1])),
                         __fmul_rn(L[3 * i + 2], wr[2]));
    }
    float tmin = -INFINITY, tmax = INFINITY;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const float inv = __fdiv_rn(1.0f, w[k]);
        const float xc = __fmul_rn(-x[k], inv);
        const float s = fabsf(inv);
        tmin = fmaxf(tmin, __fsub_rn(xc, s));
        tmax = fminf(tmax, __fadd_rn(xc, s));
    }
    if (tmax <= 0.0f || tmin > tmax) return false;
    tmin = fmaxf(0.0f, tmin);
#pragma unroll
    for (int k = 0; k < 3; ++k) x[k] = __fadd_rn(x[k], __fmul_rn(w[k], tmin));
    d = __fsub_rn(tmax, tmin);
    return true;
}

// Stages every layer once into shared memory: block of outputs o0..o0+CH-1
// as [K][CH], values rounded to the layer's operand format, zero beyond N;
// then the biases.
template <int T = kThreads>
__device__ __forceinline__ void stage_chain(const Params& p, float* wsm) {
    for (int l = 0; l < p.n_layers; ++l) {
        const Layer L = p.layer[l];
        const int nb = (L.N + L.chunk - 1) / L.chunk;
        for (int i = threadIdx.x; i < nb * L.chunk * L.K; i += T) {
            const int blk = i / (L.chunk * L.K), rem = i - blk * L.chunk * L.K;
            const int k = rem / L.chunk, j = rem - k * L.chunk;
            const int o = blk * L.chunk + j;
            wsm[L.w_off + i] = o < L.N ? stage_val(L.W[static_cast<size_t>(o) * L.K + k], L.math) : 0.0f;
        }
        for (int i = threadIdx.x; i < L.N; i += T) wsm[L.b_off + i] = L.b[i];
    }
    __syncthreads();
}

__global__ void __launch_bounds__(kThreads) transmittance_kernel(const __grid_constant__ Params p) {
    extern __shared__ float sm[];
    float* wsm = sm;                                   // weight blocks, then biases
    float* act0 = sm + ((p.w_floats + 3) & ~3) + threadIdx.x;
    float* act1 = act0 + p.maxw * kThreads;
    stage_chain(p, wsm);
    const float* bsm = wsm;  // b_off values index the same image

    long long ray = -1;
    float x[3], w[3], d = 0.0f, tau = 0.0f;
    int steps = 0;
    unsigned long long my_evals = 0;  // this thread's evaluations, added once at the end
    while (true) {
        if (ray < 0) {
            ray = atomicAdd(p.counter, 1);
            if (ray >= p.n_rays) break;
            if (!march_entry(p.rays + ray * 6, p.L, p.O, x, w, d)) {
                p.out[ray] = 1.0f;  // the ray misses the volume: fully transparent
                ray = -1;
                continue;
            }
            tau = 0.0f;
            steps = 0;
            if (!(d > 0.0f)) {
                p.out[ray] = 1.0f;  // exp(-0)
                ray = -1;
                continue;
            }
        }
        const float e = __fmul_rn(extinction(p, wsm, bsm, act0, act1, x), p.scale);
        ++steps;
        tau = __fadd_rn(tau, __fmul_rn(e, p.step));
        bool done = false;
        float result = 0.0f;
        if (tau > 16.0f) {
            done = true;
        } else {
            d = __fsub_rn(d, p.step);
#pragma unroll
            for (int k = 0; k < 3; ++k) x[k] = __fadd_rn(x[k], __fmul_rn(p.step, w[k]));
            if (!(d > 0.0f) || steps >= kSafety) {
                done = true;
                result = expf(-tau);
            }
        }
        if (done) {
            p.out[ray] = result;
            my_evals += static_cast<unsigned long long>(steps);
            ray = -1;
        }
    }
    if (my_evals) atomicAdd(p.evaluations, my_evals);
}

// ---------------------------------------------------------------------------
// RatiotrackingTransmittance (rdv/shaders/volumes/ratiotracking_transmittance.h,
// ratiotracking_transmittance_trait.h): majorant-based ratio tracking with
// Russian roulette, one persistent thread per ray.
//
// Generator: rdv/shaders/libraries/random_library.h:7-49 -- three
// Tausworthe components and an LCG, XOR-combined; random() = the low 23
// bits as a mantissa in [1, 2), minus 1. Ray r draws from the dispatch
// seeds spawned by its row index r (the reference's per-invocation init,
// random_library.h:256-268, with gl_GlobalInvocationID.x = row), so every
// ray's sequence is independent of scheduling.
// Majorant: VoxelMajorantField (rdv/shaders/volumes/voxel_majorant_field.h)
// over a [D, H, W] grid: the cell holding x, and the distance along w to
// that cell's exit.
// The loop (at most 1024 iterations):
//   maj = max(majorant, 1e-12), dist = max(exit distance, 1e-6)
//   dt = min(dist, -log(1 - random()) / (maj * density_scale))
//   d -= dt, x += dt w;  dt >= dist -> next cell;  d <= 0 -> done
//   T *= 1 - extinction(x) / maj;  T < 0.05 -> roulette: random() >= T
//   returns 0, else T = 1.
// Every operation is a separately rounded fp32 operation (no contraction);
// log is CUDA's logf.
__device__ __forceinline__ float voxel_majorant(const Params& p, const float (&x)[3], const float (&w)[3],
                                                float& dist) {
    int cell[3];
    float texit[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const float f = static_cast<float>(p.mdim[k]);
        int c = static_cast<int>(__fmul_rn(__fadd_rn(__fmul_rn(x[k], 0.5f), 0.5f), f));  // toward zero
        c = min(max(c, 0), p.mdim[k] - 1);
        cell[k] = c;
        const float vs = p.mvs[k];
        const float bmin = __fsub_rn(__fmul_rn(static_cast<float>(c), vs), 1.0f);
        const float bmax = __fadd_rn(bmin, vs);
        const float t0 = __fdiv_rn(__fsub_rn(bmin, x[k]), w[k]);
        const float t1 = __fdiv_rn(__fsub_rn(bmax, x[k]), w[k]);
        texit[k] = t0 < t1 ? t1 : t0;  // GLSL max
    }
    dist = texit[1] < texit[0] ? texit[1] : texit[0];  // GLSL min
    dist = texit[2] < dist ? texit[2] : dist;
    return __ldg(p.maj + (static_cast<long long>(cell[2]) * p.mdim[1] + cell[1]) * p.mdim[0] + cell[0]);
}

// SphereMajorantField (rdv/shaders/volumes/sphere_majorant_field.h): the
// cell holding x stores (majorant, radius in voxel units); the returned
// distance is to the exit, along w, of the box of that half-width around
// the cell's centre, at least 1e-6.
__device__ __forceinline__ float sphere_majorant(const Params& p, const float (&x)[3], const float (&w)[3],
                                                 float& dist) {
    int cell[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const float f = static_cast<float>(p.mdim[k]);
        int c = static_cast<int>(__fmul_rn(__fadd_rn(__fmul_rn(x[k], 0.5f), 0.5f), f));
        cell[k] = min(max(c, 0), p.mdim[k] - 1);
    }
    const long long idx = (static_cast<long long>(cell[2]) * p.mdim[1] + cell[1]) * p.mdim[0] + cell[0];
    const float majv = __ldg(p.maj + 2 * idx), radius = __ldg(p.maj + 2 * idx + 1);
    float texit[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const float vs = p.mvs[k];
        const float center = __fsub_rn(__fmul_rn(__fadd_rn(static_cast<float>(cell[k]), 0.5f), vs), 1.0f);
        const float half = __fmul_rn(radius, vs);
        const float t0 = __fdiv_rn(__fsub_rn(__fsub_rn(center, half), x[k]), w[k]);
        const float t1 = __fdiv_rn(__fsub_rn(__fadd_rn(center, half), x[k]), w[k]);
        texit[k] = t0 < t1 ? t1 : t0;  // GLSL max
    }
    float dd = texit[1] < texit[0] ? texit[1] : texit[0];  // GLSL min
    dd = texit[2] < dd ? texit[2] : dd;
    dist = dd < 1e-6f ? 1e-6f : dd;  // max(dist, 1e-6)
    return majv;
}

// The node's majorant field at (x, w): (majorant, max step).
__device__ __forceinline__ float field_majorant(const Params& p, const float (&x)[3], const float (&w)[3],
                                                float& dist) {
    return p.field == 1 ? sphere_majorant(p, x, w, dist) : voxel_majorant(p, x, w, dist);
}

constexpr int kRtSafety = 1024;  // ratiotracking_transmittance_trait.h's loop cap
// free flights per lane between two warp-wide extinction rounds (a
// compile-time tuning constant)
#ifndef RDVB_YIELD_FLIGHTS
#define RDVB_YIELD_FLIGHTS 16
#endif
constexpr int kYieldFlights = RDVB_YIELD_FLIGHTS;

// Work is warp-coherent: each lane advances its own ray (free flights across
// majorant cells, taking the next ray when one ends) until it reaches a
// collision; then the whole warp evaluates the extinction MLP together, each
// lane on its own collision point (lanes without rays left evaluate a dummy
// point and discard it), and applies the collision. The MLP -- nearly all of
// the arithmetic -- thus runs with the lanes converged instead of once per
// colliding lane.
template <int NT, bool ENC>
__global__ void __launch_bounds__(NT) ratiotracking_kernel(const __grid_constant__ Params p) {
    extern __shared__ float sm[];
    float* wsm = sm;
    float* act0 = sm + ((p.w_floats + 3) & ~3) + threadIdx.x;
    float* act1 = act0 + p.maxw * NT;
    stage_chain<NT>(p, wsm);
    const float* bsm = wsm;
    unsigned long long my_evals = 0;
    long long ray = -1;  // -1: take the next ray; -2: none left
    float x[3] = {0.0f, 0.0f, 0.0f}, w[3] = {0.0f, 0.0f, 0.0f}, d = 0.0f, T = 1.0f, maj = 1.0f;
    int safety = 0;
    Rng r = {0u, 0u, 0u, 0u};
    while (true) {
        bool pending = false;  // a collision at x waits for its extinction
        // at most kYieldFlights free flights per lane between two extinction
        // rounds, so that a lane stuck in a long run of free flights does
        // not hold the warp's colliding lanes back
        for (int flights = 0; ray != -2 && !pending && flights < kYieldFlights; ++flights) {
            if (ray < 0) {
                ray = atomicAdd(p.counter, 1);
                if (ray >= p.n_rays) {
                    ray = -2;
                    break;
                }
                if (!march_entry(p.rays + ray * 6, p.L, p.O, x, w, d)) {
                    p.out[ray] = 1.0f;  // the ray misses the volume: fully transparent
                    ray = -1;
                    continue;
                }
                T = 1.0f;
                safety = 0;
                r = rng_spawn(p.seeds, static_cast<unsigned>(ray));
                for (int k = 0; k < p.draws_before; ++k) rng_step(r);
            }
            if (!(d > 0.0f) || safety >= kRtSafety) {  // the loop condition
                p.out[ray] = T;
                ray = -1;
                continue;
            }
            ++safety;
            float dist;
            maj = field_majorant(p, x, w, dist);
            maj = maj < 1e-12f ? 1e-12f : maj;
            dist = dist < 1e-6f ? 1e-6f : dist;
            const float q = __fdiv_rn(-logf(__fsub_rn(1.0f, rng_uniform(r))), __fmul_rn(maj, p.scale));
            const float dt = q < dist ? q : dist;  // free-flight distance
            d = __fsub_rn(d, dt);
#pragma unroll
            for (int k = 0; k < 3; ++k) x[k] = __fadd_rn(x[k], __fmul_rn(dt, w[k]));
            if (dt >= dist) continue;  // left the majorant's cell
            if (d <= 0.0f) {           // reached the end without a collision
                p.out[ray] = T;
                ray = -1;
                continue;
            }
            pending = true;
        }
        if (!__any_sync(0xffffffffu, pending)) {
            if (__all_sync(0xffffffffu, ray == -2)) break;  // no lane has rays left
            continue;
        }
        const float sigma = extinction<NT, ENC>(p, wsm, bsm, act0, act1, x);
        if (pending) {
            ++my_evals;
            T = __fmul_rn(T, __fsub_rn(1.0f, __fdiv_rn(sigma, maj)));
            if (T < 0.05f) {
                if (rng_uniform(r) >= T) {
                    p.out[ray] = 0.0f;
                    ray = -1;
                } else {
                    T = 1.0f;  // Russian roulette survivor
                }
            }
        }
    }
    if (my_evals) atomicAdd(p.evaluations, my_evals);
}

// ---------------------------------------------------------------------------
// Rows mode of the same evaluator: the CUDA-core MLP (exact fp32 Linear
// chains, chains that mix precisions, the fp32 tail rows of LinearFast
// chains), y[row] = chain(x[row]) for row_begin <= row < row_end. Persistent
// CTAs of NT rows stage the chain's weights into shared memory once and then
// walk the rows; every thread evaluates its row in its own activation
// column, so no barrier follows the staging. The arithmetic is that of
// mlp_simt_kernel: bias first and FMAs in ascending k for exact layers,
// staged operands with the bias after for LinearFast layers. A k-step loads
// all of its operands (the row's activation, CH weights as float4 broadcast
// loads) into registers before its FMAs: with the few warps that the
// activation columns leave resident, that is what keeps shared-memory
// latency off the FMA chain (0.31 -> 0.23 ms on a 262,144-row
// 3-64-64-64-4 chain).
template <int CH, int NT>
__device__ __forceinline__ void rows_chunk(const Layer& L, const float* __restrict__ wsm, const float* __restrict__ bsm,
                                           const float* ain, float* aout, int next_math, int o0) {
    float acc[CH];
#pragma unroll
    for (int j = 0; j < CH; ++j) acc[j] = (L.math == 0 && o0 + j < L.N) ? bsm[L.b_off + o0 + j] : 0.0f;
    const float* wb = wsm + L.w_off + o0 * L.K;
    for (int k = 0; k < L.K; ++k) {
        const float a = ain[k * NT];
        const float4* wr = reinterpret_cast<const float4*>(wb + k * CH);
        float4 wk[CH / 4];
#pragma unroll
        for (int j4 = 0; j4 < CH / 4; ++j4) wk[j4] = wr[j4];
#pragma unroll
        for (int j4 = 0; j4 < CH / 4; ++j4) {
            acc[4 * j4 + 0] = fmaf(a, wk[j4].x, acc[4 * j4 + 0]);
            acc[4 * j4 + 1] = fmaf(a, wk[j4].y, acc[4 * j4 + 1]);
            acc[4 * j4 + 2] = fmaf(a, wk[j4].z, acc[4 * j4 + 2]);
            acc[4 * j4 + 3] = fmaf(a, wk[j4].w, acc[4 * j4 + 3]);
        }
    }
#pragma unroll
    for (int j = 0; j < CH; ++j) {
        const int o = o0 + j;
        if (o < L.N) {
            float v = acc[j];
            if (L.math != 0) v += bsm[L.b_off + o];
            if (L.relu) v = fmaxf(v, 0.0f);
            aout[o * NT] = stage_val(v, next_math);
        }
    }
}

template <int NT>
__global__ void __launch_bounds__(NT) chain_rows_kernel(const __grid_constant__ Params p) {
    extern __shared__ float sm[];
    float* wsm = sm;
    float* act0 = sm + ((p.w_floats + 3) & ~3) + threadIdx.x;
    float* act1 = act0 + p.maxw * NT;
    stage_chain<NT>(p, wsm);
    const float* bsm = wsm;
    const int in0 = p.layer[0].K, m0 = p.layer[0].math;
    const int outd = p.layer[p.n_layers - 1].N;
    for (long long base = p.row_begin + static_cast<long long>(blockIdx.x) * NT; base < p.row_end;
         base += static_cast<long long>(gridDim.x) * NT) {
        const long long row = base + threadIdx.x;
        const bool valid = row < p.row_end;
        for (int k = 0; k < in0; ++k) {
            float v = 0.0f;
            if (valid) {
                const long long i = row * in0 + k;
                if (p.x_dtype == 0) v = static_cast<const float*>(p.x)[i];
                else if (p.x_dtype == 1) v = __half2float(static_cast<const __half*>(p.x)[i]);
                else v = __bfloat162float(static_cast<const __nv_bfloat16*>(p.x)[i]);
                if (p.input_relu) v = fmaxf(v, 0.0f);
            }
            act0[k * NT] = stage_val(v, m0);
        }
        float* ain = act0;
        float* aout = act1;
        for (int l = 0; l < p.n_layers; ++l) {
            const Layer L = p.layer[l];
            const int next_math = l + 1 < p.n_layers ? p.layer[l + 1].math : 0;
            if (L.chunk == 4) {
                for (int o0 = 0; o0 < L.N; o0 += 4) rows_chunk<4, NT>(L, wsm, bsm, ain, aout, next_math, o0);
            } else {
                for (int o0 = 0; o0 < L.N; o0 += 32) rows_chunk<32, NT>(L, wsm, bsm, ain, aout, next_math, o0);
            }
            float* t = ain;
            ain = aout;
            aout = t;
        }
        if (valid)
            for (int o = 0; o < outd; ++o) p.y[row * outd + o] = ain[o * NT];
    }
}

// ---------------------------------------------------------------------------
// Tensor-core path (float16 / bfloat16 extinction chains): rays in batches.
//   trm_setup_kernel   one thread per ray: entry point, the exact step count
//                      of the reference's loop (d -= step while d > 0, at
//                      most 4096 steps), and a contiguous run of ceil(n/128)
//                      chunk-list entries (warp-aggregated append);
//   mlp_tc_kernel      (ray mode, march = 1) one 128-step chunk per tile:
//                      the extinction MLP on tcgen05 and the chunk's (sum,
//                      largest prefix) of tau;
//   trm_combine_kernel one thread per ray: the chunks in step order -- 0 as
//                      soon as tau + prefix > 16, else exp(-tau).
// Every step of a ray is evaluated, also past an early exit; the result is
// the reference's.
struct SetupParams {
    const float* rays;  // batch [n, 6]
    float* out;         // batch [n]
    int n;
    float L[9];
    float O[3];
    float step;
    mlp_tc::MarchRay* rec;
    int* chunk_list;
    int* n_chunks;
};

__global__ void trm_setup_kernel(const __grid_constant__ SetupParams p) {
    const int lane = threadIdx.x & 31;
    for (int base0 = blockIdx.x * blockDim.x; base0 < p.n; base0 += gridDim.x * blockDim.x) {
        const int i = base0 + threadIdx.x;
        int nch = 0;
        mlp_tc::MarchRay mr;
        if (i < p.n) {
            float x[3], w[3], d = 0.0f;
            int n = 0;
            if (march_entry(p.rays + static_cast<long long>(i) * 6, p.L, p.O, x, w, d)) {
                while (d > 0.0f && n < kSafety) {
                    d = __fsub_rn(d, p.step);
                    ++n;
                }
            }
#pragma unroll
            for (int k = 0; k < 3; ++k) {
                mr.x[k] = x[k];
                mr.w[k] = w[k];
            }
            mr.n_steps = n;
            nch = (n + mlp_tc::kTileM - 1) / mlp_tc::kTileM;
            if (n == 0) p.out[i] = 1.0f;  // miss, or an empty segment: exp(-0)
        }
        // warp-aggregated append of each ray's chunk run
        int incl = nch;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int nb = __shfl_up_sync(0xffffffffu, incl, d);
            if (lane >= d) incl += nb;
        }
        const int total = __shfl_sync(0xffffffffu, incl, 31);
        int wbase = 0;
        if (lane == 0 && total) wbase = atomicAdd(p.n_chunks, total);
        wbase = __shfl_sync(0xffffffffu, wbase, 0);
        if (i < p.n) {
            mr.base = wbase + incl - nch;
            p.rec[i] = mr;
            for (int c = 0; c < nch; ++c) p.chunk_list[mr.base + c] = i;
        }
    }
}

struct CombineParams {
    const mlp_tc::MarchRay* rec;
    const float2* chunk_out;
    float* out;
    int n;
    unsigned long long* evaluations;
};

__global__ void trm_combine_kernel(const __grid_constant__ CombineParams p) {
    for (int base0 = blockIdx.x * blockDim.x; base0 < p.n; base0 += gridDim.x * blockDim.x) {
        const int i = base0 + threadIdx.x;
        unsigned n = 0;
        if (i < p.n) {
            n = static_cast<unsigned>(p.rec[i].n_steps);
            if (n > 0) {
                const int base = p.rec[i].base;
                const int nch = (static_cast<int>(n) + mlp_tc::kTileM - 1) / mlp_tc::kTileM;
                float tau = 0.0f, T = -1.0f;
                for (int c = 0; c < nch; ++c) {
                    const float2 r = p.chunk_out[base + c];
                    if (tau + r.y > 16.0f) {
                        T = 0.0f;
                        break;
                    }
                    tau += r.x;
                }
                p.out[i] = T < 0.0f ? expf(-tau) : T;
            }
        }
        // one atomic per warp for the evaluation count
        const unsigned warp_n = __reduce_add_sync(0xffffffffu, n);
        if ((threadIdx.x & 31) == 0 && warp_n) atomicAdd(p.evaluations, static_cast<unsigned long long>(warp_n));
    }
}

}  // namespace trm
}  // namespace rdvb
