// PBVR (rdv/domain/volumes.py:257-326, rdv/shaders/volumes/pbvr.h): unbiased
// volume rendering by delta tracking through a majorant field, with an MLP
// extinction, Henyey-Greenstein scattering, an albedo, a bounce budget and
// an environment for escaped paths; one persistent thread per ray, RGB out.
//
// Per ray (x, w) -- pbvr.h:21-110:
//   object space x <- L (x - O), wo <- L w (L formed on the host); slab test
//   against [-1, 1]^3; a miss returns environment(w);
//   entry clamp, x <- x + wo tMin, d <- tMax - tMin; W = (1, 1, 1);
//   for (safety < 8192 while d > 0):
//     maj = max(majorant(x, wo, max_step), 1e-12)
//     dt = -log(1 - random()) / maj; step = min(dt, min(max_step, d))
//     x += step wo; d -= step
//     step < dt: d <= 0 -> escaped; else next iteration (a new majorant cell)
//     collision: random() >= extinction(x) / maj -> null collision
//     real collision: W *= albedo; max(W) < 1e-4 -> 0; bounces >= max -> 0;
//       w <- hg_phase_sample(w, g); wo <- L w; d <- the slab exit from x
//   escaped -> W * environment(w), else 0.
// pbvr.h calls local_majorant(mg, x, w, max_step), defined by
// volumes/majorant_field_precode.h, which the reference checkout does not
// contain. It is taken here as the field's Map[6, 2] output (x, w) ->
// (majorant, distance), read as majorant_trait.h reads it, with the distance
// floored at 1e-6 as ratiotracking_transmittance_trait.h:14 floors it --
// the "own epsilon" pbvr.h:60-61 refers to. Without a floor a ray moving
// toward -x, -y or -z stops on the first voxel face it reaches (the face
// point maps back to the voxel it leaves, whose exit distance is then 0).
// hg_phase_sample and create_ortho_basis follow
// rdv/shaders/libraries/random_library.h:224-239 and math_library.h:323-330.
// Every march operation is a separately rounded fp32 operation; log, sin,
// cos, asin and atan2 are CUDA's.
//
// Environment: a constant RGB (a Constant map), or an equirectangular image
// looked up with XRProject >> TensorSampler (math_library.h dir2xr: asin of
// w.y and atan(w.x, w.z), scaled by 1/pi and 2/pi; then the 2-D sampler).
//
// Work is warp-coherent, as in ratiotracking_kernel: each lane runs its ray's
// free flights until a tentative collision, then the warp evaluates the MLP
// together.
#pragma once
#include "sampler.cuh"
#include "transmittance.cuh"

namespace rdvb {
namespace pbvr {

using trm::Params;
constexpr int kSafety = 8192;  // pbvr.h's loop cap
constexpr float kPi = 3.14159265358979323846f;
constexpr float kInvPi = 0.318309886183790671538f;

struct Extra {
    float albedo[3];
    float g;
    int max_bounces;
    int env_kind;          // 0 constant, 1 equirectangular image
    float env_rgb[3];
    const float* env;      // [H, W, 3] fp32 (env_kind 1)
    int env_h, env_w;
    int env_clamp, env_aligned, env_linear;
    float* out;            // [n_rays, 3]
};

// dir2xr (math_library.h:265-276): a direction's equirectangular
// coordinates (atan(w.x, w.z) / pi, asin(w.y) * 2 / pi). The reference always
// adds 0 or 1e-7 to w.x, which turns a -0 x into +0 before atan.
__device__ __forceinline__ void dir2xr(const float (&w)[3], float& u, float& v) {
    const float wx = __fadd_rn(w[0], (w[0] == 0.0f && w[2] == 0.0f) ? 1e-7f : 0.0f);
    const float beta = asinf(fminf(fmaxf(w[1], -1.0f), 1.0f));
    const float alpha = atan2f(wx, w[2]);
    u = __fmul_rn(alpha, kInvPi);
    v = __fmul_rn(beta, __fmul_rn(2.0f, kInvPi));
}

// XRProject as a map of its own: [n, 3] directions -> [n, 2].
__global__ void xr_project_kernel(const float* __restrict__ dirs, long long n, float* __restrict__ out) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const float w[3] = {__ldg(dirs + 3 * i), __ldg(dirs + 3 * i + 1), __ldg(dirs + 3 * i + 2)};
        float u, v;
        dir2xr(w, u, v);
        out[2 * i] = u;
        out[2 * i + 1] = v;
    }
}

// world direction -> environment radiance
__device__ __forceinline__ void environment(const Extra& e, const float (&w)[3], float (&c)[3]) {
    if (e.env_kind == 0) {
        c[0] = e.env_rgb[0];
        c[1] = e.env_rgb[1];
        c[2] = e.env_rgb[2];
        return;
    }
    float u, v;
    dir2xr(w, u, v);
#pragma unroll
    for (int k = 0; k < 3; ++k)
        c[k] = sampler::sample2(e.env, e.env_h, e.env_w, 3, k, u, v, e.env_clamp != 0, e.env_aligned != 0,
                                e.env_linear != 0);
}

// create_ortho_basis (math_library.h:323-330)
__device__ __forceinline__ void ortho_basis(const float (&n)[3], float (&t)[3], float (&b)[3]) {
    const float sign = n[2] >= 0.0f ? 1.0f : -1.0f;
    const float a = __fdiv_rn(-1.0f, __fadd_rn(sign, n[2]));
    const float bb = __fmul_rn(__fmul_rn(n[0], n[1]), a);
    t[0] = __fadd_rn(1.0f, __fmul_rn(__fmul_rn(__fmul_rn(sign, n[0]), n[0]), a));
    t[1] = __fmul_rn(sign, bb);
    t[2] = -__fmul_rn(sign, n[0]);
    b[0] = bb;
    b[1] = __fadd_rn(sign, __fmul_rn(__fmul_rn(n[1], n[1]), a));
    b[2] = -n[1];
}

// hg_phase_sample (random_library.h:224-239): two draws (phi, then xi).
__device__ __forceinline__ void hg_sample(Rng& r, float g, float (&w)[3]) {
    const float phi = __fmul_rn(__fmul_rn(rng_uniform(r), 2.0f), kPi);
    const float xi = rng_uniform(r);
    const float g2 = __fmul_rn(g, g);
    const float one_minus_g2 = __fsub_rn(1.0f, g2);
    const float one_plus_g2 = __fadd_rn(1.0f, g2);
    const float one_over_2g = __fdiv_rn(0.5f, g);
    const float t = __fdiv_rn(one_minus_g2, __fadd_rn(__fsub_rn(1.0f, g), __fmul_rn(__fmul_rn(2.0f, g), xi)));
    const float invertcdf = __fmul_rn(one_over_2g, __fsub_rn(one_plus_g2, __fmul_rn(t, t)));
    const float cos_t = fabsf(g) < 0.001f ? __fsub_rn(__fmul_rn(2.0f, xi), 1.0f) : invertcdf;
    const float sin_t = __fsqrt_rn(fmaxf(0.0f, __fsub_rn(1.0f, __fmul_rn(cos_t, cos_t))));
    float t0[3], t1[3];
    ortho_basis(w, t0, t1);
    const float s0 = __fmul_rn(sin_t, sinf(phi)), s1 = __fmul_rn(sin_t, cosf(phi));
#pragma unroll
    for (int k = 0; k < 3; ++k)
        w[k] = __fadd_rn(__fadd_rn(__fmul_rn(s0, t0[k]), __fmul_rn(s1, t1[k])), __fmul_rn(cos_t, w[k]));
}

// wo = L w (the node's inverse 3x3, row-major), each sum rounded in order.
__device__ __forceinline__ void to_object(const float (&L)[9], const float (&w)[3], float (&wo)[3]) {
#pragma unroll
    for (int i = 0; i < 3; ++i)
        wo[i] = __fadd_rn(__fadd_rn(__fmul_rn(L[3 * i], w[0]), __fmul_rn(L[3 * i + 1], w[1])),
                          __fmul_rn(L[3 * i + 2], w[2]));
}

// ray_box_intersection (math_library.h:48-57) from x along w: tMax =
// min(min(c.x, c.y), c.z) with c = -x / w + |1 / w| (GLSL min(a, b) = b < a ?
// b : a).
__device__ __forceinline__ float slab_exit(const float (&x)[3], const float (&w)[3]) {
    float c[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const float inv = __fdiv_rn(1.0f, w[k]);
        c[k] = __fadd_rn(__fmul_rn(-x[k], inv), fabsf(inv));
    }
    const float m = c[1] < c[0] ? c[1] : c[0];
    return c[2] < m ? c[2] : m;
}

template <int NT, bool ENC>
__global__ void __launch_bounds__(NT) pbvr_kernel(const __grid_constant__ Params p, const __grid_constant__ Extra e) {
    extern __shared__ float sm[];
    float* wsm = sm;
    float* act0 = sm + ((p.w_floats + 3) & ~3) + threadIdx.x;
    float* act1 = act0 + p.maxw * NT;
    trm::stage_chain<NT>(p, wsm);
    const float* bsm = wsm;
    unsigned long long my_evals = 0;
    long long ray = -1;  // -1: take the next ray; -2: none left
    float x[3] = {0.0f, 0.0f, 0.0f}, w[3] = {0.0f, 0.0f, 1.0f}, wo[3] = {0.0f, 0.0f, 1.0f};
    float d = 0.0f, maj = 1.0f, W[3] = {1.0f, 1.0f, 1.0f};
    int safety = 0, bounces = 0;
    Rng r = {0u, 0u, 0u, 0u};
    auto finish = [&](float c0, float c1, float c2) {
        e.out[ray * 3 + 0] = c0;
        e.out[ray * 3 + 1] = c1;
        e.out[ray * 3 + 2] = c2;
        ray = -1;
    };
    while (true) {
        bool pending = false;  // a tentative collision at x waits for its extinction
        // at most kYieldFlights free flights per lane between two extinction
        // rounds, so that a lane stuck in a long run of free flights does
        // not hold the warp's colliding lanes back
        for (int flights = 0; ray != -2 && !pending && flights < trm::kYieldFlights; ++flights) {
            if (ray < 0) {
                ray = atomicAdd(p.counter, 1);
                if (ray >= p.n_rays) {
                    ray = -2;
                    break;
                }
                const float* rr = p.rays + ray * 6;
                w[0] = rr[3];
                w[1] = rr[4];
                w[2] = rr[5];
                if (!trm::march_entry(rr, p.L, p.O, x, wo, d)) {
                    float c[3];
                    environment(e, w, c);  // the ray never touches the volume
                    finish(c[0], c[1], c[2]);
                    continue;
                }
                W[0] = W[1] = W[2] = 1.0f;
                safety = 0;
                bounces = 0;
                r = rng_spawn(p.seeds, static_cast<unsigned>(ray));
                for (int k = 0; k < p.draws_before; ++k) rng_step(r);
            }
            if (!(d > 0.0f) || safety >= kSafety) {  // the loop ended without escaping
                finish(0.0f, 0.0f, 0.0f);
                continue;
            }
            ++safety;
            float max_step;
            maj = trm::field_majorant(p, x, wo, max_step);
            maj = maj < 1e-12f ? 1e-12f : maj;                      // max(majorant, 1e-12)
            max_step = max_step < 1e-6f ? 1e-6f : max_step;         // local_majorant's floor
            const float dt = __fdiv_rn(-logf(__fsub_rn(1.0f, rng_uniform(r))), maj);
            const float m = d < max_step ? d : max_step;    // min(max_step, d)
            const float step = m < dt ? m : dt;              // min(dt, .)
#pragma unroll
            for (int k = 0; k < 3; ++k) x[k] = __fadd_rn(x[k], __fmul_rn(step, wo[k]));
            d = __fsub_rn(d, step);
            if (step < dt) {
                if (d <= 0.0f) {  // reached the boundary without a collision
                    float c[3];
                    environment(e, w, c);
                    finish(__fmul_rn(W[0], c[0]), __fmul_rn(W[1], c[1]), __fmul_rn(W[2], c[2]));
                }
                continue;  // (or: a new majorant cell)
            }
            pending = true;
        }
        if (!__any_sync(0xffffffffu, pending)) {
            if (__all_sync(0xffffffffu, ray == -2)) break;  // no lane has rays left
            continue;
        }
        const float sigma = trm::extinction<NT, ENC>(p, wsm, bsm, act0, act1, x);
        if (pending) {
            ++my_evals;
            if (rng_uniform(r) >= __fdiv_rn(sigma, maj)) continue;  // null collision
#pragma unroll
            for (int k = 0; k < 3; ++k) W[k] = __fmul_rn(W[k], e.albedo[k]);
            const float wmax = fmaxf(fmaxf(W[0], W[1]), W[2]);
            if (wmax < 0.0001f || bounces >= e.max_bounces) {
                finish(0.0f, 0.0f, 0.0f);  // throughput too low, or the bounce budget spent
                continue;
            }
            hg_sample(r, e.g, w);
            to_object(p.L, w, wo);
            d = slab_exit(x, wo);
            ++bounces;
        }
    }
    if (my_evals) atomicAdd(p.evaluations, my_evals);
}

// ---------------------------------------------------------------------------
// PBVRT, PBVR_NEE and PBVR_ENV (rdv/domain/volumes.py:326-502,
// rdv/shaders/volumes/pbvrt.h, pbvr_nee.h, pbvr_env.h): delta tracking with
// next-event estimation toward a directional light (PBVR_ENV: toward a
// direction importance-sampled from the environment, env_sample), RGB. Per ray -- pbvrt.h:21-149:
//   object space; slab test (miss: tMax <= 0 or tMin >= tMax) -> 0 (PBVRT:
//   alpha 1); entry x <- x + w_o (max(0, tMin) + 1e-5), d <- tMax - tMin;
//   for (safety < 16384):
//     maj = majorant(x, w_o, dist) + 1e-5; dist <= 1e-5 -> 1e-5
//     dt = min(min(d, dist), -log(1 - random()) / (density_scale * maj))
//     x += dt w_o; d -= dt; dt >= dist -> continue; d <= 1e-7 -> break
//     random() >= extinction(x) / maj -> continue (null collision)
//     ++bounces > max_bounces -> PBVRT: W = 0, break; NEE: return
//     W *= albedo; no W[i] > 1e-4 -> PBVRT: break; NEE: return
//     out += W * transmittance_rt(x, L l, tMax from x) * hg_phase_eval(w . l, g)
//       (a ratio-tracking shadow ray: ratiotracking_transmittance_trait.h)
//     w <- hg_phase_sample(w, g); w_o <- L w; d <- slab exit from x
//   PBVRT after the loop, if bounces > 0: alpha 0,
//     out = out * light_intensity + W * environment(w).
// The majorant here is the field's raw (majorant, distance), as
// majorant_trait.h reads it. Each lane is a small state machine: the main
// path or its shadow ray; both stop at tentative collisions, where the warp
// evaluates the extinction together at each lane's point.
struct ExtraT {
    float albedo[3];
    float g;
    float density_scale;
    int max_bounces;
    int variant;             // 0 PBVRT ([n, 4]: RGB, alpha), 1 PBVR_NEE ([n, 3]), 2 PBVR_ENV ([n, 3])
    float light[3];          // normalize(light_direction), world space (host)
    float intensity[3];      // PBVRT: light_intensity
    Extra env;               // environment (PBVRT; PBVR_ENV: the sampler's) and the output pointer
    const float* densities;  // PBVR_ENV: the quadtree's cumulative child probabilities, 4 per node
    int levels;              // PBVR_ENV: its depth
};

constexpr float kPiOverTwo = 1.57079632679489661923f;

// XREnvironmentSampler.forward (rdv/domain/rendering.py:281-323,
// rdv/shaders/rendering/xr_environment_sampler.h): one draw walks the
// quadtree (rescaled to [0, 1) at every level), the leaf's probability is
// the product of the chosen children's; two more draws place the direction
// uniformly in solid angle inside the leaf pixel (usc2dir,
// math_library.h:256-263); returns the direction and the environment there
// times 1 / pdf. GLSL mix(a, b, t) = a (1 - t) + b t.
__device__ __forceinline__ void env_sample(const ExtraT& e, Rng& r, float (&dir)[3], float (&val)[3]) {
    int node = 0;
    float u0 = 0.0f, u1 = 1.0f, v0 = 0.0f, v1 = 1.0f, prob = 1.0f;
    float sel = rng_uniform(r);
    for (int i = 0; i < e.levels; ++i) {
        const float* cdf = e.densities + node * 4;
        int child = 3;
        float lo = 0.0f, hi = __ldg(cdf + 3);
        for (int c = 0; c < 3; ++c) {
            const float cc = __ldg(cdf + c);
            if (sel < cc) {
                child = c;
                hi = cc;
                break;
            }
            lo = cc;
        }
        const float span = __fsub_rn(hi, lo);
        prob = __fmul_rn(prob, 0.0f < span ? span : 0.0f);               // max(0, hi - lo)
        float q = __fdiv_rn(__fsub_rn(sel, lo), 1e-9f < span ? span : 1e-9f);
        q = q < 0.0f ? 0.0f : q;                                         // clamp(., 0, 1)
        sel = 1.0f < q ? 1.0f : q;
        const float umed = __fmul_rn(__fadd_rn(u0, u1), 0.5f), vmed = __fmul_rn(__fadd_rn(v0, v1), 0.5f);
        if (child % 2 == 0) u1 = umed; else u0 = umed;
        if (child / 2 == 0) v1 = vmed; else v0 = vmed;
        node = node * 4 + 1 + child;
    }
    const float a0 = __fmul_rn(__fsub_rn(__fmul_rn(u0, 2.0f), 1.0f), kPi);
    const float a1 = __fmul_rn(__fsub_rn(__fmul_rn(u1, 2.0f), 1.0f), kPi);
    const float b0 = __fmul_rn(__fsub_rn(__fmul_rn(v0, 2.0f), 1.0f), kPiOverTwo);
    const float b1 = __fmul_rn(__fsub_rn(__fmul_rn(v1, 2.0f), 1.0f), kPiOverTwo);
    const float sb0 = sinf(b0), sb1 = sinf(b1);
    const float solid = __fmul_rn(__fsub_rn(a1, a0), __fsub_rn(sb1, sb0));
    const float pdf = __fdiv_rn(prob, 1e-9f < solid ? solid : 1e-9f);
    const float weight = __fdiv_rn(1.0f, 1e-9f < pdf ? pdf : 1e-9f);
    const float ta = rng_uniform(r);
    const float alpha = __fadd_rn(__fmul_rn(a0, __fsub_rn(1.0f, ta)), __fmul_rn(a1, ta));
    const float ts = rng_uniform(r);
    float sv = __fadd_rn(__fmul_rn(sb0, __fsub_rn(1.0f, ts)), __fmul_rn(sb1, ts));
    sv = sv < -1.0f ? -1.0f : sv;
    sv = 1.0f < sv ? 1.0f : sv;
    const float beta = asinf(sv);
    const float rr = cosf(beta);
    dir[0] = __fmul_rn(sinf(alpha), rr);
    dir[1] = sinf(beta);
    dir[2] = __fmul_rn(cosf(alpha), rr);
    float c[3];
    environment(e.env, dir, c);
#pragma unroll
    for (int k = 0; k < 3; ++k) val[k] = __fmul_rn(c[k], weight);
}

constexpr int kSafetyT = 16384;   // pbvrt.h / pbvr_nee.h loop cap

// hg_phase_eval (random_library.h:241-249) at cos_theta
__device__ __forceinline__ float hg_eval(float cos_t, float g) {
    if (fabsf(g) < 0.001f) return __fdiv_rn(0.25f, kPi);
    const float g2 = __fmul_rn(g, g);
    const float omg2 = __fsub_rn(1.0f, g2), opg2 = __fadd_rn(1.0f, g2);
    const float base = __fsub_rn(opg2, __fmul_rn(__fmul_rn(2.0f, g), cos_t));
    return __fdiv_rn(__fmul_rn(__fdiv_rn(0.25f, kPi), omg2), powf(base, 1.5f));
}

// ENC: whether the launch has an input encoding (its sampler code is
// compiled only into those instantiations).
// VAR = e.variant at compile time: each variant keeps only its own code
// (PBVRT's escape term, PBVR_ENV's environment sampling), and every path
// end (loop_end, shadow_end) is taken at one site at the top of the flight
// loop -- the kernel measured instruction-cache bound (75 % hit rate) with
// all three variants and these ends inlined at each of their 7 call sites.
template <int NT, int VAR, bool ENC>
__global__ void __launch_bounds__(NT) pbvrt_kernel(const __grid_constant__ Params p, const __grid_constant__ ExtraT e) {
    extern __shared__ float sm[];
    float* wsm = sm;
    float* act0 = sm + ((p.w_floats + 3) & ~3) + threadIdx.x;
    float* act1 = act0 + p.maxw * NT;
    trm::stage_chain<NT>(p, wsm);
    const float* bsm = wsm;
    constexpr int n_out = VAR == 0 ? 4 : 3;
    float* out_ptr = e.env.out;
    // the NEE direction (world, object space) and the weight its term takes:
    // the directional light of PBVRT / PBVR_NEE (weight 1), or each
    // collision's environment sample of PBVR_ENV (radiance / pdf)
    float ld[3] = {e.light[0], e.light[1], e.light[2]}, lo[3], ew[3] = {1.0f, 1.0f, 1.0f};
    to_object(p.L, ld, lo);
    unsigned long long my_evals = 0;
    long long ray = -1;  // -1: take the next ray; -2: none left
    float x[3] = {0.0f, 0.0f, 0.0f}, w[3] = {0.0f, 0.0f, 1.0f}, wo[3] = {0.0f, 0.0f, 1.0f};
    float d = 0.0f, maj = 1.0f, W[3] = {1.0f, 1.0f, 1.0f}, acc[3] = {0.0f, 0.0f, 0.0f};
    int safety = 0, bounces = 0;
    // shadow ray (mode 1): point, remaining distance, transmittance, its own cap, the phase
    int mode = 0;
    float xs[3] = {0.0f, 0.0f, 0.0f}, ds = 0.0f, T = 1.0f, phase = 0.0f;
    int s_safety = 0;
    Rng r = {0u, 0u, 0u, 0u};
    auto store = [&](float a0, float a1, float a2, float alpha) {
        out_ptr[ray * n_out + 0] = a0;
        out_ptr[ray * n_out + 1] = a1;
        out_ptr[ray * n_out + 2] = a2;
        if (n_out == 4) out_ptr[ray * n_out + 3] = alpha;
        ray = -1;
    };
    // the main loop ended (cap, break): PBVRT resolves the escape term
    auto loop_end = [&]() {
        if constexpr (VAR != 0) {
            store(acc[0], acc[1], acc[2], 0.0f);
            return;
        }
        if (bounces > 0) {
            float c[3];
            environment(e.env, w, c);
            store(__fadd_rn(__fmul_rn(acc[0], e.intensity[0]), __fmul_rn(W[0], c[0])),
                  __fadd_rn(__fmul_rn(acc[1], e.intensity[1]), __fmul_rn(W[1], c[1])),
                  __fadd_rn(__fmul_rn(acc[2], e.intensity[2]), __fmul_rn(W[2], c[2])), 0.0f);
        } else {
            store(0.0f, 0.0f, 0.0f, 1.0f);
        }
    };
    // the shadow ray ended with transmittance t: add its NEE term, scatter
    auto shadow_end = [&](float t) {
        const float tr = __fmul_rn(t, phase);
        // PBVRT / NEE: out += W tr; ENV: out += (tr W) env (ew = 1 for the former)
#pragma unroll
        for (int k = 0; k < 3; ++k) acc[k] = __fadd_rn(acc[k], __fmul_rn(__fmul_rn(tr, W[k]), ew[k]));
        hg_sample(r, e.g, w);
        to_object(p.L, w, wo);
        d = slab_exit(x, wo);
        mode = 0;
    };
    // a path end to take at the top of the next flight: 1 the main loop
    // ended (loop_end), 2 the shadow ray ended with transmittance fin_t
    int fin = 0;
    float fin_t = 0.0f;
    while (true) {
        bool pending = false;
        for (int flights = 0; ray != -2 && !pending && flights < trm::kYieldFlights; ++flights) {
            if (fin != 0) {
                if (fin == 1) loop_end();
                else shadow_end(fin_t);
                fin = 0;
                continue;
            }
            if (ray < 0) {
                ray = atomicAdd(p.counter, 1);
                if (ray >= p.n_rays) {
                    ray = -2;
                    break;
                }
                const float* rr = p.rays + ray * 6;
                w[0] = rr[3];
                w[1] = rr[4];
                w[2] = rr[5];
                // object space and slab test (pbvrt.h:25-41)
                float xr[3];
#pragma unroll
                for (int k = 0; k < 3; ++k) xr[k] = __fsub_rn(rr[k], p.O[k]);
                to_object(p.L, xr, x);
                to_object(p.L, w, wo);
                float tmin = -INFINITY, tmax = INFINITY;
#pragma unroll
                for (int k = 0; k < 3; ++k) {
                    const float inv = __fdiv_rn(1.0f, wo[k]);
                    const float xc = __fmul_rn(-x[k], inv);
                    const float sabs = fabsf(inv);
                    const float lo_k = __fsub_rn(xc, sabs), hi_k = __fadd_rn(xc, sabs);
                    tmin = tmin < lo_k ? lo_k : tmin;   // GLSL max
                    tmax = hi_k < tmax ? hi_k : tmax;   // GLSL min
                }
                if (tmax <= 0.0f || tmin >= tmax) {
                    store(0.0f, 0.0f, 0.0f, 1.0f);
                    continue;
                }
                tmin = __fadd_rn(0.0f < tmin ? tmin : 0.0f, 1e-5f);
#pragma unroll
                for (int k = 0; k < 3; ++k) x[k] = __fadd_rn(x[k], __fmul_rn(wo[k], tmin));
                d = __fsub_rn(tmax, tmin);
                W[0] = W[1] = W[2] = 1.0f;
                acc[0] = acc[1] = acc[2] = 0.0f;
                safety = 0;
                bounces = 0;
                mode = 0;
                r = rng_spawn(p.seeds, static_cast<unsigned>(ray));
                for (int k = 0; k < p.draws_before; ++k) rng_step(r);
            }
            // one free flight of the main path (pbvrt.h / pbvr_nee.h: majorant
            // + 1e-5, distance floored at 1e-5) or of the shadow ray
            // (transmittance_rt, ratiotracking_transmittance_trait.h:1-31:
            // majorant floored at 1e-12, distance at 1e-6), written once for
            // both so the majorant lookup and the sample are inlined once
            const bool main_path = mode == 0;
            if (main_path) {
                if (safety >= kSafetyT) {  // the loop ran out
                    fin = 1;
                    continue;
                }
                ++safety;
            } else {
                if (!(ds > 0.0f) || s_safety >= trm::kRtSafety) {
                    fin = 2;
                    fin_t = T;
                    continue;
                }
                ++s_safety;
            }
            float qx[3], qw[3];
#pragma unroll
            for (int k = 0; k < 3; ++k) {
                qx[k] = main_path ? x[k] : xs[k];
                qw[k] = main_path ? wo[k] : lo[k];
            }
            float dist;
            float mj = trm::field_majorant(p, qx, qw, dist);
            if (main_path) {
                mj = __fadd_rn(mj, 1e-5f);
                if (dist <= 1e-5f) dist = 1e-5f;
            } else {
                mj = mj < 1e-12f ? 1e-12f : mj;
                dist = dist < 1e-6f ? 1e-6f : dist;
            }
            maj = mj;
            const float q = __fdiv_rn(-logf(__fsub_rn(1.0f, rng_uniform(r))), __fmul_rn(e.density_scale, mj));
            const float rem = main_path ? d : ds;
            const float lim = main_path ? (dist < rem ? dist : rem) : dist;  // min(d, dist) / dist
            const float dt = q < lim ? q : lim;                                // min(., q)
#pragma unroll
            for (int k = 0; k < 3; ++k) qx[k] = __fadd_rn(qx[k], __fmul_rn(dt, qw[k]));
            const float left = __fsub_rn(rem, dt);
            if (main_path) {
#pragma unroll
                for (int k = 0; k < 3; ++k) x[k] = qx[k];
                d = left;
            } else {
#pragma unroll
                for (int k = 0; k < 3; ++k) xs[k] = qx[k];
                ds = left;
            }
            if (dt >= dist) continue;
            if (main_path ? left <= 1e-7f : left <= 0.0f) {
                fin = main_path ? 1 : 2;
                fin_t = T;
                continue;
            }
            pending = true;
        }
        if (!__any_sync(0xffffffffu, pending)) {
            if (__all_sync(0xffffffffu, ray == -2)) break;  // no lane has rays left
            continue;
        }
        float pt[3];
#pragma unroll
        for (int k = 0; k < 3; ++k) pt[k] = mode == 0 ? x[k] : xs[k];
        const float sigma = trm::extinction<NT, ENC>(p, wsm, bsm, act0, act1, pt);
        if (!pending) continue;
        ++my_evals;
        if (mode == 1) {
            T = __fmul_rn(T, __fsub_rn(1.0f, __fdiv_rn(sigma, maj)));
            if (T < 0.05f) {
                if (rng_uniform(r) >= T) {
                    fin = 2;
                    fin_t = 0.0f;
                    continue;
                }
                T = 1.0f;
            }
            continue;
        }
        if (rng_uniform(r) >= __fdiv_rn(sigma, maj)) continue;  // null collision
        ++bounces;
        if (bounces > e.max_bounces) {
            if constexpr (VAR == 0) W[0] = W[1] = W[2] = 0.0f;
            fin = 1;
            continue;
        }
#pragma unroll
        for (int k = 0; k < 3; ++k) W[k] = __fmul_rn(W[k], e.albedo[k]);
        if (!(W[0] > 0.0001f || W[1] > 0.0001f || W[2] > 0.0001f)) {
            fin = 1;
            continue;
        }
        // next-event estimation toward the light (or the environment
        // sample): phase, then the shadow ray
        if constexpr (VAR == 2) {
            env_sample(e, r, ld, ew);
            to_object(p.L, ld, lo);
        }
        const float cos_t = __fadd_rn(__fadd_rn(__fmul_rn(w[0], ld[0]), __fmul_rn(w[1], ld[1])),
                                      __fmul_rn(w[2], ld[2]));
        phase = hg_eval(cos_t, e.g);
        xs[0] = x[0];
        xs[1] = x[1];
        xs[2] = x[2];
        ds = slab_exit(x, lo);
        T = 1.0f;
        s_safety = 0;
        mode = 1;
    }
    if (my_evals) atomicAdd(p.evaluations, my_evals);
}

}  // namespace pbvr
}  // namespace rdvb
