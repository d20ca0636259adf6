// Test infrastructure only (parity checker, never shipped or measured).
//
// Compiles the reference's PBVR delta-tracking body (rdv/shaders/volumes/
// pbvr.h) and its Henyey-Greenstein sampler (libraries/random_library.h) as
// C++, for the golden vectors of tests/golden/pbvr.npz. Both come from
// copies under _ref/gen/pbvr written by oracle/Makefile with two mechanical
// changes: GLSL array constructors `float[](...)` become `rdv_farr(...)`,
// and unsuffixed floating literals get an `f` (in GLSL they are float, in
// C++ double; without it `0.5 / g` would divide in double). random_library.h
// also gets the `inout uvec4` -> `uvec4&` change of libref_shaders.so.
//
// Restated here (the reference's versions do not compile as C++):
//   ray_box_intersection, create_ortho_basis   math_library.h:48-57, 323-330
//   the VoxelMajorantField                     voxel_majorant_field.h
//   the SphereMajorantField                    sphere_majorant_field.h
// local_majorant itself comes from volumes/majorant_field_precode.h, which
// the reference checkout does not contain: it is taken as the field's
// (majorant, distance) as majorant_trait.h reads a Map[6, 2], with the
// distance floored at 1e-6 as ratiotracking_transmittance_trait.h:14 does.
// The node's mat3 inverse is formed in double and rounded (GLSL leaves its
// precision to the implementation); the pins use transforms whose inverse
// is exact either way. The extinction is the analytic field
// c0 + c1 |x|^2 of libref_shaders.so's tracking pins; the environment a
// constant RGB.
#include "glsl_prelude.hpp"

#include <array>

// -- GLSL pieces the PBVR body uses on top of glsl_prelude.hpp ---------------
template <int N>
struct rdv_farr_t {
    float v[N];
    operator float*() { return v; }
};
template <typename... T>
static inline rdv_farr_t<sizeof...(T)> rdv_farr(T... a) { return {{static_cast<float>(a)...}}; }

static inline rdv_vec3 operator-(rdv_vec3 a, rdv_vec3 b) { return rdv_vec3(a.x - b.x, a.y - b.y, a.z - b.z); }
static inline rdv_vec3 operator-(rdv_vec3 a) { return rdv_vec3(-a.x, -a.y, -a.z); }
static inline rdv_vec3& operator*=(rdv_vec3& a, rdv_vec3 b) { a.x *= b.x; a.y *= b.y; a.z *= b.z; return a; }

struct rdv_mat4x3 {
    rdv_vec3 c[4];
    rdv_vec3& operator[](int i) { return c[i]; }
};
struct rdv_mat3 {
    rdv_vec3 c[3];  // columns
    rdv_mat3() {}
    explicit rdv_mat3(rdv_mat4x3 m) { c[0] = m.c[0]; c[1] = m.c[1]; c[2] = m.c[2]; }
};
// column-major product: (L v)_i = (L[0]_i v.x + L[1]_i v.y) + L[2]_i v.z
static inline rdv_vec3 operator*(rdv_mat3 L, rdv_vec3 v) {
    return rdv_vec3(L.c[0].x * v.x + L.c[1].x * v.y + L.c[2].x * v.z,
                    L.c[0].y * v.x + L.c[1].y * v.y + L.c[2].y * v.z,
                    L.c[0].z * v.x + L.c[1].z * v.y + L.c[2].z * v.z);
}
static rdv_mat3 inverse(rdv_mat3 m) {
    double M[3][3];  // M[row][col]
    const rdv_vec3* c = m.c;
    for (int j = 0; j < 3; ++j) { M[0][j] = c[j].x; M[1][j] = c[j].y; M[2][j] = c[j].z; }
    const double det = M[0][0] * (M[1][1] * M[2][2] - M[1][2] * M[2][1]) -
                       M[0][1] * (M[1][0] * M[2][2] - M[1][2] * M[2][0]) +
                       M[0][2] * (M[1][0] * M[2][1] - M[1][1] * M[2][0]);
    double I[3][3];
    I[0][0] = (M[1][1] * M[2][2] - M[1][2] * M[2][1]) / det;
    I[0][1] = (M[0][2] * M[2][1] - M[0][1] * M[2][2]) / det;
    I[0][2] = (M[0][1] * M[1][2] - M[0][2] * M[1][1]) / det;
    I[1][0] = (M[1][2] * M[2][0] - M[1][0] * M[2][2]) / det;
    I[1][1] = (M[0][0] * M[2][2] - M[0][2] * M[2][0]) / det;
    I[1][2] = (M[0][2] * M[1][0] - M[0][0] * M[1][2]) / det;
    I[2][0] = (M[1][0] * M[2][1] - M[1][1] * M[2][0]) / det;
    I[2][1] = (M[0][1] * M[2][0] - M[0][0] * M[2][1]) / det;
    I[2][2] = (M[0][0] * M[1][1] - M[0][1] * M[1][0]) / det;
    rdv_mat3 r;
    for (int j = 0; j < 3; ++j) r.c[j] = rdv_vec3((float)I[0][j], (float)I[1][j], (float)I[2][j]);
    return r;
}
#define mat4x3 rdv_mat4x3
#define mat3 rdv_mat3

// GLSL min / max: min(a, b) = b < a ? b : a, max(a, b) = a < b ? b : a
static inline float gmin(float a, float b) { return b < a ? b : a; }
static inline float gmax(float a, float b) { return a < b ? b : a; }

// math_library.h:48-57
static void ray_box_intersection(rdv_vec3 x, rdv_vec3 w, float& tMin, float& tMax) {
    const float inv[3] = {1.0f / w.x, 1.0f / w.y, 1.0f / w.z};
    const float xs[3] = {x.x, x.y, x.z};
    float lo[3], hi[3];
    for (int k = 0; k < 3; ++k) {
        const float xc = -xs[k] * inv[k];
        const float s = std::fabs(inv[k]);
        lo[k] = xc - s;
        hi[k] = xc + s;
    }
    tMin = gmax(gmax(lo[0], lo[1]), lo[2]);
    tMax = gmin(gmin(hi[0], hi[1]), hi[2]);
}

// math_library.h:323-330
static void create_ortho_basis(rdv_vec3 N, rdv_vec3& T, rdv_vec3& B) {
    const float sign = N.z >= 0 ? 1.0f : -1.0f;
    const float a = -1.0f / (sign + N.z);
    const float b = N.x * N.y * a;
    T = rdv_vec3(1.0f + sign * N.x * N.x * a, sign * b, -sign * N.x);
    B = rdv_vec3(b, sign + N.y * N.y * a, -N.y);
}

// -- the generator and its samplers (random_library.h) -----------------------
#define vec2 rdv_vec2
#define vec4 rdv_vec4
#define uvec4 rdv_uvec4
#define uvec3 rdv_uvec3
#define layout(...)
#define uniform static struct
#define pi 3.1415926535897932384626433832795f
#define two_pi 6.283185307179586476925286766559f
#define log(x) rdv_log(x)
#define random rdv_random  // stdlib's long random(void) has the same name
static float min(float a, float b) { return a < b ? a : b; }
static inline float abs(float v) { return std::fabs(v); }
// GLSL's sin / cos / sqrt / pow of a float are float: without these the
// global double overloads would round sinTheta * sin(phi) once, in double.
// Each is evaluated in double and rounded to float once (see rdv_log).
#define sin(x) static_cast<float>(std::sin(static_cast<double>(static_cast<float>(x))))
#define cos(x) static_cast<float>(std::cos(static_cast<double>(static_cast<float>(x))))
#define sqrt(x) std::sqrt(static_cast<float>(x))
#define pow(a, b) static_cast<float>(std::pow(static_cast<double>(static_cast<float>(a)), \
                                              static_cast<double>(static_cast<float>(b))))
#define RDV_NODE rdv_random_init
#include "random_library.h"
#undef RDV_NODE

// -- the majorant fields (Map[6, 2]: (x, w) -> majorant, distance) ----------
struct VoxelField {
    const float* grid;  // [D, H, W]
    int gd, gh, gw;
};
struct SphereField {
    const float* grid;  // [D, H, W, 2] (majorant, radius in voxels)
    int gd, gh, gw;
};
static void field_cell(int gd, int gh, int gw, rdv_vec3 x, int cell[3]) {
    const int dim[3] = {gw, gh, gd};
    const float xs[3] = {x.x, x.y, x.z};
    for (int k = 0; k < 3; ++k) {
        int c = (int)((xs[k] * 0.5f + 0.5f) * (float)dim[k]);
        cell[k] = c < 0 ? 0 : (c > dim[k] - 1 ? dim[k] - 1 : c);
    }
}
// voxel_majorant_field.h: the cell's majorant, the distance to the cell's exit
static float voxel_field(VoxelField f, rdv_vec3 x, rdv_vec3 w, float& max_step) {
    int cell[3];
    field_cell(f.gd, f.gh, f.gw, x, cell);
    const int dim[3] = {f.gw, f.gh, f.gd};
    const float xs[3] = {x.x, x.y, x.z}, ws[3] = {w.x, w.y, w.z};
    float texit[3];
    for (int k = 0; k < 3; ++k) {
        const float vs = 2.0f / (float)dim[k];
        const float bmin = (float)cell[k] * vs - 1.0f;
        const float bmax = bmin + vs;
        texit[k] = gmax((bmin - xs[k]) / ws[k], (bmax - xs[k]) / ws[k]);
    }
    max_step = gmin(gmin(texit[0], texit[1]), texit[2]);
    return f.grid[((long)cell[2] * f.gh + cell[1]) * f.gw + cell[0]];
}
// sphere_majorant_field.h: the distance to the exit of the box of
// half-width radius voxels around the cell's centre, at least 1e-6
static float sphere_field(SphereField f, rdv_vec3 x, rdv_vec3 w, float& max_step) {
    int cell[3];
    field_cell(f.gd, f.gh, f.gw, x, cell);
    const int dim[3] = {f.gw, f.gh, f.gd};
    const float xs[3] = {x.x, x.y, x.z}, ws[3] = {w.x, w.y, w.z};
    const long idx = ((long)cell[2] * f.gh + cell[1]) * f.gw + cell[0];
    const float majorant = f.grid[2 * idx], radius = f.grid[2 * idx + 1];
    float texit[3];
    for (int k = 0; k < 3; ++k) {
        const float vs = 2.0f / (float)dim[k];
        const float center = ((float)cell[k] + 0.5f) * vs - 1.0f;
        const float half = radius * vs;
        texit[k] = gmax(((center - half) - xs[k]) / ws[k], ((center + half) - xs[k]) / ws[k]);
    }
    max_step = gmax(gmin(gmin(texit[0], texit[1]), texit[2]), 1e-6f);
    return majorant;
}

static float local_majorant(VoxelField f, rdv_vec3 x, rdv_vec3 w, float& max_step) {
    const float m = voxel_field(f, x, w, max_step);
    max_step = gmax(max_step, 1e-6f);
    return m;
}
static float local_majorant(SphereField f, rdv_vec3 x, rdv_vec3 w, float& max_step) {
    const float m = sphere_field(f, x, w, max_step);
    max_step = gmax(max_step, 1e-6f);
    return m;
}

// -- the extinction and the environment --------------------------------------
struct ExtNode { float c0, c1; };
static void forward(ExtNode n, float* in_, float* out_) {
    out_[0] = n.c0 + n.c1 * (in_[0] * in_[0] + in_[1] * in_[1] + in_[2] * in_[2]);
}
struct EnvConst { float r, g, b; };
static void forward(EnvConst e, float*, float* out_) { out_[0] = e.r; out_[1] = e.g; out_[2] = e.b; }

// -- PBVR nodes (field order of volumes.py PBVR: s, env, mg, transform,
// albedo, g, max_bounces) -----------------------------------------------------
template <typename MG>
struct PbvrNode {
    ExtNode s;
    EnvConst env;
    MG mg;
    rdv_mat4x3 transform;
    rdv_vec3 albedo;
    float g;
    int max_bounces;
};
typedef PbvrNode<VoxelField> PbvrVoxel;
typedef PbvrNode<SphereField> PbvrSphere;

#define RDV_NODE PbvrVoxel
#include "pbvr.h"
#undef RDV_NODE
#define RDV_NODE PbvrSphere
#include "pbvr.h"
#undef RDV_NODE

// -- PBVRT and PBVR_NEE (volumes/pbvrt.h, pbvr_nee.h) -------------------------
// Their trait helpers (extinction_trait.h, majorant_trait.h,
// scattering_albedo_trait.h, environment_trait.h: one forward() each, with
// GLSL array constructors) are restated per node below; the shadow ray is
// ratiotracking_transmittance_trait.h itself (the float-literal copy of
// libref_shaders.so), instantiated per node.
static inline rdv_vec3 normalize(rdv_vec3 v) {
    const float len = sqrt((v.x * v.x + v.y * v.y) + v.z * v.z);
    return rdv_vec3(v.x / len, v.y / len, v.z / len);
}
#define SPECTRAL_DIM 3
template <typename MG>
struct PbvrtNode {
    ExtNode ext;
    MG mg;
    EnvConst env;
    float sa[3];
    rdv_mat4x3 transform;
    rdv_vec3 light_direction;
    float light_intensity[3];
    float g;
    float density_scale;
    int max_bounces;
};
typedef PbvrtNode<VoxelField> PbvrtVoxel;
typedef PbvrtNode<SphereField> PbvrtSphere;
template <typename MG>
static float extinction(PbvrtNode<MG> node, rdv_vec3 x) {
    float in_[3] = {x.x, x.y, x.z}, v[1];
    forward(node.ext, in_, v);
    return v[0];
}
// majorant_trait.h: the field's raw (majorant, distance)
static float majorant(PbvrtNode<VoxelField> node, rdv_vec3 x, rdv_vec3 w, float& distance) {
    return voxel_field(node.mg, x, w, distance);
}
static float majorant(PbvrtNode<SphereField> node, rdv_vec3 x, rdv_vec3 w, float& distance) {
    return sphere_field(node.mg, x, w, distance);
}
template <typename MG>
static void scattering_albedo(PbvrtNode<MG> node, rdv_vec3, float* sa) {
    for (int i = 0; i < 3; ++i) sa[i] = node.sa[i];
}
template <typename MG>
static void environment(PbvrtNode<MG> node, rdv_vec3, float* env) {
    env[0] = node.env.r;
    env[1] = node.env.g;
    env[2] = node.env.b;
}
#define RDV_NODE PbvrtVoxel
#include "volumes/ratiotracking_transmittance_trait.h"
#define OUT 4
#include "pbvrt.h"
#undef OUT
#undef RDV_NODE
#define RDV_NODE PbvrtSphere
#include "volumes/ratiotracking_transmittance_trait.h"
#define OUT 4
#include "pbvrt.h"
#undef OUT
#undef RDV_NODE
// PBVR_NEE: the same node fields (environment and light_intensity unused)
struct NeeVoxel : PbvrtVoxel {};
struct NeeSphere : PbvrtSphere {};
static float extinction(NeeVoxel n, rdv_vec3 x) { return extinction(static_cast<PbvrtVoxel>(n), x); }
static float extinction(NeeSphere n, rdv_vec3 x) { return extinction(static_cast<PbvrtSphere>(n), x); }
static float majorant(NeeVoxel n, rdv_vec3 x, rdv_vec3 w, float& d) { return majorant(static_cast<PbvrtVoxel>(n), x, w, d); }
static float majorant(NeeSphere n, rdv_vec3 x, rdv_vec3 w, float& d) { return majorant(static_cast<PbvrtSphere>(n), x, w, d); }
static void scattering_albedo(NeeVoxel n, rdv_vec3 x, float* sa) { scattering_albedo(static_cast<PbvrtVoxel>(n), x, sa); }
static void scattering_albedo(NeeSphere n, rdv_vec3 x, float* sa) { scattering_albedo(static_cast<PbvrtSphere>(n), x, sa); }
#define RDV_NODE NeeVoxel
#include "volumes/ratiotracking_transmittance_trait.h"
#define OUT 3
#include "pbvr_nee.h"
#undef OUT
#undef RDV_NODE
#define RDV_NODE NeeSphere
#include "volumes/ratiotracking_transmittance_trait.h"
#define OUT 3
#include "pbvr_nee.h"
#undef OUT
#undef RDV_NODE
// -- PBVR_ENV (volumes/pbvr_env.h) with its XREnvironmentSampler
// (rendering/xr_environment_sampler.h; copy: `float[3](` -> `rdv_farr(`,
// float literals). usc2dir (math_library.h:256-263) and the
// environment_sampler trait helper (environment_sampler_trait.h) are
// restated; GLSL mix(a, b, t) = a (1 - t) + b t, clamp = min(max(x, lo), hi).
#define piOverTwo 1.5707963267948966192313216916398f
#define asin(x) static_cast<float>(std::asin(static_cast<double>(static_cast<float>(x))))
static inline float mix(float a, float b, float t) { return a * (1.0f - t) + b * t; }
static inline float clamp(float x, float lo, float hi) { return gmin(gmax(x, lo), hi); }
static rdv_vec3 usc2dir(rdv_vec2 angles) {
    const float y = sin(angles.y);
    const float r = cos(angles.y);
    const float x = sin(angles.x) * r;
    const float z = cos(angles.x) * r;
    return rdv_vec3(x, y, z);
}
struct XrEnvNode {
    EnvConst environment;
    const float* densities;
};
#define RDV_NODE XrEnvNode
#define IN 6
#define OUT 7
#define LEVELS g_env_levels
static int g_env_levels = 8;
#include "xr_environment_sampler.h"
#undef LEVELS
#undef OUT
#undef IN
#undef RDV_NODE
template <typename MG>
struct EnvNodeT : PbvrtNode<MG> {
    XrEnvNode environment_sampler;
};
typedef EnvNodeT<VoxelField> EnvVoxel;
typedef EnvNodeT<SphereField> EnvSphere;
static float extinction(EnvVoxel n, rdv_vec3 x) { return extinction(static_cast<PbvrtVoxel>(n), x); }
static float extinction(EnvSphere n, rdv_vec3 x) { return extinction(static_cast<PbvrtSphere>(n), x); }
static float majorant(EnvVoxel n, rdv_vec3 x, rdv_vec3 w, float& d) { return majorant(static_cast<PbvrtVoxel>(n), x, w, d); }
static float majorant(EnvSphere n, rdv_vec3 x, rdv_vec3 w, float& d) { return majorant(static_cast<PbvrtSphere>(n), x, w, d); }
static void scattering_albedo(EnvVoxel n, rdv_vec3 x, float* sa) { scattering_albedo(static_cast<PbvrtVoxel>(n), x, sa); }
static void scattering_albedo(EnvSphere n, rdv_vec3 x, float* sa) { scattering_albedo(static_cast<PbvrtSphere>(n), x, sa); }
template <typename MG>
static rdv_vec3 environment_sampler(EnvNodeT<MG> node, rdv_vec3 x, rdv_vec3 win, float* env) {
    float in6[6] = {x.x, x.y, x.z, win.x, win.y, win.z}, result[7];
    forward(node.environment_sampler, in6, result);
    for (int i = 0; i < SPECTRAL_DIM; i++) env[i] = result[3 + i];
    return rdv_vec3(result[0], result[1], result[2]);
}
#define RDV_NODE EnvVoxel
#include "volumes/ratiotracking_transmittance_trait.h"
#define OUT 3
#include "pbvr_env.h"
#undef OUT
#undef RDV_NODE
#define RDV_NODE EnvSphere
#include "volumes/ratiotracking_transmittance_trait.h"
#define OUT 3
#include "pbvr_env.h"
#undef OUT
#undef RDV_NODE
#undef log
#undef random

template <typename Node>
static void run(Node node, const unsigned* seeds, const float* rays, long n, float* dst) {
    for (long r = 0; r < n; ++r) {
        random_seeds.seeds = rdv_uvec4(seeds[0], seeds[1], seeds[2], seeds[3]);
        rdv_random_init(rdv_uvec3{(unsigned)r, 0u, 0u});
        float in6[6];
        for (int k = 0; k < 6; ++k) in6[k] = rays[r * 6 + k];
        forward(node, in6, dst + r * 3);
    }
}

template <typename Node>
static void setup(Node& node, float c0, float c1, const float* env_rgb, const float* transform,
                  const float* albedo, float g, int max_bounces) {
    node.s = ExtNode{c0, c1};
    node.env = EnvConst{env_rgb[0], env_rgb[1], env_rgb[2]};
    for (int j = 0; j < 4; ++j)
        node.transform.c[j] = rdv_vec3(transform[3 * j], transform[3 * j + 1], transform[3 * j + 2]);
    node.albedo = rdv_vec3(albedo[0], albedo[1], albedo[2]);
    node.g = g;
    node.max_bounces = max_bounces;
}

extern "C" {

// PBVR.forward for rays [n, 6] (ray r on invocation r's generator):
// out [n, 3]. field_kind 0: voxel grid [gd, gh, gw]; 1: sphere grid
// [gd, gh, gw, 2]. transform: mat4x3, 12 floats column-major.
void ref_pbvr(float c0, float c1, int field_kind, const float* grid, int gd, int gh, int gw, const float* env_rgb,
              const float* transform, const float* albedo, float g, int max_bounces, const unsigned* seeds,
              const float* rays, long n, float* dst) {
    if (field_kind == 0) {
        PbvrVoxel node;
        setup(node, c0, c1, env_rgb, transform, albedo, g, max_bounces);
        node.mg = VoxelField{grid, gd, gh, gw};
        run(node, seeds, rays, n, dst);
    } else {
        PbvrSphere node;
        setup(node, c0, c1, env_rgb, transform, albedo, g, max_bounces);
        node.mg = SphereField{grid, gd, gh, gw};
        run(node, seeds, rays, n, dst);
    }
}

// PBVRT.forward (variant 0, dst [n, 4]) or PBVR_NEE.forward (variant 1,
// dst [n, 3]) for rays [n, 6]; fields, extinction and the constant albedo /
// environment as ref_pbvr.
void ref_pbvrt(int variant, float c0, float c1, int field_kind, const float* grid, int gd, int gh, int gw,
               const float* env_rgb, const float* transform, const float* albedo, const float* light_direction,
               const float* light_intensity, float g, float density_scale, int max_bounces, const unsigned* seeds,
               const float* rays, long n, float* dst) {
    auto fill = [&](auto& node) {
        node.ext = ExtNode{c0, c1};
        node.env = EnvConst{env_rgb[0], env_rgb[1], env_rgb[2]};
        for (int k = 0; k < 3; ++k) {
            node.sa[k] = albedo[k];
            node.light_intensity[k] = light_intensity[k];
        }
        for (int j = 0; j < 4; ++j)
            node.transform.c[j] = rdv_vec3(transform[3 * j], transform[3 * j + 1], transform[3 * j + 2]);
        node.light_direction = rdv_vec3(light_direction[0], light_direction[1], light_direction[2]);
        node.g = g;
        node.density_scale = density_scale;
        node.max_bounces = max_bounces;
    };
    const int n_out = variant == 0 ? 4 : 3;
    auto run_rays = [&](auto node) {
        for (long r = 0; r < n; ++r) {
            random_seeds.seeds = rdv_uvec4(seeds[0], seeds[1], seeds[2], seeds[3]);
            rdv_random_init(rdv_uvec3{(unsigned)r, 0u, 0u});
            float in6[6];
            for (int k = 0; k < 6; ++k) in6[k] = rays[r * 6 + k];
            forward(node, in6, dst + r * n_out);
        }
    };
    if (variant == 0 && field_kind == 0) {
        PbvrtVoxel node; fill(node); node.mg = VoxelField{grid, gd, gh, gw}; run_rays(node);
    } else if (variant == 0) {
        PbvrtSphere node; fill(node); node.mg = SphereField{grid, gd, gh, gw}; run_rays(node);
    } else if (field_kind == 0) {
        NeeVoxel node; fill(node); node.mg = VoxelField{grid, gd, gh, gw}; run_rays(node);
    } else {
        NeeSphere node; fill(node); node.mg = SphereField{grid, gd, gh, gw}; run_rays(node);
    }
}

// PBVR_ENV.forward for rays [n, 6] -> dst [n, 3]: as ref_pbvrt, the NEE
// directions from an XREnvironmentSampler over `densities` (levels deep)
// whose environment is the constant env_rgb.
void ref_pbvr_env(float c0, float c1, int field_kind, const float* grid, int gd, int gh, int gw, const float* env_rgb,
                  const float* transform, const float* albedo, const float* densities, int levels, float g,
                  float density_scale, int max_bounces, const unsigned* seeds, const float* rays, long n, float* dst) {
    g_env_levels = levels;
    auto fill = [&](auto& node) {
        node.ext = ExtNode{c0, c1};
        node.env = EnvConst{env_rgb[0], env_rgb[1], env_rgb[2]};
        node.environment_sampler = XrEnvNode{EnvConst{env_rgb[0], env_rgb[1], env_rgb[2]}, densities};
        for (int k = 0; k < 3; ++k) {
            node.sa[k] = albedo[k];
            node.light_intensity[k] = 1.0f;
        }
        for (int j = 0; j < 4; ++j)
            node.transform.c[j] = rdv_vec3(transform[3 * j], transform[3 * j + 1], transform[3 * j + 2]);
        node.light_direction = rdv_vec3(0.0f, 1.0f, 0.0f);
        node.g = g;
        node.density_scale = density_scale;
        node.max_bounces = max_bounces;
    };
    auto run_rays = [&](auto node) {
        for (long r = 0; r < n; ++r) {
            random_seeds.seeds = rdv_uvec4(seeds[0], seeds[1], seeds[2], seeds[3]);
            rdv_random_init(rdv_uvec3{(unsigned)r, 0u, 0u});
            float in6[6];
            for (int k = 0; k < 6; ++k) in6[k] = rays[r * 6 + k];
            forward(node, in6, dst + r * 3);
        }
    };
    if (field_kind == 0) {
        EnvVoxel node; fill(node); node.mg = VoxelField{grid, gd, gh, gw}; run_rays(node);
    } else {
        EnvSphere node; fill(node); node.mg = SphereField{grid, gd, gh, gw}; run_rays(node);
    }
}

// hg_phase_sample(w, g) on invocation `index`'s generator, `draws` before.
void ref_hg_phase_sample(const unsigned* seeds, int index, int draws, const float* w, float g, float* dst) {
    random_seeds.seeds = rdv_uvec4(seeds[0], seeds[1], seeds[2], seeds[3]);
    rdv_random_init(rdv_uvec3{(unsigned)index, 0u, 0u});
    for (int i = 0; i < draws; ++i) rdv_random();
    const rdv_vec3 r = hg_phase_sample(rdv_vec3(w[0], w[1], w[2]), g);
    dst[0] = r.x;
    dst[1] = r.y;
    dst[2] = r.z;
}

}  // extern "C"
