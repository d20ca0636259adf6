// Test infrastructure only (parity checker, never shipped or measured).
//
// Compiles a few of the reference's own GLSL functions as C++ (see
// glsl_prelude.hpp for which and why) and exposes them through a small
// extern "C" surface used by tests/golden/make_golden.py and by the CPU
// parity tests. The shader files are #included from the reference
// checkout (REF_SHADERS include path, set by oracle/Makefile); nothing of
// them is copied into this repository.
//
// Node layouts below mirror the field order the reference declares for each
// node type (rdv/domain/nn.py: _LinearBase.weight/bias/id,
// LinearTensorOp.x_buf/weight/bias + TensorOperation.shape/result,
// Conv2DTensorOp.x_buf/weight/bias).
#include "glsl_prelude.hpp"

// ---------------------------------------------------------------------------
// Map path: Linear (maps/linear.h), ReLU (maps/relu.h), Composite
// (maps/composite.h). Every distinct (IN, OUT) specialisation is a distinct
// node type, exactly like the reference's per-generic GLSL struct, so C++
// overload resolution plays the role of the megakernel's forward() overloads.
// ---------------------------------------------------------------------------
#define DECLARE_LINEAR(NAME, IN_, OUT_)                     \
    struct NAME { float* weight; float* bias; int id; };

DECLARE_LINEAR(Lin_3_64, 3, 64)
DECLARE_LINEAR(Lin_64_64, 64, 64)
DECLARE_LINEAR(Lin_64_4, 64, 4)
DECLARE_LINEAR(Lin_5_16, 5, 16)
DECLARE_LINEAR(Lin_16_7, 16, 7)
struct Relu_64 { int unused; };
struct Relu_16 { int unused; };

#define RDV_NODE Lin_3_64
#define IN 3
#define OUT 64
#include "maps/linear.h"
#undef IN
#undef OUT
#undef RDV_NODE

#define RDV_NODE Lin_64_64
#define IN 64
#define OUT 64
#include "maps/linear.h"
#undef IN
#undef OUT
#undef RDV_NODE

#define RDV_NODE Lin_64_4
#define IN 64
#define OUT 4
#include "maps/linear.h"
#undef IN
#undef OUT
#undef RDV_NODE

#define RDV_NODE Lin_5_16
#define IN 5
#define OUT 16
#include "maps/linear.h"
#undef IN
#undef OUT
#undef RDV_NODE

#define RDV_NODE Lin_16_7
#define IN 16
#define OUT 7
#include "maps/linear.h"
#undef IN
#undef OUT
#undef RDV_NODE

#define RDV_NODE Relu_64
#define IN 64
#define OUT 64
#include "maps/relu.h"
#undef IN
#undef OUT
#undef RDV_NODE

#define RDV_NODE Relu_16
#define IN 16
#define OUT 16
#include "maps/relu.h"
#undef IN
#undef OUT
#undef RDV_NODE

// `a >> b` builds Composite(f=b, g=a) (rdv/maths/__init__.py Map.__rshift__),
// so `L0 >> relu >> L1 >> relu >> L2 >> relu >> L3` nests left to right.
#define DECLARE_COMPOSITE(NAME, F, G, IN_, OUT_, V_)       \
    struct NAME { F f; G g; };                             \

DECLARE_COMPOSITE(C1_a, Relu_64, Lin_3_64, 3, 64, 64)
DECLARE_COMPOSITE(C1_b, Lin_64_64, C1_a, 3, 64, 64)
DECLARE_COMPOSITE(C1_c, Relu_64, C1_b, 3, 64, 64)
DECLARE_COMPOSITE(C1_d, Lin_64_64, C1_c, 3, 64, 64)
DECLARE_COMPOSITE(C1_e, Relu_64, C1_d, 3, 64, 64)
DECLARE_COMPOSITE(C1_f, Lin_64_4, C1_e, 3, 4, 64)
DECLARE_COMPOSITE(S_a, Relu_16, Lin_5_16, 5, 16, 16)
DECLARE_COMPOSITE(S_b, Lin_16_7, S_a, 5, 7, 16)

#define IN 3
#define V 64
#define OUT 64
#define RDV_NODE C1_a
#include "maps/composite.h"
#undef RDV_NODE
#define RDV_NODE C1_b
#include "maps/composite.h"
#undef RDV_NODE
#define RDV_NODE C1_c
#include "maps/composite.h"
#undef RDV_NODE
#define RDV_NODE C1_d
#include "maps/composite.h"
#undef RDV_NODE
#define RDV_NODE C1_e
#include "maps/composite.h"
#undef RDV_NODE
#undef OUT
#define OUT 4
#define RDV_NODE C1_f
#include "maps/composite.h"
#undef RDV_NODE
#undef OUT
#undef V
#undef IN

#define IN 5
#define V 16
#define OUT 16
#define RDV_NODE S_a
#include "maps/composite.h"
#undef RDV_NODE
#undef OUT
#define OUT 7
#define RDV_NODE S_b
#include "maps/composite.h"
#undef RDV_NODE
#undef OUT
#undef V
#undef IN

// ---------------------------------------------------------------------------
// TensorOperation path (fp32): LinearTensorOp, ReLUTensorOp, Conv2DTensorOp.
// ---------------------------------------------------------------------------
struct LinTO_16_24 { int shape[2]; float* result; float* x_buf; float* weight; float* bias; };
#define RDV_NODE LinTO_16_24
#define INF 16
#define OUTF 24
#include "tensors/linear_tensor_op.h"
#undef INF
#undef OUTF
#undef RDV_NODE

struct ReluTO { int shape[2]; float* result; float* x_buf; };
#define RDV_NODE ReluTO
#include "tensors/relu_tensor_op.h"
#undef RDV_NODE

struct ConvTO { int shape[2]; float* result; float* x_buf; float* weight; float* bias; };
#define RDV_NODE ConvTO
#define KH 3
#define KW 3
#define CIN 16
#define COUT 32
#define H 16
#define W 16
#include "tensors/conv2d_tensor_op.h"
#undef RDV_NODE
#undef KH
#undef KW
#undef CIN
#undef COUT
#undef H
#undef W

// Resampling and concatenation (tensors/downsample2x_tensor_op.h,
// upsample2x_tensor_op.h, concat_tensor_op.h): one 4x8 tile per invocation.
// (each reference megakernel holds one op's code; conv2d_tensor_op.h's
// helper macro is dropped so these files' own local variable of that name
// compile.)
#undef col_blocks
struct DownTO { int shape[2]; float* result; float* x_buf; int W; };
#define RDV_NODE DownTO
#include "tensors/downsample2x_tensor_op.h"
#undef RDV_NODE

struct UpTO { int shape[2]; float* result; float* x_buf; int W; };
#define RDV_NODE UpTO
#include "tensors/upsample2x_tensor_op.h"
#undef RDV_NODE

struct CatTO { int shape[2]; float* result; float* x1_buf; float* x2_buf; int C1; };
#define RDV_NODE CatTO
#include "tensors/concat_tensor_op.h"
#undef RDV_NODE

// Winograd transforms: the cooperative-matrix forward() of this file is
// compiled out (RDV_COOPERATIVE_MATRIX_SUPPORT undefined), leaving the two
// scalar transforms _winograd_fwd / _winograd_inv.
struct WinoTO { int unused; };
#define RDV_NODE WinoTO
#define CIN 16
#define COUT 16
#define H 16
#define W 16
#include "tensors/conv2d_tensor_op_winograd3x3.h"
#undef RDV_NODE
#undef CIN
#undef COUT
#undef H
#undef W

// Fixed-step transmittance (volumes/raymarching_transmittance_trait.h). The
// extinction Map is supplied here as an analytic field so the marching rule
// itself (step, early-out at tau > 16, d > 0 loop guard, safety cap) is what
// gets pinned.
struct RmNode { float c0, c1; };
static float extinction(RmNode node, vec3 x) {
    return node.c0 + node.c1 * (x.x * x.x + x.y * x.y + x.z * x.z);
}
#define RDV_NODE RmNode
#include "volumes/raymarching_transmittance_trait.h"
#undef RDV_NODE

// Ratio tracking (volumes/ratiotracking_transmittance_trait.h) with the
// reference's own Taus + LCG generator (libraries/random_library.h). The
// Makefile compiles a copy of random_library.h written into _ref/gen whose
// only change is `inout uvec4 x` -> `uvec4& x` (GLSL inout parameters are
// references; no macro can express that). The extinction is the analytic
// field above; the majorant is a voxel grid looked up as
// volumes/voxel_majorant_field.h does, restated here because that file's
// GLSL array constructors do not compile as C++.
#define vec2 rdv_vec2
#define vec4 rdv_vec4
#define uvec4 rdv_uvec4
#define uvec3 rdv_uvec3
#define layout(...)
#define uniform static struct
#define pi 3.1415926535897932384626433832795
#define two_pi 6.283185307179586476925286766559
#define log(x) rdv_log(x)
#define random rdv_random  // stdlib's long random(void) has the same name
static float min(float a, float b) { return a < b ? a : b; }
// math_library.h's create_ortho_basis is only used by the direction
// samplers, which the tracking loop never calls.
static void create_ortho_basis(vec3, vec3& T, vec3& B) { T = vec3(1, 0, 0); B = vec3(0, 0, 1); }
#define RDV_NODE rdv_random_init
#include "random_library.h"
#undef RDV_NODE

struct RtNode {
    float c0, c1;       // extinction c0 + c1 |x|^2, as RmNode
    const float* grid;  // majorant voxels [D, H, W] (z, y, x)
    int gd, gh, gw;
};
static float extinction(RtNode node, vec3 x) {
    return node.c0 + node.c1 * (x.x * x.x + x.y * x.y + x.z * x.z);
}
static float majorant(RtNode node, vec3 x, vec3 w, float& distance) {
    const int dim[3] = {node.gw, node.gh, node.gd};
    const float xs[3] = {x.x, x.y, x.z}, ws[3] = {w.x, w.y, w.z};
    int cell[3];
    float texit[3];
    for (int k = 0; k < 3; ++k) {
        int c = (int)((xs[k] * 0.5f + 0.5f) * (float)dim[k]);
        c = c < 0 ? 0 : (c > dim[k] - 1 ? dim[k] - 1 : c);
        cell[k] = c;
        const float vs = 2.0f / (float)dim[k];
        const float bmin = (float)c * vs - 1.0f;
        const float bmax = bmin + vs;
        const float t0 = (bmin - xs[k]) / ws[k], t1 = (bmax - xs[k]) / ws[k];
        texit[k] = t0 > t1 ? t0 : t1;
    }
    distance = min(min(texit[0], texit[1]), texit[2]);
    return node.grid[((long)cell[2] * node.gh + cell[1]) * node.gw + cell[0]];
}
#define RDV_NODE RtNode
#include "volumes/ratiotracking_transmittance_trait.h"
#undef RDV_NODE
#undef log
#undef random

// ---------------------------------------------------------------------------
// extern "C" surface
// ---------------------------------------------------------------------------
extern "C" {

// C1 architecture 3->64->64->64->4 with ReLU between,
// evaluated row by row through the reference's own Composite chain.
void ref_mlp_c1(const float* x, long n, float* const* W, float* const* b, float* y) {
    C1_f net;
    net.f = Lin_64_4{W[3], b[3], 0};
    net.g.f = Relu_64{0};
    net.g.g.f = Lin_64_64{W[2], b[2], 1};
    net.g.g.g.f = Relu_64{0};
    net.g.g.g.g.f = Lin_64_64{W[1], b[1], 0};
    net.g.g.g.g.g.f = Relu_64{0};
    net.g.g.g.g.g.g = Lin_3_64{W[0], b[0], 0};
    for (long r = 0; r < n; ++r) {
        float in_row[3] = {x[r * 3 + 0], x[r * 3 + 1], x[r * 3 + 2]};
        forward(net, in_row, y + r * 4);
    }
}

// Small odd-width chain 5->16->ReLU->7.
void ref_mlp_small(const float* x, long n, float* const* W, float* const* b, float* y) {
    S_b net;
    net.f = Lin_16_7{W[1], b[1], 0};
    net.g.f = Relu_16{0};
    net.g.g = Lin_5_16{W[0], b[0], 0};
    for (long r = 0; r < n; ++r) {
        float in_row[5];
        for (int k = 0; k < 5; ++k) in_row[k] = x[r * 5 + k];
        forward(net, in_row, y + r * 7);
    }
}

// LinearTensorOp fp32, INF=16, OUTF=24; batch must be a multiple of 4.
void ref_linear_tensor_op_16_24(const float* x, int batch, const float* Wt, const float* b, float* y) {
    LinTO_16_24 node;
    node.shape[0] = batch; node.shape[1] = 24;
    node.result = y; node.x_buf = const_cast<float*>(x);
    node.weight = const_cast<float*>(Wt); node.bias = const_cast<float*>(b);
    int tiles = (batch / 4) * (24 / 8);
    for (int t = 0; t < tiles; ++t) { gl_GlobalInvocationID.x = t; forward(node); }
}

void ref_relu_tensor_op(const float* x, int rows, int cols, float* y) {
    ReluTO node;
    node.shape[0] = rows; node.shape[1] = cols;
    node.result = y; node.x_buf = const_cast<float*>(x);
    int tiles = (rows / 4) * (cols / 8);
    for (int t = 0; t < tiles; ++t) { gl_GlobalInvocationID.x = t; forward(node); }
}

// Conv2DTensorOp fp32 'same' 3x3, H=W=16, CIN=16, COUT=32; x [H*W, CIN],
// weight [3, 3, CIN, COUT].
void ref_conv2d_tensor_op_3x3_16_32_16x16(const float* x, const float* w, const float* b, float* y) {
    ConvTO node;
    node.shape[0] = 16 * 16; node.shape[1] = 32;
    node.result = y; node.x_buf = const_cast<float*>(x);
    node.weight = const_cast<float*>(w); node.bias = const_cast<float*>(b);
    int tiles = (16 * 16 / 4) * (32 / 8);
    for (int t = 0; t < tiles; ++t) { gl_GlobalInvocationID.x = t; forward(node); }
}

// Downsample2xTensorOp: x [h*w, c] -> y [(h/2)*(w/2), c]; (h/2)*(w/2) a
// multiple of 4, c a multiple of 8.
void ref_downsample2x(const float* x, int h, int w, int c, float* y) {
    DownTO node;
    node.shape[0] = (h / 2) * (w / 2); node.shape[1] = c;
    node.result = y; node.x_buf = const_cast<float*>(x); node.W = w / 2;
    int tiles = (node.shape[0] / 4) * (c / 8);
    for (int t = 0; t < tiles; ++t) { gl_GlobalInvocationID.x = t; forward(node); }
}

// Upsample2xTensorOp: x [h*w, c] -> y [(2h)*(2w), c].
void ref_upsample2x(const float* x, int h, int w, int c, float* y) {
    UpTO node;
    node.shape[0] = (2 * h) * (2 * w); node.shape[1] = c;
    node.result = y; node.x_buf = const_cast<float*>(x); node.W = 2 * w;
    int tiles = (node.shape[0] / 4) * (c / 8);
    for (int t = 0; t < tiles; ++t) { gl_GlobalInvocationID.x = t; forward(node); }
}

// ConcatTensorOp: x1 [rows, c1] | x2 [rows, c2] -> y [rows, c1 + c2].
void ref_concat(const float* x1, int c1, const float* x2, int c2, int rows, float* y) {
    CatTO node;
    node.shape[0] = rows; node.shape[1] = c1 + c2;
    node.result = y; node.x1_buf = const_cast<float*>(x1); node.x2_buf = const_cast<float*>(x2); node.C1 = c1;
    int tiles = (rows / 4) * ((c1 + c2) / 8);
    for (int t = 0; t < tiles; ++t) { gl_GlobalInvocationID.x = t; forward(node); }
}

void ref_winograd_fwd(const float* d, float* V) { _winograd_fwd(const_cast<float*>(d), V); }
void ref_winograd_inv(const float* M, float* Y) { _winograd_inv(const_cast<float*>(M), Y); }

float ref_transmittance_rm(float c0, float c1, const float* x, const float* w, float d,
                           float step_size, float density_scale) {
    RmNode node{c0, c1};
    return transmittance_rm(node, vec3(x[0], x[1], x[2]), vec3(w[0], w[1], w[2]), d, step_size,
                            density_scale);
}

// The per-thread generator state of invocation `index` (random_library.h's
// init: the dispatch seeds spawned by the thread index), then n draws of
// random().
void ref_random_sequence(const unsigned* seeds, int index, int n, float* dst) {
    random_seeds.seeds = uvec4(seeds[0], seeds[1], seeds[2], seeds[3]);
    rdv_random_init(rdv_uvec3{(unsigned)index, 0u, 0u});
    for (int i = 0; i < n; ++i) dst[i] = rdv_random();
}

// transmittance_rt for one ray segment (entry point x, direction w, length
// d) on invocation `index`'s generator.
float ref_transmittance_rt(float c0, float c1, const float* grid, int gd, int gh, int gw, const unsigned* seeds,
                           int index, const float* x, const float* w, float d, float density_scale) {
    random_seeds.seeds = uvec4(seeds[0], seeds[1], seeds[2], seeds[3]);
    rdv_random_init(rdv_uvec3{(unsigned)index, 0u, 0u});
    RtNode node{c0, c1, grid, gd, gh, gw};
    return transmittance_rt(node, vec3(x[0], x[1], x[2]), vec3(w[0], w[1], w[2]), d, density_scale);
}

}  // extern "C"
