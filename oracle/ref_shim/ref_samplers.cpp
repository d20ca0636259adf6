// Test infrastructure only (parity checker, never shipped or measured).
//
// Compiles the reference's GridSampler body (rdv/shaders/samplers/
// grid_sampler.h) as C++, from a copy under _ref/gen written by
// oracle/Makefile whose only change is an `f` on unsuffixed floating
// literals (GLSL's are float: `1.0 - alpha[i]` rounds to float before the
// product, which a double literal would skip), over a dense row-major grid standing for a TensorGrid
// (grids/tensor_grid.h: the cell's OUT floats at indices_to_global(shape,
// indices) * OUT). One node type per (IN, OUT), like the reference's
// per-generic GLSL struct; the extern "C" surface samples n points.
#include "glsl_prelude.hpp"

static inline int clamp(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

#define DECLARE_GRID(IN_, OUT_)                                                             \
    struct Dense_##IN_##_##OUT_ {                                                           \
        int shape[IN_];                                                                     \
        const float* data;                                                                  \
    };                                                                                      \
    static void forward(Dense_##IN_##_##OUT_ g, int* indices, float* values) {              \
        long global = 0;                                                                    \
        for (int i = 0; i < IN_; i++) global = global * g.shape[i] + indices[i];            \
        for (int k = 0; k < OUT_; k++) values[k] = g.data[global * OUT_ + k];               \
    }                                                                                       \
    struct GridSampler_##IN_##_##OUT_ {                                                     \
        Dense_##IN_##_##OUT_ g;                                                             \
        int clamp, aligned, linear;                                                         \
    };

DECLARE_GRID(1, 3)
DECLARE_GRID(2, 3)
DECLARE_GRID(3, 3)
DECLARE_GRID(4, 3)
DECLARE_GRID(3, 5)


#define RDV_NODE GridSampler_1_3
#define IN 1
#define OUT 3
#include "samplers/grid_sampler.h"
#undef IN
#undef OUT
#undef RDV_NODE

#define RDV_NODE GridSampler_2_3
#define IN 2
#define OUT 3
#include "samplers/grid_sampler.h"
#undef IN
#undef OUT
#undef RDV_NODE

#define RDV_NODE GridSampler_3_3
#define IN 3
#define OUT 3
#include "samplers/grid_sampler.h"
#undef IN
#undef OUT
#undef RDV_NODE

#define RDV_NODE GridSampler_4_3
#define IN 4
#define OUT 3
#include "samplers/grid_sampler.h"
#undef IN
#undef OUT
#undef RDV_NODE

#define RDV_NODE GridSampler_3_5
#define IN 3
#define OUT 5
#include "samplers/grid_sampler.h"
#undef IN
#undef OUT
#undef RDV_NODE

template <typename Node, int IN_, int OUT_>
static void sample(Node node, const int* shape, const float* grid, const float* x, long n, float* dst) {
    for (int i = 0; i < IN_; ++i) node.g.shape[i] = shape[i];
    node.g.data = grid;
    for (long r = 0; r < n; ++r) {
        float in_[IN_];
        for (int i = 0; i < IN_; ++i) in_[i] = x[r * IN_ + i];
        forward(node, in_, dst + r * OUT_);
    }
}

extern "C" {

// GridSampler.forward over n points x [n, in_dim] of a dense grid
// [shape..., out_dim] -> dst [n, out_dim]; (in_dim, out_dim) one of
// (1, 3), (2, 3), (3, 3), (4, 3), (3, 5). Returns 0, or -1 for another pair.
int ref_grid_sampler(int in_dim, int out_dim, const int* shape, const float* grid, int clamp_, int aligned,
                     int linear, const float* x, long n, float* dst) {
#define CASE(IN_, OUT_)                                                                      \
    if (in_dim == IN_ && out_dim == OUT_) {                                                  \
        GridSampler_##IN_##_##OUT_ node;                                                     \
        node.clamp = clamp_;                                                                 \
        node.aligned = aligned;                                                              \
        node.linear = linear;                                                                \
        sample<GridSampler_##IN_##_##OUT_, IN_, OUT_>(node, shape, grid, x, n, dst);         \
        return 0;                                                                            \
    }
    CASE(1, 3)
    CASE(2, 3)
    CASE(3, 3)
    CASE(4, 3)
    CASE(3, 5)
#undef CASE
    return -1;
}

}  // extern "C"
