// Test infrastructure only (parity checker, never shipped or measured).
//
// Executes the reference's cooperative-matrix (float16 tensor-core) code
// paths on the CPU through coopmat_prelude.hpp, and exposes them through a
// small extern "C" surface used by tests/golden/make_golden.py:
//
//   ref_cm_mlp_c5 / ref_cm_mlp_c2   a Map chain of LinearFast and ReLU
//       nodes (maps/linear_fast.h, maps/relu.h, composed by
//       maps/composite.h, gated by libraries/cooperative_library.h), the
//       architectures of BASELINE configs 5 and 2, one invocation per row,
//       32-row workgroups (a trailing partial workgroup takes the scalar
//       fp32 path, as on the device)
//   ref_cm_small_*, ref_cm_simple_32_64, ref_cm_fast_32_64, ref_cm_mine_32_48
//       LinearTensorOp{Small,Simple,Fast,Mine}.forward
//   ref_cm_winograd_16 / ref_cm_winograd_48
//       Conv2DTensorOpWinograd3x3.forward on a 16x16 image, 16 -> 16 and
//       48 -> 48 channels
//
// The shader files are #included from copies of the reference checkout
// that oracle/Makefile writes into oracle/_ref/gen/ with their `#extension`
// lines dropped -- nothing else changes, and nothing of them is copied into
// this repository. Node structs carry the fields the shaders read (names
// from rdv/domain/nn.py's node declarations).
#include "coopmat_prelude.hpp"

// The reference's megakernel header defines this on devices with cooperative
// matrices (rdv/core/_core.py _build_code); every body below is compiled
// with it, i.e. as the tensor-core path.
#define RDV_COOPERATIVE_MATRIX_SUPPORT 1

// ----------------------------------------------------------- Map path
#include "libraries/cooperative_library.h"

#define DECLARE_LF(NAME) \
    struct NAME {        \
        float* weight;   \
        float* bias;     \
        int id;          \
    };
DECLARE_LF(LF_3_64)
DECLARE_LF(LF_64_64)
DECLARE_LF(LF_64_4)
DECLARE_LF(LF_32_128)
DECLARE_LF(LF_128_128)
DECLARE_LF(LF_128_16)
struct Relu_64 { int unused; };
struct Relu_128 { int unused; };

#define RDV_NODE LF_3_64
#define IN 3
#define OUT 64
#include "maps/linear_fast.h"
#undef OUT
#undef IN
#undef RDV_NODE
#define RDV_NODE LF_64_64
#define IN 64
#define OUT 64
#include "maps/linear_fast.h"
#undef OUT
#undef IN
#undef RDV_NODE
#define RDV_NODE LF_64_4
#define IN 64
#define OUT 4
#include "maps/linear_fast.h"
#undef OUT
#undef IN
#undef RDV_NODE
#define RDV_NODE LF_32_128
#define IN 32
#define OUT 128
#include "maps/linear_fast.h"
#undef OUT
#undef IN
#undef RDV_NODE
#define RDV_NODE LF_128_128
#define IN 128
#define OUT 128
#include "maps/linear_fast.h"
#undef OUT
#undef IN
#undef RDV_NODE
#define RDV_NODE LF_128_16
#define IN 128
#define OUT 16
#include "maps/linear_fast.h"
#undef OUT
#undef IN
#undef RDV_NODE
#define RDV_NODE Relu_64
#define IN 64
#define OUT 64
#include "maps/relu.h"
#undef OUT
#undef IN
#undef RDV_NODE
#define RDV_NODE Relu_128
#define IN 128
#define OUT 128
#include "maps/relu.h"
#undef OUT
#undef IN
#undef RDV_NODE

// Composite.forward, instantiated as a function template over the pair of
// node types: `a >> b` is Composite(f = b, g = a). V (the intermediate
// buffer) is 128, the widest hidden layer here; IN and OUT only size
// pointer parameters.
template <class F, class G>
struct Comp {
    F f;
    G g;
};
#define RDV_NODE Comp<F, G>
#define IN 1
#define V 128
#define OUT 1
template <class F, class G>
#include "maps/composite.h"
#undef OUT
#undef V
#undef IN
#undef RDV_NODE

// Layer l of a chain gets W[l], b[l] and id l, in application order.
#define FILL_LF(T)                                                      \
    static void fill(T& n, float* const* W, float* const* b, int& l) { \
        n.weight = W[l];                                                \
        n.bias = b[l];                                                  \
        n.id = l;                                                       \
        ++l;                                                            \
    }
FILL_LF(LF_3_64)
FILL_LF(LF_64_64)
FILL_LF(LF_64_4)
FILL_LF(LF_32_128)
FILL_LF(LF_128_128)
FILL_LF(LF_128_16)
static void fill(Relu_64&, float* const*, float* const*, int&) {}
static void fill(Relu_128&, float* const*, float* const*, int&) {}
template <class F, class G>
static void fill(Comp<F, G>& c, float* const* W, float* const* b, int& l) {
    fill(c.g, W, b, l);
    fill(c.f, W, b, l);
}

// config 5: 3 -> 64 (x4 hidden, ReLU) -> 4
using Chain5 =
    Comp<LF_64_4,
         Comp<Relu_64,
              Comp<LF_64_64, Comp<Relu_64, Comp<LF_64_64, Comp<Relu_64, Comp<LF_64_64, Comp<Relu_64, LF_3_64>>>>>>>>;
// config 2: 32 -> 128 (x8 hidden, ReLU) -> 16
using H1 = Comp<Relu_128, LF_32_128>;
using H2 = Comp<Relu_128, Comp<LF_128_128, H1>>;
using H3 = Comp<Relu_128, Comp<LF_128_128, H2>>;
using H4 = Comp<Relu_128, Comp<LF_128_128, H3>>;
using H5 = Comp<Relu_128, Comp<LF_128_128, H4>>;
using H6 = Comp<Relu_128, Comp<LF_128_128, H5>>;
using H7 = Comp<Relu_128, Comp<LF_128_128, H6>>;
using H8 = Comp<Relu_128, Comp<LF_128_128, H7>>;
using Chain2 = Comp<LF_128_16, H8>;

// One invocation per row (maps/map_evaluator.h: forward(map, input row,
// output row)), 32-row workgroups.
template <class Net>
static void run_chain(const float* x, long n, int in_dim, int out_dim, float* const* W, float* const* b, float* y) {
    Net net{};
    int l = 0;
    fill(net, W, b, l);
    const int groups = static_cast<int>((n + 31) / 32);
    const int live_last = static_cast<int>(n - 32L * (groups - 1));
    rdv_dispatch(groups, 32, live_last, [&] {
        const long row = gl_GlobalInvocationID.x;
        float in_row[128], out_row[128];
        for (int k = 0; k < in_dim; ++k) in_row[k] = x[row * in_dim + k];
        forward(net, in_row, out_row);
        for (int o = 0; o < out_dim; ++o) y[row * out_dim + o] = out_row[o];
    });
}

// ---------------------------------------------------------- TensorOps
// LinearTensorOpSmall, two shapes (its INF < OUTF nesting and the swapped
// one), 2 subgroups per workgroup.
struct Small_32_48 { int shape[2]; float* result; float* x_buf; float* weight; float* bias; };
struct Small_64_32 { int shape[2]; float* result; float* x_buf; float* weight; float* bias; };
#define FBUFFER float*
#define F16 float*
#define FOUT float*
#define SPT 2
#define RDV_NODE Small_32_48
#define INF 32
#define OUTF 48
#include "tensors/linear_tensor_op_small.h"
#undef OUTF
#undef INF
#undef RDV_NODE
#undef _SUBGROUPS_PER_TILE
#undef _WG_THREADS
#undef _ROWS_PER_WG
#undef _SH_X
#undef _SH_W
#undef IN_TILES
#undef OUT_TILES
#undef _ACC_T
#undef _OUT_OFF
#define RDV_NODE Small_64_32
#define INF 64
#define OUTF 32
#include "tensors/linear_tensor_op_small.h"
#undef OUTF
#undef INF
#undef RDV_NODE
#undef _SUBGROUPS_PER_TILE
#undef _WG_THREADS
#undef _ROWS_PER_WG
#undef _SH_X
#undef _SH_W
#undef IN_TILES
#undef OUT_TILES
#undef _ACC_T
#undef _OUT_OFF

// LinearTensorOpSimple: float16 weights (pre-cast), 2 subgroups.
struct Simple_32_64 { int shape[2]; float* result; float* x_buf; float16_t* weight; float* bias; };
#define F512 float*
#define RDV_NODE Simple_32_64
#define INF 32
#define OUTF 64
#include "tensors/linear_tensor_op_simple.h"
#undef OUTF
#undef INF
#undef RDV_NODE
#undef _SUBGROUPS_PER_TILE
#undef _SH_X
#undef _SH_A
#undef IN_TILES
#undef OUT_TILES
#undef _WG_THREADS
#undef SPT

// LinearTensorOpFast: float16 weights pre-tiled [n][k][16][16].
struct Fast_32_64 { int shape[2]; float* result; float* x_buf; float16_t* weight_tiled; float* bias; };
#define F256 float16_t*
#define RDV_NODE Fast_32_64
#define INF 32
#define OUTF 64
#include "tensors/linear_tensor_op_fast.h"
#undef OUTF
#undef INF
#undef RDV_NODE
#undef _SH_X0
#undef _SH_X1
#undef _SH_Y

// LinearTensorOpMine: fp32 weights, 32x16 per workgroup.
struct Mine_32_48 { int shape[2]; float* result; float* x_buf; float* weight; float* bias; };
#define RDV_NODE Mine_32_48
#define INF 32
#define OUTF 48
#include "tensors/linear_tensor_op_mine.h"
#undef OUTF
#undef INF
#undef RDV_NODE
#undef _PAD
#undef _SH_A
#undef _SH_B
#undef _SH_Y

// Conv2DTensorOpWinograd3x3 on a 16x16 image; each configuration in its
// own namespace (the file also defines the plain _winograd_fwd/_inv).
namespace wino16 {
struct Node { int shape[2]; float* result; float* x_buf; float16_t* weight_u; float* bias; };
#define RDV_NODE Node
#define H 16
#define W 16
#define CIN 16
#define COUT 16
#include "tensors/conv2d_tensor_op_winograd3x3.h"
#undef COUT
#undef CIN
#undef W
#undef H
#undef RDV_NODE
#undef _SH_V
#undef _SH_U
#undef _SH_M
#undef CIN_TILES
#undef OUT_TILES
}  // namespace wino16
namespace wino48 {
struct Node { int shape[2]; float* result; float* x_buf; float16_t* weight_u; float* bias; };
#define RDV_NODE Node
#define H 16
#define W 16
#define CIN 48
#define COUT 48
#include "tensors/conv2d_tensor_op_winograd3x3.h"
#undef COUT
#undef CIN
#undef W
#undef H
#undef RDV_NODE
#undef _SH_V
#undef _SH_U
#undef _SH_M
#undef CIN_TILES
#undef OUT_TILES
}  // namespace wino48

template <class Node>
static void run_op(Node& node, int groups, int wg_size) {
    rdv_dispatch(groups, wg_size, wg_size, [&] { forward(node); });
}

// ------------------------------------------------------ extern "C" surface
extern "C" {

void ref_cm_mlp_c5(const float* x, long n, float* const* W_, float* const* b, float* y) {
    run_chain<Chain5>(x, n, 3, 4, W_, b, y);
}

void ref_cm_mlp_c2(const float* x, long n, float* const* W_, float* const* b, float* y) {
    run_chain<Chain2>(x, n, 32, 16, W_, b, y);
}

// batch a multiple of 64 (2 subgroups x 32 rows per workgroup)
void ref_cm_small_32_48(const float* x, int batch, const float* W_, const float* b, float* y) {
    Small_32_48 node{{batch, 48}, y, const_cast<float*>(x), const_cast<float*>(W_), const_cast<float*>(b)};
    run_op(node, batch / 64, 64);
}

void ref_cm_small_64_32(const float* x, int batch, const float* W_, const float* b, float* y) {
    Small_64_32 node{{batch, 32}, y, const_cast<float*>(x), const_cast<float*>(W_), const_cast<float*>(b)};
    run_op(node, batch / 64, 64);
}

// W16: the float16 weight [64, 32] (nn.py _cast_fp16) as raw bits; batch a multiple of 32
void ref_cm_simple_32_64(const float* x, int batch, const uint16_t* W16, const float* b, float* y) {
    Simple_32_64 node{{batch, 64}, y, const_cast<float*>(x),
                      reinterpret_cast<float16_t*>(const_cast<uint16_t*>(W16)), const_cast<float*>(b)};
    run_op(node, batch / 32, 64);
}

// Wt16: [n_tiles][k_tiles][16][16] float16 bits (nn.py _tile_weight_fp16); batch a multiple of 64
void ref_cm_fast_32_64(const float* x, int batch, const uint16_t* Wt16, const float* b, float* y) {
    Fast_32_64 node{{batch, 64}, y, const_cast<float*>(x),
                    reinterpret_cast<float16_t*>(const_cast<uint16_t*>(Wt16)), const_cast<float*>(b)};
    run_op(node, (batch / 64) * (64 / 32), 32);
}

// batch a multiple of 32
void ref_cm_mine_32_48(const float* x, int batch, const float* W_, const float* b, float* y) {
    Mine_32_48 node{{batch, 48}, y, const_cast<float*>(x), const_cast<float*>(W_), const_cast<float*>(b)};
    run_op(node, (batch / 32) * (48 / 16), 32);
}

// x [256, cin] (one 16x16 image, channels last), U16 [16][cin][cout] float16 bits
void ref_cm_winograd_16(const float* x, const uint16_t* U16, const float* b, float* y) {
    wino16::Node node{{256, 16}, y, const_cast<float*>(x),
                      reinterpret_cast<float16_t*>(const_cast<uint16_t*>(U16)), const_cast<float*>(b)};
    run_op(node, 64 / 32, 32);
}

void ref_cm_winograd_48(const float* x, const uint16_t* U16, const float* b, float* y) {
    wino48::Node node{{256, 48}, y, const_cast<float*>(x),
                      reinterpret_cast<float16_t*>(const_cast<uint16_t*>(U16)), const_cast<float*>(b)};
    run_op(node, 64 / 32, 32);
}

}  // extern "C"
