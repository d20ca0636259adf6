// Test infrastructure only (parity checker, never shipped or measured).
//
// A C++ stand-in for the GLSL constructs of the reference's
// cooperative-matrix code paths (the bodies behind
// RDV_COOPERATIVE_MATRIX_SUPPORT), so that those bodies -- included from the
// reference checkout through copies whose only change is that their
// `#extension` directives are dropped (C++ has none; oracle/Makefile writes
// the copies) -- execute on the CPU:
//
//   maps/linear_fast.h                    LinearFast.forward (Map path)
//   tensors/linear_tensor_op_small.h      LinearTensorOpSmall.forward
//   tensors/linear_tensor_op_simple.h     LinearTensorOpSimple.forward
//   tensors/linear_tensor_op_fast.h       LinearTensorOpFast.forward
//   tensors/linear_tensor_op_mine.h       LinearTensorOpMine.forward
//   tensors/conv2d_tensor_op_winograd3x3.h  Conv2DTensorOpWinograd3x3.forward
//   libraries/cooperative_library.h       all_thread_sync (the fp16 gate)
//
// Execution model. A workgroup is `n` real threads (one per invocation)
// that meet at a std::barrier for every barrier(); workgroups run one
// after another, so `shared` variables (plain statics) are the running
// workgroup's shared memory. A tail workgroup runs only its live
// invocations, which is what the reference's dispatch does past the row
// count; cooperative_library.h then sees fewer than 32 lanes and sends
// LinearFast down its scalar path, as on the device.
//
// Cooperative matrices. GL_KHR_cooperative_matrix leaves the element
// distribution across a subgroup's invocations opaque; here every
// invocation of the subgroup holds the whole matrix (all of them load the
// same shared data, so they hold equal values), and coopMatStore is done
// by the subgroup's first invocation only (the reference always puts a
// barrier() between a store and any read of it). Semantics given to the
// operations (the spec leaves the last one's summation order to the
// hardware; this is the order every test here pins to):
//   coopmat<float16_t,...>  elements are float16 values (float16_t(x) is a
//                           round-to-nearest-even conversion, _Float16)
//   coopMatLoad / Store     element (r, c) at array[offset + r*stride + c]
//                           (row major) or array[offset + c*stride + r]
//                           (column major), stride in elements; stride 0
//                           broadcasts one row (the bias loads)
//   coopMatMulAdd(A, B, C)  D[i][j] = C[i][j], then for k = 0, 1, ...:
//                           D[i][j] = D[i][j] + A[i][k]*B[k][j], each
//                           product exact in fp32 (float16 x float16) and
//                           each sum rounded to fp32
#pragma once
#include <atomic>
#include <barrier>
#include <cmath>
#include <cstdint>
#include <thread>
#include <vector>

typedef unsigned int uint;
typedef _Float16 float16_t;

struct rdv_uvec3 {
    unsigned x, y, z;
};
#define uvec3 rdv_uvec3

// Per-invocation builtins (each invocation is its own thread).
static thread_local rdv_uvec3 gl_LocalInvocationID = {0, 0, 0};
static thread_local rdv_uvec3 gl_GlobalInvocationID = {0, 0, 0};
static thread_local rdv_uvec3 gl_WorkGroupID = {0, 0, 0};
static thread_local std::barrier<>* rdv_wg_barrier = nullptr;

static inline void barrier() { rdv_wg_barrier->arrive_and_wait(); }

// Shared-memory atomics of cooperative_library.h.
static inline int atomicAdd(int& v, int d) { return __atomic_fetch_add(&v, d, __ATOMIC_SEQ_CST); }
static inline uint atomicAnd(uint& v, uint m) { return __atomic_fetch_and(&v, m, __ATOMIC_SEQ_CST); }

// Runs `n_groups` workgroups of `wg_size` invocations one after another;
// the last has `live_last` live invocations. body() is one invocation.
template <class F>
static void rdv_dispatch(int n_groups, int wg_size, int live_last, F body) {
    for (int g = 0; g < n_groups; ++g) {
        const int live = (g == n_groups - 1) ? live_last : wg_size;
        std::barrier<> bar(live);
        std::vector<std::thread> ts;
        ts.reserve(live);
        for (int i = 0; i < live; ++i) {
            ts.emplace_back([&, i, g] {
                rdv_wg_barrier = &bar;
                gl_LocalInvocationID = {static_cast<unsigned>(i), 0, 0};
                gl_WorkGroupID = {static_cast<unsigned>(g), 0, 0};
                gl_GlobalInvocationID = {static_cast<unsigned>(g * wg_size + i), 0, 0};
                body();
            });
        }
        for (auto& t : ts) t.join();
    }
}

// ---------------------------------------------------- cooperative matrices
constexpr int gl_ScopeSubgroup = 3;
constexpr int gl_MatrixUseA = 0;
constexpr int gl_MatrixUseB = 1;
constexpr int gl_MatrixUseAccumulator = 2;
constexpr int gl_CooperativeMatrixLayoutRowMajor = 0;
constexpr int gl_CooperativeMatrixLayoutColumnMajor = 1;

template <typename T, int S, int R, int C, int U>
struct coopmat {
    float v[R][C];  // float16 matrices hold float16 values widened exactly
    coopmat() {
        for (int r = 0; r < R; ++r)
            for (int c = 0; c < C; ++c) v[r][c] = 0.0f;
    }
    explicit coopmat(double s) {
        const float e = static_cast<float>(static_cast<T>(s));
        for (int r = 0; r < R; ++r)
            for (int c = 0; c < C; ++c) v[r][c] = e;
    }
};

template <typename T, int S, int R, int C, int U, typename E>
static void coopMatLoad(coopmat<T, S, R, C, U>& m, const E* a, uint offset, uint stride, int layout) {
    for (int r = 0; r < R; ++r)
        for (int c = 0; c < C; ++c) {
            const uint idx = layout == gl_CooperativeMatrixLayoutRowMajor ? offset + r * stride + c
                                                                            : offset + c * stride + r;
            m.v[r][c] = static_cast<float>(static_cast<T>(a[idx]));
        }
}

template <typename T, int S, int R, int C, int U, typename E>
static void coopMatStore(const coopmat<T, S, R, C, U>& m, E* a, uint offset, uint stride, int layout) {
    if (gl_LocalInvocationID.x % 32 != 0) return;  // one store per subgroup
    for (int r = 0; r < R; ++r)
        for (int c = 0; c < C; ++c) {
            const uint idx = layout == gl_CooperativeMatrixLayoutRowMajor ? offset + r * stride + c
                                                                            : offset + c * stride + r;
            a[idx] = static_cast<E>(static_cast<T>(m.v[r][c]));
        }
}

template <typename TA, typename TC, int S, int M, int K, int N>
static coopmat<TC, S, M, N, gl_MatrixUseAccumulator> coopMatMulAdd(
    const coopmat<TA, S, M, K, gl_MatrixUseA>& A, const coopmat<TA, S, K, N, gl_MatrixUseB>& B,
    const coopmat<TC, S, M, N, gl_MatrixUseAccumulator>& Cm) {
    coopmat<TC, S, M, N, gl_MatrixUseAccumulator> D;
    for (int i = 0; i < M; ++i)
        for (int j = 0; j < N; ++j) {
            float d = Cm.v[i][j];
            for (int k = 0; k < K; ++k) d = d + A.v[i][k] * B.v[k][j];
            D.v[i][j] = d;
        }
    return D;
}

// ------------------------------------------------------ buffer references
// deref/resolve of a buffer reference is the pointer itself; address() and
// cast() move between pointers and 64-bit device addresses.
#define deref(x) (x)
#define resolve(x) (x)
#define address(p) (static_cast<uint64_t>(reinterpret_cast<uintptr_t>(p)))
#define cast(T, a) (reinterpret_cast<T>(static_cast<uintptr_t>(a)))
#define RDV_CONCAT_(a, b) a##b
#define RDV_CONCAT(a, b) RDV_CONCAT_(a, b)
#define TENSOR_OP_UNROLL
#define shared static
#define in
#define out

static inline int min(int a, int b) { return a < b ? a : b; }
static inline float max(float a, double b) { return a > static_cast<float>(b) ? a : static_cast<float>(b); }
