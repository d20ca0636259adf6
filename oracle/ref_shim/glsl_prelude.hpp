// Test infrastructure only (parity checker, never shipped or measured).
//
// A minimal C++ stand-in for the handful of GLSL constructs used by the
// reference shader functions that this directory compiles *from where they
// lie* in the reference checkout (rdv/shaders/...). Only functions whose
// bodies are plain scalar/array arithmetic are compiled this way:
//
//   maps/linear.h                       Linear.forward (exact fp32 per row)
//   maps/relu.h                         ReLU.forward
//   maps/composite.h                    Composite.forward (f(g(x)))
//   tensors/linear_tensor_op.h          LinearTensorOp.forward (fp32 4x8 tiles)
//   tensors/relu_tensor_op.h            ReLUTensorOp.forward
//   tensors/conv2d_tensor_op.h          Conv2DTensorOp.forward (fp32 direct conv)
//   tensors/conv2d_tensor_op_winograd3x3.h  _winograd_fwd / _winograd_inv
//   volumes/raymarching_transmittance_trait.h  transmittance_rm
//
// Cooperative-matrix code in those files sits behind
// RDV_COOPERATIVE_MATRIX_SUPPORT, which is never defined here, so only the
// portable scalar paths are compiled.
#pragma once
#include <cmath>
#include <cstdint>

typedef unsigned int uint;

struct rdv_uvec3 { unsigned x, y, z; };

// Per-"invocation" builtins; the wrappers set them before every call.
static rdv_uvec3 gl_LocalInvocationID = {0, 0, 0};
static rdv_uvec3 gl_GlobalInvocationID = {0, 0, 0};
static rdv_uvec3 gl_WorkGroupID = {0, 0, 0};

// One invocation at a time: the workgroup-uniformity test of
// cooperative_library.h can never see 32 live lanes, so it reports false and
// every node takes its independent (per-thread) path, exactly as a partially
// occupied workgroup does in the reference.
static inline bool all_thread_sync(uint) { return false; }

struct rdv_vec2 {
    float x, y;
    rdv_vec2() : x(0), y(0) {}
    rdv_vec2(float a, float b) : x(a), y(b) {}
};
struct rdv_vec3 {
    float x, y, z;
    rdv_vec3() : x(0), y(0), z(0) {}
    explicit rdv_vec3(float s) : x(s), y(s), z(s) {}
    rdv_vec3(float a, float b, float c) : x(a), y(b), z(c) {}
    rdv_vec3(rdv_vec2 a, float c) : x(a.x), y(a.y), z(c) {}
};
static inline rdv_vec3 operator*(float s, rdv_vec3 v) { return rdv_vec3(s * v.x, s * v.y, s * v.z); }
static inline rdv_vec3 operator*(rdv_vec3 v, float s) { return rdv_vec3(s * v.x, s * v.y, s * v.z); }
static inline rdv_vec3 operator+(rdv_vec3 a, rdv_vec3 b) { return rdv_vec3(a.x + b.x, a.y + b.y, a.z + b.z); }
static inline rdv_vec3& operator+=(rdv_vec3& a, rdv_vec3 b) { a.x += b.x; a.y += b.y; a.z += b.z; return a; }

// More GLSL vector types, for libraries/random_library.h (the Taus + LCG
// generator and its samplers): only the operations that file uses.
struct rdv_vec4 {
    float x, y, z, w;
    rdv_vec4() : x(0), y(0), z(0), w(0) {}
    rdv_vec4(float a, float b, float c, float d) : x(a), y(b), z(c), w(d) {}
    rdv_vec4(rdv_vec2 a, rdv_vec2 b) : x(a.x), y(a.y), z(b.x), w(b.y) {}
};
struct rdv_uvec4 {
    uint x, y, z, w;
    rdv_uvec4() : x(0), y(0), z(0), w(0) {}
    // GLSL's uvec4(int, ...) converts each component (two's complement wrap)
    rdv_uvec4(long long a, long long b, long long c, long long d)
        : x((uint)a), y((uint)b), z((uint)c), w((uint)d) {}
};
static inline rdv_uvec4 operator^(rdv_uvec4 a, rdv_uvec4 b) {
    rdv_uvec4 r; r.x = a.x ^ b.x; r.y = a.y ^ b.y; r.z = a.z ^ b.z; r.w = a.w ^ b.w; return r;
}
static inline rdv_uvec4 operator+(rdv_uvec4 a, int s) {
    rdv_uvec4 r; r.x = a.x + (uint)s; r.y = a.y + (uint)s; r.z = a.z + (uint)s; r.w = a.w + (uint)s; return r;
}
static inline float uintBitsToFloat(uint v) { float f; __builtin_memcpy(&f, &v, 4); return f; }
static inline uint floatBitsToUint(float f) { uint v; __builtin_memcpy(&v, &f, 4); return v; }
static inline rdv_uvec4 floatBitsToUint(rdv_vec4 v) {
    rdv_uvec4 r; r.x = floatBitsToUint(v.x); r.y = floatBitsToUint(v.y); r.z = floatBitsToUint(v.z);
    r.w = floatBitsToUint(v.w); return r;
}
static inline rdv_vec2 operator*(float s, rdv_vec2 v) { return rdv_vec2(s * v.x, s * v.y); }
static inline rdv_vec2 operator*(rdv_vec2 a, rdv_vec2 b) { return rdv_vec2(a.x * b.x, a.y * b.y); }
static inline rdv_vec2 operator+(rdv_vec2 a, rdv_vec2 b) { return rdv_vec2(a.x + b.x, a.y + b.y); }
static inline rdv_vec4 operator*(rdv_vec4 a, rdv_vec4 b) { return rdv_vec4(a.x * b.x, a.y * b.y, a.z * b.z, a.w * b.w); }
static inline rdv_vec4 operator+(rdv_vec4 a, rdv_vec4 b) { return rdv_vec4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w); }
static inline rdv_vec3 operator*(rdv_vec3 a, rdv_vec3 b) { return rdv_vec3(a.x * b.x, a.y * b.y, a.z * b.z); }
static inline rdv_vec3 operator*(double s, rdv_vec3 v) { return (float)s * v; }
static inline float dot(rdv_vec3 a, rdv_vec3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
// GLSL's float log: C++ would widen `1.0 - random()` and evaluate in double.
// Transcendentals of a float argument are evaluated in double and rounded
// once (the correctly rounded float result in practice), as the numpy
// restatements do; the pins then compare operation order, not two libm's.
static inline float rdv_log(double v) { return (float)std::log((double)(float)v); }
static inline float min(float a, double b) { return a < (float)b ? a : (float)b; }
static inline float max(int a, double b) { return (float)a > (float)b ? (float)a : (float)b; }

// GLSL max(float, float-literal) - the literal is a double in C++.
static inline float max(float a, double b) { return a > (float)b ? a : (float)b; }
static inline float max(double a, float b) { return (float)a > b ? (float)a : b; }
static inline float max(float a, float b) { return a > b ? a : b; }
static inline float max(int a, float b) { return (float)a < b ? b : (float)a; }
static inline int min(int a, int b) { return a < b ? a : b; }

#define vec3 rdv_vec3
#define shared static
#define barrier() ((void)0)
#define deref(x) (x)
#define resolve(x) (x)
#define RDV_CONCAT_(a, b) a##b
#define RDV_CONCAT(a, b) RDV_CONCAT_(a, b)
// GLSL parameter qualifiers: arrays decay to pointers, so `out float v[16]`
// still writes through to the caller.
#define in
#define out
