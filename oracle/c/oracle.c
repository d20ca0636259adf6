/*
 * Test infrastructure only: the CPU parity checker for the fused-MLP path.
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg load
 * this library; the product never does.
 *
 * Restates, row by row, the per-layer arithmetic of the reference's Map
 * nodes (rdv/shaders/...):
 *
 *   exact fp32 (Linear, maps/linear.h:28-31 and :44-48 of the fallback):
 *       acc = b[o]; for k ascending: acc += x[k] * W[o*IN + k]
 *   fp16 operands (LinearFast, maps/linear_fast.h:61-98):
 *       x and W staged as float16 (round to nearest even), products summed
 *       in fp32 starting from 0, bias added after in fp32
 *       (_output[o] = _SH_Y[...] + bias[o], :97-98)
 *   bf16 operands: same as fp16 with bfloat16 staging (a B200 extension; the
 *       reference has no bf16 path)
 *   bias first (flag bit 3): the accumulator starts from the bias and the
 *       staged products are added to it in ascending k -- the order of
 *       LinearTensorOpSmall / LinearTensorOpSimple, whose cooperative-matrix
 *       accumulators are seeded with a stride-0 load of the bias
 *       (tensors/linear_tensor_op_small.h:99, linear_tensor_op_simple.h)
 *   ReLU (maps/relu.h:1-5): max(x, 0) in fp32.
 *
 * LinearFast's workgroup fallback (linear_fast.h:44 / :102-108, and
 * cooperative_library.h:20-33): rows of a trailing partial 32-row workgroup
 * run every layer in exact fp32. `tail_exact` enables that rule.
 *
 * Built with -ffp-contract=off so every product and sum is rounded on its
 * own, the literal reading of the GLSL. Single-threaded: callers split rows
 * across threads (ctypes releases the GIL for the duration of a call).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

enum { ORACLE_MATH_F32 = 0, ORACLE_MATH_F16 = 1, ORACLE_MATH_BF16 = 2 };
#define ORACLE_FLAG_MATH_MASK 3
#define ORACLE_FLAG_RELU 4
#define ORACLE_FLAG_BIAS_FIRST 8

static float round_f16(float v) { return (float)(_Float16)v; }

static float round_bf16(float v) {
    /* round to nearest even on the upper 16 bits; NaN kept quiet */
    uint32_t u;
    memcpy(&u, &v, 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) {
        u |= 0x00400000u;
    } else {
        uint32_t lsb = (u >> 16) & 1u;
        u += 0x7fffu + lsb;
    }
    u &= 0xffff0000u;
    float r;
    memcpy(&r, &u, 4);
    return r;
}

static float stage(float v, int math) {
    if (math == ORACLE_MATH_F16) return round_f16(v);
    if (math == ORACLE_MATH_BF16) return round_bf16(v);
    return v;
}

/* dims: n_layers+1 entries; W[l] is [dims[l+1], dims[l]] row-major (PyTorch
 * nn.Linear layout); flags[l]: bits 0-1 math, bit 2 ReLU after the layer. */
void oracle_mlp_forward(const float* x, int64_t n_rows, int n_layers, const int* dims,
                        const float* const* W, const float* const* b, const int* flags,
                        int input_relu, int tail_exact, float* y) {
    int maxw = 0;
    for (int l = 0; l <= n_layers; ++l) maxw = dims[l] > maxw ? dims[l] : maxw;
    int64_t n_full = tail_exact ? (n_rows / 32) * 32 : n_rows;
    {
        float* a = (float*)malloc(sizeof(float) * (size_t)maxw);
        float* c = (float*)malloc(sizeof(float) * (size_t)maxw);
        float* ws = (float*)malloc(sizeof(float) * (size_t)maxw);
        for (int64_t r = 0; r < n_rows; ++r) {
            int in0 = dims[0];
            for (int k = 0; k < in0; ++k) {
                float v = x[r * in0 + k];
                a[k] = (input_relu && v < 0.0f) ? 0.0f : v;
            }
            for (int l = 0; l < n_layers; ++l) {
                int IN = dims[l], OUT = dims[l + 1];
                int math = flags[l] & ORACLE_FLAG_MATH_MASK;
                if (r >= n_full) math = ORACLE_MATH_F32;
                if (math == ORACLE_MATH_F32) {
                    for (int o = 0; o < OUT; ++o) {
                        float acc = b[l][o];
                        for (int k = 0; k < IN; ++k) acc += a[k] * W[l][(int64_t)o * IN + k];
                        c[o] = acc;
                    }
                } else {
                    const int bias_first = (flags[l] & ORACLE_FLAG_BIAS_FIRST) != 0;
                    for (int k = 0; k < IN; ++k) ws[k] = stage(a[k], math);
                    for (int o = 0; o < OUT; ++o) {
                        float acc = bias_first ? b[l][o] : 0.0f;
                        for (int k = 0; k < IN; ++k)
                            acc += ws[k] * stage(W[l][(int64_t)o * IN + k], math);
                        c[o] = bias_first ? acc : acc + b[l][o];
                    }
                }
                if (flags[l] & ORACLE_FLAG_RELU)
                    for (int o = 0; o < OUT; ++o) c[o] = c[o] > 0.0f ? c[o] : 0.0f;
                float* t = a; a = c; c = t;
            }
            int outd = dims[n_layers];
            for (int o = 0; o < outd; ++o) y[r * outd + o] = a[o];
        }
        free(a);
        free(c);
        free(ws);
    }
}

/* Element-wise staging used by the numpy side to emulate the same rounding. */
void oracle_round(const float* x, int64_t n, int math, float* y) {
    for (int64_t i = 0; i < n; ++i) y[i] = stage(x[i], math);
}
