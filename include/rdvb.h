/*
 * rdvb -- C ABI of the B200 (sm_100a) implementation of Rendervous's
 * data-parallel hot path: fused small-MLP evaluation, Winograd 3x3
 * convolution and the MLP volume ray-march.
 *
 * Conventions
 *  - Every entry point returns an int status: RDVB_OK (0) or a negative
 *    RDVB_ERR_* code; rdvb_last_error() gives the calling thread's message.
 *  - Tensor arguments are DEVICE pointers owned by the caller, row-major,
 *    densely packed. Small descriptor arrays (dims, flags, pointer lists) are
 *    HOST arrays read before the call returns.
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy default
 *    stream). Calls are asynchronous and stream-ordered, like the kernels
 *    they launch; they never synchronize unless documented.
 *  - The reference dispatches each operator through a Vulkan compute
 *    "megakernel" and blocks in vk.submit_and_wait
 *    (rdv/core/_core.py:2799-2886); these entry points replace that
 *    dispatch for the operators named beside each one.
 */
#ifndef RDVB_H
#define RDVB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RDVB_OK 0
#define RDVB_ERR_INVALID_ARG (-1)
#define RDVB_ERR_UNSUPPORTED (-2)
#define RDVB_ERR_CUDA (-3)
#define RDVB_ERR_DEVICE_STATUS (-4) /* a kernel reported a bounded-wait timeout */

/* element types */
#define RDVB_F32 0
#define RDVB_F16 1
#define RDVB_BF16 2

/* per-layer flags of the MLP chain: bits 0-1 arithmetic, bit 2 ReLU after */
#define RDVB_MATH_F32 0  /* Linear: exact fp32 (rdv/shaders/maps/linear.h) */
#define RDVB_MATH_F16 1  /* LinearFast: float16 operands, fp32 accumulate (maps/linear_fast.h) */
#define RDVB_MATH_BF16 2 /* bfloat16 operands, fp32 accumulate (B200 extension) */
#define RDVB_LAYER_RELU 4

/* Winograd variants */
#define RDVB_WINOGRAD_F2X2 0 /* F(2x2,3x3), the reference's algorithm */
#define RDVB_WINOGRAD_F4X4 1 /* F(4x4,3x3), B200 extension */

/* Majorant fields of the ray trackers (rdv/domain/volumes.py:172-242). */
#define RDVB_MAJORANT_VOXEL 0  /* VoxelMajorantField: grid [D, H, W] of majorants */
#define RDVB_MAJORANT_SPHERE 1 /* SphereMajorantField: grid [D, H, W, 2] of (majorant, radius in voxels) */

/* PBVR environments and the 2-D sampler flags of an equirectangular one. */
#define RDVB_ENV_CONSTANT 0 /* a Constant map: one RGB radiance for every direction */
#define RDVB_ENV_EQUIRECT 1 /* XRProject() >> TensorSampler(image [H, W, 3]) */
#define RDVB_SAMPLER_CLAMP 1
#define RDVB_SAMPLER_ALIGNED 2
#define RDVB_SAMPLER_LINEAR 4

/* Input encoding of a volume node's extinction: a sampler of a dense 3-D
 * grid in front of the chain (GridSampler / TensorSampler >> Linear ...,
 * rdv/maths/__init__.py:2018-2083), evaluated per extinction query on the
 * CUDA cores. grid: device fp32 [dims[0], dims[1], dims[2], features]
 * (z, y, x, channel); flags: RDVB_SAMPLER_* (clamp, aligned, linear). With an
 * encoding the chain maps features -> 1 (dims[0] = features), or is empty
 * (n_layers 0, features 1: the sampled value is the extinction). */
#define RDVB_ENCODING_TENSOR_SAMPLER 1
#define RDVB_ENCODING_GRID_SAMPLER 2
typedef struct rdvb_encoding {
    int kind;
    const float* grid;
    int dims[3];
    int features;
    int flags;
} rdvb_encoding;

/* rdvb_pbvrt variants */
#define RDVB_PBVRT 0    /* PBVRT: RGB + alpha, the environment after scattering */
#define RDVB_PBVR_NEE 1 /* PBVR_NEE: RGB, next-event estimation only */
#define RDVB_PBVR_ENV 2 /* PBVR_ENV: RGB, next-event estimation toward importance-sampled environment directions */

/* Library version (major*10000 + minor*100 + patch). */
int rdvb_version(void);

/* Number of kernels this library has launched in this process (all devices,
 * all threads). Lets a caller count launches inside a timed region. */
int64_t rdvb_launch_count(void);

/* Message of the last failed call on this thread ("" if none). */
const char* rdvb_last_error(void);

/* Synchronizes the current device, then reads (and, if `clear`, resets) the
 * device status word that kernels set when a bounded wait expires, and writes
 * it to *status. Returns RDVB_OK when the word is 0, RDVB_ERR_DEVICE_STATUS
 * when it is not. */
int rdvb_device_status(int clear, uint32_t* status);

/* ---------------------------------------------------------------- MLP ----
 * A chain of n_layers affine layers, dims[0] -> dims[1] -> ... -> dims[n],
 * each y = W x + b with W [dims[l+1], dims[l]] (PyTorch nn.Linear layout) and
 * b [dims[l+1]], optionally followed by ReLU.
 *
 * Replaces: Map.__call__ of a `linear(W,b,f16) >> relu >> ...` Composite
 * (rdv/maths/__init__.py:1451-1487, Composite :1700-1728, MapEvaluator
 * :1569-1610; layer arithmetic rdv/shaders/maps/linear.h:15-44 and
 * linear_fast.h:39-109) and the single-layer TensorOperations
 * LinearTensorOp{,Fast,Mine,Simple,Small} (rdv/domain/nn.py:377-411,
 * 541-605, 1153-1411).
 */

/* Bytes of the packed-weight buffer rdvb_mlp_pack writes for these dims
 * (0 if the chain cannot use the tensor-core path). */
int64_t rdvb_mlp_packed_bytes(int n_layers, const int* dims);

/* Converts fp32 weights/biases (device pointers, one per layer) into the
 * tensor-core image: float16 (operand = RDVB_F16) or bfloat16 (RDVB_BF16)
 * K-major 128-byte-swizzled weight blocks, then the fp32 biases of every
 * layer (added to the fp32 accumulator, as the reference does). `packed` must hold
 * rdvb_mlp_packed_bytes() bytes, 256-byte aligned. The reference re-reads
 * fp32 weights at every dispatch (linear_fast.h:81-82); callers that change
 * weights in place call this again. */
int rdvb_mlp_pack(int n_layers, const int* dims, const float* const* weights, const float* const* biases,
                  int operand, void* packed, void* stream);

/* y[n_rows, dims[n]] (fp32) = chain(x[n_rows, dims[0]]).
 *  x_dtype      RDVB_F32 / RDVB_F16 / RDVB_BF16
 *  layer_flags  n_layers entries: RDVB_MATH_* | (RDVB_LAYER_RELU)
 *  input_relu   apply ReLU to x first (a chain that starts with relu)
 *  tail_exact   1: rows of a trailing partial 32-row group run every layer in
 *               exact fp32, as the reference's LinearFast falls back when its
 *               32-lane workgroup is not full (linear_fast.h:44,102-108)
 *  packed       rdvb_mlp_pack output for the same weights (required when any
 *               layer is F16/BF16 and the chain fits the tensor-core path;
 *               may be NULL for all-fp32 chains)
 *  weights, biases  the fp32 device tensors (used by the CUDA-core path)
 * Chains whose every layer is F16 (or every layer BF16) with widths <= 128
 * run on the tcgen05 tensor-core kernel; other chains (widths <= 256) run on
 * the CUDA-core kernel. */
int rdvb_mlp_forward(const void* x, int x_dtype, int64_t n_rows, int n_layers, const int* dims,
                     const float* const* weights, const float* const* biases, const int* layer_flags,
                     int input_relu, int tail_exact, const void* packed, float* y, void* stream);

/* The exchange step of a sharded evaluation (B200 extension: the reference
 * runs Map.__call__, rdv/maths/__init__.py:1451-1487, on one device):
 * `bytes` from src to each of dst[0..n_dst) on `stream`, one
 * cudaMemcpyAsync per destination (n_dst 0..7). dst are other GPUs'
 * buffers mapped by rdvb_ipc_open, so the copies run on the copy engines
 * over NVLink and leave every SM to the kernels they overlap. The caller
 * orders the step with a cross-GPU barrier before any rank reads rows it
 * did not compute. */
int rdvb_peer_copy(const void* src, void* const* dst, int n_dst, int64_t bytes, void* stream);

/* The same exchange through the NVLink switch: `bytes` (a multiple of 16)
 * of this GPU's rows at src written once to mc_dst, the multicast (NVLS)
 * address of the same rows in a symmetric buffer every rank of the group
 * bound, so the switch delivers them to every GPU. A kernel of at most
 * max_ctas CTAs (the caller keeps that many SMs free of its other kernels);
 * the caller orders the step with a cross-GPU barrier after it. */
int rdvb_multicast_copy(const void* src, uint64_t mc_dst, int64_t bytes, int max_ctas, void* stream);

/* Buffers other processes on this node can map (the output buffers of a
 * sharded evaluation, filled by rdvb_peer_copy). rdvb_ipc_alloc: `bytes` of device memory on the
 * current device and its RDVB_IPC_HANDLE_BYTES-byte handle, to pass to the
 * other ranks; rdvb_ipc_free releases it. rdvb_ipc_open: another process's
 * buffer mapped into this one (peer access enabled); rdvb_ipc_close unmaps. */
#define RDVB_IPC_HANDLE_BYTES 64
int rdvb_ipc_alloc(int64_t bytes, void** ptr, void* handle);
int rdvb_ipc_free(void* ptr);
int rdvb_ipc_open(const void* handle, void** ptr);
int rdvb_ipc_close(void* ptr);

/* Which kernel rdvb_mlp_forward runs for these arguments (no reference
 * counterpart: the reference picks between its fp16 and fp32 paths inside the
 * shader, linear_fast.h:44,102-108). Returns RDVB_PATH_TENSOR_CORE when its
 * whole 32-row groups run on the tcgen05 kernel, RDVB_PATH_CUDA_CORE when the
 * call runs on the CUDA cores -- then rdvb_last_error() names the reason (an
 * fp32 layer, a misaligned x or packed image, a chain too wide ...) -- or a
 * negative RDVB_ERR_* for invalid arguments. Launches nothing; the decision
 * depends on the current device's shared-memory limit. A float16 chain whose
 * x is misaligned (e.g. a row slice x[1:] of a 3-wide fp32 tensor) runs on
 * the CUDA cores, tens of times slower: callers can check here first. */
#define RDVB_PATH_CUDA_CORE 0
#define RDVB_PATH_TENSOR_CORE 1
int rdvb_mlp_forward_path(const void* x, int x_dtype, int64_t n_rows, int n_layers, const int* dims,
                          const int* layer_flags, const void* packed, const float* y);

/* Caps the CTAs of the persistent tensor-core MLP kernel at max_ctas (0, the
 * default, = one CTA per SM), for every later launch in this process (no
 * reference counterpart). A persistent CTA holds its SM's registers, so a
 * collective launched concurrently on another stream (the NCCL all-gather
 * that overlaps a sharded map's next chunk) gets SMs only if some are left
 * free. rdvb_get_max_ctas returns the current cap. */
int rdvb_set_max_ctas(int max_ctas);
int rdvb_get_max_ctas(void);

/* Allocation-free rdvb_mlp_forward (no reference counterpart: the reference
 * re-stages weights inside every dispatch). Same arguments minus `packed`:
 * the packed weight image is written into a static device array of
 * rdvb_mlp_static_capacity() bytes (256 KiB) owned by the library, so the
 * call allocates nothing. It is for callers that cannot allocate device
 * memory (hosts driving the C ABI over buffers they do not own, loops that
 * forbid allocation between calls). Chains whose packed image exceeds the
 * capacity return RDVB_ERR_UNSUPPORTED. Nothing needs to start zeroed: each
 * call rewrites every byte the kernel reads. The array is shared by all
 * callers on a device: two calls whose work overlaps on the device (other
 * streams, other threads) race on it, so order them (one stream, or events).
 * The array's address is looked up (cudaGetSymbolAddress) on the first call
 * on each device; make that first call before any stream capture. The
 * address belongs to the device's context: after cudaDeviceReset the library
 * must be reloaded (as for its other per-device state, e.g. kernel
 * attributes). A call rejected for its arguments never writes the array, and
 * the array is written only when the tensor-core kernel will read it
 * (rdvb_mlp_forward_path). */
int64_t rdvb_mlp_static_capacity(void);
int rdvb_mlp_forward_static(const void* x, int x_dtype, int64_t n_rows, int n_layers, const int* dims,
                            const float* const* weights, const float* const* biases, const int* layer_flags,
                            int input_relu, int tail_exact, float* y, void* stream);

/* y = max(x, 0) over n floats. Replaces ReLUTensorOp
 * (rdv/domain/nn.py:362-374, rdv/shaders/tensors/relu_tensor_op.h). */
int rdvb_relu(const float* x, float* y, int64_t n, void* stream);

/* ----------------------------------------------------------- 3x3 conv ----
 * 'Same' (zero padding 1), stride-1 3x3 convolution of NHWC tensors,
 * x [n, h, w, cin] -> y [n, h, w, cout], weights [3, 3, cin, cout]
 * (channels-last, the reference TensorOp layout), bias [cout].
 *
 * Replaces: Conv2DTensorOpWinograd3x3 (rdv/domain/nn.py:1002-1087, kernel
 * rdv/shaders/tensors/conv2d_tensor_op_winograd3x3.h:95-178, filter
 * transform _winograd_transform_weight nn.py:522-538), generalised to a batch
 * of images, odd h/w and cin, cout up to 64 (multiples of 16); the reference
 * takes one image, even h and w, cin/cout <= 48.
 */

/* Bytes of the packed filter operand for (variant, cin, cout); 0 if the
 * combination is not supported. */
int64_t rdvb_winograd_packed_bytes(int variant, int cin, int cout);

/* Filter transform U = G g G^T of fp32 weights w_33io [3, 3, cin, cout]
 * (device), computed in fp32 and rounded to float16, like
 * _winograd_transform_weight (rdv/domain/nn.py:525-538).
 *  u_plain   optional (may be NULL): the reference's flat float16 array
 *            [16][cin][cout]
 *  u_packed  optional (may be NULL): the tensor-core operand consumed by
 *            rdvb_conv3x3_winograd, rdvb_winograd_packed_bytes() bytes,
 *            256-byte aligned; requires cin, cout multiples of 16, <= 64
 * RDVB_WINOGRAD_F4X4 (a B200 extension): U = G g G^T with the 6x3 Toom-Cook
 * G of the points {0, 1, -1, 2, -1/2, inf}, kept fp32; u_plain and u_packed
 * are both the plain fp32 array [36][cin][cout] (4-byte aligned), cin and
 * cout in [1, 128]. */
int rdvb_winograd_filter_transform(const float* w_33io, int cin, int cout, int variant, void* u_plain,
                                   void* u_packed, void* stream);

/* Winograd convolution: input transform (fp32, staged float16), one tcgen05
 * GEMM per transform position (fp32 accumulation), inverse transform and bias
 * (fp32), fused in one kernel.
 *  x_dtype   RDVB_F32 or RDVB_F16 (x 16-byte aligned)
 *  u_packed  rdvb_winograd_filter_transform output for these channels
 *  bias      [cout] fp32, or NULL for zero
 *  y_dtype   RDVB_F32 (the reference's output type) or RDVB_F16
 *            (y 16-byte aligned)
 * variant RDVB_WINOGRAD_F4X4: 6x6 transforms with every operand fp32 (U, V,
 * the 36 per-position reductions on CUDA cores, the inverse transform), one
 * fused kernel; cin, cout in [1, 128]; x, y aligned to their element size.
 * (float16 U and V would put F(4x4) above the 1e-2 tolerance.) */
int rdvb_conv3x3_winograd(const void* x, int x_dtype, int n, int h, int w, int cin, int cout,
                          const void* u_packed, int variant, const float* bias, void* y, int y_dtype,
                          void* stream);

/* Direct 'same' (padding kh/2, kw/2), stride-1 convolution in fp32 on CUDA
 * cores: y = bias + sum over (kh, kw, cin) of x * w, one fused multiply-add
 * per tap. Replaces Conv2DTensorOp (rdv/domain/nn.py:414-469,
 * rdv/shaders/tensors/conv2d_tensor_op.h:21-87); also the on-device check of
 * the Winograd path. x RDVB_F32 or RDVB_F16; weight [kh, kw, cin, cout] fp32;
 * cout a multiple of 8; weight and y 16-byte aligned. */
int rdvb_conv2d_direct(const void* x, int x_dtype, int n, int h, int w, int cin, int cout, int kh, int kw,
                       const float* weight, const float* bias, float* y, void* stream);

/* The same convolution with the operands rounded first: math RDVB_MATH_F16 /
 * RDVB_MATH_BF16 rounds x and w to float16 / bfloat16 (products exact in
 * fp32, fp32 accumulation), RDVB_MATH_F32 is rdvb_conv2d_direct. bias_first:
 * the bias seeds the accumulator (Conv2DTensorOpSimple, Simple3x3, Window3x3:
 * rdv/domain/nn.py:669-999, rdv/shaders/tensors/conv2d_tensor_op_simple.h,
 * conv2d_tensor_op_simple3x3.h, conv2d_tensor_op_window3x3.h) or, with 0, is
 * added after the sum (Conv2DTensorOpFast: nn.py:608-666,
 * conv2d_tensor_op_fast.h). */
int rdvb_conv2d_direct_staged(const void* x, int x_dtype, int n, int h, int w, int cin, int cout, int kh, int kw,
                              const float* weight, const float* bias, int math, int bias_first, float* y,
                              void* stream);

/* The reference's tensor-core convolutions on tcgen05 (implicit GEMM, one
 * M=128 x N=cout MMA per tap and 16 input channels, fp32 accumulation in
 * TMEM, bias added in the epilogue). Eligible shapes: cin 16..64 and cout
 * 16..256, multiples of 16, kh*kw <= 25, the taps' weights fitting shared
 * memory; rdvb_conv_tc_packed_bytes returns 0 otherwise.
 *  rdvb_conv_tc_pack: weight [kh, kw, cin, cout] fp32 (device) -> wpack
 *    (256-byte aligned, rdvb_conv_tc_packed_bytes bytes) as float16
 *    (operand RDVB_F16) or bfloat16 (RDVB_BF16).
 *  rdvb_conv2d_tc: x [n*h*w, cin] (RDVB_F32 or RDVB_F16, 16-byte aligned)
 *    -> y [n*h*w, cout] fp32 (16-byte aligned), 'same' padding, stride 1. */
int64_t rdvb_conv_tc_packed_bytes(int kh, int kw, int cin, int cout);
int rdvb_conv_tc_pack(const float* weight, int kh, int kw, int cin, int cout, int operand, void* wpack,
                      void* stream);
int rdvb_conv2d_tc(const void* x, int x_dtype, int n, int h, int w, int cin, int cout, int kh, int kw,
                   const void* wpack, int operand, const float* bias, float* y, void* stream);

/* TensorSampler (rdv/maths/__init__.py:2050-2083,
 * rdv/shaders/samplers/tensor_sampler.h): y[i] = multilinear (linear) or
 * nearest lookup of t [shape[0], ..., shape[in_dim-1], out_dim] fp32 at
 * x[i] in [-1, 1]^in_dim (x [n, in_dim] fp32; coordinate in_dim-1-d runs
 * along dimension d). clamp: corners outside t take the clamped index (else
 * they contribute 0); aligned: -1/+1 at the first/last cell centres (else at
 * the outer edges). in_dim 1..3; y [n, out_dim] fp32. */
int rdvb_tensor_sampler(const float* t, int in_dim, const int* shape, int out_dim, const float* x, int64_t n,
                        int clamp, int aligned, int linear, float* y, void* stream);

/* GridSampler (rdv/maths/__init__.py:2018-2047,
 * rdv/shaders/samplers/grid_sampler.h) over a dense grid (a TensorGrid,
 * grids/tensor_grid.h): grid [shape[0], ..., shape[in_dim-1], out_dim] fp32
 * row-major, x [n, in_dim] fp32 in [-1, 1]^in_dim (coordinate in_dim-1-d
 * along dimension d) -> y [n, out_dim] fp32. Per dimension t = x * 0.5 +
 * 0.5, pos = aligned ? t (D - 1) : t D - 0.5, voxel = floor(pos), alpha =
 * pos - voxel; linear: the 2^in_dim corners in bit-mask order, weight the
 * product of alpha / (1 - alpha) over the dimensions, corners outside the
 * grid skipped unless clamp; nearest: voxel + (alpha >= 0.5). in_dim 1..4.
 * (The TensorSampler computes its positions and blends differently, so the
 * two samplers round differently on the same tensor.) */
int rdvb_grid_sampler(const float* grid, int in_dim, const int* shape, int out_dim, const float* x, int64_t n,
                      int clamp, int aligned, int linear, float* y, void* stream);

/* 2x2 average pool, stride 2 (Downsample2xTensorOp, rdv/domain/nn.py:1090-1107,
 * rdv/shaders/tensors/downsample2x_tensor_op.h): x [h, w, c] fp32 -> y
 * [h/2, w/2, c], each output ((x00 + x01) + x10) + x11, times 0.25. h, w even;
 * c a multiple of 8; x, y 16-byte aligned. */
int rdvb_downsample2x(const float* x, int h, int w, int c, float* y, void* stream);

/* Nearest-neighbour 2x upsample (Upsample2xTensorOp, nn.py:1110-1124,
 * rdv/shaders/tensors/upsample2x_tensor_op.h): x [h, w, c] -> y [2h, 2w, c]. */
int rdvb_upsample2x(const float* x, int h, int w, int c, float* y, void* stream);

/* Channel concatenation (ConcatTensorOp, nn.py:1127-1150,
 * rdv/shaders/tensors/concat_tensor_op.h): x1 [rows, c1] | x2 [rows, c2] ->
 * y [rows, c1 + c2]; c1, c2 multiples of 8; 16-byte aligned pointers. */
int rdvb_concat_channels(const float* x1, int c1, const float* x2, int c2, int64_t rows, float* y, void* stream);

/* ---------------------------------------------------------- ray-march ----
 * Pinhole camera rays through a volume whose density and colour come from an
 * MLP, rendered front to back.
 *
 * Replaces: the reference's Cameras grid (rdv/domain/rendering.py:10-42,
 * rdv/shaders/rendering/cameras.h:1-20), its implicit [-1,1]^3 box
 * (rdv/shaders/libraries/math_library.h:48-57, miss rule and entry clamp of
 * rdv/shaders/volumes/raymarching_transmittance.h:11-19) and the per-sample
 * MLP evaluation of a Cameras >> RaymarchingTransmittance(extinction=mlp)
 * sensor (rdv/domain/volumes.py:124-141). The emission-absorption
 * compositing (softplus density, sigmoid colour, RGBA with A = 1 - T) has no
 * reference counterpart; it follows the BASELINE volume-render workload.
 */

/* Cameras: out [n_cameras, height, width, 6] = (origin, unit direction) of
 * each pixel-centre ray; poses [n_cameras, 9] = origin | target | up (device).
 * aspect <= 0 means width / height, fov <= 0 means pi / 4 (the reference's
 * defaults). */
int rdvb_camera_rays(const float* poses, int n_cameras, int width, int height, float aspect, float fov, float* out,
                     void* stream);

/* Cameras with pixel_jitter (rdv/domain/rendering.py:24-42, jitter=True;
 * rdv/shaders/rendering/cameras.h:7): as rdvb_camera_rays, but the ray of
 * pixel i = (camera, row, column) flattened passes through (column + r0,
 * row + r1) instead of the pixel centre, r0 and r1 the first two draws of
 * the reference generator (random_library.h:7-34) started from the 4 host
 * seeds spawned by index i (random_library.h:44-49, :256-268). */
int rdvb_camera_rays_jittered(const float* poses, int n_cameras, int width, int height, float aspect, float fov,
                              const uint32_t* seeds, float* out, void* stream);

/* Workspace bytes rdvb_raymarch_render needs for a width x height image. */
int64_t rdvb_raymarch_workspace_bytes(int width, int height);

/* Renders rows [row_begin, row_end) of a width x height image from the camera
 * pose9 (HOST array: origin | target | up): every ray is clipped to the
 * [-1,1]^3 box and sampled at n_samples (must be 128) midpoints
 * t_i = t0 + (i + 1/2)(t1 - t0)/n; the MLP (dims[0] = 3 -> dims[n] = 4, all
 * layers RDVB_MATH_F16 or all RDVB_MATH_BF16, `packed` from rdvb_mlp_pack)
 * gives (o0, o1, o2, o3) per sample; sigma = softplus(o0), rgb = sigmoid(o1..3),
 * alpha_i = 1 - exp(-sigma_i dt), C = sum T_i alpha_i rgb_i with
 * T_i = prod_{j<i} (1 - alpha_j). rgba [(row_end-row_begin) * width, 4] fp32,
 * 16-byte aligned: (C, 1 - T_n); rays that miss the box get 0. One fused
 * tensor-core kernel evaluates and composites every ray that hits; workspace
 * (rdvb_raymarch_workspace_bytes, 256-byte aligned) holds the hit list. */
int rdvb_raymarch_render(const float* pose9, int width, int height, float fov, float aspect, int n_samples,
                         int n_layers, const int* dims, const int* layer_flags, const void* packed, int row_begin,
                         int row_end, void* workspace, size_t workspace_bytes, float* rgba, void* stream);

/* Workspace bytes rdvb_transmittance_rm needs for n_rays rays and this
 * extinction chain: 256 for exact fp32 chains (CUDA-core march); for float16
 * / bfloat16 chains (tensor-core march) also the packed weights and the
 * per-batch ray and chunk records (about 110 MB at most). Bytes 8-15 hold
 * (uint64) the number of extinction evaluations of the last call, readable
 * once it completed. */
int64_t rdvb_transmittance_workspace_bytes(int64_t n_rays, int n_layers, const int* dims, const int* layer_flags);

/* RaymarchingTransmittance (rdv/domain/volumes.py:124-141;
 * rdv/shaders/volumes/raymarching_transmittance.h:1-21 and
 * raymarching_transmittance_trait.h:1-14; replaces the Map[6, 1] dispatch of
 * Map.__call__, rdv/maths/__init__.py:1451-1487, for this node):
 * out[i] = transmittance along ray i of rays [n_rays, 6] (origin, direction;
 * fp32, device). The ray is taken to object space by the node transform
 * (transform: HOST mat4x3, 12 floats column-major -- 3x3 part, then the
 * origin; NULL = identity), clipped to the [-1, 1]^3 box (misses give 1),
 * then marched in fixed steps of step_size from the entry point: tau +=
 * extinction(x) * density_scale * step_size, 0 as soon as tau > 16, else
 * exp(-tau) once the segment (or 4096 steps) is used up.
 * The extinction is the chain of n_layers Linear / LinearFast layers (dims[0]
 * = 3, dims[n_layers] = 1, widths <= 128; weights[l] [dims[l+1], dims[l]] and
 * biases[l] fp32 device; layer_flags as rdvb_mlp_forward; input_relu applies
 * a ReLU to the position first). workspace: 256-byte aligned,
 * rdvb_transmittance_workspace_bytes() bytes. Exact fp32 chains march one
 * ray per CUDA thread exactly like the reference's loop; float16 / bfloat16
 * chains evaluate every step of a ray in 128-step chunks on the tensor cores
 * (fused MLP kernel) and combine the chunks in step order -- same result,
 * steps past an early exit are evaluated too. encoding: NULL, or a sampler
 * in front of the chain (rdvb_encoding; then every chain runs on the CUDA
 * cores). */
int rdvb_transmittance_rm(const float* rays, int64_t n_rays, const float* transform, float step_size,
                          float density_scale, const rdvb_encoding* encoding, int n_layers, const int* dims,
                          const float* const* weights,
                          const float* const* biases, const int* layer_flags, int input_relu, void* workspace,
                          size_t workspace_bytes, float* out, void* stream);

/* RatiotrackingTransmittance (rdv/domain/volumes.py:144-170;
 * rdv/shaders/volumes/ratiotracking_transmittance.h and
 * ratiotracking_transmittance_trait.h) with a VoxelMajorantField
 * (volumes.py:196-212, rdv/shaders/volumes/voxel_majorant_field.h) or a
 * SphereMajorantField (volumes.py:215-224, sphere_majorant_field.h):
 * out[i] = the ratio-tracking estimate of the transmittance along ray i of
 * rays [n_rays, 6]. Object space, box clip and misses as
 * rdvb_transmittance_rm; then from the entry point, at most 1024 times while
 * the segment lasts: free-flight step dt = min(cell exit distance,
 * -log(1 - random()) / (majorant * density_scale)); on a collision inside the
 * cell T *= 1 - extinction(x) / majorant, and below 0.05 Russian roulette
 * (random() >= T gives 0, else T = 1).
 * majorant: fp32 device grid, majorant_dims = {D, H, W} (host); the cell of
 * x is clamp(int((x * 0.5 + 0.5) * (W, H, D)), 0, dims - 1).
 * majorant_kind RDVB_MAJORANT_VOXEL: grid [D, H, W] (z, y, x; the
 * Grid[3, 1]'s tensor without its channel); the cell's majorant, up to the
 * cell's exit. RDVB_MAJORANT_SPHERE: grid [D, H, W, 2] of (majorant, radius
 * r in voxels; 8-byte aligned); the majorant up to the exit of the box of
 * half-width r voxels around the cell's centre, at least 1e-6 ahead.
 * seeds: 4 host uint32, the dispatch's generator seeds (the reference draws
 * them per dispatch, core/_common.py:66-75); ray i draws from the seeds
 * spawned by index i (libraries/random_library.h:44-49, :256-268), the
 * Taus + LCG generator of random_library.h:7-34. draws_before (0..64):
 * draws of each ray's generator already taken upstream in the same
 * invocation -- 2 when the rays come from a jittered Cameras grid composed
 * with the node (cameras.h:7 draws the pixel offset first), else 0.
 * The extinction chain as rdvb_transmittance_rm (any Linear / LinearFast /
 * ReLU chain 3 -> ... -> 1, evaluated on the CUDA cores). workspace: 256
 * bytes, 256-byte aligned; bytes 8-15 hold the number of extinction
 * evaluations of the call. */
int rdvb_transmittance_rt(const float* rays, int64_t n_rays, const float* transform, float density_scale,
                          const float* majorant, const int* majorant_dims, int majorant_kind, const uint32_t* seeds,
                          int draws_before, const rdvb_encoding* encoding, int n_layers, const int* dims,
                          const float* const* weights, const float* const* biases, const int* layer_flags,
                          int input_relu, void* workspace, size_t workspace_bytes, float* out, void* stream);

/* XRProject (rdv/domain/rendering.py:150-160, rdv/shaders/rendering/
 * xr_project.h): out[i] = dir2xr(dirs[i]) = (atan(w.x, w.z) / pi,
 * asin(clamp(w.y, -1, 1)) * 2 / pi) for dirs [n, 3] -> out [n, 2] (fp32
 * device; math_library.h:265-276, w.x nudged by 1e-7 when w.x = w.z = 0). */
int rdvb_xr_project(const float* dirs, int64_t n, float* out, void* stream);

/* PBVR (rdv/domain/volumes.py:257-326, rdv/shaders/volumes/pbvr.h):
 * out[i] (RGB, [n_rays, 3] fp32 device) = one delta-tracking path sample of
 * the radiance arriving along ray i of rays [n_rays, 6] -- unbiased, to be
 * averaged over dispatches. Object space and box clip as
 * rdvb_transmittance_rm; a ray that misses the box returns
 * environment(w). Then at most 8192 times while the segment lasts: the
 * field's (majorant, max step) at (x, w_object) -- majorant floored at
 * 1e-12 and NOT scaled (PBVR has no density scale) --, a free flight
 * -log(1 - random()) / majorant, clipped to the max step and the segment;
 * a clipped flight that used up the segment escapes, any other starts a new
 * cell; at a tentative collision random() >= extinction(x) / majorant is a
 * null collision, else a real one: throughput *= albedo (3 host floats),
 * the path ends with 0 below 1e-4 or after max_bounces real collisions, else
 * w <- Henyey-Greenstein sample around w with anisotropy g
 * (random_library.h:224-239; two draws: azimuth, then cosine) and the
 * segment restarts at x up to the box exit. An escaped path returns
 * throughput * environment(w), a path out of iterations 0.
 * Environment: env_kind RDVB_ENV_CONSTANT (env_rgb: 3 host floats) or
 * RDVB_ENV_EQUIRECT (env_image: fp32 device [H, W, 3], env_dims = {H, W}
 * host, env_flags a mask of RDVB_SAMPLER_*), looked up at
 * (atan(w.x, w.z) / pi, asin(w.y) * 2 / pi) as XRProject() >>
 * TensorSampler (math_library.h:265-276, tensor_sampler.h).
 * Majorant field, generator (seeds, draws_before), extinction chain and
 * workspace as rdvb_transmittance_rt (bytes 8-15: extinction evaluations). */
int rdvb_pbvr(const float* rays, int64_t n_rays, const float* transform, const float* majorant,
              const int* majorant_dims, int majorant_kind, const float* albedo, float g, int max_bounces,
              int env_kind, const float* env_rgb, const float* env_image, const int* env_dims, int env_flags,
              const uint32_t* seeds, int draws_before, const rdvb_encoding* encoding, int n_layers, const int* dims,
              const float* const* weights, const float* const* biases, const int* layer_flags, int input_relu,
              void* workspace, size_t workspace_bytes, float* out, void* stream);

/* PBVRT and PBVR_NEE (rdv/domain/volumes.py:326-442,
 * rdv/shaders/volumes/pbvrt.h, pbvr_nee.h): delta tracking with
 * next-event estimation toward a directional light. Per ray: object space;
 * a ray that misses the box returns 0 (PBVRT: alpha 1); entry at
 * max(0, tMin) + 1e-5; at most 16384 times: the field's raw (majorant,
 * distance), majorant + 1e-5, distance floored at 1e-5, free flight
 * -log(1 - random()) / (density_scale * majorant) clipped to the distance
 * and the segment; segment below 1e-7 ends the loop; a tentative collision
 * is null when random() >= extinction / majorant; a real one counts a
 * bounce (past max_bounces: PBVRT zeroes the throughput and ends the loop,
 * NEE returns what it has), multiplies the throughput by albedo (3 host
 * floats; the loop ends when no channel is above 1e-4), adds throughput *
 * transmittance_rt(shadow ray toward the light) * hg_phase_eval(w . l, g),
 * then scatters (hg_phase_sample). light_direction: 3 host floats,
 * normalized here (l / sqrt((x x + y y) + z z)). PBVRT (variant
 * RDVB_PBVRT, out [n_rays, 4]): after the loop, when the ray scattered,
 * alpha 0 and RGB = NEE sum * light_intensity (3 host floats) + throughput *
 * environment(w) (environment arguments as rdvb_pbvr); else RGB 0, alpha 1.
 * PBVR_NEE (RDVB_PBVR_NEE, out [n_rays, 3]): the NEE sum; the environment
 * and light_intensity are not read. PBVR_ENV (RDVB_PBVR_ENV, out
 * [n_rays, 3], rdv/domain/volumes.py:445-502, pbvr_env.h): at each real
 * collision the NEE direction and its radiance / pdf come from an
 * XREnvironmentSampler (rendering.py:281-323, xr_environment_sampler.h):
 * env_densities (device) holds its quadtree of env_levels levels (1..12),
 * 4 cumulative child probabilities per node, child c of node n being node
 * 4 n + 1 + c; one draw walks it, two more place the direction in the leaf
 * pixel; the environment arguments are the sampler's environment map; the
 * term is (transmittance * phase * throughput) * radiance / pdf;
 * light_direction and light_intensity are not read. Majorant field, generator, chain and
 * workspace as rdvb_transmittance_rt (bytes 8-15: extinction evaluations,
 * shadow rays included). */
int rdvb_pbvrt(const float* rays, int64_t n_rays, const float* transform, float density_scale, const float* majorant,
               const int* majorant_dims, int majorant_kind, const float* albedo, float g, int max_bounces,
               const float* light_direction, const float* light_intensity, int variant, int env_kind,
               const float* env_rgb, const float* env_image, const int* env_dims, int env_flags,
               const float* env_densities, int env_levels, const uint32_t* seeds, int draws_before,
               const rdvb_encoding* encoding, int n_layers, const int* dims, const float* const* weights,
               const float* const* biases, const int* layer_flags, int input_relu, void* workspace,
               size_t workspace_bytes, float* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* RDVB_H */
