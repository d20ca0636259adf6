// C ABI of the rdv B200 hot path (declared in include/rdvb.h). One
// translation unit: the kernels are included below so that the device status
// word and the kernels share a module.
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "rdvb.h"
#include "ptx.cuh"
#include "mlp_tc.cuh"
#include "mlp_simt.cuh"
#include "winograd.cuh"
#include "winograd_f43.cuh"
#include "raymarch.cuh"
#include "transmittance.cuh"
#include "resample.cuh"
#include "conv_tc.cuh"
#include "exchange.cuh"
#include "sampler.cuh"
#include "pbvr.cuh"

namespace {

thread_local std::string g_last_error;
std::atomic<long long> g_launches{0};

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(RDVB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return RDVB_OK;
}

struct DeviceInfo {
    bool init = false;
    int sm_count = 0;
    int max_smem_optin = 0;
    size_t tc_smem_set[rdvb::mlp_tc::kMaxSlots + 1][2][3][rdvb::mlp_tc::kMaxIssuers + 1] = {};  // [slots][bf16][mode][issuers]
    size_t simt_smem_set = 0;
    size_t wino_smem_set[2] = {};
    size_t trm_smem_set = 0;
    size_t rt_smem_set[2] = {};          // per encoding (absent, present)
    size_t rt_wide_smem_set[2] = {};
    size_t pbvr_smem_set[2] = {};
    size_t pbvr_wide_smem_set[2] = {};
    size_t pbvrt_smem_set[2][3] = {};    // per (encoding, variant)
    size_t pbvrt_wide_smem_set[2][3] = {};
    size_t rows_smem_set = 0;
    size_t conv_tc_smem_set = 0;
    size_t conv_tma_smem_set = 0;
    size_t wino_tma_smem_set = 0;
    size_t wino43_smem_set[4] = {};
};
constexpr int kMaxDevices = 64;
DeviceInfo g_dev[kMaxDevices];
std::mutex g_dev_mutex;

int current_device(DeviceInfo** info) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(RDVB_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return fail(RDVB_ERR_UNSUPPORTED, "device index %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_dev_mutex);
    DeviceInfo& d = g_dev[dev];
    if (!d.init) {
        cudaDeviceProp prop;
        e = cudaGetDeviceProperties(&prop, dev);
        if (e != cudaSuccess) return fail(RDVB_ERR_CUDA, "cudaGetDeviceProperties: %s", cudaGetErrorString(e));
        if (prop.major != 10) {
            return fail(RDVB_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a (B200)", dev,
                        prop.major, prop.minor);
        }
        d.sm_count = prop.multiProcessorCount;
        d.max_smem_optin = static_cast<int>(prop.sharedMemPerBlockOptin);
        d.init = true;
    }
    *info = &d;
    return RDVB_OK;
}

inline uint32_t round_up(uint32_t v, uint32_t m) { return (v + m - 1) / m * m; }
inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// ------------------------------------------------------------- MLP layout
struct PackLayout {
    bool ok = false;
    uint32_t k_pad[rdvb::mlp_tc::kMaxLayers], n_pad[rdvb::mlp_tc::kMaxLayers];
    uint32_t w_off[rdvb::mlp_tc::kMaxLayers], w_bytes[rdvb::mlp_tc::kMaxLayers];
    uint32_t b_idx[rdvb::mlp_tc::kMaxLayers];
    uint32_t total_w = 0;  // bytes of all layer blocks
    uint32_t max_w_bytes = 0;
    uint32_t bias_gofs = 0, bias_bytes = 0;
    int64_t total_bytes = 0;
};

// Per layer the K-major SW128 weight block (n_pad rows x katoms*128 bytes, a
// 1 KB multiple since n_pad is a multiple of 16), then one fp32 bias block
// for all layers (n_pad entries each).
PackLayout pack_layout(int n_layers, const int* dims) {
    PackLayout L;
    if (n_layers < 1 || n_layers > rdvb::mlp_tc::kMaxLayers || dims == nullptr) return L;
    for (int l = 0; l <= n_layers; ++l)
        if (dims[l] < 1 || dims[l] > static_cast<int>(rdvb::mlp_tc::kMaxWidth)) return L;
    uint32_t w = 0, nb = 0;
    for (int l = 0; l < n_layers; ++l) {
        L.k_pad[l] = round_up(dims[l], 16);
        L.n_pad[l] = round_up(dims[l + 1], 16);
        const uint32_t katoms = (L.k_pad[l] + 63) / 64;
        L.w_off[l] = w;
        L.w_bytes[l] = round_up(L.n_pad[l] * katoms * 128u, 1024);
        L.b_idx[l] = nb;
        nb += L.n_pad[l];
        w += L.w_bytes[l];
        L.max_w_bytes = std::max(L.max_w_bytes, L.w_bytes[l]);
    }
    L.total_w = w;
    L.bias_gofs = w;
    L.bias_bytes = round_up(nb * 4u, 16);
    L.total_bytes = static_cast<int64_t>(w) + L.bias_bytes;
    L.ok = true;
    return L;
}

int check_chain(int n_layers, const int* dims, const int* flags) {
    if (n_layers < 1 || n_layers > rdvb::mlp_simt::kMaxLayers)
        return fail(RDVB_ERR_INVALID_ARG, "n_layers must be in [1, %d], got %d", rdvb::mlp_simt::kMaxLayers, n_layers);
    if (!dims || !flags) return fail(RDVB_ERR_INVALID_ARG, "dims and layer_flags must not be NULL");
    for (int l = 0; l <= n_layers; ++l)
        if (dims[l] < 1) return fail(RDVB_ERR_INVALID_ARG, "dims[%d] = %d must be positive", l, dims[l]);
    for (int l = 0; l < n_layers; ++l) {
        const int m = flags[l] & 3;
        if (m > RDVB_MATH_BF16 || (flags[l] & ~7))
            return fail(RDVB_ERR_INVALID_ARG, "layer_flags[%d] = %d is not a valid flag set", l, flags[l]);
    }
    return RDVB_OK;
}

// Upper bound on the CTAs of the persistent MLP kernel (0 = one per SM);
// see rdvb_set_max_ctas.
std::atomic<int> g_max_ctas{0};

// Persistent-grid size on `dev` under the rdvb_set_max_ctas cap.
int persistent_ctas(const DeviceInfo* dev) {
    const int cap = g_max_ctas.load(std::memory_order_relaxed);
    return (cap > 0 && cap < dev->sm_count) ? cap : dev->sm_count;
}

// Why the tcgen05 kernel does not take a rows-mode chain, or nullptr when
// it does as far as the arguments go (the shared-memory plan, which depends
// on the device, is checked by the launcher).
const char* mlp_tc_decline(const void* x, int n_layers, const int* dims, const int* flags, const void* packed,
                           const float* y) {
    using namespace rdvb::mlp_tc;
    if (!pack_layout(n_layers, dims).ok) return "the chain has more than 16 layers or a width above 128";
    const int math = flags[0] & 3;
    if (math == RDVB_MATH_F32) return "the chain has exact fp32 (Linear) layers";
    for (int l = 1; l < n_layers; ++l)
        if ((flags[l] & 3) != math) return "the chain mixes float16, bfloat16 and fp32 layers";
    if (packed == nullptr) return "no packed weight image was given";
    if (!aligned(packed, 256)) return "the packed weight image is not 256-byte aligned";
    if (!aligned(x, 16)) return "x is not 16-byte aligned";
    if (!aligned(y, 4)) return "y is not 4-byte aligned";
    return nullptr;
}

// --------------------------------------------------- tensor-core launcher
// Launches the tcgen05 fused-MLP kernel on rows [0, n_rows) of x, or, with
// `ray` set, in ray-march mode (tiles = the rays of ray->hit_list, count on
// the device). Sets *taken when the chain fits the kernel and it launched;
// with `dry_run` it only decides (*taken) and launches nothing.
int launch_mlp_tc(const void* x, int x_dtype, int64_t n_rows, int n_layers, const int* dims, const int* flags,
                  int input_relu, const void* packed, float* y, cudaStream_t stream, DeviceInfo* dev, bool* taken,
                  const rdvb::mlp_tc::RayParams* ray = nullptr, bool dry_run = false) {
    using namespace rdvb::mlp_tc;
    *taken = false;
    if (!ray && n_rows <= 0) return RDVB_OK;
    PackLayout L = pack_layout(n_layers, dims);
    if (!L.ok || packed == nullptr) return RDVB_OK;
    const int math = flags[0] & 3;
    if (math == RDVB_MATH_F32) return RDVB_OK;
    for (int l = 1; l < n_layers; ++l)
        if ((flags[l] & 3) != math) return RDVB_OK;
    if (!aligned(packed, 256)) return RDVB_OK;
    if (!ray && (!aligned(x, 16) || !aligned(y, 4))) return RDVB_OK;

    Params p;
    memset(&p, 0, sizeof(p));
    p.x = x;
    p.y = y;
    p.wpack = static_cast<const uint8_t*>(packed);
    p.n_rows = n_rows;
    p.n_tiles = static_cast<int>((n_rows + kTileM - 1) / kTileM);
    p.in_dim = dims[0];
    p.out_dim = dims[n_layers];
    p.x_dtype = x_dtype;
    p.relu_in = input_relu ? 1 : 0;
    const int bf16 = (math == RDVB_MATH_BF16) ? 1 : 0;
    p.n_layers = n_layers;
    p.w_total_bytes = L.total_w;
    p.bias_gofs = L.bias_gofs;
    p.bias_bytes = L.bias_bytes;
    for (int l = 0; l < n_layers; ++l) {
        p.layer[l].k_pad = L.k_pad[l];
        p.layer[l].n_pad = L.n_pad[l];
        p.layer[l].w_off = L.w_off[l];
        p.layer[l].w_bytes = L.w_bytes[l];
        p.layer[l].b_idx = L.b_idx[l];
        p.layer[l].idesc = rdvb::umma_idesc_f16(L.n_pad[l], bf16);
        p.layer[l].relu = (flags[l] & RDVB_LAYER_RELU) ? 1u : 0u;
    }
    const int esize = x_dtype == RDVB_F32 ? 4 : 2;
    p.x_stage_bytes = ray ? 0u : round_up(static_cast<uint32_t>(kTileM) * dims[0] * esize, 128);
    if (ray) p.ray = *ray;
    p.y_vec4 = (p.out_dim % 4 == 0 && aligned(y, 16)) ? 1 : 0;
    const uint32_t budget = static_cast<uint32_t>(dev->max_smem_optin);

    // TMEM per slot: the fp32 accumulator (widest layer output) and the
    // 16-bit activation tile that feeds the next layer (widest hidden input,
    // two elements per column), both in multiples of 32 columns.
    uint32_t n_max = 0, act_k_max = 16;
    for (int l = 0; l < n_layers; ++l) n_max = std::max(n_max, L.n_pad[l]);
    for (int l = 1; l < n_layers; ++l) act_k_max = std::max(act_k_max, L.k_pad[l]);
    p.acc_stride = round_up(n_max, 32);
    p.act_stride = round_up(act_k_max / 2, 32);
    p.a0_bytes = ((L.k_pad[0] + 63) / 64) * kAtomBytes;

    // Shared-memory plan for a slot count: layer-0 A tiles, weights
    // (resident when they fit, else a ring of >= 2 layer blocks), one input
    // staging buffer per slot, biases, barriers. Returns the dynamic smem
    // bytes (0 = no fit).
    auto plan = [&](int slots, Params& q) -> uint32_t {
        if (static_cast<uint32_t>(slots) * (q.acc_stride + q.act_stride) > kTmemCols) return 0;
        q.act_base = slots * q.acc_stride;
        q.off_w = slots * q.a0_bytes;
        auto place = [&](uint32_t wsize) -> uint32_t {
            q.off_x = q.off_w + wsize;
            q.off_bias = round_up(q.off_x + slots * q.x_stage_bytes, 16);
            q.off_bar = round_up(q.off_bias + q.bias_bytes, 16);
            q.off_ray = round_up(q.off_bar + kBarBlockBytes, 16);
            return q.off_ray + kRayScratchBytes + 1024u;
        };
        const uint32_t resident_size = round_up(L.total_w, 1024);
        uint32_t total = place(resident_size);
        if (total <= budget) {
            q.resident = 1;
            q.w_stages = 1;
            q.w_slot_bytes = resident_size;
            return total;
        }
        q.resident = 0;
        q.w_slot_bytes = round_up(L.max_w_bytes, 1024);
        for (int st = 3; st >= 2; --st) {
            total = place(st * q.w_slot_bytes);
            if (total <= budget) {
                q.w_stages = st;
                return total;
            }
        }
        return 0;
    };
    int slots = 0;
    uint32_t smem = 0;
    int forced = 0;
    if (const char* env = getenv("RDVB_MLP_SLOTS")) forced = atoi(env);
    for (int sl = kMaxSlots; sl >= 2; sl /= 2) {  // 4 or 2: the epilogue splits its warp groups evenly
        if (forced && sl != forced) continue;
        Params q = p;
        const uint32_t need = plan(sl, q);
        if (need) {
            p = q;
            slots = sl;
            smem = need;
            break;
        }
    }
    if (!slots) return RDVB_OK;  // does not fit: CUDA-core path
    if (dry_run) {
        *taken = true;
        return RDVB_OK;
    }

    int rc = RDVB_OK;
    const int ri = ray ? (ray->march ? kModeMarch : kModeRender) : kModeRows;
    // MMA-issuing warps: with resident weights the slots are independent --
    // one issuer per slot for 4 slots (an issuer never waits on a slot that
    // is behind while another is ready), two for 2 slots; one in-order issuer
    // for streamed weights. RDVB_MLP_ISSUERS=2 keeps two issuers for 4 slots.
    int iss = p.resident ? (slots == 4 ? 4 : 2) : 1;
    if (const char* env = getenv("RDVB_MLP_ISSUERS"))
        if (atoi(env) == 2 && iss == 4) iss = 2;
    auto go = [&](auto kernel, int sl) {
        if (dev->tc_smem_set[sl][bf16][ri][iss] < smem) {
            cudaError_t e =
                cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
            if (e != cudaSuccess) {
                rc = fail(RDVB_ERR_CUDA, "cudaFuncSetAttribute(mlp_tc<%d>): %s", sl, cudaGetErrorString(e));
                return;
            }
            dev->tc_smem_set[sl][bf16][ri][iss] = smem;
        }
        // ray mode: the tile count is only known on the device; a CTA with
        // no tile exits after loading the weights
        const int groups = (p.n_tiles + sl - 1) / sl;
        const int ctas = persistent_ctas(dev);
        const int grid = ray ? ctas : std::min(ctas, groups);
        kernel<<<grid, cta_threads(iss), smem, stream>>>(p);
    };
#define RDVB_GO(S, B, R)                                                         \
    (iss == 2 ? go(mlp_tc_kernel<S, B, R, 2>, S) : go(mlp_tc_kernel<S, B, R, 1>, S))
#define RDVB_GO4(B, R) (iss == 4 ? go(mlp_tc_kernel<4, B, R, 4>, 4) : RDVB_GO(4, B, R))
    if (ray) {
        if (ri == kModeMarch) {
            if (slots == 4) bf16 ? RDVB_GO4(1, kModeMarch) : RDVB_GO4(0, kModeMarch);
            else bf16 ? RDVB_GO(2, 1, kModeMarch) : RDVB_GO(2, 0, kModeMarch);
        } else {
            if (slots == 4) bf16 ? RDVB_GO4(1, kModeRender) : RDVB_GO4(0, kModeRender);
            else bf16 ? RDVB_GO(2, 1, kModeRender) : RDVB_GO(2, 0, kModeRender);
        }
    } else {
        if (slots == 4) bf16 ? RDVB_GO4(1, kModeRows) : RDVB_GO4(0, kModeRows);
        else bf16 ? RDVB_GO(2, 1, kModeRows) : RDVB_GO(2, 0, kModeRows);
    }
#undef RDVB_GO4
#undef RDVB_GO
    if (rc) return rc;
    *taken = true;
    return check_launch("mlp_tc_kernel");
}

// The persistent rows kernel of the chain evaluator (transmittance.cuh) when
// the chain fits it: at most 8 layers, widths <= 128, weights + activation
// columns within shared memory. *taken = false otherwise.
int launch_chain_rows(const void* x, int x_dtype, int64_t row_begin, int64_t row_end, int n_layers, const int* dims,
                      const float* const* weights, const float* const* biases, const int* flags, bool force_f32,
                      int input_relu, float* y, cudaStream_t stream, DeviceInfo* dev, bool* taken) {
    using namespace rdvb::trm;
    *taken = false;
    if (const char* env = getenv("RDVB_SIMT_PERSISTENT"))
        if (atoi(env) == 0) return RDVB_OK;
    if (n_layers > kMaxLayers) return RDVB_OK;
    int maxw = 0;
    for (int l = 0; l <= n_layers; ++l) maxw = std::max(maxw, dims[l]);
    if (maxw > kMaxWidth) return RDVB_OK;
    for (int l = 0; l < n_layers; ++l)
        if (!weights[l] || !biases[l]) return fail(RDVB_ERR_INVALID_ARG, "weights[%d]/biases[%d] is NULL", l, l);
    Params p;
    memset(&p, 0, sizeof(p));
    int off = 0;
    for (int l = 0; l < n_layers; ++l) {
        Layer& L = p.layer[l];
        L.W = weights[l];
        L.b = biases[l];
        L.K = dims[l];
        L.N = dims[l + 1];
        L.chunk = L.N <= 4 ? 4 : 32;
        L.math = force_f32 ? 0 : (flags[l] & 3);
        L.relu = (flags[l] & RDVB_LAYER_RELU) ? 1 : 0;
        L.w_off = off;
        off += ((L.N + L.chunk - 1) / L.chunk) * L.chunk * L.K;
    }
    for (int l = 0; l < n_layers; ++l) {
        p.layer[l].b_off = off;
        off += (dims[l + 1] + 3) & ~3;
    }
    p.w_floats = off;
    p.n_layers = n_layers;
    p.input_relu = input_relu ? 1 : 0;
    p.maxw = maxw;
    p.x = x;
    p.x_dtype = x_dtype;
    p.y = y;
    p.row_begin = row_begin;
    p.row_end = row_end;
    const size_t w_bytes = static_cast<size_t>((off + 3) & ~3) * 4;
    const size_t budget = static_cast<size_t>(dev->max_smem_optin);
    // 128-row CTAs, several per SM where shared memory allows: on a 262,144-row
    // 3-64-64-64-4 chain they beat one 256-row CTA per SM and two rows per thread.
    const int threads = kThreads;
    const size_t smem = w_bytes + static_cast<size_t>(2 * maxw) * threads * 4;
    if (smem > budget) return RDVB_OK;
    auto kernel = chain_rows_kernel<kThreads>;
    if (dev->rows_smem_set < smem) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return fail(RDVB_ERR_CUDA, "cudaFuncSetAttribute(chain_rows): %s", cudaGetErrorString(e));
        dev->rows_smem_set = smem;
    }
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem);
    if (e != cudaSuccess)
        return fail(RDVB_ERR_CUDA, "cudaOccupancyMaxActiveBlocksPerMultiprocessor: %s", cudaGetErrorString(e));
    per_sm = std::max(per_sm, 1);
    const long long want = (row_end - row_begin + threads - 1) / threads;
    const int grid = static_cast<int>(std::max<long long>(1, std::min<long long>(want, 1LL * dev->sm_count * per_sm)));
    kernel<<<grid, threads, smem, stream>>>(p);
    *taken = true;
    return check_launch("chain_rows_kernel");
}

int launch_mlp_simt(const void* x, int x_dtype, int64_t row_begin, int64_t row_end, int n_layers, const int* dims,
                    const float* const* weights, const float* const* biases, const int* flags, bool force_f32,
                    int input_relu, float* y, cudaStream_t stream, DeviceInfo* dev) {
    using namespace rdvb::mlp_simt;
    if (row_end <= row_begin) return RDVB_OK;
    Params p;
    memset(&p, 0, sizeof(p));
    p.x = x;
    p.x_dtype = x_dtype;
    p.y = y;
    p.row_begin = row_begin;
    p.row_end = row_end;
    p.n_layers = n_layers;
    p.relu_in = input_relu ? 1 : 0;
    int maxw = 0;
    for (int l = 0; l <= n_layers; ++l) maxw = std::max(maxw, dims[l]);
    if (maxw > kMaxWidth)
        return fail(RDVB_ERR_UNSUPPORTED, "layer width %d exceeds the CUDA-core path limit %d", maxw, kMaxWidth);
    p.maxw = maxw;
    for (int l = 0; l < n_layers; ++l) {
        if (!weights[l] || !biases[l]) return fail(RDVB_ERR_INVALID_ARG, "weights[%d]/biases[%d] is NULL", l, l);
        p.layer[l].W = weights[l];
        p.layer[l].b = biases[l];
        p.layer[l].K = dims[l];
        p.layer[l].N = dims[l + 1];
        p.layer[l].math = force_f32 ? 0 : (flags[l] & 3);
        p.layer[l].relu = (flags[l] & RDVB_LAYER_RELU) ? 1 : 0;
    }
    {
        bool taken = false;
        if (int rc = launch_chain_rows(x, x_dtype, row_begin, row_end, n_layers, dims, weights, biases, flags,
                                       force_f32, input_relu, y, stream, dev, &taken))
            return rc;
        if (taken) return RDVB_OK;
    }
    const size_t smem = (2ull * maxw * kRows + static_cast<size_t>(maxw) * kOch) * sizeof(float);
    if (smem > static_cast<size_t>(dev->max_smem_optin))
        return fail(RDVB_ERR_UNSUPPORTED, "CUDA-core MLP path needs %zu bytes of shared memory", smem);
    if (dev->simt_smem_set < smem) {
        cudaError_t e =
            cudaFuncSetAttribute(mlp_simt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return fail(RDVB_ERR_CUDA, "cudaFuncSetAttribute(mlp_simt): %s", cudaGetErrorString(e));
        dev->simt_smem_set = smem;
    }
    const int64_t rows = row_end - row_begin;
    const int64_t blocks = (rows + kRows - 1) / kRows;
    if (blocks > 0x7fffffffLL) return fail(RDVB_ERR_UNSUPPORTED, "too many rows (%lld)", (long long)rows);
    mlp_simt_kernel<<<static_cast<unsigned>(blocks), kRows, smem, stream>>>(p);
    return check_launch("mlp_simt_kernel");
}

}  // namespace

extern "C" {

int rdvb_version(void) { return 100; }

int64_t rdvb_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

const char* rdvb_last_error(void) { return g_last_error.c_str(); }

int rdvb_device_status(int clear, uint32_t* status) {
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return fail(RDVB_ERR_CUDA, "cudaDeviceSynchronize: %s", cudaGetErrorString(e));
    uint32_t v = 0;
    e = cudaMemcpyFromSymbol(&v, rdvb::g_status, sizeof(v));
    if (e != cudaSuccess) return fail(RDVB_ERR_CUDA, "reading the status word: %s", cudaGetErrorString(e));
    if (clear && v) {
        const uint32_t zero = 0;
        e = cudaMemcpyToSymbol(rdvb::g_status, &zero, sizeof(zero));
        if (e != cudaSuccess) return fail(RDVB_ERR_CUDA, "clearing the status word: %s", cudaGetErrorString(e));
    }
    if (status) *status = v;
    if (v) return fail(RDVB_ERR_DEVICE_STATUS, "a kernel's bounded wait expired (status 0x%x)", v);
    return RDVB_OK;
}

int64_t rdvb_mlp_packed_bytes(int n_layers, const int* dims) {
    PackLayout L = pack_layout(n_layers, dims);
    return L.ok ? L.total_bytes : 0;
}

int rdvb_mlp_pack(int n_layers, const int* dims, const float* const* weights, const float* const* biases, int operand,
                  void* packed, void* stream) {
    using namespace rdvb::mlp_tc;
    PackLayout L = pack_layout(n_layers, dims);
    if (!L.ok) return fail(RDVB_ERR_UNSUPPORTED, "chain not eligible for the tensor-core path (n_layers <= %d, widths <= %u)",
                           kMaxLayers, kMaxWidth);
    if (operand != RDVB_F16 && operand != RDVB_BF16)
        return fail(RDVB_ERR_INVALID_ARG, "operand must be RDVB_F16 or RDVB_BF16");
    if (!packed || !aligned(packed, 256)) return fail(RDVB_ERR_INVALID_ARG, "packed must be a 256-byte aligned pointer");
    if (!weights || !biases) return fail(RDVB_ERR_INVALID_ARG, "weights/biases must not be NULL");
    DeviceInfo* dev = nullptr;
    if (int rc = current_device(&dev)) return rc;
    PackParams pp;
    memset(&pp, 0, sizeof(pp));
    pp.n_layers = n_layers;
    pp.bf16 = operand == RDVB_BF16 ? 1 : 0;
    pp.wpack = static_cast<uint8_t*>(packed);
    uint32_t chunks = 0;
    for (int l = 0; l < n_layers; ++l) {
        if (!weights[l] || !biases[l]) return fail(RDVB_ERR_INVALID_ARG, "weights[%d]/biases[%d] is NULL", l, l);
        PackLayer& pl = pp.layer[l];
        pl.W = weights[l];
        pl.b = biases[l];
        pl.K = dims[l];
        pl.N = dims[l + 1];
        pl.n_pad = L.n_pad[l];
        pl.katoms = (L.k_pad[l] + 63) / 64;
        pl.w_off = L.w_off[l];
        pl.b_idx = L.b_idx[l];
        chunks += pl.n_pad * pl.katoms * 8;
    }
    pp.bias_gofs = L.bias_gofs;
    pp.w_chunks = chunks;
    pp.total_chunks = chunks + L.bias_bytes / 16;
    const int threads = 256;
    const int blocks = std::min<int>((chunks + threads - 1) / threads, dev->sm_count * 8);
    mlp_pack_kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(pp);
    return check_launch("mlp_pack_kernel");
}

int rdvb_mlp_forward(const void* x, int x_dtype, int64_t n_rows, int n_layers, const int* dims,
                     const float* const* weights, const float* const* biases, const int* layer_flags, int input_relu,
                     int tail_exact, const void* packed, float* y, void* stream) {
    if (int rc = check_chain(n_layers, dims, layer_flags)) return rc;
    if (x_dtype != RDVB_F32 && x_dtype != RDVB_F16 && x_dtype != RDVB_BF16)
        return fail(RDVB_ERR_INVALID_ARG, "x_dtype %d is not RDVB_F32/F16/BF16", x_dtype);
    if (n_rows < 0) return fail(RDVB_ERR_INVALID_ARG, "n_rows must be >= 0");
    if (n_rows == 0) return RDVB_OK;
    if (!x || !y) return fail(RDVB_ERR_INVALID_ARG, "x and y must not be NULL");
    if (!weights || !biases) return fail(RDVB_ERR_INVALID_ARG, "weights/biases must not be NULL");
    DeviceInfo* dev = nullptr;
    if (int rc = current_device(&dev)) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);

    bool any_low = false;
    for (int l = 0; l < n_layers; ++l) any_low |= (layer_flags[l] & 3) != RDVB_MATH_F32;
    // Rows served by the tensor-core kernel: whole 32-row groups. The rest
    // (< 32 rows) go to the CUDA-core kernel: in exact fp32 when tail_exact
    // (the reference's partial-workgroup rule), else with the same staging.
    const int64_t n_main = (n_rows / 32) * 32;
    bool taken = false;
    if (any_low) {
        if (int rc = launch_mlp_tc(x, x_dtype, n_main, n_layers, dims, layer_flags, input_relu, packed, y, st, dev,
                                   &taken))
            return rc;
    }
    if (taken) {
        return launch_mlp_simt(x, x_dtype, n_main, n_rows, n_layers, dims, weights, biases, layer_flags,
                               tail_exact != 0, input_relu, y, st, dev);
    }
    if (any_low && tail_exact) {
        if (int rc = launch_mlp_simt(x, x_dtype, 0, n_main, n_layers, dims, weights, biases, layer_flags, false,
                                     input_relu, y, st, dev))
            return rc;
        return launch_mlp_simt(x, x_dtype, n_main, n_rows, n_layers, dims, weights, biases, layer_flags, true,
                               input_relu, y, st, dev);
    }
    return launch_mlp_simt(x, x_dtype, 0, n_rows, n_layers, dims, weights, biases, layer_flags, false, input_relu, y,
                           st, dev);
}

constexpr int kMaxPeers = 7;  // peer buffers per rdvb_peer_copy call (8 GPUs per node)

int rdvb_multicast_copy(const void* src, uint64_t mc_dst, int64_t bytes, int max_ctas, void* stream) {
    if (bytes < 0 || bytes % 16) return fail(RDVB_ERR_INVALID_ARG, "bytes must be a non-negative multiple of 16");
    if (bytes == 0) return RDVB_OK;
    if (!src || !mc_dst) return fail(RDVB_ERR_INVALID_ARG, "src and mc_dst must not be NULL");
    if (!aligned(src, 16) || mc_dst % 16) return fail(RDVB_ERR_INVALID_ARG, "src and mc_dst must be 16-byte aligned");
    if (max_ctas < 1) return fail(RDVB_ERR_INVALID_ARG, "max_ctas must be >= 1");
    DeviceInfo* dev = nullptr;
    if (int rc = current_device(&dev)) return rc;
    const long long n16 = bytes / 16;
    const int threads = 512;
    const int blocks = static_cast<int>(std::max<long long>(1, std::min<long long>((n16 + threads - 1) / threads,
                                                                                 max_ctas)));
    rdvb::exchange::multicast_copy_kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4*>(src), mc_dst, n16);
    return check_launch("multicast_copy_kernel");
}

int rdvb_peer_copy(const void* src, void* const* dst, int n_dst, int64_t bytes, void* stream) {
    if (n_dst < 0 || n_dst > kMaxPeers)
        return fail(RDVB_ERR_INVALID_ARG, "n_dst must be 0..%d, got %d", kMaxPeers, n_dst);
    if (bytes < 0) return fail(RDVB_ERR_INVALID_ARG, "bytes must be >= 0");
    if (bytes == 0 || n_dst == 0) return RDVB_OK;
    if (!src || !dst) return fail(RDVB_ERR_INVALID_ARG, "src and dst must not be NULL");
    for (int k = 0; k < n_dst; ++k) {
        if (!dst[k]) return fail(RDVB_ERR_INVALID_ARG, "dst[%d] is NULL", k);
        // one copy per destination (a peer GPU's memory, mapped by rdvb_ipc_open)
        cudaError_t e = cudaMemcpyAsync(dst[k], src, static_cast<size_t>(bytes), cudaMemcpyDeviceToDevice,
                                        static_cast<cudaStream_t>(stream));
        if (e != cudaSuccess) return fail(RDVB_ERR_CUDA, "cudaMemcpyAsync to peer %d: %s", k, cudaGetErrorString(e));
    }
    return RDVB_OK;
}

static_assert(sizeof(cudaIpcMemHandle_t) == RDVB_IPC_HANDLE_BYTES, "IPC handle size");

int rdvb_ipc_alloc(int64_t bytes, void** ptr, void* handle) {
    if (bytes <= 0 || !ptr || !handle) return fail(RDVB_ERR_INVALID_ARG, "bytes > 0, ptr and handle are required");
    *ptr = nullptr;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, static_cast<size_t>(bytes));
    if (e != cudaSuccess) return fail(RDVB_ERR_CUDA, "cudaMalloc(%lld): %s", (long long)bytes, cudaGetErrorString(e));
    cudaIpcMemHandle_t h;
    e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return fail(RDVB_ERR_CUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
    }
    memcpy(handle, &h, sizeof(h));
    *ptr = p;
    return RDVB_OK;
}

int rdvb_ipc_free(void* ptr) {
    if (!ptr) return RDVB_OK;
    cudaError_t e = cudaFree(ptr);
    return e == cudaSuccess ? RDVB_OK : fail(RDVB_ERR_CUDA, "cudaFree: %s", cudaGetErrorString(e));
}

int rdvb_ipc_open(const void* handle, void** ptr) {
    if (!handle || !ptr) return fail(RDVB_ERR_INVALID_ARG, "handle and ptr are required");
    *ptr = nullptr;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return fail(RDVB_ERR_CUDA, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
    *ptr = p;
    return RDVB_OK;
}

int rdvb_ipc_close(void* ptr) {
    if (!ptr) return RDVB_OK;
    cudaError_t e = cudaIpcCloseMemHandle(ptr);
    return e == cudaSuccess ? RDVB_OK : fail(RDVB_ERR_CUDA, "cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
}

int rdvb_mlp_forward_path(const void* x, int x_dtype, int64_t n_rows, int n_layers, const int* dims,
                          const int* layer_flags, const void* packed, const float* y) {
    if (int rc = check_chain(n_layers, dims, layer_flags)) return rc;
    if (x_dtype != RDVB_F32 && x_dtype != RDVB_F16 && x_dtype != RDVB_BF16)
        return fail(RDVB_ERR_INVALID_ARG, "x_dtype %d is not RDVB_F32/F16/BF16", x_dtype);
    if (n_rows < 0) return fail(RDVB_ERR_INVALID_ARG, "n_rows must be >= 0");
    g_last_error.clear();
    if (const char* why = mlp_tc_decline(x, n_layers, dims, layer_flags, packed, y)) {
        fail(RDVB_OK, "CUDA-core path: %s", why);
        return RDVB_PATH_CUDA_CORE;
    }
    if (n_rows < 32) {
        fail(RDVB_OK, "CUDA-core path: fewer than 32 rows (no whole 32-row group)");
        return RDVB_PATH_CUDA_CORE;
    }
    DeviceInfo* dev = nullptr;
    if (int rc = current_device(&dev)) return rc;
    bool taken = false;
    if (int rc = launch_mlp_tc(x, x_dtype, (n_rows / 32) * 32, n_layers, dims, layer_flags, 0, packed,
                               const_cast<float*>(y), nullptr, dev, &taken, nullptr, true))
        return rc;
    if (!taken) {
        fail(RDVB_OK, "CUDA-core path: no shared-memory plan of the tensor-core kernel fits this chain");
        return RDVB_PATH_CUDA_CORE;
    }
    return RDVB_PATH_TENSOR_CORE;
}

int rdvb_set_max_ctas(int max_ctas) {
    if (max_ctas < 0) return fail(RDVB_ERR_INVALID_ARG, "max_ctas must be >= 0 (0 = one CTA per SM)");
    g_max_ctas.store(max_ctas, std::memory_order_relaxed);
    return RDVB_OK;
}

int rdvb_get_max_ctas(void) { return g_max_ctas.load(std::memory_order_relaxed); }

int rdvb_relu(const float* x, float* y, int64_t n, void* stream) {
    if (n < 0) return fail(RDVB_ERR_INVALID_ARG, "n must be >= 0");
    if (n == 0) return RDVB_OK;
    if (!x || !y) return fail(RDVB_ERR_INVALID_ARG, "x and y must not be NULL");
    if (!aligned(x, 16) || !aligned(y, 16)) return fail(RDVB_ERR_INVALID_ARG, "x and y must be 16-byte aligned");
    DeviceInfo* dev = nullptr;
    if (int rc = current_device(&dev)) return rc;
    const int threads = 256;
    const int64_t want = (n / 4 + threads - 1) / threads;
    const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, dev->sm_count * 16)));
    rdvb::mlp_simt::relu_kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(x, y, n);
    return check_launch("relu_kernel");
}

}  // extern "C"

// ------------------------------------------------------------- 3x3 conv
namespace {

bool wino_channels_ok(int cin, int cout) {
    using rdvb::wino::kMaxChannels;
    return cin >= 16 && cout >= 16 && cin % 16 == 0 && cout % 16 == 0 && cin <= kMaxChannels &&
           cout <= kMaxChannels;
}

bool wino43_channels_ok(int cin, int cout) {
    using rdvb::wino43::kMaxChannels;
    return cin >= 1 && cout >= 1 && cin <= kMaxChannels && cout <= kMaxChannels;
}

// F(4x4,3x3) on CUDA cores (winograd_f43.cuh); arguments validated by the caller
// except the variant-specific ones.
int conv3x3_winograd_f43(const void* x, int x_dtype, int n, int h, int w, int cin, int cout, const void* u,
                         const float* bias, void* y, int y_dtype, cudaStream_t stream) {
    using namespace rdvb::wino43;
    if (!wino43_channels_ok(cin, cout))
        return fail(RDVB_ERR_UNSUPPORTED, "F4X4 needs cin, cout in [1, %d] (got %d, %d)", kMaxChannels, cin, cout);
    if (n == 0 || h == 0 || w == 0) return RDVB_OK;
    if (!x || !y || !u) return fail(RDVB_ERR_INVALID_ARG, "x, y and u_packed must not be NULL");
    const uintptr_t xa = x_dtype == RDVB_F16 ? 2 : 4, ya = y_dtype == RDVB_F16 ? 2 : 4;
    if (!aligned(x, xa) || !aligned(y, ya) || !aligned(u, 4) || (bias && !aligned(bias, 4)))
        return fail(RDVB_ERR_INVALID_ARG, "x, y, u_packed and bias must be aligned to their element size");
    const long long tiles_h = (h + kM - 1) / kM, tiles_w = (w + kM - 1) / kM;
    if (tiles_h * tiles_w > 0x7fffffffLL) return fail(RDVB_ERR_UNSUPPORTED, "image too large (%d x %d)", h, w);
    DeviceInfo* dev = nullptr;
    if (int rc = current_device(&dev)) return rc;
    Params p;
    memset(&p, 0, sizeof(p));
    p.x = x;
    p.y = y;
    p.u = static_cast<const float*>(u);
    p.bias = bias;
    p.h = h;
    p.w = w;
    p.cin = cin;
    p.cout = cout;
    p.y_f16 = y_dtype == RDVB_F16 ? 1 : 0;
    p.tiles_w = static_cast<int>(tiles_w);
    p.tiles_per_img = static_cast<int>(tiles_h * tiles_w);
    p.n_tiles = static_cast<long long>(n) * p.tiles_per_img;
    // 8 tiles per block when their V and M fit in shared memory, else 4
    const int bt = smem_bytes(cin, cout, 8) <= static_cast<size_t>(dev->max_smem_optin) ? 8 : 4;
    const size_t smem = smem_bytes(cin, cout, bt);
    if (smem > static_cast<size_t>(dev->max_smem_optin))
        return fail(RDVB_ERR_UNSUPPORTED, "F4X4 kernel needs %zu bytes of shared memory", smem);
    const int xi = x_dtype == RDVB_F16 ? 1 : 0;
    const int ki = 2 * xi + (bt == 8 ? 1 : 0);
    const void* kernel = nullptr;
    switch (ki) {
        case 0: kernel = reinterpret_cast<const void*>(winograd_f43_kernel<false, 4>); break;
        case 1: kernel = reinterpret_cast<const void*>(winograd_f43_kernel<false, 8>); break;
        case 2: kernel = reinterpret_cast<const void*>(winograd_f43_kernel<true, 4>); break;
        default: kernel = reinterpret_cast<const void*>(winograd_f43_kernel<true, 8>); break;
    }
    if (dev->wino43_smem_set[ki] < smem) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return fail(RDVB_ERR_CUDA, "cudaFuncSetAttribute(winograd_f43): %s", cudaGetErrorString(e));
        dev->wino43_smem_set[ki] = smem;
    }
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, smem);
    if (e != cudaSuccess)
        return fail(RDVB_ERR_CUDA, "cudaOccupancyMaxActiveBlocksPerMultiprocessor: %s", cudaGetErrorString(e));
    const long long blocks = (p.n_tiles + bt - 1) / bt;
    const int grid = static_cast<int>(std::max<long long>(1, std::min<long long>(blocks, 1LL * dev->sm_count * std::max(per_sm, 1))));
    void* args[] = {&p};
    e = cudaLaunchKernel(kernel, dim3(grid), dim3(kThreads), args, smem, stream);
    if (e != cudaSuccess) return fail(RDVB_ERR_CUDA, "winograd_f43_kernel launch: %s", cudaGetErrorString(e));
    return check_launch("winograd_f43_kernel");
}

}  // namespace

extern "C" {

int64_t rdvb_winograd_packed_bytes(int variant, int cin, int cout) {
    if (variant == RDVB_WINOGRAD_F4X4)
        return wino43_channels_ok(cin, cout) ? 36LL * cin * cout * static_cast<int64_t>(sizeof(float)) : 0;
    if (variant != RDVB_WINOGRAD_F2X2 || !wino_channels_ok(cin, cout)) return 0;
    return 16LL * cout * 128;
}

int rdvb_winograd_filter_transform(const float* w_33io, int cin, int cout, int variant, void* u_plain,
                                   void* u_packed, void* stream) {
    if (variant != RDVB_WINOGRAD_F2X2 && variant != RDVB_WINOGRAD_F4X4)
        return fail(RDVB_ERR_INVALID_ARG, "unknown Winograd variant %d", variant);
    if (cin < 1 || cout < 1) return fail(RDVB_ERR_INVALID_ARG, "cin (%d) and cout (%d) must be positive", cin, cout);
    if (!w_33io) return fail(RDVB_ERR_INVALID_ARG, "w_33io must not be NULL");
    if (variant == RDVB_WINOGRAD_F4X4) {
        // the packed operand of F(4x4) is the plain [36][cin][cout] fp32 array
        if (!wino43_channels_ok(cin, cout))
            return fail(RDVB_ERR_UNSUPPORTED, "F4X4 needs cin, cout in [1, %d] (got %d, %d)",
                        rdvb::wino43::kMaxChannels, cin, cout);
        if ((u_plain && !aligned(u_plain, 4)) || (u_packed && !aligned(u_packed, 4)))
            return fail(RDVB_ERR_INVALID_ARG, "u_plain and u_packed must be 4-byte aligned");
        if (!u_plain && !u_packed) return RDVB_OK;
        DeviceInfo* dev = nullptr;
        if (int rc = current_device(&dev)) return rc;
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        const long long total = static_cast<long long>(cin) * cout;
        const int threads = 256;
        const int blocks = static_cast<int>(std::max<long long>(
            1, std::min<long long>((total + threads - 1) / threads, 4LL * dev->sm_count)));
        for (void* dst : {u_plain, u_packed}) {
            if (!dst) continue;
            rdvb::wino43::winograd_f43_filter_kernel<<<blocks, threads, 0, st>>>(w_33io, cin, cout,
                                                                                 static_cast<float*>(dst));
            if (int rc = check_launch("winograd_f43_filter_kernel")) return rc;
        }
        return RDVB_OK;
    }
    if (u_packed) {
        if (!wino_channels_ok(cin, cout))
            return fail(RDVB_ERR_UNSUPPORTED, "packed operand needs cin, cout multiples of 16 in [16, %d] (got %d, %d)",
                        rdvb::wino::kMaxChannels, cin, cout);
        if (!aligned(u_packed, 256)) return fail(RDVB_ERR_INVALID_ARG, "u_packed must be 256-byte aligned");
    }
    if (!u_plain && !u_packed) return RDVB_OK;
    DeviceInfo* dev = nullptr;
    if (int rc = current_device(&dev)) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (u_packed) {
        // the bytes of each 128-byte row past cin are never read; zero them anyway
        cudaError_t e = cudaMemsetAsync(u_packed, 0, rdvb_winograd_packed_bytes(variant, cin, cout), st);
        if (e != cudaSuccess) return fail(RDVB_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
    }
    const int total = cin * cout;
    const int threads = 256;
    const int blocks = std::max(1, std::min((total + threads - 1) / threads, dev->sm_count * 4));
    rdvb::wino::winograd_f23_filter_kernel<<<blocks, threads, 0, st>>>(
        w_33io, cin, cout, static_cast<__half*>(u_plain), static_cast<uint8_t*>(u_packed));
    return check_launch("winograd_f23_filter_kernel");
}

namespace {
// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against the driver library); null when the driver does not provide it.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    });
    return fn;
}

// The TMA-fed Winograd kernel for float16 input with 64 channels. Returns
// RDVB_OK with *taken = false when the driver or the shapes do not allow it.
int launch_winograd_tma(const void* x, int n, int h, int w, int cout, const void* u_packed, const float* bias,
                        void* y, int y_f16, cudaStream_t stream, DeviceInfo* dev, bool* taken);
}  // namespace

int rdvb_conv3x3_winograd(const void* x, int x_dtype, int n, int h, int w, int cin, int cout,
                          const void* u_packed, int variant, const float* bias, void* y, int y_dtype,
                          void* stream) {
    using namespace rdvb::wino;
    if (variant != RDVB_WINOGRAD_F2X2 && variant != RDVB_WINOGRAD_F4X4)
        return fail(RDVB_ERR_INVALID_ARG, "unknown Winograd variant %d", variant);
    if (x_dtype != RDVB_F32 && x_dtype != RDVB_F16)
        return fail(RDVB_ERR_INVALID_ARG, "x_dtype must be RDVB_F32 or RDVB_F16");
    if (y_dtype != RDVB_F32 && y_dtype != RDVB_F16)
        return fail(RDVB_ERR_INVALID_ARG, "y_dtype must be RDVB_F32 or RDVB_F16");
    if (n < 0 || h < 0 || w < 0) return fail(RDVB_ERR_INVALID_ARG, "n, h, w must be >= 0");
    if (variant == RDVB_WINOGRAD_F4X4)
        return conv3x3_winograd_f43(x, x_dtype, n, h, w, cin, cout, u_packed, bias, y, y_dtype,
                                    static_cast<cudaStream_t>(stream));
    if (!wino_channels_ok(cin, cout))
        return fail(RDVB_ERR_UNSUPPORTED, "cin, cout must be multiples of 16 in [16, %d] (got %d, %d)", kMaxChannels,
                    cin, cout);
    if (n == 0 || h == 0 || w == 0) return RDVB_OK;
    if (!x || !y || !u_packed) return fail(RDVB_ERR_INVALID_ARG, "x, y and u_packed must not be NULL");
    if (!aligned(x, 16) || !aligned(y, 16) || !aligned(u_packed, 16))
        return fail(RDVB_ERR_INVALID_ARG, "x, y and u_packed must be 16-byte aligned");
    if (bias && !aligned(bias, 4)) return fail(RDVB_ERR_INVALID_ARG, "bias must be 4-byte aligned");
    const long long tiles_w = (w + 1) / 2, tiles_h = (h + 1) / 2;
    const long long n_tiles = static_cast<long long>(n) * tiles_h * tiles_w;
    if (n_tiles > 0x7fffffffLL - kTileM) return fail(RDVB_ERR_UNSUPPORTED, "too many tiles (%lld)", n_tiles);
    DeviceInfo* dev = nullptr;
    if (int rc = current_device(&dev)) return rc;
    if (x_dtype == RDVB_F16 && cin == 64) {
        bool taken = false;
        if (int rc = launch_winograd_tma(x, n, h, w, cout, u_packed, bias, y, y_dtype == RDVB_F16 ? 1 : 0,
                                         static_cast<cudaStream_t>(stream), dev, &taken))
            return rc;
        if (taken) return RDVB_OK;
    }

    Params p;
    memset(&p, 0, sizeof(p));
    p.x = x;
    p.y = y;
    p.u_pack = static_cast<const uint8_t*>(u_packed);
    p.bias = bias;
    p.h = h;
    p.w = w;
    p.cin = cin;
    p.cout = cout;
    p.y_f16 = y_dtype == RDVB_F16 ? 1 : 0;
    p.tiles_w = static_cast<int>(tiles_w);
    p.tiles_per_img = static_cast<int>(tiles_w * tiles_h);
    p.n_tiles = static_cast<int>(n_tiles);
    p.n_blocks = static_cast<int>((n_tiles + kBlockTiles - 1) / kBlockTiles);
    p.u_bytes = static_cast<uint32_t>(rdvb_winograd_packed_bytes(variant, cin, cout));
    p.off_a = round_up(p.u_bytes, 1024);
    p.off_bar = p.off_a + 4 * kATileBytes;
    p.idesc = rdvb::umma_idesc_f16(static_cast<uint32_t>(cout), 0);
    const uint32_t smem = p.off_bar + kBarBlockBytes + 1024u;
    if (smem > static_cast<uint32_t>(dev->max_smem_optin))
        return fail(RDVB_ERR_UNSUPPORTED, "Winograd kernel needs %u bytes of shared memory", smem);
    const int xi = x_dtype == RDVB_F16 ? 1 : 0;
    auto kernel = xi ? winograd_f23_kernel<true> : winograd_f23_kernel<false>;
    if (dev->wino_smem_set[xi] < smem) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return fail(RDVB_ERR_CUDA, "cudaFuncSetAttribute(winograd): %s", cudaGetErrorString(e));
        dev->wino_smem_set[xi] = smem;
    }
    const int grid = std::min(dev->sm_count, p.n_blocks);
    kernel<<<grid, kThreads, smem, static_cast<cudaStream_t>(stream)>>>(p);
    return check_launch("winograd_f23_kernel");
}

namespace {
int launch_winograd_tma(const void* x, int n, int h, int w, int cout, const void* u_packed, const float* bias,
                        void* y, int y_f16, cudaStream_t stream, DeviceInfo* dev, bool* taken) {
    using namespace rdvb::wino;
    *taken = false;
    if (const char* env = getenv("RDVB_WINO_TMA"))
        if (atoi(env) == 0) return RDVB_OK;
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc) return RDVB_OK;
    const long long tiles_h = (h + 1) / 2, tiles_w = (w + 1) / 2;
    const long long blocks_h = (tiles_h + kTBlockTR - 1) / kTBlockTR, blocks_w = (tiles_w + kTBlockTC - 1) / kTBlockTC;
    const long long n_blocks = static_cast<long long>(n) * blocks_h * blocks_w;
    if (n_blocks > 0x7fffffffLL) return RDVB_OK;
    TmaParams p;
    memset(&p, 0, sizeof(p));
    const cuuint64_t dims[4] = {64, static_cast<cuuint64_t>(w), static_cast<cuuint64_t>(h),
                                static_cast<cuuint64_t>(n)};
    const cuuint64_t strides[3] = {128, static_cast<cuuint64_t>(w) * 128, static_cast<cuuint64_t>(h) * w * 128};
    const cuuint32_t box[4] = {64, kTBoxW, kTBoxH, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    if (enc(&p.tmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(x), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return RDVB_OK;
    p.y = y;
    p.u_pack = static_cast<const uint8_t*>(u_packed);
    p.bias = bias;
    p.h = h;
    p.w = w;
    p.cout = cout;
    p.y_f16 = y_f16;
    p.tiles_h = static_cast<int>(tiles_h);
    p.tiles_w = static_cast<int>(tiles_w);
    p.blocks_h = static_cast<int>(blocks_h);
    p.blocks_w = static_cast<int>(blocks_w);
    p.n_blocks = static_cast<int>(n_blocks);
    p.u_pos_bytes = static_cast<uint32_t>(cout) * 128u;
    p.off_v = kTBoxBytes;
    p.off_u = p.off_v + 4 * kATileBytes;
    p.off_bar = p.off_u + kURing * p.u_pos_bytes;
    p.idesc = rdvb::umma_idesc_f16(static_cast<uint32_t>(cout), 0);
    const uint32_t smem = p.off_bar + kTBarBlockBytes + 1024u;
    if (smem > static_cast<uint32_t>(dev->max_smem_optin)) return RDVB_OK;
    if (dev->wino_tma_smem_set < smem) {
        cudaError_t e = cudaFuncSetAttribute(winograd_f23_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return fail(RDVB_ERR_CUDA, "cudaFuncSetAttribute(winograd_tma): %s", cudaGetErrorString(e));
        dev->wino_tma_smem_set = smem;
    }
    const int grid = static_cast<int>(std::min<long long>(dev->sm_count, n_blocks));
    winograd_f23_tma_kernel<<<grid, kTWThreads, smem, stream>>>(p);
    *taken = true;
    return check_launch("winograd_f23_tma_kernel");
}
}  // namespace

int rdvb_conv2d_direct_staged(const void* x, int x_dtype, int n, int h, int w, int cin, int cout, int kh, int kw,
                              const float* weight, const float* bias, int math, int bias_first, float* y,
                              void* stream) {
    if (x_dtype != RDVB_F32 && x_dtype != RDVB_F16)
        return fail(RDVB_ERR_INVALID_ARG, "x_dtype must be RDVB_F32 or RDVB_F16");
    if (math != RDVB_MATH_F32 && math != RDVB_MATH_F16 && math != RDVB_MATH_BF16)
        return fail(RDVB_ERR_INVALID_ARG, "math must be RDVB_MATH_F32, _F16 or _BF16");
    if (n < 0 || h < 0 || w < 0) return fail(RDVB_ERR_INVALID_ARG, "n, h, w must be >= 0");
    if (cin < 1 || cout < 8 || cout % 8 != 0)
        return fail(RDVB_ERR_INVALID_ARG, "cin must be >= 1 and cout a positive multiple of 8 (got %d, %d)", cin, cout);
    if (kh < 1 || kw < 1) return fail(RDVB_ERR_INVALID_ARG, "kh and kw must be >= 1");
    if (n == 0 || h == 0 || w == 0) return RDVB_OK;
    if (!x || !weight || !y) return fail(RDVB_ERR_INVALID_ARG, "x, weight and y must not be NULL");
    if (!aligned(weight, 16) || !aligned(y, 16))
        return fail(RDVB_ERR_INVALID_ARG, "weight and y must be 16-byte aligned");
    DeviceInfo* dev = nullptr;
    if (int rc = current_device(&dev)) return rc;
    const long long total = static_cast<long long>(n) * h * w * (cout / 8);
    const int threads = 256;
    const int blocks = static_cast<int>(std::max<long long>(1, std::min<long long>((total + threads - 1) / threads,
                                                                               dev->sm_count * 32LL)));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    using rdvb::wino::conv2d_direct_kernel;
    const bool x16 = x_dtype == RDVB_F16;
    const bool bf = bias_first != 0;
#define RDVB_CONV(X, M, B) conv2d_direct_kernel<X, M, B><<<blocks, threads, 0, st>>>(x, weight, bias, y, n, h, w, cin, cout, kh, kw)
    if (math == RDVB_MATH_F32) {
        x16 ? RDVB_CONV(true, 0, true) : RDVB_CONV(false, 0, true);
    } else if (math == RDVB_MATH_F16) {
        if (bf) x16 ? RDVB_CONV(true, 1, true) : RDVB_CONV(false, 1, true);
        else x16 ? RDVB_CONV(true, 1, false) : RDVB_CONV(false, 1, false);
    } else {
        if (bf) x16 ? RDVB_CONV(true, 2, true) : RDVB_CONV(false, 2, true);
        else x16 ? RDVB_CONV(true, 2, false) : RDVB_CONV(false, 2, false);
    }
#undef RDVB_CONV
    return check_launch("conv2d_direct_kernel");
}

namespace {
// Shared-memory bytes of conv_tc_kernel for these shapes (0: not eligible).
uint32_t conv_tc_smem(int kh, int kw, int cin, int cout, int budget) {
    using namespace rdvb::convtc;
    if (kh < 1 || kw < 1 || kh * kw > kMaxTaps) return 0;
    if (cin < 16 || cin % 16 || cin > kMaxCin || cout < 16 || cout % 16 || cout > kMaxCout) return 0;
    const uint32_t w_bytes = static_cast<uint32_t>(kh * kw) * cout * 128u;
    const uint32_t off_a = (w_bytes + 1023u) & ~1023u;
    const uint32_t total = off_a + kRing * kATileBytes + kBarBlockBytes + 1024u;
    return total <= static_cast<uint32_t>(budget) ? total : 0u;
}
}  // namespace

int64_t rdvb_conv_tc_packed_bytes(int kh, int kw, int cin, int cout) {
    DeviceInfo* dev = nullptr;
    const int budget = current_device(&dev) == RDVB_OK ? dev->max_smem_optin : 232448;
    if (!conv_tc_smem(kh, kw, cin, cout, budget)) return 0;
    return static_cast<int64_t>(kh) * kw * cout * 128;
}

int rdvb_conv_tc_pack(const float* weight, int kh, int kw, int cin, int cout, int operand, void* wpack,
                      void* stream) {
    if (operand != RDVB_F16 && operand != RDVB_BF16) return fail(RDVB_ERR_INVALID_ARG, "operand must be RDVB_F16 or RDVB_BF16");
    if (rdvb_conv_tc_packed_bytes(kh, kw, cin, cout) <= 0)
        return fail(RDVB_ERR_UNSUPPORTED, "%dx%d x %d -> %d is outside the tensor-core convolution's limits", kh, kw,
                    cin, cout);
    if (!weight || !wpack || !aligned(wpack, 256))
        return fail(RDVB_ERR_INVALID_ARG, "weight must be set and wpack 256-byte aligned");
    DeviceInfo* dev = nullptr;
    if (int rc = current_device(&dev)) return rc;
    const long long total = static_cast<long long>(kh) * kw * cout * 64;
    const int blocks = static_cast<int>(std::min<long long>((total + 255) / 256, dev->sm_count * 8LL));
    rdvb::convtc::conv_tc_pack_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        weight, kh * kw, cin, cout, operand == RDVB_BF16 ? 1 : 0, static_cast<uint8_t*>(wpack));
    return check_launch("conv_tc_pack_kernel");
}

namespace {
// The TMA-fed kernel for float16 input with 64 channels and float16
// operands. Returns RDVB_OK with *taken = false when the shapes or the
// driver do not allow it (the caller then stages on the CUDA cores).
int launch_conv_tc_tma(const void* x, int n, int h, int w, int cout, int kh, int kw, const void* wpack,
                       const float* bias, float* y, cudaStream_t stream, DeviceInfo* dev, bool* taken) {
    using namespace rdvb::convtc;
    *taken = false;
    if (const char* env = getenv("RDVB_CONV_TMA"))
        if (atoi(env) == 0) return RDVB_OK;
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc) return RDVB_OK;
    const long long blocks_w = (w + kBoxW - 1) / kBoxW, blocks_h = (h + kBoxH - 1) / kBoxH;
    const long long n_blocks = static_cast<long long>(n) * blocks_w * blocks_h;
    if (n_blocks > 0x7fffffffLL) return RDVB_OK;
    const uint32_t w_bytes = static_cast<uint32_t>(kh * kw) * cout * 128u;
    const uint32_t off_a = (w_bytes + 1023u) & ~1023u;
    const long long room = static_cast<long long>(dev->max_smem_optin) - off_a - kTBarBlockBytes - 16 - cout * 4 - 1024;
    // tiles per stream (two streams)
    const int ring = static_cast<int>(std::min<long long>(kTmaMaxRing / 2, room > 0 ? room / (2 * kATileBytes) : 0));
    if (ring < 2) return RDVB_OK;
    TmaParams p;
    memset(&p, 0, sizeof(p));
    const cuuint64_t dims[4] = {64, static_cast<cuuint64_t>(w), static_cast<cuuint64_t>(h),
                                static_cast<cuuint64_t>(n)};
    const cuuint64_t strides[3] = {64 * 2, static_cast<cuuint64_t>(w) * 128, static_cast<cuuint64_t>(h) * w * 128};
    const cuuint32_t box[4] = {64, kBoxW, kBoxH, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    if (enc(&p.tmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(x), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return RDVB_OK;
    p.y = y;
    p.wpack = static_cast<const uint8_t*>(wpack);
    p.bias = bias;
    p.n = n;
    p.h = h;
    p.w = w;
    p.cout = cout;
    p.kh = kh;
    p.kw = kw;
    p.taps = kh * kw;
    p.blocks_w = static_cast<int>(blocks_w);
    p.blocks_h = static_cast<int>(blocks_h);
    p.n_blocks = static_cast<int>(n_blocks);
    p.ring = ring;
    p.w_bytes = w_bytes;
    p.off_a = off_a;
    p.off_bar = off_a + static_cast<uint32_t>(2 * ring) * kATileBytes;
    p.idesc = rdvb::umma_idesc_f16(static_cast<uint32_t>(cout), 0);
    p.off_bias = (p.off_bar + kTBarBlockBytes + 15u) & ~15u;
    const size_t smem = p.off_bias + static_cast<size_t>(cout) * 4 + 1024;
    if (dev->conv_tma_smem_set < smem) {
        cudaError_t e = cudaFuncSetAttribute(conv_tc_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return fail(RDVB_ERR_CUDA, "cudaFuncSetAttribute(conv_tc_tma): %s", cudaGetErrorString(e));
        dev->conv_tma_smem_set = smem;
    }
    const int grid = static_cast<int>(std::min<long long>(dev->sm_count, n_blocks));
    conv_tc_tma_kernel<<<grid, kTmaThreads, smem, stream>>>(p);
    *taken = true;
    return check_launch("conv_tc_tma_kernel");
}
}  // namespace

int rdvb_conv2d_tc(const void* x, int x_dtype, int n, int h, int w, int cin, int cout, int kh, int kw,
                   const void* wpack, int operand, const float* bias, float* y, void* stream) {
    using namespace rdvb::convtc;
    if (x_dtype != RDVB_F32 && x_dtype != RDVB_F16)
        return fail(RDVB_ERR_INVALID_ARG, "x_dtype must be RDVB_F32 or RDVB_F16");
    if (operand != RDVB_F16 && operand != RDVB_BF16) return fail(RDVB_ERR_INVALID_ARG, "operand must be RDVB_F16 or RDVB_BF16");
    if (n < 0 || h < 0 || w < 0) return fail(RDVB_ERR_INVALID_ARG, "n, h, w must be >= 0");
    DeviceInfo* dev = nullptr;
    if (int rc = current_device(&dev)) return rc;
    const uint32_t smem = conv_tc_smem(kh, kw, cin, cout, dev->max_smem_optin);
    if (!smem)
        return fail(RDVB_ERR_UNSUPPORTED, "%dx%d x %d -> %d is outside the tensor-core convolution's limits", kh, kw,
                    cin, cout);
    const long long n_pix = static_cast<long long>(n) * h * w;
    if (n_pix == 0) return RDVB_OK;
    if (n_pix > (static_cast<long long>(0x7fffffff) - 1) * kTileM)
        return fail(RDVB_ERR_UNSUPPORTED, "too many pixels (%lld)", n_pix);
    if (!x || !y || !wpack) return fail(RDVB_ERR_INVALID_ARG, "x, y and wpack must not be NULL");
    if (!aligned(x, 16) || !aligned(y, 16) || !aligned(wpack, 256))
        return fail(RDVB_ERR_INVALID_ARG, "x and y must be 16-byte and wpack 256-byte aligned");
    if (bias && !aligned(bias, 4)) return fail(RDVB_ERR_INVALID_ARG, "bias must be 4-byte aligned");
    if (x_dtype == RDVB_F16 && operand == RDVB_F16 && cin == 64) {
        bool taken = false;
        if (int rc = launch_conv_tc_tma(x, n, h, w, cout, kh, kw, wpack, bias, y, static_cast<cudaStream_t>(stream),
                                        dev, &taken))
            return rc;
        if (taken) return RDVB_OK;
    }
    Params p;
    memset(&p, 0, sizeof(p));
    p.x = x;
    p.y = y;
    p.wpack = static_cast<const uint8_t*>(wpack);
    p.bias = bias;
    p.n_pix = n_pix;
    p.h = h;
    p.w = w;
    p.cin = cin;
    p.cout = cout;
    p.kh = kh;
    p.kw = kw;
    p.taps = kh * kw;
    p.x_f16 = x_dtype == RDVB_F16 ? 1 : 0;
    p.bf16 = operand == RDVB_BF16 ? 1 : 0;
    p.n_blocks = static_cast<int>((n_pix + kTileM - 1) / kTileM);
    p.w_bytes = static_cast<uint32_t>(p.taps) * cout * 128u;
    p.off_a = (p.w_bytes + 1023u) & ~1023u;
    p.off_bar = p.off_a + kRing * kATileBytes;
    p.idesc = rdvb::umma_idesc_f16(static_cast<uint32_t>(cout), p.bf16);
    if (dev->conv_tc_smem_set < smem) {
        cudaError_t e = cudaFuncSetAttribute(conv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return fail(RDVB_ERR_CUDA, "cudaFuncSetAttribute(conv_tc): %s", cudaGetErrorString(e));
        dev->conv_tc_smem_set = smem;
    }
    const int grid = std::min(dev->sm_count, p.n_blocks);
    conv_tc_kernel<<<grid, kThreads, smem, static_cast<cudaStream_t>(stream)>>>(p);
    return check_launch("conv_tc_kernel");
}

int rdvb_conv2d_direct(const void* x, int x_dtype, int n, int h, int w, int cin, int cout, int kh, int kw,
                       const float* weight, const float* bias, float* y, void* stream) {
    return rdvb_conv2d_direct_staged(x, x_dtype, n, h, w, cin, cout, kh, kw, weight, bias, RDVB_MATH_F32, 1, y,
                                     stream);
}

namespace {
int resample_grid(long long items, DeviceInfo* dev) {
    return static_cast<int>(std::max<long long>(1, std::min<long long>((items + 255) / 256, dev->sm_count * 16LL)));
}
int check_rows_channels(const void* a, const void* b, int c) {
    if (c < 8 || c % 8 != 0) return fail(RDVB_ERR_INVALID_ARG, "channels must be a positive multiple of 8 (got %d)", c);
    if (!a || !b) return fail(RDVB_ERR_INVALID_ARG, "x and y must not be NULL");
    if (!aligned(a, 16) || !aligned(b, 16)) return fail(RDVB_ERR_INVALID_ARG, "x and y must be 16-byte aligned");
    return RDVB_OK;
}
}  // namespace

int rdvb_tensor_sampler(const float* t, int in_dim, const int* shape, int out_dim, const float* x, int64_t n,
                        int clamp, int aligned_centres, int linear, float* y, void* stream) {
    if (in_dim < 1 || in_dim > 3) return fail(RDVB_ERR_UNSUPPORTED, "in_dim must be 1, 2 or 3 (got %d)", in_dim);
    if (!shape) return fail(RDVB_ERR_INVALID_ARG, "shape must not be NULL");
    for (int d = 0; d < in_dim; ++d)
        if (shape[d] < 1) return fail(RDVB_ERR_INVALID_ARG, "shape[%d] = %d must be positive", d, shape[d]);
    if (out_dim < 1) return fail(RDVB_ERR_INVALID_ARG, "out_dim must be positive");
    if (n < 0) return fail(RDVB_ERR_INVALID_ARG, "n must be >= 0");
    if (n == 0) return RDVB_OK;
    if (!t || !x || !y) return fail(RDVB_ERR_INVALID_ARG, "t, x and y must not be NULL");
    DeviceInfo* dev = nullptr;
    if (int rc = current_device(&dev)) return rc;
    rdvb::sampler::Params p;
    memset(&p, 0, sizeof(p));
    p.t = t;
    p.x = x;
    p.y = y;
    p.n = n;
    p.out = out_dim;
    for (int d = 0; d < in_dim; ++d) p.dim[d] = shape[d];
    p.clamp = clamp ? 1 : 0;
    p.aligned = aligned_centres ? 1 : 0;
    p.linear = linear ? 1 : 0;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (in_dim == 3 && out_dim % 4 == 0 && aligned(t, 16) && aligned(y, 16)) {
        rdvb::sampler::GridParams q;
        memset(&q, 0, sizeof(q));
        q.t = t;
        q.x = x;
        q.y = y;
        q.n = n;
        q.out = out_dim;
        for (int d = 0; d < 3; ++d) q.dim[d] = shape[d];
        q.clamp = p.clamp;
        q.aligned = p.aligned;
        q.linear = p.linear;
        const long long items = n * (out_dim / 4);
        const int vb = static_cast<int>(std::max<long long>(1, std::min<long long>((items + 255) / 256,
                                                                                 dev->sm_count * 16LL)));
        rdvb::sampler::sampler3_vec4_kernel<false><<<vb, 256, 0, st>>>(q);
        return check_launch("sampler3_vec4_kernel");
    }
    const long long total = n * out_dim;
    const int blocks = static_cast<int>(std::max<long long>(1, std::min<long long>((total + 255) / 256,
                                                                               dev->sm_count * 16LL)));
    if (in_dim == 1) rdvb::sampler::tensor_sampler_kernel<1><<<blocks, 256, 0, st>>>(p);
    else if (in_dim == 2) rdvb::sampler::tensor_sampler_kernel<2><<<blocks, 256, 0, st>>>(p);
    else rdvb::sampler::tensor_sampler_kernel<3><<<blocks, 256, 0, st>>>(p);
    return check_launch("tensor_sampler_kernel");
}

int rdvb_grid_sampler(const float* grid, int in_dim, const int* shape, int out_dim, const float* x, int64_t n,
                      int clamp, int aligned_centres, int linear, float* y, void* stream) {
    if (in_dim < 1 || in_dim > 4) return fail(RDVB_ERR_UNSUPPORTED, "in_dim must be 1, 2, 3 or 4 (got %d)", in_dim);
    if (!shape) return fail(RDVB_ERR_INVALID_ARG, "shape must not be NULL");
    long long cells = 1;
    for (int d = 0; d < in_dim; ++d) {
        if (shape[d] < 1) return fail(RDVB_ERR_INVALID_ARG, "shape[%d] = %d must be positive", d, shape[d]);
        cells *= shape[d];
    }
    if (out_dim < 1) return fail(RDVB_ERR_INVALID_ARG, "out_dim must be positive");
    if (cells * out_dim > (1LL << 40)) return fail(RDVB_ERR_UNSUPPORTED, "the grid must hold at most 2^40 values");
    if (n < 0) return fail(RDVB_ERR_INVALID_ARG, "n must be >= 0");
    if (n == 0) return RDVB_OK;
    if (!grid || !x || !y) return fail(RDVB_ERR_INVALID_ARG, "grid, x and y must not be NULL");
    if (!aligned(grid, 4) || !aligned(x, 4) || !aligned(y, 4))
        return fail(RDVB_ERR_INVALID_ARG, "grid, x and y must be 4-byte aligned");
    DeviceInfo* dev = nullptr;
    if (int rc = current_device(&dev)) return rc;
    rdvb::sampler::GridParams p;
    memset(&p, 0, sizeof(p));
    p.t = grid;
    p.x = x;
    p.y = y;
    p.n = n;
    p.out = out_dim;
    for (int d = 0; d < in_dim; ++d) p.dim[d] = shape[d];
    p.clamp = clamp ? 1 : 0;
    p.aligned = aligned_centres ? 1 : 0;
    p.linear = linear ? 1 : 0;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (in_dim == 3 && out_dim % 4 == 0 && aligned(grid, 16) && aligned(y, 16)) {
        const long long items = n * (out_dim / 4);
        const int vb = static_cast<int>(std::max<long long>(1, std::min<long long>((items + 255) / 256,
                                                                                 dev->sm_count * 16LL)));
        rdvb::sampler::sampler3_vec4_kernel<true><<<vb, 256, 0, st>>>(p);
        return check_launch("sampler3_vec4_kernel");
    }
    const long long total = n * out_dim;
    const int blocks = static_cast<int>(std::max<long long>(1, std::min<long long>((total + 255) / 256,
                                                                               dev->sm_count * 16LL)));
    switch (in_dim) {
        case 1: rdvb::sampler::grid_sampler_kernel<1><<<blocks, 256, 0, st>>>(p); break;
        case 2: rdvb::sampler::grid_sampler_kernel<2><<<blocks, 256, 0, st>>>(p); break;
        case 3: rdvb::sampler::grid_sampler_kernel<3><<<blocks, 256, 0, st>>>(p); break;
        default: rdvb::sampler::grid_sampler_kernel<4><<<blocks, 256, 0, st>>>(p); break;
    }
    return check_launch("grid_sampler_kernel");
}

int rdvb_downsample2x(const float* x, int h, int w, int c, float* y, void* stream) {
    if (h < 0 || w < 0 || h % 2 || w % 2) return fail(RDVB_ERR_INVALID_ARG, "h and w must be even and >= 0");
    if (h == 0 || w == 0) return RDVB_OK;
    if (int rc = check_rows_channels(x, y, c)) return rc;
    DeviceInfo* dev = nullptr;
    if (int rc = current_device(&dev)) return rc;
    const long long items = static_cast<long long>(h / 2) * (w / 2) * (c / 8);
    rdvb::resample::downsample2x_kernel<<<resample_grid(items, dev), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        x, y, h, w, c);
    return check_launch("downsample2x_kernel");
}

int rdvb_upsample2x(const float* x, int h, int w, int c, float* y, void* stream) {
    if (h < 0 || w < 0) return fail(RDVB_ERR_INVALID_ARG, "h and w must be >= 0");
    if (h == 0 || w == 0) return RDVB_OK;
    if (int rc = check_rows_channels(x, y, c)) return rc;
    DeviceInfo* dev = nullptr;
    if (int rc = current_device(&dev)) return rc;
    const long long items = 4LL * h * w * (c / 8);
    rdvb::resample::upsample2x_kernel<<<resample_grid(items, dev), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        x, y, h, w, c);
    return check_launch("upsample2x_kernel");
}

int rdvb_concat_channels(const float* x1, int c1, const float* x2, int c2, int64_t rows, float* y, void* stream) {
    if (rows < 0) return fail(RDVB_ERR_INVALID_ARG, "rows must be >= 0");
    if (c1 < 8 || c1 % 8 || c2 < 8 || c2 % 8)
        return fail(RDVB_ERR_INVALID_ARG, "c1 and c2 must be positive multiples of 8 (got %d, %d)", c1, c2);
    if (rows == 0) return RDVB_OK;
    if (int rc = check_rows_channels(x1, y, c1 + c2)) return rc;
    if (!x2 || !aligned(x2, 16)) return fail(RDVB_ERR_INVALID_ARG, "x2 must be a 16-byte aligned pointer");
    DeviceInfo* dev = nullptr;
    if (int rc = current_device(&dev)) return rc;
    const long long items = rows * ((c1 + c2) / 8);
    rdvb::resample::concat_kernel<<<resample_grid(items, dev), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        x1, x2, y, rows, c1, c2);
    return check_launch("concat_kernel");
}

}  // extern "C"

// ------------------------------------------------------------- ray-march
namespace {

struct Vec3 {
    float x, y, z;
};
Vec3 v_sub(Vec3 a, Vec3 b) { return {a.x - b.x, a.y - b.y, a.z - b.z}; }
Vec3 v_cross(Vec3 a, Vec3 b) { return {a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x}; }
Vec3 v_norm(Vec3 a) {
    const float l = std::sqrt(a.x * a.x + a.y * a.y + a.z * a.z);
    return {a.x / l, a.y / l, a.z / l};
}

constexpr float kDefaultFov = 0.78539816339744830962f;  // pi / 4 (rendering.py:33)

}  // namespace

extern "C" {

int64_t rdvb_raymarch_workspace_bytes(int width, int height) {
    if (width < 1 || height < 1) return 0;
    return 256 + static_cast<int64_t>(width) * height * 4;
}

int rdvb_raymarch_render(const float* pose9, int width, int height, float fov, float aspect, int n_samples,
                         int n_layers, const int* dims, const int* layer_flags, const void* packed, int row_begin,
                         int row_end, void* workspace, size_t workspace_bytes, float* rgba, void* stream) {
    using namespace rdvb::mlp_tc;
    if (!pose9 || !dims || !layer_flags) return fail(RDVB_ERR_INVALID_ARG, "pose9, dims and layer_flags must not be NULL");
    if (width < 1 || height < 1) return fail(RDVB_ERR_INVALID_ARG, "width and height must be positive");
    if (row_begin < 0 || row_end > height || row_begin > row_end)
        return fail(RDVB_ERR_INVALID_ARG, "rows [%d, %d) are not inside [0, %d)", row_begin, row_end, height);
    if (n_samples != kTileM)
        return fail(RDVB_ERR_UNSUPPORTED, "n_samples must be %d (one tensor-core tile per ray), got %d", kTileM,
                    n_samples);
    if (int rc = check_chain(n_layers, dims, layer_flags)) return rc;
    if (dims[0] != 3 || dims[n_layers] != 4)
        return fail(RDVB_ERR_INVALID_ARG, "the MLP must map 3 -> 4 (density, r, g, b); got %d -> %d", dims[0],
                    dims[n_layers]);
    const int math = layer_flags[0] & 3;
    if (math == RDVB_MATH_F32) return fail(RDVB_ERR_UNSUPPORTED, "ray-march MLP layers must be RDVB_MATH_F16 or _BF16");
    for (int l = 1; l < n_layers; ++l)
        if ((layer_flags[l] & 3) != math) return fail(RDVB_ERR_UNSUPPORTED, "all layers must use the same arithmetic");
    PackLayout L = pack_layout(n_layers, dims);
    if (!L.ok) return fail(RDVB_ERR_UNSUPPORTED, "MLP widths must be <= %u", kMaxWidth);
    if (!packed || !aligned(packed, 256)) return fail(RDVB_ERR_INVALID_ARG, "packed must be a 256-byte aligned pointer");
    if (!rgba || !aligned(rgba, 16)) return fail(RDVB_ERR_INVALID_ARG, "rgba must be a 16-byte aligned pointer");
    const long long n_pix = static_cast<long long>(row_end - row_begin) * width;
    if (n_pix == 0) return RDVB_OK;
    const int64_t need = 256 + n_pix * 4;
    if (!workspace || !aligned(workspace, 256) || static_cast<int64_t>(workspace_bytes) < need)
        return fail(RDVB_ERR_INVALID_ARG, "workspace must be 256-byte aligned and hold %lld bytes", (long long)need);
    DeviceInfo* dev = nullptr;
    if (int rc = current_device(&dev)) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);

    // camera (cameras.h:1-20): look-at basis, computed once in fp32
    if (!(fov > 0.0f)) fov = kDefaultFov;
    if (!(aspect > 0.0f)) aspect = static_cast<float>(width) / static_cast<float>(height);
    const Vec3 o{pose9[0], pose9[1], pose9[2]}, t{pose9[3], pose9[4], pose9[5]}, n{pose9[6], pose9[7], pose9[8]};
    const Vec3 z = v_norm(v_sub(t, o));
    const Vec3 xa = v_norm(v_cross(n, z));
    const Vec3 ya = v_cross(z, xa);
    RayParams rp;
    memset(&rp, 0, sizeof(rp));
    rp.org[0] = o.x; rp.org[1] = o.y; rp.org[2] = o.z;
    rp.xa[0] = xa.x; rp.xa[1] = xa.y; rp.xa[2] = xa.z;
    rp.ya[0] = ya.x; rp.ya[1] = ya.y; rp.ya[2] = ya.z;
    rp.za[0] = z.x; rp.za[1] = z.y; rp.za[2] = z.z;
    rp.aspect = aspect;
    rp.sz = 1.0f / std::tan(fov * 0.5f);
    rp.width = width;
    rp.height = height;
    rp.row_begin = row_begin;
    int* n_hits = static_cast<int*>(workspace);
    int* hit_list = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + 256);
    rp.hit_list = hit_list;
    rp.n_hits = n_hits;
    rp.rgba = rgba;

    cudaError_t e = cudaMemsetAsync(n_hits, 0, sizeof(int), st);
    if (e != cudaSuccess) return fail(RDVB_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
    const int threads = 256;
    const int blocks = static_cast<int>(std::max<long long>(1, std::min<long long>((n_pix + threads - 1) / threads,
                                                                                   dev->sm_count * 16LL)));
    rdvb::ray::ray_compact_kernel<<<blocks, threads, 0, st>>>(rp, static_cast<int>(n_pix), hit_list, n_hits, rgba);
    if (int rc = check_launch("ray_compact_kernel")) return rc;
    bool taken = false;
    if (int rc = launch_mlp_tc(nullptr, RDVB_F32, 0, n_layers, dims, layer_flags, 0, packed, nullptr, st, dev, &taken,
                               &rp))
        return rc;
    if (!taken) return fail(RDVB_ERR_UNSUPPORTED, "MLP does not fit the tensor-core kernel");
    return RDVB_OK;
}

namespace {
constexpr int64_t kMarchBatch = 1 << 18;  // rays per tensor-core march batch
constexpr int64_t kMarchChunks = (rdvb::trm::kSafety + rdvb::mlp_tc::kTileM - 1) / rdvb::mlp_tc::kTileM;

// The tensor-core march takes chains whose layers all stage float16 (or all
// bfloat16) and that fit the fused kernel; exact fp32 chains run on the
// CUDA cores.
bool march_on_tensor_cores(int n_layers, const int* dims, const int* flags) {
    const int math = flags[0] & 3;
    if (math == RDVB_MATH_F32) return false;
    for (int l = 1; l < n_layers; ++l)
        if ((flags[l] & 3) != math) return false;
    return pack_layout(n_layers, dims).ok;
}

struct MarchWorkspace {
    int64_t packed_off, rec_off, list_off, out_off, total;
};

MarchWorkspace march_workspace(int64_t n_rays, int n_layers, const int* dims) {
    MarchWorkspace m;
    const int64_t batch = std::max<int64_t>(1, std::min(n_rays, kMarchBatch));
    m.packed_off = 256;
    m.rec_off = m.packed_off + ((rdvb_mlp_packed_bytes(n_layers, dims) + 255) / 256) * 256;
    m.list_off = m.rec_off + batch * static_cast<int64_t>(sizeof(rdvb::mlp_tc::MarchRay));
    m.out_off = m.list_off + ((batch * kMarchChunks * 4 + 255) / 256) * 256;
    m.total = m.out_off + batch * kMarchChunks * 8;
    return m;
}
}  // namespace

namespace {
// Object-space transform of the volume nodes: L = inverse of the 3x3 part
// of the node's mat4x3 (columns M[0..2]), O = M[3]
// (raymarching_transmittance.h:4-8, ratiotracking_transmittance.h:4-8);
// identity when NULL. The inverse is formed in double, rounded to float.
int trm_object_space(const float* transform, rdvb::trm::Params& p) {
    double M[3][3] = {{1, 0, 0}, {0, 1, 0}, {0, 0, 1}};  // M[row][col]
    if (transform) {
        for (int c = 0; c < 3; ++c)
            for (int r = 0; r < 3; ++r) M[r][c] = transform[3 * c + r];
        for (int r = 0; r < 3; ++r) p.O[r] = transform[9 + r];
    }
    const double det = M[0][0] * (M[1][1] * M[2][2] - M[1][2] * M[2][1]) -
                       M[0][1] * (M[1][0] * M[2][2] - M[1][2] * M[2][0]) +
                       M[0][2] * (M[1][0] * M[2][1] - M[1][1] * M[2][0]);
    if (!(std::fabs(det) > 0.0)) return fail(RDVB_ERR_INVALID_ARG, "the transform's 3x3 part is singular");
    double inv[3][3];
    inv[0][0] = (M[1][1] * M[2][2] - M[1][2] * M[2][1]) / det;
    inv[0][1] = (M[0][2] * M[2][1] - M[0][1] * M[2][2]) / det;
    inv[0][2] = (M[0][1] * M[1][2] - M[0][2] * M[1][1]) / det;
    inv[1][0] = (M[1][2] * M[2][0] - M[1][0] * M[2][2]) / det;
    inv[1][1] = (M[0][0] * M[2][2] - M[0][2] * M[2][0]) / det;
    inv[1][2] = (M[0][2] * M[1][0] - M[0][0] * M[1][2]) / det;
    inv[2][0] = (M[1][0] * M[2][1] - M[1][1] * M[2][0]) / det;
    inv[2][1] = (M[0][1] * M[2][0] - M[0][0] * M[2][1]) / det;
    inv[2][2] = (M[0][0] * M[1][1] - M[0][1] * M[1][0]) / det;
    for (int r = 0; r < 3; ++r)
        for (int c = 0; c < 3; ++c) p.L[3 * r + c] = static_cast<float>(inv[r][c]);
    return RDVB_OK;
}

// The extinction of a volume node: an optional input encoding (a sampler of
// a dense 3-D grid) and a chain of n_layers layers mapping 3 (or the
// encoding's features) to 1. Sets maxw, the widest activation column.
int check_extinction(const rdvb_encoding* enc, int n_layers, const int* dims, const float* const* weights,
                     const float* const* biases, const int* layer_flags, int& maxw) {
    using rdvb::trm::kMaxLayers;
    using rdvb::trm::kMaxWidth;
    const int min_layers = enc ? 0 : 1;
    if (n_layers < min_layers || n_layers > kMaxLayers)
        return fail(RDVB_ERR_INVALID_ARG, "n_layers must be in [%d, %d], got %d", min_layers, kMaxLayers, n_layers);
    if (!dims) return fail(RDVB_ERR_INVALID_ARG, "dims must not be NULL");
    int in = 3;
    if (enc) {
        if (enc->kind != RDVB_ENCODING_TENSOR_SAMPLER && enc->kind != RDVB_ENCODING_GRID_SAMPLER)
            return fail(RDVB_ERR_INVALID_ARG, "encoding kind must be RDVB_ENCODING_TENSOR_SAMPLER or "
                                              "RDVB_ENCODING_GRID_SAMPLER, got %d", enc->kind);
        if (!enc->grid || !aligned(enc->grid, 4))
            return fail(RDVB_ERR_INVALID_ARG, "the encoding grid must be a 4-byte aligned device pointer");
        long long cells = 1;
        for (int k = 0; k < 3; ++k) {
            if (enc->dims[k] < 1)
                return fail(RDVB_ERR_INVALID_ARG, "encoding dims must be positive, got %d", enc->dims[k]);
            cells *= enc->dims[k];
        }
        if (enc->features < 1 || enc->features > kMaxWidth)
            return fail(RDVB_ERR_UNSUPPORTED, "encoding features must be in [1, %d], got %d", kMaxWidth, enc->features);
        if (cells * enc->features > (1LL << 40)) return fail(RDVB_ERR_UNSUPPORTED, "encoding grid too large");
        if (enc->flags & ~(RDVB_SAMPLER_CLAMP | RDVB_SAMPLER_ALIGNED | RDVB_SAMPLER_LINEAR))
            return fail(RDVB_ERR_INVALID_ARG, "unknown encoding flag bits 0x%x", enc->flags);
        in = enc->features;
    }
    if (n_layers > 0) {
        if (int rc = check_chain(n_layers, dims, layer_flags)) return rc;
        if (!weights || !biases) return fail(RDVB_ERR_INVALID_ARG, "weights and biases must not be NULL");
        for (int l = 0; l < n_layers; ++l)
            if (!weights[l] || !biases[l]) return fail(RDVB_ERR_INVALID_ARG, "layer %d has a NULL weight or bias", l);
    }
    if (dims[0] != in || dims[n_layers] != 1)
        return fail(RDVB_ERR_INVALID_ARG, "the extinction must map %d -> 1, got %d -> %d", in, dims[0], dims[n_layers]);
    maxw = 3;
    for (int l = 0; l <= n_layers; ++l) {
        if (dims[l] > kMaxWidth) return fail(RDVB_ERR_UNSUPPORTED, "widths must be <= %d, got %d", kMaxWidth, dims[l]);
        maxw = std::max(maxw, dims[l]);
    }
    return RDVB_OK;
}

void fill_encoding(const rdvb_encoding* enc, rdvb::trm::Params& p) {
    if (!enc) return;
    p.enc = enc->kind == RDVB_ENCODING_TENSOR_SAMPLER ? 1 : 2;
    p.enc_t = enc->grid;
    for (int k = 0; k < 3; ++k) p.enc_dim[k] = enc->dims[k];
    p.enc_out = enc->features;
    p.enc_clamp = (enc->flags & RDVB_SAMPLER_CLAMP) ? 1 : 0;
    p.enc_aligned = (enc->flags & RDVB_SAMPLER_ALIGNED) ? 1 : 0;
    p.enc_linear = (enc->flags & RDVB_SAMPLER_LINEAR) ? 1 : 0;
}

// The CUDA-core march kernels: the chain's shared-memory weight image, then
// one launch of as many persistent 128-thread CTAs as fit (rays handed out
// by the counter at the start of the workspace).
enum class March { kRaymarch, kRatioTracking, kPbvr, kPbvrt };

// extra: the kernel's second argument (rdvb::pbvr::Extra for kPbvr,
// rdvb::pbvr::ExtraT for kPbvrt), else null.
int launch_simt_march(rdvb::trm::Params& p, int n_layers, const int* dims, const float* const* weights,
                      const float* const* biases, const int* layer_flags, void* workspace, DeviceInfo* dev,
                      cudaStream_t st, March kind, const void* extra = nullptr) {
    using namespace rdvb::trm;
    int off = 0;
    for (int l = 0; l < n_layers; ++l) {
        Layer& L = p.layer[l];
        L.W = weights[l];
        L.b = biases[l];
        L.K = dims[l];
        L.N = dims[l + 1];
        L.chunk = L.N <= 4 ? 4 : 32;
        L.math = layer_flags[l] & 3;
        L.relu = (layer_flags[l] & RDVB_LAYER_RELU) ? 1 : 0;
        L.w_off = off;
        off += ((L.N + L.chunk - 1) / L.chunk) * L.chunk * L.K;
    }
    for (int l = 0; l < n_layers; ++l) {
        p.layer[l].b_off = off;
        off += (dims[l + 1] + 3) & ~3;
    }
    p.w_floats = off;
    // ratio tracking and PBVR: 384 rays per CTA when their activation
    // columns fit (chains at most 64 wide), 128 otherwise -- the per-ray
    // activations bound how many warps an SM holds
    const size_t w_bytes = static_cast<size_t>((off + 3) & ~3) * 4;
    const bool wide = kind != March::kRaymarch &&
                      w_bytes + static_cast<size_t>(2 * p.maxw) * kRtWideThreads * 4 <=
                          static_cast<size_t>(dev->max_smem_optin);
    const int threads = wide ? kRtWideThreads : kThreads;
    const size_t smem = w_bytes + static_cast<size_t>(2 * p.maxw) * threads * 4;
    if (smem > static_cast<size_t>(dev->max_smem_optin))
        return fail(RDVB_ERR_UNSUPPORTED, "the extinction MLP needs %zu bytes of shared memory", smem);
    const void* kernel = nullptr;
    size_t* smem_set = nullptr;
    const char* name = nullptr;
    switch (kind) {
        case March::kRaymarch:
            kernel = reinterpret_cast<const void*>(transmittance_kernel);
            smem_set = &dev->trm_smem_set;
            name = "transmittance_kernel";
            break;
        case March::kRatioTracking: {
            // instantiations without the encoding's sampler code when there is none
            const void* const k[2][2] = {
                {reinterpret_cast<const void*>(ratiotracking_kernel<kThreads, false>),
                 reinterpret_cast<const void*>(ratiotracking_kernel<kThreads, true>)},
                {reinterpret_cast<const void*>(ratiotracking_kernel<kRtWideThreads, false>),
                 reinterpret_cast<const void*>(ratiotracking_kernel<kRtWideThreads, true>)}};
            kernel = k[wide ? 1 : 0][p.enc ? 1 : 0];
            smem_set = wide ? &dev->rt_wide_smem_set[p.enc ? 1 : 0] : &dev->rt_smem_set[p.enc ? 1 : 0];
            name = "ratiotracking_kernel";
            break;
        }
        case March::kPbvr: {
            const void* const k[2][2] = {
                {reinterpret_cast<const void*>(rdvb::pbvr::pbvr_kernel<kThreads, false>),
                 reinterpret_cast<const void*>(rdvb::pbvr::pbvr_kernel<kThreads, true>)},
                {reinterpret_cast<const void*>(rdvb::pbvr::pbvr_kernel<kRtWideThreads, false>),
                 reinterpret_cast<const void*>(rdvb::pbvr::pbvr_kernel<kRtWideThreads, true>)}};
            kernel = k[wide ? 1 : 0][p.enc ? 1 : 0];
            smem_set = wide ? &dev->pbvr_wide_smem_set[p.enc ? 1 : 0] : &dev->pbvr_smem_set[p.enc ? 1 : 0];
            name = "pbvr_kernel";
            break;
        }
        case March::kPbvrt: {
            using rdvb::pbvr::pbvrt_kernel;
            const int v = static_cast<const rdvb::pbvr::ExtraT*>(extra)->variant;
            const int enc = p.enc ? 1 : 0;
            const void* const kernels[2][2][3] = {
                {{reinterpret_cast<const void*>(pbvrt_kernel<kThreads, 0, false>),
                  reinterpret_cast<const void*>(pbvrt_kernel<kThreads, 1, false>),
                  reinterpret_cast<const void*>(pbvrt_kernel<kThreads, 2, false>)},
                 {reinterpret_cast<const void*>(pbvrt_kernel<kThreads, 0, true>),
                  reinterpret_cast<const void*>(pbvrt_kernel<kThreads, 1, true>),
                  reinterpret_cast<const void*>(pbvrt_kernel<kThreads, 2, true>)}},
                {{reinterpret_cast<const void*>(pbvrt_kernel<kRtWideThreads, 0, false>),
                  reinterpret_cast<const void*>(pbvrt_kernel<kRtWideThreads, 1, false>),
                  reinterpret_cast<const void*>(pbvrt_kernel<kRtWideThreads, 2, false>)},
                 {reinterpret_cast<const void*>(pbvrt_kernel<kRtWideThreads, 0, true>),
                  reinterpret_cast<const void*>(pbvrt_kernel<kRtWideThreads, 1, true>),
                  reinterpret_cast<const void*>(pbvrt_kernel<kRtWideThreads, 2, true>)}}};
            kernel = kernels[wide ? 1 : 0][enc][v];
            smem_set = wide ? &dev->pbvrt_wide_smem_set[enc][v] : &dev->pbvrt_smem_set[enc][v];
            name = "pbvrt_kernel";
            break;
        }
    }
    if (*smem_set < smem) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return fail(RDVB_ERR_CUDA, "cudaFuncSetAttribute(march): %s", cudaGetErrorString(e));
        *smem_set = smem;
    }
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem);
    if (e != cudaSuccess) return fail(RDVB_ERR_CUDA, "cudaOccupancyMaxActiveBlocksPerMultiprocessor: %s",
                                      cudaGetErrorString(e));
    per_sm = std::max(per_sm, 1);
    const long long want = (p.n_rays + threads - 1) / threads;
    const int grid = static_cast<int>(std::max<long long>(1, std::min<long long>(want, 1LL * dev->sm_count * per_sm)));
    e = cudaMemsetAsync(workspace, 0, 16, st);
    if (e != cudaSuccess) return fail(RDVB_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
    if (kind == March::kPbvr || kind == March::kPbvrt) {
        void* args[] = {&p, const_cast<void*>(extra)};
        e = cudaLaunchKernel(kernel, dim3(grid), dim3(threads), args, smem, st);
        if (e != cudaSuccess) return fail(RDVB_ERR_CUDA, "%s launch: %s", name, cudaGetErrorString(e));
    } else {
        void* args[] = {&p};
        e = cudaLaunchKernel(kernel, dim3(grid), dim3(threads), args, smem, st);
        if (e != cudaSuccess) return fail(RDVB_ERR_CUDA, "%s launch: %s", name, cudaGetErrorString(e));
    }
    return check_launch(name);
}
}  // namespace


int64_t rdvb_transmittance_workspace_bytes(int64_t n_rays, int n_layers, const int* dims, const int* layer_flags) {
    if (n_rays < 0 || n_layers < 1 || n_layers > rdvb::trm::kMaxLayers || !dims || !layer_flags) return 0;
    if (!march_on_tensor_cores(n_layers, dims, layer_flags)) return 256;
    return march_workspace(n_rays, n_layers, dims).total;
}

int rdvb_transmittance_rm(const float* rays, int64_t n_rays, const float* transform, float step_size,
                          float density_scale, const rdvb_encoding* encoding, int n_layers, const int* dims,
                          const float* const* weights, const float* const* biases, const int* layer_flags,
                          int input_relu, void* workspace, size_t workspace_bytes, float* out, void* stream) {
    using namespace rdvb::trm;
    if (n_rays < 0) return fail(RDVB_ERR_INVALID_ARG, "n_rays must be >= 0");
    int maxw = 3;
    if (int rc = check_extinction(encoding, n_layers, dims, weights, biases, layer_flags, maxw)) return rc;
    if (!(step_size > 0.0f)) return fail(RDVB_ERR_INVALID_ARG, "step_size must be > 0");
    if (n_rays > 0x7fffffffLL - (1LL << 24))
        return fail(RDVB_ERR_UNSUPPORTED, "at most %lld rays per call", 0x7fffffffLL - (1LL << 24));
    if (n_rays == 0) return RDVB_OK;
    if (!rays || !out) return fail(RDVB_ERR_INVALID_ARG, "rays and out must not be NULL");
    if (!aligned(rays, 4) || !aligned(out, 4)) return fail(RDVB_ERR_INVALID_ARG, "rays and out must be 4-byte aligned");
    const bool tc = !encoding && march_on_tensor_cores(n_layers, dims, layer_flags);
    const int64_t need = tc ? march_workspace(n_rays, n_layers, dims).total : 256;
    if (!workspace || !aligned(workspace, 256) || static_cast<int64_t>(workspace_bytes) < need)
        return fail(RDVB_ERR_INVALID_ARG, "workspace must be 256-byte aligned and hold %lld bytes", (long long)need);
    DeviceInfo* dev = nullptr;
    if (int rc = current_device(&dev)) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);

    Params p;
    memset(&p, 0, sizeof(p));
    p.rays = rays;
    p.out = out;
    p.n_rays = n_rays;
    p.counter = static_cast<int*>(workspace);
    p.evaluations = reinterpret_cast<unsigned long long*>(static_cast<uint8_t*>(workspace) + 8);
    p.step = step_size;
    p.scale = density_scale;
    p.n_layers = n_layers;
    p.input_relu = input_relu ? 1 : 0;
    p.maxw = maxw;
    fill_encoding(encoding, p);
    if (int rc = trm_object_space(transform, p)) return rc;
    if (tc) {
        // tensor-core march: pack the chain into the workspace, then per
        // batch of rays: setup -> fused MLP over the chunks -> combine
        using rdvb::mlp_tc::MarchRay;
        using rdvb::mlp_tc::RayParams;
        const MarchWorkspace m = march_workspace(n_rays, n_layers, dims);
        uint8_t* ws = static_cast<uint8_t*>(workspace);
        const int math = layer_flags[0] & 3;
        if (int rc = rdvb_mlp_pack(n_layers, dims, weights, biases, math == RDVB_MATH_BF16 ? RDVB_BF16 : RDVB_F16,
                                   ws + m.packed_off, stream))
            return rc;
        cudaError_t e = cudaMemsetAsync(ws, 0, 16, st);
        if (e != cudaSuccess) return fail(RDVB_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
        int* n_chunks = reinterpret_cast<int*>(ws);
        unsigned long long* evals = reinterpret_cast<unsigned long long*>(ws + 8);
        MarchRay* rec = reinterpret_cast<MarchRay*>(ws + m.rec_off);
        int* list = reinterpret_cast<int*>(ws + m.list_off);
        float2* cout2 = reinterpret_cast<float2*>(ws + m.out_off);
        for (int64_t b0 = 0; b0 < n_rays; b0 += kMarchBatch) {
            const int nb = static_cast<int>(std::min<int64_t>(kMarchBatch, n_rays - b0));
            e = cudaMemsetAsync(n_chunks, 0, sizeof(int), st);
            if (e != cudaSuccess) return fail(RDVB_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
            SetupParams sp;
            memset(&sp, 0, sizeof(sp));
            sp.rays = rays + b0 * 6;
            sp.out = out + b0;
            sp.n = nb;
            memcpy(sp.L, p.L, sizeof(sp.L));
            memcpy(sp.O, p.O, sizeof(sp.O));
            sp.step = step_size;
            sp.rec = rec;
            sp.chunk_list = list;
            sp.n_chunks = n_chunks;
            const int threads = 256;
            const int blocks = static_cast<int>(std::min<int64_t>((nb + threads - 1) / threads, dev->sm_count * 8LL));
            trm_setup_kernel<<<blocks, threads, 0, st>>>(sp);
            if (int rc = check_launch("trm_setup_kernel")) return rc;
            RayParams rp;
            memset(&rp, 0, sizeof(rp));
            rp.hit_list = list;
            rp.n_hits = n_chunks;
            rp.march = 1;
            rp.rec = rec;
            rp.chunk_out = cout2;
            rp.step = step_size;
            rp.scale = density_scale;
            bool taken = false;
            if (int rc = launch_mlp_tc(nullptr, RDVB_F32, 0, n_layers, dims, layer_flags, input_relu, ws + m.packed_off,
                                       nullptr, st, dev, &taken, &rp))
                return rc;
            if (!taken) return fail(RDVB_ERR_UNSUPPORTED, "extinction MLP does not fit the tensor-core kernel");
            CombineParams cp;
            cp.rec = rec;
            cp.chunk_out = cout2;
            cp.out = out + b0;
            cp.n = nb;
            cp.evaluations = evals;
            trm_combine_kernel<<<blocks, threads, 0, st>>>(cp);
            if (int rc = check_launch("trm_combine_kernel")) return rc;
        }
        return RDVB_OK;
    }
    return launch_simt_march(p, n_layers, dims, weights, biases, layer_flags, workspace, dev, st, March::kRaymarch);
}

int rdvb_xr_project(const float* dirs, int64_t n, float* out, void* stream) {
    if (n < 0) return fail(RDVB_ERR_INVALID_ARG, "n must be >= 0");
    if (n == 0) return RDVB_OK;
    if (!dirs || !out || !aligned(dirs, 4) || !aligned(out, 4))
        return fail(RDVB_ERR_INVALID_ARG, "dirs and out must be 4-byte aligned device pointers");
    DeviceInfo* dev = nullptr;
    if (int rc = current_device(&dev)) return rc;
    const long long blocks = std::min<long long>((n + 255) / 256, 1LL * dev->sm_count * 8);
    rdvb::pbvr::xr_project_kernel<<<static_cast<int>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(dirs, n,
                                                                                                          out);
    return check_launch("xr_project_kernel");
}

namespace {
// The arguments ratio tracking and PBVR share: the rays, the node's
// transform, the majorant field, the generator and the extinction chain.
// Fills p (all but the launch state) and reports whether there is any work.
int tracking_params(const float* rays, int64_t n_rays, const float* transform, const float* majorant,
                    const int* majorant_dims, int majorant_kind, const uint32_t* seeds, int draws_before,
                    const rdvb_encoding* encoding, int n_layers, const int* dims, const float* const* weights,
                    const float* const* biases, const int* layer_flags, int input_relu, void* workspace,
                    size_t workspace_bytes, void* out, rdvb::trm::Params& p, int out_dim) {
    using namespace rdvb::trm;
    if (draws_before < 0 || draws_before > 64)
        return fail(RDVB_ERR_INVALID_ARG, "draws_before must be in [0, 64], got %d", draws_before);
    if (n_rays < 0) return fail(RDVB_ERR_INVALID_ARG, "n_rays must be >= 0");
    int maxw = 3;
    if (int rc = check_extinction(encoding, n_layers, dims, weights, biases, layer_flags, maxw)) return rc;
    if (majorant_kind != RDVB_MAJORANT_VOXEL && majorant_kind != RDVB_MAJORANT_SPHERE)
        return fail(RDVB_ERR_INVALID_ARG, "majorant_kind must be RDVB_MAJORANT_VOXEL or RDVB_MAJORANT_SPHERE, got %d",
                    majorant_kind);
    if (!majorant_dims || !seeds) return fail(RDVB_ERR_INVALID_ARG, "majorant_dims and seeds must not be NULL");
    for (int k = 0; k < 3; ++k)
        if (majorant_dims[k] < 1)
            return fail(RDVB_ERR_INVALID_ARG, "majorant_dims must be positive, got %d", majorant_dims[k]);
    if (1LL * majorant_dims[0] * majorant_dims[1] * majorant_dims[2] > (1LL << 31))
        return fail(RDVB_ERR_UNSUPPORTED, "the majorant grid must have at most 2^31 cells");
    if (n_rays > 0x7fffffffLL - (1LL << 24))
        return fail(RDVB_ERR_UNSUPPORTED, "at most %lld rays per call", 0x7fffffffLL - (1LL << 24));
    if (n_rays == 0) return RDVB_OK;
    if (!rays || !out || !majorant) return fail(RDVB_ERR_INVALID_ARG, "rays, majorant and out must not be NULL");
    if (!aligned(rays, 4) || !aligned(out, 4) || !aligned(majorant, majorant_kind == RDVB_MAJORANT_SPHERE ? 8 : 4))
        return fail(RDVB_ERR_INVALID_ARG, "rays and out must be 4-byte aligned, a voxel majorant grid 4-byte and a "
                                          "sphere majorant grid 8-byte aligned");
    if (!workspace || !aligned(workspace, 256) || workspace_bytes < 256)
        return fail(RDVB_ERR_INVALID_ARG, "workspace must be 256-byte aligned and hold 256 bytes");
    memset(&p, 0, sizeof(p));
    p.rays = rays;
    p.out = out_dim == 1 ? static_cast<float*>(out) : nullptr;
    p.n_rays = n_rays;
    p.counter = static_cast<int*>(workspace);
    p.evaluations = reinterpret_cast<unsigned long long*>(static_cast<uint8_t*>(workspace) + 8);
    p.scale = 1.0f;
    p.n_layers = n_layers;
    p.input_relu = input_relu ? 1 : 0;
    p.maxw = maxw;
    p.maj = majorant;
    p.field = majorant_kind == RDVB_MAJORANT_SPHERE ? 1 : 0;
    p.mdim[0] = majorant_dims[2];  // x: W
    p.mdim[1] = majorant_dims[1];  // y: H
    p.mdim[2] = majorant_dims[0];  // z: D
    for (int k = 0; k < 3; ++k) p.mvs[k] = 2.0f / static_cast<float>(p.mdim[k]);
    for (int k = 0; k < 4; ++k) p.seeds[k] = seeds[k];
    p.draws_before = draws_before;
    fill_encoding(encoding, p);
    return trm_object_space(transform, p);
}

// The PBVR environment: a constant RGB or an equirectangular image [H, W, 3].
int environment_args(int env_kind, const float* env_rgb, const float* env_image, const int* env_dims, int env_flags,
                     int64_t n_rays, rdvb::pbvr::Extra& e) {
    if (env_kind == RDVB_ENV_CONSTANT) {
        if (!env_rgb) return fail(RDVB_ERR_INVALID_ARG, "a constant environment needs env_rgb");
        for (int k = 0; k < 3; ++k) e.env_rgb[k] = env_rgb[k];
    } else if (env_kind == RDVB_ENV_EQUIRECT) {
        if (!env_dims) return fail(RDVB_ERR_INVALID_ARG, "an equirectangular environment needs env_dims");
        if (env_dims[0] < 1 || env_dims[1] < 1)
            return fail(RDVB_ERR_INVALID_ARG, "env_dims must be positive, got %d x %d", env_dims[0], env_dims[1]);
        if (1LL * env_dims[0] * env_dims[1] > (1LL << 28))
            return fail(RDVB_ERR_UNSUPPORTED, "the environment image must have at most 2^28 pixels");
        if (env_flags & ~(RDVB_SAMPLER_CLAMP | RDVB_SAMPLER_ALIGNED | RDVB_SAMPLER_LINEAR))
            return fail(RDVB_ERR_INVALID_ARG, "unknown env_flags bits 0x%x", env_flags);
        if (n_rays > 0 && (!env_image || !aligned(env_image, 4)))
            return fail(RDVB_ERR_INVALID_ARG, "env_image must be a 4-byte aligned device pointer");
        e.env_kind = 1;
        e.env = env_image;
        e.env_h = env_dims[0];
        e.env_w = env_dims[1];
        e.env_clamp = (env_flags & RDVB_SAMPLER_CLAMP) ? 1 : 0;
        e.env_aligned = (env_flags & RDVB_SAMPLER_ALIGNED) ? 1 : 0;
        e.env_linear = (env_flags & RDVB_SAMPLER_LINEAR) ? 1 : 0;
    } else {
        return fail(RDVB_ERR_INVALID_ARG, "env_kind must be RDVB_ENV_CONSTANT or RDVB_ENV_EQUIRECT, got %d", env_kind);
    }
    return RDVB_OK;
}
}  // namespace

int rdvb_transmittance_rt(const float* rays, int64_t n_rays, const float* transform, float density_scale,
                          const float* majorant, const int* majorant_dims, int majorant_kind, const uint32_t* seeds,
                          int draws_before, const rdvb_encoding* encoding, int n_layers, const int* dims,
                          const float* const* weights, const float* const* biases, const int* layer_flags,
                          int input_relu, void* workspace, size_t workspace_bytes, float* out, void* stream) {
    rdvb::trm::Params p;
    if (int rc = tracking_params(rays, n_rays, transform, majorant, majorant_dims, majorant_kind, seeds, draws_before,
                                 encoding, n_layers, dims, weights, biases, layer_flags, input_relu, workspace,
                                 workspace_bytes,
                                 out, p, 1))
        return rc;
    if (n_rays == 0) return RDVB_OK;
    p.scale = density_scale;
    DeviceInfo* dev = nullptr;
    if (int rc = current_device(&dev)) return rc;
    return launch_simt_march(p, n_layers, dims, weights, biases, layer_flags, workspace, dev,
                             static_cast<cudaStream_t>(stream), March::kRatioTracking);
}

int rdvb_pbvr(const float* rays, int64_t n_rays, const float* transform, const float* majorant,
              const int* majorant_dims, int majorant_kind, const float* albedo, float g, int max_bounces,
              int env_kind, const float* env_rgb, const float* env_image, const int* env_dims, int env_flags,
              const uint32_t* seeds, int draws_before, const rdvb_encoding* encoding, int n_layers, const int* dims,
              const float* const* weights, const float* const* biases, const int* layer_flags, int input_relu,
              void* workspace, size_t workspace_bytes, float* out, void* stream) {
    rdvb::trm::Params p;
    if (int rc = tracking_params(rays, n_rays, transform, majorant, majorant_dims, majorant_kind, seeds, draws_before,
                                 encoding, n_layers, dims, weights, biases, layer_flags, input_relu, workspace,
                                 workspace_bytes,
                                 out, p, 3))
        return rc;
    if (!albedo) return fail(RDVB_ERR_INVALID_ARG, "albedo must not be NULL");
    if (max_bounces < 0) return fail(RDVB_ERR_INVALID_ARG, "max_bounces must be >= 0, got %d", max_bounces);
    if (!std::isfinite(g)) return fail(RDVB_ERR_INVALID_ARG, "g must be finite");
    rdvb::pbvr::Extra e;
    memset(&e, 0, sizeof(e));
    for (int k = 0; k < 3; ++k) e.albedo[k] = albedo[k];
    e.g = g;
    e.max_bounces = max_bounces;
    if (int rc = environment_args(env_kind, env_rgb, env_image, env_dims, env_flags, n_rays, e)) return rc;
    if (n_rays == 0) return RDVB_OK;
    e.out = out;
    DeviceInfo* dev = nullptr;
    if (int rc = current_device(&dev)) return rc;
    return launch_simt_march(p, n_layers, dims, weights, biases, layer_flags, workspace, dev,
                             static_cast<cudaStream_t>(stream), March::kPbvr, &e);
}

int rdvb_pbvrt(const float* rays, int64_t n_rays, const float* transform, float density_scale, const float* majorant,
               const int* majorant_dims, int majorant_kind, const float* albedo, float g, int max_bounces,
               const float* light_direction, const float* light_intensity, int variant, int env_kind,
               const float* env_rgb, const float* env_image, const int* env_dims, int env_flags,
               const float* env_densities, int env_levels, const uint32_t* seeds, int draws_before,
               const rdvb_encoding* encoding, int n_layers, const int* dims, const float* const* weights,
               const float* const* biases, const int* layer_flags, int input_relu, void* workspace,
               size_t workspace_bytes, float* out, void* stream) {
    rdvb::trm::Params p;
    if (int rc = tracking_params(rays, n_rays, transform, majorant, majorant_dims, majorant_kind, seeds, draws_before,
                                 encoding, n_layers, dims, weights, biases, layer_flags, input_relu, workspace,
                                 workspace_bytes,
                                 out, p, 3))
        return rc;
    if (variant != RDVB_PBVRT && variant != RDVB_PBVR_NEE && variant != RDVB_PBVR_ENV)
        return fail(RDVB_ERR_INVALID_ARG, "variant must be RDVB_PBVRT, RDVB_PBVR_NEE or RDVB_PBVR_ENV, got %d",
                    variant);
    const bool env_nee = variant == RDVB_PBVR_ENV;
    if (!albedo || (!env_nee && !light_direction) || (variant == RDVB_PBVRT && !light_intensity))
        return fail(RDVB_ERR_INVALID_ARG, "albedo, light_direction (PBVRT, NEE) and light_intensity (PBVRT) must "
                                          "not be NULL");
    if (env_nee && (env_levels < 1 || env_levels > 12))
        return fail(RDVB_ERR_INVALID_ARG, "env_levels must be in [1, 12], got %d", env_levels);
    if (env_nee && n_rays > 0 && (!env_densities || !aligned(env_densities, 4)))
        return fail(RDVB_ERR_INVALID_ARG, "env_densities must be a 4-byte aligned device pointer");
    if (max_bounces < 0) return fail(RDVB_ERR_INVALID_ARG, "max_bounces must be >= 0, got %d", max_bounces);
    if (!std::isfinite(g) || !std::isfinite(density_scale))
        return fail(RDVB_ERR_INVALID_ARG, "g and density_scale must be finite");
    rdvb::pbvr::ExtraT e;
    memset(&e, 0, sizeof(e));
    for (int k = 0; k < 3; ++k) e.albedo[k] = albedo[k];
    e.g = g;
    e.density_scale = density_scale;
    e.max_bounces = max_bounces;
    e.variant = variant == RDVB_PBVRT ? 0 : (variant == RDVB_PBVR_NEE ? 1 : 2);
    if (!env_nee) {
        // normalize(light_direction) = l / length(l), length = sqrt((x x + y y) + z z)
        const float l0 = light_direction[0], l1 = light_direction[1], l2 = light_direction[2];
        const float sq = (l0 * l0 + l1 * l1) + l2 * l2;
        const float len = std::sqrt(sq);
        if (!(len > 0.0f) || !std::isfinite(len))
            return fail(RDVB_ERR_INVALID_ARG, "light_direction must be a finite nonzero vector");
        e.light[0] = l0 / len;
        e.light[1] = l1 / len;
        e.light[2] = l2 / len;
    } else {
        e.light[1] = 1.0f;  // unused: every NEE direction is sampled
        e.densities = env_densities;
        e.levels = env_levels;
    }
    for (int k = 0; k < 3; ++k) e.intensity[k] = variant == RDVB_PBVRT ? light_intensity[k] : 0.0f;
    if (variant != RDVB_PBVR_NEE) {
        if (int rc = environment_args(env_kind, env_rgb, env_image, env_dims, env_flags, n_rays, e.env)) return rc;
    }
    if (n_rays == 0) return RDVB_OK;
    e.env.out = out;
    DeviceInfo* dev = nullptr;
    if (int rc = current_device(&dev)) return rc;
    return launch_simt_march(p, n_layers, dims, weights, biases, layer_flags, workspace, dev,
                             static_cast<cudaStream_t>(stream), March::kPbvrt, &e);
}


namespace {
int camera_rays(const float* poses, int n_cameras, int width, int height, float aspect, float fov, int jitter,
                const uint32_t* seeds, float* out, void* stream) {
    if (n_cameras < 0 || width < 0 || height < 0) return fail(RDVB_ERR_INVALID_ARG, "sizes must be >= 0");
    if (jitter && !seeds) return fail(RDVB_ERR_INVALID_ARG, "seeds must not be NULL");
    if (n_cameras == 0 || width == 0 || height == 0) return RDVB_OK;
    if (!poses || !out) return fail(RDVB_ERR_INVALID_ARG, "poses and out must not be NULL");
    DeviceInfo* dev = nullptr;
    if (int rc = current_device(&dev)) return rc;
    if (!(fov > 0.0f)) fov = kDefaultFov;
    if (!(aspect > 0.0f)) aspect = static_cast<float>(width) / static_cast<float>(height);
    const long long total = static_cast<long long>(n_cameras) * width * height;
    const int threads = 256;
    const int blocks = static_cast<int>(std::max<long long>(1, std::min<long long>((total + threads - 1) / threads,
                                                                                   dev->sm_count * 16LL)));
    const uint4 sd = jitter ? make_uint4(seeds[0], seeds[1], seeds[2], seeds[3]) : make_uint4(0u, 0u, 0u, 0u);
    rdvb::ray::camera_rays_kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
        poses, n_cameras, width, height, aspect, fov, jitter ? 1 : 0, sd, out);
    return check_launch("camera_rays_kernel");
}
}  // namespace

int rdvb_camera_rays(const float* poses, int n_cameras, int width, int height, float aspect, float fov, float* out,
                     void* stream) {
    return camera_rays(poses, n_cameras, width, height, aspect, fov, 0, nullptr, out, stream);
}

int rdvb_camera_rays_jittered(const float* poses, int n_cameras, int width, int height, float aspect, float fov,
                              const uint32_t* seeds, float* out, void* stream) {
    return camera_rays(poses, n_cameras, width, height, aspect, fov, 1, seeds, out, stream);
}

}  // extern "C"

// ---------------------------------------------------- allocation-free MLP
// A variant of rdvb_mlp_forward for callers that cannot allocate device
// memory for the packed weight image: hosts that drive the library through
// the C ABI from memory they do not own (a foreign runtime's buffers, an
// embedding with no CUDA allocator of its own), or a hot loop whose caller
// forbids allocation between calls. The image lives in a file-scope static
// device array instead.
namespace {

constexpr size_t kStaticPackBytes = 256 * 1024;  // holds chains up to ~256 KB of packed weights + biases
__device__ __align__(256) uint8_t g_static_pack[kStaticPackBytes];

void* g_static_pack_ptr[kMaxDevices] = {};
std::mutex g_static_pack_mutex;

// Address of g_static_pack on the current device, looked up once per device
// (with that device current).
int static_pack_address(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(RDVB_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return fail(RDVB_ERR_UNSUPPORTED, "device index %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_static_pack_mutex);
    if (!g_static_pack_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_static_pack);
        if (e != cudaSuccess)
            return fail(RDVB_ERR_CUDA, "cudaGetSymbolAddress(static pack): %s", cudaGetErrorString(e));
        g_static_pack_ptr[dev] = p;
    }
    *out = g_static_pack_ptr[dev];
    return RDVB_OK;
}

}  // namespace

extern "C" {

int64_t rdvb_mlp_static_capacity(void) { return static_cast<int64_t>(kStaticPackBytes); }

int rdvb_mlp_forward_static(const void* x, int x_dtype, int64_t n_rows, int n_layers, const int* dims,
                            const float* const* weights, const float* const* biases, const int* layer_flags,
                            int input_relu, int tail_exact, float* y, void* stream) {
    // The same argument checks as rdvb_mlp_forward, before anything touches
    // the shared array: a rejected call leaves it as the last good call left it.
    if (int rc = check_chain(n_layers, dims, layer_flags)) return rc;
    if (x_dtype != RDVB_F32 && x_dtype != RDVB_F16 && x_dtype != RDVB_BF16)
        return fail(RDVB_ERR_INVALID_ARG, "x_dtype %d is not RDVB_F32/F16/BF16", x_dtype);
    if (n_rows < 0) return fail(RDVB_ERR_INVALID_ARG, "n_rows must be >= 0");
    if (n_rows == 0) return RDVB_OK;
    if (!x || !y) return fail(RDVB_ERR_INVALID_ARG, "x and y must not be NULL");
    if (!weights || !biases) return fail(RDVB_ERR_INVALID_ARG, "weights/biases must not be NULL");
    for (int l = 0; l < n_layers; ++l)
        if (!weights[l] || !biases[l]) return fail(RDVB_ERR_INVALID_ARG, "weights[%d]/biases[%d] is NULL", l, l);
    const int math = layer_flags[0] & 3;
    bool uniform = true;
    for (int l = 1; l < n_layers; ++l) uniform &= (layer_flags[l] & 3) == math;
    void* packed = nullptr;
    // The image is written only when the tensor-core kernel will read it:
    // every layer float16 (or every layer bfloat16), widths <= 128, aligned
    // x and y, at least one whole 32-row group and a shared-memory plan that
    // fits. Any other call never touches the array.
    const int64_t need = rdvb_mlp_packed_bytes(n_layers, dims);
    if (uniform && math != RDVB_MATH_F32 && need > 0 && n_rows >= 32) {
        if (need > static_cast<int64_t>(kStaticPackBytes))
            return fail(RDVB_ERR_UNSUPPORTED,
                        "packed weights need %lld bytes; rdvb_mlp_forward_static holds at most %lld "
                        "(use rdvb_mlp_pack + rdvb_mlp_forward with a caller buffer)",
                        (long long)need, (long long)kStaticPackBytes);
        void* addr = nullptr;
        if (int rc = static_pack_address(&addr)) return rc;
        const int path = rdvb_mlp_forward_path(x, x_dtype, n_rows, n_layers, dims, layer_flags, addr, y);
        if (path < 0) return path;
        if (path == RDVB_PATH_TENSOR_CORE) {
            if (int rc = rdvb_mlp_pack(n_layers, dims, weights, biases,
                                       math == RDVB_MATH_BF16 ? RDVB_BF16 : RDVB_F16, addr, stream))
                return rc;
            packed = addr;
        }
    }
    return rdvb_mlp_forward(x, x_dtype, n_rows, n_layers, dims, weights, biases, layer_flags, input_relu, tail_exact,
                            packed, y, stream);
}

}  // extern "C"
