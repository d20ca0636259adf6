// Volume ray-march support kernels: the pinhole ray grid (the reference's
// Cameras node) and the ray compaction that feeds the fused-MLP kernel's ray
// mode (mlp_tc.cuh, RAY = true), which evaluates the MLP on each ray's 128
// samples and composites front to back.
#pragma once
#include "rng.cuh"
#include "mlp_tc.cuh"

namespace rdvb {
namespace ray {

// One thread per pixel of the band: rays that hit the [-1, 1]^3 box are
// appended to hit_list (one atomic per warp); pixels of missing rays get
// RGBA 0 (black background, nothing absorbed). *n_hits starts at 0.
__global__ void ray_compact_kernel(const __grid_constant__ mlp_tc::RayParams rp, int n_pix, int* __restrict__ hit_list,
                                   int* __restrict__ n_hits, float* __restrict__ rgba) {
    const int lane = threadIdx.x & 31;
    for (int base = blockIdx.x * blockDim.x; base < n_pix; base += gridDim.x * blockDim.x) {
        const int pix = base + threadIdx.x;
        bool hit = false;
        if (pix < n_pix) {
            float o[3], w[3], t0, t1;
            hit = mlp_tc::ray_setup(rp, pix, o, w, t0, t1);
            if (!hit) reinterpret_cast<float4*>(rgba)[pix] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
        const uint32_t m = __ballot_sync(0xffffffffu, hit);
        int slot0 = 0;
        if (lane == 0 && m) slot0 = atomicAdd(n_hits, __popc(m));
        slot0 = __shfl_sync(0xffffffffu, slot0, 0);
        if (hit) hit_list[slot0 + __popc(m & ((1u << lane) - 1u))] = pix;
    }
}

// Cameras (rdv/domain/rendering.py:10-42, rdv/shaders/rendering/cameras.h:1-20):
// out[cam, y, x] = (origin, unit direction) of the pixel-centre ray, 6 floats.
// poses [ncam, 9] = origin | target | up.
// Cameras grid evaluation (rdv/shaders/rendering/cameras.h:1-20). Pixel i =
// (camera, row, column) flattened. Without jitter the ray passes through the
// pixel centre; with jitter (pixel_jitter != 0) through (column + random(),
// row + random()), the two draws of pixel i's own generator (the dispatch
// seeds spawned by i; the x offset is drawn first).
__global__ void camera_rays_kernel(const float* __restrict__ poses, int ncam, int width, int height, float aspect,
                                   float fov, int jitter, uint4 seeds, float* __restrict__ out) {
    const unsigned sd[4] = {seeds.x, seeds.y, seeds.z, seeds.w};
    const long long total = static_cast<long long>(ncam) * height * width;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int x = static_cast<int>(i % width);
        const int y = static_cast<int>((i / width) % height);
        const int c = static_cast<int>(i / (static_cast<long long>(width) * height));
        const float* ps = poses + c * 9;
        const float o[3] = {ps[0], ps[1], ps[2]};
        float z[3] = {ps[3] - o[0], ps[4] - o[1], ps[5] - o[2]};
        const float zl = 1.0f / sqrtf(z[0] * z[0] + z[1] * z[1] + z[2] * z[2]);
        z[0] *= zl; z[1] *= zl; z[2] *= zl;
        const float n[3] = {ps[6], ps[7], ps[8]};
        float xa[3] = {n[1] * z[2] - n[2] * z[1], n[2] * z[0] - n[0] * z[2], n[0] * z[1] - n[1] * z[0]};
        const float xl = 1.0f / sqrtf(xa[0] * xa[0] + xa[1] * xa[1] + xa[2] * xa[2]);
        xa[0] *= xl; xa[1] *= xl; xa[2] *= xl;
        const float ya[3] = {z[1] * xa[2] - z[2] * xa[1], z[2] * xa[0] - z[0] * xa[2], z[0] * xa[1] - z[1] * xa[0]};
        float jx = 0.5f, jy = 0.5f;
        if (jitter) {
            Rng r = rng_spawn(sd, static_cast<unsigned>(i));
            jx = rng_uniform(r);
            jy = rng_uniform(r);
        }
        const float px = (static_cast<float>(x) + jx) / static_cast<float>(width) * 2.0f - 1.0f;
        const float py = (static_cast<float>(y) + jy) / static_cast<float>(height) * 2.0f - 1.0f;
        const float sx = px * aspect, sy = py, sz = 1.0f / tanf(fov * 0.5f);
        float w[3];
#pragma unroll
        for (int k = 0; k < 3; ++k) w[k] = xa[k] * sx + ya[k] * sy + z[k] * sz;
        const float wl = 1.0f / sqrtf(w[0] * w[0] + w[1] * w[1] + w[2] * w[2]);
        float* dst = out + i * 6;
        dst[0] = o[0]; dst[1] = o[1]; dst[2] = o[2];
        dst[3] = w[0] * wl; dst[4] = w[1] * wl; dst[5] = w[2] * wl;
    }
}

}  // namespace ray
}  // namespace rdvb
