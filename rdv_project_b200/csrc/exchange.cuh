// Exchange kernels of a sharded evaluation (B200 extension: the reference
// runs Map.__call__, rdv/maths/__init__.py:1451-1487, on one device).
//
// multicast_copy_kernel: this GPU's rows -> every GPU of an NVLink multicast
// group. src is this GPU's copy of the rows; dst the multicast address of
// the same rows in the group's symmetric buffer (its NVLS mapping). Each
// 16-byte chunk is read once here and written once with multimem.st: the
// switch delivers it to every GPU bound to the buffer, this one included,
// so a GPU's rows leave it once whatever the group size. A grid-stride loop
// over the chunks; no waits. Each thread's stores are performed at system
// scope (fence.sc.sys) before it exits; the caller then orders the step with
// a cross-GPU barrier on the same stream.
#pragma once
#include <cstdint>

namespace rdvb {
namespace exchange {

__global__ void multicast_copy_kernel(const uint4* __restrict__ src, uint64_t mc_dst, long long n16) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n16;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const uint4 v = __ldg(src + i);
        asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc_dst + i * 16ull),
                     "f"(__uint_as_float(v.x)), "f"(__uint_as_float(v.y)), "f"(__uint_as_float(v.z)),
                     "f"(__uint_as_float(v.w))
                     : "memory");
    }
    __threadfence_system();
}

}  // namespace exchange
}  // namespace rdvb
