// The reference's per-invocation random generator
// (rdv/shaders/libraries/random_library.h:7-49): three Tausworthe
// components and an LCG, XOR-combined; random() keeps the low 23 bits as the
// mantissa of a float in [1, 2) and subtracts 1. An invocation starts from
// the dispatch's 4 seeds spawned by its index (random_library.h:256-268:
// random_spawn(seeds, gl_GlobalInvocationID.x) for the 1-D dispatches of Map
// and grid evaluation), so every ray or pixel draws its own sequence,
// independent of scheduling.
#pragma once
#include <cstdint>

namespace rdvb {

struct Rng {
    unsigned x, y, z, w;
};

__device__ __forceinline__ unsigned taus_step(unsigned z, int s1, int s2, int s3, unsigned m) {
    const unsigned b = ((z << s1) ^ z) >> s2;
    return ((z & m) << s3) ^ b;
}

__device__ __forceinline__ void rng_step(Rng& r) {
    r.x = taus_step(r.x, 13, 19, 12, 4294967294u);
    r.y = taus_step(r.y, 2, 25, 4, 4294967288u);
    r.z = taus_step(r.z, 3, 11, 17, 4294967280u);
    r.w = 1664525u * r.w + 1013904223u;
}

__device__ __forceinline__ float rng_uniform(Rng& r) {
    rng_step(r);
    const unsigned v = r.x ^ r.y ^ r.z ^ r.w;
    return __fsub_rn(__uint_as_float((v & 0x007FFFFFu) | 0x3F800000u), 1.0f);
}

// random_spawn(seeds, index): the index's int arithmetic wraps, as unsigned.
__device__ __forceinline__ Rng rng_spawn(const unsigned (&s)[4], unsigned index) {
    Rng r;
    r.x = s[0] ^ (index ^ 17u);
    r.y = s[1] ^ (index * 123111171u);
    r.z = s[2] ^ (index + 11u);
    r.w = s[3] ^ (index ^ (s[0] + 13u * s[1]));
    rng_step(r);
    return r;
}

}  // namespace rdvb
