// synth_sm100.cuh -- counter-based N(0,1) fp16 fill (include/kf_synth.h).
//
// Element i of seed s is a pure function of (s, i): splitmix64 outputs 2k and
// 2k+1 give the two uniforms of Box-Muller pair k = i / 2, evaluated in
// binary64 and rounded once to fp16.  One thread per pair, grid-stride; the
// same definition is restated in NumPy in oracle/synth_oracle.py.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace kf {

// Output c of splitmix64 seeded with s (the state advances by the golden-ratio
// increment before each mix; Steele, Lea and Flood, OOPSLA 2014).
__device__ __forceinline__ uint64_t splitmix64_at(uint64_t s, uint64_t c) {
    uint64_t z = s + (c + 1) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__global__ void __launch_bounds__(256) fill_normal_f16_kernel(__half* dst, long long n, uint64_t seed,
                                                              long long offset) {
    const long long first = offset >> 1;               // pair holding element `offset`
    const long long end = (offset + n + 1) >> 1;       // one past the pair holding the last element
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long k = first + static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; k < end;
         k += stride) {
        const uint64_t w0 = splitmix64_at(seed, 2ull * static_cast<uint64_t>(k));
        const uint64_t w1 = splitmix64_at(seed, 2ull * static_cast<uint64_t>(k) + 1ull);
        const double u1 = static_cast<double>((w0 >> 11) + 1ull) * 0x1.0p-53;    // (0, 1]
        const double u2 = static_cast<double>(w1 >> 11) * 0x1.0p-53;            // [0, 1)
        const double r = sqrt(-2.0 * log(u1));
        const double t = 6.283185307179586 * u2;
        const double z0 = __dmul_rn(r, cos(t));
        const double z1 = __dmul_rn(r, sin(t));
        const long long e = 2 * k - offset;            // dst index of element 2k
        if (e >= 0) dst[e] = __double2half(z0);
        if (e + 1 < n) dst[e + 1] = __double2half(z1);
    }
}

}  // namespace kf
