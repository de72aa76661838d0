/*
 * kf_synth.h -- C ABI of the counter-based generator of the seeded N(0,1)
 * fp16 inputs that the benchmarks and tests feed the attention kernels.
 *
 * No counterpart in the reference: its harnesses fill inputs with mt19937
 * uniform[-1,1] (tests/test_utils.h:27-31) and its NumPy model with NumPy's
 * generator, so the same "seeded synthetic input" exists only on one side.
 * Here element i of the stream with seed s is a pure function of (s, i),
 * defined identically on the device (this entry point) and in NumPy
 * (oracle/synth_oracle.py), so a 1 GB decode cache is generated in place on
 * the GPU and any slice of it is regenerated exactly on the host.
 *
 * Definition (all integer arithmetic mod 2^64, all floating point binary64):
 *   w(c)   = splitmix64 output c of seed s, i.e. mix(s + (c + 1) * 0x9E3779B97F4A7C15)
 *            with mix(z) = z ^= z >> 30, z *= 0xBF58476D1CE4E5B9,
 *                          z ^= z >> 27, z *= 0x94D049BB133111EB, z ^ (z >> 31)
 *            (Steele, Lea and Flood, "Fast splittable pseudorandom number
 *            generators", OOPSLA 2014; Vigna's splitmix64.c);
 *   pair k: u1 = ((w(2k) >> 11) + 1) * 2^-53 in (0, 1],  u2 = (w(2k+1) >> 11) * 2^-53,
 *           r = sqrt(-2 ln u1), t = 6.283185307179586 * u2,
 *           element 2k = r cos t, element 2k+1 = r sin t   (Box and Muller, 1958);
 *   each element rounded once to fp16 (round to nearest even).
 * log, sqrt, cos and sin are the platform's binary64 functions; they agree to
 * an ulp or two, far below the fp16 rounding, so the two sides produce the
 * same bits except for a value within a few binary64 ulps of an fp16 rounding
 * boundary.
 */
#ifndef KF_SYNTH_H_
#define KF_SYNTH_H_

#include <stdint.h>

#include "kf_attn.h"

#ifdef __cplusplus
extern "C" {
#endif

/* dst[j] = element (offset + j) of the stream with `seed`, for 0 <= j < n.
 * dst: device pointer, 2-byte aligned (KF_ERR_MISALIGNED otherwise).
 * Asynchronous on `stream`; allocates nothing.  n = 0 is a no-op; n < 0,
 * offset < 0, offset + n > 2^62 or a null dst with n > 0 is
 * KF_ERR_INVALID_ARG.  All checks run before any CUDA call. */
int kf_fill_normal_f16(uint16_t* dst, long long n, unsigned long long seed, long long offset, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KF_SYNTH_H_ */
