/*
 * kf_pointwise.h -- C ABI of the B200 (sm_100a) RMSNorm, RoPE and SwiGLU
 * kernels that sit either side of the attention forward in a decoder layer.
 *
 * The reference lists these three kernels as planned and ships no code for
 * them (README.md:16-18), so there is no reference launcher to replace; the
 * entry points follow the conventions of kf_attn.h instead: device pointers,
 * plain C types, asynchronous on `stream` (a cudaStream_t, NULL = legacy
 * default stream), no allocation, KF_OK or a KF_ERR_* code (kf_attn.h) as
 * the result, argument checks before any CUDA call.
 *
 * Storage is 16-bit (fp16 unless KF_PW_BF16 is set), arithmetic fp32, and
 * the rounding points are those of the Llama-family modules in transformers:
 *   RMSNorm  y = rnd(rnd(x / sqrt(mean(x^2) + eps)) * w)
 *   SwiGLU   y = rnd(rnd(silu(g)) * u)
 * RoPE rounds once, after the rotation (transformers rounds cos/sin to the
 * storage type first; this is at least as accurate).
 * Every pointer must be 16-byte aligned and every row length a multiple of 8
 * elements (16-byte vectors); KF_ERR_MISALIGNED / KF_ERR_INVALID_ARG otherwise.
 */
#ifndef KF_POINTWISE_H_
#define KF_POINTWISE_H_

#include <stddef.h>

#include "kf_attn.h"

#ifdef __cplusplus
extern "C" {
#endif

#define KF_PW_BF16 1u       /* tensors are bf16 (default fp16) */
#define KF_ROPE_GPTJ 2u     /* kf_rope: interleaved pairs (2i, 2i+1); default NeoX (i, i + rot_dim/2) */

/* RMSNorm over the last dimension of x [rows, hidden]:
 *   out = rnd(rnd(x * rsqrt(mean(x^2) + eps)) * weight)
 * residual != NULL selects the fused residual form: s = rnd(x + residual) is
 * written to `residual` and normalised in place of x (out and residual then
 * hold the next layer's norm input and residual stream).
 * out may equal x; residual must overlap neither.  hidden: 8..32768, a
 * multiple of 8.  rows == 0 is a no-op. */
int kf_rmsnorm(const void* x, const void* weight, void* out, void* residual, long long rows, int hidden,
               float eps, unsigned flags, void* stream);

/* Rotary position embedding, in place on q [B, H_q, S, D] and k [B, H_kv, S, D]
 * addressed by element strides (the head dimension is contiguous), so
 * [B, S, H, D] storage works too.  The first rot_dim dims of each head row
 * rotate; the rest pass through.  Pair i turns by pos * inv_freq[i] with
 * pos = positions[b * S + s] (positions NULL: pos = s) and
 * inv_freq[i] = theta^(-2i / rot_dim) (inv_freq NULL) or the caller's table
 * of rot_dim / 2 floats (scaled variants).  NeoX pairs (i, i + rot_dim/2),
 * rot_dim a multiple of 16; KF_ROPE_GPTJ pairs (2i, 2i+1), rot_dim a multiple
 * of 8.  D: a multiple of 8, at most 1024.  Strides: multiples of 8, >= 0.
 * k may be NULL when H_kv == 0.  B * S == 0 is a no-op. */
int kf_rope(void* q, void* k, const int* positions, const float* inv_freq, int B, int S, int H_q, int H_kv,
            int D, int rot_dim, float theta, long long q_stride_b, long long q_stride_h, long long q_stride_s,
            long long k_stride_b, long long k_stride_h, long long k_stride_s, unsigned flags, void* stream);

/* SwiGLU on the fused gate/up projection output gate_up [rows, 2 * inter]
 * (gate columns first): out[r, j] = rnd(rnd(silu(g)) * u) with
 * g = gate_up[r, j], u = gate_up[r, inter + j].  inter: a multiple of 8.
 * out [rows, inter] must not overlap gate_up.  rows == 0 is a no-op. */
int kf_swiglu(const void* gate_up, void* out, long long rows, int inter, unsigned flags, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KF_POINTWISE_H_ */
