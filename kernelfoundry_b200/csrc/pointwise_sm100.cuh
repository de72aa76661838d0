// RMSNorm, rotary position embedding (RoPE) and SwiGLU for B200 (sm_100a).
//
// The reference lists these three kernels as planned with no code
// (README.md:16-18), so the arithmetic follows the Llama-family convention
// used by transformers' Llama modules:
//   rmsnorm : y = rnd(rnd(x * r) * w),  r = 1 / sqrt(mean(x^2) + eps)
//             (fused residual form: s = rnd(x + res) is written back to res
//             and normalised in place of x)
//   rope    : pairs (x0, x1) -> (x0 c - x1 s, x1 c + x0 s), c/s of
//             pos * theta^(-2i/rot_dim); NeoX pairing (i, i + rot_dim/2) or
//             GPT-J pairing (2i, 2i+1); one rounding at the end
//   swiglu  : y = rnd(rnd(silu(g)) * u),  silu(g) = g / (1 + e^-g)
// where rnd() rounds to the 16-bit storage type (fp16 or bf16).  Arithmetic is
// fp32 except the RoPE angle, which is formed and reduced modulo 2*pi in fp64
// so that positions up to 2^31 keep the fp32 accuracy of sincosf.
//
// All three are HBM-streaming kernels: 16-byte vector loads and stores,
// inputs read once with the evict-first hint, grids sized from the occupancy
// of the 148 SMs.  Nothing here is GEMM-shaped, so no tensor-core path.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace kf {

// ---- 8 x 16-bit <-> 8 x fp32 -------------------------------------------------
template <bool BF16>
__device__ __forceinline__ void unpack8(const uint4 v, float (&f)[8]) {
    const unsigned w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 p;
        if constexpr (BF16) {
            __nv_bfloat162 h;
            *reinterpret_cast<unsigned*>(&h) = w[i];
            p = __bfloat1622float2(h);
        } else {
            __half2 h;
            *reinterpret_cast<unsigned*>(&h) = w[i];
            p = __half22float2(h);
        }
        f[2 * i] = p.x;
        f[2 * i + 1] = p.y;
    }
}

template <bool BF16>
__device__ __forceinline__ unsigned pack2(float a, float b) {
    unsigned u;
    if constexpr (BF16) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        u = *reinterpret_cast<unsigned*>(&h);
    } else {
        __half2 h = __floats2half2_rn(a, b);
        u = *reinterpret_cast<unsigned*>(&h);
    }
    return u;
}

template <bool BF16>
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
    return make_uint4(pack2<BF16>(f[0], f[1]), pack2<BF16>(f[2], f[3]), pack2<BF16>(f[4], f[5]),
                      pack2<BF16>(f[6], f[7]));
}

// Rounds 8 fp32 values to the storage type and back.
template <bool BF16>
__device__ __forceinline__ void round8(float (&f)[8]) {
    unpack8<BF16>(pack8<BF16>(f), f);
}

__device__ __forceinline__ uint4 ld_stream(const uint4* p) { return __ldcs(p); }
__device__ __forceinline__ void st_stream(uint4* p, uint4 v) { __stcs(p, v); }

// ---- RMSNorm -------------------------------------------------------------------
// One row of `hidden` = 8 * nvec elements is owned by a group of G threads
// (G a power of two, 1..1024); thread r of the group holds vectors
// r, r + G, ..., r + (VPT-1) G (VPT <= 4) in registers between the sum of
// squares and the scaling pass, so every input byte is read from HBM once.
// All of a row's loads (x, and the residual) are issued before its first
// store.  Blocks hold max(G, 256) / G row groups and stride over the rows.
struct RmsNormParams {
    const uint4* x;        // [rows, nvec] input
    const uint4* w;        // [nvec] weight
    uint4* out;            // [rows, nvec] output (may equal x)
    uint4* res;            // [rows, nvec] residual, updated in place (RES only)
    long long rows;
    int nvec;
    int G;                 // threads per row
    float inv_hidden;
    float eps;
};

template <bool BF16, int VPT, bool RES>
__global__ void __launch_bounds__(1024) rmsnorm_kernel(const RmsNormParams p) {
    __shared__ float red[32];
    const int G = p.G;
    const int r = threadIdx.x & (G - 1);
    const int gi = threadIdx.x / G;
    const int rpb = blockDim.x / G;                      // rows per block pass
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    for (long long base = static_cast<long long>(blockIdx.x) * rpb; base < p.rows;
         base += static_cast<long long>(gridDim.x) * rpb) {
        const long long row = base + gi;
        const bool valid = row < p.rows;
        const long long off = row * p.nvec;
        uint4 v[VPT], rv[VPT];
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const int c = r + k * G;
            const bool in = valid && c < p.nvec;
            v[k] = in ? ld_stream(p.x + off + c) : make_uint4(0u, 0u, 0u, 0u);
            if constexpr (RES) rv[k] = in ? ld_stream(p.res + off + c) : make_uint4(0u, 0u, 0u, 0u);
        }
        if constexpr (RES) {
#pragma unroll
            for (int k = 0; k < VPT; ++k) {
                const int c = r + k * G;
                float a[8], b[8];
                unpack8<BF16>(v[k], a);
                unpack8<BF16>(rv[k], b);
#pragma unroll
                for (int e = 0; e < 8; ++e) a[e] += b[e];
                v[k] = pack8<BF16>(a);                   // rnd(x + res): exact sum, one rounding
                if (valid && c < p.nvec) st_stream(p.res + off + c, v[k]);
            }
        }
        float ss = 0.f;
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            float a[8];
            unpack8<BF16>(v[k], a);
#pragma unroll
            for (int e = 0; e < 8; ++e) ss = fmaf(a[e], a[e], ss);
        }
        // Sum over the row's G threads: shuffles inside a warp, then shared
        // memory across the row's warps (G > 32 only).
        const int wspan = G < 32 ? G : 32;
        for (int o = wspan >> 1; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (G > 32) {
            if (lane == 0) red[warp] = ss;
            __syncthreads();
            const int nw = G >> 5;
            const int w0 = (warp / nw) * nw;
            ss = 0.f;
            for (int j = 0; j < nw; ++j) ss += red[w0 + j];
            __syncthreads();
        }
        const float rinv = rsqrtf(fmaf(ss, p.inv_hidden, p.eps));
        if (valid) {
#pragma unroll
            for (int k = 0; k < VPT; ++k) {
                const int c = r + k * G;
                if (c < p.nvec) {
                    float a[8], wt[8];
                    unpack8<BF16>(v[k], a);
                    unpack8<BF16>(__ldg(p.w + c), wt);
#pragma unroll
                    for (int e = 0; e < 8; ++e) a[e] *= rinv;
                    round8<BF16>(a);                     // rnd(x * r)
#pragma unroll
                    for (int e = 0; e < 8; ++e) a[e] *= wt[e];   // exact in fp32; rounded once by pack8
                    st_stream(p.out + off + c, pack8<BF16>(a));
                }
            }
        }
    }
}

// ---- RoPE ----------------------------------------------------------------------
// In place on Q and K given by element strides (head_dim contiguous), so both
// [B, H, S, D] (the attention layout) and [B, S, H, D] work.  A "unit" is what
// one thread rotates per head row: NeoX, 8 pairs = the 16-byte vector at
// dims 8u.. and its partner at rot_dim/2 + 8u..; GPT-J, 4 pairs in one 16-byte
// vector at dims 8u...  Thread (u, hg, tk) of a block owns unit u of the HB
// heads hg, hg + HG, ... (HG * HB >= H_q + H_kv) of one token per pass: it
// issues all of that token's loads first, then computes the 4 or 8 angles
// once for all those heads, then rotates and stores.  The inverse
// frequencies sit in shared memory (fp64, computed once per block).
struct RopeParams {
    uint4* q;
    uint4* k;                     // nullptr when H_kv == 0
    const int* pos;               // [B, S] positions, nullptr: position = s
    const float* inv_freq;        // [rot_dim / 2], nullptr: theta^(-2i/rot_dim)
    long long q_sb, q_sh, q_ss;   // strides in 16-byte vectors
    long long k_sb, k_sh, k_ss;
    long long n_tokens;           // B * S
    int S, H_q, H_kv;
    int rot_dim;
    int U, HG, TPB;               // units per row, head groups, tokens per block pass
    double log2_theta;
};

// a mod 2*pi into [-pi, pi]: Cody-Waite reduction with 2*pi split into a
// 53-bit head and its remainder, exact for the |a| < 2^31 that int positions
// times inverse frequencies <= 1 produce.
__device__ __forceinline__ float reduce_2pi(double a) {
    const double k = rint(a * 0.15915494309189535);        // 1 / (2 pi)
    double r = fma(-k, 6.283185307179586, a);               // 2 pi, rounded to double
    r = fma(-k, 2.4492935982947064e-16, r);                 // 2 pi - its double rounding
    return static_cast<float>(r);
}

template <bool BF16, bool NEOX, int HB>
__global__ void __launch_bounds__(256) rope_kernel(const RopeParams p) {
    constexpr int NP = NEOX ? 8 : 4;                       // pairs per unit
    __shared__ double s_f[512];                            // inverse frequencies, rot_dim / 2 <= 512
    for (int i = threadIdx.x; i < p.rot_dim / 2; i += blockDim.x)
        s_f[i] = p.inv_freq ? static_cast<double>(p.inv_freq[i]) : exp2(-(2.0 * i / p.rot_dim) * p.log2_theta);
    __syncthreads();
    const int u = threadIdx.x % p.U;
    const int rest = threadIdx.x / p.U;
    const int hg = rest % p.HG;
    const int tk = rest / p.HG;
    if (tk >= p.TPB) return;
    const double* f = s_f + NP * u;
    const int H = p.H_q + p.H_kv;
    const long long half_vec = p.rot_dim / 16;             // NeoX partner offset, in vectors
    for (long long t = static_cast<long long>(blockIdx.x) * p.TPB + tk; t < p.n_tokens;
         t += static_cast<long long>(gridDim.x) * p.TPB) {
        const long long b = t / p.S;
        const long long s = t - b * p.S;
        const int pos_i = p.pos ? __ldg(p.pos + t) : static_cast<int>(s);
        for (int h0 = hg; h0 < H; h0 += HB * p.HG) {
            uint4* rowp[HB];
            uint4 a[HB], c[HB];
#pragma unroll
            for (int m = 0; m < HB; ++m) {
                const int h = h0 + m * p.HG;
                rowp[m] = nullptr;
                if (h < H) {
                    rowp[m] = h < p.H_q ? p.q + b * p.q_sb + h * p.q_sh + s * p.q_ss
                                        : p.k + b * p.k_sb + (h - p.H_q) * p.k_sh + s * p.k_ss;
                    a[m] = rowp[m][u];
                    if constexpr (NEOX) c[m] = rowp[m][half_vec + u];
                }
            }
            float cs[NP], sn[NP];
#pragma unroll
            for (int j = 0; j < NP; ++j) sincosf(reduce_2pi(static_cast<double>(pos_i) * f[j]), &sn[j], &cs[j]);
#pragma unroll
            for (int m = 0; m < HB; ++m) {
                if (!rowp[m]) continue;
                if constexpr (NEOX) {
                    float x0[8], x1[8], y0[8], y1[8];
                    unpack8<BF16>(a[m], x0);
                    unpack8<BF16>(c[m], x1);
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        y0[e] = fmaf(x0[e], cs[e], -x1[e] * sn[e]);
                        y1[e] = fmaf(x1[e], cs[e], x0[e] * sn[e]);
                    }
                    rowp[m][u] = pack8<BF16>(y0);
                    rowp[m][half_vec + u] = pack8<BF16>(y1);
                } else {
                    float x[8], y[8];
                    unpack8<BF16>(a[m], x);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        y[2 * e] = fmaf(x[2 * e], cs[e], -x[2 * e + 1] * sn[e]);
                        y[2 * e + 1] = fmaf(x[2 * e + 1], cs[e], x[2 * e] * sn[e]);
                    }
                    rowp[m][u] = pack8<BF16>(y);
                }
            }
        }
    }
}

// ---- SwiGLU --------------------------------------------------------------------
// gate_up [rows, 2 * inter] (gate columns first, then up) -> out [rows, inter].
// Blocks stride over rows; a block's threads stride over the row's vectors,
// UNR vectors per thread per pass with all 2 * UNR loads issued first.
// silu(g) = g / (1 + 2^(-g log2 e)) with the MUFU exponential and the fast
// (reciprocal-multiply) division, ~2^-21 relative error in fp32, far below
// the 16-bit rounding that follows.  The IEEE division made the kernel
// issue-bound (5.1 TB/s against 6.0).  For g < -87.3 the denominator leaves the
// fast division's range and the result is -0 (the true |silu| < 1e-36).
struct SwigluParams {
    const uint4* gu;
    uint4* out;
    long long rows;
    int ivec;                     // inter / 8
};

template <bool BF16>
__global__ void __launch_bounds__(256) swiglu_kernel(const SwigluParams p) {
    constexpr int UNR = 4;
    for (long long row = blockIdx.x; row < p.rows; row += gridDim.x) {
        const uint4* g = p.gu + row * 2 * p.ivec;
        const uint4* up = g + p.ivec;
        uint4* o = p.out + row * p.ivec;
        for (int c0 = threadIdx.x; c0 < p.ivec; c0 += UNR * blockDim.x) {
            uint4 gv[UNR], uv[UNR];
#pragma unroll
            for (int j = 0; j < UNR; ++j) {
                const int c = c0 + j * blockDim.x;
                if (c < p.ivec) {
                    gv[j] = ld_stream(g + c);
                    uv[j] = ld_stream(up + c);
                }
            }
#pragma unroll
            for (int j = 0; j < UNR; ++j) {
                const int c = c0 + j * blockDim.x;
                if (c >= p.ivec) break;
                float x[8], y[8];
                unpack8<BF16>(gv[j], x);
                unpack8<BF16>(uv[j], y);
#pragma unroll
                for (int e = 0; e < 8; ++e) x[e] = __fdividef(x[e], 1.f + __expf(-x[e]));
                round8<BF16>(x);                           // rnd(silu(g))
#pragma unroll
                for (int e = 0; e < 8; ++e) x[e] *= y[e];  // exact in fp32; rounded once by pack8
                st_stream(o + c, pack8<BF16>(x));
            }
        }
    }
}

}  // namespace kf
