// Cross-GPU exchange and merge of long-context decode partials over NVLink
// peer memory (one process per GPU, windows mapped with CUDA IPC).
//
// The KV cache of one sequence is split by ranges over `world` GPUs; each
// rank's split-KV decode writes its softmax partials (O_u, m, l) into the
// staging part of its own window.  One kernel then does the collective and
// the merge, replacing an NCCL all-gather plus a combine launch:
//   1. CTA c sends rows [r0, r1) of the staged partials to slot (parity, rank)
//      of every window (peers over NVLink, its own locally) as 8-byte words
//      {value, sequence number}: one single-copy-atomic store carries both, so
//      no fence or separate flag is needed (the low-latency protocol of
//      NCCL's LL transport, restated);
//   2. reads the same rows of every rank's slot in its own window, polling
//      each word until it carries this call's sequence number (bounded);
//   3. merges the world parts of those rows by log-sum-exp into O.
// Sequence numbers live in device memory (a per-chunk call counter in each
// window), so the kernel can be captured in a CUDA graph and replayed.  Slots
// are double-buffered by the sequence number's parity: a peer can run at most
// one call ahead (its next-but-one call needs this rank's words of the next
// call), so the slot a merge reads is never overwritten under it.  The grid is
// at most one CTA per SM, so every CTA a peer waits for is resident; a word
// that does not arrive within the configured time limit raises
// KF_DEVERR_TIMEOUT_PEER and leaves its output element unwritten.
#pragma once

#include <stdint.h>

#include "kf_ptx.cuh"

namespace kf {

constexpr int kMaxPeers = 8;

// Window layout, in 4-byte units from the base (part_stride ps a multiple of 4):
//   [0, ps)                                  staging: this rank's partials
//                                            (O_u [rows][D], then m [rows], then l [rows])
//   ps + 2 * ps * (parity * world + src)     slot[parity][src]: ps 8-byte words {value, seq}
//   ps * (1 + 4 * world)                     unit_calls[ps / 16]: call counters of the fused
//                                            decode exchange, one per (b, h_kv, row group)
//                                            (units <= rows <= ps / 18)
//   ps * (1 + 4 * world) + ps / 16           calls[n_chunks]: call counters of the
//                                            exchange-and-merge kernel, one per CTA
__host__ __device__ constexpr long long peer_slot_off(long long ps, int world, int parity, int src) {
    return ps + 2 * ps * (static_cast<long long>(parity) * world + src);
}
__host__ __device__ constexpr long long peer_unit_calls_off(long long ps, int world) {
    return ps * (1 + 4ll * world);
}
__host__ __device__ constexpr long long peer_calls_off(long long ps, int world) {
    return peer_unit_calls_off(ps, world) + ps / 16;
}
__host__ __device__ constexpr long long peer_window_words(long long ps, int world, int n_chunks) {
    return peer_calls_off(ps, world) + n_chunks;
}

struct ExchangeParams {
    float* win[kMaxPeers];        // window of each rank as mapped in this process (win[rank]: own)
    float* own;                   // win[rank] (kept apart: no run-time index into the parameters)
    int world, rank;
    long long part_stride;        // words per part
    long long rows;               // B * H_q * S_q
    int D;
    int n_chunks;                 // CTAs; CTA c owns rows [c * rows_per, ...)
    float* O;
    float* Mi;                    // nullable
    float* Li;                    // nullable
    unsigned long long timeout_ns;
};

__device__ __forceinline__ void st_ll(unsigned long long* ptr, float v, unsigned seq) {
    const unsigned long long w = (static_cast<unsigned long long>(seq) << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(ptr), "l"(w) : "memory");
}

__device__ __forceinline__ unsigned long long ld_word(const unsigned long long* ptr) {
    unsigned long long w;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(ptr) : "memory");
    return w;
}

// W = world size.  Each CTA sends and merges a contiguous range of rows; a
// thread merges output elements one at a time, issuing the 3*W word loads of
// an element together and re-polling only the words that have not arrived.
template <int W>
__global__ void __launch_bounds__(256) exchange_combine_kernel(const ExchangeParams p) {
    __shared__ unsigned s_seq;
    // Launched with programmatic stream serialization: the partial this kernel sends is the
    // previous launch's output, so nothing global is touched before that launch completes.
    grid_dep_wait();
    grid_dep_launch_dependents();
    const int c = blockIdx.x;
    const long long rows_per = (p.rows + p.n_chunks - 1) / p.n_chunks;
    const long long r0 = c * rows_per;
    const long long r1 = r0 + rows_per < p.rows ? r0 + rows_per : p.rows;
    const long long ps = p.part_stride;
    const float* own = p.own;
    unsigned* calls = reinterpret_cast<unsigned*>(p.own + peer_calls_off(ps, W));
    if (threadIdx.x == 0) s_seq = calls[c] + 1u;
    __syncthreads();
    const unsigned seq = s_seq;
    const int par = static_cast<int>(seq & 1u);
    const long long mo = p.rows * p.D;          // m after O_u, l after m
    if (r0 >= r1) {
        if (threadIdx.x == 0) calls[c] = seq;
        return;
    }

    // 1. send rows [r0, r1): O_u elements, then m and l, to every window
    const long long n_o = (r1 - r0) * p.D;
    const long long n_ml = r1 - r0;
    for (long long i = threadIdx.x; i < n_o + 2 * n_ml; i += blockDim.x) {
        const long long e = i < n_o ? r0 * p.D + i
                          : (i < n_o + n_ml ? mo + r0 + (i - n_o) : mo + p.rows + r0 + (i - n_o - n_ml));
        const float v = __ldcg(own + e);
#pragma unroll
        for (int dst = 0; dst < W; ++dst)
            st_ll(reinterpret_cast<unsigned long long*>(p.win[dst] + peer_slot_off(ps, W, par, p.rank)) + e, v, seq);
    }

    // 2 + 3. gather every rank's words of these rows from the own window and merge:
    // M = max_g m_g, O = sum_g e^(m_g - M) O_g / sum_g e^(m_g - M) l_g
    constexpr float LOG2E = 1.4426950408889634f;
    const uint64_t t0 = global_timer_ns();
    bool ok = true;
    const unsigned long long* slots =
        reinterpret_cast<const unsigned long long*>(own + peer_slot_off(ps, W, par, 0));
    for (long long it = threadIdx.x; it < n_o && ok; it += blockDim.x) {
        const long long row = r0 + it / p.D;
        const int dcol = static_cast<int>(it % p.D);
        const long long off[3] = {mo + row, mo + p.rows + row, row * p.D + dcol};
        unsigned long long w[W][3];
#pragma unroll
        for (int g = 0; g < W; ++g)
#pragma unroll
            for (int k = 0; k < 3; ++k) w[g][k] = ld_word(slots + g * ps + off[k]);
        uint32_t spins = 0;
        while (true) {
            bool all = true;
#pragma unroll
            for (int g = 0; g < W; ++g)
#pragma unroll
                for (int k = 0; k < 3; ++k)
                    if (static_cast<unsigned>(w[g][k] >> 32) != seq) {
                        all = false;
                        w[g][k] = ld_word(slots + g * ps + off[k]);
                    }
            if (all) break;
            if ((++spins & 15u) == 0u && global_timer_ns() - t0 > p.timeout_ns) { ok = false; break; }
        }
        if (!ok) break;
        float M = -CUDART_INF_F;
#pragma unroll
        for (int g = 0; g < W; ++g) M = fmaxf(M, __uint_as_float(static_cast<unsigned>(w[g][0])));
        const float Mu = (M == -CUDART_INF_F) ? 0.f : M;
        float L = 0.f, acc = 0.f;
#pragma unroll
        for (int g = 0; g < W; ++g) {
            const float wt = ex2_approx((__uint_as_float(static_cast<unsigned>(w[g][0])) - Mu) * LOG2E);
            L += wt * __uint_as_float(static_cast<unsigned>(w[g][1]));
            acc += wt * __uint_as_float(static_cast<unsigned>(w[g][2]));
        }
        p.O[row * p.D + dcol] = acc / L;
        if (dcol == 0) {
            if (p.Mi) p.Mi[row] = M;
            if (p.Li) p.Li[row] = L;
        }
    }
    if (!ok) atomicOr(&g_kf_dev_error, KF_DEVERR_TIMEOUT_PEER);
    __syncthreads();
    if (threadIdx.x == 0) calls[c] = seq;
}

}  // namespace kf
