// decode_sm100.cuh -- short-query (decode) attention forward, split-KV.
//
// Replaces the reference's flash_attn_kernel<D> launched with q_len = 1
// (tests/bench_flash_attn.cu:39-54, :153-159).  The reference gives each
// (b, h_q) one CTA that uses 1 of its 64 query rows and streams the head's
// whole KV serially, re-reading each KV head H_q/H_kv times.  Here:
//   * rows: the G = H_q/H_kv query heads sharing one KV head (times the S_q
//     query positions, S_q small) are packed as the M rows of the MMA, so
//     every K/V byte is read from HBM once per (b, h_kv);
//   * split-KV: the KV sequence of each (b, h_kv) is cut into n_split chunks,
//     one CTA each, sized by the host to fill all SMs;
//   * a producer warp streams K and V tiles (64 rows) into a shared-memory
//     ring with TMA (3-D tensor maps, swizzled boxes, zero fill past S_kv);
//     four consumer warps each take 16 rows of every tile: S = Q K^T and
//     O += P V with mma.sync m16n8k16 (the contraction is tiny; the kernel is
//     HBM-bound) and an online softmax in registers;
//   * the CTA merges its warps' (m, l, O) in shared memory, writes one
//     partial per split, and the last CTA of each (b, h_kv) to finish
//     (atomic ticket) merges the splits by log-sum-exp and writes O (and
//     Mi/Li) -- one launch, no second combine kernel.  The ticket counter is
//     reset by that CTA, so the workspace stays zeroed between calls.
// Softmax state uses the reference's convention (kernels/flash_attn.cu:
// 261-294, 575-578): m = max of scaled scores, l = sum exp(s - m), O
// un-normalised until the end.
#pragma once

#include <math_constants.h>

#include "kf_ptx.cuh"
#include "peer_sm100.cuh"

namespace kf {

// DEEP: for launches whose CTAs all fit on the SMs at once (one CTA per SM): a ring
// of twice the bytes (about 192 KB) and two groups of four consumer warps that take
// alternate stages.  A CTA's stream is bound by its consumers' warp-MMA work per stage
// (about 0.5 us per 32 KB stage with one group), so two groups double its rate.
template <int D, int MT, bool DEEP = false>
struct DecodeCfg {
    static constexpr int TK = 64;                        // KV rows per stage
    static constexpr int NW = 4;                         // consumer warps per group, 16 rows each
    static constexpr int SWB = (D >= 64) ? 128 : 2 * D;
    static constexpr int SWE = SWB / 2;
    static constexpr int NSPAN = D / SWE;
    static constexpr int TILE_BYTES = TK * D * 2;        // one K or V tile
    static constexpr int STAGE_BYTES = 2 * TILE_BYTES;
    static constexpr int NSTAGE_RAW = (DEEP ? 196608 : 98304) / STAGE_BYTES;
    static constexpr int NSTAGE = NSTAGE_RAW < 2 ? 2 : (NSTAGE_RAW > 8 ? 8 : NSTAGE_RAW);
    // Consumer groups.  Group g takes stages g, g + NG, ...; the ring depth is a
    // multiple of NG so that the stage a group waits for reuses a slot whose previous
    // stage that same group consumed (its barrier is then at most one phase behind).
    static constexpr int NG = (DEEP && NSTAGE % 2 == 0) ? 2 : 1;
    static constexpr int NCW = NW * NG;                  // consumer warps
    static constexpr int QROWS = MT * 16;
    static constexpr int QPITCH = D + 8;                 // halfs; +16 B breaks bank conflicts
    static constexpr int Q_BYTES = (QROWS * QPITCH * 2 + 15) / 16 * 16;
    static constexpr int MAX_SPLIT = 256;
    static constexpr int RED_BYTES = NW * QROWS * (D + 2) * 4;
    // split merge: weights [MAX_SPLIT][QROWS] + M, L, and two bulk-copy buffers of >= 1 split each
    static constexpr int CMB_BYTES = (MAX_SPLIT * QROWS + 2 * QROWS) * 4 + 2 * QROWS * D * 4;
    static constexpr int STAGES_BYTES = NSTAGE * STAGE_BYTES;
    // Group merge: group 1 hands its per-lane (m, l, O) fragments to group 0.
    static constexpr int GX_BYTES = NG > 1 ? NW * 32 * (MT * D / 2 + 4 * MT) * 4 : 0;
    static constexpr int RED0 = RED_BYTES > GX_BYTES ? RED_BYTES : GX_BYTES;
    static constexpr int BIG0 = STAGES_BYTES > RED0 ? STAGES_BYTES : RED0;
    static constexpr int BIG = BIG0 > CMB_BYTES ? BIG0 : CMB_BYTES;
    static constexpr int SMEM_BYTES = 1024 + BIG + Q_BYTES + 256;   // + barriers/flags
    // Cluster merge (CL kernels): the CTA's partial (O_u [QROWS][D], then (m, l) [QROWS])
    // at the end of the big region, above the CTA reduction's scratch.
    static constexpr int RED_FLOATS = NW * QROWS * (D + 3) + 2 * QROWS;
    static constexpr int CL_BYTES = QROWS * D * 4 + QROWS * 8;
    static constexpr int CL_OFF = BIG - CL_BYTES;
    static constexpr int MAX_CLUSTER = 16;
    static constexpr int THREADS = 32 * (NCW + 1);
    static_assert(NW * 16 == TK, "each consumer warp owns 16 rows of a stage");
    static_assert(NSTAGE % NG == 0, "ring depth a multiple of the consumer groups");
    static_assert(SMEM_BYTES <= 232448, "shared memory over budget");
};

struct DecodeParams {
    const uint16_t* Q;
    void* O;               // [rows][D] of out_type (fp32 when unnormalized)
    float* Mi;             // nullable
    float* Li;             // nullable
    float* part_O;         // [rows][n_split][D]   (n_split > 1)
    float* part_ml;        // [rows][n_split][2]
    unsigned* counters;    // [B*H_kv*n_rg], zero between calls
    int H_q, H_kv, S_q, S_kv, G, R, n_rg, n_split, chunk;
    float scale_log2, scale;
    int unnormalized;
    int out_type;          // KF_OUT_F32 / KF_OUT_F16 / KF_OUT_BF16
    int kv_box;            // rows per K/V TMA box: min(TK, S_kv)
    unsigned long long timeout_ns;
    // Paged KV (PAGED kernels): K/V pools [n_blocks][H_kv][block_size][D], logical
    // block j of sequence b at pool block block_table[b * max_blocks + j], and
    // seq_lens[b] keys in sequence b (clamped to [0, max_blocks * block_size]).
    const int* block_table;
    const int* seq_lens;
    int max_blocks, block_size;
    // Fused cross-GPU exchange (kernels with XW > 0, XW = world size; see xch_unit):
    // windows of every rank as mapped here (xown = the own one), part stride, rows of
    // a part (B * H_q * S_q), this rank, and the own window's per-unit call counters.
    float* xwin[kMaxPeers];
    float* xown;
    unsigned* xcalls;
    long long xps, xrows;
    int xrank;
};

// Cross-GPU exchange of one unit's softmax state, fused into the decode kernel of
// long-context decode with the KV cache split by ranges over XW GPUs.  The CTA that
// holds the unit's merged partial over this rank's keys (rows [row_base, row_base +
// nrows): O_u un-normalised per item of `acc`, raw-score max sM and sum sL per row)
// writes it into slot (parity, rank) of every rank's window as 8-byte {value, sequence
// number} words (one single-copy-atomic store each, the low-latency protocol of the
// exchange-and-merge kernel), then polls the same rows of every rank's slot in its own
// window (bounded) and merges the XW parts by log-sum-exp into O, Mi, Li.  The sequence
// number is the unit's call counter in the own window, so the launch can be replayed
// from a CUDA graph.  Called by every thread of the CTA.  The launch is a single wave
// (the deep-ring plan), so every CTA a peer waits for is resident.
template <int XW, int D, int KMAX, int THREADS>
__device__ __forceinline__ void xch_unit(const DecodeParams& p, size_t cidx, int nrows, size_t row_base,
                                         const float4 (&acc)[KMAX], const float* sM, const float* sL,
                                         volatile unsigned* s_seq, float* scratch) {
    const int tid = threadIdx.x;
    if (tid == 0) *s_seq = p.xcalls[cidx] + 1u;
    __syncthreads();
    const unsigned seq = *s_seq;
    const int par = static_cast<int>(seq & 1u);
    const long long ps = p.xps, rows = p.xrows;
    const int items = nrows * (D / 4);
    // 1. send
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
        const int it = tid + k * THREADS;
        if (it < items) {
            const long long e = static_cast<long long>(row_base + it / (D / 4)) * D + (it % (D / 4)) * 4;
#pragma unroll
            for (int dst = 0; dst < XW; ++dst) {
                unsigned long long* w =
                    reinterpret_cast<unsigned long long*>(p.xwin[dst] + peer_slot_off(ps, XW, par, p.xrank)) + e;
                st_ll(w, acc[k].x, seq);
                st_ll(w + 1, acc[k].y, seq);
                st_ll(w + 2, acc[k].z, seq);
                st_ll(w + 3, acc[k].w, seq);
            }
        }
    }
    if (tid < nrows) {
        const long long gr = static_cast<long long>(row_base) + tid;
        const float m_nat = sM[tid] * p.scale;          // natural-log units of the scaled scores
#pragma unroll
        for (int dst = 0; dst < XW; ++dst) {
            unsigned long long* w = reinterpret_cast<unsigned long long*>(p.xwin[dst] + peer_slot_off(ps, XW, par, p.xrank));
            st_ll(w + rows * D + gr, m_nat, seq);
            st_ll(w + rows * D + rows + gr, sL[tid], seq);
        }
    }
    // 2. every rank's (m, l) of these rows from the own window (one poll round for a
    // thread), the merge weights w_g = e^(m_g - M) and L = sum_g w_g l_g into scratch.
    constexpr float LOG2E = 1.4426950408889634f;
    const unsigned long long* slots =
        reinterpret_cast<const unsigned long long*>(p.xown + peer_slot_off(ps, XW, par, 0));
    float* x_w = scratch;                     // [XW][nrows] weights, then [nrows] L and M
    float* x_L = scratch + XW * nrows;
    float* x_M = x_L + nrows;
    const uint64_t t0 = global_timer_ns();
    bool ok = true;
    auto poll = [&](unsigned long long& w, const unsigned long long* addr) {
        uint32_t spins = 0;
        while (static_cast<unsigned>(w >> 32) != seq) {
            if ((++spins & 15u) == 0u && global_timer_ns() - t0 > p.timeout_ns) { ok = false; return; }
            w = ld_word(addr);
        }
    };
    __syncthreads();                          // sM / sL read by the send above
    if (tid < nrows) {
        const long long gr = static_cast<long long>(row_base) + tid;
        unsigned long long wm[XW], wl[XW];
#pragma unroll
        for (int g = 0; g < XW; ++g) {
            wm[g] = ld_word(slots + g * ps + rows * D + gr);
            wl[g] = ld_word(slots + g * ps + rows * D + rows + gr);
        }
#pragma unroll
        for (int g = 0; g < XW; ++g) {
            poll(wm[g], slots + g * ps + rows * D + gr);
            poll(wl[g], slots + g * ps + rows * D + rows + gr);
        }
        float M = -CUDART_INF_F;
#pragma unroll
        for (int g = 0; g < XW; ++g) M = fmaxf(M, __uint_as_float(static_cast<unsigned>(wm[g])));
        const float Mu = (M == -CUDART_INF_F) ? 0.f : M;
        float L = 0.f;
#pragma unroll
        for (int g = 0; g < XW; ++g) {
            const float wt = ex2_approx((__uint_as_float(static_cast<unsigned>(wm[g])) - Mu) * LOG2E);
            x_w[g * nrows + tid] = wt;
            L += wt * __uint_as_float(static_cast<unsigned>(wl[g]));
        }
        x_L[tid] = L;
        x_M[tid] = M;
        if (p.Mi) p.Mi[gr] = M;
        if (p.Li) p.Li[gr] = L;
    }
    ok = __syncthreads_and(ok) != 0;
    // 3. O = sum_g w_g O_g / L: a thread issues the 4 * XW words of its item together.
#pragma unroll 1
    for (int k = 0; k < KMAX && ok; ++k) {
        const int it = tid + k * THREADS;
        if (it >= items) continue;
        const int r = it / (D / 4);
        const long long e = static_cast<long long>(row_base + r) * D + (it % (D / 4)) * 4;
        unsigned long long w[XW][4];
#pragma unroll
        for (int g = 0; g < XW; ++g)
#pragma unroll
            for (int j = 0; j < 4; ++j) w[g][j] = ld_word(slots + g * ps + e + j);
#pragma unroll
        for (int g = 0; g < XW; ++g)
#pragma unroll
            for (int j = 0; j < 4; ++j) poll(w[g][j], slots + g * ps + e + j);
        if (!ok) break;
        float a[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int g = 0; g < XW; ++g) {
            const float wt = x_w[g * nrows + r];
#pragma unroll
            for (int j = 0; j < 4; ++j) a[j] += wt * __uint_as_float(static_cast<unsigned>(w[g][j]));
        }
        const float inv = x_L[r] > 0.f ? 1.0f / x_L[r] : 0.f;
        store_out4(p.O, e, make_float4(a[0] * inv, a[1] * inv, a[2] * inv, a[3] * inv), p.out_type);
    }
    if (!ok) atomicOr(&g_kf_dev_error, KF_DEVERR_TIMEOUT_PEER);
    __syncthreads();
    if (tid == 0) p.xcalls[cidx] = seq;
}

// PAGED: K/V come from block pools through a per-sequence block table (the maps
// are 3-D over (D, block_size, n_blocks * H_kv)); sequences have their own lengths.
// SPLIT = false: a launch with n_split == 1 (no partials, no merge), compiled
// without the split-merge code so that code does not shape the streaming loop.
// XW > 0: the unit's result is exchanged with XW - 1 peer GPUs and merged (xch_unit)
// instead of written.
// CL: the n_split CTAs of a unit form one thread-block cluster (grid x = cluster x =
// n_split): each keeps its partial in its own shared memory and, after a cluster
// barrier, merges 1/n_split of the unit's output from all the partials through
// distributed shared memory (no workspace, no ticket, no global round trip).
template <int D, int MT, bool PAGED = false, bool SPLIT = true, bool DEEP = false, int XW = 0, bool CL = false>
__global__ void __launch_bounds__(DecodeCfg<D, MT, DEEP>::THREADS)
decode_fwd_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                  const DecodeParams p) {
    using C = DecodeCfg<D, MT, DEEP>;
    constexpr int TK = C::TK, NW = C::NW, NG = C::NG, NCW = C::NCW, SWB = C::SWB, SWE = C::SWE, NSPAN = C::NSPAN;
    constexpr int NSTAGE = C::NSTAGE, QROWS = C::QROWS, QPITCH = C::QPITCH;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sBig = smem;                       // stages, later reduction scratch
    uint16_t* sQ = reinterpret_cast<uint16_t*>(smem + C::BIG);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BIG + C::Q_BYTES);
    uint64_t* empty = full + NSTAGE;
    uint64_t* merge_bar = empty + NSTAGE;      // [2] split-merge bulk copies
    volatile int* abort_flag = reinterpret_cast<volatile int*>(merge_bar + 2);
    volatile int* is_last = abort_flag + 1;
    volatile unsigned* s_seq = reinterpret_cast<volatile unsigned*>(is_last + 1);

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int split = blockIdx.x;
    const int hk = blockIdx.y / p.n_rg;
    const int rg = blockIdx.y % p.n_rg;
    const int b = blockIdx.z;
    const int r0 = rg * QROWS;
    const int nrows = min(QROWS, p.R - r0);
    // Global row index (over B*H_q*S_q) of this CTA's local row 0.
    const size_t row_base = (static_cast<size_t>(b) * p.H_q + static_cast<size_t>(hk) * p.G) * p.S_q + r0;
    const int kv_lo = split * p.chunk;
    const float c = p.scale_log2;

    if (tid == 0) {
        for (int s = 0; s < NSTAGE; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NW);
        }
        mbar_init(&merge_bar[0], 1);
        mbar_init(&merge_bar[1], 1);
        *abort_flag = 0;
        *is_last = 0;
        fence_mbar_init();
    }
    if (p.kv_box < TK) {
        // Short KV: TMA fills only kv_box rows of each tile; the rest stay zero.
        for (int i = tid; i < C::STAGES_BYTES / 16; i += C::THREADS)
            reinterpret_cast<uint4*>(sBig)[i] = make_uint4(0, 0, 0, 0);
        fence_proxy_async_smem();
    }
    // Set-up above touches shared memory only; global memory (this launch's inputs, the
    // workspace counters) is read after the previous launch on the stream has completed.
    grid_dep_wait();
    grid_dep_launch_dependents();
    int S_b = p.S_kv;                          // keys of this sequence
    if constexpr (PAGED) S_b = min(max(__ldg(p.seq_lens + b), 0), p.max_blocks * p.block_size);
    const int kv_hi = min(S_b, kv_lo + p.chunk);
    const int n_st = kv_hi > kv_lo ? (kv_hi - kv_lo + TK - 1) / TK : 0;   // 0: an empty split
    __syncthreads();
    if (warp < NCW) {
        // Consumers stage Q (padded, rows >= nrows zero) while the producer's first
        // K/V copies are already in flight.
        for (int idx = tid; idx < QROWS * (D / 8); idx += NCW * 32) {
            const int row = idx / (D / 8), ch = idx % (D / 8);
            uint4 v = make_uint4(0, 0, 0, 0);
            if (row < nrows) v = *reinterpret_cast<const uint4*>(p.Q + (row_base + row) * D + ch * 8);
            *reinterpret_cast<uint4*>(sQ + row * QPITCH + ch * 8) = v;
        }
        named_bar_sync(1, NCW * 32);
    }

    float o[MT][D / 8][4];
    float mrow[MT][2], lsum[MT][2];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
        mrow[mt][0] = mrow[mt][1] = -CUDART_INF_F;
        lsum[mt][0] = lsum[mt][1] = 0.f;
#pragma unroll
        for (int n = 0; n < D / 8; ++n) o[mt][n][0] = o[mt][n][1] = o[mt][n][2] = o[mt][n][3] = 0.f;
    }

    if (warp == NCW && PAGED) {
        // ------------------------------------------------------------ TMA producer (paged)
        // The whole warp walks the stages; lanes hold the pool-block ids of 32
        // consecutive logical blocks (one coalesced load), lane 0 issues the copies.
        if (lane == 0) {
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
        }
        const uint64_t pol = l2_policy_evict_first();
        const int BS = p.block_size;
        const int box = BS < TK ? BS : TK;
        const int n_blk = BS < TK ? TK / BS : 1;                 // pool blocks per stage
        const int used_blocks = (S_b + BS - 1) / BS;             // logical blocks holding keys
        const int* bt = p.block_table + static_cast<size_t>(b) * p.max_blocks;
        int cache_base = -(1 << 30), cache_val = -1;
        int issued = 0;
        for (int i = 0; i < n_st; ++i) {
            const int slot = i % NSTAGE, round = i / NSTAGE;
            bool ok = true;
            if (round > 0 && lane == 0)
                ok = mbar_wait_bounded(&empty[slot], (round - 1) & 1, abort_flag, p.timeout_ns);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) {
                if (lane == 0) atomicOr(&g_kf_dev_error, KF_DEVERR_TIMEOUT_SOFTMAX);
                break;
            }
            const int row = kv_lo + i * TK;
            const int lb0 = row / BS;
            const int r_in = BS < TK ? 0 : row % BS;
            if (lb0 < cache_base || lb0 + n_blk > cache_base + 32) {
                cache_base = lb0;
                const int lb = lb0 + lane;
                // Blocks past the sequence's last one read as -1: the copy then starts at
                // a negative coordinate and fills zeros (the table there may be stale).
                cache_val = lb < used_blocks ? __ldg(bt + lb) : -1;
            }
            if (lane == 0) mbar_arrive_expect_tx(&full[slot], 2 * NSPAN * TK * SWB);
            uint8_t* dK = sBig + slot * C::STAGE_BYTES;
            uint8_t* dV = dK + C::TILE_BYTES;
            for (int k = 0; k < n_blk; ++k) {
                const int pb = __shfl_sync(0xffffffffu, cache_val, lb0 + k - cache_base);
                if (lane == 0) {
                    const int c2 = pb * p.H_kv + hk;
#pragma unroll
                    for (int s2 = 0; s2 < NSPAN; ++s2) {
                        // Rows k*box .. of the stage: a multiple of 8 rows keeps the swizzle
                        // pattern of one whole-tile box.
                        tma_load_3d_hint(dK + s2 * TK * SWB + k * box * SWB, &tmK, &full[slot], s2 * SWE, r_in, c2, pol);
                        tma_load_3d_hint(dV + s2 * TK * SWB + k * box * SWB, &tmV, &full[slot], s2 * SWE, r_in, c2, pol);
                    }
                }
            }
            issued = i + 1;
        }
        if (lane == 0 && *abort_flag) {
            const int first = issued > NSTAGE ? issued - NSTAGE : 0;
            int dummy = 0;
            for (int i = first; i < issued; ++i)
                mbar_wait_bounded(&full[i % NSTAGE], (i / NSTAGE) & 1, &dummy, p.timeout_ns);
        }
    } else if (warp == NCW) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
            const uint64_t pol = l2_policy_evict_first();   // KV is streamed once
            const int bh = b * p.H_kv + hk;
            int issued = 0;
            for (int i = 0; i < n_st; ++i) {
                const int slot = i % NSTAGE, round = i / NSTAGE;
                if (round > 0 && !mbar_wait_bounded(&empty[slot], (round - 1) & 1, abort_flag, p.timeout_ns)) {
                    atomicOr(&g_kf_dev_error, KF_DEVERR_TIMEOUT_SOFTMAX);
                    break;
                }
                mbar_arrive_expect_tx(&full[slot], 2 * NSPAN * p.kv_box * SWB);
                uint8_t* dK = sBig + slot * C::STAGE_BYTES;
                uint8_t* dV = dK + C::TILE_BYTES;
                const int row = kv_lo + i * TK;
#pragma unroll
                for (int s = 0; s < NSPAN; ++s) {
                    tma_load_3d_hint(dK + s * TK * SWB, &tmK, &full[slot], s * SWE, row, bh, pol);
                    tma_load_3d_hint(dV + s * TK * SWB, &tmV, &full[slot], s * SWE, row, bh, pol);
                }
                issued = i + 1;
            }
            if (*abort_flag) {
                const int first = issued > NSTAGE ? issued - NSTAGE : 0;
                int dummy = 0;
                for (int i = first; i < issued; ++i)
                    mbar_wait_bounded(&full[i % NSTAGE], (i / NSTAGE) & 1, &dummy, p.timeout_ns);
            }
        }
    } else {
        // ------------------------------------------------------------ consumer warps
        const int cq = lane & 3;
        const int lm = lane >> 3, lr = lane & 7;
        const uint32_t sQa = smem_u32(sQ);
        const int g = warp / NW, wg = warp % NW;      // consumer group, 16-row slice of a stage
        for (int i = g; i < n_st; i += NG) {
            const int slot = i % NSTAGE;
            bool ok = mbar_wait_bounded(&full[slot], (i / NSTAGE) & 1, abort_flag, p.timeout_ns);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) { atomicOr(&g_kf_dev_error, KF_DEVERR_TIMEOUT_TMA); break; }
            const uint32_t sK = smem_u32(sBig + slot * C::STAGE_BYTES);
            const uint32_t sV = sK + C::TILE_BYTES;

            // S = Q K^T for this warp's 16 KV rows.
            float s[MT][2][4];
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) s[mt][nt][0] = s[mt][nt][1] = s[mt][nt][2] = s[mt][nt][3] = 0.f;
#pragma unroll
            for (int ks = 0; ks < D / 16; ++ks) {
                uint32_t b00, b01, b10, b11;
                const int krow = wg * 16 + lr + ((lm >> 1) << 3);
                const int kcol = ks * 16 + ((lm & 1) << 3);
                ldmatrix_x4(sK + swz_offset<SWB>(TK, krow, kcol), b00, b01, b10, b11);
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    uint32_t a0, a1, a2, a3;
                    const int qrow = mt * 16 + lr + ((lm & 1) << 3);
                    const int qcol = ks * 16 + ((lm >> 1) << 3);
                    ldmatrix_x4(sQa + (qrow * QPITCH + qcol) * 2, a0, a1, a2, a3);
                    mma_16816(s[mt][0], a0, a1, a2, a3, b00, b01);
                    mma_16816(s[mt][1], a0, a1, a2, a3, b10, b11);
                }
            }
            // Mask keys past the end of this split (only the last stage can hold them).
            if (i == n_st - 1) {
                const int kv0 = kv_lo + i * TK + wg * 16 + 2 * cq;
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            if (kv0 + nt * 8 + (e & 1) >= kv_hi) s[mt][nt][e] = -CUDART_INF_F;
            }
            // Online softmax (raw-score units; c folds in 1/sqrt(D) and log2 e).
            uint32_t pa[MT][4];
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    float mx = fmaxf(fmaxf(s[mt][0][2 * hh], s[mt][0][2 * hh + 1]),
                                     fmaxf(s[mt][1][2 * hh], s[mt][1][2 * hh + 1]));
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
                    const float m_new = fmaxf(mrow[mt][hh], mx);
                    const float m_use = (m_new == -CUDART_INF_F) ? 0.f : m_new;
                    const float f = ex2_approx((mrow[mt][hh] - m_use) * c);
                    mrow[mt][hh] = m_new;
                    const float neg = -m_use * c;
                    float ps = 0.f;
#pragma unroll
                    for (int nt = 0; nt < 2; ++nt) {
                        s[mt][nt][2 * hh] = ex2_approx(fmaf(s[mt][nt][2 * hh], c, neg));
                        s[mt][nt][2 * hh + 1] = ex2_approx(fmaf(s[mt][nt][2 * hh + 1], c, neg));
                        ps += s[mt][nt][2 * hh] + s[mt][nt][2 * hh + 1];
                    }
                    lsum[mt][hh] = lsum[mt][hh] * f + ps;
                    if (__any_sync(0xffffffffu, f != 1.0f)) {    // the row max moved (rare after the start)
#pragma unroll
                        for (int n = 0; n < D / 8; ++n) {
                            o[mt][n][2 * hh] *= f;
                            o[mt][n][2 * hh + 1] *= f;
                        }
                    }
                }
                pa[mt][0] = pack_half2(s[mt][0][0], s[mt][0][1]);
                pa[mt][1] = pack_half2(s[mt][0][2], s[mt][0][3]);
                pa[mt][2] = pack_half2(s[mt][1][0], s[mt][1][1]);
                pa[mt][3] = pack_half2(s[mt][1][2], s[mt][1][3]);
            }
            // O += P V
#pragma unroll
            for (int dp = 0; dp < D / 16; ++dp) {
                uint32_t b0a, b1a, b0b, b1b;
                const int vrow = wg * 16 + lr + ((lm & 1) << 3);
                const int vcol = dp * 16 + ((lm >> 1) << 3);
                ldmatrix_x4_trans(sV + swz_offset<SWB>(TK, vrow, vcol), b0a, b1a, b0b, b1b);
                if (PAGED && i == n_st - 1) {
                    // P is 0 for keys past the end, but 0 * (Inf or NaN) is not: clear the V
                    // halves of those keys (this lane's keys 2cq, 2cq+1, 2cq+8, 2cq+9).
                    const int k0 = kv_lo + i * TK + wg * 16 + 2 * cq;
                    const uint32_t m0 = (k0 < kv_hi ? 0x0000ffffu : 0u) | (k0 + 1 < kv_hi ? 0xffff0000u : 0u);
                    const uint32_t m1 = (k0 + 8 < kv_hi ? 0x0000ffffu : 0u) | (k0 + 9 < kv_hi ? 0xffff0000u : 0u);
                    b0a &= m0; b0b &= m0; b1a &= m1; b1b &= m1;
                }
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    mma_16816(o[mt][2 * dp], pa[mt][0], pa[mt][1], pa[mt][2], pa[mt][3], b0a, b1a);
                    mma_16816(o[mt][2 * dp + 1], pa[mt][0], pa[mt][1], pa[mt][2], pa[mt][3], b0b, b1b);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
    }
    __syncthreads();   // every stage consumed: the ring memory becomes reduction scratch
    const bool aborted = *abort_flag != 0;
    if (aborted && (!SPLIT || p.n_split == 1)) return;
    // Cluster merge: the partial of this CTA at CL_OFF, then every CTA of the cluster
    // merges the output items i with i % n_split == its rank.  Every CTA reaches both
    // cluster barriers (an aborted one publishes an empty partial: m = -inf, l = 0).
    float* cl_o = reinterpret_cast<float*>(sBig + C::CL_OFF);    // [QROWS][D]
    float2* cl_ml = reinterpret_cast<float2*>(cl_o + QROWS * D);  // [QROWS]
    auto cluster_merge = [&]() {
        cluster_sync_all();
        const uint32_t n = static_cast<uint32_t>(p.n_split);
        const uint32_t rank = cluster_ctarank();
        const uint32_t o_base = smem_u32(cl_o), ml_base = smem_u32(cl_ml);
        const int items = nrows * (D / 4);
        for (int it = static_cast<int>(rank) + static_cast<int>(n) * tid; it < items;
             it += static_cast<int>(n) * C::THREADS) {
            const int row = it / (D / 4), d = (it % (D / 4)) * 4;
            // Every peer's (m, l) and O slice are requested before any is used, so the
            // distributed-shared-memory round trips overlap.
            float2 ml[C::MAX_CLUSTER];
            float4 v[C::MAX_CLUSTER];
#pragma unroll
            for (int r = 0; r < C::MAX_CLUSTER; ++r) {
                if (r < static_cast<int>(n)) {
                    ml[r] = ld_dsmem_f2(dsmem_map(ml_base + row * 8, r));
                    v[r] = ld_dsmem_f4(dsmem_map(o_base + (row * D + d) * 4, r));
                } else {
                    ml[r] = make_float2(-CUDART_INF_F, 0.f);
                    v[r] = make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
            float M = -CUDART_INF_F;
#pragma unroll
            for (int r = 0; r < C::MAX_CLUSTER; ++r) M = fmaxf(M, ml[r].x);
            const float Mu = (M == -CUDART_INF_F) ? 0.f : M;
            float L = 0.f;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int r = 0; r < C::MAX_CLUSTER; ++r) {
                const float wt = ex2_approx((ml[r].x - Mu) * c);
                L += wt * ml[r].y;
                acc.x += wt * v[r].x; acc.y += wt * v[r].y; acc.z += wt * v[r].z; acc.w += wt * v[r].w;
            }
            const float sc = p.unnormalized ? 1.f : (L > 0.f ? 1.f / L : 0.f);
            store_out4(p.O, (row_base + row) * D + d, make_float4(acc.x * sc, acc.y * sc, acc.z * sc, acc.w * sc),
                       p.out_type);
            if (d == 0) {
                if (p.Mi) p.Mi[row_base + row] = M * p.scale;
                if (p.Li) p.Li[row_base + row] = L;
            }
        }
        cluster_sync_all();   // the other CTAs have read this CTA's partial
    };
    if constexpr (CL) {
        static_assert(SPLIT && XW == 0 && !PAGED, "cluster merge: contiguous split kernels only");
        static_assert(C::RED_FLOATS * 4 <= C::CL_OFF, "cluster partial overlaps the reduction scratch");
        if (aborted) {
            if (tid < QROWS) cl_ml[tid] = make_float2(-CUDART_INF_F, 0.f);
            cluster_merge();
            return;
        }
    } else if (aborted) {
        // A wait expired (the device error word says so).  The split still takes its
        // ticket, and the last one resets the unit's counter without merging, so the
        // counters are zero again after the call and the next call's merge is right.
        const size_t cidx = (static_cast<size_t>(b) * p.H_kv + hk) * p.n_rg + rg;
        if (tid == 0) {
            const unsigned ticket = atom_add_acq_rel_gpu(&p.counters[cidx], 1u);
            if (ticket == static_cast<unsigned>(p.n_split - 1)) p.counters[cidx] = 0u;
        }
        return;
    }

    if constexpr (NG > 1) {
        // Group 1 hands its fragments (same rows and columns as group 0's warp of the
        // same slice) to group 0, which merges them by log-sum-exp in registers.
        constexpr int PER_LANE = MT * D / 2 + 4 * MT;
        float* gx = reinterpret_cast<float*>(sBig) + ((warp % NW) * 32 + lane) * PER_LANE;
        if (warp >= NW && warp < NCW) {
            int k = 0;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) { gx[k++] = mrow[mt][hh]; gx[k++] = lsum[mt][hh]; }
#pragma unroll
                for (int n = 0; n < D / 8; ++n)
#pragma unroll
                    for (int e = 0; e < 4; ++e) gx[k++] = o[mt][n][e];
            }
        }
        __syncthreads();
        if (warp < NW) {
            int k = 0;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                float fa[2], fb[2];
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    const float mb = gx[k++], lb = gx[k++];
                    const float M = fmaxf(mrow[mt][hh], mb);
                    const float Mu = (M == -CUDART_INF_F) ? 0.f : M;
                    fa[hh] = ex2_approx((mrow[mt][hh] - Mu) * c);
                    fb[hh] = ex2_approx((mb - Mu) * c);
                    mrow[mt][hh] = M;
                    lsum[mt][hh] = lsum[mt][hh] * fa[hh] + lb * fb[hh];
                }
#pragma unroll
                for (int n = 0; n < D / 8; ++n)
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int hh = e >> 1;
                        o[mt][n][e] = o[mt][n][e] * fa[hh] + gx[k++] * fb[hh];
                    }
            }
        }
        __syncthreads();   // fragments read before the reduction below reuses the memory
    }

    float* red_m = reinterpret_cast<float*>(sBig);            // [NW][QROWS]
    float* red_l = red_m + NW * QROWS;                         // [NW][QROWS]
    float* red_o = red_l + NW * QROWS;                         // [NW][QROWS][D]
    if (warp < NW) {
        const int g = lane >> 2, cq = lane & 3;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                float l = lsum[mt][hh];
                l += __shfl_xor_sync(0xffffffffu, l, 1);
                l += __shfl_xor_sync(0xffffffffu, l, 2);
                const int row = mt * 16 + g + 8 * hh;
                if (cq == 0) {
                    red_m[warp * QROWS + row] = mrow[mt][hh];
                    red_l[warp * QROWS + row] = l;
                }
#pragma unroll
                for (int n = 0; n < D / 8; ++n)
                    *reinterpret_cast<float2*>(red_o + (warp * QROWS + row) * D + n * 8 + 2 * cq) =
                        make_float2(o[mt][n][2 * hh], o[mt][n][2 * hh + 1]);
            }
    }
    __syncthreads();
    // Per-row weights of each warp, the merged max and sum.
    float* wts = red_o + NW * QROWS * D;                       // [NW][QROWS]
    float* Mrow = wts + NW * QROWS;                            // [QROWS]
    float* Lrow = Mrow + QROWS;                                // [QROWS]
    if (tid < QROWS) {
        float M = -CUDART_INF_F;
#pragma unroll
        for (int w = 0; w < NW; ++w) M = fmaxf(M, red_m[w * QROWS + tid]);
        const float Mu = (M == -CUDART_INF_F) ? 0.f : M;
        float L = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            const float wt = ex2_approx((red_m[w * QROWS + tid] - Mu) * c);
            wts[w * QROWS + tid] = wt;
            L += wt * red_l[w * QROWS + tid];
        }
        Mrow[tid] = M;
        Lrow[tid] = L;
    }
    __syncthreads();

    if (!SPLIT || p.n_split == 1) {
        if constexpr (XW > 0) {
            constexpr int KX = (QROWS * (D / 4) + C::THREADS - 1) / C::THREADS;
            float4 acc[KX];
#pragma unroll
            for (int k = 0; k < KX; ++k) {
                const int it = tid + k * C::THREADS;
                acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (it < nrows * (D / 4)) {
                    const int row = it / (D / 4), d = (it % (D / 4)) * 4;
#pragma unroll
                    for (int w = 0; w < NW; ++w) {
                        const float wt = wts[w * QROWS + row];
                        const float4 v = *reinterpret_cast<const float4*>(red_o + (w * QROWS + row) * D + d);
                        acc[k].x += wt * v.x; acc[k].y += wt * v.y; acc[k].z += wt * v.z; acc[k].w += wt * v.w;
                    }
                }
            }
            const size_t cidx = (static_cast<size_t>(b) * p.H_kv + hk) * p.n_rg + rg;
            xch_unit<XW, D, KX, C::THREADS>(p, cidx, nrows, row_base, acc, Mrow, Lrow, s_seq,
                                            reinterpret_cast<float*>(sQ));
        } else {
        for (int idx = tid; idx < nrows * (D / 4); idx += C::THREADS) {
            const int row = idx / (D / 4), d = (idx % (D / 4)) * 4;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int w = 0; w < NW; ++w) {
                const float wt = wts[w * QROWS + row];
                const float4 v = *reinterpret_cast<const float4*>(red_o + (w * QROWS + row) * D + d);
                acc.x += wt * v.x; acc.y += wt * v.y; acc.z += wt * v.z; acc.w += wt * v.w;
            }
            const float sc = p.unnormalized ? 1.f : (Lrow[row] > 0.f ? 1.f / Lrow[row] : 0.f);
            acc.x *= sc; acc.y *= sc; acc.z *= sc; acc.w *= sc;
            store_out4(p.O, (row_base + row) * D + d, acc, p.out_type);
        }
        if (tid < nrows) {
            if (p.Mi) p.Mi[row_base + tid] = Mrow[tid] * p.scale;
            if (p.Li) p.Li[row_base + tid] = Lrow[tid];
        }
        }
        return;
    }

    if constexpr (CL) {
        for (int idx = tid; idx < nrows * (D / 4); idx += C::THREADS) {
            const int row = idx / (D / 4), d = (idx % (D / 4)) * 4;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int w = 0; w < NW; ++w) {
                const float wt = wts[w * QROWS + row];
                const float4 v = *reinterpret_cast<const float4*>(red_o + (w * QROWS + row) * D + d);
                acc.x += wt * v.x; acc.y += wt * v.y; acc.z += wt * v.z; acc.w += wt * v.w;
            }
            *reinterpret_cast<float4*>(cl_o + row * D + d) = acc;
        }
        if (tid < nrows) cl_ml[tid] = make_float2(Mrow[tid], Lrow[tid]);
        cluster_merge();
        return;
    }

    // ---- split partial: (m, l, O_u) relative to this split's max.
    // Layout: a (b, h_kv, row group) unit owns rows [row_base, row_base + nrows);
    // its partials are [split][row][D] at row_base * ns * D, so a run of splits
    // is one contiguous block the merging CTA can bulk-copy.
    const int ns = p.n_split;
    const size_t unit_off = row_base * static_cast<size_t>(ns);
    for (int idx = tid; idx < nrows * (D / 4); idx += C::THREADS) {
        const int row = idx / (D / 4), d = (idx % (D / 4)) * 4;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            const float wt = wts[w * QROWS + row];
            const float4 v = *reinterpret_cast<const float4*>(red_o + (w * QROWS + row) * D + d);
            acc.x += wt * v.x; acc.y += wt * v.y; acc.z += wt * v.z; acc.w += wt * v.w;
        }
        *reinterpret_cast<float4*>(p.part_O + (unit_off + static_cast<size_t>(split) * nrows + row) * D + d) = acc;
    }
    if (tid < nrows) {
        *reinterpret_cast<float2*>(p.part_ml + (unit_off + static_cast<size_t>(split) * nrows + tid) * 2) =
            make_float2(Mrow[tid], Lrow[tid]);
    }
    // Publication: the CTA barrier orders every thread's partial stores before
    // thread 0's ticket, a release-acquire atomic at GPU scope (one round trip,
    // no separate fence); the merging CTA's acquire and barrier order its reads
    // after all of them, and the proxy fences cover its bulk (async-proxy) copies
    // (into shared memory this CTA's threads wrote during the reduction, too).
    fence_proxy_async_global();
    fence_proxy_async_smem();
    __syncthreads();
    const size_t cidx = (static_cast<size_t>(b) * p.H_kv + hk) * p.n_rg + rg;
    if (tid == 0) {
        const unsigned ticket = atom_add_acq_rel_gpu(&p.counters[cidx], 1u);
        *is_last = (ticket == static_cast<unsigned>(ns - 1)) ? 1 : 0;
    }
    __syncthreads();
    if (!*is_last) return;
    fence_proxy_async_global();

    // ---- last CTA of this unit: merge all splits.
    // (1) per row: M = max_s m_s, weights w_s = e^{m_s - M}, L = sum_s w_s l_s
    //     (one warp per row, lanes over splits);
    // (2) O = sum_s w_s O_s / L, with runs of splits brought into shared memory
    //     by double-buffered TMA bulk copies and reduced from there.
    constexpr int WT_BYTES = (C::MAX_SPLIT * QROWS + 2 * QROWS) * 4;
    float* swt = reinterpret_cast<float*>(sBig + C::BIG - WT_BYTES);   // [ns][nrows]
    float* sM = swt + C::MAX_SPLIT * QROWS;
    float* sL = sM + QROWS;
    const float* ml = p.part_ml + unit_off * 2;
    constexpr int KMAX = (QROWS * (D / 4) + C::THREADS - 1) / C::THREADS;
    const int items = nrows * (D / 4);
    const uint32_t split_bytes = static_cast<uint32_t>(nrows) * D * 4;
    const int buf_bytes = ((C::BIG - WT_BYTES) / 2) / 16 * 16;
    int per_chunk = buf_bytes / static_cast<int>(split_bytes);
    per_chunk = per_chunk < 1 ? 1 : (per_chunk > ns ? ns : per_chunk);
    const int n_chunks = (ns + per_chunk - 1) / per_chunk;
    const float* src = p.part_O + unit_off * D;
    auto issue = [&](int ch) {
        const int s0 = ch * per_chunk;
        const int cnt = min(per_chunk, ns - s0);
        uint64_t* bar = &merge_bar[ch & 1];
        mbar_arrive_expect_tx(bar, cnt * split_bytes);
        bulk_g2s(sBig + (ch & 1) * buf_bytes, src + static_cast<size_t>(s0) * nrows * D, cnt * split_bytes, bar);
    };
    if (tid == 0) {           // the partials' copies fly while the weights are formed
        issue(0);
        if (n_chunks > 1) issue(1);
    }
    for (int r = warp; r < nrows; r += C::THREADS / 32) {
        float M = -CUDART_INF_F;
        for (int s2 = lane; s2 < ns; s2 += 32) M = fmaxf(M, __ldcg(ml + (s2 * nrows + r) * 2));
#pragma unroll
        for (int o2 = 16; o2 > 0; o2 >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o2));
        const float Mu = (M == -CUDART_INF_F) ? 0.f : M;
        float L = 0.f;
        for (int s2 = lane; s2 < ns; s2 += 32) {
            const float2 v = __ldcg(reinterpret_cast<const float2*>(ml + (s2 * nrows + r) * 2));
            const float wt = ex2_approx((v.x - Mu) * c);
            swt[s2 * nrows + r] = wt;
            L += wt * v.y;
        }
#pragma unroll
        for (int o2 = 16; o2 > 0; o2 >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o2);
        if (lane == 0) {
            sM[r] = M;
            sL[r] = L;
        }
    }
    __syncthreads();

    float4 acc[KMAX];
#pragma unroll
    for (int k = 0; k < KMAX; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    bool ok = true;
    for (int ch = 0; ch < n_chunks; ++ch) {
        int dummy = 0;
        ok = mbar_wait_bounded(&merge_bar[ch & 1], (ch >> 1) & 1, &dummy, p.timeout_ns);
        if (!ok) {   // cannot happen unless the copy engine stalls; leave the unit unwritten
            atomicOr(&g_kf_dev_error, KF_DEVERR_TIMEOUT_TMA);
            break;
        }
        const float* sb = reinterpret_cast<const float*>(sBig + (ch & 1) * buf_bytes);
        const int s0 = ch * per_chunk;
        const int cnt = min(per_chunk, ns - s0);
#pragma unroll
        for (int k = 0; k < KMAX; ++k) {
            const int it = tid + k * C::THREADS;
            if (it < items) {
                const int r = it / (D / 4), d = (it % (D / 4)) * 4;
                for (int s2 = 0; s2 < cnt; ++s2) {
                    const float wt = swt[(s0 + s2) * nrows + r];
                    const float4 v = *reinterpret_cast<const float4*>(sb + (s2 * nrows + r) * D + d);
                    acc[k].x += wt * v.x; acc[k].y += wt * v.y; acc[k].z += wt * v.z; acc[k].w += wt * v.w;
                }
            }
        }
        __syncthreads();   // buffer (ch & 1) fully read
        if (tid == 0 && ch + 2 < n_chunks) issue(ch + 2);
    }
    if constexpr (XW > 0) {
        // Every thread takes part (the exchange synchronizes the CTA); after a failed
        // copy above the error word is already set and the peers' merge is void.
        if (tid == 0) p.counters[cidx] = 0u;
        xch_unit<XW, D, KMAX, C::THREADS>(p, cidx, nrows, row_base, acc, sM, sL, s_seq,
                                          reinterpret_cast<float*>(sQ));
        return;
    }
    if (ok) {
#pragma unroll
        for (int k = 0; k < KMAX; ++k) {
            const int it = tid + k * C::THREADS;
            if (it < items) {
                const int r = it / (D / 4), d = (it % (D / 4)) * 4;
                const float sc = p.unnormalized ? 1.f : (sL[r] > 0.f ? 1.f / sL[r] : 0.f);
                store_out4(p.O, (row_base + r) * D + d, make_float4(acc[k].x * sc, acc[k].y * sc, acc[k].z * sc, acc[k].w * sc),
                           p.out_type);
            }
        }
        if (tid < nrows) {
            if (p.Mi) p.Mi[row_base + tid] = sM[tid] * p.scale;
            if (p.Li) p.Li[row_base + tid] = sL[tid];
        }
    }
    if (tid == 0) p.counters[cidx] = 0u;
}

// Merge G partial results (m in natural-log units of the scaled scores, l,
// un-normalised O) by log-sum-exp: M = max_g m_g,
// O = sum_g e^{m_g - M} O_g / sum_g e^{m_g - M} l_g.  Parts are stacked
// [G][rows] and [G][rows][D].  Used after the cross-GPU all-gather.
__global__ void combine_partials_kernel(const float* __restrict__ O_parts, const float* __restrict__ m_parts,
                                        const float* __restrict__ l_parts, int n_parts, long long rows, int D,
                                        long long stride_o, long long stride_ml,
                                        float* __restrict__ O, float* __restrict__ Mi, float* __restrict__ Li) {
    // Part g: O at O_parts + g*stride_o ([rows][D]), m/l at m_parts/l_parts + g*stride_ml ([rows]).
    const long long n4 = rows * (D / 4);
    constexpr float LOG2E = 1.4426950408889634f;
    for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < n4;
         idx += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long row = idx / (D / 4);
        const int d = static_cast<int>(idx % (D / 4)) * 4;
        float M = -CUDART_INF_F;
        for (int g = 0; g < n_parts; ++g) M = fmaxf(M, m_parts[g * stride_ml + row]);
        const float Mu = (M == -CUDART_INF_F) ? 0.f : M;
        float L = 0.f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int g = 0; g < n_parts; ++g) {
            const float wt = ex2_approx((m_parts[g * stride_ml + row] - Mu) * LOG2E);
            L += wt * l_parts[g * stride_ml + row];
            const float4 v = *reinterpret_cast<const float4*>(O_parts + g * stride_o + row * D + d);
            acc.x += wt * v.x; acc.y += wt * v.y; acc.z += wt * v.z; acc.w += wt * v.w;
        }
        const float inv = 1.f / L;
        acc.x *= inv; acc.y *= inv; acc.z *= inv; acc.w *= inv;
        *reinterpret_cast<float4*>(O + row * D + d) = acc;
        if (d == 0) {
            if (Mi) Mi[row] = M;
            if (Li) Li[row] = L;
        }
    }
}

}  // namespace kf
