// prefill_sm100.cuh -- non-causal attention forward on tcgen05 tensor cores.
//
// Replaces the reference's flash_attn_kernel<D> (kernels/flash_attn.cu:384-585)
// for query blocks of many rows (prefill).  Same math and layout contract:
// Q [B,H_q,S_q,D] fp16, K/V [B,H_kv,S_kv,D] fp16, O [B,H_q,S_q,D] fp32,
// optional Mi/Li [B,H_q,S_q] fp32 (row max of the scaled scores, sum of
// exp(score - Mi): kernels/flash_attn.cu:575-578), softmax scale 1/sqrt(D),
// GQA head map h_kv = h_q / (H_q/H_kv) (kernels/flash_attn.cu:406).
//
// One CTA owns NQ query tiles of 128 rows of one (b, h_q) and streams all of
// that head's K/V through a ring of shared-memory slots:
//   warp 0      TMA producer: Q tiles once, then K_0, V_0, K_1, V_1, ... into
//               the ring (3-D tensor maps, 128-B (or 32-B) swizzle, zero fill past
//               S_q / S_kv); every load is issued 1.5-2 KV steps before its use.
//   warp 1      TMEM owner + single-thread MMA issuer:
//                 S_t  = Q_t K_j^T        (tcgen05.mma, M=128, N=BC, fp32 in TMEM)
//                 O_t += P_t V_j          (tcgen05.mma, A = P_t from TMEM, M=128, N=D)
//               in the order PV_A(j-1), QK_A(j), PV_B(j-1), QK_B(j), so the tensor
//               core works on one tile while the other tile's softmax runs.
//   warps 4..   one softmax warpgroup per Q tile, one thread per query row:
//               tcgen05.ld of the S row, row max in registers, exp2 with the
//               scale folded in, P (fp16 pairs) written back over the first
//               BC/2 TMEM columns of S_t with tcgen05.st (the PV MMA's A operand;
//               the next QK MMA into S_t is issued after that PV, and tcgen05 MMAs
//               from one thread execute in order),
//               lazy rescale of the O row in TMEM only when the running max
//               grows by more than 2^8; epilogue O /= l straight from TMEM.
// All waits are bounded (kf_ptx.cuh); a timeout raises a device error word
// and every role unwinds, drains its in-flight copies/MMAs, frees TMEM.
#pragma once

#include <type_traits>

#include <math_constants.h>

#include "kf_ptx.cuh"

namespace kf {

// Phase trace (developer builds only: -DKF_PREFILL_TRACE, see phase_trace.py): one
// global-timer stamp per phase and CTA, for the CTA's last item.  Without the macro every
// KF_TRACE is empty and the kernels are unchanged.
enum PrefillTracePoint {
    kTrEntry, kTrSetup, kTrProdQ, kTrMmaQ, kTrMmaK0, kTrFirstS0, kTrFirstS1, kTrOFull0, kTrOFull1,
    kTrHalvesMet, kTrHalvesMerged, kTrOwnerWaited, kTrPartialWritten, kTrTicket, kTrItemEnd0,
    kTrItemEnd1, kTrExit, kTrProdRegs, kTrProdItem, kTrPassBuilt0, kTrPassStored0, kTrPassBuilt1,
    kTrPassStored1, kTrSmid, kTrSlots = 32
};
constexpr int kTraceCtas = 1024;
#ifdef KF_PREFILL_TRACE
__device__ unsigned long long g_kf_prefill_trace[kTraceCtas * kTrSlots];
#define KF_TRACE(i)                                                                                   \
    do {                                                                                              \
        if (blockIdx.x < kTraceCtas) g_kf_prefill_trace[blockIdx.x * kTrSlots + (i)] = global_timer_ns(); \
    } while (0)
#define KF_TRACE_SMID()                                                                               \
    do {                                                                                              \
        unsigned smid_;                                                                               \
        asm volatile("mov.u32 %0, %%smid;" : "=r"(smid_));                                            \
        KF_TRACE(kTrEntry);                                                                           \
        if (blockIdx.x < kTraceCtas) g_kf_prefill_trace[blockIdx.x * kTrSlots + kTrSmid] = smid_;     \
    } while (0)
#else
#define KF_TRACE(i) do { } while (0)
#define KF_TRACE_SMID() do { } while (0)
#endif

template <int D>
struct PrefillCfg {
    static constexpr int BM = 128;                     // query rows per tile (UMMA M)
    static constexpr int NQ = (D <= 128) ? 2 : 1;      // query tiles per CTA
    static constexpr int BC = (D <= 128) ? 128 : 64;   // KV rows per tile (UMMA N of QK^T)
    static constexpr int SWB = (D >= 64) ? 128 : 2 * D;  // swizzle span in bytes
    static constexpr int SWE = SWB / 2;                // fp16 elements per span
    static constexpr int NSPAN = D / SWE;              // spans (TMA boxes) per row
    static constexpr int Q_BYTES = BM * D * 2;
    static constexpr int KV_BYTES = BC * D * 2;
    static constexpr int SMEM_LIMIT = 232448;          // 227 KB opt-in per CTA
    static constexpr int BAR_BYTES = 1024;
    static constexpr int FIXED = NQ * Q_BYTES;
    static constexpr int NSLOT_RAW = (SMEM_LIMIT - 1024 - BAR_BYTES - FIXED) / KV_BYTES;
    static constexpr int NSLOT = NSLOT_RAW > 8 ? 8 : NSLOT_RAW;
    static constexpr int SMEM_BYTES = 1024 + FIXED + NSLOT * KV_BYTES + BAR_BYTES;
    static constexpr int TMEM_USED = NQ * (BC + D);
    static constexpr int TMEM_COLS = TMEM_USED <= 32 ? 32 : TMEM_USED <= 64 ? 64 : TMEM_USED <= 128 ? 128
                                   : TMEM_USED <= 256 ? 256 : 512;
    static constexpr int THREADS = 128 * (1 + NQ);
    // Epilogue: O tile staged in shared memory (128-B swizzled fp32 spans of 32
    // columns) and written by TMA stores; D = 16 keeps per-thread row stores.
    static constexpr bool TMA_STORE = D % 32 == 0;
    static_assert(!TMA_STORE || BM * D * 4 <= (NQ == 2 ? NQ * Q_BYTES : NSLOT * KV_BYTES), "O staging area");
    // Registers after rebalancing (NQ == 2: 384 threads launch with 168 each):
    // control warpgroup 128 x 112 + softmax warpgroups 256 x 192 = 63488 <= 64512.
#ifndef KF_PREFILL_L2AHEAD
#define KF_PREFILL_L2AHEAD 4
#endif
    static constexpr int L2AHEAD = KF_PREFILL_L2AHEAD;   // KV tiles of L2 prefetch lookahead
    static constexpr bool REBALANCE = NQ == 2;
    static constexpr int REG_CTRL = 112;
    static constexpr int REG_SOFTMAX = 192;
    static_assert(!REBALANCE || 128 * REG_CTRL + 256 * REG_SOFTMAX <= THREADS * (65536 / THREADS / 8 * 8),
                  "register split exceeds the launch allocation");
    static_assert(NSLOT >= 2, "K/V ring needs at least two slots");
    static_assert(SMEM_BYTES <= SMEM_LIMIT, "shared memory over budget");
    static_assert(TMEM_USED <= 512, "TMEM over budget");
};

// How long the owner chunk of a split unit waits for the other chunks' partials before
// it falls back to the ticket merge.  The chunks of a split unit run in the same last
// wave, so they normally finish within a few KV steps of each other.
constexpr uint64_t kOwnerWaitNs = 50000;

constexpr int KF_PF_UNNORMALIZED = 1;
constexpr int KF_PF_TICKET_MERGE = 2;

struct PrefillParams {
    void* O;           // [B,H_q,S_q,D] of out_type (fp32 when unnormalized)
    float* Mi;   // nullable
    float* Li;   // nullable
    int H_q, H_kv, S_q, S_kv, G;
    int B_H;            // B * H_q
    float scale_log2;   // (1/sqrt(D)) * log2(e)
    float scale;        // 1/sqrt(D)
    int flags;          // KF_PF_UNNORMALIZED: write O_u = sum exp(s - Mi) v (partial form), Mi/Li
                        // required; KF_PF_TICKET_MERGE: split units skip the owner wait
    int out_type;       // KF_OUT_F32 / KF_OUT_F16 / KF_OUT_BF16
    int q_box;          // rows per Q TMA box: min(BM, S_q)
    int kv_box;         // rows per K/V TMA box: min(BC, S_kv)
    // Work list (1-D grid).  Unit u = (b, h_q, 256-row block) with the block index
    // fastest.  Units [0, n_plain) take one CTA over all keys; each of the units
    // [n_plain, n_units) -- the partial last wave -- is split over split_k CTAs,
    // each taking `per` KV tiles: chunk 0 waits on the unit's counter in `counters`
    // until the other chunks have written softmax partials to `part` and merges them
    // with its own O (or, past a short wait, the last chunk to take a ticket merges).
    int n_qblk;         // query blocks of unit_tiles * 128 rows per (b, h_q)
    int unit_tiles;     // query tiles per unit: NQ, or 1 when two-tile units would leave most SMs idle
    int kv_off;         // S_kv - S_q (>= 0); causal kernels: query i sees keys j <= i + kv_off
    int n_units, n_plain, split_k, per;
    int n_items;        // n_plain + (n_units - n_plain) * split_k; CTAs stride over them
    float* part;        // [n_units - n_plain][split_k][NQ*BM][D + 2]
    unsigned* counters; // one ticket per split unit, zero between calls
    unsigned long long timeout_ns;
};

template <int N>
__device__ __forceinline__ void tmem_ld_chunk(uint32_t taddr, uint32_t (&r)[N]) {
    if constexpr (N == 32) tmem_ld32(taddr, r); else tmem_ld16(taddr, r);
}
template <int N>
__device__ __forceinline__ void tmem_st_chunk(uint32_t taddr, const uint32_t (&r)[N]) {
    if constexpr (N == 32) tmem_st32(taddr, r); else tmem_st16(taddr, r);
}

// Bounded wait that ignores the abort flag (used while draining).
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity, uint64_t timeout_ns) {
    int dummy = 0;
    return mbar_wait_bounded(bar, parity, &dummy, timeout_ns);
}

// One work item of the 1-D list: whole units [0, n_plain) (b, h, 256-row block),
// then the KV chunks of the split units.  KVH (one-tile units): both tiles of the CTA take
// the unit's one query tile, tile t the keys of KV tiles [t * n_kv, (t + 1) * n_kv).
struct PrefillItem {
    int unit, chunk, qblk, h, b, h_kv, q_row0, nq_active, kt0, n_kv;
    int n_kv0;          // KV steps of tile 0 (causal: one fewer where its rows end before the last tile)
    bool split;
};

template <int D, bool CAUSAL, bool SPLIT, bool KVH>
__device__ __forceinline__ PrefillItem prefill_item(const PrefillParams& p, int item) {
    using C = PrefillCfg<D>;
    PrefillItem it;
    it.chunk = 0;
    if (!SPLIT || item < p.n_plain) {
        it.unit = item;
    } else {
        it.unit = p.n_plain + (item - p.n_plain) / p.split_k;
        it.chunk = (item - p.n_plain) % p.split_k;
    }
    it.split = SPLIT && it.unit >= p.n_plain;
    // Causal: heaviest query blocks (most visible keys) first, (b, h) fastest, so the
    // long units start first; otherwise the query block is fastest.
    it.qblk = CAUSAL ? p.n_qblk - 1 - it.unit / p.B_H : it.unit % p.n_qblk;
    it.h = CAUSAL ? (it.unit % p.B_H) % p.H_q : (it.unit / p.n_qblk) % p.H_q;
    it.b = CAUSAL ? (it.unit % p.B_H) / p.H_q : it.unit / (p.n_qblk * p.H_q);
    it.h_kv = it.h / p.G;
    it.q_row0 = it.qblk * p.unit_tiles * C::BM;
    const int rows_left = p.S_q - it.q_row0;
    it.nq_active = rows_left >= p.unit_tiles * C::BM ? p.unit_tiles : (rows_left + C::BM - 1) / C::BM;
    const int n_kv_all = (p.S_kv + C::BC - 1) / C::BC;
    it.kt0 = it.split ? it.chunk * p.per : 0;                                         // first KV tile
    it.n_kv = it.split ? min(p.per, n_kv_all - it.kt0) : n_kv_all;                   // KV tiles of the item
    it.n_kv0 = it.n_kv;
    if constexpr (CAUSAL) {
        // Keys up to the unit's last (valid) query row + kv_off.
        const int last_row = min(it.q_row0 + C::NQ * C::BM, p.S_q) - 1;
        const int u = min(n_kv_all, (last_row + p.kv_off) / C::BC + 1);
        if (it.split) {
            // Split unit (chunked prefill, S_kv >= 2 S_q): the unit's own u key tiles are
            // divided evenly over the split_k chunks.  The host keeps kv_off >= 384 (split_k - 1),
            // so every row of the unit sees at least one key of every chunk.
            it.kt0 = (it.chunk * u) / p.split_k;
            it.n_kv = ((it.chunk + 1) * u) / p.split_k - it.kt0;
            it.n_kv0 = it.n_kv;
        } else {
            it.n_kv = u;
            // Tile 0 of a two-tile unit stops at the KV tile holding its own last row's
            // diagonal: the unit's last KV tile is fully masked for it.
            it.n_kv0 = it.nq_active == 2 ? min(it.n_kv, (it.q_row0 + C::BM - 1 + p.kv_off) / C::BC + 1) : it.n_kv;
        }
    }
    if constexpr (KVH) {
        it.nq_active = 2;              // two key halves of one query tile (item's tile count is even)
        it.n_kv = it.n_kv / 2;         // per tile (all keys, or the split chunk's)
        it.n_kv0 = it.n_kv;
    }
    return it;
}

// Writes a tile's O (scaled by sc) from TMEM through a free K/V ring slot: passes of
// the slot's size, each staged as 128-B swizzled spans (32 fp32 or 64 fp16/bf16
// columns, the map's box and swizzle) and TMA-stored; rows past the tensor are
// dropped.  Called by the tile's 128 softmax threads; named barrier `bar` orders the
// passes; thread row 0 waits until the last pass's stores have read the slot.
// With don.n > 0 each output element is sc * O + sum_d don.w[d] * (donor d's value):
// the owner chunk of a split unit adds the other chunks' partial rows (fp32, global
// memory, float4 q of this row at don.col[d] + q * don.stride) to its own O from TMEM.
struct DonorRows {
    int n = 0;
    int stride = 0;
    const float4* col[3] = {nullptr, nullptr, nullptr};
    float w[3] = {0.f, 0.f, 0.f};
};

template <int D, int BM, int SLOT_BYTES>
__device__ __forceinline__ void stage_store_tile(uint8_t* slot, uint32_t tO, int row, int bar, float sc, int out,
                                                 const CUtensorMap* map, int c1, int c2,
                                                 const DonorRows& don = DonorRows{}, uint8_t* slot2 = nullptr) {
    // o[0..31] = sc * O[cols c0 .. c0+31] (+ the donors' rows), in place.
    auto add_donors = [&](uint32_t (&o)[32], int c0) {
#pragma unroll
        for (int d = 0; d < 3; ++d) {
            if (d >= don.n) break;
            const float4* src = don.col[d] + static_cast<size_t>(c0 / 4) * don.stride;
            const float wd = don.w[d];
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float4 v = __ldcg(src + static_cast<size_t>(q) * don.stride);
                o[4 * q] = __float_as_uint(__uint_as_float(o[4 * q]) + wd * v.x);
                o[4 * q + 1] = __float_as_uint(__uint_as_float(o[4 * q + 1]) + wd * v.y);
                o[4 * q + 2] = __float_as_uint(__uint_as_float(o[4 * q + 2]) + wd * v.z);
                o[4 * q + 3] = __float_as_uint(__uint_as_float(o[4 * q + 3]) + wd * v.w);
            }
        }
    };
    constexpr int SPAN = BM * 128;
    constexpr int SPP = SLOT_BYTES / SPAN;                // spans per pass
    static_assert(SPP >= 1, "staging slot");
    const int cols = out == KF_OUT_F32 ? 32 : 64;         // columns per 128-B span
    const int n_spans = D / cols;
    const int n_pass = (n_spans + SPP - 1) / SPP;
#pragma unroll 1
    for (int ps = 0; ps < n_pass; ++ps) {
        // With a second slot, pass 1 is built there while pass 0's stores still read the
        // first; the wait after pass 1 covers both.
        uint8_t* sl = (slot2 != nullptr && ps == 1) ? slot2 : slot;
        const int k_end = min(SPP, n_spans - ps * SPP);
#pragma unroll 1
        for (int k = 0; k < k_end; ++k) {
            const int sp = ps * SPP + k;
            uint8_t* rowp = sl + k * SPAN + row * 128;
            if (out == KF_OUT_F32) {
                uint32_t o[32];
                tmem_ld32(tO + sp * 32, o);
                tmem_wait_ld();
#pragma unroll
                for (int k2 = 0; k2 < 32; ++k2) o[k2] = __float_as_uint(__uint_as_float(o[k2]) * sc);
                add_donors(o, sp * 32);
#pragma unroll
                for (int q = 0; q < 8; ++q)
                    *reinterpret_cast<float4*>(rowp + ((q ^ (row & 7)) << 4)) =
                        make_float4(__uint_as_float(o[4 * q]), __uint_as_float(o[4 * q + 1]),
                                    __uint_as_float(o[4 * q + 2]), __uint_as_float(o[4 * q + 3]));
            } else {
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {              // 32 columns -> 4 chunks of 16 B
                    uint32_t o[32];
                    tmem_ld32(tO + sp * 64 + hh * 32, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int k2 = 0; k2 < 32; ++k2) o[k2] = __float_as_uint(__uint_as_float(o[k2]) * sc);
                    add_donors(o, sp * 64 + hh * 32);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        uint4 w;
                        w.x = pack_out2(__uint_as_float(o[8 * q]), __uint_as_float(o[8 * q + 1]), out);
                        w.y = pack_out2(__uint_as_float(o[8 * q + 2]), __uint_as_float(o[8 * q + 3]), out);
                        w.z = pack_out2(__uint_as_float(o[8 * q + 4]), __uint_as_float(o[8 * q + 5]), out);
                        w.w = pack_out2(__uint_as_float(o[8 * q + 6]), __uint_as_float(o[8 * q + 7]), out);
                        const int cq = hh * 4 + q;
                        *reinterpret_cast<uint4*>(rowp + ((cq ^ (row & 7)) << 4)) = w;
                    }
                }
            }
        }
        if (row == 0) KF_TRACE(kTrPassBuilt0 + 2 * (ps & 1));
        fence_proxy_async_smem();
        named_bar_sync(bar, 128);
        const bool overlap = slot2 != nullptr && ps == 0 && n_pass > 1;    // pass 1 goes to slot2
        if (row == 0) {
            for (int k = 0; k < k_end; ++k) tma_store_3d(map, sl + k * SPAN, (ps * SPP + k) * cols, c1, c2);
            bulk_commit_group();
            if (!overlap) bulk_wait_group_read0();
            KF_TRACE(kTrPassStored0 + 2 * (ps & 1));
        }
        if (!overlap && ps + 1 < n_pass) named_bar_sync(bar, 128);    // slots read: next pass may write
    }
}

// Persistent CTAs: CTA c takes one item per round of gridDim.x items (snake order).  The K/V ring, TMEM and
// every barrier carry over from item to item (parities are running counts): the
// next item's Q loads as soon as the last QK MMA of the current one completes, its
// first K/V tiles stream while the current item finishes, and each tile's epilogue
// stages O through the ring slot of the item's last K (tile 0) or V (tile 1) tile,
// which the producer refills only after that epilogue's stores have read it.
// CAUSAL: bottom-right causal mask (PrefillParams::kv_off); a separate instantiation
// so the unmasked kernel carries none of its registers.  SPLIT: the work list has split
// units (a partial last wave, never causal); likewise its own instantiation, so plans
// without split units run a kernel without the split epilogue.
template <int D, bool CAUSAL, bool SPLIT, bool KVH = false>
__global__ void __launch_bounds__(PrefillCfg<D>::THREADS, 1)
prefill_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                   const PrefillParams p) {
    using C = PrefillCfg<D>;
    constexpr int BM = C::BM, BC = C::BC, NQ = C::NQ, SWB = C::SWB, SWE = C::SWE, NSPAN = C::NSPAN;
    constexpr int NSLOT = C::NSLOT;
    constexpr int OCH = D < 32 ? D : 32;   // TMEM columns per O chunk
    constexpr int RCH = D < 16 ? D : 16;   // TMEM columns per O chunk while S is held in registers

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;
    uint8_t* sKV = sQ + NQ * C::Q_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + NSLOT * C::KV_BYTES);
    uint64_t* q_full = bars;
    uint64_t* s_full = q_full + NQ;
    uint64_t* p_full = s_full + NQ;
    uint64_t* p_half = p_full + NQ;
    uint64_t* o_full = p_half + NQ;
    uint64_t* stage_free = o_full + NQ;      // tile t's epilogue has read its staging slot
    uint64_t* kv_full = stage_free + NQ;
    uint64_t* kv_empty = kv_full + NSLOT;
    uint64_t* q_empty = kv_empty + NSLOT;    // the item's last QK MMA completed
    uint64_t* mma_done = q_empty + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* ticket_last = abort_flag + 1;     // one flag per tile
    PrefillItem* first_item = reinterpret_cast<PrefillItem*>(const_cast<int*>(ticket_last) + 2);   // EARLY
    static_assert((6 * NQ + 2 * NSLOT + 2) * 8 + 16 + sizeof(PrefillItem) <= C::BAR_BYTES, "barrier area");

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0) KF_TRACE_SMID();
    // Item of round r of this CTA: rounds alternate direction over the CTAs (snake
    // order), so with items sorted heaviest first (causal) every CTA's total balances.
    auto prefill_item_index = [](int r) {
        const int G = static_cast<int>(gridDim.x), c = static_cast<int>(blockIdx.x);
        return r * G + ((r & 1) ? G - 1 - c : c);
    };

    // Key-half units (short calls, few items per CTA): the producer skips the
    // set-up barrier of the TMEM allocation, which it does not use, and its tensor maps
    // (kernel parameters) start loading at entry.  (Measured: C1 +2 %; no gain for the
    // long-unit kernels, whose prologue runs once per CTA: they keep the plain set-up.)
    constexpr bool EARLY = KVH;
    if (threadIdx.x == 0) {
        if constexpr (EARLY) {
            tma_prefetch_desc(&tmQ);
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
            // The producer's first item, decoded now (kernel parameters only) and parked in
            // shared memory: its Q load then issues as soon as the producer starts.
            if (static_cast<int>(blockIdx.x) < p.n_items)
                *first_item = prefill_item<D, CAUSAL, SPLIT, KVH>(p, static_cast<int>(blockIdx.x));
        }
        for (int t = 0; t < NQ; ++t) {
            mbar_init(&q_full[t], 1);
            mbar_init(&s_full[t], 1);
            mbar_init(&p_full[t], 128);
            mbar_init(&p_half[t], 128);
            mbar_init(&o_full[t], 1);
            mbar_init(&stage_free[t], 1);
        }
        for (int s = 0; s < NSLOT; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        mbar_init(q_empty, 1);
        mbar_init(mma_done, 1);
        *abort_flag = 0;
        for (int t = 0; t < NQ; ++t) ticket_last[t] = 0;
        fence_mbar_init();
    }
    if (p.q_box < BM || p.kv_box < BC) {
        // Short sequence: TMA writes only the first box rows of each tile; the
        // remaining rows must read as zero (zero V rows keep 0 * V finite).  The
        // host then gives every CTA a single item, so no epilogue staging lands here.
        for (int i = threadIdx.x; i < (NQ * C::Q_BYTES + NSLOT * C::KV_BYTES) / 16;
             i += blockDim.x)
            reinterpret_cast<uint4*>(sQ)[i] = make_uint4(0, 0, 0, 0);
        fence_proxy_async_smem();
    }
    if constexpr (EARLY) __syncthreads();    // barrier inits (and zero fill) seen by every thread
    // Set-up above touches shared memory only.  Global memory, and TMEM (which a CTA of
    // the previous launch on this SM may still hold), come after the previous launch on
    // the stream has completed.
    grid_dep_wait();
    grid_dep_launch_dependents();
    if constexpr (EARLY) {
        // The producer (warp 0) starts at once; the other warps wait for the TMEM
        // allocation on named barrier 1.
        if (warp != 0) {
            if (warp == 1) {
                tmem_alloc(tmem_slot, C::TMEM_COLS);
                tmem_relinquish();
            }
            tc_fence_before();
            named_bar_sync(1, C::THREADS - 32);
            tc_fence_after();
        }
    } else {
        if (warp == 1) {
            tmem_alloc(tmem_slot, C::TMEM_COLS);
            tmem_relinquish();
        }
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
    }
    if (threadIdx.x == 32) KF_TRACE(kTrSetup);         // the MMA warp, past the set-up barrier
    // The TMEM base is read from shared memory inside each role (after its setmaxnreg),
    // not held in a register across the register reallocation.
    auto tmem_base = [&]() { return *reinterpret_cast<volatile uint32_t*>(tmem_slot); };

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if constexpr (C::REBALANCE) setmaxnreg_dec<C::REG_CTRL>();
        if (lane == 0) KF_TRACE(kTrProdRegs);
        if (lane == 0) {
            if constexpr (!EARLY) {
                tma_prefetch_desc(&tmQ);
                tma_prefetch_desc(&tmK);
                tma_prefetch_desc(&tmV);
            }
            const uint32_t q_bytes = NSPAN * p.q_box * SWB;
            const uint32_t kv_bytes = NSPAN * p.kv_box * SWB;
            int pos = 0;                          // ring position of the next K/V load
            int n_done = 0;                       // items whose loads this thread issued
            uint32_t pend[NQ];                    // slots tile t's epilogue may still be reading
            int st_cnt[NQ], q_cnt[NQ];
#pragma unroll
            for (int t = 0; t < NQ; ++t) { pend[t] = 0u; st_cnt[t] = 0; q_cnt[t] = 0; }
            bool ok = true;
            for (int rnd = 0; rnd * static_cast<int>(gridDim.x) < p.n_items && ok; ++rnd) {
                const int item = prefill_item_index(rnd);
                if (item >= p.n_items) continue;
                const PrefillItem it = (EARLY && rnd == 0) ? *first_item : prefill_item<D, CAUSAL, SPLIT, KVH>(p, item);
                const int bh_q = it.b * p.H_q + it.h;
                const int bh_kv = it.b * p.H_kv + it.h_kv;
                if (n_done == 0) KF_TRACE(kTrProdItem);
                // Q of this item once the previous item's QK MMAs stopped reading Q.
                if (n_done > 0 && !mbar_wait_bounded(q_empty, (n_done - 1) & 1, abort_flag, p.timeout_ns)) {
                    atomicOr(&g_kf_dev_error, KF_DEVERR_TIMEOUT_MMA); ok = false; break;
                }
#pragma unroll
                for (int t = 0; t < NQ; ++t) {
                    if (t >= (KVH ? 1 : it.nq_active)) break;       // KVH: one query tile for both
                    mbar_arrive_expect_tx(&q_full[t], q_bytes);
                    for (int s = 0; s < NSPAN; ++s)
                        tma_load_3d(sQ + t * C::Q_BYTES + s * BM * SWB, &tmQ, &q_full[t], s * SWE,
                                    it.q_row0 + t * BM, bh_q);
                    ++q_cnt[t];
                    if (n_done == 0) KF_TRACE(kTrProdQ);
                }
                for (int i = 0; i < (KVH ? 4 : 2) * it.n_kv; ++i, ++pos) {
                    const int slot = pos % NSLOT;
                    const int round = pos / NSLOT;
                    if (round > 0 && !mbar_wait_bounded(&kv_empty[slot], (round - 1) & 1, abort_flag, p.timeout_ns)) {
                        atomicOr(&g_kf_dev_error, KF_DEVERR_TIMEOUT_MMA); ok = false; break;
                    }
#pragma unroll
                    for (int t = 0; t < NQ; ++t) {
                        if ((pend[t] >> slot) & 1u) {
                            if (!mbar_wait_bounded(&stage_free[t], st_cnt[t] & 1, abort_flag, p.timeout_ns)) {
                                atomicOr(&g_kf_dev_error, KF_DEVERR_TIMEOUT_SOFTMAX); ok = false; break;
                            }
                            ++st_cnt[t];
                            pend[t] &= ~(1u << slot);
                        }
                    }
                    if (!ok) break;
                    mbar_arrive_expect_tx(&kv_full[slot], kv_bytes);
                    // Ring order K_0, V_0, K_1, V_1, ...: a K refill takes the slot of a V freed
                    // mid-step and a V refill that of a K freed at the end of a step, so each
                    // load is issued 1.5 to 2 KV steps before its MMA needs it (TMA loads
                    // from L2 take about one step to land under full load).
                    // KVH: per step K of the first half, K of the second half, then their V.
                    const bool is_v = KVH ? (i & 3) >= 2 : (i & 1) != 0;
                    const int tile = KVH ? (i >> 2) + ((i & 1) ? it.n_kv : 0) : i >> 1;
                    const CUtensorMap* map = is_v ? &tmV : &tmK;
                    uint8_t* dst = sKV + slot * C::KV_BYTES;
                    for (int s = 0; s < NSPAN; ++s)
                        tma_load_3d(dst + s * BC * SWB, map, &kv_full[slot], s * SWE, (it.kt0 + tile) * BC, bh_kv);
                    // Warm L2 with the same operand L2AHEAD tiles ahead: the CTAs of one KV
                    // head stream it in near lockstep, so without this every tile is a
                    // first touch that waits on HBM.
                    if (C::L2AHEAD > 0 && tile + C::L2AHEAD < (KVH ? 2 : 1) * it.n_kv)
                        for (int s = 0; s < NSPAN; ++s)
                            tma_prefetch_l2_3d(map, s * SWE, (it.kt0 + tile + C::L2AHEAD) * BC, bh_kv);
                }
                if (!ok) break;
                if constexpr (KVH && C::TMA_STORE) {
                    // The merged tile is staged (by tile 0) in the slots of the last step's two
                    // K tiles: the first half's (released on stage_free[0]) and the second
                    // half's (on stage_free[1], which key-half units use for nothing else).
                    pend[0] |= 1u << ((pos - 4) % NSLOT);
                    pend[1] |= 1u << ((pos - 3) % NSLOT);
                } else if constexpr (!KVH && C::TMA_STORE) {
                    // The item's epilogue stages tile 0 in the slot of its last K and tile 1
                    // in the slot of its last V.
                    pend[0] |= 1u << ((pos - 2 - 2 * (it.n_kv - it.n_kv0)) % NSLOT);
                    if (NQ == 2 && it.nq_active == 2) pend[NQ - 1] |= 1u << ((pos - 1) % NSLOT);
                }
                ++n_done;
            }
            if (*abort_flag) {
                // Drain: every copy this thread issued must land before the CTA exits.
#pragma unroll
                for (int t = 0; t < NQ; ++t)
                    if (q_cnt[t] > 0) mbar_wait_drain(&q_full[t], (q_cnt[t] - 1) & 1, p.timeout_ns);
                for (int i = pos > NSLOT ? pos - NSLOT : 0; i < pos; ++i)
                    mbar_wait_drain(&kv_full[i % NSLOT], (i / NSLOT) & 1, p.timeout_ns);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if constexpr (C::REBALANCE) setmaxnreg_dec<C::REG_CTRL>();
        if (lane == 0) {
            const uint32_t tmem = tmem_base();
            constexpr uint32_t idesc_qk = umma_idesc_f16_f32(BM, BC, false, false);
            constexpr uint32_t idesc_pv = umma_idesc_f16_f32(BM, D, false, true);
            // Descriptors as (low, high) words: the high word is a constant and every
            // operand step is one add on the low word (the issue loop stays short).
            constexpr uint32_t DESC_HI = umma_desc_hi(8 * SWB, umma_layout_code(SWB));
            const uint32_t q_lo = (smem_u32(sQ) >> 4) + umma_desc_lbo(16);
            const uint32_t kv_lo = smem_u32(sKV) >> 4;
            // The tensor core queues only a few MMAs, so every barrier round trip this
            // thread waits on (~120 cycles even for a completed phase) idles it.  The
            // loop keeps them few: ring slot/phase are counters, K and V are tested
            // together, and a completed p_full makes the p_half wait unnecessary.
            int slotK = 0, parK = 0;        // ring position of the item's K_j
            int ring = 0;                   // KVH: ring position of the item's first load
            int q_cnt[NQ], steps[NQ];       // q_full completions, KV steps done, per tile
#pragma unroll
            for (int t = 0; t < NQ; ++t) { q_cnt[t] = 0; steps[t] = 0; }
            bool ok = true;
            for (int rnd = 0; rnd * static_cast<int>(gridDim.x) < p.n_items && ok; ++rnd) {
                const int item = prefill_item_index(rnd);
                if (item >= p.n_items) continue;
                const PrefillItem it = prefill_item<D, CAUSAL, SPLIT, KVH>(p, item);
                const int n_kv = it.n_kv, nq_active = it.nq_active;
#pragma unroll
                for (int t = 0; t < NQ; ++t) {
                    if (t >= (KVH ? 1 : nq_active) || !ok) break;
                    ok = mbar_wait_bounded(&q_full[t], q_cnt[t] & 1, abort_flag, p.timeout_ns);
                    ++q_cnt[t];
                }
                if (!ok) { atomicOr(&g_kf_dev_error, KF_DEVERR_TIMEOUT_TMA); break; }
                KF_TRACE(kTrMmaQ);
                if constexpr (KVH) {
                    // Two key halves of one query tile: step j reads K_t(j) at ring position
                    // ring + 4j + t and V_t(j - 1) at ring + 4(j - 1) + 2 + t; both tiles' QK use
                    // the one Q tile.  Same issue order as below: PV_0(j-1), QK_0(j), PV_1(j-1),
                    // QK_1(j), so each tile's MMAs overlap the other's softmax.
                    for (int j = 0; j <= n_kv && ok; ++j) {
                        int kpos[2], vpos[2];
#pragma unroll
                        for (int t = 0; t < 2; ++t) {
                            kpos[t] = ring + 4 * j + t;
                            vpos[t] = ring + 4 * (j - 1) + 2 + t;
                            if (ok && j < n_kv &&
                                !mbar_wait_bounded(&kv_full[kpos[t] % NSLOT], (kpos[t] / NSLOT) & 1, abort_flag,
                                                   p.timeout_ns))
                                ok = false;
                            if (ok && j > 0 &&
                                !mbar_wait_bounded(&kv_full[vpos[t] % NSLOT], (vpos[t] / NSLOT) & 1, abort_flag,
                                                   p.timeout_ns))
                                ok = false;
                        }
                        if (!ok) { atomicOr(&g_kf_dev_error, KF_DEVERR_TIMEOUT_TMA); break; }
                        tc_fence_after();
                        if (j == 0) KF_TRACE(kTrMmaK0);
#pragma unroll
                        for (int t = 0; t < 2; ++t) {
                            const uint32_t tS = tmem + t * BC;
                            const uint32_t tO = tmem + NQ * BC + t * D;
                            if (j > 0) {
                                const uint32_t v_lo = kv_lo + (vpos[t] % NSLOT) * (C::KV_BYTES >> 4) +
                                                      umma_desc_lbo(BC * SWB);
                                const uint32_t ppar = (steps[t] + j - 1) & 1;
#pragma unroll
                                for (int hf = 0; hf < 2; ++hf) {
                                    if (!mbar_wait_bounded(hf == 0 ? &p_half[t] : &p_full[t], ppar, abort_flag,
                                                           p.timeout_ns)) {
                                        atomicOr(&g_kf_dev_error, KF_DEVERR_TIMEOUT_SOFTMAX); ok = false; break;
                                    }
                                    tc_fence_after();
#pragma unroll
                                    for (int kk = hf * BC / 32; kk < (hf + 1) * BC / 32; ++kk)
                                        umma_ts(tO, tS + kk * 8,
                                                umma_desc_join(v_lo + ((kk * 16 * SWB) >> 4), DESC_HI), idesc_pv,
                                                (j > 1 || kk > 0) ? 1u : 0u);
                                }
                                if (!ok) break;
                                if (j == n_kv) umma_commit(&o_full[t]);
                                umma_commit(&kv_empty[vpos[t] % NSLOT]);
                            }
                            if (j < n_kv) {
                                const uint32_t k_lo = kv_lo + (kpos[t] % NSLOT) * (C::KV_BYTES >> 4) + umma_desc_lbo(16);
#pragma unroll
                                for (int kk = 0; kk < D / 16; ++kk) {
                                    const int span = (kk * 16) / SWE;
                                    const int off = ((kk * 16) % SWE) * 2;
                                    umma_ss(tS, umma_desc_join(q_lo + ((span * BM * SWB + off) >> 4), DESC_HI),
                                            umma_desc_join(k_lo + ((span * BC * SWB + off) >> 4), DESC_HI), idesc_qk,
                                            kk > 0 ? 1u : 0u);
                                }
                                umma_commit(&s_full[t]);
                                umma_commit(&kv_empty[kpos[t] % NSLOT]);
                            }
                        }
                        if (!ok) break;
                        if (j == n_kv - 1) umma_commit(q_empty);      // Q is free once these QKs complete
                    }
                    ring += 4 * n_kv;
                } else {
                const int n_kv0 = it.n_kv0;        // tile 0's steps (<= n_kv; causal only fewer)
                for (int j = 0; j <= n_kv && ok; ++j) {
                    // V_{j-1} sits at ring position 2j - 1 of the item, just before K_j.
                    int slotV = slotK - 1, parV = parK;
                    if (slotV < 0) { slotV += NSLOT; --parV; }
                    const bool k_ready = j == n_kv || mbar_test_wait(&kv_full[slotK], parK & 1);
                    const bool v_ready = j == 0 || mbar_test_wait(&kv_full[slotV], parV & 1);
                    if (!k_ready && !mbar_wait_bounded(&kv_full[slotK], parK & 1, abort_flag, p.timeout_ns)) {
                        atomicOr(&g_kf_dev_error, KF_DEVERR_TIMEOUT_TMA); ok = false; break;
                    }
                    if (!v_ready && !mbar_wait_bounded(&kv_full[slotV], parV & 1, abort_flag, p.timeout_ns)) {
                        atomicOr(&g_kf_dev_error, KF_DEVERR_TIMEOUT_TMA); ok = false; break;
                    }
                    tc_fence_after();
                    const uint32_t k_lo = kv_lo + slotK * (C::KV_BYTES >> 4) + umma_desc_lbo(16);
                    const uint32_t v_lo = kv_lo + slotV * (C::KV_BYTES >> 4) + umma_desc_lbo(BC * SWB);
#pragma unroll
                    for (int t = 0; t < NQ; ++t) {
                        if (t >= nq_active) break;
                        const uint32_t tS = tmem + t * BC;
                        const uint32_t tO = tmem + NQ * BC + t * D;
                        const int n_t = (CAUSAL && t == 0) ? n_kv0 : n_kv;
                        if (j > 0 && j <= n_t) {
                            // P_t arrives in two halves (keys [0, BC/2) then [BC/2, BC)): the
                            // first half of the PV MMAs runs while the softmax finishes the rest.
                            // Every softmax thread arrives on p_half before p_full, so a
                            // completed p_full implies p_half.  The first PV of an item also
                            // follows its softmax warpgroup's previous epilogue (which read O_t).
                            const uint32_t ppar = (steps[t] + j - 1) & 1;
                            const bool full_ready = mbar_test_wait(&p_full[t], ppar);
#pragma unroll
                            for (int hf = 0; hf < 2; ++hf) {
                                if (!full_ready) {
                                    if (!mbar_wait_bounded(hf == 0 ? &p_half[t] : &p_full[t], ppar, abort_flag,
                                                           p.timeout_ns)) {
                                        atomicOr(&g_kf_dev_error, KF_DEVERR_TIMEOUT_SOFTMAX); ok = false; break;
                                    }
                                }
                                if (hf == 0 || !full_ready) tc_fence_after();
#pragma unroll
                                for (int kk = hf * BC / 32; kk < (hf + 1) * BC / 32; ++kk) {
                                    // A = P_t in TMEM (fp16 pairs over the first BC/2 columns of S_t);
                                    // B = V: MN-major spans of SWE columns, 8-row groups of SWB bytes.
                                    umma_ts(tO, tS + kk * 8, umma_desc_join(v_lo + ((kk * 16 * SWB) >> 4), DESC_HI),
                                            idesc_pv, (j > 1 || kk > 0) ? 1u : 0u);
                                }
                            }
                            if (!ok) break;
                            if (j == n_t) umma_commit(&o_full[t]);
                            // V_{j-1} is free once the last tile's PV has read it (before QK_B(j));
                            // the last tile has all n_kv steps.
                            if (t == nq_active - 1) umma_commit(&kv_empty[slotV]);
                        }
                        if (j < n_t) {
                            const uint32_t a_lo = q_lo + t * (C::Q_BYTES >> 4);
#pragma unroll
                            for (int kk = 0; kk < D / 16; ++kk) {
                                // K-major, 128-B (or 32-B) swizzle: span s of SWE columns, +32 B per 16 columns.
                                const int span = (kk * 16) / SWE;
                                const int off = ((kk * 16) % SWE) * 2;
                                umma_ss(tS, umma_desc_join(a_lo + ((span * BM * SWB + off) >> 4), DESC_HI),
                                        umma_desc_join(k_lo + ((span * BC * SWB + off) >> 4), DESC_HI), idesc_qk,
                                        kk > 0 ? 1u : 0u);
                            }
                            umma_commit(&s_full[t]);
                        }
                    }
                    if (!ok) break;
                    if (j == n_kv - 1) umma_commit(q_empty);      // Q is free once these QKs complete
                    if (j < n_kv) {
                        umma_commit(&kv_empty[slotK]);
                        slotK += 2;                  // K_{j+1} at 2j + 2
                        if (slotK >= NSLOT) { slotK -= NSLOT; ++parK; }
                    }
                }
                }
#pragma unroll
                for (int t = 0; t < NQ; ++t)
                    if (t < nq_active) steps[t] += (t == 0) ? it.n_kv0 : n_kv;
            }
            // Every MMA issued above must complete before TMEM is released.
            umma_commit(mma_done);
            mbar_wait_drain(mma_done, 0, p.timeout_ns);
        }
    } else if (warp < 4) {
        if constexpr (C::REBALANCE) setmaxnreg_dec<C::REG_CTRL>();   // idle warps of the control group
    } else {
        // ------------------------------------------------------------ softmax warpgroups
        if constexpr (C::REBALANCE) setmaxnreg_inc<C::REG_SOFTMAX>();
        const int t = (warp - 4) >> 2;
        const int wq = warp & 3;                 // TMEM sub-partition of this warp
        const int row = wq * 32 + lane;          // query row within the tile
        const uint32_t tl = tmem_base() + (static_cast<uint32_t>(wq * 32) << 16);
        const uint32_t tS = tl + t * BC;
        const uint32_t tO = tl + NQ * BC + t * D;
        const float c = p.scale_log2;
        int pos = 0;                             // ring position of the item's K_0
        int sst = 0, o_cnt = 0;                  // this tile's KV steps and o_full completions
        bool ok = true;
        for (int rnd = 0; rnd * static_cast<int>(gridDim.x) < p.n_items && ok; ++rnd) {
            const int item = prefill_item_index(rnd);
            if (item >= p.n_items) continue;
            int n_kv, kt0, diag;
            {
                const PrefillItem it = prefill_item<D, CAUSAL, SPLIT, KVH>(p, item);
                n_kv = t == 0 ? it.n_kv0 : it.n_kv;         // this tile's KV steps
                kt0 = it.kt0 + (KVH ? t * it.n_kv : 0);     // KVH: this tile's half of the keys
                pos += (KVH ? 4 : 2) * it.n_kv;
                if (t >= it.nq_active) continue;
                // Causal: keys of tile j visible to this row are those below diag - j*BC.
                diag = CAUSAL ? it.q_row0 + t * BM + row + p.kv_off - kt0 * BC + 1 : 0;
            }
            float m_ref = -CUDART_INF_F, m_true = -CUDART_INF_F, l = 0.f;
            for (int j = 0; j < n_kv; ++j) {
                ok = mbar_wait_bounded(&s_full[t], (sst + j) & 1, abort_flag, p.timeout_ns);
                ok = __all_sync(0xffffffffu, ok);
                if (!ok) { atomicOr(&g_kf_dev_error, KF_DEVERR_TIMEOUT_MMA); break; }
                if (j == 0 && row == 0) KF_TRACE(kTrFirstS0 + t);
                tc_fence_after();
                uint32_t sr[BC];
#pragma unroll
                for (int cc = 0; cc < BC / 32; ++cc)
                    tmem_ld32(tS + cc * 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[cc * 32]));
                tmem_wait_ld();
                // Keys of this tile visible to this row: past S_kv (ragged end) and, with
                // the causal mask, past the row's diagonal read as -inf.
                int kv_valid = p.S_kv - (kt0 + j) * BC;
                if constexpr (CAUSAL) kv_valid = min(kv_valid, diag - j * BC);
                auto mask_s = [&]() {
                    if (kv_valid < BC) {
#pragma unroll
                        for (int cc = 0; cc < BC; ++cc)
                            if (cc >= kv_valid) sr[cc] = __float_as_uint(-CUDART_INF_F);
                    }
                };
                mask_s();
#define KF_S(i) __uint_as_float(sr[i])
                // Row max: three-input max, four independent chains.
                float mx0 = KF_S(0), mx1 = KF_S(1), mx2 = KF_S(2), mx3 = KF_S(3);
#pragma unroll
                for (int cc = 4; cc + 8 <= BC; cc += 8) {
                    mx0 = fmax3f(mx0, KF_S(cc), KF_S(cc + 1));
                    mx1 = fmax3f(mx1, KF_S(cc + 2), KF_S(cc + 3));
                    mx2 = fmax3f(mx2, KF_S(cc + 4), KF_S(cc + 5));
                    mx3 = fmax3f(mx3, KF_S(cc + 6), KF_S(cc + 7));
                }
                mx0 = fmax3f(mx0, KF_S(BC - 4), KF_S(BC - 3));
                mx1 = fmax3f(mx1, KF_S(BC - 2), KF_S(BC - 1));
                const float m_new = fmax3f(m_true, fmaxf(mx0, mx1), fmaxf(mx2, mx3));
                m_true = m_new;
                // P = 2^(s*c - m_ref*c): paired FMA, MUFU ex2, paired row-sum adds;
                // packed to fp16 pairs in place (pair i/2 overwrites scores already
                // read) and written over the first BC/2 TMEM columns of S_t (this
                // thread's row), the A operand of the PV MMA.  Each half of the keys
                // is published on its own barrier (p_half, then p_full).
                constexpr int HALF = BC / 2;
                float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
                auto exps = [&](auto lo_c, auto hi_c) {
                    constexpr int LO = decltype(lo_c)::value, HI = decltype(hi_c)::value;
                    const float2 c2 = make_float2(c, c);
                    const float2 neg2 = make_float2(-m_ref * c, -m_ref * c);
#pragma unroll
                    for (int i = LO; i < HI; i += 4) {
                        const float2 x0 = ffma2(make_float2(KF_S(i), KF_S(i + 1)), c2, neg2);
                        const float2 x1 = ffma2(make_float2(KF_S(i + 2), KF_S(i + 3)), c2, neg2);
                        // D = 64: one pair in eight on the FMA pipe (ex2_fma2), the rest on
                        // MUFU (measured: C4 +1.8 %; at D = 128 it costs 5 %).
                        constexpr int EMU = D == 64 ? 1 : 0;
                        const float2 e0 = ((i / 2) % 8) < EMU ? ex2_fma2(x0)
                                                               : make_float2(ex2_approx(x0.x), ex2_approx(x0.y));
                        const float2 e1 = ((i / 2 + 1) % 8) < EMU ? ex2_fma2(x1)
                                                                   : make_float2(ex2_approx(x1.x), ex2_approx(x1.y));
                        acc0 = fadd2(acc0, e0);
                        acc1 = fadd2(acc1, e1);
                        sr[i / 2] = pack_half2(e0.x, e0.y);
                        sr[i / 2 + 1] = pack_half2(e1.x, e1.y);
                    }
                };
                using Int0 = std::integral_constant<int, 0>;
                using IntH = std::integral_constant<int, HALF>;
                using IntB = std::integral_constant<int, BC>;
                // Lazy rescale: keep the reference max unless the row max grew by
                // more than 2^8 (P <= 256 stays exact enough in fp16, l and O in fp32).
                // After the first step the first half's exps start from the current
                // reference max while the row max is formed (no data dependence
                // between them); if the check then asks for a rescale (rare), the
                // scores are reloaded from TMEM and that half is redone.
                if (j == 0) {
                    m_ref = m_new;
                    exps(Int0{}, IntH{});
                } else {
                    exps(Int0{}, IntH{});
                    const bool need = (m_new - m_ref) * c > 8.0f;
                    if (__any_sync(0xffffffffu, need)) {
                        float f = 1.0f;
                        if (need) {
                            f = ex2_approx((m_ref - m_new) * c);
                            m_ref = m_new;
                            l *= f;
                        }
                        // O_t is stable here: PV_t(j-1) completed before S_t(j) was committed.
#pragma unroll
                        for (int dc = 0; dc < D / RCH; ++dc) {
                            uint32_t o[RCH];
                            tmem_ld_chunk<RCH>(tO + dc * RCH, o);
                            tmem_wait_ld();
#pragma unroll
                            for (int k = 0; k < RCH; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) * f);
                            tmem_st_chunk<RCH>(tO + dc * RCH, o);
                        }
#pragma unroll
                        for (int cc = 0; cc < HALF / 32; ++cc)
                            tmem_ld32(tS + cc * 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[cc * 32]));
                        tmem_wait_ld();
                        mask_s();
                        acc0 = make_float2(0.f, 0.f);
                        acc1 = make_float2(0.f, 0.f);
                        exps(Int0{}, IntH{});
                    }
                }
                tmem_st_chunk<HALF / 2>(tS, *reinterpret_cast<const uint32_t(*)[HALF / 2]>(&sr[0]));
                tmem_wait_st();          // first half of P (and any rescaled O) written before the MMA reads it
                tc_fence_before();
                mbar_arrive(&p_half[t]);
                exps(IntH{}, IntB{});
                tmem_st_chunk<HALF / 2>(tS + HALF / 2,
                                        *reinterpret_cast<const uint32_t(*)[HALF / 2]>(&sr[HALF / 2]));
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(&p_full[t]);
#undef KF_S
                l += (acc0.x + acc0.y) + (acc1.x + acc1.y);
            }
            sst += n_kv;
            if (ok) {
                ok = mbar_wait_bounded(&o_full[t], o_cnt & 1, abort_flag, p.timeout_ns);
                ok = __all_sync(0xffffffffu, ok);
                if (!ok) atomicOr(&g_kf_dev_error, KF_DEVERR_TIMEOUT_MMA);
            }
            ++o_cnt;
            if (row == 0) KF_TRACE(kTrOFull0 + t);
            // Rebase to the true row max: O_t * f and l * f are relative to m_true.
            float f = ex2_approx((m_ref - m_true) * c);
            float l_true = l * f;
            // The item's fields for the epilogue, recomputed from its index (an opaque
            // copy, so the compiler does not keep them in registers across the KV loop).
            int item_e;
            asm volatile("mov.b32 %0, %1;" : "=r"(item_e) : "r"(item));
            const PrefillItem ie = prefill_item<D, CAUSAL, SPLIT, KVH>(p, item_e);
            const int q_row0 = ie.q_row0, b = ie.b, h = ie.h, unit = ie.unit, chunk = ie.chunk;
            const bool split = ie.split;
            // Staging slot of this tile: the ring slot of the item's last K (tile 0) or
            // last V (tile 1); every MMA reading it completed before o_full[t] fired.  KVH:
            // the slots of the last first-half K and second-half K (stage2), for tile 0 (the
            // one that stores): both were last read by QKs issued before tile 0's last P.V.
            // The split owner's merge stages in the first only (the second in both staged
            // stores spilled), and releases both.
            // (Causal: tile 0 stages in the slot of its own last K, whose QKs were issued before
            // its o_full; the item's later loads stay within the ring depth of it.)
            uint8_t* stage = sKV + ((KVH ? pos - 4 : t == 0 ? pos - 2 - 2 * (ie.n_kv - ie.n_kv0) : pos - 1) % NSLOT) *
                                   C::KV_BYTES;
            // (Formed where it is used, from pos: a pointer held across the merge spills.)
            auto stage2 = [&]() -> uint8_t* { return KVH ? sKV + ((pos - 3) % NSLOT) * C::KV_BYTES : nullptr; };
            const int qrow = q_row0 + (KVH ? 0 : t * BM) + row;
            const bool store = qrow < p.S_q;
            const size_t orow = ((static_cast<size_t>(b) * p.H_q + h) * p.S_q + (store ? qrow : 0)) * D;   // element index
            const size_t mi = (static_cast<size_t>(b) * p.H_q + h) * p.S_q + (store ? qrow : 0);
            if constexpr (KVH) {
                // Key halves of one query tile: tile 1 hands its row's (m_ref, m_true, l) to
                // tile 0 through the idle second Q buffer; tile 0 merges tile 1's O straight
                // from TMEM (same lanes, tile 1's columns) into its staged store.  A second
                // barrier keeps tile 1 from starting its next item (whose P.V overwrites its
                // O) before tile 0 has read that O.
                // Both barriers are reductions of ok over the two tiles, so the tiles leave
                // the item loop together after an abort (neither is left at a barrier).
                // (Addressed from sKV, which this role already holds: sQ + Q_BYTES == sKV - Q_BYTES.)
                float4* xch = reinterpret_cast<float4*>(sKV - C::Q_BYTES);
                if (t == 1) {
                    xch[row] = make_float4(m_ref, m_true, l, 0.f);
                    tc_fence_before();
                }
                ok = named_bar_and(4, 256, ok);
                if (row == 0 && t == 0) KF_TRACE(kTrHalvesMet);
                if (t == 0) {
                    tc_fence_after();
                    const float4 ob = xch[row];
                    if (ok) {
                        const float M = fmaxf(m_true, ob.y);
                        const float wa = ex2_approx((m_ref - M) * c), wb = ex2_approx((ob.x - M) * c);
                        const float L = wa * l + wb * ob.z;
                        const float osc = (p.flags & KF_PF_UNNORMALIZED) ? 1.0f : 1.0f / L;
                        // O_0 = wa * O_0 + wb * O_1 in TMEM (tile 1's O: same lanes, its columns).
                        const uint32_t tO1 = tl + NQ * BC + D;
#pragma unroll 1
                        for (int dc = 0; dc < D / RCH; ++dc) {
                            uint32_t oa[RCH], ob1[RCH];
                            tmem_ld_chunk<RCH>(tO + dc * RCH, oa);
                            tmem_ld_chunk<RCH>(tO1 + dc * RCH, ob1);
                            tmem_wait_ld();
#pragma unroll
                            for (int k2 = 0; k2 < RCH; ++k2)
                                oa[k2] = __float_as_uint(wa * __uint_as_float(oa[k2]) + wb * __uint_as_float(ob1[k2]));
                            tmem_st_chunk<RCH>(tO + dc * RCH, oa);
                        }
                        tmem_wait_st();
                        if (row == 0) KF_TRACE(kTrHalvesMerged);
                        if (split) {
                            // A split chunk: the merged tile goes on to the split epilogue below
                            // as this chunk's tile 0 (O relative to M, sum L).
                            m_ref = M;
                            m_true = M;
                            l = L;
                            f = 1.0f;
                            l_true = L;
                        } else if constexpr (C::TMA_STORE) {
                            stage_store_tile<D, BM, C::KV_BYTES>(stage, tO, row, 2, osc, p.out_type, &tmO, q_row0,
                                                                b * p.H_q + h, DonorRows{}, stage2());
                            if (row == 0) {
                                mbar_arrive(&stage_free[0]);
                                mbar_arrive(&stage_free[1]);
                            }
                        } else {
#pragma unroll
                            for (int dc = 0; dc < D / OCH; ++dc) {
                                uint32_t o[OCH];
                                tmem_ld_chunk<OCH>(tO + dc * OCH, o);
                                tmem_wait_ld();
                                if (store) {
#pragma unroll
                                    for (int k2 = 0; k2 < OCH; k2 += 4)
                                        store_out4(p.O, orow + dc * OCH + k2,
                                                   make_float4(__uint_as_float(o[k2]) * osc, __uint_as_float(o[k2 + 1]) * osc,
                                                               __uint_as_float(o[k2 + 2]) * osc,
                                                               __uint_as_float(o[k2 + 3]) * osc),
                                                   p.out_type);
                                }
                            }
                        }
                        if (store && !split) {
                            if (p.Mi) p.Mi[mi] = M * p.scale;
                            if (p.Li) p.Li[mi] = L;
                        }
                    }
                    tc_fence_before();
                }
                ok = named_bar_and(4, 256, ok);
            }
            if ((!KVH || t == 0) && split) {
                // KV chunk of a split unit.  Tile t of the unit is owned by chunk t: the
                // other chunks write their partial (O_u, m, l) of tile t, relative to their
                // own max, and add 1 to the tile's counter; the owner waits (within a short
                // limit) for the k-1 partials and merges them with its own O straight from
                // TMEM.  If that wait runs out (chunks not running at the same time), the
                // owner writes its partial too and adds 1: the add that makes the count k
                // (owner or last donor) merges the tile from the k partials.
                // Partials: O_u as float4 columns [split unit][chunk][D/4][ROWS] (lane =
                // row, so every warp access is 512 contiguous bytes), then (m, l) as float2
                // [split unit][chunk][ROWS].
                const int su = unit - p.n_plain;
                constexpr int ROWS = NQ * BM;
                const int k = p.split_k;
                const size_t n_slots = static_cast<size_t>(p.n_units - p.n_plain) * k * ROWS;
                float4* part4 = reinterpret_cast<float4*>(p.part);
                float2* part_ml = reinterpret_cast<float2*>(p.part + n_slots * D);
                const int r_u = t * BM + row;                             // row within the unit
                auto o_part = [&](int ch, int q) -> float4* {             // float4 q of row r_u, chunk ch
                    return part4 + ((static_cast<size_t>(su) * k + ch) * (D / 4) + q) * ROWS + r_u;
                };
                auto ml_part = [&](int ch) -> float2* {
                    return part_ml + (static_cast<size_t>(su) * k + ch) * ROWS + r_u;
                };
                unsigned* counter = &p.counters[su * NQ + t];
                volatile int* flag = ticket_last + t;
                const bool owner = chunk == t;
                if constexpr (C::TMA_STORE) ok = named_bar_and(2 + t, 128, ok);
                bool owner_merge = false;
                if (owner && !(p.flags & KF_PF_TICKET_MERGE)) {
                    if (row == 0) {
                        const unsigned want = static_cast<unsigned>(k - 1);
                        const uint64_t lim = p.timeout_ns < kOwnerWaitNs ? p.timeout_ns : kOwnerWaitNs;
                        const uint64_t t0 = global_timer_ns();
                        int got = 0;
                        for (unsigned spins = 0; !*abort_flag; ++spins) {
                            if (ld_acquire_gpu(counter) >= want) { got = 1; break; }
                            if ((spins & 15u) == 15u && global_timer_ns() - t0 > lim) break;
                            __nanosleep(32);
                        }
                        if (got) *counter = 0u;          // every donor has added: zero for the next call
                        *flag = got;
                        KF_TRACE(kTrOwnerWaited);
                    }
                    named_bar_sync(2 + t, 128);
                    owner_merge = *flag != 0;
                    named_bar_sync(2 + t, 128);          // flag read before it is reused
                }
                if (owner_merge) {
                    __threadfence();
                    if (ok) {
                        tc_fence_after();
                        DonorRows don;
                        don.n = k - 1;
                        float md[3], ld[3];
                        float M = m_true;
#pragma unroll
                        for (int d = 0; d < 3; ++d) {
                            const int ch = d < t ? d : d + 1;            // the chunks other than t
                            const float2 ml = d < don.n ? __ldcg(ml_part(ch)) : make_float2(-CUDART_INF_F, 0.f);
                            md[d] = ml.x;
                            ld[d] = ml.y;
                            M = fmaxf(M, ml.x);
                        }
                        const float w_own = ex2_approx((m_true - M) * c);
                        float L = w_own * l_true;
#pragma unroll
                        for (int d = 0; d < 3; ++d) {
                            don.w[d] = d < don.n ? ex2_approx((md[d] - M) * c) : 0.f;
                            L += don.w[d] * ld[d];
                        }
                        const float osc = (p.flags & KF_PF_UNNORMALIZED) ? 1.0f : 1.0f / L;
                        auto store_ml = [&]() {
                            if (store) {
                                if (p.Mi) p.Mi[mi] = M * p.scale;
                                if (p.Li) p.Li[mi] = L;
                            }
                        };
                        // Key-half units write the row's (M, L) before the O store: kept live
                        // across it, the row's index spilled in that instance.
                        if constexpr (KVH) store_ml();
#pragma unroll
                        for (int d = 0; d < 3; ++d) {
                            don.w[d] *= osc;
                            don.col[d] = o_part(d < t ? d : d + 1, 0);
                        }
                        don.stride = ROWS;
                        if constexpr (C::TMA_STORE) {
                            stage_store_tile<D, BM, C::KV_BYTES>(stage, tO, row, 2 + t, f * w_own * osc, p.out_type,
                                                                &tmO, q_row0 + t * BM, b * p.H_q + h, don);
                            if (row == 0) {
                                mbar_arrive(&stage_free[t]);
                                if constexpr (KVH) mbar_arrive(&stage_free[1]);
                            }
                        } else {
                            const float so = f * w_own * osc;
#pragma unroll
                            for (int dc = 0; dc < D / OCH; ++dc) {
                                uint32_t o[OCH];
                                tmem_ld_chunk<OCH>(tO + dc * OCH, o);
                                tmem_wait_ld();
#pragma unroll
                                for (int kk = 0; kk < OCH; kk += 4) {
                                    float4 v = make_float4(__uint_as_float(o[kk]) * so, __uint_as_float(o[kk + 1]) * so,
                                                           __uint_as_float(o[kk + 2]) * so, __uint_as_float(o[kk + 3]) * so);
#pragma unroll
                                    for (int d = 0; d < 3; ++d) {
                                        if (d < don.n) {
                                            const float4 u = __ldcg(don.col[d] + static_cast<size_t>((dc * OCH + kk) / 4) * ROWS);
                                            v.x += don.w[d] * u.x; v.y += don.w[d] * u.y;
                                            v.z += don.w[d] * u.z; v.w += don.w[d] * u.w;
                                        }
                                    }
                                    if (store) store_out4(p.O, orow + dc * OCH + kk, v, p.out_type);
                                }
                            }
                        }
                        if constexpr (!KVH) store_ml();
                    }
                } else {
                    // Donor (or an owner past its wait): this tile's partial, then a ticket.
                    if (ok) {
                        tc_fence_after();
#pragma unroll
                        for (int dc = 0; dc < D / OCH; ++dc) {
                            uint32_t o[OCH];
                            tmem_ld_chunk<OCH>(tO + dc * OCH, o);
                            tmem_wait_ld();
#pragma unroll
                            for (int kk = 0; kk < OCH; kk += 4)
                                *o_part(chunk, (dc * OCH + kk) / 4) =
                                    make_float4(__uint_as_float(o[kk]) * f, __uint_as_float(o[kk + 1]) * f,
                                                __uint_as_float(o[kk + 2]) * f, __uint_as_float(o[kk + 3]) * f);
                        }
                        *ml_part(chunk) = make_float2(m_true, l_true);
                        if (row == 0) KF_TRACE(kTrPartialWritten);
                        if constexpr (C::TMA_STORE) {
                            if (row == 0) {                    // the staging slots were not used
                                mbar_arrive(&stage_free[t]);
                                if constexpr (KVH) mbar_arrive(&stage_free[1]);
                            }
                        }
                    }
                    __threadfence();
                    named_bar_sync(2 + t, 128);          // every thread of the tile, ok or not
                    if (row == 0) {
                        int last = 0;
                        if (!*abort_flag) last = atomicAdd(counter, 1u) == static_cast<unsigned>(k - 1);
                        *flag = last;
                        KF_TRACE(kTrTicket);
                    }
                    named_bar_sync(2 + t, 128);
                    const bool last = *flag != 0;
                    named_bar_sync(2 + t, 128);          // flag read before it is reused
                    if (last) {
                        // Merge the tile from the k partials: lane = row, every access coalesced.
                        __threadfence();
                        float2 ml[4];
                        float M = -CUDART_INF_F;
#pragma unroll
                        for (int ch = 0; ch < 4; ++ch) {
                            ml[ch] = ch < k ? __ldcg(ml_part(ch)) : make_float2(-CUDART_INF_F, 0.f);
                            M = fmaxf(M, ml[ch].x);
                        }
                        float w[4], L = 0.f;
#pragma unroll
                        for (int ch = 0; ch < 4; ++ch) {
                            w[ch] = ch < k ? ex2_approx((ml[ch].x - M) * c) : 0.f;
                            L += w[ch] * ml[ch].y;
                        }
                        const float osc = (p.flags & KF_PF_UNNORMALIZED) ? 1.0f : 1.0f / L;
#pragma unroll
                        for (int ch = 0; ch < 4; ++ch) w[ch] *= osc;
#pragma unroll 1
                        for (int q = 0; q < D / 4; ++q) {
                            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                            for (int ch = 0; ch < 4; ++ch) {
                                if (ch < k) {
                                    const float4 u = __ldcg(o_part(ch, q));
                                    v.x += w[ch] * u.x; v.y += w[ch] * u.y; v.z += w[ch] * u.z; v.w += w[ch] * u.w;
                                }
                            }
                            if (store) store_out4(p.O, orow + q * 4, v, p.out_type);
                        }
                        if (store) {
                            if (p.Mi) p.Mi[mi] = M * p.scale;
                            if (p.Li) p.Li[mi] = L;
                        }
                        if (row == 0) *counter = 0u;
                    }
                }
            } else if (!KVH) {
                // Every thread of the tile reaches this barrier, ok or not, so the staged
                // epilogue below (which synchronizes the tile's threads) runs for all or none.
                if constexpr (C::TMA_STORE) ok = named_bar_and(2 + t, 128, ok);
                if (ok) {
                    tc_fence_after();
                    const float osc = (p.flags & KF_PF_UNNORMALIZED) ? f : 1.0f / l;
                    if constexpr (C::TMA_STORE) {
                        stage_store_tile<D, BM, C::KV_BYTES>(stage, tO, row, 2 + t, osc, p.out_type, &tmO,
                                                            q_row0 + t * BM, b * p.H_q + h);
                        if (row == 0) mbar_arrive(&stage_free[t]);
                    } else {
#pragma unroll
                        for (int dc = 0; dc < D / OCH; ++dc) {
                            uint32_t o[OCH];
                            tmem_ld_chunk<OCH>(tO + dc * OCH, o);
                            tmem_wait_ld();
                            if (store) {
#pragma unroll
                                for (int k = 0; k < OCH; k += 4) {
                                    float4 v = make_float4(__uint_as_float(o[k]) * osc, __uint_as_float(o[k + 1]) * osc,
                                                           __uint_as_float(o[k + 2]) * osc, __uint_as_float(o[k + 3]) * osc);
                                    store_out4(p.O, orow + dc * OCH + k, v, p.out_type);
                                }
                            }
                        }
                    }
                    if (store) {
                        if (p.Mi) p.Mi[mi] = m_true * p.scale;
                        if (p.Li) p.Li[mi] = l_true;
                    }
                }
            }
            if (row == 0) KF_TRACE(kTrItemEnd0 + t);
            tc_fence_before();
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) KF_TRACE(kTrExit);
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base(), C::TMEM_COLS);
    }
}

}  // namespace kf
