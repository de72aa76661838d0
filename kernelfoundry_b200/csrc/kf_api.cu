// kf_api.cu -- the C ABI (include/kf_attn.h) over the sm_100a kernels.
//
// One translation unit: the kernels are included here so device code can
// name the library's device error word directly.  Host side: argument
// validation, the execution plan (tcgen05 prefill kernel vs. split-KV decode
// kernel, split count from the SM count and occupancy), TMA tensor-map
// encoding through the driver entry point (the library links the static
// CUDA runtime only, so it loads on machines without a GPU driver), launches.
#include <cudaTypedefs.h>

#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "../../include/kf_attn.h"
#include "../../include/kf_pointwise.h"
#include "../../include/kf_synth.h"
#include "decode_sm100.cuh"
#include "peer_sm100.cuh"
#include "kf_ptx.cuh"
#include "pointwise_sm100.cuh"
#include "prefill_sm100.cuh"
#include "synth_sm100.cuh"

namespace kf {

// Waits on a barrier that nothing signals; the bounded wait must expire.
__global__ void selftest_wait_kernel(unsigned long long timeout_ns) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        if (!mbar_wait_bounded(&bar, 0, &abort_flag, timeout_ns)) atomicOr(&g_kf_dev_error, KF_DEVERR_TIMEOUT_SELFTEST);
    }
}

}  // namespace kf

namespace {

constexpr unsigned long long kDefaultTimeoutNs = 1000000000ull;   // 1 s
std::atomic<unsigned long long> g_timeout_ns{kDefaultTimeoutNs};
thread_local int t_last_cuda_error = 0;

constexpr int kMaxDevices = 64;
constexpr int kCounterSlots = 16384;          // split-KV ticket counters at the workspace head
constexpr size_t kCounterBytes = kCounterSlots * sizeof(unsigned);

int cuda_fail(cudaError_t e) {
    t_last_cuda_error = static_cast<int>(e);
    return KF_ERR_CUDA;
}

struct DeviceInfo {
    bool ready = false;
    int sm_count = 0;
    int cc_major = 0, cc_minor = 0;
};
DeviceInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;

int device_info(DeviceInfo** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e);
    if (dev < 0 || dev >= kMaxDevices) return KF_ERR_UNSUPPORTED_DEVICE;
    DeviceInfo& di = g_dev[dev];
    if (!di.ready) {
        std::lock_guard<std::mutex> lk(g_dev_mu);
        if (!di.ready) {
            if ((e = cudaDeviceGetAttribute(&di.sm_count, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return cuda_fail(e);
            if ((e = cudaDeviceGetAttribute(&di.cc_major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess) return cuda_fail(e);
            if ((e = cudaDeviceGetAttribute(&di.cc_minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess) return cuda_fail(e);
            di.ready = true;
        }
    }
    if (di.cc_major != 10 || di.cc_minor != 0) return KF_ERR_UNSUPPORTED_DEVICE;
    *out = &di;
    return KF_OK;
}

// Sets the dynamic shared-memory opt-in of a kernel once per device and
// returns how many of its CTAs fit on one SM.
// Keyed by the kernel itself (a template argument): every instantiation has
// its own cache slot even though they share one function type.
template <auto Kern>
int kernel_setup(int smem_bytes, int threads, int* blocks_per_sm) {
    constexpr auto kern = Kern;
    struct Slot { std::atomic<int> bps{0}; };
    static Slot slots[kMaxDevices];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e);
    int v = slots[dev].bps.load(std::memory_order_acquire);
    if (v == 0) {
        if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes)) != cudaSuccess)
            return cuda_fail(e);
        int n = 0;
        if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, threads, smem_bytes)) != cudaSuccess)
            return cuda_fail(e);
        v = n > 0 ? n : 1;
        slots[dev].bps.store(v, std::memory_order_release);
    }
    *blocks_per_sm = v;
    return KF_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 3-D map over a [BH][S][D] 16-bit tensor (fp16 unless bf16); boxes of (swizzle span) x box_rows x 1.
int make_map(CUtensorMap* map, const void* base, int D, int S, long long BH, int box_rows, int swb,
             bool bf16 = false) {
    auto enc = encode_fn();
    if (!enc) return cuda_fail(cudaErrorNotSupported);
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(S), static_cast<cuuint64_t>(BH)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * 2, static_cast<cuuint64_t>(S) * D * 2};
    cuuint32_t box[3] = {static_cast<cuuint32_t>(swb / 2), static_cast<cuuint32_t>(box_rows), 1};
    cuuint32_t estr[3] = {1, 1, 1};
    const CUtensorMapSwizzle sw = swb == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                : swb == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B;
    CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                     const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cuda_fail(cudaErrorInvalidValue);
    return KF_OK;
}

// 3-D map over a [BH][S][D] fp32 tensor (the output); boxes of 32 x box_rows x 1,
// 128-B swizzle (D a multiple of 32).
int make_map_f32(CUtensorMap* map, void* base, int D, int S, long long BH, int box_rows) {
    auto enc = encode_fn();
    if (!enc) return cuda_fail(cudaErrorNotSupported);
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(S), static_cast<cuuint64_t>(BH)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * 4, static_cast<cuuint64_t>(S) * D * 4};
    cuuint32_t box[3] = {32, static_cast<cuuint32_t>(box_rows), 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cuda_fail(cudaErrorInvalidValue);
    return KF_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int validate(const void* Q, const void* K, const void* V, const float* O, int B, int H_q, int H_kv, int S_q,
             int S_kv, int D) {
    if (B < 0 || S_q < 0 || H_q <= 0 || H_kv <= 0 || H_q % H_kv != 0) return KF_ERR_INVALID_ARG;
    if (!(D == 16 || D == 64 || D == 128 || D == 256)) return KF_ERR_UNSUPPORTED_HEAD_DIM;
    if (B == 0 || S_q == 0) return KF_OK;
    if (S_kv <= 0) return KF_ERR_INVALID_ARG;
    if (B > 65535 || H_q > 65535) return KF_ERR_INVALID_ARG;
    if (static_cast<long long>(B) * H_q * S_q > (1ll << 40) || static_cast<long long>(B) * H_kv > (1ll << 31))
        return KF_ERR_INVALID_ARG;
    if (!Q || !K || !V || !O) return KF_ERR_INVALID_ARG;
    if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O)) return KF_ERR_MISALIGNED;
    return KF_OK;
}

// ------------------------------------------------------------------ planning
struct Plan {
    int path = 0;        // 0 prefill, 1 decode
    int mt = 1;          // decode: 16-row MMA tiles per CTA
    int n_rg = 1;        // decode: row groups per (b, h_kv)
    int n_split = 1;     // decode: KV splits
    bool deep = false;   // decode: the deep-ring kernel (one CTA per SM, all CTAs resident)
    bool cluster = false;  // decode: a unit's splits form a thread-block cluster (merge in DSMEM)
    int chunk = 0;       // decode: KV rows per split
    size_t ws_bytes = 0; // workspace the plan uses
    long long ctas = 0;
    // prefill work list: units = B * H_q * q-blocks; the last (units - plain)
    // units (a partial last wave) are split over split_k CTAs of `per` KV tiles
    int pf_qblk = 1, pf_units = 0, pf_plain = 0, pf_k = 1, pf_per = 0;
    int pf_tiles = 2;    // prefill: 128-row query tiles per unit
    bool pf_kvh = false; // prefill, one-tile units: the CTA's two tiles take the keys' two halves
};

int decode_max_mt(int D) { return D <= 128 ? 2 : 1; }

// Decode (packed-rows) path when G * S_q rows fit in two row groups.
bool use_decode(int G, int S_q, int D) {
    const long long R = static_cast<long long>(G) * S_q;
    return R <= 2ll * 16 * decode_max_mt(D);
}

size_t split_ws_bytes(long long rows, int n_split, int D) {
    const size_t part = static_cast<size_t>(rows) * n_split * (static_cast<size_t>(D) + 2) * sizeof(float);
    return kCounterBytes + ((part + 255) / 256) * 256;
}

template <int D, int MT>
int decode_blocks_per_sm(int* bps) {
    using C = kf::DecodeCfg<D, MT>;
    return kernel_setup<kf::decode_fwd_kernel<D, MT>>(C::SMEM_BYTES, C::THREADS, bps);
}

// Cluster-merge decode: for each cluster size s (2..16) of split CTAs, how many such
// clusters of the (D, MT, DEEP) cluster-merge kernel the device can hold at once
// (cudaOccupancyMaxActiveClusters; 0: not launchable).  Cached per device.
struct ClusterCaps {
    int act[2][17];      // [deep][s]
};

template <int D, int MT, bool DEEP>
int decode_cluster_act(int* act) {      // act[0..16]
    using C = kf::DecodeCfg<D, MT, DEEP>;
    constexpr auto kern = kf::decode_fwd_kernel<D, MT, false, true, DEEP, 0, true>;
    struct Slot { std::atomic<int> ready{0}; int act[17]; };
    static Slot slots[kMaxDevices];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e);
    Slot& sl = slots[dev];
    if (!sl.ready.load(std::memory_order_acquire)) {
        if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES)) != cudaSuccess ||
            (e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1)) != cudaSuccess)
            return cuda_fail(e);
        int tmp[17] = {0};
        for (int cs = 2; cs <= C::MAX_CLUSTER; ++cs) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(static_cast<unsigned>(cs));
            cfg.blockDim = dim3(C::THREADS);
            cfg.dynamicSmemBytes = C::SMEM_BYTES;
            cudaLaunchAttribute at[1];
            at[0].id = cudaLaunchAttributeClusterDimension;
            at[0].val.clusterDim.x = static_cast<unsigned>(cs);
            at[0].val.clusterDim.y = 1;
            at[0].val.clusterDim.z = 1;
            cfg.attrs = at;
            cfg.numAttrs = 1;
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess) tmp[cs] = n;
            else cudaGetLastError();   // a size the device cannot place is not an error of the call
        }
        for (int i = 0; i < 17; ++i) sl.act[i] = tmp[i];
        sl.ready.store(1, std::memory_order_release);
    }
    for (int i = 0; i < 17; ++i) act[i] = sl.act[i];
    return KF_OK;
}

// The deep-ring kernel exists for 16-row tiles only (act[1] stays zero for MT = 2).
int decode_cluster_caps(int D, int mt, ClusterCaps* caps) {
    std::memset(caps, 0, sizeof(*caps));
#define KF_CAPS(DV, MTV)                                                               \
    {                                                                                  \
        int rc = decode_cluster_act<DV, MTV, false>(caps->act[0]);                     \
        if (rc == KF_OK && MTV == 1) rc = decode_cluster_act<DV, 1, true>(caps->act[1]); \
        return rc;                                                                     \
    }
    switch (D) {
        case 16: if (mt == 2) KF_CAPS(16, 2) KF_CAPS(16, 1)
        case 64: if (mt == 2) KF_CAPS(64, 2) KF_CAPS(64, 1)
        case 128: if (mt == 2) KF_CAPS(128, 2) KF_CAPS(128, 1)
        default: KF_CAPS(256, 1)
    }
#undef KF_CAPS
}

int decode_bps(int D, int mt, int* bps) {
    switch (D) {
        case 16: return mt == 2 ? decode_blocks_per_sm<16, 2>(bps) : decode_blocks_per_sm<16, 1>(bps);
        case 64: return mt == 2 ? decode_blocks_per_sm<64, 2>(bps) : decode_blocks_per_sm<64, 1>(bps);
        case 128: return mt == 2 ? decode_blocks_per_sm<128, 2>(bps) : decode_blocks_per_sm<128, 1>(bps);
        default: return decode_blocks_per_sm<256, 1>(bps);
    }
}

int make_plan(int B, int H_q, int H_kv, int S_q, int S_kv, int D, size_t ws_bytes, int sm_count,
              int blocks_per_sm, Plan* pl, bool causal = false, double cta_rate = 1.0, bool allow_deep = true,
              bool deep_only = false, const ClusterCaps* caps = nullptr) {
    const int G = H_q / H_kv;
    // Causal with several query rows takes the prefill kernel (the decode kernel has
    // no per-row mask); with one row the mask keeps every key, so decode is exact.
    if (!use_decode(G, S_q, D) || (causal && S_q > 1)) {
        pl->path = 0;
        const int nq = D <= 128 ? 2 : 1;
        const int bc = D <= 128 ? 128 : 64;
        // Units of one 128-row tile instead of two when the two-tile units would leave
        // over half the SMs idle, the one-tile units still fit one wave and the keys are
        // too few for a KV split (S = 512 at B = 1: 64 two-tile units on 148 SMs).
        const long long u2 = static_cast<long long>((S_q + 255) / 256) * H_q * B;
        const long long u1 = static_cast<long long>((S_q + 127) / 128) * H_q * B;
        const int n_kv_tiles = (S_kv + bc - 1) / bc;
        pl->pf_tiles = (nq == 2 && !causal && u1 > u2 && u1 <= sm_count && n_kv_tiles < 8) ? 1 : nq;
        if (const char* ov = std::getenv("KF_PREFILL_UNIT_TILES")) {       // tuning sweeps
            const int t = std::atoi(ov);
            if (t == 1 || t == nq) pl->pf_tiles = t;
        }
        // One-tile units run the tile's two key halves as the CTA's two tiles (two chains in
        // ping-pong instead of one), merged in TMEM; KF_PREFILL_KVH=0 turns it off.
        // Also S_q <= 128 (every two-tile unit would have one tile): one-tile units whose
        // two chains take the keys' halves, split along KV as below when few.
        const char* kvh = std::getenv("KF_PREFILL_KVH");
        const bool kvh_off = kvh && std::atoi(kvh) == 0;
        if (nq == 2 && !causal && S_q <= 128 && n_kv_tiles >= 4 && n_kv_tiles % 2 == 0 && !kvh_off)
            pl->pf_tiles = 1;
        pl->pf_kvh = pl->pf_tiles == 1 && nq == 2 && !causal && n_kv_tiles >= 2 && n_kv_tiles % 2 == 0 && !kvh_off;
        const int rows_per_cta = pl->pf_tiles * 128;
        pl->pf_qblk = (S_q + rows_per_cta - 1) / rows_per_cta;
        const long long units = static_cast<long long>(pl->pf_qblk) * H_q * B;
        if (units > (1ll << 31) - 1) return KF_ERR_INVALID_ARG;
        pl->pf_units = static_cast<int>(units);
        pl->pf_plain = pl->pf_units;
        // One CTA per SM: a last wave at most half full is split along KV so it
        // finishes in 1/k of a unit's time (chunk t merges tile t of the unit).
        const int cap = sm_count;
        const int rem = static_cast<int>(units % cap);
        const int n_kv = (S_kv + bc - 1) / bc;
        // Causal units differ in size; with a long cache (S_kv >= 2 S_q, chunked prefill)
        // they differ little, and each split unit's keys are divided evenly over its chunks.
        const int kv_off = S_kv - S_q;
        const bool causal_split = causal && S_kv >= 2 * S_q;
        int k = (rem > 0 && (!causal || causal_split) && (pl->pf_tiles == nq || pl->pf_kvh)) ? cap / rem : 1;
        // Causal: every row must see a key of every chunk (kv_off >= 384 (k - 1): the lightest
        // unit's last chunk starts at most 384 (k - 1) keys past its first row's diagonal).
        if (causal && k > kv_off / 384 + 1) k = kv_off / 384 + 1;
        k = k > 4 ? 4 : k;
        // Each chunk keeps >= 4 KV tiles: writing and merging the partials costs about
        // as much as 3 KV steps (measured: S = 512, 4 tiles in 2 chunks, took 21 us
        // against 16 us unsplit).
        int min_chunk = 4;
        if (const char* ov = std::getenv("KF_PREFILL_MIN_CHUNK_TILES")) {  // tuning sweeps
            const int m = std::atoi(ov);
            if (m >= 1) min_chunk = m;
        }
        // (Causal: the lightest unit's tile count, that of the first query block.)
        const int n_kv_min = causal ? ((rows_per_cta < S_q ? rows_per_cta : S_q) - 1 + kv_off) / bc + 1 : n_kv;
        k = k > n_kv_min / min_chunk ? n_kv_min / min_chunk : k;
        if (k >= 2) {
            int per = (n_kv + k - 1) / k;
            if (pl->pf_kvh) per += per & 1;         // key-half units: even chunks (n_kv is even)
            const int k_eff = causal ? k : (n_kv + per - 1) / per;   // causal: even division, k chunks
            // Partials are laid out per full unit (nq tiles of 128 rows) in the kernel.
            const size_t part = static_cast<size_t>(rem) * k_eff * (nq * 128) * (D + 2) * sizeof(float);
            const size_t need = kCounterBytes + ((part + 255) / 256) * 256;
            if (k_eff >= 2 && need <= ws_bytes) {
                pl->pf_plain = pl->pf_units - rem;
                pl->pf_k = k_eff;
                pl->pf_per = per;
                pl->ws_bytes = need;
            }
        }
        pl->ctas = pl->pf_plain + static_cast<long long>(pl->pf_units - pl->pf_plain) * pl->pf_k;
        return KF_OK;
    }
    pl->path = 1;
    const int R = G * S_q;
    const int maxmt = decode_max_mt(D);
    pl->mt = R <= 16 ? 1 : maxmt;
    const int qrows = 16 * pl->mt;
    pl->n_rg = (R + qrows - 1) / qrows;
    const long long units = static_cast<long long>(B) * H_kv * pl->n_rg;
    const int TK = 64;
    const int total_stages = (S_kv + TK - 1) / TK;
    const double cap = static_cast<double>(sm_count) * blocks_per_sm;
    // Cost model (microseconds): HBM-bound streaming of all K/V bytes, a fixed
    // start-up per CTA wave, a per-CTA rate limit (bytes a CTA keeps in flight
    // / latency), plus the split merge (one CTA per unit bulk-copies
    // n_split partials of nrows x D floats).
    // Constants fitted to a split-count sweep on B200 (KV=4096 at B=1/16/64, KV=131072 at B=1).
    // cta_rate < 1: a CTA streams slower (paged KV: one small TMA copy per page).
    // Split merge: ~3 us of round trips (partials out, ticket, partials back) measured on
    // B200 (KV=512, B=1: 8 one-stage splits 6.4 us against 3.3 us for one stage alone);
    // the 32-row kernel (MT = 2) merges far slower (MQA, KV=512: 1 split 10.5 us, 8 splits
    // 19.8 us), so its splits must buy more streaming time.
    const double kBwMerge = 200.0;   // GB/s == bytes/ns -> x1e-3 per us
    const double kT0 = 2.0, kMerge0 = pl->mt == 1 ? 3.0 : 10.0;
    // Cluster merge (splits of a unit in one thread-block cluster, partials in shared
    // memory, two cluster barriers and distributed-shared-memory loads): no workspace, and
    // measured 0.3 us below the workspace merge at 16-row tiles (B=1, KV=4096: 8.85 against
    // 9.15 us); at 32-row tiles far below it (MQA, KV=4096: 11.0 against 33.6 us).
    const double kMergeCl = 2.7;
    const double stage_bytes = 2.0 * TK * D * 2;
    const double total_bytes = static_cast<double>(units) * total_stages * stage_bytes;
    const int nrows = R < 16 * pl->mt ? R : 16 * pl->mt;
    int best_s = 1;
    bool best_deep = false, best_cl = false;
    double best_cost = 1e300;
    const int max_s = total_stages < kf::DecodeCfg<128, 1>::MAX_SPLIT ? total_stages : kf::DecodeCfg<128, 1>::MAX_SPLIT;
    const long long rows = static_cast<long long>(B) * H_q * S_q;
    // The deep-ring kernel (contiguous K/V, 16-row tiles only: one CTA per SM, two
    // consumer groups) is a candidate when every CTA of the launch is resident.
    // Measured against the one-group kernel on B200 (B=1, 16 splits): a whole launch
    // reaches ~6.6 instead of ~6.0 TB/s, for ~0.6 us more fixed cost (the groups'
    // merge, the larger ring's set-up): it wins from about 8K keys at B=1 and at B=16,
    // KV=4096.
    const char* deep_env = std::getenv("KF_DECODE_DEEP");
    const bool plan_debug = std::getenv("KF_PLAN_DEBUG") != nullptr;
    int deep_opt = (allow_deep && pl->mt == 1) ? (deep_env ? std::atoi(deep_env) : -1) : 0;
    if (deep_only) deep_opt = 1;                     // the caller rejects a plan that is not deep
    for (int deep = 0; deep < 2; ++deep) {
        if ((deep == 1 && deep_opt == 0) || (deep == 0 && deep_opt == 1)) continue;
        // Per-CTA stream rate (GB/s): one consumer group ~51, two (deep) 68 (84 measured with
        // 32 CTAs streaming, about 67 with 96).
        const double kBwCta = (deep ? 68.0 : 50.0) * cta_rate;
        const double kBwTotal = deep ? 6.6e3 : 6.0e3;
        const double cap_d = deep ? static_cast<double>(sm_count) : cap;
        for (int s = 1; s <= max_s; ++s) {
            const int nst = (total_stages + s - 1) / s;
            const int s_eff = (total_stages + nst - 1) / nst;
            if (s_eff != s) continue;
            // Cluster merge: a launchable cluster size; the deep kernel also needs every
            // cluster resident at once (its CTAs all fit on the SMs).
            const bool cl = caps && s >= 2 && s <= 16 && caps->act[deep][s] > 0 &&
                            (!deep || caps->act[1][s] >= units);
            if (s > 1 && !cl && (units > kCounterSlots || split_ws_bytes(rows, s, D) > ws_bytes)) break;
            const double ctas = static_cast<double>(units) * s;
            if (deep && ctas > cap_d) break;
            // The deep kernel pays its larger set-up only when each CTA streams at least 8
            // stages and the launch keeps at least 85 % of the SMs busy (B=1 sweep: KV=512 in
            // 8 one-stage splits 5.9 us deep against 4.6 one group; KV=131072 in 12 splits
            // 83.0 us against 81.0 in 16).
            // (A deep-only plan -- the fused exchange -- takes the deep kernel regardless.)
            if (deep && !deep_only && (nst < 8 || ctas < 0.85 * sm_count)) continue;
            const double bw = ctas * kBwCta < kBwTotal ? ctas * kBwCta : kBwTotal;
            const double t_stream = total_bytes / (bw * 1e3) + kT0 * std::ceil(ctas / cap_d);
            const double t_cta = kT0 + nst * stage_bytes / (kBwCta * 1e3);
            const double t_merge = s == 1 ? 0.0 : cl ? kMergeCl : kMerge0 + s * nrows * D * 4.0 / (kBwMerge * 1e3);
            // The deep kernel's extra fixed cost (group merge, larger ring set-up).
            const double t_fixed = deep ? (cl ? 0.2 : 0.4) : 0.0;
            const double cost = (t_stream > t_cta ? t_stream : t_cta) + t_merge + t_fixed;
            if (plan_debug)                          // tuning aid: every candidate to stderr
                std::fprintf(stderr, "decode plan: deep %d splits %d cluster %d act %d cost %.3f us\n", deep, s,
                             cl ? 1 : 0, caps ? caps->act[deep][s < 17 ? s : 0] : -1, cost);
            if (cost < best_cost * 0.999) {
                best_cost = cost;
                best_s = s;
                best_deep = deep != 0;
                best_cl = cl;
            }
        }
    }
    // Tuning override (benchmark sweeps): KF_DECODE_NSPLIT=<n> forces the split
    // count when the workspace allows it.
    if (const char* ov = std::getenv("KF_DECODE_NSPLIT")) {
        int want = std::atoi(ov);
        const int s_ov = want >= 1 ? (total_stages + ((total_stages + want - 1) / want) - 1) /
                                         ((total_stages + want - 1) / want) : 0;
        const bool cl_ov = caps && s_ov >= 2 && s_ov <= 16 && caps->act[best_deep][s_ov] > 0 &&
                           (!best_deep || caps->act[1][s_ov] >= units);
        if (want >= 1 && want <= max_s && (want == 1 || cl_ov || (units <= kCounterSlots &&
                                                                 split_ws_bytes(rows, want, D) <= ws_bytes))) {
            best_s = s_ov;
            best_cl = cl_ov;
        }
    }
    const int nst = (total_stages + best_s - 1) / best_s;
    if (best_deep && static_cast<long long>(units) * best_s > sm_count) best_deep = false;   // after an override
    if (best_cl)
        best_cl = caps && best_s >= 2 && best_s <= 16 && caps->act[best_deep][best_s] > 0 &&
                  (!best_deep || caps->act[1][best_s] >= units);
    pl->deep = best_deep;
    pl->cluster = best_cl && best_s >= 2;
    pl->n_split = best_s;
    pl->chunk = nst * TK;
    pl->ws_bytes = (best_s > 1 && !pl->cluster) ? split_ws_bytes(rows, best_s, D) : 0;
    pl->ctas = units * best_s;
    return KF_OK;
}

int plan_for_call(int B, int H_q, int H_kv, int S_q, int S_kv, int D, size_t ws_bytes, Plan* pl,
                  bool causal = false, double cta_rate = 1.0, bool deep_only = false) {
    DeviceInfo* di = nullptr;
    int rc = device_info(&di);
    if (rc != KF_OK) return rc;
    const int G = H_q / H_kv;
    int bps = 1;
    ClusterCaps caps;
    bool have_caps = false;
    if (use_decode(G, S_q, D) && !(causal && S_q > 1)) {
        const int R = G * S_q;
        const int mt = R <= 16 ? 1 : decode_max_mt(D);
        rc = decode_bps(D, mt, &bps);
        if (rc != KF_OK) return rc;
        // KF_DECODE_CLUSTER=0: no cluster-merge plans (the workspace ticket merge only).
        const char* ce = std::getenv("KF_DECODE_CLUSTER");
        if (cta_rate >= 1.0 && !deep_only && !(ce && std::atoi(ce) == 0)) {
            if ((rc = decode_cluster_caps(D, mt, &caps)) != KF_OK) return rc;
            have_caps = true;
        }
    }
    return make_plan(B, H_q, H_kv, S_q, S_kv, D, ws_bytes, di->sm_count, bps, pl, causal, cta_rate,
                     cta_rate >= 1.0,    // paged K/V (cta_rate < 1): no deep-ring or cluster kernel
                     deep_only, have_caps ? &caps : nullptr);
}

// ------------------------------------------------------------------ launches
// Kernel launch with programmatic stream serialization (programmatic dependent launch)
// unless KF_PDL=0: the kernel's CTAs may be dispatched while the previous kernel on the
// stream drains.  Every kernel launched this way runs griddepcontrol.wait before its first
// global-memory (and TMEM) access, so results do not depend on it.
// cluster_x > 0: thread-block clusters of (cluster_x, 1, 1) CTAs.  pdl = false: no
// early dispatch (the deep-ring decode, one CTA per SM, measured slower with it:
// B=16 42.6 against 41.6 us, KV=131072 83.9 against 80.7 us).
template <typename... KArgs, typename... Args>
cudaError_t launch_ex(void (*kern)(KArgs...), dim3 grid, int threads, int smem_bytes, cudaStream_t s,
                      unsigned cluster_x, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(static_cast<unsigned>(threads));
    cfg.dynamicSmemBytes = static_cast<size_t>(smem_bytes);
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    unsigned n = 0;
    const char* e = std::getenv("KF_PDL");
    if (pdl && !(e && std::atoi(e) == 0)) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    if (cluster_x > 0) {
        attr[n].id = cudaLaunchAttributeClusterDimension;
        attr[n].val.clusterDim.x = cluster_x;
        attr[n].val.clusterDim.y = 1;
        attr[n].val.clusterDim.z = 1;
        ++n;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, int threads, int smem_bytes, cudaStream_t s,
                       Args... args) {
    return launch_ex(kern, grid, threads, smem_bytes, s, 0u, true, args...);
}

template <int D>
int launch_prefill(const Plan& pl, const void* Q, const void* K, const void* V, void* O, float* Mi, float* Li,
                   int unnorm, int B, int H_q, int H_kv, int S_q, int S_kv, void* ws, cudaStream_t s,
                   bool causal, int out_type) {
    using C = kf::PrefillCfg<D>;
    int bps = 0;
    const bool split = pl.pf_plain < pl.pf_units;
    const bool kvh = C::NQ == 2 && pl.pf_kvh;
    if (kvh && causal) return KF_ERR_INVALID_ARG;
    int rc;
    if constexpr (C::NQ == 2) {
        if (kvh)
            rc = split ? kernel_setup<kf::prefill_fwd_kernel<D, false, true, true>>(C::SMEM_BYTES, C::THREADS, &bps)
                       : kernel_setup<kf::prefill_fwd_kernel<D, false, false, true>>(C::SMEM_BYTES, C::THREADS, &bps);
    }
    if (!kvh)
        rc = causal  ? (split ? kernel_setup<kf::prefill_fwd_kernel<D, true, true>>(C::SMEM_BYTES, C::THREADS, &bps)
                              : kernel_setup<kf::prefill_fwd_kernel<D, true, false>>(C::SMEM_BYTES, C::THREADS, &bps))
             : split ? kernel_setup<kf::prefill_fwd_kernel<D, false, true>>(C::SMEM_BYTES, C::THREADS, &bps)
                     : kernel_setup<kf::prefill_fwd_kernel<D, false, false>>(C::SMEM_BYTES, C::THREADS, &bps);
    if (rc != KF_OK) return rc;
    // A TMA box may not exceed the tensor: short sequences load S rows and the
    // kernel keeps the remaining tile rows zero.
    const int q_box = S_q < C::BM ? S_q : C::BM;
    const int kv_box = S_kv < C::BC ? S_kv : C::BC;
    CUtensorMap mq, mk, mv, mo;
    if ((rc = make_map(&mq, Q, D, S_q, static_cast<long long>(B) * H_q, q_box, C::SWB)) != KF_OK) return rc;
    if ((rc = make_map(&mk, K, D, S_kv, static_cast<long long>(B) * H_kv, kv_box, C::SWB)) != KF_OK) return rc;
    if ((rc = make_map(&mv, V, D, S_kv, static_cast<long long>(B) * H_kv, kv_box, C::SWB)) != KF_OK) return rc;
    if (C::TMA_STORE && out_type == kf::KF_OUT_F32) {
        if ((rc = make_map_f32(&mo, O, D, S_q, static_cast<long long>(B) * H_q, q_box)) != KF_OK) return rc;
    } else if (C::TMA_STORE) {
        // 16-bit O: 64-column (128-B) spans, 128-B swizzle.
        if ((rc = make_map(&mo, O, D, S_q, static_cast<long long>(B) * H_q, q_box, 128,
                           out_type == kf::KF_OUT_BF16)) != KF_OK)
            return rc;
    } else {
        std::memset(&mo, 0, sizeof(mo));
    }
    kf::PrefillParams p;
    p.O = O;
    p.Mi = Mi;
    p.Li = Li;
    p.H_q = H_q;
    p.H_kv = H_kv;
    p.S_q = S_q;
    p.S_kv = S_kv;
    p.G = H_q / H_kv;
    p.scale = 1.0f / std::sqrt(static_cast<float>(D));
    p.scale_log2 = p.scale * 1.4426950408889634f;
    // KF_PREFILL_TICKET_MERGE=1: split units merge by ticket only (no owner wait).
    const char* tm = std::getenv("KF_PREFILL_TICKET_MERGE");
    p.flags = (unnorm ? kf::KF_PF_UNNORMALIZED : 0) | (tm && std::atoi(tm) ? kf::KF_PF_TICKET_MERGE : 0);
    p.out_type = out_type;
    p.timeout_ns = g_timeout_ns.load();
    p.q_box = q_box;
    p.kv_box = kv_box;
    p.n_qblk = pl.pf_qblk;
    p.unit_tiles = pl.pf_tiles;
    p.B_H = B * H_q;
    p.kv_off = S_kv - S_q;
    p.n_units = pl.pf_units;
    p.n_plain = pl.pf_plain;
    p.split_k = pl.pf_k;
    p.per = pl.pf_per;
    p.counters = split ? static_cast<unsigned*>(ws) : nullptr;
    p.part = split ? reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + kCounterBytes) : nullptr;
    const long long n_items = pl.ctas;          // whole units + KV chunks of split units
    if (n_items <= 0 || n_items > 0x7fffffffll) return KF_ERR_INVALID_ARG;
    p.n_items = static_cast<int>(n_items);
    // Persistent CTAs (one per SM, striding over the items) when every tile is full
    // size; short sequences rely on zero-filled tile rows, so each CTA then takes one item.
    DeviceInfo* di = nullptr;
    if ((rc = device_info(&di)) != KF_OK) return rc;
    const bool persistent = q_box == C::BM && kv_box == C::BC;
    const long long ctas = persistent && n_items > di->sm_count ? di->sm_count : n_items;
    const dim3 grid(static_cast<unsigned>(ctas));
    cudaError_t e = cudaSuccess;
    if constexpr (C::NQ == 2) {
        if (kvh && split)
            e = launch_pdl(kf::prefill_fwd_kernel<D, false, true, true>, grid, C::THREADS, C::SMEM_BYTES, s, mq, mk, mv,
                           mo, p);
        else if (kvh)
            e = launch_pdl(kf::prefill_fwd_kernel<D, false, false, true>, grid, C::THREADS, C::SMEM_BYTES, s, mq, mk, mv,
                           mo, p);
    }
    if (kvh) {
    } else if (causal && split)
        e = launch_pdl(kf::prefill_fwd_kernel<D, true, true>, grid, C::THREADS, C::SMEM_BYTES, s, mq, mk, mv, mo, p);
    else if (causal)
        e = launch_pdl(kf::prefill_fwd_kernel<D, true, false>, grid, C::THREADS, C::SMEM_BYTES, s, mq, mk, mv, mo, p);
    else if (split)
        e = launch_pdl(kf::prefill_fwd_kernel<D, false, true>, grid, C::THREADS, C::SMEM_BYTES, s, mq, mk, mv, mo, p);
    else
        e = launch_pdl(kf::prefill_fwd_kernel<D, false, false>, grid, C::THREADS, C::SMEM_BYTES, s, mq, mk, mv, mo, p);
    return e == cudaSuccess ? KF_OK : cuda_fail(e);
}

// Paged KV description (kf_attn_fwd_paged); null for contiguous K/V.
struct Paged {
    const int* block_table;
    const int* seq_lens;
    int n_blocks, block_size, max_blocks;
};

// Fused cross-GPU exchange arguments (kf_attn_fwd_exchange); null otherwise.
struct Xch {
    void* const* windows;
    int world, rank;
    long long part_stride;
};

template <int D, int MT, bool DEEP, int XW = 0>
int launch_decode_t(const Plan& pl, const void* Q, const void* K, const void* V, void* O, float* Mi, float* Li,
                    int unnorm, int B, int H_q, int H_kv, int S_q, int S_kv, void* ws, cudaStream_t s,
                    const Paged* pg, int out_type, const Xch* xa = nullptr) {
    using C = kf::DecodeCfg<D, MT, DEEP>;
    int bps = 0;
    const bool split = pl.n_split > 1;
    int rc;
    if constexpr (XW > 0) {
        static_assert(DEEP, "the fused exchange runs as a single wave (deep-ring plan)");
        if (pg || !xa) return KF_ERR_INVALID_ARG;
        rc = split ? kernel_setup<kf::decode_fwd_kernel<D, MT, false, true, true, XW>>(C::SMEM_BYTES, C::THREADS, &bps)
                   : kernel_setup<kf::decode_fwd_kernel<D, MT, false, false, true, XW>>(C::SMEM_BYTES, C::THREADS, &bps);
    } else if constexpr (DEEP) {
        // No deep-ring paged kernel: with one producer per SM issuing 2 KB page copies it
        // measured 80 us against 47 us one group (B=16, KV=4096, 16-row pages).
        if (pg) return KF_ERR_INVALID_ARG;
        rc = split ? kernel_setup<kf::decode_fwd_kernel<D, MT, false, true, true>>(C::SMEM_BYTES, C::THREADS, &bps)
                   : kernel_setup<kf::decode_fwd_kernel<D, MT, false, false, true>>(C::SMEM_BYTES, C::THREADS, &bps);
    } else {
        rc = pg ? (split ? kernel_setup<kf::decode_fwd_kernel<D, MT, true, true>>(C::SMEM_BYTES, C::THREADS, &bps)
                         : kernel_setup<kf::decode_fwd_kernel<D, MT, true, false>>(C::SMEM_BYTES, C::THREADS, &bps))
                : (split ? kernel_setup<kf::decode_fwd_kernel<D, MT, false, true>>(C::SMEM_BYTES, C::THREADS, &bps)
                         : kernel_setup<kf::decode_fwd_kernel<D, MT, false, false>>(C::SMEM_BYTES, C::THREADS, &bps));
    }
    if (rc != KF_OK) return rc;
    const int kv_box = S_kv < C::TK ? S_kv : C::TK;
    CUtensorMap mk, mv;
    if (pg) {
        // Pools [n_blocks][H_kv][block_size][D]: 3-D maps (D, block_size, n_blocks * H_kv).
        const int box = pg->block_size < C::TK ? pg->block_size : C::TK;
        const long long planes = static_cast<long long>(pg->n_blocks) * H_kv;
        if ((rc = make_map(&mk, K, D, pg->block_size, planes, box, C::SWB)) != KF_OK) return rc;
        if ((rc = make_map(&mv, V, D, pg->block_size, planes, box, C::SWB)) != KF_OK) return rc;
    } else {
        if ((rc = make_map(&mk, K, D, S_kv, static_cast<long long>(B) * H_kv, kv_box, C::SWB)) != KF_OK) return rc;
        if ((rc = make_map(&mv, V, D, S_kv, static_cast<long long>(B) * H_kv, kv_box, C::SWB)) != KF_OK) return rc;
    }
    kf::DecodeParams p;
    p.block_table = pg ? pg->block_table : nullptr;
    p.seq_lens = pg ? pg->seq_lens : nullptr;
    p.max_blocks = pg ? pg->max_blocks : 0;
    p.block_size = pg ? pg->block_size : 0;
    p.Q = static_cast<const uint16_t*>(Q);
    p.O = O;
    p.Mi = Mi;
    p.Li = Li;
    p.counters = static_cast<unsigned*>(ws);
    p.part_O = ws ? reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + kCounterBytes) : nullptr;
    const long long rows = static_cast<long long>(B) * H_q * S_q;
    p.part_ml = p.part_O ? p.part_O + rows * pl.n_split * D : nullptr;
    p.H_q = H_q;
    p.H_kv = H_kv;
    p.S_q = S_q;
    p.S_kv = S_kv;
    p.G = H_q / H_kv;
    p.R = p.G * S_q;
    p.n_rg = pl.n_rg;
    p.n_split = pl.n_split;
    p.chunk = pl.chunk;
    p.scale = 1.0f / std::sqrt(static_cast<float>(D));
    p.scale_log2 = p.scale * 1.4426950408889634f;
    p.unnormalized = unnorm;
    p.out_type = out_type;
    p.timeout_ns = g_timeout_ns.load();
    p.kv_box = pg ? C::TK : kv_box;
    for (int r = 0; r < kf::kMaxPeers; ++r) p.xwin[r] = nullptr;
    p.xown = nullptr;
    p.xcalls = nullptr;
    p.xps = 0;
    p.xrows = rows;
    p.xrank = 0;
    if (xa) {
        for (int r = 0; r < xa->world; ++r) p.xwin[r] = static_cast<float*>(xa->windows[r]);
        p.xown = p.xwin[xa->rank];
        p.xps = xa->part_stride;
        p.xrank = xa->rank;
        p.xcalls = reinterpret_cast<unsigned*>(p.xown + kf::peer_unit_calls_off(xa->part_stride, xa->world));
    }
    dim3 grid(pl.n_split, H_kv * pl.n_rg, B);
    cudaError_t e;
    if constexpr (XW > 0) {
        // The exchange waits on peer GPUs: a plain launch (no early dispatch next to the
        // previous kernel).
        if (split)
            kf::decode_fwd_kernel<D, MT, false, true, true, XW><<<grid, C::THREADS, C::SMEM_BYTES, s>>>(mk, mv, p);
        else
            kf::decode_fwd_kernel<D, MT, false, false, true, XW><<<grid, C::THREADS, C::SMEM_BYTES, s>>>(mk, mv, p);
        e = cudaGetLastError();
    } else if constexpr (DEEP) {
        if (split && pl.cluster) {
            int act[17];
            if ((rc = decode_cluster_act<D, MT, true>(act)) != KF_OK) return rc;
            if (pl.n_split > 16 || act[pl.n_split] <= 0) return KF_ERR_INVALID_ARG;
            e = launch_ex(kf::decode_fwd_kernel<D, MT, false, true, true, 0, true>, grid, C::THREADS, C::SMEM_BYTES, s,
                          static_cast<unsigned>(pl.n_split), false, mk, mv, p);
            return e == cudaSuccess ? KF_OK : cuda_fail(e);
        }
        e = split ? launch_ex(kf::decode_fwd_kernel<D, MT, false, true, true>, grid, C::THREADS, C::SMEM_BYTES, s, 0u,
                              false, mk, mv, p)
                  : launch_ex(kf::decode_fwd_kernel<D, MT, false, false, true>, grid, C::THREADS, C::SMEM_BYTES, s, 0u,
                              false, mk, mv, p);
    } else if (pg) {
        e = split ? launch_pdl(kf::decode_fwd_kernel<D, MT, true, true>, grid, C::THREADS, C::SMEM_BYTES, s, mk, mv, p)
                  : launch_pdl(kf::decode_fwd_kernel<D, MT, true, false>, grid, C::THREADS, C::SMEM_BYTES, s, mk, mv, p);
    } else if (split && pl.cluster) {
        int act[17];
        if ((rc = decode_cluster_act<D, MT, false>(act)) != KF_OK) return rc;
        if (pl.n_split > 16 || act[pl.n_split] <= 0) return KF_ERR_INVALID_ARG;   // the planner keeps within it
        e = launch_ex(kf::decode_fwd_kernel<D, MT, false, true, false, 0, true>, grid, C::THREADS, C::SMEM_BYTES, s,
                      static_cast<unsigned>(pl.n_split), true, mk, mv, p);
    } else {
        e = split ? launch_pdl(kf::decode_fwd_kernel<D, MT, false, true>, grid, C::THREADS, C::SMEM_BYTES, s, mk, mv, p)
                  : launch_pdl(kf::decode_fwd_kernel<D, MT, false, false>, grid, C::THREADS, C::SMEM_BYTES, s, mk, mv,
                               p);
    }
    return e == cudaSuccess ? KF_OK : cuda_fail(e);
}

int launch_decode(const Plan& pl, int D, const void* Q, const void* K, const void* V, void* O, float* Mi,
                  float* Li, int unnorm, int B, int H_q, int H_kv, int S_q, int S_kv, void* ws, cudaStream_t s,
                  const Paged* pg = nullptr, int out_type = kf::KF_OUT_F32) {
    // The deep-ring kernel exists for 16-row tiles only (the planner offers it for mt == 1).
#define KF_DEC(DV, MTV)                                                                                          \
    if constexpr (MTV == 1) {                                                                                     \
        if (pl.deep)                                                                                              \
            return launch_decode_t<DV, MTV, true>(pl, Q, K, V, O, Mi, Li, unnorm, B, H_q, H_kv, S_q, S_kv, ws, s, \
                                                  pg, out_type);                                                  \
    } else {                                                                                                      \
        if (pl.deep) return KF_ERR_INVALID_ARG;                                                                   \
    }                                                                                                             \
    return launch_decode_t<DV, MTV, false>(pl, Q, K, V, O, Mi, Li, unnorm, B, H_q, H_kv, S_q, S_kv, ws, s, pg,    \
                                           out_type)
    switch (D) {
        case 16: if (pl.mt == 2) { KF_DEC(16, 2); } KF_DEC(16, 1);
        case 64: if (pl.mt == 2) { KF_DEC(64, 2); } KF_DEC(64, 1);
        case 128: if (pl.mt == 2) { KF_DEC(128, 2); } KF_DEC(128, 1);
        default: KF_DEC(256, 1);
    }
#undef KF_DEC
}

int attn_core(const void* Q, const void* K, const void* V, void* O, float* Mi, float* Li, int unnorm, int B,
              int H_q, int H_kv, int S_q, int S_kv, int D, void* ws, size_t ws_bytes, void* stream,
              unsigned flags = 0) {
    int rc = validate(Q, K, V, static_cast<const float*>(O), B, H_q, H_kv, S_q, S_kv, D);
    if (rc != KF_OK) return rc;
    if (flags & ~static_cast<unsigned>(KF_FLAG_CAUSAL | KF_FLAG_OUT_F16 | KF_FLAG_OUT_BF16)) return KF_ERR_INVALID_ARG;
    if ((flags & KF_FLAG_OUT_F16) && (flags & KF_FLAG_OUT_BF16)) return KF_ERR_INVALID_ARG;
    const bool causal = (flags & KF_FLAG_CAUSAL) != 0;
    const int out_type = (flags & KF_FLAG_OUT_F16) ? kf::KF_OUT_F16
                       : (flags & KF_FLAG_OUT_BF16) ? kf::KF_OUT_BF16 : kf::KF_OUT_F32;
    if (unnorm && out_type != kf::KF_OUT_F32) return KF_ERR_INVALID_ARG;   // partials stay fp32
    if (causal && S_q > S_kv) return KF_ERR_INVALID_ARG;   // rows with no visible key
    if (B == 0 || S_q == 0) return KF_OK;
    if (!ws) ws_bytes = 0;
    if (ws && !aligned16(ws)) return KF_ERR_MISALIGNED;
    Plan pl;
    if ((rc = plan_for_call(B, H_q, H_kv, S_q, S_kv, D, ws_bytes, &pl, causal)) != KF_OK) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (pl.path == 0) {
        switch (D) {
            case 16: return launch_prefill<16>(pl, Q, K, V, O, Mi, Li, unnorm, B, H_q, H_kv, S_q, S_kv, ws, s, causal, out_type);
            case 64: return launch_prefill<64>(pl, Q, K, V, O, Mi, Li, unnorm, B, H_q, H_kv, S_q, S_kv, ws, s, causal, out_type);
            case 128: return launch_prefill<128>(pl, Q, K, V, O, Mi, Li, unnorm, B, H_q, H_kv, S_q, S_kv, ws, s, causal, out_type);
            default: return launch_prefill<256>(pl, Q, K, V, O, Mi, Li, unnorm, B, H_q, H_kv, S_q, S_kv, ws, s, causal, out_type);
        }
    }
    return launch_decode(pl, D, Q, K, V, O, Mi, Li, unnorm, B, H_q, H_kv, S_q, S_kv, pl.n_split > 1 ? ws : nullptr, s,
                         nullptr, out_type);
}

int paged_core(const void* Q, const void* K_pool, const void* V_pool, const int* block_table, const int* seq_lens,
               float* O, float* Mi, float* Li, int B, int H_q, int H_kv, int S_q, int D, int n_blocks,
               int block_size, int max_blocks, void* ws, size_t ws_bytes, void* stream) {
    if (B < 0 || S_q < 0 || H_q <= 0 || H_kv <= 0 || H_q % H_kv != 0) return KF_ERR_INVALID_ARG;
    if (!(D == 16 || D == 64 || D == 128 || D == 256)) return KF_ERR_UNSUPPORTED_HEAD_DIM;
    if (n_blocks <= 0 || max_blocks <= 0) return KF_ERR_INVALID_ARG;
    // block_size: a power of two in [16, 256] (a stage of 64 rows is whole blocks or part of one).
    if (block_size < 16 || block_size > 256 || (block_size & (block_size - 1))) return KF_ERR_INVALID_ARG;
    if (static_cast<long long>(n_blocks) * H_kv >= (1ll << 31) ||
        static_cast<long long>(max_blocks) * block_size >= (1ll << 31))
        return KF_ERR_INVALID_ARG;
    if (!use_decode(H_q / H_kv, S_q, D)) return KF_ERR_INVALID_ARG;    // decode shapes only
    if (B == 0 || S_q == 0) return KF_OK;
    if (!Q || !K_pool || !V_pool || !block_table || !seq_lens || !O) return KF_ERR_INVALID_ARG;
    if (!aligned16(Q) || !aligned16(K_pool) || !aligned16(V_pool) || !aligned16(O)) return KF_ERR_MISALIGNED;
    if (!ws) ws_bytes = 0;
    if (ws && !aligned16(ws)) return KF_ERR_MISALIGNED;
    const int S_max = max_blocks * block_size;
    Plan pl;
    // Per-CTA streaming rate relative to contiguous K/V, measured on B200 at B=16,
    // KV=4096: 16-row pages 0.52, 64-row pages 0.88.
    const double rate = block_size >= 64 ? 0.88 : (block_size >= 32 ? 0.7 : 0.52);
    int rc = plan_for_call(B, H_q, H_kv, S_q, S_max, D, ws_bytes, &pl, false, rate);
    if (rc != KF_OK) return rc;
    if (pl.path != 1) return KF_ERR_INVALID_ARG;
    const Paged pg{block_table, seq_lens, n_blocks, block_size, max_blocks};
    return launch_decode(pl, D, Q, K_pool, V_pool, O, Mi, Li, 0, B, H_q, H_kv, S_q, S_max,
                         pl.n_split > 1 ? ws : nullptr, static_cast<cudaStream_t>(stream), &pg);
}

// ------------------------------------------------------------------ fixed scratch (kf_attn_fwd_noalloc)
// The split-KV decode needs scratch for its per-split partials and ticket
// counters.  kf_attn_fwd_noalloc takes that scratch from this fixed array
// instead of a caller workspace: every GPU that loads the library holds these
// 2 MiB until the process exits.  In host code the array's name is only a
// host-side stand-in; its device address comes from cudaGetSymbolAddress,
// fetched once per device with that device current.
constexpr size_t kNoAllocScratchBytes = size_t(2) << 20;
std::atomic<void*> g_noalloc_scratch[kMaxDevices];

}  // namespace

static __device__ __align__(256) unsigned char g_kf_noalloc_scratch[kNoAllocScratchBytes];

namespace {

int noalloc_scratch(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e);
    if (dev < 0 || dev >= kMaxDevices) return KF_ERR_UNSUPPORTED_DEVICE;
    void* ptr = g_noalloc_scratch[dev].load(std::memory_order_acquire);
    if (!ptr) {
        std::lock_guard<std::mutex> lk(g_dev_mu);
        ptr = g_noalloc_scratch[dev].load(std::memory_order_acquire);
        if (!ptr) {
            if ((e = cudaGetSymbolAddress(&ptr, g_kf_noalloc_scratch)) != cudaSuccess) return cuda_fail(e);
            if (!ptr) return cuda_fail(cudaErrorInvalidSymbol);
            g_noalloc_scratch[dev].store(ptr, std::memory_order_release);
        }
    }
    *out = ptr;
    return KF_OK;
}

}  // namespace

namespace {
// Plan of a fused exchange call: the deep-ring decode kernel as one wave (D = 128, one
// 16-row tile per (b, h_kv): H_q / H_kv * S_q <= 16).
int exchange_plan(int B, int H_q, int H_kv, int S_q, int S_kv, int D, size_t ws_bytes, Plan* pl) {
    if (D != 128 || static_cast<long long>(H_q / H_kv) * S_q > 16) return KF_ERR_INVALID_ARG;
    int rc = plan_for_call(B, H_q, H_kv, S_q, S_kv, D, ws_bytes, pl, false, 1.0, true);
    if (rc != KF_OK) return rc;
    return (pl->path == 1 && pl->deep && pl->mt == 1) ? KF_OK : KF_ERR_INVALID_ARG;
}
}  // namespace

extern "C" {

const char* kf_strerror(int code) {
    switch (code) {
        case KF_OK: return "ok";
        case KF_ERR_INVALID_ARG: return "invalid argument (shape, null pointer or H_q % H_kv != 0)";
        case KF_ERR_UNSUPPORTED_HEAD_DIM: return "unsupported head dimension (D must be 16, 64, 128 or 256)";
        case KF_ERR_MISALIGNED: return "pointer not 16-byte aligned";
        case KF_ERR_CUDA: return "CUDA runtime error (see kf_last_cuda_error)";
        case KF_ERR_DEVICE_TIMEOUT: return "a bounded in-kernel wait expired";
        case KF_ERR_UNSUPPORTED_DEVICE: return "current device is not an sm_100 (B200) GPU";
        case KF_ERR_WORKSPACE:
            return "workspace too small (for kf_attn_fwd_noalloc: the call needs more than its fixed 2 MiB scratch)";
        default: return "unknown status";
    }
}

int kf_last_cuda_error(void) { return t_last_cuda_error; }

const char* kf_version(void) { return "kernelfoundry-b200 0.1.0 (sm_100a)"; }

int kf_attn_fwd(const void* Q, const void* K, const void* V, float* O, int B, int H_q, int H_kv, int S_q, int S_kv,
                int D, void* workspace, size_t workspace_bytes, void* stream) {
    return attn_core(Q, K, V, O, nullptr, nullptr, 0, B, H_q, H_kv, S_q, S_kv, D, workspace, workspace_bytes, stream);
}

int kf_attn_fwd_lse(const void* Q, const void* K, const void* V, float* O, float* Mi, float* Li, int B, int H_q,
                    int H_kv, int S_q, int S_kv, int D, void* workspace, size_t workspace_bytes, void* stream) {
    return attn_core(Q, K, V, O, Mi, Li, 0, B, H_q, H_kv, S_q, S_kv, D, workspace, workspace_bytes, stream);
}

int kf_attn_fwd_ex(const void* Q, const void* K, const void* V, void* O, float* Mi, float* Li, int B, int H_q,
                   int H_kv, int S_q, int S_kv, int D, unsigned flags, void* workspace, size_t workspace_bytes,
                   void* stream) {
    return attn_core(Q, K, V, O, Mi, Li, 0, B, H_q, H_kv, S_q, S_kv, D, workspace, workspace_bytes, stream, flags);
}

int kf_attn_fwd_paged(const void* Q, const void* K_pool, const void* V_pool, const int* block_table,
                      const int* seq_lens, float* O, float* Mi, float* Li, int B, int H_q, int H_kv, int S_q, int D,
                      int n_blocks, int block_size, int max_blocks, void* workspace, size_t workspace_bytes,
                      void* stream) {
    return paged_core(Q, K_pool, V_pool, block_table, seq_lens, O, Mi, Li, B, H_q, H_kv, S_q, D, n_blocks, block_size,
                      max_blocks, workspace, workspace_bytes, stream);
}

size_t kf_attn_paged_workspace_bytes(int B, int H_q, int H_kv, int S_q, int D, int block_size, int max_blocks) {
    if (B <= 0 || S_q <= 0 || H_q <= 0 || H_kv <= 0 || H_q % H_kv != 0 || max_blocks <= 0 || block_size <= 0) return 0;
    if (!use_decode(H_q / H_kv, S_q, D)) return 0;
    Plan pl;
    const double rate = block_size >= 64 ? 0.88 : (block_size >= 32 ? 0.7 : 0.52);
    if (plan_for_call(B, H_q, H_kv, S_q, max_blocks * block_size, D, static_cast<size_t>(-1), &pl, false, rate) != KF_OK)
        return 0;
    return pl.ws_bytes;
}

int kf_attn_fwd_partial(const void* Q, const void* K, const void* V, float* O_u, float* m, float* l, int B, int H_q,
                        int H_kv, int S_q, int S_kv, int D, void* workspace, size_t workspace_bytes, void* stream) {
    if (B > 0 && S_q > 0 && (!m || !l)) return KF_ERR_INVALID_ARG;
    return attn_core(Q, K, V, O_u, m, l, 1, B, H_q, H_kv, S_q, S_kv, D, workspace, workspace_bytes, stream);
}

namespace {
int combine_launch(const float* O_parts, const float* m_parts, const float* l_parts, int n_parts,
                   long long stride_o, long long stride_ml, float* O, float* Mi, float* Li, long long rows, int D,
                   void* stream) {
    DeviceInfo* di = nullptr;
    int rc = device_info(&di);
    if (rc != KF_OK) return rc;
    const long long n4 = rows * (D / 4);
    const int threads = 256;
    long long blocks = (n4 + threads - 1) / threads;
    const long long maxb = static_cast<long long>(di->sm_count) * 8;
    if (blocks > maxb) blocks = maxb;
    kf::combine_partials_kernel<<<static_cast<unsigned>(blocks), threads, 0, static_cast<cudaStream_t>(stream)>>>(
        O_parts, m_parts, l_parts, n_parts, rows, D, stride_o, stride_ml, O, Mi, Li);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? KF_OK : cuda_fail(e);
}
}  // namespace

int kf_attn_combine(const float* O_parts, const float* m_parts, const float* l_parts, int n_parts, float* O,
                    float* Mi, float* Li, int B, int H_q, int S_q, int D, void* stream) {
    if (n_parts <= 0 || B < 0 || H_q <= 0 || S_q < 0) return KF_ERR_INVALID_ARG;
    if (!(D == 16 || D == 64 || D == 128 || D == 256)) return KF_ERR_UNSUPPORTED_HEAD_DIM;
    const long long rows = static_cast<long long>(B) * H_q * S_q;
    if (rows == 0) return KF_OK;
    if (!O_parts || !m_parts || !l_parts || !O) return KF_ERR_INVALID_ARG;
    if (!aligned16(O_parts) || !aligned16(O)) return KF_ERR_MISALIGNED;
    return combine_launch(O_parts, m_parts, l_parts, n_parts, rows * D, rows, O, Mi, Li, rows, D, stream);
}

int kf_attn_combine_packed(const float* parts, long long part_stride, int n_parts, float* O, float* Mi, float* Li,
                           int B, int H_q, int S_q, int D, void* stream) {
    if (n_parts <= 0 || B < 0 || H_q <= 0 || S_q < 0) return KF_ERR_INVALID_ARG;
    if (!(D == 16 || D == 64 || D == 128 || D == 256)) return KF_ERR_UNSUPPORTED_HEAD_DIM;
    const long long rows = static_cast<long long>(B) * H_q * S_q;
    if (rows == 0) return KF_OK;
    if (!parts || !O) return KF_ERR_INVALID_ARG;
    if (part_stride < rows * (D + 2) || part_stride % 4 != 0) return KF_ERR_INVALID_ARG;
    if (!aligned16(parts) || !aligned16(O)) return KF_ERR_MISALIGNED;
    return combine_launch(parts, parts + rows * D, parts + rows * D + rows, n_parts, part_stride, part_stride, O, Mi,
                          Li, rows, D, stream);
}

size_t kf_peer_window_bytes(int world, long long part_stride, int n_chunks) {
    if (world < 1 || world > KF_MAX_PEERS || part_stride <= 0 || part_stride % 4 != 0 || n_chunks < 1) return 0;
    return static_cast<size_t>(kf::peer_window_words(part_stride, world, n_chunks)) * 4;
}

int kf_peer_window_alloc(size_t bytes, void** window, void* handle_out) {
    if (bytes == 0 || !window || !handle_out) return KF_ERR_INVALID_ARG;
    static_assert(sizeof(cudaIpcMemHandle_t) == KF_PEER_HANDLE_BYTES, "IPC handle size");
    DeviceInfo* di = nullptr;
    int rc = device_info(&di);
    if (rc != KF_OK) return rc;
    void* ptr = nullptr;
    cudaError_t e = cudaMalloc(&ptr, bytes);
    if (e != cudaSuccess) return cuda_fail(e);
    // The window must be zero before its handle leaves this process: a peer that
    // opens it may write its first {value, sequence} words at once, and a zero fill
    // still queued behind them would erase them.  cudaMemset does not block the
    // host for device memory, so wait for the fill explicitly.
    if ((e = cudaMemsetAsync(ptr, 0, bytes, 0)) != cudaSuccess || (e = cudaStreamSynchronize(0)) != cudaSuccess) {
        cudaFree(ptr);
        return cuda_fail(e);
    }
    cudaIpcMemHandle_t h;
    if ((e = cudaIpcGetMemHandle(&h, ptr)) != cudaSuccess) { cudaFree(ptr); return cuda_fail(e); }
    std::memcpy(handle_out, &h, sizeof(h));
    *window = ptr;
    return KF_OK;
}

int kf_peer_window_open(const void* handle, void** peer_window) {
    if (!handle || !peer_window) return KF_ERR_INVALID_ARG;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* ptr = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e);
    *peer_window = ptr;
    return KF_OK;
}

int kf_peer_window_close(void* peer_window) {
    if (!peer_window) return KF_ERR_INVALID_ARG;
    cudaError_t e = cudaIpcCloseMemHandle(peer_window);
    return e == cudaSuccess ? KF_OK : cuda_fail(e);
}

int kf_peer_window_free(void* window) {
    if (!window) return KF_ERR_INVALID_ARG;
    cudaError_t e = cudaFree(window);
    return e == cudaSuccess ? KF_OK : cuda_fail(e);
}

int kf_attn_exchange_combine(void* const* windows, int world, int rank, long long part_stride, int n_chunks,
                             float* O, float* Mi, float* Li, int B, int H_q, int S_q, int D, void* stream) {
    if (!windows || world < 1 || world > KF_MAX_PEERS || rank < 0 || rank >= world) return KF_ERR_INVALID_ARG;
    if (B < 0 || H_q <= 0 || S_q < 0 || n_chunks < 1) return KF_ERR_INVALID_ARG;
    if (!(D == 16 || D == 64 || D == 128 || D == 256)) return KF_ERR_UNSUPPORTED_HEAD_DIM;
    const long long rows = static_cast<long long>(B) * H_q * S_q;
    if (part_stride < rows * (D + 2) || part_stride % 4 != 0) return KF_ERR_INVALID_ARG;
    if (!O) return KF_ERR_INVALID_ARG;
    for (int r = 0; r < world; ++r) {
        if (!windows[r]) return KF_ERR_INVALID_ARG;
        if (!aligned16(windows[r])) return KF_ERR_MISALIGNED;
    }
    if (!aligned16(O)) return KF_ERR_MISALIGNED;
    if (rows == 0) return KF_OK;
    DeviceInfo* di = nullptr;
    int rc = device_info(&di);
    if (rc != KF_OK) return rc;
    // One CTA per SM at most: every chunk a peer waits for is resident.
    if (n_chunks > di->sm_count) return KF_ERR_INVALID_ARG;
    kf::ExchangeParams p;
    for (int r = 0; r < kf::kMaxPeers; ++r) p.win[r] = r < world ? static_cast<float*>(windows[r]) : nullptr;
    p.own = static_cast<float*>(windows[rank]);
    p.world = world;
    p.rank = rank;
    p.part_stride = part_stride;
    p.rows = rows;
    p.D = D;
    p.n_chunks = n_chunks;
    p.O = O;
    p.Mi = Mi;
    p.Li = Li;
    p.timeout_ns = g_timeout_ns.load();
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const dim3 grid(static_cast<unsigned>(n_chunks));
    cudaError_t e;
    switch (world) {
        case 1: e = launch_pdl(kf::exchange_combine_kernel<1>, grid, 256, 0, st, p); break;
        case 2: e = launch_pdl(kf::exchange_combine_kernel<2>, grid, 256, 0, st, p); break;
        case 3: e = launch_pdl(kf::exchange_combine_kernel<3>, grid, 256, 0, st, p); break;
        case 4: e = launch_pdl(kf::exchange_combine_kernel<4>, grid, 256, 0, st, p); break;
        case 5: e = launch_pdl(kf::exchange_combine_kernel<5>, grid, 256, 0, st, p); break;
        case 6: e = launch_pdl(kf::exchange_combine_kernel<6>, grid, 256, 0, st, p); break;
        case 7: e = launch_pdl(kf::exchange_combine_kernel<7>, grid, 256, 0, st, p); break;
        default: e = launch_pdl(kf::exchange_combine_kernel<8>, grid, 256, 0, st, p); break;
    }
    return e == cudaSuccess ? KF_OK : cuda_fail(e);
}

size_t kf_attn_exchange_workspace_bytes(int B, int H_q, int H_kv, int S_q, int S_kv, int D) {
    if (validate(reinterpret_cast<const void*>(16), reinterpret_cast<const void*>(16),
                 reinterpret_cast<const void*>(16), reinterpret_cast<const float*>(16), B, H_q, H_kv, S_q, S_kv,
                 D) != KF_OK || B == 0 || S_q == 0)
        return 0;
    Plan pl;
    if (exchange_plan(B, H_q, H_kv, S_q, S_kv, D, static_cast<size_t>(-1), &pl) != KF_OK) return 0;
    return pl.ws_bytes;
}

int kf_attn_fwd_exchange(const void* Q, const void* K, const void* V, void* const* windows, int world, int rank,
                         long long part_stride, float* O, float* Mi, float* Li, int B, int H_q, int H_kv, int S_q,
                         int S_kv, int D, void* workspace, size_t workspace_bytes, void* stream) {
    int rc = validate(Q, K, V, O, B, H_q, H_kv, S_q, S_kv, D);
    if (rc != KF_OK) return rc;
    if (!windows || !(world == 1 || world == 2 || world == 4 || world == 8) || rank < 0 || rank >= world)
        return KF_ERR_INVALID_ARG;
    const long long rows = static_cast<long long>(B) * H_q * S_q;
    if (part_stride < rows * (D + 2) || part_stride % 4 != 0) return KF_ERR_INVALID_ARG;
    for (int r = 0; r < world; ++r) {
        if (!windows[r]) return KF_ERR_INVALID_ARG;
        if (!aligned16(windows[r])) return KF_ERR_MISALIGNED;
    }
    if (B == 0 || S_q == 0) return KF_OK;
    if (!workspace) workspace_bytes = 0;
    if (workspace && !aligned16(workspace)) return KF_ERR_MISALIGNED;
    Plan pl;
    if ((rc = exchange_plan(B, H_q, H_kv, S_q, S_kv, D, workspace_bytes, &pl)) != KF_OK) return rc;
    const Xch xa{windows, world, rank, part_stride};
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    void* ws = pl.n_split > 1 ? workspace : nullptr;
    switch (world) {
        case 1: return launch_decode_t<128, 1, true, 1>(pl, Q, K, V, O, Mi, Li, 0, B, H_q, H_kv, S_q, S_kv, ws, s,
                                                       nullptr, kf::KF_OUT_F32, &xa);
        case 2: return launch_decode_t<128, 1, true, 2>(pl, Q, K, V, O, Mi, Li, 0, B, H_q, H_kv, S_q, S_kv, ws, s,
                                                       nullptr, kf::KF_OUT_F32, &xa);
        case 4: return launch_decode_t<128, 1, true, 4>(pl, Q, K, V, O, Mi, Li, 0, B, H_q, H_kv, S_q, S_kv, ws, s,
                                                       nullptr, kf::KF_OUT_F32, &xa);
        default: return launch_decode_t<128, 1, true, 8>(pl, Q, K, V, O, Mi, Li, 0, B, H_q, H_kv, S_q, S_kv, ws, s,
                                                        nullptr, kf::KF_OUT_F32, &xa);
    }
}

size_t kf_attn_workspace_bytes(int B, int H_q, int H_kv, int S_q, int S_kv, int D) {
    if (validate(reinterpret_cast<const void*>(16), reinterpret_cast<const void*>(16),
                 reinterpret_cast<const void*>(16), reinterpret_cast<const float*>(16), B, H_q, H_kv, S_q, S_kv,
                 D) != KF_OK || B == 0 || S_q == 0)
        return 0;
    Plan pl;
    if (plan_for_call(B, H_q, H_kv, S_q, S_kv, D, static_cast<size_t>(-1), &pl) != KF_OK) return 0;
    return pl.ws_bytes;
}

int kf_attn_workspace_init(void* workspace, size_t workspace_bytes, void* stream) {
    if (!workspace || workspace_bytes == 0) return KF_OK;
    cudaError_t e = cudaMemsetAsync(workspace, 0, workspace_bytes, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? KF_OK : cuda_fail(e);
}

int kf_attn_plan(int B, int H_q, int H_kv, int S_q, int S_kv, int D, size_t workspace_bytes, int* path, int* n_split,
                 int* grid_ctas) {
    int rc = validate(reinterpret_cast<const void*>(16), reinterpret_cast<const void*>(16),
                      reinterpret_cast<const void*>(16), reinterpret_cast<const float*>(16), B, H_q, H_kv, S_q, S_kv,
                      D);
    if (rc != KF_OK) return rc;
    Plan pl;
    if (B > 0 && S_q > 0 && (rc = plan_for_call(B, H_q, H_kv, S_q, S_kv, D, workspace_bytes, &pl)) != KF_OK) return rc;
    if (path) *path = pl.path;
    if (n_split) *n_split = pl.n_split;
    if (grid_ctas) *grid_ctas = static_cast<int>(pl.ctas);
    return KF_OK;
}

int kf_launch_flash_attn(const uint16_t* Q, const uint16_t* K, const uint16_t* V, float* O, int B, int S, int H_q,
                         int H_kv, int D, void* stream) {
    int rc = attn_core(Q, K, V, O, nullptr, nullptr, 0, B, H_q, H_kv, S, S, D, nullptr, 0, stream);
    if (rc != KF_OK) return rc;
    cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e);
    unsigned raw = 0;
    e = cudaMemcpyFromSymbol(&raw, kf::g_kf_dev_error, sizeof(raw));
    if (e != cudaSuccess) return cuda_fail(e);
    return raw ? KF_ERR_DEVICE_TIMEOUT : KF_OK;
}

int kf_device_error(int clear, unsigned* raw) {
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e);
    unsigned v = 0;
    if ((e = cudaMemcpyFromSymbol(&v, kf::g_kf_dev_error, sizeof(v))) != cudaSuccess) return cuda_fail(e);
    if (raw) *raw = v;
    if (clear && v) {
        const unsigned zero = 0;
        if ((e = cudaMemcpyToSymbol(kf::g_kf_dev_error, &zero, sizeof(zero))) != cudaSuccess) return cuda_fail(e);
    }
    return v ? KF_ERR_DEVICE_TIMEOUT : KF_OK;
}

void kf_set_wait_timeout_ns(unsigned long long ns) { g_timeout_ns.store(ns ? ns : kDefaultTimeoutNs); }

int kf_attn_fwd_noalloc(const void* Q, const void* K, const void* V, float* O, int B, int H_q, int H_kv, int S_q,
                        int S_kv, int D, void* stream) {
    int rc = validate(Q, K, V, O, B, H_q, H_kv, S_q, S_kv, D);
    if (rc != KF_OK) return rc;
    if (B == 0 || S_q == 0) return KF_OK;
    if (!use_decode(H_q / H_kv, S_q, D)) return KF_ERR_INVALID_ARG;   // short-query (decode) shapes only
    // The plan kf_attn_fwd makes with a workspace of the fixed scratch's size: the
    // planner keeps the split count whose partials fit (n_split = 1 needs none).
    Plan pl;
    if ((rc = plan_for_call(B, H_q, H_kv, S_q, S_kv, D, kNoAllocScratchBytes, &pl)) != KF_OK) return rc;
    if (pl.ws_bytes > kNoAllocScratchBytes) return KF_ERR_WORKSPACE;   // not reached: the plan fits
    void* scratch = nullptr;
    if (pl.n_split > 1) {
        // The ticket counters at the head of the array start at zero (a __device__
        // array is zero-initialised when the module loads) and every launch leaves
        // them at zero: the merging CTA of each unit resets its counter, also after
        // an expired wait.  The partials are overwritten before they are read.
        if ((rc = noalloc_scratch(&scratch)) != KF_OK) return rc;
    }
    return launch_decode(pl, D, Q, K, V, O, nullptr, nullptr, 0, B, H_q, H_kv, S_q, S_kv, scratch,
                         static_cast<cudaStream_t>(stream));
}

}  // extern "C"

// ---- RMSNorm / RoPE / SwiGLU -------------------------------------------------
namespace {

// Grid for a grid-stride pointwise kernel: as many blocks as are resident on
// all SMs at once (occupancy cached per device and block size), at most
// `needed`.  Block sizes are 256, 512 or 1024 threads.
template <auto Kern>
int pw_grid(int threads, long long needed, int* grid) {
    static std::atomic<int> bps[kMaxDevices][3];
    DeviceInfo* di = nullptr;
    int rc = device_info(&di);
    if (rc != KF_OK) return rc;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e);
    const int slot = threads >= 1024 ? 2 : threads >= 512 ? 1 : 0;
    int v = bps[dev][slot].load(std::memory_order_acquire);
    if (v == 0) {
        int n = 0;
        if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, Kern, threads, 0)) != cudaSuccess)
            return cuda_fail(e);
        v = n > 0 ? n : 1;
        bps[dev][slot].store(v, std::memory_order_release);
    }
    const long long cap = static_cast<long long>(di->sm_count) * v;
    *grid = static_cast<int>(needed < cap ? needed : cap);
    return KF_OK;
}

int launch_status() {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? KF_OK : cuda_fail(e);
}

template <bool BF16, int VPT, bool RES>
int rmsnorm_t(const kf::RmsNormParams& p, int threads, cudaStream_t s) {
    const int rpb = threads / p.G;
    int grid = 0;
    int rc = pw_grid<kf::rmsnorm_kernel<BF16, VPT, RES>>(threads, (p.rows + rpb - 1) / rpb, &grid);
    if (rc != KF_OK) return rc;
    kf::rmsnorm_kernel<BF16, VPT, RES><<<grid, threads, 0, s>>>(p);
    return launch_status();
}

template <bool BF16, bool RES>
int rmsnorm_vpt(const kf::RmsNormParams& p, int vpt, int threads, cudaStream_t s) {
    switch (vpt) {
        case 1: return rmsnorm_t<BF16, 1, RES>(p, threads, s);
        case 2: return rmsnorm_t<BF16, 2, RES>(p, threads, s);
        default: return rmsnorm_t<BF16, 4, RES>(p, threads, s);
    }
}

template <bool BF16>
int rmsnorm_dispatch(const kf::RmsNormParams& p, int vpt, int threads, cudaStream_t s) {
    return p.res ? rmsnorm_vpt<BF16, true>(p, vpt, threads, s) : rmsnorm_vpt<BF16, false>(p, vpt, threads, s);
}

template <bool BF16, bool NEOX, int HB>
int rope_hb(const kf::RopeParams& p, cudaStream_t s) {
    int grid = 0;
    int rc = pw_grid<kf::rope_kernel<BF16, NEOX, HB>>(256, (p.n_tokens + p.TPB - 1) / p.TPB, &grid);
    if (rc != KF_OK) return rc;
    kf::rope_kernel<BF16, NEOX, HB><<<grid, 256, 0, s>>>(p);
    return launch_status();
}

template <bool BF16, bool NEOX>
int rope_t(const kf::RopeParams& p, int hb, cudaStream_t s) {
    switch (hb) {
        case 1: return rope_hb<BF16, NEOX, 1>(p, s);
        case 4: return rope_hb<BF16, NEOX, 4>(p, s);
        default: return rope_hb<BF16, NEOX, 8>(p, s);
    }
}

template <bool BF16>
int swiglu_t(const kf::SwigluParams& p, cudaStream_t s) {
    int grid = 0;
    int rc = pw_grid<kf::swiglu_kernel<BF16>>(256, p.rows, &grid);
    if (rc != KF_OK) return rc;
    kf::swiglu_kernel<BF16><<<grid, 256, 0, s>>>(p);
    return launch_status();
}

bool stride_ok(long long st) { return st >= 0 && st % 8 == 0; }

}  // namespace

extern "C" {

int kf_rmsnorm(const void* x, const void* weight, void* out, void* residual, long long rows, int hidden,
               float eps, unsigned flags, void* stream) {
    if (flags & ~static_cast<unsigned>(KF_PW_BF16)) return KF_ERR_INVALID_ARG;
    if (rows < 0 || hidden < 8 || hidden > 32768 || hidden % 8 != 0) return KF_ERR_INVALID_ARG;
    if (!(eps >= 0.f) || !std::isfinite(eps)) return KF_ERR_INVALID_ARG;
    if (!x || !weight || !out) return KF_ERR_INVALID_ARG;
    if (!aligned16(x) || !aligned16(weight) || !aligned16(out) || (residual && !aligned16(residual)))
        return KF_ERR_MISALIGNED;
    if (rows == 0) return KF_OK;
    kf::RmsNormParams p;
    p.x = static_cast<const uint4*>(x);
    p.w = static_cast<const uint4*>(weight);
    p.out = static_cast<uint4*>(out);
    p.res = static_cast<uint4*>(residual);
    p.rows = rows;
    p.nvec = hidden / 8;
    // Threads per row: enough for at most 8 vectors each up to 256 threads,
    // at most 4 each beyond (1024 x 4 x 8 = 32768 elements).
    // Threads per row: enough for at most 4 vectors each (1024 x 4 x 8 = 32768
    // elements), which keeps a thread's row data at 16 registers (32 with
    // the residual) and the SM's warps high enough to cover HBM latency.
    int G = 1;
    while (G * 4 < p.nvec) G <<= 1;
    const int per = (p.nvec + G - 1) / G;
    int vpt = 1;
    while (vpt < per) vpt <<= 1;                            // <= 4
    p.G = G;
    p.inv_hidden = 1.f / static_cast<float>(hidden);
    p.eps = eps;
    const int threads = G > 256 ? G : 256;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return (flags & KF_PW_BF16) ? rmsnorm_dispatch<true>(p, vpt, threads, s)
                                : rmsnorm_dispatch<false>(p, vpt, threads, s);
}

int kf_rope(void* q, void* k, const int* positions, const float* inv_freq, int B, int S, int H_q, int H_kv,
            int D, int rot_dim, float theta, long long q_stride_b, long long q_stride_h, long long q_stride_s,
            long long k_stride_b, long long k_stride_h, long long k_stride_s, unsigned flags, void* stream) {
    if (flags & ~static_cast<unsigned>(KF_PW_BF16 | KF_ROPE_GPTJ)) return KF_ERR_INVALID_ARG;
    const bool neox = !(flags & KF_ROPE_GPTJ);
    if (B < 0 || S < 0 || H_q < 0 || H_kv < 0 || H_q + H_kv < 1) return KF_ERR_INVALID_ARG;
    if (D < 8 || D > 1024 || D % 8 != 0) return KF_ERR_INVALID_ARG;
    if (rot_dim <= 0 || rot_dim > D || rot_dim % (neox ? 16 : 8) != 0) return KF_ERR_INVALID_ARG;
    if (!inv_freq && !(theta > 0.f && std::isfinite(theta))) return KF_ERR_INVALID_ARG;
    if (H_q > 0 && (!q || !stride_ok(q_stride_b) || !stride_ok(q_stride_h) || !stride_ok(q_stride_s)))
        return KF_ERR_INVALID_ARG;
    if (H_kv > 0 && (!k || !stride_ok(k_stride_b) || !stride_ok(k_stride_h) || !stride_ok(k_stride_s)))
        return KF_ERR_INVALID_ARG;
    if ((H_q > 0 && !aligned16(q)) || (H_kv > 0 && !aligned16(k))) return KF_ERR_MISALIGNED;
    const long long n_tokens = static_cast<long long>(B) * S;
    if (n_tokens == 0) return KF_OK;
    kf::RopeParams p;
    p.q = H_q > 0 ? static_cast<uint4*>(q) : nullptr;
    p.k = H_kv > 0 ? static_cast<uint4*>(k) : nullptr;
    p.pos = positions;
    p.inv_freq = inv_freq;
    p.q_sb = q_stride_b / 8; p.q_sh = q_stride_h / 8; p.q_ss = q_stride_s / 8;
    p.k_sb = k_stride_b / 8; p.k_sh = k_stride_h / 8; p.k_ss = k_stride_s / 8;
    p.n_tokens = n_tokens;
    p.S = S;
    p.H_q = H_q;
    p.H_kv = H_kv;
    p.rot_dim = rot_dim;
    p.U = neox ? rot_dim / 16 : rot_dim / 8;                // 1..128
    // About 64 threads per token; each thread loads all of its HB head rows
    // (HB in {1, 4, 8}) before it computes the token's angles, so one round
    // trip to HBM covers the token whenever H <= 8 * (64 / U).
    const int H = H_q + H_kv;
    int hg_target = 64 / p.U;
    if (hg_target < 1) hg_target = 1;
    const int need = (H + hg_target - 1) / hg_target;
    const int hb = need <= 1 ? 1 : need <= 4 ? 4 : 8;
    p.HG = (H + hb - 1) / hb;
    p.TPB = 256 / (p.U * p.HG);
    if (p.TPB < 1) p.TPB = 1;
    p.log2_theta = inv_freq ? 0.0 : std::log2(static_cast<double>(theta));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool bf16 = flags & KF_PW_BF16;
    if (neox) return bf16 ? rope_t<true, true>(p, hb, s) : rope_t<false, true>(p, hb, s);
    return bf16 ? rope_t<true, false>(p, hb, s) : rope_t<false, false>(p, hb, s);
}

int kf_swiglu(const void* gate_up, void* out, long long rows, int inter, unsigned flags, void* stream) {
    if (flags & ~static_cast<unsigned>(KF_PW_BF16)) return KF_ERR_INVALID_ARG;
    if (rows < 0 || inter < 8 || inter % 8 != 0) return KF_ERR_INVALID_ARG;
    if (!gate_up || !out) return KF_ERR_INVALID_ARG;
    if (!aligned16(gate_up) || !aligned16(out)) return KF_ERR_MISALIGNED;
    if (rows == 0) return KF_OK;
    kf::SwigluParams p;
    p.gu = static_cast<const uint4*>(gate_up);
    p.out = static_cast<uint4*>(out);
    p.rows = rows;
    p.ivec = inter / 8;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return (flags & KF_PW_BF16) ? swiglu_t<true>(p, s) : swiglu_t<false>(p, s);
}

int kf_fill_normal_f16(uint16_t* dst, long long n, unsigned long long seed, long long offset, void* stream) {
    if (n < 0 || offset < 0 || (n > 0 && !dst)) return KF_ERR_INVALID_ARG;
    if (n > (1ll << 62) - offset) return KF_ERR_INVALID_ARG;     // element indices stay below 2^62
    if (n == 0) return KF_OK;
    if (reinterpret_cast<uintptr_t>(dst) & 1u) return KF_ERR_MISALIGNED;
    DeviceInfo* di = nullptr;
    int rc = device_info(&di);
    if (rc != KF_OK) return rc;
    const long long pairs = ((offset + n + 1) >> 1) - (offset >> 1);
    const long long want = (pairs + 255) / 256, cap = 8ll * di->sm_count;
    const unsigned grid = static_cast<unsigned>(want < cap ? want : cap);
    kf::fill_normal_f16_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<__half*>(dst), n, static_cast<uint64_t>(seed), offset);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? KF_OK : cuda_fail(e);
}

#ifdef KF_PREFILL_TRACE
// Developer builds only (python -m kernelfoundry_b200.phase_trace): the prefill kernels'
// per-CTA phase stamps (kf::PrefillTracePoint slots of kf::kTrSlots words per CTA, global
// timer ns, 0 = phase not reached).  Not declared in include/: the shipped library lacks them.
int kf_prefill_trace_read(unsigned long long* host, int n_ctas) {
    if (!host || n_ctas <= 0 || n_ctas > kf::kTraceCtas) return KF_ERR_INVALID_ARG;
    cudaError_t e = cudaMemcpyFromSymbol(host, kf::g_kf_prefill_trace,
                                         static_cast<size_t>(n_ctas) * kf::kTrSlots * sizeof(unsigned long long));
    return e == cudaSuccess ? KF_OK : cuda_fail(e);
}

int kf_prefill_trace_clear(void) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, kf::g_kf_prefill_trace);
    if (e == cudaSuccess) e = cudaMemset(ptr, 0, sizeof(kf::g_kf_prefill_trace));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    return e == cudaSuccess ? KF_OK : cuda_fail(e);
}
#endif

int kf_selftest_wait_timeout(unsigned long long timeout_ns, void* stream) {
    DeviceInfo* di = nullptr;
    int rc = device_info(&di);
    if (rc != KF_OK) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    kf::selftest_wait_kernel<<<1, 32, 0, s>>>(timeout_ns);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    if ((e = cudaStreamSynchronize(s)) != cudaSuccess) return cuda_fail(e);
    return kf_device_error(1, nullptr);
}

}  // extern "C"
