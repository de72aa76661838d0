/*
 * kf_attn.h -- C ABI of the B200 (sm_100a) attention forward.
 *
 * Drop-in boundary for the host launchers of sviraaj/kernelfoundry's
 * flash-attention kernel.  Tensor layout and numerics are the reference's:
 *   Q  [B, H_q,  S_q,  D]  fp16 (IEEE binary16 bits), row-major, device memory
 *   K  [B, H_kv, S_kv, D]  fp16
 *   V  [B, H_kv, S_kv, D]  fp16
 *   O  [B, H_q,  S_q,  D]  fp32 output
 *   Mi [B, H_q, S_q] fp32  row max of the scaled scores  (optional)
 *   Li [B, H_q, S_q] fp32  sum of exp(score - Mi)         (optional)
 *   score = (q . k) / sqrt(D); query head h uses KV head h / (H_q / H_kv).
 * D must be 16, 64, 128 or 256 (the reference's instantiations,
 * kernels/flash_attn.cu:589-600).  All pointers are device pointers (16-byte
 * aligned for Q, K, V, O); `stream` is a cudaStream_t (NULL = legacy default
 * stream).  Plain C types only: no CUDA or torch types in any signature.
 *
 * Every call returns KF_OK (0) or a KF_ERR_* code; none calls exit().
 * kf_attn_* calls are asynchronous on `stream` and allocate nothing.
 */
#ifndef KF_ATTN_H_
#define KF_ATTN_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define KF_OK 0
#define KF_ERR_INVALID_ARG 1          /* bad shape, null pointer, H_q % H_kv != 0, ... */
#define KF_ERR_UNSUPPORTED_HEAD_DIM 2 /* D not in {16, 64, 128, 256} */
#define KF_ERR_MISALIGNED 3           /* Q/K/V/O not 16-byte aligned */
#define KF_ERR_CUDA 4                 /* a CUDA runtime call failed: kf_last_cuda_error() */
#define KF_ERR_DEVICE_TIMEOUT 5       /* a bounded in-kernel wait expired */
#define KF_ERR_UNSUPPORTED_DEVICE 6   /* the current device is not sm_100 */
#define KF_ERR_WORKSPACE 7            /* workspace too small for an explicit request */

/* Human-readable text for a status code (static storage, never NULL). */
const char* kf_strerror(int code);

/* cudaError_t value (as int) of the most recent failing CUDA call on this thread. */
int kf_last_cuda_error(void);

/* Library version string. */
const char* kf_version(void);

/* ---- attention forward --------------------------------------------------
 * Replaces: launch_flash_attn(Q, K, V, O, B, S, H_q, H_kv, D, stream)
 *           (tests/test_flash_attn.cu:52-113) and the general q_len/kv_len
 *           launch of flash_attn_kernel<D> (tests/bench_flash_attn.cu:39-54,
 *           raw kernel signature kernels/flash_attn.cu:384-398).
 * Differences, by design: asynchronous (no stream synchronize), no per-call
 * cudaMalloc of Mi/Li scratch (the softmax state stays on chip; split partials
 * stay in shared memory or go to the caller's workspace).  Kernels are launched
 * with programmatic stream serialization: their CTAs may be dispatched while the
 * previous kernel on the stream drains, and they read and write global memory
 * only after that kernel has completed (KF_PDL=0 in the environment: plain
 * launches).
 *
 * workspace: optional device buffer used by split-KV decode plans that merge
 * through global memory (more than 16 splits per KV head, paged K/V) and by the
 * prefill's split last wave; decode splits that merge inside a thread-block
 * cluster need none (kf_attn_workspace_bytes then returns 0).  Size it with
 * kf_attn_workspace_bytes(); zero-fill it once before its first use
 * (kf_attn_workspace_init); every successful call leaves it ready for the
 * next.  Two calls that overlap on the GPU must not share a workspace.
 * workspace == NULL (or too small) is valid: decode then merges in a cluster or
 * uses fewer KV splits, and the prefill's last wave is not split (same results).
 */
int kf_attn_fwd(const void* Q, const void* K, const void* V, float* O,
                int B, int H_q, int H_kv, int S_q, int S_kv, int D,
                void* workspace, size_t workspace_bytes, void* stream);

/* Same, also writing the reference kernel's softmax state Mi/Li
 * (kernels/flash_attn.cu:575-578).  Mi and/or Li may be NULL. */
int kf_attn_fwd_lse(const void* Q, const void* K, const void* V, float* O,
                    float* Mi, float* Li,
                    int B, int H_q, int H_kv, int S_q, int S_kv, int D,
                    void* workspace, size_t workspace_bytes, void* stream);

/* Flags for kf_attn_fwd_ex. */
#define KF_FLAG_CAUSAL 1u    /* bottom-right causal mask (below) */
#define KF_FLAG_OUT_F16 2u   /* O is fp16 (default fp32) */
#define KF_FLAG_OUT_BF16 4u  /* O is bf16 */

/* kf_attn_fwd_lse with options (Mi/Li may be NULL; O points to fp32 data unless an
 * output flag says otherwise).  KF_FLAG_OUT_F16 / KF_FLAG_OUT_BF16: O is written as
 * fp16 / bf16 (round to nearest; half the bytes of the reference's fp32 O; Mi/Li
 * stay fp32; not both).  KF_FLAG_CAUSAL: query row i
 * of S_q sits at absolute position S_kv - S_q + i and attends keys
 * j <= S_kv - S_q + i (chunked prefill over a KV cache; S_q == S_kv is the usual
 * lower-triangular mask, S_q == 1 keeps every key); requires S_q <= S_kv, else
 * KF_ERR_INVALID_ARG.  Unknown flag bits are KF_ERR_INVALID_ARG.  No reference
 * counterpart: the reference has no mask and names it as required for decoder
 * use (docs/flash_attn.md:105). */
int kf_attn_fwd_ex(const void* Q, const void* K, const void* V,
                   void* O, float* Mi, float* Li,
                   int B, int H_q, int H_kv, int S_q, int S_kv, int D, unsigned flags,
                   void* workspace, size_t workspace_bytes, void* stream);

/* Decode over a paged KV cache (decode shapes: H_q/H_kv * S_q as for the decode
 * kernel, else KF_ERR_INVALID_ARG).  Pools K_pool/V_pool are fp16
 * [n_blocks][H_kv][block_size][D] (the layout of the reference's paged
 * benchmark, reference_benchmarks/bench_flash_attn2.py:153-215); logical block j
 * of sequence b lives at pool block block_table[b*max_blocks + j] (int32);
 * sequence b has seq_lens[b] keys (int32, device memory, clamped to
 * [0, max_blocks*block_size]; 0 gives O = 0).  block_size is a power of two in
 * [16, 256].  Q/O/Mi/Li as kf_attn_fwd_lse (non-causal: every query row sees the
 * sequence's keys).  Table entries past a sequence's last block are not read; an
 * entry outside [0, n_blocks) reads zeros.  Workspace as kf_attn_fwd, sized by
 * kf_attn_paged_workspace_bytes.  The reference has only the gather-then-attend
 * path; this reads the pages inside the kernel. */
int kf_attn_fwd_paged(const void* Q, const void* K_pool, const void* V_pool,
                      const int* block_table, const int* seq_lens,
                      float* O, float* Mi, float* Li,
                      int B, int H_q, int H_kv, int S_q, int D,
                      int n_blocks, int block_size, int max_blocks,
                      void* workspace, size_t workspace_bytes, void* stream);
size_t kf_attn_paged_workspace_bytes(int B, int H_q, int H_kv, int S_q, int D,
                                     int block_size, int max_blocks);

/* Partial attention over the given K/V (e.g. one GPU's slice of a long KV
 * cache): O_u = sum_j exp(s_j - m) v_j (un-normalised), m = max_j s_j,
 * l = sum_j exp(s_j - m), with s_j the scaled scores.  Merge partials of
 * disjoint KV slices with kf_attn_combine.  m and l must be non-NULL.
 * No reference counterpart: the reference has no split-KV; this is the
 * (Mi, Li, un-normalised O) state of its online softmax
 * (kernels/flash_attn.cu:261-294) exported for a cross-GPU merge. */
int kf_attn_fwd_partial(const void* Q, const void* K, const void* V,
                        float* O_u, float* m, float* l,
                        int B, int H_q, int H_kv, int S_q, int S_kv, int D,
                        void* workspace, size_t workspace_bytes, void* stream);

/* Log-sum-exp merge of n_parts partials stacked as
 *   O_parts [n_parts][B*H_q*S_q][D], m_parts/l_parts [n_parts][B*H_q*S_q]
 * into O [B,H_q,S_q,D] (normalised) and optional Mi/Li of the union.
 * No reference counterpart (see kf_attn_fwd_partial). */
int kf_attn_combine(const float* O_parts, const float* m_parts, const float* l_parts,
                    int n_parts, float* O, float* Mi, float* Li,
                    int B, int H_q, int S_q, int D, void* stream);

/* The same merge over partials packed back to back, part g at
 *   parts + g*part_stride = [O_u: B*H_q*S_q*D][m: B*H_q*S_q][l: B*H_q*S_q],
 * part_stride >= B*H_q*S_q*(D+2) floats and a multiple of 4: the layout of an
 * all-gather of each rank's kf_attn_fwd_partial output written into its slot,
 * merged without an unpacking copy.  No reference counterpart (see
 * kf_attn_fwd_partial). */
int kf_attn_combine_packed(const float* parts, long long part_stride, int n_parts,
                           float* O, float* Mi, float* Li,
                           int B, int H_q, int S_q, int D, void* stream);

/* ---- cross-GPU exchange over NVLink peer memory --------------------------
 * No reference counterpart (the reference is single-GPU).  For long-context
 * decode with the KV cache split by ranges over `world` GPUs (one process per
 * GPU), one kernel replaces the all-gather + kf_attn_combine_packed pair: it
 * writes this rank's partials into every peer's window over NVLink as 8-byte
 * {value, sequence number} words, polls the peers' words in its own window
 * and merges.
 *
 * Setup (once, outside the decode loop; these calls allocate):
 *   kf_peer_window_bytes     size of a window for world ranks, parts of
 *                            part_stride floats (>= B*H_q*S_q*(D+2), multiple
 *                            of 4) and n_chunks CTAs (1 <= n_chunks <= SMs):
 *                            staging part + 2 x world slots of 8-byte words +
 *                            per-unit and n_chunks call counters
 *   kf_peer_window_alloc     cudaMalloc + zero fill + CUDA IPC export; writes
 *                            KF_PEER_HANDLE_BYTES opaque bytes to handle_out
 *   kf_peer_window_open      maps another process's window (from its handle)
 *   kf_peer_window_close / kf_peer_window_free
 * Per decode step:
 *   kf_attn_fwd_partial(..., O = window, Mi = window + rows*D,
 *                       Li = window + rows*D + rows, ...)   staging part at the base
 *   kf_attn_exchange_combine(windows, world, rank, part_stride, n_chunks, O, ...)
 * windows[r] is rank r's window as mapped in this process (windows[rank] is
 * the own one).  Every rank makes the same sequence of calls with the same
 * shapes; each call's sequence number is kept in device memory, so both calls
 * can be captured in a CUDA graph and replayed.  Waits are bounded: a peer
 * that never arrives leaves this rank's O rows unwritten and
 * kf_device_error() reporting KF_ERR_DEVICE_TIMEOUT. */
#define KF_PEER_HANDLE_BYTES 64
#define KF_MAX_PEERS 8
size_t kf_peer_window_bytes(int world, long long part_stride, int n_chunks);
int kf_peer_window_alloc(size_t bytes, void** window, void* handle_out);
int kf_peer_window_open(const void* handle, void** peer_window);
int kf_peer_window_close(void* peer_window);
int kf_peer_window_free(void* window);
int kf_attn_exchange_combine(void* const* windows, int world, int rank, long long part_stride, int n_chunks,
                             float* O, float* Mi, float* Li, int B, int H_q, int S_q, int D, void* stream);

/* The same exchange fused into the decode kernel: one launch per decode step.  Q is
 * replicated, K/V [B, H_kv, S_kv, D] hold this rank's contiguous KV range; the kernel
 * CTA that merges a (b, h_kv) unit's KV splits writes the unit's partial straight into
 * every rank's window as {value, sequence} words, polls its own window for the other
 * ranks' words of that unit and writes the merged O (and Mi/Li) of the whole KV cache.
 * No staging part, no second launch.  Windows as above (kf_peer_window_bytes with any
 * n_chunks); each (b, h_kv) unit keeps its own call counter in the window, so this call
 * and kf_attn_exchange_combine may share windows.  Supported: D = 128, world 1, 2, 4
 * or 8, H_q/H_kv * S_q <= 16, and shapes whose launch fits the SMs in one wave (every
 * CTA a peer waits for is then resident); other shapes return KF_ERR_INVALID_ARG (use
 * kf_attn_fwd_partial + kf_attn_exchange_combine).  Workspace for the KV splits, sized
 * by kf_attn_exchange_workspace_bytes (NULL: fewer splits).  Waits are bounded as above.
 * No reference counterpart (the reference is single-GPU). */
int kf_attn_fwd_exchange(const void* Q, const void* K, const void* V, void* const* windows, int world, int rank,
                         long long part_stride, float* O, float* Mi, float* Li,
                         int B, int H_q, int H_kv, int S_q, int S_kv, int D,
                         void* workspace, size_t workspace_bytes, void* stream);
size_t kf_attn_exchange_workspace_bytes(int B, int H_q, int H_kv, int S_q, int S_kv, int D);

/* Bytes of workspace the call with these arguments would use (0 if none). */
size_t kf_attn_workspace_bytes(int B, int H_q, int H_kv, int S_q, int S_kv, int D);

/* Zero-fill a workspace before its first use (cudaMemsetAsync on stream). */
int kf_attn_workspace_init(void* workspace, size_t workspace_bytes, void* stream);

/* Execution plan the call would use, for tests and benchmarks:
 *   *path = 0 prefill (tcgen05 kernel) or 1 decode (split-KV kernel);
 *   *n_split = KV splits per (b, h_kv) (decode), *grid_ctas = work items: one CTA
 *   each, except that a prefill whose Q and K/V tiles are all full size launches
 *   min(items, SM count) persistent CTAs that stride over the items. */
int kf_attn_plan(int B, int H_q, int H_kv, int S_q, int S_kv, int D, size_t workspace_bytes,
                 int* path, int* n_split, int* grid_ctas);

/* Blocking, reference-compatible launcher: same arguments and semantics as
 * launch_flash_attn (tests/test_flash_attn.cu:52-113): S_q = S_kv = S,
 * synchronizes `stream` before returning, returns KF_* codes (the C++
 * header kf_attn_compat.h maps them to cudaError_t).  Allocates nothing. */
int kf_launch_flash_attn(const uint16_t* Q, const uint16_t* K, const uint16_t* V, float* O,
                         int B, int S, int H_q, int H_kv, int D, void* stream);

/* Short-query (decode) attention that allocates nothing and takes no workspace.
 * No counterpart in the reference (its launcher cudaMallocs Mi/Li on every
 * call, tests/test_flash_attn.cu:60-70); this entry exists for callers that
 * cannot allocate device memory at call time: serving loops that gave all free
 * device memory to a KV-cache pool at start-up and have no allocator left to
 * call, and latency-bound decode loops that must not call cudaMalloc because
 * it can synchronize the device and stall work queued on other streams.
 *   - Same arguments and results as kf_attn_fwd, for shapes that take the
 *     split-KV decode kernel (H_q/H_kv * S_q <= 64 for D <= 128, <= 32 for
 *     D = 256); other shapes return KF_ERR_INVALID_ARG.
 *   - The split partials and ticket counters live in a fixed 2 MiB array inside
 *     the library, held by every GPU that loads it until the process exits.  The
 *     KV split count is planned to fit it: where kf_attn_fwd with a larger
 *     workspace would split further (many rows at long KV), this call splits
 *     less (same results, possibly slower); nothing is allocated either way.
 *   - The ticket counters start at zero and every launch leaves them at zero
 *     (also after an expired wait), so no call clears the array.
 *   - The first call on a device looks up that array's device address (once per
 *     device, with the device current); make that first call before any stream
 *     capture.
 *   - Every call shares the one array: calls whose kernels overlap on the GPU
 *     (different streams, or different host threads on one device) race and
 *     corrupt each other's results.  Serialize them (one stream). */
int kf_attn_fwd_noalloc(const void* Q, const void* K, const void* V, float* O,
                        int B, int H_q, int H_kv, int S_q, int S_kv, int D, void* stream);

/* ---- device error word / bounded waits ----------------------------------
 * Kernels never spin forever: each wait gives up after a wall-clock limit
 * (default 1 s), records the failure in a per-device error word and unwinds.
 * No reference counterpart (the reference has no waits that can time out). */

/* Synchronizes the current device, returns KF_ERR_DEVICE_TIMEOUT if any
 * kernel recorded an expired wait since the last clear (else KF_OK).
 * clear != 0 resets the word.  *raw (nullable) receives the raw bits. */
int kf_device_error(int clear, unsigned* raw);

/* Set the in-kernel wait limit in nanoseconds (0 restores the default). */
void kf_set_wait_timeout_ns(unsigned long long ns);

/* Launch a one-CTA kernel that waits on a barrier nothing ever signals, with
 * limit timeout_ns, then synchronizes.  Returns KF_ERR_DEVICE_TIMEOUT when the
 * bounded wait expired as designed (and clears the error word): it proves
 * the unwind path without faulting or hanging the GPU. */
int kf_selftest_wait_timeout(unsigned long long timeout_ns, void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* KF_ATTN_H_ */
