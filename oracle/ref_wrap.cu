// oracle/ref_wrap.cu -- C-ABI wrapper around the UNMODIFIED reference sources.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file with the
// reference tree on the include path, so the reference's own
// tests/test_flash_attn.cu (which itself includes kernels/flash_attn.cu) is
// compiled exactly as shipped; nothing from it is copied into this
// repository.  The result, oracle/_ref/libkfref.so, is used
//   * here (no GPU): to produce golden vectors from the reference's own
//     fill_random_f32 (tests/test_utils.h:27-31) and cpu_attn
//     (tests/test_flash_attn.cu:119-169);
//   * on a B200: as the reference CUDA kernel that parity tests compare
//     against (flash_attn_kernel<D>, kernels/flash_attn.cu:384-585), through
//     its own launcher launch_flash_attn (tests/test_flash_attn.cu:52-113)
//     and, for q_len != kv_len, a launch identical in shape to the
//     reference benchmark's launch_once (tests/bench_flash_attn.cu:39-54).

#define main kfref_reference_test_main
#include "test_flash_attn.cu"
#undef main

#include <cstring>

extern "C" {

void kfref_fill_random_f32(float* out, size_t n, float lo, float hi, uint32_t seed) {
    std::vector<float> v(n);
    fill_random_f32(v, lo, hi, seed);
    std::memcpy(out, v.data(), n * sizeof(float));
}

int kfref_cpu_attn(const float* Q, const float* K, const float* V, float* O,
                   int B, int S, int H_q, int H_kv, int D) {
    const size_t qn = static_cast<size_t>(B) * H_q * S * D;
    const size_t kn = static_cast<size_t>(B) * H_kv * S * D;
    std::vector<float> q(Q, Q + qn), k(K, K + kn), v(V, V + kn), o;
    cpu_attn(q, k, v, o, nullptr, B, S, H_q, H_kv, D);
    std::memcpy(O, o.data(), qn * sizeof(float));
    return 0;
}

int kfref_launch_flash_attn(const uint16_t* Q, const uint16_t* K, const uint16_t* V, float* O,
                            int B, int S, int H_q, int H_kv, int D, void* stream) {
    return static_cast<int>(launch_flash_attn(Q, K, V, O, B, S, H_q, H_kv, D,
                                              static_cast<cudaStream_t>(stream)));
}

// General q_len/kv_len launch of the reference kernel (the shape the
// reference benchmark uses for decode).  Mi/Li are caller-provided device
// buffers of B*H_q*q_len floats.  Asynchronous on `stream`.
int kfref_launch_general(const uint16_t* Q, const uint16_t* K, const uint16_t* V, float* O,
                         float* Mi, float* Li, int B, int q_len, int kv_len,
                         int H_q, int H_kv, int D, void* stream) {
    const int bc = select_flash_bc(D);
    if (bc < 0) return static_cast<int>(cudaErrorInvalidValue);
    const size_t smem = flash_smem_bytes_for(bc, D);
    const dim3 grid(B, H_q, (q_len + kFlashBr - 1) / kFlashBr);
    const dim3 block(kFlashWarps * 32);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t err = cudaSuccess;
#define KFREF_LAUNCH(DV)                                                                  \
    do {                                                                                  \
        err = cudaFuncSetAttribute(flash_attn_kernel<DV>,                                 \
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,           \
                                   static_cast<int>(smem));                               \
        if (err != cudaSuccess) return static_cast<int>(err);                             \
        flash_attn_kernel<DV><<<grid, block, smem, s>>>(Q, K, V, O, Mi, Li, B, q_len,     \
                                                        kv_len, H_q, H_kv, bc);          \
    } while (0)
    if (D == 16) KFREF_LAUNCH(16);
    else if (D == 64) KFREF_LAUNCH(64);
    else if (D == 128) KFREF_LAUNCH(128);
    else if (D == 256) KFREF_LAUNCH(256);
    else return static_cast<int>(cudaErrorInvalidValue);
#undef KFREF_LAUNCH
    return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
