// legacy18.cu -- the reference's 18-case end-to-end harness, driven through
// the drop-in header include/kf_attn_compat.h.
//
// Same cases, generator, oracle and tolerance as sviraaj/kernelfoundry's
// tests/test_flash_attn.cu:290-326: inputs are std::mt19937(seed) +
// std::uniform_real_distribution<float>(-1, 1) with seeds s, s+1, s+2
// (tests/test_utils.h:27-31); the GPU gets their round-to-nearest fp16
// copies; the check is max-abs error <= 5e-2 against an fp32 CPU SDPA on the
// un-rounded inputs (the C restatement of cpu_attn in oracle/cpu_attn.c).
// The only change a maintainer makes to their harness is the include: the
// launcher call `launch_flash_attn(d_Q, d_K, d_V, d_O, B, S, H_q, H_kv, D)`
// is untouched.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <random>
#include <vector>

#include "kf_attn_compat.h"

extern "C" int kfo_cpu_attn(const float* Q, const float* K, const float* V, float* O, int B, int S_q, int S_kv,
                            int H_q, int H_kv, int D, float* scores_scratch);

namespace {

constexpr float kTol = 5e-2f;

#define CHECK_CUDA(x)                                                                      \
    do {                                                                                   \
        cudaError_t e_ = (x);                                                              \
        if (e_ != cudaSuccess) {                                                           \
            std::fprintf(stderr, "CUDA error %s at %s:%d\n", cudaGetErrorString(e_), __FILE__, __LINE__); \
            std::exit(2);                                                                  \
        }                                                                                  \
    } while (0)

void uniform_fill(std::vector<float>& v, float lo, float hi, uint32_t seed) {
    std::mt19937 gen(seed);
    std::uniform_real_distribution<float> dist(lo, hi);
    for (auto& x : v) x = dist(gen);
}

std::vector<uint16_t> to_half_bits(const std::vector<float>& v) {
    std::vector<uint16_t> out(v.size());
    for (size_t i = 0; i < v.size(); ++i) {
        __half h = __float2half(v[i]);
        out[i] = *reinterpret_cast<uint16_t*>(&h);
    }
    return out;
}

bool run_case(int B, int S, int H_q, int H_kv, int D, uint32_t seed) {
    const size_t qn = static_cast<size_t>(B) * H_q * S * D, kn = static_cast<size_t>(B) * H_kv * S * D;
    std::vector<float> q(qn), k(kn), v(kn), ref(qn), got(qn), scratch(S);
    uniform_fill(q, -1.f, 1.f, seed);
    uniform_fill(k, -1.f, 1.f, seed + 1);
    uniform_fill(v, -1.f, 1.f, seed + 2);
    kfo_cpu_attn(q.data(), k.data(), v.data(), ref.data(), B, S, S, H_q, H_kv, D, scratch.data());
    auto q16 = to_half_bits(q), k16 = to_half_bits(k), v16 = to_half_bits(v);
    uint16_t *dQ, *dK, *dV;
    float* dO;
    CHECK_CUDA(cudaMalloc(&dQ, qn * 2));
    CHECK_CUDA(cudaMalloc(&dK, kn * 2));
    CHECK_CUDA(cudaMalloc(&dV, kn * 2));
    CHECK_CUDA(cudaMalloc(&dO, qn * 4));
    CHECK_CUDA(cudaMemcpy(dQ, q16.data(), qn * 2, cudaMemcpyHostToDevice));
    CHECK_CUDA(cudaMemcpy(dK, k16.data(), kn * 2, cudaMemcpyHostToDevice));
    CHECK_CUDA(cudaMemcpy(dV, v16.data(), kn * 2, cudaMemcpyHostToDevice));
    CHECK_CUDA(launch_flash_attn(dQ, dK, dV, dO, B, S, H_q, H_kv, D));
    CHECK_CUDA(cudaMemcpy(got.data(), dO, qn * 4, cudaMemcpyDeviceToHost));
    cudaFree(dQ);
    cudaFree(dK);
    cudaFree(dV);
    cudaFree(dO);
    float err = 0.f;
    for (size_t i = 0; i < qn; ++i) err = std::fmax(err, std::fabs(ref[i] - got[i]));
    const bool ok = err <= kTol;
    std::printf("  B=%d S=%d H_q=%d H_kv=%d D=%d ... %s (max_abs_err=%g)\n", B, S, H_q, H_kv, D,
                ok ? "PASS" : "FAIL", err);
    return ok;
}

}  // namespace

int main() {
    std::printf("=== kernelfoundry-b200: reference harness cases via launch_flash_attn ===\n");
    const int cases[18][6] = {
        {1, 16, 1, 1, 16, 100},   {1, 16, 1, 1, 64, 101},  {1, 64, 1, 1, 128, 102}, {1, 17, 1, 1, 128, 103},
        {1, 129, 1, 1, 128, 202}, {1, 255, 1, 1, 128, 203}, {1, 256, 1, 1, 64, 200}, {1, 256, 1, 1, 128, 201},
        {1, 64, 4, 2, 64, 300},   {1, 64, 8, 2, 64, 301},   {1, 64, 32, 8, 128, 302}, {1, 64, 40, 8, 128, 303},
        {1, 64, 8, 1, 128, 304},  {1, 16, 1, 1, 256, 305},  {2, 64, 4, 4, 64, 400},  {2, 128, 4, 2, 128, 401},
        {3, 33, 4, 4, 128, 402},  {2, 129, 32, 8, 128, 403},
    };
    int failed = 0;
    for (const auto& c : cases)
        if (!run_case(c[0], c[1], c[2], c[3], c[4], static_cast<uint32_t>(c[5]))) ++failed;
    if (failed) {
        std::printf("%d case(s) FAILED\n", failed);
        return 1;
    }
    std::printf("All 18 cases PASSED.\n");
    return 0;
}
