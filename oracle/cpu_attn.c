/*
 * oracle/cpu_attn.c -- CPU restatement of the reference's C++ test oracle.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links or calls
 * this file; only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg load it, and only as the checker.
 *
 * What it restates (sviraaj/kernelfoundry):
 *   - kfo_mt19937_uniform_f32: tests/test_utils.h:27-31 (fill_random_f32),
 *     i.e. std::mt19937(seed) fed through libstdc++'s
 *     std::uniform_real_distribution<float>(lo, hi).  The generator is the
 *     published MT19937 algorithm (Matsumoto & Nishimura 1998, init_genrand
 *     seeding); the float mapping is libstdc++'s generate_canonical<float,24>
 *     (one 32-bit draw, converted to float with round-to-nearest, divided by
 *     2^32, clamped below 1) followed by u * (hi - lo) + lo in float.
 *   - kfo_cpu_attn: tests/test_flash_attn.cu:119-169 (cpu_attn), the fp32
 *     scaled-dot-product attention used by the reference's 18-case harness,
 *     generalised to S_q != S_kv (the reference uses one S for both).
 *     Loop order, accumulation order and float types follow the reference so
 *     that results are bit-identical when compiled without FMA contraction.
 *
 * Pinning: tests/test_oracle.py checks both functions against vectors that
 * tests/golden/make_golden.py produced by running the reference's own
 * fill_random_f32 and cpu_attn (compiled from the reference sources).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

/* ---- MT19937 (published algorithm) ------------------------------------- */
typedef struct {
    uint32_t mt[624];
    int idx;
} kfo_mt19937;

static void mt_seed(kfo_mt19937* s, uint32_t seed) {
    s->mt[0] = seed;
    for (int i = 1; i < 624; ++i) {
        uint32_t prev = s->mt[i - 1];
        s->mt[i] = 1812433253u * (prev ^ (prev >> 30)) + (uint32_t)i;
    }
    s->idx = 624;
}

static void mt_twist(kfo_mt19937* s) {
    for (int i = 0; i < 624; ++i) {
        uint32_t y = (s->mt[i] & 0x80000000u) | (s->mt[(i + 1) % 624] & 0x7fffffffu);
        uint32_t v = s->mt[(i + 397) % 624] ^ (y >> 1);
        if (y & 1u) v ^= 0x9908b0dfu;
        s->mt[i] = v;
    }
    s->idx = 0;
}

static uint32_t mt_next(kfo_mt19937* s) {
    if (s->idx >= 624) mt_twist(s);
    uint32_t y = s->mt[s->idx++];
    y ^= (y >> 11);
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= (y >> 18);
    return y;
}

/* One uniform float in [lo, hi) exactly as libstdc++ maps a 32-bit draw. */
static float canonical_to_range(uint32_t draw, float lo, float hi) {
    float u = (float)draw / 4294967296.0f;
    if (u >= 1.0f) u = nextafterf(1.0f, 0.0f);
    return u * (hi - lo) + lo;
}

void kfo_mt19937_uniform_f32(float* out, size_t n, float lo, float hi, uint32_t seed) {
    kfo_mt19937 s;
    mt_seed(&s, seed);
    for (size_t i = 0; i < n; ++i) out[i] = canonical_to_range(mt_next(&s), lo, hi);
}

void kfo_mt19937_raw(uint32_t* out, size_t n, uint32_t seed) {
    kfo_mt19937 s;
    mt_seed(&s, seed);
    for (size_t i = 0; i < n; ++i) out[i] = mt_next(&s);
}

/* ---- fp32 attention (reference cpu_attn, S_q/S_kv generalised) --------- */
/* Q [B,H_q,S_q,D], K/V [B,H_kv,S_kv,D], O [B,H_q,S_q,D]; h_kv = h / (H_q/H_kv).
 * scores_scratch must hold S_kv floats.  Returns 0, or -1 on bad shapes. */
int kfo_cpu_attn(const float* Q, const float* K, const float* V, float* O,
                 int B, int S_q, int S_kv, int H_q, int H_kv, int D,
                 float* scores_scratch) {
    if (B < 0 || S_q < 0 || S_kv <= 0 || H_q <= 0 || H_kv <= 0 || D <= 0) return -1;
    if (H_q % H_kv != 0) return -1;
    const float scale = 1.0f / sqrtf((float)D);
    const int gqa_ratio = H_q / H_kv;
    float* scores = scores_scratch;
    memset(O, 0, sizeof(float) * (size_t)B * H_q * S_q * D);
    for (int b = 0; b < B; ++b) {
        for (int h = 0; h < H_q; ++h) {
            const int h_kv = h / gqa_ratio;
            for (int i = 0; i < S_q; ++i) {
                const float* q_row = Q + (((size_t)b * H_q + h) * S_q + i) * D;
                for (int j = 0; j < S_kv; ++j) {
                    const float* k_row = K + (((size_t)b * H_kv + h_kv) * S_kv + j) * D;
                    float dot = 0.0f;
                    for (int d = 0; d < D; ++d) dot += q_row[d] * k_row[d];
                    scores[j] = dot * scale;
                }
                /* std::max_element: first maximum, strict '<' comparisons */
                float maxval = scores[0];
                for (int j = 1; j < S_kv; ++j)
                    if (maxval < scores[j]) maxval = scores[j];
                float sumexp = 0.0f;
                for (int j = 0; j < S_kv; ++j) {
                    scores[j] = expf(scores[j] - maxval);
                    sumexp += scores[j];
                }
                for (int j = 0; j < S_kv; ++j) scores[j] /= sumexp;
                float* o_row = O + (((size_t)b * H_q + h) * S_q + i) * D;
                for (int j = 0; j < S_kv; ++j) {
                    const float* v_row = V + (((size_t)b * H_kv + h_kv) * S_kv + j) * D;
                    for (int d = 0; d < D; ++d) o_row[d] += scores[j] * v_row[d];
                }
            }
        }
    }
    return 0;
}
