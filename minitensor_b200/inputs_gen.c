/* inputs_gen.c -- seeded synthetic inputs with the exact values a C++ program gets from
 * std::mt19937(seed) through libstdc++'s std::normal_distribution<float>.
 *
 * The reference fills its tensors this way (include/Module.hpp:226-232 for the first
 * Conv2D's He-normal weights, :96-105 for Linear), and the workload configurations draw
 * their normal inputs the same way, so the benchmark sees the reference's own numbers.
 *
 * Generator: MT19937 (Matsumoto & Nishimura 1998) with the init_genrand seeding that
 * std::mt19937(seed) uses. Canonical float: one 32-bit draw x, u = float(x) / 2^32, clamped
 * below 1 (libstdc++'s generate_canonical<float, 24>: 24 bits need one 32-bit draw).
 * Normal: the Marsaglia polar method as libstdc++ applies it -- draw x, y = 2u - 1 until
 * 0 < x^2 + y^2 <= 1, m = sqrt(-2 log(r2) / r2), return y*m and keep x*m for the next
 * call; every value is then scaled as v * stddev + mean. All arithmetic is float, as in
 * normal_distribution<float>, and log is the C library's logf -- the function std::log(float)
 * calls -- because a correctly rounded log differs from it in the last bit for about one
 * input in 5000. Built with -ffp-contract=off (no fused multiply-add), like the reference's
 * x86-64 build.
 *
 * Host-only data generation; no device code.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>

enum { MT_N = 624, MT_M = 397 };

typedef struct {
    uint32_t s[MT_N];
    int i;
} mt19937_state;

static void mt_seed(mt19937_state* g, uint32_t seed) {
    g->s[0] = seed;
    for (int i = 1; i < MT_N; ++i) g->s[i] = 1812433253u * (g->s[i - 1] ^ (g->s[i - 1] >> 30)) + (uint32_t)i;
    g->i = MT_N;
}

static uint32_t mt_next(mt19937_state* g) {
    if (g->i >= MT_N) {
        for (int k = 0; k < MT_N; ++k) {
            const uint32_t y = (g->s[k] & 0x80000000u) | (g->s[(k + 1) % MT_N] & 0x7fffffffu);
            g->s[k] = g->s[(k + MT_M) % MT_N] ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
        }
        g->i = 0;
    }
    uint32_t y = g->s[g->i++];
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return y;
}

static float canonical(mt19937_state* g) {
    const float u = (float)mt_next(g) / 4294967296.0f;
    return u >= 1.0f ? nextafterf(1.0f, 0.0f) : u;
}

/* out[0..n) = the first n values of normal_distribution<float>(mean, stddev) on mt19937(seed). */
void mtin_normal_f32(uint32_t seed, float mean, float stddev, float* out, size_t n) {
    mt19937_state g;
    mt_seed(&g, seed);
    int have_saved = 0;
    float saved = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        float v;
        if (have_saved) {
            have_saved = 0;
            v = saved;
        } else {
            float x, y, r2;
            do {
                x = 2.0f * canonical(&g) - 1.0f;
                y = 2.0f * canonical(&g) - 1.0f;
                r2 = x * x + y * y;
            } while (r2 > 1.0f || r2 == 0.0f);
            const float mult = sqrtf(-2.0f * logf(r2) / r2);
            saved = x * mult;
            have_saved = 1;
            v = y * mult;
        }
        out[i] = v * stddev + mean;
    }
}

/* out[0..n) = the first n values of uniform_real_distribution<float>(lo, hi) on mt19937(seed). */
void mtin_uniform_f32(uint32_t seed, float lo, float hi, float* out, size_t n) {
    mt19937_state g;
    mt_seed(&g, seed);
    for (size_t i = 0; i < n; ++i) out[i] = canonical(&g) * (hi - lo) + lo;
}
