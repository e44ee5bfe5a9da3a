/* Deterministic synthetic-input generator shared by the golden-vector
 * harnesses, the C oracle and (as a numpy restatement in
 * neuralscript_b200/synth.py) the Python tests and bench.
 *
 * Element i of stream `seed` is a pure function of (seed, i), so the same
 * arrays can be regenerated anywhere without storing them:
 *   raw(seed, i)     = splitmix64 finaliser of seed + (i + 1) * 0x9E3779B97F4A7C15
 *   unit(seed, i)    = (raw >> 40) * 2^-24                    (exact 24-bit value)
 *   uniform(lo, hi)  = (float)(lo + unit * (hi - lo))          (double arithmetic)
 *   normal(mu, sd)   = (float)(mu + sd * (sum_{j<12} unit(seed, 12 i + j) - 6))
 * The normal is the Irwin-Hall sum of twelve uniforms: variance 1, and every
 * intermediate is exact in double, so C and numpy agree bit for bit.
 * Files including this header must be built with -ffp-contract=off.
 */
#ifndef NS_ORACLE_NSRAND_H
#define NS_ORACLE_NSRAND_H

#include <stddef.h>
#include <stdint.h>

static inline uint64_t nsr_raw(uint64_t seed, uint64_t i) {
    uint64_t z = seed + (i + 1ull) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static inline double nsr_unit(uint64_t seed, uint64_t i) {
    return (double)(nsr_raw(seed, i) >> 40) * (1.0 / 16777216.0);
}

static inline void nsr_fill_uniform(float* out, size_t n, uint64_t seed, double lo, double hi) {
    const double w = hi - lo;
    for (size_t i = 0; i < n; i++) {
        double t = nsr_unit(seed, i) * w;
        out[i] = (float)(lo + t);
    }
}

static inline void nsr_fill_normal(float* out, size_t n, uint64_t seed, double mu, double sd) {
    for (size_t i = 0; i < n; i++) {
        double s = 0.0;
        for (int j = 0; j < 12; j++) s += nsr_unit(seed, 12ull * i + (uint64_t)j);
        double t = sd * (s - 6.0);
        out[i] = (float)(mu + t);
    }
}

/* Integer tokens drawn uniformly from [0, vocab), delivered as fp32 ids the
 * way the reference ABI carries them. */
static inline void nsr_fill_tokens(float* out, size_t n, uint64_t seed, int64_t vocab) {
    for (size_t i = 0; i < n; i++)
        out[i] = (float)(int64_t)(nsr_unit(seed, i) * (double)vocab);
}

#endif
