/* Exports of the shared synthetic-input generator (see nsrand.h). Built with
 * -ffp-contract=off so the double arithmetic matches numpy exactly. */
#include "nsrand.h"
#include "ns_oracle.h"

void orc_fill_uniform(float* out, size_t n, uint64_t seed, double lo, double hi) {
    nsr_fill_uniform(out, n, seed, lo, hi);
}
void orc_fill_normal(float* out, size_t n, uint64_t seed, double mu, double sd) {
    nsr_fill_normal(out, n, seed, mu, sd);
}
void orc_fill_tokens(float* out, size_t n, uint64_t seed, int64_t vocab) {
    nsr_fill_tokens(out, n, seed, vocab);
}
