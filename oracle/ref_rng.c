/* ref_rng.c -- TEST INFRASTRUCTURE ONLY (built into oracle/_ref/libtqref_rng.so).
 *
 * Exposes the reference bench's own input generator, the static xorshift64 +
 * Box-Muller `normal_sample` of tools/bench_forward.c:82,199-210, by compiling
 * that file in place (its main renamed) inside this translation unit, so that the
 * restated generator of the library (tqk_fill_normal) can be checked against the
 * reference's code itself rather than against a second restatement. */
#define main tqref_bench_forward_main
#include "tools/bench_forward.c"
#undef main

/* n samples of the reference's normal_sample() from the generator state *state
 * (the reference starts at 88172645463325252); *state is advanced past them. */
void tqref_normal_fill(uint64_t *state, float *out, size_t n) {
    g_rng = *state;
    for (size_t i = 0; i < n; i++) out[i] = normal_sample();
    *state = g_rng;
}

/* The same generator's uniform_open() values. */
void tqref_uniform_fill(uint64_t *state, float *out, size_t n) {
    g_rng = *state;
    for (size_t i = 0; i < n; i++) out[i] = uniform_open();
    *state = g_rng;
}
