// tqk_inputs.cu -- host-side input generator: the reference benches' N(0,1)
// stream, generated in parallel with results identical to the reference's
// sequential generator.
//
// The reference's benches draw every synthetic input from one xorshift64 state
// (seed 88172645463325252) through `uniform_open` / `normal_sample`
// (tools/bench_forward.c:82,199-210; the same in tools/bench.c:102,119-130):
// three shift-xor steps per uniform, the top 24 bits mapped to (0, 1], and one
// Box-Muller cosine branch per normal, from two consecutive uniforms.
//
// That generator is sequential, but its step is linear over GF(2): a 64x64 bit
// matrix T.  Sample i of the normal stream starts from T^(2i) applied to the
// seed, so every thread computes its own start state by square-and-multiply and
// fills a contiguous chunk; the output does not depend on the thread count.
// The float arithmetic is the reference's, evaluated the same way (IEEE single
// precision, no contraction, the C library's logf / cosf / sqrtf), so the values
// are bit-identical to the reference's on the same C library.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "tqk_internal.h"

namespace {

inline uint64_t xs_step(uint64_t x) {
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    return x;
}

// A linear map on 64-bit states: col[i] is the image of bit i.
struct BitMatrix {
    uint64_t col[64];
};

inline uint64_t bm_apply(const BitMatrix &m, uint64_t v) {
    uint64_t r = 0;
    while (v) {
        r ^= m.col[__builtin_ctzll(v)];
        v &= v - 1;
    }
    return r;
}

BitMatrix bm_square(const BitMatrix &m) {
    BitMatrix r;
    for (int i = 0; i < 64; i++) r.col[i] = bm_apply(m, m.col[i]);
    return r;
}

// The state `steps` generator steps after `state`.
uint64_t xs_jump(uint64_t state, uint64_t steps) {
    BitMatrix p;
    for (int i = 0; i < 64; i++) p.col[i] = xs_step(1ull << i);
    while (steps) {
        if (steps & 1) state = bm_apply(p, state);
        steps >>= 1;
        if (steps) p = bm_square(p);
    }
    return state;
}

// One uniform in (0, 1]: the top 24 bits of the next state, plus one, over the
// float the reference writes as 16777217.0f.  That decimal lies halfway between
// two floats and rounds to even, 2^24, in C; nvcc's front end rounds the same
// literal in host code up to 16777218, so the value is written here exactly.
// 2^24 / 2^24 = 1 can occur.
inline float xs_uniform(uint64_t &x) {
    x = xs_step(x);
    return (float)((x >> 40) + 1) / 16777216.0f;
}

inline float xs_normal(uint64_t &x) {
    const float u1 = xs_uniform(x);
    const float u2 = xs_uniform(x);
    return sqrtf(-2.0f * logf(u1)) * cosf(6.2831853f * u2);
}

constexpr size_t kMinChunk = 1 << 16;

template <typename Fill>
int fill_parallel(size_t n, int threads, Fill fill) {
    if (n == 0) return TQK_OK;
    size_t t = threads > 0 ? (size_t)threads : (size_t)std::thread::hardware_concurrency();
    if (t < 1) t = 1;
    if (t > 256) t = 256;
    if (t > (n + kMinChunk - 1) / kMinChunk) t = (n + kMinChunk - 1) / kMinChunk;
    const size_t chunk = (n + t - 1) / t;
    if (t == 1) {
        fill(0, n);
        return TQK_OK;
    }
    std::vector<std::thread> pool;
    bool started = true;
    try {
        pool.reserve(t);
        for (size_t i = 0; i < t; i++) {
            const size_t a = i * chunk, b = a + chunk < n ? a + chunk : n;
            if (a >= b) break;
            pool.emplace_back([=] { fill(a, b); });
        }
    } catch (...) {
        started = false;  // the chunks whose threads did not start stay unfilled
    }
    for (auto &th : pool) th.join();
    return started ? TQK_OK : tqk::fail(TQK_EINVAL, "tqk_fill_*: could not start the worker threads");
}

}  // namespace

extern "C" {

TQK_API uint64_t tqk_xorshift_jump(uint64_t state, uint64_t steps) { return xs_jump(state, steps); }

TQK_API int tqk_fill_normal(uint64_t seed, uint64_t first, float *out, size_t n, float scale, int threads) {
    if (seed == 0 || (!out && n)) return tqk::fail(TQK_EINVAL, "tqk_fill_normal: zero seed or NULL output");
    if (first > (UINT64_MAX >> 1)) return tqk::fail(TQK_EINVAL, "tqk_fill_normal: first sample out of range");
    return fill_parallel(n, threads, [=](size_t a, size_t b) {
        uint64_t x = xs_jump(seed, 2 * (first + a));
        for (size_t i = a; i < b; i++) out[i] = xs_normal(x) * scale;
    });
}

TQK_API int tqk_fill_uniform(uint64_t seed, uint64_t first, float *out, size_t n, int threads) {
    if (seed == 0 || (!out && n)) return tqk::fail(TQK_EINVAL, "tqk_fill_uniform: zero seed or NULL output");
    return fill_parallel(n, threads, [=](size_t a, size_t b) {
        uint64_t x = xs_jump(seed, first + a);
        for (size_t i = a; i < b; i++) out[i] = xs_uniform(x);
    });
}

}  // extern "C"
