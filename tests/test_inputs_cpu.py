"""The synthetic-input generator of the library (tqk_fill_normal / tqk_fill_uniform,
host code, no GPU) against the reference benches' own generator: the static
uniform_open / normal_sample of tools/bench_forward.c:82,199-210, compiled in place
into oracle/_ref/libtqref_rng.so (oracle/ref_rng.c).  The values must be identical
bit for bit, from the seed and from any later position, on any thread count."""
import ctypes
import os

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_RNG = os.path.join(ROOT, "oracle", "_ref", "libtqref_rng.so")
MASK = (1 << 64) - 1


def _ref_stream(kind: str, n: int, state: int):
    if not os.path.exists(REF_RNG):
        pytest.skip("oracle/_ref/libtqref_rng.so not built (needs the reference tree at build time)")
    lib = ctypes.CDLL(REF_RNG)
    st = ctypes.c_uint64(state)
    out = np.empty(n, np.float32)
    fn = lib.tqref_normal_fill if kind == "normal" else lib.tqref_uniform_fill
    fn(ctypes.byref(st), ctypes.c_void_p(out.ctypes.data), ctypes.c_size_t(n))
    return out, st.value


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_uniforms_follow_the_generator_in_python():
    """No reference build needed: the first uniforms from the xorshift64 steps written out
    in Python (three shift-xors, the top 24 bits plus one, over 2^24)."""
    from tailorquantkernel_b200 import tqk
    x, want = tqk.REF_SEED, []
    for _ in range(64):
        x ^= (x << 13) & MASK
        x ^= x >> 7
        x ^= (x << 17) & MASK
        want.append(np.float32((x >> 40) + 1) / np.float32(1 << 24))
    assert np.array_equal(_bits(tqk.fill_uniform(0, 64, threads=1)), _bits(np.array(want, np.float32)))
    assert tqk.tqk_xorshift_jump(tqk.REF_SEED, 64) == x


@pytest.mark.parametrize("threads", [1, 3, 0])
def test_normal_stream_is_the_reference_generator(threads):
    from tailorquantkernel_b200 import tqk
    n = 1_500_000
    want, state_after = _ref_stream("normal", n, tqk.REF_SEED)
    got = tqk.fill_normal(0, n, threads=threads)
    assert np.array_equal(_bits(got), _bits(want))
    # a window from the middle (the threads' jump-ahead), and the state after n samples
    assert np.array_equal(_bits(tqk.fill_normal(654_321, 70_001, threads=threads)), _bits(want[654_321:724_322]))
    assert tqk.tqk_xorshift_jump(tqk.REF_SEED, 2 * n) == state_after
    # a scale is one float multiply of each sample (the reference's weights: normal_sample() * 0.02f)
    assert np.array_equal(_bits(tqk.fill_normal(0, 1000, scale=0.02)), _bits(want[:1000] * np.float32(0.02)))


def test_uniform_stream_and_other_seeds():
    from tailorquantkernel_b200 import tqk
    want, _ = _ref_stream("uniform", 300_000, tqk.REF_SEED)
    assert np.array_equal(_bits(tqk.fill_uniform(0, 300_000, threads=4)), _bits(want))
    assert np.array_equal(_bits(tqk.fill_uniform(123_457, 1000)), _bits(want[123_457:124_457]))
    assert want.min() > 0 and want.max() <= 1
    seed = tqk.tqk_xorshift_jump(12345, 1000)
    want2, _ = _ref_stream("normal", 200_000, seed)
    assert np.array_equal(_bits(tqk.fill_normal(0, 200_000, seed=seed)), _bits(want2))


def test_guards():
    from tailorquantkernel_b200 import tqk
    assert tqk.tqk_fill_normal(0, 0, None, 10, 1.0, 1) == tqk.EINVAL  # a zero seed never leaves zero
    assert tqk.tqk_fill_normal(tqk.REF_SEED, 0, None, 10, 1.0, 1) == tqk.EINVAL
    assert tqk.tqk_fill_normal(tqk.REF_SEED, 0, None, 0, 1.0, 1) == tqk.OK  # nothing to fill
    assert tqk.tqk_fill_uniform(0, 0, None, 10, 1) == tqk.EINVAL
