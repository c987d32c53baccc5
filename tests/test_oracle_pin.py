"""Pins the oracle (CPU, no GPU needed).

The scalar restatement oracle/tq_oracle.c must reproduce, bit for bit, the
golden fixtures that tests/golden/make_golden.py generated from the reference's
own scalar build, and -- where oracle/_ref was built from the reference tree --
the reference build itself on fresh inputs.
"""
import os

import numpy as np
import pytest

import oracle
from _cases import (decode_case, digest, head_inputs, layer_inputs, matmul_inputs, norm_rope_inputs,
                    prefill_inputs, quant_edge_rows, sweep_inputs, tolerance_ok)

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def port():
    if not oracle.available("port"):
        oracle.build()
    return oracle.Oracle("port")


def _load(name):
    return np.load(os.path.join(GOLDEN, name))


def test_quantiser_golden(port):
    g = _load("quant_edge.npz")
    x = quant_edge_rows(np.random.default_rng(1))
    assert np.array_equal(x.view(np.uint32), g["x"].view(np.uint32))
    assert np.array_equal(port.quantize_rows(x), g["blocks"])


def _decode_cases():
    g = _load("decode.npz")
    return sorted({k.split("__")[0] for k in g.files})


@pytest.mark.parametrize("name", _decode_cases())
def test_decode_golden(port, name):
    g = _load("decode.npz")
    seed, nq, nkv, hd, mt, pos, of, rp = (int(v) for v in g[f"{name}__params"])
    kf, vf, q = decode_case(seed, nq, nkv, hd, mt, pos + 1, outlier_frac=of / 1e6, rope_pos=None if rp < 0 else rp)
    assert digest(kf, vf, q) == str(g[f"{name}__in_sha"]), "input stream changed"
    kp, vp = port.quantize_rows(kf), port.quantize_rows(vf)
    assert digest(kp, vp) == str(g[f"{name}__planes_sha"])
    out = port.attend(kp, vp, nq, nkv, hd, mt, pos, q)
    assert np.array_equal(out, g[f"{name}__out"])


def test_prefill_golden(port):
    g = _load("prefill.npz")
    seed, nq, nkv, hd, mt, pos0, n = (int(v) for v in g["params"])
    kf, vf, qn, kn, vn = prefill_inputs(seed, nq, nkv, hd, mt, pos0, n)
    assert digest(kf, vf, qn, kn, vn) == str(g["in_sha"])
    kp, vp = port.quantize_rows(kf), port.quantize_rows(vf)
    out = port.prefill(kp, vp, nq, nkv, hd, mt, pos0, n, qn, kn, vn)
    assert np.array_equal(out, g["out"])
    assert np.array_equal(kp[:, pos0:pos0 + n], g["kp"]) and np.array_equal(vp[:, pos0:pos0 + n], g["vp"])


def test_prefill_tc_golden(port):
    """The restatement reproduces the reference's attention_layer_batch chunks on the tensor-core
    prefill's shapes (head_dim 128, groups 1/2/4/8, a chunk at position 0, x30 scores, x8 outliers)
    bit for bit."""
    g = _load("prefill_tc.npz")
    names = sorted({k.split("__")[0] for k in g.files})
    assert len(names) == 8
    for name in names:
        seed, nq, nkv, hd, mt, pos0, n, qs, of = (int(v) for v in g[f"{name}__params"])
        kf, vf, qn, kn, vn = prefill_inputs(seed, nq, nkv, hd, mt, pos0, n, float(qs), of / 1e6)
        assert digest(kf, vf, qn, kn, vn) == str(g[f"{name}__in_sha"]), name
        kp, vp = port.quantize_rows(kf), port.quantize_rows(vf)
        out = port.prefill(kp, vp, nq, nkv, hd, mt, pos0, n, qn, kn, vn).reshape(n, nq * hd)
        assert np.array_equal(out, g[f"{name}__out"]), name
        assert np.array_equal(kp[:, pos0:pos0 + n], g[f"{name}__kp"]), name
        assert np.array_equal(vp[:, pos0:pos0 + n], g[f"{name}__vp"]), name


def test_ops_sweep_golden(port):
    g = _load("ops_sweep.npz")
    keys = sorted({k.split("__")[0] for k in g.files})
    assert len(keys) == 24
    for key in keys:
        gg, n, hd = (int(p[1:] if p[0] == "g" or p[0] == "n" else p[2:]) for p in key.split("_"))
        nb = hd // 32
        qf, kf, vf, w = sweep_inputs(gg, n, hd)
        qb, kb, vb = port.quantize_rows(qf), port.quantize_rows(kf), port.quantize_rows(vf)
        assert digest(qb, kb, vb, w) == str(g[key + "__in_sha"])
        scale = float(np.float32(1.0) / np.sqrt(np.float32(hd)))
        sc = port.attn_scores(qb, gg, kb, n, nb, scale, n + 4).reshape(gg, n + 4)
        assert np.array_equal(sc[:, :n], g[key + "__scores"]), key
        assert np.isnan(sc[:, n:]).all(), "scores written past n"
        acc = port.attn_accum(w, n + 4, gg, vb, n, nb, hd + 8).reshape(gg, hd + 8)
        assert np.array_equal(acc[:, :hd], g[key + "__accum"]), key
        assert np.isnan(acc[:, hd:]).all(), "accum written past head_dim"


def test_head_q8_golden(port):
    g = _load("head_q8.npz")
    for hd, n, seed in ((32, 1, 60), (128, 100, 70), (128, 16, 90)):
        q, kf, vf = head_inputs(hd, n, seed)
        kb, vb = port.quantize_rows(kf), port.quantize_rows(vf)
        key = f"hd{hd}_n{n}_s{seed}"
        assert digest(q, kb, vb) == str(g[key + "__in_sha"])
        o, qq, sc = port.attention_head(q, kb, vb, n, hd)
        assert np.array_equal(o, g[key + "__out"])
        assert np.array_equal(qq, g[key + "__qq"])
        assert np.array_equal(sc, g[key + "__scores"])


def test_quantiser_against_reference_build(port):
    if not oracle.available("ref_scalar"):
        pytest.skip("oracle/_ref not built (needs the reference tree)")
    ref = oracle.Oracle("ref_scalar")
    rng = np.random.default_rng(123)
    x = np.concatenate([quant_edge_rows(rng, 256),
                        rng.standard_normal((200, 256), dtype=np.float32) * np.float32(1e-3),
                        (rng.integers(-300, 300, (64, 256)) / 2).astype(np.float32)])
    assert np.array_equal(port.quantize_rows(x), ref.quantize_rows(x))


@pytest.mark.parametrize("shape", [(32, 8, 128, 300, 257), (16, 2, 64, 90, 33), (12, 4, 32, 40, 1)])
def test_attend_against_reference_build(port, shape):
    if not oracle.available("ref_scalar"):
        pytest.skip("oracle/_ref not built (needs the reference tree)")
    ref = oracle.Oracle("ref_scalar")
    nq, nkv, hd, mt, n = shape
    kf, vf, q = decode_case(7 + n, nq, nkv, hd, mt, n)
    kp, vp = port.quantize_rows(kf), port.quantize_rows(vf)
    a = port.attend(kp, vp, nq, nkv, hd, mt, n - 1, q)
    b = ref.attend(kp, vp, nq, nkv, hd, mt, n - 1, q)
    assert np.array_equal(a, b)


def test_avx2_baseline_matches_oracle():
    """The timed CPU baseline (reference AVX2 build) computes the same attention."""
    if not oracle.available("ref_avx2"):
        pytest.skip("oracle/_ref not built (needs the reference tree)")
    avx = oracle.Oracle("ref_avx2")
    g = np.load(os.path.join(GOLDEN, "decode.npz"))
    seed, nq, nkv, hd, mt, pos, _, _ = (int(v) for v in g["cfg1__params"])
    kf, vf, q = decode_case(seed, nq, nkv, hd, mt, pos + 1)
    kp, vp = avx.quantize_rows(kf), avx.quantize_rows(vf)
    out = avx.attend(kp, vp, nq, nkv, hd, mt, pos, q, threads=4)
    ok, max_abs, rel = tolerance_ok(out, g["cfg1__out"], 1e-5, 1e-5)
    assert ok, (max_abs, rel)


def test_prefill_equals_sequential_decode(port):
    """attention_layer_batch semantics: a chunk equals per-token store + attend."""
    nq, nkv, hd, mt, pos0, n = 8, 2, 64, 48, 20, 7
    kf, vf, qn, kn, vn = prefill_inputs(5, nq, nkv, hd, mt, pos0, n)
    kp, vp = port.quantize_rows(kf), port.quantize_rows(vf)
    kp2, vp2 = kp.copy(), vp.copy()
    out = port.prefill(kp, vp, nq, nkv, hd, mt, pos0, n, qn, kn, vn).reshape(n, -1)
    for i in range(n):
        assert port.store_kv(kp2, vp2, nkv, hd, mt, pos0 + i, kn[i], vn[i]) == 0
        assert np.array_equal(port.attend(kp2, vp2, nq, nkv, hd, mt, pos0 + i, qn[i]), out[i])
    assert np.array_equal(kp, kp2) and np.array_equal(vp, vp2)


def test_store_kv_rejects_bad_pos(port):
    kp = np.full((2, 4, 36), 7, np.uint8)
    vp = kp.copy()
    k = np.ones(64, np.float32)
    for pos in (-1, 4, 9):
        assert port.store_kv(kp, vp, 2, 32, 4, pos, k, k) == -1
    assert (kp == 7).all() and (vp == 7).all()


# name: (seed, n_items, n_q, n_kv, hd, first_pos, theta, eps, per_item_weights, norm); mirrors
# NORM_ROPE_CASES of tests/golden/make_golden.py.
NORM_ROPE = {
    "qwen3_like": (41, 1, 32, 8, 128, 4096, 1000000.0, 1e-6, False, True),
    "llama3_rope_only": (42, 1, 32, 8, 128, 4096, 500000.0, 1e-5, False, False),
    "batch3_hd64": (43, 3, 6, 2, 64, 17, 10000.0, 1e-6, True, True),
}


@pytest.mark.parametrize("name", sorted(NORM_ROPE))
def test_norm_rope_golden(port, name):
    """rmsnorm + rope (model/rmsnorm.c:4-19, model/rope.c:4-22) bit-exact with the reference's outputs."""
    g = _load("norm_rope.npz")
    seed, items, nq, nkv, hd, p0, theta, eps, per_item, norm = NORM_ROPE[name]
    q, k, qw, kw = norm_rope_inputs(seed, items, nq, nkv, hd, per_item)
    assert digest(q, k, qw, kw) == str(g[name + "__in_sha"])
    for it in range(items):
        c, s = port.rope_table(hd, p0 + it, theta)
        assert np.array_equal(c, g[name + "__cos"][it]) and np.array_equal(s, g[name + "__sin"][it])
        wi = it if per_item else 0
        qo = port.qk_norm_rope(q[it], nq, hd, qw[wi] if norm else None, eps, c, s)
        ko = port.qk_norm_rope(k[it], nkv, hd, kw[wi] if norm else None, eps, c, s)
        assert np.array_equal(qo.view(np.uint32), g[name + "__q"][it].view(np.uint32))
        assert np.array_equal(ko.view(np.uint32), g[name + "__k"][it].view(np.uint32))


def test_norm_rope_against_reference_build(port):
    if not oracle.available("ref_scalar"):
        pytest.skip("oracle/_ref not built (needs the reference tree)")
    ref = oracle.Oracle("ref_scalar")
    rng = np.random.default_rng(5)
    for hd, pos, theta in ((32, 0, 10000.0), (128, 131071, 500000.0), (256, 777, 1000000.0)):
        c, s = port.rope_table(hd, pos, theta)
        cr, sr = ref.rope_table(hd, pos, theta)
        assert np.array_equal(c, cr) and np.array_equal(s, sr)
        x = rng.standard_normal((5, hd), dtype=np.float32) * np.float32(50.0)
        x[0] = 0.0                       # rms = sqrt(eps)
        x[1, ::3] = np.float32(3e18)     # sum of squares overflows to inf: output 0 * w
        w = rng.standard_normal(hd, dtype=np.float32)
        a = port.qk_norm_rope(x, 5, hd, w, 1e-6, c, s)
        b = ref.qk_norm_rope(x, 5, hd, w, 1e-6, cr, sr)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


# (rows, cols, x kind) of tests/golden/make_golden.py MATMUL_CASES, seeds 500 + index
MATMUL_CASES = [(rows, cols, "random") for rows, cols in
                ((256, 512), (7, 64), (10, 32), (1027, 96), (1024, 1024), (3072, 1024), (1024, 3072))] + \
               [(256, 512, "constant"), (256, 512, "zero")]


@pytest.mark.parametrize("i", range(len(MATMUL_CASES)))
@pytest.mark.parametrize("fmt", ["8", "4"])
def test_matmul_golden(port, i, fmt):
    """pack_matrix + matmul_q{8,4}_scalar (packer/packer.c, kernel/q8_scalar.c, q4_scalar.c)
    bit-exact with the reference's outputs on the reference test's shapes."""
    rows, cols, kind = MATMUL_CASES[i]
    g = _load("matmul.npz")
    key = f"{rows}x{cols}_{kind}"
    w, x = matmul_inputs(500 + i, rows, cols, kind)
    assert digest(w, x) == str(g[key + "__in_sha"])
    wp = port.pack_matrix(w, fmt)
    assert digest(wp) == str(g[f"{key}__q{fmt}_packed_sha"])
    y = port.matmul(wp, fmt, port.quantize_rows(x[None])[0], rows, cols)
    assert np.array_equal(y.view(np.uint32), g[f"{key}__q{fmt}_y"].view(np.uint32))
    if kind == "zero":
        assert not np.any(y)


def test_matmul_against_reference_build(port):
    if not oracle.available("ref_scalar"):
        pytest.skip("oracle/_ref not built (needs the reference tree)")
    ref = oracle.Oracle("ref_scalar")
    rng = np.random.default_rng(77)
    for rows, cols in ((33, 128), (5, 4096)):
        w = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(3.0)
        w[0, :32] = 0.0  # an all-zero block: scale 1.0
        x = rng.standard_normal(cols, dtype=np.float32)
        xq = port.quantize_rows(x[None])[0]
        for fmt in "84":
            wp = port.pack_matrix(w, fmt)
            assert np.array_equal(wp, ref.pack_matrix(w, fmt))
            assert np.array_equal(port.matmul(wp, fmt, xq, rows, cols).view(np.uint32),
                                  ref.matmul(wp, fmt, xq, rows, cols).view(np.uint32))


# tests/golden/make_golden.py LAYER_CASES
LAYER_CASES = {
    "small_g4": (61, 8, 2, 64, 256, 40, 25, 1000000.0, 1e-6),
    "llama_heads": (62, 32, 8, 128, 512, 70, 64, 500000.0, 1e-5),
}


@pytest.mark.parametrize("name", sorted(LAYER_CASES))
@pytest.mark.parametrize("fmt", ["8", "4"])
def test_attention_layer_golden(port, name, fmt):
    """The port's composition of attention_layer's steps equals the reference's attention_layer
    bit for bit: output and appended cache rows."""
    seed, nq, nkv, hd, hidden, mt, pos, theta, eps = LAYER_CASES[name]
    g = _load("layer.npz")
    key = f"{name}_q{fmt}"
    w, qn, kn, kp, vp, xn = layer_inputs(seed, nq, nkv, hd, hidden, mt, pos, fmt, port)
    assert digest(*[w[n] for n in ("wq", "wk", "wv", "wo")], qn, kn, kp, vp, xn) == str(g[key + "__in_sha"])
    y = port.attention_layer(w, fmt, qn, kn, nq, nkv, hd, hidden, theta, eps, kp, vp, mt, pos, xn)
    assert np.array_equal(y.view(np.uint32), g[key + "__out"].view(np.uint32))
    assert np.array_equal(kp[:, pos], g[key + "__k_row"]) and np.array_equal(vp[:, pos], g[key + "__v_row"])


def test_pack_edges_against_reference_build(port):
    """pack_matrix on edge values (zero blocks, exact .5 products, NaN / Inf, tiny and huge
    values): the restatement equals the reference build byte for byte."""
    if not oracle.available("ref_scalar"):
        pytest.skip("oracle/_ref not built (needs the reference tree)")
    import importlib.util
    spec = importlib.util.spec_from_file_location("gpu_pack", os.path.join(os.path.dirname(__file__), "test_gpu_pack.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    w = mod._edge_rows()
    ref = oracle.Oracle("ref_scalar")
    for fmt in "84":
        assert np.array_equal(port.pack_matrix(w, fmt), ref.pack_matrix(w, fmt))


def test_reference_forward_runs_through_the_oracle_binding():
    """Oracle.forward_tokens drives the reference's own tq_ctx_init / tq_forward_token
    (model/context.c:6-122): finite logits, its guards (a token past the vocabulary and a full
    cache both return -1) and a deterministic result."""
    import oracle
    from _cases import forward_model
    if not oracle.available("ref_scalar"):
        pytest.skip("oracle/_ref not built (needs the reference tree)")
    ref, port = oracle.Oracle("ref_scalar"), oracle.Oracle("port")
    model = forward_model(71, "8", port)
    logits, rcs, planes = ref.forward_tokens(model, [3, 17, 17, 42], max_tokens=4)
    assert rcs == [0, 0, 0, 0] and np.isfinite(logits).all()
    again, _, planes2 = ref.forward_tokens(model, [3, 17, 17, 42], max_tokens=4)
    assert np.array_equal(logits, again) and all(np.array_equal(a[0], b[0]) for a, b in zip(planes, planes2))
    _, rcs, _ = ref.forward_tokens(model, [3, 96], max_tokens=4)
    assert rcs == [0, -1]
    _, rcs, _ = ref.forward_tokens(model, [1, 2, 3], max_tokens=2)
    assert rcs == [0, 0, -1]
