"""The drop-in boundary end to end: the reference's own unit-test program
(tools/test_model.c, unchanged) linked against libtq_attn_b200.so in place of
the reference's model/attn_q8.c, model/attention_layer.c and model/kv_cache.c
(oracle/Makefile target _ref/test_model_dropin, built where the reference tree
is present and carried with the repository).  Every Q8 attention test of the
reference suite -- the kernel sweep with guards, the layer tests with garbage
sentinels, the forward-pass tests -- then runs on the GPU path and must pass."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(ROOT, "oracle", "_ref", "test_model_dropin")

pytestmark = pytest.mark.gpu


def test_reference_suite_passes_through_the_dropin(cuda):
    if not os.path.exists(EXE):
        pytest.skip("oracle/_ref/test_model_dropin not built (needs the reference tree at build time)")
    res = subprocess.run([EXE], capture_output=True, text=True, timeout=600)
    lines = res.stdout.splitlines()
    failed = [l for l in lines if l.endswith("FAIL")]
    assert res.returncode == 0 and not failed, "\n".join(failed + lines[-5:] + [res.stderr[-2000:]])
    assert "All tests passed." in res.stdout
    for name in ("attention q8 kernels (dispatched and scalar): PASS",
                 "attention layer q8 cache vs f32 cache: PASS",
                 "tq_forward_token vs reference (kv q8): ok"):
        assert name in res.stdout


# ---------------------------------------------------------------------------
# device-resident layers through the drop-in: tq_b200_register_attn_weights
# ---------------------------------------------------------------------------
HARNESS = os.path.join(ROOT, "oracle", "_ref", "libtqref_dropin.so")
LAYER = (62, 32, 8, 128, 512, 70, 64, 500000.0, 1e-5)  # tests/golden/make_golden.py LAYER_CASES["llama_heads"]


def _layer_structs(oracle_mod, w, fmt, qn, kn, nq, nkv, hd, hidden, theta, eps):
    import ctypes
    import numpy as np
    f = 0 if fmt == "8" else 1
    vp = lambda a: ctypes.c_void_p(a.ctypes.data)  # noqa: E731
    q_dim, kv_dim = nq * hd, nkv * hd
    mats = [oracle_mod._TqMatrix(vp(w["wq"]), f, q_dim, hidden), oracle_mod._TqMatrix(vp(w["wk"]), f, kv_dim, hidden),
            oracle_mod._TqMatrix(vp(w["wv"]), f, kv_dim, hidden), oracle_mod._TqMatrix(vp(w["wo"]), f, hidden, q_dim)]
    aw = oracle_mod._TqAttnWeights(*mats, vp(qn), vp(kn))
    cfg = oracle_mod._TqAttnConfig(nq, nkv, hd, hidden, theta, eps)
    return aw, cfg


@pytest.mark.parametrize("fmt", ["8", "4"])
def test_registered_weights_run_the_layer_on_the_device(cuda, fmt):
    """attention_layer / attention_layer_batch of the drop-in with the layer's weights registered:
    the appended host cache rows are bit-exact with the reference's, the outputs within the
    layer tolerance (max |diff| <= 1e-3 * max |reference|), token after token and for a chunk."""
    import ctypes

    import numpy as np

    import oracle
    from _cases import layer_inputs
    if not os.path.exists(HARNESS):
        pytest.skip("oracle/_ref/libtqref_dropin.so not built (needs the reference tree at build time)")
    lib = ctypes.CDLL(HARNESS)
    port = oracle.Oracle("port")
    seed, nq, nkv, hd, hidden, mt, pos, theta, eps = LAYER
    w, qn, kn, kp, vp_, xn = layer_inputs(seed, nq, nkv, hd, hidden, mt, pos, fmt, port)
    aw, cfg = _layer_structs(oracle, w, fmt, qn, kn, nq, nkv, hd, hidden, theta, eps)
    cache = oracle._TqKvCache()
    lib.tq_kv_cache_init.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int]
    assert lib.tq_kv_cache_init(ctypes.byref(cache), 1, ctypes.byref(cfg), mt) == 0
    plane = kp.nbytes
    ctypes.memmove(cache.k_q8, kp.ctypes.data, plane)
    ctypes.memmove(cache.v_q8, vp_.ctypes.data, plane)
    host_k = np.ctypeslib.as_array(ctypes.cast(cache.k_q8, ctypes.POINTER(ctypes.c_uint8)), shape=kp.shape)
    host_v = np.ctypeslib.as_array(ctypes.cast(cache.v_q8, ctypes.POINTER(ctypes.c_uint8)), shape=vp_.shape)
    kp_ref, vp_ref = kp.copy(), vp_.copy()
    assert lib.tq_b200_register_attn_weights(ctypes.byref(aw), ctypes.byref(cfg)) == 0
    fn = lib.attention_layer
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_void_p]
    scores = np.zeros(nq * mt, np.float32)
    rng = np.random.default_rng(17)
    xs = [xn] + [rng.standard_normal(hidden, dtype=np.float32) for _ in range(2)]
    for i, x in enumerate(xs):  # three tokens on the device, the cache evolving
        out = np.zeros(hidden, np.float32)
        assert fn(ctypes.byref(aw), ctypes.byref(cfg), ctypes.byref(cache), pos + i, x.ctypes.data,
                  scores.ctypes.data, out.ctypes.data) == 0
        want = port.attention_layer(w, fmt, qn, kn, nq, nkv, hd, hidden, theta, eps, kp_ref, vp_ref, mt, pos + i, x)
        assert np.array_equal(host_k[:, pos + i], kp_ref[:, pos + i]) and np.array_equal(host_v[:, pos + i],
                                                                                         vp_ref[:, pos + i]), i
        assert np.abs(out - want).max() <= 1e-3 * np.abs(want).max(), i

    # a chunk of 2 tokens through attention_layer_batch (the prefill path)
    class BatchWs(ctypes.Structure):
        _fields_ = [("cap", ctypes.c_int)] + [(n, ctypes.c_void_p) for n in
                                               ("x", "xn", "sub", "gate", "up", "q", "attn", "k", "v", "xq", "hq")]
    ws = BatchWs()
    ws.cap = 8
    n, p0 = 2, pos + 3  # positions 67, 68; the unregistered call below takes 69 (max_tokens 70)
    xb = rng.standard_normal((n, hidden), dtype=np.float32)
    outb = np.zeros((n, hidden), np.float32)
    fb = lib.attention_layer_batch
    fb.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    assert fb(ctypes.byref(aw), ctypes.byref(cfg), ctypes.byref(cache), p0, n, xb.ctypes.data, scores.ctypes.data,
              outb.ctypes.data, ctypes.byref(ws)) == 0
    for i in range(n):
        want = port.attention_layer(w, fmt, qn, kn, nq, nkv, hd, hidden, theta, eps, kp_ref, vp_ref, mt, p0 + i, xb[i])
        assert np.array_equal(host_k[:, p0 + i], kp_ref[:, p0 + i]), i
        assert np.abs(outb[i] - want).max() <= 2e-3 * np.abs(want).max(), i

    # unregistered: the host-projection path takes over with the same results
    lib.tq_b200_unregister_attn_weights(ctypes.byref(aw))
    x = rng.standard_normal(hidden, dtype=np.float32)
    out = np.zeros(hidden, np.float32)
    assert fn(ctypes.byref(aw), ctypes.byref(cfg), ctypes.byref(cache), p0 + n, x.ctypes.data, scores.ctypes.data,
              out.ctypes.data) == 0
    want = port.attention_layer(w, fmt, qn, kn, nq, nkv, hd, hidden, theta, eps, kp_ref, vp_ref, mt, p0 + n, x)
    assert np.array_equal(host_k[:, p0 + n], kp_ref[:, p0 + n])
    assert np.abs(out - want).max() <= 1e-3 * np.abs(want).max()
    lib.tq_kv_cache_free.argtypes = [ctypes.c_void_p]
    lib.tq_kv_cache_free(ctypes.byref(cache))


def test_device_error_word_reaches_the_dropin_caller(cuda):
    """A failure that a kernel records in the device error word (here a bounded wait that
    gave up, made without any fault: a two-rank exchange whose peer never raises its flag)
    comes back from the next drop-in attention_layer call as TQK_ETIMEOUT, with the host
    cache rows untouched; the word is cleared and the call after that succeeds, bit-exact
    in the appended rows and within the layer tolerance in the output."""
    import ctypes

    import numpy as np
    import torch

    import oracle
    from _cases import layer_inputs
    from tailorquantkernel_b200 import tqk
    if not os.path.exists(HARNESS):
        pytest.skip("oracle/_ref/libtqref_dropin.so not built (needs the reference tree at build time)")
    lib = ctypes.CDLL(HARNESS)
    port = oracle.Oracle("port")
    seed, nq, nkv, hd, hidden, mt, pos, theta, eps = LAYER
    fmt = "8"
    w, qn, kn, kp, vp_, xn = layer_inputs(seed, nq, nkv, hd, hidden, mt, pos, fmt, port)
    aw, cfg = _layer_structs(oracle, w, fmt, qn, kn, nq, nkv, hd, hidden, theta, eps)
    cache = oracle._TqKvCache()
    lib.tq_kv_cache_init.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int]
    assert lib.tq_kv_cache_init(ctypes.byref(cache), 1, ctypes.byref(cfg), mt) == 0
    ctypes.memmove(cache.k_q8, kp.ctypes.data, kp.nbytes)
    ctypes.memmove(cache.v_q8, vp_.ctypes.data, vp_.nbytes)
    host_k = np.ctypeslib.as_array(ctypes.cast(cache.k_q8, ctypes.POINTER(ctypes.c_uint8)), shape=kp.shape)
    fn = lib.attention_layer
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_void_p]
    scores = np.zeros(nq * mt, np.float32)
    out = np.zeros(hidden, np.float32)
    # the drop-in's first call binds its context; then the error word is set by a timed-out wait
    assert fn(ctypes.byref(aw), ctypes.byref(cfg), ctypes.byref(cache), pos, xn.ctypes.data, scores.ctypes.data,
              out.ctypes.data) == 0
    kp_ref, vp_ref = kp.copy(), vp_.copy()
    port.attention_layer(w, fmt, qn, kn, nq, nkv, hd, hidden, theta, eps, kp_ref, vp_ref, mt, pos, xn)
    nbytes = tqk.tqk_exchange_mailbox_bytes(2, nq, hd)
    boxes = [tqk.peer_buffer_alloc(nbytes), tqk.peer_buffer_alloc(nbytes)]
    try:
        assert tqk.device_status(clear=True) == 0
        junk = torch.empty(nq * hd, device="cuda")
        tqk.exchange_merge(nq, hd, 2, 0, boxes, 1, junk)
        torch.cuda.synchronize()
        row_before = host_k[:, pos + 1].copy()
        x = np.random.default_rng(3).standard_normal(hidden, dtype=np.float32)
        rc = fn(ctypes.byref(aw), ctypes.byref(cfg), ctypes.byref(cache), pos + 1, x.ctypes.data, scores.ctypes.data,
                out.ctypes.data)
        assert rc == tqk.ETIMEOUT, rc
        assert np.array_equal(host_k[:, pos + 1], row_before)  # no rows written back
        assert tqk.device_status() == 0  # the drop-in cleared the word
        out[:] = np.nan
        assert fn(ctypes.byref(aw), ctypes.byref(cfg), ctypes.byref(cache), pos + 1, x.ctypes.data,
                  scores.ctypes.data, out.ctypes.data) == 0
        want = port.attention_layer(w, fmt, qn, kn, nq, nkv, hd, hidden, theta, eps, kp_ref, vp_ref, mt, pos + 1, x)
        assert np.array_equal(host_k[:, pos + 1], kp_ref[:, pos + 1])
        assert np.abs(out - want).max() <= 1e-3 * np.abs(want).max()
    finally:
        for b in boxes:
            tqk.peer_buffer_free(b)
        lib.tq_kv_cache_free.argtypes = [ctypes.c_void_p]
        lib.tq_kv_cache_free(ctypes.byref(cache))


@pytest.mark.parametrize("registered", [True, False])
def test_rewritten_last_row_is_noticed_without_invalidate(cuda, registered):
    """A caller that rewrites the cache row the previous call appended (here: K and V of
    every kv head at that position replaced by rows ten times larger, so that this token
    dominates the softmax) and calls again WITHOUT tq_b200_cache_invalidate: the drop-in
    compares that row with the copy it wrote, re-uploads the planes, and the output follows
    the rewritten cache (the reference reads the host planes on every call)."""
    import ctypes

    import numpy as np

    import oracle
    from _cases import layer_inputs
    if not os.path.exists(HARNESS):
        pytest.skip("oracle/_ref/libtqref_dropin.so not built (needs the reference tree at build time)")
    lib = ctypes.CDLL(HARNESS)
    port = oracle.Oracle("port")
    seed, nq, nkv, hd, hidden, mt, pos, theta, eps = LAYER
    fmt = "8"
    w, qn, kn, kp, vp_, xn = layer_inputs(seed, nq, nkv, hd, hidden, mt, pos, fmt, port)
    aw, cfg = _layer_structs(oracle, w, fmt, qn, kn, nq, nkv, hd, hidden, theta, eps)
    cache = oracle._TqKvCache()
    lib.tq_kv_cache_init.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int]
    assert lib.tq_kv_cache_init(ctypes.byref(cache), 1, ctypes.byref(cfg), mt) == 0
    ctypes.memmove(cache.k_q8, kp.ctypes.data, kp.nbytes)
    ctypes.memmove(cache.v_q8, vp_.ctypes.data, vp_.nbytes)
    host_k = np.ctypeslib.as_array(ctypes.cast(cache.k_q8, ctypes.POINTER(ctypes.c_uint8)), shape=kp.shape)
    host_v = np.ctypeslib.as_array(ctypes.cast(cache.v_q8, ctypes.POINTER(ctypes.c_uint8)), shape=vp_.shape)
    if registered:
        assert lib.tq_b200_register_attn_weights(ctypes.byref(aw), ctypes.byref(cfg)) == 0
    fn = lib.attention_layer
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_void_p]
    scores = np.zeros(nq * mt, np.float32)
    out = np.zeros(hidden, np.float32)
    kp_ref, vp_ref = kp.copy(), vp_.copy()
    try:
        assert fn(ctypes.byref(aw), ctypes.byref(cfg), ctypes.byref(cache), pos, xn.ctypes.data, scores.ctypes.data,
                  out.ctypes.data) == 0
        port.attention_layer(w, fmt, qn, kn, nq, nkv, hd, hidden, theta, eps, kp_ref, vp_ref, mt, pos, xn)
        rng = np.random.default_rng(29)
        new_k = port.quantize_rows(10.0 * rng.standard_normal((nkv, hd), dtype=np.float32))
        new_v = port.quantize_rows(10.0 * rng.standard_normal((nkv, hd), dtype=np.float32))
        host_k[:, pos] = new_k
        host_v[:, pos] = new_v
        kp_ref[:, pos] = new_k
        vp_ref[:, pos] = new_v
        x = rng.standard_normal(hidden, dtype=np.float32)
        assert fn(ctypes.byref(aw), ctypes.byref(cfg), ctypes.byref(cache), pos + 1, x.ctypes.data,
                  scores.ctypes.data, out.ctypes.data) == 0
        want = port.attention_layer(w, fmt, qn, kn, nq, nkv, hd, hidden, theta, eps, kp_ref, vp_ref, mt, pos + 1, x)
        assert np.array_equal(host_k[:, pos + 1], kp_ref[:, pos + 1])
        assert np.abs(out - want).max() <= 1e-3 * np.abs(want).max()
    finally:
        if registered:
            lib.tq_b200_unregister_attn_weights(ctypes.byref(aw))
        lib.tq_kv_cache_free.argtypes = [ctypes.c_void_p]
        lib.tq_kv_cache_free(ctypes.byref(cache))
