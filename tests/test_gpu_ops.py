"""GPU parity of the reference-shaped per-op kernels (attn_scores_q8,
attn_accum_q8, softmax; model/attn_q8.c:17-76, model/softmax.c:4-23) over the
shape grid of the reference's kernel sweep (tools/test_model.c:1612-1697):
scores and accum bit-exact with the reference's scalar kernels, nothing written
past n or head_dim (strided, padded outputs as in AK_SPAD / AK_OPAD)."""
import os

import numpy as np
import pytest

import oracle
from _cases import digest, head_inputs, sweep_inputs, tolerance_ok

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
GUARD = np.float32(12345.0)


@pytest.fixture(scope="module")
def tqk(cuda):
    from tailorquantkernel_b200 import tqk as t
    return t


@pytest.fixture(scope="module")
def port():
    return oracle.Oracle("port")


def _keys():
    g = np.load(os.path.join(GOLDEN, "ops_sweep.npz"))
    return sorted({k.split("__")[0] for k in g.files})


@pytest.mark.parametrize("key", _keys())
def test_scores_and_accum_bit_exact(tqk, port, cuda, key):
    import torch
    g = np.load(os.path.join(GOLDEN, "ops_sweep.npz"))
    gg, n, hd = (int(p.lstrip("ghdn")) for p in key.split("_"))
    nb = hd // 32
    qf, kf, vf, w = sweep_inputs(gg, n, hd)
    qb, kb, vb = port.quantize_rows(qf), port.quantize_rows(kf), port.quantize_rows(vf)
    assert digest(qb, kb, vb, w) == str(g[key + "__in_sha"])
    scale = float(np.float32(1.0) / np.sqrt(np.float32(hd)))
    sstride, ostride = n + 4, hd + 8
    sc = torch.full((gg * sstride,), float(GUARD), device=cuda)
    tqk.attn_scores(torch.from_numpy(qb).to(cuda), gg, torch.from_numpy(kb).to(cuda), n, nb, scale, sc, sstride)
    sc = sc.cpu().numpy().reshape(gg, sstride)
    assert np.array_equal(sc[:, :n], g[key + "__scores"])
    assert (sc[:, n:] == GUARD).all(), "scores written past n"
    out = torch.full((gg * ostride,), float(GUARD), device=cuda)
    tqk.attn_accum(torch.from_numpy(w).to(cuda), n + 4, gg, torch.from_numpy(vb).to(cuda), n, nb, out, ostride)
    out = out.cpu().numpy().reshape(gg, ostride)
    assert np.array_equal(out[:, :hd], g[key + "__accum"])
    assert (out[:, hd:] == GUARD).all(), "accum written past head_dim"


@pytest.mark.parametrize("rows,n", [(1, 1), (4, 7), (8, 300), (3, 5000)])
def test_softmax_rows(tqk, port, cuda, rows, n):
    import torch
    x = (np.random.default_rng(n).standard_normal((rows, n + 3), dtype=np.float32) * 20).astype(np.float32)
    xd = torch.from_numpy(x).to(cuda)
    tqk.softmax_rows(xd, rows, n, n + 3)
    got = xd.cpu().numpy()
    for r in range(rows):
        ref = port.softmax(x[r, :n])
        assert np.abs(got[r, :n] - ref).max() <= 1e-6
        assert np.array_equal(got[r, n:], x[r, n:])


def test_head_q8_composition_matches_golden(tqk, port, cuda):
    """attention_head_q8 (model/attn_q8.c:78-90) as quantise -> scores -> softmax -> accum on the device."""
    import torch
    g = np.load(os.path.join(GOLDEN, "head_q8.npz"))
    for hd, n, seed in ((32, 1, 60), (128, 100, 70), (128, 16, 90)):
        key = f"hd{hd}_n{n}_s{seed}"
        q, kf, vf = head_inputs(hd, n, seed)
        kb, vb = port.quantize_rows(kf), port.quantize_rows(vf)
        nb = hd // 32
        qq = tqk.quantize_rows(torch.from_numpy(q).to(cuda).view(1, hd))
        assert np.array_equal(qq.cpu().numpy().reshape(-1), g[key + "__qq"])
        sc = torch.empty(n, device=cuda)
        tqk.attn_scores(qq, 1, torch.from_numpy(kb).to(cuda), n, nb, float(np.float32(1) / np.sqrt(np.float32(hd))), sc, n)
        tqk.softmax_rows(sc, 1, n, n)
        out = torch.empty(hd, device=cuda)
        tqk.attn_accum(sc, n, 1, torch.from_numpy(vb).to(cuda), n, nb, out, hd)
        assert np.abs(sc.cpu().numpy() - g[key + "__scores"]).max() <= 1e-6
        ok, max_abs, rel = tolerance_ok(out.cpu().numpy(), g[key + "__out"], 1e-5, 1e-5)
        assert ok, (key, max_abs, rel)
