"""GPU parity of the projections' matrix-vector products (tqk_matmul_q8/q4,
their _batch forms and the fused tqk_project) through the C ABI.

Bar: bit-exact with the reference's scalar kernels (kernel/q8_scalar.c,
kernel/q4_scalar.c): the golden fixture tests/golden/matmul.npz holds the
reference's own outputs on the shapes of its tools/test_kernel.c; larger and
batched cases compare with the pinned oracle restatement.  The fused
tqk_project also quantises the activations (bit-exact with quantize_row_q8).
"""
import os

import numpy as np
import pytest

import oracle
from _cases import digest, matmul_inputs

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")

# the cases of tests/golden/make_golden.py MATMUL_CASES (seed 500 + index)
MATMUL_CASES = [(rows, cols, "random") for rows, cols in
                ((256, 512), (7, 64), (10, 32), (1027, 96), (1024, 1024), (3072, 1024), (1024, 3072))] + \
               [(256, 512, "constant"), (256, 512, "zero")]


@pytest.fixture(scope="module")
def tqk(cuda):
    from tailorquantkernel_b200 import tqk as t
    return t


@pytest.fixture(scope="module")
def port():
    return oracle.Oracle("port")


def _bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def _dev(a, cuda):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


@pytest.mark.parametrize("i", range(len(MATMUL_CASES)))
@pytest.mark.parametrize("fmt", ["8", "4"])
def test_matmul_matches_golden(tqk, port, cuda, i, fmt):
    import torch
    rows, cols, kind = MATMUL_CASES[i]
    g = np.load(os.path.join(GOLDEN, "matmul.npz"))
    key = f"{rows}x{cols}_{kind}"
    w, x = matmul_inputs(500 + i, rows, cols, kind)
    assert digest(w, x) == str(g[key + "__in_sha"])
    wp = port.pack_matrix(w, fmt)
    assert digest(wp) == str(g[f"{key}__q{fmt}_packed_sha"])
    xq = port.quantize_rows(x[None])[0]
    y = torch.full((rows,), float("nan"), device=cuda)
    tqk.matmul(_dev(wp, cuda), tqk.FMT_Q8 if fmt == "8" else tqk.FMT_Q4, _dev(xq, cuda), y, rows, cols)
    torch.cuda.synchronize()
    assert np.array_equal(_bits(y.cpu().numpy()), _bits(g[f"{key}__q{fmt}_y"]))


@pytest.mark.parametrize("fmt", ["8", "4"])
@pytest.mark.parametrize("rows,cols,n_tok", [
    (4096, 4096, 1),     # Llama-3-8B wq / wo
    (1024, 4096, 3),     # wk / wv, a few tokens
    (512, 4096, 8),      # one full token group
    (300, 1024, 11),     # two launches (8 + 3 tokens)
    (64, 14336, 2),      # a long row (MLP down shape): one row per group
    (97, 160, 5),        # 5 blocks per row: rows are not whole 16-byte units (lane copies)
])
def test_matmul_batch_vs_oracle(tqk, port, cuda, fmt, rows, cols, n_tok):
    import torch
    rng = np.random.default_rng(rows + cols + n_tok)
    w = rng.uniform(-1.0, 1.0, (rows, cols)).astype(np.float32)
    x = rng.standard_normal((n_tok, cols), dtype=np.float32)
    wp = port.pack_matrix(w, fmt)
    xq = port.quantize_rows(x)
    want = np.stack([port.matmul(wp, fmt, xq[t], rows, cols) for t in range(n_tok)])
    y = torch.full((n_tok, rows), float("nan"), device=cuda)
    tqk.matmul(_dev(wp, cuda), tqk.FMT_Q8 if fmt == "8" else tqk.FMT_Q4, _dev(xq, cuda), y, rows, cols, n_tok)
    torch.cuda.synchronize()
    assert np.array_equal(_bits(y.cpu().numpy()), _bits(want))


@pytest.mark.parametrize("fmt", ["8", "4"])
@pytest.mark.parametrize("n_tok", [1, 4])
def test_project_qkv_fused_quantisation(tqk, port, cuda, fmt, n_tok):
    """project_qkv (attention_layer.c:38-46) in one launch: x quantised in the kernel, then
    wq / wk / wv (Llama-3-8B shapes) -- bit-exact with quantize_row_q8 + matmul per token."""
    import torch
    hidden, q_dim, kv_dim = 4096, 4096, 1024
    rng = np.random.default_rng(31 + n_tok)
    mats = {n: rng.uniform(-1.0, 1.0, (r, hidden)).astype(np.float32)
            for n, r in (("q", q_dim), ("k", kv_dim), ("v", kv_dim))}
    x = rng.standard_normal((n_tok, hidden), dtype=np.float32)
    xq = port.quantize_rows(x)
    packed = {n: port.pack_matrix(m, fmt) for n, m in mats.items()}
    outs = {n: torch.full((n_tok, m.shape[0]), float("nan"), device=cuda) for n, m in mats.items()}
    dw = {n: _dev(p, cuda) for n, p in packed.items()}
    tqk.project([(dw[n], outs[n], mats[n].shape[0]) for n in ("q", "k", "v")],
                tqk.FMT_Q8 if fmt == "8" else tqk.FMT_Q4, _dev(x, cuda), hidden, n_tok)
    torch.cuda.synchronize()
    for n, m in mats.items():
        want = np.stack([port.matmul(packed[n], fmt, xq[t], m.shape[0], hidden) for t in range(n_tok)])
        assert np.array_equal(_bits(outs[n].cpu().numpy()), _bits(want)), n


def test_unaligned_weights_take_the_copy_path(tqk, port, cuda):
    """Weights 4 bytes off a 16-byte boundary: same results through the lane-copy path."""
    import torch
    rows, cols = 130, 512
    rng = np.random.default_rng(9)
    w = rng.uniform(-1.0, 1.0, (rows, cols)).astype(np.float32)
    x = rng.standard_normal(cols, dtype=np.float32)
    wp = port.pack_matrix(w, "8")
    xq = port.quantize_rows(x[None])[0]
    buf = torch.zeros(wp.size + 16, dtype=torch.uint8, device=cuda)
    buf[4:4 + wp.size] = _dev(wp.reshape(-1), cuda)
    y = torch.empty(rows, device=cuda)
    tqk.check(tqk.tqk_matmul_q8(buf.data_ptr() + 4, _dev(xq, cuda).data_ptr(), y.data_ptr(), rows, cols,
                                torch.cuda.current_stream().cuda_stream), "tqk_matmul_q8")
    torch.cuda.synchronize()
    assert np.array_equal(_bits(y.cpu().numpy()), _bits(port.matmul(wp, "8", xq, rows, cols)))


def test_matmul_argument_errors(tqk, cuda):
    import torch
    w = torch.zeros(4 * 36, dtype=torch.uint8, device=cuda)
    xq = torch.zeros(36, dtype=torch.uint8, device=cuda)
    y = torch.zeros(4, device=cuda)
    s = torch.cuda.current_stream().cuda_stream
    assert tqk.tqk_matmul_q8(w.data_ptr(), xq.data_ptr(), y.data_ptr(), 4, 33, s) == tqk.EINVAL   # cols % 32
    assert tqk.tqk_matmul_q8(None, xq.data_ptr(), y.data_ptr(), 4, 32, s) == tqk.EINVAL
    assert tqk.tqk_matmul_q8(w.data_ptr() + 2, xq.data_ptr(), y.data_ptr(), 4, 32, s) == tqk.EINVAL  # alignment
    assert tqk.tqk_matmul_q8(w.data_ptr(), xq.data_ptr(), y.data_ptr(), 0, 32, s) == tqk.OK       # nothing to do
    jobs = (tqk.ProjJob * 5)()
    assert tqk.tqk_project(jobs, 5, tqk.FMT_Q8, y.data_ptr(), 32, 1, s) == tqk.EINVAL           # > 4 jobs
