"""GPU parity of tqk_pack_matrix: the reference's weight packer (pack_matrix,
packer/packer.c:4-88) on the device, bit-exact.  The packed bytes of the
reference's own test shapes are pinned by the SHA-256 digests in
tests/golden/matmul.npz (made by the reference build); edge rows (zero blocks,
exact .5 products, NaN / Inf, tiny and huge values) compare with the pinned
oracle restatement."""
import os

import numpy as np
import pytest

import oracle
from _cases import digest, matmul_inputs

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")

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


@pytest.mark.parametrize("i", range(len(MATMUL_CASES)))
@pytest.mark.parametrize("fmt", ["8", "4"])
def test_pack_matches_reference_digest(tqk, cuda, i, fmt):
    import torch
    rows, cols, kind = MATMUL_CASES[i]
    g = np.load(os.path.join(GOLDEN, "matmul.npz"))
    key = f"{rows}x{cols}_{kind}"
    w, x = matmul_inputs(500 + i, rows, cols, kind)
    packed = tqk.pack_matrix(torch.from_numpy(w).to(cuda), fmt)
    torch.cuda.synchronize()
    assert digest(packed.cpu().numpy()) == str(g[f"{key}__q{fmt}_packed_sha"])


def _edge_rows():
    rng = np.random.default_rng(12)
    rows = [rng.standard_normal(256, dtype=np.float32) * np.float32(s) for s in (1.0, 1e-30, 1e30, 3e-39)]
    z = np.zeros(256, np.float32)
    z[40:64] = rng.standard_normal(24, dtype=np.float32)  # block 0 all zero (scale 1.0), block 1 partly
    rows.append(z)
    ties8 = np.full(256, 0.0, np.float32)
    ties8[0::32] = 127.0                                   # scale 1.0 in every block
    ties8[1::32], ties8[2::32], ties8[3::32], ties8[4::32] = 2.5, -2.5, 126.5, -0.5
    rows.append(ties8)
    ties4 = np.full(256, 0.0, np.float32)
    ties4[0::32] = 7.0
    ties4[1::32], ties4[2::32], ties4[17::32], ties4[18::32] = 3.5, -3.5, 0.5, -6.5
    rows.append(ties4)
    bad = rng.standard_normal(256, dtype=np.float32)
    bad[5], bad[40], bad[70], bad[71] = np.nan, np.inf, -np.inf, np.nan
    rows.append(bad)
    return np.stack(rows)


@pytest.mark.parametrize("fmt", ["8", "4"])
@pytest.mark.parametrize("offset", [0, 4])
def test_pack_edges_vs_oracle(tqk, port, cuda, fmt, offset):
    """Edge values, with W 16-byte aligned (vector loads) or 4 bytes off (scalar loads)."""
    import torch
    w = _edge_rows()
    rows, cols = w.shape
    buf = torch.zeros(w.size + 4, device=cuda)
    dw = buf[offset // 4: offset // 4 + w.size].view(rows, cols)
    dw.copy_(torch.from_numpy(w))
    got = tqk.pack_matrix(dw, fmt).cpu().numpy()
    assert np.array_equal(got, port.pack_matrix(w, fmt))


def test_pack_argument_errors(tqk, cuda):
    import torch
    w = torch.zeros(4, 64, device=cuda)
    out = torch.zeros(4 * 2 * 36, dtype=torch.uint8, device=cuda)
    s = torch.cuda.current_stream().cuda_stream
    assert tqk.tqk_pack_matrix(w.data_ptr(), 4, 48, out.data_ptr(), b"8", s) == tqk.EINVAL   # cols % 32
    assert tqk.tqk_pack_matrix(w.data_ptr(), 4, 64, out.data_ptr(), b"5", s) == tqk.EINVAL   # bit type
    assert tqk.tqk_pack_matrix(None, 4, 64, out.data_ptr(), b"8", s) == tqk.EINVAL
    assert tqk.tqk_pack_matrix(w.data_ptr(), 4, 64, out.data_ptr(), b"8", s) == tqk.OK
