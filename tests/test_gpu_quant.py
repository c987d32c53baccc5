"""GPU parity of the quantiser and the KV append: bit-exact with the reference
(kernel/quant_x.c:5-34, model/attention_layer.c:62-90), through the C ABI."""
import os

import numpy as np
import pytest

import oracle
from _cases import quant_edge_rows

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def tqk(cuda):
    from tailorquantkernel_b200 import tqk as t
    return t


@pytest.fixture(scope="module")
def port():
    return oracle.Oracle("port")


def test_quantiser_edge_rows_bit_exact(tqk, cuda):
    import torch
    g = np.load(os.path.join(GOLDEN, "quant_edge.npz"))
    x = torch.from_numpy(g["x"]).to(cuda)
    out = tqk.quantize_rows(x).cpu().numpy()
    assert np.array_equal(out, g["blocks"])


@pytest.mark.parametrize("rows,n,scale", [(1, 32, 1.0), (3, 96, 1e-3), (4096, 128, 1.0), (20000, 256, 50.0)])
def test_quantiser_random_bit_exact(tqk, port, cuda, rows, n, scale):
    import torch
    rng = np.random.default_rng(rows + n)
    x = (rng.standard_normal((rows, n), dtype=np.float32) * np.float32(scale))
    x[::7, 3] *= 8
    out = tqk.quantize_rows(torch.from_numpy(x).to(cuda)).cpu().numpy()
    assert np.array_equal(out, port.quantize_rows(x))


def test_quantiser_unaligned_rows(tqk, port, cuda):
    """Source rows that are only 4-byte aligned take the scalar-load path."""
    import torch
    x = np.random.default_rng(3).standard_normal(32 * 9 + 1, dtype=np.float32)
    xt = torch.from_numpy(x).to(cuda)
    # the rows read in place at a 4-byte offset from a 16-byte aligned allocation
    out2 = torch.empty(9 * 36, dtype=torch.uint8, device=cuda)
    tqk.check(tqk.tqk_quantize_rows_q8(xt.data_ptr() + 4, out2.data_ptr(), 9, 32, tqk._stream(None)), "quantize")
    assert np.array_equal(out2.cpu().numpy().reshape(9, 36), port.quantize_rows(x[1:].reshape(9, 32)))


@pytest.mark.parametrize("n_kv,hd,max_tokens,pos", [(8, 128, 64, 0), (8, 128, 64, 63), (2, 32, 7, 3), (4, 64, 300, 299)])
def test_store_kv_bit_exact_and_only_touches_its_slot(tqk, port, cuda, n_kv, hd, max_tokens, pos):
    import torch
    rng = np.random.default_rng(pos + hd)
    k = rng.standard_normal(n_kv * hd, dtype=np.float32)
    v = rng.standard_normal(n_kv * hd, dtype=np.float32)
    row = hd // 32 * 36
    # garbage-filled planes like the reference tests (d = 999, q = 127: tools/test_model.c:593-600)
    garbage = np.zeros((n_kv, max_tokens, row), np.uint8)
    blk = garbage.reshape(n_kv, max_tokens, hd // 32, 36)
    blk[..., :4] = np.frombuffer(np.float32(999.0).tobytes(), np.uint8)
    blk[..., 4:] = 127
    kp_ref, vp_ref = garbage.copy(), garbage.copy()
    assert port.store_kv(kp_ref, vp_ref, n_kv, hd, max_tokens, pos, k, v) == 0
    kp = torch.from_numpy(garbage).to(cuda)
    vp = torch.from_numpy(garbage).to(cuda)
    tqk.store_kv(kp, vp, n_kv, hd, max_tokens, pos, torch.from_numpy(k).to(cuda), torch.from_numpy(v).to(cuda))
    assert np.array_equal(kp.cpu().numpy(), kp_ref)
    assert np.array_equal(vp.cpu().numpy(), vp_ref)


def test_store_kv_batch_matches_sequential(tqk, port, cuda):
    import torch
    n_kv, hd, mt, pos0, n = 8, 128, 100, 40, 33
    rng = np.random.default_rng(9)
    k = rng.standard_normal((n, n_kv * hd), dtype=np.float32)
    v = rng.standard_normal((n, n_kv * hd), dtype=np.float32)
    kp_ref = np.zeros((n_kv, mt, hd // 32 * 36), np.uint8)
    vp_ref = kp_ref.copy()
    for i in range(n):
        port.store_kv(kp_ref, vp_ref, n_kv, hd, mt, pos0 + i, k[i], v[i])
    kp = torch.zeros_like(torch.from_numpy(kp_ref)).to(cuda)
    vp = torch.zeros_like(kp)
    tqk.store_kv_batch(kp, vp, n_kv, hd, mt, pos0, n, torch.from_numpy(k).to(cuda), torch.from_numpy(v).to(cuda))
    assert np.array_equal(kp.cpu().numpy(), kp_ref) and np.array_equal(vp.cpu().numpy(), vp_ref)


def test_store_kv_bad_pos_writes_nothing(tqk, cuda):
    import torch
    kp = torch.full((2, 4, 36), 7, dtype=torch.uint8, device=cuda)
    vp = kp.clone()
    k = torch.ones(64, device=cuda)
    for pos in (-1, 4):
        with pytest.raises(tqk.TQKError) as e:
            tqk.store_kv(kp, vp, 2, 32, 4, pos, k, k)
        assert e.value.status == tqk.EPOS
    torch.cuda.synchronize()
    assert bool((kp == 7).all()) and bool((vp == 7).all())
    assert tqk.device_status() == 0
