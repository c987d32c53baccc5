"""The allocation-free decode entry point (tqk_decode_q8_static) against the
workspace one (tqk_decode_q8), through the C ABI.

Same inputs, same tolerance as the decode parity tests (max abs error <= 1e-3
and max |diff| / max |ref| <= 1e-3); each case calls the static entry twice in
a row, and repeated calls must not change the device's free memory.
"""
import ctypes

import numpy as np
import pytest

from _cases import tolerance_ok

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tqk(cuda):
    from tailorquantkernel_b200 import tqk as t
    return t


def _planes(tqk, gen, shape):
    import torch
    return tqk.quantize_rows(torch.randn(shape, device="cuda", generator=gen))


def _both(tqk, make_args, n_out):
    """Runs tqk_decode_q8 once and tqk_decode_q8_static twice on fresh output buffers."""
    import torch
    ref = torch.full((n_out,), float("nan"), device="cuda")
    tqk.decode(make_args(ref))
    outs = []
    for _ in range(2):
        o = torch.full((n_out,), float("nan"), device="cuda")
        rc = tqk.tqk_decode_q8_static(ctypes.byref(make_args(o)), None)
        assert rc == 0, tqk.tqk_last_error()
        outs.append(o)
    torch.cuda.synchronize()
    return ref.cpu().numpy(), [o.cpu().numpy() for o in outs]


@pytest.mark.parametrize("nq,nkv,n_items,n", [(32, 8, 4, 4097), (64, 8, 1, 20000), (16, 2, 3, 700), (8, 8, 2, 100)])
def test_static_matches_workspace_entry(tqk, cuda, nq, nkv, n_items, n):
    import torch
    hd = 128
    gen = torch.Generator(device="cuda").manual_seed(nq + n)
    kp = _planes(tqk, gen, (n_items, nkv, n, hd))
    vp = _planes(tqk, gen, (n_items, nkv, n, hd))
    q = torch.randn(n_items, nq * hd, device="cuda", generator=gen)
    kn = torch.randn(n_items, nkv * hd, device="cuda", generator=gen)
    vn = torch.randn(n_items, nkv * hd, device="cuda", generator=gen)

    def args(out):  # fused append at n - 1: writing the same row again leaves the cache unchanged
        return tqk.decode_args(kp, vp, nq, nkv, hd, n, q, out, n_items=n_items, item_stride_blocks=nkv * n * 4,
                               len0=n, q_item_stride=nq * hd, out_item_stride=nq * hd, k_new=kn, v_new=vn,
                               kv_new_item_stride=nkv * hd)
    ref, outs = _both(tqk, args, n_items * nq * hd)
    for o in outs:
        ok, max_abs, rel = tolerance_ok(o, ref)
        assert ok, f"max abs {max_abs:.3g} rel {rel:.3g}"


def test_static_ragged_device_lengths(tqk, cuda):
    import torch
    nq, nkv, hd, mt = 32, 8, 128, 3000
    lens = torch.tensor([3000, 1, 0, 2048, 65, 1500], dtype=torch.int32, device="cuda")
    B = lens.numel()
    gen = torch.Generator(device="cuda").manual_seed(7)
    kp = _planes(tqk, gen, (B, nkv, mt, hd))
    vp = _planes(tqk, gen, (B, nkv, mt, hd))
    q = torch.randn(B, nq * hd, device="cuda", generator=gen)

    def args(out):
        return tqk.decode_args(kp, vp, nq, nkv, hd, mt, q, out, n_items=B, item_stride_blocks=nkv * mt * 4, lens=lens,
                               max_len=3000, q_item_stride=nq * hd, out_item_stride=nq * hd)
    ref, outs = _both(tqk, args, B * nq * hd)
    for o in outs:
        ok, max_abs, rel = tolerance_ok(o, ref)
        assert ok, f"max abs {max_abs:.3g} rel {rel:.3g}"


def test_static_allocates_nothing_after_setup(tqk, cuda):
    import torch
    nq, nkv, hd, n = 32, 8, 128, 4097
    gen = torch.Generator(device="cuda").manual_seed(9)
    kp = _planes(tqk, gen, (nkv, n, hd))
    vp = _planes(tqk, gen, (nkv, n, hd))
    q = torch.randn(nq * hd, device="cuda", generator=gen)
    out = torch.empty(nq * hd, device="cuda")
    a = tqk.decode_args(kp, vp, nq, nkv, hd, n, q, out, len0=n)
    assert tqk.tqk_decode_q8_static(ctypes.byref(a), None) == 0, tqk.tqk_last_error()
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        assert tqk.tqk_decode_q8_static(ctypes.byref(a), None) == 0, tqk.tqk_last_error()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0


def test_static_rejects_oversized_split(tqk, cuda):
    import torch
    nq, nkv, hd, n, items = 32, 8, 128, 128, 5000
    gen = torch.Generator(device="cuda").manual_seed(10)
    kp = _planes(tqk, gen, (nkv, n, hd))  # one shared set of planes (item stride 0)
    vp = _planes(tqk, gen, (nkv, n, hd))
    q = torch.randn(items, nq * hd, device="cuda", generator=gen)
    out = torch.empty(items, nq * hd, device="cuda")
    a = tqk.decode_args(kp, vp, nq, nkv, hd, n, q, out, n_items=items, len0=n, q_item_stride=nq * hd,
                        out_item_stride=nq * hd, split_tokens=64)  # 2 splits x 20000 units
    assert tqk.tqk_decode_q8_static(ctypes.byref(a), None) == tqk.EWORKSPACE
    assert b"16384" in tqk.tqk_last_error()
    tqk.decode(a)  # the workspace entry takes the same call
    torch.cuda.synchronize()
