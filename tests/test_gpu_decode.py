"""GPU parity of the fused decode attention (attend_q8 + store_kv,
model/attention_layer.c:62-150) through the C ABI, against the oracle.

Tolerance (the north star's): max abs error <= 1e-3 and relative error
(max |diff| / max |ref|) <= 1e-3 in FP32 (tests/_cases.py:tolerance_ok); the Q8
append is bit-exact.  Small cases compare with the golden fixtures made by the
reference itself; BASELINE.json's full configurations compare with the oracle
restatement on GPU-generated inputs.
"""
import os

import numpy as np
import pytest

import oracle
from _cases import decode_case, digest, tolerance_ok

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def tqk(cuda):
    from tailorquantkernel_b200 import tqk as t
    return t


@pytest.fixture(scope="module")
def port():
    return oracle.Oracle("port")


def _golden_names():
    g = np.load(os.path.join(GOLDEN, "decode.npz"))
    return sorted({k.split("__")[0] for k in g.files})


def _golden(name):
    g = np.load(os.path.join(GOLDEN, "decode.npz"))
    seed, nq, nkv, hd, mt, pos, of, rp = (int(v) for v in g[f"{name}__params"])
    kf, vf, q = decode_case(seed, nq, nkv, hd, mt, pos + 1, outlier_frac=of / 1e6, rope_pos=None if rp < 0 else rp)
    assert digest(kf, vf, q) == str(g[f"{name}__in_sha"])
    return (nq, nkv, hd, mt, pos), kf, vf, q, g[f"{name}__out"], str(g[f"{name}__planes_sha"])


@pytest.mark.parametrize("name", _golden_names())
def test_attend_matches_golden(tqk, cuda, name):
    import torch
    (nq, nkv, hd, mt, pos), kf, vf, q, ref, planes_sha = _golden(name)
    kp = tqk.quantize_rows(torch.from_numpy(kf).to(cuda))
    vp = tqk.quantize_rows(torch.from_numpy(vf).to(cuda))
    assert digest(kp.cpu().numpy(), vp.cpu().numpy()) == planes_sha  # device quantiser == reference
    out = torch.empty(nq * hd, device=cuda)
    tqk.attend(kp, vp, nq, nkv, hd, mt, pos, torch.from_numpy(q).to(cuda), out)
    ok, max_abs, rel = tolerance_ok(out.cpu().numpy(), ref)
    assert ok, f"{name}: max abs {max_abs:.3g} rel {rel:.3g}"


@pytest.mark.parametrize("name", _golden_names())
def test_fused_append_attend_matches_golden(tqk, cuda, name):
    """store_kv + attend_q8 in one launch: the appended row is bit-exact and the
    attention sees it."""
    import torch
    (nq, nkv, hd, mt, pos), kf, vf, q, ref, planes_sha = _golden(name)
    k_new = np.ascontiguousarray(kf[:, pos])
    v_new = np.ascontiguousarray(vf[:, pos])
    kf2, vf2 = kf.copy(), vf.copy()
    kf2[:, pos] = 0
    vf2[:, pos] = 0
    kp = tqk.quantize_rows(torch.from_numpy(kf2).to(cuda))
    vp = tqk.quantize_rows(torch.from_numpy(vf2).to(cuda))
    out = torch.empty(nq * hd, device=cuda)
    tqk.append_attend(kp, vp, nq, nkv, hd, mt, pos, torch.from_numpy(q).to(cuda), torch.from_numpy(k_new).to(cuda),
                      torch.from_numpy(v_new).to(cuda), out)
    assert digest(kp.cpu().numpy(), vp.cpu().numpy()) == planes_sha
    ok, max_abs, rel = tolerance_ok(out.cpu().numpy(), ref)
    assert ok, f"{name}: max abs {max_abs:.3g} rel {rel:.3g}"


def _gpu_planes(gen, shape_f32, tqk, outlier_frac=0.0):
    """N(0,1) fp32 on the device (optionally 1% x8 outliers), quantised to Q8 by the device quantiser."""
    import torch
    x = torch.randn(shape_f32, device="cuda", generator=gen)
    if outlier_frac:
        x = torch.where(torch.rand(shape_f32, device="cuda", generator=gen) < outlier_frac, x * 8, x)
    return tqk.quantize_rows(x)


def test_config2_all_layers_fused_append(tqk, port, cuda):
    """Config 2: 32 layers, 32 q / 8 kv heads, context 4096 + the appended token
    at position 4096, q with RoPE at 4096 -- one multi-item launch."""
    import torch
    from _cases import rope
    L, nq, nkv, hd, pos = 32, 32, 8, 128, 4096
    mt = pos + 1
    gen = torch.Generator(device="cuda").manual_seed(2)
    kp = _gpu_planes(gen, (L, nkv, mt, hd), tqk)
    vp = _gpu_planes(gen, (L, nkv, mt, hd), tqk)
    rng = np.random.default_rng(2)
    q = rope(rng.standard_normal((L, nq * hd), dtype=np.float32), hd, pos, 500000.0)
    k_new = rng.standard_normal((L, nkv * hd), dtype=np.float32)
    v_new = rng.standard_normal((L, nkv * hd), dtype=np.float32)
    out = torch.empty(L, nq * hd, device=cuda)
    args = tqk.decode_args(kp, vp, nq, nkv, hd, mt, torch.from_numpy(q).to(cuda), out, n_items=L,
                           item_stride_blocks=nkv * mt * (hd // 32), len0=pos + 1, q_item_stride=nq * hd,
                           out_item_stride=nq * hd, k_new=torch.from_numpy(k_new).to(cuda),
                           v_new=torch.from_numpy(v_new).to(cuda), kv_new_item_stride=nkv * hd)
    tqk.decode(args)
    got = out.cpu().numpy()
    kh, vh = kp.cpu().numpy(), vp.cpu().numpy()
    for layer in range(L):
        # the oracle appends from fp32 itself; the device's append must be bit-exact
        kref, vref = kh[layer].copy(), vh[layer].copy()
        assert port.store_kv(kref, vref, nkv, hd, mt, pos, k_new[layer], v_new[layer]) == 0
        assert np.array_equal(kref, kh[layer]) and np.array_equal(vref, vh[layer]), f"append layer {layer}"
        ref = port.attend(kref, vref, nq, nkv, hd, mt, pos, q[layer])
        ok, max_abs, rel = tolerance_ok(got[layer], ref)
        assert ok, f"layer {layer}: max abs {max_abs:.3g} rel {rel:.3g}"
    assert tqk.device_status() == 0


def test_config1_on_the_reference_generator(tqk, port, cuda):
    """Config 1 (one layer, 32 q / 8 kv heads, n = 1024) on inputs drawn the way the reference's
    benches draw theirs: the xorshift64 + Box-Muller stream from 88172645463325252
    (tools/bench_forward.c:82,199-210), here through tqk_fill_normal, which
    tests/test_inputs_cpu.py pins bit for bit to the reference's own normal_sample.  K then V
    ([kv head][position][head_dim]), then q; K/V quantised by the oracle's reference quantiser."""
    import torch
    nq, nkv, hd, n = 32, 8, 128, 1024
    kf = tqk.fill_normal(0, nkv * n * hd).reshape(nkv, n, hd)
    vf = tqk.fill_normal(nkv * n * hd, nkv * n * hd).reshape(nkv, n, hd)
    q = tqk.fill_normal(2 * nkv * n * hd, nq * hd)
    kp, vp = port.quantize_rows(kf), port.quantize_rows(vf)
    out = torch.empty(nq * hd, device=cuda)
    args = tqk.decode_args(torch.from_numpy(kp).to(cuda), torch.from_numpy(vp).to(cuda), nq, nkv, hd, n,
                           torch.from_numpy(q).to(cuda), out, len0=n)
    tqk.decode(args)
    ref = port.attend(kp, vp, nq, nkv, hd, n, n - 1, q)
    ok, max_abs, rel = tolerance_ok(out.cpu().numpy(), ref)
    assert ok, f"max abs {max_abs:.3g} rel {rel:.3g}"
    assert tqk.device_status() == 0


@pytest.mark.parametrize("out_mode", [0, 1])
def test_cluster_merge_every_size(tqk, port, cuda, out_mode):
    """The packed kernel's split merge for every split count from 2 to 16: with equal lengths
    (len_step 0) it runs through a thread-block cluster of the unit's splits -- three items of the
    same length with a fused append, in both output modes; with device lengths (a long item, a
    300-token and a one-token item whose later splits are empty) it runs through the tickets;
    then an empty item without an append.  The appended rows bit-exact, the outputs within the
    tolerance."""
    import torch
    nq, nkv, hd, mt = 32, 8, 128, 4097
    rng = np.random.default_rng(31)
    gen = torch.Generator(device="cuda").manual_seed(31)
    B = 3
    kp0 = _gpu_planes(gen, (B, nkv, mt, hd), tqk)
    vp0 = _gpu_planes(gen, (B, nkv, mt, hd), tqk)
    q = rng.standard_normal((B, nq * hd), dtype=np.float32)
    k_new = rng.standard_normal((B, nkv * hd), dtype=np.float32)
    v_new = rng.standard_normal((B, nkv * hd), dtype=np.float32)
    kh0, vh0 = kp0.cpu().numpy(), vp0.cpu().numpy()
    width = hd + 2 if out_mode == 1 else hd
    qd = torch.from_numpy(q).to(cuda)

    def n_splits_of(n, split):
        return n // split + (1 if n % split > split // 4 else 0)

    cases = [(4097, 2048), (4097, 1408), (4097, 1024), (4097, 832), (4097, 704), (4097, 640), (4097, 512),
             (4097, 448), (2560, 256), (4097, 384), (3072, 256), (4097, 320), (3584, 256), (3840, 256), (4097, 256)]
    assert [n_splits_of(n, sp) for n, sp in cases] == list(range(2, 17))
    for (n0, split), device_lens in [(c, dl) for c in cases for dl in (False, True)]:
        lens = np.array([n0, 300, 1] if device_lens else [n0] * B, dtype=np.int32)
        kp, vp = kp0.clone(), vp0.clone()
        out = torch.full((B, nq * width), 7.0, device=cuda)
        length = dict(lens=torch.from_numpy(lens).to(cuda), max_len=n0) if device_lens else dict(len0=n0)
        args = tqk.decode_args(kp, vp, nq, nkv, hd, mt, qd, out, n_items=B, item_stride_blocks=nkv * mt * (hd // 32),
                               q_item_stride=nq * hd, out_item_stride=nq * width, out_mode=out_mode,
                               k_new=torch.from_numpy(k_new).to(cuda), v_new=torch.from_numpy(v_new).to(cuda),
                               kv_new_item_stride=nkv * hd, split_tokens=split, **length)
        tqk.decode(args)
        got = out.cpu().numpy()
        kh, vh = kp.cpu().numpy(), vp.cpu().numpy()
        for b in range(B):
            n = int(lens[b])
            kref, vref = kh0[b].copy(), vh0[b].copy()
            assert port.store_kv(kref, vref, nkv, hd, mt, n - 1, k_new[b], v_new[b]) == 0
            assert np.array_equal(kref, kh[b]) and np.array_equal(vref, vh[b]), (n0, split, b)
            g = got[b].reshape(nq, width)
            if out_mode == 1:
                g = g[:, :hd] / g[:, hd + 1:hd + 2]
            ok, max_abs, rel = tolerance_ok(g.reshape(-1), port.attend(kref, vref, nq, nkv, hd, mt, n - 1, q[b]))
            assert ok, f"{n_splits_of(n0, split)} splits, item {b}: max abs {max_abs:.3g} rel {rel:.3g}"
    # an empty item next to full ones, no append
    lens = np.array([4097, 0, 300], dtype=np.int32)
    out = torch.full((B, nq * width), 7.0, device=cuda)
    tqk.decode(tqk.decode_args(kp0, vp0, nq, nkv, hd, mt, qd, out, n_items=B, item_stride_blocks=nkv * mt * (hd // 32),
                               lens=torch.from_numpy(lens).to(cuda), max_len=4097, q_item_stride=nq * hd,
                               out_item_stride=nq * width, out_mode=out_mode, split_tokens=256))
    got = out.cpu().numpy()
    for b in (0, 2):
        g = got[b].reshape(nq, width)
        if out_mode == 1:
            g = g[:, :hd] / g[:, hd + 1:hd + 2]
        ref = port.attend(kh0[b], vh0[b], nq, nkv, hd, mt, int(lens[b]) - 1, q[b])
        ok, max_abs, rel = tolerance_ok(g.reshape(-1), ref)
        assert ok, f"item {b}: max abs {max_abs:.3g} rel {rel:.3g}"
    e = got[1].reshape(nq, width)
    assert (e[:, :hd] == 0).all()
    if out_mode == 1:
        assert (e[:, hd] == -np.inf).all() and (e[:, hd + 1] == 0).all()
    assert tqk.device_status() == 0


def test_config3_ragged_batch_device_lens(tqk, port, cuda):
    """Config 3: batch 64, lengths ~U[512, 8192], 1% x8 outliers, device lens array."""
    import torch
    B, nq, nkv, hd, mt = 64, 32, 8, 128, 8192
    rng = np.random.default_rng(3)
    lens = rng.integers(512, 8193, B).astype(np.int32)
    gen = torch.Generator(device="cuda").manual_seed(3)
    kp = _gpu_planes(gen, (B, nkv, mt, hd), tqk, 0.01)
    vp = _gpu_planes(gen, (B, nkv, mt, hd), tqk, 0.01)
    q = rng.standard_normal((B, nq * hd), dtype=np.float32)
    out = torch.empty(B, nq * hd, device=cuda)
    lens_d = torch.from_numpy(lens).to(cuda)
    args = tqk.decode_args(kp, vp, nq, nkv, hd, mt, torch.from_numpy(q).to(cuda), out, n_items=B,
                           item_stride_blocks=nkv * mt * (hd // 32), lens=lens_d, max_len=int(lens.max()),
                           q_item_stride=nq * hd, out_item_stride=nq * hd, split_tokens=1024)
    tqk.decode(args)
    got = out.cpu().numpy()
    kh, vh = kp.cpu().numpy(), vp.cpu().numpy()
    for b in range(B):
        ref = port.attend(kh[b], vh[b], nq, nkv, hd, mt, int(lens[b]) - 1, q[b])
        ok, max_abs, rel = tolerance_ok(got[b], ref)
        assert ok, f"seq {b} (len {lens[b]}): max abs {max_abs:.3g} rel {rel:.3g}"
    assert tqk.device_status() == 0


def test_config4_long_context_and_sequence_split_merge(tqk, port, cuda):
    """Config 4: 64 q / 8 kv heads, context 131072.  Also the sequence-split path
    of the multi-GPU version emulated on one device: 4 disjoint token ranges
    written as partials, then the log-sum-exp merge."""
    import torch
    nq, nkv, hd, n = 64, 8, 128, 131072
    gen = torch.Generator(device="cuda").manual_seed(4)
    kp = _gpu_planes(gen, (nkv, n, hd), tqk)
    vp = _gpu_planes(gen, (nkv, n, hd), tqk)
    q = np.random.default_rng(4).standard_normal(nq * hd, dtype=np.float32)
    qd = torch.from_numpy(q).to(cuda)
    out = torch.empty(nq * hd, device=cuda)
    tqk.attend(kp, vp, nq, nkv, hd, n, n - 1, qd, out)
    ref = port.attend(kp.cpu().numpy(), vp.cpu().numpy(), nq, nkv, hd, n, n - 1, q)
    ok, max_abs, rel = tolerance_ok(out.cpu().numpy(), ref)
    assert ok, f"max abs {max_abs:.3g} rel {rel:.3g}"

    parts_n = 4
    shard = n // parts_n
    parts = torch.empty(parts_n, nq * (hd + 2), device=cuda)
    for r in range(parts_n):
        kr = kp[:, r * shard:(r + 1) * shard].contiguous()
        vr = vp[:, r * shard:(r + 1) * shard].contiguous()
        args = tqk.decode_args(kr, vr, nq, nkv, hd, shard, qd, parts[r], len0=shard, out_mode=tqk.OUT_PARTIAL)
        tqk.decode(args)
    merged = torch.empty(nq * hd, device=cuda)
    tqk.merge_partials(parts, parts_n, nq * (hd + 2), nq, hd, merged)
    ok, max_abs, rel = tolerance_ok(merged.cpu().numpy(), ref)
    assert ok, f"merged: max abs {max_abs:.3g} rel {rel:.3g}"


def test_split_invariance_and_caller_workspace(tqk, cuda):
    """The result does not depend on how the sequence is split, and a caller
    workspace gives the same bytes as the library's."""
    import torch
    nq, nkv, hd, n = 32, 8, 128, 5000
    gen = torch.Generator(device="cuda").manual_seed(5)
    kp = _gpu_planes(gen, (nkv, n, hd), tqk)
    vp = _gpu_planes(gen, (nkv, n, hd), tqk)
    q = torch.randn(nq * hd, device=cuda, generator=gen)
    outs = []
    for split in (0, 64, 192, 1024, 4096, 5056):
        out = torch.empty(nq * hd, device=cuda)
        tqk.decode(tqk.decode_args(kp, vp, nq, nkv, hd, n, q, out, len0=n, split_tokens=split))
        outs.append(out.cpu().numpy())
    for o in outs[1:]:
        assert np.abs(o - outs[0]).max() <= 2e-6 * max(1.0, np.abs(outs[0]).max())
    args = tqk.decode_args(kp, vp, nq, nkv, hd, n, q, torch.empty(1, device=cuda), len0=n, split_tokens=64)
    ws = torch.empty(tqk.decode_workspace_size(args), dtype=torch.uint8, device=cuda)
    tqk.workspace_init(ws)
    for _ in range(2):  # the workspace is left reusable
        out = torch.empty(nq * hd, device=cuda)
        args.out = out.data_ptr()
        tqk.decode(args, workspace=ws)
        assert np.array_equal(out.cpu().numpy(), outs[1])


def test_zero_length_items_and_partial_output(tqk, port, cuda):
    import torch
    nq, nkv, hd, mt = 8, 2, 64, 300
    kf, vf, q = decode_case(6, nq, nkv, hd, mt, mt)
    kp = tqk.quantize_rows(torch.from_numpy(kf).to(cuda)).unsqueeze(0).repeat(3, 1, 1, 1).contiguous()
    vp = tqk.quantize_rows(torch.from_numpy(vf).to(cuda)).unsqueeze(0).repeat(3, 1, 1, 1).contiguous()
    lens = torch.tensor([0, 1, 257], dtype=torch.int32, device=cuda)
    qd = torch.from_numpy(q).to(cuda).repeat(3)
    out = torch.full((3, nq * hd), 5.0, device=cuda)
    args = tqk.decode_args(kp, vp, nq, nkv, hd, mt, qd, out, n_items=3, item_stride_blocks=nkv * mt * hd // 32,
                           lens=lens, max_len=257, q_item_stride=nq * hd, out_item_stride=nq * hd, split_tokens=64)
    tqk.decode(args)
    got = out.cpu().numpy()
    assert (got[0] == 0).all()
    kh, vh = kp[0].cpu().numpy(), vp[0].cpu().numpy()
    for i, n in ((1, 1), (2, 257)):
        ok, max_abs, rel = tolerance_ok(got[i], port.attend(kh, vh, nq, nkv, hd, mt, n - 1, q))
        assert ok, (n, max_abs, rel)


@pytest.mark.parametrize("out_mode", [0, 1])
@pytest.mark.parametrize("split", [0, -1])
def test_auto_schedule_ragged_append(tqk, port, cuda, out_mode, split):
    """The automatic split (0) and the balanced schedule (-1, TQK_SPLIT_BALANCED) for 4 q heads
    per kv head (the packed kernel): ragged device lengths with empty items, tile-edge lengths, a
    fused append, both output modes, and a single short sequence."""
    import torch
    nq, nkv, hd, mt = 16, 4, 128, 4200
    lens = np.array([0, 1, 31, 32, 33, 4097, 0, 2048, 100, 4200, 64, 7], dtype=np.int32)
    B = len(lens)
    rng = np.random.default_rng(11)
    gen = torch.Generator(device="cuda").manual_seed(11)
    kp = _gpu_planes(gen, (B, nkv, mt, hd), tqk, 0.01)
    vp = _gpu_planes(gen, (B, nkv, mt, hd), tqk, 0.01)
    q = rng.standard_normal((B, nq * hd), dtype=np.float32)
    k_new = rng.standard_normal((B, nkv * hd), dtype=np.float32)
    v_new = rng.standard_normal((B, nkv * hd), dtype=np.float32)
    kh0, vh0 = kp.cpu().numpy(), vp.cpu().numpy()
    width = hd + 2 if out_mode == 1 else hd
    out = torch.full((B, nq * width), 7.0, device=cuda)
    nonzero = torch.from_numpy(np.maximum(lens, 1)).to(cuda)
    args = tqk.decode_args(kp, vp, nq, nkv, hd, mt, torch.from_numpy(q).to(cuda), out, n_items=B,
                           item_stride_blocks=nkv * mt * (hd // 32), lens=nonzero, max_len=int(lens.max()),
                           q_item_stride=nq * hd, out_item_stride=nq * width, k_new=torch.from_numpy(k_new).to(cuda),
                           v_new=torch.from_numpy(v_new).to(cuda), kv_new_item_stride=nkv * hd, out_mode=out_mode, split_tokens=split)
    tqk.decode(args)
    got = out.cpu().numpy()
    kh, vh = kp.cpu().numpy(), vp.cpu().numpy()
    for b in range(B):
        n = max(int(lens[b]), 1)
        kref, vref = kh0[b].copy(), vh0[b].copy()
        assert port.store_kv(kref, vref, nkv, hd, mt, n - 1, k_new[b], v_new[b]) == 0
        assert np.array_equal(kref, kh[b]) and np.array_equal(vref, vh[b]), f"append item {b}"
        ref = port.attend(kref, vref, nq, nkv, hd, mt, n - 1, q[b])
        g = got[b].reshape(nq, width)
        if out_mode == 1:  # acc, m (natural log), l per head
            g = g[:, :hd] / g[:, hd + 1:hd + 2]
        ok, max_abs, rel = tolerance_ok(g.reshape(-1), ref)
        assert ok, f"item {b} (len {n}): max abs {max_abs:.3g} rel {rel:.3g}"

    # zero-length items without an append, and the single-item case with fewer tiles than CTAs
    lens_d = torch.from_numpy(lens).to(cuda)
    out = torch.full((B, nq * hd), 7.0, device=cuda)
    args = tqk.decode_args(kp, vp, nq, nkv, hd, mt, torch.from_numpy(q).to(cuda), out, n_items=B,
                           item_stride_blocks=nkv * mt * (hd // 32), lens=lens_d, max_len=int(lens.max()),
                           q_item_stride=nq * hd, out_item_stride=nq * hd, split_tokens=split)
    tqk.decode(args)
    got = out.cpu().numpy()
    for b in range(B):
        if lens[b] == 0:
            assert (got[b] == 0).all()
        else:
            ok, max_abs, rel = tolerance_ok(got[b], port.attend(kh[b], vh[b], nq, nkv, hd, mt, int(lens[b]) - 1, q[b]))
            assert ok, f"item {b}: max abs {max_abs:.3g} rel {rel:.3g}"
    one = torch.empty(nq * hd, device=cuda)
    tqk.attend(kp[9], vp[9], nq, nkv, hd, mt, 39, torch.from_numpy(q[9]).to(cuda), one)
    ok, max_abs, rel = tolerance_ok(one.cpu().numpy(), port.attend(kh[9], vh[9], nq, nkv, hd, mt, 39, q[9]))
    assert ok, (max_abs, rel)
    assert tqk.device_status() == 0


@pytest.mark.parametrize("n_items", [256, 300])
def test_balanced_schedule_items_and_workspace_reuse(tqk, port, cuda, n_items):
    """The packed kernel's balanced schedule (TQK_SPLIT_BALANCED): up to 256 items the units'
    tiles are cut into equal per-CTA runs that cross unit boundaries (256 here, with empty and
    one-token items); above that it falls back to the fixed split (300).  Checked against the oracle on a sample
    of items; repeated calls through one caller workspace give identical bytes (the tickets
    are left at zero), and so does a fixed-split call in between."""
    import torch
    nq, nkv, hd, mt = 8, 2, 128, 300
    rng = np.random.default_rng(21 + n_items)
    lens = rng.integers(1, mt + 1, n_items).astype(np.int32)
    lens[::37] = 0
    lens[5] = 1
    lens[6] = mt
    gen = torch.Generator(device="cuda").manual_seed(21)
    kp = _gpu_planes(gen, (n_items, nkv, mt, hd), tqk)
    vp = _gpu_planes(gen, (n_items, nkv, mt, hd), tqk)
    q = torch.from_numpy(rng.standard_normal((n_items, nq * hd), dtype=np.float32)).to(cuda)
    lens_d = torch.from_numpy(lens).to(cuda)

    def call(split, ws=None):
        out = torch.full((n_items, nq * hd), 3.0, device=cuda)
        a = tqk.decode_args(kp, vp, nq, nkv, hd, mt, q, out, n_items=n_items,
                            item_stride_blocks=nkv * mt * (hd // 32), lens=lens_d, max_len=int(lens.max()),
                            q_item_stride=nq * hd, out_item_stride=nq * hd, split_tokens=split)
        tqk.decode(a, workspace=ws)
        return out.cpu().numpy(), a

    bal = tqk.SPLIT_BALANCED
    first, a = call(bal)
    ws = torch.empty(max(tqk.decode_workspace_size(a), 1 << 24), dtype=torch.uint8, device=cuda)
    tqk.workspace_init(ws)
    assert np.array_equal(call(bal, ws)[0], first)
    fixed = call(64, ws)[0]
    assert np.array_equal(call(bal, ws)[0], first)
    assert np.abs(call(0, ws)[0] - first).max() <= 2e-6 * max(1.0, np.abs(first).max())  # the automatic choice
    assert np.abs(fixed - first).max() <= 2e-6 * max(1.0, np.abs(first).max())
    kh, vh, qh = kp.cpu().numpy(), vp.cpu().numpy(), q.cpu().numpy()
    for b in (0, 5, 6, 37, 100, n_items - 1):
        if lens[b] == 0:
            assert (first[b] == 0).all(), b
            continue
        ok, max_abs, rel = tolerance_ok(first[b], port.attend(kh[b], vh[b], nq, nkv, hd, mt, int(lens[b]) - 1, qh[b]))
        assert ok, f"item {b} (len {lens[b]}): max abs {max_abs:.3g} rel {rel:.3g}"
    assert tqk.device_status() == 0


def test_balanced_schedule_long_ragged_two_level_merge(tqk, port, cuda):
    """Two items of very different lengths on the balanced schedule: the long one's units are
    each covered by dozens of CTAs, so their partials go through the two-level (group, then
    final) merge; the short one's units sit inside one CTA's run.  With a fused append."""
    import torch
    nq, nkv, hd, mt = 32, 8, 128, 20000
    lens = np.array([20000, 100], dtype=np.int32)
    rng = np.random.default_rng(23)
    gen = torch.Generator(device="cuda").manual_seed(23)
    kp = _gpu_planes(gen, (2, nkv, mt, hd), tqk)
    vp = _gpu_planes(gen, (2, nkv, mt, hd), tqk)
    q = rng.standard_normal((2, nq * hd), dtype=np.float32)
    k_new = rng.standard_normal((2, nkv * hd), dtype=np.float32)
    v_new = rng.standard_normal((2, nkv * hd), dtype=np.float32)
    kh0, vh0 = kp.cpu().numpy(), vp.cpu().numpy()
    out = torch.empty(2, nq * hd, device=cuda)
    args = tqk.decode_args(kp, vp, nq, nkv, hd, mt, torch.from_numpy(q).to(cuda), out, n_items=2,
                           item_stride_blocks=nkv * mt * (hd // 32), lens=torch.from_numpy(lens).to(cuda),
                           max_len=int(lens.max()), q_item_stride=nq * hd, out_item_stride=nq * hd,
                           k_new=torch.from_numpy(k_new).to(cuda), v_new=torch.from_numpy(v_new).to(cuda),
                           kv_new_item_stride=nkv * hd, split_tokens=tqk.SPLIT_BALANCED)
    tqk.decode(args)
    got = out.cpu().numpy()
    kh, vh = kp.cpu().numpy(), vp.cpu().numpy()
    for b in range(2):
        n = int(lens[b])
        kref, vref = kh0[b].copy(), vh0[b].copy()
        assert port.store_kv(kref, vref, nkv, hd, mt, n - 1, k_new[b], v_new[b]) == 0
        assert np.array_equal(kref, kh[b]) and np.array_equal(vref, vh[b]), f"append item {b}"
        ok, max_abs, rel = tolerance_ok(got[b], port.attend(kref, vref, nq, nkv, hd, mt, n - 1, q[b]))
        assert ok, f"item {b} (len {n}): max abs {max_abs:.3g} rel {rel:.3g}"
    assert tqk.device_status() == 0


def test_config3_auto_schedule(tqk, port, cuda):
    """Config 3 through the automatic split, checked against an explicit split
    and, on a sample of sequences, the oracle."""
    import torch
    B, nq, nkv, hd, mt = 64, 32, 8, 128, 8192
    rng = np.random.default_rng(13)
    lens = rng.integers(512, 8193, B).astype(np.int32)
    gen = torch.Generator(device="cuda").manual_seed(13)
    kp = _gpu_planes(gen, (B, nkv, mt, hd), tqk, 0.01)
    vp = _gpu_planes(gen, (B, nkv, mt, hd), tqk, 0.01)
    q = torch.from_numpy(rng.standard_normal((B, nq * hd), dtype=np.float32)).to(cuda)
    lens_d = torch.from_numpy(lens).to(cuda)
    outs = []
    for split in (0, tqk.SPLIT_BALANCED, 1024):
        out = torch.empty(B, nq * hd, device=cuda)
        tqk.decode(tqk.decode_args(kp, vp, nq, nkv, hd, mt, q, out, n_items=B,
                                   item_stride_blocks=nkv * mt * (hd // 32), lens=lens_d, max_len=int(lens.max()),
                                   q_item_stride=nq * hd, out_item_stride=nq * hd, split_tokens=split))
        outs.append(out.cpu().numpy())
    # schedules differ only in where fp32 partials are merged
    for o in outs[:2]:
        assert np.abs(o - outs[2]).max() <= 1e-5 * max(1.0, np.abs(outs[2]).max())
    kh, vh, qh = kp.cpu().numpy(), vp.cpu().numpy(), q.cpu().numpy()
    for b in (0, 17, 63):
        ok, max_abs, rel = tolerance_ok(outs[0][b], port.attend(kh[b], vh[b], nq, nkv, hd, mt, int(lens[b]) - 1, qh[b]))
        assert ok, f"seq {b}: max abs {max_abs:.3g} rel {rel:.3g}"
    assert tqk.device_status() == 0


def test_prefill_matches_golden_and_sequential(tqk, port, cuda):
    import torch
    from _cases import prefill_inputs
    g = np.load(os.path.join(GOLDEN, "prefill.npz"))
    seed, nq, nkv, hd, mt, pos0, n = (int(v) for v in g["params"])
    kf, vf, qn, kn, vn = prefill_inputs(seed, nq, nkv, hd, mt, pos0, n)
    kp = tqk.quantize_rows(torch.from_numpy(kf).to(cuda))
    vp = tqk.quantize_rows(torch.from_numpy(vf).to(cuda))
    out = torch.empty(n * nq * hd, device=cuda)
    tqk.prefill(kp, vp, nq, nkv, hd, mt, pos0, n, torch.from_numpy(qn).to(cuda), torch.from_numpy(kn).to(cuda),
                torch.from_numpy(vn).to(cuda), out)
    assert np.array_equal(kp.cpu().numpy()[:, pos0:pos0 + n], g["kp"])
    assert np.array_equal(vp.cpu().numpy()[:, pos0:pos0 + n], g["vp"])
    ok, max_abs, rel = tolerance_ok(out.cpu().numpy(), g["out"])
    assert ok, (max_abs, rel)


PREFILL_TC = ["g4", "g4_at0_n1", "g4_at0", "g4_x30", "g4_outliers", "g8", "g2", "g1"]


@pytest.mark.parametrize("name", PREFILL_TC)
def test_prefill_tensor_core_golden(tqk, port, cuda, name):
    """The tcgen05 prefill (head_dim 128, 1/2/4/8 q heads per kv head) against chunks the
    reference's own attention_layer_batch produced (tests/golden/prefill_tc.npz): appended rows
    bit-exact, attention within the 1e-3 tolerance -- including one token at position 0, a chunk
    over an empty cache, the reference's x30 large-score scaling and x8 outlier blocks."""
    import torch
    from _cases import prefill_inputs
    g = np.load(os.path.join(GOLDEN, "prefill_tc.npz"))
    seed, nq, nkv, hd, mt, pos0, n, qs, of = (int(v) for v in g[f"{name}__params"])
    kf, vf, qn, kn, vn = prefill_inputs(seed, nq, nkv, hd, mt, pos0, n, float(qs), of / 1e6)
    kp = tqk.quantize_rows(torch.from_numpy(kf).to(cuda))
    vp = tqk.quantize_rows(torch.from_numpy(vf).to(cuda))
    out = torch.full((n, nq * hd), float("nan"), device=cuda)
    tqk.prefill(kp, vp, nq, nkv, hd, mt, pos0, n, torch.from_numpy(qn).to(cuda), torch.from_numpy(kn).to(cuda),
                torch.from_numpy(vn).to(cuda), out)
    assert np.array_equal(kp.cpu().numpy()[:, pos0:pos0 + n], g[f"{name}__kp"])
    assert np.array_equal(vp.cpu().numpy()[:, pos0:pos0 + n], g[f"{name}__vp"])
    ok, max_abs, rel = tolerance_ok(out.cpu().numpy(), g[f"{name}__out"])
    print(f"prefill {name}: max abs {max_abs:.3g} rel {rel:.3g}")
    assert ok, f"{name}: max abs {max_abs:.3g} rel {rel:.3g}"
    assert tqk.device_status() == 0


@pytest.mark.parametrize("nq,nkv,pos0,n,mt", [
    (8, 8, 0, 1, 64),        # one token, group 1
    (16, 8, 5, 77, 100),     # group 2, ragged last CTA
    (32, 8, 2000, 40, 2100), # group 4, partial key tiles
    (32, 4, 100, 300, 500),  # group 8
    (32, 32, 64, 130, 200),  # group 1, 128 tokens per CTA
    (32, 2, 10, 20, 40),     # group 16: not a tensor-core shape, decode kernel
])
def test_prefill_tensor_core_shapes(tqk, port, cuda, nq, nkv, pos0, n, mt):
    """tqk_prefill_q8 (the tcgen05 prefill kernel for head_dim 128) against the
    oracle's attention_layer_batch restatement: appended rows bit-exact,
    attention within tolerance, for several group sizes and ragged tiles."""
    import torch
    hd = 128
    rng = np.random.default_rng(nq * 1000 + n)
    kf = np.zeros((nkv, mt, hd), np.float32)
    vf = np.zeros((nkv, mt, hd), np.float32)
    kf[:, :pos0] = rng.standard_normal((nkv, pos0, hd))
    vf[:, :pos0] = rng.standard_normal((nkv, pos0, hd))
    qn = rng.standard_normal((n, nq * hd)).astype(np.float32)
    kn = rng.standard_normal((n, nkv * hd)).astype(np.float32)
    vn = rng.standard_normal((n, nkv * hd)).astype(np.float32)
    kp = tqk.quantize_rows(torch.from_numpy(kf).to(cuda))
    vp = tqk.quantize_rows(torch.from_numpy(vf).to(cuda))
    kh, vh = kp.cpu().numpy(), vp.cpu().numpy()
    out = torch.full((n, nq * hd), float("nan"), device=cuda)
    tqk.prefill(kp, vp, nq, nkv, hd, mt, pos0, n, torch.from_numpy(qn).to(cuda), torch.from_numpy(kn).to(cuda),
                torch.from_numpy(vn).to(cuda), out)
    ref = port.prefill(kh, vh, nq, nkv, hd, mt, pos0, n, qn, kn, vn).reshape(n, nq * hd)
    assert np.array_equal(kp.cpu().numpy(), kh) and np.array_equal(vp.cpu().numpy(), vh)  # oracle appended in place
    got = out.cpu().numpy()
    ok, max_abs, rel = tolerance_ok(got, ref)
    assert ok, f"max abs {max_abs:.3g} rel {rel:.3g}"
    assert tqk.device_status() == 0


def test_config5_prefill_full(tqk, port, cuda):
    """Config 5: 2048 new tokens at positions 2048..4095 over a 2048-token Q8
    cache, 32 q / 8 kv heads, causal -- checked on a spread of query tokens."""
    import torch
    nq, nkv, hd, pos0, n = 32, 8, 128, 2048, 2048
    mt = pos0 + n
    gen = torch.Generator(device="cuda").manual_seed(55)
    kfull = torch.zeros(nkv, mt, hd, device=cuda)
    vfull = torch.zeros(nkv, mt, hd, device=cuda)
    kfull[:, :pos0] = torch.randn(nkv, pos0, hd, device=cuda, generator=gen)
    vfull[:, :pos0] = torch.randn(nkv, pos0, hd, device=cuda, generator=gen)
    kp, vp = tqk.quantize_rows(kfull), tqk.quantize_rows(vfull)
    qn = torch.randn(n, nq * hd, device=cuda, generator=gen)
    kn = torch.randn(n, nkv * hd, device=cuda, generator=gen)
    vn = torch.randn(n, nkv * hd, device=cuda, generator=gen)
    out = torch.empty(n, nq * hd, device=cuda)
    tqk.prefill(kp, vp, nq, nkv, hd, mt, pos0, n, qn, kn, vn, out)
    kh, vh = kp.cpu().numpy(), vp.cpu().numpy()
    # the appended K and V rows are the reference quantiser's
    assert np.array_equal(kh[:, pos0:], port.quantize_rows(kn.cpu().numpy().reshape(n, nkv, hd).transpose(1, 0, 2)))
    assert np.array_equal(vh[:, pos0:], port.quantize_rows(vn.cpu().numpy().reshape(n, nkv, hd).transpose(1, 0, 2)))
    got, qh = out.cpu().numpy(), qn.cpu().numpy()
    for i in (0, 1, 17, 511, 1024, 2046, 2047):
        ref = port.attend(kh, vh, nq, nkv, hd, mt, pos0 + i, qh[i])
        ok, max_abs, rel = tolerance_ok(got[i], ref)
        assert ok, f"token {i}: max abs {max_abs:.3g} rel {rel:.3g}"
    assert tqk.device_status() == 0


def test_bad_arguments_are_rejected(tqk, cuda):
    import torch
    kp = torch.zeros(8, 16, 144, dtype=torch.uint8, device=cuda)
    q = torch.zeros(32 * 128, device=cuda)
    out = torch.zeros(32 * 128, device=cuda)
    with pytest.raises(tqk.TQKError) as e:
        tqk.attend(kp, kp, 32, 8, 128, 16, 16, q, out)
    assert e.value.status == tqk.EPOS
    args = tqk.decode_args(kp.view(-1)[4:], kp, 32, 8, 128, 15, q, out, len0=3)  # 4-byte offset planes
    with pytest.raises(tqk.TQKError) as e:
        tqk.decode(args)
    assert e.value.status == tqk.EALIGN
