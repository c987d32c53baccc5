"""GPU parity of the attention prologue tqk_qk_norm_rope: per-head RMSNorm of q
and k (norm_heads, model/attention_layer.c:48-60 over model/rmsnorm.c:4-19)
followed by RoPE (rope_heads with the table of model/rope.c:4-22), as
attention_layer.c:183-189 applies them before store_kv and attend_q8.

Bar: bit-exact with the reference's outputs (tests/golden/norm_rope.npz) and
with the pinned oracle restatement; composed with the decode's fused append,
the appended Q8 rows are bit-exact and the attention meets the decode
tolerance (max abs <= 1e-3, rel <= 1e-3).
"""
import os

import numpy as np
import pytest

import oracle
from _cases import digest, norm_rope_inputs, tolerance_ok

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")

# name: (seed, n_items, n_q, n_kv, hd, first_pos, theta, eps, per_item_weights, norm); the cases of
# tests/golden/make_golden.py.
GOLDEN_CASES = {
    "qwen3_like": (41, 1, 32, 8, 128, 4096, 1000000.0, 1e-6, False, True),
    "llama3_rope_only": (42, 1, 32, 8, 128, 4096, 500000.0, 1e-5, False, False),
    "batch3_hd64": (43, 3, 6, 2, 64, 17, 10000.0, 1e-6, True, True),
}


@pytest.fixture(scope="module")
def tqk(cuda):
    from tailorquantkernel_b200 import tqk as t
    return t


@pytest.fixture(scope="module")
def port():
    return oracle.Oracle("port")


def _bits(x):
    return np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)


@pytest.mark.parametrize("name", sorted(GOLDEN_CASES))
def test_norm_rope_matches_golden(tqk, cuda, name):
    import torch
    g = np.load(os.path.join(GOLDEN, "norm_rope.npz"))
    seed, items, nq, nkv, hd, p0, theta, eps, per_item, norm = GOLDEN_CASES[name]
    q, k, qw, kw = norm_rope_inputs(seed, items, nq, nkv, hd, per_item)
    assert digest(q, k, qw, kw) == str(g[name + "__in_sha"])
    dq, dk = torch.from_numpy(q).to(cuda), torch.from_numpy(k).to(cuda)
    cos = torch.from_numpy(g[name + "__cos"]).to(cuda)
    sin = torch.from_numpy(g[name + "__sin"]).to(cuda)
    qn = torch.from_numpy(qw).to(cuda) if norm else None
    kn = torch.from_numpy(kw).to(cuda) if norm else None
    tqk.qk_norm_rope(dq, dk, items, nq, nkv, hd, qn, kn, eps, cos, sin,
                     norm_item_stride=hd if per_item else 0, rope_item_stride=hd // 2)
    torch.cuda.synchronize()
    assert np.array_equal(_bits(dq.cpu().numpy()), _bits(g[name + "__q"]))
    assert np.array_equal(_bits(dk.cpu().numpy()), _bits(g[name + "__k"]))


@pytest.mark.parametrize("items,nq,nkv,hd,norm,rope,pad", [
    (32, 32, 8, 128, True, True, 0),      # config 2: every layer of one token, per-layer weights
    (32, 32, 8, 128, False, True, 0),     # Llama-3: RoPE only
    (4, 64, 8, 128, True, False, 0),      # norm only
    (5, 4, 2, 32, True, True, 96),        # strided items
    (2, 2, 2, 256, True, True, 0),
    (7, 6, 1, 64, True, True, 64),
])
def test_norm_rope_sweep_vs_oracle(tqk, port, cuda, items, nq, nkv, hd, norm, rope, pad):
    import torch
    rng = np.random.default_rng(1000 + items * 10 + hd)
    qs, ks = nq * hd + pad, nkv * hd + pad
    q = rng.standard_normal((items, qs), dtype=np.float32) * np.float32(3.0)
    k = rng.standard_normal((items, ks), dtype=np.float32)
    q[0, :hd] = 0.0                                   # a zero head: rms = sqrt(eps)
    qw = rng.standard_normal((items, hd), dtype=np.float32)
    kw = rng.standard_normal((items, hd), dtype=np.float32)
    cos = np.zeros((items, hd // 2), np.float32)
    sin = np.zeros((items, hd // 2), np.float32)
    for it in range(items):
        cos[it], sin[it] = port.rope_table(hd, 4096 + 97 * it, 500000.0)
    eq, ek = q.copy(), k.copy()
    for it in range(items):
        eq[it, :nq * hd] = port.qk_norm_rope(q[it, :nq * hd], nq, hd, qw[it] if norm else None, 1e-6,
                                             cos[it] if rope else None, sin[it])
        ek[it, :nkv * hd] = port.qk_norm_rope(k[it, :nkv * hd], nkv, hd, kw[it] if norm else None, 1e-6,
                                              cos[it] if rope else None, sin[it])
    dq, dk = torch.from_numpy(q).to(cuda), torch.from_numpy(k).to(cuda)
    dev = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    tqk.qk_norm_rope(dq, dk, items, nq, nkv, hd, dev(qw) if norm else None, dev(kw) if norm else None, 1e-6,
                     dev(cos) if rope else None, dev(sin) if rope else None, q_item_stride=qs, k_item_stride=ks,
                     norm_item_stride=hd, rope_item_stride=hd // 2)
    torch.cuda.synchronize()
    assert np.array_equal(_bits(dq.cpu().numpy()), _bits(eq))   # padding untouched too
    assert np.array_equal(_bits(dk.cpu().numpy()), _bits(ek))


def test_norm_rope_then_fused_append(tqk, port, cuda):
    """The layer's order (attention_layer.c:183-190): norm + RoPE of q and k, then store_kv + attend_q8
    as one decode launch.  The appended Q8 row equals the oracle's quantisation of the normed k."""
    import torch
    nq, nkv, hd, pos = 32, 8, 128, 300
    mt = pos + 1
    rng = np.random.default_rng(77)
    kf = rng.standard_normal((nkv, mt, hd), dtype=np.float32)
    vf = rng.standard_normal((nkv, mt, hd), dtype=np.float32)
    kf[:, pos] = 0
    vf[:, pos] = 0
    q, k, qw, kw = norm_rope_inputs(78, 1, nq, nkv, hd, False)
    v = rng.standard_normal(nkv * hd, dtype=np.float32)
    cos, sin = port.rope_table(hd, pos, 1000000.0)
    qe = port.qk_norm_rope(q[0], nq, hd, qw[0], 1e-6, cos, sin)
    ke = port.qk_norm_rope(k[0], nkv, hd, kw[0], 1e-6, cos, sin)
    kp_e, vp_e = port.quantize_rows(kf), port.quantize_rows(vf)
    kp_e[:, pos] = port.quantize_rows(ke.reshape(nkv, 1, hd))[:, 0]
    vp_e[:, pos] = port.quantize_rows(v.reshape(nkv, 1, hd))[:, 0]
    ref = port.attend(kp_e, vp_e, nq, nkv, hd, mt, pos, qe)

    kp = tqk.quantize_rows(torch.from_numpy(kf).to(cuda))
    vp = tqk.quantize_rows(torch.from_numpy(vf).to(cuda))
    dq, dk, dv = (torch.from_numpy(np.ascontiguousarray(a)).to(cuda) for a in (q[0], k[0], v))
    tqk.qk_norm_rope(dq, dk, 1, nq, nkv, hd, torch.from_numpy(qw[0]).to(cuda), torch.from_numpy(kw[0]).to(cuda),
                     1e-6, torch.from_numpy(cos).to(cuda), torch.from_numpy(sin).to(cuda))
    out = torch.empty(nq * hd, device=cuda)
    tqk.append_attend(kp, vp, nq, nkv, hd, mt, pos, dq, dk, dv, out)
    torch.cuda.synchronize()
    assert np.array_equal(kp.cpu().numpy(), kp_e) and np.array_equal(vp.cpu().numpy(), vp_e)
    ok, max_abs, rel = tolerance_ok(out.cpu().numpy(), ref)
    assert ok, (max_abs, rel)


def test_norm_rope_argument_errors(tqk, cuda):
    import torch
    q = torch.zeros(4 * 64, device=cuda)
    k = torch.zeros(2 * 64, device=cuda)
    w = torch.ones(64, device=cuda)
    for kwargs in (dict(head_dim=63), dict(n_items=0), dict(q_norm=w), dict(rope_cos=w)):
        args = dict(n_items=1, n_q=4, n_kv=2, head_dim=64)
        args.update(kwargs)
        with pytest.raises(tqk.TQKError):
            tqk.qk_norm_rope(q, k, **args)


@pytest.mark.parametrize("nq,nkv,hd,items,n,split", [
    (32, 8, 128, 3, 300, 0),      # packed kernel (4 q heads per kv head), per-item weights and tables
    (32, 8, 128, 2, 1000, 64),    # packed kernel, 16 splits: every split CTA normalises its q rows
    (64, 8, 128, 2, 257, 0),      # tensor-core kernel, group 8
    (16, 2, 256, 1, 130, 64),     # tensor-core kernel, head_dim 256
    (8, 2, 64, 2, 90, 0),         # CUDA-core kernel
    (4, 4, 32, 3, 40, 0),         # CUDA-core kernel, head_dim 32: RoPE pairs cross lanes
])
@pytest.mark.parametrize("mode", ["norm+rope", "rope", "norm"])
def test_fused_prologue_decode(tqk, port, cuda, nq, nkv, hd, items, n, split, mode):
    """tqk_decode_q8 with the prologue fields set == tqk_qk_norm_rope followed by the plain decode,
    bit for bit (output and appended rows); the appended rows equal the oracle's quantisation of
    the normed k and the output meets the decode tolerance against the oracle; q and k_new are
    left untouched."""
    import torch
    norm, rope = "norm" in mode, "rope" in mode
    mt = n + 3
    rng = np.random.default_rng(4000 + nq + hd + n)
    gen = torch.Generator(device="cuda").manual_seed(n)
    kf = torch.randn((items, nkv, mt, hd), device=cuda, generator=gen)
    vf = torch.randn((items, nkv, mt, hd), device=cuda, generator=gen)
    kf[:, :, n - 1:] = 0
    vf[:, :, n - 1:] = 0
    q = torch.from_numpy(rng.standard_normal((items, nq * hd), dtype=np.float32) * np.float32(3)).to(cuda)
    kn = torch.from_numpy(rng.standard_normal((items, nkv * hd), dtype=np.float32)).to(cuda)
    vn = torch.from_numpy(rng.standard_normal((items, nkv * hd), dtype=np.float32)).to(cuda)
    qw = torch.from_numpy(1 + 0.2 * rng.standard_normal((items, hd), dtype=np.float32)).to(cuda) if norm else None
    kw = torch.from_numpy(1 + 0.2 * rng.standard_normal((items, hd), dtype=np.float32)).to(cuda) if norm else None
    cos = np.zeros((items, hd // 2), np.float32)
    sin = np.zeros((items, hd // 2), np.float32)
    for it in range(items):
        cos[it], sin[it] = port.rope_table(hd, n - 1, 1000000.0)
    dcos = torch.from_numpy(cos).to(cuda) if rope else None
    dsin = torch.from_numpy(sin).to(cuda) if rope else None
    plane = nkv * mt * (hd // 32)  # Q8 blocks per item
    common = dict(n_items=items, item_stride_blocks=plane, len0=n, q_item_stride=nq * hd, out_item_stride=nq * hd,
                  kv_new_item_stride=nkv * hd, split_tokens=split)
    pro = dict(q_norm=qw, k_norm=kw, norm_item_stride=hd, norm_eps=1e-6, rope_cos=dcos, rope_sin=dsin,
               rope_item_stride=hd // 2)

    # fused
    kp, vp = tqk.quantize_rows(kf), tqk.quantize_rows(vf)
    q0, kn0 = q.clone(), kn.clone()
    out = torch.empty(items, nq * hd, device=cuda)
    tqk.decode(tqk.decode_args(kp, vp, nq, nkv, hd, mt, q, out, k_new=kn, v_new=vn, **common, **pro))
    # two steps
    kp2, vp2 = tqk.quantize_rows(kf), tqk.quantize_rows(vf)
    q2, kn2 = q.clone(), kn.clone()
    tqk.qk_norm_rope(q2, kn2, items, nq, nkv, hd, qw, kw, 1e-6, dcos, dsin, norm_item_stride=hd,
                     rope_item_stride=hd // 2)
    out2 = torch.empty(items, nq * hd, device=cuda)
    tqk.decode(tqk.decode_args(kp2, vp2, nq, nkv, hd, mt, q2, out2, k_new=kn2, v_new=vn, **common))
    torch.cuda.synchronize()
    assert torch.equal(q, q0) and torch.equal(kn, kn0)
    assert torch.equal(kp, kp2) and torch.equal(vp, vp2)
    assert torch.equal(out.view(torch.int32), out2.view(torch.int32))

    kpn, vpn, qn = kp.cpu().numpy(), vp.cpu().numpy(), q.cpu().numpy()
    for it in range(items):
        w_q = qw[it].cpu().numpy() if norm else None
        w_k = kw[it].cpu().numpy() if norm else None
        c, s = (cos[it], sin[it]) if rope else (None, None)
        ke = port.qk_norm_rope(kn[it].cpu().numpy(), nkv, hd, w_k, 1e-6, c, s)
        assert np.array_equal(kpn[it, :, n - 1], port.quantize_rows(ke.reshape(nkv, hd)))
        qe = port.qk_norm_rope(qn[it], nq, hd, w_q, 1e-6, c, s)
        ref = port.attend(kpn[it], vpn[it], nq, nkv, hd, mt, n - 1, qe)
        ok, max_abs, rel = tolerance_ok(out[it].cpu().numpy(), ref)
        assert ok, (it, max_abs, rel)
