"""GPU parity of tqk_attention_layer: one token through one attention layer
on the device (attention_layer, model/attention_layer.c:169-194).

Bar: the appended cache rows are bit-exact with the reference's (the q/k/v
projections, norm, RoPE and quantisation are all bit-exact); the output goes
through the decode attention (within 1e-3 of the reference) and the output
projection, so it is held to max |diff| <= 1e-3 * max |reference output|.
References: tests/golden/layer.npz (the reference's own attention_layer) and
the pinned oracle composition for multi-token runs.
"""
import os

import numpy as np
import pytest

import oracle
from _cases import digest, layer_inputs

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")

# tests/golden/make_golden.py LAYER_CASES: (seed, n_q, n_kv, hd, hidden, max_tokens, pos, theta, eps)
LAYER_CASES = {
    "small_g4": (61, 8, 2, 64, 256, 40, 25, 1000000.0, 1e-6),
    "llama_heads": (62, 32, 8, 128, 512, 70, 64, 500000.0, 1e-5),
}
OUT_RTOL = 1e-3


@pytest.fixture(scope="module")
def tqk(cuda):
    from tailorquantkernel_b200 import tqk as t
    return t


@pytest.fixture(scope="module")
def port():
    return oracle.Oracle("port")


def _dev(a, cuda):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def _out_ok(got, ref):
    return float(np.abs(got - ref).max()) <= OUT_RTOL * float(np.abs(ref).max())


class _Layer:
    """Device copies of one layer case (weights, norms, cache planes, buffers)."""

    def __init__(self, tqk, port, cuda, case, fmt):
        import torch
        seed, nq, nkv, hd, hidden, mt, pos, theta, eps = case
        self.shape = (nq, nkv, hd, hidden, mt, theta, eps)
        w, qn, kn, kp, vp, xn = layer_inputs(seed, nq, nkv, hd, hidden, mt, pos, fmt, port)
        self.host = dict(w=w, qn=qn, kn=kn, kp=kp, vp=vp, xn=xn)
        self.w = {n: _dev(a, cuda) for n, a in w.items()}
        self.qn, self.kn = _dev(qn, cuda), _dev(kn, cuda)
        self.kp, self.vp = _dev(kp, cuda), _dev(vp, cuda)
        self.xn = _dev(xn, cuda)
        self.out = torch.empty(hidden, device=cuda)
        self.scratch = torch.empty(tqk.layer_scratch_floats(nq, nkv, hd), device=cuda)
        self.cos = torch.empty(hd // 2, device=cuda)
        self.sin = torch.empty(hd // 2, device=cuda)
        self.fmt = tqk.FMT_Q8 if fmt == "8" else tqk.FMT_Q4

    def args(self, tqk, pos, len_dev=None):
        nq, nkv, hd, hidden, mt, theta, eps = self.shape
        return tqk.attention_layer_args(self.w, self.fmt, self.qn, self.kn, nq, nkv, hd, hidden, eps, self.kp,
                                        self.vp, mt, pos, self.cos, self.sin, self.xn, self.out, self.scratch,
                                        len_dev)


@pytest.mark.parametrize("name", sorted(LAYER_CASES))
@pytest.mark.parametrize("fmt", ["8", "4"])
@pytest.mark.parametrize("device_len", [False, True])
def test_layer_matches_golden(tqk, port, cuda, name, fmt, device_len):
    import torch
    case = LAYER_CASES[name]
    seed, nq, nkv, hd, hidden, mt, pos, theta, eps = case
    g = np.load(os.path.join(GOLDEN, "layer.npz"))
    key = f"{name}_q{fmt}"
    lay = _Layer(tqk, port, cuda, case, fmt)
    h = lay.host
    assert digest(*[h["w"][n] for n in ("wq", "wk", "wv", "wo")], h["qn"], h["kn"], h["kp"], h["vp"],
                  h["xn"]) == str(g[key + "__in_sha"])
    c, s = port.rope_table(hd, pos, theta)
    lay.cos.copy_(torch.from_numpy(c))
    lay.sin.copy_(torch.from_numpy(s))
    len_dev = torch.tensor([pos + 1], dtype=torch.int32, device=cuda) if device_len else None
    tqk.attention_layer(lay.args(tqk, pos, len_dev))
    torch.cuda.synchronize()
    assert np.array_equal(lay.kp.cpu().numpy()[:, pos], g[key + "__k_row"])
    assert np.array_equal(lay.vp.cpu().numpy()[:, pos], g[key + "__v_row"])
    assert _out_ok(lay.out.cpu().numpy(), g[key + "__out"])


@pytest.mark.parametrize("fmt", ["8", "4"])
def test_layer_graph_replay_over_tokens(tqk, port, cuda, fmt):
    """A CUDA graph of one tqk_attention_layer call replayed for consecutive tokens: the position
    comes from a device int and the RoPE table / input from device buffers updated before each
    replay.  Every token's appended rows are bit-exact and its output within tolerance of the
    oracle's attention_layer on the same evolving cache."""
    import torch
    case = LAYER_CASES["llama_heads"]
    seed, nq, nkv, hd, hidden, mt, pos0, theta, eps = case
    lay = _Layer(tqk, port, cuda, case, fmt)
    kp_ref, vp_ref = lay.host["kp"].copy(), lay.host["vp"].copy()
    len_dev = torch.tensor([pos0 + 1], dtype=torch.int32, device=cuda)
    ws = torch.zeros(1 << 22, dtype=torch.uint8, device=cuda)
    stream = torch.cuda.Stream()
    steps = 4
    args = lay.args(tqk, pos0 + steps - 1, len_dev)  # pos bounds the grid; the device int is the length
    rng = np.random.default_rng(5)
    xs = [rng.standard_normal(hidden, dtype=np.float32) for _ in range(steps)]
    with torch.cuda.stream(stream):
        tqk.workspace_init(ws, stream)
        lay.xn.copy_(torch.from_numpy(xs[0]))
        c, s = port.rope_table(hd, pos0, theta)
        lay.cos.copy_(torch.from_numpy(c))
        lay.sin.copy_(torch.from_numpy(s))
        # one eager call first (sets up the kernels' attributes outside capture); it appends
        # at pos0 exactly what the first replay appends again
        tqk.attention_layer(args, ws, stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            tqk.attention_layer(args, ws, stream)
    stream.synchronize()
    # capture does not run the kernels: replay once per token
    for i in range(steps):
        pos = pos0 + i
        c, s = port.rope_table(hd, pos, theta)
        with torch.cuda.stream(stream):
            lay.cos.copy_(torch.from_numpy(c))
            lay.sin.copy_(torch.from_numpy(s))
            lay.xn.copy_(torch.from_numpy(xs[i]))
            len_dev.fill_(pos + 1)
            graph.replay()
        stream.synchronize()
        want = port.attention_layer(lay.host["w"], fmt, lay.host["qn"], lay.host["kn"], nq, nkv, hd, hidden, theta,
                                    eps, kp_ref, vp_ref, mt, pos, xs[i])
        kp = lay.kp.cpu().numpy()
        assert np.array_equal(kp[:, pos], kp_ref[:, pos]), i
        assert np.array_equal(lay.vp.cpu().numpy()[:, pos], vp_ref[:, pos]), i
        assert _out_ok(lay.out.cpu().numpy(), want), i
    del graph


def test_layer_argument_errors(tqk, cuda):
    a = tqk.AttnLayerArgs()
    assert tqk.tqk_attention_layer(None, None, 0, None) == tqk.EINVAL
    a.n_q_heads, a.n_kv_heads, a.head_dim, a.hidden_size, a.max_tokens, a.pos = 8, 2, 64, 256, 16, 16
    assert tqk.tqk_attention_layer(a, None, 0, None) == tqk.EPOS
    a.pos = 3
    assert tqk.tqk_attention_layer(a, None, 0, None) == tqk.EINVAL  # NULL pointers
