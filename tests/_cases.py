"""Seeded synthetic inputs for the parity tests and the golden fixtures.

The reference publishes no dataset for this path; its configs
define shapes and distributions: q, K, V ~ N(0,1) fp32, K/V quantised to Q8 by
the reference quantiser, config 2's q rotated by RoPE (theta 500000) at its
position, config 3's K/V with 1% of entries scaled x8.  numpy's PCG64 stream
stands in for the reference benches' xorshift64 Box-Muller stream; every
fixture stores a SHA-256 of its generated inputs so a changed stream is caught.
"""
from __future__ import annotations

import hashlib

import numpy as np

QK = 32
BLOCK_BYTES = 36


def normal(rng: np.random.Generator, shape, outlier_frac: float = 0.0) -> np.ndarray:
    x = rng.standard_normal(shape, dtype=np.float32)
    if outlier_frac > 0:
        mask = rng.random(shape, dtype=np.float32) < outlier_frac
        x[mask] *= 8.0
    return x


def rope(x: np.ndarray, head_dim: int, pos: int, theta: float) -> np.ndarray:
    """Half-split rotation of model/rope.c:4-22 applied to every head of x [..., heads*hd]."""
    i = np.arange(head_dim // 2, dtype=np.float64)
    freq = np.power(theta, -2.0 * i / head_dim)
    a = pos * freq
    c, s = np.cos(a), np.sin(a)
    h = x.reshape(-1, head_dim).astype(np.float64)
    x0, x1 = h[:, : head_dim // 2].copy(), h[:, head_dim // 2:].copy()
    h[:, : head_dim // 2] = x0 * c - x1 * s
    h[:, head_dim // 2:] = x0 * s + x1 * c
    return h.astype(np.float32).reshape(x.shape)


def digest(*arrays: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def quant_edge_rows(rng: np.random.Generator, n: int = 128) -> np.ndarray:
    """Rows exercising the quantiser's corners (kernel/quant_x.c:5-34)."""
    rows = []
    rows.append(rng.standard_normal(n, dtype=np.float32))
    rows.append(np.zeros(n, np.float32))                                  # zero scale
    rows.append(np.full(n, 3.25, np.float32))                             # constant
    r = rng.standard_normal(n, dtype=np.float32); r[::17] *= 8; rows.append(r)  # outliers
    # exact ties after scaling: max 127 -> inv 1, values k + 0.5 round half to even
    r = np.concatenate([np.array([127.0], np.float32), (np.arange(n - 1) % 9 - 4 + 0.5).astype(np.float32)])
    rows.append(r)
    r = rng.standard_normal(n, dtype=np.float32) * 1e-39; rows.append(r.astype(np.float32))  # denormals
    r = np.clip(rng.standard_normal(n), -1, 1).astype(np.float32) * np.float32(3e38); rows.append(r)  # near overflow
    r = rng.standard_normal(n, dtype=np.float32); r[5] = np.inf; rows.append(r)
    r = rng.standard_normal(n, dtype=np.float32); r[40] = -np.inf; r[41] = np.nan; rows.append(r)
    r = rng.standard_normal(n, dtype=np.float32); r[70] = np.nan; rows.append(r)
    rows.append(np.full(n, np.nan, np.float32))
    r = np.zeros(n, np.float32); r[3] = 1e-45; rows.append(r)             # smallest denormal
    r = rng.standard_normal(n, dtype=np.float32)                           # NaN payloads: quiet and signalling
    r[[2, 33, 70, 101]] = np.array([0x7FC000AB, 0xFFC00012, 0x7F8000CD, 0xFF800001], np.uint32).view(np.float32)
    rows.append(r)
    r = rng.standard_normal(n, dtype=np.float32); r[:32] = -0.0; rows.append(r)
    for k in range(8):
        rows.append((rng.standard_normal(n, dtype=np.float32) * (10.0 ** rng.uniform(-6, 6))).astype(np.float32))
    return np.stack(rows).astype(np.float32)


def decode_case(seed: int, n_q: int, n_kv: int, hd: int, max_tokens: int, n: int, *, outlier_frac: float = 0.0,
                rope_pos: int | None = None, rope_theta: float = 500000.0, q_scale: float = 1.0):
    """fp32 K/V [n_kv, max_tokens, hd] (rows >= n left zero), q [n_q*hd]."""
    rng = np.random.default_rng(seed)
    kf = np.zeros((n_kv, max_tokens, hd), np.float32)
    vf = np.zeros((n_kv, max_tokens, hd), np.float32)
    kf[:, :n] = normal(rng, (n_kv, n, hd), outlier_frac)
    vf[:, :n] = normal(rng, (n_kv, n, hd), outlier_frac)
    q = normal(rng, (n_q * hd,)) * np.float32(q_scale)
    if rope_pos is not None:
        q = rope(q, hd, rope_pos, rope_theta)
    return kf, vf, q.astype(np.float32)


def tolerance_ok(got: np.ndarray, ref: np.ndarray, atol: float = 1e-3, rtol: float = 1e-3):
    """The attention tolerance of the north star: max abs error <= 1e-3 and
    relative error (max |diff| / max |ref|) <= 1e-3, in FP32."""
    diff = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    max_abs = float(diff.max()) if diff.size else 0.0
    scale = float(np.abs(ref).max()) if ref.size else 0.0
    rel = max_abs / scale if scale > 0 else max_abs
    return (max_abs <= atol and rel <= rtol and bool(np.isfinite(got).all())), max_abs, rel


def sweep_inputs(g: int, n: int, hd: int):
    """Inputs of one per-op sweep case (the shape grid of tools/test_model.c:1677-1697)."""
    rng = np.random.default_rng(900 + g * 100 + n * 10 + hd)
    qf = rng.standard_normal((g, hd), dtype=np.float32)
    kf = rng.standard_normal((n, hd), dtype=np.float32)
    vf = rng.standard_normal((n, hd), dtype=np.float32)
    w = rng.standard_normal((g, n + 4), dtype=np.float32)
    return qf, kf, vf, w


def head_inputs(hd: int, n: int, seed: int):
    """Inputs of one attention_head_q8 case (tools/test_model.c:584-728 style; seed 90 = x30 scores)."""
    rng = np.random.default_rng(seed)
    s = np.float32(30.0 if seed == 90 else 1.0)
    q = rng.standard_normal(hd, dtype=np.float32) * s
    kf = rng.standard_normal((n, hd), dtype=np.float32) * s
    vf = rng.standard_normal((n, hd), dtype=np.float32)
    return q, kf, vf


def prefill_inputs(seed: int, n_q: int, n_kv: int, hd: int, max_tokens: int, pos0: int, n: int,
                   qk_scale: float = 1.0, outlier_frac: float = 0.0):
    """One attention_layer_batch chunk (model/attention_layer.c:221-236): cache rows [0, pos0) and n
    new tokens' q, k, v.  qk_scale multiplies q and every K row (the reference's large-score case,
    tools/test_model.c:725-728, uses 30); outlier_frac of the K and V entries are x8 (config 3's
    outlier blocks)."""
    rng = np.random.default_rng(seed)
    kf = rng.standard_normal((n_kv, max_tokens, hd), dtype=np.float32)
    vf = rng.standard_normal((n_kv, max_tokens, hd), dtype=np.float32)
    kf[:, pos0:] = 0
    vf[:, pos0:] = 0
    qn = rng.standard_normal((n, n_q * hd), dtype=np.float32)
    kn = rng.standard_normal((n, n_kv * hd), dtype=np.float32)
    vn = rng.standard_normal((n, n_kv * hd), dtype=np.float32)
    if qk_scale != 1.0:
        s = np.float32(qk_scale)
        kf, qn, kn = kf * s, qn * s, kn * s
    if outlier_frac > 0.0:
        for a in (kf, vf, kn, vn):
            a *= np.where(rng.random(a.shape) < outlier_frac, np.float32(8.0), np.float32(1.0))
    return kf, vf, qn, kn, vn


def norm_rope_inputs(seed: int, n_items: int, n_q: int, n_kv: int, hd: int, per_item_weights: bool):
    """q [items, n_q*hd], k [items, n_kv*hd] and the q/k norm weights (per item when asked) of one
    attention_layer.c:183-189 prologue case; q is scaled x4 so the norm does real work."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((n_items, n_q * hd), dtype=np.float32) * np.float32(4.0)
    k = rng.standard_normal((n_items, n_kv * hd), dtype=np.float32)
    nw = n_items if per_item_weights else 1
    qw = (np.float32(1.0) + np.float32(0.1) * rng.standard_normal((nw, hd), dtype=np.float32))
    kw = (np.float32(1.0) + np.float32(0.1) * rng.standard_normal((nw, hd), dtype=np.float32))
    return q, k, qw, kw


def matmul_inputs(seed: int, rows: int, cols: int, x_kind: str = "random"):
    """W [rows, cols] and x [cols] of one matmul case (tools/test_kernel.c:52-75 style: uniform in
    [-1, 1); x constant 1 or all zero for the edge cases)."""
    rng = np.random.default_rng(seed)
    w = rng.uniform(-1.0, 1.0, (rows, cols)).astype(np.float32)
    if x_kind == "random":
        x = rng.uniform(-1.0, 1.0, cols).astype(np.float32)
    elif x_kind == "constant":
        x = np.ones(cols, np.float32)
    else:
        x = np.zeros(cols, np.float32)
    return w, x


def layer_inputs(seed: int, n_q: int, n_kv: int, hd: int, hidden: int, max_tokens: int, pos: int, fmt: str, port):
    """One attention_layer case (model/attention_layer.c:169-194): packed wq/wk/wv/wo (uniform in
    [-1, 1), packed by the pinned oracle packer), q/k norm weights, Q8 cache planes holding
    positions [0, pos) and the input xn."""
    rng = np.random.default_rng(seed)
    shapes = {"wq": (n_q * hd, hidden), "wk": (n_kv * hd, hidden), "wv": (n_kv * hd, hidden),
              "wo": (hidden, n_q * hd)}
    w = {n: port.pack_matrix(rng.uniform(-1.0, 1.0, sh).astype(np.float32), fmt) for n, sh in shapes.items()}
    qn = (1.0 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kn = (1.0 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kf = rng.standard_normal((n_kv, max_tokens, hd), dtype=np.float32)
    vf = rng.standard_normal((n_kv, max_tokens, hd), dtype=np.float32)
    kf[:, pos:] = 0.0
    vf[:, pos:] = 0.0
    xn = rng.standard_normal(hidden, dtype=np.float32)
    return w, qn, kn, port.quantize_rows(kf), port.quantize_rows(vf), xn


def forward_model(seed: int, fmt: str, port, n_layers: int = 2, n_q: int = 8, n_kv: int = 2, hd: int = 128,
                  hidden: int = 256, inter: int = 512, vocab: int = 96, theta: float = 500000.0,
                  eps: float = 1e-5) -> dict:
    """A small decoder stack for tq_forward_token (model/context.c:104-122): packed weights
    (uniform in [-1, 1), packed by the pinned oracle packer; the embedding x0.5), norm weights
    1 + 0.1 N(0,1), in the layout of Oracle.forward_tokens."""
    rng = np.random.default_rng(seed)
    q_dim, kv_dim = n_q * hd, n_kv * hd

    def packed(rows, cols, scale=1.0):
        return port.pack_matrix((rng.uniform(-1.0, 1.0, (rows, cols)) * scale).astype(np.float32), fmt)

    def norm(n):
        return (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)

    layers = []
    for _ in range(n_layers):
        layers.append({"input_norm": norm(hidden), "post_norm": norm(hidden), "q_norm": norm(hd), "k_norm": norm(hd),
                       "wq": packed(q_dim, hidden), "wk": packed(kv_dim, hidden), "wv": packed(kv_dim, hidden),
                       "wo": packed(hidden, q_dim), "wgate": packed(inter, hidden), "wup": packed(inter, hidden),
                       "wdown": packed(hidden, inter)})
    cfg = {"n_q_heads": n_q, "n_kv_heads": n_kv, "head_dim": hd, "hidden_size": hidden, "rope_theta": theta,
           "rms_eps": eps, "n_layers": n_layers, "intermediate_size": inter, "vocab_size": vocab}
    return {"cfg": cfg, "fmt": fmt, "embed": packed(vocab, hidden, 0.5), "final_norm": norm(hidden), "layers": layers}
