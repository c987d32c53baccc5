"""CPU checkers for the Q8 attention path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference leg
may import this package.  It binds, with ctypes and numpy:

* ``port``       -- oracle/libtq_oracle.so, the scalar restatement (tq_oracle.c);
* ``ref_scalar`` -- oracle/_ref/libtqref_scalar.so, the reference's own sources
                    compiled without TQ_HAVE_AVX2 (its scalar path), plus
                    ref_attend.c composing attend_q8 from its exported functions;
* ``ref_avx2``   -- oracle/_ref/libtqref_avx2.so, the reference's AVX2/FMA build.

All three expose the same methods.  Planes are numpy uint8 arrays of shape
[n_kv, max_tokens, nb*36] (the reference layout, model/kv_cache.c:33-39).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
QK = 32
BLOCK_BYTES = 36

_LIBS = {
    "port": os.path.join(HERE, "libtq_oracle.so"),
    "ref_scalar": os.path.join(HERE, "_ref", "libtqref_scalar.so"),
    "ref_avx2": os.path.join(HERE, "_ref", "libtqref_avx2.so"),
}

# symbol names per build: (port name, reference name)
_NAMES = {
    "quantize_row": ("tqo_quantize_row_q8", "quantize_row_q8"),
    "softmax": ("tqo_softmax", "softmax"),
    "scores": ("tqo_attn_scores_q8", "attn_scores_q8_scalar"),
    "accum": ("tqo_attn_accum_q8", "attn_accum_q8_scalar"),
    "scores_dispatch": ("tqo_attn_scores_q8", "attn_scores_q8"),
    "accum_dispatch": ("tqo_attn_accum_q8", "attn_accum_q8"),
    "head": ("tqo_attention_head_q8", "attention_head_q8"),
    "store_kv": ("tqo_store_kv_q8", "refdrv_store_kv_q8"),
    "attend": ("tqo_attend_q8", "refdrv_attend_q8"),
    "prefill": ("tqo_prefill_q8", "refdrv_prefill_q8"),
    "rmsnorm": ("tqo_rmsnorm", "rmsnorm"),
    "rope_table": ("tqo_rope_table", "rope_table"),
    "rope_apply": ("tqo_rope_apply", "rope_apply"),
    "pack": ("tqo_pack_matrix", "pack_matrix"),
    "matmul_q8": ("tqo_matmul_q8", "matmul_q8_scalar"),
    "matmul_q4": ("tqo_matmul_q4", "matmul_q4_scalar"),
}


def available(kind: str) -> bool:
    return os.path.exists(_LIBS[kind])


def build(reference: str | None = None) -> None:
    """make -C oracle [ref]: the restatement always, the reference builds when its tree exists."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)
    ref = reference or os.environ.get("TQK_REFERENCE") or os.path.join(os.path.dirname(os.path.dirname(HERE)),
                                                                        "reference")
    if os.path.isdir(ref):
        subprocess.run(["make", "-s", "-C", HERE, f"REF={ref}", "ref"], check=True)


def _f32p(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _vp(a):
    return ctypes.c_void_p(a.ctypes.data)

class _TqMatrix(ctypes.Structure):
    """tq_matrix (model/model_ops.h): packed rows, tq_format (0 = Q8, 1 = Q4), rows, cols."""
    _fields_ = [("data", ctypes.c_void_p), ("format", ctypes.c_int), ("rows", ctypes.c_int), ("cols", ctypes.c_int)]


class _TqAttnWeights(ctypes.Structure):
    """tq_attn_weights (model/model_ops.h)."""
    _fields_ = [("wq", _TqMatrix), ("wk", _TqMatrix), ("wv", _TqMatrix), ("wo", _TqMatrix),
                ("q_norm", ctypes.c_void_p), ("k_norm", ctypes.c_void_p)]


class _TqAttnConfig(ctypes.Structure):
    """tq_attn_config (model/model_ops.h)."""
    _fields_ = [("n_q_heads", ctypes.c_int), ("n_kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int),
                ("hidden_size", ctypes.c_int), ("rope_theta", ctypes.c_float), ("rms_eps", ctypes.c_float)]


class _TqKvCache(ctypes.Structure):
    """tq_kv_cache (model/model_ops.h): type (0 = F32, 1 = Q8), four plane pointers, max_tokens."""
    _fields_ = [("type", ctypes.c_int), ("k_f32", ctypes.c_void_p), ("v_f32", ctypes.c_void_p),
                ("k_q8", ctypes.c_void_p), ("v_q8", ctypes.c_void_p), ("max_tokens", ctypes.c_int)]



class _TqMlpWeights(ctypes.Structure):
    """tq_mlp_weights (model/model_ops.h)."""
    _fields_ = [("wgate", _TqMatrix), ("wup", _TqMatrix), ("wdown", _TqMatrix)]


class _TqLayerWeights(ctypes.Structure):
    """tq_layer_weights (model/model_ops.h)."""
    _fields_ = [("input_norm", ctypes.c_void_p), ("attn", _TqAttnWeights), ("post_norm", ctypes.c_void_p),
                ("mlp", _TqMlpWeights)]


class _TqModelConfig(ctypes.Structure):
    """tq_model_config (model/model_ops.h)."""
    _fields_ = [("attn", _TqAttnConfig), ("n_layers", ctypes.c_int), ("intermediate_size", ctypes.c_int),
                ("vocab_size", ctypes.c_int)]


class _TqModel(ctypes.Structure):
    """tq_model = {tq_model_config cfg; tq_model_weights w = {embed, final_norm, layers}} (model/model_ops.h)."""
    _fields_ = [("cfg", _TqModelConfig), ("embed", _TqMatrix), ("final_norm", ctypes.c_void_p),
                ("layers", ctypes.POINTER(_TqLayerWeights))]


class _TqCtx(ctypes.Structure):
    """tq_ctx (model/model_ops.h)."""
    _fields_ = [("model", ctypes.c_void_p), ("caches", ctypes.POINTER(_TqKvCache)), ("pos", ctypes.c_int),
                ("max_tokens", ctypes.c_int)] + \
               [(n, ctypes.c_void_p) for n in ("x", "xn", "attn_out", "mlp_out", "gate", "up", "xq", "hq", "scores",
                                               "logits")]


class Oracle:
    def __init__(self, kind: str = "port"):
        path = _LIBS[kind]
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} not built (run `make -C oracle` / `make -C oracle ref`)")
        self.kind = kind
        self.lib = ctypes.CDLL(path)
        idx = 0 if kind == "port" else 1
        self._fn = {k: getattr(self.lib, v[idx]) for k, v in _NAMES.items()}
        for f in self._fn.values():
            f.restype = None
        for k in ("store_kv", "prefill"):
            self._fn[k].restype = ctypes.c_int
        vp, i, f, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
        self._fn["quantize_row"].argtypes = [vp, vp, i]
        self._fn["softmax"].argtypes = [vp, i]
        for k in ("scores", "scores_dispatch"):
            self._fn[k].argtypes = [vp, i, vp, i, i, f, vp, sz]
        for k in ("accum", "accum_dispatch"):
            self._fn[k].argtypes = [vp, sz, i, vp, i, i, vp, sz]
        self._fn["head"].argtypes = [vp, vp, vp, vp, i, i, vp, vp]
        self._fn["store_kv"].argtypes = [vp, vp, i, i, i, i, vp, vp]
        self._fn["attend"].argtypes = [vp, vp, i, i, i, i, i, vp, vp, vp, i]
        self._fn["prefill"].argtypes = [vp, vp, i, i, i, i, i, i, vp, vp, vp, vp, vp, i]
        self._fn["rmsnorm"].argtypes = [vp, vp, vp, i, f]
        self._fn["rope_table"].argtypes = [vp, vp, i, i, f]
        self._fn["rope_apply"].argtypes = [vp, i, vp, vp]
        for k in ("rmsnorm", "rope_table", "rope_apply"):
            self._fn[k].restype = None
        self._fn["pack"].argtypes = [vp, i, i, vp, ctypes.c_char]
        self._fn["pack"].restype = i
        for k in ("matmul_q8", "matmul_q4"):
            self._fn[k].argtypes = [vp, vp, vp, i, i]
            self._fn[k].restype = None
        if kind != "port":
            self.lib.refdrv_max_threads.restype = i
            self.lib.refdrv_quantize_rows.argtypes = [vp, vp, i, i]
            self.lib.refdrv_quantize_rows.restype = None
        else:
            self.lib.tqo_quantize_rows_q8.argtypes = [vp, vp, i, i]
            self.lib.tqo_quantize_rows_q8.restype = None

    # --- quantiser -------------------------------------------------------
    def quantize_rows(self, x: np.ndarray) -> np.ndarray:
        """quantize_row_q8 per row of x [..., n] -> uint8 [..., n/32*36]."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        n = x.shape[-1]
        rows = x.reshape(-1, n)
        out = np.zeros((rows.shape[0], n // QK * BLOCK_BYTES), dtype=np.uint8)
        if self.kind == "port":  # one C call for all rows
            self.lib.tqo_quantize_rows_q8(_vp(rows), _vp(out), ctypes.c_int(rows.shape[0]), ctypes.c_int(n))
            return out.reshape(*x.shape[:-1], n // QK * BLOCK_BYTES)
        for r in range(rows.shape[0]):
            self._fn["quantize_row"](ctypes.c_void_p(rows[r:].ctypes.data), ctypes.c_void_p(out[r:].ctypes.data), n)
        return out.reshape(*x.shape[:-1], n // QK * BLOCK_BYTES)

    def quantize_rows_bulk(self, x: np.ndarray) -> np.ndarray:
        """Same as quantize_rows, with the row loop in C for both builds."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        n = x.shape[-1]
        rows = x.reshape(-1, n)
        out = np.empty((rows.shape[0], n // QK * BLOCK_BYTES), dtype=np.uint8)
        fn = self.lib.tqo_quantize_rows_q8 if self.kind == "port" else self.lib.refdrv_quantize_rows
        fn(_vp(rows), _vp(out), ctypes.c_int(rows.shape[0]), ctypes.c_int(n))
        return out.reshape(*x.shape[:-1], n // QK * BLOCK_BYTES)

    def softmax(self, x: np.ndarray) -> np.ndarray:
        y = np.ascontiguousarray(x, dtype=np.float32).copy()
        self._fn["softmax"](_vp(y), y.shape[-1])
        return y

    # --- per-op kernels ----------------------------------------------------
    def attn_scores(self, qb, g, kb, n, nb, scale, stride, dispatched=False, fill=np.nan):
        sc = np.full(g * stride, fill, dtype=np.float32)
        self._fn["scores_dispatch" if dispatched else "scores"](_vp(np.ascontiguousarray(qb)), g,
                                                               _vp(np.ascontiguousarray(kb)), n, nb,
                                                               ctypes.c_float(scale), _vp(sc), stride)
        return sc

    def attn_accum(self, w, w_stride, g, vb, n, nb, out_stride, dispatched=False, fill=np.nan):
        out = np.full(g * out_stride, fill, dtype=np.float32)
        w = np.ascontiguousarray(w, dtype=np.float32)
        self._fn["accum_dispatch" if dispatched else "accum"](_vp(w), w_stride, g, _vp(np.ascontiguousarray(vb)), n,
                                                             nb, _vp(out), out_stride)
        return out

    def attention_head(self, q, kb, vb, n, head_dim):
        q = np.ascontiguousarray(q, dtype=np.float32)
        qq = np.zeros(head_dim // QK * BLOCK_BYTES, dtype=np.uint8)
        sc = np.zeros(max(n, 1), dtype=np.float32)
        out = np.zeros(head_dim, dtype=np.float32)
        self._fn["head"](_vp(q), _vp(qq), _vp(np.ascontiguousarray(kb)), _vp(np.ascontiguousarray(vb)), n, head_dim,
                         _vp(sc), _vp(out))
        return out, qq, sc[:n]

    # --- cache + attention ---------------------------------------------------
    def store_kv(self, kp, vp, n_kv, head_dim, max_tokens, pos, k, v) -> int:
        return self._fn["store_kv"](_vp(kp), _vp(vp), n_kv, head_dim, max_tokens, pos,
                                    _vp(np.ascontiguousarray(k, dtype=np.float32)),
                                    _vp(np.ascontiguousarray(v, dtype=np.float32)))

    def attend(self, kp, vp, n_q, n_kv, head_dim, max_tokens, pos, q, threads=1) -> np.ndarray:
        q = np.ascontiguousarray(q, dtype=np.float32)
        scores = np.zeros(n_q * max_tokens, dtype=np.float32)
        out = np.zeros(n_q * head_dim, dtype=np.float32)
        self._fn["attend"](_vp(kp), _vp(vp), n_q, n_kv, head_dim, max_tokens, pos, _vp(q), _vp(scores), _vp(out),
                           threads)
        return out

    def prefill(self, kp, vp, n_q, n_kv, head_dim, max_tokens, pos0, n, q, k, v, threads=1) -> np.ndarray:
        q = np.ascontiguousarray(q, dtype=np.float32)
        scores = np.zeros(n_q * max_tokens, dtype=np.float32)
        out = np.zeros(n * n_q * head_dim, dtype=np.float32)
        rc = self._fn["prefill"](_vp(kp), _vp(vp), n_q, n_kv, head_dim, max_tokens, pos0, n, _vp(q),
                                 _vp(np.ascontiguousarray(k, dtype=np.float32)),
                                 _vp(np.ascontiguousarray(v, dtype=np.float32)), _vp(scores), _vp(out), threads)
        if rc != 0:
            raise ValueError(f"prefill returned {rc}")
        return out

    def rope_table(self, head_dim: int, pos: int, theta: float):
        """(cos, sin) tables of rope_table (model/rope.c:4-12)."""
        c = np.zeros(head_dim // 2, np.float32)
        s = np.zeros(head_dim // 2, np.float32)
        self._fn["rope_table"](_vp(c), _vp(s), head_dim, pos, theta)
        return c, s

    def qk_norm_rope(self, x, n_heads, head_dim, weight, eps, cos_t, sin_t):
        """norm_heads + rope_heads as attention_layer applies them (attention_layer.c:183-189):
        rmsnorm in place per head row, then rope_apply with the table.  weight / cos_t may
        be None to skip that part.  Returns a new array."""
        y = np.ascontiguousarray(x, dtype=np.float32).copy()
        rows = y.reshape(-1, head_dim)
        for r in range(rows.shape[0]):
            row = rows[r]
            if weight is not None:
                w = np.ascontiguousarray(weight, dtype=np.float32)
                self._fn["rmsnorm"](_vp(row), _vp(w), _vp(row), head_dim, eps)
            if cos_t is not None:
                self._fn["rope_apply"](_vp(row), head_dim, _vp(np.ascontiguousarray(cos_t, dtype=np.float32)),
                                       _vp(np.ascontiguousarray(sin_t, dtype=np.float32)))
        return y

    def pack_matrix(self, w: np.ndarray, fmt: str) -> np.ndarray:
        """pack_matrix (packer/packer.c:77-88) of fp32 W [rows, cols]: '8' -> Q8, '4' -> Q4 rows (uint8)."""
        w = np.ascontiguousarray(w, dtype=np.float32)
        rows, cols = w.shape
        nb = cols // QK
        out = np.zeros((rows, nb * (BLOCK_BYTES if fmt == "8" else 20)), dtype=np.uint8)
        rc = self._fn["pack"](_vp(w), rows, cols, _vp(out), fmt.encode())
        if rc != 0:
            raise ValueError(f"pack_matrix returned {rc}")
        return out

    def matmul(self, w_packed: np.ndarray, fmt: str, xq: np.ndarray, rows: int, cols: int) -> np.ndarray:
        """matmul_q8_scalar / matmul_q4_scalar (kernel/q8_scalar.c:15-22, q4_scalar.c:17-24) of one Q8
        activation row xq (uint8 [cols/32*36]); matmul_*_scalar_batch is this per token."""
        y = np.zeros(rows, dtype=np.float32)
        self._fn["matmul_q8" if fmt == "8" else "matmul_q4"](_vp(np.ascontiguousarray(w_packed)),
                                                             _vp(np.ascontiguousarray(xq)), _vp(y), rows, cols)
        return y

    def attention_layer(self, w: dict, fmt: str, q_norm, k_norm, n_q: int, n_kv: int, head_dim: int,
                        hidden: int, theta: float, eps: float, kp, vp, max_tokens: int, pos: int, xn):
        """One attention_layer step (model/attention_layer.c:169-194) for one token at pos: w holds the
        packed 'wq', 'wk', 'wv', 'wo' rows; kp/vp (the layer's Q8 cache planes) get the appended rows
        in place.  The reference kinds call the reference's own attention_layer; the port composes the
        restated steps (quantize_row_q8, matmul, norm_heads + rope_heads, store_kv, attend_q8,
        quantize_row_q8, matmul).  Returns the output [hidden]."""
        q_dim, kv_dim = n_q * head_dim, n_kv * head_dim
        xn = np.ascontiguousarray(xn, dtype=np.float32)
        if self.kind == "port":
            xq = self.quantize_rows(xn[None])[0]
            q = self.matmul(w["wq"], fmt, xq, q_dim, hidden)
            k = self.matmul(w["wk"], fmt, xq, kv_dim, hidden)
            v = self.matmul(w["wv"], fmt, xq, kv_dim, hidden)
            c, s = self.rope_table(head_dim, pos, theta)
            q = self.qk_norm_rope(q, n_q, head_dim, q_norm, eps, c, s)
            k = self.qk_norm_rope(k, n_kv, head_dim, k_norm, eps, c, s)
            if self.store_kv(kp, vp, n_kv, head_dim, max_tokens, pos, k, v) != 0:
                raise ValueError("store_kv refused the position")
            attn = self.attend(kp, vp, n_q, n_kv, head_dim, max_tokens, pos, q)
            aq = self.quantize_rows(attn[None])[0]
            return self.matmul(w["wo"], fmt, aq, hidden, q_dim)
        f = 0 if fmt == "8" else 1
        keep = [np.ascontiguousarray(w[n]) for n in ("wq", "wk", "wv", "wo")]
        qn = np.ascontiguousarray(q_norm, dtype=np.float32)
        kn = np.ascontiguousarray(k_norm, dtype=np.float32)
        mats = [_TqMatrix(_vp(keep[0]), f, q_dim, hidden), _TqMatrix(_vp(keep[1]), f, kv_dim, hidden),
                _TqMatrix(_vp(keep[2]), f, kv_dim, hidden), _TqMatrix(_vp(keep[3]), f, hidden, q_dim)]
        aw = _TqAttnWeights(*mats, _vp(qn), _vp(kn))
        cfg = _TqAttnConfig(n_q, n_kv, head_dim, hidden, theta, eps)
        cache = _TqKvCache(1, None, None, _vp(kp), _vp(vp), max_tokens)
        scores = np.zeros(n_q * max_tokens, dtype=np.float32)  # one slice per q head (model/context.c:34)
        out = np.zeros(hidden, dtype=np.float32)
        fn = self.lib.attention_layer
        fn.argtypes = [ctypes.POINTER(_TqAttnWeights), ctypes.POINTER(_TqAttnConfig), ctypes.POINTER(_TqKvCache),
                       ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        fn.restype = ctypes.c_int
        rc = fn(ctypes.byref(aw), ctypes.byref(cfg), ctypes.byref(cache), pos, _vp(xn), _vp(scores), _vp(out))
        if rc != 0:
            raise ValueError(f"attention_layer returned {rc}")
        return out

    def forward_tokens(self, model: dict, tokens, max_tokens: int, start_planes=None):
        """The reference's own tq_ctx_init + tq_forward_token (model/context.c:6-122) over `tokens`
        with a Q8 KV cache (reference builds only).  model: cfg (n_q_heads, n_kv_heads, head_dim,
        hidden_size, rope_theta, rms_eps, n_layers, intermediate_size, vocab_size), fmt ("8" / "4"),
        embed (packed rows), final_norm, and layers: dicts with input_norm, post_norm, q_norm, k_norm
        and the packed wq, wk, wv, wo, wgate, wup, wdown.  Returns (logits per token [n][vocab],
        return codes, the K and V planes of every layer after the last token).  start_planes: (pos,
        [(k, v) per layer]) to start from a cache that already holds positions [0, pos) (copied into
        the context's planes) instead of an empty one."""
        if self.kind == "port":
            raise ValueError("forward_tokens runs the reference's own runtime: a reference build is needed")
        c = model["cfg"]
        f = 0 if model["fmt"] == "8" else 1
        hidden, inter, vocab, hd = c["hidden_size"], c["intermediate_size"], c["vocab_size"], c["head_dim"]
        q_dim, kv_dim = c["n_q_heads"] * hd, c["n_kv_heads"] * hd
        keep = []

        def mat(a, rows, cols):
            a = np.ascontiguousarray(a)
            keep.append(a)
            return _TqMatrix(_vp(a), f, rows, cols)

        def vec(a):
            a = np.ascontiguousarray(a, dtype=np.float32)
            keep.append(a)
            return _vp(a)

        layers = (_TqLayerWeights * c["n_layers"])()
        for i, lw in enumerate(model["layers"]):
            attn = _TqAttnWeights(mat(lw["wq"], q_dim, hidden), mat(lw["wk"], kv_dim, hidden),
                                  mat(lw["wv"], kv_dim, hidden), mat(lw["wo"], hidden, q_dim), vec(lw["q_norm"]),
                                  vec(lw["k_norm"]))
            mlp = _TqMlpWeights(mat(lw["wgate"], inter, hidden), mat(lw["wup"], inter, hidden),
                                mat(lw["wdown"], hidden, inter))
            layers[i] = _TqLayerWeights(vec(lw["input_norm"]), attn, vec(lw["post_norm"]), mlp)
        cfg = _TqModelConfig(_TqAttnConfig(c["n_q_heads"], c["n_kv_heads"], hd, hidden, c["rope_theta"],
                                           c["rms_eps"]), c["n_layers"], inter, vocab)
        m = _TqModel(cfg, mat(model["embed"], vocab, hidden), vec(model["final_norm"]),
                     ctypes.cast(layers, ctypes.POINTER(_TqLayerWeights)))
        ctx = _TqCtx()
        self.lib.tq_ctx_init.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
        self.lib.tq_ctx_init.restype = ctypes.c_int
        self.lib.tq_forward_token.argtypes = [ctypes.c_void_p, ctypes.c_int]
        self.lib.tq_forward_token.restype = ctypes.c_int
        self.lib.tq_ctx_free.argtypes = [ctypes.c_void_p]
        if self.lib.tq_ctx_init(ctypes.byref(ctx), ctypes.byref(m), 1, max_tokens) != 0:
            raise ValueError("tq_ctx_init refused the model")
        try:
            if start_planes is not None:
                pos0, planes0 = start_planes
                for i, (kp, vp) in enumerate(planes0):
                    cache = ctx.caches[i]
                    ctypes.memmove(cache.k_q8, np.ascontiguousarray(kp).ctypes.data, kp.nbytes)
                    ctypes.memmove(cache.v_q8, np.ascontiguousarray(vp).ctypes.data, vp.nbytes)
                ctx.pos = pos0
            logits, rcs = [], []
            for t in tokens:
                rcs.append(self.lib.tq_forward_token(ctypes.byref(ctx), int(t)))
                logits.append(np.ctypeslib.as_array(ctypes.cast(ctx.logits, ctypes.POINTER(ctypes.c_float)),
                                                    shape=(vocab,)).copy())
            row = hd // QK * BLOCK_BYTES
            planes = []
            for i in range(c["n_layers"]):
                cache = ctx.caches[i]
                shape = (c["n_kv_heads"], max_tokens, row)
                planes.append((np.ctypeslib.as_array(ctypes.cast(cache.k_q8, ctypes.POINTER(ctypes.c_uint8)),
                                                     shape=shape).copy(),
                               np.ctypeslib.as_array(ctypes.cast(cache.v_q8, ctypes.POINTER(ctypes.c_uint8)),
                                                     shape=shape).copy()))
            return np.stack(logits), rcs, planes
        finally:
            self.lib.tq_ctx_free(ctypes.byref(ctx))

    def max_threads(self) -> int:
        return self.lib.refdrv_max_threads() if self.kind != "port" else os.cpu_count() or 1


def dequantize(blocks: np.ndarray) -> np.ndarray:
    """uint8 [..., nb*36] -> float32 [..., nb*32]: d * q per block."""
    b = np.ascontiguousarray(blocks).reshape(*blocks.shape[:-1], -1, BLOCK_BYTES)
    d = b[..., :4].copy().view(np.float32)
    q = b[..., 4:].view(np.int8).astype(np.float32)
    return (d * q).reshape(*blocks.shape[:-1], -1)


def attention_f64(q: np.ndarray, k: np.ndarray, v: np.ndarray) -> np.ndarray:
    """float64 softmax attention of one head (tools/test_model.c:424-454 semantics)."""
    q = q.astype(np.float64)
    s = (k.astype(np.float64) @ q) / np.sqrt(q.shape[-1])
    p = np.exp(s - s.max())
    return (p[:, None] * v.astype(np.float64)).sum(0) / p.sum()
