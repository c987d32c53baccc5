"""ctypes binding of libtqk.so (the C ABI in include/tqk.h).

All functions take torch CUDA tensors (or raw device addresses) and launch on the
current torch stream unless a stream is given.  Nothing here computes on the
CPU: a missing libtqk.so raises at import time and a failing call raises
:class:`TQKError` carrying the library's status code and message.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libtqk.so")

if not os.path.exists(LIB_PATH):
    raise ImportError(
        f"{LIB_PATH} is missing: build it with `python -m tailorquantkernel_b200.build` "
        "(there is no CPU fallback)")

_lib = ctypes.CDLL(LIB_PATH)

QK = 32
BLOCK_BYTES = 36

OK = 0
EPOS = -1
EINVAL = -20
EALIGN = -21
EWORKSPACE = -22
ECUDA = -23
ENODEV = -24
ETIMEOUT = -25
EUNSUPPORTED = -26
EDEVLEN = -27

SPLIT_BALANCED = -1  # TQK_SPLIT_BALANCED
OUT_NORMALIZED = 0
OUT_PARTIAL = 1

_vp = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_f = ctypes.c_float
_sz = ctypes.c_size_t


class DecodeArgs(ctypes.Structure):
    """Mirror of tqk_decode_args (include/tqk.h)."""
    _fields_ = [
        ("k", _vp), ("v", _vp),
        ("item_stride", _i64),
        ("n_items", _i),
        ("n_q_heads", _i), ("n_kv_heads", _i), ("head_dim", _i), ("max_tokens", _i),
        ("lens", _vp),
        ("len0", _i), ("len_step", _i),
        ("max_len", _i),
        ("q", _vp), ("q_item_stride", _i64),
        ("out", _vp), ("out_item_stride", _i64),
        ("k_new", _vp), ("v_new", _vp),
        ("kv_new_item_stride", _i64),
        ("out_mode", _i),
        ("split_tokens", _i),
        ("q_norm", _vp), ("k_norm", _vp),
        ("norm_item_stride", _i64),
        ("norm_eps", _f),
        ("rope_cos", _vp), ("rope_sin", _vp),
        ("rope_item_stride", _i64),
    ]


def _sig(name, argtypes, restype=_i):
    fn = getattr(_lib, name)
    fn.argtypes = argtypes
    fn.restype = restype
    return fn


tqk_status_string = _sig("tqk_status_string", [_i], ctypes.c_char_p)
tqk_last_error = _sig("tqk_last_error", [], ctypes.c_char_p)
tqk_version = _sig("tqk_version", [], ctypes.c_char_p)
tqk_device_status = _sig("tqk_device_status", [ctypes.POINTER(_i), _i])
tqk_device_status_async = _sig("tqk_device_status_async", [_vp, _vp])
tqk_device_error_status = _sig("tqk_device_error_status", [_i])
tqk_quantize_rows_q8 = _sig("tqk_quantize_rows_q8", [_vp, _vp, _i, _i, _vp])
tqk_store_kv_q8 = _sig("tqk_store_kv_q8", [_vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp])
tqk_store_kv_q8_batch = _sig("tqk_store_kv_q8_batch", [_vp, _vp, _i, _i, _i, _i, _i, _vp, _vp, _vp])
tqk_attn_scores_q8 = _sig("tqk_attn_scores_q8", [_vp, _i, _vp, _i, _i, _f, _vp, _sz, _vp])
tqk_attn_accum_q8 = _sig("tqk_attn_accum_q8", [_vp, _sz, _i, _vp, _i, _i, _vp, _sz, _vp])
tqk_softmax_rows = _sig("tqk_softmax_rows", [_vp, _i, _i, _sz, _vp])
tqk_decode_workspace_size = _sig("tqk_decode_workspace_size", [ctypes.POINTER(DecodeArgs), ctypes.POINTER(_sz)])
tqk_workspace_init = _sig("tqk_workspace_init", [_vp, _sz, _vp])
tqk_decode_q8 = _sig("tqk_decode_q8", [ctypes.POINTER(DecodeArgs), _vp, _sz, _vp])
tqk_decode_q8_static = _sig("tqk_decode_q8_static", [ctypes.POINTER(DecodeArgs), _vp])
tqk_qk_norm_rope = _sig("tqk_qk_norm_rope", [_vp, _vp, _i, _i64, _i64, _i, _i, _i, _vp, _vp, _i64, _f, _vp, _vp,
                                              _i64, _vp])
tqk_packed_matrix_bytes = _sig("tqk_packed_matrix_bytes", [_i, _i, ctypes.c_char], _sz)
tqk_pack_matrix = _sig("tqk_pack_matrix", [_vp, _i, _i, _vp, ctypes.c_char, _vp])
tqk_matmul_q8 = _sig("tqk_matmul_q8", [_vp, _vp, _vp, _i, _i, _vp])
tqk_matmul_q4 = _sig("tqk_matmul_q4", [_vp, _vp, _vp, _i, _i, _vp])
tqk_matmul_q8_batch = _sig("tqk_matmul_q8_batch", [_vp, _vp, _vp, _i, _i, _i, _vp])
tqk_matmul_q4_batch = _sig("tqk_matmul_q4_batch", [_vp, _vp, _vp, _i, _i, _i, _vp])


class ProjJob(ctypes.Structure):
    """Mirror of tqk_proj_job (include/tqk.h)."""
    _fields_ = [("w", _vp), ("y", _vp), ("rows", _i)]


tqk_project = _sig("tqk_project", [ctypes.POINTER(ProjJob), _i, _i, _vp, _i, _i, _vp])


class AttnLayerArgs(ctypes.Structure):
    """Mirror of tqk_attn_layer_args (include/tqk.h)."""
    _fields_ = [
        ("wq", _vp), ("wk", _vp), ("wv", _vp), ("wo", _vp),
        ("format", _i),
        ("q_norm", _vp), ("k_norm", _vp),
        ("n_q_heads", _i), ("n_kv_heads", _i), ("head_dim", _i), ("hidden_size", _i),
        ("rms_eps", _f),
        ("k", _vp), ("v", _vp),
        ("max_tokens", _i),
        ("pos", _i),
        ("len", _vp),
        ("rope_cos", _vp), ("rope_sin", _vp),
        ("xn", _vp),
        ("out", _vp),
        ("scratch", _vp),
    ]


tqk_attention_layer = _sig("tqk_attention_layer", [ctypes.POINTER(AttnLayerArgs), _vp, _sz, _vp])


class LayerWeights(ctypes.Structure):
    """Mirror of tqk_layer_weights (include/tqk.h)."""
    _fields_ = [("input_norm", _vp), ("post_norm", _vp), ("wq", _vp), ("wk", _vp), ("wv", _vp), ("wo", _vp),
                ("q_norm", _vp), ("k_norm", _vp), ("wgate", _vp), ("wup", _vp), ("wdown", _vp),
                ("k_cache", _vp), ("v_cache", _vp)]


class Model(ctypes.Structure):
    """Mirror of tqk_model (include/tqk.h)."""
    _fields_ = [("n_layers", _i), ("n_q_heads", _i), ("n_kv_heads", _i), ("head_dim", _i), ("hidden_size", _i),
                ("intermediate_size", _i), ("vocab_size", _i), ("max_tokens", _i), ("rms_eps", _f), ("format", _i),
                ("embed", _vp), ("final_norm", _vp), ("rope_cos", _vp), ("rope_sin", _vp),
                ("layers", ctypes.POINTER(LayerWeights))]


tqk_forward_scratch_bytes = _sig("tqk_forward_scratch_bytes", [ctypes.POINTER(Model)], _sz)
tqk_forward_token = _sig("tqk_forward_token", [ctypes.POINTER(Model), _i, _i, _vp, _vp, _vp, _vp, _sz, _vp])
tqk_attend_q8 = _sig("tqk_attend_q8", [_vp, _vp, _i, _i, _i, _i, _i, _vp, _vp, _vp])
tqk_append_attend_q8 = _sig("tqk_append_attend_q8", [_vp, _vp, _i, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp])
tqk_prefill_q8 = _sig("tqk_prefill_q8", [_vp, _vp, _i, _i, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp])
tqk_merge_partials = _sig("tqk_merge_partials", [_vp, _i, _i64, _i, _i, _vp, _vp])
tqk_exchange_mailbox_bytes = _sig("tqk_exchange_mailbox_bytes", [_i, _i, _i], _sz)
tqk_peer_buffer_alloc = _sig("tqk_peer_buffer_alloc", [_sz, ctypes.POINTER(_vp)])
tqk_peer_buffer_free = _sig("tqk_peer_buffer_free", [_vp])
tqk_ipc_get_handle = _sig("tqk_ipc_get_handle", [_vp, ctypes.c_char_p])
tqk_ipc_open_handle = _sig("tqk_ipc_open_handle", [ctypes.c_char_p, ctypes.POINTER(_vp)])
tqk_ipc_close_handle = _sig("tqk_ipc_close_handle", [_vp])
tqk_exchange_slot_offset = _sig("tqk_exchange_slot_offset", [_i, _i, _i], _sz)
tqk_exchange_merge = _sig("tqk_exchange_merge", [_i, _i, _i, _i, ctypes.POINTER(_vp), _i, _vp, _vp])
class GatherDst(ctypes.Structure):
    """Mirror of tqk_gather_dst (include/tqk.h)."""
    _fields_ = [("world", _i), ("rank", _i), ("out", _vp * 8), ("chunk_heads", _i), ("epoch", _i)]


tqk_decode_q8_gather = _sig("tqk_decode_q8_gather", [ctypes.POINTER(DecodeArgs), ctypes.POINTER(GatherDst), _vp, _sz,
                                                      _vp])
tqk_decode_unit_count = _sig("tqk_decode_unit_count", [ctypes.POINTER(DecodeArgs), ctypes.POINTER(_i)])
tqk_gather_collect = _sig("tqk_gather_collect", [_vp, _sz, _i, _vp, _vp])
tqk_gather_mailbox_bytes = _sig("tqk_gather_mailbox_bytes", [_i, _i, _i], _sz)
tqk_gather_slot_offset = _sig("tqk_gather_slot_offset", [_i, _i, _i], _sz)
tqk_exchange_gather = _sig("tqk_exchange_gather", [_i, _i, _i, _i, ctypes.POINTER(_vp), _i, _vp, _vp])
tqk_fill_normal = _sig("tqk_fill_normal", [ctypes.c_uint64, ctypes.c_uint64, _vp, _sz, _f, _i])
tqk_fill_uniform = _sig("tqk_fill_uniform", [ctypes.c_uint64, ctypes.c_uint64, _vp, _sz, _i])
tqk_xorshift_jump = _sig("tqk_xorshift_jump", [ctypes.c_uint64, ctypes.c_uint64], ctypes.c_uint64)
IPC_HANDLE_BYTES = 64
REF_SEED = 88172645463325252  # TQK_REF_SEED: the reference benches' generator seed

EXPORTED = [
    "tqk_status_string", "tqk_last_error", "tqk_version", "tqk_device_status", "tqk_device_status_async",
    "tqk_device_error_status",
    "tqk_quantize_rows_q8", "tqk_store_kv_q8", "tqk_store_kv_q8_batch",
    "tqk_attn_scores_q8", "tqk_attn_accum_q8", "tqk_softmax_rows",
    "tqk_decode_workspace_size", "tqk_workspace_init", "tqk_decode_q8",
    "tqk_attend_q8", "tqk_append_attend_q8", "tqk_prefill_q8", "tqk_merge_partials",
    "tqk_decode_q8_static", "tqk_qk_norm_rope",
    "tqk_matmul_q8", "tqk_matmul_q4", "tqk_matmul_q8_batch", "tqk_matmul_q4_batch", "tqk_project",
    "tqk_attention_layer", "tqk_pack_matrix", "tqk_packed_matrix_bytes",
    "tqk_exchange_mailbox_bytes", "tqk_exchange_slot_offset", "tqk_peer_buffer_alloc", "tqk_peer_buffer_free",
    "tqk_ipc_get_handle",
    "tqk_ipc_open_handle", "tqk_ipc_close_handle", "tqk_exchange_merge",
    "tqk_gather_mailbox_bytes", "tqk_gather_slot_offset", "tqk_exchange_gather",
    "tqk_decode_q8_gather", "tqk_decode_unit_count", "tqk_gather_collect",
    "tqk_forward_scratch_bytes", "tqk_forward_token",
    "tqk_fill_normal", "tqk_fill_uniform", "tqk_xorshift_jump",
]


class TQKError(RuntimeError):
    def __init__(self, status: int, where: str):
        self.status = status
        msg = tqk_last_error().decode(errors="replace")
        super().__init__(f"{where}: {tqk_status_string(status).decode()} ({status}): {msg}")


def check(status: int, where: str) -> None:
    if status != OK:
        raise TQKError(status, where)


# ---------------------------------------------------------------------------
# torch helpers (torch is imported lazily: the library itself does not need it)
# ---------------------------------------------------------------------------
def _ptr(t) -> Optional[int]:
    if t is None:
        return None
    if isinstance(t, int):
        return t
    if not t.is_cuda:
        raise ValueError("tensor must live on a CUDA device")
    if not t.is_contiguous():
        raise ValueError("tensor must be contiguous")
    return t.data_ptr()


def _stream(stream) -> int:
    import torch
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def q8_bytes(rows: int, n: int) -> int:
    return rows * (n // QK) * BLOCK_BYTES


def empty_planes(n_kv: int, max_tokens: int, head_dim: int, device="cuda", leading=()):
    """Uninitialised uint8 tensor for a Q8 plane [*leading, n_kv, max_tokens, nb*36]."""
    import torch
    return torch.empty((*leading, n_kv, max_tokens, head_dim // QK * BLOCK_BYTES), dtype=torch.uint8, device=device)


def quantize_rows(x, out=None, stream=None):
    """quantize_row_q8 over the rows of a CUDA fp32 tensor [..., n] -> uint8 [..., n/32*36]."""
    import torch
    n = x.shape[-1]
    rows = x.numel() // n if n else 0
    if out is None:
        out = torch.empty((*x.shape[:-1], n // QK * BLOCK_BYTES), dtype=torch.uint8, device=x.device)
    check(tqk_quantize_rows_q8(_ptr(x), _ptr(out), rows, n, _stream(stream)), "tqk_quantize_rows_q8")
    return out


def store_kv(k_plane, v_plane, n_kv, head_dim, max_tokens, pos, k, v, stream=None):
    check(tqk_store_kv_q8(_ptr(k_plane), _ptr(v_plane), n_kv, head_dim, max_tokens, pos, _ptr(k), _ptr(v),
                          _stream(stream)), "tqk_store_kv_q8")


def store_kv_batch(k_plane, v_plane, n_kv, head_dim, max_tokens, pos0, n, k, v, stream=None):
    check(tqk_store_kv_q8_batch(_ptr(k_plane), _ptr(v_plane), n_kv, head_dim, max_tokens, pos0, n, _ptr(k),
                                _ptr(v), _stream(stream)), "tqk_store_kv_q8_batch")


def attend(k_plane, v_plane, n_q, n_kv, head_dim, max_tokens, pos, q, out, stream=None):
    check(tqk_attend_q8(_ptr(k_plane), _ptr(v_plane), n_q, n_kv, head_dim, max_tokens, pos, _ptr(q), _ptr(out),
                        _stream(stream)), "tqk_attend_q8")


def append_attend(k_plane, v_plane, n_q, n_kv, head_dim, max_tokens, pos, q, k, v, out, stream=None):
    check(tqk_append_attend_q8(_ptr(k_plane), _ptr(v_plane), n_q, n_kv, head_dim, max_tokens, pos, _ptr(q),
                               _ptr(k), _ptr(v), _ptr(out), _stream(stream)), "tqk_append_attend_q8")


def prefill(k_plane, v_plane, n_q, n_kv, head_dim, max_tokens, pos0, n, q, k, v, out, stream=None):
    check(tqk_prefill_q8(_ptr(k_plane), _ptr(v_plane), n_q, n_kv, head_dim, max_tokens, pos0, n, _ptr(q), _ptr(k),
                         _ptr(v), _ptr(out), _stream(stream)), "tqk_prefill_q8")


def attn_scores(q_blocks, g, k_blocks, n, nb, scale, scores, stride, stream=None):
    check(tqk_attn_scores_q8(_ptr(q_blocks), g, _ptr(k_blocks), n, nb, scale, _ptr(scores), stride,
                             _stream(stream)), "tqk_attn_scores_q8")


def attn_accum(w, w_stride, g, v_blocks, n, nb, out, out_stride, stream=None):
    check(tqk_attn_accum_q8(_ptr(w), w_stride, g, _ptr(v_blocks), n, nb, _ptr(out), out_stride, _stream(stream)),
          "tqk_attn_accum_q8")


def softmax_rows(x, rows, n, stride, stream=None):
    check(tqk_softmax_rows(_ptr(x), rows, n, stride, _stream(stream)), "tqk_softmax_rows")


def decode_args(k, v, n_q, n_kv, head_dim, max_tokens, q, out, *, n_items=1, item_stride_blocks=0, lens=None,
                len0=0, len_step=0, max_len=0, q_item_stride=0, out_item_stride=0, k_new=None, v_new=None,
                kv_new_item_stride=0, out_mode=OUT_NORMALIZED, split_tokens=0, q_norm=None, k_norm=None,
                norm_item_stride=0, norm_eps=1e-6, rope_cos=None, rope_sin=None, rope_item_stride=0) -> DecodeArgs:
    a = DecodeArgs()
    a.k, a.v = _ptr(k), _ptr(v)
    a.item_stride = item_stride_blocks
    a.n_items = n_items
    a.n_q_heads, a.n_kv_heads, a.head_dim, a.max_tokens = n_q, n_kv, head_dim, max_tokens
    a.lens = _ptr(lens)
    a.len0, a.len_step, a.max_len = len0, len_step, max_len
    a.q, a.q_item_stride = _ptr(q), q_item_stride
    a.out, a.out_item_stride = _ptr(out), out_item_stride
    a.k_new, a.v_new = _ptr(k_new), _ptr(v_new)
    a.kv_new_item_stride = kv_new_item_stride
    a.out_mode = out_mode
    a.split_tokens = split_tokens
    a.q_norm, a.k_norm = _ptr(q_norm), _ptr(k_norm)
    a.norm_item_stride, a.norm_eps = norm_item_stride, norm_eps
    a.rope_cos, a.rope_sin = _ptr(rope_cos), _ptr(rope_sin)
    a.rope_item_stride = rope_item_stride
    return a


def decode(args: DecodeArgs, workspace=None, stream=None) -> None:
    ws = _ptr(workspace) if workspace is not None else None
    nbytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    check(tqk_decode_q8(ctypes.byref(args), ws, nbytes, _stream(stream)), "tqk_decode_q8")


def qk_norm_rope(q, k, n_items, n_q, n_kv, head_dim, q_norm=None, k_norm=None, eps=1e-6, rope_cos=None,
                 rope_sin=None, q_item_stride=0, k_item_stride=0, norm_item_stride=0, rope_item_stride=0,
                 stream=None) -> None:
    """tqk_qk_norm_rope: in-place per-head RMSNorm and RoPE of q and k (the reference's norm_heads + rope_heads)."""
    check(tqk_qk_norm_rope(_ptr(q), _ptr(k), n_items, q_item_stride, k_item_stride, n_q, n_kv, head_dim,
                           _ptr(q_norm), _ptr(k_norm), norm_item_stride, eps, _ptr(rope_cos), _ptr(rope_sin),
                           rope_item_stride, _stream(stream)), "tqk_qk_norm_rope")


FMT_Q8, FMT_Q4 = 0, 1
Q4_BLOCK_BYTES = 20


def pack_matrix(w, fmt: str, out=None, stream=None):
    """tqk_pack_matrix: fp32 CUDA tensor W [rows, cols] -> packed Q8 ('8') / Q4 ('4') rows (uint8)."""
    import torch
    rows, cols = w.shape
    nbytes = tqk_packed_matrix_bytes(rows, cols, fmt.encode())
    if out is None:
        out = torch.empty(nbytes, dtype=torch.uint8, device=w.device)
    check(tqk_pack_matrix(_ptr(w), rows, cols, _ptr(out), fmt.encode(), _stream(stream)), "tqk_pack_matrix")
    return out.view(rows, -1)


def matmul(w, fmt, xq, y, rows, cols, n_tok=1, stream=None) -> None:
    """tqk_matmul_{q8,q4}[_batch]: y[t*rows + r] = W[r] . xq[t] (fmt FMT_Q8 / FMT_Q4; device tensors)."""
    fn = tqk_matmul_q8_batch if fmt == FMT_Q8 else tqk_matmul_q4_batch
    check(fn(_ptr(w), _ptr(xq), _ptr(y), rows, cols, n_tok, _stream(stream)), "tqk_matmul")


def project(jobs, fmt, x, cols, n_tok=1, stream=None) -> None:
    """tqk_project: quantise the n_tok fp32 rows of x and run every (w, y, rows) job in one launch."""
    arr = (ProjJob * len(jobs))(*[ProjJob(_ptr(w), _ptr(y), rows) for (w, y, rows) in jobs])
    check(tqk_project(arr, len(jobs), fmt, _ptr(x), cols, n_tok, _stream(stream)), "tqk_project")


def layer_scratch_floats(n_q, n_kv, head_dim) -> int:
    """Floats of scratch tqk_attention_layer needs (q, k, v, attention)."""
    return 2 * n_q * head_dim + 2 * n_kv * head_dim


def attention_layer_args(w, fmt, q_norm, k_norm, n_q, n_kv, head_dim, hidden, eps, k, v, max_tokens, pos,
                         rope_cos, rope_sin, xn, out, scratch, len_dev=None) -> AttnLayerArgs:
    """tqk_attn_layer_args from device tensors; w maps 'wq', 'wk', 'wv', 'wo' to packed rows."""
    a = AttnLayerArgs()
    a.wq, a.wk, a.wv, a.wo = (_ptr(w[n]) for n in ("wq", "wk", "wv", "wo"))
    a.format = fmt
    a.q_norm, a.k_norm = _ptr(q_norm), _ptr(k_norm)
    a.n_q_heads, a.n_kv_heads, a.head_dim, a.hidden_size = n_q, n_kv, head_dim, hidden
    a.rms_eps = eps
    a.k, a.v = _ptr(k), _ptr(v)
    a.max_tokens, a.pos = max_tokens, pos
    a.len = _ptr(len_dev)
    a.rope_cos, a.rope_sin = _ptr(rope_cos), _ptr(rope_sin)
    a.xn, a.out, a.scratch = _ptr(xn), _ptr(out), _ptr(scratch)
    return a


def attention_layer(args: AttnLayerArgs, workspace=None, stream=None) -> None:
    """tqk_attention_layer: one token through one attention layer on the device."""
    ws = _ptr(workspace) if workspace is not None else None
    nbytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    check(tqk_attention_layer(ctypes.byref(args), ws, nbytes, _stream(stream)), "tqk_attention_layer")


def model_struct(cfg: dict, layers: list, embed, final_norm, rope_cos, rope_sin, fmt: int = 0) -> Model:
    """tqk_model from device tensors.  cfg: n_layers, n_q_heads, n_kv_heads, head_dim, hidden_size,
    intermediate_size, vocab_size, max_tokens, rms_eps; layers: one dict per layer with the keys of
    tqk_layer_weights.  The returned struct keeps its layer array alive."""
    arr = (LayerWeights * len(layers))()
    for i, lw in enumerate(layers):
        for k, _t in LayerWeights._fields_:
            setattr(arr[i], k, _ptr(lw[k]))
    m = Model()
    for k in ("n_layers", "n_q_heads", "n_kv_heads", "head_dim", "hidden_size", "intermediate_size", "vocab_size",
              "max_tokens"):
        setattr(m, k, int(cfg[k]))
    m.rms_eps = float(cfg["rms_eps"])
    m.format = fmt
    m.embed, m.final_norm, m.rope_cos, m.rope_sin = _ptr(embed), _ptr(final_norm), _ptr(rope_cos), _ptr(rope_sin)
    m.layers = ctypes.cast(arr, ctypes.POINTER(LayerWeights))
    m._keep = arr  # noqa: SLF001  (the layer array must outlive the struct)
    return m


def forward_scratch_bytes(model: Model) -> int:
    return tqk_forward_scratch_bytes(ctypes.byref(model))


def forward_token(model: Model, token: int, pos: int, scratch, logits, next_token=None, workspace=None,
                  stream=None) -> None:
    """tqk_forward_token: one token through the whole stack on the device."""
    ws = _ptr(workspace) if workspace is not None else None
    nbytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    check(tqk_forward_token(ctypes.byref(model), token, pos, _ptr(scratch), _ptr(logits), _ptr(next_token), ws,
                            nbytes, _stream(stream)), "tqk_forward_token")


def decode_static(args: DecodeArgs, stream=None) -> None:
    """tqk_decode_q8_static: the decode with the library's static scratch (no device allocation)."""
    check(tqk_decode_q8_static(ctypes.byref(args), _stream(stream)), "tqk_decode_q8_static")


def decode_workspace_size(args: DecodeArgs) -> int:
    out = _sz(0)
    check(tqk_decode_workspace_size(ctypes.byref(args), ctypes.byref(out)), "tqk_decode_workspace_size")
    return out.value


def workspace_init(workspace, stream=None) -> None:
    check(tqk_workspace_init(_ptr(workspace), workspace.numel() * workspace.element_size(), _stream(stream)),
          "tqk_workspace_init")


def merge_partials(parts, n_parts, part_stride, n_heads, head_dim, out, stream=None):
    check(tqk_merge_partials(_ptr(parts), n_parts, part_stride, n_heads, head_dim, _ptr(out), _stream(stream)),
          "tqk_merge_partials")


def peer_buffer_alloc(nbytes: int) -> int:
    """A zeroed device buffer that is one whole allocation (so that its IPC handle maps exactly it)."""
    p = _vp()
    check(tqk_peer_buffer_alloc(nbytes, ctypes.byref(p)), "tqk_peer_buffer_alloc")
    return p.value


def peer_buffer_free(ptr: int) -> None:
    check(tqk_peer_buffer_free(ptr), "tqk_peer_buffer_free")


def ipc_get_handle(ptr: int) -> bytes:
    buf = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    check(tqk_ipc_get_handle(ptr, buf), "tqk_ipc_get_handle")
    return buf.raw


def ipc_open_handle(handle: bytes) -> int:
    if len(handle) != IPC_HANDLE_BYTES:
        raise ValueError("an IPC handle is 64 bytes")
    p = _vp()
    check(tqk_ipc_open_handle(handle, ctypes.byref(p)), "tqk_ipc_open_handle")
    return p.value


def ipc_close_handle(ptr: int) -> None:
    check(tqk_ipc_close_handle(ptr), "tqk_ipc_close_handle")


def exchange_merge(n_heads, head_dim, world, rank, mailboxes, epoch, out, stream=None):
    """tqk_exchange_merge: mailboxes is the list of every rank's mailbox address in this process;
    this rank's records of the epoch must already be in its slot (exchange_slot)."""
    arr = (_vp * len(mailboxes))(*mailboxes)
    check(tqk_exchange_merge(n_heads, head_dim, world, rank, arr, epoch, _ptr(out), _stream(stream)),
          "tqk_exchange_merge")


def exchange_gather(n_groups, chunk_floats, world, rank, mailboxes, epoch, out, stream=None):
    """tqk_exchange_gather: out[g][r][:] = rank r's group g of the epoch, on every rank."""
    arr = (_vp * len(mailboxes))(*mailboxes)
    check(tqk_exchange_gather(n_groups, chunk_floats, world, rank, arr, epoch, _ptr(out), _stream(stream)),
          "tqk_exchange_gather")


def gather_dst(world: int, rank: int, outs, chunk_heads: int, epoch: int) -> GatherDst:
    """tqk_gather_dst: every rank's pair buffer as mapped in this process, for the step `epoch` (>= 1)."""
    d = GatherDst()
    d.world, d.rank, d.chunk_heads, d.epoch = world, rank, chunk_heads, epoch
    for r in range(world):
        d.out[r] = outs[r]
    return d


def decode_gather(args: DecodeArgs, dst: GatherDst, workspace=None, stream=None) -> None:
    """tqk_decode_q8_gather: the decode with every unit's output pushed to every rank's buffer."""
    ws = _ptr(workspace) if workspace is not None else None
    nbytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    check(tqk_decode_q8_gather(ctypes.byref(args), ctypes.byref(dst), ws, nbytes, _stream(stream)),
          "tqk_decode_q8_gather")


def decode_unit_count(args: DecodeArgs) -> int:
    n = _i(0)
    check(tqk_decode_unit_count(ctypes.byref(args), ctypes.byref(n)), "tqk_decode_unit_count")
    return n.value


def gather_collect(pairs: int, n: int, epoch: int, out, stream=None) -> None:
    """tqk_gather_collect: waits until the n {value, epoch} pairs at device address `pairs` show the
    epoch and writes the values to out."""
    check(tqk_gather_collect(pairs, n, epoch, _ptr(out), _stream(stream)), "tqk_gather_collect")


class _DeviceArray:
    """A raw device address seen through __cuda_array_interface__ (torch.as_tensor views it without a copy)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


def device_array(ptr: int, shape, dtype="float32"):
    """A torch CUDA tensor viewing `shape` elements at device address ptr (memory owned elsewhere, for
    instance a tqk_peer_buffer_alloc buffer)."""
    import torch
    typestr = {"float32": "<f4", "uint8": "|u1", "int32": "<i4", "int64": "<i8"}[dtype]
    return torch.as_tensor(_DeviceArray(ptr, shape, typestr), device="cuda")


def gather_slot(mailbox: int, n_groups: int, chunk_floats: int, epoch: int) -> int:
    """Address of the epoch's slot in a gather mailbox."""
    return mailbox + tqk_gather_slot_offset(n_groups, chunk_floats, epoch)


def exchange_slot(mailbox: int, n_heads: int, head_dim: int, epoch: int) -> int:
    """Address of the epoch's partial-record slot in a mailbox."""
    return mailbox + tqk_exchange_slot_offset(n_heads, head_dim, epoch)


def device_status(clear: bool = False) -> int:
    v = _i(0)
    check(tqk_device_status(ctypes.byref(v), int(clear)), "tqk_device_status")
    return v.value


def fill_normal(first: int, n: int, scale: float = 1.0, seed: int = REF_SEED, threads: int = 0, out=None):
    """tqk_fill_normal: samples first .. first + n - 1 of the reference benches' N(0,1)
    stream (xorshift64 + Box-Muller), times scale, as a float32 numpy array (or into
    `out`, a C-contiguous float32 numpy array of n values)."""
    import numpy as np
    if out is None:
        out = np.empty(n, np.float32)
    assert out.dtype == np.float32 and out.flags.c_contiguous and out.size == n
    check(tqk_fill_normal(seed, first, out.ctypes.data, n, scale, threads), "tqk_fill_normal")
    return out


def fill_uniform(first: int, n: int, seed: int = REF_SEED, threads: int = 0, out=None):
    """tqk_fill_uniform: uniforms first .. first + n - 1 of the same generator, in (0, 1]."""
    import numpy as np
    if out is None:
        out = np.empty(n, np.float32)
    assert out.dtype == np.float32 and out.flags.c_contiguous and out.size == n
    check(tqk_fill_uniform(seed, first, out.ctypes.data, n, threads), "tqk_fill_uniform")
    return out
