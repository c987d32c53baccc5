"""The C ABI: both libraries load, export exactly what include/*.h declares,
and reject bad arguments with the documented status codes before touching a
device (so these run on any machine, GPU or not)."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "tailorquantkernel_b200")


def _declared(header, macro):
    lines = open(os.path.join(ROOT, "include", header)).read().splitlines()
    text = "\n".join(l for l in lines if not l.lstrip().startswith("#"))
    return sorted(set(re.findall(macro + r"\s+[\w\s\*]*?\b(\w+)\s*\(", text)))


def _exported(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", lib], capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


def test_tqk_exports_every_declared_symbol():
    lib = os.path.join(PKG, "libtqk.so")
    declared = _declared("tqk.h", "TQK_API")
    assert len(declared) >= 17
    exported = _exported(lib)
    assert set(declared) <= exported, set(declared) - exported
    # nothing else leaks out of the library (hidden visibility)
    assert exported == set(declared), exported - set(declared)
    ctypes.CDLL(lib)  # loads without a GPU


def test_dropin_exports_the_reference_entry_points():
    lib = os.path.join(PKG, "libtq_attn_b200.so")
    declared = _declared("tq_attn_b200.h", "TQ_B200_API")
    reference_names = {"tq_kv_cache_init", "tq_kv_cache_free", "tq_attn_validate", "tq_attn_validate_cache",
                       "attention_layer", "attention_layer_batch", "attention_head_q8", "attn_scores_q8",
                       "attn_accum_q8"}
    assert reference_names <= set(declared)
    assert set(declared) == _exported(lib)


def test_python_binding_covers_the_abi():
    from tailorquantkernel_b200 import tqk
    assert set(tqk.EXPORTED) == set(_declared("tqk.h", "TQK_API"))


def test_decode_args_layout_matches_c(tmp_path):
    """The ctypes mirror of tqk_decode_args has the C layout (size and offsets)."""
    from tailorquantkernel_b200 import tqk
    fields = [f for f, _ in tqk.DecodeArgs._fields_]
    src = tmp_path / "layout.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "tqk.h"\nint main(void){\n'
                   'printf("%zu\\n", sizeof(tqk_decode_args));\n' +
                   "".join(f'printf("%zu\\n", offsetof(tqk_decode_args, {f}));\n' for f in fields) + "return 0;}\n")
    exe = tmp_path / "layout"
    subprocess.run(["/usr/bin/gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    vals = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    assert vals[0] == ctypes.sizeof(tqk.DecodeArgs)
    assert vals[1:] == [getattr(tqk.DecodeArgs, f).offset for f in fields]


def test_attn_layer_args_layout_matches_c(tmp_path):
    """The ctypes mirror of tqk_attn_layer_args has the C layout (size and offsets)."""
    from tailorquantkernel_b200 import tqk
    fields = [f for f, _ in tqk.AttnLayerArgs._fields_]
    src = tmp_path / "layout.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "tqk.h"\nint main(void){\n'
                   'printf("%zu\\n", sizeof(tqk_attn_layer_args));\n' +
                   "".join(f'printf("%zu\\n", offsetof(tqk_attn_layer_args, {f}));\n' for f in fields) +
                   "return 0;}\n")
    exe = tmp_path / "layout"
    subprocess.run(["/usr/bin/gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    vals = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    assert vals[0] == ctypes.sizeof(tqk.AttnLayerArgs)
    assert vals[1:] == [getattr(tqk.AttnLayerArgs, f).offset for f in fields]


def test_decode_prologue_arguments_checked_before_the_device():
    """q_norm/k_norm and rope_cos/rope_sin come in pairs; the check precedes any device work."""
    from tailorquantkernel_b200 import tqk
    fake = ctypes.c_void_p(4096)
    for kw in (dict(q_norm=fake), dict(k_norm=fake), dict(rope_cos=fake), dict(rope_sin=fake)):
        a = tqk.DecodeArgs()
        a.k = a.v = a.q = a.out = fake
        a.n_items, a.n_q_heads, a.n_kv_heads, a.head_dim, a.max_tokens, a.len0 = 1, 32, 8, 128, 64, 10
        for f, v in kw.items():
            setattr(a, f, v)
        assert tqk.tqk_decode_q8(ctypes.byref(a), None, 0, None) == tqk.EINVAL


def test_packed_matrix_bytes_without_device():
    """packed_matrix_bytes (packer/packer.c:63-75): 36 / 20 bytes per 32 columns, 0 when invalid."""
    from tailorquantkernel_b200 import tqk
    assert tqk.tqk_packed_matrix_bytes(3, 64, b"8") == 3 * 2 * 36
    assert tqk.tqk_packed_matrix_bytes(3, 64, b"4") == 3 * 2 * 20
    assert tqk.tqk_packed_matrix_bytes(3, 48, b"8") == 0
    assert tqk.tqk_packed_matrix_bytes(0, 64, b"8") == 0
    assert tqk.tqk_packed_matrix_bytes(3, 64, b"x") == 0


def test_exchange_mailbox_without_device():
    """tqk_exchange_mailbox_bytes: two parity slots of every rank's records plus flags and
    tickets, 0 outside 1..8 ranks; tqk_exchange_merge rejects bad arguments before any
    device work."""
    from tailorquantkernel_b200 import tqk
    for world in (1, 2, 8):
        b = tqk.tqk_exchange_mailbox_bytes(world, 64, 128)
        assert b >= 2 * 64 * 130 * 4 + 2 * world * 4 and b % 256 == 0
    assert tqk.tqk_exchange_slot_offset(64, 128, 1) == 64 * 130 * 4  # odd epochs in the second slot
    assert tqk.tqk_exchange_slot_offset(64, 128, 2) == 0
    assert tqk.tqk_exchange_slot_offset(64, 128, 0) == 0
    assert tqk.tqk_exchange_mailbox_bytes(0, 64, 128) == 0
    assert tqk.tqk_exchange_mailbox_bytes(9, 64, 128) == 0
    boxes = (ctypes.c_void_p * 2)(None, None)
    assert tqk.tqk_exchange_merge(64, 128, 2, 0, boxes, 1, None, None) == tqk.EINVAL
    assert tqk.tqk_exchange_merge(64, 128, 2, 2, boxes, 1, 1, None) == tqk.EINVAL  # rank outside the world
    assert tqk.tqk_exchange_merge(64, 128, 2, 0, boxes, 0, 1, None) == tqk.EINVAL  # epochs start at 1


def test_error_codes_without_device():
    from tailorquantkernel_b200 import tqk
    # position checks come first and never touch a device (reference: -1 on bad pos)
    assert tqk.tqk_store_kv_q8(None, None, 8, 128, 16, -1, None, None, None) == tqk.EPOS
    assert tqk.tqk_store_kv_q8(None, None, 8, 128, 16, 16, None, None, None) == tqk.EPOS
    assert tqk.tqk_attend_q8(None, None, 32, 8, 128, 16, 16, None, None, None) == tqk.EPOS
    assert tqk.tqk_append_attend_q8(None, None, 32, 8, 128, 16, -3, None, None, None, None, None) == tqk.EPOS
    assert tqk.tqk_prefill_q8(None, None, 32, 8, 128, 16, 10, 7, None, None, None, None, None) == tqk.EPOS
    assert tqk.tqk_quantize_rows_q8(None, None, 4, 33, None) == tqk.EINVAL
    assert b"multiple of 32" in tqk.tqk_last_error()
    a = tqk.DecodeArgs()
    a.n_items, a.n_q_heads, a.n_kv_heads, a.head_dim, a.max_tokens = 1, 6, 4, 128, 16
    assert tqk.tqk_decode_q8(ctypes.byref(a), None, 0, None) == tqk.EINVAL  # 6 % 4 != 0
    a.n_q_heads, a.head_dim = 8, 96
    assert tqk.tqk_decode_q8(ctypes.byref(a), None, 0, None) == tqk.EUNSUPPORTED
    assert tqk.tqk_status_string(tqk.EALIGN) == b"device pointer not 16-byte aligned"


def test_product_has_no_cpu_path():
    """The package binds only libtqk.so; nothing under tailorquantkernel_b200 imports the oracle."""
    for dirpath, _, files in os.walk(PKG):
        for f in files:
            if f.endswith((".py", ".c", ".cu", ".h", ".cuh")):
                text = open(os.path.join(dirpath, f), errors="replace").read()
                assert "import oracle" not in text and "tq_oracle" not in text, f
