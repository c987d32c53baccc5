"""Build recipe for the native libraries of tailorquantkernel_b200.

Produces, in-tree (so they travel with the repository snapshot):
  tailorquantkernel_b200/libtqk.so           CUDA kernels + C ABI (include/tqk.h), sm_100a only
  tailorquantkernel_b200/libtq_attn_b200.so  plain-C drop-in for the reference's attention
                                             entry points (include/tq_attn_b200.h), over libtqk.so

Flags: -gencode arch=compute_100a,code=sm_100a, -O3, -lineinfo, IEEE division and
square root (nvcc defaults; never --use_fast_math, which would break the bit-exact
quantiser).  Run as ``python -m tailorquantkernel_b200.build``.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")

CUDA_SOURCES = ["tqk_runtime.cu", "tqk_quant.cu", "tqk_decode.cu", "tqk_prefill.cu", "tqk_prologue.cu",
                "tqk_matvec.cu", "tqk_layer.cu", "tqk_pack.cu", "tqk_ref_ops.cu", "tqk_exchange.cu",
                "tqk_forward.cu", "tqk_inputs.cu"]
DROPIN_SOURCES = ["dropin/tq_attn_b200.c"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-Xptxas", "-warn-spills",
]

HOST_CC = "/usr/bin/gcc"  # the image's $CC (/opt/gcc) lacks libgomp


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build tailorquantkernel_b200")


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout)
        raise RuntimeError(f"build step failed ({res.returncode}): {' '.join(cmd[:3])} ...")
    if verbose and res.stdout.strip():
        print(res.stdout)


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _deps(names: list[str]) -> list[str]:
    out = [os.path.join(CSRC, n) for n in names]
    for d in (CSRC, os.path.join(CSRC, "dropin"), INCLUDE):
        if os.path.isdir(d):
            out += [os.path.join(d, f) for f in os.listdir(d) if f.endswith((".h", ".cuh"))]
    return out


def build_tqk(verbose: bool = False, force: bool = False) -> str:
    out = os.path.join(PKG, "libtqk.so")
    srcs = [os.path.join(CSRC, s) for s in CUDA_SOURCES]
    if force or _stale(out, _deps(CUDA_SOURCES)):
        cmd = [_nvcc(), *NVCC_FLAGS, "-shared", "-o", out + ".tmp", *srcs]
        _run(cmd, verbose)
        os.replace(out + ".tmp", out)
    return out


def build_dropin(verbose: bool = False, force: bool = False) -> str:
    out = os.path.join(PKG, "libtq_attn_b200.so")
    srcs = [os.path.join(CSRC, s) for s in DROPIN_SOURCES]
    deps = _deps(DROPIN_SOURCES) + [os.path.join(PKG, "libtqk.so")]
    if force or _stale(out, deps):
        cuda = os.path.dirname(os.path.dirname(_nvcc()))
        # cudart is linked statically and kept private (--exclude-libs), so the
        # library carries no runtime dependency beyond libtqk.so and the driver
        cmd = [HOST_CC, "-std=gnu11", "-O2", "-fPIC", "-shared", "-ffp-contract=off",
               "-Wall", "-Wno-unused-function", f"-I{INCLUDE}", f"-I{cuda}/include", "-o", out + ".tmp", *srcs,
               f"-L{PKG}", "-ltqk", "-Wl,-rpath,$ORIGIN", f"-L{cuda}/lib64", "-l:libcudart_static.a",
               "-Wl,--exclude-libs,ALL", "-ldl", "-lpthread", "-lrt", "-lm"]
        _run(cmd, verbose)
        os.replace(out + ".tmp", out)
    return out


def build_oracle(verbose: bool = False) -> None:
    """Builds the CPU checkers (oracle/): always the restatement, and the
    reference builds when the reference tree is present on this machine."""
    oracle = os.path.join(ROOT, "oracle")
    _run(["make", "-s", "-C", oracle, "all"], verbose)
    # the reference tree: $TQK_REFERENCE, else a "reference" directory beside the repository
    ref = os.environ.get("TQK_REFERENCE") or os.path.join(os.path.dirname(ROOT), "reference")
    if os.path.isdir(ref):
        _run(["make", "-s", "-C", oracle, f"REF={ref}", "ref"], verbose)
        if os.path.exists(os.path.join(PKG, "libtq_attn_b200.so")):
            _run(["make", "-s", "-C", oracle, f"REF={ref}", "_ref/test_model_dropin", "_ref/libtqref_dropin.so"],
                 verbose)


def build_all(verbose: bool = False, force: bool = False) -> None:
    build_tqk(verbose, force)
    if all(os.path.exists(os.path.join(CSRC, s)) for s in DROPIN_SOURCES):
        build_dropin(verbose, force)
    build_oracle(verbose)


if __name__ == "__main__":
    build_all(verbose="-v" in sys.argv, force="-f" in sys.argv)
