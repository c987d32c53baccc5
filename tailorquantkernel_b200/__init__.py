"""tailorquantkernel_b200 -- B200 (sm_100a) Q8 GQA attention behind a C ABI.

The product is two native libraries built in-tree by ``tailorquantkernel_b200.build``:

* ``libtqk.so`` -- the CUDA kernels and their C ABI (``include/tqk.h``);
* ``libtq_attn_b200.so`` -- a plain-C drop-in for the reference's attention entry
  points (``include/tq_attn_b200.h``), linked by C callers in place of the
  reference's ``model/attn_q8.c``, ``model/attention_layer.c`` and ``model/kv_cache.c``.

This Python module only binds ``libtqk.so`` with ctypes for the tests and the
benchmark (torch supplies device memory and streams).  There is no CPU path:
importing :mod:`tailorquantkernel_b200.tqk` raises when the library is missing.
"""

__all__ = ["tqk", "build"]
