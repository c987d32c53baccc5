"""The drop-in boundary end to end: the reference's own unit-test program
(tools/test_model.c, unchanged) linked against libtq_attn_b200.so in place of
the reference's model/attn_q8.c, model/attention_layer.c and model/kv_cache.c
(oracle/Makefile target _ref/test_model_dropin, built where the reference tree
is present and carried with the repository).  Every Q8 attention test of the
reference suite -- the kernel sweep with guards, the layer tests with garbage
sentinels, the forward-pass tests -- then runs on the GPU path and must pass."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(ROOT, "oracle", "_ref", "test_model_dropin")

pytestmark = pytest.mark.gpu


def test_reference_suite_passes_through_the_dropin(cuda):
    if not os.path.exists(EXE):
        pytest.skip("oracle/_ref/test_model_dropin not built (needs the reference tree at build time)")
    res = subprocess.run([EXE], capture_output=True, text=True, timeout=600)
    lines = res.stdout.splitlines()
    failed = [l for l in lines if l.endswith("FAIL")]
    assert res.returncode == 0 and not failed, "\n".join(failed + lines[-5:] + [res.stderr[-2000:]])
    assert "All tests passed." in res.stdout
    for name in ("attention q8 kernels (dispatched and scalar): PASS",
                 "attention layer q8 cache vs f32 cache: PASS",
                 "tq_forward_token vs reference (kv q8): ok"):
        assert name in res.stdout
