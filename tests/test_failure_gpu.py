"""The device failure path without a GPU fault: a bounded wait that runs out.

vkb_context_selftest_bounded_wait launches a kernel whose mbarrier wait can
never complete (nothing arrives), bounded by a poll count exactly like every
pipeline wait in the tensor-core GEMMs and the streaming GEMV. The kernel
gives up, records the device error flag and returns; the host reads the flag
and reports VKB_ERROR_OTHER, and the same context keeps computing correctly.
"""
import numpy as np
import pytest

from oracle import py as o
from vokra_b200 import _lib, synth

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_context_survives(ctx):
    from vokra_b200 import ops
    L = _lib.load()
    for polls in (1, 1000):
        st = L.vkb_context_selftest_bounded_wait(ctx.h, polls)
        assert st == _lib.ERROR_OTHER, st
        assert "gave up" in L.vkb_last_error().decode()
    assert L.vkb_context_selftest_bounded_wait(ctx.h, 0) == _lib.ERROR_INVALID_ARGUMENT
    # the context still works, and the flag was cleared (gemm_q_f32 checks it)
    n, k, m = 256, 512, 3
    rng = np.random.default_rng(1)
    wq = synth.quantize(synth.Q8_0, rng.standard_normal(n * k).astype(np.float32) * np.float32(0.02))
    a = rng.standard_normal((m, k)).astype(np.float32)
    out = np.zeros((m, n), np.float32)
    ops.gemm_q_f32(ctx, m, n, k, a, wq, synth.Q8_0, None, out)
    ref = o.linear_q(synth.Q8_0, a, wq, n, k)
    assert np.max(np.abs(out - ref)) <= 1e-4
