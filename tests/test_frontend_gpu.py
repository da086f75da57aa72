"""vkb_log_mel (vokra_b200/csrc/frontend.cu) against the oracle's log_mel and the
reference's golden log-mel features."""
import numpy as np
import pytest

from oracle import py as o
from vokra_b200 import _lib

from test_frontend_oracle import golden

pytestmark = pytest.mark.gpu


def _dev(ctx, pcm_rows, n_mels, stride, lengths=None):
    import torch
    from vokra_b200 import ops
    x = torch.zeros((len(pcm_rows), stride), dtype=torch.float32)
    for i, r in enumerate(pcm_rows):
        x[i, :min(len(r), stride)] = torch.from_numpy(np.asarray(r[:stride], np.float32))
    x = x.cuda()
    lt = None if lengths is None else torch.tensor(lengths, dtype=torch.int32, device="cuda")
    out = ops.log_mel(ctx, x, n_mels, lengths=lt)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def test_log_mel_golden(ctx):
    # crates/vokra-models/tests/parity_whisper.rs:279-299: first 100 frames within atol 0.01
    pcm, ref, atol = golden()
    got = _dev(ctx, [pcm], 80, pcm.size)[0]
    assert np.max(np.abs(got[:, :ref.shape[1]] - ref)) <= atol
    want = o.log_mel(pcm, 80)
    # same f64 DFT, f32 power and mel sums in the oracle's order: only log10 rounding differs
    assert np.max(np.abs(got - want)) <= 2e-5


def test_log_mel_batch_ragged(ctx):
    rng = np.random.default_rng(12)
    sr = 16000
    t = np.arange(8 * sr) / sr
    tones = (0.1 * rng.standard_normal(t.size) + sum(0.05 * np.sin(2 * np.pi * f * t + p) for f, p in
             zip(rng.uniform(100, 4000, 3), rng.uniform(0, 2 * np.pi, 3)))).astype(np.float32)
    pcm, _, _ = golden()
    over = (0.2 * rng.standard_normal(480000 + 5000)).astype(np.float32)
    rows = [pcm, tones, np.zeros(0, np.float32), over, tones[:1]]
    stride = 485000
    lengths = [pcm.size, tones.size, 0, over.size, 1]
    for n_mels in (80, 128):
        got = _dev(ctx, rows, n_mels, stride, lengths)
        assert got.shape == (5, n_mels, 3000)
        for i, r in enumerate(rows):
            want = o.log_mel(r, n_mels)
            assert np.max(np.abs(got[i] - want)) <= 2e-5, (n_mels, i)


def test_log_mel_rejections(ctx):
    import ctypes as C
    import torch
    L = _lib.load()
    x = torch.zeros((1, 16000), device="cuda")
    out = torch.empty((1, 80, 3000), device="cuda")
    p, o_ = C.c_void_p(x.data_ptr()), C.c_void_p(out.data_ptr())
    assert L.vkb_log_mel(ctx.h, p, 1, 16000, None, 0, o_) == _lib.ERROR_INVALID_ARGUMENT
    assert L.vkb_log_mel(ctx.h, p, 1, 16000, None, 300, o_) == _lib.ERROR_INVALID_ARGUMENT
    assert L.vkb_log_mel(ctx.h, p, 0, 16000, None, 80, o_) == _lib.ERROR_INVALID_ARGUMENT
    assert L.vkb_log_mel(ctx.h, p, 1, -1, None, 80, o_) == _lib.ERROR_INVALID_ARGUMENT
    assert L.vkb_log_mel(ctx.h, None, 1, 16000, None, 80, o_) == _lib.ERROR_INVALID_ARGUMENT
