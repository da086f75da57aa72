"""The log-mel frontend oracle (oracle/vkb_oracle.cpp, orc_log_mel) against the
reference's golden features and its frontend unit tests (CPU only)."""
import os

import numpy as np

from oracle import py as o

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "whisper_base_frontend.npz")


def golden():
    z = np.load(GOLDEN)
    return (z["pcm"].astype(np.float32) / np.float32(32768.0)), z["logmel"], float(z["atol"])


def test_log_mel_matches_reference_golden():
    # crates/vokra-models/tests/parity_whisper.rs:279-299 (log_mel_parity): first 100 frames, atol 0.01
    pcm, ref, atol = golden()
    got = o.log_mel(pcm, ref.shape[0])
    assert got.shape == (80, 3000)
    assert np.max(np.abs(got[:, :ref.shape[1]] - ref)) <= atol
    # the restatement is far inside the reference tolerance
    assert np.max(np.abs(got[:, :ref.shape[1]] - ref)) <= 1e-4


def test_log_mel_unit_cases():
    # crates/vokra-models/src/whisper/mel.rs tests: silence, a 440 Hz tone, empty and oversized input
    s = o.log_mel(np.zeros(16000, np.float32), 80)
    assert s.shape == (80, 3000) and np.isfinite(s).all()
    assert np.all(s == np.float32(-1.5))  # log10(1e-10) = -10 -> (-10 + 4) / 4
    tone = np.sin(2 * np.pi * 440.0 * np.arange(16000) / 16000.0).astype(np.float32)
    t = o.log_mel(tone, 80)
    assert np.isfinite(t).all() and t.min() > -2.0 and t.max() < 2.0
    e = o.log_mel(np.zeros(0, np.float32), 80)
    assert e.shape == (80, 3000) and np.isfinite(e).all()
    big = o.log_mel(np.full(480000 + 5000, 0.1, np.float32), 80)
    assert np.isfinite(big).all()
    # trimming: samples past 30 s do not change the features
    pcm, _, _ = golden()
    longer = np.concatenate([pcm, np.ones(3000, np.float32)])
    assert np.array_equal(o.log_mel(longer, 80), o.log_mel(pcm, 80))


def test_mel_filterbank_cases():
    # crates/vokra-ops/src/mel.rs tests: shape, non-negativity, support of every filter
    fb = o.mel_filterbank(80)
    assert fb.shape == (80, 201)
    assert np.all(fb >= 0.0)
    assert np.all(fb.max(axis=1) > 0.0)
    fb128 = o.mel_filterbank(128)
    assert fb128.shape == (128, 201) and np.all(fb128.max(axis=1) > 0.0)
    # apply_projects_frames: a flat spectrum projects to non-negative energies
    assert np.all(fb @ np.ones(201, np.float32) >= 0.0)


def test_hann_periodic():
    # crates/vokra-ops/src/window.rs tests: periodic Hann of length 4 = [0, 0.5, 1, 0.5]
    assert np.allclose(o.hann_periodic(4), [0.0, 0.5, 1.0, 0.5], atol=1e-7)
    w = o.hann_periodic(400)
    assert w[0] == 0.0 and abs(w[200] - 1.0) < 1e-7
