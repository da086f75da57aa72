"""End-to-end Whisper forward on the B200 against the oracle forward
(route R1 with the self-attention cache in Q8_0 pages and the cross K/V in Q8_0)."""
import os

import numpy as np
import pytest

from oracle import whisper_ref
from vokra_b200 import _lib, synth

pytestmark = pytest.mark.gpu


def _rel_rms(a, b):
    return float(np.sqrt(np.mean((a - b) ** 2)) / (np.sqrt(np.mean(b ** 2)) + 1e-30))


@pytest.fixture(scope="module", params=[synth.Q8_0, synth.Q4_0, synth.Q4_K, synth.Q5_K, synth.Q6_K, synth.F32])
def tiny(request, tmp_path_factory):
    path = str(tmp_path_factory.mktemp("w") / f"tiny_{request.param}.gguf")
    synth.write_synthetic_whisper(path, synth.WHISPER_TINY_TEST, request.param, seed=1)
    return path


def _run(ctx, path, n_streams=3, n_steps=6, cross_q8=True, arch=synth.WHISPER_TINY_TEST, seed=2, self_kv="q8"):
    import torch
    from vokra_b200 import whisper
    rng = np.random.default_rng(seed)
    a = arch
    logmel = rng.uniform(-1.0, 1.5, (n_streams, a.n_mels, 2 * a.n_audio_ctx)).astype(np.float32)
    model = whisper.WhisperModel(ctx, path)
    from vokra_b200 import _lib
    modes = {"q8": _lib.SELF_KV_Q8_0, "f32": _lib.SELF_KV_F32, "q4": _lib.SELF_KV_Q4_0, "q5": _lib.SELF_KV_Q5_0}
    sess = whisper.Session(model, max_streams=n_streams, max_clips=n_streams, cross_kv_q8=cross_q8,
                           self_kv=modes[self_kv])
    sess.encode(torch.from_numpy(logmel).cuda(), list(range(n_streams)))
    enc = sess.encoder_output(n_streams)
    ref = whisper_ref.RefWhisper(path)
    ref_enc = [ref.encode(logmel[i]) for i in range(n_streams)]
    decs = [ref.decoder(ref_enc[i], kv_mode=self_kv, cross_mode="q8" if cross_q8 else "f16") for i in range(n_streams)]
    toks = rng.integers(0, a.n_vocab, (n_streams, n_steps)).tolist()
    V = a.n_vocab
    results = []
    # prefix step: the start ids for every stream in one step
    prefix = list(a.start_ids)
    streams = [s for s in range(n_streams) for _ in prefix]
    positions = [p for _ in range(n_streams) for p in range(len(prefix))]
    tokens = prefix * n_streams
    out = torch.zeros((len(tokens), V), dtype=torch.float32, device="cuda:0")
    sess.step(streams, positions, tokens, logits_dev=out)
    torch.cuda.synchronize()
    got = out.cpu().numpy().reshape(n_streams, len(prefix), V)
    for s in range(n_streams):
        results.append((got[s], decs[s].step(prefix)))
    pos = len(prefix)
    for t in range(n_steps):
        out = torch.zeros((n_streams, V), dtype=torch.float32, device="cuda:0")
        sess.step(list(range(n_streams)), [pos] * n_streams, [toks[s][t] for s in range(n_streams)], logits_dev=out)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        for s in range(n_streams):
            results.append((got[s:s + 1], decs[s].step([toks[s][t]])))
        pos += 1
    return enc, np.stack(ref_enc), results


def test_tiny_whisper_matches_oracle(ctx, tiny):
    enc, ref_enc, results = _run(ctx, tiny)
    assert _rel_rms(enc, ref_enc) <= 2e-3
    worst_abs, worst_rms = 0.0, 0.0
    mism = 0
    for got, ref in results:
        worst_abs = max(worst_abs, float(np.max(np.abs(got - ref))))
        worst_rms = max(worst_rms, _rel_rms(got, ref))
        for r in range(ref.shape[0]):
            top2 = np.sort(ref[r])[-2:]
            if top2[1] - top2[0] > 1e-3 and int(np.argmax(got[r])) != int(np.argmax(ref[r])):
                mism += 1
    print(f"logits max-abs {worst_abs:.3e} rel-rms {worst_rms:.3e}")
    assert worst_abs <= 1e-2
    assert worst_rms <= 1e-3
    assert mism == 0


@pytest.mark.parametrize("self_kv", ["f32", "q4", "q5"])
def test_tiny_whisper_self_kv_modes(ctx, tiny, self_kv):
    """The session with f32, Q4_0 or Q5_0 self-attention pages against the
    oracle keeping the same cache (prefix steps and decode steps take the
    unfused append + paged attention kernels for these modes).

    The packs themselves are bit-exact (test_kv_gpu); end to end, the device's
    K/V rows differ from the oracle's in their last bits (split-precision
    GEMMs), and a 4- or 5-bit pack turns a value that sits on a rounding
    boundary into a whole quantum (1/7 or 1/15 of the block's amax). For
    those two modes the bars are 1e-2 relative RMS and 5e-2 max-abs (a wrong
    page or a wrong block decode moves logits by O(1)); f32 pages keep the
    1e-3 / 1e-2 budget and identical argmax ids."""
    enc, ref_enc, results = _run(ctx, tiny, n_streams=2, n_steps=5, self_kv=self_kv)
    rms_tol, abs_tol = (1e-3, 1e-2) if self_kv == "f32" else (1e-2, 5e-2)
    for got, ref in results:
        assert np.max(np.abs(got - ref)) <= abs_tol
        assert _rel_rms(got, ref) <= rms_tol
        if self_kv == "f32":
            assert np.array_equal(np.argmax(got, axis=-1), np.argmax(ref, axis=-1))


def test_tiny_whisper_f16_cross_store(ctx, tiny):
    enc, ref_enc, results = _run(ctx, tiny, n_streams=2, n_steps=3, cross_q8=False)
    for got, ref in results:
        assert np.max(np.abs(got - ref)) <= 1e-2
        assert _rel_rms(got, ref) <= 1e-3


def _decode_fixed_buffer(ctx, path, n_streams, n_steps, graphs, seed=7):
    """Prefix + n_steps decode steps writing into one logits buffer, so that
    every decode step after the second replays the recorded step."""
    import torch
    from vokra_b200 import whisper
    a = synth.WHISPER_TINY_TEST
    rng = np.random.default_rng(seed)
    logmel = rng.uniform(-1.0, 1.5, (n_streams, a.n_mels, 2 * a.n_audio_ctx)).astype(np.float32)
    old = os.environ.get("VKB_STEP_GRAPHS")
    os.environ["VKB_STEP_GRAPHS"] = "1" if graphs else "0"
    try:
        model = whisper.WhisperModel(ctx, path)
        sess = whisper.Session(model, max_streams=n_streams, max_clips=n_streams)
    finally:
        if old is None:
            del os.environ["VKB_STEP_GRAPHS"]
        else:
            os.environ["VKB_STEP_GRAPHS"] = old
    sess.encode(torch.from_numpy(logmel).cuda(), list(range(n_streams)))
    prefix = list(a.start_ids)
    sess.step([s for s in range(n_streams) for _ in prefix], [p for _ in range(n_streams) for p in range(len(prefix))],
              prefix * n_streams)
    out = torch.zeros((n_streams, a.n_vocab), dtype=torch.float32, device="cuda:0")
    toks = rng.integers(0, a.n_vocab, (n_steps, n_streams))
    got = []
    for t in range(n_steps):
        sess.step(list(range(n_streams)), [len(prefix) + t] * n_streams, toks[t].tolist(), logits_dev=out)
        got.append(out.cpu().numpy().copy())
    sess.close()
    model.close()
    return np.stack(got)


def test_recorded_decode_step_replays_bit_exact(ctx, tiny):
    """A decode step recorded as a CUDA graph and replayed gives the same
    logits, bit for bit, as the same steps launched one kernel at a time
    (the replays read the new tokens, positions and page-table entries)."""
    eager = _decode_fixed_buffer(ctx, tiny, n_streams=3, n_steps=20, graphs=False)
    replay = _decode_fixed_buffer(ctx, tiny, n_streams=3, n_steps=20, graphs=True)
    assert np.isfinite(eager).all()
    assert np.array_equal(eager, replay)


def test_whisper_full_window_matches_oracle(ctx, tmp_path):
    """A one-layer model at Whisper's real window (1500 encoder frames) with 8
    heads: the tensor-core encoder attention over 12 key tiles with a ragged
    last tile, the streaming cross-attention over 1500 keys, and the fused
    decode self-attention over two head groups, against the oracle forward."""
    arch = synth.WhisperArch(80, 1500, 512, 8, 1, 64, 8, 1, 1000, 2048, 999, (1, 2, 3, 4))
    path = str(tmp_path / "window.gguf")
    synth.write_synthetic_whisper(path, arch, synth.Q8_0, seed=4)
    enc, ref_enc, results = _run(ctx, path, n_streams=2, n_steps=12, arch=arch, seed=9)
    assert _rel_rms(enc, ref_enc) <= 2e-3
    for got, ref in results:
        assert np.max(np.abs(got - ref)) <= 1e-2
        assert _rel_rms(got, ref) <= 1e-3


def test_whisper_full_window_persistent_gemm(ctx, tmp_path, monkeypatch):
    """The same window with every unsplit-K GEMM on the persistent kernel
    (conv stem GELU to f16 hi+lo planes, scaled QKV to f16, residual f32,
    cross K/V f32), against the oracle forward."""
    monkeypatch.setenv("VKB_GEMM_PERSIST", "force")
    arch = synth.WhisperArch(80, 1500, 512, 8, 1, 64, 8, 1, 1000, 2048, 999, (1, 2, 3, 4))
    path = str(tmp_path / "window_p.gguf")
    synth.write_synthetic_whisper(path, arch, synth.Q8_0, seed=4)
    enc, ref_enc, results = _run(ctx, path, n_streams=2, n_steps=4, arch=arch, seed=9)
    assert _rel_rms(enc, ref_enc) <= 2e-3
    for got, ref in results:
        assert np.max(np.abs(got - ref)) <= 1e-2
        assert _rel_rms(got, ref) <= 1e-3


def _cross_store(sess, layer, rows, d):
    """Host copies of a session's Q8_0 cross K/V store of one decoder layer."""
    import ctypes as C
    from cuda.bindings import runtime as rt
    from vokra_b200 import _lib
    ptr = [C.c_void_p() for _ in range(4)]
    _lib.check(_lib.load().vkb_session_cross_kv(sess.h, layer, *[C.byref(p) for p in ptr]))
    out = []
    for p, n in zip(ptr, (rows * d, rows * d, rows * d // 16, rows * d // 16)):
        h = np.empty(n, np.uint8)
        err, = rt.cudaMemcpy(h.ctypes.data, p.value, n, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)
        assert int(err) == 0
        out.append(h)
    return out


@pytest.mark.parametrize("prec", ["split", "encoder_f16"])
def test_fused_cross_kv_q8_bytes(ctx, tmp_path, monkeypatch, prec):
    """The cross K/V projection with Q8_0 packing in the persistent GEMM's
    epilogue writes the same store bytes as the f32 projection followed by
    the quantize kernel (BlockQ8_0::pack), clips remapped to stream slots.
    Split precision: the TMEM-operand kernel; encoder-f16: the shared-operand
    kernel on CTA pairs (weights as a once-per-call f16 plane)."""
    import torch
    from vokra_b200 import whisper
    monkeypatch.setenv("VKB_GEMM_PERSIST", "force")
    if prec == "encoder_f16":
        _lib.check(_lib.load().vkb_context_set_precision(ctx.h, _lib.PREC_ENCODER_F16))
    try:
        _fused_cross_kv_q8_bytes(ctx, tmp_path, monkeypatch)
    finally:
        _lib.check(_lib.load().vkb_context_set_precision(ctx.h, _lib.PREC_SPLIT))


def _fused_cross_kv_q8_bytes(ctx, tmp_path, monkeypatch):
    import torch
    from vokra_b200 import whisper
    arch = synth.WhisperArch(80, 1500, 512, 8, 1, 64, 8, 2, 1000, 2048, 999, (1, 2, 3, 4))
    path = str(tmp_path / "xq.gguf")
    synth.write_synthetic_whisper(path, arch, synth.Q4_0, seed=6)
    rng = np.random.default_rng(3)
    logmel = torch.from_numpy(rng.uniform(-1.0, 1.5, (2, 80, 3000)).astype(np.float32)).cuda()
    model = whisper.WhisperModel(ctx, path)
    stores = []
    for fused in ("1", "0"):
        monkeypatch.setenv("VKB_FUSED_CROSS_Q8", fused)
        sess = whisper.Session(model, max_streams=3, max_clips=2, cross_kv_q8=True)
        sess.encode(logmel, [2, 0])  # clips land in stream slots 2 and 0
        torch.cuda.synchronize()
        stores.append([_cross_store(sess, layer, 3 * 1500, 512) for layer in range(2)])
        sess.close()
    rows = np.r_[0:1500, 3000:4500]  # the written slots
    for layer in range(2):
        for a, b, per_row in zip(stores[0][layer], stores[1][layer], (512, 512, 32, 32)):
            a2, b2 = a.reshape(-1, per_row)[rows], b.reshape(-1, per_row)[rows]
            assert np.array_equal(a2, b2), layer
