"""Continuous batching (vokra_b200/batching.py): every utterance's greedy ids
under batching, with streams joining and leaving between steps, equal those of
the same utterance decoded alone in the same session kernels."""
import numpy as np
import pytest

from vokra_b200 import synth

pytestmark = pytest.mark.gpu


def test_continuous_batching_matches_one_at_a_time(ctx, tmp_path):
    import torch
    from vokra_b200 import whisper
    from vokra_b200.batching import ContinuousBatcher, Utterance
    arch = synth.WhisperArch(80, 1500, 512, 8, 1, 64, 8, 1, 1000, 2048, 999, (1, 2, 3, 4))
    path = str(tmp_path / "cb.gguf")
    synth.write_synthetic_whisper(path, arch, synth.Q8_0, seed=8)
    rng = np.random.default_rng(4)
    pcm = torch.from_numpy((0.1 * rng.standard_normal((6, 480000))).astype(np.float32)).cuda()
    lengths = [int(x) for x in rng.integers(1000, 480000, 9)]
    news = [int(x) for x in rng.integers(2, 9, 9)]
    model = whisper.WhisperModel(ctx, path)

    def run(n_slots, encode_batch):
        sess = whisper.Session(model, max_streams=n_slots, max_step_tokens=8 * n_slots, max_clips=encode_batch)
        utts = [Utterance(i % 6, lengths[i], news[i]) for i in range(9)]
        b = ContinuousBatcher(ctx, sess, n_slots, encode_batch, arch.start_ids, arch.n_mels)
        b.run(utts, pcm)
        sess.close()
        return [u.ids for u in utts], b

    batched, b = run(4, 2)
    alone, _ = run(1, 1)
    assert b.tokens == sum(news)
    assert all(len(i) == n for i, n in zip(batched, news))
    assert batched == alone
