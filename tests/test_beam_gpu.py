"""Beam search on the device decode session (SessionBeamScorer: beams are
decode streams stepped together, branched with vkb_session_copy_stream)
against the same search run on the oracle decoder."""
import copy

import numpy as np
import pytest

from oracle import whisper_ref
from vokra_b200 import synth
from vokra_b200.beam import BeamSearchConfig, SessionBeamScorer, beam_search, log_softmax

pytestmark = pytest.mark.gpu


class OracleScorer:
    def __init__(self, dec, vocab):
        self.root, self.vocab_size, self.cache = dec, vocab, {}

    def logprobs_batch(self, prefixes):
        out, new = [], {}
        for p in prefixes:
            if not self.cache:
                d = self.root
                row = d.step(list(p))[-1]
            else:
                d = copy.copy(self.cache[tuple(p[:-1])])
                d.k, d.v = list(d.k), list(d.v)
                row = d.step([p[-1]])[-1]
            new[tuple(p)] = d
            out.append(log_softmax(row))
        self.cache = new
        return out


def test_beam_search_matches_oracle(ctx, tmp_path):
    import torch
    from vokra_b200 import whisper
    arch = synth.WHISPER_TINY_TEST
    path = str(tmp_path / "beam.gguf")
    synth.write_synthetic_whisper(path, arch, synth.Q8_0, seed=3)
    rng = np.random.default_rng(11)
    logmel = rng.uniform(-1.0, 1.5, (1, arch.n_mels, 2 * arch.n_audio_ctx)).astype(np.float32)
    W = 3
    model = whisper.WhisperModel(ctx, path)
    sess = whisper.Session(model, max_streams=2 * W + 1, max_clips=1, cross_kv_q8=True)
    sess.encode(torch.from_numpy(logmel).cuda(), [6])
    cfg = BeamSearchConfig.new(W, 8).with_(n_best=3, early_stopping=False)
    prefix = list(arch.start_ids)
    dev = beam_search(SessionBeamScorer(sess, 6, list(range(2 * W)), W), prefix, arch.eot, cfg)
    ref = whisper_ref.RefWhisper(path)
    dec = ref.decoder(ref.encode(logmel[0]), kv_mode="q8", cross_mode="q8")
    orc = beam_search(OracleScorer(dec, arch.n_vocab), prefix, arch.eot, cfg)
    assert len(dev) == len(orc) > 0
    # the device logits are within 1e-2 of the oracle's: same hypotheses, scores within that budget
    for a, b in zip(dev, orc):
        assert a.tokens == b.tokens
        assert abs(a.score - b.score) <= 1e-2 * len(a.tokens)
    # a second search on the same session reuses the slots (pages released and re-acquired)
    again = beam_search(SessionBeamScorer(sess, 6, list(range(2 * W)), W), prefix, arch.eot, cfg)
    assert [h.tokens for h in again] == [h.tokens for h in dev]
    sess.close()
