"""Host logic of the continuous batcher (vokra_b200/batching.py) on CPU, against
a fake session that checks every step the way the device session does
(vkb_session_step: each stream's tokens at consecutive positions, continuing
where the stream stopped) and answers each stream with a token derived from
its own history, so any mix-up between streams shows in the ids."""
import numpy as np
import torch

from vokra_b200 import batching, ops


class Dims:
    n_audio_ctx = 1500


class Model:
    dims = Dims()


class FakeSession:
    def __init__(self, n_slots, max_step):
        self.model = Model()
        self.hist = {}
        self.encoded = {}
        self.max_step, self.max_active, self.steps = max_step, 0, 0

    def encode(self, lm, slots):
        for s in slots:
            assert s not in self.hist, "encode into a busy slot"
            self.encoded[s] = True

    def step(self, streams, positions, tokens, ids_dev=None):
        assert len(streams) <= self.max_step
        self.steps += 1
        self.max_active = max(self.max_active, len(set(streams)))
        out = []
        for s, p, t in zip(streams, positions, tokens):
            h = self.hist.setdefault(s, [])
            assert self.encoded.get(s), "step on a stream that was never encoded"
            assert p == len(h), f"stream {s}: position {p}, expected {len(h)}"
            h.append(int(t))
            out.append((sum(h) * 31 + len(h)) % 997)
        ids_dev[:len(out)] = torch.tensor(out, dtype=torch.int32)

    def step_feed(self, streams, positions, tokens, feed_rows, feed_ids, ids_dev=None):
        toks = [int(feed_ids[f]) if f >= 0 else t for t, f in zip(tokens, feed_rows)]
        self.step(streams, positions, toks, ids_dev=ids_dev)

    def release(self, slot):
        del self.hist[slot]
        self.encoded.pop(slot)


def expected_ids(prefix, n):
    h, ids = list(prefix), []
    nxt = (sum(h) * 31 + len(h)) % 997
    for _ in range(n):
        ids.append(nxt)
        h.append(nxt)
        nxt = (sum(h) * 31 + len(h)) % 997
    return ids


def test_batcher_schedules_streams(monkeypatch):
    monkeypatch.setattr(ops, "log_mel", lambda ctx, pcm, n_mels, out=None, lengths=None: out)
    rng = np.random.default_rng(0)
    news = [int(x) for x in rng.integers(1, 12, 23)]
    utts = [batching.Utterance(i % 3, 16000, n) for i, n in enumerate(news)]
    prefix = [5, 6, 7, 8]
    sess = FakeSession(5, max_step=40)
    b = batching.ContinuousBatcher(None, sess, 5, 2, prefix, 80, device="cpu")
    b.run(utts, torch.zeros((3, 16000)))
    assert b.tokens == sum(news)
    assert sess.max_active <= 5
    assert not sess.hist  # every slot released
    for u in utts:
        assert u.ids == expected_ids(prefix, u.n_new_tokens)


def test_batcher_stops_at_eot(monkeypatch):
    monkeypatch.setattr(ops, "log_mel", lambda ctx, pcm, n_mels, out=None, lengths=None: out)
    prefix = [5, 6, 7, 8]
    full = expected_ids(prefix, 30)
    eot = full[3]
    sess = FakeSession(2, max_step=16)
    u = batching.Utterance(0, 100, 30)
    b = batching.ContinuousBatcher(None, sess, 2, 1, prefix, 80, eot=eot, stop_at_eot=True, device="cpu")
    b.run([u], torch.zeros((1, 100)))
    assert u.ids == full[:full.index(eot) + 1]


def test_batcher_rejects_encode_batch_above_slots():
    """An encode batch larger than the slot count could never be admitted (the
    loop would spin with nothing active), so the constructor refuses it."""
    import pytest
    sess = FakeSession(2, max_step=16)
    for bad in (0, 3):
        with pytest.raises(ValueError):
            batching.ContinuousBatcher(None, sess, 2, bad, [5], 80, device="cpu")
