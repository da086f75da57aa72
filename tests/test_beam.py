"""beam_search (vokra_b200/beam.py) against the reference's own beam-search unit
cases (crates/vokra-core/src/decode/beam_search.rs:520-800), restated with the
same mock scorer: vocab {0=start, 1='a', 2='b', 3=eot}, a fixed transition table."""
import numpy as np
import pytest

from vokra_b200.beam import BeamSearchConfig, beam_search, ngram_block_mask, top_k

EOT = 3


class Table:
    def __init__(self, table):
        self.table = [np.array(r, np.float32) for r in table]
        self.vocab_size = len(table[0])

    def logprobs_batch(self, prefixes):
        return [self.table[p[-1]] for p in prefixes]


def scorer():
    ln = lambda p: np.log(np.float32(p))
    return Table([[ln(0.001), ln(0.6), ln(0.399), ln(0.001)],
                  [ln(0.001), ln(0.001), ln(0.098), ln(0.9)],
                  [ln(0.001), ln(0.02), ln(0.001), ln(0.95)],
                  [ln(0.001), ln(0.001), ln(0.001), ln(0.997)]])


class Const:
    def __init__(self, row):
        self.row = np.array(row, np.float32)
        self.vocab_size = len(row)

    def logprobs_batch(self, prefixes):
        return [self.row for _ in prefixes]


def test_width_one_is_greedy():
    h = beam_search(scorer(), [0], EOT, BeamSearchConfig.greedy(8))
    assert len(h) == 1 and h[0].tokens == [0, 1, 3]


def test_wider_beam_does_not_reduce_best_score():
    g = beam_search(scorer(), [0], EOT, BeamSearchConfig.greedy(8))
    b = beam_search(scorer(), [0], EOT, BeamSearchConfig.new(3, 8))
    assert b[0].score >= g[0].score - 1e-5


def test_n_best_is_sorted_unique_and_capped():
    h = beam_search(scorer(), [0], EOT, BeamSearchConfig.new(3, 8).with_(n_best=3))
    assert len(h) <= 3
    assert all(a.normalized_score >= b.normalized_score for a, b in zip(h, h[1:]))
    assert len({tuple(x.tokens) for x in h}) == len(h)


def test_early_stopping_keeps_the_same_best():
    on = BeamSearchConfig.new(3, 8)
    a = beam_search(scorer(), [0], EOT, on)
    b = beam_search(scorer(), [0], EOT, on.with_(early_stopping=False))
    assert a[0].tokens == b[0].tokens


def test_length_normalization_zero_is_raw_score():
    h = beam_search(scorer(), [0], EOT, BeamSearchConfig.new(3, 8).with_(length_normalization=0.0, n_best=3))
    assert all(abs(x.normalized_score - x.score) < 1e-6 for x in h)


def test_rejections_and_edges():
    with pytest.raises(ValueError):
        beam_search(scorer(), [], EOT, BeamSearchConfig.greedy(4))
    with pytest.raises(ValueError):
        beam_search(scorer(), [0], EOT, BeamSearchConfig.greedy(4).with_(beam_width=0))
    assert beam_search(scorer(), [0], EOT, BeamSearchConfig.new(10, 6))  # wider than the vocabulary
    assert beam_search(Const([-np.inf, 0.0]), [0], 1, BeamSearchConfig.greedy(5))[0].tokens == [0, 1]
    # never-finishing model: the best unfinished beam is returned
    h = beam_search(Const([-np.inf, 0.0]), [7], 0, BeamSearchConfig.greedy(3))
    assert h[0].tokens == [7, 1, 1, 1]


def test_helpers():
    assert top_k([1.0, 3.0, 3.0, 2.0], 3) == [(1, 3.0), (2, 3.0), (3, 2.0)]
    m = ngram_block_mask([5, 6, 5], 2, 8)  # bigram (5, 6) seen: after 5, 6 is blocked
    assert m[6] and m.sum() == 1
    assert not ngram_block_mask([5], 3, 8).any()


def _row(hist, vocab):
    # a deterministic log-probability row that depends on the whole history
    rng = np.random.default_rng(abs(hash(tuple(hist))) % (2 ** 32))
    x = rng.standard_normal(vocab).astype(np.float32) * 2.0
    return x


class HistoryScorer:
    def __init__(self, vocab):
        self.vocab_size = vocab

    def logprobs_batch(self, prefixes):
        from vokra_b200.beam import log_softmax
        return [log_softmax(_row(list(p), self.vocab_size)) for p in prefixes]


class FakeBeamSession:
    """Keeps each stream's token history the way the device KV would: step
    appends at the given positions, copy_stream copies the first n positions."""

    class model:
        class dims:
            n_vocab = 11

    def __init__(self):
        self.hist = {}

    def copy_stream(self, src, dst, n, cross):
        self.hist[dst] = list(self.hist.get(src, []))[:n]

    def release(self, slot):
        self.hist.pop(slot, None)

    def step(self, streams, positions, tokens, logits_dev=None):
        rows = {}
        for i, (s, p, t) in enumerate(zip(streams, positions, tokens)):
            h = self.hist.setdefault(s, [])
            assert p == len(h), (s, p, len(h))
            h.append(int(t))
            rows[i] = _row(h, 11)
        for i, r in rows.items():
            logits_dev[i] = __import__("torch").from_numpy(r)


def test_session_scorer_banks_match_history_scorer():
    from vokra_b200.beam import SessionBeamScorer
    cfg = BeamSearchConfig.new(3, 7).with_(n_best=3, early_stopping=False)
    fake = FakeBeamSession()
    fake.hist[9] = []
    sc = SessionBeamScorer(fake, 9, list(range(6)), 3, copy_stream=fake.copy_stream, device="cpu")
    got = beam_search(sc, [1, 2], 10, cfg)
    want = beam_search(HistoryScorer(11), [1, 2], 10, cfg)
    assert [h.tokens for h in got] == [h.tokens for h in want]
    assert all(abs(a.score - b.score) < 1e-6 for a, b in zip(got, want))


def test_ngram_block_mask_reference_cases():
    # crates/vokra-models/src/voxtral/beam_search.rs:889-930 (the same semantics as decode/beam_search.rs:442)
    for n in (0, 1):
        assert not ngram_block_mask([1, 2, 3, 1, 2], n, 5).any()
    m = ngram_block_mask([1, 2, 3, 1], 2, 5)
    assert m[2] and not m[3]
    m = ngram_block_mask([1, 2, 3, 1, 2], 3, 5)
    assert m[3] and not m[4]
    assert not ngram_block_mask([1], 3, 5).any()


def test_no_repeat_ngram_blocks_repeats():
    # a scorer that always prefers token 1 then 2: without blocking the beam loops 1,2,1,2,...
    row = np.log(np.array([0.01, 0.6, 0.38, 0.01], np.float32))
    h = beam_search(Const(row), [0], 3, BeamSearchConfig.greedy(8).with_(no_repeat_ngram_size=2))
    toks = h[0].tokens
    bigrams = list(zip(toks, toks[1:]))
    assert len(bigrams) == len(set(bigrams))


def test_session_scorer_long_prefix():
    """A prompt longer than the scorer's initial logits buffer (a Whisper prompt
    of previous text can be 224 tokens) is scored without writing past it."""
    from vokra_b200.beam import SessionBeamScorer
    cfg = BeamSearchConfig.new(2, 3).with_(n_best=2, early_stopping=False)
    prefix = [int(t) for t in np.random.default_rng(1).integers(0, 10, 150)]
    fake = FakeBeamSession()
    fake.hist[9] = []
    sc = SessionBeamScorer(fake, 9, list(range(4)), 2, copy_stream=fake.copy_stream, device="cpu")
    got = beam_search(sc, prefix, 10, cfg)
    want = beam_search(HistoryScorer(11), prefix, 10, cfg)
    assert [h.tokens for h in got] == [h.tokens for h in want]
