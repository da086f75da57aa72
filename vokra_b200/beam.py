"""Beam search over the device decode session.

`beam_search` restates the reference's search loop
(crates/vokra-core/src/decode/beam_search.rs:246-420): every active beam is
expanded by its top `beam_width` log-probabilities (after optional no-repeat
n-gram masking), the best `beam_width` candidates overall survive, candidates
ending in `eot` complete, and the result is ranked by `score / len^alpha`,
de-duplicated and cut to `n_best`. It asks its scorer for log-probabilities
through `logprobs_batch(prefixes)`, the reference's BeamScorer interface
(beam_search.rs:91-123), so one call scores every active beam.

`SessionBeamScorer` is the B200 scorer: the beams of one clip are decode
streams of a `whisper.Session`, scored in ONE batched session step per search
step. Beams live in two banks of stream slots; each call writes the new
beams into the bank the previous call did not use, branching each child from
its parent with `vkb_session_copy_stream` (a device copy of the parent's
self-attention pages), where the reference deep-copies its host cache
(whisper/decoder.rs:343-368). The clip's cross-attention rows are copied to
every slot once, at construction. Log-probabilities are the reference's
log-softmax of the step's f32 logits (whisper/beam_glue.rs:204-207).
"""
from __future__ import annotations

from dataclasses import dataclass, replace

import numpy as np

from . import _lib


@dataclass
class BeamSearchConfig:
    """BeamSearchConfig (beam_search.rs:137-214) without the LM-fusion and word-timestamp options."""
    beam_width: int
    max_new_tokens: int
    length_normalization: float = 1.0
    early_stopping: bool = True
    n_best: int = 1
    no_repeat_ngram_size: int = 0

    @staticmethod
    def greedy(max_new_tokens: int) -> "BeamSearchConfig":
        return BeamSearchConfig(1, max_new_tokens, length_normalization=0.0)

    @staticmethod
    def new(beam_width: int, max_new_tokens: int) -> "BeamSearchConfig":
        return BeamSearchConfig(beam_width, max_new_tokens)

    def with_(self, **kw) -> "BeamSearchConfig":
        return replace(self, **kw)


@dataclass
class BeamHypothesis:
    tokens: list
    score: float             # cumulative log-probability of the generated tokens (f32 sums)
    normalized_score: float  # score / len^alpha


def log_softmax(logits) -> np.ndarray:
    """f32 log-softmax of one logits row: x - max - log(sum(exp(x - max)))."""
    x = np.asarray(logits, dtype=np.float32)
    m = np.max(x)
    return (x - m - np.log(np.sum(np.exp(x - m), dtype=np.float32))).astype(np.float32)


def top_k(values, k: int):
    """The k largest (index, value) pairs, value-descending; ties keep the lower
    index first, as the reference's single-pass insertion does (beam_search.rs:478-502)."""
    v = np.asarray(values, dtype=np.float32)
    order = np.lexsort((np.arange(v.size), -v))[:k]
    return [(int(i), np.float32(v[i])) for i in order]


def ngram_block_mask(tokens, n: int, vocab: int) -> np.ndarray:
    """Tokens that would complete an n-gram already present in `tokens` (beam_search.rs:442-476)."""
    mask = np.zeros(vocab, dtype=bool)
    if n <= 1 or len(tokens) < n:
        return mask
    suffix = list(tokens[len(tokens) - (n - 1):])
    for i in range(len(tokens) - n + 1):
        if list(tokens[i:i + n - 1]) == suffix:
            f = tokens[i + n - 1]
            if f < vocab:
                mask[f] = True
    return mask


def beam_search(scorer, prefix, eot: int, config: BeamSearchConfig) -> list:
    """Beam search from `prefix` until `eot`, every beam finished, or max_new_tokens."""
    if len(prefix) == 0:
        raise ValueError("beam_search: prefix must not be empty")
    if config.beam_width <= 0 or config.n_best <= 0:
        raise ValueError("beam_search: beam_width and n_best must be >= 1")
    prefix_len = len(prefix)
    active = [(list(prefix), np.float32(0.0))]
    completed = []
    for _ in range(config.max_new_tokens):
        if not active:
            break
        if config.early_stopping and len(completed) >= config.beam_width:
            break
        all_lp = scorer.logprobs_batch([h[0] for h in active])
        vocab = scorer.vocab_size
        if len(all_lp) != len(active):
            raise ValueError("beam_search: logprobs_batch returned the wrong number of rows")
        cands = []
        for (toks, score), lp in zip(active, all_lp):
            lp = np.array(lp, dtype=np.float32)
            if lp.size != vocab:
                raise ValueError("beam_search: scorer returned a row of the wrong size")
            if config.no_repeat_ngram_size > 0:
                lp[ngram_block_mask(toks, config.no_repeat_ngram_size, vocab)] = -np.inf
            for tok, delta in top_k(lp, config.beam_width):
                if not np.isfinite(delta):
                    continue
                cands.append((toks + [tok], np.float32(score + delta)))
        # stable sort by score, descending (sort_by_score_desc)
        cands.sort(key=lambda h: -float(h[1]))
        cands = cands[:config.beam_width]
        active = []
        for c in cands:
            (completed if c[0][-1] == eot else active).append(c)
    finals = completed if completed else active
    alpha = np.float32(config.length_normalization)
    out = []
    for toks, score in finals:
        gen = np.float32(max(len(toks) - prefix_len, 1))
        out.append(BeamHypothesis(toks, float(score), float(np.float32(score / np.float32(gen ** alpha)))))
    out.sort(key=lambda h: -h.normalized_score)
    seen, uniq = [], []
    for h in out:
        if h.tokens not in seen:
            seen.append(h.tokens)
            uniq.append(h)
    return uniq[:config.n_best]


class SessionBeamScorer:
    """Scores the beams of one encoded clip on the device (see the module docstring).

    session: a whisper.Session; clip_stream: the stream slot the clip was encoded
    into; slots: 2 * beam_width free stream slots (may include clip_stream).
    copy_stream(src, dst, n_pos, copy_cross) defaults to vkb_session_copy_stream;
    device is where the step's logits are written."""

    def __init__(self, session, clip_stream: int, slots, beam_width: int, copy_stream=None, device: str = "cuda"):
        import torch
        if len(slots) < 2 * beam_width:
            raise ValueError("SessionBeamScorer: needs 2 * beam_width stream slots")
        self.s, self.W = session, beam_width
        self.slots = list(slots[:2 * beam_width])
        self.vocab_size = session.model.dims.n_vocab
        if copy_stream is None:
            L = _lib.load()
            copy_stream = lambda src, dst, n, cross: _lib.check(L.vkb_session_copy_stream(session.h, src, dst, n, cross))
        self._copy, self._device = copy_stream, device
        for slot in self.slots:
            if slot != clip_stream:
                self._copy(clip_stream, slot, 0, 1)
        self.calls = 0
        self.cache = {}  # token tuple -> slot, for the beams of the last call
        self._logits = torch.empty((max(4 * beam_width, 64), self.vocab_size), dtype=torch.float32, device=device)

    def logprobs_batch(self, prefixes):
        import torch
        bank = self.slots[(self.calls % 2) * self.W:(self.calls % 2 + 1) * self.W]
        if len(prefixes) > self.W:
            raise ValueError("SessionBeamScorer: more beams than beam_width")
        new_cache = {}
        if self.calls == 0 and len(prefixes) == 1 and tuple(prefixes[0]) not in self.cache:
            toks = list(prefixes[0])
            slot = bank[0]
            self.s.release(slot)
            n = len(toks)
            if n > self._logits.shape[0]:
                # the prefix step writes one logits row per prefix token
                self._logits = torch.empty((n, self.vocab_size), dtype=torch.float32, device=self._device)
            self.s.step([slot] * n, list(range(n)), toks, logits_dev=self._logits)
            if self._device != "cpu":
                torch.cuda.synchronize()
            rows = [self._logits[n - 1].cpu().numpy()]
            new_cache[tuple(toks)] = slot
        else:
            streams, pos, last = [], [], []
            for i, toks in enumerate(prefixes):
                parent = tuple(toks[:-1])
                if parent not in self.cache:
                    raise ValueError("SessionBeamScorer: a prefix does not extend a beam of the previous call")
                self._copy(self.cache[parent], bank[i], len(parent), 0)
                streams.append(bank[i])
                pos.append(len(toks) - 1)
                last.append(int(toks[-1]))
                new_cache[tuple(toks)] = bank[i]
            self.s.step(streams, pos, last, logits_dev=self._logits)
            if self._device != "cpu":
                torch.cuda.synchronize()
            rows = list(self._logits[:len(prefixes)].cpu().numpy())
        self.cache = new_cache
        self.calls += 1
        return [log_softmax(r) for r in rows]
