"""Continuous batching of utterances over one decode session.

Utterances wait in a queue; whenever `encode_batch` stream slots are free (or
the queue holds fewer), the next clips go through the log-mel frontend and the
encoder into those slots, and their decoder prefixes join the very next
batched step next to the single greedy tokens of every running stream. A
stream stops after its own number of new tokens (or at `eot` when
`stop_at_eot`), and its self-attention pages go back to the pool at once, so
the slot takes the next clip.

The host never waits for a step before launching the next one: each running
stream's next token is the greedy id the previous step wrote on the device
(vkb_session_step_feed), and the ids of step t are copied to pinned memory
and read while step t+1 runs. Token counts are known on the host, so a stream
never runs past its length; a stream that emits `eot` (when stopping there)
has already been fed one more step, whose id is dropped before its slot is
released.

This is the serving loop a throughput run needs (up to 128 sequences per GPU,
decode lengths that differ per utterance); the reference decodes one utterance
per DecoderStepSession (crates/vokra-models/src/compute.rs:2892-3140).
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field

import numpy as np


@dataclass
class Utterance:
    pcm_index: int          # row of the caller's PCM tensor
    n_samples: int          # valid samples of that row (the rest reads as silence)
    n_new_tokens: int       # tokens to decode after the prefix
    ids: list = field(default_factory=list)  # greedy ids, filled by run()


class ContinuousBatcher:
    def __init__(self, ctx, session, n_slots: int, encode_batch: int, prefix, n_mels: int, eot: int | None = None,
                 stop_at_eot: bool = False, device: str = "cuda"):
        import torch
        if not 0 < encode_batch <= n_slots:
            raise ValueError(f"ContinuousBatcher: encode_batch must be in [1, n_slots={n_slots}], got {encode_batch}")
        if 2 * session.model.dims.n_audio_ctx != 3000:
            raise ValueError("ContinuousBatcher: the log-mel frontend feeds models with a 30 s window (1500 frames)")
        self.ctx, self.s = ctx, session
        self.n_slots, self.encode_batch = n_slots, encode_batch
        self.prefix = [int(t) for t in prefix]
        self.n_mels, self.eot, self.stop_at_eot = n_mels, eot, stop_at_eot
        self.device = device
        rows = n_slots * (len(self.prefix) + 1)
        self.ids = [torch.zeros(rows, dtype=torch.int32, device=device) for _ in range(2)]
        self.ids_host = [torch.zeros(rows, dtype=torch.int32, pin_memory=device != "cpu") for _ in range(2)]
        self.logmel = torch.empty((encode_batch, n_mels, 3000), dtype=torch.float32, device=device)
        self.steps = 0
        self.tokens = 0

    def run(self, utterances, pcm_dev):
        """Decodes every utterance; pcm_dev is an f32 [rows, samples] tensor on the batcher's device."""
        import torch
        from . import ops
        queue = deque(utterances)
        free = list(range(self.n_slots))
        # slot -> [utterance, ids requested so far, stopped at eot, last step holding it]
        active = {}
        P = len(self.prefix)
        prev = None  # (step index, ids buffer, [(slot, row)], event) of the step in flight
        t = 0
        while queue or active or prev is not None:
            new = []
            if queue and len(free) >= min(self.encode_batch, len(queue)):
                batch = [queue.popleft() for _ in range(min(self.encode_batch, len(queue), len(free)))]
                slots = [free.pop(0) for _ in batch]
                rows = torch.tensor([u.pcm_index for u in batch], dtype=torch.long, device=self.device)
                lens = torch.tensor([u.n_samples for u in batch], dtype=torch.int32, device=self.device)
                pcm = pcm_dev.index_select(0, rows).contiguous()
                lm = self.logmel[:len(batch)]
                ops.log_mel(self.ctx, pcm, self.n_mels, out=lm, lengths=lens)
                self.s.encode(lm, slots)
                new = list(zip(slots, batch))
            # this step: the fed-back id of every running stream, the prefix of each new one
            prev_row = dict(prev[2]) if prev else {}
            streams, pos, toks, feed, rows_out = [], [], [], [], []
            for slot, st in active.items():
                u, asked, stopped, _ = st
                if stopped or asked >= u.n_new_tokens:
                    continue
                streams.append(slot)
                pos.append(P + asked - 1)  # where the id being fed back goes
                toks.append(0)
                feed.append(prev_row[slot])
                rows_out.append((slot, len(streams) - 1))
                st[1] = asked + 1
                st[3] = t
            for slot, u in new:
                for i, tk in enumerate(self.prefix):
                    streams.append(slot)
                    pos.append(i)
                    toks.append(tk)
                    feed.append(-1)
                rows_out.append((slot, len(streams) - 1))
                active[slot] = [u, 1, False, t]
            cur = None
            if streams:
                b = t % 2
                if any(f >= 0 for f in feed):
                    self.s.step_feed(streams, pos, toks, feed, self.ids[prev[1]], ids_dev=self.ids[b])
                else:
                    self.s.step(streams, pos, toks, ids_dev=self.ids[b])
                self.ids_host[b][:len(streams)].copy_(self.ids[b][:len(streams)], non_blocking=True)
                ev = None
                if self.device != "cpu":
                    ev = torch.cuda.Event()
                    ev.record()
                cur = (t, b, rows_out, ev)
                self.steps += 1
                t += 1
            if prev is not None:  # read the previous step's ids while this one runs
                self._collect(prev, active, free)
            prev = cur
        return utterances

    def _collect(self, step, active, free):
        k, b, rows_out, ev = step
        if ev is not None:
            ev.synchronize()
        got = self.ids_host[b].numpy()
        for slot, row in rows_out:
            st = active.get(slot)
            if st is None:
                continue
            u = st[0]
            if not st[2]:
                nxt = int(got[row])
                u.ids.append(nxt)
                self.tokens += 1
                if self.stop_at_eot and nxt == self.eot:
                    st[2] = True
            # finished, and no later step in flight holds the stream: its slot is free
            if (len(u.ids) >= u.n_new_tokens or st[2]) and st[3] <= k:
                del active[slot]
                self.s.release(slot)
                free.append(slot)
