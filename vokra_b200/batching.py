"""Continuous batching of utterances over one decode session.

Utterances wait in a queue; whenever `encode_batch` stream slots are free (or
the queue holds fewer), the next clips go through the log-mel frontend and the
encoder into those slots, and their decoder prefixes join the very next
batched step next to the single greedy tokens of every running stream. A
stream stops after its own number of new tokens (or at `eot` when
`stop_at_eot`), and its self-attention pages go back to the pool at once, so
the slot takes the next clip. Greedy ids come from the device argmax of the
step; the host reads them back each step to feed them forward.

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
        self.ids = torch.zeros(n_slots * (len(self.prefix) + 1), dtype=torch.int32, device=device)
        self.logmel = torch.empty((encode_batch, n_mels, 3000), dtype=torch.float32, device=device)
        self.steps = 0
        self.tokens = 0

    def run(self, utterances, pcm_dev):
        """Decodes every utterance; pcm_dev is an f32 [rows, samples] tensor on the batcher's device."""
        import torch
        from . import ops
        queue = deque(utterances)
        free = list(range(self.n_slots))
        active = {}   # slot -> [utterance, position, last token]
        P = len(self.prefix)
        while queue or active:
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
            streams, pos, toks, last_row = [], [], [], {}
            for slot, st in active.items():
                streams.append(slot)
                pos.append(st[1])
                toks.append(st[2])
                last_row[slot] = len(streams) - 1
            for slot, u in new:
                for i, t in enumerate(self.prefix):
                    streams.append(slot)
                    pos.append(i)
                    toks.append(t)
                last_row[slot] = len(streams) - 1
            if not streams:
                continue
            self.s.step(streams, pos, toks, ids_dev=self.ids)
            got = self.ids[:len(streams)].cpu().numpy()
            self.steps += 1
            for slot, u in new:
                active[slot] = [u, P, None]
            done = []
            for slot, st in active.items():
                u = st[0]
                nxt = int(got[last_row[slot]])
                u.ids.append(nxt)
                self.tokens += 1
                st[1] = P + len(u.ids) - 1  # position of the token just produced
                st[2] = nxt
                if len(u.ids) >= u.n_new_tokens or (self.stop_at_eot and nxt == self.eot):
                    done.append(slot)
            for slot in done:
                del active[slot]
                self.s.release(slot)
                free.append(slot)
        return utterances
