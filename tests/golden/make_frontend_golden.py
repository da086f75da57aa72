"""Writes tests/golden/whisper_base_frontend.npz from the reference's own
log-mel parity fixture (tests/parity/whisper_base/ in the reference
repository, checked by crates/vokra-models/tests/parity_whisper.rs:279-299,
log_mel_parity):
  pcm     input_pcm.f32 (480000 samples of 16 kHz mono PCM, every value an
          integer / 32768, so it is stored here as int16 without loss);
  logmel  logmel.f32, the first `mel_frames` frames of the [n_mels, 3000]
          features, [80, 100];
  atol    the manifest's tolerance for the base size (0.01).
Run once where the reference checkout is available:
  python tests/golden/make_frontend_golden.py <reference-root>
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def main(root: str) -> None:
    d = os.path.join(root, "tests", "parity", "whisper_base")
    man = {}
    for line in open(os.path.join(d, "manifest.txt")):
        line = line.strip()
        if line and not line.startswith("#") and "=" in line:
            k, v = line.split("=", 1)
            man[k.strip()] = v.strip()
    pcm = np.fromfile(os.path.join(d, "input_pcm.f32"), dtype=np.float32)
    assert pcm.size == int(man["pcm_len"])
    q = np.round(pcm.astype(np.float64) * 32768.0)
    assert np.array_equal(q / 32768.0, pcm.astype(np.float64)), "PCM is not int16-exact"
    n_mels, frames = int(man["n_mels"]), int(man["mel_frames"])
    logmel = np.fromfile(os.path.join(d, "logmel.f32"), dtype=np.float32).reshape(n_mels, frames)
    np.savez_compressed(os.path.join(HERE, "whisper_base_frontend.npz"), pcm=q.astype(np.int16), logmel=logmel,
                        atol=np.float32(float(man["atol"])), sha256=np.array(man["pcm_sha256"]))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("VOKRA_REFERENCE_ROOT", "."))
