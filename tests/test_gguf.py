"""The GGUF reader's rejections, host side (vkb_gguf_inspect, no device work).

Each malformed image below is one of the reference reader's own test cases
(crates/vokra-core/src/gguf/reader.rs:512-800) or a defect the loader must
catch (truncated data, misaligned offsets, a non-power-of-two alignment):
the call returns VKB_ERROR_MODEL_LOAD and names the GgufError variant the
reference returns. The GPU tests check that vkb_whisper_load reports the
same defects through a whole model file.
"""
import ctypes as C
import struct

import numpy as np
import pytest

from vokra_b200 import _lib, synth


def inspect(data: bytes):
    """(status, message, n_tensors, n_metadata) of vkb_gguf_inspect over `data`."""
    L = _lib.load()
    nt, nk = C.c_int64(-1), C.c_int64(-1)
    buf = C.create_string_buffer(data, len(data))
    st = L.vkb_gguf_inspect(buf, len(data), C.byref(nt), C.byref(nk))
    msg = L.vkb_last_error().decode("utf-8", "replace") if st else ""
    return st, msg, nt.value, nk.value


def header(n_t, n_kv, version=3, magic=b"GGUF"):
    return magic + struct.pack("<IQQ", version, n_t, n_kv)


def gstr(s: bytes):
    return struct.pack("<Q", len(s)) + s


def tinfo(name: bytes, dims, tag, off):
    return gstr(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims) + \
        struct.pack("<IQ", tag, off)


def pad_to(b: bytes, a=32):
    return b + b"\0" * ((-len(b)) % a)


def rejected(data, variant):
    st, msg, _, _ = inspect(data)
    assert st == _lib.ERROR_MODEL_LOAD, (st, msg)
    assert f"({variant})" in msg, msg
    return msg


def test_hand_built_empty_header_parses():
    assert inspect(header(0, 0))[::2] == (0, 0)
    assert inspect(header(0, 0))[3] == 0


def test_one_tensor_file_parses():
    body = pad_to(header(1, 1) + gstr(b"general.alignment") + struct.pack("<II", 4, 32) +
                  tinfo(b"t", [4], 0, 0)) + struct.pack("<4f", 1, 2, 3, 4)
    st, msg, nt, nk = inspect(body)
    assert (st, nt, nk) == (0, 1, 1), msg


def test_bad_magic():
    rejected(header(0, 0, magic=b"GGUX"), "BadMagic")


def test_unsupported_version():
    msg = rejected(header(0, 0, version=2), "UnsupportedVersion")
    assert "version 2" in msg


def test_truncated_header():
    rejected(b"GGUF", "Truncated")
    rejected(header(0, 0)[:-3], "Truncated")


def test_oversized_counts_rejected_without_allocating():
    rejected(header(0, 2 ** 64 - 1), "Truncated")
    rejected(header(2 ** 64 - 1, 0), "Truncated")


def test_oversized_string_length():
    rejected(header(0, 1) + struct.pack("<Q", 2 ** 64 - 1), "Truncated")


def test_unsupported_dtype():
    # tag 3 (ggml Q4_1) has no reader in the reference nor here
    rejected(header(1, 0) + tinfo(b"bad", [4], 3, 0), "UnsupportedDtype")


def test_tensor_offset_out_of_bounds():
    rejected(pad_to(header(1, 0) + tinfo(b"t", [4], 0, 4096)), "OffsetOutOfBounds")


def test_tensor_data_truncated():
    body = pad_to(header(1, 0) + tinfo(b"t", [64], 0, 0)) + b"\0" * 255  # 256 bytes declared
    rejected(body, "OffsetOutOfBounds")


def test_kquant_partial_block():
    body = pad_to(header(1, 0) + tinfo(b"q", [100], synth.Q4_K, 0)) + b"\0" * 144
    rejected(body, "BlockSizeMisaligned")


def test_duplicate_tensor():
    body = pad_to(header(2, 0) + tinfo(b"t", [8], 0, 0) + tinfo(b"t", [8], 0, 32)) + b"\0" * 64
    rejected(body, "DuplicateTensor")


def test_misaligned_offset():
    body = pad_to(header(1, 0) + tinfo(b"t", [8], 0, 4)) + b"\0" * 64
    rejected(body, "UnalignedTensorOffset")


@pytest.mark.parametrize("align", [0, 3, 48])
def test_alignment_not_power_of_two(align):
    body = header(0, 1) + gstr(b"general.alignment") + struct.pack("<II", 4, align)
    rejected(body, "InvalidAlignment")


def test_too_many_dimensions():
    rejected(header(1, 0) + tinfo(b"t", [1] * 9, 0, 0), "TooManyDimensions")


def test_invalid_bool():
    rejected(header(0, 1) + gstr(b"flag") + struct.pack("<IB", 7, 2), "InvalidBool")


def test_whisper_file_and_its_truncations(tmp_path):
    """A whole synthetic Whisper GGUF parses; cut anywhere inside its header or
    its last tensor, it is rejected, never read out of bounds."""
    path = str(tmp_path / "tiny.gguf")
    synth.write_synthetic_whisper(path, synth.WHISPER_TINY_TEST, synth.Q4_0, seed=1)
    data = open(path, "rb").read()
    st, msg, nt, nk = inspect(data)
    assert st == 0, msg
    assert nt == len(synth.whisper_tensor_decls(synth.WHISPER_TINY_TEST, synth.Q4_0))
    assert nk == len(synth.whisper_metadata(synth.WHISPER_TINY_TEST))
    rng = np.random.default_rng(0)
    for cut in sorted(set([1, 3, 4, 8, 23, len(data) - 1] + [int(x) for x in rng.integers(5, len(data) - 1, 40)])):
        st, msg, _, _ = inspect(data[:cut])
        assert st == _lib.ERROR_MODEL_LOAD, (cut, msg)


def _write_with(path, decls, meta):
    w = synth.GgufStreamWriter(path, meta, [synth.TensorDecl(n, t, d) for n, t, d in decls])
    w.begin()
    for name, tag, dims in decls:
        w.write(synth.quantize(tag, np.zeros(int(np.prod(dims)), np.float32)))
    w.finish()


@pytest.mark.gpu
def test_whisper_load_reports_defects(ctx, tmp_path):
    """vkb_whisper_load over whole model files with one defect each: the exact
    status and the variant or the offending tensor in the message."""
    from vokra_b200 import whisper
    a = synth.WHISPER_TINY_TEST
    decls = synth.whisper_tensor_decls(a, synth.Q8_0)
    meta = synth.whisper_metadata(a)
    cases = []
    # a Linear with the wrong shape
    bad = [(n, t, [d[0], d[1] + 64]) if n == "model.decoder.layers.1.fc2.weight" else (n, t, d) for n, t, d in decls]
    cases.append((bad, meta, "model.decoder.layers.1.fc2.weight"))
    # a missing tensor
    cases.append(([x for x in decls if x[0] != "model.encoder.layers.0.self_attn.q_proj.bias"], meta, "MissingTensor"))
    # another architecture
    cases.append((decls, dict(meta, **{"general.architecture": "llama"}), "architecture"))
    for i, (dl, mt, needle) in enumerate(cases):
        path = str(tmp_path / f"bad{i}.gguf")
        _write_with(path, dl, mt)
        with pytest.raises(_lib.VkbError) as e:
            whisper.WhisperModel(ctx, path)
        assert e.value.code == _lib.ERROR_MODEL_LOAD, e.value
        assert needle in str(e.value), str(e.value)
    # truncated data and bad magic: the reader's own checks
    good = str(tmp_path / "good.gguf")
    _write_with(good, decls, meta)
    data = open(good, "rb").read()
    for i, (blob, variant) in enumerate([(data[:-100], "OffsetOutOfBounds"), (b"GGUX" + data[4:], "BadMagic")]):
        path = str(tmp_path / f"blob{i}.gguf")
        open(path, "wb").write(blob)
        with pytest.raises(_lib.VkbError) as e:
            whisper.WhisperModel(ctx, path)
        assert e.value.code == _lib.ERROR_MODEL_LOAD and f"({variant})" in str(e.value), str(e.value)
    with pytest.raises(_lib.VkbError) as e:
        whisper.WhisperModel(ctx, str(tmp_path / "absent.gguf"))
    assert e.value.code == _lib.ERROR_IO


def test_seeded_mutations_never_crash(tmp_path):
    """A seeded mutation harness over a whole model file: 400 images with 1-8
    random bytes overwritten (header, metadata, tensor infos or data), cut,
    or with a block of bytes duplicated. Every image either parses or is
    rejected as VKB_ERROR_MODEL_LOAD; none crashes or reads out of bounds."""
    path = str(tmp_path / "tiny.gguf")
    synth.write_synthetic_whisper(path, synth.WHISPER_TINY_TEST, synth.Q8_0, seed=2)
    data = open(path, "rb").read()
    head = 4096  # mutations concentrate on the header, where the parser's decisions are
    rng = np.random.default_rng(1234)
    seen = {0: 0, _lib.ERROR_MODEL_LOAD: 0}
    for _ in range(400):
        b = bytearray(data)
        kind = rng.integers(0, 3)
        if kind == 0:
            for _ in range(int(rng.integers(1, 9))):
                b[int(rng.integers(0, head))] = int(rng.integers(0, 256))
        elif kind == 1:
            b = b[:int(rng.integers(0, len(b)))]
        else:
            i = int(rng.integers(0, head))
            n = int(rng.integers(1, 64))
            b = b[:i] + b[i:i + n] + b[i:]
        st, msg, _, _ = inspect(bytes(b))
        assert st in seen, (st, msg)
        seen[st] += 1
    assert seen[_lib.ERROR_MODEL_LOAD] > 0
    print("mutations:", seen)
