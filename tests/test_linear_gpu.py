"""Quantized Linear on the B200 (GEMV and tcgen05 GEMM paths) against the CPU
oracle's route R1 (dequantize, then the ascending-k FMA chain of gemm_f32)."""
import numpy as np
import pytest

from oracle import py as o
from vokra_b200 import _lib, synth

pytestmark = pytest.mark.gpu

# Q4_0 / Q8_0 / Q4_K run dequant-fused; Q5_K and Q6_K too (the reference
# dequantizes them at load, whisper/weights.rs:400-410, so route R1 is their
# oracle); F32 and BF16 are kept as hi + lo f16 planes, F16 as one plane.
TAGS = [synth.Q4_0, synth.Q8_0, synth.Q4_K, synth.Q5_K, synth.Q6_K, synth.F32, synth.BF16]


def _weights(tag, n, k, seed, rnd=False):
    rng = np.random.default_rng(seed)
    if tag in (synth.Q5_K, synth.Q6_K) and rnd:
        return synth.random_kquant_blocks(tag, n * k, rng)  # every sub-scale, min and high bit random
    w = (rng.standard_normal(n * k).astype(np.float32) * np.float32(0.02))
    return synth.quantize(tag, w)


def _rel_rms(a, b):
    return float(np.sqrt(np.mean((a - b) ** 2)) / (np.sqrt(np.mean(b ** 2)) + 1e-30))


def _run(ctx, tag, n, k, m, seed=0, bias=True, a_f16=False, out_f16=False, epi=_lib.EPI_NONE, scale=1.0, rnd=False):
    import torch
    from vokra_b200 import ops
    wq = _weights(tag, n, k, seed, rnd)
    rng = np.random.default_rng(seed + 1)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = (rng.standard_normal(n).astype(np.float32) * np.float32(0.1)) if bias else None
    res = rng.standard_normal((m, n)).astype(np.float32)
    w = ops.Weight(ctx, tag, n, k, wq)
    dev = "cuda:0"
    at = torch.from_numpy(a).to(dev)
    if a_f16:
        at = at.half()
    bt = None if b is None else torch.from_numpy(b).to(dev)
    out = torch.zeros((m, n), dtype=torch.float16 if out_f16 else torch.float32, device=dev)
    rt = torch.from_numpy(res).to(dev) if epi == _lib.EPI_RESIDUAL else None
    ops.linear(ctx, w, at, out, bias=bt, epilogue=epi, residual=rt, scale=scale)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    a_ref = at.float().cpu().numpy()
    ref = o.linear_q(tag, a_ref, wq, n, k, b)
    if epi == _lib.EPI_GELU:
        ref = o.gelu(ref)
    elif epi == _lib.EPI_SCALE:
        ref = ref * np.float32(scale)
    elif epi == _lib.EPI_RESIDUAL:
        ref = res + ref
    return got, ref


@pytest.mark.parametrize("tag", TAGS)
@pytest.mark.parametrize("m", [1, 2, 3, 4, 5, 8])
def test_gemv_path_matches_oracle(ctx, tag, m):
    # Q4_0 / Q8_0 / Q4_K at m = 1: the bulk-staged streaming GEMV with its in-kernel
    # split-K reduction; other formats at m <= 4: the row-per-thread GEMV; fp32
    # arithmetic either way. Elsewhere the tensor-core GEMM (its own bar).
    gv2 = tag in (synth.Q4_0, synth.Q8_0, synth.Q4_K)
    for i, (k, n) in enumerate([(256, 128), (512, 300), (1280, 1280)]):
        got, ref = _run(ctx, tag, n, k, m, seed=k + n, rnd=i % 2 == 1)
        if (gv2 and m > 1) or m > 4:
            assert _rel_rms(got, ref) <= 1e-3
            continue
        assert np.max(np.abs(got - ref)) <= 1e-4 * max(1.0, np.max(np.abs(ref)))
        assert _rel_rms(got, ref) <= 1e-5


@pytest.mark.parametrize("tag", TAGS)
@pytest.mark.parametrize("m", [5, 8, 33, 64, 100, 256, 300, 1500])
def test_tensor_core_path_matches_oracle(ctx, tag, m):
    # f16 operands on tcgen05 with fp32 accumulation: 1e-3 relative RMS, 1e-2 max-abs.
    for i, (k, n) in enumerate([(256, 128), (1280, 384)]):
        got, ref = _run(ctx, tag, n, k, m, seed=7 * k + n, rnd=i % 2 == 1)
        assert _rel_rms(got, ref) <= 1e-3, (k, n)
        assert np.max(np.abs(got - ref)) <= 1e-2, (k, n)


@pytest.mark.parametrize("tag", TAGS)
def test_tensor_core_large_k_and_ragged_n(ctx, tag):
    got, ref = _run(ctx, tag, 1300, 5120, 96, seed=11, rnd=True)
    assert _rel_rms(got, ref) <= 1e-3
    assert np.max(np.abs(got - ref)) <= 2e-2


@pytest.mark.parametrize("m", [1, 2, 64])
@pytest.mark.parametrize("epi", [_lib.EPI_GELU, _lib.EPI_SCALE, _lib.EPI_RESIDUAL])
def test_epilogues(ctx, m, epi):
    got, ref = _run(ctx, synth.Q4_0, 256, 512, m, epi=epi, scale=0.125)
    tol = 1e-5 if m == 1 else 1e-3
    assert _rel_rms(got, ref) <= tol


def test_f16_in_f16_out_no_bias(ctx):
    got, ref = _run(ctx, synth.Q8_0, 384, 512, 128, bias=False, a_f16=True, out_f16=True)
    assert _rel_rms(got, ref) <= 2e-3


def test_host_gemm_q_f32_contract(ctx):
    from vokra_b200 import ops
    n, k, m = 256, 512, 3
    wq = _weights(synth.Q4_K, n, k, 3)
    rng = np.random.default_rng(4)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    out = np.zeros((m, n), np.float32)
    ops.gemm_q_f32(ctx, m, n, k, a, wq, synth.Q4_K, b, out)
    ref = o.linear_q(synth.Q4_K, a, wq, n, k, b)
    assert np.max(np.abs(out - ref)) <= 1e-4


def test_rejections(ctx):
    from vokra_b200 import ops
    with pytest.raises(ops.VkbError) as e:
        ops.Weight(ctx, synth.Q4_0, 4, 96, synth.quantize(synth.Q4_0, np.zeros(4 * 96, np.float32)))
    assert e.value.code == _lib.ERROR_UNSUPPORTED_OP
    with pytest.raises(ops.VkbError) as e:
        ops.Weight(ctx, synth.Q4_0, 4, 64, b"\0" * 10)
    assert e.value.code == _lib.ERROR_INVALID_ARGUMENT
    with pytest.raises(ops.VkbError) as e:
        ops.Weight(ctx, 6, 4, 64, b"\0" * 10)
    assert e.value.code == _lib.ERROR_UNSUPPORTED_OP


# Large M (encoder-sized): the persistent tensor-core GEMM with the double-
# buffered accumulator takes these (>= 4 tiles per SM; 192-token tiles, so
# m = 11000 leaves a ragged last tile and n = 1300 a ragged weight tile).
@pytest.mark.parametrize("tag", TAGS)
def test_persistent_gemm_matches_oracle(ctx, tag):
    for k in (1280, 768):
        got, ref = _run(ctx, tag, 1300, k, 11000, seed=5 + k)
        assert _rel_rms(got, ref) <= 1e-4, k
        assert np.max(np.abs(got - ref)) <= 2e-3, k


@pytest.mark.parametrize("epi,out_f16", [(_lib.EPI_GELU, True), (_lib.EPI_SCALE, True), (_lib.EPI_RESIDUAL, False),
                                         (_lib.EPI_NONE, True)])
def test_persistent_gemm_epilogues(ctx, epi, out_f16):
    got, ref = _run(ctx, synth.Q4_0, 1280, 1280, 12000, epi=epi, out_f16=out_f16, scale=0.125)
    tol = 1e-3 if out_f16 else 1e-4  # an f16 output rounds at 2^-11 relative
    assert _rel_rms(got, ref) <= tol


def test_persistent_gemm_long_k(ctx, monkeypatch):
    # K = 5120 runs on the classic kernel by default; forced onto the persistent one here
    monkeypatch.setenv("VKB_GEMM_PERSIST", "force")
    got, ref = _run(ctx, synth.Q4_0, 1280, 5120, 11000, seed=9)
    assert _rel_rms(got, ref) <= 1e-4
    assert np.max(np.abs(got - ref)) <= 5e-3


@pytest.mark.parametrize("tag", [synth.Q4_0, synth.Q8_0, synth.Q4_K])
@pytest.mark.parametrize("m", [1, 2, 3, 4])
def test_streaming_gemv_wide_weight(ctx, tag, m):
    """A logits-head-wide weight (N >= 16384 rows) at m <= 4: the streaming GEMV
    for every m, its split partials summed in the kernel, fp32 arithmetic."""
    got, ref = _run(ctx, tag, 16500, 512, m, seed=21 + m)
    assert _rel_rms(got, ref) <= 1e-5
    assert np.max(np.abs(got - ref)) <= 1e-4 * max(1.0, np.max(np.abs(ref)))


@pytest.mark.parametrize("tag", [synth.Q4_0, synth.Q8_0, synth.Q4_K])
def test_persistent_gemm_single_f16(ctx, tag):
    """Large M with a single f16 activation plane (the encoder in
    VKB_PREC_ENCODER_F16): the persistent kernel at one MMA per K step;
    weights rounded to f16 once, so 2e-3 relative RMS like the other f16 path."""
    got, ref = _run(ctx, tag, 1300, 1280, 12000, seed=13, a_f16=True)
    assert _rel_rms(got, ref) <= 2e-3
    assert np.max(np.abs(got - ref)) <= 3e-2


@pytest.mark.parametrize("tag,n,k,epi,out_f16", [
    (synth.Q4_0, 1300, 1280, _lib.EPI_GELU, True),
    (synth.Q8_0, 1280, 1280, _lib.EPI_SCALE, False),
    (synth.Q4_K, 1280, 1280, _lib.EPI_NONE, True),
    (synth.Q4_0, 1280, 5120, _lib.EPI_RESIDUAL, False),
])
def test_persistent_gemm_shared_operands_match_tmem_path(ctx, monkeypatch, tag, n, k, epi, out_f16):
    """Single-f16 large-M GEMM on the kernel whose weight tile arrives by TMA
    from an f16 plane dequantized once per call (both MMA operands in shared
    memory, 256-token tiles) against the kernel that dequantizes into tensor
    memory per tile: the same f16 weights and the same K order, so the same
    values; and both against the oracle. M = 12001 leaves a ragged last tile."""
    import torch
    outs = []
    # shared operands on CTA pairs (cta_group::2), on one CTA, then the TMEM-operand kernel
    for ss, pair in (("1", "1"), ("1", "0"), ("0", "0")):
        monkeypatch.setenv("VKB_GEMM_SS", ss)
        monkeypatch.setenv("VKB_GEMM_PAIR", pair)
        monkeypatch.setenv("VKB_GEMM_PERSIST", "force")
        got, ref = _run(ctx, tag, n, k, 12001, seed=31, a_f16=True, out_f16=out_f16, epi=epi, scale=0.125)
        outs.append(got)
        assert _rel_rms(got, ref) <= 2e-3
    for o in outs[:2]:
        assert np.max(np.abs(o - outs[2])) <= 1e-5 * max(1.0, float(np.max(np.abs(outs[2]))))
