"""GPU parity of the speech decoder, decode_to_audio (decoder.rs:395-582),
through the C ABI (qora_decode_to_audio / qora_decode_to_audio_device), with
the CPU oracle (oracle/pydecoder.py) as the checker.

The GPU sums every convolution and projection in the reference's term order
but with fused multiply-adds, and its sin / exp / tanh are CUDA's, so samples
agree to f32 rounding carried through ~80 layers, not bit for bit: every
case is held to max |gpu - oracle| <= 1e-4 on samples in [-1, 1] and to an
RMS difference <= 1e-4 of the signal's RMS (measured on a B200: CUDA-core
convolutions max 6.9e-6 at the tiny dims and 1.5e-5 at the real dims;
tensor-core 3 x TF32 convolutions max 4.3e-5 and 4.4e-5, relative RMS
1.9e-5 and 3.3e-5).

Cases: the tiny dims (real strides, kernels and structure, small channel
counts) with and without a warm-up prefix; the real 12 Hz tokenizer dims on
a few frames; a long case past the real 72-position attention window and the
64-query attention tiles (real transformer dims, small Vocos); the reference's
edge behaviour (no frames, an out-of-codebook code).  The parity cases run
twice: every convolution on the CUDA cores (tensor-core mode 0), and every
convolution that has a tensor-core form on the tcgen05 3 x TF32 kernel
(mode 2; the default mode 1 picks per launch by estimated time, checked
against the other two on a longer real-dims decode)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL_MAX = 1e-4
TOL_RMS = 1e-4


@pytest.fixture(scope="module")
def ctx():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("-m gpu tests need a CUDA device")
    from qora_b200 import engine
    return engine.Context(0)


def _codes(dims, T, seed):
    return np.random.default_rng(seed).integers(0, dims.codebook_size, (dims.num_quantizers, T)).astype(np.uint32)


def _compare(got, ref, what):
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    err = np.abs(got.astype(np.float64) - ref)
    worst = float(err.max()) if err.size else 0.0
    rel = float(np.sqrt(np.mean(err ** 2)) / max(1e-30, np.sqrt(np.mean(ref.astype(np.float64) ** 2))))
    print(f"{what}: {got.size} samples, max |diff| {worst:.3e}, relative RMS diff {rel:.3e}, "
          f"clamped {float((np.abs(ref) >= 1).mean()):.4f}")
    assert worst <= TOL_MAX, (what, worst)
    assert rel <= TOL_RMS, (what, rel)


def _setup(ctx, dims, seed=4321, tc=1):
    from qora_b200.decoder import SpeechDecoder, synth_decoder
    W = synth_decoder(dims, seed)
    dec = SpeechDecoder(ctx, dims, W)
    dec.use_tensor_cores(tc)
    return W, dec


@pytest.mark.parametrize("tc", [0, 2])
def test_tiny_matches_oracle(ctx, tc):
    import pydecoder as D
    from qora_b200.decoder import DecoderDims
    dims = DecoderDims.tiny()
    W, dec = _setup(ctx, dims, tc=tc)
    for T, seed in ((1, 1), (12, 2), (65, 3)):
        codes = _codes(dims, T, seed)
        got = dec.decode_to_audio(codes)
        ctx.check_device_error()
        assert got.size == T * dims.hop
        _compare(got, D.decode_to_audio(W, codes, dims=dims), f"tiny T={T} tc={tc}")


def test_tiny_warmup_prefix_is_trimmed(ctx):
    """decode_to_audio's warm-up (decoder.rs:405-430, 548-552): the warm-up
    codes are decoded in front and their share of the samples cut."""
    import pydecoder as D
    from qora_b200.decoder import DecoderDims
    dims = DecoderDims.tiny()
    W, dec = _setup(ctx, dims)
    codes, wu = _codes(dims, 20, 5), _codes(dims, 7, 6)
    got = dec.decode_to_audio(codes, warmup=wu)
    assert got.size == 20 * dims.hop
    ref = D.decode_to_audio(W, codes, warmup=wu, dims=dims)
    _compare(got, ref, "tiny warm-up 7 + 20")
    # an empty warm-up block is ignored (decoder.rs:412-417)
    np.testing.assert_array_equal(dec.decode_to_audio(codes, warmup=np.zeros((16, 0), np.uint32)),
                                  dec.decode_to_audio(codes))


@pytest.mark.parametrize("tc", [0, 2])
def test_real_dims_match_oracle(ctx, tc):
    import pydecoder as D
    from qora_b200.decoder import DecoderDims
    dims = DecoderDims()
    W, dec = _setup(ctx, dims, tc=tc)
    codes = _codes(dims, 6, 7)
    got = dec.decode_to_audio(codes)
    ctx.check_device_error()
    assert got.size == 6 * 1920
    _compare(got, D.decode_to_audio(W, codes, dims=dims), f"real dims T=6 tc={tc}")


@pytest.mark.parametrize("tc", [0, 2])
def test_long_sequence_past_the_window(ctx, tc):
    """150 frames (3 attention query tiles, positions past the 72-position
    sliding window) with a 30-frame warm-up, real transformer and upsample
    dims, small Vocos channels (the oracle's run time)."""
    import pydecoder as D
    from qora_b200.decoder import DecoderDims
    dims = DecoderDims(vocos_channels=(96, 48, 24, 12, 8))
    W, dec = _setup(ctx, dims, seed=99, tc=tc)
    codes, wu = _codes(dims, 150, 8), _codes(dims, 30, 9)
    got = dec.decode_to_audio(codes, warmup=wu)
    ctx.check_device_error()
    _compare(got, D.decode_to_audio(W, codes, warmup=wu, dims=dims), f"long 30 + 150 tc={tc}")


def test_default_mode_matches_both_kernels(ctx):
    """Mode 1 mixes the two kernels by estimated time; on a 60-frame real-dims
    decode (where the big Vocos convolutions go to the tensor cores and the
    small ones stay on the CUDA cores) it agrees with all-CUDA-core and
    all-tensor-core decodes within the parity tolerance."""
    from qora_b200.decoder import DecoderDims
    dims = DecoderDims()
    _, dec = _setup(ctx, dims, seed=5)
    codes = _codes(dims, 60, 13)
    out = {}
    for tc in (0, 1, 2):
        dec.use_tensor_cores(tc)
        out[tc] = dec.decode_to_audio(codes)
    ctx.check_device_error()
    _compare(out[1], out[0].astype(np.float64), "60 frames mode 1 vs 0")
    _compare(out[1], out[2].astype(np.float64), "60 frames mode 1 vs 2")


def test_device_entry_matches_host_entry(ctx):
    import torch
    from qora_b200.decoder import DecoderDims
    dims = DecoderDims.tiny()
    _, dec = _setup(ctx, dims)
    codes, wu = _codes(dims, 9, 10), _codes(dims, 4, 11)
    host = dec.decode_to_audio(codes, warmup=wu)
    cd = torch.from_numpy(np.concatenate([wu, codes], axis=1).astype(np.int32)).cuda()
    out = torch.empty(9 * dims.hop, dtype=torch.float32, device="cuda")
    n = dec.decode_device(cd, 9, out, warmup_frames=4)
    torch.cuda.synchronize()
    assert n > 10
    np.testing.assert_array_equal(out.cpu().numpy(), host)


def test_edges(ctx):
    import qora_b200
    from qora_b200.decoder import DecoderDims
    dims = DecoderDims.tiny()
    _, dec = _setup(ctx, dims)
    # no frames: no samples (decoder.rs:401-404)
    assert dec.decode_to_audio(np.zeros((16, 0), np.uint32)).size == 0
    # a code outside the codebook: the reference's slice panics; here the
    # device flag reports it
    codes = _codes(dims, 3, 12)
    codes[5, 1] = dims.codebook_size
    dec.decode_to_audio(codes)
    with pytest.raises(qora_b200._lib.QoraError) as e:
        ctx.check_device_error()
    assert e.value.status == 5
    ctx.check_device_error()      # cleared
