"""Host-side pieces around the speech decoder (no GPU): the warm-up tail a
chunk hands to decode_to_audio and the VCOD codes file, held to the
reference's own unit tests (generate_new.rs:971-983 test_warmup_tail,
1009-1030 test_codes_roundtrip), and the decoder dims' frame length."""
import numpy as np
import pytest

from qora_b200.decoder import DecoderDims, read_codes_file, warmup_tail, write_codes_file


def test_warmup_tail_known_answers():
    codes = np.array([[1, 2, 3, 4, 5], [6, 7, 8, 9, 10]], np.uint32)
    for k in (0, 5, 99):                       # passthrough
        np.testing.assert_array_equal(warmup_tail(codes, k), codes)
    np.testing.assert_array_equal(warmup_tail(codes, 2), [[4, 5], [9, 10]])
    assert warmup_tail([], 3).size == 0        # empty
    t = warmup_tail(codes, 2)
    t[0, 0] = 77                               # a copy, not a view
    assert codes[0, 3] == 4


def test_codes_file_known_bytes(tmp_path):
    p = tmp_path / "rt.vcod"
    write_codes_file(p, [[1, 2047, 0], [4095, 7, 13]])
    raw = p.read_bytes()
    assert raw[:4] == b"VCOD"
    assert int.from_bytes(raw[4:8], "little") == 2
    assert int.from_bytes(raw[8:12], "little") == 3
    vals = [int.from_bytes(raw[12 + 2 * i:14 + 2 * i], "little") for i in range(6)]
    assert vals == [1, 2047, 0, 4095, 7, 13]
    assert len(raw) == 24
    np.testing.assert_array_equal(read_codes_file(p), [[1, 2047, 0], [4095, 7, 13]])


def test_codes_file_roundtrip_and_errors(tmp_path):
    codes = np.random.default_rng(0).integers(0, 2048, (16, 241)).astype(np.uint32)
    p = tmp_path / "a.vcod"
    write_codes_file(p, codes)
    got = read_codes_file(p)
    assert got.dtype == np.uint32 and got.shape == (16, 241)
    np.testing.assert_array_equal(got, codes)
    # a code keeps its low 16 bits (the reference's `as u16`)
    write_codes_file(p, [[0x12345]])
    assert read_codes_file(p)[0, 0] == 0x2345
    bad = tmp_path / "bad.vcod"
    bad.write_bytes(b"XCOD" + bytes(8))
    with pytest.raises(ValueError, match="magic"):
        read_codes_file(bad)
    short = tmp_path / "short.vcod"
    short.write_bytes(b"VCOD" + np.array([2, 3], "<u4").tobytes() + bytes(10))
    with pytest.raises(ValueError):
        read_codes_file(short)


def test_hop_is_1920_samples_per_frame():
    # 2 upsample stages of 2, Vocos strides 8, 5, 4, 3: 12.5 Hz frames at 24 kHz
    assert DecoderDims().hop == 1920
    assert DecoderDims.tiny().hop == 1920


def test_decoder_warmup_selection():
    """generate_new.rs:695-712: a chained tail wins; then the reference
    clip's codes when decode_warmup is set (trimmed to warmup_frames > 0);
    otherwise no warm-up."""
    from qora_b200 import generate as G
    ref = np.arange(2 * 6, dtype=np.uint32).reshape(2, 6)
    chain = np.full((2, 3), 9, np.uint32)
    off = G.TTSParams()
    assert off.decode_warmup is False and off.warmup_frames == 0      # defaults (generate_new.rs:64-78)
    on_all, on_tail = G.TTSParams(decode_warmup=True), G.TTSParams(decode_warmup=True, warmup_frames=2)
    for p in (off, on_all, on_tail):
        np.testing.assert_array_equal(G.decoder_warmup(p, chain, ref), chain)
    assert G.decoder_warmup(off, None, ref) is None
    assert G.decoder_warmup(off, np.zeros((2, 0), np.uint32), ref) is None
    np.testing.assert_array_equal(G.decoder_warmup(on_all, None, ref), ref)
    np.testing.assert_array_equal(G.decoder_warmup(on_tail, np.zeros((2, 0), np.uint32), ref), ref[:, 4:])
    assert G.decoder_warmup(on_tail, None, None) is None
