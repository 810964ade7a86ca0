"""After the decoder: chunk assembly and WAV output (qora_b200/audio.py),
held to the reference's own unit tests, restated: wav.rs:222-270 (trim
silence), chunk.rs:327-357 (crossfade), chunk.rs:359-444 (pad tail and the
main.rs seam pipeline); and the 16-bit WAV layout of wav.rs:7-46, read back
with the standard library."""
import wave

import numpy as np

from qora_b200 import audio as A

F32 = np.float32


def speech_frame():
    return np.full(480, 0.1, F32)             # wav.rs:222-224: energy 0.01 >> 1e-4


def speech(n, amp):
    """chunk.rs:369-378: mixed 220 / 440 Hz sines, in f32."""
    t = np.arange(n, dtype=F32) / F32(24000.0)
    tau = F32(2.0) * F32(np.pi)
    return (F32(amp) * (F32(0.6) * np.sin(tau * F32(220.0) * t) + F32(0.4) * np.sin(tau * F32(440.0) * t))).astype(F32)


# ---- wav.rs:226-270 ------------------------------------------------------
def test_trim_silence_compresses_gap():
    x = np.concatenate([speech_frame(), np.zeros(480 * 50, F32), speech_frame()])
    assert A.trim_silence(x, 24000, 0.25).size == 480 * 15       # 1 + 13 + 1 frames


def test_trim_silence_cuts_trailing():
    x = np.concatenate([speech_frame(), np.zeros(480 * 50, F32)])
    assert A.trim_silence(x, 24000, 0.25).size == 480 * 14       # 1 speech + 13 gap


def test_trim_silence_short_gap_untouched():
    x = np.concatenate([speech_frame(), np.zeros(480 * 10, F32), speech_frame()])
    np.testing.assert_array_equal(A.trim_silence(x, 24000, 0.25), x)


def test_trim_silence_all_silence():
    assert A.trim_silence(np.zeros(480 * 5, F32), 24000, 0.25).size == 0


def test_trim_silence_leading_kept():
    x = np.concatenate([np.zeros(480 * 5, F32), speech_frame()])
    np.testing.assert_array_equal(A.trim_silence(x, 24000, 0.25), x)


def test_trim_silence_off_and_empty():
    x = np.concatenate([speech_frame(), np.zeros(480 * 50, F32)])
    np.testing.assert_array_equal(A.trim_silence(x, 24000, 0.0), x)
    assert A.trim_silence(np.zeros(0, F32), 24000, 0.25).size == 0


# ---- chunk.rs:327-357 ----------------------------------------------------
def test_crossfade_len_and_blend():
    y = A.crossfade_concat([np.ones(1000, F32), np.zeros(1000, F32)], 100)
    assert y.size == 1900
    assert y[899] == 1.0
    assert abs(y[900] - 1.0) < 1e-6              # t = 0: a
    assert abs(y[949] - 0.51) < 0.02             # t = 0.49
    assert abs(y[999] - 0.01) < 1e-5             # t = 0.99
    assert y[1000] == 0.0


def test_crossfade_three_chunks():
    y = A.crossfade_concat([np.full(500, 1.0, F32), np.full(500, 2.0, F32), np.full(500, 3.0, F32)], 50)
    assert y.size == 1400
    assert abs(y[0] - 1.0) < 1e-6 and abs(y[1399] - 3.0) < 1e-6


def test_crossfade_edge_cases():
    assert A.crossfade_concat([], 10).size == 0
    np.testing.assert_array_equal(A.crossfade_concat([np.array([1.0, 2.0], F32)], 10), [1.0, 2.0])
    assert A.crossfade_concat([np.ones(10, F32), np.zeros(10, F32)], 100).size == 11   # fade clamped


def test_crossfade_blend_is_f32_in_reference_order():
    a, b = speech(3000, 0.3), speech(3000, 0.2)[::-1].copy()
    y = A.crossfade_concat([a, b], 720)
    k = np.arange(720)
    t = (k.astype(F32) / F32(720))
    want = a[-720:] * (F32(1.0) - t) + b[:720] * t
    assert np.array_equal(y[3000 - 720:3000].view(np.uint32), want.view(np.uint32))


# ---- chunk.rs:359-444 ----------------------------------------------------
def test_trim_then_join_silent_seam():
    a = np.concatenate([np.full(12000, 0.1, F32), np.full(7200, 0.15, F32)])
    b = np.concatenate([np.full(7200, 0.15, F32), np.full(12000, 0.1, F32)])
    raw = A.crossfade_concat([a, b], 720)
    seam = raw[12000 + 7200 - 720:12000 + 7200 + 720]
    assert float(np.mean(seam.astype(np.float64) ** 2)) > 0.005
    fixed = A.crossfade_concat([A.trim_silence(a, 24000, 0.25), A.trim_silence(b, 24000, 0.25)], 720)
    assert fixed.size > 1440


def test_pad_tail_stays_untouched_when_silent():
    a = np.concatenate([speech(12000, 0.2), np.zeros(4800, F32)])   # 0.2 s of silence already
    p = A.pad_tail(a, 24000, 0.15)
    assert np.array_equal(p.view(np.uint32), a.view(np.uint32))


def test_pad_tail_hot_gets_digital_silence():
    a = speech(12000, 0.2)
    p = A.pad_tail(a, 24000, 0.15)
    assert p.size == 12000 + 3600                  # round(0.15 * 24000 in f32), not ceil
    assert np.all(p[12000:] == 0.0)
    np.testing.assert_array_equal(p[:12000], a)


def test_seam_pipeline_hot_hot():
    a, b = speech(19200, 0.2), speech(19200, 0.2)
    pa = A.pad_tail(A.trim_silence(a, 24000, 0.25), 24000, 0.15)
    tb = A.trim_silence(b, 24000, 0.25)
    joined = A.crossfade_concat([pa, tb], 720)
    assert np.all(pa[-720:] == 0.0)
    assert joined[pa.size - 720] == 0.0
    assert joined.size == pa.size + tb.size - 720


def test_join_chunks_follows_main_rs():
    a, b = speech(19200, 0.2), speech(9600, 0.1)
    np.testing.assert_array_equal(A.join_chunks([a]), a)
    np.testing.assert_array_equal(A.join_chunks([a], 0.25), A.trim_silence(a, 24000, 0.25))
    want = A.crossfade_concat([A.pad_tail(a), A.pad_tail(b)], 720)
    np.testing.assert_array_equal(A.join_chunks([a, b]), want)
    want = A.crossfade_concat([A.pad_tail(A.trim_silence(x, 24000, 0.25)) for x in (a, b)], 720)
    np.testing.assert_array_equal(A.join_chunks([a, b], 0.25), want)


# ---- wav.rs:7-46 ---------------------------------------------------------
def test_write_wav_layout(tmp_path):
    x = np.array([0.0, 0.5, -0.5, 1.0, -1.0, 2.0, -3.0, 1e-5, -0.99999, np.nan], F32)
    p = tmp_path / "a.wav"
    A.write_wav(p, x, 24000)
    raw = p.read_bytes()
    assert raw[:4] == b"RIFF" and raw[8:16] == b"WAVEfmt " and raw[36:40] == b"data"
    assert int.from_bytes(raw[4:8], "little") == 36 + 2 * x.size
    assert len(raw) == 44 + 2 * x.size
    with wave.open(str(p)) as w:
        assert (w.getnchannels(), w.getsampwidth(), w.getframerate(), w.getnframes()) == (1, 2, 24000, x.size)
        pcm = np.frombuffer(w.readframes(x.size), "<i2")
    # clamp, * 32767, truncate toward zero; NaN -> 0
    assert pcm.tolist() == [0, 16383, -16383, 32767, -32767, 32767, -32767, 0, -32766, 0]
