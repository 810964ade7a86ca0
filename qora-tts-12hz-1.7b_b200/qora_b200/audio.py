"""After decode_to_audio: the reference's chunk assembly and WAV output.

main.rs:647-689 joins the chunks of a long text: each chunk's silences are
trimmed (when asked), its tail padded to 0.15 s of digital silence, and the
chunks crossfaded over 720 samples (30 ms); a single chunk is only trimmed.
The result is written as 16-bit PCM mono (wav.rs:7-46).  Restated here on
host arrays in the reference's f32 arithmetic: frame energies are summed in
order in f32 (20 ms frames, speech when the mean square is >= 1e-4), and the
f32 products, divisions, ceil and round of the reference are kept, so the
frame decisions and sample counts are the reference's own.
"""
from __future__ import annotations

import math

import numpy as np

F32 = np.float32
SAMPLE_RATE = 24000
CHUNK_FADE = 720          # main.rs:674: 30 ms at 24 kHz
CHUNK_TAIL_SECS = 0.15    # main.rs:665, 671
_SPEECH_ENERGY = F32(1e-4)


def _frame_energies(audio: np.ndarray, frame: int) -> np.ndarray:
    """Mean square of each 20 ms frame (the last may be short), each sum
    taken in order in f32 as the reference's iterator sum."""
    n = audio.size
    nf = -(-n // frame)
    out = np.empty(nf, F32)
    full = n // frame
    if full:
        sq = audio[:full * frame].reshape(full, frame) ** 2
        out[:full] = np.cumsum(sq, axis=1, dtype=F32)[:, -1] / F32(frame)
    if nf > full:
        seg = audio[full * frame:]
        out[full] = np.cumsum(seg * seg, dtype=F32)[-1] / F32(seg.size)
    return out


def _f32_audio(audio) -> np.ndarray:
    return np.ascontiguousarray(audio, dtype=F32).reshape(-1)


def trim_silence(audio, sample_rate: int = SAMPLE_RATE, max_gap_secs: float = 0.25) -> np.ndarray:
    """trim_silence (wav.rs:271-320): internal silences longer than
    max_gap_secs are cut to max_gap_secs and trailing silence beyond it is
    dropped; leading silence is kept.  All silence gives no samples."""
    x = _f32_audio(audio)
    if x.size == 0 or max_gap_secs <= 0.0:
        return x.copy()
    frame = max(sample_rate // 50, 1)
    max_gap = math.ceil(float((F32(max_gap_secs) * F32(sample_rate)) / F32(frame)))
    speech = _frame_energies(x, frame) >= _SPEECH_ENERGY
    if not speech.any():
        return np.zeros(0, F32)
    last = int(np.flatnonzero(speech)[-1])
    keep_frames = min(last + 1 + max_gap, speech.size)
    keep = np.zeros(speech.size, bool)
    run = 0
    for i in range(keep_frames):
        if speech[i]:
            keep[i], run = True, 0
        else:
            keep[i] = run < max_gap
            run += 1
    parts = [x[i * frame:(i + 1) * frame] for i in np.flatnonzero(keep)]
    return np.concatenate(parts).astype(F32, copy=False) if parts else np.zeros(0, F32)


def pad_tail(audio, sample_rate: int = SAMPLE_RATE, min_tail_secs: float = CHUNK_TAIL_SECS) -> np.ndarray:
    """pad_tail (chunk.rs:154-186): make the chunk end in at least
    min_tail_secs of silence, appending exact zeros for the deficit (a tail
    already silent that long is returned unchanged)."""
    x = _f32_audio(audio)
    if x.size == 0 or min_tail_secs <= 0.0:
        return x.copy()
    frame = max(sample_rate // 50, 1)
    e = _frame_energies(x, frame)
    loud = np.flatnonzero(e >= _SPEECH_ENERGY)
    sil = e.size - 1 - int(loud[-1]) if loud.size else e.size
    have_secs = (F32(sil) * F32(frame)) / F32(sample_rate)
    if have_secs >= F32(min_tail_secs):
        return x.copy()
    target = int(math.floor(float(F32(min_tail_secs) * F32(sample_rate)) + 0.5))   # f32 round, half away
    need = max(target - min(sil * frame, x.size), 0)
    if need == 0:
        return x.copy()
    return np.concatenate([x, np.zeros(need, F32)])


def crossfade_concat(chunks, fade_len: int = CHUNK_FADE) -> np.ndarray:
    """crossfade_concat (chunk.rs:187-214): the chunks joined with a linear
    crossfade of fade_len samples at each seam (clamped below the shortest
    chunk); length = sum - fade * (n - 1)."""
    cs = [_f32_audio(c) for c in chunks]
    if not cs:
        return np.zeros(0, F32)
    if len(cs) == 1:
        return cs[0].copy()
    fade = min(fade_len, max(min(c.size for c in cs) - 1, 0))
    if fade == 0:
        return np.concatenate(cs)
    t = np.arange(fade, dtype=F32) / F32(fade)
    parts = [cs[0][:cs[0].size - fade]]
    for i in range(len(cs) - 1):
        a, b = cs[i], cs[i + 1]
        parts.append(a[a.size - fade:] * (F32(1.0) - t) + b[:fade] * t)
        parts.append(b[fade:b.size if i + 2 == len(cs) else b.size - fade])
    return np.concatenate(parts).astype(F32, copy=False)


def join_chunks(audios, trim_silence_secs: float = 0.0, sample_rate: int = SAMPLE_RATE) -> np.ndarray:
    """main.rs:647-689: several chunks are each trimmed (trim_silence_secs >
    0), tail-padded to 0.15 s and crossfaded over 720 samples; a single
    chunk is trimmed only."""
    audios = [_f32_audio(a) for a in audios]
    if len(audios) > 1:
        if trim_silence_secs > 0.0:
            audios = [trim_silence(a, sample_rate, trim_silence_secs) for a in audios]
        return crossfade_concat([pad_tail(a, sample_rate, CHUNK_TAIL_SECS) for a in audios], CHUNK_FADE)
    if not audios:
        return np.zeros(0, F32)
    a = audios[0]
    return trim_silence(a, sample_rate, trim_silence_secs) if trim_silence_secs > 0.0 else a.copy()


def write_wav(path, samples, sample_rate: int = SAMPLE_RATE) -> None:
    """write_wav (wav.rs:7-46): 16-bit PCM mono; a sample is clamped to
    [-1, 1], scaled by 32767 and truncated toward zero (NaN -> 0, as the
    reference's saturating cast)."""
    x = _f32_audio(samples)
    v = np.clip(x, F32(-1.0), F32(1.0)) * F32(32767.0)
    pcm = np.where(np.isnan(v), F32(0.0), v).astype("<i2")
    data = pcm.tobytes()
    hdr = b"".join([
        b"RIFF", (36 + len(data)).to_bytes(4, "little"), b"WAVE",
        b"fmt ", (16).to_bytes(4, "little"), (1).to_bytes(2, "little"), (1).to_bytes(2, "little"),
        int(sample_rate).to_bytes(4, "little"), (int(sample_rate) * 2).to_bytes(4, "little"),
        (2).to_bytes(2, "little"), (16).to_bytes(2, "little"),
        b"data", len(data).to_bytes(4, "little"),
    ])
    with open(path, "wb") as f:
        f.write(hdr)
        f.write(data)
