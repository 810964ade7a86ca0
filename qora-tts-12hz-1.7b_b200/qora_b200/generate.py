"""Host mirror of the reference's prompt construction and per-frame schedule
(generate_new.rs:24-128, 140-316, 361-466, 756-768).

The reference builds every prompt row on the CPU, calling embed_text_token once
per token.  Here the builders return row *recipes* (text token, codec codes or
the voice embedding); `PromptAssembler.assemble` projects all distinct text
tokens of the prompt in one qora_text_proj_embed call and builds every row in
one qora_prompt_assemble call, on the device.  Summation order follows the
reference, so rows match it bit for bit given the same text rows.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib

# Special token ids (generate_new.rs:24-35)
IM_START = 151644
ASSISTANT = 77091
NEWLINE = 198
TTS_PAD = 151671
TTS_BOS = 151672
TTS_EOS = 151673
CODEC_THINK = 2154
CODEC_THINK_BOS = 2156
CODEC_THINK_EOS = 2157
CODEC_PAD = 2148
CODEC_BOS = 2149
CODEC_EOS = 2150


@dataclass
class TTSParams:
    """TTSParams (generate_new.rs:38-79), the fields of the talker/predictor path."""
    max_codes: int = 1000
    temperature: float = 0.9
    top_k: int = 50
    top_p: float = 1.0
    repetition_penalty: float = 1.05
    codec_eos_id: int = CODEC_EOS
    codec_bos_id: int = CODEC_BOS
    onset_frames: int = 0
    onset_temperature: float = 0.3
    decode_warmup: bool = False      # warm the decoder up on the reference clip's codes
    warmup_frames: int = 0           # only their last N frames (0: all)

    def sample_params(self) -> _lib.SampleParams:
        return _lib.SampleParams(self.temperature, self.top_k, self.top_p, self.repetition_penalty)


def decoder_warmup(params: TTSParams, chain_codes=None, ref_codes=None):
    """The warm-up codes decode_to_audio gets (generate_new.rs:695-712):
    the previous chunk's tail of the same voice when there is one; else, with
    decode_warmup set, the reference clip's codes (their last warmup_frames
    frames when that is above 0); else None.  Codes are [num_quantizers][T]."""
    from .decoder import warmup_tail
    if chain_codes is not None:
        cc = np.asarray(chain_codes, dtype=np.uint32)
        if cc.ndim == 2 and cc.shape[0] > 0 and cc.shape[1] > 0:
            return cc
    if params.decode_warmup and ref_codes is not None:
        rc = np.asarray(ref_codes, dtype=np.uint32)
        return warmup_tail(rc, params.warmup_frames) if params.warmup_frames > 0 else rc
    return None


def frame_temperature(params: TTSParams, frame_idx: int) -> float:
    """frame_temperature (generate_new.rs:82-88): the onset schedule."""
    return params.onset_temperature if frame_idx < params.onset_frames else params.temperature


@dataclass
class IclLayout:
    icl_len: int
    remainder_len: int


def icl_block_layout(ref_t: int, text_t: int, tv: int) -> IclLayout:
    """icl_block_layout (generate_new.rs:120-128): text side R + T + 1 rows,
    codec side Tv + 1; a longer text side leaves a remainder."""
    text_len, codec_len = ref_t + text_t + 1, tv + 1
    return IclLayout(codec_len, text_len - codec_len if text_len > codec_len else 0)


def prefix_suffix_split(block_len: int, r: int, prefix_len: int) -> int | None:
    """prefix_suffix_split (generate_new.rs:307-316): the suffix to prefill on
    top of a cached 9 + R prefix, or None when the cache is unusable."""
    if prefix_len != 9 + r or r >= block_len:
        return None
    return block_len - r


@dataclass(frozen=True)
class Row:
    """One prompt row: text + codec (either optional).  `codes`: one talker
    codec token, or a reference frame of 16 codes (group 0 talker, 1..15
    predictor); `voice`: the voice embedding is the codec part."""
    text: int | None = None
    codes: tuple = ()
    voice: bool = False


def build_role_prefix() -> list:
    """build_role_prefix (generate_new.rs:91-97)."""
    return [Row(IM_START), Row(ASSISTANT), Row(NEWLINE)]


def build_tts_pad_bos(pad_count: int) -> list:
    """build_tts_pad_bos (generate_new.rs:100-108)."""
    return [Row(TTS_PAD)] * pad_count + [Row(TTS_BOS)]


def _frame(ref_codes, t) -> tuple:
    return tuple(int(ref_codes[g][t]) for g in range(16))


def _check_codes(ref_codes) -> int:
    if len(ref_codes) != 16:
        raise ValueError("ref_codes must have 16 codebooks")
    tv = len(ref_codes[0])
    if tv == 0 or any(len(c) != tv for c in ref_codes):
        raise ValueError("ref_codes must be non-empty and not ragged")
    return tv


def build_icl_block(ref_tokens, text_tokens, ref_codes):
    """build_icl_block (generate_new.rs:140-193): (icl rows, remainder rows)."""
    tv = _check_codes(ref_codes)
    text_full = [int(t) for t in list(ref_tokens) + list(text_tokens)] + [TTS_EOS]
    codec_full = [(CODEC_BOS,)] + [_frame(ref_codes, t) for t in range(tv)]
    if len(text_full) > len(codec_full):
        icl = [Row(a, b) for a, b in zip(text_full, codec_full)]
        rem = [Row(a) for a in text_full[len(codec_full):]]
    else:
        icl = [Row(text_full[i] if i < len(text_full) else TTS_PAD, b)
               for i, b in enumerate(codec_full)]
        rem = []
    return icl, rem


def build_codec_prefix_voice(language_id: int) -> list:
    """build_codec_prefix_voice (generate_new.rs:200-226): the voice row is
    position 4."""
    rows = [Row(TTS_PAD, (t,)) for t in (CODEC_THINK, CODEC_THINK_BOS, language_id,
                                         CODEC_THINK_EOS)]
    return rows + [Row(TTS_PAD, voice=True), Row(TTS_BOS, (CODEC_PAD,))]


def build_codec_prefix_builtin(speaker_id: int, language_id: int) -> list:
    """build_codec_prefix_builtin (generate_new.rs:229-242)."""
    toks = (CODEC_THINK, CODEC_THINK_BOS, language_id, CODEC_THINK_EOS, speaker_id, CODEC_PAD)
    ov = build_tts_pad_bos(5)
    return [Row(ov[i].text, (t,)) for i, t in enumerate(toks)]


def build_prefill_head(speaker_id: int, language_id: int, voice: bool) -> list:
    """build_prefill_head (generate_new.rs:245-259)."""
    return build_role_prefix() + (build_codec_prefix_voice(language_id) if voice
                                  else build_codec_prefix_builtin(speaker_id, language_id))


def build_icl_prefix(ref_tokens, ref_codes) -> list:
    """build_icl_prefix (generate_new.rs:266-300)."""
    tv = _check_codes(ref_codes)
    rows = []
    for i, tok in enumerate(ref_tokens):
        if i == 0:
            c = (CODEC_BOS,)
        elif i - 1 < tv:
            c = _frame(ref_codes, i - 1)
        else:  # R > Tv, never hit in practice (generate_new.rs:279-281)
            c = (CODEC_PAD,)
        rows.append(Row(int(tok), c))
    return rows


def prefill_custom_voice_rows(text_tokens, speaker_id: int, language_id: int, voice: bool,
                              icl_rows=None) -> list:
    """The rows prefill_custom_voice (generate_new.rs:361-466) prefills: role
    prefix, codec header, then the ICL block (voice path with ICL) or the
    BOS + first-text row (when there is text)."""
    rows = build_prefill_head(speaker_id, language_id, voice)
    if voice and icl_rows is not None:
        return rows + list(icl_rows)
    if len(text_tokens):
        rows.append(Row(int(text_tokens[0]), (CODEC_BOS,)))
    return rows


def build_trailing_text(text_tokens) -> list:
    """build_trailing_text (generate_new.rs:756-768)."""
    return [Row(int(t)) for t in list(text_tokens)[1:]] + [Row(TTS_EOS)]


def encode_rows(rows):
    """The recipes as qora_prompt_row structs (include/qora_cuda.h): returns
    (the distinct text tokens in ascending order, whose projected rows the
    structs index, and the struct array)."""
    toks = sorted({r.text for r in rows if r.text is not None})
    index = {t: i for i, t in enumerate(toks)}
    recs = (_lib.PromptRow * max(1, len(rows)))()
    for i, r in enumerate(rows):
        if len(r.codes) > 16 or (r.voice and r.codes):
            raise ValueError(f"row {i}: at most 16 codes, and none with the voice embedding")
        recs[i].text = -1 if r.text is None else index[r.text]
        if r.voice:
            recs[i].codes_n = -1
        else:
            recs[i].codes_n = len(r.codes)
            for g, c in enumerate(r.codes):
                recs[i].codes[g] = int(c)
    return toks, recs


class PromptAssembler:
    """Builds recipe rows on the device: `text_proj` an engine.TextProjection,
    `talker` an engine.Talker, `predictor` an engine.CodePredictor (needed for
    rows with reference frames)."""

    def __init__(self, text_proj, talker, predictor=None):
        self.tp, self.talker, self.predictor = text_proj, talker, predictor
        self.hidden = talker.cfg.t_hidden
        if text_proj.hidden != self.hidden:
            raise ValueError(f"text projection width {text_proj.hidden} != talker hidden {self.hidden}")

    # ---- device ----------------------------------------------------------
    def text_rows(self, tokens, stream=None):
        """embed_text_token of each token, [len(tokens)][hidden] on the device."""
        return self.tp.embed_text_tokens(tokens, stream=stream)

    def assemble(self, rows, voice=None, stream=None):
        """Every row of `rows` on the device, [len(rows)][hidden] f32.  `voice`:
        a device f32 vector (the voice embedding), needed when a row has
        voice=True."""
        import torch
        from .engine import _dp, _stream
        toks, recs = encode_rows(rows)
        dev = f"cuda:{self.talker.ctx.device}"
        text = self.text_rows(toks, stream=stream) if toks else None
        out = torch.empty(len(rows), self.hidden, device=dev)
        vlen = 0
        if voice is not None:
            voice = voice.reshape(-1).to(device=dev, dtype=torch.float32).contiguous()
            vlen = voice.numel()
        _lib.call("qora_prompt_assemble", self.talker.h,
                  self.predictor.h if self.predictor is not None else None,
                  _dp(text), len(toks), _dp(voice), vlen, C.addressof(recs), len(rows),
                  _dp(out), _stream(stream))
        return out

