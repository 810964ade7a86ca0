"""Prompt assembly ORACLE: the reference's talker-prompt builders
(swordreforge/QORA-TTS-12Hz-1.7B, src/generate_new.rs:82-466, 756-768)
restated in numpy float32, with the reference's summation order.

TEST INFRASTRUCTURE ONLY.  Only tests/ may import this module, as the checker
of the engine's prompt assembly; the product never calls it.

Parity pin: the reference's own unit tests of the pure layout rules
(generate_new.rs:868-899 icl_block_layout, 957-969 frame_temperature,
985-1005 prefix_suffix_split) are restated as known-answer tests in
tests/test_prompt_host.py.  The row builders have no golden vectors in the
reference; they are restated line by line from the cited code.

Embedding sources are callables so that the checker can run on the oracle's
own text projection or on rows the device produced:
  text(token)          -> f32[hidden]  embed_text_token (talker.rs:104-116)
  codec(token)         -> f32[hidden]  embed_codec_token (talker.rs:152-154)
  acoustic(g, code)    -> f32[hidden]  get_acoustic_embedding (code_predictor.rs:279-282)
"""
from __future__ import annotations

import numpy as np

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


def frame_temperature(temperature: float, onset_frames: int, onset_temperature: float,
                      frame_idx: int) -> float:
    """generate_new.rs:82-88."""
    return onset_temperature if frame_idx < onset_frames else temperature


def icl_block_layout(ref_t: int, text_t: int, tv: int):
    """generate_new.rs:120-128: (icl_len, remainder_len)."""
    text_len = ref_t + text_t + 1
    codec_len = tv + 1
    if text_len > codec_len:
        return codec_len, text_len - codec_len
    return codec_len, 0


def prefix_suffix_split(block_len: int, r: int, prefix_len: int):
    """generate_new.rs:307-316: suffix length, or None."""
    if prefix_len != 9 + r:
        return None
    return block_len - r if r < block_len else None


class PromptRef:
    def __init__(self, text, codec, acoustic, hidden: int):
        self.text, self.codec, self.acoustic, self.hidden = text, codec, acoustic, hidden

    def _t(self, tok):
        return np.asarray(self.text(tok), np.float32)

    def _c(self, tok):
        return np.asarray(self.codec(tok), np.float32)

    def _frame_sum(self, ref_codes, t):
        """codec side of one reference frame (generate_new.rs:164-169)."""
        s = self._c(ref_codes[0][t]).copy()
        for g in range(1, 16):
            s += np.asarray(self.acoustic(g - 1, ref_codes[g][t]), np.float32)
        return s

    def role_prefix(self):
        """build_role_prefix (generate_new.rs:91-97)."""
        return [self._t(IM_START), self._t(ASSISTANT), self._t(NEWLINE)]

    def tts_pad_bos(self, pad_count):
        """build_tts_pad_bos (generate_new.rs:100-108)."""
        pad = self._t(TTS_PAD)
        return [pad.copy() for _ in range(pad_count)] + [self._t(TTS_BOS)]

    def icl_block(self, ref_tokens, text_tokens, ref_codes):
        """build_icl_block (generate_new.rs:140-193): (icl, remainder)."""
        assert len(ref_codes) == 16
        tv = len(ref_codes[0])
        assert tv > 0 and all(len(c) == tv for c in ref_codes)
        tts_pad = self._t(TTS_PAD)
        tts_eos = self._t(TTS_EOS)
        text_full = [self._t(t) for t in list(ref_tokens) + list(text_tokens)] + [tts_eos]
        codec_full = [self._c(CODEC_BOS)] + [self._frame_sum(ref_codes, t) for t in range(tv)]
        if len(text_full) > len(codec_full):
            icl = [a + b for a, b in zip(text_full[:len(codec_full)], codec_full)]
            rem = text_full[len(codec_full):]
        else:
            icl = [(text_full[i] if i < len(text_full) else tts_pad) + b
                   for i, b in enumerate(codec_full)]
            rem = []
        assert (len(icl), len(rem)) == icl_block_layout(len(ref_tokens), len(text_tokens), tv)
        return icl, rem

    def codec_prefix_voice(self, language_id, voice):
        """build_codec_prefix_voice (generate_new.rs:200-226)."""
        h = self.hidden
        pad, bos = self._t(TTS_PAD), self._t(TTS_BOS)
        out = [self._c(t) + pad for t in (CODEC_THINK, CODEC_THINK_BOS, language_id, CODEC_THINK_EOS)]
        pos4 = np.zeros(h, np.float32)
        n = min(h, len(voice))
        pos4[:n] = np.asarray(voice, np.float32)[:n] + pad[:n]
        out.append(pos4)
        out.append(self._c(CODEC_PAD) + bos)
        return out

    def codec_prefix_builtin(self, speaker_id, language_id):
        """build_codec_prefix_builtin (generate_new.rs:229-242)."""
        toks = (CODEC_THINK, CODEC_THINK_BOS, language_id, CODEC_THINK_EOS, speaker_id, CODEC_PAD)
        emb = [self._c(t) for t in toks]
        ov = self.tts_pad_bos(5)
        return [emb[i] + ov[i] for i in range(6)]

    def prefill_head(self, speaker_id, language_id, voice=None):
        """build_prefill_head (generate_new.rs:245-259)."""
        head = self.role_prefix()
        if voice is not None:
            head += self.codec_prefix_voice(language_id, voice)
        else:
            head += self.codec_prefix_builtin(speaker_id, language_id)
        return head

    def icl_prefix(self, ref_tokens, ref_codes):
        """build_icl_prefix (generate_new.rs:266-300)."""
        tv = len(ref_codes[0])
        out = []
        for i, tok in enumerate(ref_tokens):
            if i == 0:
                c = self._c(CODEC_BOS)
            elif i - 1 < tv:
                c = self._frame_sum(ref_codes, i - 1)
            else:
                c = self._c(CODEC_PAD)
            out.append(self._t(tok) + c)
        return out

    def prefill_rows(self, text_tokens, speaker_id, language_id, voice=None, icl=None):
        """The rows prefill_custom_voice (generate_new.rs:361-466) prefills."""
        rows = self.role_prefix()
        if voice is not None:
            rows += self.codec_prefix_voice(language_id, voice)
            if icl is not None:
                rows += [r.copy() for r in icl]
            elif len(text_tokens):
                rows.append(self._c(CODEC_BOS) + self._t(text_tokens[0]))
        else:
            toks = (CODEC_THINK, CODEC_THINK_BOS, language_id, CODEC_THINK_EOS, speaker_id, CODEC_PAD)
            emb = [self._c(t) for t in toks]
            ov = self.tts_pad_bos(5)
            rows += [emb[i] + ov[i] for i in range(6)]
            if len(text_tokens):
                rows.append(self._c(CODEC_BOS) + self._t(text_tokens[0]))
        return rows

    def trailing_text(self, text_tokens):
        """build_trailing_text (generate_new.rs:756-768)."""
        return [self._t(t) for t in list(text_tokens)[1:]] + [self._t(TTS_EOS)]
