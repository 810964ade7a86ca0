"""Host side of prompt construction (generate_new.rs:82-128, 140-316,
361-466, 756-768), on the CPU.

1. The reference's own unit tests of the layout rules (generate_new.rs:868-899
   icl_block_layout, 957-969 frame_temperature, 985-1005 prefix_suffix_split),
   restated as known answers, for the product and for the oracle.
2. Every recipe builder, evaluated with the qora_prompt_row rule (row = text +
   codec; a frame's codec part summed group 0 first) in numpy, equals the
   oracle's restatement of the reference builder bit for bit.
"""
import numpy as np
import pytest

import prompt_ref as R
from qora_b200 import generate as G

LAYOUT = [((8, 8, 23), (24, 0)), ((30, 30, 23), (24, 37)), ((11, 11, 22), (23, 0)),
          ((1, 1, 23), (24, 0))]                              # generate_new.rs:868-899
SPLIT = [((162, 35, 44), 127), ((162, 35, 43), None), ((35, 35, 44), None),
         ((30, 35, 44), None), ((162, 0, 9), 162)]            # generate_new.rs:985-1005


@pytest.mark.parametrize("args,want", LAYOUT)
def test_icl_block_layout_known_answers(args, want):
    l = G.icl_block_layout(*args)
    assert (l.icl_len, l.remainder_len) == want
    assert R.icl_block_layout(*args) == want


@pytest.mark.parametrize("args,want", SPLIT)
def test_prefix_suffix_split_known_answers(args, want):
    assert G.prefix_suffix_split(*args) == want
    assert R.prefix_suffix_split(*args) == want


def test_frame_temperature_known_answers():
    """generate_new.rs:957-969."""
    p = G.TTSParams(temperature=0.8, onset_frames=8, onset_temperature=0.3)
    for f, want in ((0, 0.3), (7, 0.3), (8, 0.8), (500, 0.8)):
        assert G.frame_temperature(p, f) == want
        assert R.frame_temperature(0.8, 8, 0.3, f) == want
    p.onset_frames = 0
    assert G.frame_temperature(p, 0) == 0.8
    assert G.TTSParams().onset_frames == 0 and G.TTSParams().temperature == 0.9


H = 48


def _vec(kind, *key):
    seed = abs(hash((kind,) + key)) % (2 ** 32)
    return np.random.default_rng(seed).standard_normal(H).astype(np.float32)


def _text(t):
    return _vec("text", int(t))


def _codec(t):
    return _vec("codec", int(t))


def _acoustic(g, c):
    return _vec("acoustic", int(g), int(c))


def _eval(rows, voice=None):
    """qora_prompt_row semantics (include/qora_cuda.h) in numpy float32."""
    out = []
    for r in rows:
        text = _text(r.text) if r.text is not None else None
        if r.voice:
            v = np.zeros(H, np.float32)
            n = min(H, len(voice))
            v[:n] = voice[:n] + text[:n] if text is not None else voice[:n]
        elif r.codes:
            c = _codec(r.codes[0]).copy()
            for g in range(1, len(r.codes)):
                c += _acoustic(g - 1, r.codes[g])
            v = text + c if text is not None else c
        else:
            v = text.copy() if text is not None else np.zeros(H, np.float32)
        out.append(v)
    return out


def _same(rows_a, rows_b):
    assert len(rows_a) == len(rows_b)
    for i, (a, b) in enumerate(zip(rows_a, rows_b)):
        assert np.array_equal(a, b), i


@pytest.fixture(scope="module")
def ref():
    return R.PromptRef(_text, _codec, _acoustic, H)


def _codes(tv, seed=3):
    rng = np.random.default_rng(seed)
    return [list(rng.integers(0, 2048, size=tv)) for _ in range(16)]


def test_role_prefix_and_overlay(ref):
    _same(_eval(G.build_role_prefix()), ref.role_prefix())
    _same(_eval(G.build_tts_pad_bos(5)), ref.tts_pad_bos(5))


@pytest.mark.parametrize("vlen", [H, H - 17, H + 9])
def test_codec_headers(ref, vlen):
    voice = np.random.default_rng(vlen).standard_normal(vlen).astype(np.float32)
    _same(_eval(G.build_codec_prefix_voice(2050), voice), ref.codec_prefix_voice(2050, voice))
    _same(_eval(G.build_codec_prefix_builtin(3001, 2050)), ref.codec_prefix_builtin(3001, 2050))
    _same(_eval(G.build_prefill_head(3001, 2050, True), voice), ref.prefill_head(3001, 2050, voice))
    _same(_eval(G.build_prefill_head(3001, 2050, False)), ref.prefill_head(3001, 2050))


@pytest.mark.parametrize("r,t,tv", [(2, 3, 9), (4, 9, 5), (11, 11, 22), (1, 0, 1)])
def test_icl_block_both_branches(ref, r, t, tv):
    rt = list(range(100, 100 + r))
    tt = list(range(500, 500 + t))
    codes = _codes(tv)
    icl, rem = G.build_icl_block(rt, tt, codes)
    ricl, rrem = ref.icl_block(rt, tt, codes)
    _same(_eval(icl), ricl)
    _same(_eval(rem), rrem)
    l = G.icl_block_layout(r, t, tv)
    assert (len(icl), len(rem)) == (l.icl_len, l.remainder_len)


@pytest.mark.parametrize("r,tv", [(5, 9), (6, 3), (1, 4)])
def test_icl_prefix(ref, r, tv):
    """Includes R > Tv, where rows past the frames take CODEC_PAD."""
    rt = list(range(300, 300 + r))
    codes = _codes(tv, seed=r)
    _same(_eval(G.build_icl_prefix(rt, codes)), ref.icl_prefix(rt, codes))


def test_prefill_rows_every_mode(ref):
    voice = np.random.default_rng(9).standard_normal(H).astype(np.float32)
    text = [901, 902, 903]
    codes = _codes(4)
    icl, _ = G.build_icl_block([77, 78], text, codes)
    ricl, _ = ref.icl_block([77, 78], text, codes)
    for tokens in (text, []):
        _same(_eval(G.prefill_custom_voice_rows(tokens, 3001, 2050, False)),
              ref.prefill_rows(tokens, 3001, 2050))
        _same(_eval(G.prefill_custom_voice_rows(tokens, 3001, 2050, True), voice),
              ref.prefill_rows(tokens, 3001, 2050, voice))
    _same(_eval(G.prefill_custom_voice_rows(text, 3001, 2050, True, icl), voice),
          ref.prefill_rows(text, 3001, 2050, voice, ricl))
    # the prefix cache's chunk-independent head: prefill head + ICL prefix
    # equals the first 9 + R rows of the full ICL prefill (generate_new.rs:330-355)
    full = G.prefill_custom_voice_rows(text, 3001, 2050, True, icl)
    head = G.build_prefill_head(3001, 2050, True) + G.build_icl_prefix([77, 78], codes)
    _same(_eval(head, voice), _eval(full[:len(head)], voice))


def test_trailing_text(ref):
    _same(_eval(G.build_trailing_text([5, 6, 7])), ref.trailing_text([5, 6, 7]))
    _same(_eval(G.build_trailing_text([])), ref.trailing_text([]))


def test_bad_reference_codes_are_errors():
    with pytest.raises(ValueError):
        G.build_icl_block([1], [2], _codes(3)[:15])
    ragged = _codes(3)
    ragged[4] = ragged[4][:2]
    with pytest.raises(ValueError):
        G.build_icl_prefix([1, 2], ragged)


def test_recipes_encode_as_prompt_rows():
    """encode_rows: the qora_prompt_row structs the device assembly reads
    (text index into the sorted distinct tokens, -1 none; codes_n 1 / 16 /
    0, -1 for the voice row)."""
    codes = _codes(2, 7)
    rows = G.build_codec_prefix_voice(2050) + G.build_icl_prefix([9, 5], codes) + [G.Row()]
    toks, recs = G.encode_rows(rows)
    assert toks == sorted({G.TTS_PAD, G.TTS_BOS, 9, 5})
    got = [(recs[i].text, recs[i].codes_n, list(recs[i].codes)[:max(recs[i].codes_n, 0)])
           for i in range(len(rows))]
    ix = {t: i for i, t in enumerate(toks)}
    assert got[0] == (ix[G.TTS_PAD], 1, [G.CODEC_THINK])
    assert got[4] == (ix[G.TTS_PAD], -1, [])                  # the voice row
    assert got[5] == (ix[G.TTS_BOS], 1, [G.CODEC_PAD])
    assert got[6] == (ix[9], 1, [G.CODEC_BOS])                # ICL prefix row 0
    assert got[7] == (ix[5], 16, [int(codes[g][0]) for g in range(16)])
    assert got[8] == (-1, 0, [])
    with pytest.raises(ValueError):
        G.encode_rows([G.Row(1, tuple(range(17)))])
