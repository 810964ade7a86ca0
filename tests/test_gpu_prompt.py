"""GPU parity of prompt assembly (generate_new.rs:91-466, 756-768): rows built
on the device by qora_text_proj_embed + qora_prompt_assemble against the
oracle's restatement of the reference builders (oracle/prompt_ref.py).

With the oracle fed the device's own text-projection rows the assembled rows
are bit-identical (the assembly is elementwise f32 adds in the reference's
order); with the oracle's text projection they agree within the GEMV
tolerance.  The assembled prompt then drives prefill and frames, matching the
oracle's frame loop on the same rows."""
import numpy as np
import pytest

import prompt_ref as R

pytestmark = pytest.mark.gpu

TEXT_VOCAB = 151936  # config.rs:138: the special tokens sit at its top


@pytest.fixture(scope="module")
def setup(orc):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("-m gpu tests need a CUDA device")
    import qora_b200
    from qora_b200 import engine as E
    from qora_b200 import generate as G
    kw = dict(t_vocab=3072, p_vocab=2048)  # the reference's codec vocabularies
    cfg = qora_b200.ModelConfig.tiny(**kw)
    tw, pw = qora_b200.synth_talker(cfg), qora_b200.synth_predictor(cfg)
    tpo = orc.TextProj.synth(77, TEXT_VOCAB, cfg.t_hidden, cfg.t_hidden, sigma=0.05)
    q = lambda w: qora_b200.Q4Weight(w.packed, w.scales, w.k, w.n)
    tpw = qora_b200.TextProjWeights(q(tpo.text_embedding), q(tpo.fc1), tpo.fc1_bias, q(tpo.fc2),
                                    tpo.fc2_bias)
    ctx = E.Context(0)
    talker, pred = E.Talker(ctx, tw), E.CodePredictor(ctx, pw)
    tp = E.TextProjection(ctx, tpw)
    asm = G.PromptAssembler(tp, talker, pred)
    om = orc.OracleModel(orc.Model.synth(orc.ModelConfig.tiny(**kw)))
    codec = lambda t: orc.embed_lookup(om.m.codec_embedding, int(t))
    acoustic = lambda g, c: orc.embed_lookup(om.m.codec_embeddings[g], int(c))
    return dict(E=E, G=G, cfg=cfg, ctx=ctx, talker=talker, pred=pred, tp=tp, tpo=tpo, asm=asm,
                om=om, codec=codec, acoustic=acoustic)


SPECIAL = [R.IM_START, R.ASSISTANT, R.NEWLINE, R.TTS_PAD, R.TTS_BOS, R.TTS_EOS]


def _device_ref(s, tokens):
    """The oracle builders over the device's text rows of `tokens` (every text
    token the builders under test can ask for)."""
    toks = sorted(set(int(t) for t in tokens) | set(SPECIAL))
    dev = s["asm"].text_rows(toks).cpu().numpy()
    table = {t: dev[i] for i, t in enumerate(toks)}
    return R.PromptRef(lambda t: table[int(t)], s["codec"], s["acoustic"], s["cfg"].t_hidden)


def _codes(tv, seed):
    rng = np.random.default_rng(seed)
    return [list(rng.integers(0, 3072 if g == 0 else 2048, size=tv)) for g in range(16)]


def _same(got, want):
    assert got.shape[0] == len(want)
    for i, w in enumerate(want):
        assert np.array_equal(got[i], w), i


def test_every_builder_bit_exact(setup):
    import torch
    s = setup
    G, asm, H = s["G"], s["asm"], s["cfg"].t_hidden
    text = [9707, 11, 1879, 0, 151643]
    codes = _codes(6, 1)
    ref = _device_ref(s, text + [5, 6, 7] + list(range(30, 49)))
    for vlen in (H, H - 40, H + 24):
        voice = np.random.default_rng(vlen).standard_normal(vlen).astype(np.float32)
        vt = torch.from_numpy(voice).cuda()
        cases = [
            (G.build_role_prefix(), lambda r: r.role_prefix()),
            (G.build_tts_pad_bos(5), lambda r: r.tts_pad_bos(5)),
            (G.build_codec_prefix_voice(2050), lambda r: r.codec_prefix_voice(2050, voice)),
            (G.build_codec_prefix_builtin(3001, 2050), lambda r: r.codec_prefix_builtin(3001, 2050)),
            (G.build_prefill_head(3001, 2050, True), lambda r: r.prefill_head(3001, 2050, voice)),
            (G.build_icl_prefix([5, 6, 7], codes), lambda r: r.icl_prefix([5, 6, 7], codes)),
            (G.build_icl_prefix(list(range(40, 49)), codes),          # R > Tv: PAD rows
             lambda r: r.icl_prefix(list(range(40, 49)), codes)),
            (G.build_trailing_text(text), lambda r: r.trailing_text(text)),
            (G.prefill_custom_voice_rows(text, 3001, 2050, False),
             lambda r: r.prefill_rows(text, 3001, 2050)),
            (G.prefill_custom_voice_rows(text, 3001, 2050, True),
             lambda r: r.prefill_rows(text, 3001, 2050, voice)),
            (G.prefill_custom_voice_rows([], 3001, 2050, True),
             lambda r: r.prefill_rows([], 3001, 2050, voice)),
        ]
        for ref_t, txt in (([5, 6], text), (list(range(30, 42)), text)):   # pad / remainder branch
            icl, rem = G.build_icl_block(ref_t, txt, codes)
            cases.append((icl + rem, lambda r, a=ref_t, b=txt: sum(r.icl_block(a, b, codes), [])))
            cases.append((G.prefill_custom_voice_rows(txt, 3001, 2050, True, icl),
                          lambda r, a=ref_t, b=txt: r.prefill_rows(
                              b, 3001, 2050, voice, r.icl_block(a, b, codes)[0])))
        for rows, build in cases:
            got = asm.assemble(rows, voice=vt).cpu().numpy()
            _same(got, build(ref))
    s["ctx"].check_device_error()


def test_rows_match_oracle_text_projection(setup):
    """End to end against the oracle's own embed_text_token (GEMV tolerance)."""
    s = setup
    G = s["G"]
    text = [4, 151000, 88]
    codes = _codes(3, 2)
    icl, rem = G.build_icl_block([17, 18], text, codes)
    rows = G.prefill_custom_voice_rows(text, 3001, 2050, False) + icl + rem
    got = s["asm"].assemble(rows).cpu().numpy()
    ref = R.PromptRef(s["tpo"].embed_text_token, s["codec"], s["acoustic"], s["cfg"].t_hidden)
    want = np.stack(ref.prefill_rows(text, 3001, 2050) + sum(ref.icl_block([17, 18], text, codes), []))
    scale = max(1.0, float(np.max(np.abs(want))))
    assert float(np.max(np.abs(got - want))) <= 1e-4 * scale


def test_bad_rows_are_errors(setup):
    import torch
    from qora_b200 import _lib
    s = setup
    G, E = s["G"], s["E"]
    asm = s["asm"]
    bad = [
        ([G.Row(None, (3072,))], 5),                       # codec token past the table
        ([G.Row(None, (1,) + (2048,) + (0,) * 14)], 5),     # acoustic code past its table
        ([G.Row(TEXT_VOCAB)], 5),                           # text token past the vocabulary
        ([G.Row(None, voice=True)], 1),                     # voice row, no voice given
    ]
    for rows, status in bad:
        with pytest.raises(_lib.QoraError) as ei:
            asm.assemble(rows)
        assert ei.value.status == status, rows
    no_pred = G.PromptAssembler(s["tp"], s["talker"], None)
    with pytest.raises(_lib.QoraError) as ei:
        no_pred.assemble(G.build_icl_prefix([1, 2], _codes(2, 3)))
    assert ei.value.status == 1
    assert no_pred.assemble(G.build_role_prefix()).shape == (3, s["cfg"].t_hidden)
    s["ctx"].check_device_error()


def test_assembled_prompt_drives_frames(setup, orc):
    """ICL prompt -> prefill -> 4 frames with the remainder as trailing text:
    the engine's codes equal the oracle frame loop's on the same rows."""
    import torch
    s = setup
    G, E, om, cfg = s["G"], s["E"], s["om"], s["cfg"]
    text = [12, 13, 14, 15, 16, 17, 18]
    codes = _codes(3, 4)
    voice = np.random.default_rng(5).standard_normal(cfg.t_hidden).astype(np.float32)
    icl, rem = G.build_icl_block([21, 22], text, codes)
    prompt = G.prefill_custom_voice_rows(text, 3001, 2050, True, icl)
    x = s["asm"].assemble(prompt, voice=torch.from_numpy(voice).cuda()).cpu().numpy()
    trailing = s["asm"].assemble(rem + [G.Row(G.TTS_PAD)]).cpu().numpy()
    T = x.shape[0]
    eng = E.Engine(s["talker"], s["pred"], 1, max_pos=T + 8)
    eng.prefill(x.reshape(1, T, -1), [31])
    tkv, pkv = om.talker_kv(T + 8), om.predictor_kv()
    hdn = om.talker_prefill(x, tkv, 0)
    st = {"logits": om.codec_head(hdn), "hidden": hdn.copy(), "prev": np.zeros(16, np.uint32),
          "rng": 31}
    oparams = orc.SampleParams(0.9, 50, 1.0, 1.05)   # TTSParams::default (engine default)
    out = np.zeros((1, 16), np.int32)
    for f in range(4):
        row = trailing[min(f, len(trailing) - 1)]   # remainder rows, then TTS_PAD
        eng.frame_host(row.reshape(1, -1).copy(), out)
        ref = om.frame(tkv, pkv, oparams, row, T + f, st)
        assert list(out[0]) == list(ref), f
