"""Model-level checks of the CPU oracle (tiny config, CPU only).

The reference ships no model-level golden vectors, so the oracle's talker
step (talker.rs:263-360), prefill (talker.rs:379-482) and predictor frame
(code_predictor.rs:218-513) are cross-checked against an independent float64
numpy restatement (np_ref.py) and against their own structural identities.
"""
import numpy as np
import pytest

import np_ref


@pytest.fixture(scope="module")
def tiny(orc):
    m = orc.Model.synth(orc.ModelConfig.tiny())
    return m, orc.OracleModel(m), np_ref.NpModel(m)


def test_talker_step_matches_numpy(orc, tiny):
    m, om, nm = tiny
    c = m.cfg
    kv = om.talker_kv()
    nkv = np_ref.NpKV(c.t_layers)
    for pos in range(6):
        emb = orc.synth_normal(100 + pos, 1.0, c.t_hidden)
        h, lg = om.talker_step(emb, kv, pos)
        hr, lr = nm.talker_step(emb, nkv, pos)
        assert np.max(np.abs(h - hr)) < 2e-4
        assert np.max(np.abs(lg - lr)) < 2e-4
    assert kv.len(0) == 6 and kv.len(c.t_layers - 1) == 6


def test_prefill_equals_stepwise_decode(orc, tiny):
    """prefill_talker_raw_from over T tokens == T single steps (tiny GEMVs are
    single-pass, so gemm and gemv share op order: bit-identical)."""
    m, om, _ = tiny
    c = m.cfg
    T = 5
    x = orc.synth_normal(7, 1.0, T * c.t_hidden).reshape(T, c.t_hidden)
    kv1 = om.talker_kv()
    h1 = om.talker_prefill(x, kv1, 0)
    kv2 = om.talker_kv()
    for t in range(T):
        h2, _ = om.talker_step(x[t], kv2, t)
    assert np.array_equal(h1, h2)
    for layer in range(c.t_layers):
        assert np.array_equal(kv1.k(layer)[:T], kv2.k(layer)[:T])
        assert np.array_equal(kv1.v(layer)[:T], kv2.v(layer)[:T])


def test_prefill_from_prefix_is_bit_identical(orc, tiny):
    """talker.rs:373-378: prefix-cache reuse gives the same bits as one full prefill."""
    m, om, _ = tiny
    c = m.cfg
    x = orc.synth_normal(8, 1.0, 9 * c.t_hidden).reshape(9, c.t_hidden)
    kv1 = om.talker_kv()
    h1 = om.talker_prefill(x, kv1, 0)
    kv2 = om.talker_kv()
    om.talker_prefill(x[:4], kv2, 0)
    h2 = om.talker_prefill(x[4:], kv2, 4)
    assert np.array_equal(h1, h2)


def test_predictor_frame_matches_numpy(orc, tiny):
    m, om, nm = tiny
    c = m.cfg
    hid = orc.synth_normal(11, 1.0, c.t_hidden)
    sem = om.embed_codec(17)
    kv = om.predictor_kv()
    codes, logits = om.predictor_frame(hid, sem, kv)
    # teacher-force numpy with the oracle's codes so both see the same inputs
    rcodes, rlogits = nm.predictor_frame(hid, sem, forced=codes)
    assert np.max(np.abs(logits - rlogits)) < 2e-4
    assert codes.shape == (c.p_groups,) and codes.max() < c.p_vocab
    assert kv.len(0) == c.p_groups + 1


def test_predictor_resets_kv(orc, tiny):
    m, om, _ = tiny
    c = m.cfg
    hid = orc.synth_normal(12, 1.0, c.t_hidden)
    sem = om.embed_codec(3)
    kv = om.predictor_kv()
    a, la = om.predictor_frame(hid, sem, kv)
    b, lb = om.predictor_frame(hid, sem, kv)
    assert np.array_equal(a, b) and np.array_equal(la, lb)


def test_frame_loop_runs(orc, tiny):
    m, om, _ = tiny
    c = m.cfg
    tkv, pkv = om.talker_kv(), om.predictor_kv()
    x = orc.synth_normal(13, 1.0, 4 * c.t_hidden).reshape(4, c.t_hidden)
    hidden = om.talker_prefill(x, tkv, 0)
    st = {"logits": om.codec_head(hidden), "hidden": hidden.copy(),
          "prev": np.zeros(16, np.uint32), "rng": 42}
    params = orc.SampleParams(0.9, 50, 1.0, 1.05)
    text = orc.synth_normal(14, 1.0, c.t_hidden)
    seen = []
    for f in range(3):
        codes = om.frame(tkv, pkv, params, text, 4 + f, st)
        assert codes[0] < c.t_vocab and codes[1:].max() < c.p_vocab
        assert np.array_equal(st["prev"], codes)
        seen.append(codes)
    assert tkv.len(0) == 7


def test_attend_step_matches_numpy(orc):
    """oq_attend_step (the attention block, talker.rs:285-331) vs the float64
    numpy restatement over a growing cache."""
    import np_ref
    heads, kvh, hd, steps = 4, 2, 64, 9
    rng = np.random.default_rng(3)
    qn = (1.0 + 0.1 * rng.standard_normal(hd)).astype(np.float16).view(np.uint16)
    kn = (1.0 + 0.1 * rng.standard_normal(hd)).astype(np.float16).view(np.uint16)
    cos, sin = orc.rope_tables(hd, 64, 1e6)
    kv = orc.KV(1, kvh, hd, 16)
    K, V = [], []
    for s in range(steps):
        q = rng.standard_normal(heads * hd).astype(np.float32)
        k = rng.standard_normal(kvh * hd).astype(np.float32)
        v = rng.standard_normal(kvh * hd).astype(np.float32)
        pos = 5 + 2 * s
        got = orc.attend_step(kv, 0, q, k, v, heads, kvh, hd, qn, kn, cos, sin, pos)
        qr = np_ref.rope(np_ref.qknorm(q.astype(np.float64), heads, hd, qn), heads, hd, pos)
        kr = np_ref.rope(np_ref.qknorm(k.astype(np.float64), kvh, hd, kn), kvh, hd, pos)
        K.append(kr.reshape(kvh, hd))
        V.append(v.astype(np.float64).reshape(kvh, hd))
        Ks, Vs = np.stack(K), np.stack(V)
        ref = np.zeros(heads * hd)
        for h in range(heads):
            sc = Ks[:, h // (heads // kvh)] @ qr[h * hd:(h + 1) * hd] / np.sqrt(hd)
            p = np.exp(sc - sc.max())
            ref[h * hd:(h + 1) * hd] = (p / p.sum()) @ Vs[:, h // (heads // kvh)]
        assert np.max(np.abs(got - ref)) < 1e-5
    assert kv.len(0) == steps


def test_embed_text_token_matches_numpy(orc):
    """oq_embed_text_token (talker.rs:104-116) against the float64 restatement,
    with fc1 widening the text hidden size (mid != text_hidden)."""
    tp = orc.TextProj.synth(61, text_vocab=50, text_hidden=128, hidden=96, mid=160, sigma=0.05)
    for tok in (0, 1, 17, 49):
        got = tp.embed_text_token(tok)
        ref = np_ref.embed_text_token(tp, tok)
        assert got.shape == (96,)
        assert np.max(np.abs(got - ref)) < 1e-5 * max(1.0, np.max(np.abs(ref)))


def test_talker_decode_is_embed_then_step(orc, tiny):
    """forward_talker_decode (talker.rs:161-258) = embed (text or codec path)
    then the layers of forward_with_embedding: same bits as composing them."""
    m, om, _ = tiny
    c = m.cfg
    tp = orc.TextProj.synth(62, 300, c.t_hidden, c.t_hidden)
    kv_a, kv_b = om.talker_kv(), om.talker_kv()
    for pos, (tok, is_text) in enumerate([(5, True), (17, False), (299, True), (0, False)]):
        got = om.talker_decode(tok, is_text, kv_a, pos, tp)
        emb = tp.embed_text_token(tok) if is_text else om.embed_codec(tok)
        want, _ = om.talker_step(emb, kv_b, pos)
        assert np.array_equal(got, want), pos
