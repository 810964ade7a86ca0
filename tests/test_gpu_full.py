"""Full-size parity at the BASELINE configs (1.7B dims, random-init Q4 weights).

Config 0: 28-layer talker, 32-token N(0,1) prefill
(seed 42), then 256 decode steps teacher-forced on the oracle's greedy argmax
(the step input is embed_codec_token(argmax), talker.rs:170-174, run through
forward_with_embedding, talker.rs:263-360).  Logits are compared at every
step: max-abs <= 2e-3, relative (max-abs / max |logit|) <= 1e-3, and >= 99.5 %
greedy-argmax agreement.

Config 2: all 512 code-predictor frames at head_dim 64
(BASELINE) and 128 (the reference's config.json), batch 1, teacher-forced on
the oracle's codes, same logit tolerances; code 0 per frame from xorshift64
(seed 7) mod 2048, talker hidden N(0,1) from seed 7 + frame.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ABS_TOL = 2e-3
REL_TOL = 1e-3
FRAMES2 = 512   # config 2: 512 predictor frames


@pytest.fixture(scope="module")
def E():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("-m gpu tests need a CUDA device")
    from qora_b200 import engine
    return engine


@pytest.fixture(scope="module")
def ctx(E):
    return E.Context(0)


def _cuda(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _cmp(got, ref):
    err = float(np.max(np.abs(got.astype(np.float64) - ref)))
    rel = err / max(1e-30, float(np.max(np.abs(ref))))
    return err, rel


def _oracle_from(orc, cfg, tw, pw):
    """Oracle view of the engine's host weights (same arrays, reference layout)."""
    def q(w):
        return orc.Q4Weight(w.packed, w.scales, w.k, w.n)

    def lay(lw):
        return orc.LayerWeights(q(lw.q_proj), q(lw.k_proj), q(lw.v_proj), q(lw.o_proj),
                                q(lw.gate_proj), q(lw.up_proj), q(lw.down_proj), lw.q_norm,
                                lw.k_norm, lw.input_norm, lw.post_attn_norm)

    ocfg = orc.ModelConfig(**{k: getattr(cfg, k) for k in orc.ModelConfig.__dataclass_fields__})
    half = cfg.t_head_dim // 2
    m = orc.Model(cfg=ocfg, t_layers=[lay(x) for x in tw.layers] if tw else [],
                  codec_embedding=q(tw.codec_embedding) if tw else None,
                  codec_head=q(tw.codec_head) if tw else None,
                  t_final_norm=tw.final_norm if tw else None,
                  t_rope=orc.rope_tables(cfg.t_head_dim, cfg.t_max_pos, cfg.rope_theta,
                                         [24, 20, 20] if half == 64 else [half]),
                  p_layers=[lay(x) for x in pw.layers] if pw else [],
                  input_proj=q(pw.input_proj) if pw and pw.input_proj is not None else None,
                  input_proj_bias=pw.input_proj_bias if pw else None,
                  codec_embeddings=[q(e) for e in pw.codec_embeddings] if pw else [],
                  lm_heads=[q(h) for h in pw.lm_heads] if pw else [],
                  p_final_norm=pw.final_norm if pw else None,
                  p_rope=orc.rope_tables(cfg.p_head_dim, cfg.p_max_pos, cfg.rope_theta))
    return m


def test_config0_talker_teacher_forced(E, ctx, orc):
    import qora_b200
    cfg = qora_b200.ModelConfig(t_max_pos=512)
    tw = qora_b200.synth_talker(cfg)
    om = orc.OracleModel.__new__(orc.OracleModel)
    om.m = _oracle_from(orc, cfg, tw, None)
    om.t = om.m.talker_struct()
    talker = E.Talker(ctx, tw, max_batch=1)
    kv, okv = talker.new_kv(max_pos=300), om.talker_kv(300)
    T, STEPS = 32, 256
    x = orc.synth_normal(42, 1.0, T * cfg.t_hidden).reshape(T, cfg.t_hidden)
    h = talker.prefill_talker_raw_from(_cuda(x), kv, 0)
    rh = om.talker_prefill(x, okv, 0)
    e, r = _cmp(h.cpu().numpy(), rh)
    assert e <= ABS_TOL, e
    rl = om.codec_head(rh)
    lg = talker.apply_codec_head(h).cpu().numpy()[0]
    worst_abs, worst_rel, agree = 0.0, 0.0, 0
    for step in range(STEPS):
        e, r = _cmp(lg, rl)
        worst_abs, worst_rel = max(worst_abs, e), max(worst_rel, r)
        agree += int(np.argmax(lg) == np.argmax(rl))
        tok = int(np.argmax(rl))                      # teacher forcing on the oracle
        emb = om.embed_codec(tok)
        _, glg = talker.forward_with_embedding(_cuda(emb), kv, [T + step])
        _, rl = om.talker_step(emb, okv, T + step)
        lg = glg.cpu().numpy()[0]
    e, r = _cmp(lg, rl)
    worst_abs, worst_rel = max(worst_abs, e), max(worst_rel, r)
    agree += int(np.argmax(lg) == np.argmax(rl))
    print(f"config0: worst abs {worst_abs:.3e} rel {worst_rel:.3e} argmax {agree}/{STEPS + 1}")
    assert worst_abs <= ABS_TOL and worst_rel <= REL_TOL
    assert agree / (STEPS + 1) >= 0.995
    assert list(kv.lengths()) == [T + STEPS]


@pytest.mark.parametrize("hd", [64, 128])
def test_config2_predictor_teacher_forced(E, ctx, orc, hd):
    import qora_b200
    cfg = qora_b200.ModelConfig(p_head_dim=hd)
    pw = qora_b200.synth_predictor(cfg)
    om = orc.OracleModel.__new__(orc.OracleModel)
    om.m = _oracle_from(orc, cfg, None, pw)
    om.p = om.m.predictor_struct()
    pred = E.CodePredictor(ctx, pw, max_batch=1)
    kv, okv = pred.new_kv(), om.predictor_kv()
    # semantic embeddings come from a codec_embedding table (talker.rs:152);
    # a dedicated random table of the same shape stands in here
    semtab = qora_b200.synth_q4(cfg.seed * 1000 + 900, cfg.sigma, cfg.t_vocab, cfg.t_hidden)
    st = 7
    worst_abs, worst_rel, agree, total = 0.0, 0.0, 0, 0
    for frame in range(FRAMES2):
        hid = orc.synth_normal(7 + frame, 1.0, cfg.t_hidden)
        st ^= (st << 13) & 0xFFFFFFFFFFFFFFFF
        st ^= st >> 7
        st ^= (st << 17) & 0xFFFFFFFFFFFFFFFF
        code0 = st % 2048
        sem = orc.embed_lookup(orc.Q4Weight(semtab.packed, semtab.scales, semtab.k, semtab.n), code0)
        rcodes, rlog = om.predictor_frame(hid, sem, okv)
        codes, glog = pred.generate_acoustic_codes(_cuda(hid[None]), _cuda(sem[None]), kv,
                                                   forced=rcodes.astype(np.int32)[None],
                                                   want_logits=True)
        glog = glog.cpu().numpy()[0]
        for g in range(cfg.p_groups):
            e, r = _cmp(glog[g], rlog[g])
            worst_abs, worst_rel = max(worst_abs, e), max(worst_rel, r)
        agree += int(np.sum(codes.cpu().numpy()[0] == rcodes))
        total += cfg.p_groups
    print(f"config2 hd{hd}: worst abs {worst_abs:.3e} rel {worst_rel:.3e} argmax {agree}/{total}")
    assert worst_abs <= ABS_TOL and worst_rel <= REL_TOL
    assert agree / total >= 0.995
