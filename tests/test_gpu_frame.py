"""The persistent frame kernel (one launch per batch-1 frame) against the CPU
oracle's frame loop (generate_new.rs:606-665) and against the per-op kernel
sequence, through the C ABI.

Codes (sampled code 0 + 15 greedy acoustic codes) must be identical; the
talker logits the next frame samples from are held to the same tolerances as
the other model tests (tiny model 2e-4 absolute; 1.7B dims max-abs 2e-3 and
relative 1e-3)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TINY_TOL = 2e-4
ABS_TOL, REL_TOL = 2e-3, 1e-3


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


def _run(E, orc, ctx, cfg, tw, pw, om, T, F, persistent, seed=500, check_logits=None):
    import torch
    talker = E.Talker(ctx, tw, max_batch=1)
    pred = E.CodePredictor(ctx, pw, max_batch=1)
    eng = E.Engine(talker, pred, 1, max_pos=T + F + 4)
    eng.use_persistent(persistent)
    x = orc.synth_normal(seed, 1.0, T * cfg.t_hidden).reshape(1, T, cfg.t_hidden)
    eng.prefill(x, [seed + 1])
    text = orc.synth_normal(seed + 2, 1.0, cfg.t_hidden).reshape(1, cfg.t_hidden)
    tkv, pkv = om.talker_kv(T + F + 4), om.predictor_kv()
    hdn = om.talker_prefill(x[0], tkv, 0)
    st = {"logits": om.codec_head(hdn), "hidden": hdn.copy(), "prev": np.zeros(16, np.uint32),
          "rng": seed + 1}
    codes = torch.zeros(1, 16, dtype=torch.int32, device="cuda")
    for f in range(F):
        eng.frame(_cuda(text), codes)
        ref = om.frame(tkv, pkv, orc.SampleParams(0.9, 50, 1.0, 1.05), text[0], T + f, st)
        got = codes.cpu().numpy()[0]
        assert list(got) == list(ref), (f, list(got), list(ref))
        state = eng.state()
        if check_logits is not None:
            check_logits(state["logits"].cpu().numpy()[0], st["logits"])
        assert int(state["positions"].cpu()[0]) == T + f + 1
        assert state["prev"].cpu().numpy()[0].astype(np.uint32).tolist() == st["prev"].tolist()
    ctx.check_device_error()
    return eng


def _tiny_check(got, ref):
    assert float(np.max(np.abs(got - ref))) < TINY_TOL


def _full_check(got, ref):
    err = float(np.max(np.abs(got.astype(np.float64) - ref)))
    assert err <= ABS_TOL and err / float(np.max(np.abs(ref))) <= REL_TOL, err


@pytest.mark.parametrize("persistent", [True, False])
def test_tiny_frames_match_oracle(E, ctx, orc, persistent):
    import qora_b200
    cfg = qora_b200.ModelConfig.tiny()
    tw, pw = qora_b200.synth_talker(cfg), qora_b200.synth_predictor(cfg)
    om = orc.OracleModel(orc.Model.synth(orc.ModelConfig.tiny()))
    eng = _run(E, orc, ctx, cfg, tw, pw, om, T=5, F=8, persistent=persistent,
               check_logits=_tiny_check)
    if persistent:
        assert eng.kernels_per_frame() == 1


def test_tiny_long_context_uses_attention_splits(E, ctx, orc):
    """600 cached positions: 16 position splits per kv head and their merge
    inside the frame kernel."""
    import qora_b200
    cfg = qora_b200.ModelConfig.tiny(t_max_pos=1024)
    tw, pw = qora_b200.synth_talker(cfg), qora_b200.synth_predictor(cfg)
    om = orc.OracleModel(orc.Model.synth(orc.ModelConfig.tiny(t_max_pos=1024)))
    _run(E, orc, ctx, cfg, tw, pw, om, T=600, F=3, persistent=True, seed=700,
         check_logits=_tiny_check)


def test_trace_records_every_op(E, ctx, orc):
    import qora_b200
    cfg = qora_b200.ModelConfig.tiny()
    tw, pw = qora_b200.synth_talker(cfg), qora_b200.synth_predictor(cfg)
    om = orc.OracleModel(orc.Model.synth(orc.ModelConfig.tiny()))
    talker = E.Talker(ctx, tw, max_batch=1)
    pred = E.CodePredictor(ctx, pw, max_batch=1)
    eng = E.Engine(talker, pred, 1, max_pos=16)
    eng.prefill(orc.synth_normal(3, 1.0, 4 * cfg.t_hidden).reshape(1, 4, cfg.t_hidden), [9])
    eng.trace(True)
    eng.frame(_cuda(orc.synth_normal(4, 1.0, cfg.t_hidden)[None]),
              __import__("torch").zeros(1, 16, dtype=__import__("torch").int32, device="cuda"))
    ops, st = eng.trace(False)
    L_t, L_p, G = cfg.t_layers, cfg.p_layers, cfg.p_groups
    assert len(ops) == 1 + (G + 1) * (1 + 5 * L_p) + G + 5 * L_t + 1
    assert ops[0] == 2 and (ops == 1).sum() == (G + 1) * L_p + L_t
    ready0 = (~st[:, 0]).astype(np.int64)
    ready1, done = st[:, 1].astype(np.int64), st[:, 2].astype(np.int64)
    assert np.all(st[:, 2] > 0) and np.all(ready1[ops == 0] >= ready0[ops == 0])
    assert np.all(done[ops == 0] >= ready1[ops == 0])
    assert np.all(st[ops == 0, 7] > 0)      # every GEMV op's item 0 consumed weight slots


@pytest.mark.parametrize("hd", [128, 64])
def test_full_size_frames_match_oracle(E, ctx, orc, hd):
    """1.7B dims (28-layer talker, 5-layer predictor at head_dim 128 as the
    reference config and 64 as BASELINE config 2)."""
    import qora_b200
    from test_gpu_full import _oracle_from
    cfg = qora_b200.ModelConfig(t_max_pos=256, p_head_dim=hd)
    tw, pw = qora_b200.synth_talker(cfg), qora_b200.synth_predictor(cfg)
    om = orc.OracleModel.__new__(orc.OracleModel)
    om.m = _oracle_from(orc, cfg, tw, pw)
    om.t, om.p = om.m.talker_struct(), om.m.predictor_struct()
    _run(E, orc, ctx, cfg, tw, pw, om, T=16, F=3, persistent=True, seed=800,
         check_logits=_full_check)


def _follow(E, orc, ctx, cfg, tw, pw, om, B, T, F, seed, graph):
    """The engine's frame loop for B streams against the oracle teacher-forced
    with the engine's own codes (generate_new.rs:606-665 step by step):
      - code 0 must equal the oracle's sample_token (generate_new.rs:771-862)
        drawn from the engine's own logits, previous codes and RNG state (the
        sampler exactly), and the RNG states must agree after the draw;
      - codes 1..15 must agree with the oracle's greedy argmax of its own
        predictor logits (code_predictor.rs:218-273) fed the engine's codes,
        >= 99.5 % of them (near-ties may flip);
      - the talker logits after the step (forward_with_embedding on
        E_talker[c0] + acoustic sum + text) within max-abs 2e-3 / rel 1e-3 of
        the oracle's.
    Following the engine keeps a legitimate near-tie from derailing the rest."""
    import torch
    talker = E.Talker(ctx, tw, max_batch=B)
    pred = E.CodePredictor(ctx, pw, max_batch=B)
    eng = E.Engine(talker, pred, B, max_pos=T + F + 4)
    if graph:
        eng.use_graph(True)
    H = cfg.t_hidden
    xs = np.stack([orc.synth_normal(seed + b, 1.0, T * H).reshape(T, H) for b in range(B)])
    seeds = [seed + 100 + b for b in range(B)]
    eng.prefill(xs, seeds)
    texts = orc.synth_normal(seed + 200, 1.0, B * H).reshape(B, H)
    params = orc.SampleParams(0.9, 50, 1.0, 1.05)
    okv = [om.talker_kv(T + F + 4) for _ in range(B)]
    pkv = om.predictor_kv()
    hid = [om.talker_prefill(xs[b], okv[b], 0) for b in range(B)]
    codes = torch.zeros(B, 16, dtype=torch.int32, device="cuda")
    text_d = _cuda(texts)
    worst_abs, worst_rel, agree, total = 0.0, 0.0, 0, 0
    for f in range(F):
        before = eng.state()
        eng.frame(text_d, codes)
        after = eng.state()
        got = codes.cpu().numpy().astype(np.uint32)
        glog = after["logits"].cpu().numpy()
        for b in range(B):
            lg0 = before["logits"].cpu().numpy()[b]
            prev = before["prev"].cpu().numpy()[b].astype(np.uint32)
            rng0 = int(before["rng"].cpu().numpy()[b]) & 0xFFFFFFFFFFFFFFFF
            tok, rng1 = orc.sample_token(lg0, params, prev, rng0)
            assert tok == got[b, 0], (f, b, tok, got[b, 0])
            assert rng1 == int(after["rng"].cpu().numpy()[b]) & 0xFFFFFFFFFFFFFFFF
            sem = om.embed_codec(int(got[b, 0]))
            rc, _ = om.predictor_frame(hid[b], sem, pkv, forced=got[b, 1:])
            agree += int(np.sum(rc == got[b, 1:]))
            total += cfg.p_groups
            emb = sem + om.acoustic_sum(got[b, 1:]) + texts[b]
            hid[b], rl = om.talker_step(emb, okv[b], T + f)
            err = float(np.max(np.abs(glog[b].astype(np.float64) - rl)))
            worst_abs = max(worst_abs, err)
            worst_rel = max(worst_rel, err / float(np.max(np.abs(rl))))
            assert after["prev"].cpu().numpy()[b].astype(np.uint32).tolist() == got[b].tolist()
        assert after["positions"].cpu().numpy().tolist() == [T + f + 1] * B
    ctx.check_device_error()
    print(f"B={B} frames={F}: worst abs {worst_abs:.3e} rel {worst_rel:.3e} "
          f"predictor argmax {agree}/{total}")
    assert worst_abs <= ABS_TOL and worst_rel <= REL_TOL
    assert agree / total >= 0.995
    return eng


def _full_model(orc, hd=128):
    import qora_b200
    from test_gpu_full import _oracle_from
    cfg = qora_b200.ModelConfig(t_max_pos=256, p_head_dim=hd)
    tw, pw = qora_b200.synth_talker(cfg), qora_b200.synth_predictor(cfg)
    om = orc.OracleModel.__new__(orc.OracleModel)
    om.m = _oracle_from(orc, cfg, tw, pw)
    om.t, om.p = om.m.talker_struct(), om.m.predictor_struct()
    return cfg, tw, pw, om


def test_full_size_64_frames_follow_oracle(E, ctx, orc):
    """Batch 1 at 1.7B dims for 64 frames: one persistent-kernel launch per frame."""
    cfg, tw, pw, om = _full_model(orc)
    eng = _follow(E, orc, ctx, cfg, tw, pw, om, B=1, T=16, F=64, seed=810, graph=False)
    assert eng.kernels_per_frame() == 1


def test_full_size_batch32_frames_follow_oracle(E, ctx, orc):
    """Batch 32 at 1.7B dims for 8 frames: the per-op kernels (tensor-core
    GEMVs for every 32-row projection) captured in one CUDA graph per frame."""
    cfg, tw, pw, om = _full_model(orc)
    eng = _follow(E, orc, ctx, cfg, tw, pw, om, B=32, T=16, F=8, seed=820, graph=True)
    assert eng.kernels_per_frame() > 100
