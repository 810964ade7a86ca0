"""GPU parity of the talker step, prefill, code predictor, sampler and frame
loop against the CPU oracle on a tiny random-init model (same bytes on both
sides: the engine's synthetic generator equals the oracle's, see
tests/test_capi.py::test_model_synth_matches_oracle)."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-4  # tiny model: logits are O(1); fp32 with a different summation order


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


@pytest.fixture(scope="module")
def tiny(E, ctx, orc):
    import qora_b200
    cfg = qora_b200.ModelConfig.tiny()
    tw, pw = qora_b200.synth_talker(cfg), qora_b200.synth_predictor(cfg)
    om = orc.OracleModel(orc.Model.synth(orc.ModelConfig.tiny()))
    talker = E.Talker(ctx, tw, max_batch=4)
    pred = E.CodePredictor(ctx, pw, max_batch=4)
    return cfg, om, talker, pred


def _cuda(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _maxerr(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))


def test_talker_steps(orc, tiny):
    cfg, om, talker, _ = tiny
    kv = talker.new_kv()
    okv = om.talker_kv()
    for pos in range(12):
        emb = orc.synth_normal(300 + pos, 1.0, cfg.t_hidden)
        h, lg = talker.forward_with_embedding(_cuda(emb), kv, [pos])
        rh, rl = om.talker_step(emb, okv, pos)
        assert _maxerr(h.cpu().numpy()[0], rh) < TOL
        assert _maxerr(lg.cpu().numpy()[0], rl) < TOL
    assert list(kv.lengths()) == [12]
    # cache contents vs the oracle's token-major cache
    K, V = kv.layer_tensors(1)
    assert _maxerr(K.cpu().numpy()[0][:, :12].transpose(1, 0, 2), okv.k(1)[:12]) < TOL
    assert _maxerr(V.cpu().numpy()[0][:, :12].transpose(1, 0, 2), okv.v(1)[:12]) < TOL


def test_talker_batch_streams_independent(orc, tiny):
    """B streams in one step == each stream on its own (different lengths)."""
    cfg, om, talker, _ = tiny
    kv = talker.new_kv(streams=3)
    okvs = [om.talker_kv() for _ in range(3)]
    pos = [0, 0, 0]
    for step in range(5):
        embs = orc.synth_normal(400 + step, 1.0, 3 * cfg.t_hidden).reshape(3, cfg.t_hidden)
        h, lg = talker.forward_with_embedding(_cuda(embs), kv, pos)
        for s in range(3):
            rh, rl = om.talker_step(embs[s], okvs[s], pos[s])
            assert _maxerr(lg.cpu().numpy()[s], rl) < TOL
        pos = [p + 1 for p in pos]


def test_talker_prefill_and_decode(orc, tiny):
    cfg, om, talker, _ = tiny
    T = 9
    x = orc.synth_normal(500, 1.0, T * cfg.t_hidden).reshape(T, cfg.t_hidden)
    kv = talker.new_kv()
    okv = om.talker_kv()
    h = talker.prefill_talker_raw_from(_cuda(x), kv, 0)
    rh = om.talker_prefill(x, okv, 0)
    assert _maxerr(h.cpu().numpy(), rh) < TOL
    for layer in (0, cfg.t_layers - 1):
        K, V = kv.layer_tensors(layer)
        assert _maxerr(K.cpu().numpy()[0][:, :T].transpose(1, 0, 2), okv.k(layer)[:T]) < TOL
    # codec head of the prefill hidden, then decode steps after the prefix
    lg = talker.apply_codec_head(h).cpu().numpy()[0]
    assert _maxerr(lg, om.codec_head(rh)) < TOL
    for pos in range(T, T + 4):
        emb = om.embed_codec(int(np.argmax(lg)))
        g, lgt = talker.forward_with_embedding(_cuda(emb), kv, [pos])
        _, rl = om.talker_step(emb, okv, pos)
        lg = lgt.cpu().numpy()[0]
        assert _maxerr(lg, rl) < TOL


def test_prefill_from_prefix(orc, tiny):
    cfg, om, talker, _ = tiny
    x = orc.synth_normal(600, 1.0, 10 * cfg.t_hidden).reshape(10, cfg.t_hidden)
    kv = talker.new_kv()
    talker.prefill_talker_raw_from(_cuda(x[:4]), kv, 0)
    h = talker.prefill_talker_raw_from(_cuda(x[4:]), kv, 4)
    okv = om.talker_kv()
    rh = om.talker_prefill(x, okv, 0)
    assert _maxerr(h.cpu().numpy(), rh) < TOL
    with pytest.raises(Exception):
        talker.prefill_talker_raw_from(_cuda(x[:2]), kv, 3)  # wrong start_pos (talker.rs:422)


def test_embed_codec_bit_exact(orc, tiny):
    cfg, om, talker, _ = tiny
    got = talker.embed_codec_token([5, 300]).cpu().numpy()
    for i, t in enumerate([5, 300]):
        assert np.array_equal(got[i], om.embed_codec(t))


def test_predictor_frame_teacher_forced(orc, tiny):
    cfg, om, _, pred = tiny
    B = 2
    hid = orc.synth_normal(700, 1.0, B * cfg.t_hidden).reshape(B, cfg.t_hidden)
    sem = np.stack([om.embed_codec(11), om.embed_codec(250)])
    okv = om.predictor_kv()
    ref = [om.predictor_frame(hid[b], sem[b], okv) for b in range(B)]
    forced = np.stack([r[0] for r in ref]).astype(np.int32)
    kv = pred.new_kv(streams=B)
    codes, logits = pred.generate_acoustic_codes(_cuda(hid), _cuda(sem), kv, forced=forced,
                                                 want_logits=True)
    logits = logits.cpu().numpy()
    for b in range(B):
        assert _maxerr(logits[b], ref[b][1]) < TOL
    agree = np.mean(codes.cpu().numpy() == forced)
    assert agree >= 0.9, agree


def test_predictor_frame_free_running(orc, tiny):
    cfg, om, _, pred = tiny
    hid = orc.synth_normal(710, 1.0, cfg.t_hidden)
    sem = om.embed_codec(42)
    rc, _ = om.predictor_frame(hid, sem, om.predictor_kv())
    kv = pred.new_kv()
    codes = pred.generate_acoustic_codes(_cuda(hid[None]), _cuda(sem[None]), kv)
    assert list(codes.cpu().numpy()[0]) == list(rc)
    assert list(kv.lengths()) == [cfg.p_groups + 1]


def test_acoustic_embedding_sum_bit_exact(orc, tiny):
    cfg, om, _, pred = tiny
    codes = np.array([[(7 * g + 3) % cfg.p_vocab for g in range(cfg.p_groups)]], np.int32)
    got = pred.get_acoustic_embeddings_sum(_cuda(codes)).cpu().numpy()[0]
    assert np.array_equal(got, om.acoustic_sum(codes[0].astype(np.uint32)))


def test_sampler_matches_reference(E, ctx, orc):
    """Same logits, same xorshift state: identical draw unless r sits within
    float rounding of a cumulative-probability boundary."""
    import torch
    params = E.default_params()
    oparams = orc.SampleParams(0.9, 50, 1.0, 1.05)
    B, V = 64, 3072
    logits = (orc.synth_normal(800, 3.0, B * V)).reshape(B, V)
    prev = (np.arange(B * 16).reshape(B, 16) * 37 % V).astype(np.uint32)
    seeds = np.arange(1, B + 1, dtype=np.uint64) * 0x9E3779B97F4A7C15
    rng = torch.from_numpy(seeds.view(np.int64).copy()).cuda()
    got = E.sample_token(ctx, _cuda(logits), _cuda(prev.view(np.int32)), rng, params).cpu().numpy()
    new_rng = rng.cpu().numpy().view(np.uint64)
    mism = 0
    for b in range(B):
        tok, st = orc.sample_token(logits[b], oparams, prev[b], int(seeds[b]))
        assert st == int(new_rng[b])
        if tok != got[b]:
            mism += 1
            probs = orc.sample_probs(logits[b], oparams, prev[b])
            r, _ = orc.simple_rand(int(seeds[b]))
            cum = np.cumsum(probs.astype(np.float64))
            assert np.min(np.abs(cum - r)) < 1e-5, (b, tok, got[b])
    assert mism <= 2


def test_sampler_topk_ties_and_greedy_edge(E, ctx, orc):
    import torch
    params = E._lib.SampleParams(1.0, 3, 1.0, 1.0)
    logits = np.zeros((1, 64), np.float32)
    logits[0, [5, 9, 40, 41]] = 2.0          # four-way tie: top-3 keeps 5, 9, 40
    oparams = orc.SampleParams(1.0, 3, 1.0, 1.0)
    for seed in range(1, 40):
        rng = torch.tensor([seed], dtype=torch.int64).cuda()
        g = int(E.sample_token(ctx, _cuda(logits), None, rng, params).cpu().numpy()[0])
        tok, _ = orc.sample_token(logits[0], oparams, np.zeros(0, np.uint32), seed)
        assert g == tok and g in (5, 9, 40)


def test_engine_frames_match_oracle(E, orc, tiny):
    import torch
    cfg, om, talker, pred = tiny
    B, T, F = 2, 4, 5
    eng = E.Engine(talker, pred, B, max_pos=64)
    x = orc.synth_normal(900, 1.0, B * T * cfg.t_hidden).reshape(B, T, cfg.t_hidden)
    seeds = [123, 456]
    eng.prefill(x, seeds)
    text = orc.synth_normal(901, 1.0, B * cfg.t_hidden).reshape(B, cfg.t_hidden)
    params = orc.SampleParams(0.9, 50, 1.0, 1.05)
    states, kvs = [], []
    for b in range(B):
        tkv, pkv = om.talker_kv(64), om.predictor_kv()
        hdn = om.talker_prefill(x[b], tkv, 0)
        states.append({"logits": om.codec_head(hdn), "hidden": hdn.copy(),
                       "prev": np.zeros(16, np.uint32), "rng": seeds[b]})
        kvs.append((tkv, pkv))
    tt = _cuda(text)
    codes = torch.zeros(B, 16, dtype=torch.int32).cuda()
    for f in range(F):
        if f == 2:
            eng.use_graph(True)   # the graph replay must give the same frames
        eng.frame(tt, codes)
        got = codes.cpu().numpy()
        for b in range(B):
            ref = om.frame(kvs[b][0], kvs[b][1], params, text[b], T + f, states[b])
            assert list(got[b]) == list(ref), (f, b)
    assert eng.kernels_per_frame() > 0


def test_engine_host_frame(E, orc, tiny):
    cfg, om, talker, pred = tiny
    B, T = 1, 3
    eng = E.Engine(talker, pred, B, max_pos=32)
    x = orc.synth_normal(950, 1.0, B * T * cfg.t_hidden).reshape(B, T, cfg.t_hidden)
    eng.prefill(x, [7])
    text = orc.synth_normal(951, 1.0, B * cfg.t_hidden).reshape(B, cfg.t_hidden)
    out = np.zeros((B, 16), np.int32)
    eng.frame_host(text, out)
    tkv, pkv = om.talker_kv(32), om.predictor_kv()
    hdn = om.talker_prefill(x[0], tkv, 0)
    st = {"logits": om.codec_head(hdn), "hidden": hdn.copy(), "prev": np.zeros(16, np.uint32),
          "rng": 7}
    ref = om.frame(tkv, pkv, orc.SampleParams(0.9, 50, 1.0, 1.05), text[0], T, st)
    assert list(out[0]) == list(ref)


def test_position_past_rope_table_is_an_error(E, ctx, orc, tiny):
    cfg, om, talker, _ = tiny
    kv = talker.new_kv()
    emb = orc.synth_normal(960, 1.0, cfg.t_hidden)
    talker.forward_with_embedding(_cuda(emb), kv, [cfg.t_max_pos + 5])
    with pytest.raises(Exception):
        ctx.check_device_error()
    ctx.check_device_error()  # cleared


def test_engine_batch8_frames_match_oracle(E, ctx, orc):
    """Eight streams: the talker and predictor projections run on the
    tensor-core GEMV (>= 8 rows), the output heads (not a multiple of 128
    columns) on the CUDA-core kernel; frames must equal the oracle's."""
    import torch
    import qora_b200
    cfg = qora_b200.ModelConfig.tiny()
    om = orc.OracleModel(orc.Model.synth(orc.ModelConfig.tiny()))
    talker = E.Talker(ctx, qora_b200.synth_talker(cfg), max_batch=8)
    pred = E.CodePredictor(ctx, qora_b200.synth_predictor(cfg), max_batch=8)
    B, T, F = 8, 3, 3
    eng = E.Engine(talker, pred, B, max_pos=32)
    x = orc.synth_normal(960, 1.0, B * T * cfg.t_hidden).reshape(B, T, cfg.t_hidden)
    seeds = [1000 + b for b in range(B)]
    eng.prefill(x, seeds)
    text = orc.synth_normal(961, 1.0, B * cfg.t_hidden).reshape(B, cfg.t_hidden)
    params = orc.SampleParams(0.9, 50, 1.0, 1.05)
    states, kvs = [], []
    for b in range(B):
        tkv, pkv = om.talker_kv(32), om.predictor_kv()
        hdn = om.talker_prefill(x[b], tkv, 0)
        states.append({"logits": om.codec_head(hdn), "hidden": hdn.copy(),
                       "prev": np.zeros(16, np.uint32), "rng": seeds[b]})
        kvs.append((tkv, pkv))
    tt = _cuda(text)
    codes = torch.zeros(B, 16, dtype=torch.int32).cuda()
    for f in range(F):
        eng.frame(tt, codes)
        got = codes.cpu().numpy()
        for b in range(B):
            ref = om.frame(kvs[b][0], kvs[b][1], params, text[b], T + f, states[b])
            assert list(got[b]) == list(ref), (f, b)
    ctx.check_device_error()


@pytest.mark.parametrize("B", [1, 2])
def test_engine_onset_temperature_schedule(E, orc, tiny, B):
    """frame_temperature (generate_new.rs:82-88): the first frames sample at
    the onset temperature, then at the base one.  B = 1 runs the persistent
    frame kernel, B = 2 the per-op kernels in a CUDA graph (captured again
    after the change)."""
    import torch
    from qora_b200 import generate as G
    cfg, om, talker, pred = tiny
    T, F = 3, 5
    sched = G.TTSParams(temperature=1.4, onset_frames=2, onset_temperature=0.05)
    eng = E.Engine(talker, pred, B, max_pos=32, params=sched.sample_params())
    eng.use_graph(True)
    x = orc.synth_normal(960 + B, 1.0, B * T * cfg.t_hidden).reshape(B, T, cfg.t_hidden)
    seeds = [70 + b for b in range(B)]
    eng.prefill(x, seeds)
    text = orc.synth_normal(961, 1.0, B * cfg.t_hidden).reshape(B, cfg.t_hidden)
    states, kvs = [], []
    for b in range(B):
        tkv, pkv = om.talker_kv(32), om.predictor_kv()
        hdn = om.talker_prefill(x[b], tkv, 0)
        states.append({"logits": om.codec_head(hdn), "hidden": hdn.copy(),
                       "prev": np.zeros(16, np.uint32), "rng": seeds[b]})
        kvs.append((tkv, pkv))
    tt = _cuda(text)
    codes = torch.zeros(B, 16, dtype=torch.int32).cuda()
    for f in range(F):
        temp = G.frame_temperature(sched, f)
        eng.set_temperature(temp)
        eng.frame(tt, codes)
        got = codes.cpu().numpy()
        params = orc.SampleParams(temp, sched.top_k, sched.top_p, sched.repetition_penalty)
        for b in range(B):
            ref = om.frame(kvs[b][0], kvs[b][1], params, text[b], T + f, states[b])
            assert list(got[b]) == list(ref), (f, b)


def test_talker_decode_teacher_forced(E, ctx, orc, tiny):
    """forward_talker_decode (talker.rs:161-258) over a mixed text / codec token
    sequence, device against oracle, then two streams at once."""
    import qora_b200
    from qora_b200 import _lib
    cfg, om, talker, _ = tiny
    tpo = orc.TextProj.synth(63, 400, cfg.t_hidden, cfg.t_hidden, sigma=0.05)
    q = lambda w: qora_b200.Q4Weight(w.packed, w.scales, w.k, w.n)
    tp = E.TextProjection(ctx, qora_b200.TextProjWeights(q(tpo.text_embedding), q(tpo.fc1),
                                                        tpo.fc1_bias, q(tpo.fc2), tpo.fc2_bias))
    kv = talker.new_kv(max_pos=16)
    okv = om.talker_kv(16)
    seq = [(11, True), (250, False), (399, True), (0, False), (7, True), (cfg.t_vocab - 1, False)]
    for pos, (tok, is_text) in enumerate(seq):
        got = talker.forward_talker_decode([tok], is_text, kv, [pos], tp).cpu().numpy()[0]
        want = om.talker_decode(tok, is_text, okv, pos, tpo)
        assert _maxerr(got, want) < TOL, pos
    kv2 = talker.new_kv(max_pos=16, streams=2)
    got = talker.forward_talker_decode([3, 4], False, kv2, [0, 0]).cpu().numpy()
    for b, tok in enumerate((3, 4)):
        want = om.talker_decode(tok, False, om.talker_kv(16), 0)
        assert _maxerr(got[b], want) < TOL, b
    with pytest.raises(_lib.QoraError) as ei:
        talker.forward_talker_decode([cfg.t_vocab], False, kv, [len(seq)])
    assert ei.value.status == 5
    with pytest.raises(_lib.QoraError) as ei:
        talker.forward_talker_decode([1], True, kv, [len(seq)])   # text path, no projection
    assert ei.value.status == 1
    ctx.check_device_error()


def test_embed_rows_out_of_table_is_flagged(E, ctx, tiny):
    """A device token past the codec table gives a zero row and a range error
    at the next device-error check, never a read outside the table."""
    import torch
    from qora_b200 import _lib
    cfg, _, talker, _ = tiny
    out = talker.embed_codec_token([1, cfg.t_vocab + 5, 2])
    torch.cuda.synchronize()
    with pytest.raises(_lib.QoraError) as ei:
        ctx.check_device_error()
    assert ei.value.status == 5
    o = out.cpu().numpy()
    assert np.all(o[1] == 0.0) and np.any(o[0] != 0.0) and np.any(o[2] != 0.0)
    ctx.check_device_error()   # the flag was cleared


@pytest.mark.parametrize("B", [1, 2])
def test_engine_prefill_from_prefix(E, orc, tiny, B):
    """The prefix-cache path (generate_new.rs:509-530): a prefix prefilled once,
    copied into every stream, the suffix prefilled on top; frames equal the
    oracle's on the same prefix + suffix (whose prefill-from-prefix equals a
    full prefill bit for bit, tests/test_oracle_model.py)."""
    import torch
    from qora_b200 import _lib
    cfg, om, talker, pred = tiny
    P0, T, F = 5, 4, 3
    xp = orc.synth_normal(970, 1.0, P0 * cfg.t_hidden).reshape(P0, cfg.t_hidden)
    xs = orc.synth_normal(971, 1.0, B * T * cfg.t_hidden).reshape(B, T, cfg.t_hidden)
    prefix = talker.new_kv(max_pos=32)
    talker.prefill_talker_raw_from(_cuda(xp), prefix, 0)
    eng = E.Engine(talker, pred, B, max_pos=32)
    seeds = [40 + b for b in range(B)]
    eng.prefill_from(prefix, P0, xs, seeds)
    # bit-identical to prefilling prefix + suffix in one go (prefill chunks
    # plan their GEMMs independently of their row count), as the reference's
    # prefix cache is (generate_new.rs:320-322)
    full = E.Engine(talker, pred, B, max_pos=32)
    full.prefill(np.concatenate([np.broadcast_to(xp, (B, P0, cfg.t_hidden)), xs], axis=1), seeds)
    a, b_ = eng.state(), full.state()
    assert np.array_equal(a["hidden"].cpu().numpy(), b_["hidden"].cpu().numpy())
    assert np.array_equal(a["logits"].cpu().numpy(), b_["logits"].cpu().numpy())
    assert np.array_equal(a["positions"].cpu().numpy(), b_["positions"].cpu().numpy())
    text = orc.synth_normal(972, 1.0, B * cfg.t_hidden).reshape(B, cfg.t_hidden)
    states, kvs = [], []
    for b in range(B):
        tkv, pkv = om.talker_kv(32), om.predictor_kv()
        om.talker_prefill(xp, tkv, 0)
        hdn = om.talker_prefill(xs[b], tkv, P0)
        states.append({"logits": om.codec_head(hdn), "hidden": hdn.copy(),
                       "prev": np.zeros(16, np.uint32), "rng": seeds[b]})
        kvs.append((tkv, pkv))
    tt = _cuda(text)
    codes = torch.zeros(B, 16, dtype=torch.int32).cuda()
    params = orc.SampleParams(0.9, 50, 1.0, 1.05)
    for f in range(F):
        eng.frame(tt, codes)
        got = codes.cpu().numpy()
        for b in range(B):
            ref = om.frame(kvs[b][0], kvs[b][1], params, text[b], P0 + T + f, states[b])
            assert list(got[b]) == list(ref), (f, b)
    with pytest.raises(_lib.QoraError) as ei:
        eng.prefill_from(prefix, P0 + 1, xs, seeds)     # the cache holds P0 positions
    assert ei.value.status == 2
