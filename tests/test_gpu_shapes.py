"""Talker / predictor parity on small configs chosen to reach every GEMV
tiling branch (with and without split-K, batch tiles 1/2/4, all fused
prologue / epilogue modes)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-4


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


CONFIGS = {
    "talker_h128": dict(t_hidden=128, t_heads=2, t_kv_heads=1, t_head_dim=64, t_ffn=256),
    "talker_h256_ffn128": dict(t_hidden=256, t_ffn=128),
    "pred_h256": dict(p_hidden=256, p_ffn=512),
    "pred_h128_ffn512": dict(p_hidden=128, p_ffn=512),
}


@pytest.mark.parametrize("name", list(CONFIGS))
def test_small_config_parity(E, ctx, orc, name):
    import qora_b200
    kw = CONFIGS[name]
    cfg = qora_b200.ModelConfig.tiny(**kw)
    om = orc.OracleModel(orc.Model.synth(orc.ModelConfig.tiny(**kw)))
    talker = E.Talker(ctx, qora_b200.synth_talker(cfg), max_batch=2)
    pred = E.CodePredictor(ctx, qora_b200.synth_predictor(cfg), max_batch=2)
    # talker: prefill 5 + 2 steps
    x = orc.synth_normal(1, 1.0, 5 * cfg.t_hidden).reshape(5, cfg.t_hidden)
    kv, okv = talker.new_kv(), om.talker_kv()
    h = talker.prefill_talker_raw_from(_cuda(x), kv, 0).cpu().numpy()
    rh = om.talker_prefill(x, okv, 0)
    assert np.max(np.abs(h - rh)) < TOL, "talker prefill"
    for pos in (5, 6):
        emb = orc.synth_normal(10 + pos, 1.0, cfg.t_hidden)
        _, lg = talker.forward_with_embedding(_cuda(emb), kv, [pos])
        _, rl = om.talker_step(emb, okv, pos)
        assert np.max(np.abs(lg.cpu().numpy()[0] - rl)) < TOL, f"talker step {pos}"
    # predictor, B = 1 and 2, teacher forced
    for B in (1, 2):
        hid = orc.synth_normal(20 + B, 1.0, B * cfg.t_hidden).reshape(B, cfg.t_hidden)
        sem = np.stack([om.embed_codec(3 + b) for b in range(B)])
        ref = [om.predictor_frame(hid[b], sem[b], om.predictor_kv()) for b in range(B)]
        forced = np.stack([r[0] for r in ref]).astype(np.int32)
        codes, logits = pred.generate_acoustic_codes(_cuda(hid), _cuda(sem), pred.new_kv(streams=B),
                                                     forced=forced, want_logits=True)
        logits = logits.cpu().numpy()
        for b in range(B):
            errs = np.max(np.abs(logits[b] - ref[b][1]), axis=1)
            assert np.all(errs < TOL), (B, b, errs)
