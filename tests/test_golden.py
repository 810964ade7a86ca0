"""Golden fixtures (tests/golden/golden.npz, written by tests/golden/make_golden.py).

CPU tests: the oracle and the engine's host-side functions (quantiser, RoPE
tables, synthetic weights) reproduce the committed numbers bit for bit.
GPU tests: the CUDA path, called through the C ABI, reproduces them within the
tolerances stated below.
"""
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden.npz")
GEMV_CASES = ["shapes_64x2048", "shapes_64x6144", "shapes_32x1024", "shapes_16x256", "shapes_1x32",
              "sparse_48x1024", "sparse_32x2048", "tail_16x100"]
SEEDS = {"shapes_64x2048": (1, 0.0, 0.0), "shapes_64x6144": (2, 0.0, 0.0),
         "shapes_32x1024": (3, 0.0, 0.0), "shapes_16x256": (4, 0.0, 0.0),
         "shapes_1x32": (5, 0.0, 0.0), "sparse_48x1024": (11, 0.3, 0.2),
         "sparse_32x2048": (12, 0.5, 0.5), "tail_16x100": (31, 0.0, 0.0)}


@pytest.fixture(scope="module")
def g():
    return np.load(GOLDEN)


def _kat_inputs(orc, g, name):
    k, n = (int(v) for v in g[f"{name}/kn"])
    seed, iz, sz = SEEDS[name]
    r = orc.XRng(seed)
    packed = r.bytes(k * (n // 32) * 16)
    scales = r.scales(k * (n // 32), sz)
    x = r.inputs(k, iz)
    sums = [int(packed.astype(np.uint64).sum()), int(scales.astype(np.uint64).sum()),
            int(x.view(np.uint32).astype(np.uint64).sum())]
    assert sums == [int(v) for v in g[f"{name}/input_sums"]], f"{name}: generator drifted"
    return k, n, packed, scales, x


@pytest.mark.parametrize("name", GEMV_CASES)
def test_oracle_gemv_reproduces_golden(orc, g, name):
    k, n, packed, scales, x = _kat_inputs(orc, g, name)
    y = orc.gemv_scalar(x, packed, scales, n, 0, k)
    assert y.view(np.uint32).tolist() == g[f"{name}/y"].view(np.uint32).tolist()


def test_quantisers_reproduce_golden(orc, g):
    import qora_b200
    data = g["quant/data"]
    w = orc.quantize(data)
    assert np.array_equal(w.packed, g["quant/packed"]) and np.array_equal(w.scales, g["quant/scales"])
    e = qora_b200.quantize_f32_to_q4(data)          # the engine's host quantiser (C ABI)
    assert np.array_equal(e.packed, g["quant/packed"]) and np.array_equal(e.scales, g["quant/scales"])


def test_rope_tables_reproduce_golden(orc, g):
    from qora_b200 import _lib
    import ctypes as C
    for hd, n, sec in ((128, 40, [24, 20, 20]), (64, 20, None)):
        c, s = orc.rope_tables(hd, n, 1e6, sec)
        assert np.array_equal(c, g[f"rope/hd{hd}_cos"]) and np.array_equal(s, g[f"rope/hd{hd}_sin"])
        half = hd // 2
        ce = np.empty(n * half, np.float32)
        se = np.empty(n * half, np.float32)
        secs = np.asarray(sec if sec else [half], np.int32)
        _lib.call("qora_rope_tables_host", hd, n, C.c_double(1e6), secs.ctypes.data, secs.size,
                  ce.ctypes.data, se.ctypes.data)
        assert np.array_equal(ce.reshape(c.shape), c) and np.array_equal(se.reshape(s.shape), s)


def test_oracle_sampler_reproduces_golden(orc, g):
    params = orc.SampleParams(0.9, 50, 1.0, 1.05)
    for r in range(4):
        st = int(g["sample/seeds"][r])
        for i in range(8):
            t, st = orc.sample_token(g["sample/logits"][r], params, g["sample/prev"], st)
            assert t == int(g["sample/tokens"][r, i])
        assert st == int(g["sample/final_rng"][r])


def test_oracle_tiny_model_reproduces_golden(orc, g):
    cfg = orc.ModelConfig.tiny()
    om = orc.OracleModel(orc.Model.synth(cfg))
    kv = om.talker_kv()
    h0 = om.talker_prefill(g["tiny/prefill_x"], kv, 0)
    assert np.array_equal(h0, g["tiny/prefill_hidden"])
    for s in range(4):
        h, lg = om.talker_step(g["tiny/step_emb"][s], kv, 3 + s)
        assert np.array_equal(h, g["tiny/step_hidden"][s])
        assert np.array_equal(lg, g["tiny/step_logits"][s])
    codes, plog = om.predictor_frame(g["tiny/step_hidden"][3], g["tiny/pred_sem"], om.predictor_kv())
    assert np.array_equal(np.asarray(codes, np.uint32), g["tiny/pred_codes"])
    assert np.array_equal(plog, g["tiny/pred_logits"])


# ---------------------------------------------------------------- GPU side
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


# GEMV: fixed-order device summation vs the reference's k-sequential loop;
# 1e-5 of the output scale (the reference accepts 1e-3 for its own chunked
# sums, gemv.rs:806-809).
GEMV_REL = 1e-5
# Tiny model: logits O(1), fp32 with a different summation order.
MODEL_ABS = 2e-4


@pytest.mark.gpu
@pytest.mark.parametrize("name", GEMV_CASES)
def test_gpu_gemv_matches_golden(E, ctx, orc, g, name):
    from qora_b200 import Q4Weight
    k, n, packed, scales, x = _kat_inputs(orc, g, name)
    w = E.DeviceQ4(ctx, Q4Weight(packed, scales, k, n))
    got = w.gemv(_cuda(x)).cpu().numpy()[0]
    ref = g[f"{name}/y"]
    scale = max(1.0, float(np.max(np.abs(ref))))
    assert float(np.max(np.abs(got - ref))) <= GEMV_REL * scale
    if n % 32:
        assert np.all(got[(n // 32) * 32:] == 0.0)


@pytest.mark.gpu
def test_gpu_sampler_matches_golden(E, ctx, g):
    import torch
    logits = _cuda(g["sample/logits"])
    prev = _cuda(np.tile(g["sample/prev"], (4, 1)))
    rng = torch.tensor(g["sample/seeds"].astype(np.int64)).cuda()
    for i in range(8):
        tok = E.sample_token(ctx, logits, prev, rng, E.default_params())
        assert tok.cpu().numpy().astype(np.uint32).tolist() == g["sample/tokens"][:, i].tolist()
    assert rng.cpu().numpy().astype(np.uint64).tolist() == g["sample/final_rng"].tolist()


@pytest.mark.gpu
def test_gpu_tiny_model_matches_golden(E, ctx, g):
    import qora_b200
    cfg = qora_b200.ModelConfig.tiny()
    talker = E.Talker(ctx, qora_b200.synth_talker(cfg), max_batch=1)
    pred = E.CodePredictor(ctx, qora_b200.synth_predictor(cfg), max_batch=1)
    kv = talker.new_kv()
    h0 = talker.prefill_talker_raw_from(_cuda(g["tiny/prefill_x"]), kv, 0)
    assert float(np.max(np.abs(h0.cpu().numpy() - g["tiny/prefill_hidden"]))) < MODEL_ABS
    for s in range(4):
        h, lg = talker.forward_with_embedding(_cuda(g["tiny/step_emb"][s]), kv, [3 + s])
        assert float(np.max(np.abs(h.cpu().numpy()[0] - g["tiny/step_hidden"][s]))) < MODEL_ABS
        assert float(np.max(np.abs(lg.cpu().numpy()[0] - g["tiny/step_logits"][s]))) < MODEL_ABS
    codes = pred.generate_acoustic_codes(_cuda(g["tiny/step_hidden"][3][None]),
                                         _cuda(g["tiny/pred_sem"][None]), pred.new_kv())
    assert codes.cpu().numpy()[0].astype(np.uint32).tolist() == g["tiny/pred_codes"].tolist()
