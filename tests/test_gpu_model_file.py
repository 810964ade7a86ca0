"""Weights loaded from a .qora-tts checkpoint (save.rs:262-409) give the same
device model as the same weights uploaded from memory: identical talker
logits and predictor codes."""
import numpy as np
import pytest

import qora_tts_format as qf

pytestmark = pytest.mark.gpu


def test_checkpoint_model_equals_in_memory_model(tmp_path, orc):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("-m gpu tests need a CUDA device")
    import qora_b200
    from qora_b200 import engine as E
    cfg = qora_b200.ModelConfig.tiny()
    tw, pw = qora_b200.synth_talker(cfg), qora_b200.synth_predictor(cfg)
    path = tmp_path / "tiny.qora-tts"
    qf.write(path, tw, pw, cfg)
    ctx = E.Context(0)
    mf = qora_b200.ModelFile(path)
    ta, pa = E.Talker(ctx, tw), E.CodePredictor(ctx, pw)
    tb, pb = E.Talker(ctx, mf.talker), E.CodePredictor(ctx, mf.predictor)
    mf.close()
    emb = torch.from_numpy(orc.synth_normal(41, 1.0, cfg.t_hidden)).cuda().reshape(1, -1)
    outs = []
    for t, p in ((ta, pa), (tb, pb)):
        kv = t.new_kv()
        h, lg = t.forward_with_embedding(emb, kv, [0])
        outs.append((h.cpu().numpy(), lg.cpu().numpy()))
    assert np.array_equal(outs[0][0], outs[1][0]) and np.array_equal(outs[0][1], outs[1][1])
    engines = [E.Engine(t, p, 1, max_pos=16) for t, p in ((ta, pa), (tb, pb))]
    x = orc.synth_normal(42, 1.0, 3 * cfg.t_hidden).reshape(1, 3, cfg.t_hidden)
    text = torch.from_numpy(orc.synth_normal(43, 1.0, cfg.t_hidden).reshape(1, -1)).cuda()
    codes = []
    for eng in engines:
        eng.prefill(x, [9])
        c = torch.zeros(1, 16, dtype=torch.int32, device="cuda")
        got = []
        for _ in range(3):
            eng.frame(text, c)
            got.append(c.cpu().numpy().copy())
        codes.append(np.stack(got))
    assert np.array_equal(codes[0], codes[1])
    ctx.check_device_error()
