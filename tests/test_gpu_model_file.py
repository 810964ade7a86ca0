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


def test_checkpoint_decoder_equals_named_decoder(tmp_path):
    """The speech-decoder section of a .qora-tts file (save_decoder,
    save.rs:171-262: processed codebooks, transposed linear weights) gives a
    decoder that decodes bit for bit like the same weights handed over by
    checkpoint tensor name; a file whose decoder section is not one is
    refused."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("-m gpu tests need a CUDA device")
    import qora_b200
    from qora_b200 import engine as E
    from qora_b200.decoder import DecoderDims, SpeechDecoder, synth_decoder
    cfg = qora_b200.ModelConfig.tiny()
    tw, pw = qora_b200.synth_talker(cfg), qora_b200.synth_predictor(cfg)
    dims = DecoderDims.tiny(rope_max_pos=500)
    W = synth_decoder(dims, 77)
    path = tmp_path / "with_decoder.qora-tts"
    qf.write(path, tw, pw, cfg, tail=qf.decoder_section(W, dims))
    ctx = E.Context(0)
    mf = qora_b200.ModelFile(path)
    a = SpeechDecoder.from_model_file(ctx, mf)
    mf.close()
    assert a.dims == dims
    b = SpeechDecoder(ctx, dims, W)
    codes = np.random.default_rng(3).integers(0, dims.codebook_size, (16, 14)).astype(np.uint32)
    for tc in (0, 2):
        a.use_tensor_cores(tc)
        b.use_tensor_cores(tc)
        ya, yb = a.decode_to_audio(codes), b.decode_to_audio(codes)
        assert ya.size == 14 * dims.hop
        assert np.array_equal(ya.view(np.uint32), yb.view(np.uint32)), tc
    ctx.check_device_error()
    bad = tmp_path / "placeholder.qora-tts"
    qf.write(bad, tw, pw, cfg)      # bytes standing in for the decoder section
    mf = qora_b200.ModelFile(bad)
    with pytest.raises(qora_b200._lib.QoraError):
        SpeechDecoder.from_model_file(ctx, mf)
    mf.close()
