"""GPU parity of the talker's text projection, embed_text_token
(talker.rs:104-116): text-embedding row -> fc1 + bias -> SiLU -> fc2 + bias,
through qora_text_proj_embed, against the CPU oracle token by token.

The GPU sums each GEMV in a fixed order different from the reference's
k-sequential loop, so rows are compared within 1e-4 of the output scale (the
GEMV parity tolerance).  Runs of 1-7 tokens use the CUDA-core GEMV, 8 or more
the tensor-core GEMV, and runs longer than 512 tokens are cut into chunks."""
import numpy as np
import pytest

import qora_tts_format as qf

pytestmark = pytest.mark.gpu


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


def _device_weights(tp):
    import qora_b200
    q = lambda w: qora_b200.Q4Weight(w.packed, w.scales, w.k, w.n)
    return qora_b200.TextProjWeights(q(tp.text_embedding), q(tp.fc1), tp.fc1_bias, q(tp.fc2),
                                     tp.fc2_bias)


def _check(got, tp, tokens):
    ref = np.stack([tp.embed_text_token(int(t)) for t in tokens])
    scale = max(1.0, float(np.max(np.abs(ref))))
    err = float(np.max(np.abs(got - ref)))
    assert err <= 1e-4 * scale, f"max abs err {err} (scale {scale})"


@pytest.mark.parametrize("vocab,th,mid,hidden", [
    (300, 256, 384, 256),      # fc1 widens, C % 4 == 0: tensor-core GEMV from 8 rows
    (97, 128, 160, 96),        # column groups not a multiple of 4: CUDA-core GEMV only
    (4096, 2048, 2048, 2048),  # the 1.7B model's text path (config.rs:137), smaller vocabulary
])
def test_embed_matches_oracle(E, ctx, orc, vocab, th, mid, hidden):
    tp = orc.TextProj.synth(91, vocab, th, hidden, mid=mid, sigma=0.05)
    dev = E.TextProjection(ctx, _device_weights(tp))
    rng = np.random.default_rng(vocab)
    for count in (1, 5, 8, 37):
        tokens = rng.integers(0, vocab, size=count).astype(np.uint32)
        tokens[0] = vocab - 1                    # last row of the table
        got = dev.embed_text_tokens(tokens).cpu().numpy()
        _check(got, tp, tokens)
    ctx.check_device_error()


@pytest.mark.parametrize("th,mid,hidden", [(256, 384, 256), (128, 160, 96)])
def test_rows_do_not_depend_on_the_batch(E, ctx, orc, th, mid, hidden):
    """A token's row is the same bits alone, in any run and at any position
    (the reference projects one token at a time; its prefix cache relies on
    equal rows).  (128, 160, 96) has column groups that are not a multiple of
    4, so it runs one CUDA-core launch per token."""
    tp = orc.TextProj.synth(94, 500, th, hidden, mid=mid, sigma=0.05)
    dev = E.TextProjection(ctx, _device_weights(tp))
    tokens = np.random.default_rng(1).integers(0, 500, size=45).astype(np.uint32)
    full = dev.embed_text_tokens(tokens).cpu().numpy()
    for lo, hi in ((0, 1), (3, 5), (7, 15), (10, 45), (44, 45)):
        part = dev.embed_text_tokens(tokens[lo:hi]).cpu().numpy()
        assert np.array_equal(part, full[lo:hi]), (lo, hi)
    rev = dev.embed_text_tokens(tokens[::-1].copy()).cpu().numpy()
    assert np.array_equal(rev[::-1], full)


def test_long_prompt_is_chunked(E, ctx, orc):
    """600 tokens: one 512-row chunk and one of 88, same rows as the oracle."""
    tp = orc.TextProj.synth(92, 211, 256, 256, sigma=0.05)
    dev = E.TextProjection(ctx, _device_weights(tp))
    tokens = (np.arange(600, dtype=np.uint32) * 37) % 211
    got = dev.embed_text_tokens(tokens).cpu().numpy()
    _check(got, tp, tokens)
    # a chunk's rows do not depend on which chunk they fall in
    again = dev.embed_text_tokens(tokens[512:]).cpu().numpy()
    assert np.array_equal(again, got[512:])


def test_out_of_vocabulary_token_is_range_error(E, ctx, orc):
    import torch
    from qora_b200 import _lib
    tp = orc.TextProj.synth(93, 64, 128, 128)
    dev = E.TextProjection(ctx, _device_weights(tp))
    out = torch.full((3, 128), 7.0, device="cuda")
    with pytest.raises(_lib.QoraError) as ei:
        dev.embed_text_tokens([1, 64, 2], out=out)
    assert ei.value.status == 5                  # QORA_ERR_RANGE
    assert bool(torch.all(out == 7.0))           # nothing launched
    assert dev.embed_text_tokens([]).shape == (0, 128)
    ctx.check_device_error()


def test_checkpoint_text_path_equals_in_memory(E, ctx, tmp_path):
    import qora_b200
    cfg = qora_b200.ModelConfig.tiny()
    tw, pw = qora_b200.synth_talker(cfg), qora_b200.synth_predictor(cfg)
    text = qf.text_proj_for(cfg, text_vocab=200)
    path = tmp_path / "tiny.qora-tts"
    qf.write(path, tw, pw, cfg, text=text)
    mf = qora_b200.ModelFile(path)
    a = E.TextProjection(ctx, text)
    b = E.TextProjection(ctx, mf.text_proj)
    mf.close()
    tokens = np.arange(0, 200, 7, dtype=np.uint32)
    assert np.array_equal(a.embed_text_tokens(tokens).cpu().numpy(),
                          b.embed_text_tokens(tokens).cpu().numpy())
