"""The .qora-tts reader (save.rs:262-409): a checkpoint written in the
reference's layout is read back through the C ABI with every array equal to
what was written, and malformed files are errors, not crashes."""
import ctypes as C
import os

import numpy as np
import pytest

import qora_tts_format as qf


@pytest.fixture(scope="module")
def model():
    import qora_b200
    cfg = qora_b200.ModelConfig.tiny()
    return cfg, qora_b200.synth_talker(cfg), qora_b200.synth_predictor(cfg)


def _arr(ptr, n, dt):
    assert ptr
    return np.ctypeslib.as_array(C.cast(ptr, C.POINTER(np.ctypeslib.as_ctypes_type(dt))), shape=(n,))


def _same_q4(h, w):
    assert (h.k, h.n) == (w.k, w.n)
    assert np.array_equal(_arr(h.packed, w.k * w.n // 2, np.uint8), w.packed.reshape(-1))
    assert np.array_equal(_arr(h.scales, w.k * (w.n // 32), np.uint16), w.scales.reshape(-1))


def _same_layer(h, lw, hidden, hd):
    for name in ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"):
        _same_q4(getattr(h, name), getattr(lw, name))
    assert np.array_equal(_arr(h.q_norm, hd, np.uint16), lw.q_norm)
    assert np.array_equal(_arr(h.k_norm, hd, np.uint16), lw.k_norm)
    assert np.array_equal(_arr(h.input_norm, hidden, np.uint16), lw.input_norm)
    assert np.array_equal(_arr(h.post_attn_norm, hidden, np.uint16), lw.post_attn_norm)


def test_reads_back_every_array(model, tmp_path):
    import qora_b200
    from qora_b200 import _lib
    cfg, tw, pw = model
    path = tmp_path / "tiny.qora-tts"
    text = qora_b200.synth_text_proj(81, 96, cfg.t_hidden, cfg.t_hidden, mid=2 * cfg.t_hidden)
    qf.write(path, tw, pw, cfg, text=text)
    mf = qora_b200.ModelFile(path)
    c = mf.cfg
    for k in ("t_layers", "t_hidden", "t_heads", "t_kv_heads", "t_head_dim", "t_ffn", "t_vocab",
              "t_max_pos", "p_layers", "p_hidden", "p_heads", "p_kv_heads", "p_head_dim", "p_ffn",
              "p_vocab", "p_groups", "p_max_pos"):
        assert getattr(c, k) == getattr(cfg, k), k
    t, p = mf.talker_host, mf.predictor_host
    assert t.rope_theta == cfg.rope_theta and p.rope_theta == cfg.rope_theta
    tl = (_lib.LayerHost * cfg.t_layers).from_address(t.layers)
    for i, lw in enumerate(tw.layers):
        _same_layer(tl[i], lw, cfg.t_hidden, cfg.t_head_dim)
    _same_q4(t.codec_embedding, tw.codec_embedding)
    _same_q4(t.codec_head, tw.codec_head)
    assert np.array_equal(_arr(t.final_norm, cfg.t_hidden, np.uint16), tw.final_norm)
    pl = (_lib.LayerHost * cfg.p_layers).from_address(p.layers)
    for i, lw in enumerate(pw.layers):
        _same_layer(pl[i], lw, cfg.p_hidden, cfg.p_head_dim)
    _same_q4(p.input_proj, pw.input_proj)
    assert np.array_equal(_arr(p.input_proj_bias, cfg.p_hidden, np.float32), pw.input_proj_bias)
    embs = (_lib.Q4Host * cfg.p_groups).from_address(p.codec_embeddings)
    heads = (_lib.Q4Host * cfg.p_groups).from_address(p.lm_heads)
    for g in range(cfg.p_groups):
        _same_q4(embs[g], pw.codec_embeddings[g])
        _same_q4(heads[g], pw.lm_heads[g])
    assert np.array_equal(_arr(p.final_norm, cfg.p_hidden, np.uint16), pw.final_norm)
    x = mf.text_proj_host
    _same_q4(x.text_embedding, text.text_embedding)
    _same_q4(x.fc1, text.fc1)
    _same_q4(x.fc2, text.fc2)
    assert np.array_equal(_arr(x.fc1_bias, text.fc1.n, np.float32), text.fc1_bias)
    assert np.array_equal(_arr(x.fc2_bias, text.fc2.n, np.float32), text.fc2_bias)
    mf.close()


def _status(path):
    import qora_b200
    from qora_b200 import _lib
    with pytest.raises(_lib.QoraError) as ei:
        qora_b200.ModelFile(path)
    return ei.value.status


def test_malformed_files_are_errors(model, tmp_path):
    cfg, tw, pw = model
    good = tmp_path / "good.qora-tts"
    qf.write(good, tw, pw, cfg, tail=b"")
    data = good.read_bytes()
    bad = tmp_path / "bad.qora-tts"
    bad.write_bytes(b"XTTS" + data[4:])
    assert _status(bad) == 1                       # QORA_ERR_INVALID: magic
    for cut in (3, 9, 40, len(data) // 3, len(data) // 2, len(data) - 1):
        bad.write_bytes(data[:cut])
        assert _status(bad) == 1, cut              # truncated
    qf.write(bad, tw, pw, cfg, version=2)
    assert _status(bad) == 6                       # QORA_ERR_UNSUPPORTED
    qf.write(bad, tw, pw, cfg, fmt=0)
    assert _status(bad) == 6
    qf.write(bad, tw, pw, cfg, theta=1e6 + 0.25)   # tables of a non-integer base
    assert _status(bad) == 6
    import qora_b200
    text = qora_b200.synth_text_proj(82, 32, cfg.t_hidden, cfg.t_hidden + 32)
    qf.write(bad, tw, pw, cfg, text=text)          # fc2 output != talker hidden
    assert _status(bad) == 1
    assert _status(tmp_path / "missing.qora-tts") == 1
    os.remove(bad)


def test_corrupted_bytes_never_crash(model, tmp_path):
    """Seeded byte flips anywhere in the file: every open either succeeds or
    returns an error status (every length is checked before it is used)."""
    from qora_b200 import _lib
    import qora_b200
    cfg, tw, pw = model
    good = tmp_path / "good.qora-tts"
    qf.write(good, tw, pw, cfg)
    data = bytearray(good.read_bytes())
    rng = np.random.default_rng(5)
    bad = tmp_path / "flip.qora-tts"
    for _ in range(60):
        d = bytearray(data)
        for pos in rng.integers(0, len(d), size=3):
            d[pos] ^= int(rng.integers(1, 256))
        bad.write_bytes(bytes(d))
        try:
            qora_b200.ModelFile(bad).close()
        except _lib.QoraError:
            pass
