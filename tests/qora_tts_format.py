"""Writer of the reference's .qora-tts checkpoint layout (save.rs:22-138 and the
record helpers gemv.rs:595-631), for the model-file reader tests: header
"QTTS", u32 version, u8 format (1 = Q4), then the talker and code-predictor
sections, then bytes standing in for the speech decoder (not read)."""
import ctypes as C
import struct

import numpy as np


def _u8(f, v):
    f.write(struct.pack("<B", v))


def _u32(f, v):
    f.write(struct.pack("<I", v))


def _u64(f, v):
    f.write(struct.pack("<Q", v))


def _f16(f, a):
    a = np.ascontiguousarray(a, np.uint16)
    _u64(f, a.size)
    f.write(a.tobytes())


def _f32(f, a):
    a = np.ascontiguousarray(a, np.float32)
    _u64(f, a.size)
    f.write(a.tobytes())


def _q4(f, w):
    _u64(f, w.k)
    _u64(f, w.n)
    p = np.ascontiguousarray(w.packed, np.uint8)
    _u64(f, p.size)
    f.write(p.tobytes())
    _f16(f, w.scales)


def _layer(f, lw):
    for name in ("q_proj", "k_proj", "v_proj", "o_proj"):
        _q4(f, getattr(lw, name))
    _f16(f, lw.q_norm)
    _f16(f, lw.k_norm)
    for name in ("gate_proj", "up_proj", "down_proj"):
        _q4(f, getattr(lw, name))
    _f16(f, lw.input_norm)
    _f16(f, lw.post_attn_norm)


def rope_tables(head_dim, max_pos, theta):
    """build_mrope_tables (rope.rs:11-41) through the engine library."""
    from qora_b200 import _lib
    half = head_dim // 2
    cos = np.zeros(max_pos * half, np.float32)
    sin = np.zeros(max_pos * half, np.float32)
    _lib.call("qora_rope_tables_host", head_dim, max_pos, theta, None, 0,
              cos.ctypes.data_as(C.c_void_p), sin.ctypes.data_as(C.c_void_p))
    return cos, sin


def text_proj_for(cfg, text_vocab=64):
    """A random-init text path that chains with the talker of `cfg`
    (text_hidden = mid = hidden)."""
    import qora_b200
    return qora_b200.synth_text_proj(71, text_vocab, cfg.t_hidden, cfg.t_hidden)


def write(path, tw, pw, cfg, fmt=1, version=1, theta=None, tail=b"decoder section", text=None):
    theta = cfg.rope_theta if theta is None else theta
    text = text_proj_for(cfg) if text is None else text
    with open(path, "wb") as f:
        f.write(b"QTTS")
        _u32(f, version)
        _u8(f, fmt)
        # talker (save.rs:49-88)
        half = cfg.t_head_dim // 2
        sections = [half - 2 * (half // 3), half // 3, half // 3]
        for v in (cfg.t_layers, cfg.t_hidden, text.text_embedding.n, cfg.t_heads, cfg.t_kv_heads,
                  cfg.t_head_dim, cfg.t_heads // cfg.t_kv_heads, len(sections), *sections):
            _u32(f, v)
        for lw in tw.layers:
            _layer(f, lw)
        _q4(f, tw.codec_embedding)
        _q4(f, text.text_embedding)
        _q4(f, text.fc1)
        _f32(f, text.fc1_bias)
        _q4(f, text.fc2)
        _f32(f, text.fc2_bias)
        _q4(f, tw.codec_head)
        _f16(f, tw.final_norm)
        for a in rope_tables(cfg.t_head_dim, cfg.t_max_pos, theta):
            _f32(f, a)
        # code predictor (save.rs:91-138)
        for v in (cfg.p_layers, cfg.p_hidden, cfg.p_heads, cfg.p_kv_heads, cfg.p_head_dim,
                  cfg.p_heads // cfg.p_kv_heads):
            _u32(f, v)
        _u8(f, 1)
        _q4(f, pw.input_proj)
        _f32(f, pw.input_proj_bias)
        _u32(f, len(pw.codec_embeddings))
        for e in pw.codec_embeddings:
            _q4(f, e)
        for lw in pw.layers:
            _layer(f, lw)
        _u32(f, len(pw.lm_heads))
        for h in pw.lm_heads:
            _q4(f, h)
        _f16(f, pw.final_norm)
        for a in rope_tables(cfg.p_head_dim, cfg.p_max_pos, theta):
            _f32(f, a)
        f.write(tail)
