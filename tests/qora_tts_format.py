"""Writer of the reference's .qora-tts checkpoint layout (save.rs:22-262 and
the record helpers gemv.rs:595-631), for the model-file reader tests: header
"QTTS", u32 version, u8 format (1 = Q4), then the talker and code-predictor
sections, then the speech-decoder section (decoder_section) or bytes standing
in for it."""
import ctypes as C
import io
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


def decoder_section(W, dims) -> bytes:
    """The speech-decoder section as save_decoder writes it (save.rs:171-262),
    from checkpoint-named weights W after load_speech_decoder's processing
    (loader.rs:503-716): codebooks divided by max(cluster_usage, 1e-8)
    (ema_codebook), linear weights and the codebook projections transposed to
    [in][out] (read_linear_f32 / transpose_2d), ConvNeXt pointwise weights
    transposed likewise; convolutions with their headers (save.rs:139-169);
    the standard RoPE tables (loader.rs:668-682)."""
    f = io.BytesIO()
    F32 = np.float32
    lin = lambda key: np.ascontiguousarray(np.asarray(W[key], F32).reshape(W[key].shape[0], -1).T)
    ema = lambda pre: (np.asarray(W[pre + "embedding_sum"], F32)
                       / np.fmax(np.asarray(W[pre + "cluster_usage"], F32), F32(1e-8))[:, None]).astype(F32)

    def conv(key, dil=1, stride=1):
        w = np.asarray(W[key + "weight"], F32)
        for v in (w.shape[1], w.shape[0], w.shape[2], stride, 0, dil):
            _u32(f, v)
        _f32(f, w)
        _f32(f, W[key + "bias"])

    def convt(key, stride):
        w = np.asarray(W[key + "weight"], F32)
        for v in (w.shape[0], w.shape[1], w.shape[2], stride, 0):
            _u32(f, v)
        _f32(f, w)
        _f32(f, W[key + "bias"])

    for v in (dims.hidden, dims.num_heads, dims.head_dim, dims.intermediate, dims.sliding_window,
              dims.codebook_dim):
        _u32(f, v)
    q = "decoder.quantizer."
    _f32(f, ema(q + "rvq_first.vq.layers.0._codebook."))
    _f32(f, lin(q + "rvq_first.output_proj.weight"))
    _u32(f, dims.num_quantizers - 1)
    for g in range(dims.num_quantizers - 1):
        _f32(f, ema(q + f"rvq_rest.vq.layers.{g}._codebook."))
    _f32(f, lin(q + "rvq_rest.output_proj.weight"))
    conv("decoder.pre_conv.conv.")
    t = "decoder.pre_transformer."
    _f32(f, lin(t + "input_proj.weight"))
    _f32(f, W[t + "input_proj.bias"])
    _u32(f, dims.num_layers)
    for i in range(dims.num_layers):
        L = f"{t}layers.{i}."
        for n in ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                  "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj"):
            _f32(f, lin(L + n + ".weight"))
        for n in ("input_layernorm.weight", "post_attention_layernorm.weight",
                  "self_attn_layer_scale.scale", "mlp_layer_scale.scale"):
            _f32(f, W[L + n])
    _f32(f, W[t + "norm.weight"])
    _f32(f, lin(t + "output_proj.weight"))
    _f32(f, W[t + "output_proj.bias"])
    _u32(f, dims.upsample_stages)
    for i in range(dims.upsample_stages):
        ct, cn = f"decoder.upsample.{i}.0.conv.", f"decoder.upsample.{i}.1."
        _u32(f, dims.latent)
        convt(ct, 2)
        dw = np.asarray(W[cn + "dwconv.conv.weight"], F32)
        for v in (dims.latent, dw.shape[2], 3):
            _u32(f, v)
        _f32(f, dw)
        _f32(f, W[cn + "dwconv.conv.bias"])
        _f32(f, W[cn + "norm.weight"])
        _f32(f, W[cn + "norm.bias"])
        _f32(f, lin(cn + "pwconv1.weight"))
        _f32(f, W[cn + "pwconv1.bias"])
        _f32(f, lin(cn + "pwconv2.weight"))
        _f32(f, W[cn + "pwconv2.bias"])
        _f32(f, W[cn + "gamma"])
    conv("decoder.decoder.0.conv.")
    _u32(f, len(dims.vocos_strides))
    for b, s in enumerate(dims.vocos_strides):
        p = f"decoder.decoder.{b + 1}.block."
        _f32(f, W[p + "0.alpha"])
        _f32(f, W[p + "0.beta"])
        convt(p + "1.conv.", s)
        _u32(f, 3)
        for r, dil in enumerate((1, 3, 9)):
            u = f"{p}{r + 2}."
            _f32(f, W[u + "act1.alpha"])
            _f32(f, W[u + "act1.beta"])
            conv(u + "conv1.conv.", dil)
            _f32(f, W[u + "act2.alpha"])
            _f32(f, W[u + "act2.beta"])
            conv(u + "conv2.conv.")
    nb = len(dims.vocos_strides)
    _f32(f, W[f"decoder.decoder.{nb + 1}.alpha"])
    _f32(f, W[f"decoder.decoder.{nb + 1}.beta"])
    conv(f"decoder.decoder.{nb + 2}.conv.")
    for a in rope_tables(dims.head_dim, dims.rope_max_pos, dims.rope_theta):
        _f32(f, a)
    return f.getvalue()
