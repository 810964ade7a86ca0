"""ctypes binding of the speech-decoder oracle (oracle/_build/liboracle_decoder.so)
and the reference's decode_to_audio (decoder.rs:395-582) strung together from it.

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() (as
the checker) and by bench.py's CPU-baseline leg.  The product (the CUDA
library and its Python host mirror) never imports it.

Weights are a dict keyed by the checkpoint's tensor names, in the
checkpoint's layouts (what loader.rs:503-716 reads): Linear [out, in],
Conv1d [out, in, k], ConvTranspose1d [in, out, k], codebooks as
embedding_sum [size, dim] + cluster_usage [size].  Each step below follows
the reference's arithmetic per element (the C primitives keep its order;
numpy is used only for element-wise IEEE operations, which it rounds the same
way), so for the same inputs the oracle gives the reference's bits.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle_decoder.so")
_lib = None

EPS = np.float32(1e-5)     # rms_norm_f32 / layer_norm eps (decoder.rs:229, 288, 309, 346)
DILATIONS = (1, 3, 9)      # loader.rs:622
F32 = np.float32


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            subprocess.run(["make", "-s", "-C", _HERE], check=True)
        L = C.CDLL(_LIB_PATH)
        vp, i64, i32, f32 = C.c_void_p, C.c_int64, C.c_int32, C.c_float
        sig = {
            "od_causal_conv1d": (None, [vp, vp, vp, i32, i32, i32, i32, i64, vp]),
            "od_conv_transpose1d_len": (i64, [i64, i32, i32, i32]),
            "od_conv_transpose1d": (None, [vp, vp, vp, i32, i32, i32, i32, i32, i64, vp]),
            "od_depthwise_conv1d": (None, [vp, vp, vp, i32, i32, i64, vp]),
            "od_layer_norm_cf": (None, [vp, vp, vp, i32, i64, f32, vp]),
            "od_snake_beta": (None, [vp, vp, vp, i32, i64, vp]),
            "od_gelu": (None, [vp, i64]),
            "od_f32_gemm_bias": (None, [vp, vp, vp, i64, i64, i64, vp]),
            "od_f32_gemv_rows": (None, [vp, vp, vp, i64, i64, i64, vp]),
            "od_rms_norm_rows": (None, [vp, vp, i64, i64, f32, vp]),
            "od_rope_tables": (None, [i32, i32, C.c_double, vp, vp]),
            "od_rope_split_half_rows": (None, [vp, i64, i32, i32, vp, vp, i32]),
            "od_window_attention": (None, [vp, vp, vp, i64, i32, i32, i32, f32, vp]),
            "od_silu_mul": (None, [vp, vp, i64, vp]),
            "od_warmup_trim_len": (i64, [i64, i64, i64]),
            "od_xrng_vec": (None, [C.POINTER(C.c_uint64), i64, f32, vp]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        _lib = L
    return _lib


def _c(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=F32)


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


# ------------------------------------------------------------ primitives
def causal_conv1d(x, w, b, dil: int = 1) -> np.ndarray:
    """causal_conv1d (conv.rs:114-230): x [ic][L], w [oc][ic][k]."""
    x, w, b = _c(x), _c(w), _c(b)
    oc, ic, k = w.shape
    assert x.shape[0] == ic
    out = np.empty((oc, x.shape[1]), F32)
    lib().od_causal_conv1d(_p(x), _p(w), _p(b), ic, oc, k, dil, x.shape[1], _p(out))
    return out


def conv_transpose1d(x, w, b, stride: int, pad: int = 0) -> np.ndarray:
    """conv_transpose1d (conv.rs:247-349): x [ic][L], w [ic][oc][k]."""
    x, w, b = _c(x), _c(w), _c(b)
    ic, oc, k = w.shape
    assert x.shape[0] == ic
    n = lib().od_conv_transpose1d_len(x.shape[1], k, stride, pad)
    out = np.empty((oc, n), F32)
    lib().od_conv_transpose1d(_p(x), _p(w), _p(b), ic, oc, k, stride, pad, x.shape[1], _p(out))
    return out


def depthwise_conv1d(x, w, b) -> np.ndarray:
    """depthwise_conv1d (conv.rs:361-432): x [ch][L], w [ch][1][k] (or [ch][k])."""
    x, b = _c(x), _c(b)
    w = _c(w).reshape(x.shape[0], -1)
    out = np.empty_like(x)
    lib().od_depthwise_conv1d(_p(x), _p(w), _p(b), x.shape[0], w.shape[1], x.shape[1], _p(out))
    return out


def layer_norm_cf(x, gamma, beta, eps=EPS) -> np.ndarray:
    """layer_norm_channel_first (decoder.rs:657-684)."""
    x, gamma, beta = _c(x), _c(gamma), _c(beta)
    out = np.empty_like(x)
    lib().od_layer_norm_cf(_p(x), _p(gamma), _p(beta), x.shape[0], x.shape[1], eps, _p(out))
    return out


def snake_beta(x, alpha, beta) -> np.ndarray:
    """snake_beta (conv.rs:545-641)."""
    x, alpha, beta = _c(x), _c(alpha), _c(beta)
    out = np.empty_like(x)
    lib().od_snake_beta(_p(x), _p(alpha), _p(beta), x.shape[0], x.shape[1], _p(out))
    return out


def gelu(x) -> np.ndarray:
    """gelu (conv.rs:692-694), element-wise."""
    y = np.array(x, dtype=F32, copy=True, order="C")
    lib().od_gelu(_p(y), y.size)
    return y


def f32_gemm_bias(a, b, bias) -> np.ndarray:
    """f32_gemm_bias (conv.rs:434-526): a [m][k], b [k][n]."""
    a, b, bias = _c(a), _c(b), _c(bias)
    m, k = a.shape
    assert b.shape[0] == k
    out = np.empty((m, b.shape[1]), F32)
    lib().od_f32_gemm_bias(_p(a), _p(b), _p(bias), m, b.shape[1], k, _p(out))
    return out


def gemv_rows(x, w_in_major, bias=None) -> np.ndarray:
    """f32_gemv / f32_gemv_bias (decoder.rs:596-622) per row: x [rows][k],
    w [k][n] (the reference's transposed, input-major layout)."""
    x, w = _c(x), _c(w_in_major)
    rows, k = x.shape
    assert w.shape[0] == k
    bias = None if bias is None else _c(bias)
    out = np.empty((rows, w.shape[1]), F32)
    lib().od_f32_gemv_rows(_p(x), _p(w), _p(bias), rows, k, w.shape[1], _p(out))
    return out


def rms_norm_rows(x, gamma, eps=EPS) -> np.ndarray:
    """rms_norm_f32 (decoder.rs:585-594) per row."""
    x, gamma = _c(x), _c(gamma)
    out = np.empty_like(x)
    lib().od_rms_norm_rows(_p(x), _p(gamma), x.shape[0], x.shape[1], eps, _p(out))
    return out


def rope_tables(head_dim: int, max_pos: int, theta: float):
    """The decoder's RoPE tables (loader.rs:668-682)."""
    cos_t = np.empty(max_pos * (head_dim // 2), F32)
    sin_t = np.empty_like(cos_t)
    lib().od_rope_tables(head_dim, max_pos, theta, _p(cos_t), _p(sin_t))
    return cos_t, sin_t


def rope_rows(x, heads, head_dim, cos_t, sin_t, max_pos) -> np.ndarray:
    """apply_rope_split_half (decoder.rs:624-647), row r at position r."""
    y = np.array(x, dtype=F32, copy=True, order="C")
    lib().od_rope_split_half_rows(_p(y), y.shape[0], heads, head_dim, _p(cos_t), _p(sin_t), max_pos)
    return y


def window_attention(q, k, v, heads, head_dim, window, scale) -> np.ndarray:
    """Causal sliding-window attention of decoder_transformer (decoder.rs:251-284)."""
    q, k, v = _c(q), _c(k), _c(v)
    out = np.empty_like(q)
    lib().od_window_attention(_p(q), _p(k), _p(v), q.shape[0], heads, head_dim, window, scale, _p(out))
    return out


def silu_mul(gate, up) -> np.ndarray:
    """(g / (1 + exp(-g))) * up (decoder.rs:290-295)."""
    gate, up = _c(gate), _c(up)
    out = np.empty_like(gate)
    lib().od_silu_mul(_p(gate), _p(up), gate.size, _p(out))
    return out


def warmup_trim_len(tv_frames: int, total_frames: int, out_len: int) -> int:
    """warmup_trim_len (decoder.rs:649-656)."""
    return int(lib().od_warmup_trim_len(tv_frames, total_frames, out_len))


def ema_codebook(emb_sum, usage) -> np.ndarray:
    """ema_codebook (loader.rs:488-501): embedding_sum / max(cluster_usage, 1e-8)
    per row (f32::max ignores NaN, as np.fmax does)."""
    u = np.fmax(_c(usage), F32(1e-8))
    return (_c(emb_sum) / u[:, None]).astype(F32)


# ------------------------------------------------------------ the decoder
def codebook_lookup(W: dict, codes: np.ndarray) -> np.ndarray:
    """codebook_lookup (decoder.rs:142-193): codes [16][T] -> [vq_dim][T]."""
    codes = np.asarray(codes)
    nq, T = codes.shape
    q = "decoder.quantizer"
    cb0 = ema_codebook(W[f"{q}.rvq_first.vq.layers.0._codebook.embedding_sum"],
                       W[f"{q}.rvq_first.vq.layers.0._codebook.cluster_usage"])
    p0 = W[f"{q}.rvq_first.output_proj.weight"]
    p0 = _c(p0.reshape(p0.shape[0], -1).T)           # [256][512] (transpose_2d, loader.rs:527-529)
    pr = W[f"{q}.rvq_rest.output_proj.weight"]
    pr = _c(pr.reshape(pr.shape[0], -1).T)
    out = np.zeros((p0.shape[1], T), F32)
    out += gemv_rows(cb0[codes[0]], p0).T
    sum_emb = np.zeros((T, cb0.shape[1]), F32)
    for g in range(nq - 1):
        cb = ema_codebook(W[f"{q}.rvq_rest.vq.layers.{g}._codebook.embedding_sum"],
                          W[f"{q}.rvq_rest.vq.layers.{g}._codebook.cluster_usage"])
        sum_emb += cb[codes[g + 1]]
    out += gemv_rows(sum_emb, pr).T
    return out


def decoder_transformer(W: dict, x_ch: np.ndarray, dims) -> np.ndarray:
    """decoder_transformer (decoder.rs:196-333): [latent][T] -> [latent][T]."""
    p = "decoder.pre_transformer"
    lin = lambda key: _c(W[key].T)                    # read_linear_f32 (loader.rs:477-485)
    x = gemv_rows(_c(x_ch.T), lin(f"{p}.input_proj.weight"), W[f"{p}.input_proj.bias"])
    cos_t, sin_t = rope_tables(dims.head_dim, dims.rope_max_pos, dims.rope_theta)
    scale = F32(1.0) / np.sqrt(F32(dims.head_dim))
    for i in range(dims.num_layers):
        L = f"{p}.layers.{i}"
        xn = rms_norm_rows(x, W[f"{L}.input_layernorm.weight"])
        q = gemv_rows(xn, lin(f"{L}.self_attn.q_proj.weight"))
        k = gemv_rows(xn, lin(f"{L}.self_attn.k_proj.weight"))
        v = gemv_rows(xn, lin(f"{L}.self_attn.v_proj.weight"))
        q = rope_rows(q, dims.num_heads, dims.head_dim, cos_t, sin_t, dims.rope_max_pos)
        k = rope_rows(k, dims.num_heads, dims.head_dim, cos_t, sin_t, dims.rope_max_pos)
        att = window_attention(q, k, v, dims.num_heads, dims.head_dim, dims.sliding_window, scale)
        o = gemv_rows(att, lin(f"{L}.self_attn.o_proj.weight"))
        x = x + o * _c(W[f"{L}.self_attn_layer_scale.scale"])
        xn = rms_norm_rows(x, W[f"{L}.post_attention_layernorm.weight"])
        gate = gemv_rows(xn, lin(f"{L}.mlp.gate_proj.weight"))
        up = gemv_rows(xn, lin(f"{L}.mlp.up_proj.weight"))
        mlp = gemv_rows(silu_mul(gate, up), lin(f"{L}.mlp.down_proj.weight"))
        x = x + mlp * _c(W[f"{L}.mlp_layer_scale.scale"])
    x = rms_norm_rows(x, W[f"{p}.norm.weight"])
    out = gemv_rows(x, lin(f"{p}.output_proj.weight"), W[f"{p}.output_proj.bias"])
    return _c(out.T)


def convnext(W: dict, x: np.ndarray, i: int) -> np.ndarray:
    """convnext_forward (decoder.rs:337-382) of upsample stage i."""
    cn = f"decoder.upsample.{i}.1"
    dw = depthwise_conv1d(x, W[f"{cn}.dwconv.conv.weight"], W[f"{cn}.dwconv.conv.bias"])
    normed = layer_norm_cf(dw, W[f"{cn}.norm.weight"], W[f"{cn}.norm.bias"])
    h = gelu(f32_gemm_bias(W[f"{cn}.pwconv1.weight"], normed, W[f"{cn}.pwconv1.bias"]))
    y = f32_gemm_bias(W[f"{cn}.pwconv2.weight"], h, W[f"{cn}.pwconv2.bias"])
    return x + _c(W[f"{cn}.gamma"])[:, None] * y


def _crop(y: np.ndarray, k: int, s: int) -> np.ndarray:
    """Causal right-crop of kernel_size - stride positions (decoder.rs:462-474)."""
    return _c(y[:, :y.shape[1] - (k - s)]) if k > s else y


def decode_to_audio(W: dict, codes, warmup=None, dims=None) -> np.ndarray:
    """decode_to_audio (decoder.rs:395-582): codes [16][T] (and optional warm-up
    codes [16][Tv] prepended, then trimmed) -> f32 samples at 24 kHz."""
    codes = np.asarray(codes, dtype=np.int64)
    if codes.shape[1] == 0:
        return np.zeros(0, F32)
    trim = None
    if warmup is not None:
        wu = np.asarray(warmup, dtype=np.int64)
        if wu.ndim == 2 and wu.shape[0] == codes.shape[0] and wu.shape[1] > 0:
            trim = (wu.shape[1], wu.shape[1] + codes.shape[1])
            codes = np.concatenate([wu, codes], axis=1)
    sig = codebook_lookup(W, codes)
    sig = causal_conv1d(sig, W["decoder.pre_conv.conv.weight"], W["decoder.pre_conv.conv.bias"])
    sig = decoder_transformer(W, sig, dims)
    for i in range(dims.upsample_stages):
        ct = f"decoder.upsample.{i}.0.conv"
        w = W[f"{ct}.weight"]
        sig = _crop(conv_transpose1d(sig, w, W[f"{ct}.bias"], 2), w.shape[2], 2)
        sig = convnext(W, sig, i)
    sig = causal_conv1d(sig, W["decoder.decoder.0.conv.weight"], W["decoder.decoder.0.conv.bias"])
    for bi in range(len(dims.vocos_strides)):
        b = f"decoder.decoder.{bi + 1}.block"
        sig = snake_beta(sig, W[f"{b}.0.alpha"], W[f"{b}.0.beta"])
        w = W[f"{b}.1.conv.weight"]
        s = dims.vocos_strides[bi]
        sig = _crop(conv_transpose1d(sig, w, W[f"{b}.1.conv.bias"], s), w.shape[2], s)
        for ri in range(3):
            r = f"{b}.{ri + 2}"
            h = snake_beta(sig, W[f"{r}.act1.alpha"], W[f"{r}.act1.beta"])
            h = causal_conv1d(h, W[f"{r}.conv1.conv.weight"], W[f"{r}.conv1.conv.bias"], DILATIONS[ri])
            h = snake_beta(h, W[f"{r}.act2.alpha"], W[f"{r}.act2.beta"])
            h = causal_conv1d(h, W[f"{r}.conv2.conv.weight"], W[f"{r}.conv2.conv.bias"])
            sig = h + sig
    n = len(dims.vocos_strides) + 1
    sig = snake_beta(sig, W[f"decoder.decoder.{n}.alpha"], W[f"decoder.decoder.{n}.beta"])
    sig = causal_conv1d(sig, W[f"decoder.decoder.{n + 1}.conv.weight"], W[f"decoder.decoder.{n + 1}.conv.bias"])
    out = np.clip(sig[0], F32(-1.0), F32(1.0))
    if trim is not None:
        out = out[warmup_trim_len(trim[0], trim[1], out.shape[0]):]
    return _c(out)


# ------------------------------------------------------------ conv.rs test RNG
def xrng_vec(state: int, n: int, mag: float):
    """rvec of conv.rs's tests (conv.rs:700-711): xorshift64 (<<13, >>7, <<17),
    value ((x % 2000) / 1000 - 1) * mag in f32.  Returns (values, new state)."""
    out = np.empty(n, F32)
    st = C.c_uint64(state)
    lib().od_xrng_vec(C.byref(st), n, F32(mag), _p(out))
    return out, int(st.value)
