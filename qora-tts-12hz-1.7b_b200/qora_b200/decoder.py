"""The speech decoder (decoder.rs): 16 codes per 12.5 Hz frame -> 24 kHz audio.

Host mirror of the reference's SpeechDecoderWeights / load_speech_decoder /
decode_to_audio (decoder.rs:24-66, 395-582; loader.rs:503-716) over the C ABI
(qora_decoder_* in include/qora_cuda.h).  Weights are given by checkpoint
tensor name in the checkpoint's own layouts, as load_speech_decoder reads
them from the speech tokenizer's safetensors file.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib
from .weights import synth_normal


@dataclass
class DecoderDims:
    """Decoder dims; defaults are the 12 Hz speech tokenizer's (decoder.rs:1-14,
    loader.rs:503-716)."""
    codebook_dim: int = 256
    codebook_size: int = 2048
    num_quantizers: int = 16
    vq_dim: int = 512
    latent: int = 1024
    hidden: int = 512
    num_heads: int = 16
    head_dim: int = 64
    intermediate: int = 1024
    num_layers: int = 8
    sliding_window: int = 72
    upsample_stages: int = 2
    upsample_inner: int = 4096
    vocos_channels: tuple = (1536, 768, 384, 192, 96)
    vocos_kernels: tuple = (16, 10, 8, 6)
    vocos_strides: tuple = (8, 5, 4, 3)
    rope_max_pos: int = 8000
    rope_theta: float = 10000.0

    @staticmethod
    def tiny(**kw) -> "DecoderDims":
        """Small channel counts, the real strides, kernels and structure."""
        base = dict(codebook_dim=16, codebook_size=64, vq_dim=32, latent=64, hidden=64, num_heads=2,
                    intermediate=64, num_layers=2, sliding_window=6, upsample_inner=128,
                    vocos_channels=(96, 48, 24, 12, 8))
        base.update(kw)
        return DecoderDims(**base)

    @property
    def hop(self) -> int:
        """Samples per frame (1920 at the real dims: 2 x 2 x 8 x 5 x 4 x 3)."""
        h = 2 ** self.upsample_stages
        for s in self.vocos_strides:
            h *= s
        return h

    def c_struct(self) -> _lib.DecoderDims:
        d = _lib.DecoderDims()
        for n in ("codebook_dim", "codebook_size", "num_quantizers", "vq_dim", "latent", "hidden",
                  "num_heads", "head_dim", "intermediate", "num_layers", "sliding_window",
                  "upsample_stages", "upsample_inner", "rope_max_pos"):
            setattr(d, n, getattr(self, n))
        d.vocos_blocks = len(self.vocos_strides)
        for i, v in enumerate(self.vocos_channels):
            d.vocos_channels[i] = v
        for i, (k, s) in enumerate(zip(self.vocos_kernels, self.vocos_strides)):
            d.vocos_kernels[i] = k
            d.vocos_strides[i] = s
        d.rope_theta = self.rope_theta
        return d


def decoder_tensor_shapes(dims: DecoderDims) -> dict:
    """Checkpoint tensor name -> shape, for every tensor load_speech_decoder
    reads (loader.rs:503-716)."""
    d = dims
    HD = d.num_heads * d.head_dim
    q = "decoder.quantizer."
    s = {f"{q}rvq_first.vq.layers.0._codebook.embedding_sum": (d.codebook_size, d.codebook_dim),
         f"{q}rvq_first.vq.layers.0._codebook.cluster_usage": (d.codebook_size,),
         f"{q}rvq_first.output_proj.weight": (d.vq_dim, d.codebook_dim, 1)}
    for g in range(d.num_quantizers - 1):
        s[f"{q}rvq_rest.vq.layers.{g}._codebook.embedding_sum"] = (d.codebook_size, d.codebook_dim)
        s[f"{q}rvq_rest.vq.layers.{g}._codebook.cluster_usage"] = (d.codebook_size,)
    s[f"{q}rvq_rest.output_proj.weight"] = (d.vq_dim, d.codebook_dim, 1)
    s["decoder.pre_conv.conv.weight"] = (d.latent, d.vq_dim, 3)
    s["decoder.pre_conv.conv.bias"] = (d.latent,)
    t = "decoder.pre_transformer."
    s[f"{t}input_proj.weight"] = (d.hidden, d.latent)
    s[f"{t}input_proj.bias"] = (d.hidden,)
    s[f"{t}output_proj.weight"] = (d.latent, d.hidden)
    s[f"{t}output_proj.bias"] = (d.latent,)
    s[f"{t}norm.weight"] = (d.hidden,)
    for i in range(d.num_layers):
        L = f"{t}layers.{i}."
        for n in ("q_proj", "k_proj", "v_proj"):
            s[f"{L}self_attn.{n}.weight"] = (HD, d.hidden)
        s[f"{L}self_attn.o_proj.weight"] = (d.hidden, HD)
        s[f"{L}mlp.gate_proj.weight"] = (d.intermediate, d.hidden)
        s[f"{L}mlp.up_proj.weight"] = (d.intermediate, d.hidden)
        s[f"{L}mlp.down_proj.weight"] = (d.hidden, d.intermediate)
        for n in ("input_layernorm.weight", "post_attention_layernorm.weight",
                  "self_attn_layer_scale.scale", "mlp_layer_scale.scale"):
            s[L + n] = (d.hidden,)
    for i in range(d.upsample_stages):
        ct, cn = f"decoder.upsample.{i}.0.conv.", f"decoder.upsample.{i}.1."
        s[ct + "weight"] = (d.latent, d.latent, 2)
        s[ct + "bias"] = (d.latent,)
        s[cn + "dwconv.conv.weight"] = (d.latent, 1, 7)
        s[cn + "dwconv.conv.bias"] = (d.latent,)
        s[cn + "norm.weight"] = (d.latent,)
        s[cn + "norm.bias"] = (d.latent,)
        s[cn + "pwconv1.weight"] = (d.upsample_inner, d.latent)
        s[cn + "pwconv1.bias"] = (d.upsample_inner,)
        s[cn + "pwconv2.weight"] = (d.latent, d.upsample_inner)
        s[cn + "pwconv2.bias"] = (d.latent,)
        s[cn + "gamma"] = (d.latent,)
    ch = d.vocos_channels
    s["decoder.decoder.0.conv.weight"] = (ch[0], d.latent, 7)
    s["decoder.decoder.0.conv.bias"] = (ch[0],)
    for b, (k, st) in enumerate(zip(d.vocos_kernels, d.vocos_strides)):
        p = f"decoder.decoder.{b + 1}.block."
        s[p + "0.alpha"] = (ch[b],)
        s[p + "0.beta"] = (ch[b],)
        s[p + "1.conv.weight"] = (ch[b], ch[b + 1], k)
        s[p + "1.conv.bias"] = (ch[b + 1],)
        for r in range(3):
            u = f"{p}{r + 2}."
            for a in ("act1", "act2"):
                s[f"{u}{a}.alpha"] = (ch[b + 1],)
                s[f"{u}{a}.beta"] = (ch[b + 1],)
            s[u + "conv1.conv.weight"] = (ch[b + 1], ch[b + 1], 7)
            s[u + "conv1.conv.bias"] = (ch[b + 1],)
            s[u + "conv2.conv.weight"] = (ch[b + 1], ch[b + 1], 1)
            s[u + "conv2.conv.bias"] = (ch[b + 1],)
    nb = len(d.vocos_strides)
    s[f"decoder.decoder.{nb + 1}.alpha"] = (ch[nb],)
    s[f"decoder.decoder.{nb + 1}.beta"] = (ch[nb],)
    s[f"decoder.decoder.{nb + 2}.conv.weight"] = (1, ch[nb], 7)
    s[f"decoder.decoder.{nb + 2}.conv.bias"] = (1,)
    return s


def _sigma(name: str, shape) -> tuple:
    """(mean, sigma) of a synthetic tensor: fan-in scaled weights, residual
    branches damped, norms and scales near their usual values, so the
    activations stay O(1) through the stack."""
    if name.endswith("cluster_usage"):
        return 2.0, 0.5
    if name.endswith("embedding_sum"):
        return 0.0, 2.0
    if name.endswith((".alpha", ".beta")):
        return 0.0, 0.1
    if name.endswith(("layernorm.weight", "norm.weight")):
        return 1.0, 0.05
    if name.endswith("norm.bias"):
        return 0.0, 0.05
    if name.endswith(("layer_scale.scale", ".gamma")):
        return 0.1, 0.02
    if name.endswith(".bias"):
        return 0.0, 0.01
    fan_in = int(np.prod(shape[1:])) if len(shape) > 1 else 1
    if ".block.1.conv.weight" in name or name.startswith("decoder.upsample.") and ".0.conv" in name:
        fan_in = shape[0] * max(1, shape[2] // 2)          # ConvTranspose [in][out][k]
    g = 1.0
    if "conv2.conv.weight" in name:
        g = 0.5                                             # residual unit output
    elif name.startswith("decoder.decoder.") and name.endswith(".conv.weight") and shape[0] == 1:
        g = 0.15                                            # output conv: samples mostly inside [-1, 1]
    return 0.0, g / np.sqrt(fan_in)


def synth_decoder(dims: DecoderDims, seed: int = 4321) -> dict:
    """Deterministic random-init decoder weights (splitmix64 + Box-Muller, as
    the engine's other synthetic weights), keyed by checkpoint tensor name."""
    out = {}
    for i, (name, shape) in enumerate(sorted(decoder_tensor_shapes(dims).items())):
        mean, sigma = _sigma(name, shape)
        n = int(np.prod(shape))
        v = synth_normal(seed * 1000003 + i, float(sigma), n).reshape(shape)
        if name.endswith("cluster_usage"):
            v = np.abs(v) + np.float32(mean)
        elif mean:
            v = v + np.float32(mean)
        out[name] = v.astype(np.float32)
    return out


class SpeechDecoder:
    """SpeechDecoderWeights on the device (qora_decoder).  `weights` maps every
    checkpoint tensor name to its values (any array-like of the right size)."""

    def __init__(self, ctx, dims: DecoderDims, weights: dict):
        self.ctx, self.dims = ctx, dims
        self._L = _lib.load()
        h = C.c_void_p()
        cd = dims.c_struct()
        _lib.call("qora_decoder_create", ctx.h, C.byref(cd), C.byref(h))
        self.h = h
        for name, v in weights.items():
            a = np.ascontiguousarray(v, dtype=np.float32)
            _lib.call("qora_decoder_set_tensor", self.h, name.encode(), a.ctypes.data, a.size)
        _lib.call("qora_decoder_finalize", self.h)

    @classmethod
    def from_model_file(cls, ctx, mf) -> "SpeechDecoder":
        """The speech decoder of a .qora-tts checkpoint (load_decoder_weights,
        save.rs:446-552); `mf` a qora_b200.ModelFile."""
        self = cls.__new__(cls)
        self.ctx, self._L = ctx, _lib.load()
        h = C.c_void_p()
        _lib.call("qora_model_file_decoder", mf.h, ctx.h, C.byref(h))
        self.h = h
        cd = _lib.DecoderDims()
        _lib.call("qora_decoder_get_dims", self.h, C.byref(cd))
        nb = cd.vocos_blocks
        self.dims = DecoderDims(
            codebook_dim=cd.codebook_dim, codebook_size=cd.codebook_size, num_quantizers=cd.num_quantizers,
            vq_dim=cd.vq_dim, latent=cd.latent, hidden=cd.hidden, num_heads=cd.num_heads, head_dim=cd.head_dim,
            intermediate=cd.intermediate, num_layers=cd.num_layers, sliding_window=cd.sliding_window,
            upsample_stages=cd.upsample_stages, upsample_inner=cd.upsample_inner,
            vocos_channels=tuple(cd.vocos_channels[:nb + 1]), vocos_kernels=tuple(cd.vocos_kernels[:nb]),
            vocos_strides=tuple(cd.vocos_strides[:nb]), rope_max_pos=cd.rope_max_pos, rope_theta=cd.rope_theta)
        return self

    def close(self):
        if getattr(self, "h", None):
            self._L.qora_decoder_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def use_tensor_cores(self, mode: int) -> None:
        """0: every convolution on the CUDA cores; 1 (default): the tensor
        cores where the grid fills the GPU; 2: the tensor cores wherever the
        convolution has a tensor-core form."""
        _lib.call("qora_decoder_use_tensor_cores", self.h, mode)

    def samples(self, frames: int) -> int:
        n = C.c_int64()
        _lib.call("qora_decoder_samples", self.h, frames, C.byref(n))
        return int(n.value)

    def decode_to_audio(self, codes, warmup=None, stream=None) -> np.ndarray:
        """decode_to_audio (decoder.rs:395-582): codes [num_quantizers][T]
        (host), optional warm-up codes [num_quantizers][Tv] -> samples."""
        codes = np.ascontiguousarray(codes, dtype=np.uint32)
        nq, T = codes.shape
        if nq != self.dims.num_quantizers:
            raise ValueError(f"codes have {nq} quantizers, the decoder {self.dims.num_quantizers}")
        wu, tv = None, 0
        if warmup is not None:
            wu = np.ascontiguousarray(warmup, dtype=np.uint32)
            if wu.ndim == 2 and wu.shape[0] == nq and wu.shape[1] > 0:
                tv = wu.shape[1]
            else:
                wu = None
        out = np.empty(max(1, self.samples(T + tv)), np.float32)
        n = C.c_int64()
        s = 0 if stream is None else stream.cuda_stream
        _lib.call("qora_decode_to_audio", self.h, codes.ctypes.data, T,
                  None if wu is None else wu.ctypes.data, tv, out.ctypes.data, out.size, C.byref(n), s)
        return out[:n.value].copy()

    def decode_device(self, codes_dev, frames: int, samples_dev, warmup_frames: int = 0, stream=None) -> int:
        """qora_decode_to_audio_device on device buffers (torch tensors):
        codes [num_quantizers][warmup_frames + frames] uint32 / int32,
        samples >= frames * hop floats.  Returns the kernels launched."""
        n = C.c_int32()
        s = 0 if stream is None else stream.cuda_stream
        _lib.call("qora_decode_to_audio_device", self.h, codes_dev.data_ptr(), frames, warmup_frames,
                  samples_dev.data_ptr(), C.byref(n), s)
        return int(n.value)


# ------------------------------------------------- the decoder's code inputs
def warmup_tail(codes, k: int) -> np.ndarray:
    """warmup_tail (generate_new.rs:728-737): the last k frames of every
    quantizer row of codes [num_quantizers][T], the warm-up codes the next
    chunk of the same voice hands to decode_to_audio (generate_new.rs:704;
    main.rs:642).  k == 0 or k >= T gives all of codes; no rows gives none."""
    codes = np.asarray(codes, dtype=np.uint32)
    if codes.size == 0 and (codes.ndim < 2 or codes.shape[0] == 0):
        return np.zeros((0, 0), np.uint32)
    if codes.ndim != 2:
        raise ValueError(f"codes must be [num_quantizers][frames], got shape {codes.shape}")
    T = codes.shape[1]
    if k == 0 or k >= T:
        return codes.copy()
    return codes[:, T - k:].copy()


_VCOD = b"VCOD"


def write_codes_file(path, codes) -> None:
    """write_codes_file (generate_new.rs:739-753): "VCOD", u32 quantizer
    rows, u32 frames, then the codes row by row as u16, all little-endian
    (a code keeps its low 16 bits, as the reference's `as u16`)."""
    codes = np.asarray(codes, dtype=np.uint32)
    if codes.ndim != 2 or codes.shape[0] == 0:
        raise ValueError(f"codes must be [num_quantizers][frames] with at least one row, got {codes.shape}")
    with open(path, "wb") as f:
        f.write(_VCOD)
        f.write(np.array(codes.shape, dtype="<u4").tobytes())
        f.write((codes & 0xFFFF).astype("<u2").tobytes())


def read_codes_file(path) -> np.ndarray:
    """load_all_voice_codes (main.rs:697-737): a VCOD file -> codes
    [num_quantizers][frames] uint32.  A wrong magic or a short file raises
    ValueError (the reference prints and exits)."""
    with open(path, "rb") as f:
        raw = f.read()
    if raw[:4] != _VCOD:
        raise ValueError("invalid codes file (bad magic)")
    if len(raw) < 12:
        raise ValueError("codes file too short for its header")
    nq, T = (int(v) for v in np.frombuffer(raw, dtype="<u4", count=2, offset=4))
    if len(raw) < 12 + 2 * nq * T:
        raise ValueError(f"codes file holds {len(raw) - 12} code bytes, {2 * nq * T} expected")
    return np.frombuffer(raw, dtype="<u2", count=nq * T, offset=12).astype(np.uint32).reshape(nq, T)
