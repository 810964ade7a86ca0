"""Host-side weight containers in the reference layout, and synthetic weights.

Mirrors the reference's weight structs (gemv.rs:26-31 Q4Weight,
talker.rs:19-56 TalkerWeights, code_predictor.rs:14-46 CodePredictorWeights)
with numpy arrays, and builds the C-ABI host structs from them.  Synthetic
random-init weights (N(0, sigma), quantised by quantize_f32_to_q4,
gemv.rs:92-130) are produced by the engine library's host generator.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from . import _lib

F16_ONE = np.array([1.0], np.float16).view(np.uint16)[0]


def _ptr(a: np.ndarray | None) -> int | None:
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


@dataclass
class Q4Weight:
    """Q4Weight (gemv.rs:26-31): packed u8[k*n/2] (low nibble = even column),
    scales f16 bit patterns [k*n/32]; input-major [k][n]."""
    packed: np.ndarray
    scales: np.ndarray
    k: int
    n: int

    def host(self) -> _lib.Q4Host:
        return _lib.Q4Host(_ptr(self.packed), _ptr(self.scales), self.k, self.n)

    @property
    def nbytes(self) -> int:
        return self.packed.nbytes + self.scales.nbytes


def quantize_f32_to_q4(data: np.ndarray) -> Q4Weight:
    """quantize_f32_to_q4 (gemv.rs:92-130) via the engine's host quantiser."""
    data = np.ascontiguousarray(data, np.float32)
    k, n = data.shape
    packed = np.empty(k * (n // 32) * 16, np.uint8)
    scales = np.empty(k * (n // 32), np.uint16)
    _lib.call("qora_q4_quantize_host", data.ctypes.data, k, n, packed.ctypes.data,
              scales.ctypes.data)
    return Q4Weight(packed, scales, k, n)


def synth_q4(seed: int, sigma: float, k: int, n: int) -> Q4Weight:
    packed = np.empty(k * (n // 32) * 16, np.uint8)
    scales = np.empty(k * (n // 32), np.uint16)
    _lib.call("qora_synth_q4_host", seed, sigma, k, n, packed.ctypes.data, scales.ctypes.data)
    return Q4Weight(packed, scales, k, n)


def synth_normal(seed: int, sigma: float, count: int) -> np.ndarray:
    out = np.empty(count, np.float32)
    _lib.call("qora_synth_normal_host", seed, sigma, count, out.ctypes.data)
    return out


@dataclass
class ModelConfig:
    """Talker + code-predictor dims.  Defaults: the 1.7B model (config.rs:130-153,
    model/1.7B/config.json; predictor head_dim 128 as in the reference config)."""
    t_layers: int = 28
    t_hidden: int = 2048
    t_heads: int = 16
    t_kv_heads: int = 8
    t_head_dim: int = 128
    t_ffn: int = 6144
    t_vocab: int = 3072
    t_max_pos: int = 4608
    p_layers: int = 5
    p_hidden: int = 1024
    p_heads: int = 16
    p_kv_heads: int = 8
    p_head_dim: int = 128
    p_ffn: int = 3072
    p_vocab: int = 2048
    p_groups: int = 15
    p_max_pos: int = 64
    rope_theta: float = 1e6
    sigma: float = 0.02
    seed: int = 1234

    @staticmethod
    def tiny(**kw) -> "ModelConfig":
        base = dict(t_layers=2, t_hidden=256, t_heads=4, t_kv_heads=2, t_head_dim=64, t_ffn=512,
                    t_vocab=320, t_max_pos=128, p_layers=2, p_hidden=128, p_heads=4, p_kv_heads=2,
                    p_head_dim=64, p_ffn=256, p_vocab=192, p_groups=15, p_max_pos=32)
        base.update(kw)
        return ModelConfig(**base)


@dataclass
class LayerWeights:
    q_proj: Q4Weight
    k_proj: Q4Weight
    v_proj: Q4Weight
    o_proj: Q4Weight
    gate_proj: Q4Weight
    up_proj: Q4Weight
    down_proj: Q4Weight
    q_norm: np.ndarray
    k_norm: np.ndarray
    input_norm: np.ndarray
    post_attn_norm: np.ndarray

    def host(self) -> _lib.LayerHost:
        return _lib.LayerHost(*(getattr(self, n).host() for n in
                                ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj",
                                 "down_proj")),
                              _ptr(self.q_norm), _ptr(self.k_norm), _ptr(self.input_norm),
                              _ptr(self.post_attn_norm))


def synth_layer(seed: int, sigma: float, hidden: int, heads: int, kv_heads: int, hd: int,
                ffn: int) -> LayerWeights:
    """Random-init decoder layer; tensor seeds seed+1..seed+7, norms = 1.0."""
    qd, kd = heads * hd, kv_heads * hd
    return LayerWeights(
        q_proj=synth_q4(seed + 1, sigma, hidden, qd),
        k_proj=synth_q4(seed + 2, sigma, hidden, kd),
        v_proj=synth_q4(seed + 3, sigma, hidden, kd),
        o_proj=synth_q4(seed + 4, sigma, qd, hidden),
        gate_proj=synth_q4(seed + 5, sigma, hidden, ffn),
        up_proj=synth_q4(seed + 6, sigma, hidden, ffn),
        down_proj=synth_q4(seed + 7, sigma, ffn, hidden),
        q_norm=np.full(hd, F16_ONE, np.uint16),
        k_norm=np.full(hd, F16_ONE, np.uint16),
        input_norm=np.full(hidden, F16_ONE, np.uint16),
        post_attn_norm=np.full(hidden, F16_ONE, np.uint16),
    )


@dataclass
class TalkerWeights:
    """TalkerWeights hot-path fields (talker.rs:33-56)."""
    cfg: ModelConfig
    layers: list
    codec_embedding: Q4Weight  # [vocab][hidden]
    codec_head: Q4Weight       # [hidden][vocab]
    final_norm: np.ndarray
    _keep: list = field(default_factory=list)

    def host(self) -> _lib.TalkerHost:
        c = self.cfg
        layers = (_lib.LayerHost * c.t_layers)(*[lw.host() for lw in self.layers])
        self._keep.append(layers)
        return _lib.TalkerHost(c.t_layers, c.t_hidden, c.t_heads, c.t_kv_heads, c.t_head_dim,
                               c.t_ffn, c.t_vocab, c.t_max_pos, c.rope_theta,
                               C.addressof(layers), self.codec_embedding.host(),
                               self.codec_head.host(), _ptr(self.final_norm))

    @property
    def nbytes(self) -> int:
        n = self.codec_head.nbytes
        for lw in self.layers:
            n += sum(getattr(lw, k).nbytes for k in ("q_proj", "k_proj", "v_proj", "o_proj",
                                                     "gate_proj", "up_proj", "down_proj"))
        return n


@dataclass
class PredictorWeights:
    """CodePredictorWeights (code_predictor.rs:28-46)."""
    cfg: ModelConfig
    layers: list
    input_proj: Q4Weight | None
    input_proj_bias: np.ndarray | None
    codec_embeddings: list   # num_groups x [vocab][talker hidden]
    lm_heads: list           # num_groups x [hidden][vocab]
    final_norm: np.ndarray
    _keep: list = field(default_factory=list)

    def host(self) -> _lib.PredictorHost:
        c = self.cfg
        layers = (_lib.LayerHost * c.p_layers)(*[lw.host() for lw in self.layers])
        embs = (_lib.Q4Host * c.p_groups)(*[e.host() for e in self.codec_embeddings])
        heads = (_lib.Q4Host * c.p_groups)(*[h.host() for h in self.lm_heads])
        self._keep += [layers, embs, heads]
        ip = self.input_proj.host() if self.input_proj is not None else _lib.Q4Host(None, None, 0, 0)
        return _lib.PredictorHost(c.p_layers, c.p_hidden, c.p_heads, c.p_kv_heads, c.p_head_dim,
                                  c.p_ffn, c.p_vocab, c.p_groups, c.p_max_pos, c.rope_theta,
                                  C.addressof(layers), ip, _ptr(self.input_proj_bias),
                                  C.addressof(embs), C.addressof(heads), _ptr(self.final_norm))

    @property
    def nbytes_per_pass(self) -> int:
        n = sum(h.nbytes for h in self.lm_heads) // len(self.lm_heads)
        if self.input_proj is not None:
            n += self.input_proj.nbytes
        for lw in self.layers:
            n += sum(getattr(lw, k).nbytes for k in ("q_proj", "k_proj", "v_proj", "o_proj",
                                                     "gate_proj", "up_proj", "down_proj"))
        return n


@dataclass
class TextProjWeights:
    """TalkerWeights text path (talker.rs:33-56; loader.rs:280-284):
    text_embedding [text_vocab][text_hidden], text_projection fc1
    [text_hidden][mid] + bias, fc2 [mid][hidden] + bias."""
    text_embedding: Q4Weight
    fc1: Q4Weight
    fc1_bias: np.ndarray
    fc2: Q4Weight
    fc2_bias: np.ndarray

    def host(self) -> _lib.TextProjHost:
        return _lib.TextProjHost(self.text_embedding.host(), self.fc1.host(), self.fc2.host(),
                                 _ptr(self.fc1_bias), _ptr(self.fc2_bias))

    @property
    def hidden(self) -> int:
        return self.fc2.n

    @property
    def text_vocab(self) -> int:
        return self.text_embedding.k


def synth_text_proj(seed: int, text_vocab: int, text_hidden: int, hidden: int,
                    sigma: float = 0.02, mid: int | None = None) -> TextProjWeights:
    """Random-init text path (seeds seed .. seed+4).  The 1.7B model: text_vocab
    151936, text_hidden 2048 (config.rs:137-138), mid = text_hidden, hidden 2048."""
    mid = text_hidden if mid is None else mid
    return TextProjWeights(synth_q4(seed, sigma, text_vocab, text_hidden),
                           synth_q4(seed + 1, sigma, text_hidden, mid),
                           synth_normal(seed + 2, sigma, mid),
                           synth_q4(seed + 3, sigma, mid, hidden),
                           synth_normal(seed + 4, sigma, hidden))


def synth_talker(cfg: ModelConfig) -> TalkerWeights:
    """Random-init talker.  Seeds: layer i uses cfg.seed*1000 + 10*i (+1..7)."""
    s, sg = cfg.seed, cfg.sigma
    layers = [synth_layer(s * 1000 + 10 * i, sg, cfg.t_hidden, cfg.t_heads, cfg.t_kv_heads,
                          cfg.t_head_dim, cfg.t_ffn) for i in range(cfg.t_layers)]
    return TalkerWeights(cfg, layers,
                         codec_embedding=synth_q4(s * 1000 + 900, sg, cfg.t_vocab, cfg.t_hidden),
                         codec_head=synth_q4(s * 1000 + 901, sg, cfg.t_hidden, cfg.t_vocab),
                         final_norm=np.full(cfg.t_hidden, F16_ONE, np.uint16))


def synth_predictor(cfg: ModelConfig) -> PredictorWeights:
    """Random-init code predictor (seeds cfg.seed*1000 + 500.., 902.., 910.., 940..)."""
    s, sg = cfg.seed, cfg.sigma
    layers = [synth_layer(s * 1000 + 500 + 10 * i, sg, cfg.p_hidden, cfg.p_heads, cfg.p_kv_heads,
                          cfg.p_head_dim, cfg.p_ffn) for i in range(cfg.p_layers)]
    proj = cfg.t_hidden != cfg.p_hidden
    return PredictorWeights(
        cfg, layers,
        input_proj=synth_q4(s * 1000 + 902, sg, cfg.t_hidden, cfg.p_hidden) if proj else None,
        input_proj_bias=synth_normal(s * 1000 + 903, sg, cfg.p_hidden) if proj else None,
        codec_embeddings=[synth_q4(s * 1000 + 910 + g, sg, cfg.p_vocab, cfg.t_hidden)
                          for g in range(cfg.p_groups)],
        lm_heads=[synth_q4(s * 1000 + 940 + g, sg, cfg.p_hidden, cfg.p_vocab)
                  for g in range(cfg.p_groups)],
        final_norm=np.full(cfg.p_hidden, F16_ONE, np.uint16))


class _HostView:
    """Duck-typed stand-in for TalkerWeights / PredictorWeights built from a
    ModelFile: `cfg` and `host()` are what engine.Talker / CodePredictor use."""

    def __init__(self, owner, cfg: ModelConfig, host):
        self._owner, self.cfg, self._host = owner, cfg, host

    def host(self):
        return self._host


class ModelFile:
    """A .qora-tts checkpoint (save.rs:262-409), mapped read-only by the engine
    library.  `talker` / `predictor` / `text_proj` are views for
    engine.Talker(ctx, view), engine.CodePredictor(ctx, view) and
    engine.TextProjection(ctx, view); keep this object alive until those are
    created (the device copies are independent of it afterwards)."""

    def __init__(self, path: str):
        h = C.c_void_p()
        _lib.call("qora_model_file_open", str(path).encode(), C.byref(h))
        self.h = h
        self.talker_host = _lib.TalkerHost()
        self.predictor_host = _lib.PredictorHost()
        _lib.call("qora_model_file_talker", self.h, C.byref(self.talker_host))
        _lib.call("qora_model_file_predictor", self.h, C.byref(self.predictor_host))
        t, p = self.talker_host, self.predictor_host
        self.cfg = ModelConfig(
            t_layers=t.num_layers, t_hidden=t.hidden, t_heads=t.num_heads, t_kv_heads=t.num_kv_heads,
            t_head_dim=t.head_dim, t_ffn=t.ffn, t_vocab=t.vocab, t_max_pos=t.rope_max_pos,
            p_layers=p.num_layers, p_hidden=p.hidden, p_heads=p.num_heads, p_kv_heads=p.num_kv_heads,
            p_head_dim=p.head_dim, p_ffn=p.ffn, p_vocab=p.vocab, p_groups=p.num_groups,
            p_max_pos=p.rope_max_pos, rope_theta=t.rope_theta)
        self.talker = _HostView(self, self.cfg, self.talker_host)
        self.predictor = _HostView(self, self.cfg, self.predictor_host)
        self.text_proj_host = _lib.TextProjHost()
        _lib.call("qora_model_file_text_proj", self.h, C.byref(self.text_proj_host))
        self.text_proj = _HostView(self, self.cfg, self.text_proj_host)

    def close(self):
        if getattr(self, "h", None):
            _lib.load().qora_model_file_close(self.h)
            self.h = None

    def __del__(self):
        self.close()
