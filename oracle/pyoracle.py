"""ctypes binding of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() (as
the checker) and by bench.py's CPU-baseline / --impl reference legs.  The
product (the CUDA library and its Python host mirror) never imports it.

The oracle restates the reference's Rust CPU path (src/gemv.rs, src/simd.rs,
src/gpool.rs, src/rope.rs, src/talker.rs, src/code_predictor.rs,
src/generate_new.rs); see oracle.h for the per-function citations.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass, field

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None


def build() -> str:
    """Compile the oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


class Q4(C.Structure):
    _fields_ = [("packed", C.c_void_p), ("scales", C.c_void_p), ("k", C.c_int64), ("n", C.c_int64)]


class Layer(C.Structure):
    _fields_ = [(n, Q4) for n in ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj",
                                  "down_proj")] + \
               [(n, C.c_void_p) for n in ("q_norm", "k_norm", "input_norm", "post_attn_norm")]


class Talker(C.Structure):
    _fields_ = [("num_layers", C.c_int32), ("hidden", C.c_int32), ("num_heads", C.c_int32),
                ("num_kv_heads", C.c_int32), ("head_dim", C.c_int32), ("ffn", C.c_int32),
                ("vocab", C.c_int32), ("rope_max_pos", C.c_int32), ("layers", C.c_void_p),
                ("codec_embedding", Q4), ("codec_head", Q4), ("final_norm", C.c_void_p),
                ("rope_cos", C.c_void_p), ("rope_sin", C.c_void_p)]


class Predictor(C.Structure):
    _fields_ = [("num_layers", C.c_int32), ("hidden", C.c_int32), ("num_heads", C.c_int32),
                ("num_kv_heads", C.c_int32), ("head_dim", C.c_int32), ("ffn", C.c_int32),
                ("vocab", C.c_int32), ("num_groups", C.c_int32), ("rope_max_pos", C.c_int32),
                ("layers", C.c_void_p), ("input_proj", Q4), ("input_proj_bias", C.c_void_p),
                ("codec_embeddings", C.c_void_p), ("lm_heads", C.c_void_p),
                ("final_norm", C.c_void_p), ("rope_cos", C.c_void_p), ("rope_sin", C.c_void_p)]


class SampleParams(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_int32), ("top_p", C.c_float),
                ("repetition_penalty", C.c_float)]


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        vp, i64, i32, f32 = C.c_void_p, C.c_int64, C.c_int32, C.c_float
        sig = {
            "oq_f16_to_f32": (f32, [C.c_uint16]),
            "oq_f32_to_f16": (C.c_uint16, [f32]),
            "oq_f32_to_f16_array": (None, [vp, vp, i64]),
            "oq_f16_to_f32_array": (None, [vp, vp, i64]),
            "oq_quantize_f32_to_q4": (None, [vp, i64, i64, vp, vp]),
            "oq_gemv_q4_scalar": (None, [vp, vp, vp, i64, i64, i64, vp]),
            "oq_gemv_q4_avx2": (None, [vp, vp, vp, i64, i64, i64, vp]),
            "oq_gemv_q4_avx512": (None, [vp, vp, vp, i64, i64, i64, vp]),
            "oq_has_avx2": (C.c_int, []),
            "oq_has_avx512": (C.c_int, []),
            "oq_gemv_q4_inner": (None, [vp, vp, i64, i64, vp]),
            "oq_gemv": (None, [vp, vp, vp]),
            "oq_gemv_workers": (None, [vp, vp, vp, C.c_int]),
            "oq_gemm": (None, [vp, i64, vp, vp]),
            "oq_embed_lookup": (None, [vp, i64, vp]),
            "oq_rms_norm_f16": (None, [vp, vp, i64, vp]),
            "oq_softmax_raw": (None, [vp, i64]),
            "oq_silu": (f32, [f32]),
            "oq_pool_workers": (C.c_int, []),
            "oq_pool_set_workers": (None, [C.c_int]),
            "oq_set_simd": (None, [C.c_int]),
            "oq_get_simd": (C.c_int, []),
            "oq_build_rope_tables": (None, [i32, i32, C.c_double, vp, i32, vp, vp]),
            "oq_apply_rope_split": (None, [vp, i32, i32, i64, vp, vp, i64]),
            "oq_qk_norm": (None, [vp, i32, i32, vp]),
            "oq_kv_create": (vp, [i32, i32, i32, i32]),
            "oq_kv_destroy": (None, [vp]),
            "oq_kv_reset": (None, [vp]),
            "oq_kv_len": (i32, [vp, i32]),
            "oq_kv_k": (vp, [vp, i32]),
            "oq_kv_v": (vp, [vp, i32]),
            "oq_kv_copy": (C.c_int, [vp, vp]),
            "oq_talker_step": (C.c_int, [vp, vp, vp, i64, vp, vp]),
            "oq_attend_step": (C.c_int, [vp, vp, vp, i32, i32, i32, vp, vp, vp, vp, i64, i64, vp,
                                         i32, vp]),
            "oq_talker_prefill": (C.c_int, [vp, vp, i64, vp, i64, vp]),
            "oq_gemm_long": (None, [vp, i64, vp, vp]),
            "oq_talker_prefill_rows": (C.c_int, [vp, vp, i64, vp, i64, vp, vp]),
            "oq_codec_head": (None, [vp, vp, vp]),
            "oq_embed_codec_token": (None, [vp, C.c_uint32, vp]),
            "oq_embed_text_token": (None, [vp, C.c_uint32, vp]),
            "oq_talker_decode": (C.c_int, [vp, vp, C.c_uint32, C.c_int, vp, i64, vp]),
            "oq_predictor_frame": (C.c_int, [vp, vp, vp, vp, vp, vp]),
            "oq_predictor_frame_forced": (C.c_int, [vp, vp, vp, vp, vp, vp, vp]),
            "oq_acoustic_embeddings_sum": (None, [vp, vp, vp]),
            "oq_argmax": (C.c_uint32, [vp, i64]),
            "oq_project_input": (None, [vp, vp, vp]),
            "oq_simple_rand": (f32, [C.POINTER(C.c_uint64)]),
            "oq_sample_token": (C.c_uint32, [vp, i64, vp, vp, i32, C.POINTER(C.c_uint64), f32]),
            "oq_sample_probs": (None, [vp, i64, vp, vp, i32, f32, vp]),
            "oq_frame": (C.c_int, [vp, vp, vp, vp, vp, vp, i64, vp, vp, vp,
                                   C.POINTER(C.c_uint64), vp]),
            "oq_synth_normal": (None, [C.c_uint64, f32, i64, vp]),
            "oq_synth_q4": (None, [C.c_uint64, f32, i64, i64, vp, vp]),
            "oq_xrng": (C.c_uint64, [C.POINTER(C.c_uint64)]),
            "oq_test_rbytes": (None, [C.POINTER(C.c_uint64), i64, vp]),
            "oq_test_rscales": (None, [C.POINTER(C.c_uint64), i64, C.c_double, vp]),
            "oq_test_rinput": (None, [C.POINTER(C.c_uint64), i64, C.c_double, vp]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"], "array must be C-contiguous"
    return a.ctypes.data


# --------------------------------------------------------------------------
# Q4 weights and small wrappers
# --------------------------------------------------------------------------
@dataclass
class Q4Weight:
    """Reference Q4Weight (gemv.rs:26-31): packed u8[k*n/2], scales f16 bits."""
    packed: np.ndarray
    scales: np.ndarray
    k: int
    n: int

    def cstruct(self) -> Q4:
        return Q4(ptr(self.packed), ptr(self.scales), self.k, self.n)


def quantize(data: np.ndarray) -> Q4Weight:
    data = np.ascontiguousarray(data, dtype=np.float32)
    k, n = data.shape
    g = n // 32
    packed = np.zeros(k * g * 16, np.uint8)
    scales = np.zeros(k * g, np.uint16)
    lib().oq_quantize_f32_to_q4(ptr(data), k, n, ptr(packed), ptr(scales))
    return Q4Weight(packed, scales, k, n)


def synth_q4(seed: int, sigma: float, k: int, n: int) -> Q4Weight:
    g = n // 32
    packed = np.zeros(k * g * 16, np.uint8)
    scales = np.zeros(k * g, np.uint16)
    lib().oq_synth_q4(seed, sigma, k, n, ptr(packed), ptr(scales))
    return Q4Weight(packed, scales, k, n)


def synth_normal(seed: int, sigma: float, count: int) -> np.ndarray:
    out = np.zeros(count, np.float32)
    lib().oq_synth_normal(seed, sigma, count, ptr(out))
    return out


def gemv(x: np.ndarray, w: Q4Weight, workers: int = 0) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(w.n, np.float32)
    ws = w.cstruct()
    lib().oq_gemv_workers(ptr(x), C.addressof(ws), ptr(out), workers)
    return out


def gemm_long(x: np.ndarray, w: Q4Weight) -> np.ndarray:
    """oq_gemm_long: the bits of gemm (per-row single pass), blocked over rows."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1, w.k)
    out = np.zeros((x.shape[0], w.n), np.float32)
    ws = w.cstruct()
    lib().oq_gemm_long(ptr(x), x.shape[0], C.addressof(ws), ptr(out))
    return out


def gemv_single(x: np.ndarray, w: Q4Weight) -> np.ndarray:
    """Single-pass gemv_q4_inner over all k (the scalar oracle order)."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(w.n, np.float32)
    ws = w.cstruct()
    lib().oq_gemv_q4_inner(ptr(x), C.addressof(ws), 0, w.k, ptr(out))
    return out


def gemv_scalar(x, packed, scales, n, k0, k1):
    out = np.zeros(n, np.float32)
    lib().oq_gemv_q4_scalar(ptr(x), ptr(packed), ptr(scales), n, k0, k1, ptr(out))
    return out


def gemv_avx2(x, packed, scales, n, k0, k1):
    out = np.zeros(n, np.float32)
    lib().oq_gemv_q4_avx2(ptr(x), ptr(packed), ptr(scales), n, k0, k1, ptr(out))
    return out


def gemv_avx512(x, packed, scales, n, k0, k1):
    out = np.zeros(n, np.float32)
    lib().oq_gemv_q4_avx512(ptr(x), ptr(packed), ptr(scales), n, k0, k1, ptr(out))
    return out


def embed_lookup(w: Q4Weight, token: int) -> np.ndarray:
    out = np.zeros(w.n, np.float32)
    ws = w.cstruct()
    lib().oq_embed_lookup(C.addressof(ws), token, ptr(out))
    return out


class TextProjC(C.Structure):
    _fields_ = [("text_embedding", Q4), ("fc1", Q4), ("fc2", Q4), ("fc1_bias", C.c_void_p),
                ("fc2_bias", C.c_void_p)]


@dataclass
class TextProj:
    """TalkerWeights text path (talker.rs:33-56): text_embedding, fc1 + bias,
    fc2 + bias."""
    text_embedding: Q4Weight
    fc1: Q4Weight
    fc1_bias: np.ndarray
    fc2: Q4Weight
    fc2_bias: np.ndarray

    @staticmethod
    def synth(seed: int, text_vocab: int, text_hidden: int, hidden: int, sigma: float = 0.02,
              mid: int | None = None) -> "TextProj":
        mid = text_hidden if mid is None else mid
        return TextProj(synth_q4(seed, sigma, text_vocab, text_hidden),
                        synth_q4(seed + 1, sigma, text_hidden, mid),
                        synth_normal(seed + 2, sigma, mid),
                        synth_q4(seed + 3, sigma, mid, hidden),
                        synth_normal(seed + 4, sigma, hidden))

    def cstruct(self) -> TextProjC:
        return TextProjC(self.text_embedding.cstruct(), self.fc1.cstruct(), self.fc2.cstruct(),
                         ptr(self.fc1_bias), ptr(self.fc2_bias))

    def embed_text_token(self, token: int) -> np.ndarray:
        """embed_text_token (talker.rs:104-116)."""
        out = np.zeros(self.fc2.n, np.float32)
        s = self.cstruct()
        lib().oq_embed_text_token(C.addressof(s), token, ptr(out))
        return out


def rms_norm_f16(x: np.ndarray, gamma_f16: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros_like(x)
    lib().oq_rms_norm_f16(ptr(x), ptr(gamma_f16), x.size, ptr(out))
    return out


def rope_tables(head_dim: int, max_pos: int, theta: float = 1e6, sections=None):
    half = head_dim // 2
    sections = np.asarray(sections if sections is not None else [half], np.int32)
    cos = np.zeros(max_pos * half, np.float32)
    sin = np.zeros(max_pos * half, np.float32)
    lib().oq_build_rope_tables(head_dim, max_pos, theta, ptr(sections), sections.size,
                               ptr(cos), ptr(sin))
    return cos, sin


def f32_to_f16(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32)
    out = np.zeros(a.shape, np.uint16)
    lib().oq_f32_to_f16_array(ptr(a), ptr(out), a.size)
    return out


# --------------------------------------------------------------------------
# Test-generator restatements (gemv.rs:693-730)
# --------------------------------------------------------------------------
class XRng:
    def __init__(self, seed: int):
        self.state = C.c_uint64(seed)

    def bytes(self, n):
        out = np.zeros(n, np.uint8)
        lib().oq_test_rbytes(C.byref(self.state), n, ptr(out))
        return out

    def scales(self, n, zero_frac):
        out = np.zeros(n, np.uint16)
        lib().oq_test_rscales(C.byref(self.state), n, zero_frac, ptr(out))
        return out

    def inputs(self, n, zero_frac):
        out = np.zeros(n, np.float32)
        lib().oq_test_rinput(C.byref(self.state), n, zero_frac, ptr(out))
        return out


# --------------------------------------------------------------------------
# Models (random-init N(0, sigma) weights, reference layout)
# --------------------------------------------------------------------------
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

    def cstruct(self) -> Layer:
        return Layer(*(getattr(self, n).cstruct() for n in
                       ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj",
                        "down_proj")),
                     ptr(self.q_norm), ptr(self.k_norm), ptr(self.input_norm),
                     ptr(self.post_attn_norm))


@dataclass
class ModelConfig:
    """Talker + predictor dims.  Defaults are the 1.7B model (config.rs:130-153)."""
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


def _layer_synth(seed: int, sigma: float, hidden: int, heads: int, kv_heads: int, hd: int,
                 ffn: int) -> LayerWeights:
    qd, kd = heads * hd, kv_heads * hd
    one = f32_to_f16(np.ones(1, np.float32))[0]
    return LayerWeights(
        q_proj=synth_q4(seed + 1, sigma, hidden, qd),
        k_proj=synth_q4(seed + 2, sigma, hidden, kd),
        v_proj=synth_q4(seed + 3, sigma, hidden, kd),
        o_proj=synth_q4(seed + 4, sigma, qd, hidden),
        gate_proj=synth_q4(seed + 5, sigma, hidden, ffn),
        up_proj=synth_q4(seed + 6, sigma, hidden, ffn),
        down_proj=synth_q4(seed + 7, sigma, ffn, hidden),
        q_norm=np.full(hd, one, np.uint16),
        k_norm=np.full(hd, one, np.uint16),
        input_norm=np.full(hidden, one, np.uint16),
        post_attn_norm=np.full(hidden, one, np.uint16),
    )


@dataclass
class Model:
    cfg: ModelConfig
    t_layers: list
    codec_embedding: Q4Weight
    codec_head: Q4Weight
    t_final_norm: np.ndarray
    t_rope: tuple
    p_layers: list
    input_proj: Q4Weight | None
    input_proj_bias: np.ndarray | None
    codec_embeddings: list
    lm_heads: list
    p_final_norm: np.ndarray
    p_rope: tuple
    _keep: list = field(default_factory=list)

    @staticmethod
    def synth(cfg: ModelConfig) -> "Model":
        """Random-init weights.  Tensor seeds are cfg.seed + fixed offsets so the
        same config always yields the same bytes (GPU and oracle share them)."""
        s, sg = cfg.seed, cfg.sigma
        one = f32_to_f16(np.ones(1, np.float32))[0]
        t_layers = [_layer_synth(s * 1000 + 10 * i, sg, cfg.t_hidden, cfg.t_heads,
                                 cfg.t_kv_heads, cfg.t_head_dim, cfg.t_ffn)
                    for i in range(cfg.t_layers)]
        p_layers = [_layer_synth(s * 1000 + 500 + 10 * i, sg, cfg.p_hidden, cfg.p_heads,
                                 cfg.p_kv_heads, cfg.p_head_dim, cfg.p_ffn)
                    for i in range(cfg.p_layers)]
        half_t = cfg.t_head_dim // 2
        sec = [24, 20, 20] if half_t == 64 else [half_t]
        m = Model(
            cfg=cfg,
            t_layers=t_layers,
            codec_embedding=synth_q4(s * 1000 + 900, sg, cfg.t_vocab, cfg.t_hidden),
            codec_head=synth_q4(s * 1000 + 901, sg, cfg.t_hidden, cfg.t_vocab),
            t_final_norm=np.full(cfg.t_hidden, one, np.uint16),
            t_rope=rope_tables(cfg.t_head_dim, cfg.t_max_pos, cfg.rope_theta, sec),
            p_layers=p_layers,
            input_proj=(synth_q4(s * 1000 + 902, sg, cfg.t_hidden, cfg.p_hidden)
                        if cfg.t_hidden != cfg.p_hidden else None),
            input_proj_bias=(synth_normal(s * 1000 + 903, sg, cfg.p_hidden)
                             if cfg.t_hidden != cfg.p_hidden else None),
            codec_embeddings=[synth_q4(s * 1000 + 910 + g, sg, cfg.p_vocab, cfg.t_hidden)
                              for g in range(cfg.p_groups)],
            lm_heads=[synth_q4(s * 1000 + 940 + g, sg, cfg.p_hidden, cfg.p_vocab)
                      for g in range(cfg.p_groups)],
            p_final_norm=np.full(cfg.p_hidden, one, np.uint16),
            p_rope=rope_tables(cfg.p_head_dim, cfg.p_max_pos, cfg.rope_theta),
        )
        return m

    # ---- oracle structs -------------------------------------------------
    def talker_struct(self) -> Talker:
        c = self.cfg
        layers = (Layer * c.t_layers)(*[lw.cstruct() for lw in self.t_layers])
        self._keep.append(layers)
        t = Talker(c.t_layers, c.t_hidden, c.t_heads, c.t_kv_heads, c.t_head_dim, c.t_ffn,
                   c.t_vocab, c.t_max_pos, C.addressof(layers), self.codec_embedding.cstruct(),
                   self.codec_head.cstruct(), ptr(self.t_final_norm), ptr(self.t_rope[0]),
                   ptr(self.t_rope[1]))
        self._keep.append(t)
        return t

    def predictor_struct(self) -> Predictor:
        c = self.cfg
        layers = (Layer * c.p_layers)(*[lw.cstruct() for lw in self.p_layers])
        embs = (Q4 * c.p_groups)(*[e.cstruct() for e in self.codec_embeddings])
        heads = (Q4 * c.p_groups)(*[h.cstruct() for h in self.lm_heads])
        self._keep += [layers, embs, heads]
        ip = self.input_proj.cstruct() if self.input_proj is not None else Q4(None, None, 0, 0)
        p = Predictor(c.p_layers, c.p_hidden, c.p_heads, c.p_kv_heads, c.p_head_dim, c.p_ffn,
                      c.p_vocab, c.p_groups, c.p_max_pos, C.addressof(layers), ip,
                      ptr(self.input_proj_bias) if self.input_proj_bias is not None else None,
                      C.addressof(embs), C.addressof(heads), ptr(self.p_final_norm),
                      ptr(self.p_rope[0]), ptr(self.p_rope[1]))
        self._keep.append(p)
        return p


class KV:
    def __init__(self, layers: int, kv_heads: int, head_dim: int, max_pos: int):
        self.h = lib().oq_kv_create(layers, kv_heads, head_dim, max_pos)
        self.shape = (layers, kv_heads, head_dim, max_pos)

    def __del__(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.oq_kv_destroy(self.h)
            self.h = None

    def len(self, layer: int = 0) -> int:
        return lib().oq_kv_len(self.h, layer)

    def k(self, layer: int) -> np.ndarray:
        L, kvh, hd, mp = self.shape
        p = lib().oq_kv_k(self.h, layer)
        return np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_float)), (mp, kvh, hd))

    def v(self, layer: int) -> np.ndarray:
        L, kvh, hd, mp = self.shape
        p = lib().oq_kv_v(self.h, layer)
        return np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_float)), (mp, kvh, hd))

    def reset(self):
        lib().oq_kv_reset(self.h)

    def copy_from(self, other: "KV"):
        assert lib().oq_kv_copy(self.h, other.h) == 0


class OracleModel:
    """Oracle runner bound to one Model."""

    def __init__(self, model: Model):
        self.m = model
        self.t = model.talker_struct()
        self.p = model.predictor_struct()

    def talker_kv(self, max_pos=None) -> KV:
        c = self.m.cfg
        return KV(c.t_layers, c.t_kv_heads, c.t_head_dim, max_pos or c.t_max_pos)

    def predictor_kv(self) -> KV:
        c = self.m.cfg
        return KV(c.p_layers, c.p_kv_heads, c.p_head_dim, c.p_groups + 1)

    def talker_step(self, emb, kv: KV, position: int):
        c = self.m.cfg
        emb = np.ascontiguousarray(emb, np.float32)
        h = np.zeros(c.t_hidden, np.float32)
        lg = np.zeros(c.t_vocab, np.float32)
        rc = lib().oq_talker_step(C.addressof(self.t), ptr(emb), kv.h, position, ptr(h), ptr(lg))
        assert rc == 0, rc
        return h, lg

    def talker_decode(self, token: int, is_text: bool, kv: KV, position: int,
                      text_proj: "TextProj | None" = None):
        """forward_talker_decode (talker.rs:161-258): the final-normed hidden."""
        out = np.zeros(self.m.cfg.t_hidden, np.float32)
        tps = text_proj.cstruct() if text_proj is not None else None
        rc = lib().oq_talker_decode(C.addressof(self.t), C.addressof(tps) if tps is not None else None,
                                    token, 1 if is_text else 0, kv.h, position, ptr(out))
        assert rc == 0, rc
        return out

    def talker_prefill(self, x, kv: KV, start_pos: int = 0):
        c = self.m.cfg
        x = np.ascontiguousarray(x, np.float32)
        T = x.size // c.t_hidden
        h = np.zeros(c.t_hidden, np.float32)
        rc = lib().oq_talker_prefill(C.addressof(self.t), ptr(x), T, kv.h, start_pos, ptr(h))
        assert rc == 0, rc
        return h

    def talker_prefill_rows(self, x, kv: KV, start_pos: int = 0, logits: bool = False):
        """The prefill of `x` [T][hidden] on top of kv (oracle_long.c: the
        values of talker_prefill, blocked and on every host core), returning
        every row's final-normed hidden [T][hidden] and, with logits=True,
        every row's codec-head logits [T][vocab]."""
        c = self.m.cfg
        x = np.ascontiguousarray(x, np.float32).reshape(-1, c.t_hidden)
        T = x.shape[0]
        h = np.zeros((T, c.t_hidden), np.float32)
        lg = np.zeros((T, c.t_vocab), np.float32) if logits else None
        rc = lib().oq_talker_prefill_rows(C.addressof(self.t), ptr(x), T, kv.h, start_pos, ptr(h),
                                          ptr(lg) if logits else None)
        assert rc == 0, rc
        return (h, lg) if logits else h

    def codec_head(self, hidden):
        out = np.zeros(self.m.cfg.t_vocab, np.float32)
        hidden = np.ascontiguousarray(hidden, np.float32)
        lib().oq_codec_head(C.addressof(self.t), ptr(hidden), ptr(out))
        return out

    def embed_codec(self, token: int):
        out = np.zeros(self.m.cfg.t_hidden, np.float32)
        lib().oq_embed_codec_token(C.addressof(self.t), token, ptr(out))
        return out

    def predictor_frame(self, hidden, sem, kv: KV, forced=None):
        c = self.m.cfg
        hidden = np.ascontiguousarray(hidden, np.float32)
        sem = np.ascontiguousarray(sem, np.float32)
        codes = np.zeros(c.p_groups, np.uint32)
        logits = np.zeros((c.p_groups, c.p_vocab), np.float32)
        if forced is None:
            rc = lib().oq_predictor_frame(C.addressof(self.p), ptr(hidden), ptr(sem), kv.h,
                                          ptr(codes), ptr(logits))
        else:
            forced = np.ascontiguousarray(forced, np.uint32)
            rc = lib().oq_predictor_frame_forced(C.addressof(self.p), ptr(hidden), ptr(sem), kv.h,
                                                 ptr(forced), ptr(codes), ptr(logits))
        assert rc == 0, rc
        return codes, logits

    def acoustic_sum(self, codes):
        codes = np.ascontiguousarray(codes, np.uint32)
        out = np.zeros(self.m.cfg.t_hidden, np.float32)
        lib().oq_acoustic_embeddings_sum(C.addressof(self.p), ptr(codes), ptr(out))
        return out

    def frame(self, tkv: KV, pkv: KV, params: SampleParams, text_row, position, state):
        """state: dict(logits, hidden, prev (u32[16]), rng (int))."""
        c = self.m.cfg
        codes = np.zeros(16, np.uint32)
        rng = C.c_uint64(state["rng"])
        text_row = np.ascontiguousarray(text_row, np.float32)
        rc = lib().oq_frame(C.addressof(self.t), C.addressof(self.p), tkv.h, pkv.h,
                            C.byref(params), ptr(text_row), position, ptr(state["logits"]),
                            ptr(state["hidden"]), ptr(state["prev"]), C.byref(rng), ptr(codes))
        assert rc == 0, rc
        state["rng"] = rng.value
        return codes


def sample_token(logits, params: SampleParams, prev, rng_state: int, temperature=None):
    logits = np.ascontiguousarray(logits, np.float32)
    prev = np.ascontiguousarray(prev, np.uint32)
    st = C.c_uint64(rng_state)
    t = params.temperature if temperature is None else temperature
    tok = lib().oq_sample_token(ptr(logits), logits.size, C.byref(params), ptr(prev), prev.size,
                                C.byref(st), t)
    return tok, st.value


def sample_probs(logits, params: SampleParams, prev, temperature=None):
    logits = np.ascontiguousarray(logits, np.float32)
    prev = np.ascontiguousarray(prev, np.uint32)
    out = np.zeros_like(logits)
    t = params.temperature if temperature is None else temperature
    lib().oq_sample_probs(ptr(logits), logits.size, C.byref(params), ptr(prev), prev.size, t,
                          ptr(out))
    return out


def attend_step(kv: "KV", layer: int, q, k, v, heads: int, kv_heads: int, hd: int, q_norm, k_norm,
                rope_cos, rope_sin, position: int):
    """Attention block of one decode step of one layer (talker.rs:285-331)."""
    q, k, v = (np.ascontiguousarray(a, np.float32) for a in (q, k, v))
    out = np.zeros(heads * hd, np.float32)
    rc = lib().oq_attend_step(ptr(q), ptr(k), ptr(v), heads, kv_heads, hd, ptr(q_norm), ptr(k_norm),
                              ptr(rope_cos), ptr(rope_sin), rope_cos.size, position, kv.h, layer,
                              ptr(out))
    assert rc == 0, rc
    return out


def simple_rand(state: int):
    st = C.c_uint64(state)
    r = lib().oq_simple_rand(C.byref(st))
    return r, st.value
