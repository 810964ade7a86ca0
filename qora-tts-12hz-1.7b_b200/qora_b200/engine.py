"""Device-side Python mirror of the reference operator surface.

Each method names the reference function it stands in for.  Device tensors
are torch CUDA tensors (torch supplies device memory and streams only); all
compute goes through libqora_b200.so.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib
from .weights import ModelConfig, PredictorWeights, Q4Weight, TalkerWeights

_VP = C.c_void_p


def _stream(stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _dp(t: torch.Tensor | None):
    if t is None:
        return None
    assert t.is_cuda and t.is_contiguous(), "expected a contiguous CUDA tensor"
    return t.data_ptr()


class Context:
    """Per-device context (qora_ctx)."""

    def __init__(self, device: int = 0):
        self.device = device
        self._L = _lib.load()
        h = C.c_void_p()
        _lib.call("qora_ctx_create", device, C.byref(h))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            self._L.qora_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def check_device_error(self, stream=None) -> None:
        """Raises if a kernel flagged a device-side error (then clears it)."""
        _lib.call("qora_ctx_check_device_error", self.h, _stream(stream))


class DeviceQ4:
    """A Q4Weight on the device (gemv.rs:26-31), repacked on upload."""

    def __init__(self, ctx: Context, w: Q4Weight):
        self.ctx, self.k, self.n = ctx, w.k, w.n
        hs = w.host()
        self._L = _lib.load()
        h = C.c_void_p()
        _lib.call("qora_q4_weight_upload", ctx.h, C.byref(hs), C.byref(h))
        self.h = h

    def __del__(self):
        if getattr(self, "h", None):
            self._L.qora_q4_weight_destroy(self.h)
            self.h = None

    def gemv(self, x: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """gemv (gemv.rs:149): rows of x [B][k] -> [B][n]."""
        x = x.reshape(-1, self.k)
        out = out if out is not None else torch.empty(x.shape[0], self.n, device=x.device)
        _lib.call("qora_q4_gemv", self.ctx.h, self.h, _dp(x), _dp(out), x.shape[0], _stream(stream))
        return out

    def gemm(self, x: torch.Tensor, stream=None) -> torch.Tensor:
        """gemm (gemv.rs:157): seq_len token rows."""
        x = x.reshape(-1, self.k)
        out = torch.empty(x.shape[0], self.n, device=x.device)
        _lib.call("qora_q4_gemm", self.ctx.h, self.h, _dp(x), x.shape[0], _dp(out), _stream(stream))
        return out

    def embed_lookup(self, tokens: torch.Tensor, stream=None) -> torch.Tensor:
        """embed_lookup (gemv.rs:165): dequantised rows for token ids (uint32/int32)."""
        tokens = tokens.to(torch.int32).contiguous()
        out = torch.empty(tokens.numel(), self.n, device=tokens.device)
        _lib.call("qora_q4_embed_rows", self.ctx.h, self.h, _dp(tokens), tokens.numel(), _dp(out),
                  _stream(stream))
        return out


def rms_norm_f16(ctx: Context, x: torch.Tensor, gamma_f16: torch.Tensor, stream=None):
    """rms_norm_f16 (gemv.rs:445-454) over the rows of x."""
    n = x.shape[-1]
    rows = x.numel() // n
    out = torch.empty_like(x)
    _lib.call("qora_rms_norm_f16", ctx.h, _dp(x.contiguous()), _dp(gamma_f16), n, rows, _dp(out),
              _stream(stream))
    return out


def build_mrope_tables(head_dim: int, max_pos: int, theta: float, sections=None):
    """build_mrope_tables (rope.rs:11-41) on the host."""
    half = head_dim // 2
    cos = np.empty(max_pos * half, np.float32)
    sin = np.empty(max_pos * half, np.float32)
    sec = np.asarray(sections if sections is not None else [half], np.int32)
    _lib.call("qora_rope_tables_host", head_dim, max_pos, theta, sec.ctypes.data, sec.size,
              cos.ctypes.data, sin.ctypes.data)
    return cos, sin


class KvCache:
    """RawKvCache for `streams` streams (gemv.rs:75-86), preallocated on device."""

    def __init__(self, ctx: Context, layers: int, kv_heads: int, head_dim: int, max_pos: int,
                 streams: int = 1, page_positions: int = 0, pool_pages: int = 0):
        """page_positions > 0: paged storage (qora_kv_create_paged), a pool of
        pool_pages pages of page_positions positions mapped as streams grow."""
        self.ctx, self.layers, self.kv_heads, self.head_dim = ctx, layers, kv_heads, head_dim
        self.max_pos, self.streams = max_pos, streams
        self.paged = page_positions > 0
        self._L = _lib.load()
        h = C.c_void_p()
        if self.paged:
            _lib.call("qora_kv_create_paged", ctx.h, layers, kv_heads, head_dim, max_pos, streams,
                      page_positions, pool_pages, C.byref(h))
        else:
            _lib.call("qora_kv_create", ctx.h, layers, kv_heads, head_dim, max_pos, streams, C.byref(h))
        self.h = h

    def pages(self):
        """(mapped, free) pages of a paged cache."""
        m, f = C.c_int32(), C.c_int32()
        _lib.call("qora_kv_pages_host", self.h, C.byref(m), C.byref(f))
        return m.value, f.value

    def __del__(self):
        if getattr(self, "h", None):
            self._L.qora_kv_destroy(self.h)
            self.h = None

    def reset(self, ids=None, stream=None):
        if ids is None:
            _lib.call("qora_kv_reset", self.h, None, 0, _stream(stream))
        else:
            a = np.asarray(ids, np.int32)
            _lib.call("qora_kv_reset", self.h, a.ctypes.data, a.size, _stream(stream))

    def lengths(self, stream=None) -> np.ndarray:
        out = np.empty(self.streams, np.int32)
        _lib.call("qora_kv_lengths_host", self.h, out.ctypes.data, _stream(stream))
        return out

    def copy_stream_from(self, dst_stream: int, src: "KvCache", src_stream: int, stream=None):
        _lib.call("qora_kv_copy_stream", self.h, dst_stream, src.h, src_stream, _stream(stream))

    def layer_tensors(self, layer: int, stream=None):
        """Copies of one layer's (K, V) slabs, [streams][kv_heads][max_pos][head_dim]."""
        shape = (self.streams, self.kv_heads, self.max_pos, self.head_dim)
        k = torch.empty(shape, dtype=torch.float32, device="cuda")
        v = torch.empty(shape, dtype=torch.float32, device="cuda")
        _lib.call("qora_kv_export_layer", self.h, layer, _dp(k), _dp(v), _stream(stream))
        return k, v

    def attend(self, layer: int, qkv: torch.Tensor, num_heads: int, q_norm: torch.Tensor,
               k_norm: torch.Tensor, rope_cos: torch.Tensor, rope_sin: torch.Tensor,
               positions: torch.Tensor, advance: bool = False, out: torch.Tensor | None = None,
               stream=None, noalloc: bool = False) -> torch.Tensor:
        """KV append + attend of one layer (talker.rs:285-331): qkv [B][q|k|v] raw
        projections; q_norm / k_norm f16 bits as int16 tensors; rope tables
        [max_pos * head_dim/2] f32; positions int32 [B].  Returns [B][num_heads*head_dim].
        noalloc: use qora_kv_attend_noalloc, which allocates no device memory
        (its scratch is a fixed static array; B * num_heads * head_dim <= 16384)."""
        B = qkv.shape[0]
        out = out if out is not None else torch.empty(B, num_heads * self.head_dim,
                                                      device=qkv.device)
        rope_max_pos = rope_cos.numel() // (self.head_dim // 2)
        entry = "qora_kv_attend_noalloc" if noalloc else "qora_kv_attend"
        _lib.call(entry, self.h, layer, _dp(qkv), num_heads, _dp(q_norm), _dp(k_norm),
                  _dp(rope_cos), _dp(rope_sin), rope_max_pos, _dp(positions), B,
                  1 if advance else 0, _dp(out), _stream(stream))
        return out


class Talker:
    """TalkerWeights on the device (talker.rs)."""

    def __init__(self, ctx: Context, w: TalkerWeights, max_batch: int = 1):
        self.ctx, self.cfg = ctx, w.cfg
        hs = w.host()
        self._L = _lib.load()
        h = C.c_void_p()
        _lib.call("qora_talker_create", ctx.h, C.byref(hs), max_batch, C.byref(h))
        self.h = h
        self.max_batch = max_batch

    def __del__(self):
        if getattr(self, "h", None):
            self._L.qora_talker_destroy(self.h)
            self.h = None

    def new_kv(self, max_pos: int | None = None, streams: int = 1, page_positions: int = 0,
               pool_pages: int = 0) -> KvCache:
        c = self.cfg
        return KvCache(self.ctx, c.t_layers, c.t_kv_heads, c.t_head_dim, max_pos or c.t_max_pos,
                       streams, page_positions, pool_pages)

    def forward_with_embedding(self, emb: torch.Tensor, kv: KvCache, positions, stream=None):
        """forward_with_embedding (talker.rs:263-360) for B = emb.shape[0] streams.
        Returns (hidden [B][H], logits [B][V])."""
        c = self.cfg
        emb = emb.reshape(-1, c.t_hidden).contiguous()
        B = emb.shape[0]
        pos = torch.as_tensor(positions, dtype=torch.int32).reshape(-1).to(emb.device)
        hidden = torch.empty(B, c.t_hidden, device=emb.device)
        logits = torch.empty(B, c.t_vocab, device=emb.device)
        _lib.call("qora_talker_step", self.h, kv.h, _dp(emb), _dp(pos), B, _dp(hidden),
                  _dp(logits), _stream(stream))
        return hidden, logits

    def prefill_talker_raw_from(self, x: torch.Tensor, kv: KvCache, start_pos: int = 0,
                                kv_stream: int = 0, stream=None) -> torch.Tensor:
        """prefill_talker_raw_from (talker.rs:379-482): returns the last normed hidden."""
        c = self.cfg
        x = x.reshape(-1, c.t_hidden).contiguous()
        hidden = torch.empty(c.t_hidden, device=x.device)
        _lib.call("qora_talker_prefill", self.h, kv.h, kv_stream, _dp(x), x.shape[0], start_pos,
                  _dp(hidden), _stream(stream))
        return hidden

    def forward_talker_decode(self, tokens, is_text: bool, kv: KvCache, positions,
                              text_proj: "TextProjection | None" = None,
                              stream=None) -> torch.Tensor:
        """forward_talker_decode (talker.rs:161-258) for B = len(tokens) streams:
        embeds each token (text path through `text_proj`, or the codec
        embedding), runs the step and returns the final-normed hidden [B][H]."""
        c = self.cfg
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32).reshape(-1))
        dev = f"cuda:{self.ctx.device}"
        pos = torch.as_tensor(positions, dtype=torch.int32).reshape(-1).to(dev)
        hidden = torch.empty(t.size, c.t_hidden, device=dev)
        _lib.call("qora_talker_decode", self.h, kv.h, text_proj.h if text_proj is not None else None,
                  t.ctypes.data, 1 if is_text else 0, _dp(pos), t.size, _dp(hidden), _stream(stream))
        return hidden

    def apply_codec_head(self, hidden: torch.Tensor, stream=None) -> torch.Tensor:
        """apply_codec_head (talker.rs:647-649)."""
        c = self.cfg
        hidden = hidden.reshape(-1, c.t_hidden).contiguous()
        out = torch.empty(hidden.shape[0], c.t_vocab, device=hidden.device)
        _lib.call("qora_talker_codec_head", self.h, _dp(hidden), hidden.shape[0], _dp(out),
                  _stream(stream))
        return out

    def embed_codec_token(self, tokens, stream=None) -> torch.Tensor:
        """embed_codec_token (talker.rs:152-154)."""
        t = torch.as_tensor(tokens, dtype=torch.int32).reshape(-1).cuda()
        out = torch.empty(t.numel(), self.cfg.t_hidden, device="cuda")
        _lib.call("qora_talker_embed_codec", self.h, _dp(t), t.numel(), _dp(out), _stream(stream))
        return out


class TextProjection:
    """The talker's text embedding + text projection on the device
    (TalkerWeights text path, talker.rs:33-56)."""

    def __init__(self, ctx: Context, w):
        self.ctx = ctx
        hs = w.host()
        self.hidden, self.text_vocab = int(hs.fc2.n), int(hs.text_embedding.k)
        self._L = _lib.load()
        h = C.c_void_p()
        _lib.call("qora_text_proj_create", ctx.h, C.byref(hs), C.byref(h))
        self.h = h

    def __del__(self):
        if getattr(self, "h", None):
            self._L.qora_text_proj_destroy(self.h)
            self.h = None

    def embed_text_tokens(self, tokens, out: torch.Tensor | None = None,
                          stream=None) -> torch.Tensor:
        """embed_text_token (talker.rs:104-116) for every token id in `tokens`
        (host ids); returns [len(tokens)][hidden] on the device."""
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32).reshape(-1))
        if out is None:
            out = torch.empty(t.size, self.hidden, device=f"cuda:{self.ctx.device}")
        assert out.numel() == t.size * self.hidden
        _lib.call("qora_text_proj_embed", self.h, t.ctypes.data, t.size, _dp(out), _stream(stream))
        return out

    def embed_text_token(self, token: int, stream=None) -> torch.Tensor:
        """embed_text_token (talker.rs:104-116) for one token: [hidden]."""
        return self.embed_text_tokens([token], stream=stream)[0]


class CodePredictor:
    """CodePredictorWeights on the device (code_predictor.rs)."""

    def __init__(self, ctx: Context, w: PredictorWeights, max_batch: int = 1):
        self.ctx, self.cfg = ctx, w.cfg
        hs = w.host()
        self._L = _lib.load()
        h = C.c_void_p()
        _lib.call("qora_predictor_create", ctx.h, C.byref(hs), max_batch, C.byref(h))
        self.h = h

    def __del__(self):
        if getattr(self, "h", None):
            self._L.qora_predictor_destroy(self.h)
            self.h = None

    def new_kv(self, streams: int = 1) -> KvCache:
        c = self.cfg
        return KvCache(self.ctx, c.p_layers, c.p_kv_heads, c.p_head_dim, c.p_groups + 1, streams)

    def generate_acoustic_codes(self, talker_hidden: torch.Tensor, semantic_embed: torch.Tensor,
                                kv: KvCache, forced=None, want_logits: bool = False, stream=None):
        """generate_acoustic_codes (code_predictor.rs:218-273) for B streams.
        Returns codes [B][groups] (int32) and, if asked, logits [B][groups][vocab]."""
        c = self.cfg
        hid = talker_hidden.reshape(-1, c.t_hidden).contiguous()
        sem = semantic_embed.reshape(-1, c.t_hidden).contiguous()
        B = hid.shape[0]
        codes = torch.empty(B, c.p_groups, dtype=torch.int32, device=hid.device)
        logits = torch.empty(B, c.p_groups, c.p_vocab, device=hid.device) if want_logits else None
        f = None
        if forced is not None:
            f = torch.as_tensor(forced, dtype=torch.int32).reshape(B, c.p_groups).cuda().contiguous()
        _lib.call("qora_predictor_frame", self.h, kv.h, _dp(hid), _dp(sem), B, _dp(codes),
                  _dp(logits), _dp(f), _stream(stream))
        return (codes, logits) if want_logits else codes

    def get_acoustic_embeddings_sum(self, codes: torch.Tensor, stream=None) -> torch.Tensor:
        """get_acoustic_embeddings_sum (code_predictor.rs:287-300)."""
        c = self.cfg
        codes = codes.to(torch.int32).reshape(-1, c.p_groups).contiguous()
        out = torch.empty(codes.shape[0], c.t_hidden, device=codes.device)
        _lib.call("qora_predictor_embed_sum", self.h, _dp(codes), codes.shape[0], _dp(out),
                  _stream(stream))
        return out


def default_params() -> _lib.SampleParams:
    """TTSParams::default sampling fields (generate_new.rs:63-79)."""
    return _lib.SampleParams(0.9, 50, 1.0, 1.05)


def sample_token(ctx: Context, logits: torch.Tensor, prev: torch.Tensor | None,
                 rng: torch.Tensor, params: _lib.SampleParams, stream=None) -> torch.Tensor:
    """sample_token (generate_new.rs:771-862) for each row of logits.
    rng: int64 tensor [B] of xorshift64 states, updated in place."""
    logits = logits.reshape(logits.shape[0], -1).contiguous()
    B, V = logits.shape
    out = torch.empty(B, dtype=torch.int32, device=logits.device)
    n_prev = 0 if prev is None else prev.shape[-1]
    if prev is not None:
        prev = prev.to(torch.int32).reshape(B, n_prev).contiguous()
    _lib.call("qora_sample", ctx.h, _dp(logits), B, V, _dp(prev), n_prev, _dp(rng),
              C.byref(params), _dp(out), _stream(stream))
    return out


class Engine:
    """The frame loop (generate_new.rs:606-665) for B streams on one GPU."""

    def __init__(self, talker: Talker, predictor: CodePredictor, batch: int, max_pos: int,
                 params: _lib.SampleParams | None = None):
        self.talker, self.predictor, self.B = talker, predictor, batch
        self.params = params or default_params()
        self._L = _lib.load()
        h = C.c_void_p()
        _lib.call("qora_engine_create", talker.h, predictor.h, batch, max_pos,
                  C.byref(self.params), C.byref(h))
        self.h = h

    def __del__(self):
        if getattr(self, "h", None):
            self._L.qora_engine_destroy(self.h)
            self.h = None

    def prefill(self, x: np.ndarray, seeds, stream=None):
        x = np.ascontiguousarray(x, np.float32)
        T = x.shape[1]
        s = np.ascontiguousarray(np.asarray(seeds, np.uint64).reshape(self.B))
        _lib.call("qora_engine_prefill", self.h, x.ctypes.data, T, s.ctypes.data, _stream(stream))

    def prefill_from(self, prefix: KvCache, prefix_len: int, x: np.ndarray, seeds,
                     prefix_stream: int = 0, stream=None):
        """The prefix-cache path (generate_new.rs:509-530): every stream starts
        from a copy of `prefix` (holding prefix_len positions) and prefills the
        suffix x [B][T][hidden] on top."""
        x = np.ascontiguousarray(x, np.float32)
        T = x.shape[1]
        s = np.ascontiguousarray(np.asarray(seeds, np.uint64).reshape(self.B))
        _lib.call("qora_engine_prefill_from", self.h, prefix.h, prefix_stream, prefix_len,
                  x.ctypes.data, T, s.ctypes.data, _stream(stream))

    def use_persistent(self, enable: bool = True):
        """One persistent-kernel launch per frame (default where supported) or
        the per-op kernel sequence."""
        _lib.call("qora_engine_use_persistent", self.h, 1 if enable else 0)

    def trace(self, enable: bool = True):
        """Turns per-op stamps of the persistent frame kernel on/off and returns
        the last recorded frame: op types int32 [n] and uint64 [n][8]: four
        globaltimer stamps (ns); SM cycles waiting for weight slots, computing
        and reducing; slots consumed."""
        n = C.c_int32()
        _lib.call("qora_engine_trace", self.h, 1 if enable else 0, 0, C.byref(n), None, None)
        ops = np.zeros(n.value, np.int32)
        st = np.zeros((n.value, 8), np.uint64)
        _lib.call("qora_engine_trace", self.h, 1 if enable else 0, n.value, C.byref(n),
                  ops.ctypes.data, st.ctypes.data)
        return ops, st

    def use_graph(self, enable: bool = True):
        _lib.call("qora_engine_use_graph", self.h, 1 if enable else 0)

    def set_temperature(self, temperature: float):
        """The first sample_token's temperature for the following frames
        (frame_temperature, generate_new.rs:82-88)."""
        self.params.temperature = temperature
        _lib.call("qora_engine_set_temperature", self.h, float(temperature))

    def frame(self, text: torch.Tensor, codes: torch.Tensor, stream=None):
        """One frame from device buffers: text [B][H] f32 -> codes [B][16] int32."""
        _lib.call("qora_engine_frame", self.h, _dp(text), _dp(codes), _stream(stream))

    def frame_host(self, text: np.ndarray, codes: np.ndarray, stream=None):
        """One frame from host buffers (copies included; returns after the D2H copy)."""
        _lib.call("qora_engine_frame_host", self.h, text.ctypes.data, codes.ctypes.data,
                  _stream(stream))

    def kernels_per_frame(self) -> int:
        n = C.c_int32()
        _lib.call("qora_engine_kernels_per_frame", self.h, C.byref(n))
        return n.value

    def state(self) -> dict:
        """Copies of the device state (qora_engine_state): logits [B][vocab],
        hidden [B][hidden] (the talker's final-normed output, the predictor's
        next input), prev [B][16], rng [B], positions [B]."""
        ptrs = [C.c_void_p() for _ in range(5)]
        _lib.call("qora_engine_state", self.h, *[C.byref(p) for p in ptrs])
        c, B = self.talker.cfg, self.B
        hid = _device_view(ptrs[1].value, (B, 2, c.t_hidden), "<f4")[:, 0]
        return {"logits": _device_view(ptrs[0].value, (B, c.t_vocab), "<f4").clone(),
                "hidden": hid.clone(),
                "prev": _device_view(ptrs[2].value, (B, 16), "<i4").clone(),
                "rng": _device_view(ptrs[3].value, (B,), "<i8").clone(),
                "positions": _device_view(ptrs[4].value, (B,), "<i4").clone()}


class _CudaArray:
    """A raw device pointer described by __cuda_array_interface__ (no copy)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (ptr, False), "version": 3, "strides": None}


def _device_view(ptr: int, shape, typestr: str) -> torch.Tensor:
    return torch.as_tensor(_CudaArray(ptr, shape, typestr), device="cuda")
