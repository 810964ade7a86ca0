"""ctypes binding of libqora_b200.so, the engine's C ABI (include/qora_cuda.h).

There is no fallback: if the shared library is missing or a CUDA device is
absent, calls raise.  Build the library with ``make -C qora-tts-12hz-1.7b_b200``
(or ``__graft_entry__.build()``).
"""
from __future__ import annotations

import ctypes as C
import os

_PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(_PKG_DIR, "_build", "libqora_b200.so")

QORA_OK = 0
STATUS = {0: "ok", 1: "invalid argument", 2: "shape mismatch", 3: "CUDA error",
          4: "out of device memory", 5: "position out of range", 6: "unsupported configuration",
          7: "device wait timed out"}


class QoraError(RuntimeError):
    def __init__(self, status: int, where: str, message: str):
        super().__init__(f"{where}: {STATUS.get(status, status)} ({message})")
        self.status = status


class Q4Host(C.Structure):
    _fields_ = [("packed", C.c_void_p), ("scales", C.c_void_p), ("k", C.c_int64), ("n", C.c_int64)]


class LayerHost(C.Structure):
    _fields_ = [(n, Q4Host) for n in ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj",
                                      "up_proj", "down_proj")] + \
               [(n, C.c_void_p) for n in ("q_norm", "k_norm", "input_norm", "post_attn_norm")]


class TalkerHost(C.Structure):
    _fields_ = [("num_layers", C.c_int32), ("hidden", C.c_int32), ("num_heads", C.c_int32),
                ("num_kv_heads", C.c_int32), ("head_dim", C.c_int32), ("ffn", C.c_int32),
                ("vocab", C.c_int32), ("rope_max_pos", C.c_int32), ("rope_theta", C.c_double),
                ("layers", C.c_void_p), ("codec_embedding", Q4Host), ("codec_head", Q4Host),
                ("final_norm", C.c_void_p)]


class PredictorHost(C.Structure):
    _fields_ = [("num_layers", C.c_int32), ("hidden", C.c_int32), ("num_heads", C.c_int32),
                ("num_kv_heads", C.c_int32), ("head_dim", C.c_int32), ("ffn", C.c_int32),
                ("vocab", C.c_int32), ("num_groups", C.c_int32), ("rope_max_pos", C.c_int32),
                ("rope_theta", C.c_double), ("layers", C.c_void_p), ("input_proj", Q4Host),
                ("input_proj_bias", C.c_void_p), ("codec_embeddings", C.c_void_p),
                ("lm_heads", C.c_void_p), ("final_norm", C.c_void_p)]


class TextProjHost(C.Structure):
    _fields_ = [("text_embedding", Q4Host), ("fc1", Q4Host), ("fc2", Q4Host),
                ("fc1_bias", C.c_void_p), ("fc2_bias", C.c_void_p)]


class PromptRow(C.Structure):
    _fields_ = [("text", C.c_int32), ("codes_n", C.c_int32), ("codes", C.c_uint32 * 16)]


class SampleParams(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_int32), ("top_p", C.c_float),
                ("repetition_penalty", C.c_float)]


class DecoderDims(C.Structure):
    """qora_decoder_dims (include/qora_cuda.h)."""
    _fields_ = [(n, C.c_int32) for n in ("codebook_dim", "codebook_size", "num_quantizers", "vq_dim",
                                          "latent", "hidden", "num_heads", "head_dim", "intermediate",
                                          "num_layers", "sliding_window", "upsample_stages",
                                          "upsample_inner", "vocos_blocks")] + \
               [("vocos_channels", C.c_int32 * 8), ("vocos_kernels", C.c_int32 * 8),
                ("vocos_strides", C.c_int32 * 8), ("rope_max_pos", C.c_int32), ("rope_theta", C.c_double)]


# name -> (restype, argtypes); every entry point declared in include/qora_cuda.h
_vp, _i32, _i64, _f32, _u64 = C.c_void_p, C.c_int32, C.c_int64, C.c_float, C.c_uint64
_PP = C.POINTER(C.c_void_p)
SIGNATURES = {
    "qora_ctx_create": (C.c_int, [_i32, _PP]),
    "qora_ctx_destroy": (None, [_vp]),
    "qora_status_string": (C.c_char_p, [_i32]),
    "qora_last_error": (C.c_char_p, []),
    "qora_ctx_check_device_error": (C.c_int, [_vp, _vp]),
    "qora_q4_quantize_host": (C.c_int, [_vp, _i64, _i64, _vp, _vp]),
    "qora_synth_normal_host": (C.c_int, [_u64, _f32, _i64, _vp]),
    "qora_synth_q4_host": (C.c_int, [_u64, _f32, _i64, _i64, _vp, _vp]),
    "qora_q4_weight_upload": (C.c_int, [_vp, _vp, _PP]),
    "qora_q4_weight_destroy": (None, [_vp]),
    "qora_q4_gemv": (C.c_int, [_vp, _vp, _vp, _vp, _i32, _vp]),
    "qora_q4_gemm": (C.c_int, [_vp, _vp, _vp, _i64, _vp, _vp]),
    "qora_q4_embed_rows": (C.c_int, [_vp, _vp, _vp, _i32, _vp, _vp]),
    "qora_rms_norm_f16": (C.c_int, [_vp, _vp, _vp, _i64, _i32, _vp, _vp]),
    "qora_rope_tables_host": (C.c_int, [_i32, _i32, C.c_double, _vp, _i32, _vp, _vp]),
    "qora_kv_create": (C.c_int, [_vp, _i32, _i32, _i32, _i32, _i32, _PP]),
    "qora_kv_create_paged": (C.c_int, [_vp, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _PP]),
    "qora_kv_pages_host": (C.c_int, [_vp, _vp, _vp]),
    "qora_kv_destroy": (None, [_vp]),
    "qora_kv_reset": (C.c_int, [_vp, _vp, _i32, _vp]),
    "qora_kv_lengths_host": (C.c_int, [_vp, _vp, _vp]),
    "qora_kv_copy_stream": (C.c_int, [_vp, _i32, _vp, _i32, _vp]),
    "qora_kv_layer_ptrs": (C.c_int, [_vp, _i32, _PP, _PP, _PP]),
    "qora_kv_export_layer": (C.c_int, [_vp, _i32, _vp, _vp, _vp]),
    "qora_kv_attend": (C.c_int, [_vp, _i32, _vp, _i32, _vp, _vp, _vp, _vp, _i32, _vp, _i32, _i32,
                                  _vp, _vp]),
    "qora_kv_attend_noalloc": (C.c_int, [_vp, _i32, _vp, _i32, _vp, _vp, _vp, _vp, _i32, _vp, _i32,
                                          _i32, _vp, _vp]),
    "qora_model_file_open": (C.c_int, [C.c_char_p, _PP]),
    "qora_model_file_talker": (C.c_int, [_vp, _vp]),
    "qora_model_file_predictor": (C.c_int, [_vp, _vp]),
    "qora_model_file_text_proj": (C.c_int, [_vp, _vp]),
    "qora_model_file_close": (None, [_vp]),
    "qora_text_proj_create": (C.c_int, [_vp, _vp, _PP]),
    "qora_text_proj_destroy": (None, [_vp]),
    "qora_text_proj_embed": (C.c_int, [_vp, _vp, _i32, _vp, _vp]),
    "qora_prompt_assemble": (C.c_int, [_vp, _vp, _vp, _i32, _vp, _i32, _vp, _i32, _vp, _vp]),
    "qora_talker_create": (C.c_int, [_vp, _vp, _i32, _PP]),
    "qora_talker_destroy": (None, [_vp]),
    "qora_talker_step": (C.c_int, [_vp, _vp, _vp, _vp, _i32, _vp, _vp, _vp]),
    "qora_talker_prefill": (C.c_int, [_vp, _vp, _i32, _vp, _i32, _i32, _vp, _vp]),
    "qora_talker_codec_head": (C.c_int, [_vp, _vp, _i32, _vp, _vp]),
    "qora_talker_decode": (C.c_int, [_vp, _vp, _vp, _vp, _i32, _vp, _i32, _vp, _vp]),
    "qora_talker_embed_codec": (C.c_int, [_vp, _vp, _i32, _vp, _vp]),
    "qora_predictor_create": (C.c_int, [_vp, _vp, _i32, _PP]),
    "qora_predictor_destroy": (None, [_vp]),
    "qora_predictor_frame": (C.c_int, [_vp, _vp, _vp, _vp, _i32, _vp, _vp, _vp, _vp]),
    "qora_predictor_embed_sum": (C.c_int, [_vp, _vp, _i32, _vp, _vp]),
    "qora_sample": (C.c_int, [_vp, _vp, _i32, _i32, _vp, _i32, _vp, _vp, _vp, _vp]),
    "qora_engine_create": (C.c_int, [_vp, _vp, _i32, _i32, _vp, _PP]),
    "qora_engine_destroy": (None, [_vp]),
    "qora_engine_prefill": (C.c_int, [_vp, _vp, _i32, _vp, _vp]),
    "qora_engine_prefill_from": (C.c_int, [_vp, _vp, _i32, _i32, _vp, _i32, _vp, _vp]),
    "qora_engine_frame": (C.c_int, [_vp, _vp, _vp, _vp]),
    "qora_engine_frame_host": (C.c_int, [_vp, _vp, _vp, _vp]),
    "qora_engine_use_graph": (C.c_int, [_vp, _i32]),
    "qora_engine_use_persistent": (C.c_int, [_vp, _i32]),
    "qora_engine_set_temperature": (C.c_int, [_vp, _f32]),
    "qora_engine_trace": (C.c_int, [_vp, _i32, _i32, _vp, _vp, _vp]),
    "qora_engine_kernels_per_frame": (C.c_int, [_vp, C.POINTER(C.c_int32)]),
    "qora_decoder_create": (C.c_int, [_vp, _vp, _PP]),
    "qora_decoder_set_tensor": (C.c_int, [_vp, C.c_char_p, _vp, _i64]),
    "qora_decoder_finalize": (C.c_int, [_vp]),
    "qora_decoder_destroy": (None, [_vp]),
    "qora_model_file_decoder": (C.c_int, [_vp, _vp, _PP]),
    "qora_decoder_get_dims": (C.c_int, [_vp, _vp]),
    "qora_decoder_use_tensor_cores": (C.c_int, [_vp, _i32]),
    "qora_decoder_samples": (C.c_int, [_vp, _i64, C.POINTER(C.c_int64)]),
    "qora_decode_to_audio": (C.c_int, [_vp, _vp, _i64, _vp, _i64, _vp, _i64, C.POINTER(C.c_int64), _vp]),
    "qora_decode_to_audio_device": (C.c_int, [_vp, _vp, _i64, _i64, _vp, C.POINTER(C.c_int32), _vp]),
    "qora_engine_state": (C.c_int, [_vp, _PP, _PP, _PP, _PP, _PP]),
}

_lib = None


def load() -> C.CDLL:
    """Load the engine library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"libqora_b200.so not built ({LIB_PATH}); run "
                              f"`make -C {_PKG_DIR}` or __graft_entry__.build()")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int, where: str) -> None:
    if rc != QORA_OK:
        msg = load().qora_last_error()
        raise QoraError(rc, where, msg.decode() if msg else "")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)
