"""QORA-TTS decode engine for B200 (sm_100a).

Host-side mirror of the reference operator surface (gemv.rs, rope.rs,
talker.rs, code_predictor.rs, generate_new.rs) over the C ABI in
include/qora_cuda.h, implemented by libqora_b200.so.  The device API lives in
qora_b200.engine (imports torch).
"""
from . import _lib
from .weights import (ModelConfig, Q4Weight, LayerWeights, TalkerWeights, PredictorWeights,
                      TextProjWeights, ModelFile, quantize_f32_to_q4, synth_q4, synth_normal,
                      synth_talker, synth_predictor, synth_text_proj)

__all__ = ["_lib", "ModelConfig", "Q4Weight", "LayerWeights", "TalkerWeights", "PredictorWeights",
           "TextProjWeights", "ModelFile", "quantize_f32_to_q4", "synth_q4", "synth_normal",
           "synth_talker", "synth_predictor", "synth_text_proj"]
