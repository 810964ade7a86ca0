"""C-ABI checks that need no GPU: the library loads, exports every entry point
include/qora_cuda.h declares, and its host-side functions (quantiser,
synthetic weights, RoPE tables) agree bit-for-bit with the oracle."""
import ctypes as C
import os
import re
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "qora_cuda.h")


@pytest.fixture(scope="module")
def lib():
    import qora_b200
    try:
        return qora_b200._lib.load()
    except ImportError:
        subprocess.run(["make", "-s", "-j8", "-C", os.path.join(ROOT, "qora-tts-12hz-1.7b_b200")],
                       check=True)
        return qora_b200._lib.load()


def header_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(qora_[a-z0-9_]+)\s*\(", src)))


def test_header_symbols_exported(lib):
    names = header_functions()
    assert len(names) >= 35
    out = subprocess.run(["nm", "-D", "--defined-only", lib._name], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (qora_[a-z0-9_]+)", out))
    missing = [n for n in names if n not in exported]
    assert not missing, missing


def test_binding_covers_header(lib):
    import qora_b200
    names = header_functions()
    assert sorted(qora_b200._lib.SIGNATURES) == names


def test_rust_binding_covers_header():
    """The extern "C" block a Rust caller would add (include/qora_cuda_ffi.rs)
    declares exactly the header's functions."""
    src = open(os.path.join(ROOT, "include", "qora_cuda_ffi.rs")).read()
    block = src[src.index('extern "C" {'):src.index("/// Turns a status")]
    assert sorted(set(re.findall(r"pub fn (qora_\w+)", block))) == header_functions()


def test_status_strings(lib):
    assert lib.qora_status_string(0) == b"ok"
    assert lib.qora_status_string(2) == b"shape mismatch"


def test_no_device_fails_loudly(lib):
    """Without a usable CUDA device the context call returns an error, never a
    silent CPU path."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import qora_b200
    h = C.c_void_p()
    rc = lib.qora_ctx_create(0, C.byref(h))
    assert rc != 0
    with pytest.raises(qora_b200._lib.QoraError):
        qora_b200._lib.check(rc, "qora_ctx_create")


def test_quantiser_matches_oracle(lib, orc):
    import qora_b200
    rng = np.random.default_rng(11)
    data = (rng.standard_normal((96, 512)) * 0.02).astype(np.float32)
    data[0, :32] = 0.0
    data[7, 100] = 0.9
    mine = qora_b200.quantize_f32_to_q4(data)
    ref = orc.quantize(data)
    assert np.array_equal(mine.packed, ref.packed)
    assert np.array_equal(mine.scales, ref.scales)


def test_synth_matches_oracle(lib, orc):
    import qora_b200
    for seed, k, n in [(1, 64, 256), (99, 33, 96)]:
        a = qora_b200.synth_q4(seed, 0.02, k, n)
        b = orc.synth_q4(seed, 0.02, k, n)
        assert np.array_equal(a.packed, b.packed) and np.array_equal(a.scales, b.scales)
    assert np.array_equal(qora_b200.synth_normal(5, 1.0, 1001), orc.synth_normal(5, 1.0, 1001))


def test_model_synth_matches_oracle(lib, orc):
    import qora_b200
    cfg = qora_b200.ModelConfig.tiny()
    t = qora_b200.synth_talker(cfg)
    p = qora_b200.synth_predictor(cfg)
    m = orc.Model.synth(orc.ModelConfig.tiny())
    assert np.array_equal(t.layers[1].down_proj.packed, m.t_layers[1].down_proj.packed)
    assert np.array_equal(t.codec_head.scales, m.codec_head.scales)
    assert np.array_equal(p.lm_heads[14].packed, m.lm_heads[14].packed)
    assert np.array_equal(p.input_proj_bias, m.input_proj_bias)


def test_rope_tables_match_oracle(lib, orc):
    from qora_b200 import _lib as ql
    half = 64
    cos = np.empty(300 * half, np.float32)
    sin = np.empty(300 * half, np.float32)
    sec = np.array([24, 20, 20], np.int32)
    ql.call("qora_rope_tables_host", 128, 300, 1e6, sec.ctypes.data, 3, cos.ctypes.data,
            sin.ctypes.data)
    c2, s2 = orc.rope_tables(128, 300, 1e6, [24, 20, 20])
    assert np.array_equal(cos, c2) and np.array_equal(sin, s2)


def test_engine_module_imports_and_fails_loudly_without_gpu(lib):
    import torch
    from qora_b200 import engine as E
    assert hasattr(E, "Context") and hasattr(E, "Engine") and hasattr(E, "Talker")
    if not torch.cuda.is_available():
        import qora_b200
        with pytest.raises(qora_b200._lib.QoraError):
            E.Context(0)


def test_tiny_and_full_configs_agree_with_oracle(orc):
    import dataclasses
    import qora_b200
    for a, b in [(qora_b200.ModelConfig.tiny(), orc.ModelConfig.tiny()),
                 (qora_b200.ModelConfig(), orc.ModelConfig())]:
        assert dataclasses.asdict(a) == dataclasses.asdict(b)
