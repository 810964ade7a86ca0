"""Prefill GEMM (k_gemm_mma: 128-column x 128-row tensor-core tiles over all
of K) against the tensor-core GEMV it replaces on the prefill path
(k_gemv_mma without a K split, selected with QORA_PREFILL_GEMM=0).

Both keep the operands exact (two-part weights, hi / lo inputs scaled by a
power of two per row).  At the 1.7B dims the prefill plan of k_gemv_mma has
no K split, so both accumulate K in the same order and a talker prefill
(the reference's gemm over a prompt, gemv.rs:290-412, inside
prefill_talker_raw_from, talker.rs:379-482) must give the same bits with
either: last hidden, codec-head logits and every cached K / V row, for row
counts that leave partial 128-row tiles (1, 45, 300 rows) and for a prompt
longer than one 512-row chunk (700).  At the tiny dims k_gemv_mma splits K
over a cluster, so the two differ by f32 summation order only (relative
1e-5).  Each setting runs in a child process (the switch is read once per
process)."""
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

_CHILD = textwrap.dedent("""
    import sys, numpy as np, torch
    sys.path.insert(0, {pkg!r})
    import qora_b200 as qb
    from qora_b200 import engine as E
    out = {{}}
    ctx = E.Context(0)
    for name, cfg in (("tiny", qb.ModelConfig.tiny(t_max_pos=1100)),
                      ("full", qb.ModelConfig(t_layers=2, t_max_pos=1100))):
        talker = E.Talker(ctx, qb.synth_talker(cfg), max_batch=1)
        H = cfg.t_hidden
        for T in (1, 45, 300, 700):
            kv = talker.new_kv(max_pos=T, streams=1)
            x = torch.from_numpy(qb.synth_normal(900 + T, 1.0, T * H).reshape(T, H)).cuda()
            h = talker.prefill_talker_raw_from(x, kv, 0)
            out[f"{{name}}_{{T}}_h"] = h.cpu().numpy()
            out[f"{{name}}_{{T}}_lg"] = talker.apply_codec_head(h).cpu().numpy()
            k, v = kv.layer_tensors(cfg.t_layers - 1)
            out[f"{{name}}_{{T}}_k"] = k.cpu().numpy()
            out[f"{{name}}_{{T}}_v"] = v.cpu().numpy()
        del talker
    ctx.check_device_error()
    np.savez({path!r}, **out)
""")


def _run(tmp_path, flag, var="QORA_PREFILL_GEMM"):
    path = str(tmp_path / f"prefill_{var}_{flag}.npz")
    code = _CHILD.format(pkg=os.path.join(ROOT, "qora-tts-12hz-1.7b_b200"), path=path)
    env = dict(os.environ, **{var: flag})
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-3000:]
    return np.load(path)


def test_prefill_gemm_matches_split_free_gemv_bitwise(tmp_path):
    new, old = _run(tmp_path, "1"), _run(tmp_path, "0")
    assert sorted(new.files) == sorted(old.files)
    for key in new.files:
        a, b = new[key], old[key]
        assert a.shape == b.shape, key
        if key.startswith("full"):
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), key
        else:
            err = float(np.max(np.abs(a.astype(np.float64) - b)))
            assert err <= 1e-5 * max(1.0, float(np.max(np.abs(b)))), (key, err)


def test_prefill_attention_tc_matches_cuda_core(tmp_path):
    """k_prefill_attn_tc (tcgen05; Q, K, V, P as f16 hi + lo pairs) against the
    f32 CUDA-core k_prefill_attn (QORA_PREFILL_ATTN_TC=0) at head_dim 128:
    the same prefills agree to f32 summation-order differences (relative
    1e-5 of each tensor's largest magnitude, through two layers)."""
    new, old = _run(tmp_path, "1", "QORA_PREFILL_ATTN_TC"), _run(tmp_path, "0", "QORA_PREFILL_ATTN_TC")
    worst = 0.0
    for key in new.files:
        if not key.startswith("full"):
            continue                  # head_dim 64: the CUDA-core kernel either way
        a, b = new[key].astype(np.float64), old[key].astype(np.float64)
        err = float(np.max(np.abs(a - b))) / max(1e-30, float(np.max(np.abs(b))))
        worst = max(worst, err)
        assert err <= 1e-5, (key, err)
    print(f"prefill attention tc vs cuda-core: worst relative {worst:.2e}")


def test_tc_prefill_bits_do_not_depend_on_the_split():
    """The talker's cache (>= 256 positions) prefills on k_prefill_attn_tc and
    the prefill GEMM: a 300-token prompt prefilled in one call and as 120 +
    180 tokens (the prefix-cache path, generate_new.rs:320-322) gives the
    same last hidden and the same cached K / V, bit for bit."""
    import torch
    import qora_b200 as qb
    from qora_b200 import engine as E
    ctx = E.Context(0)
    cfg = qb.ModelConfig(t_layers=2, t_max_pos=512)
    talker = E.Talker(ctx, qb.synth_talker(cfg), max_batch=1)
    H, T, P = cfg.t_hidden, 300, 120
    x = torch.from_numpy(qb.synth_normal(77, 1.0, T * H).reshape(T, H)).cuda()
    whole = talker.new_kv(max_pos=512, streams=1)
    split = talker.new_kv(max_pos=512, streams=1)
    h1 = talker.prefill_talker_raw_from(x, whole, 0)
    talker.prefill_talker_raw_from(x[:P].contiguous(), split, 0)
    h2 = talker.prefill_talker_raw_from(x[P:].contiguous(), split, P)
    ctx.check_device_error()
    assert np.array_equal(h1.cpu().numpy().view(np.uint32), h2.cpu().numpy().view(np.uint32))
    for layer in range(cfg.t_layers):
        k1, v1 = whole.layer_tensors(layer)
        k2, v2 = split.layer_tensors(layer)
        assert np.array_equal(k1[:, :, :T].cpu().numpy(), k2[:, :, :T].cpu().numpy()), layer
        assert np.array_equal(v1[:, :, :T].cpu().numpy(), v2[:, :, :T].cpu().numpy()), layer
