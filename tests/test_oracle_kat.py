"""Pins the CPU oracle before anything is checked against it.

* The reference's own GEMV known-answer tests (gemv.rs:756-861), restated
  with its xorshift generators (gemv.rs:693-730): SIMD == scalar bit-exact,
  k-chunk assembly, many-chunk tolerance, tail-n behaviour.  Both SIMD ports
  (AVX2: simd.rs:76-153, AVX-512: simd.rs:203-269) are held to the scalar
  oracle (gemv.rs:249-287).
* The reference's sampler tests (generate_new.rs:918-955), restated.
* IEEE binary16 conversions (the `half` crate) checked exhaustively against
  numpy, and the quantiser (gemv.rs:92-130) against an independent numpy
  restatement.
"""
import math

import numpy as np
import pytest


def _check_case(orc, k, n, seed, in_zero, sc_zero, fn):
    r = orc.XRng(seed)
    groups = n // 32
    packed = r.bytes(k * groups * 16)
    scales = r.scales(k * groups, sc_zero)
    x = r.inputs(k, in_zero)
    expect = orc.gemv_scalar(x, packed, scales, n, 0, k)
    got = fn(x, packed, scales, n, 0, k)
    assert got.view(np.uint32).tolist() == expect.view(np.uint32).tolist(), (k, n, seed)
    return expect


SIMD = ["avx2", "avx512"]


def _simd_fn(orc, name):
    if name == "avx2":
        if not orc.lib().oq_has_avx2():
            pytest.skip("no AVX2 on this host")
        return orc.gemv_avx2
    if not orc.lib().oq_has_avx512():
        pytest.skip("no AVX-512 on this host")
    return orc.gemv_avx512


@pytest.mark.parametrize("simd", SIMD)
def test_simd_matches_scalar_shapes(orc, simd):
    # gemv.rs:758-765
    fn = _simd_fn(orc, simd)
    for k, n, seed in [(64, 2048, 1), (64, 6144, 2), (32, 1024, 3), (16, 256, 4), (1, 32, 5)]:
        _check_case(orc, k, n, seed, 0.0, 0.0, fn)


@pytest.mark.parametrize("simd", SIMD)
def test_simd_matches_scalar_sparse(orc, simd):
    # gemv.rs:769-773: zero-skipping (input==0, scale==0), negative scales
    fn = _simd_fn(orc, simd)
    _check_case(orc, 48, 1024, 11, 0.3, 0.2, fn)
    _check_case(orc, 32, 2048, 12, 0.5, 0.5, fn)


@pytest.mark.parametrize("simd", SIMD)
def test_simd_subrange_matches(orc, simd):
    # gemv.rs:777-810
    fn = _simd_fn(orc, simd)
    r = orc.XRng(21)
    k, n = 64, 1024
    packed = r.bytes(k * (n // 32) * 16)
    scales = r.scales(k * (n // 32), 0.1)
    x = r.inputs(k, 0.1)
    full = orc.gemv_scalar(x, packed, scales, n, 0, k)
    acc = np.zeros(n, np.float32)
    acc_ref = np.zeros(n, np.float32)
    for a, b in [(0, 16), (16, 48), (48, 64)]:
        acc += fn(x, packed, scales, n, a, b)
        acc_ref += orc.gemv_scalar(x, packed, scales, n, a, b)
    assert np.array_equal(acc.view(np.uint32), acc_ref.view(np.uint32))
    assert np.all(np.abs(acc - full) < 1e-3)


@pytest.mark.parametrize("simd", SIMD)
def test_simd_many_chunks_tolerance(orc, simd):
    # gemv.rs:814-842
    fn = _simd_fn(orc, simd)
    r = orc.XRng(77)
    k, n = 128, 1024
    packed = r.bytes(k * (n // 32) * 16)
    scales = r.scales(k * (n // 32), 0.1)
    x = r.inputs(k, 0.1)
    full = orc.gemv_scalar(x, packed, scales, n, 0, k)
    nc = 32
    ck = (k + nc - 1) // nc
    acc = np.zeros(n, np.float32)
    for t in range(nc):
        a, b = t * ck, min((t + 1) * ck, k)
        if a >= b:
            continue
        acc += fn(x, packed, scales, n, a, b)
    assert np.all(np.abs(acc - full) < 1e-3)


@pytest.mark.parametrize("simd", SIMD)
def test_simd_tail_n(orc, simd):
    # gemv.rs:846-861: n not a multiple of 32 -> remainder stays zero
    fn = _simd_fn(orc, simd)
    r = orc.XRng(31)
    k, n = 16, 100
    packed = r.bytes(k * (n // 32) * 16)
    scales = r.scales(k * (n // 32), 0.0)
    x = r.inputs(k, 0.0)
    expect = orc.gemv_scalar(x, packed, scales, n, 0, k)
    got = fn(x, packed, scales, n, 0, k)
    assert np.array_equal(got, expect)
    assert np.all(got[96:] == 0.0)


def test_scalar_gemv_matches_float64(orc):
    """Independent numpy restatement of the Q4 dot product (dequant w, f64 sum)."""
    r = orc.XRng(99)
    k, n = 96, 512
    packed = r.bytes(k * (n // 32) * 16)
    scales = r.scales(k * (n // 32), 0.1)
    x = r.inputs(k, 0.1)
    got = orc.gemv_scalar(x, packed, scales, n, 0, k)
    lo = (packed & 15).astype(np.int64) - 8
    hi = (packed >> 4).astype(np.int64) - 8
    q = np.stack([lo, hi], -1).reshape(k, n)
    sc = scales.view(np.float16).astype(np.float64).reshape(k, n // 32)
    w = q * np.repeat(sc, 32, axis=1)
    ref = x.astype(np.float64) @ w
    assert np.max(np.abs(got - ref)) < 1e-4


def test_f16_to_f32_exhaustive(orc):
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    got = np.zeros(65536, np.float32)
    orc.lib().oq_f16_to_f32_array(orc.ptr(bits), orc.ptr(got), 65536)
    ref = bits.view(np.float16).astype(np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), ref[~nan].view(np.uint32))


def test_f32_to_f16_rne(orc):
    rng = np.random.default_rng(5)
    vals = np.concatenate([
        rng.standard_normal(200000).astype(np.float32) * np.float32(0.01),
        rng.standard_normal(50000).astype(np.float32) * np.float32(1e-5),  # subnormal range
        rng.standard_normal(50000).astype(np.float32) * np.float32(3e4),   # near overflow
        # every f16 value and every midpoint between neighbours (ties)
        np.arange(0, 0x7c00, dtype=np.uint32).astype(np.uint16).view(np.float16).astype(np.float32),
        ((np.arange(0, 0x7bff, dtype=np.uint32).astype(np.uint16).view(np.float16).astype(np.float64)
          + np.arange(1, 0x7c00, dtype=np.uint32).astype(np.uint16).view(np.float16).astype(np.float64))
         / 2).astype(np.float32),
        np.array([65504, 65519.99, 65520, 1e9, -1e9, 0.0, -0.0, np.inf, -np.inf], np.float32),
    ]).astype(np.float32)
    vals = np.concatenate([vals, -vals])
    got = orc.f32_to_f16(vals)
    with np.errstate(over="ignore"):  # values past 65520 round to infinity, as intended
        ref = vals.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, ref)


def _np_quantize(data):
    """Independent numpy restatement of quantize_f32_to_q4 (gemv.rs:92-130)."""
    k, n = data.shape
    g = data.reshape(k, n // 32, 32)
    absmax = np.max(np.abs(g), axis=2)
    scale = (absmax / np.float32(7.0)).astype(np.float32)
    scales = scale.astype(np.float16).view(np.uint16)
    with np.errstate(divide="ignore"):
        inv = np.where(scale > 0, np.float32(1.0) / scale, np.float32(0.0)).astype(np.float32)
    v = (g * inv[:, :, None]).astype(np.float32)
    rnd = np.sign(v) * np.floor(np.abs(v) + np.float32(0.5))  # half away from zero
    # floor(|v| + 0.5) in f32 may round for |v| near 2^23; values here are tiny.
    q = (np.clip(rnd, -8, 7) + 8).astype(np.uint8).reshape(k, n // 32, 16, 2)
    packed = (q[..., 0] | (q[..., 1] << 4)).reshape(-1)
    return packed, scales.reshape(-1)


def test_quantiser_matches_numpy(orc):
    rng = np.random.default_rng(3)
    data = (rng.standard_normal((64, 256)) * 0.02).astype(np.float32)
    data[3, :32] = 0.0          # all-zero group -> scale 0, q = 8
    data[5, 40] = 0.5           # outlier group
    w = orc.quantize(data)
    p_ref, s_ref = _np_quantize(data)
    assert np.array_equal(w.scales, s_ref)
    assert np.array_equal(w.packed, p_ref)


def test_quantiser_roundtrip_error(orc):
    rng = np.random.default_rng(4)
    data = (rng.standard_normal((32, 1024)) * 0.02).astype(np.float32)
    w = orc.quantize(data)
    deq = np.stack([orc.embed_lookup(w, i) for i in range(32)])
    sc = w.scales.view(np.float16).astype(np.float32).reshape(32, 32)
    err = np.abs(deq - data).reshape(32, 32, 32)
    assert np.all(err <= sc[:, :, None] * 0.5 + 1e-4)


def test_synth_q4_equals_quantised_normals(orc):
    k, n = 16, 128
    w = orc.synth_q4(42, 0.02, k, n)
    ref = orc.quantize(orc.synth_normal(42, 0.02, k * n).reshape(k, n))
    assert np.array_equal(w.packed, ref.packed) and np.array_equal(w.scales, ref.scales)
    z = orc.synth_normal(7, 1.0, 200000)
    assert abs(z.mean()) < 0.01 and abs(z.std() - 1.0) < 0.01


def test_pool_chunking_within_reference_tolerance(orc):
    """gemv_q4 pool chunking (gemv.rs:290-346) vs single pass: the bound the
    reference's own tests accept (1e-3)."""
    w = orc.synth_q4(5, 0.02, 2048, 2048)
    x = orc.synth_normal(6, 1.0, 2048)
    single = orc.gemv_single(x, w)
    for workers in (1, 4, 16):
        got = orc.gemv(x, w, workers=workers)
        assert np.max(np.abs(got - single)) < 1e-3
    assert np.array_equal(orc.gemv(x, w, workers=1), single)


def test_rope_tables_match_libm(orc):
    hd, mp = 128, 300
    cos, sin = orc.rope_tables(hd, mp, 1e6, [24, 20, 20])
    for pos in (0, 1, 7, 299):
        for i in (0, 1, 23, 24, 47, 63):
            freq = 1.0 / math.pow(1e6, (2 * i) / hd)
            assert cos[pos * 64 + i] == np.float32(math.cos(pos * freq))
            assert sin[pos * 64 + i] == np.float32(math.sin(pos * freq))
    c2, s2 = orc.rope_tables(hd, mp, 1e6, [64])
    assert np.array_equal(cos, c2) and np.array_equal(sin, s2)


def test_argmax_last_index_on_ties(orc):
    a = np.array([1.0, 3.0, 3.0, 2.0], np.float32)
    assert orc.lib().oq_argmax(orc.ptr(a), 4) == 2  # code_predictor.rs:336-339
    b = np.array([5.0], np.float32)
    assert orc.lib().oq_argmax(orc.ptr(b), 1) == 0


# ---- sampler KATs: generate_new.rs:902-955 ----------------------------------
def _params(orc, top_p, top_k=0, temp=1.0, rep=1.0):
    return orc.SampleParams(temp, top_k, top_p, rep)


def test_top_p_off_by_default(orc):
    logits = np.array([2.0, 1.0, 0.5, 0.1], np.float32)
    for tp in (1.0, 0.0, -0.5, 2.0):
        p = _params(orc, tp)
        seen = [False] * 4
        rng = 12345
        for _ in range(200):
            t, rng = orc.sample_token(logits, p, np.zeros(0, np.uint32), rng, 1.0)
            seen[t] = True
        assert all(seen), tp


def test_top_p_cuts_tail(orc):
    logits = np.array([5.0, 1.0, 1.0, 1.0], np.float32)
    p = _params(orc, 0.5)
    rng = 999
    for _ in range(50):
        t, rng = orc.sample_token(logits, p, np.zeros(0, np.uint32), rng, 1.0)
        assert t == 0


def test_top_p_keeps_argmax_always(orc):
    logits = np.array([3.0, 2.9, 2.8], np.float32)
    p = _params(orc, 0.01)
    rng = 7
    for _ in range(20):
        t, rng = orc.sample_token(logits, p, np.zeros(0, np.uint32), rng, 1.0)
        assert t == 0


def test_simple_rand_xorshift(orc):
    # generate_new.rs:17-22: xorshift64 (13, 7, 17), r = state as f32 / u64::MAX as f32
    s = 12345
    for _ in range(100):
        r, s2 = orc.simple_rand(s)
        x = s
        x ^= (x << 13) & 0xFFFFFFFFFFFFFFFF
        x ^= x >> 7
        x ^= (x << 17) & 0xFFFFFFFFFFFFFFFF
        assert s2 == x
        assert r == np.float32(np.float32(x) / np.float32(2.0 ** 64))
        s = s2


def test_topk_stable_ties(orc):
    """Top-k keeps the first k by (prob desc, index asc) (stable sort, :806-811)."""
    logits = np.zeros(10, np.float32)
    logits[[2, 5, 7]] = 1.0
    p = _params(orc, 1.0, top_k=2)
    probs = orc.sample_probs(logits, p, np.zeros(0, np.uint32), 1.0)
    assert np.count_nonzero(probs) == 2 and probs[2] > 0 and probs[5] > 0 and probs[7] == 0
    logits = np.zeros(10, np.float32)
    p = _params(orc, 1.0, top_k=3)
    probs = orc.sample_probs(logits, p, np.zeros(0, np.uint32), 1.0)
    assert list(np.nonzero(probs)[0]) == [0, 1, 2]


def test_repetition_penalty_sign_rule(orc):
    logits = np.array([2.0, -2.0, 1.0, 0.0], np.float32)
    p = _params(orc, 1.0, temp=1.0, rep=2.0)
    probs = orc.sample_probs(logits, p, np.array([0, 1, 3], np.uint32), 1.0)
    pen = np.array([1.0, -4.0, 1.0, 0.0], np.float64)
    ref = np.exp(pen - pen.max())
    ref /= ref.sum()
    assert np.allclose(probs, ref, atol=1e-6)
