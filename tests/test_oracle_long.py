"""The long-sequence oracle (oracle/oracle_long.c) against the oracle it
speeds up (CPU only).

oq_gemm_long and oq_talker_prefill_rows reorganise gemm_q4 (gemv.rs:349-412)
and prefill_talker_raw_from (talker.rs:379-482) into blocked, vectorised,
multi-threaded loops for sequences of thousands of positions; every output
element must keep the reference's operation order, so they are held bit for
bit to oq_gemm / oq_talker_prefill (and to the scalar kernel with the SIMD
paths off)."""
import numpy as np
import pytest


@pytest.mark.parametrize("k,n,rows", [(64, 256, 1), (96, 288, 13), (128, 100, 25), (2048, 96, 40)])
def test_gemm_long_bits(orc, k, n, rows):
    w = orc.synth_q4(31 + k + n, 0.02, k, n)
    x = orc.synth_normal(5 + rows, 1.0, rows * k).reshape(rows, k)
    x[0, :7] = 0.0          # skipped rows of the weight (gemv.rs:259)
    x[rows - 1, 3] = -0.0
    got = orc.gemm_long(x, w)
    ref = np.stack([orc.gemv_single(x[r], w) for r in range(rows)])
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    if n % 32:
        assert not got[:, n // 32 * 32:].any()  # tail columns stay zero (gemv.rs:846-861)


def test_gemm_long_scalar_path_bits(orc):
    w = orc.synth_q4(77, 0.02, 256, 320)
    x = orc.synth_normal(9, 1.0, 17 * 256).reshape(17, 256)
    L = orc.lib()
    old = L.oq_get_simd()
    try:
        L.oq_set_simd(0)
        got = orc.gemm_long(x, w)
    finally:
        L.oq_set_simd(old)
    ref = np.stack([orc.gemv_scalar(x[r], w.packed, w.scales, w.n, 0, w.k) for r in range(17)])
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.fixture(scope="module")
def tiny(orc):
    m = orc.Model.synth(orc.ModelConfig.tiny())
    return m, orc.OracleModel(m)


def test_prefill_rows_equals_prefill(orc, tiny):
    """Every row's hidden, the cache and the last hidden equal oq_talker_prefill's bits
    (row j's hidden = the last hidden of a prefill of rows 0..j)."""
    m, om = tiny
    c = m.cfg
    T = 37
    x = orc.synth_normal(41, 1.0, T * c.t_hidden).reshape(T, c.t_hidden)
    kv1 = om.talker_kv()
    rows, logits = om.talker_prefill_rows(x, kv1, 0, logits=True)
    kv2 = om.talker_kv()
    last = om.talker_prefill(x, kv2, 0)
    assert np.array_equal(rows[-1], last)
    for layer in range(c.t_layers):
        assert np.array_equal(kv1.k(layer)[:T], kv2.k(layer)[:T])
        assert np.array_equal(kv1.v(layer)[:T], kv2.v(layer)[:T])
    for j in (0, 11, 24):
        kv3 = om.talker_kv()
        assert np.array_equal(rows[j], om.talker_prefill(x[:j + 1], kv3, 0))
    ref_logits = np.stack([orc.gemv_single(rows[r], m.codec_head) for r in range(T)])
    assert np.array_equal(logits, ref_logits)


def test_prefill_rows_on_a_prefix(orc, tiny):
    """A suffix prefilled on top of a cached prefix (start_pos > 0)."""
    m, om = tiny
    c = m.cfg
    x = orc.synth_normal(43, 1.0, 30 * c.t_hidden).reshape(30, c.t_hidden)
    kv1 = om.talker_kv()
    om.talker_prefill(x[:19], kv1, 0)
    rows = om.talker_prefill_rows(x[19:], kv1, 19)
    kv2 = om.talker_kv()
    om.talker_prefill(x[:19], kv2, 0)
    last = om.talker_prefill(x[19:], kv2, 19)
    assert np.array_equal(rows[-1], last)
    assert kv1.len(0) == 30
