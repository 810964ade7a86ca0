"""GPU parity of the Q4 GEMV kernels against the CPU oracle.

Inputs: the reference's own GEMV test generators and shapes (gemv.rs:693-773,
846-861) plus the talker / predictor shapes with random-init N(0, 0.02)
weights.  The GPU sums in a different (fixed) order than the reference's
k-sequential loop, so results are compared within the tolerance the
reference accepts for its own chunked summation (gemv.rs:806-809, 1e-3),
tightened here to 1e-4 relative to the output scale.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def E():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("-m gpu tests need a CUDA device")
    from qora_b200 import engine
    return engine


@pytest.fixture(scope="module")
def ctx(E):
    return E.Context(0)


def _dev(E, ctx, packed, scales, k, n):
    from qora_b200 import Q4Weight
    return E.DeviceQ4(ctx, Q4Weight(np.ascontiguousarray(packed), np.ascontiguousarray(scales), k, n))


def _close(got, ref, rel=1e-4):
    scale = max(1.0, float(np.max(np.abs(ref))))
    err = float(np.max(np.abs(got - ref)))
    assert err <= rel * scale, f"max abs err {err} (scale {scale})"
    return err


def _kat(orc, k, n, seed, in_zero, sc_zero):
    r = orc.XRng(seed)
    packed = r.bytes(k * (n // 32) * 16)
    scales = r.scales(k * (n // 32), sc_zero)
    x = r.inputs(k, in_zero)
    return packed, scales, x


@pytest.mark.parametrize("k,n,seed,iz,sz", [
    (64, 2048, 1, 0.0, 0.0), (64, 6144, 2, 0.0, 0.0), (32, 1024, 3, 0.0, 0.0),
    (16, 256, 4, 0.0, 0.0), (1, 32, 5, 0.0, 0.0),          # gemv.rs:758-765
    (48, 1024, 11, 0.3, 0.2), (32, 2048, 12, 0.5, 0.5),    # gemv.rs:769-773
])
def test_reference_kat_shapes(E, ctx, orc, k, n, seed, iz, sz):
    import torch
    packed, scales, x = _kat(orc, k, n, seed, iz, sz)
    ref = orc.gemv_scalar(x, packed, scales, n, 0, k)
    w = _dev(E, ctx, packed, scales, k, n)
    got = w.gemv(torch.from_numpy(x).cuda()).cpu().numpy()[0]
    _close(got, ref, 1e-5)


def test_tail_n_stays_zero(E, ctx, orc):
    import torch
    k, n = 16, 100                                           # gemv.rs:846-861
    r = orc.XRng(31)
    packed = r.bytes(k * (n // 32) * 16)
    scales = r.scales(k * (n // 32), 0.0)
    x = r.inputs(k, 0.0)
    ref = orc.gemv_scalar(x, packed, scales, n, 0, k)
    got = _dev(E, ctx, packed, scales, k, n).gemv(torch.from_numpy(x).cuda()).cpu().numpy()[0]
    _close(got[:96], ref[:96], 1e-5)
    assert np.all(got[96:] == 0.0)


SHAPES = [(2048, 4096), (2048, 1024), (2048, 2048), (2048, 6144), (6144, 2048), (2048, 3072),
          (1024, 2048), (1024, 1024), (3072, 1024), (1024, 3072), (1024, 512)]


@pytest.mark.parametrize("k,n", SHAPES)
def test_model_shapes_batch1(E, ctx, orc, k, n):
    import torch
    w = orc.synth_q4(7000 + k + n, 0.02, k, n)
    x = orc.synth_normal(17 + k, 1.0, k)
    ref = orc.gemv_single(x, w)
    got = _dev(E, ctx, w.packed, w.scales, k, n).gemv(torch.from_numpy(x).cuda()).cpu().numpy()[0]
    _close(got, ref)


@pytest.mark.parametrize("rows", [2, 3, 4, 5, 8, 16, 17, 32, 64])
def test_batched_rows(E, ctx, orc, rows):
    import torch
    k, n = 2048, 2048
    w = orc.synth_q4(55, 0.02, k, n)
    x = orc.synth_normal(56 + rows, 1.0, rows * k).reshape(rows, k)
    dw = _dev(E, ctx, w.packed, w.scales, k, n)
    got = dw.gemv(torch.from_numpy(x).cuda()).cpu().numpy()
    for r in range(rows):
        _close(got[r], orc.gemv_single(x[r], w))


def test_gemm_matches_tokens(E, ctx, orc):
    import torch
    k, n, T = 1024, 3072, 37
    w = orc.synth_q4(77, 0.02, k, n)
    x = orc.synth_normal(78, 1.0, T * k).reshape(T, k)
    got = _dev(E, ctx, w.packed, w.scales, k, n).gemm(torch.from_numpy(x).cuda()).cpu().numpy()
    import ctypes
    ref = np.zeros((T, n), np.float32)
    ws = w.cstruct()
    orc.lib().oq_gemm(orc.ptr(x), T, ctypes.addressof(ws), orc.ptr(ref))
    for t in range(T):
        _close(got[t], ref[t])


def test_gemv_is_deterministic(E, ctx, orc):
    import torch
    k, n = 6144, 2048
    w = orc.synth_q4(91, 0.02, k, n)
    x = torch.from_numpy(orc.synth_normal(92, 1.0, 4 * k)).cuda().reshape(4, k)
    dw = _dev(E, ctx, w.packed, w.scales, k, n)
    a = dw.gemv(x).cpu().numpy()
    b = dw.gemv(x).cpu().numpy()
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_embed_rows_bit_exact(E, ctx, orc):
    import torch
    w = orc.synth_q4(33, 0.02, 3072, 2048)
    dw = _dev(E, ctx, w.packed, w.scales, 3072, 2048)
    toks = np.array([0, 1, 2149, 3071, 17], np.int32)
    got = dw.embed_lookup(torch.from_numpy(toks).cuda()).cpu().numpy()
    for i, t in enumerate(toks):
        ref = orc.embed_lookup(w, int(t))
        assert np.array_equal(got[i].view(np.uint32), ref.view(np.uint32))


def test_rms_norm(E, ctx, orc):
    import torch
    x = orc.synth_normal(5, 1.0, 3 * 2048).reshape(3, 2048)
    gamma = orc.f32_to_f16(orc.synth_normal(6, 0.5, 2048) + 1.0)
    got = E.rms_norm_f16(ctx, torch.from_numpy(x).cuda(),
                         torch.from_numpy(gamma.view(np.int16)).cuda()).cpu().numpy()
    for r in range(3):
        ref = orc.rms_norm_f16(x[r], gamma)
        assert np.max(np.abs(got[r] - ref)) <= 1e-5 * np.max(np.abs(ref))


@pytest.mark.parametrize("k,rows", [(128, 1), (128, 2), (128, 3), (128, 4), (128, 6), (256, 2),
                                    (256, 5), (96, 2), (32, 4)])
def test_small_k_single_split(E, ctx, orc, k, rows):
    """k <= 256 runs without split-K (one CTA holds all rows of a column group)."""
    import torch
    n = 512
    w = orc.synth_q4(123 + k, 0.02, k, n)
    x = orc.synth_normal(124 + rows, 1.0, rows * k).reshape(rows, k)
    got = _dev(E, ctx, w.packed, w.scales, k, n).gemv(torch.from_numpy(x).cuda()).cpu().numpy()
    for r in range(rows):
        _close(got[r], orc.gemv_single(x[r], w))


# Batches of >= 8 rows on 128-column tiles run on the tensor cores (tcgen05,
# f16 operands split into exact weight halves and hi/lo input halves, f32
# accumulation): the same 1e-4-of-scale bound as the CUDA-core kernel.
@pytest.mark.parametrize("k,n,rows", [(2048, 6144, 32), (6144, 2048, 16), (2048, 3072, 8),
                                      (1024, 2048, 100), (2048, 1024, 512), (1024, 3072, 9)])
def test_batched_shapes_tensor_core(E, ctx, orc, k, n, rows):
    import ctypes
    import torch
    w = orc.synth_q4(600 + rows, 0.02, k, n)
    x = orc.synth_normal(601 + rows, 1.0, rows * k).reshape(rows, k)
    got = _dev(E, ctx, w.packed, w.scales, k, n).gemv(torch.from_numpy(x).cuda()).cpu().numpy()
    ctx.check_device_error()
    ref = np.zeros((rows, n), np.float32)
    ws = w.cstruct()
    orc.lib().oq_gemm(orc.ptr(x), rows, ctypes.addressof(ws), orc.ptr(ref))
    for r in range(rows):
        _close(got[r], ref[r])


def test_batched_tensor_core_is_deterministic(E, ctx, orc):
    import torch
    k, n, rows = 2048, 2048, 24
    w = orc.synth_q4(610, 0.02, k, n)
    x = torch.from_numpy(orc.synth_normal(611, 1.0, rows * k)).cuda().reshape(rows, k)
    dw = _dev(E, ctx, w.packed, w.scales, k, n)
    a = dw.gemv(x).cpu().numpy()
    b = dw.gemv(x).cpu().numpy()
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("k,n", [(2048, 1024), (6144, 2048)])
def test_batched_any_input_range(E, ctx, orc, k, n):
    """The tensor-core operands are f16 halves of each row scaled by a power of
    two chosen per row, so activation outliers (|x| up to 1e5, past the f16
    range) and rows of tiny values (|x| < 2^-14, f16 subnormals unscaled) keep
    the 1e-4-of-scale bound, each row against its own output scale."""
    import ctypes
    import torch
    rows = 16
    w = orc.synth_q4(630 + k, 0.02, k, n)
    x = orc.synth_normal(631 + k, 1.0, rows * k).reshape(rows, k)
    x[3, 100] = 1.0e5                     # one outlier in a normal row
    x[3, 7] = -7.5e4
    x[5] *= 1.0e5                         # a whole row of large values
    x[9] *= 2.0e-6                        # a row of values below 2^-14
    x[11, ::3] = 0.0                      # zeros (skipped rows of the weight)
    x[12] = 0.0                           # an all-zero row
    got = _dev(E, ctx, w.packed, w.scales, k, n).gemv(torch.from_numpy(x).cuda()).cpu().numpy()
    ctx.check_device_error()              # no range error
    ref = np.zeros((rows, n), np.float32)
    ws = w.cstruct()
    orc.lib().oq_gemm(orc.ptr(x), rows, ctypes.addressof(ws), orc.ptr(ref))
    for r in range(rows):
        scale = float(np.max(np.abs(ref[r])))
        err = float(np.max(np.abs(got[r].astype(np.float64) - ref[r])))
        assert err <= 1e-4 * scale or (scale == 0.0 and err == 0.0), (r, err, scale)


def test_batched_infinite_input_is_an_error(E, ctx, orc):
    # an infinite input has no finite scale: reported instead of propagating silently
    import torch
    from qora_b200 import _lib
    k, n, rows = 1024, 1024, 8
    w = orc.synth_q4(620, 0.02, k, n)
    x = orc.synth_normal(621, 1.0, rows * k).reshape(rows, k)
    x[3, 100] = np.inf
    _dev(E, ctx, w.packed, w.scales, k, n).gemv(torch.from_numpy(x).cuda())
    with pytest.raises(_lib.QoraError) as ei:
        ctx.check_device_error()
    assert ei.value.status == 5   # QORA_ERR_RANGE
    ctx.check_device_error()      # cleared
