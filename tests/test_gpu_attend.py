"""qora_kv_attend (KV append + attend of one layer, talker.rs:285-331) against
the oracle's restatement of the same block, through the C ABI.

Three streams at different RoPE positions, 300 steps so the position splits
of the decode kernel (32 positions per tile, up to 16 splits) and their
merge are exercised; head_dim 128 with 16/8 heads (talker) and head_dim 64
with 16/8 heads (predictor at the BASELINE's head_dim)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATOL = 2e-5   # attention outputs are O(1); fp32, online softmax vs two-pass softmax


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


def _f16(a):
    return np.asarray(a, np.float16).view(np.uint16)


# caches of 256 positions or more decode on the streamed kernel (bulk-copy
# ring, per-warp online softmax), shorter ones on the per-tile kernel
@pytest.mark.parametrize("hd,steps,heads", [(128, 300, 16), (64, 40, 16), (64, 300, 16),
                                            (128, 260, 32), (128, 270, 8)])
def test_attend_matches_oracle(E, ctx, orc, hd, steps, heads):
    import torch
    kvh, B, layers, layer = 8, 3, 2, 1
    max_pos, rope_max = steps + 8, 1024
    rng = np.random.default_rng(hd)
    qn = _f16(1.0 + 0.1 * rng.standard_normal(hd))
    kn = _f16(1.0 + 0.1 * rng.standard_normal(hd))
    cos, sin = orc.rope_tables(hd, rope_max, 1e6)
    kv = E.KvCache(ctx, layers, kvh, hd, max_pos, B)
    okv = [orc.KV(layers, kvh, hd, max_pos) for _ in range(B)]
    d_qn = torch.from_numpy(qn.view(np.int16)).cuda()
    d_kn = torch.from_numpy(kn.view(np.int16)).cuda()
    d_cos, d_sin = torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()
    base = np.array([0, 7, 500], np.int32)
    width = (heads + 2 * kvh) * hd
    worst = 0.0
    for s in range(steps):
        qkv = rng.standard_normal((B, width)).astype(np.float32)
        pos = base + s
        got = kv.attend(layer, torch.from_numpy(qkv).cuda(), heads, d_qn, d_kn, d_cos, d_sin,
                        torch.from_numpy(pos).cuda(), advance=True).cpu().numpy()
        for b in range(B):
            q, k, v = qkv[b, :heads * hd], qkv[b, heads * hd:(heads + kvh) * hd], qkv[b, (heads + kvh) * hd:]
            ref = orc.attend_step(okv[b], layer, q, k, v, heads, kvh, hd, qn, kn, cos, sin, int(pos[b]))
            worst = max(worst, float(np.max(np.abs(got[b] - ref))))
    ctx.check_device_error()
    assert worst <= ATOL, worst
    assert list(kv.lengths()) == [steps] * B
    # appended keys (normed + roped) and values match the oracle's cache
    k_dev, v_dev = (t.cpu().numpy() for t in kv.layer_tensors(layer))
    for b in range(B):
        ok = okv[b].k(layer)[:steps].transpose(1, 0, 2)
        ov = okv[b].v(layer)[:steps].transpose(1, 0, 2)
        # keys: qk-norm sums in a different order (warp tree vs sequential)
        assert float(np.max(np.abs(k_dev[b, :, :steps] - ok))) <= 4e-6
        assert np.array_equal(v_dev[b, :, :steps], ov)


def test_attend_position_past_rope_table_is_an_error(E, ctx, orc):
    import torch
    from qora_b200 import _lib
    hd, heads, kvh = 64, 4, 2
    cos, sin = orc.rope_tables(hd, 8, 1e6)
    kv = E.KvCache(ctx, 1, kvh, hd, 16, 1)
    one = torch.from_numpy(_f16(np.ones(hd)).view(np.int16)).cuda()
    qkv = torch.zeros(1, (heads + 2 * kvh) * hd, device="cuda")
    kv.attend(0, qkv, heads, one, one, torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda(),
              torch.tensor([8], dtype=torch.int32, device="cuda"))
    with pytest.raises(_lib.QoraError) as ei:
        ctx.check_device_error()
    assert ei.value.status == 5   # QORA_ERR_RANGE


def test_attend_rejects_bad_shapes(E, ctx):
    import torch
    from qora_b200 import _lib
    kv = E.KvCache(ctx, 1, 2, 64, 16, 1)
    z = torch.zeros(4, device="cuda")
    zi = torch.zeros(1, dtype=torch.int32, device="cuda")
    with pytest.raises(_lib.QoraError):      # 3 heads over 2 kv heads
        kv.attend(0, torch.zeros(1, 7 * 64, device="cuda"), 3, z, z, z, z, zi)
    with pytest.raises(_lib.QoraError):      # layer out of range
        kv.attend(5, torch.zeros(1, 8 * 64, device="cuda"), 4, z, z, z, z, zi)
