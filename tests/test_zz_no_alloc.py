"""qora_kv_attend_noalloc: the KV append + attend entry point that allocates
no device memory, for callers that cannot let a library call cudaMalloc (a
real-time audio loop that must not stall on an allocation, or a host
application whose memory manager already holds the GPU's memory).

Its scratch is a fixed array in the library's static device memory, shared
by every call.  The test runs it side by side with qora_kv_attend (which
sizes its scratch with cudaMalloc) on two caches that start identical, for
two calls in a row, and requires the same outputs, lengths and cache
contents within the tolerance of tests/test_gpu_attend.py; it also checks
that a call beyond the static array's limit is refused before any launch.

This file is collected last on purpose, so that a run stopping at the first
failure has run every other test before it."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATOL = 2e-5   # same tolerance as tests/test_gpu_attend.py


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


def test_noalloc_attend_matches_allocating_attend(E, ctx, orc):
    import torch
    heads, kvh, hd, B, layers, layer = 16, 8, 128, 4, 2, 1
    max_pos, rope_max, prefix = 128, 256, 70
    rng = np.random.default_rng(11)
    qn = torch.from_numpy(_f16(1.0 + 0.1 * rng.standard_normal(hd)).view(np.int16)).cuda()
    kn = torch.from_numpy(_f16(1.0 + 0.1 * rng.standard_normal(hd)).view(np.int16)).cuda()
    cos, sin = (torch.from_numpy(t).cuda() for t in orc.rope_tables(hd, rope_max, 1e6))
    width = (heads + 2 * kvh) * hd
    kv_a = E.KvCache(ctx, layers, kvh, hd, max_pos, B)   # qora_kv_attend
    kv_b = E.KvCache(ctx, layers, kvh, hd, max_pos, B)   # qora_kv_attend_noalloc
    base = torch.tensor([3, 40, 100, 0], dtype=torch.int32, device="cuda")
    # identical prefixes in both caches (several position splits per query)
    for s in range(prefix):
        qkv = torch.from_numpy(rng.standard_normal((B, width)).astype(np.float32)).cuda()
        kv_a.attend(layer, qkv, heads, qn, kn, cos, sin, base + s, advance=True)
        kv_b.attend(layer, qkv, heads, qn, kn, cos, sin, base + s, advance=True)
    # two calls in a row through each entry point
    for s in range(prefix, prefix + 2):
        qkv = torch.from_numpy(rng.standard_normal((B, width)).astype(np.float32)).cuda()
        ref = kv_a.attend(layer, qkv, heads, qn, kn, cos, sin, base + s, advance=True)
        got = kv_b.attend(layer, qkv, heads, qn, kn, cos, sin, base + s, advance=True,
                          noalloc=True)
        torch.cuda.synchronize()
        ctx.check_device_error()
        err = float((got - ref).abs().max())
        assert err <= ATOL, f"call {s - prefix}: max abs diff {err}"
    assert list(kv_b.lengths()) == list(kv_a.lengths()) == [prefix + 2] * B
    ka, va = kv_a.layer_tensors(layer)
    kb, vb = kv_b.layer_tensors(layer)
    assert float((ka - kb).abs().max()) == 0.0 and float((va - vb).abs().max()) == 0.0


def test_noalloc_attend_rejects_sizes_beyond_its_scratch(E, ctx, orc):
    import torch
    from qora_b200 import _lib
    heads, kvh, hd, B = 16, 8, 128, 9          # 9 * 16 * 128 > 16384
    kv = E.KvCache(ctx, 1, kvh, hd, 8, B)
    one = torch.from_numpy(_f16(np.ones(hd)).view(np.int16)).cuda()
    cos, sin = (torch.from_numpy(t).cuda() for t in orc.rope_tables(hd, 8, 1e6))
    qkv = torch.zeros(B, (heads + 2 * kvh) * hd, device="cuda")
    pos = torch.zeros(B, dtype=torch.int32, device="cuda")
    with pytest.raises(_lib.QoraError) as ei:
        kv.attend(0, qkv, heads, one, one, cos, sin, pos, noalloc=True)
    assert ei.value.status == 6                # QORA_ERR_UNSUPPORTED
    assert list(kv.lengths()) == [0] * B       # nothing ran
