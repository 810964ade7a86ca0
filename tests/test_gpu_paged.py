"""Paged KV cache (qora_kv_create_paged) through the C ABI.

The reference grows one Vec per layer per stream (RawKvCache, gemv.rs:75-86);
the paged cache draws fixed pages from a preallocated pool as streams grow.
The kernels are the same as for the slab layout and only the row addressing
differs, so a paged cache must give the slab cache's results bit for bit:
talker prefill + steps (tiny model), the standalone attend at short and long
capacities, a prefix copied into other streams (full pages shared, the
partial page copied), pool exhaustion reported before any launch, and pages
returned by reset."""
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


@pytest.fixture(scope="module")
def tiny(E, ctx):
    import qora_b200
    cfg = qora_b200.ModelConfig.tiny(t_max_pos=512)
    return cfg, E.Talker(ctx, qora_b200.synth_talker(cfg), max_batch=4)


def _run_talker(orc, talker, kv, cfg, B, T, steps, seed):
    """Per-stream prefill of T rows, then `steps` batched steps; returns every
    step's hidden and logits."""
    import torch
    H = cfg.t_hidden
    for b in range(B):
        x = orc.synth_normal(seed + b, 1.0, T * H).reshape(T, H)
        talker.prefill_talker_raw_from(torch.from_numpy(x).cuda(), kv, 0, kv_stream=b)
    out = []
    for s in range(steps):
        emb = torch.from_numpy(orc.synth_normal(seed + 100 + s, 1.0, B * H).reshape(B, H)).cuda()
        h, lg = talker.forward_with_embedding(emb, kv, [T + s] * B)
        out.append((h.cpu().numpy(), lg.cpu().numpy()))
    return out


@pytest.mark.parametrize("page", [32, 64])
def test_paged_talker_equals_slab_bitwise(E, ctx, orc, tiny, page):
    cfg, talker = tiny
    B, T, steps = 3, 45, 30
    slab = talker.new_kv(max_pos=128, streams=B)
    paged = talker.new_kv(max_pos=128, streams=B, page_positions=page, pool_pages=3 * (128 // page))
    a = _run_talker(orc, talker, slab, cfg, B, T, steps, 300)
    b = _run_talker(orc, talker, paged, cfg, B, T, steps, 300)
    ctx.check_device_error()
    for (h1, l1), (h2, l2) in zip(a, b):
        assert np.array_equal(h1.view(np.uint32), h2.view(np.uint32))
        assert np.array_equal(l1.view(np.uint32), l2.view(np.uint32))
    assert list(paged.lengths()) == [T + steps] * B
    mapped, free = paged.pages()
    assert mapped == B * ((T + steps + page - 1) // page)
    k1, v1 = slab.layer_tensors(1)
    k2, v2 = paged.layer_tensors(1)       # gathered into the slab layout
    n = T + steps
    assert np.array_equal(k1[:, :, :n].cpu().numpy(), k2[:, :, :n].cpu().numpy())
    assert np.array_equal(v1[:, :, :n].cpu().numpy(), v2[:, :, :n].cpu().numpy())


def test_paged_prefix_copy_shares_full_pages(E, ctx, orc, tiny):
    """A 70-position prefix (two full 32-position pages and 6 rows) copied to
    three streams: the full pages are shared, the partial page is copied; each
    stream then grows on its own pages, and every step equals the slab cache's."""
    import torch
    cfg, talker = tiny
    H, P0, steps = cfg.t_hidden, 70, 12
    x = orc.synth_normal(400, 1.0, P0 * H).reshape(P0, H)
    caches = {}
    for name, kw in (("slab", {}), ("paged", {"page_positions": 32, "pool_pages": 16})):
        kv = talker.new_kv(max_pos=128, streams=4, **kw)
        talker.prefill_talker_raw_from(torch.from_numpy(x).cuda(), kv, 0, kv_stream=0)
        for d in (1, 2, 3):
            kv.copy_stream_from(d, kv, 0)
        caches[name] = kv
    mapped, _ = caches["paged"].pages()
    assert mapped == 3 + 3          # stream 0's three pages + one copied partial page per copy
    assert list(caches["paged"].lengths()) == [P0] * 4
    outs = {}
    for name, kv in caches.items():
        res = []
        for s in range(steps):
            emb = torch.from_numpy(orc.synth_normal(500 + s, 1.0, 4 * H).reshape(4, H)).cuda()
            h, lg = talker.forward_with_embedding(emb, kv, [P0 + s] * 4)
            res.append(lg.cpu().numpy())
        outs[name] = res
    ctx.check_device_error()
    for l1, l2 in zip(outs["slab"], outs["paged"]):
        assert np.array_equal(l1.view(np.uint32), l2.view(np.uint32))
    mapped, _ = caches["paged"].pages()
    assert mapped == 3 + 3          # 82 positions still fit the third page of each stream


def test_paged_pool_exhaustion_and_reset(E, ctx, orc, tiny):
    import torch
    from qora_b200 import _lib
    cfg, talker = tiny
    H = cfg.t_hidden
    kv = talker.new_kv(max_pos=256, streams=2, page_positions=32, pool_pages=3)
    x = torch.from_numpy(orc.synth_normal(600, 1.0, 64 * H).reshape(64, H)).cuda()
    talker.prefill_talker_raw_from(x, kv, 0, kv_stream=0)       # two pages
    with pytest.raises(_lib.QoraError) as ei:                     # two more do not fit
        talker.prefill_talker_raw_from(x, kv, 0, kv_stream=1)
    assert ei.value.status == 4                                   # QORA_ERR_OOM, before any launch
    assert list(kv.lengths()) == [64, 0]
    kv.reset([0])
    assert kv.pages() == (0, 3)
    talker.prefill_talker_raw_from(x, kv, 0, kv_stream=1)
    assert list(kv.lengths()) == [0, 64] and kv.pages() == (2, 1)
    ctx.check_device_error()


@pytest.mark.parametrize("max_pos,page", [(48, 32), (300, 64)])
def test_paged_attend_equals_slab(E, ctx, orc, max_pos, page):
    """qora_kv_attend on the short-cache and the streamed kernel."""
    import torch
    hd, heads, kvh, B, layers, steps = 128, 16, 8, 3, 2, max_pos - 8
    rng = np.random.default_rng(page)
    gam = torch.from_numpy(np.full(hd, 0x3C00, np.uint16).view(np.int16)).cuda()
    cos, sin = orc.rope_tables(hd, 1024, 1e6)
    d_cos, d_sin = torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()
    slab = E.KvCache(ctx, layers, kvh, hd, max_pos, B)
    paged = E.KvCache(ctx, layers, kvh, hd, max_pos, B, page_positions=page,
                      pool_pages=B * ((max_pos + page - 1) // page))
    width = (heads + 2 * kvh) * hd
    for s in range(steps):
        qkv = torch.from_numpy(rng.standard_normal((B, width)).astype(np.float32)).cuda()
        pos = torch.full((B,), s, dtype=torch.int32, device="cuda")
        a = slab.attend(1, qkv, heads, gam, gam, d_cos, d_sin, pos, advance=True).cpu().numpy()
        b = paged.attend(1, qkv, heads, gam, gam, d_cos, d_sin, pos, advance=True).cpu().numpy()
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), s
    ctx.check_device_error()
    assert list(paged.lengths()) == [steps] * B
