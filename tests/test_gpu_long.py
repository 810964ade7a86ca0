"""Config 3: the long-context KV stress at full size.

The 28-layer talker (1.7B dims, random-init Q4 weights) takes an ICL-style
prefill of 2048 N(0,1) positions per stream (seed 42 + stream), then 2048
greedy decode steps to 4096 positions, for 2 streams with caches of their
own (the configuration runs 32 streams; two suffice for parity, the bench
times 32), held in a paged cache (64-position pages mapped as they grow).
Each step's input is embed_codec_token of the engine's own argmax (last index on ties, code_predictor.rs:335-341) fed back through
forward_with_embedding (talker.rs:263-360): the greedy loop itself runs on
the device.  The oracle is then teacher-forced with exactly those inputs:
one pass over all 4096 rows (prefill_talker_raw_from arithmetic,
talker.rs:379-482, through oracle/oracle_long.c), giving every position's
codec-head logits.  The decode rows therefore use the reference's gemm
rounding instead of its threaded gemv chunking (gemv.rs:290-346); the two
differ by f32 summation order, well inside the tolerance below.

Held to the north-star tolerance at every one of the 2049 logit vectors per
stream: max-abs <= 2e-3, relative (max-abs / max |logit|) <= 1e-3, and
>= 99.5 % greedy-argmax agreement.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ABS_TOL = 2e-3
REL_TOL = 1e-3
STREAMS = 2
PREFILL = 2048
STEPS = 2048


@pytest.fixture(scope="module")
def E():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("-m gpu tests need a CUDA device")
    from qora_b200 import engine
    return engine


def _last_argmax(torch, logits):
    """Argmax with the last index winning ties (code_predictor.rs:335-341)."""
    V = logits.shape[-1]
    return (V - 1) - torch.argmax(torch.flip(logits, [-1]), dim=-1)


def test_config3_long_context(E, orc):
    import torch
    import qora_b200
    from test_gpu_full import _oracle_from
    cfg = qora_b200.ModelConfig()
    H, V = cfg.t_hidden, cfg.t_vocab
    tw = qora_b200.synth_talker(cfg)
    ctx = E.Context(0)
    talker = E.Talker(ctx, tw, max_batch=STREAMS)
    # the paged cache: 64-position pages mapped as the streams grow
    kv = talker.new_kv(max_pos=PREFILL + STEPS, streams=STREAMS, page_positions=64,
                       pool_pages=STREAMS * (PREFILL + STEPS) // 64)
    xs = [orc.synth_normal(42 + s, 1.0, PREFILL * H).reshape(PREFILL, H) for s in range(STREAMS)]
    hid = torch.stack([talker.prefill_talker_raw_from(torch.from_numpy(x).cuda(), kv, 0, kv_stream=s)
                       for s, x in enumerate(xs)])
    logits = talker.apply_codec_head(hid)
    got = np.zeros((STREAMS, STEPS + 1, V), np.float32)
    toks = np.zeros((STREAMS, STEPS), np.int64)
    got[:, 0] = logits.cpu().numpy()
    for step in range(STEPS):
        tok = _last_argmax(torch, logits)
        toks[:, step] = tok.cpu().numpy()
        emb = talker.embed_codec_token(tok)
        _, logits = talker.forward_with_embedding(emb, kv, [PREFILL + step] * STREAMS)
        got[:, step + 1] = logits.cpu().numpy()
    ctx.check_device_error()
    assert list(kv.lengths()) == [PREFILL + STEPS] * STREAMS
    assert kv.pages() == (STREAMS * (PREFILL + STEPS) // 64, 0)
    del kv, talker
    torch.cuda.empty_cache()

    om = orc.OracleModel.__new__(orc.OracleModel)
    om.m = _oracle_from(orc, cfg, tw, None)
    om.t = om.m.talker_struct()
    worst_abs, worst_rel, agree, total = 0.0, 0.0, 0, 0
    for s in range(STREAMS):
        okv = om.talker_kv(PREFILL + STEPS)
        fed = np.stack([om.embed_codec(int(t)) for t in toks[s]])
        _, rl = om.talker_prefill_rows(np.concatenate([xs[s], fed]), okv, 0, logits=True)
        ref = rl[PREFILL - 1:].astype(np.float64)   # the prefill's last row, then every step
        del okv
        err = np.max(np.abs(got[s] - ref), axis=1)
        rel = err / np.maximum(1e-30, np.max(np.abs(ref), axis=1))
        worst_abs, worst_rel = max(worst_abs, float(err.max())), max(worst_rel, float(rel.max()))
        g_arg = (V - 1) - np.argmax(got[s][:, ::-1], axis=1)
        r_arg = (V - 1) - np.argmax(ref[:, ::-1], axis=1)
        agree += int(np.sum(g_arg == r_arg))
        total += STEPS + 1
    print(f"config3: {STREAMS} streams to {PREFILL + STEPS} positions: worst abs {worst_abs:.3e} "
          f"rel {worst_rel:.3e} argmax {agree}/{total}")
    assert worst_abs <= ABS_TOL and worst_rel <= REL_TOL
    assert agree / total >= 0.995
