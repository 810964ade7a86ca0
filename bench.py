#!/usr/bin/env python
"""QORA-TTS decode-path benchmark (one JSON line on rank 0).

Workload (BASELINE.json metric "talker+predictor frames/s per B200 (batch 1 &
32) and Q4 GEMV HBM GB/s vs roofline"): the per-frame loop of
generate_new.rs:606-665 on the 1.7B dims (28-layer talker, 5-layer code
predictor with head_dim 128 as in the reference config), random-init
N(0, 0.02) Q4 weights, 64-token N(0,1) prefill per stream, sampling with
top-k 50 / temperature 0.9 / repetition penalty 1.05, EOS ignored.
One step = one frame for every stream on the GPU: talker step + 15-code
predictor + sampling, replayed as one CUDA graph.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl ours|reference]

Multi-GPU: one process per GPU (torchrun); each GPU runs its own B streams
(replicas, no data-path collective); value = all frames / max-over-ranks time.
--impl reference times the reference's CPU algorithm (the oracle port of the
Rust path: AVX-512 Q4 GEMV + worker pool) on the host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "qora-tts-12hz-1.7b_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import numpy as np  # noqa: E402

METRIC = "talker+predictor frames/s per B200 (batch 1 & 32) and Q4 GEMV HBM GB/s vs roofline"
PREFILL = 64
REF_FRAMES_PER_S = 1.0 / 0.35   # README.md:272-280: 0.35 s/frame talker+predictor, laptop CPU
L2_BYTES = 126 * 1024 * 1024


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-batch32", action="store_true")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-roofline", action="store_true")
    ap.add_argument("--no-config3", action="store_true")
    ap.add_argument("--no-decoder", action="store_true")
    ap.add_argument("--frames", type=int, default=None, help="frames of the decoder profile case")
    ap.add_argument("--profile-case", default=None,
                    choices=["gemv", "frame_trace", "batch_frame", "attn_decode", "prefill", "decoder"],
                    help="small fixed workload for an ncu capture instead of the bench")
    return ap.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ----------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------- CPU arm
def oracle_model_from(tw, pw):
    """Wrap the engine's host weight arrays (reference layout) for the oracle."""
    import pyoracle as po
    c = tw.cfg

    def q(w):
        return po.Q4Weight(w.packed, w.scales, w.k, w.n)

    def lay(lw):
        return po.LayerWeights(q(lw.q_proj), q(lw.k_proj), q(lw.v_proj), q(lw.o_proj),
                               q(lw.gate_proj), q(lw.up_proj), q(lw.down_proj), lw.q_norm,
                               lw.k_norm, lw.input_norm, lw.post_attn_norm)

    ocfg = po.ModelConfig(**{k: getattr(c, k) for k in po.ModelConfig.__dataclass_fields__})
    half = c.t_head_dim // 2
    return po.Model(cfg=ocfg, t_layers=[lay(x) for x in tw.layers],
                    codec_embedding=q(tw.codec_embedding), codec_head=q(tw.codec_head),
                    t_final_norm=tw.final_norm,
                    t_rope=po.rope_tables(c.t_head_dim, c.t_max_pos, c.rope_theta,
                                          [24, 20, 20] if half == 64 else [half]),
                    p_layers=[lay(x) for x in pw.layers],
                    input_proj=q(pw.input_proj) if pw.input_proj is not None else None,
                    input_proj_bias=pw.input_proj_bias,
                    codec_embeddings=[q(e) for e in pw.codec_embeddings],
                    lm_heads=[q(h) for h in pw.lm_heads], p_final_norm=pw.final_norm,
                    p_rope=po.rope_tables(c.p_head_dim, c.p_max_pos, c.rope_theta))


def cpu_frames(model, frames: int, warmup: int, budget_s: float | None = None):
    """Times the oracle frame loop (batch 1) on the host; returns frames/s."""
    import pyoracle as po
    om = po.OracleModel(model)
    c = model.cfg
    tkv = om.talker_kv(PREFILL + warmup + frames + 8)
    pkv = om.predictor_kv()
    x = po.synth_normal(1000, 1.0, PREFILL * c.t_hidden).reshape(PREFILL, c.t_hidden)
    hidden = om.talker_prefill(x, tkv, 0)
    st = {"logits": om.codec_head(hidden), "hidden": hidden.copy(),
          "prev": np.zeros(16, np.uint32), "rng": 1000}
    text = po.synth_normal(77, 1.0, c.t_hidden)
    params = po.SampleParams(0.9, 50, 1.0, 1.05)
    pos = PREFILL
    for _ in range(warmup):
        om.frame(tkv, pkv, params, text, pos, st)
        pos += 1
    t0 = time.perf_counter()
    done = 0
    while done < frames:
        om.frame(tkv, pkv, params, text, pos, st)
        pos += 1
        done += 1
        if budget_s is not None and time.perf_counter() - t0 > budget_s and done >= 3:
            break
    dt = time.perf_counter() - t0
    return done / dt, done, dt, po.lib().oq_pool_workers()


class Ranks:
    """One process per GPU as torchrun starts them (RANK / LOCAL_RANK /
    WORLD_SIZE / MASTER_* from the environment): the barrier that brackets the
    timed region and the max over ranks of a device-timed duration.  Replicas
    only: no collective touches the data path.  backend "nccl" (device
    tensors) for the bench; "gloo" (CPU tensors) for the host-side tests."""

    def __init__(self, backend: str = "nccl", device=None, timeout_s: int = 300):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.backend, self.device, self.dist = backend, device, None
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            kw = {"device_id": device} if backend == "nccl" else {}
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
            self.dist = dist

    def barrier(self):
        if self.dist is not None:
            self.dist.barrier()

    def max(self, v: float) -> float:
        """The largest of every rank's v (each rank's own time when alone)."""
        if self.dist is None:
            return v
        import torch
        t = torch.tensor([v], dtype=torch.float64,
                         device=self.device if self.backend == "nccl" else "cpu")
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def stream_seed(self, base: int, batch: int, b: int) -> int:
        """Seed of stream b of this rank: every stream of the job distinct."""
        return base + self.rank * batch + b

    def close(self):
        if self.dist is not None:
            self.dist.barrier()
            self.dist.destroy_process_group()
            self.dist = None


def aggregate_rate(units_per_rank: int, world: int, ms_max: float) -> float:
    """Whole-job rate: the units every rank processed over the slowest rank's time."""
    return units_per_rank * world / (ms_max / 1000.0)


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import pyoracle as po
    po.build()
    cfg = po.ModelConfig()
    model = po.Model.synth(cfg)
    fps, done, dt, cores = cpu_frames(model, args.steps, args.warmup)
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": fps, "unit": "frames/s",
        "n_gpus": args.gpus, "steps": done, "warmup": args.warmup, "ms_per_step": 1000.0 * dt / done,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": fps / REF_FRAMES_PER_S,
        "dtype": "f32 (Q4 weights)", "data": "synthetic: random-init N(0,0.02) Q4 weights",
        "config": {"workload": "frame loop batch 1 (talker step + 15-code predictor + top-k 50 "
                               "sampling), 1.7B dims, predictor head_dim 128, 64-token prefill",
                   "batch_per_gpu": 1},
        "cpu_baseline": {"value": fps, "unit": "frames/s", "cores": cores, "kind": "port",
                         "sample": f"{done} frames after {args.warmup} warm-up and a 64-token prefill"},
        "e2e": {"value": fps, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ----------------------------------------------------------------- GPU arm
def _graph_time_ms(torch, fn, reps):
    """Capture fn() (a sequence of engine launches) in a CUDA graph and return
    the average replay time in ms (CUDA events on the replay stream)."""
    fn()                                  # warm-up: sizes scratch outside capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            fn()
    torch.cuda.synchronize()
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st = torch.cuda.current_stream()
    e0.record(st)
    for _ in range(reps):
        g.replay()
    e1.record(st)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def frame_algorithmic_bytes(cfg, positions):
    """Algorithmic bytes of one batch-1 frame: talker step (Q4 weights, f16
    norms, K/V read over `positions` + 1 cached positions and the appended
    row, the embedding row) plus the predictor's 15 weight passes (one
    2-token prefill + 14 steps, each with the input projection and one
    head), Q4 at 0.5625 B per weight."""
    q4 = 0.5625
    H, F = cfg.t_hidden, cfg.t_ffn
    qd, kd = cfg.t_heads * cfg.t_head_dim, cfg.t_kv_heads * cfg.t_head_dim
    t_w = cfg.t_layers * (H * (qd + 2 * kd) + qd * H + 2 * H * F + F * H) + H * cfg.t_vocab
    t_norm = 2 * (cfg.t_layers * (2 * H + 2 * cfg.t_head_dim) + H)
    kv_pos = cfg.t_layers * 2 * kd * 4
    Hp, Fp = cfg.p_hidden, cfg.p_ffn
    pq, pk = cfg.p_heads * cfg.p_head_dim, cfg.p_kv_heads * cfg.p_head_dim
    p_layer = Hp * (pq + 2 * pk) + pq * Hp + 2 * Hp * Fp + Fp * Hp
    p_pass = cfg.p_layers * p_layer + H * Hp + Hp * cfg.p_vocab
    return (q4 * t_w + t_norm + kv_pos * (positions + 1) + kv_pos + 1152
            + q4 * cfg.p_groups * p_pass)


def gemv_stream_roofline(E, ctx, tw, torch, reps=5):
    """k_gemv over the whole talker weight set at batch 1, back to back in one
    CUDA graph (197 launches, 796 MB > L2): algorithmic bytes and time."""
    mats = []
    for lw in tw.layers:
        for nm in ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"):
            mats.append(E.DeviceQ4(ctx, getattr(lw, nm)))
    mats.append(E.DeviceQ4(ctx, tw.codec_head))
    xs = {k: torch.randn(1, k, device="cuda") for k in {m.k for m in mats}}
    ys = {n: torch.empty(1, n, device="cuda") for n in {m.n for m in mats}}
    byts = sum(0.5625 * m.k * m.n + 4 * (m.k + m.n) for m in mats)

    def run():
        for m in mats:
            m.gemv(xs[m.k], ys[m.n])

    ms = _graph_time_ms(torch, run, reps)
    del mats
    return byts, ms


def gemv_sweep(E, ctx, torch, qb):
    """Config 1: per-shape GB/s at batch 1/4/16; each replay walks weight copies
    totalling >= 4x L2 so every launch streams from HBM."""
    shapes = [(2048, 4096), (2048, 1024), (2048, 2048), (2048, 6144), (6144, 2048), (2048, 3072)]
    out = {}
    for k, n in shapes:
        w = qb.synth_q4(4242 + k + n, 0.02, k, n)
        wbytes = 0.5625 * k * n
        copies = max(4, int(np.ceil(4 * L2_BYTES / wbytes)))
        devs = [E.DeviceQ4(ctx, w) for _ in range(copies)]
        res = {}
        for B in (1, 4, 16):
            x = torch.randn(B, k, device="cuda")
            y = torch.empty(B, n, device="cuda")

            def run():
                for d in devs:
                    d.gemv(x, y)

            ms = _graph_time_ms(torch, run, 3)
            us = 1000.0 * ms / copies
            gbs = (wbytes + 4 * B * (k + n)) / (us * 1e-6) / 1e9
            res[f"b{B}"] = {"us": round(us, 2), "GB/s": round(gbs, 1)}
        out[f"{k}x{n}"] = res
        del devs
        torch.cuda.empty_cache()
    return out


def config3_rate(E, ctx, tw, torch, qb, K, W, seed0, peak):
    """Config 3: 32 streams, each with its own cache.
    Times the 2048-token N(0,1) prefill of all 32 streams (per stream, 512-row
    chunks), tops every cache up to 4064 positions with a second prefill (an
    ICL prompt of that length fills the same cache), then times K batched
    decode steps (forward_with_embedding for the 32 streams) at positions
    4064 .. 4064+K-1 and, on its own, the decode attention of one layer over
    that cache (qora_kv_attend without advancing: the same append slot and
    the same K/V read every call)."""
    cfg = tw.cfg
    S, P1, P2 = 32, 2048, 4064
    H = cfg.t_hidden
    talker = E.Talker(ctx, tw, max_batch=S)
    kv = talker.new_kv(max_pos=P2 + K + W + 8, streams=S)
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    xs = [torch.from_numpy(qb.synth_normal(seed0 + s, 1.0, P1 * H).reshape(P1, H)).cuda() for s in range(S)]
    torch.cuda.synchronize()
    e0.record(st)
    for s in range(S):
        talker.prefill_talker_raw_from(xs[s], kv, 0, kv_stream=s)
    e1.record(st)
    torch.cuda.synchronize()
    prefill_ms = e0.elapsed_time(e1)
    del xs
    for s in range(S):
        x2 = torch.from_numpy(qb.synth_normal(seed0 + 100 + s, 1.0, (P2 - P1) * H).reshape(P2 - P1, H)).cuda()
        talker.prefill_talker_raw_from(x2, kv, P1, kv_stream=s)
    emb = torch.from_numpy(qb.synth_normal(seed0 + 999, 1.0, S * H).reshape(S, H)).cuda()
    pos = P2
    for _ in range(W):
        talker.forward_with_embedding(emb, kv, [pos] * S)
        pos += 1
    torch.cuda.synchronize()
    p_start = pos
    e0.record(st)
    for _ in range(K):
        talker.forward_with_embedding(emb, kv, [pos] * S)
        pos += 1
    e1.record(st)
    torch.cuda.synchronize()
    step_ms = e0.elapsed_time(e1) / K
    # the decode attention of layer 0 alone, over the cache as it stands
    c = cfg
    qkv = torch.randn(S, (c.t_heads + 2 * c.t_kv_heads) * c.t_head_dim, device="cuda")
    lw = tw.layers[0]
    qn = torch.from_numpy(lw.q_norm.view(np.int16).copy()).cuda()
    kn = torch.from_numpy(lw.k_norm.view(np.int16).copy()).cuda()
    cos, sin = E.build_mrope_tables(c.t_head_dim, c.t_max_pos, c.rope_theta, [24, 20, 20])
    cos, sin = torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()
    posd = torch.full((S,), pos, dtype=torch.int32, device="cuda")
    out = torch.empty(S, c.t_heads * c.t_head_dim, device="cuda")
    reps = 20
    for _ in range(3):
        kv.attend(0, qkv, c.t_heads, qn, kn, cos, sin, posd, out=out)
    torch.cuda.synchronize()
    e0.record(st)
    for _ in range(reps):
        kv.attend(0, qkv, c.t_heads, qn, kn, cos, sin, posd, out=out)
    e1.record(st)
    torch.cuda.synchronize()
    attn_us = 1000.0 * e0.elapsed_time(e1) / reps
    P = pos  # cached positions read per stream (+1 appended row)
    kv_bytes = S * c.t_kv_heads * (P + 1) * c.t_head_dim * 4 * 2
    io_bytes = S * 4 * ((c.t_heads + 2 * c.t_kv_heads) * c.t_head_dim + c.t_heads * c.t_head_dim)
    attn_gbs = (kv_bytes + io_bytes) / (attn_us * 1e-6) / 1e9
    ctx.check_device_error()
    del kv, talker
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return {"streams": S, "prefill_tokens_per_stream": P1,
            "prefill_ms_all_streams": round(prefill_ms, 1),
            "prefill_tokens_per_s": round(S * P1 / (prefill_ms / 1000.0), 1),
            "decode_positions": [p_start, p_start + K - 1], "decode_steps": K,
            "ms_per_step": round(step_ms, 3), "stream_steps_per_s": round(S / (step_ms / 1000.0), 1),
            "attention": {"kernel": "k_attention (decode, 32 streams, one layer)",
                          "positions": P + 1, "us_per_launch": round(attn_us, 2),
                          "algorithmic_bytes_per_launch": int(kv_bytes + io_bytes),
                          "achieved": round(attn_gbs, 1), "peak": peak, "unit": "GB/s",
                          "frac": round(attn_gbs / peak, 4)}}


def engine_rate(E, talker, pred, torch, qb, B, K, W, seed0, with_e2e=False, prefill=PREFILL):
    cfg = talker.cfg
    max_pos = prefill + W + (2 * K if with_e2e else K) + 8
    eng = E.Engine(talker, pred, B, max_pos)
    x = np.stack([qb.synth_normal(seed0 + b, 1.0, prefill * cfg.t_hidden).reshape(prefill, cfg.t_hidden)
                  for b in range(B)])
    eng.prefill(x, [seed0 + b for b in range(B)])
    eng.use_graph(True)
    text = torch.from_numpy(qb.synth_normal(77, 1.0, B * cfg.t_hidden).reshape(B, cfg.t_hidden)).cuda()
    codes = torch.zeros(B, 16, dtype=torch.int32, device="cuda")
    for _ in range(W):
        eng.frame(text, codes)
    torch.cuda.synchronize()
    return eng, text, codes


# DRAM bytes per launch from the committed ncu captures (text copied here,
# never read at run time): k_frame on the bench's batch-1 frame workload, and
# k_gemv's DRAM bytes per algorithmic byte on the talker gate/up shape.
KFRAME_DRAM_BYTES = 946941952        # profiles/k_frame_b1_frame.md
KGEMV_DRAM_PER_ALG_BYTE = 1.0058     # profiles/k_gemv_b1_2048x6144.md


def predictor_rate(E, ctx, qb, torch, hd, frames):
    """Config 2: the code predictor alone at batch 1 -
    one generate_acoustic_codes per frame (2-token prefill + 14 steps, 15
    heads with argmax), the per-op kernels of a frame captured in one CUDA
    graph and replayed; talker hidden N(0,1) (seed 7), semantic row from a
    codec-embedding-shaped table."""
    cfg = qb.ModelConfig(p_head_dim=hd)
    pw = qb.synth_predictor(cfg)
    pred = E.CodePredictor(ctx, pw, max_batch=1)
    kv = pred.new_kv()
    hid = torch.from_numpy(qb.synth_normal(7, 1.0, cfg.t_hidden)).cuda().reshape(1, -1)
    sem = torch.from_numpy(qb.synth_normal(8, 1.0, cfg.t_hidden)).cuda().reshape(1, -1)
    codes = torch.zeros(1, cfg.p_groups, dtype=torch.int32, device="cuda")
    from qora_b200 import _lib

    def run():
        _lib.call("qora_predictor_frame", pred.h, kv.h, hid.data_ptr(), sem.data_ptr(), 1,
                  codes.data_ptr(), None, None, torch.cuda.current_stream().cuda_stream)

    ms = _graph_time_ms(torch, run, frames)
    del pred, kv
    return {"head_dim": hd, "frames": frames, "ms_per_frame": round(ms, 4),
            "frames_per_s": round(1000.0 / ms, 1)}


def talker_step_rate(E, ctx, tw, torch, qb, steps=256, prefill=32):
    """Config 0: the talker alone at batch 1 - a 32-token
    prefill, then `steps` forward_with_embedding steps (per-op kernels of one
    step captured in a CUDA graph; each replay appends a position, so the
    replays walk positions 32 .. 32 + steps - 1 as config 0 does)."""
    cfg = tw.cfg
    talker = E.Talker(ctx, tw, max_batch=1)
    kv = talker.new_kv(max_pos=prefill + steps + 8)
    x = torch.from_numpy(qb.synth_normal(42, 1.0, prefill * cfg.t_hidden).reshape(prefill, -1)).cuda()
    emb = torch.from_numpy(qb.synth_normal(43, 1.0, cfg.t_hidden)).cuda().reshape(1, -1)
    pos = torch.full((1,), prefill, dtype=torch.int32, device="cuda")
    hidden = torch.empty(1, cfg.t_hidden, device="cuda")
    logits = torch.empty(1, cfg.t_vocab, device="cuda")
    from qora_b200 import _lib

    def run():
        _lib.call("qora_talker_step", talker.h, kv.h, emb.data_ptr(), pos.data_ptr(), 1,
                  hidden.data_ptr(), logits.data_ptr(), torch.cuda.current_stream().cuda_stream)

    talker.prefill_talker_raw_from(x, kv, 0)
    # _graph_time_ms runs one eager step and one replay before timing: start the
    # timed replays two positions in, and time steps - 2 of them
    ms = _graph_time_ms(torch, run, steps - 2)
    del talker, kv
    return {"prefill_tokens": prefill, "steps": steps, "ms_per_step": round(ms, 4),
            "steps_per_s": round(1000.0 / ms, 1)}


DECODER_FRAMES = 241          # the reference's decode measurement (alynaze.txt:17-22: 241 frames)
FP32_PEAK_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12   # nominal: SMs x FP32 lanes x 2 x clocks.max.sm


def decoder_flops(d, frames: int) -> int:
    """Algorithmic FLOPs (2 per multiply-add) of decode_to_audio over `frames`
    frames: every projection and convolution term, the attention's scores and
    weighted sums over each position's window; element-wise ops not counted."""
    F = frames
    HD = d.num_heads * d.head_dim
    f = 2 * 2 * d.codebook_dim * d.vq_dim * F                 # codebook output projections
    f += 2 * d.vq_dim * d.latent * 3 * F                      # pre-conv
    f += 2 * d.latent * d.hidden * F                          # input projection
    keys = sum(min(t + 1, d.sliding_window) for t in range(F))
    f += d.num_layers * (2 * F * (d.hidden * 3 * HD + HD * d.hidden + 2 * d.hidden * d.intermediate
                                  + d.intermediate * d.hidden) + 2 * 2 * HD * keys)
    f += 2 * d.hidden * d.latent * F                          # output projection
    L = F
    for _ in range(d.upsample_stages):
        L *= 2
        f += 2 * d.latent * d.latent * L + 2 * d.latent * 7 * L + 2 * 2 * d.latent * d.upsample_inner * L
    ch = d.vocos_channels
    f += 2 * d.latent * ch[0] * 7 * L
    for b, (k, s) in enumerate(zip(d.vocos_kernels, d.vocos_strides)):
        L *= s
        f += 2 * ch[b] * ch[b + 1] * (k // s) * L + 3 * (2 * ch[b + 1] * ch[b + 1] * 8 * L)
    f += 2 * ch[-1] * 7 * L
    return f


def decoder_rate(ctx, torch, frames=DECODER_FRAMES, reps=5, cpu_frames_n=None):
    """The speech decoder (decode_to_audio, decoder.rs:395-582) at the 12 Hz
    tokenizer dims on `frames` frames of uniform random codes (seed 5),
    random-init f32 weights: device time per decode (codes resident, CUDA
    events over `reps` decodes after 2 untimed ones), end to end through
    qora_decode_to_audio (host codes in, host samples out), the implicit-GEMM
    roofline, and the oracle's time per frame on a few frames (CPU)."""
    from qora_b200.decoder import DecoderDims, SpeechDecoder, synth_decoder
    d = DecoderDims()
    W = synth_decoder(d)
    dec = SpeechDecoder(ctx, d, W)
    codes = np.random.default_rng(5).integers(0, d.codebook_size, (d.num_quantizers, frames)).astype(np.uint32)
    cd = torch.from_numpy(codes.astype(np.int32)).cuda()
    out = torch.empty(frames * d.hop, dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream()
    launches = 0
    for _ in range(2):
        launches = dec.decode_device(cd, frames, out, stream=st)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        dec.decode_device(cd, frames, out, stream=st)
    e1.record(st)
    torch.cuda.synchronize()
    ctx.check_device_error()
    ms = e0.elapsed_time(e1) / reps
    dec.decode_to_audio(codes)
    t0 = time.perf_counter()
    for _ in range(reps):
        host = dec.decode_to_audio(codes)
    e2e_ms = 1000.0 * (time.perf_counter() - t0) / reps
    flops = decoder_flops(d, frames)
    tf = flops / (ms * 1e-3) / 1e12
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            tf32x3, tf32_src = float(json.load(f)["bf16_tflops"]) / 2 / 3, "measured bf16 burst"
    except Exception:
        tf32x3, tf32_src = 1590.0 / 2 / 3, "fallback bf16 1590"
    audio_s = frames * d.hop / 24000.0
    res = {"workload": f"decode_to_audio of {frames} frames ({audio_s:.2f} s of 24 kHz audio), 12 Hz tokenizer "
                       "dims, random-init f32 weights, uniform random codes; largest activation "
                       f"{d.vocos_channels[-1] * frames * d.hop * 4 / 1e6:.0f} MB > L2",
           "frames": frames, "ms_per_decode": round(ms, 3), "frames_per_s": round(frames / (ms * 1e-3), 1),
           "audio_s_per_s": round(audio_s / (ms * 1e-3), 1), "gpu_launches_per_decode": launches,
           "e2e": {"ms_per_decode": round(e2e_ms, 3), "frames_per_s": round(frames / (e2e_ms * 1e-3), 1),
                   "h2d_bytes_per_decode": int(codes.nbytes), "d2h_bytes_per_decode": int(host.nbytes)},
           "roofline": {"bound": "tensor (f32-exact as 3 TF32 products)",
                        "kernel": "whole decode (k_dec_conv_tc dominant)",
                        "achieved": round(tf, 2), "peak": round(tf32x3, 1), "unit": "TFLOP/s",
                        "frac": round(tf / tf32x3, 4),
                        "peak_source": f"{tf32_src}: TF32 dense = half the bf16 GEMM rate, / 3 products per "
                                       "f32-exact term",
                        "fp32_cuda_core_peak": round(FP32_PEAK_TFLOPS, 1),
                        "flops_per_decode": flops},
           "vs_published_cpu": "the reference decodes 241 frames in ~15 s on its 22-thread laptop CPU "
                               "(alynaze.txt:22)"}
    if cpu_frames_n:
        import pydecoder as pd
        cc = codes[:, :cpu_frames_n]
        t0 = time.perf_counter()
        pd.decode_to_audio(W, cc, dims=d)
        dt = time.perf_counter() - t0
        res["cpu_baseline"] = {"value": round(cpu_frames_n / dt, 3), "unit": "frames/s", "cores": 1,
                               "kind": "port", "sample": f"{cpu_frames_n} frames through the oracle's "
                                                         "decode_to_audio (single-threaded C restatement)"}
    del dec
    return res


def run_ours(args):
    import torch
    import qora_b200 as qb
    from qora_b200 import engine as E

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    ranks = Ranks("nccl", torch.device("cuda", local))
    world, rank = ranks.world, ranks.rank

    K, W, B = args.steps, max(3, args.warmup), args.batch
    cfg = qb.ModelConfig()
    tw, pw = qb.synth_talker(cfg), qb.synth_predictor(cfg)
    ctx = E.Context(local)
    maxb = max(B, 1 if args.no_batch32 else 32)
    talker = E.Talker(ctx, tw, max_batch=maxb)
    pred = E.CodePredictor(ctx, pw, max_batch=maxb)
    peak, peak_src = peaks()

    def barrier():
        ranks.barrier()
        torch.cuda.synchronize()

    max_over_ranks = ranks.max
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed_frames(eng, text, codes, n):
        barrier()
        e0.record(st)
        for _ in range(n):
            eng.frame(text, codes)
        e1.record(st)
        torch.cuda.synchronize()
        return max_over_ranks(e0.elapsed_time(e1))

    # the clock sampler runs across every timed GPU leg below
    clk = ClockSampler(local).__enter__()

    # ---- device-resident frame loop (value)
    eng, text, codes = engine_rate(E, talker, pred, torch, qb, B, K, W, ranks.stream_seed(1000, B, 0), True)
    ms = timed_frames(eng, text, codes, K)
    kernels = eng.kernels_per_frame()
    ctx.check_device_error()
    frames = B * K * world
    value = aggregate_rate(B * K, world, ms)

    # ---- end to end through the public host API (pinned host buffers), on the
    # same workload: the cache is prefilled again (untimed) so these frames sit
    # at the same positions as the device-resident ones above
    x = np.stack([qb.synth_normal(ranks.stream_seed(1000, B, b), 1.0, PREFILL * cfg.t_hidden).reshape(PREFILL, cfg.t_hidden)
                  for b in range(B)])
    eng.prefill(x, [ranks.stream_seed(1000, B, b) for b in range(B)])
    for _ in range(W):
        eng.frame(text, codes)
    torch.cuda.synchronize()
    text_pin = text.cpu().pin_memory()
    codes_pin = torch.zeros(B, 16, dtype=torch.int32).pin_memory()
    text_h, codes_h = text_pin.numpy(), codes_pin.numpy()
    barrier()
    e0.record(st)
    for _ in range(K):
        eng.frame_host(text_h, codes_h)
    e1.record(st)
    torch.cuda.synchronize()
    ms_e2e = max_over_ranks(e0.elapsed_time(e1))
    e2e = {"value": frames / (ms_e2e / 1000.0), "unit": "frames/s",
           "h2d_bytes_per_step": int(B * cfg.t_hidden * 4), "d2h_bytes_per_step": int(B * 16 * 4)}
    del eng
    torch.cuda.synchronize()

    # ---- batch 32 (same positions), then batch 1 and 32 at config 4's mean
    # cache position (1000 frames after a 64-token prefill: ~564)
    b32, c4 = None, None
    if not args.no_batch32:
        K32 = max(10, min(K, 60))
        eng32, text32, codes32 = engine_rate(E, talker, pred, torch, qb, 32, K32, W,
                                             ranks.stream_seed(50000, 32, 0))
        ms32 = timed_frames(eng32, text32, codes32, K32)
        b32 = {"value": 32 * K32 * world / (ms32 / 1000.0), "unit": "frames/s", "steps": K32,
               "ms_per_step": ms32 / K32, "positions": [PREFILL + W, PREFILL + W + K32 - 1]}
        del eng32
        torch.cuda.synchronize()
        c4 = {"positions_from": 564}
        for bb, kk in ((1, K), (32, K32)):
            e4, t4, c4d = engine_rate(E, talker, pred, torch, qb, bb, kk, W,
                                      ranks.stream_seed(90000, bb, 0), prefill=564 - W)
            m4 = timed_frames(e4, t4, c4d, kk)
            c4[f"b{bb}"] = {"value": round(bb * kk * world / (m4 / 1000.0), 2), "unit": "frames/s",
                            "ms_per_step": round(m4 / kk, 4), "steps": kk}
            del e4
            torch.cuda.synchronize()
        c4["note"] = ("config 4's per-GPU step at its mean cache position (the cache is "
                      "prefilled to 564 - warm-up positions instead of decoding 500 frames)")

    if rank != 0:
        clk.__exit__(None, None, None)
        ranks.close()
        return

    # ---- roofline of the dominant kernel: at batch 1 the whole frame is one
    # k_frame launch (talker step + 15-code predictor + sampler), so its
    # launch duration is the CUDA-event time per frame measured above
    roof, gemv_stream = None, None
    if not args.no_roofline:
        pos_avg = PREFILL + W + 0.5 * K  # cache positions during the timed frames
        fb = frame_algorithmic_bytes(cfg, pos_avg)
        us = 1000.0 * ms / K
        achieved = fb / (us * 1e-6) / 1e9
        roof = {"bound": "hbm", "kernel": "k_frame (persistent frame kernel, batch 1)",
                "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_source": peak_src,
                "traffic": KFRAME_DRAM_BYTES,
                "traffic_source": "ncu capture of one launch on this workload (profiles/k_frame_b1_frame.md)",
                "launches_per_step": kernels, "us_per_launch": round(us, 2),
                "algorithmic_bytes_per_launch": round(fb),
                "bytes_model": "talker weights 796,262,400 + norms + KV read 229,376 B x (P+1) + "
                               "KV write + predictor weight passes (15 x per-pass weights x 0.5625 B)"}
        # the per-launch Q4 GEMV kernel over the talker weights, back to back
        byts, gms = gemv_stream_roofline(E, ctx, tw, torch)
        n_launch = 7 * len(tw.layers) + 1
        g_ach = byts / (gms / 1000.0) / 1e9
        gemv_stream = {"kernel": "k_gemv (talker Q4 GEMVs, batch 1, back-to-back launches)",
                       "achieved": round(g_ach, 1), "peak": peak, "unit": "GB/s",
                       "frac": round(g_ach / peak, 4),
                       "traffic": round(KGEMV_DRAM_PER_ALG_BYTE * byts / n_launch),
                       "traffic_source": "DRAM bytes per algorithmic byte of the ncu capture "
                                         "profiles/k_gemv_b1_2048x6144.md, scaled to the launch mix",
                       "launches": n_launch,
                       "us_per_launch": round(1000.0 * gms / n_launch, 2),
                       "algorithmic_bytes_per_launch": round(byts / n_launch)}

    sweep = None if args.no_sweep else gemv_sweep(E, ctx, torch, qb)

    cfg3 = cfg2 = cfg0 = None
    if world == 1 and not args.no_config3:
        cfg3 = config3_rate(E, ctx, tw, torch, qb, max(5, min(K, 20)), 3, 42, peak)
    if world == 1 and not args.no_sweep:
        cfg2 = [predictor_rate(E, ctx, qb, torch, hd, 64) for hd in (64, 128)]
        cfg0 = talker_step_rate(E, ctx, tw, torch, qb)
    dec = None
    if world == 1 and not args.no_decoder:
        dec = decoder_rate(ctx, torch, cpu_frames_n=None if args.no_cpu else 2)
    clk.__exit__(None, None, None)

    cpu = None
    if world == 1 and not args.no_cpu:
        model = oracle_model_from(tw, pw)
        fps, done, dt, cores = cpu_frames(model, 60, 1, budget_s=20.0)
        cpu = {"value": round(fps, 3), "unit": "frames/s", "cores": cores, "kind": "port",
               "sample": f"{done} frames (batch 1) after 1 warm-up frame and a 64-token prefill, "
                         f"oracle port of the reference AVX-512 GEMV + worker pool"}

    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "frames/s", "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": round(ms / K, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": round(value / REF_FRAMES_PER_S, 2), "dtype": "f32 (Q4 weights)",
        "data": "synthetic: random-init N(0,0.02) Q4 weights, N(0,1) prefill and text rows",
        "config": {"workload": "frame loop: talker step + 15-code predictor + top-k 50 sampling "
                               "(one persistent-kernel launch per batch-1 frame)",
                   "batch_per_gpu": B, "prefill_tokens": PREFILL, "talker_layers": cfg.t_layers,
                   "predictor_head_dim": cfg.p_head_dim, "parallelism": f"replicas x{world}",
                   "l2": "per-frame weight stream 0.95 GB > 126 MB L2, no flush",
                   "vs_baseline_ref": "README.md:280 0.35 s/frame (laptop CPU)",
                   "reference_arm": "one CPU process on rank 0 (the reference is a single-host "
                                    "CPU program); at N > 1 the arms' ratio compares N GPUs "
                                    "with that one process"},
        "e2e": {k: (round(v, 2) if isinstance(v, float) else v) for k, v in e2e.items()},
        "gpu_launches": int(kernels * K),
        "kernels_per_step": kernels,
        "roofline": roof,
        "gemv_stream": gemv_stream,
        "cpu_baseline": cpu,
        "clocks": clk.summary(),
        "batch32": b32,
        "config4_positions": c4,
        "config3": cfg3,
        "config2_predictor": cfg2,
        "config0_talker": cfg0,
        "decoder": dec,
        "gemv_sweep": sweep,
    }
    print(json.dumps(line), flush=True)
    ranks.close()


def profile_case_gemv():
    """ncu case: the isolated batch-1 Q4 GEMV on the talker gate/up shape
    (in 2048 x out 6144, 7.08 MB of Q4 weights).  24 weight copies (170 MB >
    126 MB L2) are swept twice without a graph; capture launches 25.. (second
    sweep), whose weights have left L2."""
    import torch
    import qora_b200 as qb
    from qora_b200 import engine as E
    torch.cuda.set_device(0)
    ctx = E.Context(0)
    w = qb.synth_q4(4242 + 2048 + 6144, 0.02, 2048, 6144)
    devs = [E.DeviceQ4(ctx, w) for _ in range(24)]
    x = torch.randn(1, 2048, device="cuda")
    y = torch.empty(1, 6144, device="cuda")
    for _ in range(2):
        for d in devs:
            d.gemv(x, y)
    torch.cuda.synchronize()
    ctx.check_device_error()
    print(json.dumps({"profile_case": "gemv", "launches": 2 * len(devs), "k": 2048, "n": 6144}))


def profile_case_frame_trace():
    """Per-op stamps of the persistent frame kernel (batch 1, 1.7B dims, 64-token
    prefill): one JSON line with the phase split of a frame.  Phases per op, on
    the SM running the op's first item: wait (previous op's signal -> this op's
    dependency met), input (input vector built), items (GEMV / attention /
    sampler work), signal (completion counter)."""
    import torch
    import qora_b200 as qb
    from qora_b200 import engine as E
    torch.cuda.set_device(0)
    cfg = qb.ModelConfig()
    ctx = E.Context(0)
    talker = E.Talker(ctx, qb.synth_talker(cfg), max_batch=1)
    pred = E.CodePredictor(ctx, qb.synth_predictor(cfg), max_batch=1)
    eng = E.Engine(talker, pred, 1, PREFILL + 16)
    x = qb.synth_normal(1000, 1.0, PREFILL * cfg.t_hidden).reshape(1, PREFILL, cfg.t_hidden)
    eng.prefill(x, [1000])
    text = torch.from_numpy(qb.synth_normal(77, 1.0, cfg.t_hidden).reshape(1, cfg.t_hidden)).cuda()
    codes = torch.zeros(1, 16, dtype=torch.int32, device="cuda")
    for _ in range(3):
        eng.frame(text, codes)
    eng.trace(True)
    for _ in range(2):
        eng.frame(text, codes)
    ops, st = eng.trace(False)
    ctx.check_device_error()
    st = st.astype(np.uint64)
    n = len(ops)
    ready0 = (~st[:, 0]).astype(np.int64)          # earliest input ready over SMs
    ready1, done, start = (st[:, k].astype(np.int64) for k in (1, 2, 3))
    t_begin = int(min(start.min(), ready0.min()))
    total = int(done.max() - t_begin)
    prev_done = np.r_[t_begin, done[:-1]]
    phases = {"gap": ready0 - prev_done,            # previous op done everywhere -> first input ready
              "spread": ready1 - ready0,            # first -> last SM with its input ready
              "work": done - ready1,                # last input ready -> last item done
              "slot_wait": st[:, 4].astype(np.int64) / 1.965,
              "compute": st[:, 5].astype(np.int64) / 1.965, "reduce": st[:, 6].astype(np.int64) / 1.965}
    # op labels in program order (frame.cu frame_build)
    layer = ["qkv", "attn", "o", "gate_up", "down"]
    labels = ["sample"]
    for tk in range(cfg.p_groups + 1):
        labels += ["p_proj"] + ["p_" + x for x in layer] * cfg.p_layers + (["p_head"] if tk else [])
    labels += ["t_" + x for x in layer] * cfg.t_layers + ["t_head"]
    assert len(labels) == n, (len(labels), n)
    labels = np.array(labels)
    by_label = {}
    for lb in dict.fromkeys(labels.tolist()):
        m = labels == lb
        by_label[lb] = {"ops": int(m.sum()),
                        **{k: round(float(v[m].mean()) / 1000.0, 3) for k, v in phases.items()}}
    t0 = n - 5 * cfg.t_layers - 1
    print(json.dumps({"profile_case": "frame_trace", "ops": n, "frame_us": round(total / 1000.0, 1),
                      "us_per_op": round(total / n / 1000.0, 3),
                      "talker_us": round(float(done[-1] - done[t0 - 1]) / 1000.0, 1),
                      "phase_share": {k: round(float(v.sum()) / total, 3) for k, v in phases.items()
                                      if k in ("gap", "spread", "work")},
                      "mean_us_by_op": by_label}))


def profile_case_batch_frame(B):
    """ncu case: one frame of B streams (1.7B dims, 64-token prefill, graph
    replay after 3 warm-up frames), bracketed by cudaProfilerStart/Stop so
    that `ncu --profile-from-start off` captures exactly that frame."""
    import torch
    import qora_b200 as qb
    from qora_b200 import engine as E
    torch.cuda.set_device(0)
    cfg = qb.ModelConfig()
    ctx = E.Context(0)
    talker = E.Talker(ctx, qb.synth_talker(cfg), max_batch=B)
    pred = E.CodePredictor(ctx, qb.synth_predictor(cfg), max_batch=B)
    eng, text, codes = engine_rate(E, talker, pred, torch, qb, B, 1, 3, 3000)
    torch.cuda.profiler.start()
    eng.frame(text, codes)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    ctx.check_device_error()
    print(json.dumps({"profile_case": "batch_frame", "batch": B,
                      "kernels_per_frame": eng.kernels_per_frame()}))


def profile_case_prefill(tokens=2048):
    """ncu case: one stream's config-3 prefill (1.7B dims, random-init Q4
    weights, `tokens` N(0,1) rows in 512-row chunks), after one untimed
    prefill of another stream, bracketed by cudaProfilerStart/Stop; prints
    its CUDA-event time as one JSON line."""
    import torch
    import qora_b200 as qb
    from qora_b200 import engine as E
    torch.cuda.set_device(0)
    cfg = qb.ModelConfig()
    ctx = E.Context(0)
    talker = E.Talker(ctx, qb.synth_talker(cfg), max_batch=1)
    kv = talker.new_kv(max_pos=tokens, streams=2)
    xs = [torch.from_numpy(qb.synth_normal(42 + s, 1.0, tokens * cfg.t_hidden)
                           .reshape(tokens, cfg.t_hidden)).cuda() for s in range(2)]
    talker.prefill_talker_raw_from(xs[0], kv, 0, kv_stream=0)
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.profiler.start()
    e0.record(st)
    talker.prefill_talker_raw_from(xs[1], kv, 0, kv_stream=1)
    e1.record(st)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    ctx.check_device_error()
    print(json.dumps({"profile_case": "prefill", "tokens": tokens,
                      "ms": round(e0.elapsed_time(e1), 3)}))


def profile_case_decoder(frames=DECODER_FRAMES):
    """ncu case: one decode_to_audio of `frames` frames at the 12 Hz tokenizer
    dims (as the bench's decoder leg), after one untimed decode, bracketed by
    cudaProfilerStart/Stop; prints its CUDA-event time as one JSON line."""
    import torch
    from qora_b200 import engine as E
    from qora_b200.decoder import DecoderDims, SpeechDecoder, synth_decoder
    torch.cuda.set_device(0)
    ctx = E.Context(0)
    d = DecoderDims()
    dec = SpeechDecoder(ctx, d, synth_decoder(d))
    codes = np.random.default_rng(5).integers(0, d.codebook_size, (d.num_quantizers, frames)).astype(np.int32)
    cd = torch.from_numpy(codes).cuda()
    out = torch.empty(frames * d.hop, dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream()
    dec.decode_device(cd, frames, out, stream=st)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.profiler.start()
    e0.record(st)
    n = dec.decode_device(cd, frames, out, stream=st)
    e1.record(st)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    ctx.check_device_error()
    print(json.dumps({"profile_case": "decoder", "frames": frames, "launches": n,
                      "ms": round(e0.elapsed_time(e1), 3)}))


def profile_case_attn_decode(streams=32, positions=4096, reps=8):
    """ncu case: the decode attention of one talker layer (16 q / 8 kv heads,
    head_dim 128) for `streams` streams over `positions` cached positions each
    (one-layer cache, 1.07 GB at 32 x 4096; K / V filled with N(0,1)), the
    kernel the config-3 step spends most of its time in.  Times `reps`
    launches after 3 warm-up launches (CUDA events) and prints one JSON line."""
    import ctypes as C
    import torch
    from qora_b200 import engine as E, _lib
    torch.cuda.set_device(0)
    ctx = E.Context(0)
    H, KV, HD = 16, 8, 128
    kv = E.KvCache(ctx, 1, KV, HD, positions, streams)
    kp, vp, lp = C.c_void_p(), C.c_void_p(), C.c_void_p()
    _lib.call("qora_kv_layer_ptrs", kv.h, 0, C.byref(kp), C.byref(vp), C.byref(lp))
    n = streams * KV * positions * HD
    for p in (kp, vp):
        E._device_view(p.value, (n,), "<f4").copy_(torch.randn(n, device="cuda"))
    E._device_view(lp.value, (streams,), "<i4").fill_(positions - 1)
    qkv = torch.randn(streams, (H + 2 * KV) * HD, device="cuda")
    gam = torch.from_numpy(np.full(HD, 0x3C00, np.uint16).view(np.int16)).cuda()
    cos, sin = E.build_mrope_tables(HD, positions + 1, 1e6, [24, 20, 20])
    cos, sin = torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()
    pos = torch.full((streams,), positions - 1, dtype=torch.int32, device="cuda")
    out = torch.empty(streams, H * HD, device="cuda")
    for _ in range(3):
        kv.attend(0, qkv, H, gam, gam, cos, sin, pos, out=out)
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        kv.attend(0, qkv, H, gam, gam, cos, sin, pos, out=out)
    e1.record(st)
    torch.cuda.synchronize()
    ctx.check_device_error()
    us = 1000.0 * e0.elapsed_time(e1) / reps
    byts = streams * KV * positions * HD * 4 * 2
    print(json.dumps({"profile_case": "attn_decode", "streams": streams, "positions": positions,
                      "us_per_launch": round(us, 2), "kv_bytes": byts,
                      "GB/s": round(byts / (us * 1e-6) / 1e9, 1)}))


def main():
    args = parse()
    if args.profile_case == "decoder":
        profile_case_decoder(args.frames or DECODER_FRAMES)
        return
    if args.profile_case == "prefill":
        profile_case_prefill()
        return
    if args.profile_case == "attn_decode":
        profile_case_attn_decode()
        return
    if args.profile_case == "gemv":
        profile_case_gemv()
        return
    if args.profile_case == "batch_frame":
        profile_case_batch_frame(args.batch)
        return
    if args.profile_case == "frame_trace":
        profile_case_frame_trace()
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
