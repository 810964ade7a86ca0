"""The multi-GPU host logic of bench.py (one process per GPU, replicas only),
run as two gloo ranks on the CPU: the timing barrier, the max over ranks of
each rank's duration, the whole-job rate, per-rank stream seeds, rank-0-only
output, and the reference arm, which only rank 0 runs."""
import json
import os
import socket
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    sys.path.insert(0, ROOT)
    import bench
    r = bench.Ranks("gloo", timeout_s=60)
    r.barrier()
    ms = 10.0 + 5.0 * rank             # each rank's own device time
    ms_max = r.max(ms)
    res = {"rank": r.rank, "world": r.world, "ms_max": ms_max,
           "rate": bench.aggregate_rate(100, r.world, ms_max),
           "seeds": [r.stream_seed(1000, 4, b) for b in range(4)]}
    with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
        json.dump(res, f)
    r.close()


def test_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp
    port = _free_port()
    mp.spawn(_rank_main, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    res = [json.load(open(tmp_path / f"rank{i}.json")) for i in range(2)]
    for i, r in enumerate(res):
        assert r["rank"] == i and r["world"] == 2
        assert r["ms_max"] == 15.0                      # the slower rank's time, on every rank
        assert r["rate"] == pytest.approx(100 * 2 / 0.015)
    seeds = res[0]["seeds"] + res[1]["seeds"]
    assert len(set(seeds)) == 8                         # every stream of the job distinct


def test_single_process_needs_no_process_group(monkeypatch):
    sys.path.insert(0, ROOT)
    import bench
    monkeypatch.delenv("WORLD_SIZE", raising=False)
    r = bench.Ranks("gloo")
    assert r.world == 1 and r.dist is None and r.max(3.0) == 3.0
    r.barrier()
    r.close()


def test_reference_arm_runs_on_rank_zero_only():
    """Under torchrun every rank runs `bench.py --impl reference`; ranks other
    than 0 exit 0 at once, without work or output."""
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    p = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                        "--gpus", "2", "--steps", "1", "--warmup", "3"],
                       env=env, capture_output=True, text=True, timeout=120)
    assert p.returncode == 0, p.stderr
    assert p.stdout.strip() == ""


def test_algorithmic_bytes_model_matches_the_published_figures():
    """The roofline's per-unit figures (1.7B dims): talker step weights
    796,262,400 B (28 x 50,331,648 + 6,291,456 codec-head weights at
    0.5625 B), predictor weight passes 698,941,440 B (15 passes, head_dim
    128), 229,376 B of K/V per cached position."""
    sys.path.insert(0, ROOT)
    import bench
    import qora_b200
    cfg = qora_b200.ModelConfig()
    q4 = 0.5625
    talker_w = 28 * 50_331_648 + 6_291_456
    assert q4 * talker_w == 796_262_400
    kv_pos = cfg.t_layers * 2 * cfg.t_kv_heads * cfg.t_head_dim * 4
    assert kv_pos == 229_376
    norms = 2 * (cfg.t_layers * (2 * cfg.t_hidden + 2 * cfg.t_head_dim) + cfg.t_hidden)
    for P in (0, 64, 300):
        total = bench.frame_algorithmic_bytes(cfg, P)
        pred = total - (796_262_400 + norms + kv_pos * (P + 1) + kv_pos + 1152)
        assert pred == 698_941_440, (P, pred)
    assert bench.aggregate_rate(400, 8, 1000.0) == 3200.0
