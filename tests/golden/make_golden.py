"""Writes the committed golden fixtures (tests/golden/*.npz) from the CPU oracle.

The reference is a Rust crate and no Rust toolchain exists in this image, so
it cannot be run to produce vectors.  Its own tests for this path hold no
stored outputs either: they are differential (gemv.rs:735-861 compares the
AVX2 kernel with the scalar one on xorshift-generated inputs).  The pin is
therefore: (1) those differential known-answer tests, restated against the
oracle in tests/test_oracle_kat.py, and (2) these fixtures, produced by the
pinned oracle on the reference's own generators (gemv.rs:693-730) and on the
seeded synthetic model, so every later run of the oracle and of the CUDA
engine is compared against fixed numbers rather than against a moving
restatement.

Run from the repository root:  python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import pyoracle as po  # noqa: E402

# gemv.rs:758-773 (shapes, seeds, zero fractions) and gemv.rs:846-861 (tail n)
GEMV_CASES = [
    ("shapes_64x2048", 64, 2048, 1, 0.0, 0.0),
    ("shapes_64x6144", 64, 6144, 2, 0.0, 0.0),
    ("shapes_32x1024", 32, 1024, 3, 0.0, 0.0),
    ("shapes_16x256", 16, 256, 4, 0.0, 0.0),
    ("shapes_1x32", 1, 32, 5, 0.0, 0.0),
    ("sparse_48x1024", 48, 1024, 11, 0.3, 0.2),
    ("sparse_32x2048", 32, 2048, 12, 0.5, 0.5),
    ("tail_16x100", 16, 100, 31, 0.0, 0.0),
]


def gemv_cases():
    out = {}
    for name, k, n, seed, iz, sz in GEMV_CASES:
        r = po.XRng(seed)
        groups = n // 32
        packed = r.bytes(k * groups * 16)
        scales = r.scales(k * groups, sz)
        x = r.inputs(k, iz)
        y = po.gemv_scalar(x, packed, scales, n, 0, k)
        # inputs are regenerated from the restated xorshift generators; their
        # checksums pin those generators
        out[f"{name}/input_sums"] = np.array(
            [int(packed.astype(np.uint64).sum()), int(scales.astype(np.uint64).sum()),
             int(x.view(np.uint32).astype(np.uint64).sum())], np.uint64)
        out[f"{name}/y"] = y
        out[f"{name}/kn"] = np.array([k, n], np.int64)
    return out


def quantiser_case():
    data = po.synth_normal(99, 0.02, 8 * 64).reshape(8, 64)
    data[0, :32] = 0.0                      # all-zero group: scale 0, nibbles 8
    data[1, 5] = 0.5                        # one large value dominating a group
    w = po.quantize(data)
    return {"quant/data": data, "quant/packed": w.packed, "quant/scales": w.scales}


def rope_case():
    cos, sin = po.rope_tables(128, 40, 1e6, [24, 20, 20])
    c64, s64 = po.rope_tables(64, 20, 1e6)
    return {"rope/hd128_cos": cos, "rope/hd128_sin": sin, "rope/hd64_cos": c64, "rope/hd64_sin": s64}


def sampler_case():
    logits = po.synth_normal(5, 3.0, 4 * 3072).reshape(4, 3072).astype(np.float32)
    logits[1, 100:160] = 7.5                # a block of exact ties inside the top-k
    prev = np.array([17, 100, 2150, 5, 5, 9, 3000, 42, 0, 1, 2, 3, 4, 6, 7, 8], np.uint32)
    params = po.SampleParams(0.9, 50, 1.0, 1.05)
    toks, states = [], []
    for r in range(4):
        st = 1000 + r
        row = []
        for _ in range(8):
            t, st = po.sample_token(logits[r], params, prev, st)
            row.append(t)
        toks.append(row)
        states.append(st)
    return {"sample/logits": logits, "sample/prev": prev,
            "sample/tokens": np.array(toks, np.uint32),
            "sample/final_rng": np.array(states, np.uint64),
            "sample/seeds": np.arange(1000, 1004, dtype=np.uint64)}


def tiny_model_case():
    """Tiny-config talker prefill + steps, one predictor frame (oracle weights
    come from the shared splitmix64 generator, so the engine builds the same
    model from ModelConfig.tiny())."""
    cfg = po.ModelConfig.tiny()
    om = po.OracleModel(po.Model.synth(cfg))
    T = 3
    x = po.synth_normal(1, 1.0, T * cfg.t_hidden).reshape(T, cfg.t_hidden)
    kv = om.talker_kv()
    h0 = om.talker_prefill(x, kv, 0)
    embs, hid, logit = [], [], []
    for s in range(4):
        e = po.synth_normal(2 + s, 1.0, cfg.t_hidden)
        h, lg = om.talker_step(e, kv, T + s)
        embs.append(e)
        hid.append(h)
        logit.append(lg)
    sem = om.embed_codec(int(np.argmax(logit[-1])))
    codes, plog = om.predictor_frame(hid[-1], sem, om.predictor_kv())
    return {"tiny/prefill_x": x, "tiny/prefill_hidden": h0, "tiny/step_emb": np.stack(embs),
            "tiny/step_hidden": np.stack(hid), "tiny/step_logits": np.stack(logit),
            "tiny/pred_sem": sem, "tiny/pred_codes": np.asarray(codes, np.uint32),
            "tiny/pred_logits": np.asarray(plog, np.float32)}


def main():
    po.build()
    fixtures = {}
    for part in (gemv_cases, quantiser_case, rope_case, sampler_case, tiny_model_case):
        fixtures.update(part())
    path = os.path.join(HERE, "golden.npz")
    np.savez_compressed(path, **fixtures)
    print(f"wrote {path}: {len(fixtures)} arrays, {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()
