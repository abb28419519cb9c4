"""Regenerate the golden fixtures under tests/golden/ from the CPU oracle.

The reference crate cannot be built in this image and ships no golden
vectors for the decode loop, so these fixtures come from the oracle
(oracle/qtts_oracle.c, a line-by-line restatement of the Rust source) run on
the seeded synthetic weights.  They pin the GPU path to the oracle and the
oracle to itself across machines (parity with the Rust crate stays
unpinned).  Weights are identified by the sha256 of the synthetic file.

    python tests/golden/make_golden.py [--skip-1p7b] [--only NAME[,NAME...]]

--only regenerates just the named fixtures (tiny_long_kv, p1p7b_config3_2000,
p1p7b_config4_64); the long 1.7B cases take tens of minutes on 8 cores.

The oracle uses 8 K-split chunks for the large talker GEMVs (the reference's
threading policy, gemv.rs:268-309, on an 8-thread host).
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys
import time

import numpy as np

REPO = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "qora-tts-12hz-1.7b_b200"))

from oracle import oracle as O  # noqa: E402
from qtts_b200 import make_params as QP  # noqa: E402
from qtts_b200 import workload as W  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))
THREADS = 8


def sha256(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for blk in iter(lambda: f.read(1 << 24), b""):
            h.update(blk)
    return h.hexdigest()


def oracle_model(kind):
    path = os.path.join(W.MODEL_DIR, f"qtts_{kind}_seed0.oracle.qora-tts")
    os.makedirs(W.MODEL_DIR, exist_ok=True)
    if not os.path.exists(path):
        O.synth_write(path, O.dims_1p7b() if kind == "1p7b" else O.dims_tiny(), 0)
    return path


def topk(lg, k=5):
    idx = np.argsort(-lg, axis=-1, kind="stable")[..., :k]
    return idx.astype(np.int32), np.take_along_axis(lg, idx, axis=-1)


def run_case(m, utt, frames, keep_frames=None):
    p = O.make_params(frames, float(utt["params"].temperature), int(utt["params"].top_k),
                      float(utt["params"].repetition_penalty))
    t0 = time.time()
    n, codes, lg, hid = m.generate(utt["text"], p, utt["seed"], speaker_id=utt.get("speaker_id", 0),
                                   language_id=utt.get("language_id", 2050), voice=utt.get("voice"),
                                   ignore_eos=True, dump_logits=True, dump_hidden=True)
    dt = time.time() - t0
    ti, tv = topk(lg)
    out = dict(codes=codes, frames=np.int32(n), top_idx=ti, top_val=tv,
               absmax=np.abs(lg).max(axis=1).astype(np.float32), seconds=np.float64(dt))
    if keep_frames is None:
        out["logits"] = lg
        out["hidden"] = hid
        out["logit_frames"] = np.arange(frames, dtype=np.int32)
    else:
        kf = np.array(keep_frames, np.int32)
        out["logits"] = lg[kf]
        out["hidden"] = hid[kf]
        out["logit_frames"] = kf
    return out


def sampler_kats():
    rng = np.random.default_rng(7)
    cases = []
    for i in range(32):
        V = 3072
        lg = (rng.standard_normal(V) * 4).astype(np.float32)
        if i % 8 == 1:  # exact ties in the logits
            lg[rng.integers(0, V, 40)] = lg.max()
        if i % 8 == 2:  # coarse values -> many equal probabilities
            lg = np.round(lg).astype(np.float32)
        T, k = [(1.0, 1), (0.8, 50), (0.9, 50), (1.0, 0), (0.7, 3071), (1.3, 5), (0.8, 1), (1.0, 3072)][i % 8]
        prev = rng.integers(0, V, 16).astype(np.uint32)
        if i % 4 == 3:
            prev[:] = prev[0]  # duplicates are penalised repeatedly
        state = int(rng.integers(1, 2**63))
        p = O.make_params(1, T, k, 1.05)
        tok, st2 = O.sample_token(lg, p, prev, state)
        cases.append((lg, T, k, prev, state, tok, st2))
    return dict(logits=np.stack([c[0] for c in cases]), temperature=np.array([c[1] for c in cases], np.float32),
                top_k=np.array([c[2] for c in cases], np.int32), prev=np.stack([c[3] for c in cases]),
                state=np.array([c[4] for c in cases], np.uint64), token=np.array([c[5] for c in cases], np.uint32),
                state_out=np.array([c[6] for c in cases], np.uint64))


def tiny_long_kv(m):
    """Tiny model, config-3 sampling (T=0.8, top-k 50, seed 42), 2000 frames:
    the talker attention runs over ~2010 cached positions (talker.rs:305-331)."""
    u3, frames = W.config3(m.dims.t_hidden)
    return run_case(m, u3, frames, keep_frames=[0, 1, 999, 1500, frames - 1])


def p1p7b_config3_2000(m):
    """1.7B, benchmark config 3 in full: 96-token prompt, T=0.8 / top-k 50 /
    seed 42, 2000 frames (KV to ~2010 positions)."""
    u3, frames = W.config3(2048)
    return run_case(m, u3, frames, keep_frames=[0, 999, frames - 1])


def p1p7b_config4_64(m, frames=3):
    """1.7B, benchmark config 4's 64 utterances (ragged 16-256-token prompts,
    own voice and seed each, T=0.8 / top-k 50), `frames` frames each, one
    oracle run per utterance; stacked along a leading utterance axis."""
    utts, _ = W.config4(64, 2048)
    runs = [run_case(m, u, frames, keep_frames=[0, frames - 1]) for u in utts]
    out = {k: np.stack([r[k] for r in runs]) for k in runs[0] if k != "seconds"}
    out["seconds"] = np.float64(sum(float(r["seconds"]) for r in runs))
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--skip-1p7b", action="store_true")
    ap.add_argument("--only", default="", help="comma-separated fixture names")
    args = ap.parse_args()
    if args.only:
        O.set_threads(THREADS)
        only = set(args.only.split(","))
        if "tiny_long_kv" in only:
            m = O.Model(oracle_model("tiny"))
            r = tiny_long_kv(m)
            np.savez_compressed(os.path.join(OUT, "tiny_long_kv.npz"), **r)
            print("tiny_long_kv frames", int(r["frames"]), "s", float(r["seconds"]), flush=True)
            m.close()
        big = [n for n in ("p1p7b_config3_2000", "p1p7b_config4_64") if n in only]
        if big:
            m = O.Model(oracle_model("1p7b"))
            for name in big:
                r = globals()[name](m)
                np.savez_compressed(os.path.join(OUT, f"{name}.npz"), **r)
                print(name, "s", float(r["seconds"]), flush=True)
            m.close()
        return
    meta_path = os.path.join(OUT, "meta.npz")
    old_meta = dict(np.load(meta_path)) if os.path.exists(meta_path) else {}
    O.set_threads(THREADS)
    np.savez_compressed(os.path.join(OUT, "sampler_kats.npz"), **sampler_kats())

    tiny = oracle_model("tiny")
    m = O.Model(tiny)
    H = m.dims.t_hidden
    u1, _ = W.config1(H)
    cases = {"tiny_greedy": (u1, 24)}
    u3, _ = W.config3(H)
    cases["tiny_sampled"] = (u3, 24)
    nv = dict(text=W.tokens(11, 7), voice=None, speaker_id=3001, language_id=2055, seed=9,
              params=QP(0.9, 20, 1.05))
    cases["tiny_speaker"] = (nv, 12)
    et = dict(text=np.zeros(0, np.uint32), voice=W.voice_embedding(5, H), seed=3, params=QP(1.0, 1, 1.05))
    cases["tiny_notext"] = (et, 8)
    meta = dict(old_meta)
    meta.update(threads=np.int32(THREADS), tiny_sha256=np.array(sha256(tiny)))
    for name, (u, f) in cases.items():
        r = run_case(m, u, f, keep_frames=sorted({0, 1, 2, f // 2, f - 1}))
        np.savez_compressed(os.path.join(OUT, f"{name}.npz"), **r)
        print(name, "frames", int(r["frames"]), "s", float(r["seconds"]), flush=True)
    m.close()

    if not args.skip_1p7b:
        big = oracle_model("1p7b")
        meta["p1p7b_sha256"] = np.array(sha256(big))
        m = O.Model(big)
        u1, f1 = W.config1(2048)
        r = run_case(m, u1, f1, keep_frames=[0, 1, 50, 99])
        np.savez_compressed(os.path.join(OUT, "p1p7b_config1.npz"), **r)
        print("1p7b config1", int(r["frames"]), "s", float(r["seconds"]), flush=True)
        u3, _ = W.config3(2048)
        r = run_case(m, u3, 24, keep_frames=[0, 23])
        np.savez_compressed(os.path.join(OUT, "p1p7b_config3_24f.npz"), **r)
        print("1p7b config3 24f", int(r["frames"]), "s", float(r["seconds"]), flush=True)
        m.close()
    np.savez(meta_path, **meta)


if __name__ == "__main__":
    main()
