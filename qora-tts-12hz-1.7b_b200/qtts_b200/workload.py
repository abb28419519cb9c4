"""Seeded synthetic inputs for the benchmark configs (no datasets, no
checkpoints: weights are the seeded synthetic .qora-tts, inputs are seeded
token ids and speaker embeddings with the configs' shapes).

config 1: 32 prompt ids ~U[0, 151936), a 2048-d N(0,1) L2-normalised voice
          embedding, language 2050, greedy (T=1, top_k=1), rep 1.05, 100 frames
config 3: 96 prompt ids, T=0.8, top_k=50, rng seed 42, 2000 frames
config 4: 64 utterances, prompt lengths ~U[16, 256], own voice and seed each,
          T=0.8, top_k=50, 500 frames
config 5: 512 utterances from the config-4 generator, 64 per GPU
decoder:  16 code streams of T frames ~U[0, 2048) (the speech decoder's
          first stage; T = 500, an utterance of config 4/5)
"""
from __future__ import annotations

import os

import numpy as np

from . import Dims, dims_1p7b, dims_tiny, file_probe, make_params, synth_write, synth_write_with_decoder

TEXT_VOCAB = 151936
LANG_ENGLISH = 2050  # config.json codec_language_id.english
MODEL_DIR = os.environ.get("QTTS_MODEL_DIR", "/tmp/qtts_models")


def model_path(kind: str = "1p7b", seed: int = 0) -> str:
    """Path of the seeded synthetic model, written on first use: "1p7b",
    "tiny", or "decoder" (the tiny talker/predictor with a full-size speech
    decoder section)."""
    os.makedirs(MODEL_DIR, exist_ok=True)
    path = os.path.join(MODEL_DIR, f"qtts_{kind}_seed{seed}.qora-tts")
    if not os.path.exists(path):
        d: Dims = dims_1p7b() if kind == "1p7b" else dims_tiny()
        tmp = path + f".tmp{os.getpid()}"
        if kind == "decoder":
            synth_write_with_decoder(tmp, d, seed)
        else:
            synth_write(tmp, d, seed)
        os.replace(tmp, path)
    file_probe(path)
    return path


def voice_embedding(seed: int, dim: int = 2048) -> np.ndarray:
    v = np.random.default_rng(seed).standard_normal(dim)
    return (v / np.linalg.norm(v)).astype(np.float32)


def tokens(seed: int, n: int) -> np.ndarray:
    return np.random.default_rng(seed).integers(0, TEXT_VOCAB, size=n, dtype=np.int64).astype(np.uint32)


def config1(hidden: int = 2048):
    return dict(text=tokens(101, 32), voice=voice_embedding(102, hidden), language_id=LANG_ENGLISH,
                speaker_id=0, seed=1, params=make_params(1.0, 1, 1.05)), 100


def config3(hidden: int = 2048):
    return dict(text=tokens(301, 96), voice=voice_embedding(302, hidden), language_id=LANG_ENGLISH,
                speaker_id=0, seed=42, params=make_params(0.8, 50, 1.05)), 2000


def config4(n_utt: int = 64, hidden: int = 2048, base_seed: int = 400):
    rng = np.random.default_rng(base_seed)
    lens = rng.integers(16, 257, size=n_utt)
    utts = []
    for i in range(n_utt):
        utts.append(dict(text=tokens(base_seed * 1000 + i, int(lens[i])),
                         voice=voice_embedding(base_seed * 1000 + 500 + i, hidden),
                         language_id=LANG_ENGLISH, speaker_id=0, seed=1000 + i,
                         params=make_params(0.8, 50, 1.05)))
    return utts, 500


def config5_shard(rank: int, world: int, total: int = 512, hidden: int = 2048):
    """Contiguous block of the 512 config-5 utterances owned by `rank`."""
    utts, frames = config4(total, hidden)
    per = (total + world - 1) // world
    return utts[rank * per:(rank + 1) * per], frames


def decoder_codes(T: int, seed: int = 700) -> np.ndarray:
    """16 code streams of T frames, uniform over the 2048-entry codebooks."""
    return np.random.default_rng(seed).integers(0, 2048, size=(16, T), dtype=np.int64).astype(np.uint32)
