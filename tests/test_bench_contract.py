"""bench.py on the CPU: the module imports (every name its GPU path uses at
import time exists), the config-5 schedule defaults, the timed window and the
wave split.  Nothing here launches a GPU kernel."""
import importlib.util
import os

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(REPO, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_imports_and_constants(bench):
    assert bench.METRIC == "codec frames/sec"
    assert bench.WAVE == 64  # config 4: 64 concurrent utterances
    assert (bench.WAVE5, bench.LANES5) == (256, 2)
    assert bench.UTT_FRAMES["config5"] == 500
    assert 7.0 <= bench.TC_TRAFFIC_RATIO < 8.5  # expanded tiles: ~4 / 0.5625 B per weight
    assert callable(bench.roofline_tc) and callable(bench.roofline_dec) and callable(bench.frame_roofline)


def test_timed_window_is_centred(bench):
    # 20 timed frames of 500-frame utterances start at frame 240 (KV ~260)
    assert bench.timed_window("config5", 20, 5) == 240
    assert bench.timed_window("config5", 600, 5) == 5  # longer than the utterance: right after warm-up
    assert bench.timed_window("config1", 50, 5) == 25


def test_waves_split_utterances(bench):
    # the wave split of Waves.__init__: contiguous blocks of up to `wave`
    utts = list(range(512))
    waves = [utts[i:i + bench.WAVE5] for i in range(0, len(utts), bench.WAVE5)]
    assert [len(w) for w in waves] == [256, 256]
    assert sum(waves, []) == utts


def test_roofline_tc_overlap_fields(bench):
    ft = {"ms": 10.0, "flops": 1e12, "launches": 400, "weight_bytes": 4e9}
    r = bench.roofline_tc(ft, {"bf16_tflops_sustained": 1400.0}, 20.0, 2, 256)
    assert r["bound"] == "tensor" and r["unit"] == "TFLOP/s"
    assert abs(r["achieved"] - 100.0) < 1e-9  # 1e12 FLOP in 10 ms
    assert abs(r["overlapped"]["lanes_overlap"] - 1.0) < 1e-9  # 2 waves x 10 ms over a 20 ms step
    assert r["traffic"] == pytest.approx(bench.TC_TRAFFIC_RATIO * 4e9 / 400)


def test_decoder_launch_count(bench):
    # CUDA cores below 16 frames: 79 kernels; tensor cores from 16 frames,
    # with one row-split kernel (the input projection's) above 64 frames
    assert bench.decoder_launches(5) == 79
    assert bench.decoder_launches(40) == 72
    assert bench.decoder_launches(500) == 73
