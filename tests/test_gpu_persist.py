"""The opt-in persistent code predictor (QTTS_PERSIST=1, pred_persist.cu)
against the oracle fixtures: the environment switch is read once per process,
so the checks run in a child process."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))

CHILD = r"""
import sys
sys.path.insert(0, {tests!r})
import numpy as np
from conftest import golden
import qtts_b200 as Q
from qtts_b200 import workload as W
from test_gpu_model import tiny_case, _check_forced
m = Q.Model(W.model_path("tiny"), 0)
for case in ["tiny_greedy", "tiny_sampled", "tiny_notext"]:
    g = golden(case)
    F = g["codes"].shape[0]
    s = Q.Session(m, 1, 10 + F)
    codes, frames, lg, _ = Q.generate(s, [tiny_case(case, m.dims.t_hidden)], F, forced=g["codes"][None],
                                      dump_logits=True)
    _check_forced(codes[0], g, lg[0])
    s.close()
print("persistent predictor parity ok")
"""


def test_persistent_predictor_teacher_forced_tiny():
    env = dict(os.environ, QTTS_PERSIST="1")
    r = subprocess.run([sys.executable, "-c", CHILD.format(tests=HERE)], env=env, capture_output=True, text=True,
                       timeout=600, cwd=os.path.dirname(HERE))
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "parity ok" in r.stdout
