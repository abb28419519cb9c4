"""The opt-in staged decode GEMV (QTTS_STAGED=1: the CTA's weight slice in
shared memory, gemv.cu gemv_dec_kernel<..., STG = true>) on the 1.7B config-1
fixture.  With the global split-K plan off (QTTS_GLOBAL_SPLIT=0) the
talker's gate/up pair is the projection it takes over; the planner log must
show it, and the teacher-forced codes and logits must match
the oracle as on the default path.  The environment switch is read once per
process, so the run is a child process."""
import os
import subprocess
import sys

import pytest

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

HERE = os.path.dirname(os.path.abspath(__file__))

CHILD = r"""
import sys
sys.path.insert(0, {tests!r})
from conftest import golden
import qtts_b200 as Q
from qtts_b200 import workload as W
from test_gpu_model import _check_forced
m = Q.Model(W.model_path("1p7b"), 0)
g = golden("p1p7b_config1")
u, F = W.config1(2048)
s = Q.Session(m, 1, 10 + F)
codes, frames, lg, _ = Q.generate(s, [u], F, forced=g["codes"][None], dump_logits=True)
assert frames[0] == F
_check_forced(codes[0], g, lg[0], max_ties=1)
s.close()
print("staged decode parity ok")
"""


def test_staged_decode_gemv_1p7b_config1():
    env = dict(os.environ, QTTS_STAGED="1", QTTS_GLOBAL_SPLIT="0", QTTS_PLAN_LOG="1")
    r = subprocess.run([sys.executable, "-c", CHILD.format(tests=HERE)], env=env, capture_output=True, text=True,
                       timeout=900, cwd=os.path.dirname(HERE))
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "parity ok" in r.stdout
    assert "cuda-core staged" in r.stderr, "no projection took the staged kernel"
