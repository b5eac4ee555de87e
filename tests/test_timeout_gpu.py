"""A bounded device wait that runs out is reported, not hung on: with the
test knob IQ_QMV_TEST_TIMEOUT one warp's first weight copy is never
requested, its slot wait gives up after a short bound, the warp drains its
other copies and stops, and the pass fails with IQ_ETIMEDOUT (-6) on the
host.  No GPU fault, trap or hang is involved: the wait is on a barrier that
nothing completes, and every copy that was started lands before the CTA
exits.  Runs in a child process so the knob does not leak into other tests."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

CHILD = r"""
import numpy as np
from inferq_b200 import synth
from inferq_b200._lib import IqError
from inferq_b200.model import Model, State
cfg = synth.tiny()
m = Model(cfg, list(synth.generate(cfg, seed=1)))
st = State(m, 64)
try:
    st.forward([1, 2, 3])
    print("NO-ERROR")
except IqError as e:
    print("ERROR", e.code, e)
"""


def test_gemv_wait_timeout_reaches_the_host(cuda):
    env = dict(os.environ, IQ_QMV_TEST_TIMEOUT="1")
    r = subprocess.run([sys.executable, "-c", CHILD], env=env, capture_output=True, text=True, timeout=300,
                       cwd=os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    assert r.returncode == 0, r.stderr[-2000:]
    line = [l for l in r.stdout.splitlines() if l.startswith(("ERROR", "NO-ERROR"))][-1]
    assert line.startswith("ERROR -6"), line
    assert "gave up" in line


WIDE_CHILD = r"""
import numpy as np
import torch
from inferq_b200 import _lib
from inferq_b200 import quants as Q
w = Q.encode(torch.randn(256, 512) * 0.02, Q.Q8_0).numpy()
m = _lib.Matrix(Q.Q8_0, w, 256, 512)
m.forward_wide(torch.randn(64, 512, device="cuda"))
try:
    _lib.status()
    print("NO-ERROR")
except _lib.IqError as e:
    print("ERROR", e.code, e)
_lib.status()  # the record was cleared by the first check
print("CLEARED")
"""


def test_wide_product_wait_timeout_reaches_the_host(cuda):
    """IQ_WIDE_TEST_TIMEOUT: the MMA thread skips the first stage, the
    epilogue's first TMEM-buffer wait runs out, every role winds down (TMA
    copies and MMAs drained, TMEM freed) and iq_matrix_status reports
    IQ_ETIMEDOUT; the context stays usable."""
    env = dict(os.environ, IQ_WIDE_TEST_TIMEOUT="1")
    r = subprocess.run([sys.executable, "-c", WIDE_CHILD], env=env, capture_output=True, text=True, timeout=300,
                       cwd=os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith(("ERROR", "NO-ERROR", "CLEARED"))]
    assert lines[0].startswith("ERROR -6") and "gave up" in lines[0], lines
    assert lines[-1] == "CLEARED"
