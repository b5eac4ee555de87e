"""One host thread driving matrices on two GPUs in turn: the operator entry
points keep their scratch per device, so each GPU's kernels only ever see
that GPU's memory (narrow GEMV through host buffers, and the wide product)."""
import numpy as np
import pytest
import torch

import oracle
from inferq_b200 import _lib
from inferq_b200 import quants as Q

pytestmark = pytest.mark.gpu


def test_one_thread_alternates_between_two_gpus(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    rows, cols = 384, 1024
    g = torch.Generator().manual_seed(12)
    w = Q.encode(torch.randn(rows, cols, generator=g) * 0.02, Q.Q8_0).numpy()
    mats = []
    for dev in (0, 1):
        torch.cuda.set_device(dev)
        mats.append(_lib.Matrix(Q.Q8_0, w, rows, cols))
    x = np.random.default_rng(3).standard_normal((5, cols)).astype(np.float32)
    want = oracle.qmatvec(Q.Q8_0, w, rows, cols, x, order=1, ksplit=_lib.ksplit(Q.Q8_0, rows, cols))
    xw = np.random.default_rng(4).standard_normal((70, cols)).astype(np.float32)
    want_wide = oracle.qmatvec(Q.Q8_0, w, rows, cols, xw, order=1, ksplit=1)
    try:
        for _ in range(3):
            for dev in (0, 1):
                torch.cuda.set_device(dev)
                y = mats[dev].forward_rows(x)
                assert np.array_equal(y.view(np.uint32), want.view(np.uint32)), dev
                yw = mats[dev].forward_wide(torch.from_numpy(xw).cuda(dev)).cpu().numpy()
                assert np.array_equal(yw.view(np.uint32), want_wide.view(np.uint32)), dev
                _lib.status()
    finally:
        torch.cuda.set_device(0)
