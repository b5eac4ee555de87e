"""The algorithmic byte counts behind the bench line's roofline figures,
checked against the figures the path's scope fixes for the 35B shapes
(Q4_K_M mix): per expert 2,039,808 B; a verify pass at ctx 1024 of about
2.42 GB at k=1 with 8 experts per layer, 3.54 GB at k=4 with 21.7 and
4.38 GB with all 32 (every weight byte read once, KV and DeltaNet state
included).  CPU only: the counts are arithmetic over the configuration."""
import numpy as np
import pytest

import bench
from inferq_b200 import quants as Q
from inferq_b200 import synth


@pytest.fixture(scope="module")
def cfg():
    return synth.qwen36_35b()


def test_expert_bytes(cfg):
    H, F = cfg.hidden_size, cfg.moe_intermediate_size
    per_expert = (F * Q.row_bytes(cfg.dtype("exp_gate"), H) + F * Q.row_bytes(cfg.dtype("exp_up"), H) +
                  H * Q.row_bytes(cfg.dtype("exp_down"), F))
    assert per_expert == 2_039_808


@pytest.mark.parametrize("k,union,gb", [(1, 8, 2.42), (4, 21.7, 3.54), (4, 32, 4.38)])
def test_pass_bytes(cfg, k, union, gb):
    u = np.full(cfg.num_hidden_layers, union)
    total = bench.pass_bytes(cfg, u, 1024, k)
    assert abs(total / 1e9 - gb) <= 0.01 * gb, total
    # the GEMV's share (weights only) is the pass minus state, KV, router and embedding rows
    g = bench.gemv_bytes(cfg, u, k)
    assert 0.85 * total < g < total


def test_gemv_bytes_grow_by_one_expert_per_layer_and_union(cfg):
    L = cfg.num_hidden_layers
    a = bench.gemv_bytes(cfg, np.full(L, 10.0), 4)
    b = bench.gemv_bytes(cfg, np.full(L, 11.0), 4)
    assert b - a == pytest.approx(L * 2_039_808)
