"""Stage statistics of the diagnose dump (no GPU): the reference's readDiag
record (packages/core/src/nn/model.ts:534-573) and the stage diff."""
import importlib.util
import math
import os

import numpy as np

_path = os.path.join(os.path.dirname(__file__), "..", "0xbitnet_b200", "diagnose.py")
_spec = importlib.util.spec_from_file_location("obn_diagnose", _path)
dg = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(dg)


def test_stage_stats_counts_and_moments():
    v = np.array([1.0, -2.0, 0.0, np.nan, np.inf, 3.0], np.float32)
    s = dg.stage_stats("x", v)
    assert s["length"] == 6 and s["nan_count"] == 1 and s["inf_count"] == 1
    assert s["zero_count"] == 1 and s["min"] == -2.0 and s["max"] == 3.0
    # mean and rms divide by the full length, as the reference does
    assert math.isclose(s["mean"], 2.0 / 6.0)
    assert math.isclose(s["rms"], math.sqrt(14.0 / 6.0))
    assert s["first8"][:3] == [1.0, -2.0, 0.0] and math.isnan(s["first8"][3])


def test_stage_stats_all_nonfinite():
    s = dg.stage_stats("x", np.array([np.nan, -np.inf]))
    assert s["min"] == math.inf and s["max"] == -math.inf
    assert s["nan_count"] == 1 and s["inf_count"] == 1 and s["mean"] == 0.0


def test_first_divergence():
    rng = np.random.default_rng(0)
    arrs = {n: rng.standard_normal(64) for n in dg.STAGES}
    a = [dg.stage_stats(n, arrs[n]) for n in dg.STAGES]
    b = [dg.stage_stats(n, arrs[n] * (1 + 1e-6)) for n in dg.STAGES]
    assert dg.first_divergence(a, b) is None
    c = [dict(s) for s in b]
    c[4]["max"] += 1.0
    assert dg.first_divergence(a, c) == "final_norm"
    d = [dict(s) for s in b]
    d[1]["nan_count"] = 3
    assert dg.first_divergence(a, d) == "layer_0"
    assert dg.first_divergence(a[:2], b) == "layer_1"  # a missing stage
    assert "embedding" in dg.format_stats(a)
