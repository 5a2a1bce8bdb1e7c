"""Stage statistics for diffing a forward against the oracle, stage by stage.

The reference's `diagnose()` (packages/core/src/nn/model.ts:449-531, readDiag at
:534-573, DiagnosticResult in packages/core/src/types.ts:100-111) reads back
the embedding, the outputs of layers 0 and 1 and of the last layer, the final
norm, the LM-head input and the first 100 logits, and reports per stage the
length, min / max / mean / rms over the finite values (mean and rms divided by
the full length, as the reference does), the NaN / Inf / zero counts and the
first eight values. `stage_stats` computes the same record from a host array;
`BitNetDecoder.diagnose` (decoder.py) produces the stages of a decode step and
`first_divergence` names the first stage whose statistics leave a tolerance
against another run's (the oracle's) stages.

Pure numpy: importing this module does not load libobn.
"""
from __future__ import annotations

import math
from typing import Iterable, Sequence

import numpy as np

# Stage names of a decode step, in the reference's order.
STAGES = ("embedding", "layer_0", "layer_1", "last_layer", "final_norm", "lm_input",
          "logits_first100")


def stage_stats(name: str, values) -> dict:
    """readDiag's record for one stage (float64 accumulation over the values)."""
    a = np.asarray(values, dtype=np.float64).ravel()
    n = int(a.size)
    nan = np.isnan(a)
    inf = np.isinf(a)
    fin = a[~(nan | inf)]
    out = {
        "name": name,
        "length": n,
        "min": float(fin.min()) if fin.size else math.inf,
        "max": float(fin.max()) if fin.size else -math.inf,
        "mean": float(fin.sum() / n) if n else math.nan,
        "rms": float(math.sqrt(float((fin * fin).sum()) / n)) if n else math.nan,
        "nan_count": int(nan.sum()),
        "inf_count": int(inf.sum()),
        "zero_count": int((fin == 0).sum()),
        "first8": [float(v) for v in a[:8]],
    }
    return out


def _close(a: float, b: float, rtol: float, atol: float) -> bool:
    if math.isinf(a) or math.isinf(b) or math.isnan(a) or math.isnan(b):
        return (a == b) or (math.isnan(a) and math.isnan(b))
    return abs(a - b) <= atol + rtol * abs(b)


def first_divergence(got: Sequence[dict], want: Sequence[dict], rtol: float = 1e-3,
                     atol: float = 1e-4,
                     fields: Iterable[str] = ("min", "max", "mean", "rms")) -> str | None:
    """Name of the first stage (in `want`'s order) whose counts differ or whose
    statistics leave rtol / atol, or None when every stage agrees."""
    by_name = {s["name"]: s for s in got}
    for w in want:
        g = by_name.get(w["name"])
        if g is None or g["length"] != w["length"]:
            return w["name"]
        if any(g[k] != w[k] for k in ("nan_count", "inf_count")):
            return w["name"]
        if not all(_close(g[f], w[f], rtol, atol) for f in fields):
            return w["name"]
    return None


def format_stats(stats: Sequence[dict]) -> str:
    """One line per stage, for logs."""
    lines = []
    for s in stats:
        lines.append(
            f"{s['name']:16s} n={s['length']:8d} min={s['min']:+.5g} max={s['max']:+.5g} "
            f"mean={s['mean']:+.5g} rms={s['rms']:.5g} nan={s['nan_count']} "
            f"inf={s['inf_count']} zero={s['zero_count']}")
    return "\n".join(lines)
