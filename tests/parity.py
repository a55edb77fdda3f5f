"""Parity helpers shared by the tests.

The parity rule for top-k results: returned ids must be identical except at
score ties within a relative tolerance (1e-5 for fp32 data, 1e-2 for
fp16 / bf16), and the returned scores must agree within the same tolerance.
"""
from __future__ import annotations

import numpy as np

RTOL_FP32 = 1e-5
RTOL_HALF = 1e-2


def _close(a, b, rtol, atol):
    return np.abs(a - b) <= atol + rtol * np.maximum(np.abs(a), np.abs(b))


def assert_topk_match(ref_d, ref_i, got_d, got_i, rtol=RTOL_FP32, atol=1e-6, name=""):
    """Sorted scores equal within rtol; ids equal except inside tie groups.

    * a position whose id differs must hold an id the reference ranks at a
      score tied (within rtol) with the reference score at that position;
    * an id missing from the result must be tied with the reference's k-th
      (last kept) score, i.e. the difference is only which tied row was cut.
    """
    ref_d = np.asarray(ref_d, np.float64)
    got_d = np.asarray(got_d, np.float64)
    ref_i = np.asarray(ref_i)
    got_i = np.asarray(got_i)
    assert ref_d.shape == got_d.shape, (name, ref_d.shape, got_d.shape)
    assert ref_i.shape == got_i.shape, (name, ref_i.shape, got_i.shape)
    ok = _close(ref_d, got_d, rtol, atol)
    assert ok.all(), (f"{name}: scores differ at {np.argwhere(~ok)[:5].tolist()}, "
                      f"max |diff| {np.abs(ref_d - got_d)[~ok].max()}")
    for r in range(ref_i.shape[0]):
        if np.array_equal(ref_i[r], got_i[r]):
            continue
        pos = {int(v): j for j, v in enumerate(ref_i[r])}
        last = ref_d[r, -1]
        for j in np.nonzero(ref_i[r] != got_i[r])[0]:
            g = int(got_i[r, j])
            if g in pos:
                assert _close(ref_d[r, pos[g]], ref_d[r, j], rtol, atol), (
                    f"{name}: row {r} pos {j}: id {g} ranked at score {ref_d[r, pos[g]]} by the "
                    f"reference, returned at score {ref_d[r, j]}")
            else:
                assert _close(got_d[r, j], last, rtol, atol), (
                    f"{name}: row {r} pos {j}: extra id {g} (score {got_d[r, j]}) is not tied "
                    f"with the k-th score {last}")
        for m in set(ref_i[r].tolist()) - set(got_i[r].tolist()):
            assert _close(ref_d[r, pos[int(m)]], last, rtol, atol), (
                f"{name}: row {r}: id {m} (score {ref_d[r, pos[int(m)]]}) missing and not tied "
                f"with the k-th score {last}")


def recall(pred, truth):
    """Mean set overlap per row (rapidadb.utils.compute_recall,
    python/rapidadb/utils.py:29-57)."""
    pred = np.asarray(pred)
    truth = np.asarray(truth)
    tot = 0.0
    for p, t in zip(pred, truth):
        ts = set(t.tolist())
        tot += len(set(p.tolist()) & ts) / max(len(ts), 1)
    return tot / max(len(pred), 1)
