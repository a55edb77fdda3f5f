"""Comparison of a multi-iteration Lloyd run with the reference's.

The reference's update kernel sums points with float atomics
(csrc/kernels/kmeans.cu:73-80), so its centroids are reproducible only up to
summation order, and a point whose two nearest centroids are (nearly) equally
far may switch between them.  The pin: centroids within ``rtol`` (relative to
the largest centroid coordinate), labels identical except at near-ties
(squared distances to the two centroids, in fp64 against the reference's
centroids, within ``tie_rtol``).
"""
from __future__ import annotations

import numpy as np


def assert_lloyd_match(x, cent_ref, lab_ref, cent, lab, rtol=1e-4, tie_rtol=1e-4, name=""):
    cent_ref = np.asarray(cent_ref, np.float64)
    cent = np.asarray(cent, np.float64)
    scale = np.abs(cent_ref).max()
    np.testing.assert_allclose(cent, cent_ref, rtol=rtol, atol=rtol * scale, err_msg=f"{name}: centroids")
    lab_ref = np.asarray(lab_ref).astype(np.int64)
    lab = np.asarray(lab).astype(np.int64)
    diff = np.nonzero(lab != lab_ref)[0]
    if len(diff):
        xd = np.asarray(x, np.float64)[diff]
        a = ((xd - cent_ref[lab_ref[diff]]) ** 2).sum(1)
        b = ((xd - cent_ref[lab[diff]]) ** 2).sum(1)
        ok = np.abs(a - b) <= tie_rtol * np.maximum(a, b) + 1e-9
        assert ok.all(), (f"{name}: {int((~ok).sum())} of {len(diff)} differing labels are not near-ties, "
                          f"e.g. point {int(diff[~ok][0])}: {a[~ok][0]} vs {b[~ok][0]}")
    assert len(diff) <= max(2, len(lab) // 1000), f"{name}: {len(diff)} labels differ"
