"""Comparison helpers shared by the parity tests.

Pass bar: selected expert indices bit-exact except where
two router scores tie within one bf16 ulp; block outputs within max-abs 2e-2
and cosine >= 0.9999 of the reference.
"""
from __future__ import annotations

import numpy as np

MAX_ABS_TOL = 2e-2
COSINE_MIN = 0.9999


def bf16_to_f32(b):
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def ulp_bf16(v):
    v = np.abs(np.asarray(v, np.float64))
    v = np.where(v == 0, np.finfo(np.float32).tiny, v)
    return np.exp2(np.floor(np.log2(v)) - 7)


def router_index_check(idx_got, idx_ref, scores_ref):
    """Return (n_mismatch_rows, n_exempt_rows).

    A row whose indices differ is exempt only if, at every position where they
    differ, the two competing experts' reference scores are within one bf16
    ulp of each other (a tie the f32 summation order may break either way).
    """
    idx_got = np.asarray(idx_got)
    idx_ref = np.asarray(idx_ref)
    bad = exempt = 0
    for t in range(idx_ref.shape[0]):
        if np.array_equal(idx_got[t], idx_ref[t]):
            continue
        ok = True
        for k in np.nonzero(idx_got[t] != idx_ref[t])[0]:
            a, b = idx_ref[t, k], idx_got[t, k]
            if not (0 <= b < scores_ref.shape[1]):
                ok = False
                break
            sa, sb = scores_ref[t, a], scores_ref[t, b]
            if abs(float(sa) - float(sb)) > ulp_bf16(max(abs(sa), abs(sb))):
                ok = False
                break
        if ok:
            exempt += 1
        else:
            bad += 1
    return bad, exempt


def exempt_rows(idx_got, idx_ref, scores_ref):
    rows = []
    for t in range(idx_ref.shape[0]):
        if not np.array_equal(idx_got[t], idx_ref[t]):
            rows.append(t)
    return rows


def block_close(got, ref, max_abs=MAX_ABS_TOL, cos_min=COSINE_MIN):
    """max-abs and cosine check; returns (ok, max_abs, cosine)."""
    g = np.asarray(got, np.float64).ravel()
    r = np.asarray(ref, np.float64).ravel()
    if g.size == 0:
        return True, 0.0, 1.0
    ma = float(np.max(np.abs(g - r)))
    den = np.linalg.norm(g) * np.linalg.norm(r)
    cos = float(np.dot(g, r) / den) if den > 0 else (1.0 if ma == 0 else 0.0)
    return (ma <= max_abs and cos >= cos_min), ma, cos
