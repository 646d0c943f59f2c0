"""Comparison rules shared by the parity tests.

Index rule (rows i >= K-1): the retrieved index SETS must be equal.  A row
whose sets differ is exempt only when every differing key's exact (fp64) score
lies within REL_TIE * |s_K| of the K-th best exact score s_K, i.e. the
difference is a near-tie at the top-K boundary; exempt rows are counted and
reported.  Rows i < K-1 must contain every key 0..i (their pad slots are
compared separately).
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

from oracle import wayfinder_oracle as oracle  # noqa: E402

REL_TIE = 1e-6
GOLDEN = Path(__file__).resolve().parent / "golden"


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


def compare_indices(got: np.ndarray, want: np.ndarray, q_addr: np.ndarray, k_addr: np.ndarray,
                    rows: np.ndarray | None = None, rel_tie: float = REL_TIE) -> dict:
    """Compare (B, n, K) index tensors row by row under the index rule.

    ``rows`` gives the sequence position of each compared row (default 0..n-1).
    Returns {"rows": n_checked, "exempt": n_near_tie, "bad": [(b, i), ...]}.
    """
    B, n, K = got.shape
    assert want.shape == got.shape, (got.shape, want.shape)
    rows = np.arange(n) if rows is None else np.asarray(rows)
    bad, exempt = [], 0
    for b in range(B):
        for r in range(n):
            i = int(rows[r])
            nv = min(i + 1, K)
            g = got[b, r]
            w = want[b, r]
            gs = set(int(x) for x in g if 0 <= x <= i)
            ws = set(int(x) for x in w if 0 <= x <= i)
            if nv < K:
                full = set(range(i + 1))
                if gs != full or ws != full:
                    bad.append((b, i))
                continue
            if len(set(g.tolist())) != K:
                bad.append((b, i))
                continue
            if gs == ws:
                continue
            s = oracle.exact_scores_f64(q_addr, k_addr, b, i)
            sk = np.sort(s)[::-1][K - 1]
            diff = gs.symmetric_difference(ws)
            if all(abs(s[j] - sk) <= rel_tie * abs(sk) for j in diff):
                exempt += 1
            else:
                bad.append((b, i))
    return {"rows": B * n, "exempt": exempt, "bad": bad}


def same_selection(got: np.ndarray, want: np.ndarray) -> bool:
    """(..., T, K) index tensors select the same keys per row (in any slot order) and
    agree exactly on the pad slots that follow the i + 1 keys of rows i < K-1."""
    if got.shape != want.shape:
        return False
    T, K = got.shape[-2], got.shape[-1]
    for i in range(T):
        n = min(i + 1, K)
        g, w = got[..., i, :], want[..., i, :]
        if not (np.sort(g[..., :n], axis=-1) == np.sort(w[..., :n], axis=-1)).all():
            return False
        if not (g[..., n:] == w[..., n:]).all():
            return False
    return True


def reference_pads(i: int, K: int, T: int) -> list[int]:
    """Pad indices of row i under the sorted-slot convention (causal_topk.py:37-57)."""
    return [(i + K + s + 1) % T for s in range(i + 1, K)]
