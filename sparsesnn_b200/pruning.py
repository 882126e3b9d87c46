"""2:4 magnitude pruning for conv/linear weights (host, numpy).

Same rule as reference ``sparse/pruning.py:28-76`` (``prune_n_m``, n=2, m=4):
in every group of 4 consecutive weights along C_in inside one (kh, kw) tap
(reference ``sengine/optimizer.py:499-523`` order), the two of smallest
magnitude are zeroed.
"""
from __future__ import annotations

import numpy as np


def prune_2_4_last(w: np.ndarray) -> np.ndarray:
    """Zero the 2 smallest-|w| of each group of 4 along the last dim."""
    w = np.asarray(w)
    shape = w.shape
    w2 = w.reshape(-1, shape[-1])
    rows, cols = w2.shape
    pad = (-cols) % 4
    if pad:
        w2 = np.concatenate([w2, np.zeros((rows, pad), w2.dtype)], axis=1)
    g = w2.reshape(rows, -1, 4)
    drop = np.argsort(np.abs(g), axis=2, kind="stable")[:, :, :2]
    out = g.copy()
    np.put_along_axis(out, drop, 0, axis=2)
    out = out.reshape(rows, -1)[:, :cols]
    return out.reshape(shape)


def prune_conv_2_4(w_fchw: np.ndarray) -> np.ndarray:
    """2:4-prune ``[F, C, KH, KW]`` along C inside each tap."""
    p = prune_2_4_last(np.transpose(w_fchw, (0, 2, 3, 1)))
    return np.ascontiguousarray(np.transpose(p, (0, 3, 1, 2)))


def is_2_4(w_fchw: np.ndarray) -> bool:
    """At most 2 non-zeros in every group of 4 along C per tap."""
    f = w_fchw.shape[0]
    g = np.transpose(w_fchw, (0, 2, 3, 1)).reshape(f, -1, 4)
    return bool(((g != 0).sum(axis=2) <= 2).all())
