"""Add + neuron and MaxPool + neuron oracles in numpy.

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.

Restates the graph patterns the reference fuses into
``add_lif_fused_kernel`` (``sengine/kernels/add_lif_fused.py:19-75``:
``Add(a, b) -> LIF``) and ``maxpool_lif_fused_kernel``
(``sengine/kernels/pool_lif_fused.py:15-79``: ``MaxPool2d -> LIF``) with the
model semantics: ``torch.nn.MaxPool2d`` (padding never wins the max) per
timestep, then ``MultiStepLIFNeuron`` / ``MultiStepIFNeuron``
(``models/neurons.py:121-146,187-211``, via ``lif_layer.multistep_lif``).
"""
from __future__ import annotations

import numpy as np

from .lif_layer import multistep_lif


def maxpool2d(x: np.ndarray, k: int, s: int, p: int) -> np.ndarray:
    """``x [N, C, H, W]`` -> ``[N, C, OH, OW]``, padded positions at -inf."""
    n, c, h, w = x.shape
    oh = (h + 2 * p - k) // s + 1
    ow = (w + 2 * p - k) // s + 1
    xp = np.full((n, c, h + 2 * p, w + 2 * p), -np.inf, np.float32)
    xp[:, :, p:p + h, p:p + w] = x
    out = np.full((n, c, oh, ow), -np.inf, np.float32)
    for i in range(k):
        for j in range(k):
            out = np.maximum(out, xp[:, :, i:i + s * oh:s, j:j + s * ow:s])
    return out


def maxpool_lif(x_seq, k, s, p, *, tau=2.0, v_th=1.0, v_reset=0.0, neuron="lif", v0=None):
    """``x_seq [T, B, C, H, W]`` -> ``(spikes, h, v_final)`` over the pooled map."""
    t, b = x_seq.shape[:2]
    pooled = maxpool2d(np.asarray(x_seq, np.float32).reshape((t * b,) + x_seq.shape[2:]), k, s, p)
    return multistep_lif(pooled.reshape((t, b) + pooled.shape[1:]), tau, v_th, v_reset, v0=v0,
                         neuron=neuron)


def add_lif(a_seq, b_seq, *, tau=2.0, v_th=1.0, v_reset=0.0, neuron="lif", v0=None):
    """``a_seq + b_seq`` (``[T, ...]``, float32) through the neuron."""
    x = (np.asarray(a_seq, np.float32) + np.asarray(b_seq, np.float32)).astype(np.float32)
    return multistep_lif(x, tau, v_th, v_reset, v0=v0, neuron=neuron)
