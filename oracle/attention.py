"""Spikformer attention core + attention LIF oracle in numpy.

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.

Restates the reference's spiking self-attention core
(``models/spikformer.py:122-127``): per timestep, image and head,
``attn = (q @ k^T) * scale`` and ``x = attn @ v`` with the heads merged back
into channels, then ``attn_lif = MultiStepLIFNeuron(tau=2, v_threshold=0.5)``
(``:97``) over the T timesteps.  The fused graph op that replaces this
subgraph, ``FusedSpikformerAttention``, computes the same thing
(``sengine/tdl/attention_ops.py:50-82``).

With spike inputs every product is an integer count, so the float64 matrix
products here are exact and so is their float32 cast; the neuron update
follows ``lif_layer.multistep_lif`` (float32, division form of the reference
LIF, ``models/neurons.py:121-146``).
"""
from __future__ import annotations

import numpy as np

from .lif_layer import multistep_lif


def spikformer_attn_lif(q, k, v, *, T: int, heads: int, scale: float = 0.125, tau: float = 2.0,
                        v_th: float = 0.5, v_reset: float = 0.0, v0=None):
    """``q, k, v``: ``(T*B, N, C)`` arrays of spikes.

    Returns ``(spikes (T*B,N,C), x (T*B,N,C) float32 neuron input,
    h (T*B,N,C) pre-reset membrane, v_final (B,N,C))``.
    """
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    tb, n, c = q.shape
    hd = c // heads
    b = tb // T

    def split(a):
        return a.reshape(tb, n, heads, hd).transpose(0, 2, 1, 3)     # (TB, heads, N, hd)

    qh, kh, vh = split(q), split(k), split(v)
    attn = (qh @ kh.transpose(0, 1, 3, 2)) * scale
    x = (attn @ vh).transpose(0, 2, 1, 3).reshape(tb, n, c).astype(np.float32)
    v0_ = None if v0 is None else np.asarray(v0, np.float32)
    spikes, h, v_final = multistep_lif(x.reshape(T, b, n, c), tau, v_th, v_reset, v0=v0_)
    return (spikes.reshape(tb, n, c), x, h.reshape(tb, n, c), v_final)
