"""Fused Conv/Linear + BN + LIF (+SEW add) oracle in numpy.

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.

Restates the reference PyTorch path for one layer:

* ``SeqToANNContainer(Conv2d, BatchNorm2d)`` (reference ``models/layers.py:26-31``):
  merge T and B, run the conv (``bias=False``, ``models/sewresnet.py:18-24``)
  and eval-mode BatchNorm2d, split back.
* ``MultiStepLIFNeuron`` (reference ``models/neurons.py:187-211``) over
  ``LIFNeuron.forward`` (``:121-146``): state starts at 0 every forward
  (``:207``); per step
  ``v = v*(1-1/tau) + x/tau``; ``spike = (v - v_th >= 0)`` (``heaviside``,
  ``:69-78``, forward is ``x.ge(0)``); hard reset
  ``v = (1-spike)*v + spike*v_reset``.
* ``MultiStepIFNeuron``: ``v = v + x`` then the same fire/reset.
* SEW ``ADD`` connect: ``out = spike + identity`` (``models/sewresnet.py:50-66``).
* The other residual epilogues of the reference's fused templates
  (``sengine/kernels/interleaved_templates.py``): Add before the neuron,
  ``neuron(bn + residual)`` (``conv1x1_bn_add_lif``, ``:163-221``), and two
  neurons around the Add, ``neuron2(neuron(bn) + residual)``
  (``conv1x1_bn_if_add_lif``, ``:297-364``).  Each neuron follows the
  module semantics above (LIF with its decay, IF without); the reference
  templates integrate without decay in both places (their ``TODO: add LIF
  decay``, ``:378-381``), which is the IF case here.

The conv is an im2col matrix product accumulated in float64 and rounded to
float32 once, which is at least as accurate as the reference's float32 conv.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass
class BNParams:
    gamma: np.ndarray
    beta: np.ndarray
    mean: np.ndarray
    var: np.ndarray
    eps: float = 1e-5

    def scale_bias(self):
        """Per-channel ``(scale, bias)`` with ``bn(y) = y*scale + bias``.

        Restates reference ``sengine/optimizer.py:160-183`` (float64 math,
        stored as float32; conv bias 0): ``scale = gamma/sqrt(var+eps)``,
        ``bias = scale*(0-mean) + beta``.
        """
        g = self.gamma.astype(np.float64)
        s = g / np.sqrt(self.var.astype(np.float64) + self.eps)
        b = s * (0.0 - self.mean.astype(np.float64)) + self.beta.astype(np.float64)
        return s.astype(np.float32), b.astype(np.float32)


def conv2d_nchw(x: np.ndarray, w: np.ndarray, stride: int = 1, pad: int = 0) -> np.ndarray:
    """``x [N,C,H,W]`` * ``w [F,C,KH,KW]`` -> ``[N,F,OH,OW]`` float32."""
    n, c, h, wd = x.shape
    f, c2, kh, kw = w.shape
    assert c == c2
    oh = (h + 2 * pad - kh) // stride + 1
    ow = (wd + 2 * pad - kw) // stride + 1
    xp = np.zeros((n, c, h + 2 * pad, wd + 2 * pad), np.float64)
    xp[:, :, pad:pad + h, pad:pad + wd] = x
    cols = np.empty((n, oh, ow, kh, kw, c), np.float64)
    for i in range(kh):
        for j in range(kw):
            patch = xp[:, :, i:i + stride * oh:stride, j:j + stride * ow:stride]
            cols[:, :, :, i, j, :] = np.transpose(patch, (0, 2, 3, 1))
    wk = np.transpose(w.astype(np.float64), (0, 2, 3, 1)).reshape(f, -1)
    y = cols.reshape(n * oh * ow, -1) @ wk.T
    return np.ascontiguousarray(
        np.transpose(y.reshape(n, oh, ow, f), (0, 3, 1, 2))).astype(np.float32)


def batchnorm_eval(y: np.ndarray, bn: BNParams) -> np.ndarray:
    """Eval-mode BatchNorm2d/1d on channel dim 1, float32 result."""
    shp = (1, -1) + (1,) * (y.ndim - 2)
    inv = 1.0 / np.sqrt(bn.var.astype(np.float64) + bn.eps)
    out = (y.astype(np.float64) - bn.mean.reshape(shp)) * (inv * bn.gamma).reshape(shp) \
        + bn.beta.reshape(shp)
    return out.astype(np.float32)


def multistep_lif(x_seq: np.ndarray, tau: float = 2.0, v_th: float = 1.0,
                  v_reset: float = 0.0, v0: np.ndarray | None = None,
                  neuron: str = "lif"):
    """Run the neuron over ``x_seq [T, ...]`` (float32 arithmetic).

    Returns ``(spikes [T,...], h [T,...] pre-reset membrane, v_final)``.
    """
    x_seq = x_seq.astype(np.float32)
    v = np.zeros_like(x_seq[0]) if v0 is None else v0.astype(np.float32).copy()
    decay = np.float32(1.0 - 1.0 / tau)
    tau32 = np.float32(tau)
    spikes = np.empty_like(x_seq)
    hs = np.empty_like(x_seq)
    for t in range(x_seq.shape[0]):
        if neuron == "lif":
            v = (v * decay + x_seq[t] / tau32).astype(np.float32)
        else:
            v = (v + x_seq[t]).astype(np.float32)
        hs[t] = v
        s = ((v - np.float32(v_th)) >= 0).astype(np.float32)
        v = ((np.float32(1.0) - s) * v + s * np.float32(v_reset)).astype(np.float32)
        spikes[t] = s
    return spikes, hs, v


def fused_layer(x_seq: np.ndarray, w: np.ndarray, bn: BNParams, *, stride: int = 1,
                pad: int | None = None, tau: float = 2.0, v_th: float = 1.0,
                v_reset: float = 0.0, residual: np.ndarray | None = None,
                neuron: str = "lif", v0: np.ndarray | None = None,
                res_mode: str = "add_after", neuron2: str = "lif", tau2: float = 2.0,
                v_th2: float = 1.0, v_reset2: float = 0.0, v0_2: np.ndarray | None = None):
    """One fused layer over ``x_seq [T,B,C,H,W]``.

    Returns dict with ``out`` (spikes, plus ``residual`` when given),
    ``spikes``, ``h`` (pre-reset membrane per step), ``v`` (final membrane
    ``[B,F,OH,OW]``) and ``bn_out`` (BN output per step, the neuron input).
    ``res_mode`` places the residual: ``add_after`` (SEW, ``out = spike +
    residual``), ``add_before`` (the neuron integrates ``bn + residual``) or
    ``two_neuron`` (``out = neuron2(spike + residual)``; adds ``spikes2``,
    ``h2`` and ``v2``, and ``spikes``/``h``/``v`` stay the first neuron's).
    """
    t, b = x_seq.shape[:2]
    if pad is None:
        pad = w.shape[2] // 2
    y = conv2d_nchw(x_seq.reshape((t * b,) + x_seq.shape[2:]), w, stride, pad)
    z = batchnorm_eval(y, bn).reshape((t, b) + y.shape[1:])
    if residual is not None and res_mode == "add_before":
        x_in = (z + residual.astype(np.float32)).astype(np.float32)
    else:
        x_in = z
    spikes, h, v = multistep_lif(x_in, tau, v_th, v_reset, v0=v0, neuron=neuron)
    if residual is None:
        return {"out": spikes, "spikes": spikes, "h": h, "v": v, "bn_out": z}
    if res_mode == "add_before":
        return {"out": spikes, "spikes": spikes, "h": h, "v": v, "bn_out": z}
    if res_mode == "two_neuron":
        x2 = (spikes + residual.astype(np.float32)).astype(np.float32)
        s2, h2, v2 = multistep_lif(x2, tau2, v_th2, v_reset2, v0=v0_2, neuron=neuron2)
        return {"out": s2, "spikes": spikes, "h": h, "v": v, "bn_out": z,
                "spikes2": s2, "h2": h2, "v2": v2}
    if res_mode != "add_after":
        raise ValueError(f"unknown res_mode {res_mode!r}")
    out = spikes + residual.astype(np.float32)
    return {"out": out, "spikes": spikes, "h": h, "v": v, "bn_out": z}


def make_config0(seed: int = 0, T: int = 4, B: int = 16, C: int = 128, F: int = 128,
                 H: int = 32, W: int = 32, k: int = 3, p_spike: float = 0.2):
    """Seeded config-0 style inputs (numpy RNG; shapes per the layer spec).

    Spikes ~ Bernoulli(p); W Kaiming-normal (fan_out, relu gain) then 2:4
    pruned along C per tap; BN gamma~U(.5,1.5), beta~N(0,.1),
    mean~N(0,.1), var~U(.5,1.5).
    """
    from .pack24 import prune_conv_weight
    rng = np.random.default_rng(seed)
    x = (rng.random((T, B, C, H, W)) < p_spike).astype(np.float32)
    std = np.sqrt(2.0 / (F * k * k))
    w = (rng.standard_normal((F, C, k, k)) * std).astype(np.float32)
    w = prune_conv_weight(w)
    bn = BNParams(gamma=rng.uniform(0.5, 1.5, F).astype(np.float32),
                  beta=(rng.standard_normal(F) * 0.1).astype(np.float32),
                  mean=(rng.standard_normal(F) * 0.1).astype(np.float32),
                  var=rng.uniform(0.5, 1.5, F).astype(np.float32))
    return x, w, bn


def spike_agreement(spk_gpu: np.ndarray, spk_ref: np.ndarray, h_ref: np.ndarray,
                    v_th: float = 1.0, band: float = 1e-2, stats: dict | None = None):
    """Parity rule for spikes over ``[T, ...]`` arrays.

    Returns ``(fraction_equal, all_explained, n_mismatch, diverged_mask)``.
    A neuron's FIRST mismatching step must lie at ``|h_ref - v_th| < band``
    (``h_ref`` = oracle pre-reset membrane); after that step the two
    trajectories legitimately differ (the reset happened on one side only),
    so later steps of that neuron are counted but not re-judged.
    ``diverged_mask`` marks neurons with any mismatch (excluded from the
    final-membrane comparison).

    ``stats`` (optional dict) receives the counts that make the relaxation
    visible: ``first`` (first mismatches, each judged against the band),
    ``later`` (mismatches after a neuron's first, not judged), ``later_off_band``
    (those of them whose reference membrane lies outside the band: the
    mismatches the strict per-position rule would reject), ``neurons`` and
    ``diverged`` (neurons with any mismatch).
    """
    mism = spk_gpu != spk_ref
    frac = 1.0 - float(mism.mean()) if mism.size else 1.0
    near = np.abs(h_ref - v_th) < band
    seen = np.zeros(mism.shape[1:], bool)
    ok = True
    n_first = n_later = n_later_off = 0
    for t in range(mism.shape[0]):
        first = mism[t] & ~seen
        later = mism[t] & seen
        if (first & ~near[t]).any():
            ok = False
        n_first += int(first.sum())
        n_later += int(later.sum())
        n_later_off += int((later & ~near[t]).sum())
        seen |= mism[t]
    if stats is not None:
        stats.update(first=n_first, later=n_later, later_off_band=n_later_off,
                     neurons=int(seen.size), diverged=int(seen.sum()))
    return frac, ok, int(mism.sum()), seen


def fused_layer_torch(x_seq, w: np.ndarray, bn: BNParams, *, stride: int = 1,
                      pad: int | None = None, tau: float = 2.0, v_th: float = 1.0,
                      v_reset: float = 0.0, neuron: str = "lif", threads: int | None = None):
    """:func:`fused_layer` for model-sized inputs: torch CPU fp32 conv and
    eval BatchNorm (the reference's own ops, ``SeqToANNContainer(Conv2d,
    BatchNorm2d)``, ``models/layers.py:26-31``), then the same multi-step
    neuron in float32 (``models/neurons.py:121-146,187-211``).

    ``x_seq`` is ``[T,B,C,H,W]`` (numpy or a CPU torch tensor).  Returns numpy
    ``spikes``, ``h`` (pre-reset membrane per step) and ``v`` (final).
    """
    import torch
    import torch.nn.functional as F

    if threads:
        torch.set_num_threads(threads)
    xs = torch.as_tensor(np.asarray(x_seq, np.float32)) if not isinstance(x_seq, torch.Tensor) \
        else x_seq.float()
    t, b = xs.shape[:2]
    if pad is None:
        pad = w.shape[2] // 2
    with torch.no_grad():
        y = F.conv2d(xs.flatten(0, 1), torch.from_numpy(np.ascontiguousarray(w)),
                     stride=stride, padding=pad)
        z = F.batch_norm(y, torch.from_numpy(bn.mean), torch.from_numpy(bn.var),
                         torch.from_numpy(bn.gamma), torch.from_numpy(bn.beta),
                         training=False, eps=bn.eps)
        z = z.view(t, b, *z.shape[1:])
        v = torch.zeros_like(z[0])
        decay = float(np.float32(1.0 - 1.0 / tau))
        spikes = torch.empty_like(z)
        hs = torch.empty_like(z)
        for k in range(t):
            v = v * decay + z[k] / tau if neuron == "lif" else v + z[k]
            hs[k] = v
            s = (v - v_th).ge(0).to(z.dtype)
            v = (1.0 - s) * v + s * v_reset
            spikes[k] = s
    return {"spikes": spikes.numpy(), "h": hs.numpy(), "v": v.numpy()}
