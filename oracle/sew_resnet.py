"""SEW-ResNet-18 (CIFAR stem) CPU port of the reference PyTorch forward.

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.  Used by the GPU
model tests as the end-to-end checker and by ``bench.py``'s CPU baseline /
reference arm as the timed "reference CPU path".

Follows reference ``models/sewresnet.py``:
* ``SEWResNet.forward`` (``:190-210``): stem conv + BN once, repeat over T
  (``:199-201``), ``sn1``, maxpool (Identity for the CIFAR stem), 4 stages,
  ``AdaptiveAvgPool2d(1)`` per step, flatten, mean over T, ``fc``.
* ``BasicBlock.forward`` (``:50-66``): ``sn1(bn1(conv1 x))``,
  ``sn2(bn2(conv2 .))``, identity = ``downsample(x)`` when present
  (conv1x1 stride s + BN + neuron, ``:172-179``), ``out += identity`` (ADD).
* Geometry per the benchmark config: 3x3 stride-1 stem with 64 channels, no
  maxpool, stages 64/128/256/512 with [2,2,2,2] blocks, 100 classes, LIF
  neurons (tau 2, v_th 1, hard reset 0) everywhere.

Weights are generated here from a seed (numpy RNG) so that the GPU model,
the oracle and the golden fixture (``tests/golden/make_golden.py``, which
loads them into the real reference model) all see the same parameters.
"""
from __future__ import annotations

import numpy as np

from .pack24 import prune_conv_weight

STAGES = (64, 128, 256, 512)
BLOCKS = (2, 2, 2, 2)


# Kaiming-normal, fan-in, ReLU gain, scaled by 1/sqrt(E[x^2]) of the layer's
# input (spikes firing at about 11%: gain 3), so that random weights keep the
# network firing through every stage (the reference's fan-out init with
# threshold-1 neurons leaves an untrained network nearly silent).
SPIKE_GAIN = 3.0


def _conv_w(rng, f, c, k, gain=SPIKE_GAIN):
    return (rng.standard_normal((f, c, k, k)) * gain * np.sqrt(2.0 / (c * k * k))).astype(np.float32)


def _bn(rng, f):
    return {"gamma": rng.uniform(0.5, 1.5, f).astype(np.float32),
            "beta": (rng.standard_normal(f) * 0.1).astype(np.float32),
            "mean": (rng.standard_normal(f) * 0.1).astype(np.float32),
            "var": rng.uniform(0.5, 1.5, f).astype(np.float32)}


def make_params(seed: int = 0, num_classes: int = 100, in_channels: int = 3,
                stem_channels: int = 64, stem_kernel: int = 3, input_moment: float = 1.0):
    """Seeded SEW-ResNet-18 parameters; every non-stem conv 2:4-pruned along Cin
    (``stem_kernel`` 7: the ImageNet / DVS stem; ``input_moment``: E[x^2] of
    the stem's input, 0.05 for Bernoulli(0.05) event frames)."""
    rng = np.random.default_rng(seed)
    P = {"stem": {"w": _conv_w(rng, stem_channels, in_channels, stem_kernel,
                               1.0 / np.sqrt(input_moment)),
                  "bn": _bn(rng, stem_channels)},
         "blocks": []}
    inpl = stem_channels
    for si, (planes, nb) in enumerate(zip(STAGES, BLOCKS)):
        for bi in range(nb):
            stride = 2 if (si > 0 and bi == 0) else 1
            blk = {"stride": stride, "cin": inpl, "planes": planes,
                   "w1": prune_conv_weight(_conv_w(rng, planes, inpl, 3)), "bn1": _bn(rng, planes),
                   "w2": prune_conv_weight(_conv_w(rng, planes, planes, 3)), "bn2": _bn(rng, planes)}
            if stride != 1 or inpl != planes:
                blk["wd"] = prune_conv_weight(_conv_w(rng, planes, inpl, 1))
                blk["bnd"] = _bn(rng, planes)
            P["blocks"].append(blk)
            inpl = planes
    bound = 1.0 / np.sqrt(inpl)
    P["fc_w"] = rng.uniform(-bound, bound, (num_classes, inpl)).astype(np.float32)
    P["fc_b"] = rng.uniform(-bound, bound, num_classes).astype(np.float32)
    return P


def make_input(seed: int, B: int, H: int = 32, W: int = 32, C: int = 3):
    rng = np.random.default_rng(seed + 1000)
    return rng.standard_normal((B, C, H, W)).astype(np.float32)


def make_dvs_input(seed: int, B: int, T: int = 16, H: int = 128, W: int = 128, C: int = 2,
                   p: float = 0.05):
    """Event frames: Bernoulli(p) {0,1} per polarity, pixel and timestep, in
    the reference's DVS layout ``[B, T, C, H, W]``."""
    rng = np.random.default_rng(seed + 2000)
    return (rng.random((B, T, C, H, W)) < p).astype(np.float32)


def forward_torch(P, x, T: int = 4, tau: float = 2.0, v_th: float = 1.0, threads: int | None = None,
                  return_trace: bool = False, stem_stride: int = 1, maxpool: bool = False):
    """Reference-path forward in torch (CPU, fp32).

    ``x`` is ``[B,C,H,W]`` (direct encoding: the stem's BN output repeated
    over T, ``models/sewresnet.py:197-201``) or ``[B,T,C,H,W]`` event frames
    (the stem runs on every timestep, ``:191-196``).  ``stem_stride=2,
    maxpool=True`` is the ImageNet/DVS stem (7x7/2, MaxPool(3,2,1) after the
    neuron, ``:140-143,202-203``).

    Returns logits ``[B, classes]`` (numpy); with ``return_trace`` also the
    per-layer spike tensors ``[T,B,C,H,W]`` keyed by layer name.
    """
    import torch
    import torch.nn.functional as F

    if threads:
        torch.set_num_threads(threads)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))  # noqa: E731
    trace = {}

    def bn(y, p):
        return F.batch_norm(y, t(p["mean"]), t(p["var"]), t(p["gamma"]), t(p["beta"]),
                            training=False, eps=1e-5)

    def lif(z_seq):
        v = torch.zeros_like(z_seq[0])
        out = []
        decay = 1.0 - 1.0 / tau
        for k in range(z_seq.shape[0]):
            v = v * decay + z_seq[k] / tau
            s = (v - v_th).ge(0).to(z_seq.dtype)
            v = (1.0 - s) * v + s * 0.0
            out.append(s)
        return torch.stack(out, 0)

    def seq_conv_bn(x_seq, w, p, stride, pad):
        Tn, Bn = x_seq.shape[:2]
        y = F.conv2d(x_seq.flatten(0, 1), t(w), stride=stride, padding=pad)
        y = bn(y, p)
        return y.view(Tn, Bn, *y.shape[1:])

    with torch.no_grad():
        xt = t(x)
        w0 = P["stem"]["w"]
        pad0 = w0.shape[2] // 2
        if xt.dim() == 5:                                  # [B,T,C,H,W] -> [T,B,C,H,W]
            xs = xt.transpose(0, 1).contiguous()
            Tn, Bn = xs.shape[:2]
            y = bn(F.conv2d(xs.flatten(0, 1), t(w0), stride=stem_stride, padding=pad0),
                   P["stem"]["bn"])
            h = lif(y.view(Tn, Bn, *y.shape[1:]))
        else:
            y = bn(F.conv2d(xt, t(w0), stride=stem_stride, padding=pad0), P["stem"]["bn"])
            h = lif(y.unsqueeze(0).repeat(T, 1, 1, 1, 1))
        trace["stem"] = h
        if maxpool:
            Tn, Bn = h.shape[:2]
            h = F.max_pool2d(h.flatten(0, 1), 3, 2, 1)
            h = h.view(Tn, Bn, *h.shape[1:])
            trace["maxpool"] = h
        for i, blk in enumerate(P["blocks"]):
            ident = h
            o = lif(seq_conv_bn(h, blk["w1"], blk["bn1"], blk["stride"], 1))
            trace[f"b{i}.sn1"] = o
            o = lif(seq_conv_bn(o, blk["w2"], blk["bn2"], 1, 1))
            trace[f"b{i}.sn2"] = o
            if "wd" in blk:
                ident = lif(seq_conv_bn(h, blk["wd"], blk["bnd"], blk["stride"], 0))
                trace[f"b{i}.ds"] = ident
            h = o + ident
            trace[f"b{i}.out"] = h
        feat = h.mean(dim=(3, 4))            # AdaptiveAvgPool2d(1) + flatten(2)
        logits = F.linear(feat.mean(dim=0), t(P["fc_w"]), t(P["fc_b"]))
    if return_trace:
        return logits.numpy(), {k: v.numpy() for k, v in trace.items()}
    return logits.numpy()
