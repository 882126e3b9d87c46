"""MS-ResNet-34 (membrane shortcut) CPU port of the reference PyTorch forward.

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.

Follows reference ``models/msresnet.py``:
* ``MSResNet18.forward`` (``:154-171``): the input repeated over T, the stem
  ``TDBNContainer(Conv2d 7x7/2 pad 3, BatchNorm3d)`` with NO neuron
  (``:135-138``), stages ``conv2_x .. conv5_x`` built by ``_make_layer`` with
  stride 2 in the first block of EVERY stage (``:140-152``), ``sn_out``, mean
  over T, ``adaptive_avg_pool2d(1)``, ``fc``.
* ``BasicBlock18.forward`` (``:119-123``): ``out = conv_bn1(sn1(x))``,
  ``out = conv_bn2(sn2(out))``, ``sc = shortcut(x)`` -- a 1x1/stride conv + BN
  on the REAL-valued x when the shape changes, else x -- and ``out + sc``.
* ``TDBNContainer`` (``:61-87``): conv on the flattened ``(T*B)`` batch, then
  BatchNorm3d over ``(B, C, T, H, W)``; in eval that is the per-channel affine
  ``y*scale + bias``.
* Neurons: the benchmark configuration uses LIF (tau 2, v_th 1, hard reset
  to 0, ``models/neurons.py:121-146``) in place of the reference's
  ``MSNeuron`` (decay 0.25, threshold 0.5, ``:28-58``) -- a deliberate
  deviation that follows the benchmark's stated neuron.

Weights come from a seed so that the GPU model, this port and the golden
fixture (``tests/golden/make_golden.py`` loads them into the reference model
class with its neurons swapped for ``MultiStepLIFNeuron``) all see the same
network.
"""
from __future__ import annotations

import numpy as np

from .pack24 import prune_conv_weight
from .sew_resnet import SPIKE_GAIN, _bn, _conv_w

LAYERS_34 = (3, 4, 6, 3)
STAGES = (64, 128, 256, 512)


def make_params(seed: int = 0, num_classes: int = 1000, layers=LAYERS_34, in_channels: int = 3):
    """Seeded MS-ResNet parameters.  Every conv but the stem 2:4-pruned along
    Cin.  Spike-input convs get the spike gain; the stem (N(0,1) images) and
    the shortcut convs (real-valued membrane stream) Kaiming fan-in."""
    rng = np.random.default_rng(seed)
    P = {"stem": {"w": _conv_w(rng, 64, in_channels, 7, 1.0), "bn": _bn(rng, 64)}, "blocks": []}
    inpl = 64
    for planes, nb in zip(STAGES, layers):
        for bi in range(nb):
            stride = 2 if bi == 0 else 1
            blk = {"stride": stride, "cin": inpl, "planes": planes,
                   "w1": prune_conv_weight(_conv_w(rng, planes, inpl, 3, SPIKE_GAIN)),
                   "bn1": _bn(rng, planes),
                   "w2": prune_conv_weight(_conv_w(rng, planes, planes, 3, SPIKE_GAIN)),
                   "bn2": _bn(rng, planes)}
            if stride != 1 or inpl != planes:
                blk["wsc"] = prune_conv_weight(_conv_w(rng, planes, inpl, 1, 1.0))
                blk["bnsc"] = _bn(rng, planes)
            P["blocks"].append(blk)
            inpl = planes
    bound = 1.0 / np.sqrt(inpl)
    P["fc_w"] = rng.uniform(-bound, bound, (num_classes, inpl)).astype(np.float32)
    P["fc_b"] = rng.uniform(-bound, bound, num_classes).astype(np.float32)
    return P


def make_input(seed: int, B: int, H: int = 224, W: int = 224, C: int = 3):
    rng = np.random.default_rng(seed + 3000)
    return rng.standard_normal((B, C, H, W)).astype(np.float32)


def forward_torch(P, x, T: int = 4, tau: float = 2.0, v_th: float = 1.0,
                  threads: int | None = None, return_trace: bool = False):
    """Reference-path forward in torch (CPU, fp32); ``x`` is ``[B,C,H,W]``.

    Returns logits (numpy); with ``return_trace`` also every block's tensors
    ``[T,B,C,H,W]``: ``stem`` (real), ``b{i}.s1`` (sn1 spikes), ``b{i}.o1``
    (sn2 spikes = conv_bn1 -> sn2), ``b{i}.sc`` (real shortcut, when a conv),
    ``b{i}.out`` (real block output) and ``sn_out``.
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
        y = bn(F.conv2d(t(x), t(P["stem"]["w"]), stride=2, padding=3), P["stem"]["bn"])
        h = y.unsqueeze(0).repeat(T, 1, 1, 1, 1)
        trace["stem"] = h
        for i, blk in enumerate(P["blocks"]):
            s1 = lif(h)
            o1 = lif(seq_conv_bn(s1, blk["w1"], blk["bn1"], blk["stride"], 1))
            out = seq_conv_bn(o1, blk["w2"], blk["bn2"], 1, 1)
            if "wsc" in blk:
                sc = seq_conv_bn(h, blk["wsc"], blk["bnsc"], blk["stride"], 0)
                trace[f"b{i}.sc"] = sc
            else:
                sc = h
            trace[f"b{i}.s1"] = s1
            trace[f"b{i}.o1"] = o1
            h = out + sc
            trace[f"b{i}.out"] = h
        s = lif(h)
        trace["sn_out"] = s
        feat = s.mean(dim=0).mean(dim=(2, 3))
        logits = F.linear(feat, t(P["fc_w"]), t(P["fc_b"]))
    if return_trace:
        return logits.numpy(), {k: v.numpy() for k, v in trace.items()}
    return logits.numpy()
