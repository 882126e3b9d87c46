"""MS-ResNet-34 inference on the B200 fused layers (membrane shortcut).

Mirrors the reference model (``models/msresnet.py``):
* stem ``TDBNContainer(Conv2d 7x7/2, BatchNorm3d)`` without a neuron
  (``:135-138``): ``snn_stem_forward_dual`` writes the fp16 BN output,
  computed once and repeated over T (direct encoding, ``:156-158``), and in
  the same pass block 0's ``sn1`` (the LIF of that output);
* ``BasicBlock18`` (``:94-123``) as three fused launches: the LIF of the
  real-valued stream (``sn1``, ``snn_lif_forward``); conv1 + BN + LIF
  (``conv_bn1`` then ``sn2``, one fused sparse layer); conv2 + BN with the
  shortcut added in the epilogue (``conv_bn2(...) + sc``: fp16 BN output plus
  the residual, rounded once).  The shortcut is the stream itself or a fused
  1x1/stride conv + BN of it (no neuron: its input is real-valued, so the
  sparse MMA's B operand carries fp16 membranes, not spikes);
* ``sn_out`` (LIF), mean over T, avgpool, ``fc`` (``:166-171``) as a neuron
  launch and the head kernel.

The benchmark configuration's neuron is LIF (tau 2, v_th 1) everywhere in
place of the reference's ``MSNeuron`` (decay 0.25, threshold 0.5).
"""
from __future__ import annotations

import numpy as np

from . import runtime as rt
from .layer import SparseConvBNLIF, fold_bn
from .netplan import CONV, HEAD, INPUT, LIF, LOGITS, STEM, Node, PlanModel, glue_desc
from .pruning import prune_conv_2_4
from .sew_resnet import SPIKE_GAIN, _bn_params

LAYERS_34 = (3, 4, 6, 3)
STAGES = (64, 128, 256, 512)


def init_params(seed=0, num_classes=1000, layers=LAYERS_34, in_channels=3):
    """Random-init MS-ResNet parameters (same draws as the oracle's
    ``make_params``): Kaiming-normal fan-in convs, the spike gain on convs
    fed by spikes, BN as config 0, every conv but the stem 2:4-pruned."""
    rng = np.random.default_rng(seed)

    def conv(f, c, k, gain):
        return (rng.standard_normal((f, c, k, k)) * gain * np.sqrt(2.0 / (c * k * k))).astype(np.float32)

    P = {"stem": {"w": conv(64, in_channels, 7, 1.0), "bn": _bn_params(rng, 64)}, "blocks": []}
    inpl = 64
    for planes, nb in zip(STAGES, layers):
        for bi in range(nb):
            stride = 2 if bi == 0 else 1
            blk = {"stride": stride, "cin": inpl, "planes": planes,
                   "w1": prune_conv_2_4(conv(planes, inpl, 3, SPIKE_GAIN)), "bn1": _bn_params(rng, planes),
                   "w2": prune_conv_2_4(conv(planes, planes, 3, SPIKE_GAIN)),
                   "bn2": _bn_params(rng, planes)}
            if stride != 1 or inpl != planes:
                blk["wsc"] = prune_conv_2_4(conv(planes, inpl, 1, 1.0))
                blk["bnsc"] = _bn_params(rng, planes)
            P["blocks"].append(blk)
            inpl = planes
    bound = 1.0 / np.sqrt(inpl)
    P["fc_w"] = rng.uniform(-bound, bound, (num_classes, inpl)).astype(np.float32)
    P["fc_b"] = rng.uniform(-bound, bound, num_classes).astype(np.float32)
    return P


class MSResNet34(PlanModel):
    """One replica of MS-ResNet (default [3,4,6,3]) for fixed (T, batch, H, W).
    Input ``[B, C, H, W]`` fp32 images, repeated over T."""

    def __init__(self, params, *, T=4, batch=64, H=224, W=224, tau=2.0, v_threshold=1.0,
                 device="cuda"):
        st = params["stem"]
        cout, cin, kh, kw = st["w"].shape
        super().__init__(T=T, batch=batch, in_shape=(batch, cin, H, W),
                         num_classes=params["fc_w"].shape[0], device=device)
        dev = self.device
        s, b = fold_bn(**st["bn"])
        # The stem writes its fp16 BN output AND block 0's sn1 (the LIF of that
        # output over T) in one pass (snn_stem_forward_dual).
        self.stem_desc = rt.make_desc(T=T, B=batch, Cin=cin, H=H, W=W, Cout=cout, KH=kh, KW=kw,
                                      stride=2, pad=kh // 2, tau=tau, v_threshold=v_threshold)
        h = (H + 2 * (kh // 2) - kh) // 2 + 1
        w_ = (W + 2 * (kw // 2) - kw) // 2 + 1
        s1_stem = self.buf((T * batch, h, w_, cout))
        x = self.add(Node(STEM, "stem", [INPUT], self.buf((T * batch, h, w_, cout)), self.stem_desc,
                          (self.param(st["w"]), self.param(s), self.param(b)), (1, 0, 0, 0, 0),
                          out2=s1_stem))
        nkw = dict(T=T, B=batch, tau=tau, v_threshold=v_threshold, device=dev)
        c = cout
        for i, blk in enumerate(params["blocks"]):
            stride = blk["stride"]
            if i == 0:
                s1 = s1_stem
            else:
                s1 = self.add(Node(LIF, f"b{i}.sn1", [x], self.buf((T * batch, h, w_, c)),
                                   glue_desc(T=T, B=batch, C=c, H=h, W=w_, tau=tau,
                                             v_threshold=v_threshold)))
            l1 = SparseConvBNLIF(blk["w1"], *fold_bn(**blk["bn1"]), H=h, W=w_, stride=stride,
                                 pad=1, **nkw)
            o1 = self.add(Node(CONV, f"b{i}.conv1", [s1], self.buf(l1.out_shape()), layer=l1))
            sc = x
            if "wsc" in blk:
                lsc = SparseConvBNLIF(blk["wsc"], *fold_bn(**blk["bnsc"]), H=h, W=w_,
                                      stride=stride, pad=0, neuron="none_f16", T=T, B=batch,
                                      device=dev)
                sc = self.add(Node(CONV, f"b{i}.sc", [x], self.buf(lsc.out_shape()), layer=lsc))
            l2 = SparseConvBNLIF(blk["w2"], *fold_bn(**blk["bn2"]), H=l1.OH, W=l1.OW, stride=1,
                                 pad=1, neuron="none_f16", T=T, B=batch, device=dev)
            x = self.add(Node(CONV, f"b{i}.conv2", [o1, sc], self.buf(l2.out_shape()), layer=l2))
            h, w_, c = l1.OH, l1.OW, blk["planes"]
        sout = self.add(Node(LIF, "sn_out", [x], self.buf((T * batch, h, w_, c)),
                             glue_desc(T=T, B=batch, C=c, H=h, W=w_, tau=tau,
                                       v_threshold=v_threshold)))
        self.feat_hw, self.feat_c = h * w_, c
        self.add(Node(HEAD, "head", [sout], LOGITS, None,
                      (self.param(params["fc_w"]), self.param(params["fc_b"])),
                      (T, batch, h * w_, c, self.num_classes)))
