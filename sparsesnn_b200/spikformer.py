"""Spikformer-8-384 inference on the B200 fused layers.

Mirrors the reference model (``models/spikformer.py``) in the benchmark
geometry (a stride-2 pool after each of the four patch-splitting stages:
224x224 -> 14x14 = 196 tokens, 12 heads of 32 channels):
* ``SPS`` (``:159-206``): the stem conv (Cin = 3, dense) + BN + LIF, then
  three dense 3x3 convs + BN + LIF as fused layers with unpruned weights
  (``SNN_FLAG_DENSE``); a plain spike max pool after every stage; the RPE
  conv + BN + LIF with ``x + x_feat`` fused as its SEW add;
* ``Block`` (``:140-152``) x 8: q, k, v = Linear + BN1d + LIF as ONE fused
  2:4 layer over the T*B*N token rows (the three weights stacked, 3E output
  channels, each row q | k | v); the attention core + attention LIF (v_th
  0.5, one kernel) reading q, k, v as packed blocks; proj = Linear + BN1d + LIF with ``x + ...`` in its
  epilogue; MLP fc1 / fc2 likewise, fc2 adding ``x1``;
* the head (mean over tokens and T, Linear) in the head kernel.

Activations keep their real channel counts (48, 96, ...): a fused layer's
last 64-channel k-block reads zeros past its input channels.
"""
from __future__ import annotations

import numpy as np
import torch

from . import runtime as rt
from .layer import SparseConvBNLIF, fold_bn
from .netplan import (ATTN, CONV, HEAD, INPUT, LOGITS, MAXPOOL, STEM, Node, PlanModel,
                      glue_desc, pool_out)
from .pruning import prune_2_4_last
from .sew_resnet import SPIKE_GAIN, _bn_params

STREAM_GAIN = 1.0


def init_params(seed=0, embed=384, depth=8, mlp_ratio=4, num_classes=1000, in_channels=3):
    """Random-init Spikformer parameters (same draws as the oracle's
    ``make_params``): dense SPS convs, Linear weights 2:4-pruned along the
    input dim with nn.Linear-style biases, BN as config 0; Kaiming fan-in
    scaled by the input's second moment (spike inputs ``SPIKE_GAIN``)."""
    rng = np.random.default_rng(seed)

    def w(f, c, k, gain):
        shape = (f, c, k, k) if k else (f, c)
        return (rng.standard_normal(shape) * gain * np.sqrt(2.0 / (c * (k * k if k else 1)))).astype(np.float32)

    def linear(f, c, gain):
        wt = prune_2_4_last(w(f, c, 0, gain))
        bound = 1.0 / np.sqrt(c)
        return {"w": wt, "b": rng.uniform(-bound, bound, f).astype(np.float32), "bn": _bn_params(rng, f)}

    e = embed
    chans = (in_channels, e // 8, e // 4, e // 2, e)
    sps = []
    for i in range(4):
        sps.append({"w": w(chans[i + 1], chans[i], 3, 1.0 if i == 0 else SPIKE_GAIN),
                    "bn": _bn_params(rng, chans[i + 1])})
    rpe = {"w": w(e, e, 3, SPIKE_GAIN), "bn": _bn_params(rng, e)}
    blocks = []
    for _ in range(depth):
        blocks.append({"q": linear(e, e, STREAM_GAIN), "k": linear(e, e, STREAM_GAIN),
                       "v": linear(e, e, STREAM_GAIN), "proj": linear(e, e, SPIKE_GAIN),
                       "fc1": linear(mlp_ratio * e, e, STREAM_GAIN),
                       "fc2": linear(e, mlp_ratio * e, SPIKE_GAIN)})
    bound = 1.0 / np.sqrt(e)
    return {"sps": sps, "rpe": rpe, "blocks": blocks,
            "fc_w": rng.uniform(-bound, bound, (num_classes, e)).astype(np.float32),
            "fc_b": rng.uniform(-bound, bound, num_classes).astype(np.float32),
            "embed": e, "heads": 12}


class Spikformer(PlanModel):
    """One replica of Spikformer (default 8-384, 12 heads) for fixed (T,
    batch, H, W).  Input ``[B, C, H, W]`` fp32 images, repeated over T."""

    def __init__(self, params, *, T=4, batch=32, H=224, W=224, tau=2.0, v_threshold=1.0,
                 attn_v_threshold=0.5, device="cuda"):
        E, heads = params["embed"], params["heads"]
        st = params["sps"][0]
        c0, cin = st["w"].shape[:2]
        super().__init__(T=T, batch=batch, in_shape=(batch, cin, H, W),
                         num_classes=params["fc_w"].shape[0], device=device)
        dev = self.device
        TB = T * batch
        lif = dict(tau=tau, v_threshold=v_threshold)
        s, b = fold_bn(**st["bn"])
        self.stem_desc = rt.make_desc(T=T, B=batch, Cin=cin, H=H, W=W, Cout=c0, KH=3, KW=3,
                                      stride=1, pad=1, **lif)
        # The stem's spikes go only to the first max pool: they travel
        # bit-packed (an eighth of the fp16 bytes at full resolution).
        bits = rt.SNN_FLAG_SPIKE_BITS if c0 % 16 == 0 else 0
        self.stem_desc.flags = bits
        sps0 = self.buf((TB, H, W, c0 // 8), torch.uint8) if bits else self.buf((TB, H, W, c0))
        x = self.add(Node(STEM, "sps0", [INPUT], sps0, self.stem_desc,
                          (self.param(st["w"]), self.param(s), self.param(b)), (1, 0, 0, 0, 0)))
        h, w_, c = H, W, c0
        for i in range(4):
            if i > 0:
                p = params["sps"][i]
                layer = SparseConvBNLIF(p["w"], *fold_bn(**p["bn"]), T=T, B=batch, H=h, W=w_,
                                        pad=1, dense=True, device=dev, **lif)
                x = self.add(Node(CONV, f"sps{i}", [x], self.buf(layer.out_shape()), layer=layer))
                c = layer.Cout
            ph, pw = pool_out(h, 3, 2, 1), pool_out(w_, 3, 2, 1)
            pd = glue_desc(T=T, B=batch, C=c, H=h, W=w_, neuron="none", k=3, stride=2, pad=1)
            if i == 0:
                pd.flags = bits
            x = self.add(Node(MAXPOOL, f"pool{i}", [x], self.buf((TB, ph, pw, c)), pd))
            h, w_ = ph, pw
        p = params["rpe"]
        rpe = SparseConvBNLIF(p["w"], *fold_bn(**p["bn"]), T=T, B=batch, H=h, W=w_, pad=1,
                              dense=True, device=dev, **lif)
        x0 = self.add(Node(CONV, "rpe", [x, x], self.buf(rpe.out_shape()), layer=rpe))
        N = h * w_
        self.tokens = N
        rows = batch * N

        def lin(pp, name, src, res=None, out_c=None):
            if isinstance(pp, (list, tuple)):
                # Linears over the same input as one layer: weights stacked
                # along the output channels, BN folded per part.
                folds = [fold_bn(**x["bn"], conv_bias=x["b"]) for x in pp]
                w = np.concatenate([np.asarray(x["w"]) for x in pp], 0)
                sc = np.concatenate([f[0] for f in folds])
                bi = np.concatenate([f[1] for f in folds])
            else:
                w, (sc, bi) = pp["w"], fold_bn(**pp["bn"], conv_bias=pp["b"])
            layer = SparseConvBNLIF(w, sc, bi, T=T, B=1, H=1, W=rows, device=dev, **lif)
            out = self.buf(layer.out_shape())
            ins = [src.view(T, 1, rows, src.shape[-1])]
            if res is not None:
                ins.append(res.view(T, 1, rows, res.shape[-1]))
            self.add(Node(CONV, name, ins, out, layer=layer))
            return out

        xs = x0.view(T, 1, rows, E)
        attn_desc = rt.make_desc(T=T, B=batch, Cin=E, H=1, W=N, Cout=E, KH=1, KW=1, tau=tau,
                                 v_threshold=attn_v_threshold)
        for i, blk in enumerate(params["blocks"]):
            # q, k, v: one launch of the three Linears (3E output channels,
            # rows of q | k | v), read by the attention core as packed blocks.
            qkv = lin([blk["q"], blk["k"], blk["v"]], f"b{i}.qkv", xs)
            a = self.add(Node(ATTN, f"b{i}.attn", [qkv.view(TB, N, 3 * E)], self.buf((TB, N, E)),
                              attn_desc, attn={"N": N, "heads": heads, "head_dim": E // heads,
                                               "scale": 0.125, "packed": True}))
            x1 = lin(blk["proj"], f"b{i}.proj", a, res=xs)
            hm = lin(blk["fc1"], f"b{i}.fc1", x1)
            xs = lin(blk["fc2"], f"b{i}.fc2", hm, res=x1)
        self.feat_hw, self.feat_c = N, E
        self.add(Node(HEAD, "head", [xs], LOGITS, None,
                      (self.param(params["fc_w"]), self.param(params["fc_b"])),
                      (T, batch, N, E, self.num_classes)))
