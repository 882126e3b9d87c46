"""Spikformer-8-384 CPU port of the reference PyTorch forward.

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.

Follows reference ``models/spikformer.py``:
* ``SPS`` (``:159-206``): conv 3x3 (no bias) + BatchNorm2d + LIF per stage,
  channels E/8, E/4, E/2, E; a MaxPool2d(3, 2, 1) after the neuron; the RPE
  conv + BN + LIF whose spikes are added to its input (``x + x_feat``);
  tokens ``x.flatten(-2).transpose(-1, -2)``.  The benchmark geometry has a
  pool after EACH of the four stages (224 -> 14x14 tokens); the reference
  module pools after the last two only (56x56 tokens at 224).
* ``Block`` (``:140-152``): ``x + SSA(x)`` then ``x + MLP(x)``.
* ``SSA`` (``:76-130``): q, k, v = LIF(BN1d(Linear(x))); per head
  ``(q k^T * 0.125) v``; ``attn_lif`` (v_th 0.5); ``proj`` = LIF(BN1d(Linear)).
* ``MLP`` (``:47-73``): LIF(BN1d(fc1)), LIF(BN1d(fc2)), hidden 4E.
* head (``:254-264``): mean over tokens, mean over T, Linear.
All neurons LIF tau 2, hard reset to 0 (``models/neurons.py:121-146``).

Weights come from a seed so that the GPU model, this port and the golden
fixture (``tests/golden/make_golden.py`` loads them into the reference's own
``SPS`` sub-modules and ``Block`` modules) all see the same network.
"""
from __future__ import annotations

import numpy as np

from .pack24 import prune_2_4
from .sew_resnet import SPIKE_GAIN, _bn

# Input gains (1/sqrt(E[x^2]) of each layer's input) that keep a random
# network firing: spike inputs SPIKE_GAIN; the residual token stream (small
# non-negative integers) gain 1.
STREAM_GAIN = 1.0


def _w(rng, f, c, k, gain):
    shape = (f, c, k, k) if k else (f, c)
    return (rng.standard_normal(shape) * gain * np.sqrt(2.0 / (c * (k * k if k else 1)))).astype(np.float32)


def _linear(rng, f, c, gain):
    w = prune_2_4(_w(rng, f, c, 0, gain))          # 2:4 along the input dim
    bound = 1.0 / np.sqrt(c)
    b = rng.uniform(-bound, bound, f).astype(np.float32)
    return {"w": w, "b": b, "bn": _bn(rng, f)}


def make_params(seed: int = 0, embed: int = 384, depth: int = 8, mlp_ratio: int = 4,
                num_classes: int = 1000, in_channels: int = 3):
    """Seeded Spikformer parameters.  SPS convs dense (only Linear / 1x1
    weights are 2:4-pruned, along the input dim)."""
    rng = np.random.default_rng(seed)
    e = embed
    chans = (in_channels, e // 8, e // 4, e // 2, e)
    sps = []
    for i in range(4):
        gain = 1.0 if i == 0 else SPIKE_GAIN
        sps.append({"w": _w(rng, chans[i + 1], chans[i], 3, gain), "bn": _bn(rng, chans[i + 1])})
    rpe = {"w": _w(rng, e, e, 3, SPIKE_GAIN), "bn": _bn(rng, e)}
    blocks = []
    for _ in range(depth):
        blocks.append({"q": _linear(rng, e, e, STREAM_GAIN), "k": _linear(rng, e, e, STREAM_GAIN),
                       "v": _linear(rng, e, e, STREAM_GAIN), "proj": _linear(rng, e, e, SPIKE_GAIN),
                       "fc1": _linear(rng, mlp_ratio * e, e, STREAM_GAIN),
                       "fc2": _linear(rng, e, mlp_ratio * e, SPIKE_GAIN)})
    bound = 1.0 / np.sqrt(e)
    return {"sps": sps, "rpe": rpe, "blocks": blocks,
            "fc_w": rng.uniform(-bound, bound, (num_classes, e)).astype(np.float32),
            "fc_b": rng.uniform(-bound, bound, num_classes).astype(np.float32),
            "embed": e, "heads": 12}


def make_input(seed: int, B: int, H: int = 224, W: int = 224, C: int = 3):
    rng = np.random.default_rng(seed + 4000)
    return rng.standard_normal((B, C, H, W)).astype(np.float32)


def forward_torch(P, x, T: int = 4, heads: int = 12, threads: int | None = None,
                  return_trace: bool = False):
    """Reference-path forward in torch (CPU, fp32); ``x`` is ``[B,C,H,W]``
    repeated over T.  Returns logits (numpy); with ``return_trace`` also
    ``sps{i}`` (spikes before the pool), ``pool{i}``, ``x0`` (tokens after the
    RPE add, ``[T,B,N,C]``) and per block ``b{i}.q/k/v/attn/x1/h/x2``."""
    import torch
    import torch.nn.functional as F

    if threads:
        torch.set_num_threads(threads)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))  # noqa: E731
    trace = {}

    def bn(y, p):
        return F.batch_norm(y, t(p["mean"]), t(p["var"]), t(p["gamma"]), t(p["beta"]),
                            training=False, eps=1e-5)

    def lif(z, v_th=1.0, tau=2.0):
        v = torch.zeros_like(z[0])
        out = []
        for k in range(z.shape[0]):
            v = v * (1.0 - 1.0 / tau) + z[k] / tau
            s = (v - v_th).ge(0).to(z.dtype)
            v = (1.0 - s) * v
            out.append(s)
        return torch.stack(out, 0)

    def conv_bn(xs, p):
        Tn, Bn = xs.shape[:2]
        y = bn(F.conv2d(xs.flatten(0, 1), t(p["w"]), padding=1), p["bn"])
        return y.view(Tn, Bn, *y.shape[1:])

    def pool(xs):
        Tn, Bn = xs.shape[:2]
        y = F.max_pool2d(xs.flatten(0, 1), 3, 2, 1)
        return y.view(Tn, Bn, *y.shape[1:])

    def lin(xs, p):
        # Linear over (T*B*N, C), then BatchNorm1d over channels (models/spikformer.py:108-110)
        Tn, Bn, N, C = xs.shape
        y = F.linear(xs.flatten(0, 2), t(p["w"]), t(p["b"]))
        y = F.batch_norm(y, t(p["bn"]["mean"]), t(p["bn"]["var"]), t(p["bn"]["gamma"]),
                         t(p["bn"]["beta"]), training=False, eps=1e-5)
        return y.view(Tn, Bn, N, -1)

    with torch.no_grad():
        xt = t(x)
        y = bn(F.conv2d(xt, t(P["sps"][0]["w"]), padding=1), P["sps"][0]["bn"])
        h = lif(y.unsqueeze(0).repeat(T, 1, 1, 1, 1))
        for i in range(4):
            if i > 0:
                h = lif(conv_bn(h, P["sps"][i]))
            trace[f"sps{i}"] = h
            h = pool(h)
            trace[f"pool{i}"] = h
        x_feat = h
        r = lif(conv_bn(x_feat, P["rpe"]))
        trace["rpe"] = r
        xs = r + x_feat
        Tn, Bn, C, Hh, Ww = xs.shape
        xs = xs.flatten(-2).transpose(-1, -2).contiguous()        # (T, B, N, C)
        trace["x0"] = xs
        N, dh = Hh * Ww, C // heads
        for i, b in enumerate(P["blocks"]):
            q = lif(lin(xs, b["q"]))
            k = lif(lin(xs, b["k"]))
            v = lif(lin(xs, b["v"]))
            qh, kh, vh = (a.reshape(Tn, Bn, N, heads, dh).permute(0, 1, 3, 2, 4) for a in (q, k, v))
            att = (qh @ kh.transpose(-2, -1)) * 0.125
            o = (att @ vh).transpose(2, 3).reshape(Tn, Bn, N, C)
            a = lif(o, v_th=0.5)
            x1 = xs + lif(lin(a, b["proj"]))
            hmid = lif(lin(x1, b["fc1"]))
            x2 = x1 + lif(lin(hmid, b["fc2"]))
            for nm, val in (("q", q), ("k", k), ("v", v), ("attn", a), ("x1", x1), ("h", hmid),
                            ("x2", x2)):
                trace[f"b{i}.{nm}"] = val
            xs = x2
        feat = xs.mean(2).mean(0)
        logits = F.linear(feat, t(P["fc_w"]), t(P["fc_b"]))
    if return_trace:
        return logits.numpy(), {k: v.numpy() for k, v in trace.items()}
    return logits.numpy()
