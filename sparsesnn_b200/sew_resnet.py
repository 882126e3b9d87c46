"""SEW-ResNet-18 inference on the B200 fused layers (CIFAR stem, T steps).

Mirrors the reference model (``models/sewresnet.py``):
* stem conv+BN computed once and repeated over T (``:199-201``) -> LIF
  (``snn_stem_forward``, dense: the reference never prunes the stem);
* ``BasicBlock`` (``:50-66``): conv1+BN+LIF and conv2+BN+LIF as fused 2:4
  layers; the SEW ``ADD`` (``out += identity``) is fused into conv2's
  epilogue; the downsample (conv1x1 stride s + BN + LIF, ``:172-179``) is a
  fused 1x1 layer whose output is conv2's residual;
* avgpool + mean over T + fc (``:207-210``) in one head kernel.

All activations live in preallocated device buffers, so ``forward`` does not
allocate and can be captured in a CUDA graph.  The product path has no CPU
fallback: every op is a libsnnb200 launch.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import runtime as rt
from .layer import SparseConvBNLIF, fold_bn
from .netplan import CONV, HEAD, INPUT, LOGITS, MAXPOOL, STEM, Node, PlanModel, glue_desc, pool_out
from .pruning import prune_conv_2_4

STAGES = (64, 128, 256, 512)
BLOCKS = (2, 2, 2, 2)


def _bn_params(rng, f):
    return {"gamma": rng.uniform(0.5, 1.5, f).astype(np.float32),
            "beta": (rng.standard_normal(f) * 0.1).astype(np.float32),
            "mean": (rng.standard_normal(f) * 0.1).astype(np.float32),
            "var": rng.uniform(0.5, 1.5, f).astype(np.float32)}


# Kaiming-normal (fan-in, ReLU gain) scaled by 1/sqrt(E[x^2]) of the layer's
# input, so that a random-weight network keeps firing through every stage:
# spike inputs firing at about 11% (E[x^2] = 1/9, gain 3); the stem sees
# N(0,1) images (gain 1) or event frames of density p (gain 1/sqrt(p)).
SPIKE_GAIN = 3.0


def init_params(seed=0, num_classes=100, in_channels=3, stem_channels=64, stem_kernel=3,
                input_moment=1.0):
    """Random-init parameters of the benchmark configuration (``stem_kernel``
    7 for the ImageNet / DVS stem, ``models/sewresnet.py:140``;
    ``input_moment`` = E[x^2] of the stem's input).

    Kaiming-normal convs (fan-in, ReLU gain, scaled by 1/sqrt(E[x^2]) of the
    layer's input, see ``SPIKE_GAIN``), BN gamma~U(.5,1.5), beta~N(0,.1),
    mean~N(0,.1), var~U(.5,1.5); every conv except the stem 2:4-pruned along
    C_in; nn.Linear-style uniform head.
    """
    rng = np.random.default_rng(seed)

    def conv(f, c, k, gain=SPIKE_GAIN):
        return (rng.standard_normal((f, c, k, k)) * gain * np.sqrt(2.0 / (c * k * k))).astype(np.float32)

    P = {"stem": {"w": conv(stem_channels, in_channels, stem_kernel, 1.0 / np.sqrt(input_moment)),
                  "bn": _bn_params(rng, stem_channels)},
         "blocks": []}
    inpl = stem_channels
    for si, (planes, nb) in enumerate(zip(STAGES, BLOCKS)):
        for bi in range(nb):
            stride = 2 if (si > 0 and bi == 0) else 1
            blk = {"stride": stride, "cin": inpl, "planes": planes,
                   "w1": prune_conv_2_4(conv(planes, inpl, 3)), "bn1": _bn_params(rng, planes),
                   "w2": prune_conv_2_4(conv(planes, planes, 3)), "bn2": _bn_params(rng, planes)}
            if stride != 1 or inpl != planes:
                blk["wd"] = prune_conv_2_4(conv(planes, inpl, 1))
                blk["bnd"] = _bn_params(rng, planes)
            P["blocks"].append(blk)
            inpl = planes
    bound = 1.0 / np.sqrt(inpl)
    P["fc_w"] = rng.uniform(-bound, bound, (num_classes, inpl)).astype(np.float32)
    P["fc_b"] = rng.uniform(-bound, bound, num_classes).astype(np.float32)
    return P


def params_from_state_dict(sd, prune=False):
    """Map a reference ``SEWResNet`` state_dict (``sew_resnet18`` with a 3x3
    stem) to the parameter dict used here.  Keys follow the reference module
    tree: ``conv1``, ``bn1``, ``layerX.Y.conv{1,2}.module.{0,1}``,
    ``layerX.0.downsample.0.module.{0,1}``, ``fc``."""
    g = lambda k: sd[k].detach().cpu().numpy().astype(np.float32)  # noqa: E731

    def bn(prefix):
        return {"gamma": g(prefix + ".weight"), "beta": g(prefix + ".bias"),
                "mean": g(prefix + ".running_mean"), "var": g(prefix + ".running_var")}

    pr = prune_conv_2_4 if prune else (lambda w: w)
    P = {"stem": {"w": g("conv1.weight"), "bn": bn("bn1")}, "blocks": []}
    inpl = P["stem"]["w"].shape[0]
    for li in range(1, 5):
        bi = 0
        while f"layer{li}.{bi}.conv1.module.0.weight" in sd:
            pre = f"layer{li}.{bi}"
            w1 = g(pre + ".conv1.module.0.weight")
            planes = w1.shape[0]
            blk = {"cin": inpl, "planes": planes,
                   "stride": 2 if (li > 1 and bi == 0) else 1,
                   "w1": pr(w1), "bn1": bn(pre + ".conv1.module.1"),
                   "w2": pr(g(pre + ".conv2.module.0.weight")), "bn2": bn(pre + ".conv2.module.1")}
            if pre + ".downsample.0.module.0.weight" in sd:
                blk["wd"] = pr(g(pre + ".downsample.0.module.0.weight"))
                blk["bnd"] = bn(pre + ".downsample.0.module.1")
            P["blocks"].append(blk)
            inpl = planes
            bi += 1
    P["fc_w"] = g("fc.weight")
    P["fc_b"] = g("fc.bias")
    return P


class SEWResNet18:
    """One replica of SEW-ResNet-18 for a fixed (T, batch, H, W)."""

    def __init__(self, params, *, T=4, batch=128, H=32, W=32, tau=2.0, v_threshold=1.0,
                 device="cuda"):
        self.T, self.B, self.H, self.W = T, batch, H, W
        self.device = torch.device(device)
        dev = self.device
        lib = rt.load()
        rt.check(lib.snn_init())
        st = params["stem"]
        self.stem_w = torch.from_numpy(st["w"]).to(dev)
        s, b = fold_bn(**st["bn"])
        self.stem_scale = torch.from_numpy(s).to(dev)
        self.stem_bias = torch.from_numpy(b).to(dev)
        cout, cin, kh, kw = st["w"].shape
        self.stem_desc = rt.make_desc(T=T, B=batch, Cin=cin, H=H, W=W, Cout=cout, KH=kh, KW=kw,
                                      stride=1, pad=kh // 2, tau=tau, v_threshold=v_threshold)
        # Two input buffers: the host->device copy of the next call's images
        # (on a copy stream) overlaps the forward that reads the other one.
        self.x_ins = [torch.empty((batch, cin, H, W), dtype=torch.float32, device=dev)
                      for _ in range(2)]
        self.x_in = self.x_ins[0]
        self._in_sel = 0                  # input buffer the launches read
        self._next_buf = 0
        self._copy_stream = torch.cuda.Stream(dev)
        self._buf_free = [None, None]     # event: last forward reading buffer k is done
        self.a0 = torch.empty((T * batch, H, W, cout), dtype=torch.float16, device=dev)
        kw_ = dict(T=T, B=batch, tau=tau, v_threshold=v_threshold, device=dev)
        self.blocks = []
        h, w, c = H, W, cout
        for blk in params["blocks"]:
            stride = blk["stride"]
            l1 = SparseConvBNLIF(blk["w1"], *fold_bn(**blk["bn1"]), H=h, W=w, stride=stride,
                                 pad=1, **kw_)
            oh, ow = l1.OH, l1.OW
            l2 = SparseConvBNLIF(blk["w2"], *fold_bn(**blk["bn2"]), H=oh, W=ow, stride=1,
                                 pad=1, **kw_)
            ds = None
            if "wd" in blk:
                ds = SparseConvBNLIF(blk["wd"], *fold_bn(**blk["bnd"]), H=h, W=w, stride=stride,
                                     pad=0, **kw_)
            planes = l1.Cout
            o1 = torch.empty(l1.out_shape(), dtype=torch.float16, device=dev)
            idb = torch.empty(ds.out_shape(), dtype=torch.float16, device=dev) if ds else None
            out = torch.empty(l2.out_shape(), dtype=torch.float16, device=dev)
            self.blocks.append({"l1": l1, "l2": l2, "ds": ds, "o1": o1, "id": idb, "out": out})
            h, w, c = oh, ow, planes
        self.feat_hw, self.feat_c = h * w, c
        self.fc_w = torch.from_numpy(params["fc_w"]).to(dev)
        self.fc_b = torch.from_numpy(params["fc_b"]).to(dev)
        self.num_classes = self.fc_w.shape[0]
        # One logits buffer per input buffer (each captured graph writes its
        # own), so a consumer of one forward's logits -- a copy to the host, a
        # collective -- can overlap the next forward.
        self.logits_bufs = [torch.empty((batch, self.num_classes), dtype=torch.float32, device=dev)
                            for _ in range(2)]
        self.logits = self.logits_bufs[0]
        self._graph = None

    # --------------------------------------------------------------- launches
    def conv_layers(self):
        for blk in self.blocks:
            yield blk["l1"]
            if blk["ds"] is not None:
                yield blk["ds"]
            yield blk["l2"]

    def launches(self):
        """(name, callable) for every kernel launch of one forward, in order."""
        lib = rt.load()
        ops = []

        def stem():
            s = torch.cuda.current_stream(self.device).cuda_stream
            rt.check(lib.snn_stem_forward(self.stem_desc, 1, self.x_ins[self._in_sel].data_ptr(),
                                          self.stem_w.data_ptr(), self.stem_scale.data_ptr(),
                                          self.stem_bias.data_ptr(), self.a0.data_ptr(), s))
        ops.append(("stem", stem))
        h = self.a0
        for i, blk in enumerate(self.blocks):
            hin = h
            ops.append((f"b{i}.conv1", lambda blk=blk, hin=hin: blk["l1"](hin, out=blk["o1"])))
            if blk["ds"] is not None:
                ops.append((f"b{i}.ds", lambda blk=blk, hin=hin: blk["ds"](hin, out=blk["id"])))
                ident = blk["id"]
            else:
                ident = hin
            ops.append((f"b{i}.conv2", lambda blk=blk, ident=ident:
                        blk["l2"](blk["o1"], residual=ident, out=blk["out"])))
            h = blk["out"]

        def head(h=h):
            s = torch.cuda.current_stream(self.device).cuda_stream
            rt.check(lib.snn_head_forward(self.T, self.B, self.feat_hw, self.feat_c,
                                          self.num_classes, h.data_ptr(), self.fc_w.data_ptr(),
                                          self.fc_b.data_ptr(),
                                          self.logits_bufs[self._in_sel].data_ptr(), s))
        ops.append(("head", head))
        return ops

    def run(self):
        """One forward from input buffer ``_in_sel`` (``self.x_in`` unless a
        call selected the other) into its logits buffer (no allocation)."""
        for _, op in self._ops():
            op()
        return self.logits_bufs[self._in_sel]

    def _ops(self):
        if not hasattr(self, "_ops_cache"):
            self._ops_cache = self.launches()
        return self._ops_cache

    def capture(self, warmup=3):
        """Capture the forward into CUDA graphs (after eager warm-ups), one
        per input buffer; returns the graph that reads ``x_in``."""
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self.run()
        torch.cuda.current_stream(self.device).wait_stream(s)
        self._graphs = []
        for k in range(2):
            self._in_sel = k
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.run()
            self._graphs.append(g)
        self._in_sel = 0
        self._graph = self._graphs[0]
        return self._graph

    def replay(self, buf=0):
        """Replay the forward on the images in input buffer ``buf`` (0 is
        ``x_in``); returns that buffer's logits."""
        self._graphs[buf].replay()
        return self.logits_bufs[buf]

    def __call__(self, x):
        """Public API: images ``[B, C, H, W]`` fp32 (host or device) -> logits
        (device tensor on the current stream, valid until the call after
        next: consecutive calls alternate between two logits buffers).

        The images go to the device on a copy stream into the input buffer
        the previous forward is not reading, so when calls follow each other
        the copy of one batch overlaps the forward of the previous one; the
        forward itself is ordered after its copy on the current stream.
        ``x`` (pinned host memory for an asynchronous copy) must stay
        unchanged until the forward that reads it has started."""
        cur = torch.cuda.current_stream(self.device)
        k = self._next_buf
        self._next_buf ^= 1
        cs = self._copy_stream
        if self._buf_free[k] is not None:
            cs.wait_event(self._buf_free[k])
        else:
            cs.wait_stream(cur)
        with torch.cuda.stream(cs):
            self.x_ins[k].copy_(x, non_blocking=True)
            copied = torch.cuda.Event()
            copied.record(cs)
        cur.wait_event(copied)
        if self._graph is not None:
            self._graphs[k].replay()
        else:
            self._in_sel = k
            self.run()
            self._in_sel = 0
        done = torch.cuda.Event()
        done.record(cur)
        self._buf_free[k] = done
        return self.logits_bufs[k]

    def spikes(self, name):
        """Device buffer of a layer output by trace name (for tests)."""
        if name == "stem":
            return self.a0
        i, kind = name[1:].split(".")
        blk = self.blocks[int(i)]
        return {"sn1": blk["o1"], "ds": blk["id"], "out": blk["out"]}[kind]


def conv_layer_flops(layer: SparseConvBNLIF) -> int:
    """Dense-equivalent FLOPs 2*M*N*K of one fused layer (M = T*B*OH*OW)."""
    d = layer.desc
    m = d.T * d.B * layer.OH * layer.OW
    return 2 * m * d.Cout * d.KH * d.KW * d.Cin


def conv_layer_bytes(layer: SparseConvBNLIF, residual: bool, act_bytes: int = 2,
                     binary_out: bool = False) -> int:
    """Algorithmic HBM bytes of one fused layer: activations in (once), packed
    weights + metadata, outputs out, residual in.  Defaults count this
    library's fp16 tensors; ``act_bytes=1, binary_out=True`` counts the byte
    convention of 1-byte (FP8) activations and residuals and 1-bit spikes for
    a layer whose output is binary."""
    d = layer.desc
    n_in = d.T * d.B * d.H * d.W * d.Cin
    n_out = d.T * d.B * layer.OH * layer.OW * d.Cout
    w = rt.weight_bytes(d)
    out = n_out // 8 if binary_out else n_out * act_bytes
    return n_in * act_bytes + w + out + (n_out * act_bytes if residual else 0)


class SEWResNet18DVS(PlanModel):
    """SEW-ResNet-18 with the reference's ImageNet stem on event frames (the
    DVS configuration): ``models/sewresnet.py:140-143,190-210`` --
    conv1 7x7/2 (pad 3) + BN + LIF on every timestep's frame, MaxPool(3,2,1)
    of the spikes, four SEW stages (64/128/256/512, ADD), avgpool + mean over
    T + fc.

    Input ``[T, B, C, H, W]`` fp32 (time-major; the reference's 5-D input is
    ``[B, T, C, H, W]`` and is transposed first, ``:192-193``).
    """

    def __init__(self, params, *, T=16, batch=4, H=128, W=128, tau=2.0, v_threshold=1.0,
                 device="cuda", split_t=True):
        st = params["stem"]
        cout, cin, kh, kw = st["w"].shape
        super().__init__(T=T, batch=batch, in_shape=(T, batch, cin, H, W),
                         num_classes=params["fc_w"].shape[0], device=device)
        dev = self.device
        s, b = fold_bn(**st["bn"])
        self.stem_desc = rt.make_desc(T=T, B=batch, Cin=cin, H=H, W=W, Cout=cout, KH=kh, KW=kw,
                                      stride=2, pad=kh // 2, tau=tau, v_threshold=v_threshold)
        sh, sw = (H + 2 * (kh // 2) - kh) // 2 + 1, (W + 2 * (kw // 2) - kw) // 2 + 1
        # The stem's spikes go only to the max pool: bit-packed between the
        # two where the tensor-core stem serves it (up to 64 channels, K <= 192).
        bits = (rt.SNN_FLAG_SPIKE_BITS
                if cout % 16 == 0 and cout <= 64 and cin * kh * kw <= 192 else 0)
        self.stem_desc.flags = bits
        a0 = (self.buf((T * batch, sh, sw, cout // 8), torch.uint8) if bits
              else self.buf((T * batch, sh, sw, cout)))
        self.add(Node(STEM, "stem", [INPUT], a0, self.stem_desc,
                      (self.param(st["w"]), self.param(s), self.param(b)), (T, 0, 0, 0, 0)))
        ph, pw = pool_out(sh, 3, 2, 1), pool_out(sw, 3, 2, 1)
        p0 = self.buf((T * batch, ph, pw, cout))
        pd = glue_desc(T=T, B=batch, C=cout, H=sh, W=sw, neuron="none", k=3, stride=2, pad=1)
        pd.flags = bits
        self.add(Node(MAXPOOL, "maxpool", [a0], p0, pd))
        kw_ = dict(T=T, B=batch, tau=tau, v_threshold=v_threshold, device=dev)
        h, w_, x = ph, pw, p0

        def conv(name, layer, ins):
            # Long T on few images: 3x3 layers of >= 128 channels run in the
            # timestep-split form (all T*B images' GEMMs spread over the SMs,
            # then the neuron scan), measured 1.2-4.6x faster at T = 16 on 4
            # images, as are the 1x1 downsamples to >= 256 channels (1.4x);
            # the 64-channel layers and the first 1x1 downsample stay one-pass.
            ws = None
            d = layer.desc
            if split_t and T >= 8 and ((d.KH * d.KW > 1 and layer.Cout >= 128) or layer.Cout >= 256):
                ws = self.split_workspace(layer)
            return self.add(Node(CONV, name, ins, self.buf(layer.out_shape()), layer=layer,
                                 workspace=ws))

        for i, blk in enumerate(params["blocks"]):
            stride = blk["stride"]
            l1 = SparseConvBNLIF(blk["w1"], *fold_bn(**blk["bn1"]), H=h, W=w_, stride=stride,
                                 pad=1, **kw_)
            o1 = conv(f"b{i}.conv1", l1, [x])
            ident = x
            if "wd" in blk:
                ds = SparseConvBNLIF(blk["wd"], *fold_bn(**blk["bnd"]), H=h, W=w_,
                                     stride=stride, pad=0, **kw_)
                ident = conv(f"b{i}.ds", ds, [x])
            l2 = SparseConvBNLIF(blk["w2"], *fold_bn(**blk["bn2"]), H=l1.OH, W=l1.OW, stride=1,
                                 pad=1, **kw_)
            x = conv(f"b{i}.conv2", l2, [o1, ident])
            h, w_ = l1.OH, l1.OW
        c = params["blocks"][-1]["planes"]
        self.feat_hw, self.feat_c = h * w_, c
        self.add(Node(HEAD, "head", [x], LOGITS, None,
                      (self.param(params["fc_w"]), self.param(params["fc_b"])),
                      (T, batch, h * w_, c, self.num_classes)))
