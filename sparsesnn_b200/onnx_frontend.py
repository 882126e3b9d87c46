"""Plugin-mode ONNX front end: SNN graphs with the reference's fused neuron
ops in and out of this library's node plans.

* ``export_sew_resnet18(params, path, T)`` writes a SEW-ResNet-18 in the
  layout the reference's exporter produces in plugin mode
  (``sengine/tdl/transforms.py:899-…``, ``sengine/tdl/neuron_ops.py:62-68``):
  4-D ``(T*B, C, H, W)`` tensors, the stem's BN output repeated over T by a
  ``Tile``, one ``FusedLIFNeuron`` (attributes ``T_i, tau_f, v_threshold_f,
  v_reset_f, hard_reset_i``) after every BN, the SEW ``Add``, and the
  classifier tail ``GlobalAveragePool -> Flatten -> Gemm -> Reshape ->
  ReduceMean`` over T.
* ``load_plan(path, batch)`` parses such a file -- the op set the
  reference's parser reads (``sengine/parser.py:152-210``, neurons
  ``:327-368``) -- into a :class:`~sparsesnn_b200.netplan.PlanModel`:
  Conv -> BatchNormalization -> neuron [-> Add] chains become fused sparse
  layers (2:4 weights detected per ``validate_2_4_pattern``,
  ``sengine/optimizer.py:499-523``; other weights run dense), a stem conv
  with fewer than 4 input channels (the reference never prunes it,
  ``sengine/graph_slicer.py:106``) the stem kernel, MaxPool after a neuron the
  plain pool, ``Add -> neuron`` the Add+LIF glue, the tail the head kernel.

The ONNX bytes go through ``onnx_io`` (no ``onnx`` package here).
"""
from __future__ import annotations

import numpy as np

from . import onnx_io
from . import runtime as rt
from .layer import SparseConvBNLIF, fold_bn
from .netplan import ADD_LIF, CONV, HEAD, INPUT, LOGITS, LIF, MAXPOOL, STEM, Node, PlanModel, glue_desc

NEURON_OPS = {"FusedLIFNeuron": "lif", "FusedIFNeuron": "if"}


# ------------------------------------------------------------------ export
def export_sew_resnet18(params, path, T=4, batch=1, H=32, W=32, tau=2.0, v_threshold=1.0):
    """Write SEW-ResNet-18 (CIFAR stem; ``sew_resnet.init_params`` layout) as a
    plugin-mode ONNX file."""
    g = onnx_io.GraphWriter("sew_resnet18")
    cin = params["stem"]["w"].shape[1]
    g.input("input", (batch, cin, H, W))
    n = [0]

    def name(p):
        n[0] += 1
        return f"{p}_{n[0]}"

    def conv(x, w, stride, pad):
        wn = g.init(name("conv.weight"), w.astype(np.float32))
        y = name("conv")
        k = w.shape[2]
        g.node("Conv", [x, wn], [y], name=y, kernel_shape=[k, k], strides=[stride, stride],
               pads=[pad, pad, pad, pad], dilations=[1, 1], group=1)
        return y

    def bn(x, p):
        ins = [x] + [g.init(name(f"bn.{k}"), p[k].astype(np.float32))
                     for k in ("gamma", "beta", "mean", "var")]
        y = name("bn")
        g.node("BatchNormalization", ins, [y], name=y, epsilon=1e-5)
        return y

    def lif(x):
        y = name("lif")
        g.node("FusedLIFNeuron", [x], [y], name=y, domain="sengine", T_i=T, tau_f=float(tau),
               v_threshold_f=float(v_threshold), v_reset_f=0.0, hard_reset_i=1)
        return y

    st = params["stem"]
    h = bn(conv("input", st["w"], 1, st["w"].shape[2] // 2), st["bn"])
    reps = g.init("tile.repeats", np.array([T, 1, 1, 1], np.int64))
    tiled = name("tile")
    g.node("Tile", [h, reps], [tiled], name=tiled)
    h = lif(tiled)
    for blk in params["blocks"]:
        s = blk["stride"]
        o1 = lif(bn(conv(h, blk["w1"], s, 1), blk["bn1"]))
        o2 = lif(bn(conv(o1, blk["w2"], 1, 1), blk["bn2"]))
        ident = lif(bn(conv(h, blk["wd"], s, 0), blk["bnd"])) if "wd" in blk else h
        y = name("add")
        g.node("Add", [o2, ident], [y], name=y)
        h = y
    gp, fl, gm, rs = name("gap"), name("flatten"), name("gemm"), name("reshape")
    g.node("GlobalAveragePool", [h], [gp], name=gp)
    g.node("Flatten", [gp], [fl], name=fl, axis=1)
    fw = g.init("fc.weight", params["fc_w"].astype(np.float32))
    fb = g.init("fc.bias", params["fc_b"].astype(np.float32))
    g.node("Gemm", [fl, fw, fb], [gm], name=gm, alpha=1.0, beta=1.0, transB=1)
    shp = g.init("reshape.shape", np.array([T, -1, params["fc_w"].shape[0]], np.int64))
    g.node("Reshape", [gm, shp], [rs], name=rs)
    g.node("ReduceMean", [rs], ["output"], name="temporal_mean", axes=[0], keepdims=0)
    g.output("output", (batch, params["fc_w"].shape[0]))
    return g.save(path, custom_domains=("", "sengine"))


# ------------------------------------------------------------------ import
def _attrs(node):
    out = {}
    for a in node.attribute:
        if a.type == onnx_io.A_FLOAT:
            out[a.name] = a.f
        elif a.type == onnx_io.A_INT:
            out[a.name] = a.i
        elif a.type == onnx_io.A_INTS:
            out[a.name] = list(a.ints)
        elif a.type == onnx_io.A_FLOATS:
            out[a.name] = list(a.floats)
    return out


def neuron_params(node):
    """(kind, T, tau, v_threshold, v_reset) of a fused neuron node, with the
    reference parser's attribute names and defaults (``sengine/parser.py:327-368``)."""
    a = _attrs(node)
    kind = NEURON_OPS[node.op_type]
    T = int(a.get("T_i", a.get("T", 4)))
    tau = float(a.get("tau_f", a.get("tau", 2.0))) if kind == "lif" else float("inf")
    if not int(a.get("hard_reset_i", a.get("hard_reset", 1))):
        raise ValueError(f"{node.name}: soft reset is not supported")
    return (kind, T, tau, float(a.get("v_threshold_f", a.get("v_threshold", 1.0))),
            float(a.get("v_reset_f", a.get("v_reset", 0.0))))


def is_2_4(w, tol=1e-10):
    """The reference's 2:4 test: groups of four along C_in within each tap
    ('columnslast' order), ``|w| < tol`` counting as zero."""
    f = w.shape[0]
    g = np.transpose(w, (0, 2, 3, 1)).reshape(f, -1)
    if g.shape[1] % 4:
        return False
    return bool(((np.abs(g.reshape(f, -1, 4)) >= tol).sum(axis=2) <= 2).all())


class OnnxPlanModel(PlanModel):
    """A node plan parsed from a plugin-mode ONNX file (see module doc)."""

    def __init__(self, path, *, batch, device="cuda"):
        m = onnx_io.load(path)
        g = m.graph
        inits = {t.name: onnx_io.to_array(t) for t in g.initializer}
        consumers = {}
        for nd in g.node:
            for x in nd.input:
                consumers.setdefault(x, []).append(nd)
        producer = {o: nd for nd in g.node for o in nd.output}
        in_dims = [d.dim_value for d in g.input[0].type.tensor_type.shape.dim]
        _, cin, H, W = in_dims
        T = next(neuron_params(nd)[1] for nd in g.node if nd.op_type in NEURON_OPS)
        fc = next(nd for nd in g.node if nd.op_type == "Gemm")
        nc = inits[fc.input[1]].shape[0]
        super().__init__(T=T, batch=batch, in_shape=(batch, cin, H, W), num_classes=nc,
                         device=device)
        dev = self.device
        self.onnx_nodes = len(g.node)
        shapes = {}                  # tensor name -> (C, H, W) of one (t, b) image
        bufs = {}                    # tensor name -> device buffer
        done = set()

        def only_consumer(x, op):
            cs = consumers.get(x, [])
            return cs[0] if len(cs) == 1 and cs[0].op_type in op else None

        def neuron_kw(nd):
            kind, _, tau, vth, vr = neuron_params(nd)
            return dict(neuron=kind, tau=tau if kind == "lif" else 2.0, v_threshold=vth, v_reset=vr)

        for nd in g.node:
            if id(nd) in done:
                continue
            op = nd.op_type
            if op == "Conv":
                a = _attrs(nd)
                w = inits[nd.input[1]].astype(np.float32)
                k, s = w.shape[2], a.get("strides", [1, 1])[0]
                pad = a.get("pads", [0, 0, 0, 0])[0]
                bnn = only_consumer(nd.output[0], ("BatchNormalization",))
                if bnn is None:
                    raise ValueError(f"{nd.name}: a conv must feed a BatchNormalization")
                bp = [inits[x] for x in bnn.input[1:5]]
                eps = _attrs(bnn).get("epsilon", 1e-5)
                conv_bias = inits[nd.input[2]] if len(nd.input) > 2 and nd.input[2] else None
                scale, bias = fold_bn(*bp, eps=eps, conv_bias=conv_bias)
                nxt = only_consumer(bnn.output[0], ("Tile",) + tuple(NEURON_OPS))
                src = nd.input[0]
                if src == g.input[0].name:
                    # stem: conv + BN [+ Tile over T] + neuron on the images
                    tile = nxt if nxt is not None and nxt.op_type == "Tile" else None
                    neu = only_consumer(tile.output[0], tuple(NEURON_OPS)) if tile else nxt
                    kw = neuron_kw(neu)
                    desc = rt.make_desc(T=T, B=batch, Cin=cin, H=H, W=W, Cout=w.shape[0], KH=k, KW=k,
                                        stride=s, pad=pad, neuron=kw["neuron"], tau=kw["tau"],
                                        v_threshold=kw["v_threshold"], v_reset=kw["v_reset"])
                    oh, ow = (H + 2 * pad - k) // s + 1, (W + 2 * pad - k) // s + 1
                    out = self.buf((T * batch, oh, ow, w.shape[0]))
                    self.add(Node(STEM, nd.name, [INPUT], out, desc,
                                  (self.param(w), self.param(scale), self.param(bias)),
                                  (1 if tile else T, 0, 0, 0, 0)))
                    done.update({id(bnn), id(neu)} | ({id(tile)} if tile else set()))
                    bufs[neu.output[0]] = out
                    shapes[neu.output[0]] = (w.shape[0], oh, ow)
                    continue
                neu = nxt
                if neu is None or neu.op_type not in NEURON_OPS:
                    raise ValueError(f"{nd.name}: BN must feed a fused neuron")
                c, h, w_ = shapes[src]
                dense = not is_2_4(w)
                layer = SparseConvBNLIF(w, scale, bias, T=T, B=batch, H=h, W=w_, stride=s, pad=pad,
                                        device=dev, dense=dense, **neuron_kw(neu))
                ins = [bufs[src]]
                out_name = neu.output[0]
                add = only_consumer(out_name, ("Add",))
                if add is not None:
                    # SEW Add: fused into whichever of its two operands' convs
                    # comes second (the sum is exact either way)
                    other = [x for x in add.input if x != out_name][0]
                    if other in bufs:
                        ins.append(bufs[other])
                        out_name = add.output[0]
                        done.add(id(add))
                out = self.buf(layer.out_shape())
                self.add(Node(CONV, nd.name, ins, out, layer=layer))
                done.update({id(bnn), id(neu)})
                bufs[out_name] = out
                shapes[out_name] = (w.shape[0], layer.OH, layer.OW)
            elif op in NEURON_OPS:
                src = nd.input[0]
                prod = producer.get(src)
                c, h, w_ = shapes[src]
                kw = neuron_kw(nd)
                d = glue_desc(T=T, B=batch, C=c, H=h, W=w_, **kw)
                out = self.buf((T * batch, h, w_, c))
                if prod is not None and prod.op_type == "Add":
                    a, b = prod.input
                    self.add(Node(ADD_LIF, nd.name, [bufs[a], bufs[b]], out, d))
                else:
                    self.add(Node(LIF, nd.name, [bufs[src]], out, d))
                bufs[nd.output[0]] = out
                shapes[nd.output[0]] = (c, h, w_)
            elif op == "Add":
                # an Add not fused into a conv: fused with the neuron that follows it
                if only_consumer(nd.output[0], tuple(NEURON_OPS)) is None:
                    raise ValueError(f"{nd.name}: an unfused Add must feed a neuron")
                shapes[nd.output[0]] = shapes[nd.input[0]]
            elif op == "MaxPool":
                a = _attrs(nd)
                k, s = a["kernel_shape"][0], a.get("strides", [1, 1])[0]
                pad = a.get("pads", [0, 0, 0, 0])[0]
                c, h, w_ = shapes[nd.input[0]]
                oh, ow = (h + 2 * pad - k) // s + 1, (w_ + 2 * pad - k) // s + 1
                out = self.buf((T * batch, oh, ow, c))
                self.add(Node(MAXPOOL, nd.name, [bufs[nd.input[0]]], out,
                              glue_desc(T=T, B=batch, C=c, H=h, W=w_, neuron="none", k=k, stride=s,
                                        pad=pad)))
                bufs[nd.output[0]] = out
                shapes[nd.output[0]] = (c, oh, ow)
            elif op == "GlobalAveragePool":
                c, h, w_ = shapes[nd.input[0]]
                fw, fb = inits[fc.input[1]], inits[fc.input[2]]
                if not _attrs(fc).get("transB", 0):
                    fw = fw.T
                self.feat_hw, self.feat_c = h * w_, c
                self.add(Node(HEAD, "head", [bufs[nd.input[0]]], LOGITS, None,
                              (self.param(np.ascontiguousarray(fw, np.float32)),
                               self.param(fb.astype(np.float32))),
                              (T, batch, h * w_, c, nc)))
            elif op in ("Flatten", "Gemm", "Reshape", "ReduceMean", "Tile", "BatchNormalization"):
                continue            # the head tail, or consumed above
            else:
                raise ValueError(f"unsupported op {op} ({nd.name})")


def load_plan(path, batch, device="cuda"):
    """A node-plan model from a plugin-mode ONNX file."""
    return OnnxPlanModel(path, batch=batch, device=device)
