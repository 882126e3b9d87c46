"""Whole-network forwards as a plan of fused nodes over preallocated buffers.

A model driver lists its forward as :class:`Node` records -- stem, fused
sparse conv (+ residual), max pool (+ neuron), neuron, Add + neuron,
attention core, head -- over device buffers it allocates once.  The same plan
serves the Python launch loop (one libsnnb200 call per node, capturable in a
CUDA graph) and the engine file of the native C++ executor
(``engine_file.save_engine``), so both run identical launches.

The counterpart in the reference is the sengine plan that
``sengine/build/buffer_planner.py`` assigns and ``sengine/csrc/cpp_executor.cu``
(``sengine_execute``, :883-1194) walks node by node.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import runtime as rt

# Node kinds (the engine file's op codes, csrc/snn_engine.cuh).
STEM, CONV, HEAD, ADD_LIF, MAXPOOL, LIF, ATTN = 1, 2, 3, 4, 5, 6, 7

INPUT = "input"      # the forward's images (input buffer of the current call)
LOGITS = "logits"    # the forward's logits buffer


@dataclass
class Node:
    kind: int
    name: str
    ins: list                      # input tensors (or INPUT)
    out: object                    # output tensor (or LOGITS)
    desc: rt.SnnConvDesc | None = None
    params: tuple = ()             # parameter tensors (device)
    ints: tuple = (0, 0, 0, 0, 0)
    layer: object = None           # CONV: the SparseConvBNLIF
    attn: dict = field(default_factory=dict)   # ATTN: N, heads, head_dim, scale
    workspace: object = None       # CONV: fp32 workspace of the timestep-split form, or None
    out2: object = None            # STEM: spikes of desc.neuron on the fp16 BN output (dual form)


class PlanModel:
    """A forward over a node plan: eager launch loop, two CUDA graphs (one per
    input buffer, each writing its own logits buffer) and the public call with
    the host-to-device copy on a copy stream."""

    def __init__(self, *, T, batch, in_shape, num_classes, device):
        self.T, self.B = T, batch
        self.device = torch.device(device)
        dev = self.device
        rt.check(rt.load().snn_init())
        self.in_shape = tuple(in_shape)
        self.x_ins = [torch.empty(self.in_shape, dtype=torch.float32, device=dev) for _ in range(2)]
        self.x_in = self.x_ins[0]
        self.num_classes = num_classes
        self.logits_bufs = [torch.empty((batch, num_classes), dtype=torch.float32, device=dev)
                            for _ in range(2)]
        self.logits = self.logits_bufs[0]
        self._in_sel = 0
        self._next_buf = 0
        self._copy_stream = torch.cuda.Stream(dev)
        self._buf_free = [None, None]
        self._graph = None
        self._graphs = []
        self.nodes: list[Node] = []

    # ------------------------------------------------------------ building
    def buf(self, shape, dtype=torch.float16):
        return torch.empty(tuple(shape), dtype=dtype, device=self.device)

    def param(self, arr):
        return torch.as_tensor(arr).to(self.device).contiguous()

    def add(self, node: Node):
        self.nodes.append(node)
        return node.out

    def split_workspace(self, layer):
        """The model's workspace for timestep-split layers, grown to fit
        ``layer`` (one buffer shared by every such layer: they run in turn)."""
        need = (layer.workspace_bytes() + 3) // 4
        if getattr(self, "_ws", None) is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.float32, device=self.device)
            for n in self.nodes:
                if n.workspace is not None:
                    n.workspace = self._ws
        return self._ws

    # ------------------------------------------------------------ launching
    def _t(self, x):
        if x is INPUT:
            return self.x_ins[self._in_sel]
        if x is LOGITS:
            return self.logits_bufs[self._in_sel]
        return x

    def _launch(self, n: Node):
        lib = rt.load()
        s = torch.cuda.current_stream(self.device).cuda_stream
        ins = [self._t(x) for x in n.ins]
        out = self._t(n.out)
        if n.kind == CONV:
            n.layer(ins[0], residual=ins[1] if len(ins) > 1 else None, out=out,
                    workspace=n.workspace)
        elif n.kind == STEM:
            w, sc, bi = n.params
            if n.out2 is not None:
                rt.check(lib.snn_stem_forward_dual(n.desc, n.ints[0], ins[0].data_ptr(),
                                                   w.data_ptr(), sc.data_ptr(), bi.data_ptr(),
                                                   out.data_ptr(), n.out2.data_ptr(), s))
            else:
                rt.check(lib.snn_stem_forward(n.desc, n.ints[0], ins[0].data_ptr(), w.data_ptr(),
                                              sc.data_ptr(), bi.data_ptr(), out.data_ptr(), s))
        elif n.kind == HEAD:
            fw, fb = n.params
            T, B, HW, C, NC = n.ints
            rt.check(lib.snn_head_forward(T, B, HW, C, NC, ins[0].data_ptr(), fw.data_ptr(),
                                          fb.data_ptr(), out.data_ptr(), s))
        elif n.kind == ADD_LIF:
            rt.check(lib.snn_add_lif_forward(n.desc, ins[0].data_ptr(), ins[1].data_ptr(), None,
                                             out.data_ptr(), s))
        elif n.kind == MAXPOOL:
            rt.check(lib.snn_maxpool_lif_forward(n.desc, ins[0].data_ptr(), None, out.data_ptr(), s))
        elif n.kind == LIF:
            rt.check(lib.snn_lif_forward(n.desc, ins[0].data_ptr(), None, out.data_ptr(), s))
        elif n.kind == ATTN:
            a, d = n.attn, n.desc
            if a.get("packed"):                          # one [T*B][N][3C] q | k | v tensor
                cb = a["heads"] * a["head_dim"] * 2
                q = ins[0].data_ptr()
                qkv, flags = (q, q + cb, q + 2 * cb), rt.SNN_FLAG_QKV_PACKED
            else:
                qkv, flags = tuple(x.data_ptr() for x in ins), 0
            rt.check(lib.snn_spikformer_attn_forward(
                d.T, d.B, a["N"], a["heads"], a["head_dim"], a["scale"], d.tau, d.v_threshold,
                d.v_reset, flags, *qkv, None, out.data_ptr(), s))
        else:
            raise ValueError(f"unknown node kind {n.kind}")

    def launches(self):
        """(name, callable) for every kernel launch of one forward, in order."""
        return [(n.name, (lambda n=n: self._launch(n))) for n in self.nodes]

    def conv_layers(self):
        return [n.layer for n in self.nodes if n.kind == CONV]

    def run(self):
        """One forward from input buffer ``_in_sel`` into its logits buffer."""
        for n in self.nodes:
            self._launch(n)
        return self.logits_bufs[self._in_sel]

    def capture(self, warmup=3):
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
        self._graphs[buf].replay()
        return self.logits_bufs[buf]

    def __call__(self, x):
        """Public API: images (host or device, fp32, ``in_shape``) -> logits
        (device tensor on the current stream, valid until the call after next).
        Pinned host images are copied on a copy stream into the input buffer
        the previous forward is not reading."""
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

    def buffer(self, name):
        """Output tensor of the node called ``name`` (for tests)."""
        for n in self.nodes:
            if n.name == name:
                return self._t(n.out)
        raise KeyError(name)


def glue_desc(*, T, B, C, H, W, neuron="lif", k=1, stride=1, pad=0, tau=2.0, v_threshold=1.0,
              v_reset=0.0):
    """Descriptor of a glue node (C channels, window k for pools)."""
    return rt.make_desc(T=T, B=B, Cin=C, H=H, W=W, Cout=C, KH=k, KW=k, stride=stride, pad=pad,
                        neuron=neuron, tau=tau, v_threshold=v_threshold, v_reset=v_reset)


def pool_out(h, k, s, p):
    return (h + 2 * p - k) // s + 1


def conv_flops(layer) -> int:
    """Dense-equivalent FLOPs 2*M*N*K of one fused layer (M = T*B*OH*OW)."""
    d = layer.desc
    return 2 * d.T * d.B * layer.OH * layer.OW * d.Cout * d.KH * d.KW * d.Cin


def desc_copy(d):
    return rt.SnnConvDesc.from_buffer_copy(bytes(d))


__all__ = ["Node", "PlanModel", "STEM", "CONV", "HEAD", "ADD_LIF", "MAXPOOL", "LIF", "ATTN",
           "INPUT", "LOGITS", "glue_desc", "pool_out", "conv_flops", "desc_copy"]
