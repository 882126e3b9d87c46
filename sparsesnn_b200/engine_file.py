"""Engine files for the native executor (``snn_engine_*`` in libsnnb200).

``save_engine(model, path)`` writes a model replica as an engine file: the
fused nodes of one forward in execution order (for SEW-ResNet-18: stem, per
block conv1 / downsample / conv2 with the SEW residual, head; for the
node-plan models -- DVS SEW-ResNet-18, MS-ResNet-34, Spikformer -- their
plan), the byte size of every activation, and one blob with the packed 2:4
weights, folded BN scale/bias, stem and FC parameters.  ``Engine`` loads such a file
through the C-ABI and runs it without Python in the loop (the node loop and
its CUDA graph are C++).

The layout is this library's own (the reference's ``.sengine``,
``sengine/build/sengine_io.py:33-38``, binds TileLang kernels rebuilt from
tuning caches); see ``csrc/snn_engine.cuh`` for the record formats.
"""
from __future__ import annotations

import ctypes
import struct
from pathlib import Path

import numpy as np

from . import runtime as rt

MAGIC = b"SNNE"
VERSION = 2
NO_TENSOR = 0xFFFFFFFF
OP_STEM, OP_CONV, OP_HEAD, OP_ADD_LIF, OP_MAXPOOL_LIF, OP_LIF, OP_ATTN = 1, 2, 3, 4, 5, 6, 7
OP_CONV_TSPLIT = 8
F16, F32 = 0, 1
_ALIGN = 256


class _Writer:
    def __init__(self):
        self.tensors = []          # (bytes, dtype)
        self.nodes = []            # packed node records
        self.blob = bytearray()

    def tensor(self, nbytes, dtype):
        self.tensors.append((int(nbytes), dtype))
        return len(self.tensors) - 1

    def param(self, arr):
        off = (len(self.blob) + _ALIGN - 1) // _ALIGN * _ALIGN
        self.blob.extend(b"\0" * (off - len(self.blob)))
        self.blob.extend(np.ascontiguousarray(arr).tobytes())
        return off

    def node(self, op, in0, in1, out, desc=None, p=(0, 0, 0, 0), i=(0, 0, 0, 0, 0)):
        d = bytes(desc) if desc is not None else bytes(ctypes.sizeof(rt.SnnConvDesc))
        rec = struct.pack("<4I", op, in0, in1, out) + d + struct.pack("<4Q", *p) + \
            struct.pack("<5i", *i) + b"\0" * 12
        assert len(rec) == 160
        self.nodes.append(rec)

    def write(self, path, inp, outp, T, B):
        tens = b"".join(struct.pack("<QII", n, dt, 0) for n, dt in self.tensors)
        body = tens + b"".join(self.nodes) + bytes(self.blob)
        total = 64 + len(body)
        hdr = MAGIC + struct.pack("<7I", VERSION, len(self.tensors), len(self.nodes), inp, outp, T, B)
        hdr += struct.pack("<2Q", len(self.blob), total) + b"\0" * 16
        assert len(hdr) == 64
        Path(path).write_bytes(hdr + body)


def _conv_desc(layer):
    d = rt.SnnConvDesc.from_buffer_copy(bytes(layer.desc))
    # the layer's own flags (dense weights, general kernel), no membrane
    # flags: the membrane starts at zero every forward
    d.flags = layer.base_flags
    return d


def save_plan(model, path):
    """Write a node-plan model (``netplan.PlanModel``: SEW-ResNet-18 DVS,
    MS-ResNet-34, Spikformer) as an engine file: one engine tensor per device
    buffer (views of a buffer map to it), the nodes in plan order."""
    from . import netplan as npl
    w = _Writer()
    T, B = model.T, model.B
    ids = {}

    def tid(x):
        if x is npl.INPUT:
            key = ("input",)
            if key not in ids:
                ids[key] = w.tensor(model.x_ins[0].numel() * 4, F32)
            return ids[key]
        if x is npl.LOGITS:
            key = ("logits",)
            if key not in ids:
                ids[key] = w.tensor(model.logits.numel() * 4, F32)
            return ids[key]
        st = x.untyped_storage()
        if x.storage_offset() != 0 or x.numel() * x.element_size() != st.nbytes():
            raise ValueError("plan tensors must be whole buffers (or views of whole buffers)")
        key = st.data_ptr()
        if key not in ids:
            ids[key] = w.tensor(st.nbytes(), F32 if x.dtype.is_floating_point and x.element_size() == 4
                                else F16)
        return ids[key]

    P = lambda t: w.param(t.detach().cpu().numpy())  # noqa: E731
    kinds = {npl.STEM: OP_STEM, npl.CONV: OP_CONV, npl.HEAD: OP_HEAD, npl.ADD_LIF: OP_ADD_LIF,
             npl.MAXPOOL: OP_MAXPOOL_LIF, npl.LIF: OP_LIF, npl.ATTN: OP_ATTN}
    for n in model.nodes:
        ins = [tid(x) for x in n.ins]
        out = tid(n.out)
        in1 = ins[1] if len(ins) > 1 else NO_TENSOR
        if n.kind == npl.CONV:
            L = n.layer
            if n.workspace is not None:
                w.node(OP_CONV_TSPLIT, ins[0], in1, out, _conv_desc(L),
                       (P(L.weight_blob), P(L.bn_scale), P(L.bn_bias), 0),
                       (tid(n.workspace), 0, 0, 0, 0))
            else:
                w.node(OP_CONV, ins[0], in1, out, _conv_desc(L),
                       (P(L.weight_blob), P(L.bn_scale), P(L.bn_bias), 0))
        elif n.kind == npl.STEM:                         # dual form: in1 = the spike output
            w.node(OP_STEM, ins[0], NO_TENSOR if n.out2 is None else tid(n.out2), out, n.desc,
                   tuple(P(t) for t in n.params) + (0,), n.ints)
        elif n.kind == npl.HEAD:
            w.node(OP_HEAD, ins[0], NO_TENSOR, out, None, (P(n.params[0]), P(n.params[1]), 0, 0),
                   n.ints)
        elif n.kind == npl.ATTN:
            d = rt.SnnConvDesc.from_buffer_copy(bytes(n.desc))
            d.tau2 = n.attn["scale"]
            if n.attn.get("packed"):                     # q | k | v blocks of one tensor
                d.flags = rt.SNN_FLAG_QKV_PACKED
                w.node(OP_ATTN, ins[0], ins[0], out, d,
                       i=(ins[0], n.attn["N"], n.attn["heads"], n.attn["head_dim"], 0))
            else:
                d.flags = 0
                w.node(OP_ATTN, ins[0], ins[1], out, d,
                       i=(ins[2], n.attn["N"], n.attn["heads"], n.attn["head_dim"], 0))
        else:
            d = rt.SnnConvDesc.from_buffer_copy(bytes(n.desc))
            d.flags = n.desc.flags & rt.SNN_FLAG_SPIKE_BITS   # a pool of bit-packed spikes
            w.node(kinds[n.kind], ins[0], in1, out, d)
    w.write(path, tid(npl.INPUT), tid(npl.LOGITS), T, B)
    return path


def save_engine(model, path):
    """Write ``model`` as an engine file at ``path`` (a SEWResNet18 replica,
    or any node-plan model)."""
    if hasattr(model, "nodes"):
        return save_plan(model, path)
    w = _Writer()
    T, B = model.T, model.B
    cin = model.x_in.shape[1]
    images = w.tensor(B * cin * model.H * model.W * 4, F32)
    a0 = w.tensor(model.a0.numel() * 2, F16)
    sd = model.stem_desc
    w.node(OP_STEM, images, NO_TENSOR, a0, sd,
           (w.param(model.stem_w.cpu().numpy()), w.param(model.stem_scale.cpu().numpy()),
            w.param(model.stem_bias.cpu().numpy()), 0), (1, 0, 0, 0, 0))

    def conv(layer, src, res, dst):
        w.node(OP_CONV, src, NO_TENSOR if res is None else res, dst, _conv_desc(layer),
               (w.param(layer.weight_blob.cpu().numpy()), w.param(layer.bn_scale.cpu().numpy()),
                w.param(layer.bn_bias.cpu().numpy()), 0))

    h = a0
    for blk in model.blocks:
        o1 = w.tensor(blk["o1"].numel() * 2, F16)
        conv(blk["l1"], h, None, o1)
        ident = h
        if blk["ds"] is not None:
            ident = w.tensor(blk["id"].numel() * 2, F16)
            conv(blk["ds"], h, None, ident)
        out = w.tensor(blk["out"].numel() * 2, F16)
        conv(blk["l2"], o1, ident, out)
        h = out
    logits = w.tensor(B * model.num_classes * 4, F32)
    w.node(OP_HEAD, h, NO_TENSOR, logits, None,
           (w.param(model.fc_w.cpu().numpy()), w.param(model.fc_b.cpu().numpy()), 0, 0),
           (T, B, model.feat_hw, model.feat_c, model.num_classes))
    w.write(path, images, logits, T, B)
    return path


def check_file(path):
    """(nodes, tensors) of a valid engine file; raises SnnError otherwise."""
    lib = rt.load()
    n = ctypes.c_int32(0)
    t = ctypes.c_int32(0)
    rt.check(lib.snn_engine_check_file(str(path).encode(), ctypes.byref(n), ctypes.byref(t)))
    return n.value, t.value


class Engine:
    """A loaded engine file (C++ node loop, optional CUDA graph)."""

    def __init__(self, path):
        self._lib = rt.load()
        h = ctypes.c_void_p()
        rt.check(self._lib.snn_engine_load(str(path).encode(), ctypes.byref(h)))
        self._h = h
        T, B = ctypes.c_int32(), ctypes.c_int32()
        ib, ob = ctypes.c_size_t(), ctypes.c_size_t()
        rt.check(self._lib.snn_engine_io(h, ctypes.byref(T), ctypes.byref(B), ctypes.byref(ib),
                                         ctypes.byref(ob)))
        self.T, self.B, self.image_bytes, self.logit_bytes = T.value, B.value, ib.value, ob.value

    def capture(self, stream):
        """Capture the node loop on ``stream`` (a torch.cuda.Stream or raw
        handle) into a CUDA graph that later runs replay."""
        s = getattr(stream, "cuda_stream", stream)
        rt.check(self._lib.snn_engine_capture(self._h, ctypes.c_void_p(s)))

    def run(self, images_ptr, logits_ptr, stream):
        """One forward: raw pointers (host or device; 0 = engine buffer) and a
        stream handle; asynchronous on that stream."""
        s = getattr(stream, "cuda_stream", stream)
        rt.check(self._lib.snn_engine_run(self._h, ctypes.c_void_p(images_ptr or None),
                                          ctypes.c_void_p(logits_ptr or None), ctypes.c_void_p(s)))

    def close(self):
        if self._h:
            self._lib.snn_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
