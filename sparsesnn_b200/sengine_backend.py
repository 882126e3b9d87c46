"""sengine-facing backend: a drop-in for the reference's fused-kernel compile
and export steps, targeting libsnnb200.so.

Reference boundary (all paths inside the SparseSNN repo):

* ``TileLangCompiler.compile_all`` (``sengine/build/tilelang_compiler.py:404-491``)
  returns ``{node_id: callable}``; for fused anchors it calls
  ``_get_fused_conv_bn_if`` (``:542-651``) whose callable has the TileLang
  ``out_idx=[-1]`` shape ``kern(data, weight, state, bn_scale, bn_bias) -> out``.
  ``B200Compiler.compile_all`` / ``get_fused_conv_bn_lif`` return callables with
  the same argument order and meaning (``weight`` is the packed 2:4 blob, see
  ``FusedKernel.pack``).
* ``export_all_kernels(kernels, ir, build_dir, nvcc, arch)``
  (``sengine/build/export_standalone.py:106-210``) writes one ``.so`` per kernel
  exporting ``int init(void)`` and ``int call(data, weight, state, scale,
  bias, out, cudaStream_t)`` -- the ABI the C executor dlopens
  (``sengine/csrc/cpp_executor.cu:631-662``, call site ``:909-913``).
  ``export_all_kernels`` here writes a tiny C shim per node that binds the
  layer geometry and forwards to ``snn_conv_forward``; the shim links
  libsnnb200.so and keeps the exact reference symbol names.

Fusion decisions are read from the reference IR annotations set by
``apply_fusion`` (``sengine/fusion_strategy.py:55-179``):
``node.assigned_kernel`` and ``node.extra_attrs['absorbed_nids' |
'residual_nid']``.  Nodes are duck-typed (``id``, ``conv_params``,
``input_shapes``, ``neuron_params``), so the reference ``sengine.ir.Node`` or
any object with the same fields works.
"""
from __future__ import annotations

import os
import subprocess
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from . import runtime as rt

# Reference KernelVariant names (sengine/ir.py:51-95) this backend implements.
FUSED_CONV_VARIANTS = ("TileLangFusedConvBNIF", "TileLangFusedConv1x1BNIF",
                       "FusedSparseConvBNLIF", "TileLangLinearBNLIF")
PKG_DIR = Path(__file__).resolve().parent


def _variant_name(v) -> str:
    return getattr(v, "name", str(v)).split(".")[-1]


def _neurons_of(node, ir=None):
    """Neuron kinds/params of a fused anchor, in slice order: its own
    ``neuron_params``, then the absorbed LIF/IF nodes' (reference
    ``tilelang_compiler.py:566-575``).  Each is ``(kind, tau, v_threshold,
    v_reset)``; a slice without a neuron gets the default LIF."""
    cands = []
    if getattr(node, "neuron_params", None) is not None:
        cands.append(node.neuron_params)
    if ir is not None:
        for a in node.extra_attrs.get("absorbed_nids", []):
            n = ir.nodes.get(a) if hasattr(ir, "nodes") else None
            if n is not None and getattr(n, "neuron_params", None) is not None:
                cands.append(n.neuron_params)
    out = []
    for npar in cands:
        kind = _variant_name(getattr(npar, "neuron_type", "LIF")).upper()
        if kind in ("LIF", "IF"):
            tau = float(getattr(npar, "tau", 2.0) or 2.0)
            out.append((kind.lower(), tau, float(npar.v_threshold), float(npar.v_reset)))
    return out or [("lif", 2.0, 1.0, 0.0)]


def _neuron_of(node, ir=None):
    """The first neuron of a fused anchor (see ``_neurons_of``)."""
    return _neurons_of(node, ir)[0]


_NEURON_OPS = ("LIF", "IF")


def _res_mode_of(node):
    """Residual epilogue of a fused anchor from the slicer's pattern string
    (``extra_attrs['fusion_slice']``, op names joined by ``+``,
    ``sengine/graph_slicer.py:152-177``; template table
    ``sengine/kernels/interleaved_templates.py:371-397``): ``None`` without
    an absorbed Add, ``"add_after"`` for ``X+LIF+Add``, ``"add_before"`` for
    ``X+Add+LIF`` and ``"two_neuron"`` for ``X+IF+Add+LIF``.  An anchor with a
    residual but no pattern string is the SEW ``add_after``."""
    if node.extra_attrs.get("residual_nid") is None:
        return None
    pat = node.extra_attrs.get("fusion_slice")
    if not pat:
        return "add_after"
    ops = [o for o in str(pat).split("+")[1:] if o in _NEURON_OPS or o == "Add"]
    if len(ops) == 2 and ops[0] in _NEURON_OPS and ops[1] == "Add":
        return "add_after"
    if len(ops) == 2 and ops[0] == "Add" and ops[1] in _NEURON_OPS:
        return "add_before"
    if len(ops) == 3 and ops[1] == "Add" and ops[0] in _NEURON_OPS and ops[2] in _NEURON_OPS:
        return "two_neuron"
    raise NotImplementedError(f"fused pattern {pat!r} has no B200 epilogue")


@dataclass
class LayerGeometry:
    T: int
    B: int
    Cin: int
    H: int
    W: int
    Cout: int
    KH: int
    KW: int
    stride: int
    pad: int


class FusedKernel:
    """Callable with the reference TileLang kernel signatures
    ``kern(data, weight, state, bn_scale, bn_bias[, residual]) -> out``
    (``interleaved_templates.py:95-288``) and, for two neurons around the
    Add, ``kern(data, weight, state1, state2, bn_scale, bn_bias, residual)
    -> out`` (``:297-364``).

    ``data`` (T*B, H, W, Cin) fp16; ``state`` (B*OH*OW, Cout) fp32 membrane,
    read at start and overwritten with the final v (the reference kernels'
    behaviour, ``interleaved_templates.py:127-151``); output allocated by the
    callee (``out_idx=[-1]``).  ``res_mode`` (``None`` without a residual,
    else ``"add_after"``, ``"add_before"`` or ``"two_neuron"``) places the Add.
    """

    def __init__(self, geom: LayerGeometry, neuron="lif", tau=2.0, v_threshold=1.0,
                 v_reset=0.0, residual=False, res_mode=None, neuron2=None):
        self.geom = geom
        self.res_mode = res_mode or ("add_after" if residual else None)
        self.residual = self.res_mode is not None
        kind2, tau2, vth2, vr2 = neuron2 or ("lif", 2.0, 1.0, 0.0)
        self.desc = rt.make_desc(T=geom.T, B=geom.B, Cin=geom.Cin, H=geom.H, W=geom.W,
                                 Cout=geom.Cout, KH=geom.KH, KW=geom.KW, stride=geom.stride,
                                 pad=geom.pad, neuron=neuron, tau=tau,
                                 v_threshold=v_threshold, v_reset=v_reset,
                                 res_mode=self.res_mode or "add_after", neuron2=kind2,
                                 tau2=tau2, v_threshold2=vth2, v_reset2=vr2)
        self.OH, self.OW = rt.out_shape(self.desc)

    @property
    def key(self) -> str:
        g, d = self.geom, self.desc
        res = {None: "", "add_after": "_res", "add_before": "_addres",
               "two_neuron": f"_res2n{d.neuron2}t{d.tau2:g}v{d.v_threshold2:g}"}[self.res_mode]
        return (f"b200_sparse_conv_{g.Cin}_{g.Cout}_{g.KH}x{g.KW}_{g.H}x{g.W}_s{g.stride}"
                f"_B{g.B}_T{g.T}_n{d.neuron}t{d.tau:g}v{d.v_threshold:g}{res}")

    def pack(self, weight_fchw) -> np.ndarray:
        """Pruned fp32 ``[Cout, Cin, KH, KW]`` -> packed 2:4 blob (host uint8)."""
        w = np.asarray(weight_fchw, np.float32)
        if w.ndim == 2:
            w = w[:, :, None, None]
        return rt.pack_weight_24(self.desc, w)

    def __call__(self, data, weight, *args, out=None):
        import torch
        g = self.geom
        if out is None:
            out = torch.empty((g.T * g.B, self.OH, self.OW, g.Cout), dtype=torch.float16,
                              device=data.device)
        self.desc.flags = rt.SNN_FLAG_READ_STATE | rt.SNN_FLAG_WRITE_STATE
        s = torch.cuda.current_stream(data.device).cuda_stream
        lib = rt.load()
        if self.res_mode == "two_neuron":
            if len(args) != 5:
                raise TypeError("two-neuron kernel takes (data, weight, state1, state2, "
                                "bn_scale, bn_bias, residual)")
            state, state2, bn_scale, bn_bias, residual = args
            rt.check(lib.snn_conv_forward_res2(self.desc, data.data_ptr(), weight.data_ptr(),
                                               state.data_ptr(), state2.data_ptr(),
                                               bn_scale.data_ptr(), bn_bias.data_ptr(),
                                               residual.data_ptr(), out.data_ptr(), s))
            return out
        if len(args) not in (3, 4):
            raise TypeError("kernel takes (data, weight, state, bn_scale, bn_bias[, residual])")
        state, bn_scale, bn_bias = args[:3]
        residual = args[3] if len(args) == 4 else None
        if self.residual:
            if residual is None:
                raise ValueError("this fused node absorbed an Add: residual required")
            rt.check(lib.snn_conv_forward_res(self.desc, data.data_ptr(), weight.data_ptr(),
                                              state.data_ptr(), bn_scale.data_ptr(),
                                              bn_bias.data_ptr(), residual.data_ptr(),
                                              out.data_ptr(), s))
        else:
            rt.check(lib.snn_conv_forward(self.desc, data.data_ptr(), weight.data_ptr(),
                                          state.data_ptr(), bn_scale.data_ptr(),
                                          bn_bias.data_ptr(), out.data_ptr(), s))
        return out


class B200Compiler:
    """Builds fused-layer callables for the IR's fused anchors (the
    ``TileLangCompiler`` role for the fused sparse variants)."""

    def __init__(self, ir, T: int = 4, batch_size: int = 1):
        self.ir = ir
        self.T = T
        self.B = batch_size
        self._cache: dict[str, FusedKernel] = {}

    def _spatial(self, node):
        shp = node.input_shapes[0] if node.input_shapes else None
        if shp is None or len(shp) < 4:
            raise ValueError(f"node {node.id}: input shape unknown")
        return int(shp[-2]), int(shp[-1])          # NCHW (H, W), as the reference IR records

    def get_fused_conv_bn_lif(self, node) -> FusedKernel:
        """Mirror of ``_get_fused_conv_bn_if`` (``tilelang_compiler.py:542-651``)
        with the LIF semantics kept for 3x3 anchors too (the reference compiles
        IF there, ``:610-631``, which drops the absorbed neuron's decay)."""
        cp = node.conv_params
        H, W = self._spatial(node)
        neurons = _neurons_of(node, self.ir)
        kind, tau, vth, vr = neurons[0]
        geom = LayerGeometry(self.T, self.B, cp.in_channels, H, W, cp.out_channels,
                             cp.kernel_h, cp.kernel_w, cp.stride_h, cp.pad_h)
        res_mode = _res_mode_of(node)
        neuron2 = None
        if res_mode == "two_neuron":
            if len(neurons) < 2:
                raise ValueError(f"node {node.id}: two-neuron pattern without two neurons")
            neuron2 = neurons[1]
        k = FusedKernel(geom, kind, tau, vth, vr, res_mode=res_mode, neuron2=neuron2)
        return self._cache.setdefault(k.key, k)

    def compile_all(self) -> dict:
        """``{node_id: FusedKernel}`` for every fused anchor of the IR."""
        out = {}
        for nid, node in self.ir.nodes.items():
            if _variant_name(getattr(node, "assigned_kernel", "")) in FUSED_CONV_VARIANTS:
                out[nid] = self.get_fused_conv_bn_lif(node)
        return out


_SHIM = r"""/* Generated by sparsesnn_b200.sengine_backend.export_all_kernels: binds one
 * fused layer's geometry to libsnnb200 behind the reference's per-kernel ABI. */
#include "snn_b200.h"
static const snn_conv_desc D = {%(T)d, %(B)d, %(Cin)d, %(H)d, %(W)d, %(Cout)d, %(KH)d, %(KW)d,
                                %(stride)d, %(pad)d, %(neuron)d,
                                SNN_FLAG_READ_STATE | SNN_FLAG_WRITE_STATE,
                                (float)%(tau).9g, (float)%(vth).9g, (float)%(vr).9g,
                                %(res_mode)d, %(neuron2)d,
                                (float)%(tau2).9g, (float)%(vth2).9g, (float)%(vr2).9g};
int init(void) { return snn_init(); }
int call(void* data, void* weight, float* state, float* bn_scale, float* bn_bias, void* out,
         void* stream) {
  return snn_conv_forward(&D, data, weight, state, bn_scale, bn_bias, out, stream);
}
int call_res(void* data, void* weight, float* state, float* bn_scale, float* bn_bias,
             void* residual, void* out, void* stream) {
  return snn_conv_forward_res(&D, data, weight, state, bn_scale, bn_bias, residual, out, stream);
}
int call_res2(void* data, void* weight, float* state1, float* state2, float* bn_scale,
              float* bn_bias, void* residual, void* out, void* stream) {
  return snn_conv_forward_res2(&D, data, weight, state1, state2, bn_scale, bn_bias, residual,
                               out, stream);
}
"""


def write_shim(kern: FusedKernel, path: Path) -> Path:
    d = kern.desc
    path.write_text(_SHIM % dict(T=d.T, B=d.B, Cin=d.Cin, H=d.H, W=d.W, Cout=d.Cout, KH=d.KH,
                                 KW=d.KW, stride=d.stride, pad=d.pad, neuron=d.neuron,
                                 tau=d.tau, vth=d.v_threshold, vr=d.v_reset,
                                 res_mode=d.res_mode, neuron2=d.neuron2, tau2=d.tau2,
                                 vth2=d.v_threshold2, vr2=d.v_reset2))
    return path


def export_all_kernels(kernels: dict, ir=None, build_dir: str = "build/b200",
                       cc: str | None = None, arch: str = "sm_100a") -> dict:
    """Write and compile one shim ``.so`` per distinct kernel; returns
    ``{node_id: so_path}`` (reference ``export_standalone.py:106-210``).  The
    shims export ``init`` and ``call`` (plus ``call_res`` for the residual
    epilogues and ``call_res2`` for two neurons around the Add, whose
    argument order is the reference template's: data, weight, state1,
    state2, bn_scale, bn_bias, residual, out, stream) and load libsnnb200.so
    through an rpath."""
    if arch != "sm_100a":
        raise ValueError("libsnnb200 targets sm_100a only")
    cc = cc or os.environ.get("CC", "gcc")
    out_dir = Path(build_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    lib = rt.LIB_PATH
    include = PKG_DIR.parent / "include"
    by_key: dict[str, str] = {}
    result = {}
    for nid, kern in kernels.items():
        if kern.key not in by_key:
            src = write_shim(kern, out_dir / f"{kern.key}.c")
            so = out_dir / f"{kern.key}.so"
            subprocess.run([cc, "-shared", "-fPIC", "-O2", "-I", str(include), str(src), "-o", str(so),
                            "-L", str(lib.parent), "-l:" + lib.name,
                            "-Wl,-rpath," + str(lib.parent)], check=True)
            by_key[kern.key] = str(so)
        result[nid] = by_key[kern.key]
    return result
