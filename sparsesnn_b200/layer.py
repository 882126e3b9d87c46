"""Torch-facing wrappers of the fused layer (device memory via torch tensors).

``SparseConvBNLIF`` owns one layer's packed 2:4 weight blob and BN
scale/bias on the GPU and launches the fused kernel on the current torch
stream.  The data layouts are the reference sengine ones:
data ``(T*B, H, W, Cin)`` fp16, state ``(B*OH*OW, Cout)`` fp32,
output ``(T*B, OH, OW, Cout)`` (reference
``sengine/kernels/interleaved_templates.py:95-154``).
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import runtime as rt


def fold_bn(gamma, beta, mean, var, eps=1e-5, conv_bias=None):
    """BN -> per-channel ``(scale, bias)`` kept out of the weights.

    Restates reference ``sengine/optimizer.py:160-183``: float64 math,
    ``scale = gamma/sqrt(var+eps)``, ``bias = scale*(b - mean) + beta``,
    stored as float32; the weight is NOT scaled (``:168``).
    """
    g = np.asarray(gamma, np.float64)
    s = g / np.sqrt(np.asarray(var, np.float64) + eps)
    b = np.zeros_like(s) if conv_bias is None else np.asarray(conv_bias, np.float64)
    bias = s * (b - np.asarray(mean, np.float64)) + np.asarray(beta, np.float64)
    return s.astype(np.float32), bias.astype(np.float32)


def _np(x):
    if isinstance(x, torch.Tensor):
        return x.detach().cpu().numpy()
    return np.asarray(x)


class SparseConvBNLIF:
    """One fused 2:4-sparse Conv(+Linear) + BN + LIF/IF layer over T steps.

    ``res_mode`` says where a residual passed to ``__call__`` enters:
    ``"add_after"`` (SEW ADD, ``out = spike + residual``), ``"add_before"``
    (the neuron integrates ``bn + residual``) or ``"two_neuron"`` (``out =
    neuron2(spike + residual)``, second membrane ``state2``; ``neuron2``,
    ``tau2``, ``v_threshold2``, ``v_reset2`` describe that neuron).

    ``neuron="none"`` gives the fp32 BN output, ``"none_f16"`` the fp16 BN
    output (with a residual: ``out = bn + residual``).  ``dense=True`` takes
    an unpruned weight and runs it as two 2:4 halves (``SNN_FLAG_DENSE``).
    """

    def __init__(self, weight, bn_scale, bn_bias, *, T, B, H, W, stride=1, pad=None,
                 neuron="lif", tau=2.0, v_threshold=1.0, v_reset=0.0, device="cuda",
                 force_generic=False, res_mode="add_after", neuron2="lif", tau2=2.0,
                 v_threshold2=1.0, v_reset2=0.0, dense=False):
        w = _np(weight).astype(np.float32)
        if w.ndim == 2:                       # Linear [out, in] -> 1x1 conv
            w = w[:, :, None, None]
        cout, cin, kh, kw = w.shape
        self.base_flags = (rt.SNN_FLAG_FORCE_GENERIC if force_generic else 0) | \
            (rt.SNN_FLAG_DENSE if dense else 0)
        self.dense = dense
        self.neuron = neuron
        self.desc = rt.make_desc(T=T, B=B, Cin=cin, H=H, W=W, Cout=cout, KH=kh, KW=kw,
                                 flags=self.base_flags,
                                 stride=stride, pad=(kh // 2 if pad is None else pad),
                                 neuron=neuron, tau=tau, v_threshold=v_threshold,
                                 v_reset=v_reset, res_mode=res_mode, neuron2=neuron2,
                                 tau2=tau2, v_threshold2=v_threshold2, v_reset2=v_reset2)
        self.res_mode = res_mode
        self.OH, self.OW = rt.out_shape(self.desc)
        blob = rt.pack_weight_24(self.desc, w)
        self.device = torch.device(device)
        self.weight_blob = torch.from_numpy(blob).to(self.device)
        self.bn_scale = torch.as_tensor(_np(bn_scale), dtype=torch.float32, device=self.device)
        self.bn_bias = torch.as_tensor(_np(bn_bias), dtype=torch.float32, device=self.device)
        self.T, self.B, self.Cin, self.Cout = T, B, cin, cout
        self.H, self.W = H, W
        self.out_dtype = torch.float32 if neuron == "none" else torch.float16

    def out_shape(self):
        return (self.T * self.B, self.OH, self.OW, self.Cout)

    def state_shape(self):
        return (self.B * self.OH * self.OW, self.Cout)

    def workspace_bytes(self):
        """Bytes of the workspace the timestep-split form needs."""
        n = ctypes.c_size_t()
        rt.check(rt.load().snn_conv_tsplit_workspace_bytes(self.desc, ctypes.byref(n)))
        return n.value

    def __call__(self, data, state=None, residual=None, out=None, *, read_state=None,
                 write_state=None, stream=None, state2=None, workspace=None):
        """Run the layer; returns ``out``.

        ``state`` (optional) is the membrane buffer: read at start unless
        ``read_state=False`` and final v written unless ``write_state=False``.
        ``state2`` is the second neuron's membrane (``res_mode="two_neuron"``,
        same shape and flags as ``state``).  With ``workspace`` (a device
        tensor of at least ``workspace_bytes()`` bytes) the layer runs in its
        timestep-split form (``snn_conv_forward_tsplit``).
        """
        if data.dtype != torch.float16 or not data.is_contiguous():
            raise ValueError("data must be contiguous fp16 (T*B, H, W, Cin)")
        if tuple(data.shape) != (self.T * self.B, self.H, self.W, self.Cin):
            raise ValueError(f"data shape {tuple(data.shape)} does not match layer")
        if out is None:
            out = torch.empty(self.out_shape(), dtype=self.out_dtype, device=data.device)
        flags = self.base_flags
        if state is not None:
            if tuple(state.shape) != self.state_shape() or state.dtype != torch.float32:
                raise ValueError("state must be fp32 (B*OH*OW, Cout)")
            if read_state is not False:
                flags |= rt.SNN_FLAG_READ_STATE
            if write_state is not False:
                flags |= rt.SNN_FLAG_WRITE_STATE
        self.desc.flags = flags
        s = stream if stream is not None else torch.cuda.current_stream(data.device).cuda_stream
        lib = rt.load()
        sp = state.data_ptr() if state is not None else None
        if self.res_mode == "two_neuron":
            if residual is None:
                raise ValueError("res_mode two_neuron needs a residual")
            if (state is None) != (state2 is None):
                raise ValueError("two_neuron takes both membranes or neither")
            if state2 is not None and (tuple(state2.shape) != self.state_shape()
                                       or state2.dtype != torch.float32):
                raise ValueError("state2 must be fp32 (B*OH*OW, Cout)")
        if residual is not None:
            if residual.dtype != torch.float16 or tuple(residual.shape) != self.out_shape():
                raise ValueError("residual must be fp16 (T*B, OH, OW, Cout)")
        if workspace is not None:
            if self.res_mode == "two_neuron":
                raise ValueError("the timestep-split form has no two-neuron epilogue")
            nbytes = workspace.numel() * workspace.element_size()
            rt.check(lib.snn_conv_forward_tsplit(
                self.desc, data.data_ptr(), self.weight_blob.data_ptr(), sp,
                self.bn_scale.data_ptr(), self.bn_bias.data_ptr(),
                residual.data_ptr() if residual is not None else None, out.data_ptr(),
                workspace.data_ptr(), nbytes, s))
        elif self.res_mode == "two_neuron":
            rt.check(lib.snn_conv_forward_res2(
                self.desc, data.data_ptr(), self.weight_blob.data_ptr(), sp,
                state2.data_ptr() if state2 is not None else None,
                self.bn_scale.data_ptr(), self.bn_bias.data_ptr(), residual.data_ptr(),
                out.data_ptr(), s))
        elif residual is not None:
            rt.check(lib.snn_conv_forward_res(
                self.desc, data.data_ptr(), self.weight_blob.data_ptr(), sp,
                self.bn_scale.data_ptr(), self.bn_bias.data_ptr(), residual.data_ptr(),
                out.data_ptr(), s))
        else:
            rt.check(lib.snn_conv_forward(
                self.desc, data.data_ptr(), self.weight_blob.data_ptr(), sp,
                self.bn_scale.data_ptr(), self.bn_bias.data_ptr(), out.data_ptr(), s))
        return out
