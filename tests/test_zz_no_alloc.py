"""The allocation-free form of the timestep-split layer
(``snn_conv_forward_tsplit_static``), for callers that cannot allocate device
memory themselves: its fp32 intermediate lives in a fixed array inside the
library instead of a caller workspace.

Called through the C-ABI twice in a row on different inputs, its spikes and
final membranes must match the workspace form's (``snn_conv_forward_tsplit``)
within the tolerance the timestep-split tests use; a layer whose
intermediate exceeds the array is rejected.  This file sorts last so that a
run stopping at the first failure has run every other test first; it also
passes on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest

from oracle import lif_layer as L

pytestmark = pytest.mark.gpu


def to_nhwc(x):
    t, b, c, h, w = x.shape
    return np.ascontiguousarray(np.transpose(x, (0, 1, 3, 4, 2)).reshape(t * b, h, w, c))


def test_static_scratch_matches_workspace_form(cuda_device):
    import torch
    from sparsesnn_b200 import runtime as rt
    from sparsesnn_b200.layer import SparseConvBNLIF, fold_bn
    lib = rt.load()
    # A DVS SEW-ResNet-18 stage-3 conv with its SEW residual: T = 16, 4 images.
    T, B, C, F, H = 16, 4, 256, 256, 8
    x, w, bn = L.make_config0(seed=77, T=T, B=B, C=C, F=F, H=H, W=H)
    w = (w * 2.0).astype(np.float32)
    layer = SparseConvBNLIF(w, *fold_bn(bn.gamma, bn.beta, bn.mean, bn.var), T=T, B=B, H=H, W=H)
    need = layer.workspace_bytes()
    assert 0 < need <= lib_max_bytes()
    ws = torch.empty(need // 4, dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(5)
    flags = rt.SNN_FLAG_WRITE_STATE
    for call in range(2):                       # two calls in a row, different inputs
        xs = (rng.random(x.shape) < 0.2 + 0.1 * call).astype(np.float32)
        xd = torch.from_numpy(to_nhwc(xs)).to("cuda", torch.float16)
        res = torch.from_numpy(to_nhwc(rng.integers(0, 3, (T, B, F, H, H)).astype(np.float32))).to(
            "cuda", torch.float16)
        outs, states = [], []
        for static in (False, True):
            out = torch.full(layer.out_shape(), 5.0, dtype=torch.float16, device="cuda")
            st = torch.full(layer.state_shape(), -3.0, dtype=torch.float32, device="cuda")
            d = rt.SnnConvDesc.from_buffer_copy(bytes(layer.desc))
            d.flags = flags
            args = (ctypes.byref(d), xd.data_ptr(), layer.weight_blob.data_ptr(), st.data_ptr(),
                    layer.bn_scale.data_ptr(), layer.bn_bias.data_ptr(), res.data_ptr(),
                    out.data_ptr())
            if static:
                rc = lib.snn_conv_forward_tsplit_static(*args, s)
            else:
                rc = lib.snn_conv_forward_tsplit(*args, ws.data_ptr(), need, s)
            assert rc == 0, lib.snn_last_error_message()
            outs.append(out)
            states.append(st)
        torch.cuda.synchronize()
        assert rt.device_error() == 0
        agree = float((outs[0] == outs[1]).float().mean())
        v0, v1 = states[0].cpu().numpy(), states[1].cpu().numpy()
        print(f"call {call}: outputs equal at {agree:.6f}, max |dv| {np.abs(v0 - v1).max():.3e}")
        assert agree >= 0.999
        assert (np.abs(v0 - v1) <= 1e-2 * np.abs(v0) + 1e-3).all()
        assert float(outs[1].float().mean()) > 0.05     # the layer fires


def lib_max_bytes():
    """SNN_TSPLIT_STATIC_MAX_BYTES of include/snn_b200.h."""
    return 8 << 20


def test_static_scratch_rejects_oversized_layer(cuda_device):
    import torch
    from sparsesnn_b200 import runtime as rt
    from sparsesnn_b200.layer import SparseConvBNLIF, fold_bn
    lib = rt.load()
    T, B, C, F, H = 16, 8, 128, 128, 16          # 16 MiB of intermediate
    x, w, bn = L.make_config0(seed=3, T=2, B=1, C=C, F=F, H=4, W=4)
    layer = SparseConvBNLIF(w, *fold_bn(bn.gamma, bn.beta, bn.mean, bn.var), T=T, B=B, H=H, W=H)
    assert layer.workspace_bytes() > lib_max_bytes()
    xd = torch.zeros((T * B, H, H, C), dtype=torch.float16, device="cuda")
    out = torch.empty(layer.out_shape(), dtype=torch.float16, device="cuda")
    rc = lib.snn_conv_forward_tsplit_static(ctypes.byref(layer.desc), xd.data_ptr(),
                                            layer.weight_blob.data_ptr(), None,
                                            layer.bn_scale.data_ptr(), layer.bn_bias.data_ptr(),
                                            None, out.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream)
    assert rc == rt.SNN_E_INVALID
    assert b"static array" in lib.snn_last_error_message()
