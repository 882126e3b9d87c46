"""GPU parity of the timestep-split fused layer (snn_conv_forward_tsplit):
conv + BN of all T*B images at once into an fp32 workspace, then the neuron
over T.  DVS-configuration shapes (T = 16, 4 images) on every stage, strided
and 1x1 layers, both residual modes, IF, odd T; against the oracle by the
layer parity rule and against the one-pass layer."""
import numpy as np
import pytest

from oracle import lif_layer as L

pytestmark = pytest.mark.gpu


def to_nhwc(x):
    t, b, c, h, w = x.shape
    return np.ascontiguousarray(np.transpose(x, (0, 1, 3, 4, 2)).reshape(t * b, h, w, c))


def from_nhwc(y, T, B):
    tb, h, w, c = y.shape
    return np.transpose(y.reshape(T, B, h, w, c), (0, 1, 4, 2, 3))


@pytest.mark.parametrize("T, B, C, F, H, k, stride, neuron, res", [
    (16, 4, 64, 64, 32, 3, 1, "lif", None),
    (16, 4, 128, 128, 16, 3, 1, "lif", "add_after"),
    (16, 4, 256, 256, 8, 3, 1, "lif", "add_after"),
    (16, 4, 512, 512, 4, 3, 1, "lif", None),
    (16, 4, 256, 512, 8, 3, 2, "lif", None),
    (16, 4, 128, 256, 16, 1, 2, "if", None),
    (5, 3, 128, 128, 8, 3, 1, "lif", "add_before"),
])
def test_tsplit_layer(cuda_device, T, B, C, F, H, k, stride, neuron, res):
    import torch
    from sparsesnn_b200 import runtime as rt
    from sparsesnn_b200.layer import SparseConvBNLIF, fold_bn
    x, w, bn = L.make_config0(seed=T + C + F + H + k, T=T, B=B, C=C, F=F, H=H, W=H, k=k)
    w = (w * 2.0).astype(np.float32)                     # busier neurons
    scale, bias = fold_bn(bn.gamma, bn.beta, bn.mean, bn.var)
    layer = SparseConvBNLIF(w, scale, bias, T=T, B=B, H=H, W=H, stride=stride, pad=k // 2,
                            neuron=neuron, res_mode=res or "add_after")
    oh, ow = layer.OH, layer.OW
    rng = np.random.default_rng(T + F)
    res_np, rd = None, None
    if res == "add_after":
        res_np = rng.integers(0, 3, (T, B, F, oh, ow)).astype(np.float32)
    elif res == "add_before":
        res_np = (rng.standard_normal((T, B, F, oh, ow)) * 0.5).astype(np.float16).astype(np.float32)
    if res_np is not None:
        rd = torch.from_numpy(to_nhwc(res_np)).to("cuda", torch.float16)
    xd = torch.from_numpy(to_nhwc(x)).to("cuda", torch.float16)
    ws = torch.empty(layer.workspace_bytes() // 4, dtype=torch.float32, device="cuda")
    st = torch.full(layer.state_shape(), 9.0, dtype=torch.float32, device="cuda")
    y = layer(xd, state=st, residual=rd, read_state=False, workspace=ws)
    st1 = torch.full_like(st, 9.0)
    y1 = layer(xd, state=st1, residual=rd, read_state=False)       # one-pass form
    torch.cuda.synchronize()
    assert rt.device_error() == 0
    w16 = w.astype(np.float16).astype(np.float32)
    ref = L.fused_layer_torch(x if res != "add_before" else x, w16, bn, stride=stride, pad=k // 2,
                              neuron=neuron) if res != "add_before" else None
    if res == "add_before":
        r = L.fused_layer(x, w16, bn, stride=stride, pad=k // 2, neuron=neuron, residual=res_np,
                          res_mode="add_before")
        ref = {"spikes": r["spikes"], "h": r["h"], "v": r["v"]}
    ys = from_nhwc(y.float().cpu().numpy(), T, B)
    spk = ys - res_np if res == "add_after" else ys
    assert set(np.unique(spk)) <= {0.0, 1.0}
    st_ = {}
    frac, ok, _, div = L.spike_agreement(spk, ref["spikes"], ref["h"], stats=st_)
    print(f"tsplit agreement {frac:.6f} rate {ref['spikes'].mean():.3f} {st_}")
    assert frac >= 0.995 and ok
    v = np.transpose(st.cpu().numpy().reshape(B, oh, ow, F), (0, 3, 1, 2))
    err = np.abs(v - ref["v"])[~div]
    assert (err <= 1e-2 * np.abs(ref["v"][~div]) + 1e-3).all()
    # against the one-pass form: the same spikes but where a BN output sits
    # within rounding of the threshold
    agree = float((y == y1).float().mean())
    print(f"one-pass vs split: {agree:.6f} equal")
    assert agree >= 0.999
    assert 0.02 < ref["spikes"].mean() < 0.9


def test_tsplit_rejects_small_workspace(cuda_device):
    import torch
    from sparsesnn_b200 import runtime as rt
    from sparsesnn_b200.layer import SparseConvBNLIF, fold_bn
    x, w, bn = L.make_config0(seed=1, T=4, B=2, C=64, F=64, H=8, W=8)
    layer = SparseConvBNLIF(w, *fold_bn(bn.gamma, bn.beta, bn.mean, bn.var), T=4, B=2, H=8, W=8)
    xd = torch.from_numpy(to_nhwc(x)).to("cuda", torch.float16)
    ws = torch.empty(layer.workspace_bytes() // 4 - 4, dtype=torch.float32, device="cuda")
    with pytest.raises(rt.SnnError) as e:
        layer(xd, workspace=ws)
    assert e.value.code == rt.SNN_E_INVALID
