"""GPU parity of the layer modes the Spikformer, MS-ResNet and DVS SEW-ResNet
models add to the fused path:

* dense (unpruned) weights run as two 2:4 halves (``SNN_FLAG_DENSE``), with
  and without the SEW residual, four- and two-timestep accumulators, and
  zero-padded channels (48 -> 64 inputs, 96 -> 128 outputs, as a Spikformer
  patch-splitting stage stores them);
* the fp16 BN output without neuron, plain and plus a real-valued residual
  (MS-ResNet's ``conv_bn2(...) + shortcut``, ``models/msresnet.py:119-123``);
* the plain max pool after a neuron (``models/sewresnet.py:202-203``,
  ``models/spikformer.py:192-197``) and the neuron of one real-valued input
  (``models/msresnet.py:119-121``), both exact;
* the dense stem without neuron (MS-ResNet's 7x7/2 stem, ``:135-138``).
"""
import numpy as np
import pytest

from oracle import lif_layer as L
from oracle.glue import maxpool2d

pytestmark = pytest.mark.gpu


def to_nhwc(x):
    t, b, c, h, w = x.shape
    return np.ascontiguousarray(np.transpose(x, (0, 1, 3, 4, 2)).reshape(t * b, h, w, c))


def from_nhwc(y, T, B):
    tb, h, w, c = y.shape
    return np.transpose(y.reshape(T, B, h, w, c), (0, 1, 4, 2, 3))


def _bn(rng, f):
    return L.BNParams(rng.uniform(0.5, 1.5, f).astype(np.float32),
                      (rng.standard_normal(f) * 0.1).astype(np.float32),
                      (rng.standard_normal(f) * 0.1).astype(np.float32),
                      rng.uniform(0.5, 1.5, f).astype(np.float32))


def check_spikes(spk, v, ref):
    st = {}
    frac, ok, _, div = L.spike_agreement(spk, ref["spikes"], ref["h"], stats=st)
    print(f"agreement {frac:.6f} {st}")
    assert frac >= 0.995 and ok, frac
    err = np.abs(v - ref["v"])[~div]
    assert (err <= 1e-2 * np.abs(ref["v"][~div]) + 1e-3).all(), err.max()


@pytest.mark.parametrize("cin, cout, hw, stride, T", [
    (64, 128, 16, 1, 4),      # 64-pixel tiles, four timesteps per accumulator
    (128, 192, 14, 1, 4),     # 56-pixel tiles (two timesteps per accumulator)
    (192, 384, 28, 1, 4),
    (384, 384, 8, 1, 3),      # partial last chunk of timesteps
    (64, 128, 16, 2, 4),      # strided
])
@pytest.mark.parametrize("residual", [False, True], ids=["plain", "res"])
def test_dense_layer(cuda_device, cin, cout, hw, stride, T, residual):
    import torch
    from sparsesnn_b200 import runtime as rt
    from sparsesnn_b200.layer import SparseConvBNLIF, fold_bn
    rng = np.random.default_rng(cin + cout + hw + T)
    B = 4
    x = (rng.random((T, B, cin, hw, hw)) < 0.2).astype(np.float32)
    # Kaiming scale x 4: inputs large enough that a good share of neurons fire
    w = (rng.standard_normal((cout, cin, 3, 3)) * 4 * np.sqrt(2.0 / (cout * 9))).astype(np.float32)
    bn = _bn(rng, cout)
    scale, bias = fold_bn(bn.gamma, bn.beta, bn.mean, bn.var)
    layer = SparseConvBNLIF(w, scale, bias, T=T, B=B, H=hw, W=hw, stride=stride, pad=1, dense=True)
    assert rt.variant(layer.desc) == rt.SNN_VARIANT_GENERIC
    oh, ow = layer.OH, layer.OW
    res_np, rd = None, None
    if residual:
        res_np = rng.integers(0, 3, (T, B, cout, oh, ow)).astype(np.float32)
        rd = torch.from_numpy(to_nhwc(res_np)).to("cuda", torch.float16)
    st = torch.full(layer.state_shape(), 2.0, dtype=torch.float32, device="cuda")
    y = layer(torch.from_numpy(to_nhwc(x)).to("cuda", torch.float16), state=st, residual=rd,
              read_state=False)
    torch.cuda.synchronize()
    assert rt.device_error() == 0
    ref = L.fused_layer_torch(x, w.astype(np.float16).astype(np.float32), bn, stride=stride, pad=1)
    ys = from_nhwc(y.float().cpu().numpy(), T, B)
    spk = ys - res_np if residual else ys
    assert set(np.unique(spk)) <= {0.0, 1.0}
    v = np.transpose(st.cpu().numpy().reshape(B, oh, ow, cout), (0, 3, 1, 2))
    check_spikes(spk, v, ref)
    assert 0.01 < ref["spikes"].mean() < 0.9


def test_dense_zero_padded_channels(cuda_device):
    """48 real input channels stored as 64, 96 real outputs as 128: padded
    inputs are zero, padded output rows have zero weights and BN scale/bias,
    so they never spike; the real channels match the 48 -> 96 oracle."""
    import torch
    from sparsesnn_b200.layer import SparseConvBNLIF, fold_bn
    rng = np.random.default_rng(3)
    T, B, H = 4, 2, 16
    x = (rng.random((T, B, 48, H, H)) < 0.3).astype(np.float32)
    w = (rng.standard_normal((96, 48, 3, 3)) * 4 * np.sqrt(2.0 / (96 * 9))).astype(np.float32)
    bn = _bn(rng, 96)
    s, b = fold_bn(bn.gamma, bn.beta, bn.mean, bn.var)
    xp = np.zeros((T, B, 64, H, H), np.float32); xp[:, :, :48] = x
    wp = np.zeros((128, 64, 3, 3), np.float32); wp[:96, :48] = w
    sp = np.zeros(128, np.float32); sp[:96] = s
    bp = np.zeros(128, np.float32); bp[:96] = b
    layer = SparseConvBNLIF(wp, sp, bp, T=T, B=B, H=H, W=H, dense=True)
    st = torch.zeros(layer.state_shape(), dtype=torch.float32, device="cuda")
    y = layer(torch.from_numpy(to_nhwc(xp)).to("cuda", torch.float16), state=st)
    torch.cuda.synchronize()
    ys = from_nhwc(y.float().cpu().numpy(), T, B)
    assert not ys[:, :, 96:].any()
    ref = L.fused_layer_torch(x, w.astype(np.float16).astype(np.float32), bn, pad=1)
    v = np.transpose(st.cpu().numpy().reshape(B, H, H, 128), (0, 3, 1, 2))[:, :96]
    check_spikes(ys[:, :, :96], v, ref)
    assert 0.01 < ref["spikes"].mean() < 0.9


@pytest.mark.parametrize("cin, cout, hw, k, stride", [
    (64, 64, 14, 3, 1), (128, 128, 7, 3, 1), (64, 128, 28, 1, 2), (256, 256, 8, 3, 1)])
@pytest.mark.parametrize("residual", [False, True], ids=["plain", "res"])
def test_bn_f16_output(cuda_device, cin, cout, hw, k, stride, residual):
    """No neuron, fp16 output: bn (+ residual) computed in fp32 and rounded
    once; compared with the oracle on the same fp16 weights and inputs."""
    import torch
    from sparsesnn_b200 import runtime as rt
    from sparsesnn_b200.layer import SparseConvBNLIF, fold_bn
    rng = np.random.default_rng(cin + hw + k)
    T, B = 4, 3
    x, w, bn = L.make_config0(seed=cin + hw + k, T=T, B=B, C=cin, F=cout, H=hw, W=hw, k=k)
    x = (x * rng.standard_normal(x.shape)).astype(np.float16).astype(np.float32)   # real-valued
    scale, bias = fold_bn(bn.gamma, bn.beta, bn.mean, bn.var)
    layer = SparseConvBNLIF(w, scale, bias, T=T, B=B, H=hw, W=hw, stride=stride, pad=k // 2,
                            neuron="none_f16")
    oh, ow = layer.OH, layer.OW
    res_np, rd = None, None
    if residual:
        res_np = rng.standard_normal((T, B, cout, oh, ow)).astype(np.float16).astype(np.float32)
        rd = torch.from_numpy(to_nhwc(res_np)).to("cuda", torch.float16)
    y = layer(torch.from_numpy(to_nhwc(x)).to("cuda", torch.float16), residual=rd)
    torch.cuda.synchronize()
    assert rt.device_error() == 0
    assert y.dtype == torch.float16
    got = from_nhwc(y.float().cpu().numpy(), T, B)
    ref = L.fused_layer(x, w.astype(np.float16).astype(np.float32), bn, stride=stride,
                        pad=k // 2)["bn_out"]
    if residual:
        ref = ref + res_np
    tol = 2.0 ** -10 * np.abs(ref) + 1e-3 * max(1.0, float(np.abs(ref).max()) * 1e-2)
    assert (np.abs(got - ref) <= tol).all(), np.abs(got - ref).max()


def test_plain_maxpool_after_neuron(cuda_device):
    """snn_maxpool_lif_forward with neuron NONE: the max pool alone, exact."""
    import torch
    from sparsesnn_b200 import runtime as rt
    rng = np.random.default_rng(1)
    for (T, B, C, H, k, s, p) in ((4, 2, 64, 17, 3, 2, 1), (16, 1, 64, 64, 3, 2, 1),
                                  (4, 3, 48, 28, 3, 2, 1), (2, 2, 384, 28, 2, 2, 0)):
        x = (rng.random((T, B, C, H, H)) < 0.3).astype(np.float32)
        d = rt.make_desc(T=T, B=B, Cin=C, H=H, W=H, Cout=C, KH=k, KW=k, stride=s, pad=p,
                         neuron="none")
        oh = (H + 2 * p - k) // s + 1
        out = torch.full((T * B, oh, oh, C), 9.0, dtype=torch.float16, device="cuda")
        xd = torch.from_numpy(to_nhwc(x)).to("cuda", torch.float16)
        rt.check(rt.load().snn_maxpool_lif_forward(d, xd.data_ptr(), None, out.data_ptr(),
                                                  torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        ref = maxpool2d(x.reshape((T * B, C, H, H)), k, s, p).reshape(T, B, C, oh, oh)
        assert np.array_equal(from_nhwc(out.float().cpu().numpy(), T, B), ref)


@pytest.mark.parametrize("neuron, tau", [("lif", 2.0), ("lif", 3.0), ("if", 2.0)])
def test_single_input_neuron(cuda_device, neuron, tau):
    """snn_lif_forward: the neuron of one real-valued fp16 input, exact
    (spikes and final membrane) against the oracle on the same fp16 values."""
    import torch
    from sparsesnn_b200 import runtime as rt
    rng = np.random.default_rng(2)
    T, B, C, H = 4, 3, 64, 9
    x = (rng.standard_normal((T, B, C, H, H)) * 1.5).astype(np.float16).astype(np.float32)
    d = rt.make_desc(T=T, B=B, Cin=C, H=H, W=H, Cout=C, KH=1, KW=1, neuron=neuron, tau=tau,
                     flags=rt.SNN_FLAG_WRITE_STATE)
    out = torch.empty((T * B, H, H, C), dtype=torch.float16, device="cuda")
    st = torch.empty((B * H * H, C), dtype=torch.float32, device="cuda")
    xd = torch.from_numpy(to_nhwc(x)).to("cuda", torch.float16)
    rt.check(rt.load().snn_lif_forward(d, xd.data_ptr(), st.data_ptr(), out.data_ptr(),
                                      torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    spk, _, v = L.multistep_lif(x, tau=tau, neuron=neuron)
    assert np.array_equal(from_nhwc(out.float().cpu().numpy(), T, B), spk)
    assert np.array_equal(np.transpose(st.cpu().numpy().reshape(B, H, H, C), (0, 3, 1, 2)), v)


def test_stem_without_neuron(cuda_device):
    """7x7 stride-2 stem with BN and no neuron: fp16 BN output repeated over T."""
    import torch
    from sparsesnn_b200 import runtime as rt
    rng = np.random.default_rng(4)
    T, B, Cin, H, Cout = 4, 2, 3, 30, 64
    x = rng.standard_normal((B, Cin, H, H)).astype(np.float32)
    w = (rng.standard_normal((Cout, Cin, 7, 7)) * 0.1).astype(np.float32)
    scale = rng.uniform(0.5, 1.5, Cout).astype(np.float32)
    bias = rng.normal(0, 0.1, Cout).astype(np.float32)
    d = rt.make_desc(T=T, B=B, Cin=Cin, H=H, W=H, Cout=Cout, KH=7, KW=7, stride=2, pad=3,
                     neuron="none")
    oh = (H + 6 - 7) // 2 + 1
    out = torch.empty((T * B, oh, oh, Cout), dtype=torch.float16, device="cuda")
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    xd, wd, sd, bd = dev(x), dev(w), dev(scale), dev(bias)
    rt.check(rt.load().snn_stem_forward(d, 1, xd.data_ptr(), wd.data_ptr(), sd.data_ptr(),
                                       bd.data_ptr(), out.data_ptr(),
                                       torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    z = L.conv2d_nchw(x, w, 2, 3) * scale[None, :, None, None] + bias[None, :, None, None]
    got = from_nhwc(out.float().cpu().numpy(), T, B)
    for t in range(T):
        assert (np.abs(got[t] - z) <= 2.0 ** -10 * np.abs(z) + 1e-4).all()


@pytest.mark.parametrize("cin, cout, hw, dense, variant", [
    (48, 96, 16, True, 0),        # a Spikformer patch-splitting conv, 48 channels stored as 48
    (96, 192, 14, True, 0),
    (48, 64, 16, False, 1),       # four-timestep halo kernel, one partial input block
    (96, 128, 16, False, 1),      # 128-channel halo kernel
    (200, 256, 8, False, 2),      # streaming halo kernel, partial fourth block
    (72, 128, 16, False, 0),      # general kernel (strided)
])
def test_partial_input_channel_block(cuda_device, cin, cout, hw, dense, variant):
    """Cin a multiple of 8 but not of 64: the activations keep Cin channels
    in HBM, the last 64-channel k-block reads TMA zero fill past Cin and its
    weight columns are zero."""
    import torch
    from sparsesnn_b200 import runtime as rt
    from sparsesnn_b200.layer import SparseConvBNLIF, fold_bn
    rng = np.random.default_rng(cin + cout)
    T, B = 4, 3
    stride = 2 if (variant == 0 and not dense) else 1
    x = (rng.random((T, B, cin, hw, hw)) < 0.25).astype(np.float32)
    w = (rng.standard_normal((cout, cin, 3, 3)) * 3 * np.sqrt(2.0 / (cin * 9))).astype(np.float32)
    if not dense:
        from oracle.pack24 import prune_conv_weight
        w = prune_conv_weight(w)
    bn = _bn(rng, cout)
    scale, bias = fold_bn(bn.gamma, bn.beta, bn.mean, bn.var)
    layer = SparseConvBNLIF(w, scale, bias, T=T, B=B, H=hw, W=hw, stride=stride, pad=1, dense=dense)
    assert rt.variant(layer.desc) == variant
    st = torch.zeros(layer.state_shape(), dtype=torch.float32, device="cuda")
    y = layer(torch.from_numpy(to_nhwc(x)).to("cuda", torch.float16), state=st)
    torch.cuda.synchronize()
    assert rt.device_error() == 0
    ref = L.fused_layer_torch(x, w.astype(np.float16).astype(np.float32), bn, stride=stride, pad=1)
    oh, ow = layer.OH, layer.OW
    v = np.transpose(st.cpu().numpy().reshape(B, oh, ow, cout), (0, 3, 1, 2))
    check_spikes(from_nhwc(y.float().cpu().numpy(), T, B), v, ref)
    assert 0.01 < ref["spikes"].mean() < 0.9


@pytest.mark.parametrize("T, hw, cout", [(4, 56, 64), (3, 20, 48), (6, 16, 64)])
@pytest.mark.parametrize("residual", [False, True], ids=["plain", "res"])
def test_bn_f16_four_timestep_halo(cuda_device, T, hw, cout, residual):
    """The fp16 BN output (+ real residual) in the four-timestep halo kernel
    (MS-ResNet's stage-1 conv2 with its membrane shortcut): several pixel
    tiles per CTA, T not a multiple of four, fewer than 64 channels."""
    import torch
    from sparsesnn_b200 import runtime as rt
    from sparsesnn_b200.layer import SparseConvBNLIF, fold_bn
    rng = np.random.default_rng(T + hw + cout)
    B = 4
    x, w, bn = L.make_config0(seed=T + hw, T=T, B=B, C=64, F=cout, H=hw, W=hw)
    scale, bias = fold_bn(bn.gamma, bn.beta, bn.mean, bn.var)
    layer = SparseConvBNLIF(w, scale, bias, T=T, B=B, H=hw, W=hw, neuron="none_f16")
    assert rt.variant(layer.desc) == rt.SNN_VARIANT_HALO_RESIDENT
    res_np, rd = None, None
    if residual:
        res_np = (rng.standard_normal((T, B, cout, hw, hw)) * 2).astype(np.float16).astype(np.float32)
        rd = torch.from_numpy(to_nhwc(res_np)).to("cuda", torch.float16)
    y = layer(torch.from_numpy(to_nhwc(x)).to("cuda", torch.float16), residual=rd)
    torch.cuda.synchronize()
    assert rt.device_error() == 0
    got = from_nhwc(y.float().cpu().numpy(), T, B)
    ref = L.fused_layer_torch(x, w.astype(np.float16).astype(np.float32), bn, pad=1, neuron="lif")
    # BN output of the oracle: recompute without the neuron
    import torch.nn.functional as F
    with torch.no_grad():
        z = F.conv2d(torch.from_numpy(x.reshape((T * B,) + x.shape[2:])),
                     torch.from_numpy(w.astype(np.float16).astype(np.float32)), padding=1)
        z = z * torch.from_numpy(scale)[None, :, None, None] + torch.from_numpy(bias)[None, :, None, None]
    zr = z.numpy().reshape(T, B, cout, hw, hw)
    if residual:
        zr = zr + res_np
    assert ref is not None
    tol = 2.0 ** -10 * np.abs(zr) + 2e-3
    assert (np.abs(got - zr) <= tol).all(), np.abs(got - zr).max()
