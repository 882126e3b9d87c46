"""GPU parity of the dense stem (conv + BN + neuron over T) through the C ABI:
the row-tiled kernel (3x3 s1 p1, 64 channels, input repeated over T) on
widths that do and do not divide its 128-pixel tile, and the general kernel
(per-timestep input, other channel counts)."""
import ctypes

import numpy as np
import pytest

from oracle import lif_layer as L

pytestmark = pytest.mark.gpu

GUARD, SENTINEL = 4096, -3.0


def run_stem(x, w, scale, bias, T, neuron, tau, Tin, stride=1):
    import torch
    from sparsesnn_b200 import runtime as rt
    lib = rt.load()
    B, Cin, H, W = x.shape[1:]
    Cout, k = w.shape[0], w.shape[2]
    d = rt.make_desc(T=T, B=B, Cin=Cin, H=H, W=W, Cout=Cout, KH=k, KW=k, stride=stride, pad=k // 2,
                     neuron=neuron, tau=tau)
    H = (H + 2 * (k // 2) - k) // stride + 1
    W = (W + 2 * (k // 2) - k) // stride + 1
    xd = torch.from_numpy(x).cuda()
    wd = torch.from_numpy(w).cuda()
    sd = torch.from_numpy(scale).cuda()
    bd = torch.from_numpy(bias).cuda()
    # The output is followed by a guard tail of sentinels: TMA stores clip at
    # the tensor map's extent, so nothing past the tensor may change.
    n_out = T * B * H * W * Cout
    buf = torch.full((n_out + GUARD,), SENTINEL, dtype=torch.float16, device="cuda")
    out = buf[:n_out]
    rc = lib.snn_stem_forward(ctypes.byref(d), Tin, xd.data_ptr(), wd.data_ptr(), sd.data_ptr(),
                              bd.data_ptr(), out.data_ptr(), None)
    assert rc == 0, lib.snn_last_error_message()
    torch.cuda.synchronize()
    assert rt.device_error() == 0
    assert bool((buf[n_out:] == SENTINEL).all()), "stem wrote past its output"
    return np.transpose(out.float().cpu().numpy().reshape(T, B, H, W, Cout), (0, 1, 4, 2, 3))


def reference(x, w, scale, bias, T, neuron, tau, stride=1):
    k = w.shape[2]
    z = np.stack([L.conv2d_nchw(x[t], w, stride, k // 2) for t in range(x.shape[0])])
    z = (z * scale[None, None, :, None, None] + bias[None, None, :, None, None]).astype(np.float32)
    if z.shape[0] == 1:
        z = np.repeat(z, T, 0)
    return L.multistep_lif(z, tau=tau, neuron=neuron)


@pytest.mark.parametrize("case", [
    dict(H=32, W=32, Cout=64, neuron="lif", tau=2.0, Tin=1),     # CIFAR stem (row-tiled)
    dict(H=12, W=40, Cout=64, neuron="lif", tau=3.0, Tin=1),     # 128 % 40 != 0, general tau
    dict(H=9, W=7, Cout=64, neuron="if", tau=2.0, Tin=1),       # IF, short image
    dict(H=16, W=16, Cout=32, neuron="lif", tau=2.0, Tin=1),     # general kernel (32 channels)
    dict(H=16, W=16, Cout=64, neuron="lif", tau=2.0, Tin=4),     # general kernel (input per timestep)
    # general tensor-core stem (K <= 192): a 7x7/2 event-frame stem (2 channels, a frame
    # per timestep), a 48-channel stem on rows wider than 128 pixels, a 7x7/2
    # RGB stem with an IF neuron
    dict(H=30, W=34, Cout=64, neuron="lif", tau=2.0, Tin=8, Cin=2, k=7, stride=2, binary=True),
    dict(H=12, W=140, Cout=48, neuron="lif", tau=2.0, Tin=1),
    dict(H=29, W=29, Cout=64, neuron="if", tau=2.0, Tin=1, k=7, stride=2),
    # CUDA-core stem (more than 64 channels)
    dict(H=16, W=16, Cout=96, neuron="lif", tau=2.0, Tin=1),
], ids=["cifar", "w40_tau3", "if_9x7", "c32_general", "tin4_general", "dvs7x7s2", "c48_w140",
        "rgb7x7s2_if", "c96_cudacore"])
def test_stem_parity(cuda_device, case):
    rng = np.random.default_rng(7)
    Cin, k, stride = case.get("Cin", 3), case.get("k", 3), case.get("stride", 1)
    T, B = max(4, case["Tin"]), 3
    H, W, Cout = case["H"], case["W"], case["Cout"]
    if case.get("binary"):
        x = (rng.random((case["Tin"], B, Cin, H, W)) < 0.3).astype(np.float32)
        w = (rng.standard_normal((Cout, Cin, k, k)) * 0.6).astype(np.float32)
    else:
        x = rng.standard_normal((case["Tin"], B, Cin, H, W)).astype(np.float32)
        w = (rng.standard_normal((Cout, Cin, k, k)) * 0.3 * 3 / k).astype(np.float32)
    scale = rng.uniform(0.5, 1.5, Cout).astype(np.float32)
    bias = rng.normal(0, 0.1, Cout).astype(np.float32)
    got = run_stem(x, w, scale, bias, T, case["neuron"], case["tau"], case["Tin"], stride)
    spk, h, _ = reference(x, w, scale, bias, T, case["neuron"], case["tau"], stride)
    assert 0.02 < spk.mean() < 0.9
    assert set(np.unique(got)) <= {0.0, 1.0}
    frac, ok, _, _ = L.spike_agreement(got, spk, h)
    assert frac >= 0.995 and ok, frac


@pytest.mark.parametrize("case", [
    dict(H=40, W=40, Cout=64, k=7, stride=2, Tin=1, neuron="lif", tau=2.0),     # TMA windows
    dict(H=29, W=29, Cout=64, k=7, stride=2, Tin=1, neuron="lif", tau=3.0),     # cp.async windows
    dict(H=30, W=36, Cout=64, k=7, stride=2, Tin=8, Cin=2, neuron="if", tau=2.0),
    dict(H=12, W=140, Cout=48, k=3, stride=1, Tin=1, neuron="lif", tau=2.0),
], ids=["rgb7x7s2_tma", "rgb7x7s2_cpasync_tau3", "frames_if", "c48_w140"])
def test_stem_dual_output(cuda_device, case):
    """snn_stem_forward_dual: its fp16 BN output equals the no-neuron stem's
    bit for bit, and its spikes equal the neuron over T run on that output
    (the standalone LIF node after MS-ResNet's stem), bit for bit."""
    import torch
    from sparsesnn_b200 import runtime as rt
    lib = rt.load()
    rng = np.random.default_rng(21)
    Cin, k, stride, Tin = case.get("Cin", 3), case["k"], case["stride"], case["Tin"]
    T, B = max(4, Tin), 3
    H, W, Cout = case["H"], case["W"], case["Cout"]
    x = rng.standard_normal((Tin, B, Cin, H, W)).astype(np.float32)
    w = (rng.standard_normal((Cout, Cin, k, k)) * 0.6 / k).astype(np.float32)
    scale = rng.uniform(0.5, 1.5, Cout).astype(np.float32)
    bias = rng.normal(0.3, 0.2, Cout).astype(np.float32)
    plain = run_stem(x, w, scale, bias, T, "none", 2.0, Tin, stride)      # [T][B][C][OH][OW]
    d = rt.make_desc(T=T, B=B, Cin=Cin, H=H, W=W, Cout=Cout, KH=k, KW=k, stride=stride,
                     pad=k // 2, neuron=case["neuron"], tau=case["tau"])
    OH, OW = plain.shape[3], plain.shape[4]
    n_out = T * B * OH * OW * Cout
    bufs = [torch.full((n_out + GUARD,), SENTINEL, dtype=torch.float16, device="cuda")
            for _ in range(2)]
    xd, wd, sd, bd = (torch.from_numpy(a).cuda() for a in (x, w, scale, bias))
    rc = lib.snn_stem_forward_dual(ctypes.byref(d), Tin, xd.data_ptr(), wd.data_ptr(),
                                   sd.data_ptr(), bd.data_ptr(), bufs[0].data_ptr(),
                                   bufs[1].data_ptr(), None)
    assert rc == 0, lib.snn_last_error_message()
    torch.cuda.synchronize()
    assert rt.device_error() == 0
    for b in bufs:
        assert bool((b[n_out:] == SENTINEL).all()), "dual stem wrote past an output"
    conv = lambda t: np.transpose(t[:n_out].float().cpu().numpy().reshape(T, B, OH, OW, Cout),  # noqa: E731
                                  (0, 1, 4, 2, 3))
    bn, spikes = conv(bufs[0]), conv(bufs[1])
    assert np.array_equal(bn, plain)
    ref, _, _ = L.multistep_lif(bn, tau=case["tau"], neuron=case["neuron"])
    assert np.array_equal(spikes, ref)
    assert 0.02 < ref.mean() < 0.9


@pytest.mark.parametrize("case", [
    dict(H=12, W=140, Cout=48, k=3, stride=1, Tin=1, neuron="lif", tau=2.0),     # Spikformer's
    dict(H=29, W=29, Cout=64, k=7, stride=2, Tin=1, neuron="if", tau=2.0),
    dict(H=30, W=36, Cout=32, k=7, stride=2, Tin=8, Cin=2, neuron="lif", tau=3.0),
    dict(H=16, W=16, Cout=16, k=3, stride=1, Tin=1, neuron="lif", tau=2.0),
    dict(H=32, W=32, Cout=64, k=3, stride=1, Tin=1, neuron="lif", tau=2.0),     # CIFAR geometry
], ids=["c48_w140", "rgb7x7s2_if", "frames_tau3", "c16", "cifar"])
def test_stem_bit_packed_output(cuda_device, case):
    """SNN_FLAG_SPIKE_BITS: the stem's spikes bit-packed ([T*B][OH][OW][C/8]
    bytes, channel c in bit c%8 of byte c/8) unpack to the fp16 spikes of the
    same general stem bit for bit (the CIFAR geometry's fp16 spikes come
    from the row-tiled kernel: there the oracle's parity rule), and nothing
    past the packed tensor is written."""
    import torch
    from sparsesnn_b200 import runtime as rt
    lib = rt.load()
    rng = np.random.default_rng(33)
    Cin, k, stride, Tin = case.get("Cin", 3), case["k"], case["stride"], case["Tin"]
    T, B = max(4, Tin), 3
    H, W, Cout = case["H"], case["W"], case["Cout"]
    x = rng.standard_normal((Tin, B, Cin, H, W)).astype(np.float32)
    w = (rng.standard_normal((Cout, Cin, k, k)) * 0.9 / k).astype(np.float32)
    scale = rng.uniform(0.5, 1.5, Cout).astype(np.float32)
    bias = rng.normal(0.3, 0.2, Cout).astype(np.float32)
    fp16 = run_stem(x, w, scale, bias, T, case["neuron"], case["tau"], Tin, stride)
    d = rt.make_desc(T=T, B=B, Cin=Cin, H=H, W=W, Cout=Cout, KH=k, KW=k, stride=stride,
                     pad=k // 2, neuron=case["neuron"], tau=case["tau"],
                     flags=rt.SNN_FLAG_SPIKE_BITS)
    OH, OW = fp16.shape[3], fp16.shape[4]
    n_out = T * B * OH * OW * Cout // 8
    buf = torch.full((n_out + GUARD,), 0xA5, dtype=torch.uint8, device="cuda")
    xd, wd, sd, bd = (torch.from_numpy(a).cuda() for a in (x, w, scale, bias))
    rc = lib.snn_stem_forward(ctypes.byref(d), Tin, xd.data_ptr(), wd.data_ptr(), sd.data_ptr(),
                              bd.data_ptr(), buf.data_ptr(), None)
    assert rc == 0, lib.snn_last_error_message()
    torch.cuda.synchronize()
    assert rt.device_error() == 0
    assert bool((buf[n_out:] == 0xA5).all()), "bit-packed stem wrote past its output"
    packed = buf[:n_out].cpu().numpy().reshape(T, B, OH, OW, Cout // 8)
    got = np.transpose(np.unpackbits(packed, axis=-1, bitorder="little").astype(np.float32),
                       (0, 1, 4, 2, 3))
    if Cout == 64 and k == 3 and stride == 1 and Tin == 1:      # fp16 from the row-tiled kernel
        spk, h, _ = reference(x, w, scale, bias, T, case["neuron"], case["tau"], stride)
        frac, ok, _, _ = L.spike_agreement(got, spk, h)
        assert frac >= 0.995 and ok, frac
    else:
        assert np.array_equal(got, fp16)
    assert 0.02 < got.mean() < 0.9
