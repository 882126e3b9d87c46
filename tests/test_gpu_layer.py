"""GPU parity of the fused 2:4-sparse Conv/Linear + BN + LIF layer.

Checks, on every reference golden case and at the config-0 full size:
* spikes agree at >= 99.5% of positions, and every neuron's first mismatch
  lies at |h - v_th| < 1e-2 (h = reference pre-reset membrane);
* final membrane within rtol 1e-2 (+ atol 1e-3) on neurons whose spike
  trains agree;
* BN pre-activations (neuron disabled) within the error of FP16 weight
  rounding of the fp32 reference, and within 1e-5 relative of the oracle
  run with the same FP16-rounded weights (accumulation order only).
"""
import numpy as np
import pytest

from conftest import LAYER_CASES, RES_CASES, load_layer_case
from oracle import lif_layer as L

pytestmark = pytest.mark.gpu

V_RTOL, V_ATOL = 1e-2, 1e-3
SPIKE_MIN_AGREE = 0.995


def to_nhwc(x_tbchw):
    t, b, c, h, w = x_tbchw.shape
    return np.ascontiguousarray(np.transpose(x_tbchw, (0, 1, 3, 4, 2)).reshape(t * b, h, w, c))


def from_nhwc(y, T, B):
    tb, oh, ow, f = y.shape
    return np.transpose(y.reshape(T, B, oh, ow, f), (0, 1, 4, 2, 3))


def build_layer(g, neuron=None, device="cuda", force_generic=False):
    from sparsesnn_b200.layer import SparseConvBNLIF, fold_bn
    mean = g["mean"] - g["lin_bias"] if g["linear"] else g["mean"]
    scale, bias = fold_bn(g["gamma"], g["beta"], mean, g["var"])
    neuron = neuron or g["neuron"]
    if g["linear"]:
        # Spikformer Linear over N = H*W tokens: rows = B*N, one "image" row.
        return SparseConvBNLIF(g["w"][:, :, 0, 0], scale, bias, T=g["T"], B=1, H=1,
                               W=g["B"] * g["H"] * g["W"], neuron=neuron, device=device,
                               force_generic=force_generic)
    return SparseConvBNLIF(g["w"], scale, bias, T=g["T"], B=g["B"], H=g["H"], W=g["W"],
                           stride=g["stride"], pad=g["pad"], neuron=neuron, device=device,
                           force_generic=force_generic)


def layer_input(g):
    x = g["x"].astype(np.float32)
    if g["linear"]:
        T, B, C = x.shape[:3]
        tok = np.transpose(x.reshape(T, B, C, -1), (0, 1, 3, 2))       # (T,B,N,C)
        return np.ascontiguousarray(tok.reshape(T, 1, B * tok.shape[2], C))
    return to_nhwc(x)


def run_case(g, neuron=None, residual=None, force_generic=False):
    import torch
    from sparsesnn_b200 import runtime as rt
    layer = build_layer(g, neuron, force_generic=force_generic)
    x = torch.from_numpy(layer_input(g)).to("cuda", torch.float16)
    state = torch.full(layer.state_shape(), 123.0, dtype=torch.float32, device="cuda")
    res = None
    if residual is not None:
        res = torch.from_numpy(to_nhwc(residual.astype(np.float32))).to("cuda", torch.float16)
    out = layer(x, state=state, residual=res, read_state=False)
    torch.cuda.synchronize()
    assert rt.device_error() == 0
    return out.float().cpu().numpy(), state.cpu().numpy(), layer


def unflatten(g, y, state=None):
    """Kernel layouts -> reference layouts: y (T,B,F,OH,OW), v (B,F,OH,OW)."""
    T, B, F = g["T"], g["B"], g["F"]
    if g["linear"]:
        H, W = g["H"], g["W"]
        ys = np.transpose(y.reshape(T, B, H, W, F), (0, 1, 4, 2, 3))
    else:
        ys = from_nhwc(y, T, B)
    oh, ow = ys.shape[3:]
    v = None if state is None else np.transpose(state.reshape(B, oh, ow, F), (0, 3, 1, 2))
    return ys, v


def check_spikes_and_v(spk, v, ref_spk, ref_h, ref_v):
    st = {}
    frac, explained, nmis, diverged = L.spike_agreement(spk, ref_spk, ref_h, stats=st)
    # The first-mismatch rule excuses a diverged neuron's later steps: report them.
    print(f"spikes: agreement {frac:.6f}, {st['first']} first mismatches (in band), "
          f"{st['later']} later excused ({st['later_off_band']} off band), "
          f"{st['diverged']}/{st['neurons']} neurons diverged")
    assert frac >= SPIKE_MIN_AGREE, f"spike agreement {frac:.5f}"
    assert explained, "a spike mismatch lies away from the threshold band"
    keep = ~diverged
    err = np.abs(v - ref_v)[keep]
    assert (err <= V_RTOL * np.abs(ref_v[keep]) + V_ATOL).all(), f"max v err {err.max()}"
    return frac, nmis


@pytest.mark.parametrize("generic", [False, True], ids=["auto", "generic"])
@pytest.mark.parametrize("name", LAYER_CASES)
def test_golden_layer_parity(cuda_device, name, generic):
    """Every golden case through the kernel the library picks (the halo
    kernel for stride-1 3x3 layers on images >= 8 rows) and through the
    general kernel."""
    g = load_layer_case(name)
    res = g.get("residual")
    y, state, _ = run_case(g, residual=res, force_generic=generic)
    ys, v = unflatten(g, y, state)
    if res is not None:
        spk = ys - res.astype(np.float32)
        assert np.isin(spk, (0.0, 1.0)).all()
        assert np.isin(ys, (0, 1, 2, 3)).all()
    else:
        spk = ys
        assert np.isin(spk, (0.0, 1.0)).all()
    check_spikes_and_v(spk, v, g["spikes"].astype(np.float32), g["h"], g["v"])


@pytest.mark.parametrize("generic", [False, True], ids=["auto", "generic"])
@pytest.mark.parametrize("name", ["c3s1", "c3s2", "c1s2", "c3res", "lin"])
def test_golden_preactivation(cuda_device, name, generic):
    g = load_layer_case(name)
    y, _, _ = run_case(g, neuron="none", force_generic=generic)
    z, _ = unflatten(g, y)
    ref = g["bn_out"]
    # vs the fp32 reference: FP16 weight rounding bounds the error.
    scale = np.abs(ref).max()
    assert np.abs(z - ref).max() <= 5e-3 * scale
    # vs the oracle on FP16-rounded weights: accumulation order only.
    w16 = g["w"].astype(np.float16).astype(np.float32)
    mean = g["mean"] - g["lin_bias"] if g["linear"] else g["mean"]
    bn = L.BNParams(g["gamma"], g["beta"], mean, g["var"])
    x = g["x"].astype(np.float32)
    if g["linear"]:
        r = L.fused_layer(x, w16, bn, stride=1, pad=0)["bn_out"]
    else:
        r = L.fused_layer(x, w16, bn, stride=g["stride"], pad=g["pad"])["bn_out"]
    assert np.abs(z - r).max() <= 1e-5 * max(scale, 1.0)


def test_state_read_and_two_calls(cuda_device):
    """Running T=4 as two T=2 calls with the membrane carried through state
    equals one T=4 call (reads v0 from state, writes final v)."""
    import torch
    g = load_layer_case("c3s1")
    full, state_full, _ = run_case(g)
    g2 = dict(g, T=2)
    layer = build_layer(g2)
    x = torch.from_numpy(layer_input(g)).to("cuda", torch.float16)
    half = x.shape[0] // 2
    state = torch.zeros(layer.state_shape(), dtype=torch.float32, device="cuda")
    o1 = layer(x[:half].contiguous(), state=state)
    o2 = layer(x[half:].contiguous(), state=state)
    torch.cuda.synchronize()
    got = torch.cat([o1, o2]).float().cpu().numpy()
    assert np.array_equal(got, full)
    assert np.array_equal(state.cpu().numpy(), state_full)


def test_long_t_chunking(cuda_device):
    """T=10 (> 4 timesteps per tensor-memory chunk) against the oracle."""
    import torch
    g = load_layer_case("c3s1")
    rng = np.random.default_rng(11)
    T = 10
    x = (rng.random((T, g["B"], g["C"], g["H"], g["W"])) < 0.2).astype(np.float32)
    gg = dict(g, T=T, x=x)
    y, state, _ = run_case(gg)
    ys, v = unflatten(gg, y, state)
    bn = L.BNParams(g["gamma"], g["beta"], g["mean"], g["var"])
    r = L.fused_layer(x, g["w"], bn, stride=1, pad=1)
    check_spikes_and_v(ys, v, r["spikes"], r["h"], r["v"])


def _torch_reference(x_tbchw, w, scale, bias, stride, pad, tau=2.0, v_th=1.0):
    """Plain PyTorch fp32 reference of the same op (TF32 off), on the GPU."""
    import torch
    import torch.nn.functional as F
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False
    T, B = x_tbchw.shape[:2]
    z = F.conv2d(x_tbchw.flatten(0, 1), w, stride=stride, padding=pad)
    z = z * scale[None, :, None, None] + bias[None, :, None, None]
    z = z.view(T, B, *z.shape[1:])
    v = torch.zeros_like(z[0])
    spk, hs = [], []
    for t in range(T):
        v = v * (1.0 - 1.0 / tau) + z[t] / tau
        hs.append(v)
        s = (v - v_th).ge(0).float()
        v = (1.0 - s) * v
        spk.append(s)
    return torch.stack(spk), torch.stack(hs), v


@pytest.mark.parametrize("generic", [False, True], ids=["halo", "generic"])
def test_config0_full_size(cuda_device, generic):
    """Config 0: 3x3 s1 p1, Cin=Cout=128, 32x32, B=16, T=4."""
    import torch
    from sparsesnn_b200.layer import SparseConvBNLIF, fold_bn
    x, w, bn = L.make_config0(seed=0)
    scale, bias = fold_bn(bn.gamma, bn.beta, bn.mean, bn.var)
    layer = SparseConvBNLIF(w, scale, bias, T=4, B=16, H=32, W=32, force_generic=generic)
    xd = torch.from_numpy(to_nhwc(x)).to("cuda", torch.float16)
    state = torch.zeros(layer.state_shape(), dtype=torch.float32, device="cuda")
    y = layer(xd, state=state, read_state=False)
    torch.cuda.synchronize()
    from sparsesnn_b200 import runtime as rt
    assert rt.device_error() == 0
    xt = torch.from_numpy(x).cuda()
    spk, h, v = _torch_reference(xt, torch.from_numpy(w).cuda(), torch.from_numpy(scale).cuda(),
                                 torch.from_numpy(bias).cuda(), 1, 1)
    ys = from_nhwc(y.float().cpu().numpy(), 4, 16)
    vg = np.transpose(state.cpu().numpy().reshape(16, 32, 32, 128), (0, 3, 1, 2))
    frac, nmis = check_spikes_and_v(ys, vg, spk.cpu().numpy(), h.cpu().numpy(), v.cpu().numpy())
    print(f"config0 spike agreement {frac:.6f} ({nmis} mismatches)")


def test_size_independent_properties(cuda_device):
    """Large-batch properties: outputs are exact {0,1}, a zero input gives the
    BN-bias-only trajectory, and batch images are independent (permuting the
    batch permutes the output)."""
    import torch
    from sparsesnn_b200.layer import SparseConvBNLIF, fold_bn
    x, w, bn = L.make_config0(seed=1, B=32, C=256, F=256, H=16, W=16)
    scale, bias = fold_bn(bn.gamma, bn.beta, bn.mean, bn.var)
    layer = SparseConvBNLIF(w, scale, bias, T=4, B=32, H=16, W=16)
    xd = torch.from_numpy(to_nhwc(x)).to("cuda", torch.float16)
    y = layer(xd)
    perm = torch.randperm(32, generator=torch.Generator().manual_seed(0))
    xp = xd.view(4, 32, 16, 16, 256)[:, perm].reshape_as(xd).contiguous()
    yp = layer(xp)
    torch.cuda.synchronize()
    assert torch.equal(y.view(4, 32, 16, 16, 256)[:, perm], yp.view(4, 32, 16, 16, 256))
    assert set(torch.unique(y).tolist()) <= {0.0, 1.0}
    y0 = layer(torch.zeros_like(xd))
    torch.cuda.synchronize()
    # zero input: every pixel of a channel follows the same bias-driven trajectory
    y0 = y0.view(4, -1, 256).float()
    assert torch.equal(y0.amax(dim=1), y0.amin(dim=1))
    z = torch.from_numpy(bias)
    v = torch.zeros_like(z)
    for t in range(4):
        v = v * 0.5 + z / 2.0
        s = (v - 1.0).ge(0).float()
        v = (1.0 - s) * v
        assert torch.equal(y0[t, 0].cpu(), s)


@pytest.mark.parametrize("T", [1, 2, 3, 4])
@pytest.mark.parametrize("residual", [False, True], ids=["plain", "res"])
def test_halo_stream_variant(cuda_device, T, residual):
    """Streaming-weight halo kernel (Cin=256 on 12x12, 8x12, 8x8 and 4x4
    images; 4x4 takes four images per tile from three column-shifted boxes,
    here with a ragged last tile of 3 images) against the oracle, for every
    timestep count it serves (one N = 64*T MMA per tap) and with the SEW
    residual."""
    import torch
    from sparsesnn_b200 import runtime as rt
    from sparsesnn_b200.layer import SparseConvBNLIF, fold_bn
    for (H, W) in ((12, 12), (8, 12), (8, 8), (4, 4)):
        x, w, bn = L.make_config0(seed=10 + T, T=T, B=3, C=256, F=256, H=H, W=W)
        scale, bias = fold_bn(bn.gamma, bn.beta, bn.mean, bn.var)
        layer = SparseConvBNLIF(w, scale, bias, T=T, B=3, H=H, W=W)
        assert rt.variant(layer.desc) == rt.SNN_VARIANT_HALO_STREAM
        xd = torch.from_numpy(to_nhwc(x)).to("cuda", torch.float16)
        res_np = None
        res = None
        if residual:
            rng = np.random.default_rng(T)
            res_np = rng.integers(0, 3, (T, 3, 256, H, W)).astype(np.float32)
            res = torch.from_numpy(to_nhwc(res_np)).to("cuda", torch.float16)
        state = torch.zeros(layer.state_shape(), dtype=torch.float32, device="cuda")
        y = layer(xd, state=state, residual=res, read_state=False)
        torch.cuda.synchronize()
        assert rt.device_error() == 0
        r = L.fused_layer(x, w, bn, stride=1, pad=1)
        ys = from_nhwc(y.float().cpu().numpy(), T, 3)
        spk = ys - res_np if residual else ys
        v = np.transpose(state.cpu().numpy().reshape(3, H, W, 256), (0, 3, 1, 2))
        check_spikes_and_v(spk, v, r["spikes"], r["h"], r["v"])


@pytest.mark.parametrize("T", [1, 3, 4])
@pytest.mark.parametrize("residual", [False, True], ids=["plain", "res"])
def test_m64_halo_path(cuda_device, T, residual):
    """Layers with at most 64 output channels run M = 64 MMAs (metadata
    remapped to the M = 64 TMEM layout, spikes through tiles shared by four
    warps).  Odd T checks partial passes across pixel tiles; a second call
    with the membrane carried over checks the state read/write."""
    import torch
    from sparsesnn_b200 import runtime as rt
    from sparsesnn_b200.layer import SparseConvBNLIF, fold_bn
    B, H, W = 3, 16, 24
    for F in (64, 32):
        x, w, bn = L.make_config0(seed=20 + T + F, T=2 * T, B=B, C=64, F=F, H=H, W=W)
        scale, bias = fold_bn(bn.gamma, bn.beta, bn.mean, bn.var)
        layer = SparseConvBNLIF(w, scale, bias, T=T, B=B, H=H, W=W)
        assert rt.variant(layer.desc) == rt.SNN_VARIANT_HALO_RESIDENT
        res_np = None
        if residual:
            rng = np.random.default_rng(T + F)
            res_np = rng.integers(0, 3, (2 * T, B, F, H, W)).astype(np.float32)
        state = torch.zeros(layer.state_shape(), dtype=torch.float32, device="cuda")
        outs = []
        for half in range(2):                 # two calls, membrane carried over
            sl = slice(half * T, (half + 1) * T)
            xd = torch.from_numpy(to_nhwc(x[sl])).to("cuda", torch.float16)
            res = (torch.from_numpy(to_nhwc(res_np[sl])).to("cuda", torch.float16)
                   if residual else None)
            outs.append(layer(xd, state=state, residual=res).float().cpu().numpy())
        torch.cuda.synchronize()
        assert rt.device_error() == 0
        r = L.fused_layer(x, w, bn, stride=1, pad=1)
        ys = np.concatenate([from_nhwc(o, T, B) for o in outs], axis=0)
        spk = ys - res_np if residual else ys
        v = np.transpose(state.cpu().numpy().reshape(B, H, W, F), (0, 3, 1, 2))
        check_spikes_and_v(spk, v, r["spikes"], r["h"], r["v"])


@pytest.mark.parametrize("cin, F, H, W, T, neuron, tau", [
    (64, 64, 8, 8, 4, "lif", 2.0),        # one tile per image
    (64, 64, 12, 20, 5, "lif", 2.0),      # ragged tiles, a second pass with one timestep
    (64, 48, 17, 9, 6, "lif", 3.0),       # Cout < 64, general tau, two passes
    (128, 64, 10, 16, 3, "if", 2.0),      # two 64-channel input blocks, IF
    (64, 32, 16, 16, 8, "lif", 2.0),      # two full passes
], ids=["8x8", "ragged_T5", "c48_tau3_T6", "cin128_if_T3", "c32_T8"])
@pytest.mark.parametrize("residual", [False, True], ids=["plain", "res"])
def test_halo4_path(cuda_device, cin, F, H, W, T, neuron, tau, residual):
    """Spiking layers with at most 64 output channels run the four-timestep
    halo kernel: N = 256 MMAs over 8 x 8 pixels x 4 timesteps from a
    (C, W, T, H, B) tensor map.  Ragged images, T not a multiple of four
    (timesteps past T read as zero and are not stored), Cin of two blocks,
    both neurons and a membrane carried between two calls."""
    import torch
    from sparsesnn_b200 import runtime as rt
    from sparsesnn_b200.layer import SparseConvBNLIF, fold_bn
    B = 2
    x, w, bn = L.make_config0(seed=7 * T + F + cin, T=2 * T, B=B, C=cin, F=F, H=H, W=W)
    scale, bias = fold_bn(bn.gamma, bn.beta, bn.mean, bn.var)
    layer = SparseConvBNLIF(w, scale, bias, T=T, B=B, H=H, W=W, neuron=neuron, tau=tau)
    assert rt.variant(layer.desc) == rt.SNN_VARIANT_HALO_RESIDENT
    res_np = None
    if residual:
        rng = np.random.default_rng(T + F)
        res_np = rng.integers(0, 3, (2 * T, B, F, H, W)).astype(np.float32)
    state = torch.zeros(layer.state_shape(), dtype=torch.float32, device="cuda")
    outs = []
    for part in range(2):                     # two calls, membrane carried over
        sl = slice(part * T, (part + 1) * T)
        xd = torch.from_numpy(to_nhwc(x[sl])).to("cuda", torch.float16)
        res = (torch.from_numpy(to_nhwc(res_np[sl])).to("cuda", torch.float16)
               if residual else None)
        outs.append(layer(xd, state=state, residual=res).float().cpu().numpy())
    torch.cuda.synchronize()
    assert rt.device_error() == 0
    # The oracle on the kernel's fp16-rounded weights: an IF membrane integrates
    # the weight rounding error of K = 1152 without decay.
    w16 = w.astype(np.float16).astype(np.float32)
    r = L.fused_layer(x, w16, bn, stride=1, pad=1, neuron=neuron, tau=tau)
    ys = np.concatenate([from_nhwc(o, T, B) for o in outs], axis=0)
    spk = ys - res_np if residual else ys
    assert set(np.unique(spk)) <= {0.0, 1.0}
    v = np.transpose(state.cpu().numpy().reshape(B, H, W, F), (0, 3, 1, 2))
    check_spikes_and_v(spk, v, r["spikes"], r["h"], r["v"])


@pytest.mark.parametrize("cin, cout", [(384, 1536), (1536, 384), (384, 384)],
                         ids=["fc1", "fc2", "qkv"])
def test_spikformer_linear_shapes(cuda_device, cin, cout):
    """The Linear + BN + LIF twin at Spikformer-8-384 feature sizes (tokens of
    4 images x 196 patches as rows; 2:4 along the input dim) against the
    oracle run as a 1x1 conv over the rows."""
    import torch
    from sparsesnn_b200 import runtime as rt
    from sparsesnn_b200.layer import SparseConvBNLIF, fold_bn
    T, rows = 4, 4 * 196
    x, w, bn = L.make_config0(seed=31 + cin, T=T, B=1, C=cin, F=cout, H=1, W=rows, k=1)
    scale, bias = fold_bn(bn.gamma, bn.beta, bn.mean, bn.var)
    layer = SparseConvBNLIF(w[:, :, 0, 0], scale, bias, T=T, B=1, H=1, W=rows)
    xd = torch.from_numpy(to_nhwc(x)).to("cuda", torch.float16)
    state = torch.zeros(layer.state_shape(), dtype=torch.float32, device="cuda")
    y = layer(xd, state=state, read_state=False)
    torch.cuda.synchronize()
    assert rt.device_error() == 0
    r = L.fused_layer(x, w, bn, stride=1, pad=0)
    ys = from_nhwc(y.float().cpu().numpy(), T, 1)
    v = np.transpose(state.cpu().numpy().reshape(1, 1, rows, cout), (0, 3, 1, 2))
    check_spikes_and_v(ys, v, r["spikes"], r["h"], r["v"])


# ------------------------------------------------------------- residual modes
BAND = 1e-2


def check_two_neuron(out, v1, v2, ref, v_th=1.0, v_th2=1.0):
    """Parity rule for neuron2(neuron(bn) + residual): a neuron's first output
    mismatch must lie where the second neuron's pre-reset membrane is within
    the band of its threshold, or where the first neuron was within its band
    at this or an earlier step (its spike may have flipped there).  Final
    membranes are compared on neurons that never came near either threshold."""
    s2 = ref["spikes2"].astype(np.float32)
    mism = out != s2
    frac = 1.0 - float(mism.mean())
    assert frac >= SPIKE_MIN_AGREE, f"spike agreement {frac:.5f}"
    near1 = np.maximum.accumulate(np.abs(ref["h"] - v_th) < BAND, axis=0)
    near2 = np.abs(ref["h2"] - v_th2) < BAND
    seen = np.zeros(mism.shape[1:], bool)
    for t in range(mism.shape[0]):
        first = mism[t] & ~seen
        assert not (first & ~near1[t] & ~near2[t]).any(), f"unexplained mismatch at t={t}"
        seen |= mism[t]
    clean1 = ~near1[-1]
    clean2 = clean1 & ~seen & ~near2.any(axis=0)
    for v, rv, keep in ((v1, ref["v"], clean1), (v2, ref["v2"], clean2)):
        err = np.abs(v - rv)[keep]
        assert (err <= V_RTOL * np.abs(rv[keep]) + V_ATOL).all(), f"max v err {err.max()}"


def run_res_layer(x, w, bn, res, *, T, B, H, W, stride=1, pad=None, neuron="lif", tau=2.0,
                  res_mode="add_before", neuron2="lif", tau2=2.0, force_generic=False,
                  state_init=None):
    import torch
    from sparsesnn_b200 import runtime as rt
    from sparsesnn_b200.layer import SparseConvBNLIF, fold_bn
    scale, bias = fold_bn(bn.gamma, bn.beta, bn.mean, bn.var)
    layer = SparseConvBNLIF(w, scale, bias, T=T, B=B, H=H, W=W, stride=stride, pad=pad,
                            neuron=neuron, tau=tau, res_mode=res_mode, neuron2=neuron2,
                            tau2=tau2, force_generic=force_generic)
    assert rt.variant(layer.desc) == rt.SNN_VARIANT_GENERIC
    xd = torch.from_numpy(to_nhwc(x)).to("cuda", torch.float16)
    rd = torch.from_numpy(to_nhwc(res)).to("cuda", torch.float16)
    st = torch.full(layer.state_shape(), 123.0, dtype=torch.float32, device="cuda")
    st2 = torch.full(layer.state_shape(), -7.0, dtype=torch.float32, device="cuda") \
        if res_mode == "two_neuron" else None
    y = layer(xd, state=st, residual=rd, read_state=False, state2=st2)
    torch.cuda.synchronize()
    assert rt.device_error() == 0
    oh, ow = layer.OH, layer.OW
    F = w.shape[0]
    ys = from_nhwc(y.float().cpu().numpy(), T, B)
    to_bfhw = lambda s: np.transpose(s.cpu().numpy().reshape(B, oh, ow, F), (0, 3, 1, 2))
    return ys, to_bfhw(st), (to_bfhw(st2) if st2 is not None else None)


@pytest.mark.parametrize("generic", [False, True], ids=["auto", "generic"])
@pytest.mark.parametrize("name", RES_CASES)
def test_golden_residual_modes(cuda_device, name, generic):
    """The reference's Add-before-LIF and IF+Add+LIF epilogues against its
    own modules' outputs (golden fixtures)."""
    g = load_layer_case(name)
    bn = L.BNParams(g["gamma"], g["beta"], g["mean"], g["var"])
    ys, v, v2 = run_res_layer(g["x"].astype(np.float32), g["w"], bn, g["residual"], T=g["T"],
                              B=g["B"], H=g["H"], W=g["W"], pad=g["pad"], neuron=g["neuron"],
                              res_mode=g["res_mode"], neuron2=g["neuron2"],
                              force_generic=generic)
    assert np.isin(ys, (0.0, 1.0)).all()
    if g["res_mode"] == "two_neuron":
        check_two_neuron(ys, v, v2, g)
    else:
        check_spikes_and_v(ys, v, g["spikes"].astype(np.float32), g["h"], g["v"])


@pytest.mark.parametrize("T", [4, 3], ids=["T4", "T3"])
@pytest.mark.parametrize("mode, neuron, tau, neuron2, tau2", [
    ("add_before", "lif", 2.0, "lif", 2.0),
    ("add_before", "lif", 3.0, "lif", 2.0),
    ("add_before", "if", 2.0, "lif", 2.0),
    ("two_neuron", "if", 2.0, "lif", 2.0),
    ("two_neuron", "lif", 2.0, "lif", 3.0),
    ("two_neuron", "lif", 3.0, "if", 2.0),
], ids=["addlif", "addlif_tau3", "addif", "if_add_lif", "lif_add_lif3", "lif3_add_if"])
@pytest.mark.parametrize("k", [3, 1])
def test_residual_modes_vs_oracle(cuda_device, T, mode, neuron, tau, neuron2, tau2, k):
    """Every neuron combination of both epilogues, 3x3 and 1x1, with four
    timesteps per accumulator (T=4) and two (T=3), 192 output channels (a
    partial 128-channel tile), real-valued residual."""
    B, C, F, H, W = 2, 64, 192, 8, 8
    x, w, bn = L.make_config0(seed=40 + T + k, T=T, B=B, C=C, F=F, H=H, W=W, k=k)
    rng = np.random.default_rng(50 + T)
    res = (rng.standard_normal((T, B, F, H, W)) * 0.5).astype(np.float16).astype(np.float32)
    ys, v, v2 = run_res_layer(x, w, bn, res, T=T, B=B, H=H, W=W, pad=k // 2, neuron=neuron,
                              tau=tau, res_mode=mode, neuron2=neuron2, tau2=tau2)
    r = L.fused_layer(x, w, bn, stride=1, pad=k // 2, tau=tau, neuron=neuron, residual=res,
                      res_mode=mode, neuron2=neuron2, tau2=tau2)
    assert np.isin(ys, (0.0, 1.0)).all()
    if mode == "two_neuron":
        check_two_neuron(ys, v, v2, r)
    else:
        check_spikes_and_v(ys, v, r["spikes"], r["h"], r["v"])


@pytest.mark.parametrize("cin, cout, hw, k, stride", [(256, 256, 8, 3, 1), (512, 512, 4, 3, 1),
                                                     (256, 512, 8, 3, 2)],
                         ids=["s3", "s4", "s4_strided"])
@pytest.mark.parametrize("residual", [False, True], ids=["plain", "res"])
@pytest.mark.parametrize("neuron", ["lif", "if"])
def test_cta_pair_path(cuda_device, cin, cout, hw, k, stride, residual, neuron):
    """Stage-3/4 shapes with an even number of 128-channel tiles on CTA pairs
    (SNN_FLAG_CTA_PAIR: one M = 256 MMA per 2-CTA cluster); parity with the
    oracle, and the same spikes and membranes as the one-CTA path."""
    import torch
    from sparsesnn_b200 import runtime as rt
    from sparsesnn_b200.layer import SparseConvBNLIF, fold_bn
    T, B = 4, 8
    x, w, bn = L.make_config0(seed=cin + cout + hw + k, T=T, B=B, C=cin, F=cout, H=hw, W=hw, k=k)
    scale, bias = fold_bn(bn.gamma, bn.beta, bn.mean, bn.var)
    outs = []
    for pair in (True, False):
        layer = SparseConvBNLIF(w, scale, bias, T=T, B=B, H=hw, W=hw, stride=stride, pad=k // 2,
                                neuron=neuron)
        if pair:
            layer.base_flags |= rt.SNN_FLAG_CTA_PAIR
        oh, ow = layer.OH, layer.OW
        rng = np.random.default_rng(7)
        res_np = rng.integers(0, 3, (T, B, cout, oh, ow)).astype(np.float32) if residual else None
        xd = torch.from_numpy(to_nhwc(x)).to("cuda", torch.float16)
        rd = torch.from_numpy(to_nhwc(res_np)).to("cuda", torch.float16) if residual else None
        st = torch.full(layer.state_shape(), 3.0, dtype=torch.float32, device="cuda")
        y = layer(xd, state=st, residual=rd, read_state=False)
        torch.cuda.synchronize()
        assert rt.device_error() == 0
        outs.append((y.float().cpu().numpy(), st.cpu().numpy()))
    (y_pair, st_pair), (y_one, st_one) = outs
    assert np.array_equal(y_pair, y_one)
    assert np.array_equal(st_pair, st_one)
    # The oracle on the kernel's fp16-rounded weights (K up to 4608: with IF
    # the fp32-weight reference drifts by the weight rounding alone).
    w16 = w.astype(np.float16).astype(np.float32)
    r = L.fused_layer(x, w16, bn, stride=stride, pad=k // 2, neuron=neuron)
    ys = from_nhwc(y_pair, T, B)
    spk = ys - res_np if residual else ys
    v = np.transpose(st_pair.reshape(B, oh, ow, cout), (0, 3, 1, 2))
    check_spikes_and_v(spk, v, r["spikes"], r["h"], r["v"])
