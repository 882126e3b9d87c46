"""Persistent conv kernels walking several pixel tiles per CTA.

Each kernel launches at most one CTA per SM (per 128-channel slice) and a CTA
walks pixel tiles until they run out, so the second and later tiles of a CTA
reuse its staging buffers, accumulators and mbarrier phases.  These cases
have several times more tiles than CTAs for every variant the library routes
SEW-ResNet-18 layers to, and compare spikes and final membranes with the
torch-CPU oracle (``oracle.lif_layer.fused_layer_torch``) under the same
parity rule as the golden cases.
"""
import numpy as np
import pytest

from oracle import lif_layer as L

pytestmark = pytest.mark.gpu

SMS = 148


def to_nhwc(x):
    t, b, c, h, w = x.shape
    return np.ascontiguousarray(np.transpose(x, (0, 1, 3, 4, 2)).reshape(t * b, h, w, c))


def from_nhwc(y, T, B):
    tb, h, w, c = y.shape
    return np.transpose(y.reshape(T, B, h, w, c), (0, 1, 4, 2, 3))


def check(spk, v, ref):
    st = {}
    frac, ok, nmis, div = L.spike_agreement(spk, ref["spikes"], ref["h"], stats=st)
    print(f"agreement {frac:.6f}: {st['first']} first mismatches, {st['later']} later excused "
          f"({st['later_off_band']} off band), {st['diverged']}/{st['neurons']} neurons diverged")
    assert frac >= 0.995 and ok, frac
    keep = ~div
    err = np.abs(v - ref["v"])[keep]
    assert (err <= 1e-2 * np.abs(ref["v"][keep]) + 1e-3).all(), err.max()


@pytest.mark.parametrize("name, T, B, C, F, H, stride, k, variant, tiles", [
    # four-timestep halo kernel (<= 64 channels): 8x8-pixel tiles, grid <= 148
    ("halo4", 4, 32, 64, 64, 32, 1, 3, 1, 32 * 16),
    # 128-channel resident halo kernel: 8x16-pixel tiles, one 128-channel slice
    ("halo_m128", 4, 160, 128, 128, 16, 1, 3, 1, 160 * 2),
    # streaming halo kernel, 8x8 images: one tile per image, 74 CTAs per slice
    ("halo_stream_8x8", 4, 160, 256, 256, 8, 1, 3, 2, 160),
    # streaming halo kernel, 4x4 images: four images per tile, 37 CTAs per slice
    ("halo_stream_4x4", 4, 400, 512, 512, 4, 1, 3, 2, 100),
    # general kernel, strided 3x3 (TC = 4, 64-pixel tiles of whole rows)
    ("general_s2", 4, 200, 128, 256, 16, 2, 3, 0, 200),
    # general kernel, 1x1 stride-2 downsample
    ("general_1x1", 4, 128, 64, 128, 32, 2, 1, 0, 128 * 4),
])
@pytest.mark.parametrize("residual", [False, True], ids=["plain", "res"])
def test_many_tiles_per_cta(cuda_device, name, T, B, C, F, H, stride, k, variant, tiles,
                            residual):
    import torch
    from sparsesnn_b200 import runtime as rt
    from sparsesnn_b200.layer import SparseConvBNLIF, fold_bn
    x, w, bn = L.make_config0(seed=B + C + F + H, T=T, B=B, C=C, F=F, H=H, W=H, k=k)
    scale, bias = fold_bn(bn.gamma, bn.beta, bn.mean, bn.var)
    layer = SparseConvBNLIF(w, scale, bias, T=T, B=B, H=H, W=H, stride=stride, pad=k // 2)
    assert rt.variant(layer.desc) == variant
    n_m = (F + 127) // 128
    per_cta = tiles / min(tiles, SMS // n_m)
    assert per_cta >= 2, "the case must give each CTA at least two tiles on average"
    oh, ow = layer.OH, layer.OW
    res_np = None
    rd = None
    if residual:
        rng = np.random.default_rng(B)
        res_np = rng.integers(0, 3, (T, B, F, oh, ow)).astype(np.float32)
        rd = torch.from_numpy(to_nhwc(res_np)).to("cuda", torch.float16)
    xd = torch.from_numpy(to_nhwc(x)).to("cuda", torch.float16)
    st = torch.full(layer.state_shape(), 5.0, dtype=torch.float32, device="cuda")
    y = layer(xd, state=st, residual=rd, read_state=False)
    torch.cuda.synchronize()
    assert rt.device_error() == 0
    # fp16-rounded weights: the kernel's operand (K up to 4608)
    w16 = w.astype(np.float16).astype(np.float32)
    ref = L.fused_layer_torch(x, w16, bn, stride=stride, pad=k // 2)
    ys = from_nhwc(y.float().cpu().numpy(), T, B)
    spk = ys - res_np if residual else ys
    assert set(np.unique(spk)) <= {0.0, 1.0}
    v = np.transpose(st.cpu().numpy().reshape(B, oh, ow, F), (0, 3, 1, 2))
    check(spk, v, ref)
