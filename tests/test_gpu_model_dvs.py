"""DVS SEW-ResNet-18 (config 4: 2-channel 128x128 event frames, T=16, the
reference's 7x7/2 stem + MaxPool(3,2,1)) on the B200 kernels at the per-GPU
batch of the 8-GPU run (4 images), against the CPU port of the reference
forward (pinned to the reference model class by ``sew18_dvs_logits.npz``).

* the stem (conv + BN + LIF on every timestep's frame) and the spike max
  pool against the oracle (the pool bit for bit);
* per-layer teacher forcing on all 19 fused conv launches over T=16 (four
  accumulator chunks of four timesteps, the membrane carried on chip);
* end to end: logits by the reference validator's rule, and the golden
  reference logits.
"""
import os

import numpy as np
import pytest

from oracle import lif_layer as L

pytestmark = pytest.mark.gpu

T, B = 16, 4


def to_nhwc(x):
    t, b, c, h, w = x.shape
    return np.ascontiguousarray(np.transpose(x, (0, 1, 3, 4, 2)).reshape(t * b, h, w, c))


def from_nhwc(y, T_, B_):
    tb, h, w, c = y.shape
    return np.transpose(y.reshape(T_, B_, h, w, c), (0, 1, 4, 2, 3))


def _bn(p):
    return L.BNParams(p["gamma"], p["beta"], p["mean"], p["var"])


def _params():
    from sparsesnn_b200.sew_resnet import init_params
    return init_params(seed=0, num_classes=11, in_channels=2, stem_kernel=7, input_moment=0.05)


@pytest.fixture(scope="module")
def setup(cuda_device):
    import torch
    from oracle.sew_resnet import forward_torch, make_dvs_input
    from sparsesnn_b200.sew_resnet import SEWResNet18DVS
    threads = os.cpu_count() or 1
    P = _params()
    x = make_dvs_input(seed=3, B=B, T=T)                       # [B, T, C, H, W]
    logits_ref, trace = forward_torch(P, x, T=T, stem_stride=2, maxpool=True,
                                      return_trace=True, threads=threads)
    model = SEWResNet18DVS(P, T=T, batch=B, device="cuda:0")
    x_tb = np.ascontiguousarray(np.transpose(x, (1, 0, 2, 3, 4)))   # time-major model input
    return P, x, x_tb, logits_ref, trace, model, torch, threads


def test_dvs_stem_and_pool(setup):
    import torch
    import torch.nn.functional as F
    P, x, x_tb, logits_ref, trace, model, torch, threads = setup
    model(torch.from_numpy(x_tb))
    torch.cuda.synchronize()
    from sparsesnn_b200 import runtime as rt
    stem = model.buffer("stem")
    if model.stem_desc.flags & rt.SNN_FLAG_SPIKE_BITS:       # bit-packed stem spikes
        got = from_nhwc(np.unpackbits(stem.cpu().numpy(), axis=-1, bitorder="little")
                        .astype(np.float32), T, B)
    else:
        got = from_nhwc(stem.float().cpu().numpy(), T, B)
    st = P["stem"]
    with torch.no_grad():
        z = F.conv2d(torch.from_numpy(x_tb).flatten(0, 1), torch.from_numpy(st["w"]), stride=2,
                     padding=3)
        s, b = _bn(st["bn"]).scale_bias()
        z = (z * torch.from_numpy(s)[None, :, None, None] + torch.from_numpy(b)[None, :, None, None])
    z = z.numpy().reshape((T, B) + z.shape[1:])
    _, h, _ = L.multistep_lif(z)
    stats = {}
    frac, ok, _, _ = L.spike_agreement(got, trace["stem"], h, stats=stats)
    print(f"stem agreement {frac:.6f} {stats}")
    assert frac >= 0.995 and ok
    # the pool of the GPU's own stem spikes, exactly
    pooled = from_nhwc(model.buffer("maxpool").float().cpu().numpy(), T, B)
    ref_pool = F.max_pool2d(torch.from_numpy(got).flatten(0, 1), 3, 2, 1).numpy()
    assert np.array_equal(pooled, ref_pool.reshape(pooled.shape))


def test_dvs_teacher_forced_layers(setup):
    from sparsesnn_b200 import runtime as rt
    P, x, x_tb, logits_ref, trace, model, torch, threads = setup
    convs = {n.name: n.layer for n in model.nodes if n.layer is not None}
    assert len(convs) == 19
    prev = trace["maxpool"]
    worst = (1.0, "")
    for i, p in enumerate(P["blocks"]):
        xin = torch.from_numpy(to_nhwc(prev)).to("cuda:0", torch.float16)
        pairs = [(f"b{i}.conv1", prev, p["w1"], p["bn1"], p["stride"], 1, None)]
        if "wd" in p:
            pairs.append((f"b{i}.ds", prev, p["wd"], p["bnd"], p["stride"], 0, None))
            ident = trace[f"b{i}.ds"]
        else:
            ident = prev
        pairs.append((f"b{i}.conv2", trace[f"b{i}.sn1"], p["w2"], p["bn2"], 1, 1, ident))
        for name, inp, w, bnp, stride, pad, res in pairs:
            layer = convs[name]
            xi = xin if inp is prev else torch.from_numpy(to_nhwc(inp)).to("cuda:0", torch.float16)
            rd = None if res is None else torch.from_numpy(to_nhwc(res)).to("cuda:0", torch.float16)
            y = layer(xi, residual=rd)
            got = from_nhwc(y.float().cpu().numpy(), T, B)
            if res is not None:
                got = got - res
            ref = L.fused_layer_torch(inp, w, _bn(bnp), stride=stride, pad=pad, threads=threads)
            st = {}
            frac, ok, _, _ = L.spike_agreement(got, ref["spikes"], ref["h"], stats=st)
            print(f"{name} ({rt.variant(layer.desc)}): agreement {frac:.6f} rate "
                  f"{ref['spikes'].mean():.3f} {st}")
            assert frac >= 0.995 and ok, (name, frac)
            worst = min(worst, (frac, name))
        prev = trace[f"b{i}.out"]
    torch.cuda.synchronize()
    assert rt.device_error() == 0
    print(f"worst layer {worst}")


def test_dvs_end_to_end_logits(setup):
    P, x, x_tb, logits_ref, trace, model, torch, _ = setup
    out = model(torch.from_numpy(x_tb)).cpu().numpy()
    a, b = out.ravel(), logits_ref.ravel()
    cos_all = float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))
    print(f"dvs logits cosine {cos_all:.6f}; top-1 {out.argmax(1)} vs {logits_ref.argmax(1)}")
    assert cos_all > 0.99
    assert (out.argmax(1) == logits_ref.argmax(1)).mean() >= 0.75


def test_dvs_golden_reference_logits(cuda_device):
    """Batch 1 against the reference model class's own logits."""
    import torch
    from conftest import GOLDEN
    from sparsesnn_b200.sew_resnet import SEWResNet18DVS
    m = np.load(GOLDEN / "sew18_dvs_logits.npz")
    shape = tuple(int(v) for v in m["x_shape"])
    x = np.unpackbits(m["x_bits"])[: int(np.prod(shape))].reshape(shape).astype(np.float32)
    model = SEWResNet18DVS(_params(), T=shape[1], batch=shape[0], device="cuda:0")
    out = model(torch.from_numpy(np.ascontiguousarray(np.transpose(x, (1, 0, 2, 3, 4))))).cpu().numpy()
    ref = m["logits"]
    cos = float((out * ref).sum() / (np.linalg.norm(out) * np.linalg.norm(ref)))
    print(f"dvs golden cosine {cos:.6f}")
    assert cos > 0.99 and out.argmax() == ref.argmax()


def test_dvs_graph_replay_matches_eager(setup):
    P, x, x_tb, logits_ref, trace, model, torch, _ = setup
    xt = torch.from_numpy(x_tb)
    eager = model(xt).clone()
    model.capture(warmup=1)
    try:
        graphed = model(xt).clone()
    finally:
        model._graph = None
    assert torch.equal(eager, graphed)
