"""MS-ResNet-34 (config 2: 224x224, T=4, LIF neurons, real-valued membrane
shortcut) on the B200 kernels against the CPU port of the reference forward
(pinned to the reference model class by ``msresnet34_logits.npz``).

Batch 4 gives every persistent conv kernel more pixel tiles than CTAs at the
first stage.  Per block, with the oracle's tensors as inputs (teacher
forcing):
* ``sn1``: the LIF of the fp16 stream, bit for bit;
* ``conv1`` (+ BN + LIF): the layer parity rule;
* the shortcut conv (+ BN, no neuron, fp16 out) and ``conv2`` (+ BN + the
  shortcut, fp16 out): within fp16 rounding of the oracle run on the same
  fp16 inputs and weights.
End to end: logits by the reference validator's rule, and the golden
reference logits at batch 1.
"""
import os

import numpy as np
import pytest

from oracle import lif_layer as L

pytestmark = pytest.mark.gpu

T, B = 4, 4


def to_nhwc(x):
    t, b, c, h, w = x.shape
    return np.ascontiguousarray(np.transpose(x, (0, 1, 3, 4, 2)).reshape(t * b, h, w, c))


def from_nhwc(y, T_, B_):
    tb, h, w, c = y.shape
    return np.transpose(y.reshape(T_, B_, h, w, c), (0, 1, 4, 2, 3))


def f16(a):
    return a.astype(np.float16).astype(np.float32)


def _bn(p):
    return L.BNParams(p["gamma"], p["beta"], p["mean"], p["var"])


def bn_conv_torch(x, w, bnp, stride, pad, threads):
    """BN(conv(x)) over [T,B,C,H,W] in torch CPU fp32 (the reference's
    TDBNContainer in eval)."""
    import torch
    import torch.nn.functional as F
    torch.set_num_threads(threads)
    t, b = x.shape[:2]
    with torch.no_grad():
        y = F.conv2d(torch.from_numpy(np.ascontiguousarray(x)).flatten(0, 1),
                     torch.from_numpy(np.ascontiguousarray(w)), stride=stride, padding=pad)
        s, bb = _bn(bnp).scale_bias()
        y = y * torch.from_numpy(s)[None, :, None, None] + torch.from_numpy(bb)[None, :, None, None]
    return y.numpy().reshape((t, b) + y.shape[1:])


@pytest.fixture(scope="module")
def setup(cuda_device):
    import torch
    from oracle.ms_resnet import forward_torch, make_input
    from sparsesnn_b200.ms_resnet import MSResNet34, init_params
    threads = os.cpu_count() or 1
    P = init_params(seed=0)
    x = make_input(seed=5, B=B)
    logits_ref, trace = forward_torch(P, x, T=T, return_trace=True, threads=threads)
    model = MSResNet34(P, T=T, batch=B, device="cuda:0")
    return P, x, logits_ref, trace, model, torch, threads


def test_msresnet_stem(setup):
    P, x, logits_ref, trace, model, torch, _ = setup
    model(torch.from_numpy(x))
    torch.cuda.synchronize()
    got = from_nhwc(model.buffer("stem").float().cpu().numpy(), T, B)
    ref = trace["stem"]
    assert (np.abs(got - ref) <= 2.0 ** -10 * np.abs(ref) + 1e-4).all()
    # The same pass writes block 0's sn1: the LIF of the stem's own fp16
    # output over T, bit for bit.
    stem = next(n for n in model.nodes if n.name == "stem")
    s1 = from_nhwc(stem.out2.float().cpu().numpy(), T, B)
    spk, _, _ = L.multistep_lif(got)
    assert np.array_equal(s1, spk)
    assert 0.01 < s1.mean() < 0.9


def test_msresnet_teacher_forced_blocks(setup):
    from sparsesnn_b200 import runtime as rt
    P, x, logits_ref, trace, model, torch, threads = setup
    nodes = {n.name: n for n in model.nodes}
    dev = lambda a: torch.from_numpy(to_nhwc(a)).to("cuda:0", torch.float16)  # noqa: E731
    lib = rt.load()
    stream = torch.cuda.current_stream().cuda_stream
    prev = trace["stem"]
    worst_rel = 0.0
    for i, p in enumerate(P["blocks"]):
        xin = f16(prev)                               # the stream as the kernels store it
        # sn1: LIF of the fp16 stream, exact (block 0's comes from the stem's
        # dual pass, checked in test_msresnet_stem)
        if i > 0:
            n = nodes[f"b{i}.sn1"]
            s1 = torch.empty_like(dev(xin))
            rt.check(lib.snn_lif_forward(n.desc, dev(xin).data_ptr(), None, s1.data_ptr(), stream))
            spk, _, _ = L.multistep_lif(xin)
            assert np.array_equal(from_nhwc(s1.float().cpu().numpy(), T, B), spk), f"b{i}.sn1"
        # conv1 + BN + LIF on the oracle's sn1 spikes
        l1 = nodes[f"b{i}.conv1"].layer
        got = from_nhwc(l1(dev(trace[f"b{i}.s1"])).float().cpu().numpy(), T, B)
        r1 = L.fused_layer_torch(trace[f"b{i}.s1"], p["w1"], _bn(p["bn1"]), stride=p["stride"],
                                 pad=1, threads=threads)
        st = {}
        frac, ok, _, _ = L.spike_agreement(got, r1["spikes"], r1["h"], stats=st)
        print(f"b{i}.conv1 ({rt.variant(l1.desc)}): agreement {frac:.6f} {st}")
        assert frac >= 0.995 and ok, (i, frac)
        # shortcut conv (real input) and conv2 + shortcut, fp16 outputs
        if "wsc" in p:
            lsc = nodes[f"b{i}.sc"].layer
            got = from_nhwc(lsc(dev(xin)).float().cpu().numpy(), T, B)
            ref = bn_conv_torch(xin, f16(p["wsc"]), p["bnsc"], p["stride"], 0, threads)
            err = np.abs(got - ref)
            assert (err <= 2.0 ** -10 * np.abs(ref) + 2e-3).all(), (i, "sc", err.max())
            sc = f16(trace[f"b{i}.sc"])
        else:
            sc = xin
        l2 = nodes[f"b{i}.conv2"].layer
        got = from_nhwc(l2(dev(trace[f"b{i}.o1"]), residual=dev(sc)).float().cpu().numpy(), T, B)
        ref = bn_conv_torch(trace[f"b{i}.o1"], f16(p["w2"]), p["bn2"], 1, 1, threads) + sc
        err = np.abs(got - ref)
        worst_rel = max(worst_rel, float((err / (np.abs(ref) + 1e-3)).max()))
        assert (err <= 2.0 ** -10 * np.abs(ref) + 2e-3).all(), (i, "conv2", err.max())
        prev = trace[f"b{i}.out"]
    torch.cuda.synchronize()
    assert rt.device_error() == 0
    print(f"worst relative error of a block output {worst_rel:.2e}")


def test_msresnet_end_to_end_logits(setup):
    P, x, logits_ref, trace, model, torch, _ = setup
    out = model(torch.from_numpy(x)).cpu().numpy()
    a, b = out.ravel(), logits_ref.ravel()
    cos_all = float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))
    cos = (out * logits_ref).sum(1) / (np.linalg.norm(out, axis=1) * np.linalg.norm(logits_ref, axis=1))
    print(f"msresnet logits cosine {cos_all:.6f} (per image {np.round(cos, 5)}); top-1 "
          f"{out.argmax(1)} vs {logits_ref.argmax(1)}")
    assert cos_all > 0.99 and cos.min() > 0.95


def test_msresnet_golden_reference_logits(cuda_device):
    import torch
    from conftest import GOLDEN
    from oracle.ms_resnet import make_input
    from sparsesnn_b200.ms_resnet import MSResNet34, init_params
    m = np.load(GOLDEN / "msresnet34_logits.npz")
    x = make_input(seed=int(m["seed"]), B=int(m["batch"]))
    model = MSResNet34(init_params(seed=0), T=4, batch=x.shape[0], device="cuda:0")
    out = model(torch.from_numpy(x)).cpu().numpy()
    ref = m["logits"]
    cos = float((out * ref).sum() / (np.linalg.norm(out) * np.linalg.norm(ref)))
    print(f"msresnet golden cosine {cos:.6f}")
    assert cos > 0.99


def test_msresnet_graph_replay_matches_eager(setup):
    P, x, logits_ref, trace, model, torch, _ = setup
    xt = torch.from_numpy(x)
    eager = model(xt).clone()
    model.capture(warmup=1)
    try:
        graphed = model(xt).clone()
    finally:
        model._graph = None
    assert torch.equal(eager, graphed)
