"""SEW-ResNet-18 on the B200 layers vs the reference forward.

* Per-layer teacher forcing: each fused layer gets the ORACLE's input
  spikes and its output is judged by the layer parity rule (spikes >= 99.5%
  equal, first mismatch of every neuron within |h - v_th| < 1e-2).
* End to end: logits vs the reference model's (golden fixture), cosine >= 0.99
  and identical top-1, the acceptance rule of the reference's own validator
  (sengine/scripts/verify_correctness.py:99-151).  Spike flips compound with
  depth, so this is the looser check.
"""
import numpy as np
import pytest

from conftest import GOLDEN
from oracle import lif_layer as L

pytestmark = pytest.mark.gpu


def to_nhwc(x):
    t, b, c, h, w = x.shape
    return np.ascontiguousarray(np.transpose(x, (0, 1, 3, 4, 2)).reshape(t * b, h, w, c))


def from_nhwc(y, T, B):
    tb, h, w, c = y.shape
    return np.transpose(y.reshape(T, B, h, w, c), (0, 1, 4, 2, 3))


@pytest.fixture(scope="module")
def setup(cuda_device):
    import torch
    from oracle.sew_resnet import forward_torch, make_params
    from sparsesnn_b200.sew_resnet import SEWResNet18
    m = np.load(GOLDEN / "sew18_logits.npz")
    P = make_params(0)
    logits_ref, trace = forward_torch(P, m["x"], T=4, return_trace=True)
    model = SEWResNet18(P, T=4, batch=2, device="cuda:0")
    return P, m, logits_ref, trace, model, torch


def _bn(p):
    return L.BNParams(p["gamma"], p["beta"], p["mean"], p["var"])


def test_end_to_end_logits(setup):
    P, m, logits_ref, trace, model, torch = setup
    out = model(torch.from_numpy(m["x"])).cpu().numpy()
    ref = m["logits"]
    cos = (out * ref).sum(1) / (np.linalg.norm(out, axis=1) * np.linalg.norm(ref, axis=1))
    assert (cos >= 0.99).all(), cos
    assert (out.argmax(1) == ref.argmax(1)).all()


def test_stem_exact_spikes(setup):
    P, m, logits_ref, trace, model, torch = setup
    model(torch.from_numpy(m["x"]))
    torch.cuda.synchronize()
    got = from_nhwc(model.a0.float().cpu().numpy(), 4, 2)
    ref = trace["stem"]
    z = L.batchnorm_eval(L.conv2d_nchw(m["x"], P["stem"]["w"], 1, 1), _bn(P["stem"]["bn"]))
    _, h, _ = L.multistep_lif(np.repeat(z[None], 4, 0))
    frac, ok, nmis, _ = L.spike_agreement(got, ref, h)
    assert frac >= 0.995 and ok


def test_teacher_forced_layers(setup):
    P, m, logits_ref, trace, model, torch = setup
    prev = trace["stem"]
    worst = 1.0
    for i, (blk, p) in enumerate(zip(model.blocks, P["blocks"])):
        xin = torch.from_numpy(to_nhwc(prev)).to("cuda:0", torch.float16)
        o1 = blk["l1"](xin)
        r = L.fused_layer(prev, p["w1"], _bn(p["bn1"]), stride=p["stride"], pad=1)
        got = from_nhwc(o1.float().cpu().numpy(), 4, 2)
        frac, ok, _, _ = L.spike_agreement(got, r["spikes"], r["h"])
        assert frac >= 0.995 and ok, (i, "conv1", frac)
        worst = min(worst, frac)
        if "wd" in p:
            ident_ref = trace[f"b{i}.ds"]
            d = blk["ds"](xin)
            rd = L.fused_layer(prev, p["wd"], _bn(p["bnd"]), stride=p["stride"], pad=0)
            got = from_nhwc(d.float().cpu().numpy(), 4, 2)
            frac, ok, _, _ = L.spike_agreement(got, rd["spikes"], rd["h"])
            assert frac >= 0.995 and ok, (i, "ds", frac)
        else:
            ident_ref = prev
        sn1 = trace[f"b{i}.sn1"]
        o2 = blk["l2"](torch.from_numpy(to_nhwc(sn1)).to("cuda:0", torch.float16),
                       residual=torch.from_numpy(to_nhwc(ident_ref)).to("cuda:0", torch.float16))
        r2 = L.fused_layer(sn1, p["w2"], _bn(p["bn2"]), stride=1, pad=1)
        got = from_nhwc(o2.float().cpu().numpy(), 4, 2) - ident_ref
        frac, ok, _, _ = L.spike_agreement(got, r2["spikes"], r2["h"])
        assert frac >= 0.995 and ok, (i, "conv2", frac)
        prev = trace[f"b{i}.out"]
    print(f"worst teacher-forced layer agreement {worst:.6f}")


def test_graph_replay_matches_eager(setup):
    P, m, logits_ref, trace, model, torch = setup
    x = torch.from_numpy(m["x"])
    eager = model(x).clone()
    model.capture(warmup=1)
    try:
        graphed = model(x).clone()
    finally:
        model._graph = None
    assert torch.equal(eager, graphed)
