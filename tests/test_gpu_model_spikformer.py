"""Spikformer-8-384 (config 3: 224x224, T=4, 14x14 tokens, 12 heads) on the
B200 kernels against the CPU port of the reference forward (pinned to the
reference's own modules by ``spikformer_logits.npz``).

Teacher forcing, every node fed the oracle's input:
* the stem and the three dense patch-splitting convs (+ BN + LIF) and the
  RPE conv with its ``x + x_feat``: the layer parity rule;
* the four spike max pools and the attention cores: bit for bit;
* every Linear + BN1d + LIF (q, k, v, proj with ``x + ...``, fc1, fc2 with
  ``x1 + ...``) of the eight blocks: the layer parity rule.
End to end: logits by the reference validator's rule (batch 2) and the
golden reference logits (batch 1).
"""
import os

import numpy as np
import pytest

from oracle import lif_layer as L

pytestmark = pytest.mark.gpu

T, B = 4, 2


def to_nhwc(x):
    t, b, c, h, w = x.shape
    return np.ascontiguousarray(np.transpose(x, (0, 1, 3, 4, 2)).reshape(t * b, h, w, c))


def from_nhwc(y, T_, B_):
    tb, h, w, c = y.shape
    return np.transpose(y.reshape(T_, B_, h, w, c), (0, 1, 4, 2, 3))


def pack_bits(y_nhwc):
    """fp16 0/1 spikes [.., C] -> bit-packed bytes [.., C/8] (channel c in bit c%8 of byte c/8)."""
    return np.packbits(y_nhwc.astype(np.uint8), axis=-1, bitorder="little")


def unpack_bits(b_nhwc):
    return np.unpackbits(b_nhwc, axis=-1, bitorder="little").astype(np.float32)


def _bn(p):
    return L.BNParams(p["gamma"], p["beta"], p["mean"], p["var"])


def judge(got, ref_spk, h, tag, v_th=1.0):
    st = {}
    frac, ok, _, _ = L.spike_agreement(got, ref_spk, h, v_th=v_th, stats=st)
    print(f"{tag}: agreement {frac:.6f} rate {ref_spk.mean():.3f} {st}")
    assert frac >= 0.995 and ok, (tag, frac)


def linear_h(x_tbnc, p, threads):
    """Pre-reset membranes of LIF(BN1d(Linear(x))) over (T, B, N, C)."""
    import torch
    import torch.nn.functional as F
    torch.set_num_threads(threads)
    with torch.no_grad():
        z = F.linear(torch.from_numpy(np.ascontiguousarray(x_tbnc)), torch.from_numpy(p["w"]),
                     torch.from_numpy(p["b"]))
        bn = p["bn"]
        z = F.batch_norm(z.flatten(0, 2), torch.from_numpy(bn["mean"]), torch.from_numpy(bn["var"]),
                         torch.from_numpy(bn["gamma"]), torch.from_numpy(bn["beta"]), training=False,
                         eps=1e-5).view(z.shape)
    return L.multistep_lif(z.numpy())


@pytest.fixture(scope="module")
def setup(cuda_device):
    import torch
    from oracle.spikformer import forward_torch, make_input
    from sparsesnn_b200.spikformer import Spikformer, init_params
    threads = os.cpu_count() or 1
    P = init_params(seed=0)
    x = make_input(seed=9, B=B)
    logits_ref, trace = forward_torch(P, x, T=T, return_trace=True, threads=threads)
    model = Spikformer(P, T=T, batch=B, device="cuda:0")
    return P, x, logits_ref, trace, model, torch, threads


def test_spikformer_patch_splitting(setup):
    from sparsesnn_b200 import runtime as rt
    P, x, logits_ref, trace, model, torch, threads = setup
    nodes = {n.name: n for n in model.nodes}
    lib = rt.load()
    s = torch.cuda.current_stream().cuda_stream
    model(torch.from_numpy(x))
    torch.cuda.synchronize()
    # stem
    sps0 = model.buffer("sps0")
    if nodes["sps0"].desc.flags & rt.SNN_FLAG_SPIKE_BITS:   # bit-packed stem spikes
        got = from_nhwc(unpack_bits(sps0.cpu().numpy()), T, B)
    else:
        got = from_nhwc(sps0.float().cpu().numpy(), T, B)
    z = L.batchnorm_eval(L.conv2d_nchw(x, P["sps"][0]["w"], 1, 1), _bn(P["sps"][0]["bn"]))
    _, h, _ = L.multistep_lif(np.repeat(z[None], T, 0))
    judge(got, trace["sps0"], h, "sps0")
    dev = lambda a: torch.from_numpy(to_nhwc(a)).to("cuda:0", torch.float16)  # noqa: E731
    for i in range(4):
        if i > 0:
            layer = nodes[f"sps{i}"].layer
            got = from_nhwc(layer(dev(trace[f"pool{i - 1}"])).float().cpu().numpy(), T, B)
            ref = L.fused_layer_torch(trace[f"pool{i - 1}"], P["sps"][i]["w"], _bn(P["sps"][i]["bn"]),
                                      pad=1, threads=threads)
            judge(got, ref["spikes"], ref["h"], f"sps{i} (dense)")
        # pool of the oracle's spikes, exact
        n = nodes[f"pool{i}"]
        src = dev(trace[f"sps{i}"])
        if n.desc.flags & rt.SNN_FLAG_SPIKE_BITS:            # the pool reads packed spikes
            src = torch.from_numpy(pack_bits(to_nhwc(trace[f"sps{i}"]))).to("cuda:0")
        out = torch.empty_like(dev(trace[f"pool{i}"]))
        rt.check(lib.snn_maxpool_lif_forward(n.desc, src.data_ptr(), None, out.data_ptr(), s))
        torch.cuda.synchronize()
        assert np.array_equal(from_nhwc(out.float().cpu().numpy(), T, B), trace[f"pool{i}"]), i
    # RPE conv + LIF + x_feat
    rpe = nodes["rpe"].layer
    xf = trace["pool3"]
    got = from_nhwc(rpe(dev(xf), residual=dev(xf)).float().cpu().numpy(), T, B) - xf
    ref = L.fused_layer_torch(xf, P["rpe"]["w"], _bn(P["rpe"]["bn"]), pad=1, threads=threads)
    judge(got, ref["spikes"], ref["h"], "rpe (dense, + x_feat)")
    assert rt.device_error() == 0


def test_spikformer_teacher_forced_blocks(setup):
    from sparsesnn_b200 import runtime as rt
    P, x, logits_ref, trace, model, torch, threads = setup
    nodes = {n.name: n for n in model.nodes}
    N, E = model.tokens, P["embed"]
    rows = B * N
    tok = lambda a: torch.from_numpy(np.ascontiguousarray(a.reshape(T, 1, rows, -1))).to(  # noqa: E731
        "cuda:0", torch.float16)
    back = lambda y: y.float().cpu().numpy().reshape(T, B, N, -1)  # noqa: E731
    lib = rt.load()
    s = torch.cuda.current_stream().cuda_stream
    xs = trace["x0"]
    for i, p in enumerate(P["blocks"]):
        # q, k, v: one fused layer whose output rows are q | k | v
        got = back(nodes[f"b{i}.qkv"].layer(tok(xs)))
        for j, nm in enumerate(("q", "k", "v")):
            spk, h, _ = linear_h(xs, p[nm], threads)
            judge(got[..., j * E:(j + 1) * E], spk, h, f"b{i}.{nm}")
        # attention core + attention LIF on the oracle's q, k, v packed the
        # same way: exact
        n = nodes[f"b{i}.attn"]
        qkv = tok(np.concatenate([trace[f"b{i}.{nm}"] for nm in ("q", "k", "v")], -1))
        out = torch.empty((T, 1, rows, E), dtype=torch.float16, device="cuda:0")
        a = n.attn
        assert a["packed"]
        cb = E * 2
        rt.check(lib.snn_spikformer_attn_forward(T, B, N, a["heads"], a["head_dim"], a["scale"],
                                                 n.desc.tau, n.desc.v_threshold, 0.0,
                                                 rt.SNN_FLAG_QKV_PACKED, qkv.data_ptr(),
                                                 qkv.data_ptr() + cb, qkv.data_ptr() + 2 * cb,
                                                 None, out.data_ptr(), s))
        torch.cuda.synchronize()
        assert np.array_equal(back(out), trace[f"b{i}.attn"]), f"b{i}.attn"
        # proj + x, fc1, fc2 + x1
        got = back(nodes[f"b{i}.proj"].layer(tok(trace[f"b{i}.attn"]), residual=tok(xs))) - xs
        spk, h, _ = linear_h(trace[f"b{i}.attn"], p["proj"], threads)
        judge(got, spk, h, f"b{i}.proj")
        x1 = trace[f"b{i}.x1"]
        got = back(nodes[f"b{i}.fc1"].layer(tok(x1)))
        spk, h, _ = linear_h(x1, p["fc1"], threads)
        judge(got, spk, h, f"b{i}.fc1")
        hm = trace[f"b{i}.h"]
        got = back(nodes[f"b{i}.fc2"].layer(tok(hm), residual=tok(x1))) - x1
        spk, h, _ = linear_h(hm, p["fc2"], threads)
        judge(got, spk, h, f"b{i}.fc2")
        xs = trace[f"b{i}.x2"]
    assert rt.device_error() == 0


def test_spikformer_end_to_end_logits(setup):
    P, x, logits_ref, trace, model, torch, _ = setup
    out = model(torch.from_numpy(x)).cpu().numpy()
    a, b = out.ravel(), logits_ref.ravel()
    cos_all = float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))
    cos = (out * logits_ref).sum(1) / (np.linalg.norm(out, axis=1) * np.linalg.norm(logits_ref, axis=1))
    print(f"spikformer logits cosine {cos_all:.6f} (per image {np.round(cos, 5)}); top-1 "
          f"{out.argmax(1)} vs {logits_ref.argmax(1)}")
    assert cos_all > 0.99 and cos.min() > 0.95


def test_spikformer_golden_reference_logits(cuda_device):
    import torch
    from conftest import GOLDEN
    from oracle.spikformer import make_input
    from sparsesnn_b200.spikformer import Spikformer, init_params
    m = np.load(GOLDEN / "spikformer_logits.npz")
    x = make_input(seed=int(m["seed"]), B=int(m["batch"]))
    model = Spikformer(init_params(seed=0), T=4, batch=x.shape[0], device="cuda:0")
    out = model(torch.from_numpy(x)).cpu().numpy()
    ref = m["logits"]
    cos = float((out * ref).sum() / (np.linalg.norm(out) * np.linalg.norm(ref)))
    print(f"spikformer golden cosine {cos:.6f}")
    assert cos > 0.99


def test_spikformer_graph_replay_matches_eager(setup):
    P, x, logits_ref, trace, model, torch, _ = setup
    xt = torch.from_numpy(x)
    eager = model(xt).clone()
    model.capture(warmup=1)
    try:
        graphed = model(xt).clone()
    finally:
        model._graph = None
    assert torch.equal(eager, graphed)
