"""The oracle is pinned to fixtures made by the real reference PyTorch path.

Fixtures: ``tests/golden/make_golden.py`` (imports the reference's
``sparse/pruning.py``, ``models/neurons.py``, ``models/layers.py`` and
``models/sewresnet.py``).
"""
import numpy as np
import pytest

from conftest import ATTN_CASES, GOLDEN, LAYER_CASES, RES_CASES, load_attn_case, load_layer_case
from oracle import lif_layer as L
from oracle import pack24 as P


def test_prune_matches_reference():
    d = np.load(GOLDEN / "prune.npz")
    assert np.array_equal(P.prune_conv_weight(d["w"]), d["pruned"])
    assert np.array_equal(P.prune_2_4(d["w2"]), d["pruned2"])   # padded last dim


@pytest.mark.parametrize("name", LAYER_CASES)
def test_layer_matches_reference(name):
    g = load_layer_case(name)
    x = g["x"].astype(np.float32)
    if g["linear"]:
        # Linear bias enters like a shifted BN mean: bn(Wx + b) == bn'(Wx).
        bn = L.BNParams(g["gamma"], g["beta"], g["mean"] - g["lin_bias"], g["var"])
    else:
        bn = L.BNParams(g["gamma"], g["beta"], g["mean"], g["var"])
    res = g.get("residual")
    r = L.fused_layer(x, g["w"], bn, stride=g["stride"], pad=g["pad"], neuron=g["neuron"],
                      residual=None if res is None else res.astype(np.float32))
    # float64-accumulated conv vs the reference's float32 conv: a few ulps.
    np.testing.assert_allclose(r["bn_out"], g["bn_out"], rtol=0, atol=1e-5)
    np.testing.assert_allclose(r["h"], g["h"], rtol=0, atol=1e-5)
    np.testing.assert_allclose(r["v"], g["v"], rtol=0, atol=1e-5)
    frac, explained, _, _ = L.spike_agreement(r["spikes"], g["spikes"].astype(np.float32), g["h"])
    assert frac == 1.0 and explained
    if res is not None:
        assert np.array_equal(r["out"], g["out"].astype(np.float32))


@pytest.mark.parametrize("name", RES_CASES)
def test_residual_modes_match_reference(name):
    """Add-before-neuron and two-neuron epilogues against the reference
    modules (Conv -> BN -> Add -> LIF; Conv -> BN -> IF -> Add -> LIF)."""
    g = load_layer_case(name)
    bn = L.BNParams(g["gamma"], g["beta"], g["mean"], g["var"])
    r = L.fused_layer(g["x"].astype(np.float32), g["w"], bn, stride=g["stride"], pad=g["pad"],
                      neuron=g["neuron"], residual=g["residual"], res_mode=g["res_mode"],
                      neuron2=g["neuron2"])
    np.testing.assert_allclose(r["bn_out"], g["bn_out"], rtol=0, atol=1e-5)
    np.testing.assert_allclose(r["h"], g["h"], rtol=0, atol=1e-5)
    np.testing.assert_allclose(r["v"], g["v"], rtol=0, atol=1e-5)
    assert np.array_equal(r["spikes"], g["spikes"].astype(np.float32))
    if g["res_mode"] == "two_neuron":
        np.testing.assert_allclose(r["h2"], g["h2"], rtol=0, atol=1e-5)
        np.testing.assert_allclose(r["v2"], g["v2"], rtol=0, atol=1e-5)
    assert np.array_equal(r["out"], g["out"].astype(np.float32))


@pytest.mark.parametrize("name", ATTN_CASES)
def test_attention_matches_reference(name):
    """Spikformer attention core + attention LIF: exact (integer counts)."""
    from oracle.attention import spikformer_attn_lif
    g = load_attn_case(name)
    spk, x, _, _ = spikformer_attn_lif(g["q"], g["k"], g["v"], T=g["T"], heads=g["heads"])
    assert np.array_equal(x, g["x"])
    assert np.array_equal(spk, g["spikes"].astype(np.float32))


def test_glue_matches_reference():
    """MaxPool2d -> LIF and Add -> LIF / IF against the reference modules."""
    from oracle.glue import add_lif, maxpool2d, maxpool_lif
    g = np.load(GOLDEN / "glue.npz")
    x = g["x"]
    t, b = x.shape[:2]
    pooled = maxpool2d(x.reshape((t * b,) + x.shape[2:]), 3, 2, 1)
    assert np.array_equal(pooled.reshape(g["pooled"].shape), g["pooled"])
    assert np.array_equal(maxpool_lif(x, 3, 2, 1)[0], g["s_pool"].astype(np.float32))
    assert np.array_equal(add_lif(g["a"], g["b"])[0], g["s_add"].astype(np.float32))
    assert np.array_equal(add_lif(g["a"], g["b"], neuron="if")[0], g["s_add_if"].astype(np.float32))


def test_sew18_forward_matches_reference_model():
    from oracle.sew_resnet import forward_torch, make_params
    m = np.load(GOLDEN / "sew18_logits.npz")
    logits, trace = forward_torch(make_params(0), m["x"], T=4, return_trace=True)
    np.testing.assert_allclose(logits, m["logits"], rtol=0, atol=1e-5)
    # every stage fires (random weights scaled to keep the network active)
    for name in ("stem", "b1.sn1", "b3.sn1", "b5.sn1", "b7.sn1"):
        assert trace[name].mean() > 0.01, name


def test_bench_weights_equal_oracle_weights():
    """The product's init_params and the oracle's make_params draw the same
    weights (the GPU model and the oracle forward see one network)."""
    from oracle.sew_resnet import make_params
    from sparsesnn_b200.sew_resnet import init_params
    for kw in ({}, dict(num_classes=11, in_channels=2, stem_kernel=7, input_moment=0.05)):
        a, b = init_params(seed=0, **kw), make_params(0, **kw)
        assert np.array_equal(a["stem"]["w"], b["stem"]["w"])
        for x, y in zip(a["blocks"], b["blocks"]):
            for k in ("w1", "w2", "wd"):
                if k in x:
                    assert np.array_equal(x[k], y[k])
        assert np.array_equal(a["fc_w"], b["fc_w"])


def test_bn_fold_matches_batchnorm():
    rng = np.random.default_rng(0)
    f = 32
    bn = L.BNParams(rng.uniform(0.5, 1.5, f).astype(np.float32),
                    (rng.standard_normal(f) * 0.1).astype(np.float32),
                    (rng.standard_normal(f) * 0.1).astype(np.float32),
                    rng.uniform(0.5, 1.5, f).astype(np.float32))
    y = rng.standard_normal((3, f, 5, 5)).astype(np.float32)
    s, b = bn.scale_bias()
    np.testing.assert_allclose(y * s[None, :, None, None] + b[None, :, None, None],
                               L.batchnorm_eval(y, bn), rtol=1e-6, atol=1e-6)


def test_spike_agreement_rule_flags_far_mismatch():
    # A planted mismatch far from threshold must be rejected; one near the
    # threshold is accepted, and later steps of a diverged neuron are ignored.
    h = np.array([[0.2, 0.995], [0.3, 0.4]], np.float32)      # [T=2, N=2]
    ref = (h >= 1.0).astype(np.float32)
    near = ref.copy(); near[0, 1] = 1.0; near[1, 1] = 1.0
    frac, ok, n, div = L.spike_agreement(near, ref, h)
    assert ok and n == 2 and div.tolist() == [False, True]
    far = ref.copy(); far[0, 0] = 1.0
    assert not L.spike_agreement(far, ref, h)[1]


def test_spike_agreement_reports_excused_mismatches():
    # The later mismatch of a diverged neuron is not judged, but it is
    # counted, and counted as off-band when its reference membrane is far
    # from the threshold.
    h = np.array([[0.2, 0.995], [0.3, 0.4]], np.float32)
    ref = (h >= 1.0).astype(np.float32)
    got = ref.copy(); got[0, 1] = 1.0; got[1, 1] = 1.0
    st = {}
    L.spike_agreement(got, ref, h, stats=st)
    assert st == {"first": 1, "later": 1, "later_off_band": 1, "neurons": 2, "diverged": 1}


def load_dvs_golden():
    m = np.load(GOLDEN / "sew18_dvs_logits.npz")
    shape = tuple(int(v) for v in m["x_shape"])
    x = np.unpackbits(m["x_bits"])[: int(np.prod(shape))].reshape(shape).astype(np.float32)
    return x, m["logits"]


def test_oracle_dvs_sew18_matches_reference_logits():
    """DVS SEW-ResNet-18 (7x7/2 stem per timestep, MaxPool(3,2,1), T=16) port
    against the reference model class's logits; the spikes reach the last
    stage (the network is not silent)."""
    from oracle.sew_resnet import forward_torch, make_params
    x, ref = load_dvs_golden()
    P = make_params(0, num_classes=11, in_channels=2, stem_kernel=7, input_moment=0.05)
    logits, trace = forward_torch(P, x, T=16, stem_stride=2, maxpool=True, return_trace=True)
    np.testing.assert_allclose(logits, ref, rtol=0, atol=1e-5)
    assert trace["b7.sn1"].mean() > 0.01
    print("spike rates:", {k: round(float(v.mean()), 3) for k, v in trace.items()})


def test_oracle_msresnet34_matches_reference_logits():
    """MS-ResNet-34 port (LIF neurons, real-valued membrane shortcut) against
    the reference model class with its neurons set to the same LIF; the
    spikes keep firing through the last stage."""
    from oracle.ms_resnet import forward_torch, make_input, make_params
    m = np.load(GOLDEN / "msresnet34_logits.npz")
    x = make_input(seed=int(m["seed"]), B=int(m["batch"]))
    logits, trace = forward_torch(make_params(0), x, T=4, return_trace=True)
    np.testing.assert_allclose(logits, m["logits"], rtol=0, atol=1e-5)
    assert trace["b15.o1"].mean() > 0.05 and trace["sn_out"].mean() > 0.05


def test_msresnet_weights_equal_oracle_weights():
    from oracle.ms_resnet import make_params
    from sparsesnn_b200.ms_resnet import init_params
    a, b = init_params(seed=0), make_params(0)
    assert np.array_equal(a["stem"]["w"], b["stem"]["w"])
    for x, y in zip(a["blocks"], b["blocks"]):
        for k in ("w1", "w2", "wsc"):
            assert (k in x) == (k in y)
            if k in x:
                assert np.array_equal(x[k], y[k])
    assert np.array_equal(a["fc_w"], b["fc_w"])


def test_oracle_spikformer_matches_reference_modules():
    """Spikformer-8-384 port (14x14 tokens, 12 heads) against the reference's
    own SPS sub-modules and Block modules; every block keeps firing."""
    from oracle.spikformer import forward_torch, make_input, make_params
    m = np.load(GOLDEN / "spikformer_logits.npz")
    x = make_input(seed=int(m["seed"]), B=int(m["batch"]))
    logits, trace = forward_torch(make_params(0), x, T=4, return_trace=True)
    np.testing.assert_allclose(logits, m["logits"], rtol=0, atol=2e-5)
    for b in range(8):
        assert 0.02 < trace[f"b{b}.attn"].mean() < 0.9 and trace[f"b{b}.h"].mean() > 0.02


def test_spikformer_weights_equal_oracle_weights():
    from oracle.spikformer import make_params
    from sparsesnn_b200.spikformer import init_params
    a, b = init_params(seed=0), make_params(0)
    for x, y in zip(a["sps"] + [a["rpe"]], b["sps"] + [b["rpe"]]):
        assert np.array_equal(x["w"], y["w"])
    for x, y in zip(a["blocks"], b["blocks"]):
        for k in ("q", "k", "v", "proj", "fc1", "fc2"):
            assert np.array_equal(x[k]["w"], y[k]["w"]) and np.array_equal(x[k]["b"], y[k]["b"])
    assert np.array_equal(a["fc_w"], b["fc_w"])
