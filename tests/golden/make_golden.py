"""Generate golden fixtures by running the REAL reference PyTorch path.

Run in a container that has the reference checkout (it is not needed at
test time and never on the GPU box):

    python tests/golden/make_golden.py --ref /path/to/SparseSNN

It imports the reference's own modules -- ``sparse/pruning.py``
(``prune_2_4``), ``models/neurons.py`` (``MultiStepLIFNeuron`` /
``MultiStepIFNeuron``), ``models/layers.py`` (``SeqToANNContainer``) and
``models/sewresnet.py`` (``sew_resnet18``) -- and records, for small seeded
cases, the inputs, the reference-pruned weights, BN parameters and the
reference outputs (spikes, pre-reset membrane per step, final membrane).
The files it writes are committed next to this script and read by
``tests/test_oracle_golden.py`` and the GPU parity tests.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def layer_case(ref, name, *, T, B, C, F, H, W, k, stride, pad, neuron="lif", x_max=1,
               residual=False, seed=0, linear=False):
    import torch
    import torch.nn as nn
    prune_2_4 = ref["prune_2_4"]
    SeqToANNContainer = ref["SeqToANNContainer"]
    g = torch.Generator().manual_seed(seed)
    if x_max == 1:
        x = (torch.rand((T, B, C, H, W), generator=g) < 0.2).float()
    else:
        x = torch.randint(0, x_max + 1, (T, B, C, H, W), generator=g).float()
    std = (2.0 / (F * k * k)) ** 0.5
    w = torch.randn((F, C, k, k), generator=g) * std
    w = prune_2_4(w.permute(0, 2, 3, 1)).permute(0, 3, 1, 2).contiguous()
    gamma = torch.rand(F, generator=g) + 0.5
    beta = torch.randn(F, generator=g) * 0.1
    mean = torch.randn(F, generator=g) * 0.1
    var = torch.rand(F, generator=g) + 0.5
    lin_bias = (torch.randn(F, generator=g) * 0.05) if linear else None

    if linear:
        # Spikformer MLP/SSA projection: Linear + BatchNorm1d + LIF on (T,B,N,C)
        # (models/spikformer.py:63-71).  Tokens are the H*W positions.
        lin = nn.Linear(C, F)
        lin.weight.data.copy_(w[:, :, 0, 0])
        lin.bias.data.copy_(lin_bias)
        bnm = nn.BatchNorm1d(F)
        bnm.weight.data.copy_(gamma); bnm.bias.data.copy_(beta)
        bnm.running_mean.copy_(mean); bnm.running_var.copy_(var)
        lin.eval(); bnm.eval()
        xs = x.flatten(3).transpose(2, 3)                 # (T,B,N,C)
        with torch.no_grad():
            z = lin(xs.flatten(0, 1))
            z = bnm(z.transpose(-1, -2)).transpose(-1, -2).reshape(T, B, H * W, F)
            z = z.transpose(2, 3).reshape(T, B, F, H, W)  # back to (T,B,F,H,W)
    else:
        conv = nn.Conv2d(C, F, k, stride=stride, padding=pad, bias=False)
        conv.weight.data.copy_(w)
        bnm = nn.BatchNorm2d(F)
        bnm.weight.data.copy_(gamma); bnm.bias.data.copy_(beta)
        bnm.running_mean.copy_(mean); bnm.running_var.copy_(var)
        seq = SeqToANNContainer(conv, bnm).eval()
        with torch.no_grad():
            z = seq(x)
    neuron_mod = ref["MultiStepLIFNeuron"](tau=2.0, v_threshold=1.0, v_reset=0.0) \
        if neuron == "lif" else ref["MultiStepIFNeuron"](v_threshold=1.0, v_reset=0.0)
    cell = neuron_mod.neuron
    cell.reset()
    spikes, hs = [], []
    with torch.no_grad():
        for t in range(T):
            # Same steps as the cell's forward, recording the pre-reset membrane.
            if neuron == "lif":
                cell.neuronal_charge(z[t])
                hs.append(cell.v.clone())
                s = cell.neuronal_fire()
                cell.neuronal_reset(s)
            else:
                s = cell(z[t])
                # IF: v after charge equals v_reset where it fired, else kept v.
                hs.append(None)
            spikes.append(s)
        v_final = cell.v.clone()
        # Cross-check against the unmodified multi-step module.
        ref_spk = neuron_mod(z)
    spikes = torch.stack(spikes)
    assert torch.equal(spikes, ref_spk)
    if neuron != "lif":
        # Recompute h for IF with the same float32 ops as IFNeuron.forward.
        v = torch.zeros_like(z[0]); hs = []
        for t in range(T):
            v = v + z[t]; hs.append(v.clone())
            sp = (v - 1.0).ge(0).float(); v = (1.0 - sp) * v + sp * 0.0
    h = torch.stack(hs)
    out = {"x": x.numpy().astype(np.uint8), "w": w.numpy(), "gamma": gamma.numpy(),
           "beta": beta.numpy(), "mean": mean.numpy(), "var": var.numpy(),
           "spikes": spikes.numpy().astype(np.uint8), "h": h.numpy(),
           "v": v_final.numpy(), "bn_out": z.numpy(),
           "meta": np.array([T, B, C, F, H, W, k, stride, pad, int(neuron == "lif"),
                             int(linear)], np.int64)}
    if linear:
        out["lin_bias"] = lin_bias.numpy()
    if residual:
        r = torch.randint(0, 3, spikes.shape, generator=g).float()
        out["residual"] = r.numpy().astype(np.uint8)
        out["out"] = (spikes + r).numpy().astype(np.uint8)
    np.savez_compressed(HERE / f"layer_{name}.npz", **out)
    print("wrote", name, {k: v.shape for k, v in out.items()})


def run_neuron(ref, kind, inp):
    """Reference multi-step neuron (tau 2 / v_th 1 / v_reset 0) over ``inp``
    ``(T, ...)``: spikes, pre-reset membrane per step and final membrane,
    cross-checked against the unmodified multi-step module."""
    import torch
    mod = ref["MultiStepLIFNeuron"](tau=2.0, v_threshold=1.0, v_reset=0.0) \
        if kind == "lif" else ref["MultiStepIFNeuron"](v_threshold=1.0, v_reset=0.0)
    cell = mod.neuron
    cell.reset()
    spikes, hs = [], []
    with torch.no_grad():
        for t in range(inp.shape[0]):
            if kind == "lif":
                cell.neuronal_charge(inp[t])
                hs.append(cell.v.clone())
                s = cell.neuronal_fire()
                cell.neuronal_reset(s)
            else:
                s = cell(inp[t])
            spikes.append(s)
        v_final = cell.v.clone()
        ref_spk = mod(inp)
    spikes = torch.stack(spikes)
    assert torch.equal(spikes, ref_spk)
    if kind != "lif":
        v = torch.zeros_like(inp[0]); hs = []
        for t in range(inp.shape[0]):
            v = v + inp[t]; hs.append(v.clone())
            sp = (v - 1.0).ge(0).float(); v = (1.0 - sp) * v + sp * 0.0
    return spikes, torch.stack(hs), v_final


def residual_case(ref, name, *, mode, neuron, neuron2="lif", T, B, C, F, H, W, k, seed):
    """The reference's other residual epilogues, run through its modules:
    ``mode="add_before"``: Conv -> BN -> Add(residual) -> neuron (pattern
    ``Conv2d+Add+LIF``, ``sengine/kernels/interleaved_templates.py:163-221``);
    ``mode="two_neuron"``: Conv -> BN -> neuron -> Add(residual) -> neuron2
    (``Conv2d+IF+Add+LIF``, ``:297-364``).  The residual is a real-valued
    fp16-representable tensor (an MS-ResNet style skip input)."""
    import torch
    import torch.nn as nn
    pad = k // 2
    g = torch.Generator().manual_seed(seed)
    x = (torch.rand((T, B, C, H, W), generator=g) < 0.2).float()
    std = (2.0 / (F * k * k)) ** 0.5
    w = torch.randn((F, C, k, k), generator=g) * std
    w = ref["prune_2_4"](w.permute(0, 2, 3, 1)).permute(0, 3, 1, 2).contiguous()
    gamma = torch.rand(F, generator=g) + 0.5
    beta = torch.randn(F, generator=g) * 0.1
    mean = torch.randn(F, generator=g) * 0.1
    var = torch.rand(F, generator=g) + 0.5
    conv = nn.Conv2d(C, F, k, stride=1, padding=pad, bias=False)
    conv.weight.data.copy_(w)
    bnm = nn.BatchNorm2d(F)
    bnm.weight.data.copy_(gamma); bnm.bias.data.copy_(beta)
    bnm.running_mean.copy_(mean); bnm.running_var.copy_(var)
    seq = ref["SeqToANNContainer"](conv, bnm).eval()
    with torch.no_grad():
        z = seq(x)
    r = (torch.randn(z.shape, generator=g) * 0.5).half().float()
    out = {"x": x.numpy().astype(np.uint8), "w": w.numpy(), "gamma": gamma.numpy(),
           "beta": beta.numpy(), "mean": mean.numpy(), "var": var.numpy(), "bn_out": z.numpy(),
           "residual_f": r.numpy(),
           "meta": np.array([T, B, C, F, H, W, k, 1, pad, int(neuron == "lif"), 0], np.int64)}
    if mode == "add_before":
        spikes, h, v = run_neuron(ref, neuron, z + r)
        out.update(spikes=spikes.numpy().astype(np.uint8), h=h.numpy(), v=v.numpy(),
                   out=spikes.numpy().astype(np.uint8),
                   res_meta=np.array([1, int(neuron2 == "lif")], np.int64))
    else:
        s1, h1, v1 = run_neuron(ref, neuron, z)
        s2, h2, v2 = run_neuron(ref, neuron2, s1 + r)
        out.update(spikes=s1.numpy().astype(np.uint8), h=h1.numpy(), v=v1.numpy(),
                   spikes2=s2.numpy().astype(np.uint8), h2=h2.numpy(), v2=v2.numpy(),
                   out=s2.numpy().astype(np.uint8),
                   res_meta=np.array([2, int(neuron2 == "lif")], np.int64))
    np.savez_compressed(HERE / f"layer_{name}.npz", **out)
    print("wrote", name, {k: v.shape for k, v in out.items()})


def attention_case(ref_path, name, *, T, B, N, heads, hd, p_spike, seed):
    """Spikformer attention core + attention LIF from the reference: the
    fused graph op's forward (``sengine/tdl/attention_ops.py:50-82``) and,
    as a cross-check, the model's own formulation (``models/spikformer.py:
    122-127``: matmuls in float32, then ``MultiStepLIFNeuron(tau=2,
    v_threshold=0.5)``)."""
    import importlib.util
    import torch
    from models.neurons import MultiStepLIFNeuron
    spec = importlib.util.spec_from_file_location(
        "attention_ops", str(Path(ref_path) / "sengine" / "tdl" / "attention_ops.py"))
    ops = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ops)
    g = torch.Generator().manual_seed(seed)
    C = heads * hd
    q, k, v = ((torch.rand((T * B, N, C), generator=g) < p_spike).float() for _ in range(3))
    with torch.no_grad():
        fused = ops._spikformer_attn_forward(None, q, k, v, T, heads, hd, 0.125, 2.0, 0.5)
        qh, kh, vh = (a.reshape(T, B, N, heads, hd).permute(0, 1, 3, 2, 4) for a in (q, k, v))
        x = ((qh @ kh.transpose(-2, -1)) * 0.125) @ vh
        x = x.transpose(2, 3).reshape(T, B, N, C)
        model = MultiStepLIFNeuron(tau=2.0, v_threshold=0.5)(x).reshape(T * B, N, C)
    assert torch.equal(fused, model)
    np.savez_compressed(HERE / f"attn_{name}.npz", q=q.numpy().astype(np.uint8),
                        k=k.numpy().astype(np.uint8), v=v.numpy().astype(np.uint8),
                        x=x.reshape(T * B, N, C).numpy(), spikes=model.numpy().astype(np.uint8),
                        meta=np.array([T, B, N, heads, hd], np.int64))
    print("wrote attn", name, tuple(q.shape), "spike rate", float(model.mean()))


def glue_case(ref):
    """MaxPool2d(3, 2, 1) -> MultiStepLIFNeuron and Add -> MultiStepLIFNeuron /
    MultiStepIFNeuron through the reference modules (the patterns of
    ``sengine/kernels/pool_lif_fused.py`` and ``add_lif_fused.py``)."""
    import torch
    import torch.nn as nn
    g = torch.Generator().manual_seed(21)
    T, B, C, H, W = 4, 2, 64, 9, 10
    x = (torch.randn((T, B, C, H, W), generator=g) * 1.5).half().float()
    pool = ref["SeqToANNContainer"](nn.MaxPool2d(3, 2, 1))
    with torch.no_grad():
        pooled = pool(x)
        s_pool = ref["MultiStepLIFNeuron"](tau=2.0, v_threshold=1.0, v_reset=0.0)(pooled)
    a = (torch.randn((T, B, C, H, W), generator=g)).half().float()
    b = torch.randint(0, 3, (T, B, C, H, W), generator=g).float()
    with torch.no_grad():
        s_add = ref["MultiStepLIFNeuron"](tau=2.0, v_threshold=1.0, v_reset=0.0)(a + b)
        s_add_if = ref["MultiStepIFNeuron"](v_threshold=1.0, v_reset=0.0)(a + b)
    np.savez_compressed(HERE / "glue.npz", x=x.numpy(), pooled=pooled.numpy(),
                        s_pool=s_pool.numpy().astype(np.uint8), a=a.numpy(), b=b.numpy(),
                        s_add=s_add.numpy().astype(np.uint8),
                        s_add_if=s_add_if.numpy().astype(np.uint8))
    print("wrote glue", tuple(x.shape), "pool rate", float(s_pool.mean()), "add rate",
          float(s_add.mean()))


def prune_case(ref):
    import torch
    g = torch.Generator().manual_seed(7)
    w = torch.randn((16, 8, 3, 3), generator=g)
    p = ref["prune_2_4"](w.permute(0, 2, 3, 1)).permute(0, 3, 1, 2).contiguous()
    w2 = torch.randn((6, 10), generator=g)          # last dim not a multiple of 4
    p2 = ref["prune_2_4"](w2)
    np.savez_compressed(HERE / "prune.npz", w=w.numpy(), pruned=p.numpy(), w2=w2.numpy(),
                        pruned2=p2.numpy())
    print("wrote prune")


def model_case(ref, repo):
    """SEW-ResNet-18 CIFAR-stem logits from the reference model class."""
    import torch
    import torch.nn as nn
    sys.path.insert(0, str(repo))
    from oracle.sew_resnet import make_params, make_input
    P = make_params(seed=0)
    m = ref["sew_resnet18"](in_channels=3, neuron_type="lif", num_classes=100, T=4)
    m.conv1 = nn.Conv2d(3, 64, 3, 1, 1, bias=False)
    m.maxpool = nn.Identity()
    t = torch.from_numpy

    def set_bn(bnm, p):
        bnm.weight.data.copy_(t(p["gamma"])); bnm.bias.data.copy_(t(p["beta"]))
        bnm.running_mean.copy_(t(p["mean"])); bnm.running_var.copy_(t(p["var"]))

    m.conv1.weight.data.copy_(t(P["stem"]["w"])); set_bn(m.bn1, P["stem"]["bn"])
    blocks = [b for layer in (m.layer1, m.layer2, m.layer3, m.layer4) for b in layer]
    for blk, p in zip(blocks, P["blocks"]):
        blk.conv1.module[0].weight.data.copy_(t(p["w1"])); set_bn(blk.conv1.module[1], p["bn1"])
        blk.conv2.module[0].weight.data.copy_(t(p["w2"])); set_bn(blk.conv2.module[1], p["bn2"])
        if "wd" in p:
            ds = blk.downsample[0].module
            ds[0].weight.data.copy_(t(p["wd"])); set_bn(ds[1], p["bnd"])
    m.fc.weight.data.copy_(t(P["fc_w"])); m.fc.bias.data.copy_(t(P["fc_b"]))
    m.eval()
    x = make_input(seed=0, B=2)
    with torch.no_grad():
        logits = m(t(x)).numpy()
    np.savez_compressed(HERE / "sew18_logits.npz", x=x, logits=logits)
    print("wrote sew18 logits", logits.shape)


def dvs_case(ref, repo):
    """DVS SEW-ResNet-18 logits (7x7/2 stem on 2-channel 128x128 event frames,
    MaxPool(3,2,1), T=16) from the reference model class as it is
    (``sew_resnet18(in_channels=2)``, ``models/sewresnet.py:140-143,190-210``)."""
    import torch
    sys.path.insert(0, str(repo))
    from oracle.sew_resnet import make_dvs_input, make_params
    P = make_params(seed=0, num_classes=11, in_channels=2, stem_kernel=7, input_moment=0.05)
    m = ref["sew_resnet18"](in_channels=2, neuron_type="lif", num_classes=11, T=16)
    _load_sew_params(m, P)
    x = make_dvs_input(seed=0, B=1, T=16)
    with torch.no_grad():
        logits = m(torch.from_numpy(x)).numpy()
    np.savez_compressed(HERE / "sew18_dvs_logits.npz", x_bits=np.packbits(x.astype(np.uint8)),
                        x_shape=np.array(x.shape), logits=logits)
    print("wrote sew18 dvs logits", logits.shape)


def _load_sew_params(m, P):
    import torch
    t = torch.from_numpy

    def set_bn(bnm, p):
        bnm.weight.data.copy_(t(p["gamma"])); bnm.bias.data.copy_(t(p["beta"]))
        bnm.running_mean.copy_(t(p["mean"])); bnm.running_var.copy_(t(p["var"]))

    m.conv1.weight.data.copy_(t(P["stem"]["w"])); set_bn(m.bn1, P["stem"]["bn"])
    blocks = [b for layer in (m.layer1, m.layer2, m.layer3, m.layer4) for b in layer]
    for blk, p in zip(blocks, P["blocks"]):
        blk.conv1.module[0].weight.data.copy_(t(p["w1"])); set_bn(blk.conv1.module[1], p["bn1"])
        blk.conv2.module[0].weight.data.copy_(t(p["w2"])); set_bn(blk.conv2.module[1], p["bn2"])
        if "wd" in p:
            ds = blk.downsample[0].module
            ds[0].weight.data.copy_(t(p["wd"])); set_bn(ds[1], p["bnd"])
    m.fc.weight.data.copy_(t(P["fc_w"])); m.fc.bias.data.copy_(t(P["fc_b"]))
    m.eval()


def msresnet_case(ref, repo):
    """MS-ResNet-34 logits from the reference model class (``ms_resnet34``,
    ``models/msresnet.py:126-171,335``) with every ``MSNeuron`` replaced by the
    reference's ``MultiStepLIFNeuron(tau=2, v_threshold=1)`` (the benchmark's
    neuron), at 224x224, T=4."""
    import torch
    sys.path.insert(0, str(repo))
    from oracle.ms_resnet import make_input, make_params
    import models.msresnet as msr
    P = make_params(seed=0)
    m = msr.ms_resnet34(num_classes=1000, in_channels=3, T=4)
    lif = lambda: ref["MultiStepLIFNeuron"](tau=2.0, v_threshold=1.0, v_reset=0.0)  # noqa: E731

    def swap(mod):
        for name, child in mod.named_children():
            if isinstance(child, msr.MSNeuron):
                setattr(mod, name, lif())
            else:
                swap(child)
    swap(m)
    t = torch.from_numpy

    def set_bn(bnm, p):
        bnm.weight.data.copy_(t(p["gamma"])); bnm.bias.data.copy_(t(p["beta"]))
        bnm.running_mean.copy_(t(p["mean"])); bnm.running_var.copy_(t(p["var"]))

    m.conv1.module[0].weight.data.copy_(t(P["stem"]["w"])); set_bn(m.conv1.module[1], P["stem"]["bn"])
    blocks = [b for st in (m.conv2_x, m.conv3_x, m.conv4_x, m.conv5_x) for b in st]
    assert len(blocks) == len(P["blocks"])
    for blk, p in zip(blocks, P["blocks"]):
        blk.conv_bn1.module[0].weight.data.copy_(t(p["w1"])); set_bn(blk.conv_bn1.module[1], p["bn1"])
        blk.conv_bn2.module[0].weight.data.copy_(t(p["w2"])); set_bn(blk.conv_bn2.module[1], p["bn2"])
        if "wsc" in p:
            blk.shortcut.module[0].weight.data.copy_(t(p["wsc"]))
            set_bn(blk.shortcut.module[1], p["bnsc"])
    m.fc.weight.data.copy_(t(P["fc_w"])); m.fc.bias.data.copy_(t(P["fc_b"]))
    m.eval()
    x = make_input(seed=0, B=1)
    with torch.no_grad():
        logits = m(t(x)).numpy()
    # the input is regenerated from its seed (oracle.ms_resnet.make_input)
    np.savez_compressed(HERE / "msresnet34_logits.npz", seed=np.array(0), batch=np.array(1),
                        logits=logits)
    print("wrote msresnet34 logits", logits.shape)


def spikformer_case(repo):
    """Spikformer-8-384 logits from the reference's own modules
    (``models/spikformer.py``): the ``SPS`` sub-modules (convs, BatchNorm2d,
    ``MultiStepLIFNeuron``s, ``MaxPool2d``) run in the benchmark geometry --
    a pool after each of the four stages, 224x224 -> 14x14 tokens -- then
    eight reference ``Block``s (12 heads) and the mean / Linear head, at
    T=4 on one 224x224 image."""
    import torch
    import torch.nn as nn
    sys.path.insert(0, str(repo))
    from oracle.spikformer import make_input, make_params
    import models.spikformer as sf
    P = make_params(seed=0)
    E, T, heads = P["embed"], 4, P["heads"]
    t = torch.from_numpy

    def set_bn(bnm, p):
        bnm.weight.data.copy_(t(p["gamma"])); bnm.bias.data.copy_(t(p["beta"]))
        bnm.running_mean.copy_(t(p["mean"])); bnm.running_var.copy_(t(p["var"]))

    def set_lin(lin, bnm, p):
        lin.weight.data.copy_(t(p["w"])); lin.bias.data.copy_(t(p["b"])); set_bn(bnm, p["bn"])

    sps = sf.SPS(img_size_h=224, img_size_w=224, patch_size=16, in_channels=3, embed_dims=E)
    stages = [(sps.proj_conv, sps.proj_bn, sps.proj_lif), (sps.proj_conv1, sps.proj_bn1, sps.proj_lif1),
              (sps.proj_conv2, sps.proj_bn2, sps.proj_lif2), (sps.proj_conv3, sps.proj_bn3, sps.proj_lif3)]
    for (conv, bnm, _), p in zip(stages, P["sps"]):
        conv.weight.data.copy_(t(p["w"])); set_bn(bnm, p["bn"])
    sps.rpe_conv.weight.data.copy_(t(P["rpe"]["w"])); set_bn(sps.rpe_bn, P["rpe"]["bn"])
    blocks = [sf.Block(dim=E, num_heads=heads, mlp_ratio=4) for _ in P["blocks"]]
    for blk, p in zip(blocks, P["blocks"]):
        a = blk.attn
        set_lin(a.q_linear, a.q_bn, p["q"]); set_lin(a.k_linear, a.k_bn, p["k"])
        set_lin(a.v_linear, a.v_bn, p["v"]); set_lin(a.proj_linear, a.proj_bn, p["proj"])
        set_lin(blk.mlp.fc1_linear, blk.mlp.fc1_bn, p["fc1"])
        set_lin(blk.mlp.fc2_linear, blk.mlp.fc2_bn, p["fc2"])
    head = nn.Linear(E, P["fc_w"].shape[0])
    head.weight.data.copy_(t(P["fc_w"])); head.bias.data.copy_(t(P["fc_b"]))
    for mod in [sps, head] + blocks:
        mod.eval()
    x = make_input(seed=0, B=1)
    with torch.no_grad():
        xs = t(x).unsqueeze(0).repeat(T, 1, 1, 1, 1)
        Tn, B, _, H, W = xs.shape
        y = xs.flatten(0, 1)
        pools = [sps.maxpool2, sps.maxpool2, sps.maxpool2, sps.maxpool3]
        for (conv, bnm, lif), pool in zip(stages, pools):
            y = bnm(conv(y)).reshape(Tn, B, -1, H, W)
            y = pool(lif(y).flatten(0, 1))
            H, W = H // 2, W // 2
        x_feat = y.reshape(Tn, B, -1, H, W)
        r = sps.rpe_lif(sps.rpe_bn(sps.rpe_conv(y)).reshape(Tn, B, -1, H, W))
        xt = (r + x_feat).flatten(-2).transpose(-1, -2)
        for blk in blocks:
            xt = blk(xt)
        logits = head(xt.mean(2).mean(0)).numpy()
    np.savez_compressed(HERE / "spikformer_logits.npz", seed=np.array(0), batch=np.array(1),
                        logits=logits)
    print("wrote spikformer logits", logits.shape)


CASES = ("prune", "layers", "residual", "attention", "glue", "sew18", "dvs", "msresnet",
         "spikformer")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of the SparseSNN reference checkout")
    ap.add_argument("--only", nargs="*", choices=CASES, help="regenerate only these fixtures")
    a = ap.parse_args()
    only = set(a.only or CASES)
    sys.path.insert(0, a.ref)
    from sparse.pruning import prune_2_4
    from models.neurons import MultiStepLIFNeuron, MultiStepIFNeuron
    from models.layers import SeqToANNContainer
    from models.sewresnet import sew_resnet18
    ref = dict(prune_2_4=prune_2_4, MultiStepLIFNeuron=MultiStepLIFNeuron,
               MultiStepIFNeuron=MultiStepIFNeuron, SeqToANNContainer=SeqToANNContainer,
               sew_resnet18=sew_resnet18)
    import torch
    torch.set_num_threads(4)
    if "prune" in only:
        prune_case(ref)
    if "layers" in only:
        layer_cases(ref)
    if "residual" in only:
        residual_case(ref, "c3addlif", mode="add_before", neuron="lif", T=4, B=2, C=64, F=128,
                      H=8, W=8, k=3, seed=9)
        residual_case(ref, "c1twon", mode="two_neuron", neuron="if", neuron2="lif", T=4, B=2,
                      C=128, F=64, H=8, W=8, k=1, seed=10)
    if "attention" in only:
        attention_case(a.ref, "n64", T=4, B=2, N=64, heads=2, hd=32, p_spike=0.13, seed=11)
        attention_case(a.ref, "n196", T=4, B=2, N=196, heads=2, hd=32, p_spike=0.09, seed=12)
        attention_case(a.ref, "n100h64", T=3, B=2, N=100, heads=2, hd=64, p_spike=0.09, seed=13)
    if "glue" in only:
        glue_case(ref)
    repo = HERE.parent.parent
    if "sew18" in only:
        model_case(ref, repo)
    if "dvs" in only:
        dvs_case(ref, repo)
    if "msresnet" in only:
        msresnet_case(ref, repo)
    if "spikformer" in only:
        spikformer_case(repo)


def layer_cases(ref):
    layer_case(ref, "c3s1", T=4, B=2, C=64, F=128, H=8, W=8, k=3, stride=1, pad=1, seed=1)
    layer_case(ref, "c3s2", T=2, B=2, C=64, F=128, H=8, W=8, k=3, stride=2, pad=1, seed=2)
    layer_case(ref, "c1s2", T=4, B=2, C=64, F=128, H=8, W=8, k=1, stride=2, pad=0, seed=3)
    layer_case(ref, "c3res", T=4, B=2, C=128, F=128, H=4, W=4, k=3, stride=1, pad=1, x_max=2,
               residual=True, seed=4)
    layer_case(ref, "c3f64", T=4, B=2, C=64, F=64, H=8, W=8, k=3, stride=1, pad=1, seed=5)
    layer_case(ref, "c3if", T=4, B=2, C=64, F=128, H=8, W=8, k=3, stride=1, pad=1, neuron="if",
               seed=6)
    layer_case(ref, "lin", T=4, B=2, C=128, F=256, H=4, W=4, k=1, stride=1, pad=0, seed=8,
               linear=True)


if __name__ == "__main__":
    main()
