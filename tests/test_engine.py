"""Native whole-model executor (snn_engine_*) and its engine file.

CPU: the file layout written by ``engine_file`` is what the C++ parser reads,
and damaged files (magic, version, size, offsets, node kinds, tensor ids)
are rejected with SNN_E_INVALID.  GPU: an engine saved from a SEW-ResNet-18
replica gives the Python driver's logits exactly (the same kernels on the
same data), eagerly and replayed from its CUDA graph, with host and device
buffers, call after call; an engine with the glue node kinds gives the
logits of the same entry points called one by one.
"""
import ctypes
import struct

import numpy as np
import pytest

from sparsesnn_b200 import runtime as rt
from sparsesnn_b200 import engine_file as ef


@pytest.fixture(scope="module")
def lib():
    from sparsesnn_b200 import build
    build.build()
    return rt.load()


def _small_file(path, *, T=4, B=2, cin=64, cout=128, hw=8, nc=10):
    """One 3x3 conv node and a head, with zero parameters."""
    w = ef._Writer()
    d = rt.make_desc(T=T, B=B, Cin=cin, H=hw, W=hw, Cout=cout, KH=3, KW=3)
    nbytes = ctypes.c_size_t()
    rt.check(rt.load().snn_conv_weight_bytes(d, ctypes.byref(nbytes)))
    x = w.tensor(T * B * hw * hw * cin * 2, ef.F16)
    images = w.tensor(B * 4, ef.F32)
    y = w.tensor(T * B * hw * hw * cout * 2, ef.F16)
    logits = w.tensor(B * nc * 4, ef.F32)
    w.node(ef.OP_CONV, x, ef.NO_TENSOR, y, d,
           (w.param(np.zeros(nbytes.value, np.uint8)), w.param(np.ones(cout, np.float32)),
            w.param(np.zeros(cout, np.float32)), 0))
    w.node(ef.OP_HEAD, y, ef.NO_TENSOR, logits, None,
           (w.param(np.zeros((nc, cout), np.float32)), w.param(np.zeros(nc, np.float32)), 0, 0),
           (T, B, hw * hw, cout, nc))
    w.write(path, images, logits, T, B)
    return path


def test_engine_file_round_trip(lib, tmp_path):
    p = _small_file(tmp_path / "small.snne")
    assert ef.check_file(p) == (2, 4)


def _corrupt(src, dst, offset, data):
    b = bytearray(src.read_bytes())
    b[offset:offset + len(data)] = data
    dst.write_bytes(bytes(b))
    return dst


@pytest.mark.parametrize("what", ["magic", "version", "truncated", "offset", "kind", "tensor_id",
                                  "flags"])
def test_damaged_engine_file_rejected(lib, tmp_path, what):
    src = _small_file(tmp_path / "ok.snne")
    raw = src.read_bytes()
    node0 = 64 + 4 * 16                       # first node record
    bad = tmp_path / "bad.snne"
    if what == "magic":
        _corrupt(src, bad, 0, b"XXXX")
    elif what == "version":
        _corrupt(src, bad, 4, struct.pack("<I", 99))
    elif what == "truncated":
        bad.write_bytes(raw[:-8])
    elif what == "offset":                    # weight offset past the blob
        _corrupt(src, bad, node0 + 96, struct.pack("<Q", 1 << 40))
    elif what == "kind":
        _corrupt(src, bad, node0, struct.pack("<I", 77))
    elif what == "tensor_id":
        _corrupt(src, bad, node0 + 4, struct.pack("<I", 1000))
    elif what == "flags":                     # engines keep no membrane between forwards
        _corrupt(src, bad, node0 + 16 + 11 * 4, struct.pack("<i", rt.SNN_FLAG_READ_STATE))
    with pytest.raises(rt.SnnError) as ei:
        ef.check_file(bad)
    assert ei.value.code == rt.SNN_E_INVALID


def _stem_file(path, *, H, kh, pad, stride, out_hw, T=2, B=1, cout=16):
    """A stem node whose output tensor holds out_hw x out_hw pixels, and a head."""
    w = ef._Writer()
    d = rt.make_desc(T=T, B=B, Cin=3, H=H, W=H, Cout=cout, KH=kh, KW=kh, stride=stride, pad=pad)
    images = w.tensor(B * 3 * H * H * 4, ef.F32)
    a0 = w.tensor(T * B * out_hw * out_hw * cout * 2, ef.F16)
    logits = w.tensor(B * 4 * 4, ef.F32)
    w.node(ef.OP_STEM, images, ef.NO_TENSOR, a0, d,
           (w.param(np.zeros((cout, 3, kh, kh), np.float32)), w.param(np.ones(cout, np.float32)),
            w.param(np.zeros(cout, np.float32)), 0), (1, 0, 0, 0, 0))
    w.node(ef.OP_HEAD, a0, ef.NO_TENSOR, logits, None,
           (w.param(np.zeros((4, cout), np.float32)), w.param(np.zeros(4, np.float32)), 0, 0),
           (T, B, out_hw * out_hw, cout, 4))
    w.write(path, images, logits, T, B)
    return path


def test_stem_output_size_checked_from_its_geometry(lib, tmp_path):
    """The stem check sizes the output from OH x OW: a 1x1 stem with pad 2
    writes (H+4)^2 pixels, so an H x H output tensor is rejected; a 7x7
    stride-2 stem needs only its (H/2)^2 pixels."""
    bad = _stem_file(tmp_path / "pad2.snne", H=8, kh=1, pad=2, stride=1, out_hw=8)
    with pytest.raises(rt.SnnError) as ei:
        ef.check_file(bad)
    assert ei.value.code == rt.SNN_E_INVALID
    ok = _stem_file(tmp_path / "pad2ok.snne", H=8, kh=1, pad=2, stride=1, out_hw=12)
    assert ef.check_file(ok) == (2, 3)
    s2 = _stem_file(tmp_path / "s2.snne", H=16, kh=7, pad=3, stride=2, out_hw=8)
    assert ef.check_file(s2) == (2, 3)
    neg = _stem_file(tmp_path / "neg.snne", H=16, kh=7, pad=-1, stride=2, out_hw=8)
    with pytest.raises(rt.SnnError):
        ef.check_file(neg)


def _bits_file(path, *, stem_flags, pool_flags, a0_bytes_per_px, pool_op=ef.OP_MAXPOOL_LIF,
               T=2, B=1, H=16, cout=16):
    """Stem -> plain max pool (3x3/2/1) -> head; the stem output tensor holds
    a0_bytes_per_px bytes a pixel."""
    w = ef._Writer()
    d = rt.make_desc(T=T, B=B, Cin=3, H=H, W=H, Cout=cout, KH=3, KW=3, stride=1, pad=1,
                     flags=stem_flags)
    images = w.tensor(B * 3 * H * H * 4, ef.F32)
    a0 = w.tensor(T * B * H * H * a0_bytes_per_px, ef.F16)
    P = (H + 2 - 3) // 2 + 1
    p0 = w.tensor(T * B * P * P * cout * 2, ef.F16)
    logits = w.tensor(B * 4 * 4, ef.F32)
    w.node(ef.OP_STEM, images, ef.NO_TENSOR, a0, d,
           (w.param(np.zeros((cout, 3, 3, 3), np.float32)), w.param(np.ones(cout, np.float32)),
            w.param(np.zeros(cout, np.float32)), 0), (1, 0, 0, 0, 0))
    pd = rt.make_desc(T=T, B=B, Cin=cout, H=H, W=H, Cout=cout, KH=3, KW=3, stride=2, pad=1,
                      neuron="none", flags=pool_flags)
    w.node(pool_op, a0, a0 if pool_op == ef.OP_ADD_LIF else ef.NO_TENSOR, p0, pd)
    w.node(ef.OP_HEAD, p0, ef.NO_TENSOR, logits, None,
           (w.param(np.zeros((4, cout), np.float32)), w.param(np.zeros(4, np.float32)), 0, 0),
           (T, B, P * P, cout, 4))
    w.write(path, images, logits, T, B)
    return path


def test_bit_packed_stem_and_pool_nodes(lib, tmp_path):
    """SNN_FLAG_SPIKE_BITS between a stem and its max pool: the tensor needs
    only Cout/8 bytes a pixel when both nodes carry the flag; without it the
    same tensor is too small, and no other glue node may take the flag."""
    bits = rt.SNN_FLAG_SPIKE_BITS
    ok = _bits_file(tmp_path / "bits.snne", stem_flags=bits, pool_flags=bits, a0_bytes_per_px=2)
    assert ef.check_file(ok) == (3, 4)
    for name, kw in [("stem_fp16", dict(stem_flags=0, pool_flags=bits)),
                     ("pool_fp16", dict(stem_flags=bits, pool_flags=0)),
                     ("add_bits", dict(stem_flags=bits, pool_flags=bits, pool_op=ef.OP_ADD_LIF))]:
        bad = _bits_file(tmp_path / f"{name}.snne", a0_bytes_per_px=2, **kw)
        with pytest.raises(rt.SnnError) as ei:
            ef.check_file(bad)
        assert ei.value.code == rt.SNN_E_INVALID, name
    fp16 = _bits_file(tmp_path / "fp16.snne", stem_flags=0, pool_flags=0, a0_bytes_per_px=32)
    assert ef.check_file(fp16) == (3, 4)


def test_missing_engine_file(lib, tmp_path):
    with pytest.raises(rt.SnnError):
        ef.check_file(tmp_path / "absent.snne")


@pytest.mark.gpu
def test_engine_matches_python_driver(cuda_device, tmp_path):
    import torch
    from sparsesnn_b200.sew_resnet import SEWResNet18, init_params
    T, B = 4, 8
    model = SEWResNet18(init_params(seed=3), T=T, batch=B)
    path = ef.save_engine(model, tmp_path / "sew18.snne")
    assert ef.check_file(path) == (21, 1 + 1 + 8 * 2 + 3 + 1)
    rng = np.random.default_rng(5)
    imgs = [torch.from_numpy(rng.standard_normal((B, 3, 32, 32)).astype(np.float32)).pin_memory()
            for _ in range(2)]
    ref = []
    for x in imgs:
        ref.append(model(x).clone())
    torch.cuda.synchronize()
    eng = ef.Engine(path)
    assert (eng.T, eng.B, eng.image_bytes, eng.logit_bytes) == (T, B, B * 3 * 32 * 32 * 4, B * 100 * 4)
    s = torch.cuda.Stream()
    out_h = torch.empty((B, 100), dtype=torch.float32).pin_memory()
    out_d = torch.empty((B, 100), dtype=torch.float32, device="cuda")
    # eager node loop, host buffers, two calls in a row
    for x, r in zip(imgs, ref):
        eng.run(x.data_ptr(), out_h.data_ptr(), s)
        s.synchronize()
        assert torch.equal(out_h, r.cpu())
    # captured graph, device buffers
    eng.capture(s)
    for x, r in zip(imgs, ref):
        xd = x.to("cuda")
        torch.cuda.synchronize()
        eng.run(xd.data_ptr(), out_d.data_ptr(), s)
        s.synchronize()
        assert torch.equal(out_d, r)
    assert rt.device_error() == 0
    eng.close()


@pytest.mark.gpu
def test_engine_glue_nodes_match_direct_calls(cuda_device, tmp_path):
    """An engine with the other node kinds -- stem, MaxPool(3,2,1)+LIF, Add+LIF,
    a 3x3 conv with the SEW residual, head -- gives the logits of the same
    entry points called one by one."""
    import torch
    from sparsesnn_b200.layer import SparseConvBNLIF
    from sparsesnn_b200.pruning import prune_conv_2_4
    lib = rt.load()
    T, B, H, C, F, NC = 4, 4, 32, 64, 64, 10
    rng = np.random.default_rng(9)
    f32 = lambda *sh: rng.standard_normal(sh).astype(np.float32)  # noqa: E731
    stem_w = f32(C, 3, 3, 3) * 0.3
    stem_s, stem_b = np.abs(f32(C)) + 0.5, f32(C) * 0.1
    stem_d = rt.make_desc(T=T, B=B, Cin=3, H=H, W=H, Cout=C, KH=3, KW=3, pad=1)
    # IF for the pooled spikes (a tau = 2 LIF fed 0/1 never reaches 1.0 in 4 steps)
    pool_d = rt.make_desc(T=T, B=B, Cin=C, H=H, W=H, Cout=C, KH=3, KW=3, stride=2, pad=1,
                          neuron="if")
    P = H // 2
    add_d = rt.make_desc(T=T, B=B, Cin=C, H=P, W=P, Cout=C, KH=1, KW=1, pad=0, neuron="if",
                         v_threshold=1.5)
    conv = SparseConvBNLIF(prune_conv_2_4(f32(F, C, 3, 3) * 0.1), np.ones(F, np.float32),
                           np.zeros(F, np.float32), T=T, B=B, H=P, W=P)
    fc_w, fc_b = f32(NC, F) * 0.1, f32(NC) * 0.1

    w = ef._Writer()
    images = w.tensor(B * 3 * H * H * 4, ef.F32)
    a0 = w.tensor(T * B * H * H * C * 2, ef.F16)
    p0 = w.tensor(T * B * P * P * C * 2, ef.F16)
    q0 = w.tensor(T * B * P * P * C * 2, ef.F16)
    r0 = w.tensor(T * B * P * P * F * 2, ef.F16)
    logits = w.tensor(B * NC * 4, ef.F32)
    w.node(ef.OP_STEM, images, ef.NO_TENSOR, a0, stem_d,
           (w.param(stem_w), w.param(stem_s), w.param(stem_b), 0), (1, 0, 0, 0, 0))
    w.node(ef.OP_MAXPOOL_LIF, a0, ef.NO_TENSOR, p0, pool_d)
    w.node(ef.OP_ADD_LIF, p0, p0, q0, add_d)
    w.node(ef.OP_CONV, q0, p0, r0, ef._conv_desc(conv),
           (w.param(conv.weight_blob.cpu().numpy()), w.param(conv.bn_scale.cpu().numpy()),
            w.param(conv.bn_bias.cpu().numpy()), 0))
    w.node(ef.OP_HEAD, r0, ef.NO_TENSOR, logits, None, (w.param(fc_w), w.param(fc_b), 0, 0),
           (T, B, P * P, F, NC))
    path = tmp_path / "glue.snne"
    w.write(path, images, logits, T, B)
    assert ef.check_file(path) == (5, 6)

    x = torch.from_numpy(f32(B, 3, H, H)).cuda()
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    sw, ss, sb, fw, fb = dev(stem_w), dev(stem_s), dev(stem_b), dev(fc_w), dev(fc_b)
    a = torch.empty((T * B, H, H, C), dtype=torch.float16, device="cuda")
    p = torch.empty((T * B, P, P, C), dtype=torch.float16, device="cuda")
    q = torch.empty_like(p)
    r = torch.empty((T * B, P, P, F), dtype=torch.float16, device="cuda")
    ref = torch.empty((B, NC), dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    rt.check(lib.snn_stem_forward(stem_d, 1, x.data_ptr(), sw.data_ptr(), ss.data_ptr(), sb.data_ptr(),
                                  a.data_ptr(), s))
    rt.check(lib.snn_maxpool_lif_forward(pool_d, a.data_ptr(), None, p.data_ptr(), s))
    rt.check(lib.snn_add_lif_forward(add_d, p.data_ptr(), p.data_ptr(), None, q.data_ptr(), s))
    conv(q, residual=p, out=r)
    rt.check(lib.snn_head_forward(T, B, P * P, F, NC, r.data_ptr(), fw.data_ptr(), fb.data_ptr(),
                                  ref.data_ptr(), s))
    torch.cuda.synchronize()
    assert p.float().abs().sum() > 0 and q.float().abs().sum() > 0     # spikes at every stage

    eng = ef.Engine(path)
    st = torch.cuda.Stream()
    out = torch.empty_like(ref)
    for _ in range(2):
        eng.run(x.data_ptr(), out.data_ptr(), st)
        st.synchronize()
        assert torch.equal(out, ref)
    assert rt.device_error() == 0
    eng.close()


@pytest.mark.gpu
@pytest.mark.parametrize("which", ["dvs", "msresnet", "spikformer"])
def test_plan_models_through_the_engine(cuda_device, tmp_path, which):
    """An engine file saved from a node-plan model (plain max pool, single-input
    LIF, fp16 BN output with the membrane shortcut, dense weights, attention
    nodes) gives the Python driver's logits exactly, eagerly and replayed from
    its CUDA graph, two calls in a row."""
    import torch
    rng = np.random.default_rng(11)
    if which == "dvs":
        from sparsesnn_b200.sew_resnet import SEWResNet18DVS, init_params
        model = SEWResNet18DVS(init_params(seed=1, num_classes=11, in_channels=2, stem_kernel=7,
                                           input_moment=0.05), T=8, batch=1, H=64, W=64)
        xs = [(rng.random((8, 1, 2, 64, 64)) < 0.05).astype(np.float32) for _ in range(2)]
    elif which == "msresnet":
        from sparsesnn_b200.ms_resnet import MSResNet34, init_params
        model = MSResNet34(init_params(seed=1, num_classes=10), T=4, batch=2, H=64, W=64)
        xs = [rng.standard_normal((2, 3, 64, 64)).astype(np.float32) for _ in range(2)]
    else:
        from sparsesnn_b200.spikformer import Spikformer, init_params
        model = Spikformer(init_params(seed=1, depth=2, num_classes=10), T=4, batch=2, H=64, W=64)
        xs = [rng.standard_normal((2, 3, 64, 64)).astype(np.float32) for _ in range(2)]
    imgs = [torch.from_numpy(x).pin_memory() for x in xs]
    ref = [model(x).clone() for x in imgs]
    torch.cuda.synchronize()
    path = ef.save_engine(model, tmp_path / f"{which}.snne")
    assert ef.check_file(path)[0] == len(model.nodes)
    eng = ef.Engine(path)
    s = torch.cuda.Stream()
    out = torch.empty_like(ref[0])
    for graph in (False, True):
        if graph:
            eng.capture(s)
        for x, r in zip(imgs, ref):
            eng.run(x.data_ptr(), out.data_ptr(), s)
            s.synchronize()
            assert torch.equal(out, r), (which, graph)
    assert rt.device_error() == 0
    eng.close()
