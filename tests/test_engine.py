"""Native whole-model executor (snn_engine_*) and its engine file.

CPU: the file layout written by ``engine_file`` is what the C++ parser reads,
and damaged files (magic, version, size, offsets, node kinds, tensor ids)
are rejected with SNN_E_INVALID.  GPU: an engine saved from a SEW-ResNet-18
replica gives the Python driver's logits exactly (the same kernels on the
same data), eagerly and replayed from its CUDA graph, with host and device
buffers, call after call.
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
