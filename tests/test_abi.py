"""The C-ABI library loads and exports every symbol include/snn_b200.h
declares; descriptor validation works without a GPU."""
import ctypes
import re
import subprocess

import pytest

from conftest import ROOT
from sparsesnn_b200 import build, runtime as rt


@pytest.fixture(scope="module", autouse=True)
def _lib():
    build.build()
    return rt.load()


def header_functions():
    text = (ROOT / "include" / "snn_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(snn_[a-z0-9_]+)\s*\(", text)))


def test_exports_every_declared_symbol(_lib):
    names = header_functions()
    assert names and set(names) == set(rt.EXPORTED)
    out = subprocess.run(["nm", "-D", "--defined-only", str(rt.LIB_PATH)],
                         capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    for n in names:
        assert n in exported, n
        assert hasattr(_lib, n)


def test_abi_version(_lib):
    assert _lib.snn_abi_version() == 3


def test_desc_struct_layout():
    assert ctypes.sizeof(rt.SnnConvDesc) == 20 * 4
    assert rt.SnnConvDesc.res_mode.offset == 15 * 4


def test_residual_entry_points_validate_mode(_lib):
    """forward_res takes ADD_AFTER / ADD_BEFORE, forward_res2 only TWO_NEURON;
    the checks come before any device work."""
    d = rt.make_desc(T=4, B=2, Cin=64, H=8, W=8, Cout=128, KH=3, KW=3, res_mode="two_neuron")
    rc = _lib.snn_conv_forward_res(d, 16, 16, None, 16, 16, 16, 16, None)
    assert rc == rt.SNN_E_INVALID
    d = rt.make_desc(T=4, B=2, Cin=64, H=8, W=8, Cout=128, KH=3, KW=3, res_mode="add_before")
    rc = _lib.snn_conv_forward_res2(d, 16, 16, None, None, 16, 16, 16, 16, None)
    assert rc == rt.SNN_E_INVALID
    rc = _lib.snn_conv_forward_res2(d, 16, 16, None, None, 16, 16, None, 16, None)
    assert rc == rt.SNN_E_INVALID


@pytest.mark.parametrize("kw, msg", [
    (dict(Cin=36), "multiple of 8"),
    (dict(stride=3), "stride"),
    (dict(H=9, stride=2), "even"),
    (dict(Cin=64 * 150), "exceeds"),
])
def test_invalid_descriptors(kw, msg):
    base = dict(T=4, B=2, Cin=64, H=8, W=8, Cout=128, KH=3, KW=3)
    base.update(kw)
    d = rt.make_desc(**base)
    with pytest.raises(rt.SnnError) as e:
        rt.weight_bytes(d)
    assert e.value.code == rt.SNN_E_INVALID and msg in str(e.value)


def test_out_shape_and_weight_bytes():
    d = rt.make_desc(T=4, B=16, Cin=128, H=32, W=32, Cout=128, KH=3, KW=3)
    assert rt.out_shape(d) == (32, 32)
    # values 128 x 576 fp16 + meta 1 x 36 x 128 words
    assert rt.weight_bytes(d) == 128 * 576 * 2 + 36 * 128 * 4
    d = rt.make_desc(T=4, B=16, Cin=64, H=32, W=32, Cout=128, KH=1, KW=1, stride=2, pad=0)
    assert rt.out_shape(d) == (16, 16)


def test_forward_without_device_fails_loudly(_lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    d = rt.make_desc(T=1, B=1, Cin=64, H=8, W=8, Cout=128, KH=3, KW=3)
    rc = _lib.snn_conv_forward(d, 16, 16, None, 16, 16, 16, None)
    assert rc in (rt.SNN_E_NO_DEVICE, rt.SNN_E_CUDA)


@pytest.mark.parametrize("kw, expect", [
    (dict(Cin=128, H=32, W=32), rt.SNN_VARIANT_HALO_RESIDENT),      # config 0
    (dict(Cin=64, H=32, W=32, Cout=64), rt.SNN_VARIANT_HALO_RESIDENT),
    (dict(Cin=256, H=12, W=12, Cout=256), rt.SNN_VARIANT_HALO_STREAM),
    (dict(Cin=512, H=8, W=12, Cout=512), rt.SNN_VARIANT_HALO_STREAM),
    (dict(Cin=256, H=8, W=8, Cout=256), rt.SNN_VARIANT_HALO_STREAM),
    (dict(Cin=512, H=16, W=16, Cout=512), rt.SNN_VARIANT_HALO_STREAM),
    (dict(Cin=256, H=8, W=8, T=5), rt.SNN_VARIANT_GENERIC),          # T > 4
    (dict(Cin=512, H=4, W=4), rt.SNN_VARIANT_HALO_STREAM),           # 4x4: four images per tile
    (dict(Cin=512, H=6, W=6), rt.SNN_VARIANT_GENERIC),               # other images < 8x8
    (dict(Cin=64, H=32, W=32, stride=2), rt.SNN_VARIANT_GENERIC),
    (dict(Cin=64, H=32, W=32, KH=1, KW=1, pad=0), rt.SNN_VARIANT_GENERIC),
    (dict(Cin=128, H=32, W=32, flags=rt.SNN_FLAG_FORCE_GENERIC), rt.SNN_VARIANT_GENERIC),
    # only the general kernel has the Add-before-neuron and two-neuron epilogues
    (dict(Cin=128, H=32, W=32, res_mode="add_before"), rt.SNN_VARIANT_GENERIC),
    (dict(Cin=256, H=12, W=12, Cout=256, res_mode="two_neuron"), rt.SNN_VARIANT_GENERIC),
])
def test_variant_selection(kw, expect):
    base = dict(T=4, B=2, Cin=64, H=8, W=8, Cout=128, KH=3, KW=3)
    base.update(kw)
    assert rt.variant(rt.make_desc(**base)) == expect
