"""2:4 packing: the C++ packer in libsnnb200.so is bit-exact with the oracle.

Runs on CPU: the packer is host code and needs no GPU.
"""
import itertools

import numpy as np
import pytest

from conftest import LAYER_CASES, load_layer_case
from oracle import pack24 as P
from sparsesnn_b200 import build, runtime as rt

PATTERNS = list(itertools.combinations(range(4), 2))     # the 6 legal pairs


@pytest.fixture(scope="module", autouse=True)
def _lib():
    build.build()
    rt.load()


def split_blob(blob, f_pad, k):
    nv = f_pad * (k // 2) * 2
    off = (nv + 255) // 256 * 256
    return blob[:nv].view(np.float16).reshape(f_pad, k // 2), \
        blob[off:].view(np.uint32).reshape(f_pad // 128, k // 32, 128)


def c_pack(w_fchw):
    f, c, kh, kw = w_fchw.shape
    d = rt.make_desc(T=1, B=1, Cin=c, H=8, W=8, Cout=f, KH=kh, KW=kw)
    blob = rt.pack_weight_24(d, w_fchw)
    return split_blob(blob, -(-f // 128) * 128, c * kh * kw)


@pytest.mark.parametrize("name", LAYER_CASES)
def test_c_packer_bit_exact_on_reference_pruned_weights(name):
    g = load_layer_case(name)
    vals, meta = c_pack(g["w"])
    wfk = P.conv_weight_to_fk(g["w"])
    assert np.array_equal(vals, P.pack_values(wfk))
    assert np.array_equal(meta, P.pack_meta(wfk))


def test_roundtrip_unpack_equals_fp16_weight():
    rng = np.random.default_rng(3)
    w = P.prune_conv_weight(rng.standard_normal((192, 128, 3, 3)).astype(np.float32))
    vals, meta = c_pack(w)
    wfk = P.conv_weight_to_fk(w)
    dense = P.unpack(vals, meta, 192, wfk.shape[1])
    assert np.array_equal(dense, wfk.astype(np.float16).astype(np.float32))


def _pattern_weight(f=128, c=64):
    """Row r, group g keeps PATTERNS[(r + g) % 6] with value (r+1) + g/64."""
    w = np.zeros((f, c, 1, 1), np.float32)
    for r in range(f):
        for gi in range(c // 4):
            i0, i1 = PATTERNS[(r + gi) % 6]
            w[r, 4 * gi + i0, 0, 0] = r + 1 + gi / 64
            w[r, 4 * gi + i1, 0, 0] = -(r + 1) - gi / 64
    return w


def test_known_answer_all_six_patterns():
    w = _pattern_weight()
    vals, meta = c_pack(w)
    nib = {p: p[0] | (p[1] << 2) for p in PATTERNS}
    assert sorted(nib.values()) == [0x4, 0x8, 0x9, 0xC, 0xD, 0xE]
    # Independent re-derivation of a few words, written out by hand:
    # lane 0 covers rows 0 (low half) and 8 (high half), groups 0..3.
    expect = 0
    for q in range(4):
        expect |= nib[PATTERNS[(0 + q) % 6]] << (4 * q)
        expect |= nib[PATTERNS[(8 + q) % 6]] << (16 + 4 * q)
    assert meta[0, 0, 0] == expect
    # lane 8 covers the same rows, groups 4..7.
    expect = 0
    for q in range(4):
        expect |= nib[PATTERNS[(0 + 4 + q) % 6]] << (4 * q)
        expect |= nib[PATTERNS[(8 + 4 + q) % 6]] << (16 + 4 * q)
    assert meta[0, 0, 8] == expect
    # lane 29 -> rows 16*(29//16) + 29%8 = 21 and 29; (29//8) odd -> groups 4..7
    expect = 0
    for q in range(4):
        expect |= nib[PATTERNS[(21 + 4 + q) % 6]] << (4 * q)
        expect |= nib[PATTERNS[(29 + 4 + q) % 6]] << (16 + 4 * q)
    assert meta[0, 0, 29] == expect
    # row 0 low half and row 8 high half of lane 0, as literal hex
    assert meta[0, 0, 0] == 0xED9C9C84
    # values keep ascending index order
    assert vals[0, 0] == np.float16(1.0) and vals[0, 1] == np.float16(-1.0)


def test_constant_patterns_literal_words():
    w = np.zeros((128, 64, 1, 1), np.float32)
    w[:, 2::4] = 1.0
    w[:, 3::4] = 2.0
    _, meta = c_pack(w)
    assert (meta == 0xEEEEEEEE).all()                  # (2,3) everywhere
    _, meta = c_pack(np.zeros((128, 64, 1, 1), np.float32))
    assert (meta == 0x44444444).all()                  # all-zero groups -> (0,1)


def test_tie_rule_fewer_than_two_nonzeros():
    w = np.zeros((128, 64, 1, 1), np.float32)
    w[0, 2] = 5.0          # group 0 of row 0: only position 2 -> (0,2) -> 0x8
    w[0, 4 + 0] = 3.0      # group 1: only position 0 -> (0,1) -> 0x4
    w[0, 8 + 3] = 1.0      # group 2: only position 3 -> (0,3) -> 0xC
    vals, meta = c_pack(w)
    assert meta[0, 0, 0] & 0xFFF == 0xC48
    assert vals[0, 0] == 0 and vals[0, 1] == np.float16(5.0)
    assert vals[0, 2] == np.float16(3.0) and vals[0, 3] == 0
    assert np.array_equal(meta, P.pack_meta(P.conv_weight_to_fk(w)))


def test_padding_rows_and_multi_tile():
    rng = np.random.default_rng(5)
    w = P.prune_conv_weight(rng.standard_normal((200, 64, 3, 3)).astype(np.float32))
    vals, meta = c_pack(w)
    assert vals.shape == (256, 288) and meta.shape == (2, 18, 128)
    assert (vals[200:] == 0).all()
    assert np.array_equal(meta, P.pack_meta(P.conv_weight_to_fk(w)))


def test_rejects_dense_group():
    w = np.zeros((128, 64, 1, 1), np.float32)
    w[3, 4:7] = 1.0        # three non-zeros in one group
    d = rt.make_desc(T=1, B=1, Cin=64, H=8, W=8, Cout=128, KH=1, KW=1)
    with pytest.raises(rt.SnnError) as e:
        rt.pack_weight_24(d, w)
    assert e.value.code == rt.SNN_E_NOT_24
    with pytest.raises(ValueError):
        P.pack_meta(P.conv_weight_to_fk(w))


@pytest.mark.parametrize("f, c, k", [(96, 64, 3), (192, 128, 3), (136, 192, 1)])
def test_dense_split_packer_bit_exact(f, c, k):
    """Dense weights (SNN_FLAG_DENSE): the C packer's two 2:4 halves per
    activation k-block equal the numpy restatement, zeros included, and the
    halves sum back to the fp16 dense weight."""
    from oracle.pack24 import conv_weight_to_fk, pack_dense_split, unpack
    rng = np.random.default_rng(f + c + k)
    w = rng.standard_normal((f, c, k, k)).astype(np.float32)
    w[0, :8] = 0.0                                    # whole zero groups keep their fixed pairs
    d = rt.make_desc(T=1, B=1, Cin=c, H=8, W=8, Cout=f, KH=k, KW=k, flags=rt.SNN_FLAG_DENSE)
    blob = rt.pack_weight_24(d, w)
    f_pad = -(-f // 128) * 128
    K = c * k * k
    vals, meta = split_blob(blob, f_pad, 2 * K)
    rv, rm = pack_dense_split(w)
    assert np.array_equal(vals.view(np.uint16), rv.view(np.uint16))
    assert np.array_equal(meta, rm)
    virt = unpack(vals, meta, f, 2 * K).reshape(f, K // 64, 2, 64)
    dense = conv_weight_to_fk(w).astype(np.float16).astype(np.float32).reshape(f, K // 64, 64)
    assert np.array_equal(virt.sum(axis=2), dense)


def test_dense_flag_doubles_weight_bytes_and_limits_k():
    d = rt.make_desc(T=1, B=1, Cin=128, H=8, W=8, Cout=128, KH=3, KW=3)
    dd = rt.make_desc(T=1, B=1, Cin=128, H=8, W=8, Cout=128, KH=3, KW=3, flags=rt.SNN_FLAG_DENSE)
    n1, n2 = rt.weight_bytes(d), rt.weight_bytes(dd)
    assert n2 == 2 * n1
    big = rt.make_desc(T=1, B=1, Cin=512, H=8, W=8, Cout=128, KH=3, KW=3, flags=rt.SNN_FLAG_DENSE)
    with pytest.raises(rt.SnnError):
        rt.weight_bytes(big)                          # 2 * 4608 > 8192 weight columns


@pytest.mark.parametrize("dense", [False, True], ids=["sparse", "dense"])
@pytest.mark.parametrize("c", [8, 48, 96, 200])
def test_partial_input_block_packs_zero_columns(c, dense):
    """Cin not a multiple of 64: the GEMM K is padded to whole 64-channel
    k-blocks, the padding columns carry zero weights (the activations there
    are TMA zero fill), and the blob equals the numpy restatement of the
    weight zero-padded to those channels."""
    rng = np.random.default_rng(c)
    w = rng.standard_normal((96, c, 3, 3)).astype(np.float32)
    if not dense:
        w = P.prune_conv_weight(w)
    flags = rt.SNN_FLAG_DENSE if dense else 0
    d = rt.make_desc(T=1, B=1, Cin=c, H=8, W=8, Cout=96, KH=3, KW=3, flags=flags)
    cp = -(-c // 64) * 64
    wp = np.zeros((96, cp, 3, 3), np.float32)
    wp[:, :c] = w
    dp = rt.make_desc(T=1, B=1, Cin=cp, H=8, W=8, Cout=96, KH=3, KW=3, flags=flags)
    assert rt.weight_bytes(d) == rt.weight_bytes(dp)
    assert np.array_equal(rt.pack_weight_24(d, w), rt.pack_weight_24(dp, wp))
    if not dense:
        vals, meta = split_blob(rt.pack_weight_24(d, w), 128, 9 * cp)
        wfk = P.conv_weight_to_fk(w)
        assert wfk.shape == (96, 9 * cp)
        assert np.array_equal(meta, P.pack_meta(wfk))
        assert np.array_equal(vals.view(np.uint16), P.pack_values(wfk).view(np.uint16))
