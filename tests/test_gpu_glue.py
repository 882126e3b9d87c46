"""GPU parity of the fused Add + neuron and MaxPool + neuron glue kernels.

Max pooling, fp16 + fp16 sums and the neuron update are exact in the kernel
and the oracle alike, so spikes and final membranes must match bit for bit."""
import numpy as np
import pytest

from conftest import GOLDEN
from oracle.glue import add_lif, maxpool_lif

pytestmark = pytest.mark.gpu


def nhwc(a):
    t, b, c, h, w = a.shape
    return np.ascontiguousarray(np.transpose(a, (0, 1, 3, 4, 2)).reshape(t * b, h, w, c))


def from_nhwc(y, T, B):
    tb, h, w, c = y.shape
    return np.transpose(y.reshape(T, B, h, w, c), (0, 1, 4, 2, 3))


def run(kind, x, b=None, *, k=3, s=2, pad=1, neuron="lif", tau=2.0, v_th=1.0, state0=None):
    import torch
    from sparsesnn_b200 import runtime as rt
    T, B, C, H, W = x.shape
    flags = rt.SNN_FLAG_WRITE_STATE | (rt.SNN_FLAG_READ_STATE if state0 is not None else 0)
    d = rt.make_desc(T=T, B=B, Cin=C, H=H, W=W, Cout=C, KH=k, KW=k, stride=s, pad=pad,
                     neuron=neuron, tau=tau, v_threshold=v_th, flags=flags)
    xd = torch.from_numpy(nhwc(x)).cuda().half()
    if kind == "pool":
        OH, OW = (H + 2 * pad - k) // s + 1, (W + 2 * pad - k) // s + 1
    else:
        OH, OW = H, W
    out = torch.full((T * B, OH, OW, C), 7.0, dtype=torch.float16, device="cuda")
    st = (torch.from_numpy(np.ascontiguousarray(np.transpose(state0, (0, 2, 3, 1)).reshape(-1, C)))
          .cuda().float() if state0 is not None
          else torch.zeros((B * OH * OW, C), device="cuda"))
    lib = rt.load()
    stream = torch.cuda.current_stream().cuda_stream
    if kind == "pool":
        rt.check(lib.snn_maxpool_lif_forward(d, xd.data_ptr(), st.data_ptr(), out.data_ptr(), stream))
    else:
        bd = torch.from_numpy(nhwc(b)).cuda().half()
        rt.check(lib.snn_add_lif_forward(d, xd.data_ptr(), bd.data_ptr(), st.data_ptr(),
                                         out.data_ptr(), stream))
    torch.cuda.synchronize()
    assert rt.device_error() == 0
    y = from_nhwc(out.float().cpu().numpy(), T, B)
    v = np.transpose(st.cpu().numpy().reshape(B, OH, OW, C), (0, 3, 1, 2))
    return y, v


def test_golden_glue(cuda_device):
    g = np.load(GOLDEN / "glue.npz")
    y, _ = run("pool", g["x"])
    assert np.array_equal(y, g["s_pool"].astype(np.float32))
    y, _ = run("add", g["a"], g["b"])
    assert np.array_equal(y, g["s_add"].astype(np.float32))
    y, _ = run("add", g["a"], g["b"], neuron="if")
    assert np.array_equal(y, g["s_add_if"].astype(np.float32))


@pytest.mark.parametrize("k, s, pad, H, W", [(3, 2, 1, 16, 16), (2, 2, 0, 7, 9), (3, 1, 1, 5, 6),
                                             (1, 1, 0, 4, 4)])
@pytest.mark.parametrize("neuron, tau", [("lif", 2.0), ("lif", 3.0), ("if", 2.0)])
def test_maxpool_lif_vs_oracle(cuda_device, k, s, pad, H, W, neuron, tau):
    rng = np.random.default_rng(k * 100 + H)
    T, B, C = 3, 2, 72
    x = (rng.standard_normal((T, B, C, H, W)) * 1.5).astype(np.float16).astype(np.float32)
    v0 = (rng.standard_normal((B, C, (H + 2 * pad - k) // s + 1, (W + 2 * pad - k) // s + 1)) * 0.3
          ).astype(np.float32)
    y, v = run("pool", x, k=k, s=s, pad=pad, neuron=neuron, tau=tau, state0=v0)
    ref, _, rv = maxpool_lif(x, k, s, pad, neuron=neuron, tau=tau, v0=v0)
    assert np.array_equal(y, ref)
    assert np.array_equal(v, rv)


@pytest.mark.parametrize("neuron, tau, v_th", [("lif", 2.0, 1.0), ("lif", 1.5, 0.7), ("if", 2.0, 1.0)])
def test_add_lif_vs_oracle(cuda_device, neuron, tau, v_th):
    rng = np.random.default_rng(3)
    T, B, C, H, W = 4, 3, 128, 5, 7
    a = rng.standard_normal((T, B, C, H, W)).astype(np.float16).astype(np.float32)
    b = rng.integers(0, 3, (T, B, C, H, W)).astype(np.float32)
    y, v = run("add", a, b, neuron=neuron, tau=tau, v_th=v_th)
    ref, _, rv = add_lif(a, b, neuron=neuron, tau=tau, v_th=v_th)
    assert np.array_equal(y, ref)
    assert np.array_equal(v, rv)


@pytest.mark.parametrize("k, s, pad, H, W, C", [(3, 2, 1, 17, 23, 48), (2, 2, 0, 8, 6, 32),
                                                (3, 1, 1, 5, 7, 16), (1, 1, 0, 3, 4, 64)])
def test_maxpool_of_bit_packed_spikes(cuda_device, k, s, pad, H, W, C):
    """SNN_FLAG_SPIKE_BITS: the plain max pool of bit-packed spikes
    ([T*B][H][W][C/8] bytes, channel c in bit c%8 of byte c/8) equals the
    pool of the same spikes as fp16, bit for bit, and writes nothing past
    its output."""
    import torch
    from sparsesnn_b200 import runtime as rt
    rng = np.random.default_rng(k * 1000 + H * 10 + C)
    T, B = 3, 2
    x = (rng.random((T, B, C, H, W)) < 0.2).astype(np.float32)
    ref, _ = run("pool", x, k=k, s=s, pad=pad, neuron="none")
    packed = np.packbits(nhwc(x).astype(np.uint8), axis=-1, bitorder="little")
    d = rt.make_desc(T=T, B=B, Cin=C, H=H, W=W, Cout=C, KH=k, KW=k, stride=s, pad=pad,
                     neuron="none", flags=rt.SNN_FLAG_SPIKE_BITS)
    OH, OW = (H + 2 * pad - k) // s + 1, (W + 2 * pad - k) // s + 1
    n_out = T * B * OH * OW * C
    buf = torch.full((n_out + 4096,), 7.0, dtype=torch.float16, device="cuda")
    src = torch.from_numpy(packed).cuda()
    lib = rt.load()
    rt.check(lib.snn_maxpool_lif_forward(d, src.data_ptr(), None, buf.data_ptr(),
                                         torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert rt.device_error() == 0
    assert bool((buf[n_out:] == 7.0).all()), "bit-packed pool wrote past its output"
    y = from_nhwc(buf[:n_out].float().cpu().numpy().reshape(T * B, OH, OW, C), T, B)
    assert np.array_equal(y, ref)
    assert 0.1 < y.mean() < 0.95
