"""GPU parity of the fused Spikformer attention core + attention LIF.

Spike products are integer counts, so the kernel's x is exact and its
spikes must equal the reference's bit for bit (golden fixtures from the
reference's fused op and model formulation, and the oracle at the
Spikformer-8-384 size)."""
import numpy as np
import pytest

from conftest import ATTN_CASES, load_attn_case
from oracle.attention import spikformer_attn_lif

pytestmark = pytest.mark.gpu

GUARD = 8192


def run_attn(q, k, v, *, T, heads, scale=0.125, tau=2.0, v_th=0.5, state=None, flags=0):
    import torch
    from sparsesnn_b200 import runtime as rt
    tb, n, c = q.shape
    dev = "cuda"
    qd, kd, vd = (torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev, torch.float16)
                  for a in (q, k, v))
    # Output followed by a guard tail of sentinels: the spike tiles' TMA
    # stores clip tokens past N at the tensor map's extent.
    n_out = tb * n * c
    buf = torch.full((n_out + GUARD,), 7.0, dtype=torch.float16, device=dev)
    out = buf[:n_out].view(tb, n, c)
    s = torch.cuda.current_stream().cuda_stream
    sp = state.data_ptr() if state is not None else None
    rt.check(rt.load().snn_spikformer_attn_forward(T, tb // T, n, heads, c // heads, scale, tau,
                                                   v_th, 0.0, flags, qd.data_ptr(), kd.data_ptr(),
                                                   vd.data_ptr(), sp, out.data_ptr(), s))
    torch.cuda.synchronize()
    assert bool((buf[n_out:] == 7.0).all()), "attention wrote past its output"
    return out.float().cpu().numpy()


@pytest.mark.parametrize("name", ATTN_CASES)
def test_golden_attention_exact(cuda_device, name):
    from sparsesnn_b200 import runtime as rt
    g = load_attn_case(name)
    y = run_attn(g["q"], g["k"], g["v"], T=g["T"], heads=g["heads"])
    assert rt.device_error() == 0
    assert np.array_equal(y, g["spikes"].astype(np.float32))


def test_state_chaining(cuda_device):
    """T=4 as two T=2 calls with the membrane carried in state equals one
    call; the final membrane equals the oracle's."""
    import torch
    from sparsesnn_b200 import runtime as rt
    g = load_attn_case("n196")
    T, B, N, heads = g["T"], g["B"], g["N"], g["heads"]
    C = g["q"].shape[-1]
    st = torch.zeros((B * N * C,), dtype=torch.float32, device="cuda")
    outs = []
    for half in range(2):
        sl = slice(half * 2 * B, (half + 1) * 2 * B)
        outs.append(run_attn(g["q"][sl], g["k"][sl], g["v"][sl], T=2, heads=heads, state=st,
                             flags=rt.SNN_FLAG_READ_STATE | rt.SNN_FLAG_WRITE_STATE))
    assert rt.device_error() == 0
    assert np.array_equal(np.concatenate(outs), g["spikes"].astype(np.float32))
    _, _, _, v_final = spikformer_attn_lif(g["q"], g["k"], g["v"], T=T, heads=heads)
    assert np.array_equal(st.cpu().numpy().reshape(B, N, C), v_final)


@pytest.mark.parametrize("tau, v_th", [(2.0, 0.5), (3.0, 0.3)], ids=["tau2", "tau3"])
def test_spikformer_8_384_full_size(cuda_device, tau, v_th):
    """Spikformer-8-384 on 224x224 (T=4, B=32, 196 tokens, 12 heads of 32)."""
    from sparsesnn_b200 import runtime as rt
    rng = np.random.default_rng(5)
    T, B, N, heads, hd = 4, 32, 196, 12, 32
    q, k, v = ((rng.random((T * B, N, heads * hd)) < 0.09).astype(np.float32) for _ in range(3))
    y = run_attn(q, k, v, T=T, heads=heads, tau=tau, v_th=v_th)
    assert rt.device_error() == 0
    ref, _, _, _ = spikformer_attn_lif(q, k, v, T=T, heads=heads, tau=tau, v_th=v_th)
    assert np.array_equal(y, ref)
    assert 0.05 < ref.mean() < 0.95


def test_single_token_and_small_heads(cuda_device):
    """Edge sizes: N = 1, N = 129 (a one-row second M-tile), N = 256, head_dim
    64, several 64-channel groups per image."""
    from sparsesnn_b200 import runtime as rt
    rng = np.random.default_rng(9)
    for N, hd, heads, p in ((1, 32, 2, 0.9), (129, 32, 4, 0.1), (33, 64, 3, 0.2),
                            (256, 64, 1, 0.06), (256, 32, 6, 0.06)):
        T, B = 2, 3
        q, k, v = ((rng.random((T * B, N, heads * hd)) < p).astype(np.float32) for _ in range(3))
        y = run_attn(q, k, v, T=T, heads=heads)
        assert rt.device_error() == 0
        ref, _, _, _ = spikformer_attn_lif(q, k, v, T=T, heads=heads)
        assert np.array_equal(y, ref), (N, hd)


def test_packed_qkv_layout(cuda_device):
    """SNN_FLAG_QKV_PACKED: q, k, v as the channel blocks of one
    [T*B][N][3C] tensor (a fused q|k|v Linear's output) give the same spikes
    as three separate tensors, at the Spikformer-8-384 size and an edge size."""
    import torch
    from sparsesnn_b200 import runtime as rt
    rng = np.random.default_rng(12)
    for T, B, N, heads, hd in ((4, 32, 196, 12, 32), (2, 3, 129, 3, 64)):
        C = heads * hd
        q, k, v = ((rng.random((T * B, N, C)) < 0.09).astype(np.float32) for _ in range(3))
        qkv = torch.from_numpy(np.concatenate([q, k, v], -1)).to("cuda", torch.float16)
        n_out = T * B * N * C
        buf = torch.full((n_out + GUARD,), 7.0, dtype=torch.float16, device="cuda")
        out = buf[:n_out]
        cb = C * 2
        rt.check(rt.load().snn_spikformer_attn_forward(
            T, B, N, heads, hd, 0.125, 2.0, 0.5, 0.0, rt.SNN_FLAG_QKV_PACKED, qkv.data_ptr(),
            qkv.data_ptr() + cb, qkv.data_ptr() + 2 * cb, None, out.data_ptr(),
            torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        assert rt.device_error() == 0
        assert bool((buf[n_out:] == 7.0).all()), "attention wrote past its output"
        ref, _, _, _ = spikformer_attn_lif(q, k, v, T=T, heads=heads)
        assert np.array_equal(out.float().cpu().numpy().reshape(T * B, N, C), ref), (N, hd)
