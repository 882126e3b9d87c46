import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

LAYER_CASES = ["c3s1", "c3s2", "c1s2", "c3res", "c3f64", "c3if", "lin"]
# Residual epilogues other than the SEW ADD (Add before the neuron; two
# neurons around the Add).
RES_CASES = ["c3addlif", "c1twon"]
RES_MODES = {0: "add_after", 1: "add_before", 2: "two_neuron"}
ATTN_CASES = ["n64", "n196", "n100h64"]


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def load_layer_case(name):
    g = dict(np.load(GOLDEN / f"layer_{name}.npz"))
    T, B, C, F, H, W, k, s, pad, islif, lin = (int(v) for v in g["meta"])
    g.update(T=T, B=B, C=C, F=F, H=H, W=W, k=k, stride=s, pad=pad,
             neuron="lif" if islif else "if", linear=bool(lin), res_mode="add_after",
             neuron2="lif")
    if "res_meta" in g:
        mode, lif2 = (int(v) for v in g["res_meta"])
        g.update(res_mode=RES_MODES[mode], neuron2="lif" if lif2 else "if",
                 residual=g["residual_f"])
    return g


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.skip(f"device sm_{major}{minor} is not sm_100")
    from sparsesnn_b200 import build
    build.build()
    return torch.device("cuda:0")


def load_attn_case(name):
    g = dict(np.load(GOLDEN / f"attn_{name}.npz"))
    T, B, N, heads, hd = (int(v) for v in g["meta"])
    g.update(T=T, B=B, N=N, heads=heads, hd=hd)
    return g
