"""SEW-ResNet-18 (T=4, CIFAR 32x32, batch 128 per GPU) inference throughput.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One process per GPU (torchrun for N > 1), one model replica per GPU, batch 128
per GPU (weak scaling), NCCL all-gather of the logits after every forward (the
only collective, as in the data-parallel design), pipelined on a side stream
under the next forward.  Prints ONE JSON line on rank 0.

* A step is ``--batches-per-step`` (default 100) forwards of one batch of 128
  images each, so that K steps span about a second of device time.
* value: images/s of the whole job, inputs resident in HBM, each forward one
  CUDA-graph replay, timed with CUDA events between barriers, max over ranks.
* e2e: the same through the C-ABI native executor (``snn_engine_run`` on an
  engine file saved from the replica) with the images copied from pinned host
  memory and the logits read back to host every forward; ``python_driver`` is
  the same measurement through the Python call ``model(x_host)``.
* roofline: the fused sparse conv kernels (19 launches per forward): their
  share of the forward measured INSIDE a CUDA graph (timing-event nodes
  between launches), applied to the timed forward; FLOPs are
  dense-equivalent 2*M*N*K.  ``layers`` gives every launch's time and its
  fraction of the tensor ceiling and of HBM.
* strong_scaling: the same forward at a fixed global batch (``--global-batch``,
  default 128) split over the ranks.
* cpu_baseline (rank 0, N = 1): the CPU port of the reference PyTorch path
  (``oracle/sew_resnet.py``) on a bounded sample of images, all host threads.
* --impl reference: only that CPU path, as the reference arm.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "SEW-ResNet-18 T=4 images/s"
UNIT = "images/s"
BATCH = 128
T_STEPS = 4
HW = 32
CPU_SAMPLE = 64          # images per CPU-baseline forward


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=BATCH)
    ap.add_argument("--batches-per-step", type=int, default=100)
    ap.add_argument("--global-batch", type=int, default=BATCH)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the Spikformer / MS-ResNet / DVS configurations")
    ap.add_argument("--profile-config", default=None,
                    help="only run eager forwards of one configuration (sew_resnet18, "
                         "spikformer_8_384, msresnet34, dvs_sew_resnet18) at --batch, for a "
                         "profiler; prints nothing")
    ap.add_argument("--cpu-steps", type=int, default=5)
    return ap.parse_args()


def config(args, world):
    return {"workload": f"SEW-ResNet-18 CIFAR stem (3x3 s1, no maxpool), stages 64/128/256/512, "
                        f"ADD, 100 classes, T={T_STEPS}, 3x{HW}x{HW}, batch {args.batch} per GPU",
            "model": "sew_resnet18_cifar", "global_batch": args.batch * world,
            "forwards_per_step": args.batches_per_step,
            "seq_len": T_STEPS, "parallelism": f"dp{world}",
            "weights": "random init (Kaiming, BN stats as config 0), 2:4 pruned except stem",
            "l2": "working set per step > 126 MB L2 (activations ~600 MB), no flush"}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


def spikformer_linear_layers(dev, stream, sparse_peak, iters=10):
    """The Linear + BN + LIF twin at Spikformer-8-384 shapes (T=4, batch 32,
    196 tokens: 6272 rows per timestep; one of q/k/v and proj 384->384, the
    fused q|k|v layer the model runs 384->1152, fc1 384->1536, fc2
    1536->384), random 2:4 weights and Bernoulli(0.2) spikes: per-layer
    CUDA-event time and dense-equivalent TFLOP/s against the 2:4 ceiling."""
    import numpy as np
    import torch
    from sparsesnn_b200.layer import SparseConvBNLIF
    from sparsesnn_b200.pruning import prune_2_4_last
    T, rows = 4, 32 * 196
    out = {}
    for name, cin, cout in (("q", 384, 384), ("qkv_fused", 384, 1152), ("fc1", 384, 1536),
                            ("fc2", 1536, 384)):
        rng = np.random.default_rng(0)
        w = prune_2_4_last(rng.standard_normal((cout, cin)).astype(np.float32) * (2.0 / cin) ** 0.5)
        layer = SparseConvBNLIF(w, np.ones(cout, np.float32), np.zeros(cout, np.float32),
                                T=T, B=1, H=1, W=rows, device=dev)
        x = (torch.rand((T, 1, rows, cin), device=dev) < 0.2).half()
        y = torch.empty((T, 1, rows, cout), dtype=torch.float16, device=dev)
        for _ in range(3):
            layer(x, out=y)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(iters):
            layer(x, out=y)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / iters
        tflops = 2.0 * T * rows * cin * cout / (ms / 1000.0) / 1e12
        out[name] = {"us": round(ms * 1000.0, 2), "tflops": round(tflops, 1),
                     "frac": round(tflops / sparse_peak, 4), "rows": T * rows, "cin": cin, "cout": cout}
    return out


def spikformer_attention(dev, stream, hbm_peak, iters=12, sets=4):
    """The fused attention core + attention LIF at the Spikformer-8-384 shape
    (T=4, batch 32, 196 tokens, 12 heads of 32) on Bernoulli(0.09) q/k/v
    spikes: CUDA-event time per call, rotating over `sets` input sets
    (together larger than L2), and HBM throughput of the algorithmic bytes
    (q, k, v read once, spikes written once, fp16)."""
    import torch
    from sparsesnn_b200 import runtime as rt
    T, B, N, heads, hd = 4, 32, 196, 12, 32
    C = heads * hd
    lib = rt.load()
    ins = [[(torch.rand((T * B, N, C), device=dev) < 0.09).half() for _ in range(3)]
           for _ in range(sets)]
    out = torch.empty((T * B, N, C), dtype=torch.float16, device=dev)
    s = stream.cuda_stream

    def call(i):
        q, k, v = ins[i % sets]
        rt.check(lib.snn_spikformer_attn_forward(T, B, N, heads, hd, 0.125, 2.0, 0.5, 0.0, 0,
                                                 q.data_ptr(), k.data_ptr(), v.data_ptr(), None,
                                                 out.data_ptr(), s))
    for i in range(3):
        call(i)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for i in range(iters):
        call(i)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / iters
    nbytes = 4 * T * B * N * C * 2
    gbs = nbytes / (ms / 1000.0) / 1e9
    return {"us": round(ms * 1000.0, 2), "GB/s": round(gbs, 1), "frac": round(gbs / hbm_peak, 4),
            "bytes": nbytes, "shape": {"T": T, "B": B, "N": N, "heads": heads, "head_dim": hd},
            "l2": f"{sets} input sets rotated"}


def glue_kernels(dev, stream, hbm_peak, iters=10):
    """The fused MaxPool + LIF (SEW/MS-ResNet ImageNet stem shape: T=4, batch
    32, 64 channels, 112x112 -> 56x56, 3x3 s2 p1) and Add + LIF (T=4, batch
    128, 64 channels, 32x32) kernels: CUDA-event time per call and HBM
    throughput of the algorithmic bytes (inputs read once, spikes written
    once; every buffer set is larger than L2 or rotated)."""
    import torch
    from sparsesnn_b200 import runtime as rt
    lib = rt.load()
    s = stream.cuda_stream
    res = {}
    T, B, C, H = 4, 32, 64, 112
    d = rt.make_desc(T=T, B=B, Cin=C, H=H, W=H, Cout=C, KH=3, KW=3, stride=2, pad=1)
    x = torch.randn((T * B, H, H, C), device=dev).half()
    y = torch.empty((T * B, H // 2, H // 2, C), dtype=torch.float16, device=dev)
    nbytes = x.numel() * 2 + y.numel() * 2
    runs = {"maxpool_lif": (lambda: rt.check(lib.snn_maxpool_lif_forward(d, x.data_ptr(), None,
                                                                         y.data_ptr(), s)), nbytes)}
    T2, B2, H2 = 4, 128, 32
    d2 = rt.make_desc(T=T2, B=B2, Cin=C, H=H2, W=H2, Cout=C, KH=1, KW=1)
    ab = [[torch.randn((T2 * B2, H2, H2, C), device=dev).half() for _ in range(2)] for _ in range(2)]
    z = torch.empty((T2 * B2, H2, H2, C), dtype=torch.float16, device=dev)
    cnt = [0]

    def add_call():
        a, b = ab[cnt[0] % 2]
        cnt[0] += 1
        rt.check(lib.snn_add_lif_forward(d2, a.data_ptr(), b.data_ptr(), None, z.data_ptr(), s))
    runs["add_lif"] = (add_call, 3 * z.numel() * 2)
    for name, (fn, nb) in runs.items():
        for _ in range(3):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(iters):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / iters
        gbs = nb / (ms / 1000.0) / 1e9
        res[name] = {"us": round(ms * 1000.0, 2), "GB/s": round(gbs, 1),
                     "frac": round(gbs / hbm_peak, 4), "bytes": nb}
    return res


def cpu_reference_images_per_s(steps, sample, threads, warmup=1):
    """Time the oracle's port of the reference PyTorch forward on CPU."""
    import torch
    from oracle.sew_resnet import forward_torch, make_input
    from sparsesnn_b200.sew_resnet import init_params
    torch.set_num_threads(threads)
    P = init_params(seed=0)
    x = make_input(seed=0, B=sample)
    for _ in range(warmup):
        forward_torch(P, x, T=T_STEPS)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        forward_torch(P, x, T=T_STEPS)
        times.append(time.perf_counter() - t0)
    return sample / (sum(times) / len(times)), times


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        # nvidia-smi indices are physical and ignore CUDA_VISIBLE_DEVICES:
        # select the GPU by its UUID.
        import torch
        self.gpu = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu, f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in (self.out or "").splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1])); mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def run_reference(args, rank):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    ips, times = cpu_reference_images_per_s(max(1, args.steps), CPU_SAMPLE, threads,
                                            warmup=max(1, args.warmup))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    line = {"impl": "reference", "metric": METRIC, "value": ips, "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000.0 * sum(times) / len(times), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config(args, world),
            "cpu_baseline": {"value": ips, "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"{CPU_SAMPLE} images per step, torch CPU fp32 port of "
                                       f"the reference forward (oracle/sew_resnet.py)"},
            "e2e": {"value": ips, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit(line)


def segment_times(model, stream, replays=50):
    """Per-launch device time of one forward INSIDE a CUDA graph: the forward
    is captured with a timing event (an event-record node) between every two
    launches and replayed; returns ({launch name: mean ms}, total ms).  The
    event nodes cut the programmatic-dependent-launch overlap between
    neighbours, so the segments sum to a little more than the plain graph's
    step; shares are what this measures."""
    import torch
    ops = model.launches()
    evs = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(len(ops) + 1)]
    g = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(model.device)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        model._in_sel = 0
        with torch.cuda.graph(g):
            evs[0].record()
            for (_, op), e in zip(ops, evs[1:]):
                op()
                e.record()
    stream.wait_stream(side)
    acc = [0.0] * len(ops)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    for _ in range(replays):
        g.replay()
        torch.cuda.synchronize()
        for i in range(len(ops)):
            acc[i] += evs[i].elapsed_time(evs[i + 1])
    del g
    per = {name: a / replays for (name, _), a in zip(ops, acc)}
    return per, sum(per.values())


# The other configurations of the benchmark (one replica per GPU each), built
# on the node-plan drivers; measured after the headline and reported under
# "configs".  (name, per-GPU batch, T, builder, CPU-baseline forward)
def _other_configs():
    def dvs(dev, batch):
        from sparsesnn_b200.sew_resnet import SEWResNet18DVS, init_params
        P = init_params(seed=0, num_classes=11, in_channels=2, stem_kernel=7, input_moment=0.05)
        m = SEWResNet18DVS(P, T=16, batch=batch, H=128, W=128, device=dev)
        return m, P

    def msr(dev, batch):
        from sparsesnn_b200.ms_resnet import MSResNet34, init_params
        P = init_params(seed=0)
        return MSResNet34(P, T=4, batch=batch, H=224, W=224, device=dev), P

    def spk(dev, batch):
        from sparsesnn_b200.spikformer import Spikformer, init_params
        P = init_params(seed=0)
        return Spikformer(P, T=4, batch=batch, H=224, W=224, device=dev), P

    def cpu_dvs(P, n):
        from oracle.sew_resnet import forward_torch, make_dvs_input
        x = make_dvs_input(seed=0, B=n, T=16)
        return lambda: forward_torch(P, x, T=16, stem_stride=2, maxpool=True)

    def cpu_msr(P, n):
        from oracle.ms_resnet import forward_torch, make_input
        x = make_input(seed=0, B=n)
        return lambda: forward_torch(P, x, T=4)

    def cpu_spk(P, n):
        from oracle.spikformer import forward_torch, make_input
        x = make_input(seed=0, B=n)
        return lambda: forward_torch(P, x, T=4)

    return [
        ("spikformer_8_384", 32, 4, spk, cpu_spk,
         "Spikformer-8-384: SPS with a stride-2 pool after each of 4 stages (224x224 -> 14x14 "
         "tokens), 8 blocks, 12 heads, MLP ratio 4, T=4, 3x224x224, 1000 classes; Linear weights "
         "2:4, SPS convs dense"),
        ("msresnet34", 64, 4, msr, cpu_msr,
         "MS-ResNet-34 (LIF -> conv -> BN, membrane shortcut; [3,4,6,3], 64/128/256/512), T=4, "
         "3x224x224, 1000 classes; non-stem convs 2:4"),
        ("dvs_sew_resnet18", 4, 16, dvs, cpu_dvs,
         "DVS SEW-ResNet-18 (7x7/2 stem + MaxPool(3,2,1) on 2x128x128 Bernoulli(0.05) event "
         "frames, ADD), T=16, 11 classes, 4 per GPU (batch 32 at 8 GPUs); non-stem convs 2:4"),
    ]


def measure_config(name, batch, T, build, cpu_fn, workload, *, dev, stream, world, rank,
                   sparse_peak, dense_peak, forwards, cpu, threads):
    """One configuration: device-resident forwards (graph replays, logits
    gathered on a side stream at N > 1), the same through the public call
    with host images, per-launch time inside the graph, the conv layers'
    fraction of their tensor-core ceilings, and (rank 0, N = 1) a bounded CPU
    sample of the reference path."""
    import torch
    from sparsesnn_b200 import dist as sd
    from sparsesnn_b200.netplan import CONV, conv_flops
    model, P = build(dev, batch)
    g = torch.Generator().manual_seed(77 + rank)
    if name == "dvs_sew_resnet18":
        x_host = (torch.rand(model.in_shape, generator=g) < 0.05).float().pin_memory()
    else:
        x_host = torch.randn(model.in_shape, generator=g).pin_memory()
    for k in range(2):
        model.x_ins[k].copy_(x_host.to(dev))
    model.run()
    model.capture(warmup=2)
    gath = sd.OverlappedGather(tuple(model.logits.shape), world, dev) if world > 1 else None

    def fw(n, public=False):
        for i in range(n):
            if gath is not None:
                gath.reuse(i & 1)
            out = model(x_host) if public else model.replay(i & 1)
            if gath is not None:
                gath.submit(out, i & 1)
        if gath is not None:
            gath.drain()

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    res = {"workload": workload, "per_gpu_batch": batch, "global_batch": batch * world, "T": T}
    for public in (False, True):
        fw(3, public)
        if world > 1:
            torch.distributed.barrier(device_ids=[dev.index])
        torch.cuda.synchronize()
        e0.record(stream)
        fw(forwards, public)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = sd.max_over_ranks(e0.elapsed_time(e1) / forwards, device=dev)
        if public:
            py_e2e = batch * world / (ms / 1000.0)
        else:
            res.update(value=batch * world / (ms / 1000.0), unit=UNIT, ms_per_forward=ms)
    # End to end through the C-ABI executor, as for the headline: an engine
    # file saved from this plan, snn_engine_run with the pinned host images
    # (H2D inside the call) and the logits read back to pinned host memory.
    import os
    import tempfile
    from sparsesnn_b200 import engine_file as ef
    eng_dir = tempfile.mkdtemp()
    eng_path = os.path.join(eng_dir, f"{name}_rank{rank}.snne")
    ef.save_engine(model, eng_path)
    eng = ef.Engine(eng_path)
    logits_host = torch.empty(tuple(model.logits.shape), dtype=torch.float32).pin_memory()
    eng_logits = [torch.empty_like(model.logits) for _ in range(2)]

    def eng_fw(n):
        for i in range(n):
            k = i & 1
            if gath is None:
                eng.run(x_host.data_ptr(), logits_host.data_ptr(), es)
                continue
            gath.reuse(k)
            eng.run(x_host.data_ptr(), eng_logits[k].data_ptr(), es)
            gath.submit(eng_logits[k], k)
            logits_host.copy_(eng_logits[k], non_blocking=True)
        if gath is not None:
            gath.drain()

    es = torch.cuda.Stream(dev)                          # capture needs a non-default stream
    with torch.cuda.stream(es):
        eng.capture(es)
        eng_fw(3)
        if world > 1:
            torch.distributed.barrier(device_ids=[dev.index])
        torch.cuda.synchronize()
        e0.record(es)
        eng_fw(forwards)
        e1.record(es)
        torch.cuda.synchronize()
    ms = sd.max_over_ranks(e0.elapsed_time(e1) / forwards, device=dev)
    eng.close()
    os.remove(eng_path)
    os.rmdir(eng_dir)
    res["e2e"] = {"value": batch * world / (ms / 1000.0), "unit": UNIT,
                  "path": "snn_engine_run (C-ABI executor, CUDA graph): pinned H2D of the images "
                          "and D2H of the logits in every call",
                  "h2d_bytes_per_forward": int(x_host.numel() * 4),
                  "d2h_bytes_per_forward": int(logits_host.numel() * 4),
                  "python_driver": py_e2e}
    per_launch, seg_total = segment_times(model, stream, replays=20)
    scale_t = res["ms_per_forward"] / seg_total
    busy, conv_ms, n_conv = 0.0, 0.0, 0
    for n in model.nodes:
        if n.kind != CONV:
            continue
        t_s = per_launch[n.name] * scale_t / 1000.0
        peak = dense_peak if n.layer.dense else sparse_peak
        busy += conv_flops(n.layer) / (peak * 1e12)
        conv_ms += t_s * 1000.0
        n_conv += 1
    res["roofline"] = {"bound": "tensor", "frac": busy / (conv_ms / 1000.0), "unit": "TFLOP/s",
                       "conv_launches": n_conv, "conv_ms_per_forward": conv_ms,
                       "conv_share": conv_ms / res["ms_per_forward"],
                       "note": "sum over fused conv launches of FLOPs / ceiling (2:4 sparse ceiling "
                               "for 2:4 layers, dense bf16 peak for dense ones) over their time "
                               "inside the graph"}
    res["launches"] = {k: round(v * scale_t * 1000.0, 2) for k, v in per_launch.items()}
    if cpu and rank == 0 and world == 1:
        import time
        torch.set_num_threads(threads)
        f = cpu_fn(P, 1)
        f()
        t0 = time.perf_counter()
        f()
        dt = time.perf_counter() - t0
        res["cpu_baseline"] = {"value": 1.0 / dt, "unit": UNIT, "cores": threads, "kind": "port",
                               "sample": "1 image x 1 forward (after one warm-up), torch CPU fp32 "
                                         "port of the reference forward (oracle/)"}
    del model
    torch.cuda.empty_cache()
    return res


def profile_config(args):
    """Eager forwards of one configuration on cuda:0 at ``--batch`` images
    (``--warmup`` + ``--steps`` forwards), for ncu captures of its kernels."""
    import torch
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if args.profile_config == "sew_resnet18":
        from sparsesnn_b200.sew_resnet import SEWResNet18, init_params
        model = SEWResNet18(init_params(seed=0), T=T_STEPS, batch=args.batch, H=HW, W=HW, device=dev)
    else:
        build = {c[0]: c[3] for c in _other_configs()}[args.profile_config]
        model, _ = build(dev, args.batch)
    for k in range(2):
        shape = model.x_ins[k].shape
        if args.profile_config == "dvs_sew_resnet18":
            model.x_ins[k].copy_((torch.rand(shape, device=dev) < 0.05).float())
        else:
            model.x_ins[k].copy_(torch.randn(shape, device=dev))
    for _ in range(args.warmup + args.steps):
        model.run()
    torch.cuda.synchronize()
    from sparsesnn_b200 import runtime as rt
    if rt.device_error() != 0:
        raise RuntimeError("a kernel reported a device error")


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from sparsesnn_b200 import dist as sd
    from sparsesnn_b200.sew_resnet import SEWResNet18, conv_layer_bytes, conv_layer_flops, init_params

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    R = args.batches_per_step
    P = init_params(seed=0)
    model = SEWResNet18(P, T=T_STEPS, batch=args.batch, H=HW, W=HW, device=dev)
    g = torch.Generator().manual_seed(1234 + rank)
    x_host = torch.randn((args.batch, 3, HW, HW), generator=g).pin_memory()
    x_dev = x_host.to(dev)
    logits_host = torch.empty((args.batch, model.num_classes), dtype=torch.float32).pin_memory()
    gath = sd.OverlappedGather(tuple(model.logits.shape), world, dev) if world > 1 else None

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    # Warm-up (eager), then capture the forward into CUDA graphs (one per
    # input buffer; both buffers hold this rank's resident batch).
    for k in range(2):
        model.x_ins[k].copy_(x_dev)
    for _ in range(max(3, args.warmup)):
        model.run()
    torch.cuda.synchronize()
    model.capture(warmup=1)
    stream = torch.cuda.current_stream(dev)

    def forwards(n):
        """n forwards on the resident batch, alternating the two graphs; at
        N > 1 each forward's logits are gathered on a side stream under the
        next forward."""
        for i in range(n):
            k = i & 1
            if gath is not None:
                gath.reuse(k)
            out = model.replay(k)
            if gath is not None:
                gath.submit(out, k)
        if gath is not None:
            gath.drain()

    for _ in range(max(3, args.warmup)):
        forwards(R)
    torch.cuda.synchronize()
    n_launch = len(model.launches())

    # ---------------- timed region A: device-resident inputs, graph replay
    # A step is R forwards of one batch each.  The clock sampler runs across
    # the timed region plus a second of identical replays before it.
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clk:
        forwards(2 * R)
        torch.cuda.synchronize()
        barrier(); torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            forwards(R)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
    ms = sd.max_over_ranks(e0.elapsed_time(e1) / args.steps, device=dev)
    value = args.batch * R * world / (ms / 1000.0)

    # ---------------- timed region B: end to end through the Python call
    def e2e_forwards(n):
        for i in range(n):
            if gath is not None:
                gath.reuse(i & 1)
            out = model(x_host)                          # H2D from pinned memory + replay
            if gath is not None:
                gath.submit(out, i & 1)
            logits_host.copy_(out, non_blocking=True)    # D2H of the forward's result
        if gath is not None:
            gath.drain()

    e2e_forwards(4)
    barrier(); torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.steps):
        e2e_forwards(R)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms_e2e = sd.max_over_ranks(e0.elapsed_time(e1) / args.steps, device=dev)
    e2e_driver = args.batch * R * world / (ms_e2e / 1000.0)

    # ---------------- timed region C: the native executor through the C-ABI
    # (snn_engine_run: pinned host images in, logits out, the C++ node loop
    # replayed from its CUDA graph), on an engine file saved from the same
    # replica.
    import tempfile
    from sparsesnn_b200 import engine_file as ef
    eng_dir = tempfile.mkdtemp()
    eng_path = os.path.join(eng_dir, f"sew18_rank{rank}.snne")
    ef.save_engine(model, eng_path)
    eng = ef.Engine(eng_path)
    eng_logits = [torch.empty_like(model.logits) for _ in range(2)]
    es = torch.cuda.Stream(dev)

    def eng_forwards(n):
        for i in range(n):
            k = i & 1
            if gath is None:
                # H2D of the images, graph replay, D2H of the logits into pinned host memory
                eng.run(x_host.data_ptr(), logits_host.data_ptr(), es)
                continue
            gath.reuse(k)
            eng.run(x_host.data_ptr(), eng_logits[k].data_ptr(), es)   # H2D + graph replay
            gath.submit(eng_logits[k], k)
            logits_host.copy_(eng_logits[k], non_blocking=True)        # D2H of the result
        if gath is not None:
            gath.drain()

    with torch.cuda.stream(es):
        eng.capture(es)
        eng_forwards(max(3, args.warmup))
        es.synchronize()
        barrier()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(es)
        for _ in range(args.steps):
            eng_forwards(R)
        c1.record(es)
        es.synchronize()
    barrier()
    ms_eng = sd.max_over_ranks(c0.elapsed_time(c1) / args.steps, device=dev)
    e2e = args.batch * R * world / (ms_eng / 1000.0)
    eng.close()
    os.remove(eng_path)
    os.rmdir(eng_dir)

    # ---------------- strong scaling: a fixed global batch split over ranks
    strong = None
    if args.global_batch % world == 0:
        per = args.global_batch // world
        sm_model = model if per == args.batch else SEWResNet18(P, T=T_STEPS, batch=per, H=HW, W=HW,
                                                               device=dev)
        for k in range(2):
            sm_model.x_ins[k].copy_(x_dev[:per])
        if sm_model is not model:
            sm_model.capture(warmup=2)
        sg = sd.OverlappedGather(tuple(sm_model.logits.shape), world, dev) if world > 1 else None

        def sm_forwards(n):
            for i in range(n):
                if sg is not None:
                    sg.reuse(i & 1)
                out = sm_model.replay(i & 1)
                if sg is not None:
                    sg.submit(out, i & 1)
            if sg is not None:
                sg.drain()

        sm_forwards(R)
        barrier(); torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            sm_forwards(R)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        ms_s = sd.max_over_ranks(e0.elapsed_time(e1) / args.steps, device=dev)
        strong = {"global_batch": args.global_batch, "per_gpu_batch": per,
                  "ms_per_step": ms_s, "forwards_per_step": R,
                  "value": args.global_batch * R / (ms_s / 1000.0), "unit": UNIT}
        if sm_model is not model:
            del sm_model

    # ---------------- roofline: per-launch time inside the graph
    per_launch, seg_total = segment_times(model, stream)
    conv_names = [n for n, _ in model.launches() if n not in ("stem", "head")]
    conv_share = sum(per_launch[n] for n in conv_names) / seg_total
    ms_fwd = ms / R                                  # one forward of the timed region
    conv_ms = ms_fwd * conv_share                    # the conv launches' part of it
    layers = list(model.conv_layers())
    flops = sum(conv_layer_flops(l) for l in layers)
    hbm_peak, bf16_peak, peak_kind = peaks()
    sparse_peak = 2.0 * bf16_peak
    achieved = flops / (conv_ms / 1000.0) / 1e12
    traffic = None
    tf = ROOT / "profiles" / "sew18_traffic.txt"
    if tf.exists():
        for line in tf.read_text().splitlines():
            if line.startswith("fused_conv_dram_bytes_per_forward:"):
                traffic = int(float(line.split(":")[1]))
    # Per conv launch: time = its graph segment scaled so the segments sum to
    # the timed forward; fractions of the 2:4 tensor ceiling and of HBM, the
    # latter for the bytes the fp16 format moves and for the byte convention
    # of 1-byte activations / 1-bit spikes.
    scale_t = ms_fwd / seg_total
    per_layer = {}
    res_of = {}
    for i, blk in enumerate(model.blocks):
        res_of[f"b{i}.conv1"] = (blk["l1"], False)
        if blk["ds"] is not None:
            res_of[f"b{i}.ds"] = (blk["ds"], False)
        res_of[f"b{i}.conv2"] = (blk["l2"], True)
    for name, t_ms in per_launch.items():
        ent = {"us": round(t_ms * scale_t * 1000.0, 2)}
        if name in res_of:
            layer, has_res = res_of[name]
            t_s = t_ms * scale_t / 1000.0
            fl = conv_layer_flops(layer)
            b16 = conv_layer_bytes(layer, has_res)
            b8 = conv_layer_bytes(layer, has_res, act_bytes=1, binary_out=not has_res)
            from sparsesnn_b200 import runtime as rt
            ent.update(variant={0: "general", 1: "halo", 2: "halo_stream"}[rt.variant(layer.desc)],
                       tflops=round(fl / t_s / 1e12, 1), frac_tensor=round(fl / t_s / 1e12 / sparse_peak, 4),
                       frac_hbm_f16=round(b16 / t_s / 1e9 / hbm_peak, 4),
                       frac_hbm_s8d=round(b8 / t_s / 1e9 / hbm_peak, 4))
        per_layer[name] = ent
    alg_bytes = sum(conv_layer_bytes(*res_of[n]) for n in conv_names)
    from sparsesnn_b200 import runtime as rt
    if rt.device_error() != 0:
        raise RuntimeError("fused kernel reported a device error")

    linear = spikformer_linear_layers(dev, stream, sparse_peak) if rank == 0 else None
    attn = spikformer_attention(dev, stream, hbm_peak) if rank == 0 else None
    glue = glue_kernels(dev, stream, hbm_peak) if rank == 0 else None
    if rt.device_error() != 0:
        raise RuntimeError("a kernel reported a device error")

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        ips, _ = cpu_reference_images_per_s(args.cpu_steps, CPU_SAMPLE, threads)
        cpu = {"value": ips, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{CPU_SAMPLE} images x {args.cpu_steps} forwards (after one warm-up), "
                         f"torch CPU fp32 port of the reference forward (oracle/sew_resnet.py)"}
    others = {}
    if not args.no_configs:
        for name, batch, T, build, cpu_fn, workload in _other_configs():
            others[name] = measure_config(
                name, batch, T, build, cpu_fn, workload, dev=dev, stream=stream, world=world,
                rank=rank, sparse_peak=sparse_peak, dense_peak=bf16_peak, forwards=20,
                cpu=not args.no_cpu_baseline, threads=os.cpu_count() or 1)
        if rt.device_error() != 0:
            raise RuntimeError("a kernel reported a device error")
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "f16", "data": "synthetic", "config": config(args, world),
                "e2e": {"value": e2e, "unit": UNIT,
                        "h2d_bytes_per_step": int(x_host.numel() * 4) * R,
                        "d2h_bytes_per_step": int(logits_host.numel() * 4) * R,
                        "path": "snn_engine_run (C-ABI native executor, CUDA graph), pinned host buffers",
                        "python_driver": e2e_driver},
                "gpu_launches": n_launch * args.steps * R,
                "roofline": {"bound": "tensor", "achieved": achieved, "peak": sparse_peak,
                             "unit": "TFLOP/s", "frac": achieved / sparse_peak,
                             "traffic": traffic,
                             "kernel": "fused sparse conv+BN+LIF kernels, 19 launches/forward "
                                       "(halo4 x4, halo x3, halo_stream x6, general x6)",
                             "peak_note": f"2:4 sparse ceiling = 2 x {peak_kind} dense bf16 "
                                          f"{bf16_peak} TFLOP/s; FLOPs dense-equivalent",
                             "timing": "conv launches' share of the forward, measured inside the "
                                       "CUDA graph (event-record nodes between launches), times the "
                                       "timed forward (ms_per_step / forwards per step)",
                             "flops_per_forward": flops, "kernel_ms_per_forward": conv_ms,
                             "forward_ms": ms_fwd, "conv_share": conv_share,
                             "step_frac": flops / (ms_fwd / 1000.0) / 1e12 / sparse_peak,
                             "hbm_view": {"achieved": alg_bytes / (conv_ms / 1000.0) / 1e9,
                                          "peak": hbm_peak, "unit": "GB/s",
                                          "frac": alg_bytes / (conv_ms / 1000.0) / 1e9 / hbm_peak,
                                          "algorithmic_bytes_per_forward": alg_bytes}},
                "layers": per_layer,
                "strong_scaling": strong,
                "spikformer_linear": linear,
                "spikformer_attention": attn,
                "glue": glue,
                "configs": others,
                "clocks": dict(clk.summary(), window="timed region plus two steps of replays before it"),
                "cpu_baseline": cpu}
        emit(line)


_JSON_FD = None     # original stdout when it is redirected (N > 1)


def emit(line):
    """Print the one JSON result line on the original stdout."""
    text = json.dumps(line) + "\n"
    if _JSON_FD is None:
        print(text, end="", flush=True)
    else:
        os.write(_JSON_FD, text.encode())


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        # Libraries write to file descriptor 1 directly (NCCL prints its
        # version banner there); send all of that to stderr and keep the
        # original stdout for the one JSON line.
        global _JSON_FD
        sys.stdout.flush()
        _JSON_FD = os.dup(1)
        os.dup2(2, 1)
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.profile_config:
        profile_config(args)
        return
    import torch
    import torch.distributed as dist
    from sparsesnn_b200 import dist as sd
    if world > 1:
        torch.cuda.set_device(local_rank)
        sd.init_from_env("nccl", timeout_s=120.0, device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
