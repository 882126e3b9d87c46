"""SEW-ResNet-18 (T=4, CIFAR 32x32, batch 128 per GPU) inference throughput.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One process per GPU (torchrun for N > 1), one model replica per GPU, batch 128
per GPU (weak scaling), NCCL all-gather of the logits each step (the only
collective, as in the data-parallel design).  Prints ONE JSON line on rank 0.

* value: images/s of the whole job, inputs resident in HBM, each step = one
  CUDA-graph replay of the forward (+ logits gather when N > 1), timed with
  CUDA events between barriers, max over ranks.
* e2e: the same through the C-ABI native executor (``snn_engine_run`` on an
  engine file saved from the replica) with the input copied from pinned host
  memory and the logits read back to host every step; ``python_driver`` is
  the same measurement through the Python call ``model(x_host)``.
* roofline: the fused sparse conv kernel (19 launches per forward), timed
  with CUDA events around each launch over K eager forwards run right after
  the timed region; FLOPs are dense-equivalent 2*M*N*K.
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
CPU_SAMPLE = 8           # images per CPU-baseline step


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=BATCH)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-steps", type=int, default=3)
    return ap.parse_args()


def config(args, world):
    return {"workload": f"SEW-ResNet-18 CIFAR stem (3x3 s1, no maxpool), stages 64/128/256/512, "
                        f"ADD, 100 classes, T={T_STEPS}, 3x{HW}x{HW}, batch {args.batch} per GPU",
            "model": "sew_resnet18_cifar", "global_batch": args.batch * world,
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
    196 tokens: 6272 rows per timestep; q/k/v/proj 384->384, fc1 384->1536,
    fc2 1536->384), random 2:4 weights and Bernoulli(0.2) spikes: per-layer
    CUDA-event time and dense-equivalent TFLOP/s against the 2:4 ceiling."""
    import numpy as np
    import torch
    from sparsesnn_b200.layer import SparseConvBNLIF
    from sparsesnn_b200.pruning import prune_2_4_last
    T, rows = 4, 32 * 196
    out = {}
    for name, cin, cout in (("qkv", 384, 384), ("fc1", 384, 1536), ("fc2", 1536, 384)):
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

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
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


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from sparsesnn_b200.sew_resnet import SEWResNet18, conv_layer_bytes, conv_layer_flops, init_params

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    P = init_params(seed=0)
    model = SEWResNet18(P, T=T_STEPS, batch=args.batch, H=HW, W=HW, device=dev)
    g = torch.Generator().manual_seed(1234 + rank)
    x_host = torch.randn((args.batch, 3, HW, HW), generator=g).pin_memory()
    x_dev = x_host.to(dev)
    logits_host = torch.empty((args.batch, model.num_classes), dtype=torch.float32).pin_memory()
    gathered = torch.empty((world * args.batch, model.num_classes), dtype=torch.float32,
                           device=dev) if world > 1 else None

    from sparsesnn_b200 import dist as sd

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    def gather():
        if world > 1:
            sd.gather_logits(model.logits, gathered)

    # Warm-up (eager), then capture the forward into a CUDA graph.
    model.x_in.copy_(x_dev)
    for _ in range(max(3, args.warmup)):
        model.run()
        gather()
    torch.cuda.synchronize()
    model.capture(warmup=1)
    for _ in range(max(3, args.warmup)):
        model.replay()
        gather()
    torch.cuda.synchronize()
    n_launch = len(model.launches())

    # ---------------- timed region A: device-resident inputs, graph replay
    # The clock sampler runs across the timed region plus 300 / 200 identical
    # replays before / after it, so that even a short timed region has
    # samples taken under the same load.
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def roll(iters):
        # Fixed iteration counts: every rank issues the same collectives.
        for i in range(iters):
            model.replay()
            gather()
            if i % 20 == 19:
                torch.cuda.synchronize()
        torch.cuda.synchronize()

    with ClockSampler(local_rank) as clk:
        roll(300)
        barrier(); torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            model.replay()
            gather()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        roll(200)
    ms = sd.max_over_ranks(e0.elapsed_time(e1) / args.steps, device=dev)
    value = args.batch * world / (ms / 1000.0)

    # ---------------- timed region B: end to end through the public call
    barrier(); torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.steps):
        out = model(x_host)                         # H2D from pinned memory + graph replay
        gather()
        logits_host.copy_(out, non_blocking=True)   # D2H of the step's result
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms_e2e = sd.max_over_ranks(e0.elapsed_time(e1) / args.steps, device=dev)
    e2e_driver = args.batch * world / (ms_e2e / 1000.0)

    # ---------------- timed region C: the native executor through the C-ABI
    # (snn_engine_run: pinned host images in, host logits out, the C++ node
    # loop replayed from its CUDA graph), on an engine file saved from the
    # same replica.
    import tempfile
    from sparsesnn_b200 import engine_file as ef
    eng_dir = tempfile.mkdtemp()
    eng_path = os.path.join(eng_dir, f"sew18_rank{rank}.snne")
    ef.save_engine(model, eng_path)
    eng = ef.Engine(eng_path)
    eng_logits = torch.empty_like(model.logits)
    es = torch.cuda.Stream(dev)
    with torch.cuda.stream(es):
        eng.capture(es)
        for _ in range(max(3, args.warmup)):
            eng.run(x_host.data_ptr(), eng_logits.data_ptr(), es)
            if world > 1:
                sd.gather_logits(eng_logits, gathered)
        es.synchronize()
        barrier()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(es)
        for _ in range(args.steps):
            eng.run(x_host.data_ptr(), eng_logits.data_ptr(), es)   # H2D + graph replay
            if world > 1:
                sd.gather_logits(eng_logits, gathered)
            logits_host.copy_(eng_logits, non_blocking=True)         # D2H of the step's result
        c1.record(es)
        es.synchronize()
    barrier()
    ms_eng = sd.max_over_ranks(c0.elapsed_time(c1) / args.steps, device=dev)
    e2e = args.batch * world / (ms_eng / 1000.0)
    eng.close()
    os.remove(eng_path)
    os.rmdir(eng_dir)

    # ---------------- per-launch CUDA-event timing of the fused conv kernel
    ops = model.launches()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in ops]
    conv_ms = 0.0
    per_layer = {name: 0.0 for name, _ in ops}
    for _ in range(args.steps):
        for (name, op), (a, b) in zip(ops, evs):
            a.record(stream); op(); b.record(stream)
        torch.cuda.synchronize()
        for (name, _), (a, b) in zip(ops, evs):
            dt = a.elapsed_time(b)
            per_layer[name] += dt / args.steps
    conv_names = [n for n, _ in ops if n not in ("stem", "head")]
    conv_ms = sum(per_layer[n] for n in conv_names)
    flops = sum(conv_layer_flops(l) for l in model.conv_layers())
    alg_bytes = sum(conv_layer_bytes(blk["l1"], False) + conv_layer_bytes(blk["l2"], True) +
                    (conv_layer_bytes(blk["ds"], False) if blk["ds"] is not None else 0)
                    for blk in model.blocks)
    hbm_peak, bf16_peak, peak_kind = peaks()
    sparse_peak = 2.0 * bf16_peak
    achieved = flops / (conv_ms / 1000.0) / 1e12
    traffic = None
    tf = ROOT / "profiles" / "sew18_traffic.txt"
    if tf.exists():
        for line in tf.read_text().splitlines():
            if line.startswith("fused_conv_dram_bytes_per_forward:"):
                traffic = int(float(line.split(":")[1]))
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
               "sample": f"{CPU_SAMPLE} images x {args.cpu_steps} forwards, torch CPU fp32 "
                         f"port of the reference forward (oracle/sew_resnet.py)"}
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "f16", "data": "synthetic", "config": config(args, world),
                "e2e": {"value": e2e, "unit": UNIT,
                        "h2d_bytes_per_step": int(x_host.numel() * 4),
                        "d2h_bytes_per_step": int(logits_host.numel() * 4),
                        "path": "snn_engine_run (C-ABI native executor, CUDA graph), pinned host buffers",
                        "python_driver": e2e_driver},
                "gpu_launches": n_launch * args.steps,
                "roofline": {"bound": "tensor", "achieved": achieved, "peak": sparse_peak,
                             "unit": "TFLOP/s", "frac": achieved / sparse_peak,
                             "traffic": traffic,
                             "kernel": "fused sparse conv+BN+LIF kernels, 19 launches/forward "
                                       "(halo4 x4, halo x3, halo_stream x6, general x6)",
                             "peak_note": f"2:4 sparse ceiling = 2 x {peak_kind} dense bf16 "
                                          f"{bf16_peak} TFLOP/s; FLOPs dense-equivalent",
                             "flops_per_forward": flops, "kernel_ms_per_forward": conv_ms,
                             "hbm_view": {"achieved": alg_bytes / (conv_ms / 1000.0) / 1e9,
                                          "peak": hbm_peak, "unit": "GB/s",
                                          "frac": alg_bytes / (conv_ms / 1000.0) / 1e9 / hbm_peak,
                                          "algorithmic_bytes_per_forward": alg_bytes}},
                "layer_ms": {k: round(v, 4) for k, v in per_layer.items()},
                "spikformer_linear": linear,
                "spikformer_attention": attn,
                "glue": glue,
                "clocks": dict(clk.summary(), window="timed region plus 300 replays before and 200 after"),
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
