#!/usr/bin/env python
"""W4A4 linear benchmark on B200 (Llama-2-7B linear shapes).

One step = the seven W4A4 linears of one Llama-2-7B decoder layer at M tokens
(q, k, v, o: 4096 -> 4096; gate, up: 4096 -> 11008; down: 11008 -> 4096 with the
172 x 64 Hadamard-product rotation), each one fused rotate+quantize of its
input (shared by q/k/v and by gate/up) plus one tcgen05 W4A4 GEMM with the
dequant epilogue: 4 + 7 kernel launches. Metric: W4A4 linear TOPS
(2*M*N*K integer ops per linear) over the whole step.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 (under torchrun): every rank runs the same layer on its own token batch
(data parallel over tokens, no collective on the data path), weak scaling;
elapsed time is the max over ranks. `--impl reference` times the CPU W4A4
linear of the oracle restatement (the reference's own path is PyTorch CPU
fake-quant; its arithmetic is restated in oracle/) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

LAYER = [("q", 4096, 4096), ("k", 4096, 4096), ("v", 4096, 4096), ("o", 4096, 4096),
         ("gate", 4096, 11008), ("up", 4096, 11008), ("down", 11008, 4096)]
# which quantised input each linear consumes (q/k/v share one, gate/up share one)
INPUT_OF = {"q": "attn", "k": "attn", "v": "attn", "o": "o", "gate": "mlp", "up": "mlp", "down": "down"}
INPUT_K = {"attn": 4096, "o": 4096, "mlp": 4096, "down": 11008}
METRIC = "W4A4 linear TOPS at Llama-2-7B shapes (M=1..2048), % of int8 TC peak"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--workload", default="llama2-7b", choices=["llama2-7b", "llama2-70b-tp"],
                   help="llama2-7b: config 1 layer, data parallel over tokens (default); "
                        "llama2-70b-tp: config 4 layer, column-parallel over N with the fused all-gather")
    p.add_argument("--tp-mode", default="fused", choices=["fused", "nccl"])
    p.add_argument("--tokens", type=int, default=2048)
    p.add_argument("--replicas", type=int, default=4, help="layer replicas cycled so the working set exceeds L2")
    p.add_argument("--activations", default="packed", choices=["packed", "int8"],
                   help="activation codes handed from the quantizer to the GEMM: packed nibbles (dscq_matmul, "
                        "the reference's format) or one int8 code per element (dscq_matmul_a8); same result bits")
    p.add_argument("--no-sweep", action="store_true")
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--kernel-case", choices=["gemm", "quant", "headrot"], default=None,
                   help="run REPS launches of one kernel on [M, K] x [N, K] (for profilers) and exit")
    p.add_argument("--M", type=int, default=8192)
    p.add_argument("--K", type=int, default=4096)
    p.add_argument("--N", type=int, default=11008)
    p.add_argument("--reps", type=int, default=3)
    p.add_argument("--variant", type=int, default=0,
                   help="--kernel-case gemm: dscq_matmul variant 0-6, or dscq_matmul_a8 (int8 activation codes): "
                        "7 = AUTO (CTA pairs), 8 = the 1-CTA kernel")
    p.add_argument("--qvariant", default="auto", choices=["auto", "tc", "legacy"],
                   help="rotate+quantize kernel for --kernel-case quant")
    p.add_argument("--graph", action="store_true",
                   help="--kernel-case gemm: time REPS launches replayed from one CUDA graph (device time per launch, "
                        "no host launch overhead), cycling weight copies so the launches stream weights from HBM")
    return p.parse_args()


def _graph_time(fn, R: int, dev) -> float:
    """Median device time (ms) per call of fn(i), i = 0..R-1, replayed from one CUDA graph."""
    import torch

    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for i in range(R):
            fn(i)
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(R):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    ts = []
    for _ in range(5):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1) / R)
    del g
    return statistics.median(ts)


def kernel_case(args) -> None:
    """A few launches of one kernel on synthetic data, timed with CUDA events (used under ncu)."""
    import numpy as np
    import torch

    from dscquant_b200 import ops, synthetic

    dev = torch.device("cuda", 0)
    bf = lambda b: torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(torch.bfloat16).to(dev)  # noqa: E731
    x = bf(synthetic.activations_bf16(args.M, args.K, seed=1))
    if args.kernel_case == "headrot":  # online per-head rotation + quantisation, heads = K / 128
        g = torch.Generator().manual_seed(5)
        a = torch.randn(args.K // 128, 128, 128, generator=g, dtype=torch.float64) * 0.05
        hi, lo = ops.head_rotation_operands(torch.matrix_exp(a - a.transpose(1, 2)).float().to(dev))
        units = args.M * args.K * 2.5 + 4 * args.M
        copies = max(1, min(64, -(-(256 << 20) // (args.M * args.K * 2)))) if args.graph else 1
        xs = [x] + [x.clone() for _ in range(copies - 1)]

        def fn(i=0):
            return ops.rowquant_headrot(xs[i % copies], hi, lo, "act_sym")
        if args.graph:
            t = _graph_time(fn, max(args.reps, copies), dev)
            print(json.dumps({"kernel_case": "headrot", "M": args.M, "K": args.K, "ms": t,
                              "rate": units / (t * 1e-3) / 1e9, "unit": "GB/s", "input_copies": copies}))
            return
    elif args.kernel_case == "quant":
        units = args.M * args.K * 2.5 + 4 * args.M
        # input copies: enough that consecutive graph launches never find their rows in the 126 MB L2
        copies = max(1, min(64, -(-(256 << 20) // (args.M * args.K * 2)))) if args.graph else 1
        xs = [x] + [x.clone() for _ in range(copies - 1)]

        def fn(i=0):
            return ops.rowquant(xs[i % copies], "act_sym", rotate=True, KP=args.K, variant=args.qvariant)
        if args.graph:
            t = _graph_time(fn, max(args.reps, copies), dev)
            print(json.dumps({"kernel_case": "quant", "qvariant": args.qvariant, "M": args.M, "K": args.K, "ms": t,
                              "rate": units / (t * 1e-3) / 1e9, "unit": "GB/s", "graph_launches": max(args.reps, copies),
                              "input_copies": copies}))
            return
    else:
        w = bf(synthetic.weights_bf16(args.N, args.K, seed=2))
        qw = ops.rowquant(w, "weight_sym", rotate=True, KP=args.K)
        qx = ops.rowquant(x, "act_sym", rotate=True, KP=args.K, codes=args.variant in (7, 8))
        out = torch.empty((args.M, args.N), dtype=torch.bfloat16, device=dev)
        from dscquant_b200 import _lib

        # weight copies: enough that consecutive launches never find their weights in the 126 MB L2
        wbytes = qw.packed.numel()
        copies = max(1, min(64, -(-(256 << 20) // wbytes))) if args.graph else 1
        wcopies = [qw.packed] + [qw.packed.clone() for _ in range(copies - 1)]
        lib = _lib.load()

        def fn(i=0):
            if args.variant in (7, 8):  # int8 activation codes: AUTO (CTA pairs) / the 1-CTA kernel
                v = _lib.GEMM_AUTO if args.variant == 7 else _lib.GEMM_LARGE_M
                _lib.check(lib.dscq_matmul_a8_variant(ops._ptr(qx.codes), args.K, ops._ptr(wcopies[i % copies]),
                                                      ops._ptr(qx.scales), ops._ptr(qw.scales), None, None, args.M,
                                                      args.N, args.K, _lib.BF16, ops._ptr(out), None, v,
                                                      ops._stream(dev)), "matmul_a8")
                return
            _lib.check(lib.dscq_matmul(ops._ptr(qx.packed), ops._ptr(wcopies[i % copies]), ops._ptr(qx.scales), None,
                                       ops._ptr(qw.scales), None, None, None, args.M, args.N, args.K,
                                       _lib.BF16, ops._ptr(out), None, args.variant, ops._stream(dev)),
                       "matmul")
        units = 2.0 * args.M * args.N * args.K
        if args.graph:
            R = max(args.reps, copies)
            t = _graph_time(fn, R, dev)
            print(json.dumps({"kernel_case": "gemm", "variant": args.variant, "M": args.M, "K": args.K, "N": args.N,
                              "ms": t, "rate": units / (t * 1e-3) / 1e12, "unit": "TOPS", "graph_launches": R,
                              "weight_copies": copies,
                              "weight_GBps": wbytes / (t * 1e-3) / 1e9}))
            return
    fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(args.reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    t = min(ts)
    rate = units / (t * 1e-3) / (1e12 if args.kernel_case == "gemm" else 1e9)
    print(json.dumps({"kernel_case": args.kernel_case, "variant": args.variant, "M": args.M, "K": args.K, "N": args.N, "ms": t,
                      "rate": rate, "unit": "TOPS" if args.kernel_case == "gemm" else "GB/s"}))


def layer_ops(M: int) -> float:
    return float(sum(2 * M * n * k for _, k, n in LAYER))


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        return {"hbm_gbs": float(pk["hbm_gbs"]), "bf16_tflops": float(pk["bf16_tflops"]),
                "bf16_tflops_sustained": float(pk.get("bf16_tflops_sustained", pk["bf16_tflops"])),
                "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ---------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, gpu_index: int):
        self.samples = []
        self.window = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(gpu_index), "-lms", "100"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.time(), line.strip()))

    def mark(self, t0, t1):
        self.window = (t0, t1)

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for t, line in self.samples:
            if self.window and not (self.window[0] - 0.15 <= t <= self.window[1] + 0.15):
                continue
            parts = [s.strip() for s in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        if not rows:
            rows = [[s.strip() for s in line.split(",")] for _, line in self.samples[-3:]]
            rows = [r for r in rows if len(r) >= 9]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        reasons = sorted({self.NAMES[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------- reference arm / CPU baseline
def ref_layer_sample(rows: int, seed: int = 0):
    """The reference's own CPU path as shipped -- QuantLinear.forward (core/linear.py:48-52: weight and
    activation fake quantisation every call, bf16 F.linear), restated bit-exactly in oracle/oracle_torch.py --
    over the 7 Llama-2-7B layer linears on `rows` tokens, with every host core torch can use.
    Returns (step, stage_split, threads): step() runs the 7 linears; stage_split() runs them once and returns
    seconds per stage."""
    import numpy as np
    import torch

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle_torch

    from dscquant_b200 import synthetic

    torch.set_num_threads(os.cpu_count() or 1)
    bf = lambda b: torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(torch.bfloat16)  # noqa: E731
    xs = {key: bf(synthetic.activations_bf16(rows, K, seed=3000 + K + 7 * i)) for i, (key, K) in enumerate(INPUT_K.items())}
    layers = [(xs[INPUT_OF[name]], bf(synthetic.weights_bf16(N, K, seed=1000 + i))) for i, (name, K, N) in enumerate(LAYER)]

    def step():
        for x, w in layers:
            oracle_torch.quantlinear_forward(x, w)

    def stage_split():
        tot = {}
        for x, w in layers:
            for k, v in oracle_torch.timed_stages(x, w).items():
                tot[k] = tot.get(k, 0.0) + v
        return tot

    return step, stage_split, torch.get_num_threads()


def cpu_port_sample(rows: int, seed: int = 0):
    """The oracle's C W4A4 linear (benchmark scheme: Hadamard rotation, symmetric int4 codes, int32 GEMM on
    pre-packed int4 weights, epilogue) on `rows` tokens, pthreads over every host core."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import oracle

    from dscquant_b200 import synthetic

    f32 = lambda b: (b.astype(np.uint32) << 16).view(np.float32)  # noqa: E731
    layers = []
    for i, (name, K, N) in enumerate(LAYER):
        w = synthetic.weights_bf16(N, K, seed=1000 + i)
        q = oracle.quant_rows(oracle.rotate_c(f32(w)), oracle.WEIGHT_SYM, 1.0, KP=K)
        layers.append((synthetic.activations_bf16(rows, K, seed=2000 + i), q["packed"], q["scales"], N))

    def step():
        for x, wp, sw, N in layers:
            oracle.w4a4_linear(x, wp, sw, N)

    return step, oracle.num_threads()


def _time_bounded(step, min_steps: int, min_s: float, max_s: float) -> tuple[float, int]:
    step()  # warm-up
    n, t0 = 0, time.perf_counter()
    while n < min_steps or (time.perf_counter() - t0 < min_s and time.perf_counter() - t0 < max_s):
        step()
        n += 1
    return (time.perf_counter() - t0) / n, n


def cpu_baseline_record(tokens: int) -> dict:
    """cpu_baseline for the GPU arm: a bounded sample (about 10-30 s) of the same workload on the host cores."""
    step, split, threads = ref_layer_sample(tokens)
    dt, n = _time_bounded(step, 2, 8.0, 30.0)
    stages = split()
    rec = {"value": layer_ops(tokens) / dt / 1e12, "unit": "TOPS", "cores": threads, "kind": "port",
           "sample": (f"{n} steps of the reference's QuantLinear.forward as shipped (oracle/oracle_torch.py, bit-exact "
                      f"restatement of core/linear.py:48-52) over the 7 Llama-2-7B layer linears at {tokens} tokens"),
           "ms_per_step": dt * 1e3, "tokens": tokens,
           "stage_ms": {k: round(v * 1e3, 2) for k, v in stages.items()}}
    cstep, cthreads = cpu_port_sample(16)
    cdt, cn = _time_bounded(cstep, 2, 3.0, 15.0)
    rec["c_port_benchmark_scheme"] = {"value": layer_ops(16) / cdt / 1e12, "unit": "TOPS", "cores": cthreads,
                                      "tokens": 16, "steps": cn,
                                      "what": "oracle C W4A4 linear: rotation, symmetric codes, int32 GEMM, epilogue"}
    return rec


def run_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    rows = args.tokens
    step, split, threads = ref_layer_sample(rows)
    for _ in range(max(args.warmup, 0)):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / max(args.steps, 1)
    tops = layer_ops(rows) / dt / 1e12
    stages = split()
    sample = (f"{rows} tokens per step through the 7 Llama-2-7B layer linears, the reference's QuantLinear.forward as "
              "shipped (per-call weight fake quantisation, asymmetric per-token activations, bf16 F.linear; "
              "oracle/oracle_torch.py restates core/linear.py:48-52 bit-exactly)")
    line = {"impl": "reference", "metric": METRIC, "value": tops, "unit": "TOPS", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16 fake-quant (int4 codes held in bf16)",
            "data": "synthetic (seeded N(0,1) activations with 1% x20 outlier channels, N(0,0.02) weights)",
            "config": {"workload": "llama2-7b-layer-linears", "tokens_per_gpu": rows,
                       "shapes_KxN": [[k, n] for _, k, n in LAYER], "parallelism": "host cores"},
            "cpu_baseline": {"value": tops, "unit": "TOPS", "cores": threads, "kind": "port", "sample": sample,
                             "stage_ms": {k: round(v * 1e3, 2) for k, v in stages.items()}},
            "e2e": {"value": tops, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- config 4: column-parallel 70B layer
LAYER70 = [("qkv", 8192, 10240), ("o", 8192, 8192), ("gate", 8192, 28672), ("up", 8192, 28672), ("down", 28672, 8192)]


def run_tp(args) -> None:
    """Llama-2-70B layer linears at M = 4096 tokens, column-parallel over N on every
    rank of the job; the shards are exchanged inside the GEMM epilogue (fused) or by NCCL all-gather.
    Strong scaling: the total work is fixed; value = layer ops / max-over-ranks step time."""
    import datetime

    import torch
    import torch.distributed as tdist

    from dscquant_b200 import _lib, ops, parallel, synthetic  # noqa: F401

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29531")
    tdist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                             device_id=dev)
    M = 4096
    gen = torch.Generator(device=dev)
    layers = []
    for i, (name, K, N) in enumerate(LAYER70):
        lo, hi = parallel.shard_bounds(N, world, rank)
        gen.manual_seed(7000 + 31 * i + rank)
        w = (torch.randn((hi - lo, K), generator=gen, device=dev, dtype=torch.float32) * 0.02).to(torch.bfloat16)
        layers.append((name, K, N, parallel.ColumnParallelQuantLinear(w, N, mode=args.tp_mode, max_tokens=M)))
        del w
    xs = {}
    for K in sorted({k for _, k, _ in LAYER70}):
        gen.manual_seed(9000 + K)
        xs[K] = torch.randn((M, K), generator=gen, device=dev, dtype=torch.float32).to(torch.bfloat16)
    stream = torch.cuda.current_stream(dev)

    def step():
        for name, K, N, layer in layers:
            layer(xs[K])

    for _ in range(max(args.warmup, 1)):
        step()
    tdist.barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / args.steps
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
    ms = float(t.item())
    ops_ = float(sum(2 * M * n * k for _, k, n in LAYER70))
    if rank == 0:
        print(json.dumps({"metric": "W4A4 linear TOPS, Llama-2-70B layer linears, column-parallel over N",
                          "value": ops_ / (ms * 1e-3) / 1e12, "unit": "TOPS", "n_gpus": world, "steps": args.steps,
                          "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
                          "vs_baseline": None, "dtype": "int4 x int4 -> int32 (bf16 in/out)",
                          "data": "synthetic (seeded normal activations and weights)",
                          "config": {"workload": "llama2-70b-tp", "tokens": M, "tp_mode": args.tp_mode,
                                     "shapes_KxN": [[k, n] for _, k, n in LAYER70],
                                     "parallelism": f"tp{world} column-parallel over N"}}), flush=True)
    del layers
    tdist.barrier()
    tdist.destroy_process_group()


# ---------------------------------------------------------------- GPU arm
def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = world > 1 and "RANK" in os.environ
    if args.kernel_case:
        kernel_case(args)
        return
    if args.workload == "llama2-70b-tp" and args.impl == "ours":
        run_tp(args)
        return
    if args.impl == "reference":
        if dist:
            pass  # other ranks exit without work
        run_reference(args, rank, world)
        return

    import numpy as np
    import torch

    import dscquant_b200 as dq
    from dscquant_b200 import _lib, ops, synthetic

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if dist:
        import datetime

        import torch.distributed as tdist

        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = tdist
    _lib.load()
    peaks = load_peaks()
    M, R = args.tokens, args.replicas

    # ---- model state: R replicas of one layer's weights (packed once) and inputs
    def bf(bits):
        return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(dev)

    reps = []
    for r in range(R):
        mods = {}
        for i, (name, K, N) in enumerate(LAYER):
            base = torch.nn.Linear(K, N, bias=False, dtype=torch.bfloat16, device=dev)
            with torch.no_grad():
                base.weight.copy_(bf(synthetic.weights_bf16(N, K, seed=1000 + i + 17 * r)))
            ql = dq.QuantLinear(base, dq.QuantConfig())
            ql.enabled = True
            ql.prepare()
            ql.base.weight.data = torch.empty(0, device=dev, dtype=torch.bfloat16)  # only packed weights stay
            mods[name] = ql
        xs = {k: bf(synthetic.activations_bf16(M, K, seed=3000 + 31 * r + K + rank)) for k, K in INPUT_K.items()}
        reps.append((mods, xs))
    outs = {name: torch.empty((M, N), dtype=torch.bfloat16, device=dev) for name, _, N in LAYER}

    a8 = args.activations == "int8"
    stream = torch.cuda.current_stream(dev)
    gemm_events = []  # (start, end, ops) of GEMM launches in the timed region
    quant_events = []  # (start, end, bytes)

    def step(i, record=False):
        mods, xs = reps[i % R]
        qs = {}
        for key, K in INPUT_K.items():
            if record:
                e0 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
            qs[key] = ops.rowquant(xs[key], "act_sym", rotate=True, KP=K, codes=a8, packed_out=not a8)
            if record:
                e1 = torch.cuda.Event(enable_timing=True)
                e1.record(stream)
                quant_events.append((e0, e1, M * K * 2 + (M * K if a8 else M * K // 2) + 4 * M))
        for name, K, N in LAYER:
            ql = mods[name]
            q = qs[INPUT_OF[name]]
            p = ql._prep
            if record:
                e0 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
            if a8:
                rc = _lib.load().dscq_matmul_a8(ops._ptr(q.codes), K, ops._ptr(p["packed"]), ops._ptr(q.scales),
                                                ops._ptr(p["sw"]), None, None, M, N, K, _lib.BF16,
                                                ops._ptr(outs[name]), None, ops._stream(dev))
            else:
                rc = _lib.load().dscq_matmul(ops._ptr(q.packed), ops._ptr(p["packed"]), ops._ptr(q.scales), None,
                                             ops._ptr(p["sw"]), None, None, None, M, N, K, _lib.BF16,
                                             ops._ptr(outs[name]), None, 0, ops._stream(dev))
            _lib.check(rc, "matmul")
            if record:
                e1 = torch.cuda.Event(enable_timing=True)
                e1.record(stream)
                gemm_events.append((e0, e1, 2.0 * M * N * K))

    def barrier():
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize(dev)

    for i in range(args.warmup):
        step(i)
    barrier()
    sampler = ClockSampler(local)
    time.sleep(0.3)
    barrier()
    t_start = time.time()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for i in range(args.steps):
        step(i, record=True)
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    t_end = time.time()
    barrier()
    elapsed_ms = ev0.elapsed_time(ev1)
    sampler.mark(t_start, t_end)
    clocks = sampler.stop()
    if pg is not None:
        t = torch.tensor([elapsed_ms], device=dev, dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        elapsed_ms = float(t.item())
    ms_per_step = elapsed_ms / args.steps
    value = layer_ops(M) * world / (ms_per_step * 1e-3) / 1e12

    gemm_ms = sum(a.elapsed_time(b) for a, b, _ in gemm_events)
    gemm_ops = sum(o for _, _, o in gemm_events)
    quant_ms = sum(a.elapsed_time(b) for a, b, _ in quant_events)
    quant_bytes = sum(o for _, _, o in quant_events)
    gemm_tops = gemm_ops / (gemm_ms * 1e-3) / 1e12
    quant_gbs = quant_bytes / (quant_ms * 1e-3) / 1e9
    int8_peak = 2.0 * peaks["bf16_tflops"]  # kind::i8 issues at twice the kind::f16 rate

    status = ops.device_status(dev)

    # ---- e2e through the public API (QuantLinear.forward) with pinned host buffers
    mods = reps[0][0]
    # one pinned host input per distinct layer input (q/k/v share one, gate/up another), copied once
    host_in = {key: torch.empty((M, K), dtype=torch.bfloat16, pin_memory=True) for key, K in INPUT_K.items()}
    host_out = {name: torch.empty((M, N), dtype=torch.bfloat16, pin_memory=True) for name, _, N in LAYER}
    for key in INPUT_K:
        host_in[key].copy_(reps[0][1][key].cpu())
    h2d = sum(M * K * 2 for K in INPUT_K.values())
    d2h = sum(M * N * 2 for _, _, N in LAYER)
    from dscquant_b200.hostio import HostPipeline

    pipe = HostPipeline(dev)
    for name, _, _ in LAYER:
        mods[name].int8_activations = a8  # same activation format as the device-resident step
    e2e_mods = [mods[name] for name, _, _ in LAYER]
    e2e_in = [host_in[INPUT_OF[name]] for name, _, _ in LAYER]
    e2e_out = [host_out[name] for name, _, _ in LAYER]

    def e2e_step():
        pipe.run(e2e_mods, e2e_in, e2e_out)

    e2e_steps = max(5, min(args.steps, 30))
    for _ in range(3):
        e2e_step()
    barrier()
    a0 = torch.cuda.Event(enable_timing=True)
    a1 = torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    stream.wait_event(pipe.done_event)
    a1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = a0.elapsed_time(a1) / e2e_steps
    if pg is not None:
        t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = layer_ops(M) * world / (e2e_ms * 1e-3) / 1e12

    # ---- sweep over M for the three shapes (kernel-level, L2 flushed before each timed call)
    sweep = []
    if not args.no_sweep and rank == 0:
        flush = torch.empty(512 * 1024 * 1024, dtype=torch.uint8, device=dev)
        for (K, N) in ((4096, 4096), (4096, 11008), (11008, 4096)):
            base = torch.nn.Linear(K, N, bias=False, dtype=torch.bfloat16, device=dev)
            with torch.no_grad():
                base.weight.copy_(bf(synthetic.weights_bf16(N, K, seed=K + N)))
            ql = dq.QuantLinear(base, dq.QuantConfig())
            ql.enabled = True
            ql.prepare()
            for m in (1, 16, 128, 512, 2048, 8192):
                x = bf(synthetic.activations_bf16(m, K, seed=m))
                g_t, q_t = [], []
                for it in range(8):
                    flush.zero_()
                    e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
                    e[0].record(stream)
                    q = ops.rowquant(x, "act_sym", rotate=True, KP=K)
                    e[1].record(stream)
                    ops.w4a4_gemm(q.packed, ql._prep["packed"], q.scales, ql._prep["sw"], M=m, N=N)
                    e[2].record(stream)
                    torch.cuda.synchronize(dev)
                    if it >= 2:
                        q_t.append(e[0].elapsed_time(e[1]))
                        g_t.append(e[1].elapsed_time(e[2]))
                gm, qm = statistics.median(g_t), statistics.median(q_t)
                ops_ = 2.0 * m * N * K
                gbytes = m * K / 2 + N * K / 2 + 2 * m * N + 4 * m + 4 * N
                sweep.append({"M": m, "K": K, "N": N, "gemm_us": round(gm * 1e3, 2), "quant_us": round(qm * 1e3, 2),
                              "gemm_tops": round(ops_ / (gm * 1e-3) / 1e12, 1),
                              "linear_tops": round(ops_ / ((gm + qm) * 1e-3) / 1e12, 1),
                              "gemm_frac_int8_peak": round(ops_ / (gm * 1e-3) / 1e12 / int8_peak, 3),
                              "gemm_frac_hbm": round(gbytes / (gm * 1e-3) / 1e9 / peaks["hbm_gbs"], 3),
                              "quant_frac_hbm": round((m * K * 2.5 + 4 * m) / (qm * 1e-3) / 1e9 / peaks["hbm_gbs"], 3)})
        del flush

    # ---- CPU baseline (rank 0 at N = 1)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline_record(M)

    # DRAM bytes per GEMM launch from one ncu capture of each benchmark shape at M = 2048
    # (dram__bytes_read.sum + dram__bytes_write.sum), launch-weighted over the step's 7 GEMMs
    gemm_kernel = "w4a4_gemm_pair_a8" if a8 else "w4a4_gemm_pair"
    traffic = None
    if M == 2048 and not a8:
        per_shape = {(4096, 4096): 12.662e6, (4096, 11008): 26.866e6, (11008, 4096): 33.891e6}
        traffic = sum(per_shape[(k, n)] for _, k, n in LAYER) / len(LAYER)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TOPS", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int4 x int4 -> int32 (bf16 in/out)",
            "data": "synthetic (seeded N(0,1) activations with 1% x20 outlier channels, N(0,0.02) weights)",
            "config": {"workload": "llama2-7b-layer-linears", "tokens_per_gpu": M,
                       "shapes_KxN": [[k, n] for _, k, n in LAYER], "rotation": "WHT-4096 / H172xH64 (K=11008)",
                       "activation_quant": "symmetric per-token int4", "weight_quant": "symmetric per-channel int4",
                       "activation_codes": "int8 (one code per byte)" if a8 else "packed int4 nibbles",
                       "parallelism": f"dp{world} over tokens" if world > 1 else "single GPU",
                       "l2": f"{R} layer replicas cycled (working set > 126 MB L2)"},
            "gpu_launches": 11 * args.steps,
            "roofline": {"kernel": gemm_kernel, "bound": "tensor", "achieved": gemm_tops, "peak": int8_peak,
                         "unit": "TFLOP/s", "frac": gemm_tops / int8_peak, "traffic": traffic,
                         "traffic_note": f"{gemm_kernel} bytes per launch, ncu capture of each shape at M=2048 (profiles/)",
                         "peak_note": f"int8 dense = 2 x {peaks['source']} bf16 cuBLAS {peaks['bf16_tflops']} TFLOP/s; "
                                      "ops are integer ops (2 per MAC)",
                         "share_of_step": gemm_ms / elapsed_ms},
            "roofline_quantize": {"kernel": "rowquant", "bound": "hbm", "achieved": quant_gbs, "peak": peaks["hbm_gbs"],
                                  "unit": "GB/s", "frac": quant_gbs / peaks["hbm_gbs"],
                                  "share_of_step": quant_ms / elapsed_ms},
            "e2e": {"value": e2e_value, "unit": "TOPS", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "api": "HostPipeline.run over the 7 QuantLinear modules: pinned host input -> device -> "
                           "QuantLinear.forward -> pinned host output per linear, copies in both directions "
                           "overlapped with the kernels on three streams"},
            "cpu_baseline": cpu, "clocks": clocks, "device_status": status, "sweep": sweep,
        }
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()


if __name__ == "__main__":
    main()
