#!/usr/bin/env python
"""W4A4 linear benchmark on B200 (Llama-2-7B linear shapes), with the other configs
as sub-records of the same JSON line.

One step = the seven W4A4 linears of every layer of a 32-layer Llama-2-7B at M = 2048 tokens per GPU
(q, k, v, o: 4096 -> 4096; gate, up: 4096 -> 11008; down: 11008 -> 4096 with the 172 x 64
Hadamard-product rotation), each layer with its own weights and inputs resident in HBM: per layer one
fused rotate+quantize per distinct input (shared by q/k/v and by gate/up) plus one tcgen05 W4A4 GEMM
with the dequant epilogue per linear, 4 + 7 launches. Metric: W4A4 linear TOPS (2*M*N*K integer ops
per linear) over the whole step.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 (under torchrun): every rank runs the step on its own token batch (data parallel over tokens, no
collective on the data path), weak scaling; elapsed time is the max over ranks. At every N the line
also carries `config4_tp`: the Llama-2-70B layer linears split column-parallel over the N ranks
(strong scaling) with the fused NVLink exchange and the NCCL all-gather, per-phase times included.
At N = 1 rank 0 adds the kernel sweeps of configs 1 and 3, the config-2 prefill and the CPU
baseline. `--impl reference` times the reference's own CPU path (QuantLinear.forward as shipped,
restated bit-exactly in oracle/oracle_torch.py) on the host cores on the same workload.
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
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--tokens", type=int, default=2048)
    p.add_argument("--layers", type=int, default=32, help="distinct Llama-2-7B layers per step (32: the whole model)")
    p.add_argument("--no-tp", action="store_true", help="skip the config-4 column-parallel record")
    p.add_argument("--no-prefill", action="store_true", help="skip the config-2 prefill record")
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


# ---------------------------------------------------------------- synthetic model state on the GPU
LAYER3 = [("q", 4096, 4096), ("k", 4096, 1024), ("v", 4096, 1024), ("o", 4096, 4096),
          ("gate", 4096, 14336), ("up", 4096, 14336), ("down", 14336, 4096)]
INPUT_K3 = {"attn": 4096, "o": 4096, "mlp": 4096, "down": 14336}
LAYER70 = [("qkv", 8192, 10240), ("o", 8192, 8192), ("gate", 8192, 28672), ("up", 8192, 28672), ("down", 28672, 8192)]
DATA = "synthetic (seeded N(0,1) activations with 1% x20 outlier channels, N(0,0.02) weights, generated on the GPU)"


def activations_gpu(M: int, K: int, gen, dev):
    """[M, K] bf16 ~ N(0, 1) with 1% of the K channels (seeded choice) scaled x20: the benchmark distribution."""
    import torch

    x = torch.randn(M, K, generator=gen, device=dev)
    cols = torch.randperm(K, generator=gen, device=dev)[: max(1, K // 100)]
    x[:, cols] *= 20.0
    return x.to(torch.bfloat16)


class Quant:
    """Preallocated outputs of one rotate+quantize launch (C ABI, the AUTO kernel) for a [M, K] input."""

    def __init__(self, M: int, K: int, dev, a8: bool = False):
        import torch

        from dscquant_b200 import ops

        self.M, self.K, self.a8 = M, K, a8
        self.packed = None if a8 else torch.empty((M, K // 2), dtype=torch.uint8, device=dev)
        self.codes = torch.empty((M, K), dtype=torch.int8, device=dev) if a8 else None
        self.scales = torch.empty((M,), dtype=torch.float32, device=dev)
        self.rot_a, self.h = ops.rotation_factor(K, dev)
        self.dev = dev

    def __call__(self, x):
        from dscquant_b200 import _lib, ops

        rc = _lib.load().dscq_rowquant(ops._ptr(x), _lib.BF16, self.M, self.K, x.stride(0), 1, self.rot_a,
                                       ops._ptr(self.h), _lib.ACT_SYM, 1.0, self.M, self.K, ops._ptr(self.packed),
                                       0 if self.a8 else self.K // 2, ops._ptr(self.scales), None, None,
                                       ops._ptr(self.codes), self.K if self.a8 else 0, ops._stream(self.dev))
        _lib.check(rc, "rowquant")


def gemm_call(q: Quant, mod, out, M: int, N: int, K: int, dev):
    from dscquant_b200 import _lib, ops

    p = mod._prep
    if q.a8:
        rc = _lib.load().dscq_matmul_a8(ops._ptr(q.codes), K, ops._ptr(p["packed"]), ops._ptr(q.scales),
                                        ops._ptr(p["sw"]), None, None, M, N, K, _lib.BF16, ops._ptr(out), None,
                                        ops._stream(dev))
    else:
        rc = _lib.load().dscq_matmul(ops._ptr(q.packed), ops._ptr(p["packed"]), ops._ptr(q.scales), None,
                                     ops._ptr(p["sw"]), None, None, None, M, N, K, _lib.BF16, ops._ptr(out), None, 0,
                                     ops._stream(dev))
    _lib.check(rc, "matmul")


# ---------------------------------------------------------------- kernel-level sweep (configs 1 and 3)
def sweep_shapes(shapes, Ms, dev, peaks, gen):
    """rotate+quantize and GEMM of each (K, N) at each M, timed per launch with CUDA events, L2 flushed
    (512 MB written) before every timed call; median of 6 after 2 untimed."""
    import statistics

    import torch

    from dscquant_b200 import ops
    from dscquant_b200.llama import random_quant_linear

    flush = torch.empty(512 * 1024 * 1024, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    int8_peak = 2.0 * peaks["bf16_tflops"]
    out = []
    for (K, N) in shapes:
        ql = random_quant_linear(N, K, gen, dev)
        for m in Ms:
            x = activations_gpu(m, K, gen, dev)
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
            out.append({"M": m, "K": K, "N": N, "gemm_us": round(gm * 1e3, 2), "quant_us": round(qm * 1e3, 2),
                        "gemm_tops": round(ops_ / (gm * 1e-3) / 1e12, 1),
                        "linear_tops": round(ops_ / ((gm + qm) * 1e-3) / 1e12, 1),
                        "gemm_frac_int8_peak": round(ops_ / (gm * 1e-3) / 1e12 / int8_peak, 3),
                        "gemm_frac_hbm": round(gbytes / (gm * 1e-3) / 1e9 / peaks["hbm_gbs"], 3),
                        "quant_frac_hbm": round((m * K * 2.5 + 4 * m) / (qm * 1e-3) / 1e9 / peaks["hbm_gbs"], 3)})
        del ql
    del flush
    return out


def layer_from_sweep(sweep, layer, input_k):
    """Per-M layer figures from the sweep: every GEMM of the layer plus one rotate+quantize per distinct
    input (q/k/v share one, gate/up share one)."""
    res = {}
    for m in sorted({r["M"] for r in sweep}):
        rows = {(r["K"], r["N"]): r for r in sweep if r["M"] == m}
        gemm_us = sum(rows[(k, n)]["gemm_us"] for _, k, n in layer)
        quant_us = sum(next(r["quant_us"] for (kk, _), r in rows.items() if kk == K) for K in input_k.values())
        ops_ = sum(2.0 * m * n * k for _, k, n in layer)
        res[str(m)] = {"layer_tops": round(ops_ / ((gemm_us + quant_us) * 1e-6) / 1e12, 1),
                       "gemm_tops": round(ops_ / (gemm_us * 1e-6) / 1e12, 1),
                       "gemm_us": round(gemm_us, 2), "quant_us": round(quant_us, 2)}
    return res


# ---------------------------------------------------------------- config 4: Llama-2-70B layer, column-parallel
def tp70_record(dev, rank: int, world: int, steps: int = 10, warmup: int = 3) -> dict:
    """The five Llama-2-70B layer linears at M = 4096, output channels split over the `world` ranks of the
    job (strong scaling: the total work is fixed). N = 1: one GPU, no exchange. N > 1: the three exchange
    modes of parallel.ColumnParallelQuantLinear -- 'fused' (row-split quantisation into symmetric memory,
    peer reads of the other ranks' rows, GEMM epilogue storing every tile into every rank's output over
    NVLink), 'push' (the same, the epilogue storing locally and a row-block copy pushing each finished
    block to the peers beside the next GEMM launch) and 'nccl' (replicated quantisation, local GEMM,
    NCCL all-gather, reassembly); `value` is the best of them. Times are CUDA
    events on each rank's stream, max over ranks; per-phase milliseconds per step from events recorded
    at the phase boundaries of every call (max over ranks)."""
    import torch

    from dscquant_b200 import ops, parallel
    from dscquant_b200.llama import random_quant_linear

    M = 4096
    ops_total = float(sum(2 * M * n * k for _, k, n in LAYER70))
    gen = torch.Generator(device=dev)
    stream = torch.cuda.current_stream(dev)
    xs = {}
    for K in sorted({k for _, k, _ in LAYER70}):
        gen.manual_seed(9000 + K)
        xs[K] = activations_gpu(M, K, gen, dev)

    def timed(step):
        for _ in range(warmup):
            step()
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / steps
        if world > 1:
            t = torch.tensor([ms], device=dev, dtype=torch.float64)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    rec = {"workload": "llama2-70b-layer-linears", "tokens": M, "shapes_KxN": [[k, n] for _, k, n in LAYER70],
           "n_gpus": world, "scaling": "strong", "unit": "TOPS"}
    if world == 1:
        mods = []
        for i, (name, K, N) in enumerate(LAYER70):
            gen.manual_seed(7000 + 31 * i)
            mods.append((K, N, random_quant_linear(N, K, gen, dev)))

        def step():
            for K, N, ql in mods:
                q = ops.rowquant(xs[K], "act_sym", rotate=True, KP=K)
                ops.w4a4_gemm(q.packed, ql._prep["packed"], q.scales, ql._prep["sw"], M=M, N=N)

        ms = timed(step)
        rec["single"] = {"ms_per_step": ms, "value": ops_total / (ms * 1e-3) / 1e12}
        rec["value"] = rec["single"]["value"]
        return rec
    # single-GPU result of the first linear (every rank holds the full weight for this check): every
    # exchange mode's gathered [M, N] output must equal it bit for bit
    _, K0, N0 = LAYER70[0]
    gen.manual_seed(7000)
    w0 = (torch.randn((N0, K0), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
    qw0 = ops.rowquant(w0, "weight_sym", rotate=True, KP=K0)
    qx0 = ops.rowquant(xs[K0], "act_sym", rotate=True, KP=K0)
    y_ref = ops.w4a4_gemm(qx0.packed, qw0.packed, qx0.scales, qw0.scales, M=M, N=N0)
    del w0, qw0, qx0
    parity = {}
    for mode in ("fused", "push", "nccl"):
        layers = []
        for i, (name, K, N) in enumerate(LAYER70):
            lo, hi = parallel.shard_bounds(N, world, rank)
            gen.manual_seed(7000 + 31 * i)
            w = (torch.randn((N, K), generator=gen, device=dev) * 0.02).to(torch.bfloat16)[lo:hi].contiguous()
            layers.append((K, parallel.ColumnParallelQuantLinear(w, N, mode=mode, max_tokens=M, copy_out=False)))
            del w

        def step():
            for K, layer in layers:
                layer(xs[K])

        ms = timed(step)
        same = torch.tensor([1.0 if torch.equal(layers[0][1](xs[K0]), y_ref) else 0.0], device=dev)
        torch.distributed.all_reduce(same, op=torch.distributed.ReduceOp.MIN)
        parity[mode] = bool(same.item() == 1.0)
        # phase breakdown: one more instrumented pass of `steps` steps
        for _, layer in layers:
            layer.timeline = []
        for _ in range(steps):
            step()
        torch.cuda.synchronize(dev)
        phases = {}
        for _, layer in layers:
            tl = layer.timeline
            for (_, a), (name, b) in zip(tl[:-1], tl[1:]):
                if name == "start":
                    continue
                phases[name] = phases.get(name, 0.0) + a.elapsed_time(b)
            layer.timeline = None
        names = sorted(phases)
        t = torch.tensor([phases[n] / steps for n in names], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        rec[mode] = {"ms_per_step": ms, "value": ops_total / (ms * 1e-3) / 1e12,
                     "phase_ms_per_step": {n: round(float(v), 4) for n, v in zip(names, t.tolist())}}
        del layers
        torch.cuda.synchronize(dev)
        torch.distributed.barrier()
    rec["bit_exact_vs_single_gpu"] = parity  # first linear, [4096, 10240], every rank
    rec["value"] = max(rec[m]["value"] for m in ("fused", "push", "nccl"))
    rec["best_mode"] = max(("fused", "push", "nccl"), key=lambda m: rec[m]["value"])
    return rec


# ---------------------------------------------------------------- config 2: Llama-2-7B prefill
def prefill_record(dev, seq: int = 2048, reps: int = 5) -> dict:
    import torch

    from dscquant_b200.llama import LlamaConfig, LlamaW4A4

    cfg = LlamaConfig()
    model = LlamaW4A4(cfg, dev, seed=11)
    ids = torch.randint(0, cfg.vocab, (seq,), device=dev, generator=torch.Generator(device=dev).manual_seed(12))
    for _ in range(2):
        model(ids)
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)

    def timed(fn):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            out = fn(ids)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / reps, out

    ms_eager, logits = timed(model)
    graph = model.graph(seq)  # the same kernels, replayed from one CUDA graph
    graph(ids)
    ms, glogits = timed(graph)
    ok = bool(torch.isfinite(logits.float()).all()) and bool(torch.equal(glogits, logits))
    del graph
    rec = {"workload": "llama2-7b-prefill", "batch": 1, "seq_len": seq, "layers": cfg.layers, "vocab": cfg.vocab,
           "tokens_per_s": seq / (ms * 1e-3), "ms_per_prefill": ms, "reps": reps, "launch": "one CUDA graph",
           "tokens_per_s_eager": seq / (ms_eager * 1e-3), "ms_per_prefill_eager": ms_eager,
           "w4a4_linear_tops": model.linear_ops(seq) / (ms * 1e-3) / 1e12, "logits_finite_and_graph_equal": ok,
           "note": "all 224 projections + LM head W4A4 (rotate+quantize shared by q/k/v and by gate/up, residuals "
                   "added in the GEMM epilogue); RMSNorm / RoPE / SiLU-gate as single-pass bf16 kernels of this "
                   "package; causal attention bf16 torch SDPA; random-init weights, uniform random token ids"}
    del model
    torch.cuda.empty_cache()
    return rec


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
    if args.impl == "reference":
        run_reference(args, rank, world)  # rank 0 runs, other ranks exit without work
        return

    import torch

    from dscquant_b200 import _lib, ops
    from dscquant_b200.llama import random_quant_linear

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if dist:
        import datetime

        import torch.distributed as tdist

        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = tdist
    world = pg.get_world_size() if pg is not None else 1
    _lib.load()
    peaks = load_peaks()
    M, L = args.tokens, args.layers
    a8 = args.activations == "int8"

    # ---- model state: L distinct layers (packed weights) and their inputs, all resident in HBM
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    layers = []
    for li in range(L):
        mods = {name: random_quant_linear(N, K, gen, dev) for name, K, N in LAYER}
        xs = {key: activations_gpu(M, K, gen, dev) for key, K in INPUT_K.items()}
        layers.append((mods, xs))
    quants = {key: Quant(M, K, dev, a8) for key, K in INPUT_K.items()}
    outs = {name: torch.empty((M, N), dtype=torch.bfloat16, device=dev) for name, _, N in LAYER}
    stream = torch.cuda.current_stream(dev)
    gemm_events, quant_events = [], []

    def step(record_layer=-1):
        """One pass over the L layers; the launches of layer `record_layer` are bracketed by CUDA events
        (a CUDA event costs ~1-3 us of stream time, so the timed steps sample one layer each)."""
        for li, (mods, xs) in enumerate(layers):
            record = li == record_layer
            for key, K in INPUT_K.items():
                if record:
                    e0 = torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                quants[key](xs[key])
                if record:
                    e1 = torch.cuda.Event(enable_timing=True)
                    e1.record(stream)
                    quant_events.append((e0, e1, M * K * 2 + (M * K if a8 else M * K // 2) + 4 * M))
            for name, K, N in LAYER:
                if record:
                    e0 = torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                gemm_call(quants[INPUT_OF[name]], mods[name], outs[name], M, N, K, dev)
                if record:
                    e1 = torch.cuda.Event(enable_timing=True)
                    e1.record(stream)
                    gemm_events.append((e0, e1, 2.0 * M * N * K))

    def barrier():
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        step()
    barrier()
    sampler = ClockSampler(local)
    time.sleep(0.3)
    barrier()
    t_start = time.time()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for i in range(args.steps):
        step(record_layer=(7 * i + 3) % L)  # a different layer's launches timed in each step
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
    step_ops = layer_ops(M) * L
    value = step_ops * world / (ms_per_step * 1e-3) / 1e12
    gemm_ms = sum(a.elapsed_time(b) for a, b, _ in gemm_events)
    gemm_tops = sum(o for _, _, o in gemm_events) / (gemm_ms * 1e-3) / 1e12
    quant_ms = sum(a.elapsed_time(b) for a, b, _ in quant_events)
    quant_gbs = sum(o for _, _, o in quant_events) / (quant_ms * 1e-3) / 1e9
    int8_peak = 2.0 * peaks["bf16_tflops"]
    sm_mhz = (clocks or {}).get("sm_mhz") or 1965.0
    # the 2-SM tcgen05 int8 MMA rate measured on B200 (8176 MAC/clk/SM, cta_group::2 M=256 N=256) at the
    # SM clock sampled during the timed region
    mma_i8_peak = 2 * 8176 * 148 * sm_mhz * 1e6 / 1e12
    status = ops.device_status(dev)
    gemm_events_n, quant_events_n = list(gemm_events), list(quant_events)
    del gemm_events[:], quant_events[:]

    # ---- e2e through the public API (QuantLinear.forward via HostPipeline) with pinned host buffers:
    # layer 0's seven linears; median of 5 repeats
    from dscquant_b200.hostio import HostPipeline

    mods0, xs0 = layers[0]
    host_in = {key: xs0[key].cpu().pin_memory() for key in INPUT_K}
    host_out = {name: torch.empty((M, N), dtype=torch.bfloat16, pin_memory=True) for name, _, N in LAYER}
    h2d = sum(M * K * 2 for K in INPUT_K.values())
    d2h = sum(M * N * 2 for _, _, N in LAYER)
    pipe = HostPipeline(dev)
    for name, _, _ in LAYER:
        mods0[name].int8_activations = a8
    e2e_mods = [mods0[name] for name, _, _ in LAYER]
    e2e_in = [host_in[INPUT_OF[name]] for name, _, _ in LAYER]
    e2e_out = [host_out[name] for name, _, _ in LAYER]
    for _ in range(3):
        pipe.run(e2e_mods, e2e_in, e2e_out)
    barrier()
    reps = []
    for _ in range(5):
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        for _ in range(10):
            pipe.run(e2e_mods, e2e_in, e2e_out)
        stream.wait_event(pipe.done_event)
        a1.record(stream)
        torch.cuda.synchronize(dev)
        reps.append(a0.elapsed_time(a1) / 10)
    e2e_ms = sorted(reps)[len(reps) // 2]
    if pg is not None:
        t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = layer_ops(M) * world / (e2e_ms * 1e-3) / 1e12
    del layers, quants, outs
    torch.cuda.empty_cache()

    # ---- config 4 at this world size (every rank takes part)
    tp = None
    if not args.no_tp:
        tp = tp70_record(dev, rank, world)

    # ---- rank 0 extras at N = 1: kernel sweeps (configs 1 and 3), prefill (config 2), CPU baseline
    sweep7 = sweep3 = prefill = cpu = None
    if rank == 0 and world == 1:
        sgen = torch.Generator(device=dev)
        sgen.manual_seed(77)
        if not args.no_sweep:
            sweep7 = sweep_shapes(((4096, 4096), (4096, 11008), (11008, 4096)), (1, 16, 128, 512, 2048, 8192), dev,
                                  peaks, sgen)
            sweep3 = sweep_shapes(((4096, 4096), (4096, 1024), (4096, 14336), (14336, 4096)), (1, 128, 2048, 8192),
                                  dev, peaks, sgen)
        if not args.no_prefill:
            prefill = prefill_record(dev)
        if not args.no_cpu:
            cpu = cpu_baseline_record(M)

    if rank == 0:
        gemm_kernel = "w4a4_gemm_pair_a8" if a8 else "w4a4_gemm_pair"
        line = {
            "metric": METRIC, "value": value, "unit": "TOPS", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int4 x int4 -> int32 (bf16 in/out)", "data": DATA,
            "config": {"workload": "llama2-7b-linears", "layers": L, "tokens_per_gpu": M,
                       "shapes_KxN": [[k, n] for _, k, n in LAYER], "rotation": "WHT-4096 / H172xH64 (K=11008)",
                       "activation_quant": "symmetric per-token int4", "weight_quant": "symmetric per-channel int4",
                       "activation_codes": "int8 (one code per byte)" if a8 else "packed int4 nibbles",
                       "parallelism": f"dp{world} over tokens" if world > 1 else "single GPU",
                       "l2": f"{L} distinct layers per step ({L * 101} MB of packed weights, inputs per layer): "
                             "larger than the 126 MB L2"},
            "gpu_launches": 11 * L * args.steps,
            "roofline": {"kernel": gemm_kernel, "bound": "tensor", "achieved": gemm_tops, "peak": int8_peak,
                         "unit": "TFLOP/s", "frac": gemm_tops / int8_peak,
                         "peak_note": f"int8 dense = 2 x {peaks['source']} bf16 cuBLAS {peaks['bf16_tflops']} TFLOP/s; "
                                      "ops are integer ops (2 per MAC)",
                         "frac_of_mma_i8_rate": gemm_tops / mma_i8_peak, "mma_i8_rate": mma_i8_peak,
                         "mma_i8_note": "2-SM tcgen05 kind::i8 issue rate measured on B200 (8176 MAC/clk/SM) x 148 SMs "
                                        "x the sampled SM clock",
                         "traffic": 19.753e6 if (M == 2048 and not a8) else None,
                         "traffic_source": "copied from an ncu capture (dram__bytes_read.sum + dram__bytes_write.sum, "
                                           "w4a4_gemm_pair at M=2048 on the three shapes, launch-weighted), "
                                           "profiles/w4a4_gemm_persistent__dram_traffic_M2048.md; not measured in "
                                           "this run",
                         "share_of_step": gemm_ms * L / elapsed_ms,
                         "timed_launches": len(gemm_events_n),
                         "sampling": "CUDA events around every launch of one layer per timed step (a different "
                                     "layer each step)"},
            "roofline_quantize": {"kernel": "rotq_tc", "bound": "hbm", "achieved": quant_gbs, "peak": peaks["hbm_gbs"],
                                  "unit": "GB/s", "frac": quant_gbs / peaks["hbm_gbs"],
                                  "share_of_step": quant_ms * L / elapsed_ms, "timed_launches": len(quant_events_n)},
            "e2e": {"value": e2e_value, "unit": "TOPS", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "repeats_ms": [round(r, 3) for r in reps],
                    "api": "HostPipeline.run over one layer's 7 QuantLinear modules: pinned host input -> device -> "
                           "QuantLinear.forward -> pinned host output per linear, copies overlapped with the kernels "
                           "on three streams; median of 5 repeats of 10 calls"},
            "cpu_baseline": cpu, "clocks": clocks, "device_status": status,
            "config4_tp": tp, "config2_prefill": prefill,
            "config1_sweep": sweep7,
            "config3_sweep": sweep3,
            "config3_layer": layer_from_sweep(sweep3, LAYER3, INPUT_K3) if sweep3 else None,
            "config1_layer": layer_from_sweep(sweep7, LAYER, INPUT_K) if sweep7 else None,
        }
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()


if __name__ == "__main__":
    main()
