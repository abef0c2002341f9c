"""Benchmark of the quantized-matmul hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the config the headline metric is quoted
on): decode qmv, M=1, bf16 activations ~N(0,1), 4-bit g64 weights quantized
(MLX affine) from N(0, 0.02), the seven projections of a 27B-class decoder
layer: 6144x5120, 1024x5120 (x2), 5120x6144, 17408x5120 (x2), 5120x17408.
One step = one pass over the seven projections (191.7 MB of algorithmic
bytes).  Two copies of the layer's weights alternate between steps, so every
step reads 191.7 MB that is not L2 resident (383 MB > 126 MB L2).

Headline: `value` = algorithmic weight-stream GB/s (bytes = N*K*bits/8 +
2*N*(K/64)*2 + M*K*2 + M*N*2 per projection) with inputs resident in HBM;
`e2e` = the same metric through the public op (mlxturbo_b200.ops.
quantized_matmul) with each step's activations copied from pinned host memory
and the outputs copied back inside the timed region (the step's calls captured
once in a CUDA graph and replayed, as a decode loop runs them; eager figures
beside it).  Extra keys report the
M=2..16 verify sweep and the 8-bit lm_head.

Multi-GPU: the dense decode path does not shard (replicas only); each rank
runs the same layer on its own GPU, `value` sums all ranks' bytes over the max
of the per-rank device times ("scaling": "weak").

--impl reference: the reference's arithmetic has no runnable implementation
here (MLX/Metal are absent); the CPU arm times this repository's C oracle
(fp32 dequantise-then-matmul, OpenMP over all host cores) on a bounded sample
of the same workload and reports the same metric.
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

import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

LAYER = [  # (N, K) of one 27B-class decoder layer
    (6144, 5120), (1024, 5120), (1024, 5120), (5120, 6144), (17408, 5120), (17408, 5120), (5120, 17408)]
GS, BITS = 64, 4
I8_MIN_BYTES = 12 << 20  # matrices of this many bytes of codes take the integer-MMA kernel at M <= 8
# DRAM bytes (read + write) per launch of each projection's kernels, from one
# ncu capture of `python bench.py --case layer` (profiles/
# decode_layer_launches.md): the integer-MMA kernel plus its prep launch
NCU_TRAFFIC_BYTES = {"6144x5120": 17976832, "5120x6144": 17980672, "17408x5120": 50386048, "5120x17408": 50669056}
L2_BYTES = 126 * 1024 * 1024
PEAKS_PATH = os.path.join(REPO, "MEASURED_PEAKS.json")


def alg_bytes(M: int, N: int, K: int, bits: int = BITS, gs: int = GS) -> int:
    return N * K * bits // 8 + 2 * N * (K // gs) * 2 + M * K * 2 + M * N * 2


def peaks() -> dict:
    try:
        with open(PEAKS_PATH) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])),
                "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    """SM clocks and clock-event reasons, read (never set) while the GPU is
    under the benchmark's load: through NVML every 5 ms when the bindings are
    present, else `nvidia-smi` every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits: sw_power_cap, hw_slowdown, sw_thermal, hw_thermal
    NVML_BITS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
                 ("sw_power_cap", 0x4))

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples: list[list[str]] = []
        self.source = "none"
        self._stop = threading.Event()
        self._t = None

    def _run_nvml(self, nv) -> bool:
        try:
            nv.nvmlInit()
            h = nv.nvmlDeviceGetHandleByIndex(self.gpu)
            smax = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        except Exception:
            return False
        self.source = "nvml"
        try:
            while not self._stop.is_set():
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.samples.append([str(self.gpu), str(sm), str(smax), "", ""] +
                                    ["Active" if bits & b else "Not Active" for _, b in self.NVML_BITS])
                self._stop.wait(0.005)
        except Exception:
            pass
        finally:
            try:
                nv.nvmlShutdown()
            except Exception:
                pass
        return True

    def _run(self):
        try:
            import pynvml as nv
        except ImportError:
            nv = None
        if nv is not None and self._run_nvml(nv):
            return
        self.source = "nvidia-smi"
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                if out.returncode == 0 and out.stdout.strip():
                    self.samples.append([c.strip() for c in out.stdout.strip().split(",")])
            except (OSError, subprocess.SubprocessError):
                return
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join(timeout=10)

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        smax = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for s in self.samples:
            for name, v in zip(names, s[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(self.samples), "source": self.source}


# ---------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------
def make_layer(dev, seed: int, M: int, bits: int = BITS):
    from mlxturbo_b200 import ops

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    mats = []
    for (N, K) in LAYER:
        wf = torch.randn((N, K), generator=g, device=dev, dtype=torch.float32) * 0.02
        wq, s, b = ops.quantize(wf, GS, bits, dtype=torch.bfloat16)
        del wf
        x = torch.randn((M, K), generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
        y = torch.empty((M, N), device=dev, dtype=torch.bfloat16)
        mats.append((x, wq, s, b, y, N, K))
    return mats


def run_layer(mats, bits=BITS):
    from mlxturbo_b200 import ops

    for (x, wq, s, b, y, N, K) in mats:
        ops.quantized_matmul(x, wq, s, b, group_size=GS, bits=bits, out=y)


def capture(fn):
    """A CUDA graph of fn() (kernels keep their programmatic-launch edges)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
        fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return g


def time_device(fn, steps: int, warmup: int, dist_on: bool) -> float:
    """ms per step: CUDA events on the launching stream, barrier + sync both sides, max over ranks."""
    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    if dist_on:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(steps):
        fn(i)
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    if dist_on:
        t = torch.tensor([ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
        torch.distributed.barrier()
    return ms / steps


def per_launch_us(mats, bits=BITS, reps: int = 20) -> list[float]:
    """Average device time of each projection's kernel: a graph of at least
    `reps` back-to-back launches per projection, rotating through enough
    copies of its weights that they span three L2 capacities, so every launch
    reads its matrix from HBM (two copies of a 3-18 MB matrix would stay in
    the 126 MB L2 and time L2 reads)."""
    from mlxturbo_b200 import ops

    out = []
    for j in range(len(mats[0])):
        x, wq, s, b, y, N, K = mats[0][j]
        nbytes = wq.numel() * 4 + (s.numel() + b.numel()) * 2
        copies = max(2, -(-3 * L2_BYTES // nbytes))
        bank = [(wq, s, b)] + [(wq.clone(), s.clone(), b.clone()) for _ in range(copies - 1)]
        n = max(reps, copies)

        def fn(j=j):
            for r in range(n):
                w_, s_, b_ = bank[r % copies]
                ops.quantized_matmul(x, w_, s_, b_, group_size=GS, bits=bits, out=y)
        g = capture(fn)
        for _ in range(3):
            g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(5):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        out.append(e0.elapsed_time(e1) * 1e3 / (5 * n))
        del g, bank
    return out


def cpu_baseline(sample_s: float = 12.0) -> dict:
    """The C oracle (fp32 dequantise-then-matmul, OpenMP) on the host cores."""
    import numpy as np

    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle as O

    rng = np.random.default_rng(0)
    N, K = 17408, 5120  # the largest projection of the layer
    codes = rng.integers(0, 2**32, size=(N, K // 8), dtype=np.uint64).astype(np.uint32)
    s = O.to_half(rng.uniform(0, 0.02, size=(N, K // GS)))
    b = O.to_half(rng.uniform(-0.01, 0.01, size=(N, K // GS)))
    x = O.to_half(rng.normal(0, 1, size=(1, K)))
    nt = O.num_threads()
    O.qmm(x, codes, s, b, GS, BITS, "bf16", nthreads=nt)  # warm
    t0 = time.perf_counter()
    reps = 0
    while time.perf_counter() - t0 < sample_s or reps < 2:
        O.qmm(x, codes, s, b, GS, BITS, "bf16", nthreads=nt)
        reps += 1
    dt = (time.perf_counter() - t0) / reps
    gbs = alg_bytes(1, N, K) / dt / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": nt, "kind": "port",
            "sample": f"{reps} passes of the 17408x5120 M=1 projection (50.2 MB, 4-bit g64) in {reps * dt:.1f} s"}


def prefill_bench(dev, pk, warmup, dist_on) -> dict:
    """x [M, 5120] against a 4-bit g64 W [17408, 5120], M in {512, 2048, 8192}."""
    from mlxturbo_b200 import ops

    N, K = 17408, 5120
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    wq, s, b = ops.quantize(torch.randn((N, K), generator=g, device=dev) * 0.02, GS, BITS, dtype=torch.bfloat16)
    out = {}
    for M in (512, 2048, 8192):
        x = torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16)
        y = torch.empty((M, N), device=dev, dtype=torch.bfloat16)
        steps = 10 if M >= 2048 else 20
        ms = time_device(lambda i: ops.quantized_matmul(x, wq, s, b, group_size=GS, bits=BITS, out=y), steps,
                         warmup, dist_on)
        tf = 2.0 * M * N * K / (ms * 1e-3) / 1e12
        out[f"M={M}"] = {"TFLOP/s": round(tf, 1), "ms": round(ms, 4), "frac_of_bf16_peak": round(tf / pk["bf16_tflops"], 4)}
        del x, y
    err = ops.device_error()
    out["device_error"] = err
    return out


def lm_head_bench(dev, pk, warmup, world) -> dict:
    """configs[2] lm_head: 8-bit g64 W [248320, 5120], M in {1, 4, 16}, column-sharded over the
    world (P = world; each rank holds 248320/P rows) with an all-gather of the logits when P > 1."""
    from mlxturbo_b200 import distributed as D
    from mlxturbo_b200 import ops

    N, K = 248320, 5120
    rank, _ = D._group_rank_world(None)
    a, z = D.shard_range(N, rank, world)
    n_local = z - a
    g = torch.Generator(device=dev)
    g.manual_seed(11 + rank)
    wq = torch.empty((n_local, K * 8 // 32), dtype=torch.int32, device=dev)
    s = torch.empty((n_local, K // GS), dtype=torch.bfloat16, device=dev)
    b = torch.empty_like(s)
    for r0 in range(0, n_local, 32768):  # quantise in slices to bound the fp32 staging buffer
        r1 = min(n_local, r0 + 32768)
        wq[r0:r1], s[r0:r1], b[r0:r1] = ops.quantize(torch.randn((r1 - r0, K), generator=g, device=dev) * 0.02,
                                                    GS, 8, dtype=torch.bfloat16)
    head = D.ColumnShardedLMHead(wq, s, b, None, GS, 8, None, None)
    out = {"P": world, "rows_per_gpu": n_local}
    for M in (1, 4, 16):
        x = torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16)
        y = torch.empty((M, n_local), device=dev, dtype=torch.bfloat16)
        ms_local = time_device(lambda i: ops.quantized_matmul(x, wq, s, b, group_size=GS, bits=8, out=y), 10,
                               warmup, world > 1)
        ms = time_device(lambda i: head(x), 10, warmup, world > 1) if world > 1 else ms_local
        gbs = alg_bytes(M, N, K, bits=8) / (ms * 1e-3) / 1e9
        gbs_local = alg_bytes(M, n_local, K, bits=8) / (ms_local * 1e-3) / 1e9
        ms_greedy = time_device(lambda i: head.argmax(x), 10, warmup, world > 1)
        out[f"M={M}"] = {"GB/s": round(gbs, 1), "ms": round(ms, 4), "frac_of_hbm_per_gpu": round(gbs / world / pk["hbm_gbs"], 4),
                         "local_kernel_ms": round(ms_local, 4), "local_kernel_frac_of_hbm": round(gbs_local / pk["hbm_gbs"], 4),
                         "greedy_on_shards_ms": round(ms_greedy, 4)}
        del x, y
    del head, wq, s, b
    if world > 1 and rank == 0:
        # the same matrix whole on one GPU (rank 0 alone, no collective): the P = 1 time that the sharded time
        # is a speedup over (strong scaling: the same rows split P ways)
        torch.cuda.empty_cache()
        wq = torch.empty((N, K * 8 // 32), dtype=torch.int32, device=dev)
        s = torch.empty((N, K // GS), dtype=torch.bfloat16, device=dev)
        b = torch.empty_like(s)
        for r0 in range(0, N, 32768):
            r1 = min(N, r0 + 32768)
            wq[r0:r1], s[r0:r1], b[r0:r1] = ops.quantize(torch.randn((r1 - r0, K), generator=g, device=dev) * 0.02,
                                                        GS, 8, dtype=torch.bfloat16)
        for M in (1, 4, 16):
            x = torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16)
            y = torch.empty((M, N), device=dev, dtype=torch.bfloat16)
            ms1 = time_device(lambda i: ops.quantized_matmul(x, wq, s, b, group_size=GS, bits=8, out=y), 10, warmup,
                              False)
            e = out[f"M={M}"]
            e["one_gpu_ms"] = round(ms1, 4)
            e["speedup_vs_one_gpu"] = round(ms1 / e["ms"], 3)
            e["efficiency_vs_one_gpu"] = round(ms1 / e["ms"] / world, 3)
        del wq, s, b, x, y
        torch.cuda.empty_cache()
    return out


def config0_bench(dev, pk, warmup, dist_on, cpu: bool) -> dict:
    """one quantized linear, x bf16 [1, 4096] ~ N(0,1) against W [11008, 4096] ~ N(0, 0.02)
    (4-bit g64), timed on the GPU (device-resident, eight weight copies rotating so each call reads
    HBM; and end to end through the public op with x and y in pinned host memory) and, on rank 0 at
    N = 1, on the host cores through the C oracle for the same shape."""
    from mlxturbo_b200 import ops

    N, K = 11008, 4096
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    copies = 8  # 8 x 25.4 MB > L2
    mats = []
    for _ in range(copies):
        wq, s, b = ops.quantize(torch.randn((N, K), generator=g, device=dev) * 0.02, GS, BITS, dtype=torch.bfloat16)
        mats.append((wq, s, b))
    x = torch.randn((1, K), generator=g, device=dev).to(torch.bfloat16)
    y = torch.empty((1, N), dtype=torch.bfloat16, device=dev)
    reps = 40

    def fn():
        for r in range(reps):
            wq, s, b = mats[r % copies]
            ops.quantized_matmul(x, wq, s, b, group_size=GS, bits=BITS, out=y)
    gr = capture(fn)
    ms = time_device(lambda i: gr.replay(), 5, warmup, dist_on) / reps
    del gr
    nbytes = alg_bytes(1, N, K)
    x_host = torch.empty((1, K), dtype=torch.bfloat16).normal_().pin_memory()
    y_host = torch.empty((1, N), dtype=torch.bfloat16).pin_memory()

    def e2e(i):
        wq, s, b = mats[i % copies]
        x.copy_(x_host, non_blocking=True)
        ops.quantized_matmul(x, wq, s, b, group_size=GS, bits=BITS, out=y)
        y_host.copy_(y, non_blocking=True)
    ms_e2e = time_device(e2e, 200, warmup, dist_on)

    def e2e_graph():  # the same calls captured, each with its transfers as kernels (ops.copy_)
        for r in range(reps):
            wq, s, b = mats[r % copies]
            ops.copy_(x, x_host)
            ops.quantized_matmul(x, wq, s, b, group_size=GS, bits=BITS, out=y)
            ops.copy_(y_host, y)
    gr = capture(e2e_graph)
    ms_e2e_graph = time_device(lambda i: gr.replay(), 5, warmup, dist_on) / reps
    del gr
    out = {"shape": "x[1,4096] . W[11008,4096]^T, 4-bit g64 bf16",
           "gpu": {"us": round(ms * 1e3, 2), "GB/s": round(nbytes / (ms * 1e-3) / 1e9, 1),
                   "frac_of_hbm": round(nbytes / (ms * 1e-3) / 1e9 / pk["hbm_gbs"], 4),
                   "how": f"CUDA graph of {reps} calls over {copies} weight copies (L2-cold), events"},
           "gpu_e2e": {"us": round(ms_e2e * 1e3, 2), "GB/s": round(nbytes / (ms_e2e * 1e-3) / 1e9, 1),
                       "how": "eager public op, pinned H2D of x and D2H of y per call"},
           "gpu_e2e_graph": {"us": round(ms_e2e_graph * 1e3, 2),
                             "GB/s": round(nbytes / (ms_e2e_graph * 1e-3) / 1e9, 1),
                             "how": f"CUDA graph of {reps} public-op calls over {copies} weight copies, each call "
                                    "with its pinned-host transfers of x and y as kernels (ops.copy_)"}}
    if cpu:
        import numpy as np

        sys.path.insert(0, os.path.join(REPO, "oracle"))
        import oracle as O

        wq, s, b = mats[0]
        w_h = wq.cpu().numpy().view(np.uint32)
        s_h = s.cpu().view(torch.int16).numpy().view(np.uint16)
        b_h = b.cpu().view(torch.int16).numpy().view(np.uint16)
        x_h = x.cpu().view(torch.int16).numpy().view(np.uint16)
        nt = O.num_threads()
        O.qmm(x_h, w_h, s_h, b_h, GS, BITS, "bf16", nthreads=nt)
        t0, n = time.perf_counter(), 0
        while time.perf_counter() - t0 < 3.0 or n < 3:
            O.qmm(x_h, w_h, s_h, b_h, GS, BITS, "bf16", nthreads=nt)
            n += 1
        dt = (time.perf_counter() - t0) / n
        out["cpu"] = {"us": round(dt * 1e6, 1), "GB/s": round(nbytes / dt / 1e9, 2), "cores": nt,
                      "kind": "port", "sample": f"{n} calls of the same shape"}
        out["gpu_e2e_over_cpu"] = round(dt / (ms_e2e * 1e-3), 1)
        out["gpu_e2e_graph_over_cpu"] = round(dt / (ms_e2e_graph * 1e-3), 1)
    del mats
    return out


STACK_LAYERS = 64


def stack64_bench(dev, pk, warmup, dist_on) -> dict:
    """configs[4]'s 64-layer stack: 64 random-init 4-bit g64 layers of the configs[1] shapes
    (64 distinct weight sets, 12.3 GB), run layer by layer (seven projections per layer, in order)
    at decode M = 1, verify M = 4 and prefill M = 512 / 2048.  The decode pass is the reference's
    own unit of decode cost ("mlp_all (64 layers)", mlxturbo/kernels/dispatch.py:228-229)."""
    from mlxturbo_b200 import ops

    g = torch.Generator(device=dev)
    g.manual_seed(4242)
    layers = []
    for _ in range(STACK_LAYERS):
        mats = []
        for (N, K) in LAYER:
            wq, s, b = ops.quantize(torch.randn((N, K), generator=g, device=dev) * 0.02, GS, BITS,
                                    dtype=torch.bfloat16)
            mats.append((wq, s, b, N, K))
        layers.append(mats)
    out = {"layers": STACK_LAYERS, "weight_GB": round(STACK_LAYERS * sum(alg_bytes(0, N, K) for N, K in LAYER) / 1e9, 2)}
    for M in (1, 4, 512, 2048):
        xs = [torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16) for (N, K) in LAYER]
        ys = [torch.empty((M, N), dtype=torch.bfloat16, device=dev) for (N, K) in LAYER]

        def one_pass():
            for mats in layers:
                for j, (wq, s, b, N, K) in enumerate(mats):
                    ops.quantized_matmul(xs[j], wq, s, b, group_size=GS, bits=BITS, out=ys[j])
        if M <= 16:
            gr = capture(one_pass)
            ms = time_device(lambda i: gr.replay(), 3, warmup, dist_on)
            del gr
        else:
            ms = time_device(lambda i: one_pass(), 2, 1, dist_on)
        nbytes = STACK_LAYERS * sum(alg_bytes(M, N, K) for N, K in LAYER)
        flops = STACK_LAYERS * sum(2.0 * M * N * K for N, K in LAYER)
        r = {"ms_per_pass": round(ms, 3), "GB/s": round(nbytes / (ms * 1e-3) / 1e9, 1),
             "TFLOP/s": round(flops / (ms * 1e-3) / 1e12, 1)}
        if M <= 16:
            r["frac_of_hbm"] = round(nbytes / (ms * 1e-3) / 1e9 / pk["hbm_gbs"], 4)
            r["mode"] = "one CUDA graph per pass"
        else:
            r["frac_of_bf16_peak"] = round(flops / (ms * 1e-3) / 1e12 / pk["bf16_tflops"], 4)
            r["mode"] = "eager"
        out[f"M={M}"] = r
        del xs, ys
    del layers
    torch.cuda.empty_cache()
    return out


MOE_E, MOE_TOPK, MOE_HIDDEN, MOE_INTER = 512, 10, 2048, 512


def moe_bench(dev, pk, warmup, world) -> dict:
    """512 experts, top-10, hidden 2048, intermediate 512, 4-bit g64 gate/up/down from
    N(0, 0.02); T tokens per GPU in {1, 8, 64, 256}; expert ids uniform (distinct per token) or
    Zipf(1.1) over a seeded expert permutation; expert-parallel over the world (E/P experts per rank).
    GB/s counts the distinct experts' weight bytes touched on this rank plus activations in and out.
    Each case cycles through R routings (R calls per graph) so that consecutive calls' experts span about
    twice the L2: the timings read the weights from HBM."""
    import numpy as np

    from mlxturbo_b200 import _lib
    from mlxturbo_b200 import distributed as D
    from mlxturbo_b200 import nn as qnn
    from mlxturbo_b200 import ops

    rank, _ = D._group_rank_world(None)
    a, z = D.shard_range(MOE_E, rank, world)
    E_l = z - a
    g = torch.Generator(device=dev)
    g.manual_seed(21 + rank)

    def bank(n_experts):
        glu_ = qnn.SwitchGLU(MOE_HIDDEN, MOE_INTER, n_experts, device=dev)
        for proj, (n, k) in ((glu_.gate_proj, (MOE_INTER, MOE_HIDDEN)), (glu_.up_proj, (MOE_INTER, MOE_HIDDEN)),
                             (glu_.down_proj, (MOE_HIDDEN, MOE_INTER))):
            for e0 in range(0, n_experts, 64):
                e1 = min(n_experts, e0 + 64)
                wq, sc, bi = ops.quantize(torch.randn(((e1 - e0) * n, k), generator=g, device=dev) * 0.02, GS, BITS,
                                          dtype=torch.bfloat16)
                proj.weight[e0:e1] = wq.view(e1 - e0, n, -1)
                proj.scales[e0:e1] = sc.view(e1 - e0, n, -1)
                proj.biases[e0:e1] = bi.view(e1 - e0, n, -1)
        return glu_

    glu = bank(E_l)
    ep = D.ExpertParallelSwitchGLU(glu, MOE_E, None)
    # P > 1: rank 0 also holds the whole bank and times each case on its own (no collective), the one-GPU
    # rate the expert-parallel rate is compared with (weak scaling: T tokens per GPU either way)
    ep1 = D.ExpertParallelSwitchGLU(bank(MOE_E), MOE_E, None) if world > 1 and rank == 0 else None
    expert_bytes = 3 * (MOE_INTER * MOE_HIDDEN * BITS // 8 + 2 * MOE_INTER * (MOE_HIDDEN // GS) * 2)
    rng = np.random.default_rng(5 + rank)
    zipf_p = 1.0 / np.arange(1, MOE_E + 1) ** 1.1
    zipf_p /= zipf_p.sum()
    perm = np.random.default_rng(99).permutation(MOE_E)  # the same skew on every rank
    out = {"P": world, "experts_per_gpu": E_l}
    for T in (1, 8, 64, 256):
        for dist_name in ("uniform", "zipf"):
            def routing():
                if dist_name == "uniform":
                    return np.stack([rng.choice(MOE_E, MOE_TOPK, replace=False) for _ in range(T)])
                return np.stack([perm[rng.choice(MOE_E, MOE_TOPK, replace=False, p=zipf_p)] for _ in range(T)])

            # R routings per case, called in turn, so that the experts R consecutive calls touch span
            # about twice the L2 (uniform: R = 15 at T = 1, 2 at T = 8, 1 above): each call reads its
            # experts from HBM, as a decode loop whose routing changes every token does
            # (from sizes only, so every rank takes the same number of collective steps)
            R = max(1, min(16, -(-2 * L2_BYTES // (min(MOE_E, world * T * MOE_TOPK) * expert_bytes))))
            sets = []
            for r in range(R):
                ids = routing()
                sets.append((ids, torch.from_numpy(ids.astype(np.int32)).to(dev),
                             torch.randn((T, MOE_HIDDEN), generator=g, device=dev).to(torch.bfloat16),
                             torch.softmax(torch.randn((T, MOE_TOPK), generator=g, device=dev), -1)))

            def calls(fn):
                for (_, idx, x, w) in sets:
                    fn(x, idx, w)

            fired = _lib.fire_counts().get("moe_glu_decode", 0)
            ms_eager = time_device(lambda i: calls(ep), 10, warmup, world > 1) / R
            path = "one launch" if _lib.fire_counts().get("moe_glu_decode", 0) > fired else "sort + four launches"
            padded = world > 1 and world * T * MOE_TOPK * MOE_HIDDEN * 2 <= D.ExpertParallelSwitchGLU.CAPACITY_BYTES
            ms, mode = ms_eager, "eager"  # exact split sizes go through the host: eager
            if world == 1 or padded:  # no host synchronisation inside: one CUDA graph of the R block calls
                try:
                    gr = capture(lambda: calls(ep))
                except RuntimeError as err:  # a collective the runtime refuses to capture: keep eager
                    mode = f"eager (capture refused: {str(err).splitlines()[0][:80]})"
                else:
                    ms = time_device(lambda i: gr.replay(), 20, warmup, world > 1) / R
                    del gr  # before the process group goes away (it may hold NCCL work)
                    mode = "graph"
            # weight bytes of the distinct experts every rank touched (summed over ranks), mean over the R calls
            touched_sum = 0.0
            for (ids, idx, _, _) in sets:
                if world > 1:
                    allids = [torch.empty_like(idx) for _ in range(world)]
                    torch.distributed.all_gather(allids, idx)
                    touched_sum += len(np.unique(torch.cat(allids).cpu().numpy()))
                else:
                    touched_sum += len(np.unique(ids))
            touched = touched_sum / R
            nbytes = touched * expert_bytes + world * T * MOE_HIDDEN * 2 * 2
            gbs = nbytes / (ms * 1e-3) / 1e9
            e = {"us": round(ms * 1e3, 1), "us_eager": round(ms_eager * 1e3, 1), "mode": mode, "path": path,
                 "GB/s": round(gbs, 1), "frac_of_hbm_per_gpu": round(gbs / world / pk["hbm_gbs"], 4),
                 "distinct_experts": round(touched, 1), "routings_rotated": R,
                 "tokens_per_s": round(world * T / (ms * 1e-3), 1)}
            if ep1 is not None:
                gr1 = capture(lambda: calls(ep1.forward_local))
                ms1 = time_device(lambda i: gr1.replay(), 20, warmup, False) / R
                del gr1
                e["one_gpu_us"] = round(ms1 * 1e3, 1)
                e["efficiency_vs_one_gpu"] = round(ms1 / ms, 3)  # (P*T/ms) / (T/ms1) / P
            out[f"T={T} {dist_name}"] = e
    del ep, glu, ep1
    return out


# ---------------------------------------------------------------------------
# small self-contained cases for ncu captures (three calls of one op)
# ---------------------------------------------------------------------------
CASES_HELP = """--case qmv N K M [bits] | qmv_i8 N K M [bits] | prefill M N K | moe T [E] | layer
  qmv: the dispatched decode path; qmv_i8: the integer-MMA kernel called directly; prefill: the tensor-core
  kernel; moe: the 512-expert top-10 block on one GPU; layer: the seven decode projections at M=1."""


def run_case(argv: list[str]) -> None:
    from mlxturbo_b200 import ops

    dev = torch.device("cuda:0")
    kind = argv[0]
    if kind == "layer":
        mats = []
        for N, K in LAYER:
            wq, s, b = ops.quantize(torch.randn(N, K, device=dev) * 0.02, GS, BITS)
            mats.append((torch.randn(1, K, device=dev).bfloat16(), wq, s, b))
        for _ in range(3):
            for x, wq, s, b in mats:
                y = ops.quantized_matmul(x, wq, s, b, group_size=GS, bits=BITS)
    elif kind == "moe":
        from mlxturbo_b200 import distributed as D
        from mlxturbo_b200 import nn as qnn

        T, E = int(argv[1]), int(argv[2]) if len(argv) > 2 else MOE_E
        glu = qnn.SwitchGLU(MOE_HIDDEN, MOE_INTER, E, device=dev)
        for proj, (n, k) in ((glu.gate_proj, (MOE_INTER, MOE_HIDDEN)), (glu.up_proj, (MOE_INTER, MOE_HIDDEN)),
                             (glu.down_proj, (MOE_HIDDEN, MOE_INTER))):
            wq, s, b = ops.quantize(torch.randn((E * n, k), device=dev) * 0.02, GS, BITS)
            proj.weight.copy_(wq.view(E, n, -1))
            proj.scales.copy_(s.view(E, n, -1))
            proj.biases.copy_(b.view(E, n, -1))
        ep = D.ExpertParallelSwitchGLU(glu, E, None)
        g = torch.Generator(device=dev)
        g.manual_seed(0)
        idx = torch.stack([torch.randperm(E, generator=g, device=dev)[:MOE_TOPK] for _ in range(T)]).to(torch.int32)
        w = torch.softmax(torch.randn((T, MOE_TOPK), device=dev), -1)
        x = torch.randn((T, MOE_HIDDEN), device=dev).to(torch.bfloat16)
        for _ in range(3):
            y = ep(x, idx, w)
    elif kind in ("qmv", "qmv_i8", "prefill"):
        if kind == "prefill":
            M, N, K, bits = int(argv[1]), int(argv[2]), int(argv[3]), BITS
        else:
            N, K, M = int(argv[1]), int(argv[2]), int(argv[3])
            bits = int(argv[4]) if len(argv) > 4 else BITS
        wq, s, b = ops.quantize(torch.randn(N, K, device=dev) * 0.02, GS, bits)
        x = torch.randn(M, K, device=dev).bfloat16()
        for _ in range(3):
            if kind == "qmv_i8":
                y = ops.qmv_i8(x, wq, s, b, bits=bits)
            else:
                y = ops.quantized_matmul(x, wq, s, b, bits=bits)
    else:
        raise SystemExit(f"unknown case {kind!r}\n{CASES_HELP}")
    torch.cuda.synchronize()
    print("ok", float(y.float().abs().mean()), ops.device_error())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--case", nargs="+", metavar="ARG", help="run one small profiling case and exit: " + CASES_HELP)
    args = ap.parse_args()
    if args.case:
        run_case(args.case)
        return
    warmup = max(3, args.warmup)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    layer_bytes = sum(alg_bytes(1, N, K) for N, K in LAYER)
    config = {"workload": "decode qmv M=1, 27B-class layer (7 projections), 4-bit g64 bf16",
              "shapes_NxK": [f"{N}x{K}" for N, K in LAYER], "M": 1, "bits": BITS, "group_size": GS,
              "weight_copies": 2, "l2": "inputs larger than L2 (2 x 191.7 MB weight sets alternate)",
              "parallelism": f"replicas x{args.gpus}"}

    if args.impl == "reference":
        if rank != 0:
            return
        cb = cpu_baseline(sample_s=6.0)
        values = [cb["value"]]
        for _ in range(args.steps - 1 if args.steps > 1 else 0):
            values.append(cpu_baseline(sample_s=2.0)["value"])
        v = statistics.median(values)
        line = {"impl": "reference", "metric": "qmv weight-stream GB/s (decode layer, M=1)", "value": v,
                "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": warmup,
                "ms_per_step": round(layer_bytes / (v * 1e9) * 1e3, 3), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "u4 codes, fp32 accumulate", "data": "synthetic",
                "config": config,
                "cpu_baseline": {**cb, "value": v,
                                 "note": "reference CPU path (MLX CPU backend) unavailable here; C oracle port"},
                "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    dist_on = world > 1
    if dist_on:
        import datetime

        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local if dist_on else 0)
    torch.cuda.set_device(dev)
    from mlxturbo_b200 import _lib

    layers = [make_layer(dev, 1234 + rank * 7 + c, 1) for c in range(2)]
    torch.cuda.synchronize()

    # ---- headline: device-resident, the layer step replayed from CUDA graphs ----
    graphs = [capture(lambda c=c: run_layer(layers[c])) for c in range(2)]
    fire0 = _lib.fire_counts()["qmv"]
    # the clock record covers the timed steps and, on both sides of them, untimed
    # replays of the same step (a fixed count, so ranks stay in step): the timed
    # region alone is a few milliseconds, shorter than one sampling interval
    busy = 4000

    def keep_busy():
        for i in range(busy):
            graphs[i % 2].replay()
        torch.cuda.synchronize()

    with ClockSampler(torch.cuda.current_device()) as clk:
        keep_busy()
        ms = time_device(lambda i: graphs[i % 2].replay(), args.steps, warmup, dist_on)
        keep_busy()
    # kernel launches per step: one per projection, plus the activation-plane
    # prep launch where the integer-MMA kernel takes the matrix (>= 12 MiB of codes)
    per_step = sum(2 if N * K * BITS // 8 >= I8_MIN_BYTES else 1 for N, K in LAYER)
    launches_timed = per_step * args.steps
    value = layer_bytes * world / (ms * 1e-3) / 1e9

    # ---- per-kernel launch durations (graphs of back-to-back launches) ---------
    k_us = per_launch_us(layers)
    pk = peaks()
    # dominant kernel: the integer-MMA decode kernel (with its prep launch) on the
    # five projections of >= 12 MiB of codes, which take most of the step
    big = [i for i, (N, K) in enumerate(LAYER) if N * K * BITS // 8 >= I8_MIN_BYTES]
    big_bytes = sum(alg_bytes(1, *LAYER[i]) for i in big)
    achieved = big_bytes / (sum(k_us[i] for i in big) * 1e-6) / 1e9
    layer_achieved = layer_bytes / (sum(k_us) * 1e-6) / 1e9
    traffic = [NCU_TRAFFIC_BYTES.get(f"{LAYER[i][0]}x{LAYER[i][1]}") for i in big]
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved / pk["hbm_gbs"], 4),
                "traffic": (round(sum(traffic) / len(traffic)) if all(traffic) else None),
                "traffic_note": "dram read+write bytes per launch (prep + main), mean over those projections, "
                                "from one ncu capture (profiles/decode_layer_launches.md); algorithmic bytes per "
                                f"launch {round(big_bytes / len(big))}",
                "kernel": "qmv_i8_kernel<4,64,bf16,MP=1> + qmv_i8_prep_kernel (6144x5120, 5120x6144, "
                          "17408x5120 x2, 5120x17408)",
                "layer": {"achieved": round(layer_achieved, 1), "frac": round(layer_achieved / pk["hbm_gbs"], 4),
                          "kernels": "1024x5120 x2: qmv_kernel (CTA per tile); the rest: qmv_i8_kernel + prep"},
                "per_launch_us": {f"{N}x{K}#{i}": round(t, 2) for i, ((N, K), t) in enumerate(zip(LAYER, k_us))},
                "per_launch_how": "CUDA events over a graph of back-to-back launches of one projection, rotating "
                                  "weight copies that span 3x the L2, so each launch reads HBM",
                "peak_source": pk["source"]}
    del graphs

    # ---- HBM floor for one launch per projection --------------------------------
    # the same byte counts read by a plain streaming kernel, launched and timed
    # exactly like the decode layer (PDL, CUDA graphs, two alternating copies)
    lib = _lib.load()
    sizes = [(alg_bytes(1, N, K) + 15) // 16 * 16 for N, K in LAYER]
    fbuf = torch.empty(2 * sum(sizes), dtype=torch.uint8, device=dev)
    sink = torch.empty(4096, dtype=torch.uint8, device=dev)

    def floor_layer(c):
        off = c * sum(sizes)
        stream = torch.cuda.current_stream(dev).cuda_stream
        for nb in sizes:
            _lib.check(lib.qmm_stream_read(fbuf.data_ptr() + off, nb, 148 * 4, sink.data_ptr(), stream), "stream_read")
            off += nb

    fgraphs = [capture(lambda c=c: floor_layer(c)) for c in range(2)]
    ms_floor = time_device(lambda i: fgraphs[i % 2].replay(), args.steps, warmup, dist_on)
    del fgraphs, fbuf
    roofline["floor"] = {"layer_ms": round(ms_floor, 4), "GB/s": round(layer_bytes / (ms_floor * 1e-3) / 1e9, 1),
                         "what": "plain streaming reads of the seven projections' algorithmic bytes, one launch "
                                 "each, PDL + CUDA graph (qmm_stream_read)"}
    roofline["frac_of_floor"] = round(ms_floor / ms, 4)

    # ---- end to end through the public op with host buffers ---------------------
    # Each step copies the seven projections' activations from pinned host
    # memory in one transfer (one pinned buffer, the projections' rows back to
    # back), runs the public op on views of the device buffer, and copies all
    # seven outputs back in one transfer: the copies a decode loop makes per
    # layer when its inputs and outputs live on the host.
    Ks = [K for (N, K) in LAYER]
    Ns = [N for (N, K) in LAYER]
    xoff = [sum(Ks[:j]) for j in range(len(LAYER))]
    yoff = [sum(Ns[:j]) for j in range(len(LAYER))]
    xs_host = [torch.empty(sum(Ks), dtype=torch.bfloat16).normal_().pin_memory() for _ in range(2)]
    ys_host = torch.empty(sum(Ns), dtype=torch.bfloat16).pin_memory()
    h2d = sum(Ks) * 2
    d2h = sum(Ns) * 2
    x_dev = torch.empty(sum(Ks), dtype=torch.bfloat16, device=dev)
    y_dev = torch.empty(sum(Ns), dtype=torch.bfloat16, device=dev)
    x_views = [x_dev[xoff[j]:xoff[j] + Ks[j]].view(1, Ks[j]) for j in range(len(LAYER))]
    y_views = [y_dev[yoff[j]:yoff[j] + Ns[j]].view(1, Ns[j]) for j in range(len(LAYER))]

    def e2e_step(i):
        from mlxturbo_b200 import ops

        mats = layers[i % 2]
        ops.copy_(x_dev, xs_host[i % 2])  # pinned host -> device, one kernel
        for j, (x, wq, s, b, y, N, K) in enumerate(mats):
            ops.quantized_matmul(x_views[j], wq, s, b, group_size=GS, bits=BITS, out=y_views[j])
        ops.copy_(ys_host, y_dev)  # device -> pinned host, one kernel

    def e2e_step_copy_engine(i):
        from mlxturbo_b200 import ops

        mats = layers[i % 2]
        x_dev.copy_(xs_host[i % 2], non_blocking=True)
        for j, (x, wq, s, b, y, N, K) in enumerate(mats):
            ops.quantized_matmul(x_views[j], wq, s, b, group_size=GS, bits=BITS, out=y_views[j])
        ys_host.copy_(y_dev, non_blocking=True)

    # The step as a decode loop runs it: captured once in a CUDA graph (the public-op calls and both
    # transfers) and replayed per step; eager calls, with kernel and with copy-engine transfers, beside it.
    e2e_graphs = [capture(lambda c=c: e2e_step(c)) for c in range(2)]
    ms_e2e = time_device(lambda i: e2e_graphs[i % 2].replay(), args.steps, warmup, dist_on)
    del e2e_graphs
    e2e_value = layer_bytes * world / (ms_e2e * 1e-3) / 1e9
    ms_e2e_eager = time_device(e2e_step, args.steps, warmup, dist_on)
    ms_e2e_ce = time_device(e2e_step_copy_engine, args.steps, warmup, dist_on)

    # ---- verify-width sweep and 8-bit lm_head (extra context) -----------------
    sweep = {}
    for M in (2, 4, 8, 16):
        lm = [make_layer(dev, 99 + c, M) for c in range(2)]
        gm = [capture(lambda c=c: run_layer(lm[c])) for c in range(2)]
        m_ms = time_device(lambda i: gm[i % 2].replay(), max(10, args.steps // 2), warmup, dist_on)
        b_m = sum(alg_bytes(M, N, K) for N, K in LAYER)
        sweep[f"M={M}"] = {"GB/s": round(b_m / (m_ms * 1e-3) / 1e9, 1), "ms": round(m_ms, 4),
                           "frac_of_hbm": round(b_m / (m_ms * 1e-3) / 1e9 / pk["hbm_gbs"], 4)}
        del lm, gm
    torch.cuda.empty_cache()
    extra = {"verify_sweep": sweep,
             "prefill": prefill_bench(dev, pk, warmup, dist_on),
             "lm_head_8bit_column_sharded": lm_head_bench(dev, pk, warmup, world)}
    torch.cuda.empty_cache()
    extra["moe_gather_expert_parallel"] = moe_bench(dev, pk, warmup, world)
    torch.cuda.empty_cache()
    extra["config0_single_linear"] = config0_bench(dev, pk, warmup, dist_on,
                                                   cpu=(rank == 0 and world == 1 and not args.no_cpu))
    torch.cuda.empty_cache()
    extra["stack64_layer_by_layer"] = stack64_bench(dev, pk, warmup, dist_on)

    line = {"metric": "qmv weight-stream GB/s (decode layer, M=1)", "value": round(value, 1), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights through MLX affine quantisation)",
            "config": config, "roofline": roofline,
            "e2e": {"value": round(e2e_value, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": round(ms_e2e, 4),
                    "mode": "public-op calls (ops.quantized_matmul through the PyTorch operator) captured once in a "
                            "CUDA graph and replayed per step; every step copies the seven activations from pinned "
                            "host memory to the device and the seven outputs back, each transfer one kernel "
                            "(ops.copy_)",
                    "eager_value": round(layer_bytes * world / (ms_e2e_eager * 1e-3) / 1e9, 1),
                    "eager_ms_per_step": round(ms_e2e_eager, 4),
                    "eager_copy_engine_value": round(layer_bytes * world / (ms_e2e_ce * 1e-3) / 1e9, 1),
                    "eager_copy_engine_ms_per_step": round(ms_e2e_ce, 4)},
            "gpu_launches": int(launches_timed), "clocks": clk.summary(),
            "frac_of_nominal_8TBs": round(value / world / 8000.0, 4), **extra}
    if rank == 0 and world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline()
    if dist_on:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
