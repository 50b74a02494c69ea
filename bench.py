"""Benchmark of the quantized-linear hot path on B200.

One step = one pass of the hot path over one batch of synthetic, seeded input. Workloads
(`--workload`, default `int8`, the configuration the headline metric is quoted on):

  int8         INT8 W8A8 layer M=256 K=4096 N=11008: int8 activations with per-token fp32
               scales, int8 weights with per-channel fp32 scales, exact int32 accumulation,
               bf16 out (w8a8_block_int8_matmul, block [1, 4096]). Ranks run independent
               replicas (weak scaling). HBM-bound: roofline in GB/s.
  awq_prefill  AWQ W4A16 layer M=2048 K=8192 N=28672 bf16, group 128, output columns sharded
               over the ranks, the all-gather of the bf16 output inside the GEMM epilogue
               (TOB_BENCH_GATHER=nccl: an NCCL all-gather after it) (strong scaling).
               Tensor-bound: roofline in TFLOP/s.
  fp8          FP8 layer M=N=K=8192 from bf16: per-token dynamic quantisation of A, tensor-wide
               quantisation of B, per-token x per-tensor e4m3 GEMM to bf16 (replicas).
  fp8_block    FP8 block-scaled GEMM M=4096 N=K=7168, [128, 128] scale blocks, bf16 out (replicas).
  dense_bf16   dense bf16 GEMM M=2048 K=8192 N=28672 (the prefill layer, unquantized; replicas).
  awq_gemv     AWQ W4A16 decode GEMV x[1, 4096] fp16 @ int4 [4096, 4096], group 128 (replicas).
  dense_gemv   dense fp16 GEMV y = A[4096, 4096] @ x (the decode GEMV, unquantized; replicas).
  decode       32 layers x {qkv 4096->6144, o 4096->4096, gate_up 4096->28672, down 14336->4096}
               AWQ int4 group 128, fp16, M tokens (--decode-m, default 16), silu_and_mul of the
               gate_up output (in its kernel) into down; N-sharded with an all-gather after
               every linear.
               HBM GB/s over the weight bytes.

Reported on one JSON line (rank 0):
  value      device throughput of K steps replayed from a CUDA graph, inputs resident in HBM,
             weights rotated over buffers larger than L2 where a step's working set is smaller
             than L2; total over ranks; time = max over ranks.
  e2e        the same metric through the public API with host buffers: each step copies its
             activations (and their scales) from pinned host memory and reads the output back.
  roofline   the dominant kernel's algorithmic bytes or FLOPs per launch / its mean duration
             (CUDA events on its stream, timed in a graph of launches of that kernel alone),
             against MEASURED_PEAKS.json; traffic = DRAM bytes per launch from profiles/.
  cpu_baseline  the reference algorithm restated on torch CPU tensors on all host cores.
`--impl reference` runs that CPU arm alone (rank 0) on the same metric, config and unit.
Launch: python bench.py [--gpus N --steps K --warmup W]; N>1 under torch.distributed.run.
"""

from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

METRIC = "W4A16/W8A8/FP8 GEMM TFLOP/s & GEMV HBM GB/s, % of B200 roofline, 1-8 GPU"


def measured_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except Exception:
            pass
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def profile_traffic(name: str):
    """DRAM bytes per launch of a workload's dominant kernel from its committed ncu summary."""
    path = ROOT / "profiles" / name
    if not path.exists():
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9]+)", path.read_text())
    return int(m.group(1)) if m else None


class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons)}


def graph_of(fn, reps: int):
    """Captures `reps` calls of fn(i) into one CUDA graph (after an eager warm-up on a side
    stream, as torch requires)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn(0)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(reps):
            fn(i)
    return g


def timed_graph_ms(fn, reps: int, warmup: int, dist=None, clock_index=None):
    """Mean ms per call of fn over a graph of `reps` calls (max over ranks); optionally samples
    clocks while the GPU is kept busy around the timed replay."""
    g = graph_of(fn, reps)
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = ClockSampler(clock_index) if clock_index is not None else None
    if clk is not None:
        clk.__enter__()
        soak = time.perf_counter() + 1.0  # load the GPU so the 100 ms samples see the timed state
        while time.perf_counter() < soak:
            g.replay()
            torch.cuda.synchronize()
    ev0.record()
    g.replay()
    ev1.record()
    torch.cuda.synchronize()
    if clk is not None:
        soak = time.perf_counter() + 0.3
        while time.perf_counter() < soak:
            g.replay()
            torch.cuda.synchronize()
        clk.__exit__(None, None, None)
    if dist is not None:
        dist.barrier()
    ms = ev0.elapsed_time(ev1)
    if dist is not None:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    del g
    return ms / reps, (clk.summary() if clk is not None else None)


# ====================================================================== workloads
class Int8Layer:
    name = "int8"
    unit = "TOPS"
    dtype = "int8"
    bound = "hbm"
    scaling = "weak"
    profile = "w8a8_int8_m256_k4096_n11008.md"
    M, K, N = 256, 4096, 11008
    data = ("synthetic (seeded uniform int8 in [-127,127]; scales U(0.005,0.05) per token, "
            "U(0.001,0.01) per channel)")
    launches_per_step = 1

    def __init__(self, dev, rank, world):
        import tileops_b200 as tob

        self.tob = tob
        tob.set_launch_overlap(True)  # call i+1 streams its weights while call i finishes
        M, K, N = self.M, self.K, self.N
        self.kernel_bytes = M * K + N * K + 4 * M + 4 * N + 2 * M * N
        g = torch.Generator().manual_seed(1234 + 2 + rank)
        a_cpu = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8)
        a_s_cpu = torch.rand(M, 1, generator=g) * 0.045 + 0.005
        self.b_s = (torch.rand(N, 1, generator=g) * 0.009 + 0.001).to(dev)
        # 6 x 45 MB > 126 MB L2: every step streams its weights from HBM
        self.weights = [torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8).to(dev)
                        for _ in range(6)]
        self.a, self.a_s = a_cpu.to(dev), a_s_cpu.to(dev)
        self.a_host, self.a_s_host = a_cpu.pin_memory(), a_s_cpu.pin_memory()
        self.out_host = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
        self.dev = dev

    def step(self, i):
        self.tob.w8a8_block_int8_matmul(self.a, self.weights[i % 6], self.a_s, self.b_s,
                                        [1, self.K], output_dtype=torch.bfloat16)

    kernel_step = step

    def e2e_step(self, i):
        a = self.a_host.to(self.dev, non_blocking=True)
        a_s = self.a_s_host.to(self.dev, non_blocking=True)
        c = self.tob.w8a8_block_int8_matmul(a, self.weights[i % 6], a_s, self.b_s, [1, self.K],
                                            output_dtype=torch.bfloat16)
        self.out_host.copy_(c, non_blocking=True)

    def h2d_d2h(self):
        return self.a_host.numel() + 4 * self.a_s_host.numel(), 2 * self.out_host.numel()

    def total_units(self, world):
        return world * 2 * self.M * self.N * self.K / 1e12  # tera-ops per step, whole job

    def roofline_units(self):
        return "hbm", self.kernel_bytes

    def config(self, world):
        return {"workload": "int8_w8a8_gemm M=256 K=4096 N=11008 per-token x per-channel "
                            "scales -> bf16", "M": self.M, "K": self.K, "N": self.N,
                "parallelism": f"replicas x{world}",
                "l2": "rotating weights: 6 x 45 MB buffers > 126 MB L2",
                "launch_overlap": "programmatic dependent launch between consecutive calls"}

    @classmethod
    def cpu_reference(cls, threads):
        from oracle import int8 as oi8

        torch.set_num_threads(threads)
        g = torch.Generator().manual_seed(1234 + 2)
        M, K, N = cls.M, cls.K, cls.N
        a = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8)
        b = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
        a_s = torch.rand(M, 1, generator=g) * 0.045 + 0.005
        b_s = torch.rand(N, 1, generator=g) * 0.009 + 0.001
        run = lambda: oi8.block_matmul_reference_cpu_torch(a, b, a_s, b_s, (1, K), torch.bfloat16)  # noqa: E731
        return run, 2 * M * N * K / 1e12, ("the full layer per pass; torch CPU fp32 dequant + "
                                           "fp32 GEMM (reference algorithm)")


class AwqPrefill:
    name = "awq_prefill"
    unit = "TFLOP/s"
    dtype = "bf16"
    bound = "tensor"
    scaling = "strong"
    profile = "awq_prefill_m2048_k8192_n28672.md"
    M, K, N, G = 2048, 8192, 28672, 128
    data = "synthetic (seeded random packed int4 weights and zeros, scales U(0.002,0.02), x N(0,1))"
    launches_per_step = 1

    def __init__(self, dev, rank, world):
        import tileops_b200 as tob
        from tileops_b200 import sharded

        self.tob, self.sharded = tob, sharded
        M, K, N, G = self.M, self.K, self.N, self.G
        n_loc = N // world
        g = torch.Generator().manual_seed(1234 + 3 + 100 * rank)  # this rank's column shard
        self.qw = torch.randint(-2 ** 31, 2 ** 31 - 1, (K, n_loc // 8), generator=g,
                                dtype=torch.int32).to(dev)
        self.qz = torch.randint(-2 ** 31, 2 ** 31 - 1, (K // G, n_loc // 8), generator=g,
                                dtype=torch.int32).to(dev)
        self.s = (torch.rand(K // G, n_loc, generator=g) * 0.018 + 0.002).bfloat16().to(dev)
        gx = torch.Generator().manual_seed(1234 + 3)  # the same activations on every rank
        x_cpu = torch.randn(M, K, generator=gx).bfloat16()
        self.x = x_cpu.to(dev)
        self.x_host = x_cpu.pin_memory()
        self.out_host = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
        self.flops_per_rank = 2 * M * n_loc * K
        self.dev, self.world = dev, world
        self.gather = os.environ.get("TOB_BENCH_GATHER", "fused")
        self.layer = sharded.ShardedAWQLinear.from_shard(self.qw, self.s, self.qz)

    def _layer(self, x):
        if self.world > 1 and self.gather == "fused":
            return self.layer.gathered(x)
        y = self.tob.awq_gemm(x, self.qw, self.s, self.qz, 1)
        return self.sharded.gather_columns(y) if self.world > 1 else y

    def close(self):
        self.layer.close()

    def step(self, i):
        self._layer(self.x)

    def kernel_step(self, i):
        self.tob.awq_gemm(self.x, self.qw, self.s, self.qz, 1)

    def e2e_step(self, i):
        x = self.x_host.to(self.dev, non_blocking=True)
        self.out_host.copy_(self._layer(x), non_blocking=True)

    def h2d_d2h(self):
        return 2 * self.x_host.numel(), 2 * self.out_host.numel()

    def total_units(self, world):
        return 2 * self.M * self.N * self.K / 1e12  # the whole layer per step

    def roofline_units(self):
        return "tensor", self.flops_per_rank

    def config(self, world):
        gather = ("gather fused into the GEMM epilogue (tiles stored into every rank's "
                  "output over NVLink, one NCCL barrier)" if self.gather == "fused" else
                  "NCCL all-gather after the GEMM")
        return {"workload": "awq_w4a16_prefill M=2048 K=8192 N=28672 bf16 group 128, output "
                            "columns sharded over ranks",
                "gather": gather if world > 1 else None,
                "M": self.M, "K": self.K, "N": self.N, "group_size": self.G,
                "parallelism": f"tp{world} (N-sharded)",
                "l2": "per step 117 MB of bf16 output plus weights and activations > L2"}

    @classmethod
    def cpu_reference(cls, threads):
        from oracle import awq as oawq

        torch.set_num_threads(threads)
        M, K, G = cls.M, cls.K, cls.G
        n = 1792  # one 16th of the output columns per pass
        g = torch.Generator().manual_seed(1234 + 3)
        x = torch.randn(M, K, generator=g).bfloat16()
        qw = torch.randint(-2 ** 31, 2 ** 31 - 1, (K, n // 8), generator=g, dtype=torch.int32)
        qz = torch.randint(-2 ** 31, 2 ** 31 - 1, (K // G, n // 8), generator=g, dtype=torch.int32)
        s = (torch.rand(K // G, n, generator=g) * 0.018 + 0.002).bfloat16()
        run = lambda: oawq.gemm_reference_cpu_torch(x, qw, s, qz, G)  # noqa: E731
        return run, 2 * M * n * K / 1e12, ("N=1792 of 28672 columns per pass (full M, K); torch "
                                           "CPU int64 unpack + dequant + bf16 matmul (reference "
                                           "algorithm)")


class Fp8Layer:
    name = "fp8"
    unit = "TFLOP/s"
    dtype = "e4m3"
    bound = "tensor"
    scaling = "weak"
    profile = "fp8_m8192_n8192_k8192.md"
    M = N = K = 8192
    data = "synthetic (seeded bf16 N(0,1))"
    launches_per_step = 4  # group quant, amax, tensor quant, GEMM

    def __init__(self, dev, rank, world):
        import tileops_b200 as tob

        self.tob = tob
        g = torch.Generator().manual_seed(1234 + 4 + rank)
        A_cpu = torch.randn(self.M, self.K, generator=g).bfloat16()
        self.B = torch.randn(self.N, self.K, generator=g).bfloat16().to(dev)
        self.A = A_cpu.to(dev)
        self.A_host = A_cpu.pin_memory()
        self.out_host = torch.empty(self.M, self.N, dtype=torch.bfloat16).pin_memory()
        self.dev = dev
        self.flops = 2 * self.M * self.N * self.K
        qa, sa = tob.per_token_group_quant_fp8(self.A, self.K)
        qb, sb = tob.input_to_float8(self.B)
        self.qa, self.sa, self.qb, self.sb = qa, sa, qb, sb.reshape(1, 1)

    def _layer(self, A):
        qa, sa = self.tob.per_token_group_quant_fp8(A, self.K)
        qb, sb = self.tob.input_to_float8(self.B)
        return self.tob.w8a8_block_fp8_matmul(qa, qb, sa, sb.reshape(1, 1), [self.N, self.K],
                                              output_dtype=torch.bfloat16)

    def step(self, i):
        self._layer(self.A)

    def kernel_step(self, i):
        self.tob.w8a8_block_fp8_matmul(self.qa, self.qb, self.sa, self.sb, [self.N, self.K],
                                       output_dtype=torch.bfloat16)

    def e2e_step(self, i):
        A = self.A_host.to(self.dev, non_blocking=True)
        self.out_host.copy_(self._layer(A), non_blocking=True)

    def h2d_d2h(self):
        return 2 * self.A_host.numel(), 2 * self.out_host.numel()

    def total_units(self, world):
        return world * self.flops / 1e12

    def roofline_units(self):
        return "tensor", self.flops

    def config(self, world):
        return {"workload": "fp8_e4m3 layer M=N=K=8192: per-token dynamic quant of A, "
                            "tensor-wide quant of B, scaled GEMM -> bf16",
                "M": self.M, "N": self.N, "K": self.K, "parallelism": f"replicas x{world}",
                "l2": "A, B, their fp8 copies and the output are 512 MB per step > L2"}

    @classmethod
    def cpu_reference(cls, threads):
        from oracle import fp8 as ofp8

        torch.set_num_threads(threads)
        m = 512  # 512 of the 8192 rows of A per pass (B quantised in full)
        g = torch.Generator().manual_seed(1234 + 4)
        A = torch.randn(m, cls.K, generator=g).bfloat16()
        B = torch.randn(cls.N, cls.K, generator=g).bfloat16()
        run = lambda: ofp8.layer_reference_cpu_torch(A, B)  # noqa: E731
        return run, 2 * m * cls.N * cls.K / 1e12, ("M=512 of 8192 rows per pass (full N, K; B "
                                                   "quantised in full); torch CPU quantise + fp32 "
                                                   "dequant GEMM (reference algorithm)")


class DenseBf16:
    name = "dense_bf16"
    unit = "TFLOP/s"
    dtype = "bf16"
    bound = "tensor"
    scaling = "weak"
    profile = "dense_bf16_m2048_k8192_n28672.md"
    M, K, N = 2048, 8192, 28672
    data = "synthetic (seeded bf16 N(0,1) weights, activations N(0, 1/K))"
    launches_per_step = 1

    def __init__(self, dev, rank, world):
        import tileops_b200 as tob

        self.tob = tob
        M, K, N = self.M, self.K, self.N
        g = torch.Generator().manual_seed(1234 + 7 + rank)
        a_cpu = (torch.randn(M, K, generator=g) / K ** 0.5).bfloat16()
        # 2 x 470 MB of weights > 126 MB L2
        self.bs = [torch.randn(K, N, generator=g).bfloat16().to(dev) for _ in range(2)]
        self.a = a_cpu.to(dev)
        self.a_host = a_cpu.pin_memory()
        self.out_host = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
        self.dev = dev
        self.flops = 2 * M * N * K

    def step(self, i):
        self.tob.gemm(self.a, self.bs[i % 2])

    kernel_step = step

    def e2e_step(self, i):
        a = self.a_host.to(self.dev, non_blocking=True)
        self.out_host.copy_(self.tob.gemm(a, self.bs[i % 2]), non_blocking=True)

    def h2d_d2h(self):
        return 2 * self.a_host.numel(), 2 * self.out_host.numel()

    def total_units(self, world):
        return world * self.flops / 1e12

    def roofline_units(self):
        return "tensor", self.flops

    def config(self, world):
        return {"workload": "dense bf16 GEMM M=2048 K=8192 N=28672 (the AWQ prefill layer with "
                            "dense weights): the comparator of the quantized layers",
                "M": self.M, "N": self.N, "K": self.K, "parallelism": f"replicas x{world}",
                "l2": "rotating weights: 2 x 470 MB buffers > 126 MB L2"}

    @classmethod
    def cpu_reference(cls, threads):
        torch.set_num_threads(threads)
        M, K = cls.M, cls.K
        n = 7168  # a quarter of the 28672 columns per pass
        g = torch.Generator().manual_seed(1234 + 7)
        a = (torch.randn(M, K, generator=g) / K ** 0.5).bfloat16()
        b = torch.randn(K, n, generator=g).bfloat16()
        run = lambda: a @ b  # noqa: E731
        return run, 2 * M * n * K / 1e12, ("N=7168 of 28672 columns per pass (full M, K); torch "
                                           "CPU bf16 matmul")


class Fp8BlockGemm:
    name = "fp8_block"
    unit = "TFLOP/s"
    dtype = "e4m3"
    bound = "tensor"
    scaling = "weak"
    profile = "w8a8_block_scaled_m4096_n7168_k7168.md"
    M, N, K = 4096, 7168, 7168
    data = ("synthetic (seeded e4m3 codes of N(0, 50^2) values; per-(token, 128-column block) and "
            "per-(128 x 128 block) fp32 scales U(0.001, 0.051))")
    launches_per_step = 1

    def __init__(self, dev, rank, world):
        import tileops_b200 as tob

        self.tob = tob
        M, N, K = self.M, self.N, self.K
        kt = K // 128
        g = torch.Generator().manual_seed(1234 + 6 + rank)
        qa_cpu = (torch.randn(M, K, generator=g) * 50).to(torch.float8_e4m3fn)
        sa_cpu = torch.rand(M, kt, generator=g) * 0.05 + 0.001
        # 3 x 51 MB of weights > 126 MB L2: every step streams its B from HBM
        self.qbs = [(torch.randn(N, K, generator=g) * 50).to(torch.float8_e4m3fn).to(dev)
                    for _ in range(3)]
        self.sb = (torch.rand(N // 128, kt, generator=g) * 0.05 + 0.001).to(dev)
        self.qa, self.sa = qa_cpu.to(dev), sa_cpu.to(dev)
        self.qa_host, self.sa_host = qa_cpu.view(torch.uint8).pin_memory(), sa_cpu.pin_memory()
        self.out_host = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
        self.dev = dev
        self.flops = 2 * M * N * K

    def step(self, i):
        self.tob.w8a8_block_fp8_matmul(self.qa, self.qbs[i % 3], self.sa, self.sb, [128, 128],
                                       output_dtype=torch.bfloat16)

    kernel_step = step

    def e2e_step(self, i):
        qa = self.qa_host.to(self.dev, non_blocking=True).view(torch.float8_e4m3fn)
        sa = self.sa_host.to(self.dev, non_blocking=True)
        c = self.tob.w8a8_block_fp8_matmul(qa, self.qbs[i % 3], sa, self.sb, [128, 128],
                                           output_dtype=torch.bfloat16)
        self.out_host.copy_(c, non_blocking=True)

    def h2d_d2h(self):
        return self.qa_host.numel() + 4 * self.sa_host.numel(), 2 * self.out_host.numel()

    def total_units(self, world):
        return world * self.flops / 1e12

    def roofline_units(self):
        return "tensor", self.flops

    def config(self, world):
        return {"workload": "fp8_e4m3 block-scaled GEMM M=4096 N=K=7168, [128, 128] scale "
                            "blocks (DeepSeek-style) -> bf16",
                "M": self.M, "N": self.N, "K": self.K, "block": [128, 128],
                "parallelism": f"replicas x{world}",
                "l2": "rotating weights: 3 x 51 MB buffers > 126 MB L2"}

    @classmethod
    def cpu_reference(cls, threads):
        import numpy as np

        from oracle import fp8 as ofp8

        torch.set_num_threads(threads)
        m = 64  # 64 of the 4096 rows per pass
        K, N = cls.K, cls.N
        kt = K // 128
        g = torch.Generator().manual_seed(1234 + 6)
        qa = (torch.randn(m, K, generator=g) * 50).to(torch.float8_e4m3fn).view(torch.uint8)
        qb = (torch.randn(N, K, generator=g) * 50).to(torch.float8_e4m3fn).view(torch.uint8)
        sa = (torch.rand(m, kt, generator=g) * 0.05 + 0.001).numpy()
        sb = (torch.rand(N // 128, kt, generator=g) * 0.05 + 0.001).numpy()
        a, b = np.ascontiguousarray(qa.numpy()), np.ascontiguousarray(qb.numpy())
        run = lambda: ofp8.block_matmul_reference_cpu(a, b, sa, sb, (128, 128), "bf16")  # noqa: E731
        return run, 2 * m * N * K / 1e12, ("M=64 of 4096 rows per pass (full N, K); numpy CPU "
                                           "fp32 block dequant + fp32 GEMM (reference algorithm)")


class AwqGemv:
    name = "awq_gemv"
    unit = "GB/s"
    dtype = "f16"
    bound = "hbm"
    scaling = "weak"
    profile = "awq_gemv_k4096_n4096.md"
    K, N, G = 4096, 4096, 128
    SETS = 48  # 48 x 8.7 MB > L2
    data = "synthetic (seeded random packed int4, scales U(0.002,0.02), x N(0,1))"
    launches_per_step = 1

    def __init__(self, dev, rank, world):
        import tileops_b200 as tob

        self.tob = tob
        K, N, G = self.K, self.N, self.G
        g = torch.Generator().manual_seed(1234 + 1 + rank)
        self.sets = []
        for _ in range(self.SETS):
            qw = torch.randint(-2 ** 31, 2 ** 31 - 1, (K, N // 8), generator=g, dtype=torch.int32)
            qz = torch.randint(-2 ** 31, 2 ** 31 - 1, (K // G, N // 8), generator=g, dtype=torch.int32)
            s = (torch.rand(K // G, N, generator=g) * 0.018 + 0.002).half()
            self.sets.append((qw.to(dev), s.to(dev), qz.to(dev)))
        x_cpu = torch.randn(1, K, generator=g).half()
        self.x = x_cpu.to(dev)
        self.x_host = x_cpu.pin_memory()
        self.out_host = torch.empty(1, N, dtype=torch.float16).pin_memory()
        self.dev = dev
        self.kernel_bytes = K * N // 2 + (K // G) * N * 2 + (K // G) * N // 2 + 2 * K + 2 * N
        # Consecutive calls overlap through programmatic dependent launch: a call streams its
        # weights while the previous one finishes (no kernel in the chain writes weights).
        tob.set_launch_overlap(True)

    def step(self, i):
        qw, s, qz = self.sets[i % self.SETS]
        self.tob.awq_gemm(self.x, qw, s, qz, 1)

    kernel_step = step

    def e2e_step(self, i):
        qw, s, qz = self.sets[i % self.SETS]
        x = self.x_host.to(self.dev, non_blocking=True)
        self.out_host.copy_(self.tob.awq_gemm(x, qw, s, qz, 1), non_blocking=True)

    def h2d_d2h(self):
        return 2 * self.K, 2 * self.N

    def total_units(self, world):
        return world * self.kernel_bytes / 1e9  # GB per step, whole job

    def roofline_units(self):
        return "hbm", self.kernel_bytes

    def config(self, world):
        return {"workload": "awq_w4a16_gemv x[1,4096] fp16 @ int4 [4096,4096] group 128",
                "M": 1, "K": self.K, "N": self.N, "group_size": self.G,
                "parallelism": f"replicas x{world}",
                "l2": "48 rotating weight sets x 8.7 MB > L2",
                "launch_overlap": "programmatic dependent launch between consecutive calls"}

    @classmethod
    def cpu_reference(cls, threads):
        from oracle import awq as oawq

        torch.set_num_threads(threads)
        K, N, G = cls.K, cls.N, cls.G
        g = torch.Generator().manual_seed(1234 + 1)
        x = torch.randn(1, K, generator=g).half()
        qw = torch.randint(-2 ** 31, 2 ** 31 - 1, (K, N // 8), generator=g, dtype=torch.int32)
        qz = torch.randint(-2 ** 31, 2 ** 31 - 1, (K // G, N // 8), generator=g, dtype=torch.int32)
        s = (torch.rand(K // G, N, generator=g) * 0.018 + 0.002).half()
        byts = K * N // 2 + (K // G) * N * 2 + (K // G) * N // 2 + 2 * K + 2 * N
        run = lambda: oawq.gemm_reference_cpu_torch(x, qw, s, qz, G)  # noqa: E731
        return run, byts / 1e9, ("the full GEMV per pass; torch CPU int64 unpack + dequant + fp16 "
                                 "matmul (reference algorithm)")


class DenseGemv:
    name = "dense_gemv"
    unit = "GB/s"
    dtype = "f16"
    bound = "hbm"
    scaling = "weak"
    profile = "dense_gemv_m4096_k4096.md"  # no ncu summary of it yet: traffic reads as null
    M, K = 4096, 4096
    SETS = 8  # 8 x 33.6 MB > L2
    data = "synthetic (seeded fp16 A N(0,1), x N(0, 1/K))"
    launches_per_step = 1

    def __init__(self, dev, rank, world):
        import tileops_b200 as tob

        self.tob = tob
        tob.set_launch_overlap(True)  # as the int4 GEMV line: call i+1 streams A under call i
        M, K = self.M, self.K
        g = torch.Generator().manual_seed(1234 + 8 + rank)
        self.sets = [torch.randn(M, K, generator=g).half().to(dev) for _ in range(self.SETS)]
        x_cpu = (torch.randn(K, generator=g) / K ** 0.5).half()
        self.x = x_cpu.to(dev)
        self.x_host = x_cpu.pin_memory()
        self.out_host = torch.empty(M, dtype=torch.float16).pin_memory()
        self.dev = dev
        self.kernel_bytes = 2 * M * K + 2 * K + 2 * M

    def step(self, i):
        self.tob.gemv(self.sets[i % self.SETS], self.x)

    kernel_step = step

    def e2e_step(self, i):
        x = self.x_host.to(self.dev, non_blocking=True)
        self.out_host.copy_(self.tob.gemv(self.sets[i % self.SETS], x), non_blocking=True)

    def h2d_d2h(self):
        return 2 * self.K, 2 * self.M

    def total_units(self, world):
        return world * self.kernel_bytes / 1e9  # GB per step, whole job

    def roofline_units(self):
        return "hbm", self.kernel_bytes

    def config(self, world):
        return {"workload": "dense fp16 GEMV y[4096] = A[4096,4096] @ x (the AWQ GEMV layer with "
                            "dense weights): the comparator of the int4 GEMV",
                "M": self.M, "K": self.K, "parallelism": f"replicas x{world}",
                "l2": "8 rotating weight sets x 33.6 MB > L2",
                "launch_overlap": "programmatic dependent launch between consecutive calls"}

    @classmethod
    def cpu_reference(cls, threads):
        torch.set_num_threads(threads)
        M, K = cls.M, cls.K
        g = torch.Generator().manual_seed(1234 + 8)
        a = torch.randn(M, K, generator=g).half()
        x = (torch.randn(K, generator=g) / K ** 0.5).half()
        run = lambda: a @ x  # noqa: E731
        return run, (2 * M * K + 2 * K + 2 * M) / 1e9, "the full GEMV per pass; torch CPU fp16 mv"


class Decode:
    name = "decode"
    unit = "GB/s"
    dtype = "f16"
    bound = "hbm"
    scaling = "strong"
    profile = "awq_decode_step.md"
    LAYERS = 32
    SHAPES = [(4096, 6144), (4096, 4096), (4096, 28672), (14336, 4096)]  # (K, N) per linear
    G = 128
    data = "synthetic (seeded random packed int4 weights, scales U(0.002,0.02), x N(0,1))"
    launches_per_step = 128  # counted by _run: 4 linears per layer (silu_and_mul inside the
    # gate_up kernel up to 32 tokens, a second launch above), a barrier after each gathering one

    def __init__(self, dev, rank, world, m=16):
        import tileops_b200 as tob
        from tileops_b200 import sharded

        self.tob, self.sharded, self.world, self.dev = tob, sharded, world, dev
        self.bufs = None
        # 3.6 GB of weights: drawn on the device from a seeded generator
        g = torch.Generator(device=dev).manual_seed(1234 + 5 + 100 * rank)
        self.layers = []
        for _ in range(self.LAYERS):
            lins = []
            for (k, n) in self.SHAPES:
                nl = n // world
                qw = torch.randint(-2 ** 31, 2 ** 31 - 1, (k, nl // 8), generator=g,
                                   dtype=torch.int32, device=dev)
                qz = torch.randint(-2 ** 31, 2 ** 31 - 1, (k // self.G, nl // 8), generator=g,
                                   dtype=torch.int32, device=dev)
                s = (torch.rand(k // self.G, nl, generator=g, device=dev) * 0.018 + 0.002).half()
                lins.append((qw, s, qz))
            self.layers.append(lins)
        self.weight_bytes = self.LAYERS * sum(
            k * n // 2 + (k // self.G) * n * 2 + (k // self.G) * n // 2 for k, n in self.SHAPES)
        self.set_m(m)
        tob.set_launch_overlap(True)  # layer i+1 streams its weights while layer i finishes

    def set_m(self, m):
        """Switches the batch to m tokens (the same weights)."""
        self.close()
        self.m = m
        self.bufs = None
        if self.world > 1 and m > 2:
            # one set of two peer-mapped [m, N] outputs per linear of the layer ([m, N/2] for
            # gate_up, whose kernel applies silu_and_mul), shared by the 32 layers (each set
            # alternates its two buffers)
            self.bufs = [self.sharded.PeerBuffers(m, n // 2 if j == 2 else n, torch.float16)
                         for j, (_, n) in enumerate(self.SHAPES)]
        gx = torch.Generator().manual_seed(1234 + 5)
        x_cpu = torch.randn(m, 4096, generator=gx).half()
        self.x = x_cpu.to(self.dev)
        self.x_host = x_cpu.pin_memory()
        self.out_host = torch.empty(m, 4096, dtype=torch.float16).pin_memory()

    def _linear(self, x, w, j):
        # gate_up (j == 2): gate and up columns interleaved in blocks of 8
        # (awq_interleave_gate_up), silu_and_mul applied in the GEMM's epilogue
        gemm = (lambda *a: self.tob.awq_gemm_silu_and_mul(*a)) if j == 2 else \
            (lambda *a: self.tob.awq_gemm(*a, 1))
        # this library's kernels per call: the GEMM, and the activation after it where the GEMM
        # has no fused epilogue (gate_up, K = 4096: 1-2 tokens and above 32 tokens)
        own = 2 if (j == 2 and (self.m > 32 or self.m <= 2)) else 1
        if self.world == 1:
            self._launches += own
            return gemm(x, *w)
        if self.m > 2:
            # this rank's column slice, all-gathered inside the kernel (peer stores over NVLink
            # and a GPU rank barrier)
            if j == 2:
                y = self.sharded.gathered_gemm_act(x, *w, self.bufs[j])
            else:
                y = self.sharded.gathered_gemm(x, *w, self.bufs[j])
            if y is not None:
                self._launches += 2  # the gathering kernel and the rank barrier
                return y
        # 1-2 tokens (and shapes the gathering kernels do not take): the local kernel on the
        # slice, then an NCCL all-gather
        self._launches += own
        return self.sharded.gather_columns(gemm(x, *w))

    def _run(self, x):
        self._launches = 0
        for qkv, o, gu, down in self.layers:
            h = self._linear(x, qkv, 0)
            a = self._linear(h[:, :4096], o, 1)  # read in place where the kernel can
            act = self._linear(a, gu, 2)  # silu(gate) * up, [M, 14336]
            x = self._linear(act, down, 3)
        self.launches_per_step = self._launches
        return x

    def close(self):
        for b in getattr(self, "bufs", None) or []:
            b.close()  # collective
        self.bufs = None

    def step(self, i):
        self._run(self.x)

    kernel_step = step

    def e2e_step(self, i):
        x = self.x_host.to(self.dev, non_blocking=True)
        self.out_host.copy_(self._run(x), non_blocking=True)

    def h2d_d2h(self):
        return 2 * self.x_host.numel(), 2 * self.out_host.numel()

    def total_units(self, world):
        return self.weight_bytes / 1e9  # GB of weights streamed per step, whole job

    def extra(self, ms_step):
        # one step advances the M sequences of the batch by one token each
        return {"tokens_per_s": self.m / (ms_step * 1e-3)}

    def roofline_units(self):
        return "hbm", self.weight_bytes / self.world

    def config(self, world):
        return {"workload": f"awq decode step, 32 layers x 4 linears (8B-class), M={self.m} fp16, "
                            "group 128, silu_and_mul in the gate_up kernel (gate/up columns "
                            "interleaved by 8), N-sharded, each linear all-gathered (inside its "
                            "kernel where it has a gathering form, NCCL otherwise)",
                "M": self.m, "layers": self.LAYERS, "parallelism": f"tp{world} (N-sharded)",
                "l2": "3.6 GB of weights per step > L2",
                "launch_overlap": "programmatic dependent launch between consecutive layers"}

    @classmethod
    def cpu_reference(cls, threads, m=16):
        from oracle import awq as oawq

        torch.set_num_threads(threads)
        k, n, G = 4096, 4096, cls.G  # one o-projection linear per pass
        g = torch.Generator().manual_seed(1234 + 5)
        x = torch.randn(m, k, generator=g).half()
        qw = torch.randint(-2 ** 31, 2 ** 31 - 1, (k, n // 8), generator=g, dtype=torch.int32)
        qz = torch.randint(-2 ** 31, 2 ** 31 - 1, (k // G, n // 8), generator=g, dtype=torch.int32)
        s = (torch.rand(k // G, n, generator=g) * 0.018 + 0.002).half()
        byts = k * n // 2 + (k // G) * n * 2 + (k // G) * n // 2
        run = lambda: oawq.gemm_reference_cpu_torch(x, qw, s, qz, G)  # noqa: E731
        return run, byts / 1e9, (f"one 4096x4096 linear (M={m}) of the 128 per step per pass; "
                                 "torch CPU reference algorithm")


WORKLOADS = {c.name: c for c in (Int8Layer, AwqPrefill, Fp8Layer, Fp8BlockGemm, DenseBf16,
                                  AwqGemv, DenseGemv, Decode)}


def time_cpu(workload_cls, reps: int, **kw):
    threads = os.cpu_count() or 1
    run, units, sample = workload_cls.cpu_reference(threads, **kw)
    run()  # warm-up
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return units / t, t, threads, sample


def arm_config(wl_cls, world: int, decode_m: int) -> dict:
    """The `config` a workload reports, built without a device (the CPU reference arm quotes the
    same config as the GPU arm)."""
    probe = wl_cls.__new__(wl_cls)
    probe.world = world
    probe.m = decode_m
    probe.gather = os.environ.get("TOB_BENCH_GATHER", "fused")
    return probe.config(world)


# The other configurations of the scope, measured in the default run after the headline one
# and reported under "workloads": (key, workload, decode M).
SUB_WORKLOADS = [("awq_gemv", "awq_gemv", None), ("fp8", "fp8", None),
                 ("awq_prefill", "awq_prefill", None), ("decode_m1", "decode", 1),
                 ("decode_m4", "decode", 4), ("decode_m16", "decode", 16),
                 ("decode_m64", "decode", 64)]


def cpu_line(wl_cls, reps: int, decode_m: int | None = None) -> dict:
    kw = {"m": decode_m} if wl_cls is Decode and decode_m is not None else {}
    v, t, cores, sample = time_cpu(wl_cls, reps, **kw)
    return {"value": v, "unit": wl_cls.unit, "cores": cores, "kind": "port",
            "sample": f"{sample}; median {t:.3f} s per pass"}


def run_reference_arm(args, rank: int, wl) -> None:
    if rank != 0:
        return
    for _ in range(args.warmup):
        time_cpu(wl, 1)
    vals, secs = [], []
    cores, sample = os.cpu_count(), ""
    for _ in range(args.steps):
        v, t, cores, sample = time_cpu(wl, 1)
        vals.append(v)
        secs.append(t)
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": wl.unit,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "scaling": wl.scaling, "vs_baseline": None, "dtype": wl.dtype,
        "data": wl.data, "config": arm_config(wl, args.gpus, args.decode_m),
        "cpu_baseline": {"value": value, "unit": wl.unit, "cores": cores, "kind": "port",
                         "sample": f"{sample}; median {statistics.median(secs):.3f} s per pass"},
        "e2e": {"value": value, "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if args.workload == "int8" and not args.single:
        subs = {}
        for key, name, m in SUB_WORKLOADS:
            sub_cls = WORKLOADS[name]
            cb = cpu_line(sub_cls, 1, m)
            subs[key] = {"value": cb["value"], "unit": sub_cls.unit,
                         "config": arm_config(sub_cls, args.gpus, m or args.decode_m),
                         "cpu_baseline": cb}
        line["workloads"] = subs
    print(json.dumps(line), flush=True)


def measure(wl, wl_cls, args, dist, dev, rank, world, local, steps, cpu_reps=3,
            decode_m=None) -> dict | None:
    """Times one workload: device throughput (graph replay), its dominant kernel (roofline) and
    the end-to-end path through the public API. Returns rank 0's line fields."""
    from tileops_b200 import _lib

    wl.step(0)  # first call: tensor maps, kernel attributes, NCCL communicator
    torch.cuda.synchronize()

    # ---------------- device throughput: K steps from one CUDA graph, inputs resident
    ms_step, clocks = timed_graph_ms(wl.step, steps, args.warmup, dist, clock_index=local)
    value = wl.total_units(world) / (ms_step * 1e-3)

    # ---------------- the dominant kernel alone (roofline)
    k_ms, _ = timed_graph_ms(wl.kernel_step, min(steps, 60), args.warmup, dist)

    # ---------------- end to end through the public API with host buffers
    for i in range(args.warmup):
        wl.e2e_step(i)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        wl.e2e_step(i)
    e1.record()
    torch.cuda.synchronize()
    e_ms = e0.elapsed_time(e1)
    if dist is not None:
        t = torch.tensor([e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_ms = float(t.item())
    e2e_value = wl.total_units(world) / (e_ms / steps * 1e-3)
    assert _lib.device_error_word() == 0
    if rank != 0:
        return None

    peaks, peak_kind = measured_peaks()
    bound, per_launch = wl.roofline_units()
    if bound == "hbm":
        achieved = per_launch / (k_ms * 1e-3) / 1e9
        peak, unit, peak_note = float(peaks["hbm_gbs"]), "GB/s", peak_kind
    else:
        achieved = per_launch / (k_ms * 1e-3) / 1e12
        unit = "TFLOP/s"
        peak = float(peaks["bf16_tflops"])
        sustained = float(peaks.get("bf16_tflops_sustained", peak))
        peak_note = peak_kind + " bf16 burst"
        if wl.name in ("fp8", "fp8_block"):  # dense e4m3 runs at twice the bf16 rate
            peak, sustained = 2 * peak, 2 * sustained
            peak_note = peak_kind + " bf16 burst x2 (e4m3)"
    h2d, d2h = wl.h2d_d2h()
    line = {
        "value": value, "unit": wl.unit, "ms_per_step": ms_step, "scaling": wl.scaling,
        "dtype": wl.dtype, "data": wl.data, "config": wl.config(world),
        "e2e": {"value": e2e_value, "unit": wl.unit, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "roofline": {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
                     "frac": achieved / peak, "traffic": profile_traffic(wl.profile),
                     "peak_source": peak_note, "kernel_ms": k_ms,
                     "algorithmic_per_launch": per_launch},
        "cpu_baseline": cpu_line(wl_cls, cpu_reps, decode_m),
        "gpu_launches": steps * wl.launches_per_step,
        "clocks": clocks,
    }
    if bound == "tensor":  # the kernel runs for the whole step, under the power cap
        line["roofline"]["peak_sustained"] = sustained
        line["roofline"]["frac_sustained"] = achieved / sustained
    if hasattr(wl, "extra"):
        line.update(wl.extra(ms_step))
    return line


def make_workload(wl_cls, dev, rank, world, decode_m):
    return wl_cls(dev, rank, world, decode_m) if wl_cls is Decode else wl_cls(dev, rank, world)


def release(wl, dist) -> None:
    if hasattr(wl, "close"):
        wl.close()  # collective: releases buffers mapped into the peers
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="int8", choices=sorted(WORKLOADS))
    ap.add_argument("--decode-m", type=int, default=16)
    ap.add_argument("--single", action="store_true",
                    help="measure only --workload (no 'workloads' entries for the other configs)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    wl_cls = WORKLOADS[args.workload]

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference_arm(args, rank, wl_cls)
        return 0

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    wl = make_workload(wl_cls, dev, rank, world, args.decode_m)
    head = measure(wl, wl_cls, args, dist, dev, rank, world, local, args.steps,
                   decode_m=args.decode_m if wl_cls is Decode else None)
    release(wl, dist)
    del wl

    subs = {}
    if args.workload == "int8" and not args.single:
        decode = None
        for key, name, m in SUB_WORKLOADS:
            sub_cls = WORKLOADS[name]
            if sub_cls is Decode:
                if decode is None:
                    decode = make_workload(sub_cls, dev, rank, world, m)
                decode.set_m(m)
                sub = decode
            else:
                sub = make_workload(sub_cls, dev, rank, world, None)
            r = measure(sub, sub_cls, args, dist, dev, rank, world, local, args.steps, cpu_reps=2,
                        decode_m=m)
            if r is not None:
                subs[key] = r
            if sub is not decode:
                release(sub, dist)
            del sub
        if decode is not None:
            release(decode, dist)
            del decode

    if rank == 0:
        line = {"metric": METRIC, "value": head["value"], "unit": head["unit"], "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
                "higher_is_better": True, "scaling": head["scaling"], "vs_baseline": None}
        line.update({k: v for k, v in head.items() if k not in line})
        if subs:
            line["workloads"] = subs
        print(json.dumps(line), flush=True)
    if dist is not None:
        from tileops_b200 import sharded

        sharded.close_peer_barriers()  # collective
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
