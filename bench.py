"""Benchmark of the int8 dynamic-quantization hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W]
                    [--workload distilbert|bert|ffn|sweep] [--impl ours|reference]

One JSON line on stdout (rank 0).  A "step" is one pass of the hot path over
one batch of seeded synthetic input (no dataset or checkpoint exists here):

* ``distilbert`` (default, config 3): the DistilBERT-base encoder, every
  Linear int8 (DynamicQuantizeLinear -> MatMulInteger -> dequant + bias
  [-> erf-GELU]), batch 32 x seq 128, run by the graph executor
  (GpuGraphExecutor).  Metric: sequences/s.
* ``bert`` (config 4): BERT-base, 12 layers, per-column weight scales and
  zero points, batch 64 x seq 512.
* ``ffn`` (config 2): the int8 FFN block alone, M = 4096, via the per-op API.
* ``sweep`` (config 5): one large-M point of the fused chain (M=65536,
  K=N=4096).  Metric: int8 TOP/s.

Timing: W untimed warm-up steps, then K steps each bracketed by CUDA events
on the launching stream, with the L2 evicted between steps by a 256 MiB read (outside the
events); barrier + synchronize on both sides; max over ranks.  Multi-GPU runs
shard the batch: every rank processes its own batch (weak scaling, no
collective on the data path).  ``e2e`` times the same step through the public
API from pinned host memory, including the H2D copy of the input and the D2H
copy of the output (encoder workloads: ``GpuGraphExecutor.run`` with host
arrays, wall-clock).  ``roofline`` is measured for the dominant kernel (the
GELU-fused FFN GEMM of the encoder, M x 768 x 3072) by CUDA events around
back-to-back launches of that kernel.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "DistilBERT-int8 seq/s at 1/2/4/8 B200; MatMulInteger int8 TOPS vs peak"
INT8_PEAK_TOPS = 4500.0  # B200 dense int8, datasheet (no measured int8 peak on this pool)

# DRAM bytes (read + write) of one launch of the roofline kernel, from one
# ncu capture (cold cache) of `bench.py --kernel ffn1 --shape 4096,768,3072`.
# The sweep kernel (M=65536, K=N=4096) is too large to capture under the
# profiling size rule: its value is the M=8192 capture of
# `bench.py --kernel gemm --shape 8192,4096,4096` scaled by the 8x rows, which
# is how its traffic grows (A and the output scale with M).
TRAFFIC_FFN1_M4096 = 5.869056e6 + 1.025024e6
TRAFFIC_SWEEP_FROM_M8192 = 8 * (52.330496e6 + 83.63136e6)


def roofline_traffic(kdesc: str):
    """ncu DRAM bytes per launch for the roofline kernel, scaled by rows."""
    if "K=768 N=3072" in kdesc:
        m = int(kdesc.split("M=")[1].split()[0])
        return TRAFFIC_FFN1_M4096 * m / 4096
    if "K=4096 N=4096" in kdesc:
        m = int(kdesc.split("M=")[1].split()[0])
        return TRAFFIC_SWEEP_FROM_M8192 * m / 65536
    return None


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------- workloads
class FfnWorkload:
    """Config 2: int8 FFN block, batch 32 x seq 128 (M=4096), K=768, F=3072."""

    name = "ffn"

    def __init__(self, device, batch=32, seq=128, hidden=768, ffn=3072, seed_base=0):
        import torch
        from iconnx_b200 import ops, synth
        self.torch, self.ops = torch, ops
        self.device = device
        self.batch, self.seq, self.hidden, self.ffn = batch, seq, hidden, ffn
        self.M = batch * seq
        x = synth.normal((self.M, hidden), 1.0, seed_base + 0)
        w1 = synth.int8_uniform((hidden, ffn), 1)
        w2 = synth.int8_uniform((ffn, hidden), 3)
        b1 = synth.normal((ffn,), 0.02, 2)
        b2 = synth.normal((hidden,), 0.02, 102)
        self.x_host = torch.from_numpy(x).pin_memory()
        self.x = self.x_host.to(device)
        self.w1 = ops.prepare_weight(torch.from_numpy(w1).to(device))
        self.w2 = ops.prepare_weight(torch.from_numpy(w2).to(device))
        self.b1 = torch.from_numpy(b1).to(device)
        self.b2 = torch.from_numpy(b2).to(device)
        self.ws = torch.tensor([0.01], dtype=torch.float32, device=device)
        self.out_host = torch.empty((self.M, hidden), dtype=torch.float32).pin_memory()
        self.units_per_step = batch  # sequences
        self.unit = "seq/s"
        self.launches_per_step = 5   # minmax, quantize, GEMM1(+minmax of h), quantize, GEMM2
        self.gemm_ops = 2 * (2.0 * self.M * hidden * ffn)

    def step(self, x=None):
        ops = self.ops
        if not hasattr(self, "mm"):
            self.mm = ops.MinMaxPartials(self.device)
        # GEMM1's epilogue records the (min, max) partials DQL2 needs
        h, *_ = ops.dynamic_quant_linear(self.x if x is None else x, self.w1, self.ws, self.b1,
                                         gelu=True, out_minmax=self.mm)
        out, *_ = ops.dynamic_quant_linear(h, self.w2, self.ws, self.b2, x_minmax=self.mm)
        return out

    def make_replay(self):
        return _torch_graph_replay(self)

    def e2e_step(self):
        torch = self.torch
        x = self.x_host.to(self.device, non_blocking=True)
        out = self.step(x)
        self.out_host.copy_(out, non_blocking=True)
        return int(self.x_host.numel() * 4), int(self.out_host.numel() * 4)

    # dominant kernel: the GELU-fused GEMM1 (M x 768 x 3072)
    def gemm_probe(self):
        ops = self.ops
        y, s, z = ops.gpu_dynamic_quantize_linear(self.x)
        out = self.torch.empty((self.M, self.ffn), dtype=self.torch.float32, device=self.device)

        def launch():
            ops.quant_linear(y, s, z, self.w1, self.ws, self.b1, gelu=True, out=out)
        M, K, N = self.M, self.hidden, self.ffn
        ops_count = 2.0 * M * N * K
        bytes_alg = M * K + N * K + 4 * M * N + 4 * N * 2
        return launch, ops_count, bytes_alg, f"quant_linear_gelu M={M} K={K} N={N}"

    def cpu_sample(self, threads):
        """Oracle FFN block on ONE sequence (M=128)."""
        from oracle import oracle
        xs = self.x_host.numpy()[: self.seq]
        w1 = self.w1_host if hasattr(self, "w1_host") else None
        from iconnx_b200 import synth
        w1 = synth.int8_uniform((self.hidden, self.ffn), 1)
        w2 = synth.int8_uniform((self.ffn, self.hidden), 3)
        b1 = synth.normal((self.ffn,), 0.02, 2)
        b2 = synth.normal((self.hidden,), 0.02, 102)
        ws = np.array([0.01], np.float32)
        t0 = time.perf_counter()
        h = oracle.quant_linear(xs, w1, ws, b1, None, True, threads=threads)[0]
        oracle.quant_linear(h, w2, ws, b2, None, False, threads=threads)
        dt = time.perf_counter() - t0
        return 1.0 / dt, f"FFN block on 1 sequence (M={self.seq}) of the same workload"


class SweepWorkload:
    """Config 5 large-M point: DQL -> MatMulInteger -> dequant + bias."""

    name = "sweep"

    def __init__(self, device, M=65536, K=4096, N=4096, seed_base=0):
        import torch
        from iconnx_b200 import ops, synth
        self.torch, self.ops, self.device = torch, ops, device
        self.M, self.K, self.N = M, K, N
        x = synth.outlier_mix((M, K), seed_base)
        self.x_host = torch.from_numpy(x).pin_memory()
        self.x = self.x_host.to(device)
        self.w = ops.prepare_weight(torch.from_numpy(synth.int8_uniform((K, N), 1)).to(device))
        self.bias = torch.from_numpy(synth.normal((N,), 0.02, 2)).to(device)
        self.ws = torch.tensor([0.01], dtype=torch.float32, device=device)
        self.out_host = torch.empty((M, N), dtype=torch.float32).pin_memory()
        self.units_per_step = 2.0 * M * N * K / 1e12
        self.unit = "TOPS"
        self.launches_per_step = 3
        self.gemm_ops = 2.0 * M * N * K

    def step(self, x=None):
        out, *_ = self.ops.dynamic_quant_linear(self.x if x is None else x, self.w, self.ws,
                                                self.bias)
        return out

    def make_replay(self):
        return _torch_graph_replay(self)

    def e2e_step(self):
        x = self.x_host.to(self.device, non_blocking=True)
        out = self.step(x)
        self.out_host.copy_(out, non_blocking=True)
        return int(self.x_host.numel() * 4), int(self.out_host.numel() * 4)

    def gemm_probe(self):
        ops = self.ops
        y, s, z = ops.gpu_dynamic_quantize_linear(self.x)
        out = self.torch.empty((self.M, self.N), dtype=self.torch.float32, device=self.device)

        def launch():
            ops.quant_linear(y, s, z, self.w, self.ws, self.bias, out=out)
        M, K, N = self.M, self.K, self.N
        return launch, 2.0 * M * N * K, M * K + N * K + 4 * M * N, f"quant_linear M={M} K={K} N={N}"

    def cpu_sample(self, threads):
        from oracle import oracle
        m = 64
        xs = self.x_host.numpy()[:m]
        from iconnx_b200 import synth
        w = synth.int8_uniform((self.K, self.N), 1)
        b = synth.normal((self.N,), 0.02, 2)
        t0 = time.perf_counter()
        oracle.quant_linear(xs, w, np.array([0.01], np.float32), b, None, False, threads=threads)
        dt = time.perf_counter() - t0
        return 2.0 * m * self.N * self.K / dt / 1e12, f"fused chain on {m} rows of the same workload"


def _torch_graph_replay(wl):
    """Capture one per-op step in a CUDA graph on torch's current stream."""
    torch = wl.torch
    for _ in range(2):
        wl.step()
    torch.cuda.synchronize(wl.device)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        wl.step()
    wl._graph = g
    return g.replay, torch.cuda.current_stream(wl.device)


def _int_mm_reference(torch, dev, stream, n=8192, reps=20):
    """An achievable int8 tensor-core reference measured on this box: cuBLASLt's
    s8 x s8 -> s32 GEMM (torch._int_mm) at n^3, CUDA events, back-to-back."""
    a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=dev)
    b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=dev)
    for _ in range(3):
        torch._int_mm(a, b)
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_ev.record(stream)
    for _ in range(reps):
        torch._int_mm(a, b)
    e_ev.record(stream)
    torch.cuda.synchronize(dev)
    ms = s_ev.elapsed_time(e_ev) / reps
    return {"tops": 2.0 * n ** 3 / (ms / 1e3) / 1e12, "shape": f"{n}x{n}x{n}", "ms": ms}


def _ffn_gemm_probe(torch, device, M, K=768, N=3072):
    """The GELU-fused FFN1 GEMM (dominant kernel of every encoder layer)."""
    from iconnx_b200 import ops, synth
    x = torch.from_numpy(synth.normal((M, K), 1.0, 0)).to(device)
    w = ops.prepare_weight(torch.from_numpy(synth.int8_uniform((K, N), 1)).to(device))
    b = torch.from_numpy(synth.normal((N,), 0.02, 2)).to(device)
    ws = torch.tensor([0.01], dtype=torch.float32, device=device)
    y, s, z = ops.gpu_dynamic_quantize_linear(x)
    out = torch.empty((M, N), dtype=torch.float32, device=device)

    def launch():
        ops.quant_linear(y, s, z, w, ws, b, gelu=True, out=out)
    return launch, 2.0 * M * N * K, M * K + N * K + 4 * M * N + 8 * N, \
        f"quant_linear_gelu M={M} K={K} N={N}"


class L2Flush:
    """Evicts the 126 MB L2 between timed launches by READING a 256 MiB
    buffer (a sum into a scalar): the L2 then holds clean lines, so the timed
    kernel pays no write-back of flush data.  Each call is ~80 us of device
    work, which also keeps the GPU ahead of the host so that a timed launch
    never waits on the host's enqueue."""

    def __init__(self, torch, dev, mib=256):
        self.torch = torch
        self.buf = torch.ones(mib << 18, dtype=torch.float32, device=dev)
        self.acc = torch.empty((), dtype=torch.float32, device=dev)

    def __call__(self):
        self.torch.sum(self.buf, dim=0, out=self.acc)
        self.torch.sum(self.buf, dim=0, out=self.acc)


def _timed_launches(torch, dev, stream, launch, flush, reps=10):
    """Median device time (ms) of single launches, each bracketed by CUDA
    events on `stream` with the L2 flushed before it (outside the events),
    after 3 untimed launches.  Everything is enqueued before one final
    synchronize, so the flushes keep the device busy while the host enqueues
    the next launch."""
    with torch.cuda.stream(stream):
        for _ in range(3):
            launch()
        torch.cuda.synchronize(dev)
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(reps)]
        for a, b in evs:
            flush()
            a.record(stream)
            launch()
            b.record(stream)
    torch.cuda.synchronize(dev)
    return float(np.median([a.elapsed_time(b) for a, b in evs]))


def north_star_gemms(torch, dev, flush, peaks):
    """The fused MatMulInteger target of the north star ("fused MatMulInteger
    at >= 60% of dense int8 tensor peak at config-4 large M") at config 4's
    two Linear shapes (M = 64 x 512 = 32768, per-column w_scale and int8
    weight zero points) and config 5's largest point.  Each entry: CUDA-event
    time of one launch (L2 flushed before it), int8 TOP/s, the fraction of the
    4.5 POPS datasheet dense int8 peak and of 2 x the measured bf16 peak, and
    the HBM roof of the shape (algorithmic bytes at the measured copy
    bandwidth) for shapes whose f32 output makes them memory-bound."""
    from iconnx_b200 import ops, synth
    stream = torch.cuda.Stream(dev)
    bf16 = peaks.get("bf16_tflops", 1590.0)
    hbm = peaks["hbm_gbs"]
    cases = [
        ("c4_ffn2", 32768, 3072, 768, True, False, False),
        ("c4_ffn2_residual", 32768, 3072, 768, True, False, True),
        ("c4_ffn1_gelu", 32768, 768, 3072, True, True, False),
        ("c5_largest", 65536, 4096, 4096, False, False, False),
    ]
    res = {}
    for name, M, K, N, per_col, gelu, residual in cases:
        with torch.cuda.stream(stream):
            # inputs drawn on the device (torch generator, seeded) with the
            # configs' distributions: N(0,1), config 5 with 0.1% N(0,20)
            # outliers; weights int8 uniform [-127, 127]
            gen = torch.Generator(device=dev)
            gen.manual_seed(0)
            x = torch.randn((M, K), generator=gen, device=dev)
            if name.startswith("c5"):
                pick = torch.rand((M, K), generator=gen, device=dev) < 0.001
                x[pick] *= 20.0
                del pick
            wk = torch.randint(-127, 128, (K, N), generator=gen, device=dev, dtype=torch.int8)
            w = ops.prepare_weight(wk)
            del wk
            if per_col:
                ws = torch.from_numpy(synth.uniform_f32((N,), 0.005, 0.02, 41)).to(dev)
                bz = torch.from_numpy(synth.int8_uniform((N,), 51, -8, 8)).to(dev)
                y, s, z, rows = ops.gpu_dynamic_quantize_linear(x, row_len=K)
            else:
                ws = torch.tensor([0.01], dtype=torch.float32, device=dev)
                bz, rows = None, None
                y, s, z = ops.gpu_dynamic_quantize_linear(x)
            del x
            b = torch.from_numpy(synth.normal((N,), 0.02, 2)).to(dev)
            r = torch.randn((M, N), generator=gen, device=dev) if residual else None
            out = torch.empty((M, N), dtype=torch.float32, device=dev)
        torch.cuda.synchronize(dev)

        def launch():
            ops.quant_linear(y, s, z, w, ws, b, bz, rows, gelu=gelu, out=out, residual=r)
        ms = _timed_launches(torch, dev, stream, launch, flush)
        op = 2.0 * M * N * K
        tops = op / (ms / 1e3) / 1e12
        alg = M * K + N * K + 4 * M * N * (2 if residual else 1) + 4 * (M if rows is not None else 0)
        t_hbm = alg / (hbm * 1e9) * 1e3
        t_int8 = op / (INT8_PEAK_TOPS * 1e12) * 1e3
        res[name] = {"M": M, "K": K, "N": N, "per_column": per_col, "gelu": gelu,
                     "residual": residual, "ms": ms, "int8_tops": tops,
                     "frac_of_4500_datasheet": tops / INT8_PEAK_TOPS,
                     "frac_of_2x_measured_bf16": tops / (2 * bf16),
                     "hbm_roof_ms": t_hbm, "int8_roof_ms": t_int8,
                     "bound": "hbm" if t_hbm > t_int8 else "tensor",
                     "frac_of_roof": max(t_hbm, t_int8) / ms}
        del y, s, z, w, ws, bz, rows, b, r, out
        torch.cuda.empty_cache()
    return res


class EncoderWorkload:
    """Configs 3 / 4: an int8 encoder through GpuGraphExecutor."""

    def __init__(self, device, kind="distilbert", seed_base=0, batch=None):
        import torch
        from iconnx_b200 import graphs
        from iconnx_b200.engine import GpuGraphExecutor
        self.torch, self.device = torch, device
        self.name = kind
        if kind == "distilbert":
            self.cfg, self.batch, self.seq = graphs.DISTILBERT, 32, 128
            self.model = "DistilBERT-base (6 layers, int8 Linears, per-tensor)"
        else:
            self.cfg, self.batch, self.seq = graphs.BERT_BASE, 64, 512
            self.model = "BERT-base (12 layers, int8 Linears, per-column scale + zero point)"
        self.global_batch = self.batch
        if batch is not None:
            self.batch = batch
        self.M = self.batch * self.seq
        self.ex = GpuGraphExecutor.new(device.index or 0)
        self.out = graphs.build_bert(self.ex, self.cfg, self.batch, self.seq)
        self.inputs = graphs.bert_inputs(self.batch, self.seq, seed=6 + seed_base)
        # pinned host buffers: the device->host copy of the output runs at full PCIe speed
        self.host_out = torch.empty((self.batch, self.seq, self.cfg.hidden), dtype=torch.float32,
                                    pin_memory=True).numpy()
        self.host_outs = [torch.empty((self.batch, self.seq, self.cfg.hidden), dtype=torch.float32,
                                      pin_memory=True).numpy() for _ in range(2)]
        self.inputs = {k: torch.from_numpy(v).pin_memory().numpy() for k, v in self.inputs.items()}
        self.ex.run(self.inputs, [self.out])        # lower + compile + warm
        self.ex.run(self.inputs, [self.out])        # captures the CUDA graph
        self.units_per_step = self.batch
        self.unit = "seq/s"
        self.launches_per_step = self.ex.kernel_launches()
        self.gemm_ops = graphs.gemm_ops_per_sequence(self.cfg, self.seq) * self.batch

    def make_replay(self):
        stream = self.torch.cuda.ExternalStream(self.ex.stream(), device=self.device)
        return self.ex.replay, stream

    def e2e_step(self):
        self.ex.run_device(self.inputs, [self.out])
        self.ex.fetch(self.out, self.host_out)
        h2d = sum(a.nbytes for a in self.inputs.values())
        return h2d, self.host_out.nbytes

    def e2e_loop(self, steps):
        """A serving loop through the public API: GpuGraphExecutor.submit /
        wait with two submissions in flight; every step uploads its inputs
        from pinned host memory and downloads its output into pinned host
        memory, the download overlapping the next step's compute."""
        pending = []
        for i in range(steps):
            pending.append(self.ex.submit(self.inputs, [self.out], [self.host_outs[i % 2]]))
            if len(pending) == 2:
                self.ex.wait(pending.pop(0))
        for t in pending:
            self.ex.wait(t)
        h2d = sum(a.nbytes for a in self.inputs.values())
        return h2d, self.host_outs[0].nbytes

    def gemm_probe(self):
        return _ffn_gemm_probe(self.torch, self.device, self.M)

    def cpu_sample(self, threads):
        """The CPU interpreter (oracle operators) on ONE sequence, all layers."""
        from iconnx_b200 import graphs
        from oracle.graph_executor import CpuGraph
        if getattr(self, "_cpu", None) is None or self._cpu[0].threads != threads:
            cpu = CpuGraph(threads=threads)
            self._cpu = (cpu, graphs.build_bert(cpu, self.cfg, 1, self.seq))
        cpu, out = self._cpu
        inp = graphs.bert_inputs(1, self.seq)
        t0 = time.perf_counter()
        cpu.run(inp, [out])
        dt = time.perf_counter() - t0
        return 1.0 / dt, (f"{self.name} encoder, 1 sequence x {self.seq} tokens, all "
                          f"{self.cfg.layers} layers, CPU interpreter over the oracle operators")


WORKLOADS = {"ffn": FfnWorkload, "sweep": SweepWorkload,
             "distilbert": lambda dev, seed_base=0, batch=None: EncoderWorkload(dev, "distilbert",
                                                                                 seed_base, batch),
             "bert": lambda dev, seed_base=0, batch=None: EncoderWorkload(dev, "bert", seed_base, batch)}


# ------------------------------------------------------------------ helpers
def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def cpu_info():
    model = ""
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    model = ln.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return os.cpu_count() or 1, model


def run_reference(args):
    """CPU implementation of the path (the oracle restating the reference's
    single-threaded CPU operators), run with every host thread."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from oracle import oracle
    ncores, model = cpu_info()
    threads = oracle.max_threads()

    class _Host:  # CPU-only stand-in holding the same seeded inputs
        pass

    import torch
    from iconnx_b200 import synth
    if args.workload in ("distilbert", "bert"):
        from iconnx_b200 import graphs
        w = EncoderWorkload.__new__(EncoderWorkload)
        w.name = args.workload
        w.cfg, w.seq = (graphs.DISTILBERT, 128) if args.workload == "distilbert" else (graphs.BERT_BASE, 512)
        fn = lambda: EncoderWorkload.cpu_sample(w, threads)  # noqa: E731
        unit = "seq/s"
        cfg = {"workload": f"{args.workload} encoder (config {'3' if args.workload == 'distilbert' else '4'})",
               "sample": "one sequence per step"}
    elif args.workload == "ffn":
        w = FfnWorkload.__new__(FfnWorkload)
        w.batch, w.seq, w.hidden, w.ffn = 32, 128, 768, 3072
        w.x_host = torch.from_numpy(synth.normal((128, 768), 1.0, 0))
        fn = lambda: FfnWorkload.cpu_sample(w, threads)  # noqa: E731
        unit = "seq/s"
        cfg = {"workload": "C2 int8 FFN block (batch 32 x seq 128, 768->3072->768)"}
    else:
        w = SweepWorkload.__new__(SweepWorkload)
        w.M, w.K, w.N = 65536, 4096, 4096
        w.x_host = torch.from_numpy(synth.outlier_mix((64, 4096), 0))
        fn = lambda: SweepWorkload.cpu_sample(w, threads)  # noqa: E731
        unit = "TOPS"
        cfg = {"workload": "C5 fused chain M=65536 K=N=4096"}
    for _ in range(args.warmup):
        fn()
    vals = []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        v, sample = fn()
        vals.append(v)
    dt = time.perf_counter() - t0
    value = float(np.mean(vals))
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": unit,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u8xs8->s32, f32 epilogue",
            "data": "synthetic (seeded)", "config": cfg,
            "cpu_baseline": {"value": value, "unit": unit, "cores": threads, "kind": "port",
                             "sample": sample + f"; host: {ncores} cores, {model}"},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_kernel_probe(args):
    """--kernel NAME: launch one kernel of the path a few times (for ncu
    captures of a single kernel; prints no JSON line)."""
    import torch
    from iconnx_b200 import graphs, ops, synth
    dev = torch.device("cuda", 0)
    M, K, N = [int(v) for v in args.shape.split(",")]
    if args.kernel in ("ffn1", "gemm", "gemm_pc", "quant", "residual", "residual_ln"):
        x = torch.from_numpy(synth.normal((M, K), 1.0, 0)).to(dev)
        w = ops.prepare_weight(torch.from_numpy(synth.int8_uniform((K, N), 1)).to(dev))
        b = torch.from_numpy(synth.normal((N,), 0.02, 2)).to(dev)
        ws = torch.tensor([0.01], dtype=torch.float32, device=dev)
        res = (torch.from_numpy(synth.normal((M, N), 1.0, 5)).to(dev)
               if args.kernel in ("residual", "residual_ln") else None)
        bz = rows = None
        if args.kernel == "gemm_pc":
            # config 4's per-column weight scale and int8 zero point
            ws = torch.from_numpy(synth.uniform_f32((N,), 0.005, 0.02, 41)).to(dev)
            bz = torch.from_numpy(synth.int8_uniform((N,), 51, -8, 8)).to(dev)
            y, s, z, rows = ops.gpu_dynamic_quantize_linear(x, row_len=K)
        else:
            y, s, z = ops.gpu_dynamic_quantize_linear(x)
        out = torch.empty((M, N), dtype=torch.float32, device=dev)
        mm = ops.MinMaxPartials(dev)
        if args.kernel == "residual_ln":
            gamma = torch.from_numpy(synth.normal((N,), 1.0, 6)).to(dev)
            beta = torch.from_numpy(synth.normal((N,), 0.02, 7)).to(dev)
            for _ in range(3):
                ops.quant_linear_layernorm(y, s, z, w, ws, res, gamma, beta, bias=b, out=out, minmax=mm)
        for _ in range(3 if args.kernel != "residual_ln" else 0):
            ops.quant_linear(y, s, z, w, ws, b, bz, rows, gelu=args.kernel == "ffn1", out=out,
                             minmax=mm if args.kernel == "quant" else None, residual=res)
            if args.kernel == "quant":
                ops.gpu_dynamic_quantize_from_partials(out, mm)
    elif args.kernel == "attention":
        from iconnx_b200.engine import GpuGraphExecutor
        ex = GpuGraphExecutor.new(0)
        out = graphs.build_bert(ex, graphs.BertConfig(layers=1, vocab=1000), M, K)
        ex.set_cuda_graphs(False)
        inp = graphs.bert_inputs(M, K, vocab=1000)
        for _ in range(2):
            ex.run(inp, [out])
    torch.cuda.synchronize()
    print(f"kernel probe {args.kernel} {args.shape} done", file=sys.stderr)


def pin_to_gpu_numa(torch, local):
    """Restricts this process to the CPU cores NVML reports as closest to its
    GPU (matched by PCI bus id), so the pinned host buffers of the end-to-end
    loop are first touched, and later written by the copy engine, in that
    GPU's NUMA node.  A process-level setting; best effort."""
    try:
        import pynvml
        props = torch.cuda.get_device_properties(local)
        bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        words = pynvml.nvmlDeviceGetCpuAffinity(h, (os.cpu_count() + 63) // 64)
        cpus = {64 * i + b for i, w in enumerate(words) for b in range(64) if (w >> b) & 1}
        cpus &= set(range(os.cpu_count()))
        if cpus:
            os.sched_setaffinity(0, cpus)
        return len(cpus)
    except Exception:
        return None


def device_ms(torch, dev, wl, steps, warmup, flush, barrier, clocks=None):
    """Total device time (ms) of `steps` replays of the workload's step, each
    bracketed by CUDA events on the stream the step runs on, with an L2 flush
    before each (outside the events), after `warmup` untimed steps."""
    replay, wstream = wl.make_replay()
    cur = torch.cuda.current_stream(dev)
    for _ in range(warmup):
        replay()
    barrier()
    if clocks is not None:
        clocks.start()
        # keep the GPU under the same load for ~1.5 s so the 100 ms clock
        # sampler sees the clocks of this workload (untimed, like the warm-up)
        t_soak = time.time()
        while time.time() - t_soak < 1.5:
            for _ in range(10):
                replay()
            torch.cuda.synchronize(dev)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(steps)]
    for s_ev, e_ev in evs:
        flush()                             # L2 flush, outside the events
        wstream.wait_stream(cur)
        s_ev.record(wstream)
        replay()
        e_ev.record(wstream)
        cur.wait_stream(wstream)
    barrier()
    return float(np.sum([s_ev.elapsed_time(e_ev) for s_ev, e_ev in evs]))


def end_to_end_ms(torch, dev, wl, steps, warmup, barrier):
    """Wall time (ms) of `steps` steps through the public API with host
    buffers: inputs uploaded and the output downloaded every step."""
    pipelined = hasattr(wl, "e2e_loop")
    if pipelined:
        wl.e2e_loop(warmup)
    else:
        for _ in range(warmup):
            wl.e2e_step()
    barrier()
    t0 = time.perf_counter()
    if pipelined:
        h2d, d2h = wl.e2e_loop(steps)
    else:
        for _ in range(steps):
            h2d, d2h = wl.e2e_step()
    torch.cuda.synchronize(dev)
    return (time.perf_counter() - t0) * 1e3, h2d, d2h, pipelined


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="distilbert", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-north-star", action="store_true",
                    help="skip the north-star GEMM shapes and the config-4 encoder that the "
                         "default 1-GPU run measures after the headline workload")
    ap.add_argument("--global-dql", action="store_true",
                    help="encoders on N>1 GPUs: every DynamicQuantizeLinear takes (min, max) over "
                         "all ranks (8-byte NCCL all-reduce), matching one executor over the "
                         "whole batch")
    ap.add_argument("--scaling", default="weak", choices=["weak", "strong"],
                    help="weak: every GPU runs the config's batch; strong (encoders): the "
                         "config's batch is split across the GPUs")
    ap.add_argument("--kernel", choices=["ffn1", "gemm", "gemm_pc", "quant", "residual", "residual_ln",
                                                 "attention"],
                    help="launch one kernel of the path a few times and exit (ncu captures)")
    ap.add_argument("--shape", default="4096,768,3072",
                    help="M,K,N for --kernel (attention: batch,seq,0)")
    args = ap.parse_args()
    if args.kernel:
        run_kernel_probe(args)
        return
    args.warmup = max(args.warmup, 3)

    if args.impl == "reference":
        run_reference(args)
        return

    import torch
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        pin_to_gpu_numa(torch, local)
    pg = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)
        pg = dist
    strong = args.scaling == "strong" and args.workload in ("distilbert", "bert")
    if strong:
        full = 32 if args.workload == "distilbert" else 64
        if full % world:
            raise SystemExit(f"--scaling strong: batch {full} does not split over {world} GPUs")
        wl = WORKLOADS[args.workload](dev, seed_base=1000 * rank, batch=full // world)
    else:
        wl = WORKLOADS[args.workload](dev, seed_base=1000 * rank)
    global_dql = args.global_dql and world > 1 and isinstance(wl, EncoderWorkload)
    if global_dql:
        from iconnx_b200.engine import nccl_unique_id
        box = [nccl_unique_id() if rank == 0 else None]
        pg.broadcast_object_list(box, src=0)
        wl.ex.set_global_dql(box[0], world, rank)
        wl.ex.run(wl.inputs, [wl.out])     # recompile with the all-reduce steps
        wl.ex.run(wl.inputs, [wl.out])     # capture the CUDA graph
        wl.launches_per_step = wl.ex.kernel_launches()
    stream = torch.cuda.current_stream(dev)
    flush = L2Flush(torch, dev)
    if not hasattr(wl, "launches_per_step"):
        wl.launches_per_step = 0

    def barrier():
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize(dev)

    # ---- device-resident timing (value)
    clocks = ClockSampler(local)
    total_ms = device_ms(torch, dev, wl, args.steps, args.warmup, flush, barrier, clocks)
    clk = clocks.stop()
    t = torch.tensor([total_ms], device=dev)
    if pg is not None:
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
    total_ms = float(t.item())
    value = wl.units_per_step * world * args.steps / (total_ms / 1e3)

    # ---- end-to-end through the public API, host buffers (e2e)
    e2e_ms, h2d, d2h, pipelined = end_to_end_ms(torch, dev, wl, args.steps, args.warmup, barrier)
    t = torch.tensor([e2e_ms], device=dev)
    if pg is not None:
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
    e2e_ms = float(t.item())
    e2e_value = wl.units_per_step * world * args.steps / (e2e_ms / 1e3)

    # ---- roofline of the dominant kernel (fused GEMM): single launches,
    # CUDA events on the launching stream, L2 flushed before each
    launch, ops_count, bytes_alg, kdesc = wl.gemm_probe()
    k_ms = _timed_launches(torch, dev, torch.cuda.Stream(dev), launch, flush, reps=20)
    peaks, peak_kind = load_peaks()
    tops = ops_count / (k_ms / 1e3) / 1e12
    gbs = bytes_alg / (k_ms / 1e3) / 1e9
    t_tensor = ops_count / (INT8_PEAK_TOPS * 1e12)
    t_hbm = bytes_alg / (peaks["hbm_gbs"] * 1e9)
    if t_tensor >= t_hbm:
        roof = {"bound": "tensor", "achieved": tops, "peak": INT8_PEAK_TOPS, "unit": "TOP/s",
                "frac": tops / INT8_PEAK_TOPS, "peak_source": "datasheet dense int8 (no measured int8 peak)"}
    else:
        roof = {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": gbs / peaks["hbm_gbs"], "peak_source": f"{peak_kind} hbm_gbs"}
    if wl.name == "sweep":
        roof["cublaslt_int8"] = _int_mm_reference(torch, dev, stream)
        roof["frac_of_cublaslt_int8"] = tops / roof["cublaslt_int8"]["tops"]
    traffic = roofline_traffic(kdesc)
    roof.update({"traffic": traffic, "traffic_note": "ncu dram read+write bytes per launch (profiles/), "
                 "scaled by rows where the capture used a smaller M", "algorithmic_bytes": bytes_alg,
                 "kernel": kdesc, "kernel_ms": k_ms, "int8_tops": tops,
                 "tensor_frac_of_4500": tops / INT8_PEAK_TOPS})

    line = {"metric": METRIC, "value": value, "unit": wl.unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
            "higher_is_better": True, "scaling": "strong" if strong else "weak", "vs_baseline": None,
            "dtype": "u8xs8->s32, f32 epilogue", "data": "synthetic (seeded)",
            "config": {"workload": wl.name, "M_per_gpu": wl.M,
                       "l2": "L2 evicted between timed steps (256 MiB read)",
                       "parallelism": f"batch-shard x{world} (independent executors, no collective)"},
            "e2e": {"value": e2e_value, "unit": wl.unit, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "mode": ("submit/wait, 2 in flight (upload, run, download every step)"
                             if pipelined else "run + fetch per step")},
            "gpu_launches": wl.launches_per_step * args.steps,
            "roofline": roof, "clocks": clk}
    if wl.name == "ffn":
        line["config"].update({"model": "DistilBERT-base FFN block (int8)", "global_batch": 32 * world,
                               "seq_len": 128})
    if isinstance(wl, EncoderWorkload):
        line["config"].update({"model": wl.model, "global_batch": wl.batch * world,
                               "seq_len": wl.seq, "batch_per_gpu": wl.batch})
        if strong:
            line["config"]["parallelism"] += f"; strong scaling of the config's batch {wl.global_batch}"
        if global_dql:
            line["config"]["parallelism"] = (f"batch-shard x{world}, global DynamicQuantizeLinear "
                                             "(8-byte NCCL MAX all-reduce per DQL)")
        line["int8_gemm_tops_in_step"] = wl.gemm_ops / (total_ms / args.steps / 1e3) / 1e12
    if world == 1 and args.workload == "distilbert" and not args.no_north_star:
        # the north star's other targets, measured in the same run: the fused
        # GEMM at config 4's / config 5's large-M shapes, and config 4's
        # encoder (BERT-base, batch 64 x seq 512) on device and end to end
        ns_clocks = ClockSampler(local)
        ns_clocks.start()
        gemms = north_star_gemms(torch, dev, flush, peaks)
        c4 = WORKLOADS["bert"](dev)
        c4_steps = max(3, min(args.steps, 10))
        c4_ms = device_ms(torch, dev, c4, c4_steps, args.warmup, flush, barrier)
        c4_e2e, _, _, _ = end_to_end_ms(torch, dev, c4, c4_steps, args.warmup, barrier)
        line["north_star"] = {
            "fused_gemm": gemms,
            "config4_bert_base": {"seq_per_s": c4.units_per_step * c4_steps / (c4_ms / 1e3),
                                  "e2e_seq_per_s": c4.units_per_step * c4_steps / (c4_e2e / 1e3),
                                  "ms_per_step": c4_ms / c4_steps, "batch": c4.batch,
                                  "seq_len": c4.seq, "steps": c4_steps,
                                  "int8_gemm_tops_in_step": c4.gemm_ops / (c4_ms / c4_steps / 1e3) / 1e12},
            "clocks": ns_clocks.stop()}
        del c4
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle
        ncores, model = cpu_info()
        from threadpoolctl import threadpool_limits
        with threadpool_limits(limits=1):   # numpy's BLAS too: one core
            v, sample = wl.cpu_sample(1)
        line["cpu_baseline"] = {"value": v, "unit": wl.unit, "cores": 1, "kind": "port",
                                "sample": sample + f"; host {ncores} cores, {model}"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.destroy_process_group()


if __name__ == "__main__":
    main()
