"""Benchmark of the evie-b200 hot path: one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

Workloads (per GPU; with N GPUs each rank runs its own share: weak scaling, no data-path collective):
  model_decode (default) Qwen3.5-4B-shaped decode, 64 sequences = 32 steered/unsteered pairs, 4096-token prompts,
               full SwiGLU capture (--model 0.8b: the 0.8B shapes, for small profiling cases)
  gdn_decode   Gated DeltaNet decode step, B=64 sequences x 16 heads, dk=dv=128, fp32 state
  gqa_decode   gated GQA decode attention, B=64, 16 q / 4 kv heads, hd 256, ctx ~ U[1024, 32768], 256-token pages
  gdn_prefill  Gated DeltaNet prefill, B=8, T=8192, 16 heads
  proj_gemm    one projection GEMM (the 4B gate/up weight, R=64 rows; --batch sets R)
The default run also times the three isolated ops (gdn_decode, gdn_prefill, gqa_decode) after the model's timed
region and reports them under `isolated`.

Timing: W untimed warm-up steps, then K steps, each bracketed by CUDA events on the launching stream; L2 is
flushed (a 256 MiB write, then a 256 MiB read so that no dirty line is left) between timed steps whenever a step's
working set fits in L2. The K-step region is bracketed by a barrier and torch.cuda.synchronize() on both sides; the
reported time is the max over ranks.
`e2e` repeats the step through the C ABI from pinned host buffers with the host<->device copies inside the timed
region. `cpu_baseline` (rank 0, N=1) times the CPU oracle (a C++ restatement of evie-core's CPU path) on a
bounded sample of the same workload, on evie's default thread count (half the logical CPUs, at most 8).
`--impl reference` times that CPU path alone.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tokens/s/GPU (batch 64) + prefill tok/s; % of HBM/tensor roofline at 1/2/4/8"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        d["source"] = "measured"
        return d
    return dict(FALLBACK_PEAKS)


def host_cpus() -> int:
    """Logical CPUs this process may run on (what Rust's available_parallelism reports)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 4


def evie_threads() -> int:
    """evie's default compute threads: half the logical CPUs, clamped to [1, 8] (crates/evie/src/main.rs:111);
    EVIE_CPU_THREADS overrides."""
    if os.environ.get("EVIE_CPU_THREADS"):
        return max(1, int(os.environ["EVIE_CPU_THREADS"]))
    return max(1, min(8, host_cpus() // 2))


def profiled_traffic(kernel: str, algorithmic_per_launch: float | None = None):
    """DRAM bytes per launch of `kernel` from the committed ncu summaries, if one exists: the captured figure, or,
    for a launch too large to capture, the traffic-to-algorithmic ratio captured on a smaller launch of the same
    kernel times this launch's algorithmic bytes."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        v = json.load(f).get(kernel)
    if isinstance(v, dict):
        r = v.get("traffic_per_algorithmic_byte")
        return r * algorithmic_per_launch if r and algorithmic_per_launch else None
    return v


# ------------------------------------------------------------------------------------------------------------
# clocks during the timed region

class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.dev}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or not self.path:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx.append(float(parts[2]))
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------------------------------------------
# multi-GPU host logic (one process per GPU, weak scaling)

def rank_prompts(rank: int, npairs: int, P: int, V: int, count: int | None = None):
    """The prompts of `rank`'s steered/unsteered pairs: pairs [rank * npairs, (rank + 1) * npairs) of one seeded
    stream (seed 5), so that every rank draws disjoint pairs of the same global set whatever the world size. `count`
    limits how many of the rank's pairs are drawn."""
    import torch

    count = npairs if count is None else count
    g = torch.Generator().manual_seed(5)
    first = rank * npairs
    drawn = [torch.randint(0, V, (P,), generator=g) for _ in range(first + count)]
    return [p.numpy().astype(np.uint32) for p in drawn[first:]]


def max_over_ranks(values, device=None):
    """Element-wise max of a list of floats over all ranks (every rank gets the result); identity with one rank."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return list(values)
    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def gather_to_rank0(arr, device=None):
    """The equal-shaped arrays of all ranks, stacked in rank order on rank 0 ([world, ...]); None on the other ranks;
    arr[None] with one rank. Floating-point arrays (logits) move as float32, integer ones (token ids, neuron
    indices) as int32. One all-gather, the same step on every rank (NCCL on the GPUs, gloo on CPU)."""
    import torch
    import torch.distributed as dist

    arr = np.asarray(arr)
    a = np.ascontiguousarray(arr, dtype=np.float32 if arr.dtype.kind == "f" else np.int32)
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return a[None].copy()
    t = torch.from_numpy(a).to(device) if device is not None else torch.from_numpy(a)
    parts = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(parts, t)
    return np.stack([x.cpu().numpy() for x in parts]) if dist.get_rank() == 0 else None


# ------------------------------------------------------------------------------------------------------------
# workloads

class Workload:
    name = ""
    unit = "tokens/s"
    dtype = "f32"
    kernel = ""            # dominant kernel name (ncu)
    bound = "hbm"
    flush_l2 = False
    tokens_per_step = 0    # units of the metric per step per GPU

    def config(self) -> dict:
        raise NotImplementedError

    def setup(self, dev):
        raise NotImplementedError

    def step(self):
        """Enqueues one step on the current stream. Returns the number of our kernel launches."""
        raise NotImplementedError

    def algorithmic(self) -> float:
        """Bytes (hbm) or FLOPs (tensor) of the dominant kernel per step."""
        raise NotImplementedError

    def e2e_step(self):
        """One step through the C ABI with host buffers (H2D inputs, D2H result). Returns (h2d, d2h) bytes."""
        raise NotImplementedError

    def cpu_sample(self, threads: int) -> dict:
        raise NotImplementedError

    # default timing: one CUDA-event pair per step on the current stream, L2 flushed between steps if asked
    def warmup(self, w):
        for _ in range(w):
            self.step()

    def _flush(self):
        """The L2 flush between timed steps: a 256 MiB write, then a 256 MiB read of a second buffer, so that the
        write's dirty lines are written back before the timed region and L2 holds only clean, unrelated lines
        (without the read, the timed kernel pays for writing back up to 126 MB of the flush's data)."""
        import torch

        if self.flush_l2 and not hasattr(self, "_flushbuf"):
            self._flushbuf = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
            self._flushread = torch.zeros(64 << 20, dtype=torch.float32, device="cuda")
            self._flushsum = torch.empty((), dtype=torch.float32, device="cuda")
        buf = getattr(self, "_flushbuf", None)
        if buf is None:
            return None

        def flush(i):
            buf.fill_(i & 0xFF)
            torch.sum(self._flushread, dim=0, out=self._flushsum)
        return flush

    def timed(self, k):
        import torch

        stream = torch.cuda.current_stream()
        flush = self._flush()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(k)]
        launches = 0
        for i in range(k):
            if flush is not None:
                flush(i)
            ev[i][0].record(stream)
            launches += self.step()
            ev[i][1].record(stream)
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in ev), launches

    def e2e(self, k):
        import torch

        stream = torch.cuda.current_stream()
        flush = self._flush()
        for _ in range(2):
            self.e2e_step()
        torch.cuda.synchronize()
        ms = 0.0
        h2d = d2h = 0
        for i in range(k):
            if flush is not None:
                flush(i)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            h2d, d2h = self.e2e_step()
            b.record(stream)
            torch.cuda.synchronize()
            ms += a.elapsed_time(b)
        return ms, h2d, d2h


class GdnDecode(Workload):
    name = "gdn_decode"
    kernel = "gdn_decode_step_kernel"
    flush_l2 = True  # the 64 MiB state fits in the 126 MB L2

    def __init__(self, B=64, H=16, d=128):
        self.B, self.H, self.d = B, H, d
        self.tokens_per_step = B

    def config(self):
        return {"workload": f"gdn_decode_step B={self.B} H={self.H} dk=dv={self.d} fp32 state",
                "global_batch": self.B, "heads": self.H, "l2": "flushed between timed steps (256 MiB write, then 256 MiB read)"}

    def algorithmic(self):
        B, H, d = self.B, self.H, self.d
        return 2 * B * H * d * d * 4 + B * H * 3 * d * 2 + B * H * 8 + B * H * d * 4

    def setup(self, dev):
        import torch
        from tests._inputs import gdn_decode_inputs

        x = gdn_decode_inputs(self.B, self.H, 2, device=dev if getattr(self, "gen_on_device", False) else "cpu")
        self.x = {k: v.to(dev) for k, v in x.items()}
        self.o = torch.empty(self.B, self.H, self.d, device=dev)
        self.host = {k: v.cpu().pin_memory() for k, v in x.items() if k != "S"}
        self.dev_in = {k: torch.empty_like(v, device=dev) for k, v in self.host.items()}
        self.o_host = torch.empty(self.B, self.H, self.d).pin_memory()

    def step(self):
        from evie_b200 import ops

        x = self.x
        ops.gdn_decode_step(x["q"], x["k"], x["v"], x["g"], x["beta"], x["S"], self.o)
        return 1

    def e2e_step(self):
        from evie_b200 import ops

        h2d = 0
        for k, v in self.host.items():
            self.dev_in[k].copy_(v, non_blocking=True)
            h2d += v.numel() * v.element_size()
        d = self.dev_in
        ops.gdn_decode_step(d["q"], d["k"], d["v"], d["g"], d["beta"], self.x["S"], self.o)
        self.o_host.copy_(self.o, non_blocking=True)
        return h2d, self.o.numel() * 4

    def cpu_sample(self, threads):
        import oracle
        from tests._inputs import bf16_bits, gdn_decode_inputs

        oracle.set_threads(threads)
        x = gdn_decode_inputs(self.B, self.H, 2)
        S = x["S"].numpy().copy()
        args = (bf16_bits(x["q"]), bf16_bits(x["k"]), bf16_bits(x["v"]), x["g"].numpy(), x["beta"].numpy())
        oracle.gdn_decode(S, *args)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 10.0 and n < 2000:
            oracle.gdn_decode(S, *args)
            n += 1
        dt = (time.perf_counter() - t0) / n
        return {"value": self.B / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
                "sample": f"{n} full decode steps (B={self.B}, H={self.H}) of the oracle's recur_body restatement"}


class GdnPrefill(Workload):
    """Chunked Gated DeltaNet prefill, B sequences x T tokens x H heads, dk = dv = 128, S0 = 0."""
    name = "gdn_prefill"
    kernel = "gdn_chunk_prefill_kernel"
    bound = "tensor"

    def __init__(self, B=8, T=8192, H=16, d=128):
        self.B, self.T, self.H, self.d = B, T, H, d
        self.tokens_per_step = B * T

    def hbm_bytes(self):
        B, T, H, d = self.B, self.T, self.H, self.d
        return B * T * H * d * 2 * 3 + B * T * H * 8 + B * T * H * d * 2 + B * H * d * d * 4

    def config(self):
        return {"workload": f"gdn_chunk_prefill B={self.B} T={self.T} H={self.H} dk=dv={self.d} chunk=64, "
                            f"S0=0, o bf16",
                "global_batch": self.B, "seq_len": self.T, "heads": self.H,
                "hbm_bytes_per_step": self.hbm_bytes(),
                "l2": f"inputs larger than L2 ({self.hbm_bytes() / 1e9:.2f} GB)"}

    def algorithmic(self):
        """6 C d^2 + 10 C^2 d FLOP per (chunk, head), the triangular solve excluded."""
        C, d = 64, self.d
        chunks = self.B * self.H * ((self.T + C - 1) // C)
        return (6 * C * d * d + 10 * C * C * d) * chunks

    def setup(self, dev):
        import torch
        from tests._inputs import gdn_prefill_inputs

        x = gdn_prefill_inputs(self.B, self.T, self.H, 3, device=dev if getattr(self, "gen_on_device", False) else "cpu")
        self.S0 = x["S"].to(dev)
        self.x = {k: v.to(dev) for k, v in x.items()}
        self.o = torch.empty(self.B, self.T, self.H, self.d, device=dev, dtype=torch.bfloat16)
        self.host = {k: x[k].cpu().pin_memory() for k in ("q", "k", "v", "g", "beta")}
        self.dev_in = {k: torch.empty_like(v, device=dev) for k, v in self.host.items()}
        self.o_host = torch.empty(self.B, self.T, self.H, self.d, dtype=torch.bfloat16).pin_memory()

    def step(self):
        from evie_b200 import ops

        x = self.x
        x["S"].copy_(self.S0)
        ops.gdn_chunk_prefill(x["q"], x["k"], x["v"], x["g"], x["beta"], x["S"], self.o)
        return 1

    def e2e_step(self):
        from evie_b200 import ops

        h2d = 0
        for k, v in self.host.items():
            self.dev_in[k].copy_(v, non_blocking=True)
            h2d += v.numel() * v.element_size()
        d = self.dev_in
        self.x["S"].copy_(self.S0)
        ops.gdn_chunk_prefill(d["q"], d["k"], d["v"], d["g"], d["beta"], self.x["S"], self.o)
        self.o_host.copy_(self.o, non_blocking=True)
        return h2d, self.o.numel() * 2

    def cpu_sample(self, threads):
        import oracle
        from tests._inputs import bf16_bits, gdn_prefill_inputs

        oracle.set_threads(threads)
        heads = min(threads, self.B * self.H)
        Ts = min(self.T, 2048)
        x = gdn_prefill_inputs(1, Ts, heads, 3)
        args = (bf16_bits(x["q"]), bf16_bits(x["k"]), bf16_bits(x["v"]), x["g"].numpy(), x["beta"].numpy())
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 10.0 and n < 50:
            oracle.gdn_prefill(x["S"].numpy().copy(), *args)
            n += 1
        dt = (time.perf_counter() - t0) / n
        per_head_token = dt / (heads * Ts)
        return {"value": 1.0 / (per_head_token * self.H), "unit": "tokens/s", "cores": threads, "kind": "port",
                "sample": f"{n} calls of the oracle's token-sequential prefill on {heads} heads x {Ts} tokens, "
                          f"scaled to {self.H} heads per token"}


class GqaDecode(Workload):
    name = "gqa_decode"
    kernel = "gqa_decode_tma_kernel"

    def __init__(self, B=64, Hq=16, Hkv=4, hd=256, page=256):
        import torch

        self.B, self.Hq, self.Hkv, self.hd, self.page = B, Hq, Hkv, hd, page
        g = torch.Generator().manual_seed(4)
        self.ctx = torch.randint(1024, 32769, (B,), generator=g).tolist()
        self.tokens_per_step = B

    def config(self):
        return {"workload": f"gqa_decode B={self.B} Hq={self.Hq} Hkv={self.Hkv} hd={self.hd} ctx~U[1024,32768] "
                            f"(sum {sum(self.ctx)}) page={self.page} bf16 KV",
                "global_batch": self.B, "l2": f"inputs larger than L2 ({self.algorithmic() / 1e9:.2f} GB)"}

    def algorithmic(self):
        """K and V rows read once, q and gate (bf16) read, out (f32) written, page tables and lengths read."""
        kv = sum(self.ctx) * self.Hkv * self.hd * 2 * 2
        pages = sum((c + self.page - 1) // self.page for c in self.ctx)
        return kv + self.B * self.Hq * self.hd * (2 + 2 + 4) + (pages + self.B) * 4

    def setup(self, dev):
        import torch
        from tests._inputs import gqa_inputs

        x = gqa_inputs(self.B, self.Hq, self.Hkv, self.ctx, 4, hd=self.hd, page=self.page,
                       device=dev if getattr(self, "gen_on_device", False) else "cpu")
        self.x = {k: v.to(dev) for k, v in x.items()}
        self.out = torch.empty(self.B, self.Hq, self.hd, device=dev)
        self.host = {k: x[k].cpu().pin_memory() for k in ("q", "gate")}
        self.dev_in = {k: torch.empty_like(v, device=dev) for k, v in self.host.items()}
        self.out_host = torch.empty(self.B, self.Hq, self.hd).pin_memory()

    def step(self):
        from evie_b200 import ops

        x = self.x
        ops.gqa_decode_paged(x["q"], x["gate"], x["kp"], x["vp"], x["pt"], x["ctx"], 1 / 16, self.out)
        return 1

    def e2e_step(self):
        from evie_b200 import ops

        h2d = 0
        for k, v in self.host.items():
            self.dev_in[k].copy_(v, non_blocking=True)
            h2d += v.numel() * v.element_size()
        x = self.x
        ops.gqa_decode_paged(self.dev_in["q"], self.dev_in["gate"], x["kp"], x["vp"], x["pt"], x["ctx"], 1 / 16,
                             self.out)
        self.out_host.copy_(self.out, non_blocking=True)
        return h2d, self.out.numel() * 4

    def cpu_sample(self, threads):
        import oracle
        from tests._inputs import bf16_bits, gqa_inputs

        oracle.set_threads(threads)
        nb = 8
        x = gqa_inputs(nb, self.Hq, self.Hkv, self.ctx[:nb], 4, hd=self.hd, page=self.page)
        args = (bf16_bits(x["q"]), bf16_bits(x["kp"]), bf16_bits(x["vp"]), x["pt"].numpy(), x["ctx"].numpy(),
                bf16_bits(x["gate"]), 1 / 16)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 10.0 and n < 100:
            oracle.gqa_decode(*args)
            n += 1
        dt = (time.perf_counter() - t0) / n
        # scale to the full batch by context length
        per_tok = dt / sum(self.ctx[:nb])
        full = per_tok * sum(self.ctx)
        return {"value": self.B / full, "unit": "tokens/s", "cores": threads, "kind": "port",
                "sample": f"{n} calls on the first {nb} sequences (ctx {sum(self.ctx[:nb])} tokens), "
                          f"scaled to the batch by context length"}


class ProjGemm(Workload):
    """One projection of the model: y = x W^T for bf16 weights W [M][K] and f32 activations x [R][K] as split bf16
    planes, through evie_proj_gemm. Default shape: the 4B MLP gate/up projection (M = 18432, K = 2560) at the decode
    batch R = 64; --batch sets R (R > 128 runs the prefill tiles). Weights are rotated over copies that together
    exceed L2, so every step streams its weight from HBM."""
    name = "proj_gemm"
    kernel = "proj_gemm_kernel"

    def __init__(self, B=64, M=18432, K=2560):
        self.R, self.M, self.K = B, M, K
        self.tokens_per_step = B
        self.bound = "hbm" if B <= 128 else "tensor"

    def config(self):
        return {"workload": f"proj_gemm M={self.M} K={self.K} R={self.R} (bf16 weights x split-bf16 f32 operand)",
                "global_batch": self.R, "l2": "weights rotated over copies larger than L2"}

    def algorithmic(self):
        """hbm: the weight bytes plus the operand planes and the f32 output; tensor: 2 M K R useful FLOPs."""
        if self.bound == "hbm":
            return self.M * self.K * 2 + 2 * self.R * self.K * 2 + self.R * self.M * 4
        return 2 * self.M * self.K * self.R

    def setup(self, dev):
        import torch

        from evie_b200 import ops

        g = torch.Generator(device=dev).manual_seed(7)
        nbytes = self.M * self.K * 2
        self.ncopy = max(1, (300 << 20) // nbytes + 1) if self.R <= 128 else 1
        self.ws = [(torch.randn(self.M, self.K, generator=g, device=dev) * 0.02).to(torch.bfloat16)
                   for _ in range(self.ncopy)]
        self.x2 = ops.split_planes(torch.randn(self.R, self.K, generator=g, device=dev))
        self.y = torch.empty(16, self.R, self.M, device=dev) if self.R <= 128 else torch.empty(self.R, self.M,
                                                                                                device=dev)
        self.i = 0

    def step(self):
        import ctypes as C

        import torch

        from evie_b200 import check, lib

        planes = C.c_int(0)
        w = self.ws[self.i % self.ncopy]
        self.i += 1
        check(lib().evie_proj_gemm(w.data_ptr(), self.x2.data_ptr(), self.y.data_ptr(), self.y.numel(), self.M,
                                   self.K, self.R, 16, C.byref(planes), torch.cuda.current_stream().cuda_stream))
        return 1

    def e2e_step(self):
        import torch

        if not hasattr(self, "x_host"):
            self.x_host = self.x2.cpu().pin_memory()
            self.y_host = torch.empty(self.R, self.M).pin_memory()
        self.x2.copy_(self.x_host, non_blocking=True)
        self.step()
        self.y_host.copy_(self.y[0] if self.y.dim() == 3 else self.y, non_blocking=True)
        return self.x_host.numel() * 2, self.R * self.M * 4

    def cpu_sample(self, threads):
        import oracle

        oracle.set_threads(threads)
        rng = np.random.default_rng(7)
        R = min(self.R, 64)
        w = rng.integers(0, 1 << 15, (self.M, self.K), dtype=np.uint16)
        x = rng.standard_normal((R, self.K), dtype=np.float32)
        oracle.matmul(w[:64], x)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 10.0 and n < 50:
            oracle.matmul(w, x)
            n += 1
        dt = (time.perf_counter() - t0) / n
        return {"value": R / dt, "unit": "tokens/s", "cores": threads, "nproc": host_cpus(), "kind": "port",
                "sample": f"{n} calls of the oracle's matmul (kernels.rs:138-268) at M={self.M} K={self.K} R={R}"}


class ModelDecode(Workload):
    """Per GPU: Qwen3.5-4B shapes, random bf16 weights (seed 5), B sequences = B/2 steered/unsteered pairs,
    P-token uniform-random prompts, +0.6 dose Add steering on 32 seeded (layer, neuron) pairs on the steered half,
    every SwiGLU activation captured. A step is one greedy decode step of all B sequences."""
    name = "model_decode"
    kernel = "decode step (all kernels)"
    dtype = "f32"  # the arithmetic type; operands below
    dtype_detail = "f32 activations x bf16 weights (split-bf16 operands), fp32 DeltaNet state, bf16 KV"

    def __init__(self, B=64, prompt=4096, rank=0, model="4b"):
        assert B % 2 == 0 and model in ("4b", "0.8b")
        self.B, self.P, self.rank, self.model = B, prompt, rank, model
        self.tokens_per_step = B
        self.n_pairs_total = None

    def config(self):
        tag = "4B" if self.model == "4b" else "0.8B"
        return {"workload": f"Qwen3.5-{tag}-shaped decode, {self.B} sequences ({self.B // 2} steered/unsteered pairs) "
                            f"per GPU, {self.P}-token prompts, greedy, steering +0.6 dose on 32 (layer, neuron) pairs, "
                            f"full SwiGLU capture",
                "model": f"qwen3.5-{self.model}-shaped (random init, seed 5)", "global_batch": self.B, "seq_len": self.P,
                "l2": "inputs larger than L2 (8.4 GB weights + caches per step)",
                "prefill_tok_s": getattr(self, "prefill_tok_s", None),
                "prefill_ms": getattr(self, "prefill_ms", None)}

    def checkpoint(self, device):
        """The synthetic checkpoint (seed 5), written once per machine (shared by every rank and both arms)."""
        from evie_b200 import checkpoint as ck

        base = os.environ.get("EVIE_CKPT_DIR", tempfile.gettempdir())
        shape = ck.QWEN35_4B if self.model == "4b" else ck.QWEN35_0_8B
        name = "evie_qwen35_4b_seed5" if self.model == "4b" else "evie_qwen35_0p8b_seed5"
        return ck.ensure_checkpoint(os.path.join(base, name), ck.text_config(shape), seed=5, device=device)

    def setup(self, dev):
        import torch

        from evie_b200 import checkpoint as ck
        from evie_b200.gpu import GpuModel, GpuSeq

        self.ckpt = self.checkpoint("cuda")
        self.cfg = json.load(open(os.path.join(self.ckpt, "config.json")))
        L, n, V = self.cfg["num_hidden_layers"], self.cfg["intermediate_size"], self.cfg["vocab_size"]
        self.max_ctx = self.P + 1024
        # prefill feeds whole prompts, up to EVIE_PREFILL_ROWS rows per call: more sequences per call give the per-row
        # mixer and attention kernels more CTAs (rows index a grid dimension, so at most 65535)
        rows = int(os.environ.get("EVIE_PREFILL_ROWS", "32768"))
        self.m = GpuModel(self.ckpt, max_ctx=self.max_ctx, slots=self.B, max_rows=min(rows, self.B * self.P),
                          device=dev.index or 0)
        g = torch.Generator().manual_seed(5)
        self.layers = torch.randint(0, L, (32,), generator=g).tolist()
        self.neurons = torch.randint(0, n, (32,), generator=g).tolist()
        self.prompts = rank_prompts(self.rank, self.B // 2, self.P, V)
        # dose unit: median ||residual leaving layer l|| over tokens 1.. of pair 0's prompt (calib.rs:94-100),
        # divided by ||W_down[:, n]|| (engine.rs:102-104); measured on the unsteered lane of pair 0.
        out = self.m.forward([GpuSeq(1, 0, self.prompts[0])], want_logits=False, capture=True)
        resid = out.resid.reshape(self.P, L, -1).astype(np.float32)
        norms = np.linalg.norm(resid[1:], axis=-1)
        self.units = np.median(norms, axis=0)
        ops = []
        for l, nn in zip(self.layers, self.neurons):
            w = ck.read_tensor(self.ckpt, f"model.language_model.layers.{l}.mlp.down_proj.weight")
            col = float(np.sqrt((w[:, nn].astype(np.float64) ** 2).sum()))
            ops.append((l, nn, "add", float(0.6 * self.units[l] / max(col, 1e-12))))
        self.ops = ops
        for sl in range(self.B):
            self.m.set_ops(sl, ops if sl % 2 == 0 else [])
        self.m.reset_slot(1)
        # prefill every sequence (pair p: slots 2p steered, 2p+1 unsteered), timed on the context's stream
        stream = torch.cuda.ExternalStream(self.m.stream_ptr())
        per_call = max(1, min(self.B, rows // self.P))
        self.first_tokens = np.zeros(self.B, np.uint32)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for c0 in range(0, self.B, per_call):
            seqs = [GpuSeq(sl, 0, self.prompts[sl // 2]) for sl in range(c0, min(self.B, c0 + per_call))]
            o = self.m.forward(seqs, want_logits=False)
            self.first_tokens[c0:c0 + len(seqs)] = o.next_tokens
        e1.record(stream)
        torch.cuda.synchronize()
        self.prefill_ms = e0.elapsed_time(e1)
        self.prefill_tok_s = self.B * self.P / (self.prefill_ms / 1000.0)
        # Where one prefill call's time goes: the first call again, from reset slots (the same prompts, so the slots
        # end as before), with the library's profiling events around every kernel group (the eager path: a little
        # slower than the timed calls). Its greedy tokens must equal the timed call's.
        first = [GpuSeq(sl, 0, self.prompts[sl // 2]) for sl in range(min(self.B, per_call))]
        for s in first:
            self.m.reset_slot(s.slot)
        self.m.profile(True)
        o = self.m.forward(first, want_logits=False)
        groups = self.m.profile_read()
        self.m.profile(False)
        self.prefill_groups = {"rows": len(first) * self.P,
                               "same_tokens": bool(np.array_equal(o.next_tokens, self.first_tokens[:len(first)])),
                               "ms": {k: round(v[0], 3) for k, v in sorted(groups.items(), key=lambda kv: -kv[1][0])
                                      if v[1]}}
        self.pos = self.P
        self.next = self.first_tokens.copy()
        self.stream = stream
        self.frames_host = torch.empty((self.B, L * n), dtype=torch.int8).pin_memory()
        self.resid_host = torch.empty((self.B, L * self.cfg["hidden_size"]), dtype=torch.float16).pin_memory()

    def algorithmic(self):
        """Bytes one decode step must move: every weight once (incl. the tied LM head), each sequence's DeltaNet
        state and conv window read and written, its KV cache read and the new token's K/V written, the captured
        frame and residual rows written."""
        c = self.cfg
        d, n, L, V = c["hidden_size"], c["intermediate_size"], c["num_hidden_layers"], c["vocab_size"]
        hk, hv, dk, dv = (c["linear_num_key_heads"], c["linear_num_value_heads"], c["linear_key_head_dim"],
                          c["linear_value_head_dim"])
        nh, nkv, hd = c["num_attention_heads"], c["num_key_value_heads"], c["head_dim"]
        n_lin = sum(1 for t in c["layer_types"] if t == "linear_attention")
        n_full = L - n_lin
        conv_dim = 2 * hk * dk + hv * dv
        w = V * d + n_lin * ((conv_dim + hv * dv + 2 * hv) * d + d * hv * dv) + n_full * ((2 * nh + 2 * nkv) * hd * d
                                                                                          + d * nh * hd)
        w += L * 3 * n * d
        weights = 2 * w
        state = self.B * n_lin * (hv * dk * dv + (c["linear_conv_kernel_dim"] - 1) * conv_dim) * 4 * 2
        ctx = getattr(self, "pos_timed", self.pos) + 1 + self.mid_steps() // 2
        kv = self.B * n_full * nkv * hd * 2 * 2 * (ctx + 1)
        capture = self.B * L * (n + 2 * d)
        return weights + state + kv + capture

    def mid_steps(self):
        return getattr(self, "_steps", 0)

    def prefill_flops(self):
        """Useful FLOPs of the prefill of B prompts of P tokens (what the split operands double is not counted):
        2 per weight element per row for every projection (the LM head on each prompt's last row only); causal
        attention, 4 hd FLOPs per (query row, head, earlier position); the DeltaNet recurrence, 7 dk dv FLOPs per
        (row, value head) (kv = S^T k, the rank-1 update and o = S^T q)."""
        c = self.cfg
        d, n, L, V = c["hidden_size"], c["intermediate_size"], c["num_hidden_layers"], c["vocab_size"]
        hk, hv, dk, dv = (c["linear_num_key_heads"], c["linear_num_value_heads"], c["linear_key_head_dim"],
                          c["linear_value_head_dim"])
        nh, nkv, hd = c["num_attention_heads"], c["num_key_value_heads"], c["head_dim"]
        n_lin = sum(1 for t in c["layer_types"] if t == "linear_attention")
        n_full = L - n_lin
        conv_dim = 2 * hk * dk + hv * dv
        proj = n_lin * ((conv_dim + hv * dv + 2 * hv) * d + d * hv * dv) + n_full * ((2 * nh + 2 * nkv) * hd * d
                                                                                     + d * nh * hd) + L * 3 * n * d
        rows = self.B * self.P
        attn = n_full * nh * 4 * hd * self.B * (self.P * (self.P + 1) // 2)
        gdn = n_lin * hv * 7 * dk * dv * rows
        return 2 * proj * rows + 2 * V * d * self.B + attn + gdn

    def group_bytes(self, ctx):
        """Algorithmic bytes per decode step of each profiled kernel group (evie_profile groups)."""
        c = self.cfg
        d, n, L, V = c["hidden_size"], c["intermediate_size"], c["num_hidden_layers"], c["vocab_size"]
        hk, hv, dk, dv = (c["linear_num_key_heads"], c["linear_num_value_heads"], c["linear_key_head_dim"],
                          c["linear_value_head_dim"])
        nh, nkv, hd = c["num_attention_heads"], c["num_key_value_heads"], c["head_dim"]
        K = c["linear_conv_kernel_dim"]
        n_lin = sum(1 for t in c["layer_types"] if t == "linear_attention")
        n_full = L - n_lin
        conv_dim = 2 * hk * dk + hv * dv
        B = self.B
        # bf16 weights of each projection group (one cuBLAS GEMM per layer streams its weight once)
        return {
            "gemm_linear_in": 2 * n_lin * (conv_dim + hv * dv + 2 * hv) * d,
            "gemm_linear_out": 2 * n_lin * d * hv * dv,
            "gemm_attn_in": 2 * n_full * (2 * nh + 2 * nkv) * hd * d,
            "gemm_attn_out": 2 * n_full * d * nh * hd,
            "gemm_mlp_gate_up": 2 * L * 2 * n * d,
            "gemm_mlp_down": 2 * L * n * d,
            "lm_head_gemm": 2 * V * d,
            "gdn_mixer": B * n_lin * hv * dk * dv * 4 * 2,
            "conv": B * n_lin * (K - 1) * conv_dim * 4 * 2,
            "gqa_attention": B * n_full * nkv * hd * 2 * 2 * ctx,
            "attn_prep": B * n_full * nkv * hd * 2 * 2,
            # gate and up planes read, the split down_proj operand and the i8 frame written
            "swiglu": B * L * n * (2 * 2 * 4 + 2 * 2 + 1),
        }

    def profile_pass(self, k):
        """k more device-resident steps with the library's per-group CUDA events on (after the timed region). Each
        step is captured as a graph with the events as event-record nodes between the kernel groups, so a group's
        time is its device time inside a replayed step."""
        ctx = self.pos + 1 + k // 2
        self.m.profile(True)
        self.run_device_steps(k)
        prof = self.m.profile_read()
        self.m.profile(False)
        gb = self.group_bytes(ctx)
        total = sum(v[0] for v in prof.values())
        out = {}
        for name, (ms, n) in prof.items():
            if n == 0:
                continue
            per = ms / k
            e = {"ms_per_step": per, "share": ms / total, "launch_groups_per_step": n / k}
            if name in gb and gb[name] > 0:
                e["algorithmic_bytes"] = gb[name]
                e["gbs"] = gb[name] / (per / 1000.0) / 1e9
            out[name] = e
        return out

    def seqs(self):
        from evie_b200.gpu import GpuSeq

        return [GpuSeq(sl, self.pos, self.next[sl:sl + 1]) for sl in range(self.B)]

    def run_device_steps(self, k):
        """k greedy decode steps kept on the device (evie_decode_greedy), captures written on the device."""
        toks = self.m.decode_greedy(self.seqs(), k, capture=True)
        self.last_tokens = toks
        self.next = toks[-1].copy()
        self.pos += k
        return k

    def results(self, logits=False):
        """What rank 0 collects after the timed region: the timed steps' token ids [steps, B] and, as the reduced
        capture, the 16 most active neurons of each sequence's last timed step [B, 16]; with logits, also the next
        step's logits of every sequence [B, V] f32 (one more forward with want_logits)."""
        res = {"token_ids": self.last_tokens.view(np.int32), "top_active": self.m.top_active(16)}
        if logits:
            o = self.m.forward(self.seqs(), want_logits=True)
            self.next = o.next_tokens.copy()
            self.pos += 1
            res["logits"] = o.logits.astype(np.float32)
        return res

    def result_shapes(self, steps, logits=False):
        shp = {"token_ids": (steps, self.B), "top_active": (self.B, 16)}
        if logits:
            shp["logits"] = (self.B, self.cfg["vocab_size"])
        return shp

    def step(self):
        return self.run_device_steps(1)

    def warmup(self, w):
        self.run_device_steps(w)

    def timed(self, k):
        """k device-resident decode steps in one evie_decode_greedy call, timed on the context's stream."""
        import torch

        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        self.pos_timed = self.pos
        a.record(self.stream)
        self.run_device_steps(k)
        b.record(self.stream)
        torch.cuda.synchronize()
        return a.elapsed_time(b), k * self.launches_per_step()

    def launches_per_step(self):
        """Our kernels per decode step: embed+norm; per DeltaNet layer the input projection, conv (which also shifts
        the conv window), mixer, output projection, add-norm x2, gate/up projection, SwiGLU, down projection; per
        attention layer the same with prep + attention in place of conv + mixer; the LM head, logits/argmax + finish,
        row advance. The ncu launch list of the decode step counts the same 293 at 4B shapes (129 of them the
        projection GEMM)."""
        c = self.cfg
        L = c["num_hidden_layers"]
        n_lin = sum(1 for t in c["layer_types"] if t == "linear_attention")
        return 1 + n_lin * 9 + (L - n_lin) * 9 + 4

    def e2e(self, k):
        import torch

        for _ in range(2):
            self.e2e_step()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(self.stream)
        h2d = d2h = 0
        for _ in range(k):
            h2d, d2h = self.e2e_step()
        b.record(self.stream)
        torch.cuda.synchronize()
        return a.elapsed_time(b), h2d, d2h

    def e2e_step(self):
        """One decode step through evie_forward with host buffers: the step's tokens go up, the greedy tokens and
        the captured frames and residual rows come back. The batch is passed as arrays (GpuModel.forward_batch: one
        token per sequence in slot order), as a serving loop over tens of sequences would call it."""
        from evie_b200.gpu import GpuOut

        if not hasattr(self, "_out"):
            self._out = GpuOut(frames=self.frames_host.numpy(), resid=self.resid_host.numpy())
            self._slots = np.arange(self.B, dtype=np.int32)
        o = self.m.forward_batch(self._slots, self.pos, self.next, want_logits=False, capture=True, out=self._out)
        self.next = o.next_tokens.copy()
        self.pos += 1
        c = self.cfg
        return self.B * 4, self.B * 4 + self.B * c["num_hidden_layers"] * (c["intermediate_size"] + 2 * c["hidden_size"])

    def prepare_cpu(self, threads):
        """Inputs of the CPU sample when setup() (the GPU arm) has not run, e.g. for `--impl reference`: the same
        checkpoint (generated the same way, so the GPU arm finds it), pair 0's prompt and the 32 steered
        (layer, neuron) pairs; the dose unit is measured by the oracle on the 64-token sample prompt (median residual
        norm over its tokens 1..), since an oracle pass over the whole 4096-token prompt takes hours on the CPU."""
        import torch

        import oracle
        from evie_b200 import checkpoint as ck

        self.ckpt = self.checkpoint("cuda" if torch.cuda.is_available() else "cpu")
        self.cfg = json.load(open(os.path.join(self.ckpt, "config.json")))
        L, n, V = self.cfg["num_hidden_layers"], self.cfg["intermediate_size"], self.cfg["vocab_size"]
        g = torch.Generator().manual_seed(5)
        self.layers = torch.randint(0, L, (32,), generator=g).tolist()
        self.neurons = torch.randint(0, n, (32,), generator=g).tolist()
        self.prompts = rank_prompts(self.rank, self.B // 2, self.P, V, count=1)
        oracle.set_threads(threads)
        m = oracle.Model(self.ckpt)
        _, _, rs = m.forward([dict(cache=m.new_cache(), tokens=self.prompts[0][:64], resid=True)])
        resid = rs[0].view(np.float16).astype(np.float32).reshape(64, L, -1)
        units = np.median(np.linalg.norm(resid[1:], axis=-1), axis=0)
        ops = []
        for l, nn in zip(self.layers, self.neurons):
            w = ck.read_tensor(self.ckpt, f"model.language_model.layers.{l}.mlp.down_proj.weight")
            col = float(np.sqrt((w[:, nn].astype(np.float64) ** 2).sum()))
            ops.append((l, nn, "add", float(0.6 * units[l] / max(col, 1e-12))))
        self.ops = ops

    def cpu_sample(self, threads):
        """One steered/unsteered pair decoding at the GPU arm's context: the oracle's caches are put at position P
        (the prompt length) with generator-filled states and key/value rows (oracle_cache_seed), since the oracle's
        prefill of a P-token prompt at these shapes takes hours; then a few greedy steps with the steering plan and
        the capture on the steered lane."""
        import oracle

        dose_note = ""
        if not hasattr(self, "ops"):
            self.prepare_cpu(threads)
            dose_note = "; dose unit measured by the oracle on a 64-token prompt"
        oracle.set_threads(threads)
        if getattr(self, "_cpu_model", None) is None:
            self._cpu_model = oracle.Model(self.ckpt)
        m = self._cpu_model
        plan = oracle.compile_plan([dict(layer=l, neuron=nn, mode="add", value=v) for l, nn, _, v in self.ops],
                                   m.cfg.n_layers, m.cfg.intermediate, lambda l, n: 1.0)
        gate = oracle.GateState()
        ca, cb = m.seeded_cache(self.P, 1), m.seeded_cache(self.P, 2)
        nxt = [int(self.prompts[0][-1]), int(self.prompts[0][-1])]
        steps = 0
        t0 = time.perf_counter()
        while steps < 4 and time.perf_counter() - t0 < 30.0:
            lg, _, _ = m.forward([dict(cache=ca, tokens=np.array([nxt[0]], np.uint32), plan=plan, gate=gate,
                                       frames=True),
                                  dict(cache=cb, tokens=np.array([nxt[1]], np.uint32))])
            nxt = [oracle.greedy(lg[0]), oracle.greedy(lg[1])]
            steps += 1
        dt = time.perf_counter() - t0
        return {"value": 2 * steps / dt, "unit": "tokens/s", "cores": threads, "nproc": host_cpus(),
                "kind": "port", "context": self.P,
                "sample": f"1 steered/unsteered pair, {steps} greedy decode steps at context {self.P} (caches put at "
                          f"position {self.P} with generator-filled states and keys/values), steering plan and "
                          f"capture on the steered lane, 4B-shaped model; evie's default threads "
                          f"(half the logical CPUs, at most 8){dose_note}"}


WORKLOADS = {"gdn_decode": GdnDecode, "gdn_prefill": GdnPrefill, "gqa_decode": GqaDecode,
             "model_decode": ModelDecode, "proj_gemm": ProjGemm}


def make_workload(args):
    cls = WORKLOADS[args.workload]
    kw = {"B": args.batch} if args.batch else {}
    if cls is GdnPrefill and args.seq:
        kw["T"] = args.seq
    if cls is ModelDecode:
        kw["rank"] = dist_env()[0]
        kw["model"] = args.model
        if args.prompt:
            kw["prompt"] = args.prompt
    return cls(**kw)
DEFAULT_WORKLOAD = "model_decode"


# ------------------------------------------------------------------------------------------------------------

def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    w = make_workload(args)
    threads = evie_threads()
    vals = []
    for _ in range(args.warmup):
        w.cpu_sample(threads)
    for _ in range(args.steps):
        vals.append(w.cpu_sample(threads))
    v = statistics.median(x["value"] for x in vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": vals[0]["unit"], "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * w.tokens_per_step / v,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": w.dtype, "data": "synthetic",
        "config": w.config(),
        "cpu_baseline": {"value": v, "unit": vals[0]["unit"], "cores": threads, "nproc": host_cpus(),
                         "kind": "port", "sample": vals[0]["sample"]},
        "e2e": {"value": v, "unit": vals[0]["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)
    return 0


ISOLATED = (("gdn_decode", "gdn_decode_step B=64 H=16 dk=dv=128 fp32 state"),
            ("gdn_prefill", "gdn_chunk_prefill B=8 T=8192 H=16 dk=dv=128 chunk=64"),
            ("gqa_decode", "gqa_decode B=64 Hq=16 Hkv=4 hd=256 ctx~U[1024,32768] paged bf16 KV"))


def isolated_passes(dev, steps=10, warmup=3):
    """The three isolated ops of the hot path at their full sizes (the single recurrent DeltaNet step, the chunked
    DeltaNet prefill, the paged attention decode), each timed like a workload of its own after the model's timed
    region, with its roofline against the measured peaks: HBM for the two decode ops, bf16 tensor for the prefill.
    Inputs are drawn on the device (the same distributions as the parity tests' host draws, other values); L2 is
    flushed between steps where the inputs would fit in it."""
    import torch

    pk = peaks()
    out = {}
    for name, label in ISOLATED:
        try:
            w = WORKLOADS[name]()
            w.gen_on_device = True
            w.setup(dev)
            w.warmup(warmup)
            torch.cuda.synchronize()
            ms, _ = w.timed(steps)
            per = ms / steps
            alg = w.algorithmic()
            e = {"workload": label, "ms_per_step": per, "value": w.tokens_per_step / (per / 1000.0),
                 "unit": w.unit}
            if w.bound == "hbm":
                ach = alg / (per / 1000.0) / 1e9
                e["roofline"] = {"bound": "hbm", "achieved": ach, "peak": pk["hbm_gbs"], "unit": "GB/s",
                                 "frac": ach / pk["hbm_gbs"], "kernel": w.kernel, "algorithmic_bytes": alg,
                                 "peak_source": pk["source"]}
            else:
                ach = alg / (per / 1000.0) / 1e12
                e["roofline"] = {"bound": "tensor", "achieved": ach, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                                 "frac": ach / pk["bf16_tflops"], "kernel": w.kernel, "algorithmic_flops": alg,
                                 "peak_source": pk["source"]}
            out[name] = e
            del w
            torch.cuda.empty_cache()
        except Exception as ex:  # the line is still printed without this entry
            print(f"isolated pass {name} failed: {ex}", file=sys.stderr)
    return out


def run_ours(args):
    import torch
    import torch.distributed as dist

    import evie_b200

    rank, world, local = dist_env()
    if world > 1:
        import datetime

        # NCCL's communicator lines (rank count, transport) go to standard error with the rest of the log. A level
        # below INFO inherited from the environment (e.g. VERSION) would hide them, so it is raised; INFO or TRACE
        # set by the caller is kept. Standard output carries only the JSON line.
        if os.environ.get("NCCL_DEBUG", "").upper() not in ("INFO", "TRACE"):
            os.environ["NCCL_DEBUG"] = "INFO"
            os.environ["NCCL_DEBUG_SUBSYS"] = "INIT"
        os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    evie_b200.lib()
    w = make_workload(args)
    w.setup(dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    w.warmup(max(args.warmup, 3))
    torch.cuda.synchronize()
    w._steps = args.steps
    # EVIE_PROFILE_RANGE=1 brackets the timed region with cudaProfilerStart/Stop, so that
    # `ncu --profile-from-start off` lists exactly the timed launches
    prange = os.environ.get("EVIE_PROFILE_RANGE") == "1"
    with Clocks(local) as clk:
        barrier()
        if prange:
            torch.cuda.profiler.start()
        t_wall = time.perf_counter()
        total_ms, launches = w.timed(args.steps)
        barrier()
        t_wall = time.perf_counter() - t_wall
        if prange:
            torch.cuda.profiler.stop()
    clocks = clk.summary()
    barrier()
    # results to rank 0 (token ids and reduced captures), outside the timed region; every rank takes this step
    gathered = None
    if hasattr(w, "results"):
        try:
            res = w.results(logits=args.gather_logits)
        except Exception as e:  # still take the collective steps, with -1 in place of this rank's results
            print(f"results unavailable on rank {rank}: {e}", file=sys.stderr)
            res = {k: np.full(shp, -1, np.float32 if k == "logits" else np.int32)
                   for k, shp in w.result_shapes(args.steps, args.gather_logits).items()}
        gathered = {k: gather_to_rank0(v, device=dev) for k, v in res.items()}
    e2e_ms, h2d, d2h = w.e2e(args.steps)
    kernels = None
    if hasattr(w, "profile_pass"):
        try:
            kernels = w.profile_pass(args.steps)
        except Exception as e:  # the line is still printed, with the whole step as the roofline kernel
            print(f"kernel-group profile unavailable: {e}", file=sys.stderr)
    total_ms, e2e_ms = max_over_ranks([total_ms, e2e_ms], device=dev)

    pk = peaks()
    avg_s = total_ms / 1000.0 / args.steps
    units = w.tokens_per_step * world
    line = {
        "metric": METRIC,
        "value": units / avg_s,
        "unit": w.unit,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": max(args.warmup, 3),
        "ms_per_step": total_ms / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": w.dtype,
        **({"dtype_detail": w.dtype_detail} if getattr(w, "dtype_detail", None) else {}),
        "data": "synthetic",
        "config": dict(w.config(), parallelism=f"dp{world}"),
        "clocks": clocks,
        "e2e": {"value": units / (e2e_ms / 1000.0 / args.steps), "unit": w.unit, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": launches,
        "wall_s": t_wall,
    }
    alg = w.algorithmic()
    if kernels:
        line["kernels"] = kernels
        line["kernels_sum_ms_per_step"] = sum(v["ms_per_step"] for v in kernels.values())
        dom = max((k for k in kernels if "gbs" in kernels[k]), key=lambda k: kernels[k]["ms_per_step"])
        ach = kernels[dom]["gbs"]
        per_launch = kernels[dom]["algorithmic_bytes"] / kernels[dom]["launch_groups_per_step"]
        line["roofline"] = {"bound": "hbm", "achieved": ach, "peak": pk["hbm_gbs"], "unit": "GB/s",
                            "frac": ach / pk["hbm_gbs"], "traffic": profiled_traffic(dom, per_launch), "kernel": dom,
                            "algorithmic_bytes": per_launch,
                            "launch_ms": kernels[dom]["ms_per_step"] / kernels[dom]["launch_groups_per_step"],
                            "peak_source": pk["source"],
                            "step": {"achieved": alg / avg_s / 1e9, "frac": alg / avg_s / 1e9 / pk["hbm_gbs"],
                                     "algorithmic_bytes": alg}}
    elif w.bound == "hbm":
        ach = alg / avg_s / 1e9
        line["roofline"] = {"bound": "hbm", "achieved": ach, "peak": pk["hbm_gbs"], "unit": "GB/s",
                            "frac": ach / pk["hbm_gbs"], "traffic": profiled_traffic(w.kernel),
                            "kernel": w.kernel, "algorithmic_bytes": alg, "peak_source": pk["source"]}
    else:
        ach = alg / avg_s / 1e12
        line["roofline"] = {"bound": "tensor", "achieved": ach, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                            "frac": ach / pk["bf16_tflops"], "traffic": profiled_traffic(w.kernel),
                            "kernel": w.kernel, "algorithmic_flops": alg, "peak_source": pk["source"]}
    if hasattr(w, "prefill_flops") and getattr(w, "prefill_ms", None):
        pf = w.prefill_flops() / (w.prefill_ms / 1000.0) / 1e12
        line["prefill_roofline"] = {"bound": "tensor", "achieved": pf, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                                    "frac": pf / pk["bf16_tflops"], "algorithmic_flops": w.prefill_flops(),
                                    "tok_s": w.prefill_tok_s, "peak_source": pk["source"]}
        if getattr(w, "prefill_groups", None):
            line["prefill_roofline"]["groups_one_call"] = w.prefill_groups
    if rank == 0 and gathered:
        line["gathered"] = {k: list(v.shape) for k, v in gathered.items()}
    if world == 1 and args.workload == DEFAULT_WORKLOAD and not args.no_isolated:
        line["isolated"] = isolated_passes(dev)
    if rank == 0 and world == 1 and not args.no_cpu:
        line["cpu_baseline"] = w.cpu_sample(evie_threads())
    if rank == 0:
        emit(line)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


_OUT = None


def emit(line: dict) -> None:
    """Writes the run's one JSON line to the process's original standard output."""
    out = _OUT or sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def main():
    global _OUT
    # Standard output carries exactly one JSON line: keep a handle on it and send everything else that writes to
    # file descriptor 1 (NCCL's version banner under torchrun, library messages, prints) to standard error.
    sys.stdout.flush()
    _OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    sys.stdout = os.fdopen(os.dup(2), "w", buffering=1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD, choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--gather-logits", action="store_true",
                    help="after the timed region also gather every sequence's next-step logits to rank 0")
    ap.add_argument("--no-isolated", action="store_true",
                    help="skip the isolated passes of the DeltaNet step, chunked prefill and paged attention")
    ap.add_argument("--batch", type=int, default=0, help="override the batch size (small profiling cases)")
    ap.add_argument("--prompt", type=int, default=0, help="override the prompt length of model_decode")
    ap.add_argument("--model", default="4b", choices=["4b", "0.8b"],
                    help="model_decode shapes: Qwen3.5-4B (the benchmark) or 0.8B (small profiling cases)")
    ap.add_argument("--seq", type=int, default=0, help="override the sequence length of gdn_prefill")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
