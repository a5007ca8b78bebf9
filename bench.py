"""Benchmark of the GPU-resident rollout hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl mine|reference]

Workloads (synthetic, seeded):
  rollout    config 5 (default): 8,192 GRPO rollouts, the GPU-resident loop.
             Under torchrun the fixed 8,192 rollouts are split by group over
             the N GPUs (strong scaling: the total work is the same for every
             N); the only collective is the NCCL allgather of rewards.  At
             N = 1 the line also carries blocks for configs 2, 3 and 4.
  rollout_c4 config 4: 1,024 rollouts with Poisson arrivals (8 per ms), a
             shared 1,024-token copy-on-write prefix plus per-group prompts
             of U[64,1024] tokens, max_new U[32,512] (one GPU; under
             torchrun every rank runs its own replica: weak scaling).
  attention  config 2: paged GQA decode attention, B=64 ragged sequences
             L ~ U[128,4096], 32 q / 8 kv heads, d=128, bf16 16-token pages
             scattered in the arena.  Two arena copies (> L2) alternate.
  sampling   config 3: 256 rows x 32,000 fp32 logits, fused sampling.
  decode_ring  the reference's per-step CommandRing benchmark (src/main.c).
  lm_head, rollout_model  the model-decode extension (tensor-core GEMMs).
  Except for rollout, every rank runs its own replica (weak scaling).

--impl reference times the CPU implementation of the same workload on this
host's cores: the reference project has no CPU implementation of paged
attention or of the rollout loop, so it is the CPU restatement of the
reference's algorithms (oracle/), fed numpy inputs of the same shapes and
distributions, without loading this runtime or touching the GPU.  Its line
has the same config, steps and warm-up as the GPU arm; each step is a
bounded sample of the workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
import __graft_entry__ as ge  # noqa: E402

HBM_FALLBACK_GBS = 6650.0


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except OSError:
        return {"hbm_gbs": HBM_FALLBACK_GBS, "bf16_tflops": 1590.0}, "fallback"


def ncu_traffic(kernel: str, workload: str):
    """Per-launch DRAM bytes recorded from an ncu capture in profiles/ncu_traffic.txt
    (lines: <kernel> <workload> <bytes_per_launch> <commit of the capture>);
    (None, None) when not recorded."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic.txt")
    try:
        with open(path) as f:
            for line in f:
                parts = line.split()
                if (len(parts) >= 3 and not line.startswith("#") and parts[0] == kernel
                        and parts[1] == workload):
                    return float(parts[2]), (parts[3] if len(parts) > 3 else None)
    except OSError:
        pass
    return None, None


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and clock-event reasons via NVML while running."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.05):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self.period = period_s
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            import torch
            props = torch.cuda.get_device_properties(device_index)
            bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
            self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
            self.nvml = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # noqa: BLE001 - clocks are reported as unavailable
            self.nvml = None
            self.err = repr(e)

    def _sample(self):
        n = self.nvml
        self.samples.append(n.nvmlDeviceGetClockInfo(self.h, n.NVML_CLOCK_SM))
        try:
            mask = n.nvmlDeviceGetCurrentClocksEventReasons(self.h)
        except AttributeError:
            mask = n.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
        for bit, name in self.REASONS.items():
            if mask & bit and name != "gpu_idle":
                self.reasons.add(name)

    def _run(self):
        while not self._stop.is_set():
            self._sample()
            time.sleep(self.period)

    def start(self):
        if self.nvml:
            self._sample()
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()

    def stop(self):
        if self.nvml:
            self._stop.set()
            self._thread.join()
            self._sample()

    def report(self):
        if not self.nvml:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "error": self.err}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ------------------------------------------------- CPU ports (no GPU, no runtime)
def _bf16_normal(rng, shape, std=1.0):
    """bf16 bit patterns of N(0, std) values (truncated float32), generated
    in chunks to bound the float32 temporaries."""
    out = np.empty(int(np.prod(shape)), dtype=np.uint16)
    step = 1 << 24
    for i in range(0, out.size, step):
        x = rng.standard_normal(min(step, out.size - i), dtype=np.float32)
        if std != 1.0:
            x *= np.float32(std)
        out[i:i + x.size] = x.view(np.uint32) >> 16
    return out.reshape(shape)


_PORT_INPUTS = {}


def _cached(key, make):
    """Port inputs are built once per process: the reference arm calls a
    port once per step."""
    if key not in _PORT_INPUTS:
        _PORT_INPUTS[key] = make()
    return _PORT_INPUTS[key]


def _port_rollout_decode(threads, budget_s, n_rollouts, ctx, gen, vocab, seed):
    """The loop's decode step on the host for one GRPO group: `n_rollouts`
    rollouts whose first ctx tokens are one shared prompt (the same page ids
    in every page table) and whose private pages are scattered through the
    arena; per token paged GQA attention over the whole context
    (oracle/oracle.c, OpenMP over (rollout, kv head)), N(0, 2) logits, and
    the reference sampling algorithm (cu/sample.cu:40-123 restated,
    insertion top-k) per rollout on a thread pool.  Decodes until the time
    budget is spent (at least one token).  Returns (tokens, steps, seconds)."""
    from concurrent.futures import ThreadPoolExecutor
    orc = ge.load_oracle()
    B, Hq, Hkv = n_rollouts, 32, 8
    rng = np.random.default_rng(seed)
    shared = ctx // 16
    own = (ctx + gen + 15) // 16 - shared

    def make():
        n_pages = shared + B * own
        arena_pages = int(n_pages * 1.25) + 1
        perm = rng.permutation(arena_pages).astype(np.int32)
        pt = np.zeros((B, shared + own), dtype=np.int32)
        pt[:, :shared] = perm[:shared]
        pt[:, shared:] = perm[shared:shared + B * own].reshape(B, own)
        return pt, _bf16_normal(rng, arena_pages * Hkv * 2 * 16 * 128)
    pt, arena = _cached(("rollout", B, ctx, gen, seed), make)
    pool = ThreadPoolExecutor(max_workers=threads)
    t0 = time.perf_counter()
    steps = 0
    while steps == 0 or (time.perf_counter() - t0 < budget_s and steps < gen):
        q = _bf16_normal(rng, (B, Hq, 128))
        lens = np.full(B, ctx + steps + 1, dtype=np.int32)
        orc.paged_gqa_attention(q, arena, pt, lens, Hq, Hkv, 128 ** -0.5, n_threads=threads)
        logits = rng.standard_normal((B, vocab), dtype=np.float32) * np.float32(2.0)
        list(pool.map(lambda b: orc.sample_row(logits[b], 0.8, 50, 0.9,
                                               orc.sample_u24(1234, b, steps)), range(B)))
        steps += 1
    dt = time.perf_counter() - t0
    pool.shutdown()
    return B * steps, steps, dt


def _port_result(value, unit, threads, dt, sample):
    return {"value": value, "unit": unit, "cores": threads, "kind": "port", "seconds": dt,
            "sample": sample}


# ------------------------------------------------------------- workloads
class Workload:
    """Common surface: a GPU step plus class-level facts that the reference
    arm uses without the GPU (static_config, cpu_port)."""

    scaling = "weak"          # every rank runs its own replica
    dtype = "bf16"
    bound = "hbm"
    launches_per_step = 1

    @classmethod
    def line_config(cls, args, world):
        """The config object of both arms' JSON lines (GPU-independent)."""
        par = (f"dp{world} (groups split by rank)" if cls.scaling == "strong"
               else f"replicas{world}") if world > 1 else "single"
        return cls.static_config(args, world) | {"parallelism": par}

    def config(self):
        return self.line_config(self.args, self.world)

    def details(self):
        return {}

    def gpu_launches(self, steps):
        return self.launches_per_step * steps

    def check_errors(self):
        return 0


def _c2_inputs(rank):
    """Config-2 lengths and scattered page table (numpy, seeded)."""
    B = 64
    lens = np.random.default_rng(2 + 1000 * rank).integers(128, 4097, size=B).astype(np.int32)
    rng = np.random.default_rng(20 + rank)
    n_pages = (lens + 15) // 16
    P = int(n_pages.max())
    arena_pages = int(int(n_pages.sum()) * 1.25) + 1
    pt = np.full((B, P), -1, dtype=np.int32)
    perm = rng.permutation(arena_pages).astype(np.int32)
    k = 0
    for b, n in enumerate(n_pages):
        pt[b, :n] = perm[k:k + n]
        k += n
    return lens, pt, arena_pages


class AttentionWorkload(Workload):
    """BASELINE config 2 (paged GQA decode attention)."""

    name = "paged_gqa_decode_attention_c2"
    kernel = "paged_gqa_decode_kernel"
    metric = "decode-attn HBM GB/s (paged GQA, config 2)"
    unit = "GB/s"
    B, Hq, Hkv = 64, 32, 8

    @classmethod
    def static_config(cls, args, world):
        return {"workload": cls.name, "batch": cls.B, "seq_len": "U[128,4096], seed 2 (+1000 x rank)",
                "q_heads": cls.Hq, "kv_heads": cls.Hkv, "head_dim": 128, "page_tokens": 16,
                "kv_dtype": "bf16", "pages": "scattered (random permutation of a 1.25x arena)",
                "l2": "two arena copies alternate (2 x ~0.55 GB > 126 MB L2)",
                "chunk_pages": args.chunk_pages or "auto"}

    @staticmethod
    def algorithmic_bytes(lens, Hq=32, Hkv=8):
        n_pages = (lens + 15) // 16
        return (int(lens.sum()) * Hkv * 128 * 2 * 2 + len(lens) * Hq * 128 * (2 + 4)
                + int(n_pages.sum()) * 4)

    def __init__(self, args, rank, world, dev):
        import torch
        self.args, self.world = args, world
        self.torch = torch
        self.pkg = ge.load_package()
        self.dev = dev
        self.lens, pt, self.arena_pages = _c2_inputs(rank)
        self.P = pt.shape[1]
        self.page_table = torch.from_numpy(pt).to(dev)
        self.seq_lens = torch.from_numpy(self.lens).to(dev)
        elems = self.arena_pages * self.Hkv * 2 * 16 * 128
        self.arenas = []
        for _ in range(2):
            a = torch.empty(elems, dtype=torch.bfloat16, device=dev)
            self.pkg.fill_normal_bf16(a, seed=2 + rank, stream_id=1)   # same contents, two copies
            self.arenas.append(a)
        self.q = torch.empty(self.B, self.Hq, 128, dtype=torch.bfloat16, device=dev)
        self.pkg.fill_normal_bf16(self.q, seed=2 + rank, stream_id=2)
        self.out = torch.empty(self.B, self.Hq, 128, dtype=torch.float32, device=dev)
        # pure streaming (no page is shared): evict-first keeps L2 clean
        self.attn = self.pkg.PagedDecodeAttention(self.B, self.Hq, self.Hkv, self.P,
                                                  int(self.lens.max()), self.arena_pages,
                                                  chunk_pages=args.chunk_pages, evict_first=True)
        self.i = 0
        self.kv_bytes = int(self.lens.sum()) * self.Hkv * 128 * 2 * 2
        self.bytes = self.algorithmic_bytes(self.lens)
        self.flops = 4 * self.Hq * 128 * int(self.lens.sum())
        torch.cuda.synchronize()

    def step(self):
        self.attn(self.q, self.arenas[self.i & 1], self.page_table, self.seq_lens, out=self.out)
        self.i += 1

    def units_per_step(self):
        return self.bytes / 1e9  # GB

    def e2e(self, steps, warmup):
        """Same metric through the C ABI with host buffers: the step's query is
        copied from pinned host memory and the output read back each step (the
        KV arena is the resident cache)."""
        torch = self.torch
        q_h = self.q.cpu().pin_memory()
        out_h = torch.empty(self.out.shape, dtype=torch.float32).pin_memory()
        s = torch.cuda.current_stream()

        def one():
            self.q.copy_(q_h, non_blocking=True)
            self.step()
            out_h.copy_(self.out, non_blocking=True)

        for _ in range(warmup):
            one()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(steps):
            one()
        e1.record(s)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        return {"value": self.units_per_step() / (ms / 1e3), "unit": self.unit,
                "ms_per_step": ms, "h2d_bytes_per_step": int(q_h.numel() * 2),
                "d2h_bytes_per_step": int(out_h.numel() * 4)}

    def check_errors(self):
        return self.attn.error_code()

    @classmethod
    def cpu_port(cls, args, threads, budget_s):
        """The CPU restatement (oracle/oracle.c, fp64 accumulate, OpenMP over
        (sequence, kv head)) on config-2 inputs built with numpy: batches of
        8 of the 64 sequences, in turn, until the budget is spent."""
        orc = ge.load_oracle()

        def make():
            lens, pt, arena_pages = _c2_inputs(0)
            rng = np.random.default_rng(21)
            return (lens, pt, _bf16_normal(rng, arena_pages * cls.Hkv * 2 * 16 * 128),
                    _bf16_normal(rng, (cls.B, cls.Hq, 128)))
        lens, pt, arena, q = _cached("c2", make)
        t0 = time.perf_counter()
        done_bytes, k, seqs = 0, 0, 0
        while k == 0 or time.perf_counter() - t0 < budget_s:
            sl = slice(8 * (k % 8), 8 * (k % 8) + 8)
            orc.paged_gqa_attention(q[sl], arena, pt[sl], lens[sl], cls.Hq, cls.Hkv, 128 ** -0.5,
                                    n_threads=threads)
            done_bytes += cls.algorithmic_bytes(lens[sl])
            seqs += 8
            k += 1
        dt = time.perf_counter() - t0
        return _port_result(done_bytes / 1e9 / dt, cls.unit, threads, dt,
                            f"{seqs} config-2 sequences in batches of 8, oracle/oracle.c "
                            f"fp64-accumulate restatement, OpenMP")

    def details(self):
        return {"chunk_pages_used": self.attn.plan()[0], "tokens": int(self.lens.sum())}


class SamplingWorkload(Workload):
    """256 rows x 32,000 fp32 logits ~ N(0, 2), T=0.8,
    top-k 50, top-p 0.9, Philox seed 1234, counter = (rollout_id = row, step).
    Eight logits buffers (262 MB > 126 MB L2) rotate between steps."""

    name = "fused_sampling_c3"
    kernel = "sample_rows_kernel"
    metric = "sampling logits HBM GB/s (config 3)"
    unit = "GB/s"
    dtype = "fp32"
    R, V, NBUF = 256, 32000, 8

    @classmethod
    def static_config(cls, args, world):
        return {"workload": cls.name, "rows": cls.R, "vocab": cls.V, "temperature": 0.8,
                "top_k": 50, "top_p": 0.9, "seed": 1234, "logits": "N(0, 2)",
                "l2": "8 logits buffers rotate (262 MB > 126 MB L2)"}

    def __init__(self, args, rank, world, dev):
        import torch
        self.args, self.world = args, world
        self.torch = torch
        self.pkg = ge.load_package()
        self.bufs = []
        for i in range(self.NBUF):
            t = torch.empty(self.R, self.V, dtype=torch.float32, device=dev)
            self.pkg.fill_normal_f32(t, seed=3 + rank, stream_id=100 + i, std=2.0)
            self.bufs.append(t)
        rows = self.pkg.sample_row_table(0.8, 50, 0.9, np.arange(self.R, dtype=np.uint32), 0, 1234)
        self.rows = torch.from_numpy(rows.view(np.uint8)).to(dev)
        self.out = torch.empty(self.R, dtype=torch.int32, device=dev)
        self.bytes = self.R * self.V * 4 + self.R * (32 + 4)
        self.i = 0
        torch.cuda.synchronize()
        # the kernel is shorter than a Python ctypes call: steps replay one
        # captured call per buffer so the launch gaps do not set the time
        self.graphs = self._graphs(lambda i: self.pkg.sample_rows(
            self.bufs[i], self.rows, self.V, out=self.out))

    def _graphs(self, call):
        """One CUDA graph per logits buffer holding call(buffer index)."""
        torch = self.torch
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for i in range(self.NBUF):
                call(i)
        torch.cuda.current_stream().wait_stream(side)
        graphs = []
        for i in range(self.NBUF):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                call(i)
            graphs.append(g)
        torch.cuda.synchronize()
        return graphs

    def step(self):
        self.graphs[self.i % self.NBUF].replay()
        self.i += 1

    def units_per_step(self):
        return self.bytes / 1e9

    def details(self):
        """The same calls given each buffer's 16-column chunk maxima
        (rt_sample_rows_cmax, the rollout loop's path: its logits kernel
        writes them), CUDA events over 50 graph-replayed calls on the
        rotating buffers, and the standalone chunk-maximum kernel; tokens
        compared with the full-row path."""
        torch, pkg = self.torch, self.pkg
        cms = [pkg.logits_chunk_max(b, self.V) for b in self.bufs]
        full = [pkg.sample_rows(b, self.rows, self.V).clone() for b in self.bufs]
        got = [pkg.sample_rows_cmax(b, c, self.rows, self.V).clone()
               for b, c in zip(self.bufs, cms)]
        equal = all(bool(torch.equal(a, b)) for a, b in zip(full, got))
        s = torch.cuda.current_stream()

        def timed(fn, n=50):
            for i in range(5):
                fn(i)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            for i in range(n):
                fn(i)
            e1.record(s)
            torch.cuda.synchronize()
            return e0.elapsed_time(e1) * 1e3 / n

        g_s = self._graphs(lambda i: pkg.sample_rows_cmax(self.bufs[i], cms[i], self.rows,
                                                          self.V, out=self.out))
        g_c = self._graphs(lambda i: pkg.logits_chunk_max(self.bufs[i], self.V, out=cms[i]))
        us_cm = timed(lambda i: g_c[i % self.NBUF].replay())
        us = timed(lambda i: g_s[i % self.NBUF].replay())
        return {"producer_maxima": {
            "us_per_call": us, "tokens_equal_full_path": equal,
            "chunk_max_kernel_us": us_cm,
            "note": "rt_sample_rows_cmax reads each row's 2,000 chunk maxima and only the "
                    "chunks that can hold a top-k survivor; the value above is the full-row "
                    "path (rt_sample_rows)"}}

    def e2e(self, steps, warmup):
        """Logits rows copied from pinned host memory each step, tokens read back."""
        torch = self.torch
        host = self.bufs[0].cpu().pin_memory()
        tok_h = torch.empty(self.R, dtype=torch.int32).pin_memory()
        s = torch.cuda.current_stream()

        def one():
            self.bufs[0].copy_(host, non_blocking=True)
            self.pkg.sample_rows(self.bufs[0], self.rows, self.V, out=self.out)
            tok_h.copy_(self.out, non_blocking=True)

        for _ in range(warmup):
            one()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(steps):
            one()
        e1.record(s)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        return {"value": self.units_per_step() / (ms / 1e3), "unit": self.unit, "ms_per_step": ms,
                "h2d_bytes_per_step": int(host.numel() * 4), "d2h_bytes_per_step": self.R * 4}

    @classmethod
    def cpu_port(cls, args, threads, budget_s):
        """The reference algorithm (cu/sample.cu:40-123 restated in
        oracle/oracle.c, insertion top-k) over numpy N(0, 2) rows, rows in
        parallel on a thread pool, until the budget is spent."""
        from concurrent.futures import ThreadPoolExecutor
        orc = ge.load_oracle()
        rows = _cached("c3", lambda: np.random.default_rng(3).standard_normal(
            (cls.R, cls.V), dtype=np.float32) * np.float32(2.0))
        pool = ThreadPoolExecutor(max_workers=threads)
        t0 = time.perf_counter()
        n = 0
        while n == 0 or time.perf_counter() - t0 < budget_s:
            batch = [(n + j) % cls.R for j in range(threads)]
            list(pool.map(lambda r: orc.sample_row(rows[r], 0.8, 50, 0.9,
                                                   orc.sample_u24(1234, r, 0)), batch))
            n += len(batch)
        dt = time.perf_counter() - t0
        pool.shutdown()
        return _port_result(n * cls.V * 4 / 1e9 / dt, cls.unit, threads, dt,
                            f"{n} config-3 rows, reference algorithm, {threads} rows at a time")


def _traj_checksum(torch, traj, lengths):
    """Order-sensitive checksum of the written part of a trajectory buffer
    (row r holds lengths[r] tokens; the rest of the row is never written)."""
    width = traj.shape[1]
    valid = torch.arange(width, device=traj.device)[None, :] < lengths[:, None]
    w = torch.arange(1, traj.numel() + 1, device=traj.device, dtype=torch.int64) % 1000003
    return int((traj.to(torch.int64) * valid * w.view(traj.shape)).sum().item())


class RolloutWorkload(Workload):
    """BASELINE config 5 (config 2's attention shape and config-3 sampling):
    8,192 rollouts = 512 GRPO groups x 16, split by group across the N GPUs
    (strong scaling: the same 8,192 rollouts whatever N).  Each group's 16
    rollouts share a 512-token prompt held once in the KV arena
    (copy-on-write prefix); each rollout generates 256 tokens.  One step =
    one RL step: every local rollout generated to completion by the
    GPU-resident loop (requests from a device array), rewards ~ U(0,1)
    (Philox seed 5) allgathered over NCCL, group-normalised advantages."""

    name = "grpo_rollouts_c5"
    kernel = "paged_gqa_group_kernel+paged_gqa_decode_kernel"  # attention of one pass
    metric = "rollout tokens/s (config 5; value = all GPUs, per GPU = value / n_gpus)"
    unit = "tokens/s"
    scaling = "strong"
    launches_per_step = None  # counted from the loop's pass counter
    launches_per_pass = 5

    GROUPS, G, PROMPT, GEN, VOCAB = 512, 16, 512, 256, 32000
    DECODE_MODE = 1  # q, K/V and logits from Philox (the reference has no model)

    @classmethod
    def static_config(cls, args, world):
        groups = args.groups or cls.GROUPS
        return {"workload": cls.name, "rollouts": groups * cls.G, "groups": groups,
                "group_size": cls.G, "prompt_tokens": cls.PROMPT, "new_tokens": cls.GEN,
                "q_heads": 32, "kv_heads": 8, "head_dim": 128, "page_tokens": 16,
                "vocab": cls.VOCAB, "sampling": "T=0.8 top-k 50 top-p 0.9", "slots": 256,
                "reward": "U(0,1) Philox seed 5, NCCL allgather, GRPO advantages",
                "l2": "KV arena > 126 MB L2 (prompts + 256 slots x 17 private pages)"}

    def __init__(self, args, rank, world, dev):
        import torch
        self.args, self.world = args, world
        self.torch = torch
        self.pkg = pkg = ge.load_package()
        self.rank, self.dev = rank, dev
        if getattr(args, "groups", 0):
            self.GROUPS = args.groups
        self.g0, self.ng = pkg.shard_groups(self.GROUPS, world, rank)
        self.n = self.ng * self.G
        pages_prompt = self.PROMPT // 16
        priv = 256 * ((self.GEN + 16 + 15) // 16)
        self.arena = pkg.DeviceArena(self.ng * pages_prompt + priv + 64, device=dev)
        cfg = dict(num_q_heads=32, num_kv_heads=8, vocab=self.VOCAB, max_slots=256,
                   max_context=self.PROMPT + self.GEN, max_new_tokens=self.GEN, max_admit=256,
                   drop_when_full=0, decode_mode=self.DECODE_MODE, reward_mode=1, reward_seed=5,
                   logit_std=2.0,
                   max_prefixes=self.ng, max_prefix_pages=self.ng * pages_prompt,
                   max_passes=1 << 24, idle_timeout_ms=20000, chunk_pages=args.chunk_pages)
        self.eng = pkg.RolloutEngine(cfg, self.arena)
        prompt_pages = self.arena.acquire(self.ng * pages_prompt)
        self.arena.fill_pages(prompt_pages, seed=4 + rank, stream_id=0)  # synthetic prefill (untimed)
        for g in range(self.ng):
            self.eng.set_prefix(g, prompt_pages[g * pages_prompt:(g + 1) * pages_prompt], self.PROMPT)
        self._attach_model(torch, dev, rank)
        r = np.zeros(self.n, dtype=np.dtype(pkg.REQUEST_RECORD))
        gid = np.arange(self.n) // self.G                       # local group
        r["request_id"] = (np.arange(self.n, dtype=np.uint64) + np.uint64(self.g0 * self.G + 1)) | \
            ((gid.astype(np.uint64) + np.uint64(1)) << np.uint64(32))
        r["max_tokens"] = self.GEN
        r["kv_blocks"] = pages_prompt
        r["temperature"], r["top_k"], r["top_p"], r["rng_seed"] = 0.8, 50, 0.9, 1234
        self._make_buffers(torch, dev, r)
        self.arrivals = None
        self.tokens_per_step = self.n * self.GEN
        torch.cuda.synchronize()

    def _make_buffers(self, torch, dev, r):
        self.reqs_host = r
        self.req_d = torch.from_numpy(r.view(np.uint8).copy()).to(dev)
        self.dones = torch.zeros(self.n * 24, dtype=torch.uint8, device=dev)
        self.state = torch.zeros(72 * 256 + 32, dtype=torch.uint8, device=dev)
        self.traj = torch.zeros(self.n, int(r["max_tokens"].max()), dtype=torch.int32, device=dev)
        self.rewards = torch.zeros(self.n, dtype=torch.float32, device=dev)
        total = self.GROUPS * self.G if self.scaling == "strong" else self.n
        self.all_rewards = torch.zeros(total, dtype=torch.float32, device=dev)
        self.adv = torch.zeros_like(self.all_rewards)
        self.nccl = None
        if self.world > 1 and self.scaling == "strong":
            import torch.distributed as dist

            def exchange(b):
                obj = [b]
                dist.broadcast_object_list(obj, src=0)
                return obj[0]
            self.nccl = self.pkg.NcclRewards(self.rank, self.world, exchange)

    def _attach_model(self, torch, dev, rank):
        pass

    def _post(self, stream=None):
        if self.nccl:
            self.nccl.allgather(self.rewards, self.all_rewards, stream=stream)
        else:
            self.all_rewards.copy_(self.rewards)
        self.pkg.grpo_advantages(self.all_rewards, self.G, out=self.adv, stream=stream)

    def _launch(self, **kw):
        self.eng.launch(requests=self.req_d, n_requests=self.n, dones=self.dones, state=self.state,
                        trajectories=self.traj, rewards=self.rewards, n_rows=self.n,
                        arrivals=self.arrivals, arrival_unit=self.pkg.RT_ARRIVAL_NS, **kw)

    def step(self):
        self._launch()
        self._post()

    def units_per_step(self):
        return float(self.tokens_per_step)

    def check_errors(self):
        st = self.eng.wait()
        self.last_stats = st
        return st["error"] or st["attn_error"]

    def gpu_launches(self, steps):
        # per pass: schedule, prepare, attention, logits, sampler; per step:
        # one allgather (when N > 1) and one advantage kernel
        per_step = 2 if self.nccl else 1
        return int(self.last_stats["passes"]) * self.launches_per_pass * steps + per_step * steps

    def trajectory_check(self, sample_rows=64):
        """After the timed steps: the trajectories of one more step (buffer
        cleared first) equal those the timed steps left (the run is seeded
        and deterministic), and a sample of rollouts (every n/64-th) equals a
        token-by-token replay of the loop's logits through the standalone
        sampler."""
        torch = self.torch
        lengths = torch.from_numpy(self.reqs_host["max_tokens"].astype(np.int64)).to(self.traj.device)
        before = _traj_checksum(torch, self.traj, lengths)
        self.traj.fill_(-1)
        self.step()
        self.eng.wait()
        after = _traj_checksum(torch, self.traj, lengths)
        rows = range(0, self.n, max(1, self.n // sample_rows))
        total, bad = self.pkg.replay_trajectories(self.reqs_host, self.traj.cpu().numpy(), rows,
                                                  self.VOCAB)
        ok = before == after and not bad
        return {"result": "equal" if ok else "DIFFERENT", "checksum_timed": before,
                "checksum_check_step": after, "replayed_rollouts": len(rows),
                "replayed_tokens": total, "mismatches": len(bad), "first_mismatches": bad[:3]}

    def rank_diagnostics(self):
        """One more step with CUDA events around the loop and around the
        reward exchange + advantages (the allgather waits for the slowest
        rank, so its time shows imbalance), plus passes and waves."""
        torch = self.torch
        e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        e[0].record()
        self._launch()
        e[1].record()
        self._post()
        e[2].record()
        torch.cuda.synchronize()
        st = self.eng.wait()
        return {"rank": self.rank, "rollouts": self.n, "waves": -(-self.n // 256),
                "passes": int(st["passes"]), "loop_ms": e[0].elapsed_time(e[1]),
                "allgather_adv_ms": e[1].elapsed_time(e[2])}

    def e2e(self, steps, warmup):
        """Through the C ABI with host buffers: requests pushed into a mapped
        RequestRing and dones drained from a mapped DoneRing by the host C
        pump (rt_host_pump), then the trajectories and advantages copied to
        pinned host memory; all inside the timed region."""
        torch = self.torch
        rings = self.pkg.HostRings()
        traj_h = torch.empty(self.traj.shape, dtype=torch.int32).pin_memory()
        adv_h = torch.empty(self.adv.shape, dtype=torch.float32).pin_memory()
        s = torch.cuda.current_stream()

        def one():
            self.eng.launch(ring=rings.req, done_ring=rings.done, state=self.state,
                            trajectories=self.traj, rewards=self.rewards, n_rows=self.n)
            got, _ = rings.pump(self.reqs_host, self.n, send_sentinel=True, timeout_ms=120000)
            if got != self.n:
                raise RuntimeError(f"e2e pump drained {got} of {self.n}")
            self._post()
            traj_h.copy_(self.traj, non_blocking=True)
            adv_h.copy_(self.adv, non_blocking=True)

        for _ in range(min(warmup, 1)):
            one()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(steps):
            one()
        e1.record(s)
        torch.cuda.synchronize()
        self.eng.wait()
        rings.close()
        ms = e0.elapsed_time(e1) / steps
        return {"value": self.units_per_step() / (ms / 1e3), "unit": self.unit, "ms_per_step": ms,
                "h2d_bytes_per_step": self.n * 34,
                "d2h_bytes_per_step": self.n * 24 + traj_h.numel() * 4 + adv_h.numel() * 4}

    @staticmethod
    def _pct(x, scale=1e3):
        x = np.sort(np.asarray(x, dtype=np.float64))
        if not len(x):
            return None
        q = lambda f: round(float(x[min(len(x) - 1, int(f * len(x)))]) / scale, 2)
        return {"n": int(len(x)), "p50": q(0.5), "p90": q(0.9), "p99": q(0.99),
                "max": round(float(x[-1]) / scale, 2)}

    def trace_report(self):
        """One more RL step, untimed, with the device trace attached
        (rt_rollout_set_trace): device-clock latencies in the manner of the
        reference's trace report (docs/tracing.md), from the schedule
        kernel's records: rollout alloc -> trajectory done, and the interval
        between decode passes."""
        tr = self.pkg.DeviceTrace(1 << 18)
        self.eng.set_trace(tr)
        self.step()
        self.eng.wait()
        self.eng.set_trace(None)
        rec, total = tr.read()
        pk = self.pkg
        alloc = {}
        life = []
        for r in rec:
            t = int(r["type"])
            if t == pk.TRACE_ROLLOUT_ALLOC:
                alloc[int(r["rollout_id"])] = int(r["tsc"])
            elif t == pk.TRACE_TRAJECTORY_DONE and int(r["rollout_id"]) in alloc:
                life.append(int(r["tsc"]) - alloc.pop(int(r["rollout_id"])))
        passes = rec[rec["type"] == pk.TRACE_DECODE_BATCH]["tsc"].astype(np.int64)
        return {"clock": "GPU globaltimer, ns -> us", "records": int(total),
                "rollout_alloc_to_done_us": self._pct(life),
                "decode_pass_interval_us": self._pct(np.diff(passes))}

    def kernel_profile(self, n_rollouts=512):
        """Per-kernel device time from a host-stepped replay (rt_rollout_profile)
        of the first n_rollouts of the step."""
        n = min(n_rollouts, self.n)
        return self.eng.profile(requests=self.req_d, n_requests=n, dones=self.dones,
                                state=self.state, trajectories=self.traj, rewards=self.rewards,
                                n_rows=self.n)

    @classmethod
    def cpu_port(cls, args, threads, budget_s):
        tokens, steps, dt = _port_rollout_decode(threads, budget_s, cls.G, cls.PROMPT, cls.GEN,
                                                 cls.VOCAB, seed=11)
        return _port_result(tokens / dt, cls.unit, threads, dt,
                            f"1 group x 16 rollouts, {steps} decode steps from a shared 512-token "
                            f"prompt, scattered private pages (attention + logits + reference "
                            f"sampling per token)")

    def details(self):
        return {"rollouts_per_gpu": self.n,
                "arena_gb": round(self.arena.buf.numel() / 1e9, 3)}


class RolloutC4Workload(RolloutWorkload):
    """BASELINE config 4, continuous batching on one GPU: 1,024 rollouts in
    64 GRPO groups of 16 arriving as a Poisson process (exponential gaps,
    mean 1/8 ms, seed 4, in group order).  Every context starts with the
    same registered 1,024-token copy-on-write prefix followed by the group's
    prompt of U[64,1024] tokens (one per group, seed 4), so most groups'
    contexts end mid-page; each rollout generates U[32,512] tokens (seed 4).
    Attention shape of config 2, sampling of config 3, synthetic logits.

    value: one step = the loop over the 1,024 requests held in a device
    array, each admitted no earlier than its arrival time (the schedule
    kernel reads the GPU clock), then rewards and advantages; tokens/s is
    the generated tokens over that device time, so it includes the arrival
    span (~128 ms) and the drain.
    e2e: the host C pump pushes the requests into the mapped RequestRing at
    their arrival times (rt_host_pump_paced) and drains the DoneRing; the
    latency of each rollout (arrival -> done record drained) is reported."""

    name = "continuous_batching_c4"
    metric = "rollout tokens/s (config 4: Poisson arrivals, continuous batching)"
    scaling = "weak"
    N_ROLLOUTS, G, BASE, GEN, VOCAB, RATE_PER_MS = 1024, 16, 1024, 512, 32000, 8.0

    @classmethod
    def inputs(cls, seed=4):
        rng = np.random.default_rng(seed)
        prompt = rng.integers(64, 1025, size=cls.N_ROLLOUTS // cls.G)
        max_new = rng.integers(32, 513, size=cls.N_ROLLOUTS)
        gaps = rng.exponential(1e6 / cls.RATE_PER_MS, size=cls.N_ROLLOUTS)
        arrival_ns = np.cumsum(gaps) - gaps[0]
        return prompt, max_new, arrival_ns.astype(np.uint64)

    @classmethod
    def static_config(cls, args, world):
        prompt, max_new, arr = cls.inputs()
        return {"workload": cls.name, "rollouts": cls.N_ROLLOUTS, "groups": cls.N_ROLLOUTS // cls.G,
                "group_size": cls.G, "arrivals": "Poisson, mean 8 per ms (exponential gaps, seed 4)",
                "arrival_span_ms": round(float(arr[-1]) / 1e6, 2),
                "shared_prefix_tokens": cls.BASE, "prompt_tokens": "U[64,1024] per group, seed 4",
                "new_tokens": "U[32,512] per rollout, seed 4",
                "generated_tokens": int(max_new.sum()), "q_heads": 32, "kv_heads": 8,
                "head_dim": 128, "page_tokens": 16, "vocab": cls.VOCAB,
                "sampling": "T=0.8 top-k 50 top-p 0.9", "slots": 256,
                "admission": "all free slots per pass, backpressure (requests wait, none dropped)",
                "l2": "KV arena ~0.7 GB > 126 MB L2"}

    def __init__(self, args, rank, world, dev):
        import torch
        self.args, self.world = args, world
        self.torch = torch
        self.pkg = pkg = ge.load_package()
        self.rank, self.dev = rank, dev
        prompt, max_new, arrival = self.inputs()
        self.prompt, self.arrival_ns = prompt, arrival
        self.n = self.N_ROLLOUTS
        self.ng = self.n // self.G
        self.GROUPS = self.ng
        base_pages = self.BASE // 16
        grp_pages = [(int(p) + 15) // 16 for p in prompt]
        priv = 256 * ((self.GEN + 16 + 15) // 16)
        self.arena = pkg.DeviceArena(base_pages + sum(grp_pages) + priv + 64, device=dev)
        cfg = dict(num_q_heads=32, num_kv_heads=8, vocab=self.VOCAB, max_slots=256,
                   max_context=self.BASE + 1024 + self.GEN, max_new_tokens=self.GEN,
                   max_admit=256, drop_when_full=0, decode_mode=1, reward_mode=1, reward_seed=5,
                   logit_std=2.0, max_prefixes=self.ng,
                   max_prefix_pages=self.ng * (base_pages + 64), max_passes=1 << 26,
                   idle_timeout_ms=20000, chunk_pages=args.chunk_pages)
        self.eng = pkg.RolloutEngine(cfg, self.arena)
        base = self.arena.acquire(base_pages)
        self.arena.fill_pages(base, seed=4 + rank, stream_id=0)      # synthetic prefill (untimed)
        for g in range(self.ng):
            own = self.arena.acquire(grp_pages[g])
            self.arena.fill_pages(own, seed=4 + rank, stream_id=1000000 * (g + 1))
            self.eng.set_prefix(g, list(base) + list(own), self.BASE + int(prompt[g]))
        r = np.zeros(self.n, dtype=np.dtype(pkg.REQUEST_RECORD))
        gid = np.arange(self.n) // self.G
        r["request_id"] = np.arange(1, self.n + 1, dtype=np.uint64) | \
            ((gid.astype(np.uint64) + np.uint64(1)) << np.uint64(32))
        r["max_tokens"] = max_new
        r["kv_blocks"] = (self.BASE + prompt[gid] + 15) // 16
        r["temperature"], r["top_k"], r["top_p"], r["rng_seed"] = 0.8, 50, 0.9, 1234
        self._make_buffers(torch, dev, r)
        self.arrivals = torch.from_numpy(arrival.astype(np.int64)).to(dev)
        self.tokens_per_step = int(max_new.sum())
        torch.cuda.synchronize()

    def e2e(self, steps, warmup):
        """Ring-fed and paced: requests enter the mapped RequestRing at their
        arrival times (rt_host_pump_paced), dones are drained from the mapped
        DoneRing, then the trajectories and advantages are copied to pinned
        host memory; all inside the timed region."""
        torch = self.torch
        rings = self.pkg.HostRings()
        traj_h = torch.empty(self.traj.shape, dtype=torch.int32).pin_memory()
        adv_h = torch.empty(self.adv.shape, dtype=torch.float32).pin_memory()
        s = torch.cuda.current_stream()
        lat = []

        def one():
            self.eng.launch(ring=rings.req, done_ring=rings.done, state=self.state,
                            trajectories=self.traj, rewards=self.rewards, n_rows=self.n)
            got, raw, done_ns = rings.pump_paced(self.reqs_host, self.arrival_ns, self.n,
                                                 send_sentinel=True, timeout_ms=120000)
            if got != self.n:
                raise RuntimeError(f"e2e pump drained {got} of {self.n}")
            d = raw[: self.n * 24].view(np.dtype([("request_id", "<u8"), ("rollout_id", "<u4"),
                                                    ("tokens_generated", "<u4"), ("reward", "<f4"),
                                                    ("status", "<u4")]))
            idx = d["request_id"].astype(np.int64) - 1
            lat.append(done_ns[:self.n].astype(np.float64) - self.arrival_ns[idx].astype(np.float64))
            self._post()
            traj_h.copy_(self.traj, non_blocking=True)
            adv_h.copy_(self.adv, non_blocking=True)

        for _ in range(min(warmup, 1)):
            one()
        torch.cuda.synchronize()
        lat.clear()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(steps):
            one()
        e1.record(s)
        torch.cuda.synchronize()
        self.eng.wait()
        rings.close()
        ms = e0.elapsed_time(e1) / steps
        return {"value": self.units_per_step() / (ms / 1e3), "unit": self.unit, "ms_per_step": ms,
                "h2d_bytes_per_step": self.n * 34,
                "d2h_bytes_per_step": self.n * 24 + traj_h.numel() * 4 + adv_h.numel() * 4,
                "latency_arrival_to_done_ms": self._pct(np.concatenate(lat), 1e6)}

    def kernel_profile(self, n_rollouts=None):
        """Host-stepped replay of all 1,024 rollouts with the arrivals given
        in passes (arrival time / the timed run's mean pass interval), so the
        replay admits in the same rhythm as the timed loop."""
        st = getattr(self, "last_stats", None)
        pass_ns = (self.last_ms * 1e6 / st["passes"]) if st and st["passes"] else 100e3
        arr = self.torch.from_numpy((self.arrival_ns / pass_ns).astype(np.int64)).to(self.dev)
        return self.eng.profile(requests=self.req_d, n_requests=self.n, dones=self.dones,
                                state=self.state, trajectories=self.traj, rewards=self.rewards,
                                n_rows=self.n, arrivals=arr,
                                arrival_unit=self.pkg.RT_ARRIVAL_PASS)

    @classmethod
    def cpu_port(cls, args, threads, budget_s):
        prompt, _, _ = cls.inputs()
        ctx = cls.BASE + int(prompt[0])
        tokens, steps, dt = _port_rollout_decode(threads, budget_s, cls.G, ctx, cls.GEN,
                                                 cls.VOCAB, seed=12)
        return _port_result(tokens / dt, cls.unit, threads, dt,
                            f"group 0 (16 rollouts, {ctx}-token shared context), {steps} decode "
                            f"steps (attention + logits + reference sampling per token)")

    def details(self):
        return {"arena_gb": round(self.arena.buf.numel() / 1e9, 3)}


def _decode_ring_inputs(rank, N=10000, BLOCKS=128, SLOTS=4096, BLOCK=16384):
    orc = ge.load_oracle()
    rng = np.random.default_rng(7 + rank)
    arena_host = rng.standard_normal(BLOCKS * BLOCK // 2).astype(np.float16).view(np.uint8)
    q_bits = rng.standard_normal((SLOTS, 128)).astype(np.float16).view(np.uint16)
    d = np.zeros(N, orc.DESCRIPTOR_DTYPE)
    i = np.arange(N, dtype=np.uint64)
    d["seq_id"] = 1 + rank
    d["kv_block_offset"] = i % BLOCKS
    d["num_kv_blocks"] = 1
    d["output_token_offset"] = i
    d["reward_cookie"] = (np.uint64(1 + rank) << np.uint64(32)) | i
    return d, arena_host, q_bits


class DecodeRingWorkload(Workload):
    """The reference's per-step CommandRing benchmark (src/main.c:201-260):
    10,000 decode descriptors of one trajectory, kv_block_offset = i % 128
    over 16 KiB fp16 blocks, num_kv_blocks 1, output slot i & 4095 of a
    4,096-slot q / o buffer.  The q buffer is filled once with N(0,1) fp16
    (the reference's synthetic model_state / query_producer kernels are not
    part of the path).

    value: one step = the fixed128 step over the 10,000 descriptors resident
    in HBM, one rt_attention_fixed128 launch; 64 copies of the blocks, q and
    o buffers, descriptors and results (371 MB > 126 MB L2) rotate between
    steps.
    e2e: one step = launch the persistent decode worker, push the 10,000
    descriptors and a stop sentinel through the mapped CommandRing, drain
    the 10,000 Completions from the mapped CompletionRing
    (rt_host_decode_pump), join the worker."""

    name = "command_ring_decode_main_c"
    kernel = "fixed128_batch_kernel"
    metric = "decode steps/s (fixed128 step, reference src/main.c shape)"
    unit = "steps/s"
    dtype = "fp16 KV, fp32 math"
    roofline_note = ("latency-bound: 10,000 warps each stage 512 B of KV with one bulk copy "
                     "and run a one-token step; the HBM bytes are incidental")
    N, BLOCKS, SLOTS, BLOCK, COPIES = 10000, 128, 4096, 16384, 64

    @classmethod
    def static_config(cls, args, world):
        return {"workload": cls.name, "descriptors": cls.N, "kv_blocks": cls.BLOCKS,
                "block_bytes": cls.BLOCK, "num_kv_blocks": 1, "io_slots": cls.SLOTS,
                "value_step": "rt_attention_fixed128 over HBM-resident descriptors",
                "e2e_step": "decode worker launch + ring dispatch + poll + stop sentinel + join",
                "rings": "CommandRing / CompletionRing, 4,096 slots, pinned mapped host memory",
                "l2": "64 rotating copies of blocks, q, o, descriptors and results (> 126 MB L2)"}

    def __init__(self, args, rank, world, dev):
        import ctypes
        import torch
        self.args, self.world = args, world
        self.torch, self.ctypes = torch, ctypes
        self.pkg = pkg = ge.load_package()
        d, self.arena_host, self.q_bits = _decode_ring_inputs(rank)
        self.descs = d
        C = self.COPIES
        self.arena_t = torch.from_numpy(self.arena_host.copy()).to(dev).repeat(C).view(C, -1)
        self.arenas = [pkg.device_arena(self.arena_t[c], self.BLOCK) for c in range(C)]
        q1 = torch.from_numpy(self.q_bits.view(np.int16)).to(dev).view(torch.float16)
        self.q = q1.repeat(C, 1).view(C, self.SLOTS, 128)
        self.o = torch.zeros(C, self.SLOTS, 128, dtype=torch.float32, device=dev)
        self.desc_d = torch.from_numpy(d.view(np.uint8).copy()).to(dev).repeat(C).view(C, -1)
        self.res = torch.zeros(C, self.N * 24, dtype=torch.uint8, device=dev)
        self.step_count = torch.zeros(1, dtype=torch.int64, device=dev)
        self.rings = pkg.CommandRings()
        # HBM bytes per descriptor: the descriptor, the K and V rows read
        # (seq_len 1), q, o, the 24-byte result
        self.bytes = self.N * (32 + 2 * 256 + 256 + 512 + 24)
        self.i = 0
        self.last = None
        torch.cuda.synchronize()

    def step(self):
        c = self.i % self.COPIES
        self.i += 1
        rc = self.pkg.lib().rt_attention_fixed128(
            self.ctypes.c_void_p(self.desc_d[c].data_ptr()), self.N,
            self.ctypes.byref(self.arenas[c]), None, self.ctypes.c_void_p(self.q[c].data_ptr()),
            self.ctypes.c_void_p(self.o[c].data_ptr()), self.SLOTS,
            self.ctypes.c_void_p(self.res[c].data_ptr()),
            self.ctypes.c_void_p(self.torch.cuda.current_stream().cuda_stream))
        self.pkg.check(rc, "rt_attention_fixed128")

    def _ring_once(self):
        self.pkg.launch_decode_worker(self.rings, self.arenas[0], q_buffer=self.q[0],
                                      o_buffer=self.o[0], io_slots=self.SLOTS,
                                      step_count=self.step_count, stop_sentinels=1,
                                      idle_timeout_ms=20000)
        got, raw = self.rings.pump(self.descs, 1, self.N, timeout_ms=60000)
        if got != self.N:
            raise RuntimeError(f"decode ring drained {got} of {self.N}")
        self.torch.cuda.current_stream().synchronize()  # the worker exits at the sentinel
        self.last = raw

    def units_per_step(self):
        return float(self.N)

    def check_errors(self):
        """Batch results (and, after e2e, the ring's Completions) against the
        CPU restatement: records equal except token ids, which must be
        near-ties of the oracle where they differ."""
        orc = ge.load_oracle()
        want, o_orc, _ = orc.decode_steps(self.descs, self.arena_host, self.BLOCK,
                                          q_buf=self.q_bits, io_slots=self.SLOTS)
        dt = np.dtype([("path_kind", "<u4"), ("token_id", "<u4"), ("bytes_touched", "<u4"),
                       ("tile_count", "<u4"), ("cycle_estimate", "<u8")])
        res = self.res[0].cpu().numpy().view(dt)
        ok = np.array_equal(res["cycle_estimate"], want["cycles_taken"])
        ok &= self._tokens_ok(res["token_id"], want["token_id"], o_orc)
        self._want = (want, o_orc)
        return 0 if ok else -100

    def _check_ring(self):
        orc = ge.load_oracle()
        want, o_orc = self._want if getattr(self, "_want", None) else orc.decode_steps(
            self.descs, self.arena_host, self.BLOCK, q_buf=self.q_bits, io_slots=self.SLOTS)[:2]
        comps = self.last.view(orc.COMPLETION_DTYPE)[:self.N]
        ok = all(np.array_equal(comps[f], want[f]) for f in
                 ("seq_id", "kv_block_offset", "reward_cookie", "cycles_taken"))
        ok &= self._tokens_ok(comps["token_id"], want["token_id"], o_orc)
        st = self.pkg.decode_worker_stats()
        if not ok or st["error"] != 0:
            raise RuntimeError(f"decode ring completions differ from the oracle (stats {st})")

    @staticmethod
    def _tokens_ok(tok, want, o_orc):
        bad = np.nonzero(tok != want)[0]
        return all(o_orc[i][tok[i]] >= o_orc[i].max() - 2e-4 for i in bad)

    def e2e(self, steps, warmup):
        """Through the decode worker and the mapped rings (host buffers by
        construction: descriptors read from pinned host memory, Completions
        written back to it, inside every step)."""
        torch = self.torch
        s = torch.cuda.current_stream()
        for _ in range(min(warmup, 3)):
            self._ring_once()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(steps):
            self._ring_once()
        e1.record(s)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        self._check_ring()
        return {"value": self.N / (ms / 1e3), "unit": self.unit, "ms_per_step": ms,
                "h2d_bytes_per_step": (self.N + 1) * 32, "d2h_bytes_per_step": self.N * 32}

    @classmethod
    def cpu_port(cls, args, threads, budget_s):
        """The reference step on the host (oracle/oracle.c orc_decode_steps:
        process_descriptor + the fixed128 attention of test/test_bench.cu:
        109-155) over the same descriptors, split into contiguous chunks run
        on a thread pool, whole batches until the budget is spent."""
        from concurrent.futures import ThreadPoolExecutor
        orc = ge.load_oracle()
        d, arena, q = _cached("ring", lambda: _decode_ring_inputs(0))
        chunks = np.array_split(np.arange(cls.N), threads)
        pool = ThreadPoolExecutor(max_workers=threads)
        t0 = time.perf_counter()
        reps = 0
        while reps == 0 or time.perf_counter() - t0 < budget_s:
            list(pool.map(lambda c: orc.decode_steps(d[c], arena, cls.BLOCK, q_buf=q,
                                                     io_slots=cls.SLOTS), chunks))
            reps += 1
        dt = time.perf_counter() - t0
        pool.shutdown()
        return _port_result(reps * cls.N / dt, cls.unit, threads, dt,
                            f"{reps} batch(es) of the 10,000 descriptors, C restatement on "
                            f"{threads} threads")


class LmHeadWorkload(Workload):
    """The decode step's LM head as a tensor-core GEMM (rt_gemm_bf16,
    tcgen05): logits fp32 [256 slots][32,000] = hidden bf16 [256][4096] x
    W bf16 [32,000][4096]^T.  The 262 MB weight exceeds the 126 MB L2, so
    every step streams it from HBM.  The same product through cuBLAS
    (torch.matmul, bf16 output) is timed beside it for context."""

    name = "lm_head_gemm_256x4096x32000"
    kernel = "gemm_bf16_tn_kernel"
    metric = "LM-head GEMM TFLOP/s (256 x 4096 -> 32,000, bf16 in, fp32 out)"
    unit = "TFLOP/s"
    dtype = "bf16 in, fp32 accumulate and out"
    bound = "tensor"
    M, N, K = 256, 32000, 4096

    @classmethod
    def static_config(cls, args, world):
        return {"workload": cls.name, "M": cls.M, "N": cls.N, "K": cls.K,
                "tile": "256 x 224 unit, 3-stage TMA ring, double-buffered TMEM accumulator",
                "l2": "W 262 MB > 126 MB L2 (streamed from HBM every step)"}

    def __init__(self, args, rank, world, dev):
        import ctypes
        import torch
        self.args, self.world = args, world
        self.torch, self.ctypes = torch, ctypes
        self.pkg = pkg = ge.load_package()
        self.A = torch.empty(self.M, self.K, dtype=torch.bfloat16, device=dev)
        self.W = torch.empty(self.N, self.K, dtype=torch.bfloat16, device=dev)
        pkg.fill_normal_bf16(self.A, seed=21 + rank, stream_id=1)
        pkg.fill_normal_bf16(self.W, seed=21 + rank, stream_id=2, std=0.02)
        self.C = torch.empty(self.M, self.N, dtype=torch.float32, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        self.p = pkg.rt_gemm_params_t(self.M, self.N, self.K, self.K, self.K, self.N, 0, 0)
        self.flops = 2.0 * self.M * self.N * self.K
        # HBM bytes per launch: W and A read once, C written once
        self.bytes = self.N * self.K * 2 + self.M * self.K * 2 + self.M * self.N * 4
        torch.cuda.synchronize()

    def step(self):
        c = self.ctypes
        rc = self.pkg.lib().rt_gemm_bf16(c.byref(self.p), c.c_void_p(self.A.data_ptr()),
                                         c.c_void_p(self.W.data_ptr()), c.c_void_p(self.C.data_ptr()),
                                         None, 0, c.c_void_p(self.err.data_ptr()),
                                         c.c_void_p(self.torch.cuda.current_stream().cuda_stream))
        self.pkg.check(rc, "rt_gemm_bf16")

    def units_per_step(self):
        return self.flops / 1e12

    def check_errors(self):
        """Kernel error word, and 64 sampled outputs against a float64 dot."""
        torch = self.torch
        rng = np.random.default_rng(5)
        ms, ns = rng.integers(0, self.M, 64), rng.integers(0, self.N, 64)
        ref = (self.A[ms].double() * self.W[ns].double()).sum(1)
        bound = (self.A[ms].double().abs() * self.W[ns].double().abs()).sum(1) * 2.0 ** -16 + 1e-6
        got = self.C[torch.as_tensor(ms, device=self.C.device),
                     torch.as_tensor(ns, device=self.C.device)].double()
        ok = bool(((got - ref).abs() <= bound).all())
        return int(self.err.item()) or (0 if ok else -100)

    def cublas_ms(self, reps=20):
        torch = self.torch
        out = torch.empty(self.M, self.N, dtype=torch.bfloat16, device=self.A.device)
        for _ in range(3):
            torch.matmul(self.A, self.W.t(), out=out)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            torch.matmul(self.A, self.W.t(), out=out)
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    def e2e(self, steps, warmup):
        """Hidden rows copied from pinned host memory each step, logits read
        back to pinned host memory."""
        torch = self.torch
        a_h = self.A.cpu().pin_memory()
        c_h = torch.empty(self.C.shape, dtype=torch.float32).pin_memory()
        s = torch.cuda.current_stream()

        def one():
            self.A.copy_(a_h, non_blocking=True)
            self.step()
            c_h.copy_(self.C, non_blocking=True)

        for _ in range(warmup):
            one()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(steps):
            one()
        e1.record(s)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        return {"value": self.units_per_step() / (ms / 1e3), "unit": self.unit, "ms_per_step": ms,
                "h2d_bytes_per_step": self.M * self.K * 2, "d2h_bytes_per_step": self.M * self.N * 4}

    @classmethod
    def cpu_port(cls, args, threads, budget_s):
        """The same product on the host (numpy float32 matmul, multithreaded
        BLAS) over row blocks of a numpy hidden state and weight, until the
        budget is spent; the reference has no LM head."""
        def make():
            rng = np.random.default_rng(21)
            return (rng.standard_normal((cls.M, cls.K), dtype=np.float32),
                    rng.standard_normal((cls.N, cls.K), dtype=np.float32) * np.float32(0.02))
        a, w = _cached("lm", make)
        t0 = time.perf_counter()
        rows = 0
        while rows < cls.M and (rows == 0 or time.perf_counter() - t0 < budget_s):
            _ = a[rows:rows + 16] @ w.T
            rows += 16
        dt = time.perf_counter() - t0
        return _port_result(2.0 * rows * cls.N * cls.K / dt / 1e12, cls.unit, threads, dt,
                            f"{rows} of 256 rows, numpy float32 matmul")

    def details(self):
        return {"cublas_bf16_out_ms": round(self.cublas_ms(), 4)}


class RolloutModelWorkload(RolloutWorkload):
    """Config 5 with a model behind the decode step (RT_ROLLOUT_DECODE_MODEL)
    instead of Philox q / K / V and logits: per pass the slots' last-token
    embeddings (table 32,000 x 4,096 bf16), the QKV projection (4,096 ->
    6,144) and the LM head (4,096 -> 32,000) run as tensor-core GEMMs
    (rt_gemm_bf16) around the same paged attention and sampler; the
    prompts' K / V come from the same model (rt_rollout_prefill).  Weights
    are seeded N(0, s) bf16 (no checkpoint exists offline): embedding s = 1,
    QKV 1/64, LM head 0.05."""

    name = "grpo_rollouts_c5_model"
    metric = "rollout tokens/s (config 5, model decode: QKV + LM-head GEMMs)"
    DECODE_MODE = 2
    launches_per_pass = 8  # schedule, embed, QKV GEMM, prepare, attention, hidden, LM GEMM, sampler

    @classmethod
    def static_config(cls, args, world):
        return super().static_config(args, world) | {
            "workload": cls.name,
            "model": "embedding 32,000 x 4,096, QKV 4,096 -> 6,144, LM head 4,096 -> 32,000; "
                     "bf16 weights N(0, s), fp32 accumulation",
            "prompts": "seeded token ids, K / V prefilled by the model (rt_rollout_prefill, "
                       "untimed setup)"}

    def _attach_model(self, torch, dev, rank):
        D, NQKV = 32 * 128, (32 + 2 * 8) * 128
        self.emb = torch.empty(self.VOCAB, D, dtype=torch.bfloat16, device=dev)
        self.wqkv = torch.empty(NQKV, D, dtype=torch.bfloat16, device=dev)
        self.wlm = torch.empty(self.VOCAB, D, dtype=torch.bfloat16, device=dev)
        self.pkg.fill_normal_bf16(self.emb, seed=31 + rank, stream_id=1)
        self.pkg.fill_normal_bf16(self.wqkv, seed=31 + rank, stream_id=2, std=1.0 / 64)
        self.pkg.fill_normal_bf16(self.wlm, seed=31 + rank, stream_id=3, std=0.05)
        self.eng.set_model(self.emb, self.wqkv, self.wlm)
        self.gemm_flops_per_token = 2.0 * D * (NQKV + self.VOCAB)
        # the prompts' K / V from the model (seeded token ids), untimed setup,
        # its rate measured once with CUDA events
        g = torch.Generator(device=dev).manual_seed(41 + rank)
        toks = torch.randint(0, self.VOCAB, (self.ng, self.PROMPT), generator=g, device=dev,
                             dtype=torch.int32)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for gi in range(self.ng):
            self.eng.prefill(gi, toks[gi])
        e1.record()
        torch.cuda.synchronize()
        self.prefill_tokens_per_s = self.ng * self.PROMPT / (e0.elapsed_time(e1) / 1e3)

    def trajectory_check(self, sample_rows=64):
        """Model decode feeds sampled tokens back, so there is no closed-form
        replay; the check is that one more step reproduces the timed
        trajectories bit for bit."""
        torch = self.torch
        lengths = torch.from_numpy(self.reqs_host["max_tokens"].astype(np.int64)).to(self.traj.device)
        before = _traj_checksum(torch, self.traj, lengths)
        self.traj.fill_(-1)
        self.step()
        self.eng.wait()
        after = _traj_checksum(torch, self.traj, lengths)
        return {"result": "equal" if before == after else "DIFFERENT",
                "checksum_timed": before, "checksum_check_step": after}

    @classmethod
    def cpu_port(cls, args, threads, budget_s):
        """The model decode step on the host for one GRPO group (16
        rollouts, shared 512-token prompt): embedding rows, QKV and LM-head
        projections (numpy float32 matmul, multithreaded BLAS), paged GQA
        attention (oracle/oracle.c, OpenMP), the reference sampling
        algorithm per row, until the budget is spent."""
        from concurrent.futures import ThreadPoolExecutor
        orc = ge.load_oracle()
        B, Hq, Hkv, D = cls.G, 32, 8, 32 * 128
        n_pages = (cls.PROMPT + cls.GEN + 15) // 16
        rng = np.random.default_rng(11)

        def make():
            arena_b = _bf16_normal(rng, B * n_pages * Hkv * 2 * 16 * 128)
            pt = rng.permutation(B * n_pages).astype(np.int32).reshape(B, n_pages)
            pt[:, :cls.PROMPT // 16] = pt[0, :cls.PROMPT // 16]
            emb = rng.standard_normal((cls.VOCAB, D), dtype=np.float32)
            wqkv = rng.standard_normal(((Hq + 2 * Hkv) * 128, D), dtype=np.float32) / np.float32(64)
            wlm = rng.standard_normal((cls.VOCAB, D), dtype=np.float32) * np.float32(0.05)
            return arena_b, pt, emb, wqkv, wlm
        arena_b, pt, emb, wqkv, wlm = _cached("model", make)
        pool = ThreadPoolExecutor(max_workers=threads)
        tok = np.zeros(B, dtype=np.int64)
        t0 = time.perf_counter()
        steps = 0
        while steps == 0 or (time.perf_counter() - t0 < budget_s and steps < cls.GEN):
            x = emb[tok]
            qkv = x @ wqkv.T
            q = (qkv[:, :D].astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
            lens = np.full(B, cls.PROMPT + steps + 1, dtype=np.int32)
            o = orc.paged_gqa_attention(q.reshape(B, Hq, 128), arena_b, pt, lens, Hq, Hkv,
                                        128 ** -0.5, n_threads=threads)
            logits = (o.reshape(B, D) @ wlm.T).astype(np.float32)
            tok = np.array(list(pool.map(lambda b: orc.sample_row(
                logits[b], 0.8, 50, 0.9, orc.sample_u24(1234, b, steps)), range(B))))
            steps += 1
        dt = time.perf_counter() - t0
        pool.shutdown()
        return _port_result(B * steps / dt, cls.unit, threads, dt,
                            f"1 group x 16 rollouts, {steps} model decode steps from a 512-token "
                            f"prompt (embedding, QKV and LM-head matmuls, attention, sampling)")

    def details(self):
        return super().details() | {"prefill_tokens_per_s": round(self.prefill_tokens_per_s),
                                    "gemm_flops_per_token": self.gemm_flops_per_token}


WORKLOADS = {"lm_head": LmHeadWorkload, "rollout": RolloutWorkload,
             "rollout_c4": RolloutC4Workload, "rollout_model": RolloutModelWorkload,
             "attention": AttentionWorkload, "sampling": SamplingWorkload,
             "decode_ring": DecodeRingWorkload}


def config1_cpu_path(reps=5):
    """BASELINE config 1, the reference's CPU path:
    - 10,000 hw_desc_t decode descriptors (seed 0, max_tokens 2048) through
      hw_ring + hw_worker_sim, producer and worker on two host threads,
      command depth capped at 1,024;
    - host batching: the reference benchmark's 10,000 step descriptors
      (src/main.c shape) submitted by decode_batch_submit in windows of 32
      into a CommandRing and consumed by a second thread.
    The reference's own C sources (compiled unmodified into oracle/_ref) are
    timed beside this repo's C implementation of the same API, and the
    output streams (64-byte completions; CommandRing records with their
    batch stamps) are compared byte for byte."""
    orc = ge.load_oracle()
    try:
        ref = orc.Harness("ref")
    except OSError as e:
        return {"unavailable": f"reference build absent: {e}"}
    mine = orc.Harness("mine")
    descs = mine.gen_c1(10000, seed=0, max_tokens=2048)
    # the two implementations alternate, so that drift of the host's clocks
    # during the measurement falls on both alike; medians over the runs
    r, m = [], []
    for _ in range(reps):
        r.append(ref.run_c1(descs, depth_cap=1024))
        m.append(mine.run_c1(descs, depth_cap=1024))
    rs, ms = statistics.median(x[3] for x in r), statistics.median(x[3] for x in m)
    d, _, _ = _decode_ring_inputs(0)
    rb, mb = [], []
    for _ in range(8 * reps):
        rb.append(ref.run_decode_batch(d, 32))
        mb.append(mine.run_decode_batch(d, 32))
    rbs, mbs = statistics.median(x[1] for x in rb), statistics.median(x[1] for x in mb)
    return {"workload": "BASELINE config 1: 10,000 hw_desc_t, seed 0, depth 1,024",
            "kind": "reference", "cores": 2,
            "reference_descs_per_s": len(descs) / rs, "reference_tokens_per_s": r[0][1] / rs,
            "mine_descs_per_s": len(descs) / ms, "mine_tokens_per_s": m[0][1] / ms,
            "completion_stream_equal": bool(np.array_equal(r[0][0].view(np.uint8),
                                                           m[0][0].view(np.uint8))),
            "reps": reps, "order": "alternating",
            "decode_batch": {
                "workload": "10,000 src/main.c step descriptors, decode_batch_submit windows of 32, "
                            "CommandRing 4,096 slots, consumer thread",
                "reference_descs_per_s": len(d) / rbs, "mine_descs_per_s": len(d) / mbs,
                "command_ring_stream_equal": bool(rb[0][0].tobytes() == mb[0][0].tobytes()),
                "reps": 8 * reps, "order": "alternating"}}


def roofline_block(wl, achieved_gbs, ms, peaks, src, traffic, traffic_commit=None):
    """The dominant kernel against its bound: HBM GB/s, or for a tensor-core
    workload bf16 TFLOP/s against the burst GEMM peak (the kernel is timed
    alone), with its HBM fraction beside it."""
    tsrc = (f"profiles/ncu_traffic.txt (one ncu capture at commit {traffic_commit})"
            if traffic is not None else None)
    if getattr(wl, "bound", "hbm") == "tensor":
        tf = wl.flops / (ms / 1e3) / 1e12
        peak = peaks.get("bf16_tflops", 1590.0)
        return {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s",
                "frac": tf / peak,
                "peak_source": f"{src} cuBLAS bf16 burst (MEASURED_PEAKS.json bf16_tflops)"
                if src == "measured" else "fallback 1.59 PFLOP/s",
                "frac_of_nominal_2250": tf / 2250.0,
                "hbm_achieved_gbs": achieved_gbs, "hbm_frac": achieved_gbs / peaks["hbm_gbs"],
                "traffic": traffic, "traffic_source": tsrc, "kernel": wl.kernel}
    return ({"bound": "hbm", "achieved": achieved_gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
             "frac": achieved_gbs / peaks["hbm_gbs"],
             "peak_source": f"{src} copy bandwidth (MEASURED_PEAKS.json hbm_gbs)"
             if src == "measured" else "fallback 6.65 TB/s",
             "frac_of_nominal_8tbs": achieved_gbs / 8000.0, "traffic": traffic,
             "traffic_source": tsrc, "kernel": wl.kernel}
            | ({"note": wl.roofline_note} if hasattr(wl, "roofline_note") else {}))


def loop_kernel_report(prof):
    """Per-kernel averages of a host-stepped replay; attention GB/s over the
    deduplicated KV bytes (each shared prefix once per pass)."""
    attn_s = prof["ms_attention"] / 1e3
    keys = ("ms_schedule", "ms_prepare", "ms_attention", "ms_logits", "ms_sample")
    tot = sum(prof[k] for k in keys)
    return prof["attn_bytes_unique"] / attn_s / 1e9, {
        "source": "rt_rollout_profile host-stepped replay, CUDA events per kernel",
        "passes": prof["passes"],
        "avg_us": {k[3:]: 1e3 * prof[k] / max(prof["passes"], 1) for k in keys},
        "share": {k[3:]: prof[k] / tot for k in keys},
        "attn_logical_GBps": prof["attn_bytes_logical"] / attn_s / 1e9,
        "attn_unique_bytes_per_launch": prof["attn_bytes_unique"] / max(prof["attn_launches"], 1),
    }


def timed_steps(torch, wl, steps, warmup, dev_index):
    """W untimed steps, then K steps between CUDA events on the launching
    stream with a synchronize on both sides; clocks sampled meanwhile."""
    for _ in range(warmup):
        wl.step()
    torch.cuda.synchronize()
    clocks = ClockSampler(dev_index)
    clocks.start()
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(s)
    for _ in range(steps):
        wl.step()
    e1.record(s)
    torch.cuda.synchronize()
    clocks.stop()
    return e0.elapsed_time(e1) / steps, clocks.report()


def extra_block(cls, args, dev, steps, warmup, peaks, src):
    """One more BASELINE config measured in the same run (N = 1): device
    value with its roofline, e2e through host buffers, clocks, error word,
    and for config 4 the latency and trajectory checks."""
    import torch
    wl = cls(args, 0, 1, dev)
    ms, clocks = timed_steps(torch, wl, steps, warmup, 0)
    wl.last_ms = ms
    err = wl.check_errors()
    out = {"config": wl.config(), "metric": wl.metric, "unit": wl.unit,
           "value": wl.units_per_step() / (ms / 1e3), "ms_per_step": ms, "steps": steps,
           "warmup": warmup, "device_error_code": err, "clocks": clocks}
    traffic, commit = ncu_traffic(wl.kernel, wl.name)
    if isinstance(wl, RolloutWorkload):
        achieved, rep = loop_kernel_report(wl.kernel_profile())
        if isinstance(wl, RolloutModelWorkload):
            rep["note"] = ("model decode: 'prepare' = embedding gather + QKV GEMM + q/K/V "
                           "scatter, 'logits' = bf16 hidden + LM-head GEMM")
        out["kernels"] = rep
        out["gpu_launches"] = wl.gpu_launches(steps)
        out["roofline"] = roofline_block(wl, achieved, rep["avg_us"]["attention"] / 1e3, peaks, src,
                                         traffic, commit)
        out["trajectory_check"] = wl.trajectory_check()
        out["device_trace"] = wl.trace_report()
    else:
        out["roofline"] = roofline_block(wl, wl.bytes / (ms / 1e3) / 1e9, ms, peaks, src,
                                         traffic, commit)
        out["gpu_launches"] = wl.gpu_launches(steps)
    e2e = wl.e2e(max(3, min(steps, 20)), min(warmup, 3))
    out["e2e"] = {k: v for k, v in e2e.items() if k != "ms_per_step"}
    out["details"] = wl.details()
    del wl
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return out


# -------------------------------------------------------------------- main
def run_mine(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    cls = WORKLOADS[args.workload]
    wl = cls(args, rank, world, dev)
    for _ in range(args.warmup):
        wl.step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(s)
    for _ in range(args.steps):
        wl.step()
    e1.record(s)
    torch.cuda.synchronize()
    clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    wl.last_ms = ms
    # every rank's share is the same size (groups split evenly), so the
    # whole-job rate is the per-rank units over the slowest rank's time x N
    value = wl.units_per_step() / (ms / 1e3) * world
    err = wl.check_errors()
    n_launch = wl.gpu_launches(args.steps)
    traj = wl.trajectory_check() if hasattr(wl, "trajectory_check") else None
    diag = None
    if world > 1 and hasattr(wl, "rank_diagnostics"):
        mine_d = wl.rank_diagnostics()
        diag = [None] * world
        dist.all_gather_object(diag, mine_d)
    prof = wl.kernel_profile() if hasattr(wl, "kernel_profile") else None
    e2e = None if args.no_e2e else wl.e2e(args.steps, args.warmup)
    if world > 1 and e2e is not None:
        t = torch.tensor([e2e["ms_per_step"]], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e["value"] = wl.units_per_step() / (float(t.item()) / 1e3) * world
        e2e["ms_per_step"] = float(t.item())
    cpu = c1 = trace = None
    peaks, src = measured_peaks()
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cls.cpu_port(args, os.cpu_count() or 1, 10.0)
        cpu.pop("seconds", None)
        c1 = config1_cpu_path()
        if hasattr(wl, "trace_report"):
            trace = wl.trace_report()
    details = wl.details()
    if prof is not None:
        # dominant kernel of the loop: paged attention, per-launch average
        # from the host-stepped replay's CUDA events
        achieved, prof_report = loop_kernel_report(prof)
        roof_ms = prof_report["avg_us"]["attention"] / 1e3
    else:
        achieved = wl.bytes / (ms / 1e3) / 1e9
        prof_report, roof_ms = None, ms
    traffic, commit = ncu_traffic(cls.kernel, cls.name)
    roof = roofline_block(wl, achieved, roof_ms, peaks, src, traffic, commit)
    if world > 1 and getattr(wl, "nccl", None):
        wl.nccl.close()
    del wl
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    extra = {}
    if world == 1 and args.workload == "rollout" and not args.no_extra:
        extra["attention_c2"] = extra_block(AttentionWorkload, args, dev, 50, 10, peaks, src)
        extra["sampling_c3"] = extra_block(SamplingWorkload, args, dev, 50, 10, peaks, src)
        extra["continuous_batching_c4"] = extra_block(RolloutC4Workload, args, dev, 3, 3, peaks,
                                                      src)
        extra["model_decode_c5"] = extra_block(RolloutModelWorkload, args, dev, 2, 3, peaks, src)
    if rank == 0:
        line = {
            "metric": cls.metric, "value": value, "unit": cls.unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": cls.scaling, "vs_baseline": None,
            "dtype": cls.dtype, "data": "synthetic (Philox N(0,1), seeded)",
            "config": cls.line_config(args, world),
            "roofline": roof,
            "cpu_baseline": cpu,
            "cpu_path_config1": c1,
            "e2e": None if e2e is None else {k: e2e[k] for k in e2e if k != "ms_per_step"},
            "gpu_launches": n_launch,
            "trajectory_check": traj,
            "kernels": prof_report,
            "per_rank": diag,
            "device_trace": trace,
            "clocks": clocks.report(),
            "device_error_code": err,
            "details": details,
        } | extra
        print(json.dumps(line), flush=True)
    failed = bool(err) or (traj is not None and traj["result"] != "equal") or any(
        b.get("device_error_code") or (b.get("trajectory_check") or {}).get("result", "equal")
        != "equal" for b in extra.values())
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 3 if failed else 0


def run_reference(args):
    """The CPU implementation of the same workload on this host's cores,
    rank 0 only (other ranks exit without work): W warm-up samples, then K
    timed samples, each a bounded sample of the workload sized so the whole
    run stays within a few minutes; value = the median sample.  Inputs are
    numpy; this runtime is not loaded and the GPU is not touched."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    cls = WORKLOADS[args.workload]
    threads = os.cpu_count() or 1
    budget = max(0.5, min(10.0, 90.0 / (args.steps + args.warmup)))
    for _ in range(args.warmup):
        cls.cpu_port(args, threads, budget)
    samples = [cls.cpu_port(args, threads, budget) for _ in range(args.steps)]
    v = statistics.median(x["value"] for x in samples)
    cpu = samples[0] | {"value": v, "budget_s_per_step": budget}
    cpu.pop("seconds", None)
    print(json.dumps({
        "impl": "reference", "metric": cls.metric, "value": v, "unit": cls.unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "scaling": cls.scaling, "config": cls.line_config(args, world), "cpu_baseline": cpu,
        "e2e": {"value": v, "unit": cls.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--workload", default="rollout", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="mine", choices=["mine", "reference"])
    ap.add_argument("--chunk-pages", type=int, default=0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="rollout at N = 1: skip the config-2/3/4 blocks")
    ap.add_argument("--no-e2e", action="store_true",
                    help="skip the end-to-end leg (for ncu runs: the decode_ring e2e leg needs "
                         "its persistent worker to run beside the host pump)")
    ap.add_argument("--groups", type=int, default=0,
                    help="rollout only: GRPO groups (default 512; fewer keep ncu captures small)")
    ap.add_argument("--ncu-replay", type=int, default=0,
                    help="rollout workloads: run the host-stepped replay of this many rollouts "
                         "and exit (plain kernel launches, for ncu captures)")
    args = ap.parse_args()
    if args.ncu_replay:
        import torch
        torch.cuda.set_device(0)
        name = args.workload if args.workload.startswith("rollout") else "rollout"
        wl = WORKLOADS[name](args, 0, 1, torch.device("cuda", 0))
        prof = wl.kernel_profile(args.ncu_replay)
        print(json.dumps({"ncu_replay": args.ncu_replay, "profile": prof}), flush=True)
        return 0
    quick = not args.workload.startswith("rollout")   # rollout steps are whole RL steps
    if args.steps is None:
        args.steps = 200 if quick else 3
    if args.warmup is None:
        args.warmup = 10 if quick else 3
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_mine(args)


if __name__ == "__main__":
    sys.exit(main())
