#!/usr/bin/env python
"""Benchmark of the quantized projection hot path (BASELINE metric:
"Q4_K/Q8_0 GEMV HBM GB/s (% of peak); DFlash 16-token draft-block fwd/s").

With no --workload the run covers every BASELINE config and prints one JSON
line per config, the headline (config 1) last:
  gemv_q8_0     config 0: Q8_0 4096x4096 GEMV, one token
  ffn_q4k_m16   config 2: the DFlash FFN (gate/up 4096->14336, down 14336->4096) for 16 tokens
  dflash_block  config 3: the 6-layer DFlash decoder, one 16-token block over 2048 context rows
  lm_head_q8_0  config 4: lm_head Q8_0 4096->128256 for 1024 rows with the argmax
                (vocab-sharded over the ranks, MAX all-reduce of the keys)
  ffn_q4k_m1    config 1: the DFlash FFN for one token (the headline)
Each step goes through the C ABI (liblaguna_cuda.so); weights are raw GGUF
blocks rotated through a pool larger than 3x the 126 MB L2, so every step
streams its weights from HBM.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
  python bench.py --impl reference ...   # the reference's own shader code on host cores

Multi-GPU (torchrun, one rank per GPU): configs 0-3 run independent token
streams on every rank (replicas, no collective on the data path;
"scaling": "weak"); config 4 shards the vocab rows ("scaling": "strong").
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

MEASURED_PEAKS = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
L2_BYTES = 126 * 1024 * 1024

METRIC = "Q4_K/Q8_0 GEMV HBM GB/s (% of peak); DFlash 16-token draft-block fwd/s"


def _traffic(workload, kernel):
    """DRAM bytes (read + write) of one launch of the workload's dominant kernel,
    from the ncu capture summarised in profiles/ -- only when that capture was
    of the same kernel (None otherwise)."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            rec = json.load(f).get(workload)
    except Exception:
        return None
    if isinstance(rec, dict) and rec.get("kernel") == kernel:
        return rec.get("traffic")
    return None


_CPU_THREADS = [0]  # --cpu-threads; 0 = every host thread this process may use


def host_threads():
    if _CPU_THREADS[0] > 0:
        return _CPU_THREADS[0]
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def set_host_threads(n):
    """OpenMP threads of the CPU baselines: torchrun sets OMP_NUM_THREADS=1, so
    the count is set explicitly (env for libraries not loaded yet, and the
    runtime call for an OpenMP runtime already loaded)."""
    os.environ["OMP_NUM_THREADS"] = str(n)
    try:
        import ctypes

        ctypes.CDLL("libgomp.so.1").omp_set_num_threads(int(n))
    except Exception:
        pass


def peaks():
    try:
        with open(MEASURED_PEAKS) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


# ---------------------------------------------------------------------------
# Workloads: a list of projections (dtype, m, k, n) + the per-step op chain.

WORKLOADS = {
    # config 1: M=1 Q4_K GEMVs of the DFlash FFN (gate/up 4096->14336, down 14336->4096)
    "ffn_q4k_m1": dict(dtype="q4k", m=1, shapes=[("gate", 4096, 14336), ("up", 4096, 14336),
                                                  ("down", 14336, 4096)], ffn=True, config=1),
    # config 0: Q8_0 4096x4096 GEMV
    "gemv_q8_0": dict(dtype="q8_0", m=1, shapes=[("w", 4096, 4096)], ffn=False, config=0),
    # config 2: M=16 draft block through the same FFN projections (one lc_ffn call per step)
    "ffn_q4k_m16": dict(dtype="q4k", m=16, shapes=[("gate", 4096, 14336), ("up", 4096, 14336),
                                                    ("down", 14336, 4096)], ffn=True, config=2),
}


# Workloads with their own drivers (below): BASELINE config 4 (lm_head, vocab
# sharded over the ranks) and config 3 (the DFlash decoder, 16-token block).
SPECIAL = ("lm_head_q8_0", "dflash_block", "target_verify")
LM_HEAD = dict(m=1024, k=4096, vocab=128256, config=4)
DFLASH_HP = dict(n_layers=6, n_embd=4096, n_heads=32, n_kv_heads=8, head_dim=128, rope_dim=128, n_ff=14336, n_aux=5,
                 rope_base=500000.0, norm_eps=1e-5, qk_eps=1e-6)
DFLASH_CTX, DFLASH_BLOCK = 2048, 16


def weight_bytes(dtype, k, n):
    return n * (k // 256 * 144 if dtype == "q4k" else k // 32 * 34)


def step_bytes(wl):
    m = wl["m"]
    tot = 0
    for _, k, n in wl["shapes"]:
        tot += weight_bytes(wl["dtype"], k, n) + 4 * m * (k + n)
    return tot


def workload_config(name, wl):
    return {"workload": name, "baseline_config": wl["config"], "m": wl["m"],
            "projections": [f"{nm} {k}->{n}" for nm, k, n in wl["shapes"]], "bytes_per_step": step_bytes(wl)}


def launch_bytes(wl):
    """Algorithmic bytes of one projection launch (W + x + y); all shapes of a
    workload move the same bytes per launch."""
    _, k, n = wl["shapes"][0]
    return weight_bytes(wl["dtype"], k, n) + 4 * wl["m"] * (k + n)


# ---------------------------------------------------------------------------
class ClockSampler:
    """SM clock and throttle-reason sampling around the timed region.

    Polls NVML (read-only queries) every ~2 ms in a background thread so that
    even a short timed region is covered; samples taken between mark_begin()
    and mark_end() are the ones reported.  Falls back to nvidia-smi."""

    # NVML clocks-event-reason bits
    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown", 0x4: "sw_power_cap"}

    def __init__(self, dev):
        import threading

        self.samples = []  # (t, sm_mhz, reasons_bits)
        self.t_begin = self.t_end = None
        self.stop_flag = threading.Event()
        self.thread = None
        self.max_mhz = None
        self.handle = None
        try:
            import pynvml as nv

            nv.nvmlInit()
            self.nv = nv
            try:
                import torch

                uuid = str(torch.cuda.get_device_properties(dev).uuid)
                self.handle = nv.nvmlDeviceGetHandleByUUID(("GPU-" + uuid) if not uuid.startswith("GPU-") else uuid)
            except Exception:
                self.handle = nv.nvmlDeviceGetHandleByIndex(physical_gpu_index(dev.index or 0))
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(self.handle, nv.NVML_CLOCK_SM)
        except Exception:
            self.handle = None

    def _poll(self):
        nv = self.nv
        while not self.stop_flag.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                self.samples.append((time.perf_counter(), sm, rs))
            except Exception:
                pass
            time.sleep(0.002)

    def start(self):
        import threading

        if self.handle is None:
            return
        self.thread = threading.Thread(target=self._poll, daemon=True)
        self.thread.start()
        time.sleep(0.05)

    def mark_begin(self):
        self.t_begin = time.perf_counter()

    def sample_now(self):
        """One sample from the calling thread, taken after the timed work is
        enqueued and before the host waits for it, so that even a timed region
        shorter than the polling period holds a sample."""
        if self.handle is None:
            return
        nv = self.nv
        try:
            sm = nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)
            rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
            self.samples.append((time.perf_counter(), sm, rs))
        except Exception:
            pass

    def mark_end(self):
        self.t_end = time.perf_counter()

    def stop(self):
        if self.handle is None or self.thread is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.stop_flag.set()
        self.thread.join(timeout=2)
        inside = [s for s in self.samples if self.t_begin is not None and self.t_begin <= s[0] <= (self.t_end or 1e30)]
        window = inside or self.samples
        sm = [s[1] for s in window]
        bits = 0
        for s in window:
            bits |= s[2]
        reasons = sorted(name for b, name in self.REASONS.items() if bits & b)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(window), "samples_in_timed_region": len(inside), "source": "nvml"}


def physical_gpu_index(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        if local_rank < len(ids) and ids[local_rank].isdigit():
            return int(ids[local_rank])
    return local_rank


# ---------------------------------------------------------------------------
class CpuReference:
    """The reference's CPU-runnable implementation of one workload step: its
    GLSL projection shaders (kernels/proj_q4k.comp, kernels/proj_q8_0.comp) and
    kernels/activation.comp compiled for the host (oracle/_ref, OpenMP over
    the invocations), else the C restatement of the same algorithm (oracle/).

    A step is the workload's projections for all m tokens (and the SiLU gate
    of the FFN), restricted to the first `frac` of each projection's rows when
    a bounded sample is asked for."""

    def __init__(self, wl, rng):
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as orc
        from laguna_raw_halo_strix_b200 import synth

        self.orc, self.wl = orc, wl
        self.dtype = orc.Q4_K if wl["dtype"] == "q4k" else orc.Q8_0
        self.ref = orc.RefShaders() if os.path.exists(orc.REF_LIB) else None
        self.port = orc.Oracle(threads=host_threads())
        self.cores = self.port.lib.lco_get_threads()
        self.kind = "reference" if self.ref is not None else "port"
        self.w = {nm: synth.weight_blocks(self.dtype, n, k, rng) for nm, k, n in wl["shapes"]}
        self.wp = {nm: orc.pad4(w) for nm, w in self.w.items()} if self.ref is not None else None
        self.x = synth.activations(wl["m"], wl["shapes"][0][1], rng)

    def _proj(self, name, x, k, rows):
        orc, m = self.orc, x.shape[0]
        c = np.zeros((m, rows), np.float32)
        if self.ref is None:
            return self.port.proj(self.dtype, x, self.w[name][:rows], k, rows)
        shader = "proj_q4k" if self.dtype == orc.Q4_K else "proj_q8_0"
        for r in range(m):
            push = np.array([k, rows] + ([0] if self.dtype == orc.Q4_K else []), np.uint32).tobytes()
            self.ref.run(shader, [np.ascontiguousarray(x[r]), self.wp[name], c[r]], push,
                         orc.RefShaders.groups(rows))
        return c

    def step(self, frac=1.0):
        """One (sampled) step; returns the algorithmic bytes it moved."""
        wl, m = self.wl, self.wl["m"]
        nbytes = 0
        rows = {nm: max(16, int(n * frac)) for nm, k, n in wl["shapes"]}
        if wl["ffn"]:
            (_, kg, _), (_, ku, _), (_, kd, nd) = wl["shapes"]
            g = self._proj("gate", self.x, kg, rows["gate"])
            u = self._proj("up", self.x, ku, rows["up"])
            na = m * min(rows["gate"], rows["up"])
            h = np.zeros((m, kd), np.float32)
            gv, uv = g[:, :na // m].ravel().copy(), u[:, :na // m].ravel().copy()
            hv = np.zeros(na, np.float32)
            if self.ref is not None:
                self.ref.run("activation", [gv, uv, hv], np.array([na], np.uint32).tobytes(),
                             self.orc.RefShaders.groups(na))
            else:
                hv = self.port.activation(gv, uv)
            h[:, :na // m] = hv.reshape(m, -1)
            self._proj("down", h, kd, rows["down"])
            for nm, k, n in wl["shapes"]:
                nbytes += weight_bytes(wl["dtype"], k, rows[nm]) + 4 * m * (k + rows[nm])
        else:
            for nm, k, n in wl["shapes"]:
                self._proj(nm, self.x, k, rows[nm])
                nbytes += weight_bytes(wl["dtype"], k, rows[nm]) + 4 * m * (k + rows[nm])
        return nbytes

    def describe(self):
        return ("reference GLSL shaders compiled for the CPU (oracle/_ref)" if self.ref is not None
                else "C restatement of the reference algorithm (oracle/)")


def cpu_baseline(wl, min_seconds, rng):
    """Full workload steps on the host cores, repeated until min_seconds of
    CPU work; returns (GB/s, kind, cores, sample)."""
    cr = CpuReference(wl, rng)
    cr.step(0.02)  # warm (page in, thread pool)
    t0 = time.perf_counter()
    cr.step(0.05)
    est_full = (time.perf_counter() - t0) / 0.05
    frac = min(1.0, min_seconds / max(est_full, 1e-9))
    nbytes, passes = 0, 0
    t0 = time.perf_counter()
    while True:
        nbytes += cr.step(frac)
        passes += 1
        if time.perf_counter() - t0 >= min_seconds:
            break
    t = time.perf_counter() - t0
    what = "full steps" if frac >= 1.0 else f"steps sampled to {frac:.1%} of each projection's rows"
    sample = (f"{passes} {what} of {args_workload_desc(wl)}, {cr.describe()}, {t:.1f} s on {cr.cores} threads")
    return nbytes / t / 1e9, cr.kind, cr.cores, sample


def args_workload_desc(wl):
    return ", ".join(f"{nm} {k}->{n}" for nm, k, n in wl["shapes"]) + f" (m={wl['m']})"


# ---------------------------------------------------------------------------
def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    set_host_threads(host_threads())
    wl = WORKLOADS[args.workload if args.workload in WORKLOADS else "ffn_q4k_m1"]
    cr = CpuReference(wl, np.random.default_rng(0))
    # each step: the workload's step, sampled to the rows that keep the whole
    # run near 2 minutes of CPU time
    cr.step(0.02)
    t0 = time.perf_counter()
    cr.step(0.05)
    est_full = (time.perf_counter() - t0) / 0.05
    frac = min(1.0, 120.0 / (args.warmup + args.steps) / max(est_full, 1e-9))
    vals = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        nb = cr.step(frac)
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            vals.append(nb / dt / 1e9)
    value = statistics.median(vals)
    kind, cores = cr.kind, cr.cores
    what = "the full step" if frac >= 1.0 else f"the step sampled to {frac:.1%} of each projection's rows"
    sample = f"per step {what} of {args_workload_desc(wl)}, {cr.describe()}, median of {args.steps} steps"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, BASELINE distributions)",
        "config": dict(workload_config(args.workload if args.workload in WORKLOADS else "ffn_q4k_m1", wl),
                       parallelism="host cores (rank 0 only)"),
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": cores, "kind": kind, "sample": sample},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# Shared plumbing.
_PG = {"init": False}


def _dist_init():
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not _PG["init"]:
        from datetime import timedelta

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local_rank))
        _PG["init"] = True
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    return world, rank, local_rank, dev


def _max_over_ranks(v, dev, world):
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def _graph_kernel_nodes(g):
    """Kernel nodes of a captured torch CUDA graph (cudaGraphGetNodes +
    cudaGraphNodeGetType through the CUDA runtime)."""
    import ctypes as C

    try:
        import torch

        rt = None
        for name in ("libcudart.so.12", "libcudart.so"):
            try:
                rt = C.CDLL(name)
                break
            except OSError:
                pass
        if rt is None:
            import glob

            cands = glob.glob(os.path.join(os.path.dirname(torch.__file__), "..", "nvidia", "cuda_runtime", "lib",
                                           "libcudart.so*"))
            rt = C.CDLL(cands[0])
        graph = C.c_void_p(g.raw_cuda_graph())
        n = C.c_size_t(0)
        rt.cudaGraphGetNodes(graph, None, C.byref(n))
        nodes = (C.c_void_p * n.value)()
        rt.cudaGraphGetNodes(graph, nodes, C.byref(n))
        kinds = C.c_int(0)
        count = 0
        for i in range(n.value):
            rt.cudaGraphNodeGetType(C.c_void_p(nodes[i]), C.byref(kinds))
            count += kinds.value == 0  # cudaGraphNodeTypeKernel
        return count
    except Exception:
        return None


def _emit(line):
    print(json.dumps(line), flush=True)


def _timed_graph(g, stream, dev, world, rank):
    """Replay g once between barriers and synchronisation with CUDA events on
    its stream and the clocks sampled; returns (max-over-ranks ms, clocks)."""
    import torch

    _barrier(world)
    sampler = ClockSampler(dev) if rank == 0 else None
    if sampler:
        sampler.start()
    torch.cuda.synchronize(dev)
    _barrier(world)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    if sampler:
        sampler.mark_begin()
    e0.record(stream)
    g.replay()
    e1.record(stream)
    if sampler:
        sampler.sample_now()
    stream.synchronize()
    if sampler:
        sampler.mark_end()
    torch.cuda.synchronize(dev)
    _barrier(world)
    ms = _max_over_ranks(e0.elapsed_time(e1), dev, world)
    return ms, (sampler.stop() if sampler else None)


# ---------------------------------------------------------------------------
def _kernel_name(wl):
    m, q4 = wl["m"], wl["dtype"] == "q4k"
    if m <= 2:
        return "gemv_rows_kernel<Q4Lane<%d>>" % m if q4 else "gemv_rows_kernel<Q8Lane>"
    if m <= 32:
        return "x16_pack_kernel + dq_gemm_kernel"
    return "lmh_pack_kernel + lmh_kernel"


def _dtype_label(wl):
    m, w = wl["m"], ("q4k" if wl["dtype"] == "q4k" else "q8_0")
    if m <= 2:
        return w + "*f32 (f32 activations, f32 FMA accumulate)"
    if m <= 32:
        return w + "*f16x2 (activations as f16 hi+lo, ~22 bits; tcgen05 f32 accumulate)"
    return w + "*f16 (activations as one f16 after a power-of-two scale; tcgen05 f32 accumulate)"


def run_projection(args, name):
    """BASELINE configs 0, 1 and 2: projections of m tokens; the FFN workloads
    run the decoder FFN block (gate, up, SiLU-gate, down) as one lc_ffn call."""
    import torch

    from laguna_raw_halo_strix_b200 import lc, synth

    world, rank, local_rank, dev = _dist_init()
    stream = torch.cuda.Stream(dev)
    ctx = lc.Context(local_rank)
    ctx.set_stream(stream)

    wl = WORKLOADS[name]
    dtype = lc.Q4_K if wl["dtype"] == "q4k" else lc.Q8_0
    m = wl["m"]
    rng = np.random.default_rng(1000 + rank)

    # weight sets rotated through a pool > 3x L2
    set_bytes = sum(weight_bytes(wl["dtype"], k, n) for _, k, n in wl["shapes"])
    pool = max(2, -(-3 * L2_BYTES // set_bytes))
    base = {nm: torch.from_numpy(synth.weight_blocks(dtype, n, k, rng)).to(dev) for nm, k, n in wl["shapes"]}
    weights = []
    for p in range(pool):
        # distinct bytes per pool entry (flip nibbles / ints deterministically; scales stay finite)
        weights.append({nm: (t if p == 0 else t ^ torch.tensor(p * 37 % 255, dtype=torch.uint8, device=dev))
                        for nm, t in base.items()})
    k0 = wl["shapes"][0][1]
    x = torch.from_numpy(synth.activations(m, k0, rng)).to(dev)
    bufs = {nm: torch.empty(m, n, device=dev) for nm, k, n in wl["shapes"]}
    out_name = wl["shapes"][-1][0]

    def step(i):
        ws = weights[i % pool]
        if wl["ffn"]:
            (_, kg, ng), _, (_, kd, nd) = wl["shapes"]
            ctx.ffn(dtype, x, ws["gate"], ws["up"], ws["down"], bufs["down"], m, kg, ng)
        else:
            for nm, k, n in wl["shapes"]:
                ctx.proj_m(dtype, x, ws[nm], bufs[nm], m, k, n)

    # the dominant kernel alone: the first projection shape, its weights rotated
    # through their own pool > 3x L2
    dname, dk, dn = wl["shapes"][0]
    dbytes = weight_bytes(wl["dtype"], dk, dn)
    dpool = max(2, -(-3 * L2_BYTES // dbytes))
    dweights = [weights[p % pool][dname] if p < pool else
                weights[0][dname] ^ torch.tensor((p * 53 + 11) % 255, dtype=torch.uint8, device=dev)
                for p in range(dpool)]
    dx = torch.from_numpy(synth.activations(m, dk, rng)).to(dev)
    dy = torch.empty(m, dn, device=dev)

    def dominant(i):
        ctx.proj_m(dtype, dx, dweights[i % dpool], dy, m, dk, dn)

    n_dom = max(args.steps, 3 * dpool)
    with torch.cuda.stream(stream):
        for i in range(args.warmup):  # eager warm-up: sizes scratch, sets kernel attributes
            step(i)
            dominant(i)
        stream.synchronize()
        g_steps = torch.cuda.CUDAGraph(keep_graph=True)
        with torch.cuda.graph(g_steps, stream=stream):
            for i in range(args.steps):
                step(args.warmup + i)
        g_dom = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_dom, stream=stream):
            for i in range(n_dom):
                dominant(i)
        g_steps.replay()
        g_dom.replay()
        stream.synchronize()
        launches = _graph_kernel_nodes(g_steps)
        ms, clocks = _timed_graph(g_steps, stream, dev, world, rank)
        d0 = torch.cuda.Event(enable_timing=True)
        d1 = torch.cuda.Event(enable_timing=True)
        d0.record(stream)
        g_dom.replay()
        d1.record(stream)
        stream.synchronize()
        per_launch_ms = d0.elapsed_time(d1) / n_dom
        del g_steps, g_dom

        # e2e: the input copied from pinned host memory and the result read back
        # every step by the host-buffer entry points (lc_ffn_host /
        # lc_proj_m_host: upload, compute, read back and wait in one C-ABI call)
        x_host = torch.from_numpy(synth.activations(m, k0, rng)).pin_memory()
        y_host = {nm: torch.empty((m, n), dtype=torch.float32).pin_memory() for nm, k, n in wl["shapes"]}
        e2e_steps = max(100, args.steps)

        def host_step(i):
            ws = weights[i % pool]
            if wl["ffn"]:
                (_, kg, ng), _, (dn_name, kd, nd) = wl["shapes"]
                ctx.ffn_host(dtype, x_host, ws["gate"], ws["up"], ws["down"], y_host[dn_name], m, kg, ng)
            else:
                for nm, k, n in wl["shapes"]:
                    ctx.proj_m_host(dtype, x_host, ws[nm], y_host[nm], m, k, n)

        for i in range(3):
            host_step(i)
        _barrier(world)
        t0 = time.perf_counter()
        for i in range(e2e_steps):
            host_step(i)
        e2e_s = _max_over_ranks(time.perf_counter() - t0, dev, world)

    sb = step_bytes(wl)
    value = world * sb * args.steps / (ms / 1e3) / 1e9
    e2e_value = world * sb * e2e_steps / e2e_s / 1e9
    hbm, tflops, peak_src = peaks()
    lb = dbytes + 4 * m * (dk + dn)
    achieved = lb / (per_launch_ms / 1e3) / 1e9
    kernel = _kernel_name(wl)
    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            v, kind, cores, sample = cpu_baseline(wl, 10.0, np.random.default_rng(7))
            cpu = {"value": v, "unit": "GB/s", "cores": cores, "kind": kind, "sample": sample}
        _emit({
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": _dtype_label(wl),
            "data": "synthetic (seeded; BASELINE block/activation distributions)",
            "config": dict(workload_config(name, wl),
                           step=("lc_ffn: gate+up grouped, SiLU-gate fused into down" if wl["ffn"] else
                                 "lc_proj_m per projection"),
                           l2=f"weights rotated through {pool} sets of {set_bytes / 1e6:.1f} MB (> 3x the 126 MB L2)",
                           parallelism=f"replicas x{world} (independent token streams, no collective)"),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "peak_source": peak_src, "unit": "GB/s",
                         "frac": achieved / hbm, "traffic": _traffic(name, kernel), "kernel": kernel,
                         "dominant": f"{dname} {dk}->{dn}, weights rotated through {dpool} copies "
                                     f"({dpool * dbytes / 1e6:.0f} MB, > 3x L2)",
                         "per_launch_us": per_launch_ms * 1e3, "bytes_per_launch": lb},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "GB/s",
                    "h2d_bytes_per_step": int(x_host.numel() * 4) * (1 if wl["ffn"] else len(wl["shapes"])),
                    "d2h_bytes_per_step": int(y_host[out_name].numel() * 4) if wl["ffn"] else
                    int(sum(t.numel() for t in y_host.values()) * 4),
                    "steps": e2e_steps, "call": "lc_ffn_host" if wl["ffn"] else "lc_proj_m_host"},
            "clocks": clocks, "gpu_launches": None if launches is None else launches,
        })
    ctx.close()
    return 0


# ---------------------------------------------------------------------------
def lm_head_cpu_baseline(m, k, vocab, seconds, rng):
    """The reference's lm_head (target.rs:580-605: the Q8_0 projection shader
    per hidden row) and argmax on the host cores, on a sample of token rows and
    vocab rows, extrapolated to the full step; GB/s of the step's bytes."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc
    from laguna_raw_halo_strix_b200 import synth

    o = orc.Oracle(threads=host_threads())
    ref = orc.RefShaders() if os.path.exists(orc.REF_LIB) else None
    rows, toks = min(vocab, 16384), 4
    w = synth.q8_0_blocks(rows, k, rng)
    wp = orc.pad4(w) if ref is not None else None
    x = synth.activations(toks, k, rng)
    t0 = time.perf_counter()
    passes = 0
    while True:
        for r in range(toks):
            c = np.zeros(rows, np.float32)
            if ref is not None:
                ref.run("proj_q8_0", [np.ascontiguousarray(x[r]), wp, c],
                        np.array([k, rows], np.uint32).tobytes(), orc.RefShaders.groups(rows))
            else:
                c = o.proj(orc.Q8_0, x[r:r + 1], w, k, rows)[0]
            o.argmax(c)
        passes += 1
        if time.perf_counter() - t0 >= seconds:
            break
    t = (time.perf_counter() - t0) / passes
    step_s = t * (m / toks) * (vocab / rows)
    step_b = vocab * (k // 32) * 34 + 4 * m * k
    kind = "reference" if ref is not None else "port"
    sample = (f"{toks} token rows x {rows} vocab rows per pass ({passes} passes, {t * 1e3:.0f} ms each), "
              f"extrapolated to {m} rows x {vocab} vocab rows; "
              + ("reference GLSL proj_q8_0 compiled for the CPU (oracle/_ref)" if ref is not None else
                 "C restatement (oracle/)") + " + argmax")
    return step_b / step_s / 1e9, kind, o.lib.lco_get_threads(), sample


def run_lm_head(args):
    """lm_head Q8_0 4096 -> 128256 for 1024 rows (16-token
    blocks x 64 sequences) fused with argmax.  The vocab rows are split into
    contiguous shards, one per rank; each rank computes its shard's keys and one
    int64 MAX all-reduce (NCCL) gives every rank the global draft tokens.
    Total work is fixed as ranks are added ("scaling": "strong")."""
    import torch

    from laguna_raw_halo_strix_b200 import lc, synth
    from laguna_raw_halo_strix_b200.lm_head import ShardedLmHead, make_comm

    world, rank, local_rank, dev = _dist_init()
    stream = torch.cuda.Stream(dev)
    ctx = lc.Context(local_rank)
    ctx.set_stream(stream)
    m, k, vocab = LM_HEAD["m"], LM_HEAD["k"], args.vocab or LM_HEAD["vocab"]
    # the reduction through the library's own NCCL communicator (one C-ABI call per step)
    comm = make_comm(ctx, rank, world, timeout_ms=60000)
    head = ShardedLmHead(ctx, lc.Q8_0, k, vocab, rank, world, comm=comm)
    rng = np.random.default_rng(2000 + rank)
    shard = synth.q8_0_blocks(head.n_local, k, rng)
    shard_bytes = shard.nbytes
    pool = max(1, -(-3 * L2_BYTES // shard_bytes))  # weight copies so each step streams from HBM
    heads = []
    base = torch.from_numpy(shard.reshape(-1)).to(dev)
    for p in range(pool):
        h = ShardedLmHead(ctx, lc.Q8_0, k, vocab, rank, world, comm=comm)
        # distinct bytes per copy: flip only the int8 q bytes (the f16 scales stay valid)
        if p:
            w = base.view(-1, 34).clone()
            w[:, 2:] ^= (p * 37) % 255
            h.w = w.view(-1)
        else:
            h.w = base
        heads.append(h)
    x = torch.from_numpy(synth.activations(m, k, rng)).to(dev)
    keys = torch.empty(m, dtype=torch.int64, device=dev)

    def step(i):
        heads[i % pool](x, m, keys)

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            step(i)
        stream.synchronize()
        _barrier(world)
        sampler = ClockSampler(dev) if rank == 0 else None
        if sampler:
            sampler.start()
        torch.cuda.synchronize(dev)
        _barrier(world)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        if sampler:
            sampler.mark_begin()
        e0.record(stream)
        for i in range(args.steps):
            step(args.warmup + i)
        e1.record(stream)
        if sampler:
            sampler.sample_now()
        stream.synchronize()
        if sampler:
            sampler.mark_end()
        _barrier(world)
        ms = _max_over_ranks(e0.elapsed_time(e1), dev, world)
        clocks = sampler.stop() if sampler else None
        # local (kernel-only) time of one shard, for the roofline figure
        l0 = torch.cuda.Event(enable_timing=True)
        l1 = torch.cuda.Event(enable_timing=True)
        nl = max(3, min(args.steps, 20))
        l0.record(stream)
        for i in range(nl):
            heads[i % pool].local_keys(x, m, keys)
        l1.record(stream)
        stream.synchronize()
        local_ms = l0.elapsed_time(l1) / nl
        # our kernels per step: the nodes of one captured local step
        gl = torch.cuda.CUDAGraph(keep_graph=True)
        with torch.cuda.graph(gl, stream=stream):
            heads[0].local_keys(x, m, keys)
        per_step = _graph_kernel_nodes(gl)
        del gl
        # e2e: x from pinned host memory, draft tokens back to the host, every step
        x_host = torch.from_numpy(synth.activations(m, k, rng)).pin_memory()
        k_host = torch.empty(m, dtype=torch.int64).pin_memory()
        e2e_steps = max(3, min(args.steps, 20))
        _barrier(world)
        t0 = time.perf_counter()
        for i in range(e2e_steps):
            x.copy_(x_host, non_blocking=True)
            step(i)
            comm.wait()  # the bounded wait of the reduction (host deadline)
            k_host.copy_(keys, non_blocking=True)
            stream.synchronize()
        e2e_s = _max_over_ranks(time.perf_counter() - t0, dev, world)
    comm.close()

    w_total = vocab * (k // 32) * 34
    step_b = w_total + world * 4 * m * k  # every weight byte once; x read by every rank
    value = step_b * args.steps / (ms / 1e3) / 1e9
    hbm, tflops, peak_src = peaks()
    local_b = shard_bytes + 4 * m * k
    local_f = 2.0 * m * k * head.n_local
    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            v, kind, cores, sample = lm_head_cpu_baseline(m, k, vocab, 10.0, np.random.default_rng(8))
            cpu = {"value": v, "unit": "GB/s", "cores": cores, "kind": kind, "sample": sample}
        kernel = "lmh_pack_kernel + lmh_kernel"
        _emit({
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None,
            "dtype": "q8_0*f16 (activations as one f16 after a per-row power of two; tcgen05 f32 accumulate)",
            "data": "synthetic (seeded; BASELINE block/activation distributions)",
            "config": {"workload": "lm_head_q8_0", "baseline_config": LM_HEAD["config"], "m": m, "k": k,
                       "vocab": vocab, "rows_per_rank": head.n_local, "bytes_per_step": step_b,
                       "tokens_per_s": m * args.steps / (ms / 1e3),
                       "l2": f"weights rotated through {pool} copies of {shard_bytes / 1e6:.1f} MB per rank",
                       "parallelism": f"vocab-sharded x{world}, int64 MAX all-reduce of {m} keys per step "
                                      "(lc_lm_head_argmax_sharded: the library's NCCL communicator)"},
            # tensor-bound: 2 m k n_local useful flops per launch (the tcgen05 tiles)
            "roofline": {"bound": "tensor", "achieved": local_f / (local_ms / 1e3) / 1e12, "peak": tflops,
                         "peak_source": peak_src + " (dense bf16 burst)", "unit": "TFLOP/s",
                         "frac": local_f / (local_ms / 1e3) / 1e12 / tflops,
                         "traffic": _traffic("lm_head_q8_0", kernel),
                         "kernel": kernel + " (one shard)",
                         "per_launch_us": local_ms * 1e3, "flops_per_launch": local_f,
                         "hbm_gbs_per_launch": local_b / (local_ms / 1e3) / 1e9},
            "cpu_baseline": cpu,
            "e2e": {"value": step_b * e2e_steps / e2e_s / 1e9, "unit": "GB/s", "h2d_bytes_per_step": 4 * m * k,
                    "d2h_bytes_per_step": 8 * m, "steps": e2e_steps},
            "clocks": clocks, "gpu_launches": None if per_step is None else per_step * args.steps,
        })
    ctx.close()
    return 0


# ---------------------------------------------------------------------------
def dflash_cpu_baseline(seconds, rng):
    """The reference's decoder op sequence (dflash.rs:877-976, restated over
    the C kernels in oracle/dflash_oracle.py) on the host cores: one layer of
    the config-3 decoder for a sample of the block's tokens over the full
    context, extrapolated to the 6-layer 16-token block; forwards per second."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import dflash_oracle as dfo
    import oracle as orc

    hp = dict(DFLASH_HP, n_layers=1)
    o = orc.Oracle(threads=host_threads())
    t = dfo.make_model(hp, orc.Q4_K, rng)
    model = dfo.DFlashOracle(hp, t, o)
    E, KVD = hp["n_embd"], hp["n_kv_heads"] * hp["head_dim"]
    kv = [(rng.standard_normal((DFLASH_CTX, KVD)).astype(np.float32),
           rng.standard_normal((DFLASH_CTX, KVD)).astype(np.float32))]
    toks = 2
    x = rng.standard_normal((toks, E)).astype(np.float32)
    t0 = time.perf_counter()
    passes = 0
    while True:
        model.decode_block(x, kv)
        passes += 1
        if time.perf_counter() - t0 >= seconds:
            break
    per = (time.perf_counter() - t0) / passes
    fwd_s = per * DFLASH_HP["n_layers"] * (DFLASH_BLOCK / toks)
    sample = (f"one decoder layer for {toks} block tokens over {DFLASH_CTX} context rows per pass ({passes} passes, "
              f"{per:.2f} s each), extrapolated to {DFLASH_HP['n_layers']} layers x {DFLASH_BLOCK} tokens; "
              "C restatement of the reference kernels (oracle/) in the dflash.rs op order")
    return 1.0 / fwd_s, "port", o.lib.lco_get_threads(), sample


def run_dflash(args):
    """the DFlash decoder (6 layers, hidden 4096, 32 Q / 8 KV
    heads of 128, FFN 14336, Q4_K projections) for one 16-token draft block over
    2048 context rows of encoder output; a step is lc_dflash_decode_block.  The
    encoder prefill (fc 5x4096 -> 4096 over 2048 rows, context K/V) runs once
    and is timed apart.  Independent sequences on each rank ("scaling": "weak")."""
    import torch

    from laguna_raw_halo_strix_b200 import lc, synth
    from laguna_raw_halo_strix_b200.model import DFlash, hparams

    world, rank, local_rank, dev = _dist_init()
    stream = torch.cuda.Stream(dev)
    ctx = lc.Context(local_rank)
    ctx.set_stream(stream)
    hp = DFLASH_HP
    rng = np.random.default_rng(3000 + rank)
    model = DFlash(ctx, hparams(**hp), max_ctx=DFLASH_CTX, max_block=DFLASH_BLOCK)
    tensors = synth.dflash_tensors(hp, lc.Q4_K, rng, share=True)
    wbytes = 0
    for nm, (dt, a) in tensors.items():
        model.set_tensor(nm, dt, a)
        if nm.startswith("blk."):
            wbytes += a.nbytes
    E, A, M = hp["n_embd"], hp["n_aux"], DFLASH_BLOCK
    kvd = hp["n_kv_heads"] * hp["head_dim"]
    with torch.cuda.stream(stream):
        feats = torch.from_numpy(rng.standard_normal((DFLASH_CTX, A * E)).astype(np.float32)).to(dev)
        enc = torch.empty(DFLASH_CTX, E, device=dev)
        x = torch.from_numpy(rng.standard_normal((M, E)).astype(np.float32)).to(dev)
        hid = torch.empty(M, E, device=dev)
        model.encode(feats, DFLASH_CTX, enc)  # warm
        p0 = torch.cuda.Event(enable_timing=True)
        p1 = torch.cuda.Event(enable_timing=True)
        p0.record(stream)
        model.encode(feats, DFLASH_CTX, enc)
        model.set_context(enc, DFLASH_CTX)
        p1.record(stream)
        stream.synchronize()
        prefill_ms = p0.elapsed_time(p1)
        for i in range(args.warmup):
            model.decode_block(x, M, hid)
        stream.synchronize()
        g = torch.cuda.CUDAGraph(keep_graph=True)
        with torch.cuda.graph(g, stream=stream):
            for i in range(args.steps):
                model.decode_block(x, M, hid)
        g.replay()
        stream.synchronize()
        launches = _graph_kernel_nodes(g)
        ms, clocks = _timed_graph(g, stream, dev, world, rank)
        del g
        # e2e: the block's token inputs from pinned host memory, hidden states back
        x_host = torch.from_numpy(rng.standard_normal((M, E)).astype(np.float32)).pin_memory()
        h_host = torch.empty(M, E).pin_memory()
        e2e_steps = max(5, min(args.steps, 50))
        _barrier(world)
        t0 = time.perf_counter()
        for i in range(e2e_steps):
            x.copy_(x_host, non_blocking=True)
            model.decode_block(x, M, hid)
            h_host.copy_(hid, non_blocking=True)
            stream.synchronize()
        e2e_s = _max_over_ranks(time.perf_counter() - t0, dev, world)
    ok = bool(torch.isfinite(hid).all().item())
    model.close()
    kv_bytes = hp["n_layers"] * (DFLASH_CTX + M) * kvd * 2 * 4
    fwd_bytes = wbytes + kv_bytes
    fwd_s = world * args.steps / (ms / 1e3)
    hbm, _, peak_src = peaks()
    per_fwd_s = ms / 1e3 / args.steps
    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            v, kind, cores, sample = dflash_cpu_baseline(10.0, np.random.default_rng(9))
            cpu = {"value": v, "unit": "fwd/s", "cores": cores, "kind": kind, "sample": sample}
        _emit({
            "metric": METRIC, "value": fwd_s, "unit": "fwd/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None,
            "dtype": "q4k*f16x2 projections (activations as f16 hi+lo, ~22 bits; tcgen05 f32 accumulate), "
                     "f32 element-wise ops, attention f16 hi/lo on tcgen05",
            "data": "synthetic (seeded; BASELINE distributions; one set of projection weights per shape, "
                    "uploaded separately for every layer)",
            "config": {"workload": "dflash_block", "baseline_config": 3, "layers": hp["n_layers"], "hidden": E,
                       "heads": hp["n_heads"], "kv_heads": hp["n_kv_heads"], "ffn": hp["n_ff"],
                       "context": DFLASH_CTX, "block": M, "bytes_per_fwd": fwd_bytes,
                       "prefill_ms": prefill_ms, "finite": ok,
                       "l2": f"{fwd_bytes / 1e6:.0f} MB streamed per forward (> 3x the 126 MB L2)",
                       "parallelism": f"replicas x{world} (independent sequences, no collective)"},
            "roofline": {"bound": "hbm", "achieved": fwd_bytes / per_fwd_s / 1e9, "peak": hbm,
                         "peak_source": peak_src, "unit": "GB/s", "frac": fwd_bytes / per_fwd_s / 1e9 / hbm,
                         "traffic": None, "kernel": "whole decoder step (all kernels)",
                         "per_launch_us": per_fwd_s * 1e6, "bytes_per_launch": fwd_bytes},
            "cpu_baseline": cpu,
            "e2e": {"value": world * e2e_steps / e2e_s, "unit": "fwd/s", "h2d_bytes_per_step": 4 * M * E,
                    "d2h_bytes_per_step": 4 * M * E, "steps": e2e_steps},
            "clocks": clocks, "gpu_launches": launches,
        })
    ctx.close()
    return 0


# ---------------------------------------------------------------------------
# The target model's verify step (no BASELINE configuration names one): a
# Laguna-shaped model -- hidden 4096, 32 Q / 8 KV heads of 128, layer 0 dense
# (FFN 14336), layers 1-3 MoE (64 experts of 1024, 8 used, a shared expert of
# 1024), Q4_K projections, a 32000-row Q8_0 lm_head -- verifying a block of 16
# draft tokens through its K/V cache of 2048 positions, then rolled back.
TARGET_HP = dict(n_layers=4, n_embd=4096, n_heads=32, n_kv_heads=8, head_dim=128, rope_dim=128, rope_dim_swa=128,
                 n_ff=14336, n_expert=64, n_expert_used=8, n_ff_exp=1024, n_ff_shexp=1024, n_vocab=32000)
TARGET_CTX, TARGET_BLOCK = 2048, 16


def run_target_verify(args):
    """Verify throughput (draft tokens checked per second) of lc_target_forward
    with LC_TARGET_CACHED: one step = a 16-token block at positions 2048..2063
    (K/V appended, causal attention over the cache, MoE routed on the device,
    lm_head keys), the cache then truncated back to 2048."""
    import tempfile

    import torch

    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from gguf_writer import write_gguf

    from laguna_raw_halo_strix_b200 import lc, synth
    from laguna_raw_halo_strix_b200.target import Target

    world, rank, local_rank, dev = _dist_init()
    stream = torch.cuda.Stream(dev)
    ctx = lc.Context(local_rank)
    ctx.set_stream(stream)
    hp, C, M = TARGET_HP, TARGET_CTX, TARGET_BLOCK
    E = hp["n_embd"]
    rng = np.random.default_rng(4000 + rank)
    tens = synth.target_tensors(hp, rng, share=True)
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "target.gguf")
        write_gguf(path, synth.target_meta(hp),
                   [(n, dt, shape, np.ascontiguousarray(a).view(np.uint8).reshape(-1))
                    for n, (dt, a, shape) in tens.items()])
        file_bytes = os.path.getsize(path)
        t0 = time.perf_counter()
        tm = Target(ctx, path, max_ctx=C + M, max_block=M)
        load_s = time.perf_counter() - t0
    with torch.cuda.stream(stream):
        x = torch.from_numpy((0.5 * rng.standard_normal((M, E))).astype(np.float32)).to(dev)
        keys = torch.empty(M, dtype=torch.int64, device=dev)
        for _ in range(C // M):  # the cache: 2048 positions
            tm.forward(x, M, cached=True)
        for _ in range(args.warmup):
            tm.forward(x, M, cached=True, keys=keys)
            tm.truncate(C)
        stream.synchronize()
        g = torch.cuda.CUDAGraph(keep_graph=True)
        with torch.cuda.graph(g, stream=stream):
            for _ in range(args.steps):
                tm.forward(x, M, cached=True, keys=keys)
                tm.truncate(C)
        g.replay()
        stream.synchronize()
        launches = _graph_kernel_nodes(g)
        ms, clocks = _timed_graph(g, stream, dev, world, rank)
        del g
        x_host = torch.from_numpy((0.5 * rng.standard_normal((M, E))).astype(np.float32)).pin_memory()
        k_host = torch.empty(M, dtype=torch.int64).pin_memory()
        e2e_steps = max(5, min(args.steps, 50))
        _barrier(world)
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            x.copy_(x_host, non_blocking=True)
            tm.forward(x, M, cached=True, keys=keys)
            tm.truncate(C)
            k_host.copy_(keys, non_blocking=True)
            stream.synchronize()
        e2e_s = _max_over_ranks(time.perf_counter() - t0, dev, world)
        # the experts the last verify step selected, per MoE layer (lc_target_routing)
        distinct_per_layer = []
        for layer in range(1, hp["n_layers"]):
            ids, _ = tm.routing(layer)
            distinct_per_layer.append(int(torch.unique(ids[ids >= 0]).numel()))
    tm.close()
    # bytes one verify step must read: every dense projection, the router and
    # shared expert, the experts the block selected, the K/V cache and the lm_head
    q4 = 144 / 256
    H, KVD, F = hp["n_heads"], hp["n_kv_heads"] * hp["head_dim"], hp["n_ff"]
    QD = H * hp["head_dim"]
    NE, U, Fe, S, V = hp["n_expert"], hp["n_expert_used"], hp["n_ff_exp"], hp["n_ff_shexp"], hp["n_vocab"]
    attn_b = ((QD + 2 * KVD + H) * E + E * QD) * q4
    distinct = sum(distinct_per_layer)
    moe_b = (hp["n_layers"] - 1) * (E * NE * 4 + 3 * S * E * q4) + distinct * 3 * Fe * E * q4
    # what the step actually streams: a 16-row block covers the expert set
    # (16 x 8 >= 64), so every expert's gate / up / down run as dense GEMMs
    read_b = (hp["n_layers"] * attn_b + 3 * F * E * q4
              + (hp["n_layers"] - 1) * (E * NE * 4 + 3 * S * E * q4 + NE * 3 * Fe * E * q4)
              + hp["n_layers"] * (C + M) * KVD * 2 * 4 + V * E * 34 / 32)
    step_b = (hp["n_layers"] * attn_b + 3 * F * E * q4 + moe_b
              + hp["n_layers"] * (C + M) * KVD * 2 * 4 + V * E * 34 / 32)
    hbm, _, peak_src = peaks()
    per_step_s = ms / 1e3 / args.steps
    if rank == 0:
        _emit({
            "metric": METRIC, "value": world * M * args.steps / (ms / 1e3), "unit": "verified tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "q4k*f16x2 projections (tcgen05 f32 accumulate), f32 expert GEMV, f32 element-wise ops",
            "data": "synthetic (seeded; one array per distinct shape, its own device copy per layer and expert)",
            "config": {"workload": "target_verify", "baseline_config": None, "layers": hp["n_layers"],
                       "hidden": E, "heads": H, "kv_heads": hp["n_kv_heads"], "ffn_dense": F, "experts": NE,
                       "experts_used": U, "ffn_expert": Fe, "ffn_shared": S, "vocab": V, "cache": C, "block": M,
                       "bytes_per_step": step_b, "distinct_experts_per_moe_layer": distinct_per_layer,
                       "bytes_streamed_per_step": read_b,
                       "gguf_bytes": file_bytes,
                       "load_s": load_s, "load_gbs": file_bytes / load_s / 1e9,
                       "l2": f"{step_b / 1e6:.0f} MB read per step (> 3x the 126 MB L2)",
                       "parallelism": f"replicas x{world} (independent sequences, no collective)"},
            "roofline": {"bound": "hbm", "achieved": step_b / per_step_s / 1e9, "peak": hbm,
                         "peak_source": peak_src, "unit": "GB/s", "frac": step_b / per_step_s / 1e9 / hbm,
                         "traffic": None, "kernel": "whole verify step (all kernels)",
                         "per_launch_us": per_step_s * 1e6, "bytes_per_launch": step_b},
            "cpu_baseline": None,
            "e2e": {"value": world * M * e2e_steps / e2e_s, "unit": "verified tokens/s",
                    "h2d_bytes_per_step": 4 * M * E, "d2h_bytes_per_step": 8 * M, "steps": e2e_steps},
            "clocks": clocks, "gpu_launches": launches,
        })
    ctx.close()
    return 0


DEFAULT_SEQUENCE = ("gemv_q8_0", "ffn_q4k_m16", "dflash_block", "lm_head_q8_0", "ffn_q4k_m1")


def run_workload(args, name):
    if name == "target_verify":
        return run_target_verify(args)
    if name == "lm_head_q8_0":
        return run_lm_head(args)
    if name == "dflash_block":
        return run_dflash(args)
    return run_projection(args, name)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--workload", default="all", choices=["all"] + sorted(WORKLOADS) + list(SPECIAL),
                    help="one workload, or all of them with the headline (ffn_q4k_m1) last (default)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--vocab", type=int, default=0,
                    help="lm_head_q8_0 only: vocab rows (default: BASELINE config 4's 128256); a smaller vocab "
                         "keeps an ncu capture short")
    ap.add_argument("--cpu-threads", type=int, default=0,
                    help="threads of the CPU baselines and the reference arm (default: all usable host threads)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    _CPU_THREADS[0] = max(0, args.cpu_threads)

    if args.impl == "reference":
        return run_reference_arm(args)
    names = DEFAULT_SEQUENCE if args.workload == "all" else (args.workload,)
    for name in names:
        run_workload(args, name)
    if _PG["init"]:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
