"""Benchmark of the B200 GDN forward (driver contract: one JSON line on rank 0).

Headline workload: Qwen3-Next GDN layer chunked prefill,
B=1, T=8192, 16 q/k heads, 32 v heads, d=128, bf16 q/k/v, fp32 g/beta, in-kernel
q/k L2 norm, fp32 final state.  A "step" is one ``chunk_gated_delta_rule``
call over that batch.  With N GPUs (torchrun) every rank runs its own
config-1 sequence (sharding by sequence, no collective on the data path):
weak scaling, ``value`` = N * 8192 tokens / max-over-ranks time.

Also reported: recurrent decode microseconds per step and
its fraction of measured HBM bandwidth; a CPU baseline (the oracle's fp32
chunked restatement of the reference algorithm) timed on the host's cores.

``--impl reference`` times that CPU restatement alone on the same config (a
bounded token sample per step), since the reference itself targets Cambricon
MLUs and cannot run here.
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

# BASELINE config 1 / 3 shapes
CFG1 = dict(B=1, T=8192, H=16, HV=32, K=128, V=128)
CFG3 = dict(N=256, slots=1024, H=16, HV=32, K=128, V=128)
BT = 64
CPU_SAMPLE_TOKENS = 8192  # the whole config-1 sequence


def flops_per_token_head(K, V, bt=BT):
    # 2 * (BT*(3K+2V) + 3KV): KK^T, w, u, w.h, K^T v_new, q.h, qK^T, A v_new
    return 2 * (bt * (3 * K + 2 * V) + 3 * K * V)


def stage_flops_per_token_head(K, V, bt=BT, path="tc"):
    """Algorithmic FLOPs per token per v-head of each kernel (bf16 GEMMs).
    tcgen05 path: the WY kernel does KK^T, qK^T, w, u; the state kernel does
    w.h, q.h, K^T v_new and A v_new.  Generic path: wy / state / out."""
    if path == "tc":
        wy = 2 * bt * K + 2 * bt * K + 2 * bt * K + 2 * bt * V
        state = 2 * K * V * 3 + 2 * bt * V
        return {"wy": wy, "state": state, "fused": wy + state}
    return {
        "wy": 2 * bt * K + 2 * bt * K + 2 * bt * V,       # KK^T, w, u
        "state": 2 * K * V + 2 * K * V,                     # w.h, K^T v_new
        "out": 2 * K * V + 2 * bt * K + 2 * bt * V,         # q.h, qK^T, A v_new
    }


def prefill_bytes(T, H, HV, K, V, nseq, state_out=True):
    b = T * (2 * H * K * 2 + 2 * HV * V * 2 + 2 * HV * 4)
    if state_out:
        b += nseq * HV * K * V * 4
    return b


def _load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d["bf16_tflops_sustained"]), "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


def _load_traffic():
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        return json.load(open(p))
    except Exception:
        return {}


class ClockSampler:
    """SM clock and clock-event reasons sampled DURING the timed region.

    A timed region here lasts a few milliseconds, far shorter than
    nvidia-smi's sampling period, so the GPU is read through NVML (read-only
    queries) by a background thread about every millisecond while the region
    runs, and :meth:`sample` takes one more reading between step launches,
    while the GPU is still busy with queued work.  Falls back to an
    ``nvidia-smi -lms 200`` stream when NVML is unavailable.
    """

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))
    SMI_FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                  "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                  "clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid):
        self.uuid = uuid
        self.nvml = None
        self.handle = None
        self.proc = None
        self.samples = []  # (sm MHz, set of reasons)
        self.max_mhz = None
        self.source = None
        self._stop = threading.Event()
        self._lock = threading.Lock()

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByUUID(self.uuid) if self.uuid else \
                pynvml.nvmlDeviceGetHandleByIndex(0)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM))
            self.bits = [(nm, getattr(pynvml, attr)) for nm, attr in self.REASONS]
            self.source = "NVML, polled about every 1 ms during the timed region and between step launches"
            self.t = threading.Thread(target=self._poll, daemon=True)
            self.t.start()
        except Exception:
            self.nvml = None
            self._start_smi()
        return self

    def sample(self):
        """One reading now (call it right after launching a step)."""
        if self.nvml is None:
            return
        try:
            mhz = float(self.nvml.nvmlDeviceGetClockInfo(self.handle, self.nvml.NVML_CLOCK_SM))
            mask = self.nvml.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
        except Exception:
            return
        with self._lock:
            self.samples.append((mhz, {nm for nm, bit in self.bits if mask & bit}))

    def _poll(self):
        while not self._stop.is_set():
            self.sample()
            time.sleep(0.001)

    def _start_smi(self):
        cmd = ["nvidia-smi", f"--query-gpu={self.SMI_FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"]
        if self.uuid:
            cmd += ["-i", self.uuid]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.lines = []
            self.t = threading.Thread(target=lambda: [self.lines.append(l.strip()) for l in self.proc.stdout],
                                      daemon=True)
            self.t.start()
            self.source = "nvidia-smi -lms 200"
        except Exception:
            self.proc = None

    def __exit__(self, *exc):
        if self.nvml is not None:
            self._stop.set()
            self.t.join(timeout=1)
            try:
                self.nvml.nvmlShutdown()
            except Exception:
                pass
        elif self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            names = [nm for nm, _ in self.REASONS]
            for l in self.lines:
                parts = [x.strip() for x in l.split(",")]
                if len(parts) < 7:
                    continue
                try:
                    mhz, self.max_mhz = float(parts[0]), float(parts[1])
                except ValueError:
                    continue
                self.samples.append((mhz, {nm for nm, v in zip(names, parts[3:7]) if v.lower() == "active"}))

    def summary(self):
        with self._lock:
            sm = [m for m, _ in self.samples]
            reasons = set().union(*[r for _, r in self.samples]) if self.samples else set()
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(sm), "source": self.source}


# --------------------------------------------------------------------------
# CPU baseline: the oracle's fp32 chunked restatement, v-heads split over
# worker processes, the remaining cores given to each worker's BLAS
# --------------------------------------------------------------------------

def _cpu_worker(args):
    import numpy as np
    import oracle
    q, k, v, g, beta = args
    t0 = time.perf_counter()
    oracle.chunk_gated_delta_rule(q, k, v, g, beta, None, None, True, None, True, dtype=np.float32)
    return time.perf_counter() - t0


def _cpu_inputs(T, H, HV, K, V, seed=1):
    import numpy as np
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((1, T, H, K)).astype(np.float32)
    k = rng.standard_normal((1, T, H, K)).astype(np.float32)
    v = rng.standard_normal((1, T, HV, V)).astype(np.float32)
    g = -np.log1p(np.exp(-rng.standard_normal((1, T, HV)))).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((1, T, HV))))).astype(np.float32)
    G = HV // H
    parts = []
    for hv in range(HV):  # one v-head (and its q/k head) per task: the recurrences are independent
        h = hv // G
        parts.append((q[:, :, h:h + 1], k[:, :, h:h + 1], v[:, :, hv:hv + 1], g[:, :, hv:hv + 1],
                      beta[:, :, hv:hv + 1]))
    return parts


class CpuBaseline:
    def __init__(self, cfg, sample_tokens=CPU_SAMPLE_TOKENS):
        import multiprocessing as mp
        self.cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
        # one worker per v-head task up to the core count; leftover cores go to
        # each worker's BLAS threads, so every core is used without oversubscription
        self.workers = max(1, min(self.cores, cfg["HV"]))
        self.blas_threads = max(1, self.cores // self.workers)
        saved = {v: os.environ.get(v) for v in ("OPENBLAS_NUM_THREADS", "OMP_NUM_THREADS", "MKL_NUM_THREADS")}
        for var in saved:
            os.environ[var] = str(self.blas_threads)
        self.pool = mp.get_context("spawn").Pool(self.workers)
        for var, val in saved.items():
            if val is None:
                os.environ.pop(var, None)
            else:
                os.environ[var] = val
        self.parts = _cpu_inputs(sample_tokens, cfg["H"], cfg["HV"], cfg["K"], cfg["V"])
        self.tokens = sample_tokens

    def step(self):
        t0 = time.perf_counter()
        self.pool.map(_cpu_worker, self.parts, chunksize=1)
        return time.perf_counter() - t0

    def close(self):
        self.pool.close()
        self.pool.join()


def _cpu_model():
    try:
        for l in open("/proc/cpuinfo"):
            if l.startswith("model name"):
                return l.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


# --------------------------------------------------------------------------

def _dist_setup(n_gpus):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def _max_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def run_ours(a):
    import ctypes

    import torch

    import domesticated_torch_mlu_ops_b200 as ops
    from domesticated_torch_mlu_ops_b200 import _lib

    world, rank, local = _dist_setup(a.gpus)
    dev = torch.device("cuda", torch.cuda.current_device())
    hbm, tc_burst, tc_sust, peak_kind = _load_peaks()
    cfg = dict(CFG1)
    if a.tokens:
        cfg["T"] = a.tokens
    H, HV, K, V = (cfg[x] for x in ("H", "HV", "K", "V"))
    wl = _workload(a.workload, world, rank, cfg)
    B, T, cu_list, nseq_total, tokens_total = wl["B"], wl["T"], wl["cu"], wl["nseq"], wl["tokens"]
    N = B if cu_list is None else len(cu_list) - 1

    cpu = (CpuBaseline(cfg) if (rank == 0 and world == 1 and not a.no_cpu and a.workload == "cfg1")
           else None)

    gen = torch.Generator().manual_seed(wl["seed"] + rank)
    q_h = torch.randn(B, T, H, K, generator=gen).bfloat16().pin_memory()
    k_h = torch.randn(B, T, H, K, generator=gen).bfloat16().pin_memory()
    v_h = torch.randn(B, T, HV, V, generator=gen).bfloat16().pin_memory()
    g_h = torch.nn.functional.logsigmoid(torch.randn(B, T, HV, generator=gen)).pin_memory()
    b_h = torch.sigmoid(torch.randn(B, T, HV, generator=gen)).pin_memory()
    h0 = (torch.randn(N, HV, K, V, generator=gen) * 0.02).to(dev) if wl["h0"] else None
    cu = None if cu_list is None else torch.tensor(cu_list, dtype=torch.int64, device=dev)
    q, k, v, g, beta = (x.to(dev) for x in (q_h, k_h, v_h, g_h, b_h))
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    lib = _lib.load()

    def step():
        return ops.chunk_gated_delta_rule(q, k, v, g, beta, None, h0, True, cu,
                                          use_qk_l2norm_in_kernel=True)

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()

    # ---- device-resident timing (per-step events, L2 flushed between) ----
    stream = torch.cuda.current_stream(dev)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(a.steps)]
    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(dev).uuid)
        uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
    except Exception:
        pass
    _barrier(world)
    torch.cuda.synchronize()
    n0 = lib.gdn_kernel_launch_count()
    with ClockSampler(uuid) as clk:
        for i in range(a.steps):
            flush.zero_()
            evs[i][0].record(stream)
            step()
            evs[i][1].record(stream)
            clk.sample()  # the step's kernels are queued or running
        torch.cuda.synchronize()
    _barrier(world)
    launches = lib.gdn_kernel_launch_count() - n0
    step_ms = [s.elapsed_time(e) for s, e in evs]
    ms_local = sum(step_ms) / len(step_ms)
    ms = _max_over_ranks(ms_local, world)

    # ---- N > 1: the same step followed by the final gather of every rank's
    # outputs and final states onto rank 0 (NCCL gather over NVLink), and,
    # for callers that need the whole output everywhere, onto every rank ----
    gather = allgather = None
    if world > 1:
        from domesticated_torch_mlu_ops_b200 import shard
        tok_all = wl["tokens"] if wl["scaling"] == "strong" else world * B * T
        for dst in (0, None):
            plan = shard.OutputGather(wl["parts"], wl["lens"], dev, rank, state_shape=(HV, K, V), dst=dst)
            ms_g = _timed(lambda: plan(*step()), a.steps, flush, stream, world)
            res = {"value": tok_all / (ms_g / 1e3), "unit": "tokens/s", "ms_per_step": ms_g,
                   "bytes_received": plan.gathered_bytes(torch.empty(1, 1, HV, V, dtype=torch.bfloat16))}
            if dst == 0:
                res["collective"] = ("torch.distributed gather (NCCL) of the packed bf16 outputs and fp32 "
                                     "final states to rank 0, then a row permutation there")
                gather = res
            else:
                res["collective"] = ("torch.distributed all_gather_into_tensor (NCCL): every rank ends "
                                     "with the whole output")
                allgather = res

    # ---- the other ways the prefill shards (BASELINE configs 4 and 1) ----
    subs = None
    if a.workload == "cfg1" and not a.tokens and not a.no_subs:
        subs = {"cfg4": _sub_cfg4(ops, dev, world, rank, a, flush, stream)}
        if world > 1:
            subs["cfg1_heads"] = _sub_heads(ops, dev, world, rank, a, flush, stream)

    # ---- per-kernel timing with the library's stage events ----
    nst = 8
    sev = [torch.cuda.Event(enable_timing=True) for _ in range(nst)]
    for e in sev:  # torch creates the CUDA event on first record
        e.record(stream)
    torch.cuda.synchronize()
    handles = (ctypes.c_void_p * nst)(*[ctypes.c_void_p(e.cuda_event) for e in sev])
    stage_ms = {}
    names = None
    reps = max(3, min(a.steps, 10))
    for _ in range(reps):
        flush.zero_()
        o, ht, info = _chunk_with_events(ops, q, k, v, g, beta, handles, nst, cu, h0)
        torch.cuda.synchronize()
        names = info["stages"]
        for i, nm in enumerate(names):
            stage_ms.setdefault(nm, []).append(sev[i].elapsed_time(sev[i + 1]))
    stage_avg = {nm: sum(x) / len(x) for nm, x in stage_ms.items()}

    # ---- end-to-end through the public API with host buffers ----
    e2e_ms, h2d, d2h = None, 0, 0
    if not a.no_e2e:
        e2e_evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in range(a.steps)]
        h0_h = None if h0 is None else h0.cpu().pin_memory()
        cu_h = None if cu is None else cu.cpu()
        extra_h = [x for x in (h0_h, cu_h) if x is not None]

        # page-locked outputs allocated once, as a serving loop would keep them
        o_out = torch.empty(B, T, HV, V, dtype=torch.bfloat16).pin_memory()
        ht_out = torch.empty(N, HV, K, V, dtype=torch.float32).pin_memory()

        def e2e_step():
            # host buffers in, host buffers out, through the public host-memory entry point
            return ops.chunk_gated_delta_rule_from_host(q_h, k_h, v_h, g_h, b_h, None, h0_h, True, cu_h,
                                                        use_qk_l2norm_in_kernel=True, device=dev,
                                                        segment_tokens=a.segment_tokens,
                                                        o_out=o_out, final_state_out=ht_out)

        for _ in range(2):
            e2e_step()
        _barrier(world)
        torch.cuda.synchronize()
        for i in range(a.steps):
            flush.zero_()
            e2e_evs[i][0].record(stream)
            o_h, ht_h = e2e_step()
            e2e_evs[i][1].record(stream)
        torch.cuda.synchronize()
        e2e_ms = _max_over_ranks(sum(s.elapsed_time(e) for s, e in e2e_evs) / a.steps, world)
        h2d = sum(x.numel() * x.element_size() for x in [q_h, k_h, v_h, g_h, b_h] + extra_h)
        d2h = o_h.numel() * o_h.element_size() + ht_h.numel() * ht_h.element_size()

    # ---- decode (config 3) and the causal conv1d in front of the layer ----
    dec = _decode_bench(ops, dev, a, hbm, flush, peak_kind) if not a.no_decode else None
    conv = _conv_bench(ops, dev, a, hbm, flush, peak_kind) if not a.no_decode and rank == 0 else None
    bwd = _bwd_bench(ops, dev, a, flush, tc_burst, peak_kind) if not a.no_bwd and rank == 0 else None

    # ---- CPU baseline (rank 0, N=1) ----
    cpu_line = None
    if cpu is not None:
        cpu.step()  # warm-up (imports in the workers)
        t_cpu = []
        t_end = time.perf_counter() + 20.0
        while time.perf_counter() < t_end and len(t_cpu) < 5:
            t_cpu.append(cpu.step())
        cpu.close()
        best = min(t_cpu)
        cpu_line = {"value": cpu.tokens / best, "unit": "tokens/s", "cores": cpu.cores,
                    "kind": "port",
                    "sample": f"{cpu.tokens} tokens of the config-1 shape (all 32 v-heads), numpy fp32 "
                              f"chunked restatement, {cpu.workers} worker processes x {cpu.blas_threads} "
                              f"BLAS threads on {cpu.cores} cores, best of {len(t_cpu)}; host {_cpu_model()}"}

    if rank == 0:
        tokens = tokens_total if wl["scaling"] == "strong" else world * B * T
        value = tokens / (ms / 1e3)
        fl_tok = flops_per_token_head(K, V)
        total_flops = B * T * HV * fl_tok  # this rank's share (rank 0)
        sfl = stage_flops_per_token_head(K, V, path="tc" if "plan" in stage_avg and len(stage_avg) <= 3 else "generic")
        dom = max(stage_avg, key=stage_avg.get)
        dom_key = dom.split(":")[0]
        dom_flops = B * T * HV * sfl.get(dom_key, 0)
        traffic = _load_traffic().get(dom) if a.workload == "cfg1" and not a.tokens else None
        roof = {"kernel": dom, "bound": "tensor", "achieved": dom_flops / (stage_avg[dom] * 1e-3) / 1e12,
                "peak": tc_burst, "unit": "TFLOP/s", "peak_kind": f"{peak_kind} bf16 burst",
                "traffic": traffic}
        roof["frac"] = roof["achieved"] / roof["peak"]
        pbytes = prefill_bytes(B * T, H, HV, K, V, N)
        line = {
            "metric": wl["metric"],
            "value": value, "unit": "tokens/s", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": wl["scaling"],
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) q/k/v, "
            "logsigmoid/sigmoid gates; BASELINE config distributions)",
            "config": {"workload": wl["desc"], "tokens_per_gpu": B * T,
                       "parallelism": wl["par"],
                       "l2": "256 MiB buffer written between timed steps"},
            "roofline": roof,
            "path_roofline": {"flops": total_flops, "tflops": total_flops / (ms * 1e-3) / 1e12,
                              "frac_tensor": total_flops / (ms * 1e-3) / 1e12 / tc_burst,
                              "algorithmic_bytes": pbytes,
                              "frac_hbm": pbytes / (ms * 1e-3) / 1e9 / hbm},
            "stages_ms": stage_avg,
            "e2e": None if e2e_ms is None else {
                "value": tokens / (e2e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "api": f"chunk_gated_delta_rule_from_host (pinned host tensors in and out, outputs "
                       f"preallocated; {a.segment_tokens}-token pieces: copy-in, compute and copy-out "
                       f"overlap)"},
            "gpu_launches": int(launches),
            "with_gather": gather,
            "with_allgather": allgather,
            "sharded": subs,
            "clocks": clk.summary(),
            "decode": dec,
            "conv1d": conv,
            "backward": bwd,
            "cpu_baseline": cpu_line,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def _timed(fn, steps, flush, stream, world, warmup=3):
    """Mean device time (ms) of ``fn`` over ``steps`` calls, L2 flushed
    before each, barrier + synchronize around the region, max over ranks."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    _barrier(world)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for st, en in evs:
        flush.zero_()
        st.record(stream)
        fn()
        en.record(stream)
    torch.cuda.synchronize()
    _barrier(world)
    return _max_over_ranks(sum(st.elapsed_time(en) for st, en in evs) / steps, world)


def _sub_cfg4(ops, dev, world, rank, a, flush, stream):
    """BASELINE config 4 (64 sequences x 4096 tokens, seed 4) split by
    sequence, 64/N per rank (strong scaling); with the gather of outputs and
    final states to rank 0."""
    import torch
    from domesticated_torch_mlu_ops_b200 import shard
    H, HV, K, V = (CFG1[x] for x in ("H", "HV", "K", "V"))
    if 64 % world:
        return {"skipped": f"64 sequences do not split over {world} ranks"}
    b, T = 64 // world, 4096
    gen = torch.Generator().manual_seed(4 + rank)
    q = torch.randn(b, T, H, K, generator=gen).bfloat16().to(dev)
    k = torch.randn(b, T, H, K, generator=gen).bfloat16().to(dev)
    v = torch.randn(b, T, HV, V, generator=gen).bfloat16().to(dev)
    g = torch.nn.functional.logsigmoid(torch.randn(b, T, HV, generator=gen)).to(dev)
    beta = torch.sigmoid(torch.randn(b, T, HV, generator=gen)).to(dev)

    def step():
        return ops.chunk_gated_delta_rule(q, k, v, g, beta, None, None, True, use_qk_l2norm_in_kernel=True)

    steps = max(3, min(a.steps, 10))
    ms = _timed(step, steps, flush, stream, world)
    out = {"workload": "config4: 64 x 4096 tokens, H=16 HV=32 K=V=128 bf16, in-kernel q/k L2 norm",
           "parallelism": f"sequence-sharded x{world} ({b} sequences per rank)", "scaling": "strong",
           "value": 64 * T / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms,
           "tokens_per_s_per_gpu": 64 * T / (ms / 1e3) / world}
    if world > 1:
        parts = [list(range(r * b, r * b + b)) for r in range(world)]
        plan = shard.OutputGather(parts, [T] * 64, dev, rank, state_shape=(HV, K, V), dst=0)
        ms_g = _timed(lambda: plan(*step()), steps, flush, stream, world)
        out["with_gather"] = {"value": 64 * T / (ms_g / 1e3), "unit": "tokens/s", "ms_per_step": ms_g,
                              "collective": "NCCL gather of outputs and final states to rank 0",
                              "bytes_received": plan.gathered_bytes(v)}
    del q, k, v, g, beta
    return out


def _sub_heads(ops, dev, world, rank, a, flush, stream):
    """BASELINE config 1's single sequence split by v-head groups (each rank
    owns H/N q/k heads and their v-heads; shard.partition_heads): strong
    scaling of one sequence; with the gather of outputs and final states to
    rank 0."""
    import torch
    from domesticated_torch_mlu_ops_b200 import shard
    B, T, H, HV, K, V = (CFG1[x] for x in ("B", "T", "H", "HV", "K", "V"))
    if H % world:
        return {"skipped": f"{H} q/k heads do not split over {world} ranks"}
    gen = torch.Generator().manual_seed(1)
    full = (torch.randn(B, T, H, K, generator=gen).bfloat16(), torch.randn(B, T, H, K, generator=gen).bfloat16(),
            torch.randn(B, T, HV, V, generator=gen).bfloat16(),
            torch.nn.functional.logsigmoid(torch.randn(B, T, HV, generator=gen)),
            torch.sigmoid(torch.randn(B, T, HV, generator=gen)))
    rng_ = shard.partition_heads(H, HV, world)[rank]
    q, k, v, g, beta, _ = (None if x is None else x.to(dev)
                           for x in shard.head_slices(*full, None, rng_, HV // H))

    def step():
        return ops.chunk_gated_delta_rule(q, k, v, g, beta, None, None, True, use_qk_l2norm_in_kernel=True)

    steps = max(3, min(a.steps, 10))
    ms = _timed(step, steps, flush, stream, world)
    hg = shard.HeadGather(world, rank, dst=0)
    ms_g = _timed(lambda: hg(*step()), steps, flush, stream, world)
    o_, ht_ = step()
    return {"workload": "config1 (B=1 T=8192 H=16 HV=32 K=V=128 bf16) split by v-head groups",
            "parallelism": f"head-sharded x{world} ({H // world} q/k heads, {HV // world} v-heads per rank)",
            "scaling": "strong", "value": B * T / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms,
            "with_gather": {"value": B * T / (ms_g / 1e3), "unit": "tokens/s", "ms_per_step": ms_g,
                            "collective": "NCCL gather of the head groups' outputs and final states to rank 0",
                            "bytes_received": hg.gathered_bytes(o_, ht_)}}


def _workload(name, world, rank, cfg):
    """Per-rank shape of a BASELINE prefill config.

    cfg1: one B=1, T=8192 sequence per rank (weak scaling).
    cfg2: 16 sequences, lengths U[512, 8192] (seed 2), packed with cu_seqlens,
          initial states N(0, 0.02); sequences split across ranks by token
          count (strong scaling).
    cfg4: 64 sequences x 4096 tokens split evenly across ranks (strong scaling).
    """
    from domesticated_torch_mlu_ops_b200 import shard
    if name == "cfg1":
        return dict(B=1, T=cfg["T"], cu=None, nseq=world, tokens=world * cfg["T"], seed=1, h0=False,
                    lens=[cfg["T"]] * world, parts=[[r] for r in range(world)],
                    scaling="weak", par=f"sequence-sharded x{world} (one sequence per rank)",
                    metric="prefill tokens/s (Qwen3-Next GDN layer chunked prefill, BASELINE config 1)",
                    desc=f"config1: chunk_gated_delta_rule B=1 T={cfg['T']} H=16 HV=32 K=V=128 bf16, "
                         "in-kernel q/k L2 norm, fp32 final state")
    if name == "cfg4":
        if 64 % world:
            raise SystemExit("cfg4 needs the GPU count to divide 64")
        b = 64 // world
        return dict(B=b, T=4096, cu=None, nseq=64, tokens=64 * 4096, seed=4, h0=False,
                    lens=[4096] * 64, parts=[list(range(r * b, r * b + b)) for r in range(world)],
                    scaling="strong", par=f"sequence-sharded x{world} ({b} sequences per rank)",
                    metric="prefill tokens/s (GDN box-scale sharded prefill, BASELINE config 4)",
                    desc="config4: 64 x 4096 tokens, H=16 HV=32 K=V=128 bf16, in-kernel q/k L2 norm")
    if name == "cfg2":
        import numpy as np
        lens = np.random.default_rng(2).integers(512, 8193, size=16).tolist()
        parts = shard.partition_sequences(lens, world)
        mine = parts[rank]
        cu = [0]
        for i in mine:
            cu.append(cu[-1] + lens[i])
        return dict(B=1, T=cu[-1], cu=cu, nseq=16, tokens=int(sum(lens)), seed=2, h0=True,
                    lens=lens, parts=parts,
                    scaling="strong", par=f"sequences bin-packed over {world} ranks",
                    metric="prefill tokens/s (GDN varlen packed prefill, BASELINE config 2)",
                    desc=f"config2: 16 sequences U[512,8192] ({sum(lens)} tokens) packed via cu_seqlens, "
                         "h0 N(0,0.02), H=16 HV=32 K=V=128 bf16")
    raise SystemExit(f"unknown workload {name}")


def _chunk_with_events(ops, q, k, v, g, beta, handles, nst, cu=None, h0=None):
    """One chunk_gated_delta_rule call with the library's stage events set."""
    import ctypes

    import torch

    from domesticated_torch_mlu_ops_b200 import _lib, gdn
    B, T, H, K = k.shape
    HV, V = v.shape[2], v.shape[3]
    N = B if cu is None else cu.numel() - 1
    o = torch.empty_like(v)
    ht = torch.empty(N, HV, K, V, dtype=torch.float32, device=q.device)
    args = _lib.ChunkArgs(
        q=gdn._ptr(q), k=gdn._ptr(k), v=gdn._ptr(v), g=gdn._ptr(g), beta=gdn._ptr(beta),
        initial_state=gdn._ptr(h0), o=gdn._ptr(o), final_state=gdn._ptr(ht), cu_seqlens=gdn._ptr(cu),
        B=B, T=T, N=N, H=H, HV=HV, K=K, V=V, qkv_dtype=_lib.GDN_BF16, cu_dtype=_lib.GDN_I64,
        scale=0.0, use_qk_l2norm=1, state_v_first=0, force_generic=0,
        stage_events=ctypes.cast(handles, ctypes.POINTER(ctypes.c_void_p)), n_stage_events=nst)
    lib = _lib.load()
    nbytes = lib.gdn_chunk_workspace_size(ctypes.byref(args))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
    args.workspace = ctypes.c_void_p(ws.data_ptr())
    args.workspace_bytes = nbytes
    n0 = lib.gdn_kernel_launch_count()
    _lib.check(lib.gdn_chunk_fwd(ctypes.byref(args), gdn._stream(q.device)))
    n = lib.gdn_kernel_launch_count() - n0
    return o, ht, {"stages": _stage_names(n)}


def _stage_names(n):
    # launch order of the chunk paths (launchers in domesticated_torch_mlu_ops_b200/csrc/);
    # the "plan" stage is a chunk-table kernel, or only an event when sequences of
    # equal length need no table
    if n == 6:  # generic fp32 path
        return ["plan", "prep:q", "prep:k", "wy", "state", "out"]
    if n == 3:  # tcgen05 path, chunk table, separate WY and state kernels
        return ["plan", "wy", "state"]
    if n == 2 and os.environ.get("GDN_TC_FUSED", "0").startswith("1"):  # fused cluster kernel
        return ["plan", "fused"]
    if n == 2:  # tcgen05 path without a chunk table
        return ["plan", "wy", "state"]
    return [f"k{i}" for i in range(n)]


def _decode_bench(ops, dev, a, hbm, flush, peak_kind="measured"):
    import torch
    c = CFG3
    N, S, H, HV, K, V = c["N"], c["slots"], c["H"], c["HV"], c["K"], c["V"]
    gen = torch.Generator().manual_seed(3)
    q = torch.randn(1, N, H, K, generator=gen).bfloat16().to(dev)
    k = torch.randn(1, N, H, K, generator=gen).bfloat16().to(dev)
    v = torch.randn(1, N, HV, V, generator=gen).bfloat16().to(dev)
    g = torch.nn.functional.logsigmoid(torch.randn(1, N, HV, generator=gen)).to(dev)
    beta = torch.sigmoid(torch.randn(1, N, HV, generator=gen)).to(dev)
    cache = (torch.randn(S, HV, V, K, generator=gen) * 0.02).to(dev)
    idx = torch.randperm(S, generator=gen)[:N].to(dev)
    cu = torch.arange(N + 1, device=dev)

    def step():
        ops.fused_recurrent_gated_delta_rule_fn(q, k, v, g, beta, K ** -0.5, cache, True, cu, idx,
                                                None, True)

    for _ in range(max(3, a.warmup)):
        step()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(max(a.steps, 10))]
    for s, e in ev:
        flush.zero_()
        s.record()
        step()
        e.record()
    torch.cuda.synchronize()
    us = sum(s.elapsed_time(e) for s, e in ev) / len(ev) * 1e3
    nbytes = N * (2 * HV * K * V * 4 + 2 * H * K * 2 + 2 * HV * V * 2 + 2 * HV * 4 + 8)
    gbs = nbytes / (us * 1e-6) / 1e9
    return {"workload": "config3: 256 sequences x 1 token, cache [1024,32,128,128] f32",
            "us_per_step": us, "algorithmic_bytes": nbytes, "achieved_gbs": gbs,
            "peak_gbs": hbm, "frac_hbm": gbs / hbm, "peak_kind": f"{peak_kind} HBM copy",
            "kernel": "decode_stream_kernel", "traffic": _load_traffic().get("decode")}


def _conv_bench(ops, dev, a, hbm, flush, peak_kind="measured"):
    """The causal conv1d in front of the GDN layer at the config-1 prefill
    shape (q/k/v conv channels 2*16*128 + 32*128 = 8192, 8192 tokens,
    width 4, SiLU, bf16, vLLM layout with a slot cache) and one decode
    update for the config-3 batch (256 sequences)."""
    import torch
    D, T, W, N = 8192, CFG1["T"], 4, CFG3["N"]
    gen = torch.Generator().manual_seed(4)
    x = torch.randn(T, D, generator=gen).bfloat16().to(dev)
    w = (torch.randn(D, W, generator=gen) * 0.3).bfloat16().to(dev)
    b = torch.randn(D, generator=gen).bfloat16().to(dev)
    cs = torch.zeros(2, W - 1, D, dtype=torch.bfloat16, device=dev).transpose(1, 2)
    qsl = torch.tensor([0, T], dtype=torch.int32, device=dev)
    ci = torch.tensor([1], dtype=torch.int32, device=dev)
    hi = torch.tensor([True], device=dev)
    xu = torch.randn(N, D, generator=gen).bfloat16().to(dev)
    cache = torch.randn(N, D, W, generator=gen).bfloat16().to(dev)

    def timed(fn, reps):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
        for st, en in ev:
            flush.zero_()
            st.record()
            fn()
            en.record()
        torch.cuda.synchronize()
        return sum(st.elapsed_time(en) for st, en in ev) / reps * 1e3

    us_fn = timed(lambda: ops.causal_conv1d_fn(x.t(), w, b, cs, qsl, ci, hi, "silu"), max(a.steps, 10))
    # the conv and the chunked prefill of one GDN layer (config 1), as two ops
    # (the prefill reads q/k/v in place from the conv output) and fused
    H, HV = CFG1["H"], CFG1["HV"]
    g = torch.nn.functional.logsigmoid(torch.randn(1, T, HV, generator=gen)).to(dev)
    beta = torch.sigmoid(torch.randn(1, T, HV, generator=gen)).to(dev)
    h0 = (torch.randn(1, HV, 128, 128, generator=gen) * 0.02).to(dev)

    def two_ops():
        yt = ops.causal_conv1d_fn(x.t(), w, b, cs, qsl, ci, hi, "silu").t()
        q = yt[:, :H * 128].view(1, T, H, 128)
        k = yt[:, H * 128:2 * H * 128].view(1, T, H, 128)
        v = yt[:, 2 * H * 128:].view(1, T, HV, 128)
        return ops.chunk_gated_delta_rule(q, k, v, g, beta, None, h0, True, cu_seqlens=qsl,
                                          use_qk_l2norm_in_kernel=True)

    def fused():
        return ops.causal_conv1d_chunk_gated_delta_rule(x.t(), w, b, cs, qsl, g, beta, H, HV, initial_state=h0,
                                                        output_final_state=True, cache_indices=ci,
                                                        has_initial_state=hi, use_qk_l2norm_in_kernel=True)
    us_two = timed(two_ops, max(a.steps, 10))
    us_fused = timed(fused, max(a.steps, 10))
    us_up = timed(lambda: ops.causal_conv1d_update(xu, cache, None, w, b, "silu"), max(a.steps, 10))
    b_fn = 2 * T * D * 2 + D * W * 2 + D * 2 + 2 * D * (W - 1) * 2
    b_up = N * D * (2 + 2 * W * 2 + 2) + D * W * 2 + D * 2
    return {
        "prefill": {"workload": "causal_conv1d_fn: dim 8192 x 8192 tokens, width 4, SiLU, bf16, slot cache",
                    "us_per_call": us_fn, "algorithmic_bytes": b_fn,
                    "achieved_gbs": b_fn / (us_fn * 1e-6) / 1e9, "frac_hbm": b_fn / (us_fn * 1e-6) / 1e9 / hbm,
                    "kernels": "conv_fwd_kernel + conv_state_kernel"},
        "update": {"workload": "causal_conv1d_update: 256 sequences x 8192 channels, width 4, bf16 cache",
                   "us_per_call": us_up, "algorithmic_bytes": b_up,
                   "achieved_gbs": b_up / (us_up * 1e-6) / 1e9, "frac_hbm": b_up / (us_up * 1e-6) / 1e9 / hbm,
                   "kernels": "conv_update_kernel"},
        "layer_prefill": {"workload": "causal_conv1d_fn + chunk_gated_delta_rule of one GDN layer, config 1 "
                                      "(8192 tokens, 16/32 heads, d=128, bf16, in-kernel L2 norm)",
                          "us_two_ops": us_two, "us_fused": us_fused,
                          "kernels_two_ops": "conv_fwd_kernel + conv_state_kernel + chunk_plan_kernel + "
                                             "tc_wy_kernel + tc_state3_kernel",
                          "kernels_fused": "chunk_plan_kernel + tc_wy_kernel (conv applied to its tiles) + "
                                           "tc_state3_kernel + conv_state_kernel",
                          # conv reads x and writes y, the prefill reads y; fused: x read
                          # once, post-conv q/k written once for the state kernel
                          "hbm_bytes_saved": 2 * (2 * T * D) - 2 * T * 2 * H * 128},
        "peak_gbs": hbm, "peak_kind": f"{peak_kind} HBM copy"}




def bwd_flops_per_chunk_head(K, V):
    """Matmul FLOPs of one (64-token chunk, v-head) of the backward, forward
    recompute included: the products that gdn_chunk_bwd.cu and the generic
    forward's W/U/state kernels compute (2 FLOPs per multiply-add)."""
    aK, aV, b, c = 64 * 64 * K, 64 * 64 * V, 64 * K * V, 64 ** 3
    fwd = 2 * aK + aV + 2 * b                       # K K^T, W, U, W h, K^T v_new
    dvl = aK + aV                                   # Q K^T, P^T dO
    state = 3 * b                                   # K dh', [Q; W]^T [dO; dv]
    dqkw = aV + 3 * b + 2 * aK                      # dO v^T, v dh'^T, dO h^T, dv h^T, dP K, dP^T Q
    wy = 4 * aK + 2 * aV + 2 * c + 2 * aK           # K K^T, dW K^T, dv V^T, T^T dW, T^T dv, dA, dS K, dS^T K
    return 2 * (fwd + dvl + state + dqkw + wy)


def _bwd_bench(ops, dev, a, flush, tc_burst, peak_kind="measured"):
    """Backward (training) of the config-1 prefill shape: gdn_chunk_bwd with
    dO given and no final-state gradient, q/k L2 norm on."""
    import torch
    B, T, H, HV, K, V = (CFG1[x] for x in ("B", "T", "H", "HV", "K", "V"))
    gen = torch.Generator().manual_seed(5)
    q = torch.randn(B, T, H, K, generator=gen).bfloat16().to(dev)
    k = torch.randn(B, T, H, K, generator=gen).bfloat16().to(dev)
    v = torch.randn(B, T, HV, V, generator=gen).bfloat16().to(dev)
    g = torch.nn.functional.logsigmoid(torch.randn(B, T, HV, generator=gen)).to(dev)
    beta = torch.sigmoid(torch.randn(B, T, HV, generator=gen)).to(dev)
    do = torch.randn(B, T, HV, V, generator=gen).bfloat16().to(dev)

    def call():
        return ops.chunk_gated_delta_rule_bwd(q, k, v, g, beta, None, None, do, None,
                                              use_qk_l2norm_in_kernel=True)

    for _ in range(2):
        call()
    torch.cuda.synchronize()
    reps = max(3, min(a.steps, 5))
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    for st, en in ev:
        flush.zero_()
        st.record()
        call()
        en.record()
    torch.cuda.synchronize()
    ms = sum(st.elapsed_time(en) for st, en in ev) / reps
    flops = (T // 64) * B * HV * bwd_flops_per_chunk_head(K, V)
    tf = flops / (ms * 1e-3) / 1e12
    return {"workload": "chunk_gated_delta_rule backward, config-1 shape (B=1 T=8192 H=16 HV=32 K=V=128 "
                        "bf16, q/k L2 norm, dO given, no final-state gradient), forward recompute included",
            "ms_per_call": ms, "tokens_per_s": B * T / (ms * 1e-3), "flops": flops, "tflops": tf,
            "frac_tensor_bf16_measured": tf / tc_burst, "peak_kind": f"{peak_kind} bf16 burst",
            "kernels": "chunk_plan_kernel + tcgen05 recompute (tc_wy_kernel, tc_state3_kernel storing h and "
                       "v_new images) + tcgen05 tc_bwd_dvlocal, tc_bwd_state, tc_bwd_dqkw, tc_bwd_wy + "
                       "bwd_qk (v-head sums, L2-norm backward), bwd_dg"}


def run_reference(a):
    """CPU restatement of the reference algorithm (the oracle port), timed on
    the host's cores on a bounded sample of the config-1 workload."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg = dict(CFG1)
    cpu = CpuBaseline(cfg, sample_tokens=a.ref_tokens)
    for _ in range(max(1, min(a.warmup, 2))):
        cpu.step()
    t = [cpu.step() for _ in range(a.steps)]
    cpu.close()
    sec = sum(t) / len(t)
    value = cpu.tokens / sec
    line = {
        "impl": "reference",
        "metric": "prefill tokens/s (Qwen3-Next GDN layer chunked prefill, BASELINE config 1)",
        "value": value, "unit": "tokens/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config1: chunk_gated_delta_rule B=1 T=8192 H=16 HV=32 K=V=128, "
                   f"timed on a {cpu.tokens}-token sample per step"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cpu.cores, "kind": "port",
                         "sample": f"{cpu.tokens} tokens of config 1 per step, numpy fp32 chunked "
                                   f"restatement of the reference's six stages, {cpu.workers} worker "
                                   f"processes x {cpu.blas_threads} BLAS threads; host {_cpu_model()}"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-decode", action="store_true", help="skip the decode and conv1d measurements")
    ap.add_argument("--no-bwd", action="store_true", help="skip the backward measurement")
    ap.add_argument("--ref-tokens", type=int, default=CPU_SAMPLE_TOKENS)
    ap.add_argument("--tokens", type=int, default=0,
                    help="override config 1's T (small cases for ncu captures; not a bench line)")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg")
    ap.add_argument("--no-subs", action="store_true",
                    help="skip the config-4 and head-split sub-workloads of the config-1 line")
    ap.add_argument("--segment-tokens", dest="segment_tokens", type=int, default=4096,
                    help="tokens per piece of the host-streamed end-to-end leg (multiple of 64)")
    ap.add_argument("--workload", default="cfg1", choices=["cfg1", "cfg2", "cfg4"],
                    help="BASELINE prefill config (default cfg1, the headline)")
    a = ap.parse_args()
    a.warmup = max(a.warmup, 3)
    if a.impl == "reference":
        run_reference(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
