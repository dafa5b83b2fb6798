#!/usr/bin/env python
"""Prefill MUL_MAT throughput of the ggml B200 backend (the headline of BASELINE.json).

Workload (one "step"): the quantized prefill GEMM sweep's three (K, N) weight shapes,
(4096, 4096), (4096, 14336) and (14336, 4096), in Q4_K, each multiplied by a 512-token F32
activation ubatch, through --layers (default 32, a Llama-3-8B's depth) layers: distinct device
copies of the weights, as a model's layers are. Weights are N(0, 0.02) quantized to Q4_K on the host, activations
N(0, 1), seeded; all synthetic.

  value     TFLOP/s of the step on the device, inputs resident in HBM, L2 flushed (a 256 MiB
            memset) before every timed step, device time from CUDA events.
  e2e       the same metric through the plugin call a ggml host makes: graph_compute on a graph
            of the three MUL_MAT nodes with host-buffer tensors (activations and dst in the
            backend's pinned host buffers), copies in and out inside every call.
  roofline  the tcgen05 GEMM kernel alone (its CUDA-event time per launch) against the
            measured bf16/fp16 dense peak.
  check     a sample of the timed kernels' and the plugin path's outputs against the fp64 oracle.

--gpus N (under torchrun): every rank runs its own ubatch against its own copy of the
weights (replicas; weak scaling); the timed region is bracketed by barriers and the max over
ranks is reported.

--impl reference: the CPU restatement of the reference's MUL_MAT (the oracle, fp64 over the
ggml-decoded weight, rocket_cpu_matmul_slice) on all host cores, on a bounded token sample of
the same workload per step.
"""
import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "ggml-rocket_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "prefill GEMM TFLOP/s (F16/Q4_K) and prompt tokens/sec at 512-token ubatch"
SHAPES = [(4096, 4096), (4096, 14336), (14336, 4096)]   # (K, N)
M_TOKENS = 512
WTYPE = 12   # Q4_K
WORKLOAD = ("Q4_K MUL_MAT sweep (BASELINE configs[1]) at M=512: (K,N) in {(4096,4096),(4096,14336),"
            "(14336,4096)}, one op per shape per step")
CPU_SAMPLE_ROWS = 64


def step_flops(m=M_TOKENS):
    return sum(2.0 * m * n * k for (k, n) in SHAPES)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["gemm", "gemv", "moe", "fa", "glue", "layer", "crossover"], default="gemm",
                    help="gemm: the headline MUL_MAT sweep (default); gemv: the sweep's weights at decode "
                         "size (M = --decode-m, --decode-type, b200_mul_mat_vec); moe: the MUL_MAT_ID layer of "
                         "BASELINE configs[3], expert-parallel over the ranks; fa: the FLASH_ATTN_EXT "
                         "prefill of configs[2]; glue: a layer's glue ops and the MoE router at the "
                         "headline's prefill shapes (HBM-bound kernels, GB/s); layer: configs[4]'s Llama-3-8B "
                         "layer through graph_compute, prompt tokens/s; crossover: the M at which a claimed "
                         "MUL_MAT with host tensors beats the host CPU")
    ap.add_argument("--layers", type=int, default=32,
                    help="gemm workload: layers (distinct weight copies) the sweep runs through per step")
    ap.add_argument("--decode-type", choices=["q4_k", "q6_k", "q8_0"], default="q4_k",
                    help="gemv workload: weight type")
    ap.add_argument("--decode-m", type=int, default=1,
                    help="gemv workload: token rows per step (1..32)")
    ap.add_argument("--shard", action="store_true",
                    help="gemm workload on several GPUs: split every weight's rows across the ranks "
                         "(strong scaling), the output all-gathered by the GEMM epilogue's stores into "
                         "peer memory, instead of one replica per rank")
    ap.add_argument("--ep", choices=["peer", "nccl"], default="peer",
                    help="moe workload on several GPUs: exchanges by the kernels' own stores into peer "
                         "memory (default) or by NCCL all-to-all")
    return ap.parse_args()


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def profile_traffic():
    """Per-launch DRAM bytes of the GEMM kernel from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", "gemm_q4k_m512_traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get("traffic_bytes_per_launch")
    except Exception:
        return None


class ClockSampler:
    """SM clocks and throttle reasons sampled during the timed region: NVML queries (read-only) from
    a background thread every few milliseconds, so even a timed region of tens of milliseconds
    gets samples; nvidia-smi -lms is the fallback when NVML cannot be loaded."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4}

    def __init__(self, gpu_index, period_s=0.005):
        self.gpu = gpu_index
        self.period = period_s
        self.samples = []
        self.thread = None
        self.stop_flag = False
        self.proc = None
        self.out = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(gpu_index)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM))
        except Exception:
            self.nvml = None

    def _loop(self):
        n = self.nvml
        while not self.stop_flag:
            try:
                mhz = float(n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM))
                get = getattr(n, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                    n.nvmlDeviceGetCurrentClocksThrottleReasons
                mask = int(get(self.handle))
                self.samples.append((mhz, mask))
            except Exception:
                pass
            time.sleep(self.period)

    def start(self):
        if self.nvml is not None:
            import threading
            self.thread = threading.Thread(target=self._loop, daemon=True)
            self.thread.start()
            return
        try:
            self.out = tempfile.NamedTemporaryFile(mode="w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), "--query-gpu=clocks.sm,clocks.max.sm,"
                                          "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                                          "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.out, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        sm, smax, reasons = [], 0.0, set()
        if self.thread is not None:
            self.stop_flag = True
            self.thread.join(timeout=5)
            smax = self.max_mhz
            for mhz, mask in self.samples:
                sm.append(mhz)
                for name, bit in self.REASONS.items():
                    if mask & bit:
                        reasons.add(name)
            source = "nvml"
        elif self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.out.flush()
            self.out.seek(0)
            rows = [r.strip().split(",") for r in self.out.read().strip().splitlines() if r.strip()]
            os.unlink(self.out.name)
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for r in rows:
                try:
                    sm.append(float(r[0]))
                    smax = max(smax, float(r[1]))
                    for i, nm in enumerate(names):
                        if r[2 + i].strip().lower() == "active":
                            reasons.add(nm)
                except Exception:
                    continue
            source = "nvidia-smi"
        else:
            return None
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm), "source": source}


# ------------------------------------------------------------------------------------------------
# reference arm: the CPU restatement timed on the host
# ------------------------------------------------------------------------------------------------

def make_host_inputs(seed, m_rows):
    import numpy as np
    from ggml_b200 import quants
    rng = np.random.default_rng(seed)
    ws, acts = [], []
    for (k, n) in SHAPES:
        w = (rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02))
        ws.append(quants.quantize(WTYPE, w))
        acts.append(rng.standard_normal((m_rows, k), dtype=np.float32))
    return ws, acts


def cpu_oracle_step(ws, acts):
    import oracle
    for (k, n), w, a in zip(SHAPES, ws, acts):
        oracle.mul_mat(WTYPE, w, n, k, a, nthreads=0)


def cpu_path_step(ws, acts):
    import oracle
    for (k, n), w, a in zip(SHAPES, ws, acts):
        oracle.cpu_path_mul_mat_q4k(w, n, k, a, nthreads=0)


def run_reference(args):
    ws_, rank, _ = dist_env()
    if rank != 0:
        return 0
    import oracle
    oracle.build()
    ws, acts = make_host_inputs(0xB200, CPU_SAMPLE_ROWS)
    tw = time.perf_counter()
    for _ in range(args.warmup):
        cpu_oracle_step(ws, acts)
    t_step = (time.perf_counter() - tw) / max(args.warmup, 1)
    # a CPU step takes ~0.3 s: time as many of the requested steps as fit in ~30 s
    steps = max(1, min(args.steps, int(30.0 / max(t_step, 1e-3))))
    t0 = time.perf_counter()
    for _ in range(steps):
        cpu_oracle_step(ws, acts)
    dt = (time.perf_counter() - t0) / steps
    val = step_flops(CPU_SAMPLE_ROWS) / dt / 1e12
    cores = os.cpu_count()
    line = {
        "impl": "reference", "metric": METRIC, "value": val, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": steps, "steps_requested": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
        "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": WORKLOAD, "sample": f"{CPU_SAMPLE_ROWS} of the 512 tokens per step",
                   "global_batch": M_TOKENS, "parallelism": "host threads"},
        "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": cores, "kind": "port",
                         "sample": f"{CPU_SAMPLE_ROWS} token rows x 3 shapes per step, {steps} steps "
                                   f"(the requested steps that fit in ~30 s)"},
        "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------------------------
# our arm
# ------------------------------------------------------------------------------------------------

def _pinned_array(g, nbytes, dtype, shape):
    """A numpy view of pinned host memory from the backend's host buffer type (the memory a ggml
    host gets for its CPU-side tensors when it uses this backend's host buffer type)."""
    import ctypes
    import numpy as np
    ptr = g.lib().ggml_backend_b200_host_alloc(nbytes)
    if not ptr:
        raise SystemExit("ggml_backend_b200_host_alloc failed")
    buf = (ctypes.c_uint8 * nbytes).from_address(ptr)
    return np.frombuffer(buf, dtype=dtype, count=int(np.prod(shape))).reshape(shape), ptr


def check_sample(ws_host, acts_host, outs_np, rows=16):
    """max |err| / max |ref| of a seeded sample of output rows against the fp64 oracle."""
    import numpy as np
    import oracle
    oracle.build()
    worst = 0.0
    rng = np.random.default_rng(7)
    for (k, n), w, a, o in zip(SHAPES, ws_host, acts_host, outs_np):
        sel = np.unique(np.concatenate([[0, a.shape[0] - 1], rng.choice(a.shape[0], rows - 2, replace=False)]))
        ref = oracle.mul_mat(WTYPE, w, n, k, np.ascontiguousarray(a[sel]))
        worst = max(worst, float(np.max(np.abs(o[sel] - ref)) / np.max(np.abs(ref))))
    return worst


def run_e2e_plugin(args, g, ws_host, acts_host, pinned):
    """The headline step through the plugin surface a ggml host calls: one graph of the sweep's three
    MUL_MAT nodes with host-buffer tensors, computed by ggml_backend_b200_graph_compute. Weights are
    pageable host tensors (packed into the backend's device cache on first use, keyed by name and
    content); activations and outputs are in pinned host memory (pinned=True, the backend's host
    buffer type) or in pageable memory. Every call copies the activations in and the outputs out
    inside the call. Returns (seconds per call, h2d bytes, d2h bytes, outputs)."""
    import numpy as np
    be = g.Backend()
    keep, nodes, outs, pins = [], [], [], []
    h2d = d2h = 0
    for i, ((k, n), w, a) in enumerate(zip(SHAPES, ws_host, acts_host)):
        if pinned:
            a_h, a_ptr = _pinned_array(g, a.nbytes, np.float32, a.shape)
            o_h, o_ptr = _pinned_array(g, M_TOKENS * n * 4, np.float32, (M_TOKENS, n))
            pins += [a_ptr, o_ptr]
        else:
            a_h = np.empty_like(a)
            o_h = np.empty((M_TOKENS, n), np.float32)
            a_ptr, o_ptr = a_h.ctypes.data, o_h.ctypes.data
        a_h[:] = a
        wt = g.make_tensor(WTYPE, [k, n], data=w, name=f"blk.0.sweep{i}.weight")
        at = g.make_tensor(g.F32, [k, M_TOKENS], data=a_ptr, name=f"sweep{i}_in")
        dt = g.make_tensor(g.F32, [n, M_TOKENS], data=o_ptr, op=g.OP_MUL_MAT, srcs=[wt, at], name=f"sweep{i}_out")
        keep += [wt, at, dt, a_h, o_h]
        nodes.append(dt)
        outs.append(o_h)
        h2d += a.nbytes
        d2h += o_h.nbytes
    for _ in range(max(3, args.warmup)):
        if be.graph_compute(nodes) != g.STATUS_SUCCESS:
            raise SystemExit("graph_compute failed")
    t0 = time.perf_counter()
    for _ in range(args.steps):
        if be.graph_compute(nodes) != g.STATUS_SUCCESS:
            raise SystemExit("graph_compute failed")
    dt_call = (time.perf_counter() - t0) / args.steps
    res = [o.copy() for o in outs]
    if be.cpu_fallbacks() != 0:
        raise SystemExit("the plugin computed a claimed op on the CPU")
    be.close()
    del keep, outs
    for ptr in pins:
        g.lib().ggml_backend_b200_host_free(ptr)
    return dt_call, h2d, d2h, res


def run_ours(args):
    import numpy as np
    import torch
    import ggml_b200 as g

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    g.lib()
    L = args.layers

    ws_host, acts_host = make_host_inputs(0xB200 + rank, M_TOKENS)
    stream = torch.cuda.current_stream()
    # One N(0, 0.02) Q4_K weight per shape, packed once and copied into L distinct device buffers
    # (the layers of a model): a step runs the sweep through all L, and no layer's weights are still
    # in L2 when it runs (L x 75.5 MB of packed weights).
    base = []
    for (k, n), w in zip(SHAPES, ws_host):
        raw = torch.from_numpy(w.reshape(-1)).to(dev)
        packed = torch.empty(g.weight_packed_size(WTYPE, n, k), dtype=torch.uint8, device=dev)
        g.weight_pack(WTYPE, raw, n, k, packed)
        base.append(packed)
        del raw
    weights = [[base[i] if l == 0 else base[i].clone() for i in range(len(SHAPES))] for l in range(L)]
    acts, a16s, scales, outs, gws = [], [], [], [], []
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    for (k, n), a in zip(SHAPES, acts_host):
        acts.append(torch.from_numpy(a).to(dev))
        a16s.append(torch.empty((M_TOKENS, k), dtype=torch.float16, device=dev))
        scales.append(torch.empty(M_TOKENS, dtype=torch.float32, device=dev))
        outs.append(torch.empty((M_TOKENS, n), dtype=torch.float32, device=dev))
        wsz = g.gemm_packed_workspace_size(M_TOKENS, n, k, WTYPE)
        gws.append(torch.empty(max(wsz, 256), dtype=torch.uint8, device=dev))
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    launches_per_step = L * sum(g.mul_mat_plan(M_TOKENS, n, k, WTYPE)["launches"] for (k, n) in SHAPES)

    def step(ev=None):
        # ev (the kernel-timing pass only): an event pair around every GEMM launch. The timed pass
        # records no event between the kernels, so each launch may begin (programmatic dependent
        # launch) while the one before it drains.
        for l in range(L):
            for i, (k, n) in enumerate(SHAPES):
                g.act_pack(acts[i], M_TOKENS, k, a16s[i], scales[i], stream=stream)
                if ev:
                    ev[l][i][0].record(stream)
                g.gemm_packed(WTYPE, weights[l][i], n, k, a16s[i], scales[i], M_TOKENS, outs[i], gws[i], err,
                              stream=stream)
                if ev:
                    ev[l][i][1].record(stream)

    def ev_pair():
        return (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))

    # A GPU-side delay after each flush lets the host enqueue the whole step before the device
    # reaches it, so the events bracket device work only (no host launch gaps).
    slack_cycles = 2000000 * L
    for _ in range(max(3, args.warmup)):
        flush.zero_()
        torch.cuda._sleep(slack_cycles)
        step()
    torch.cuda.synchronize()
    if int(err.item()) != 0:
        raise SystemExit(f"device error {int(err.item())} during warm-up")

    sampler = ClockSampler(local) if rank == 0 else None
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    evs = []
    for si in range(args.steps):
        flush.zero_()
        torch.cuda._sleep(slack_cycles)
        e = ev_pair()
        e[0].record(stream)
        step()
        e[1].record(stream)
        evs.append(e)
        if si == 0 and sampler:
            sampler.start()
    torch.cuda.synchronize()
    clocks = sampler.stop() if sampler else None
    if world > 1:
        torch.distributed.barrier()
    if int(err.item()) != 0:
        raise SystemExit(f"device error {int(err.item())} in the timed region")
    step_ms = [e[0].elapsed_time(e[1]) for e in evs]
    outs_np = [o.cpu().numpy() for o in outs]

    # The roofline's kernel time: the same steps again with an event pair around every GEMM launch
    # (on its stream); per shape, the mean over layers and steps.
    kevs = []
    for _ in range(max(2, min(args.steps, 10))):
        flush.zero_()
        torch.cuda._sleep(slack_cycles)
        e = [[ev_pair() for _ in SHAPES] for _ in range(L)]
        step(e)
        kevs.append(e)
    torch.cuda.synchronize()
    per_shape_ms = [statistics.mean(e[l][i][0].elapsed_time(e[l][i][1]) for e in kevs for l in range(L))
                    for i in range(len(SHAPES))]
    ms_local = sum(step_ms) / len(step_ms)
    gemm_local = sum(per_shape_ms)

    # configs[0] beside the headline: the F16 MUL_MAT N = K = 4096, M = 512 (one launch, L2 flushed)
    f16_us = None
    if rank == 0:
        k0 = n0 = 4096
        w16 = (np.random.default_rng(0xB200).standard_normal((n0, k0), dtype=np.float32) * np.float32(0.02))
        w16p = torch.from_numpy(w16.astype(np.float16).view(np.uint8).reshape(-1)).to(dev)
        a0 = torch.from_numpy(acts_host[0]).to(dev)
        o0 = torch.empty((M_TOKENS, n0), dtype=torch.float32, device=dev)
        ws0 = torch.empty(max(256, g.mul_mat_workspace_size(M_TOKENS, n0, k0, g.F16)), dtype=torch.uint8, device=dev)
        t16 = []
        for it in range(13):
            flush.zero_()
            torch.cuda._sleep(400000)
            e = ev_pair()
            e[0].record(stream)
            g.mul_mat(g.F16, w16p, n0, k0, a0, M_TOKENS, o0, ws0, err, stream=stream)
            e[1].record(stream)
            if it >= 3:
                t16.append(e)
        torch.cuda.synchronize()
        f16_us = statistics.median(e[0].elapsed_time(e[1]) for e in t16) * 1e3

    # ---- e2e: the plugin call a ggml host makes, with host buffers ----
    e2e_s, h2d, d2h, e2e_outs = run_e2e_plugin(args, g, ws_host, acts_host, pinned=True)
    e2e_pg_s = None
    if rank == 0:
        e2e_pg_s, _, _, _ = run_e2e_plugin(args, g, ws_host, acts_host, pinned=False)

    vals = torch.tensor([ms_local, gemm_local, e2e_s * 1e3], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(vals, op=torch.distributed.ReduceOp.MAX)
    ms, gms, e2e_ms = [float(x) for x in vals.tolist()]

    # On several GPUs, the two paths that really use them, beside the replicas: the configs[3] MoE layer
    # with its experts split over the ranks (exchanges by kernel stores into peer memory; weak scaling:
    # 2048 tokens per rank) and the headline sweep with every weight's rows split over the ranks (strong
    # scaling), each with its one-GPU reference measured in the same run on rank 0.
    multi = None
    if world > 1:
        del weights
        torch.cuda.empty_cache()
        moe_n = run_moe(args, inside=True)
        torch.distributed.barrier()
        moe_1 = run_moe(args, world_override=1, inside=True) if rank == 0 else None
        torch.distributed.barrier()
        shard_n = {m: run_gemm_sharded(args, inside=True, m_tokens=m) for m in (M_TOKENS, 2048)}
        torch.distributed.barrier()
        shard_1 = {m: time_sweep_1gpu(args, m) for m in (M_TOKENS, 2048)} if rank == 0 else None
        torch.distributed.barrier()
        if rank == 0:
            multi = {
                "moe_expert_parallel": {
                    "workload": "BASELINE configs[3] MoE layer (gate+up+down, Q4_K, 128 experts top-8), 2048 tokens "
                                f"per rank, experts split {MOE['E']}/{world} per rank, peer-memory exchanges",
                    "ms_per_layer": moe_n["ms"], "tokens_per_s": moe_n["tokens_per_s"], "tflops": moe_n["tflops"],
                    "ms_per_layer_1gpu": moe_1["ms"], "weak_efficiency": moe_1["ms"] / moe_n["ms"]},
                "sharded_sweep": {
                    f"m{m}": {
                        "workload": f"the sweep's three shapes (one layer) at M = {m} with every weight's rows split "
                                    "over the ranks, output all-gathered by the GEMM epilogue's peer stores; L2 "
                                    "flushed before every step",
                        "ms": shard_n[m]["ms"], "tflops": shard_n[m]["tflops"], "ms_1gpu": shard_1[m],
                        "ms_1gpu_what": "b200_mul_mat of the whole weights on rank 0's GPU, timed the same way",
                        "strong_speedup": shard_1[m] / shard_n[m]["ms"]} for m in (M_TOKENS, 2048)}}

    if rank == 0:
        peaks, peak_src = measured_peaks()
        flops = step_flops() * L
        value = flops * world / (ms / 1e3) / 1e12
        achieved = step_flops() / (gms / 1e3) / 1e12
        peak = float(peaks.get("bf16_tflops", 1590.0))
        # the outputs of the timed kernels and of the plugin path, sampled against the fp64 oracle
        err_dev = check_sample(ws_host, acts_host, outs_np)
        err_e2e = check_sample(ws_host, acts_host, e2e_outs)
        # the CPU baseline: the oracle on a bounded sample, this host's cores, median of 5
        import oracle
        oracle.build()
        ws_c, acts_c = make_host_inputs(0xB200, CPU_SAMPLE_ROWS)
        cpu_oracle_step(ws_c, acts_c)
        reps = []
        for _ in range(5):
            t0 = time.perf_counter()
            cpu_oracle_step(ws_c, acts_c)
            reps.append(time.perf_counter() - t0)
        cpu_dt = statistics.median(reps)
        f64_val = step_flops(CPU_SAMPLE_ROWS) / cpu_dt / 1e12
        # the host CPU's own quantized path (8-bit activation blocks, integer dots, AVX2), the
        # stand-in for ggml's CPU backend: the primary CPU baseline
        cpu_path_step(ws_c, acts_c)
        reps = []
        for _ in range(5):
            t0 = time.perf_counter()
            cpu_path_step(ws_c, acts_c)
            reps.append(time.perf_counter() - t0)
        cpu_val = step_flops(CPU_SAMPLE_ROWS) / statistics.median(reps) / 1e12
        plans = {f"{k}x{n}": g.mul_mat_plan(M_TOKENS, n, k, WTYPE) for (k, n) in SHAPES}
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16 (fp32 accumulate)", "data": "synthetic",
            "config": {"workload": WORKLOAD, "weight_type": "Q4_K", "global_batch": M_TOKENS * world,
                       "seq_len": M_TOKENS, "parallelism": f"replicas x{world}", "layers_per_step": L,
                       "weights": f"one N(0,0.02) Q4_K weight per shape, packed and copied into {L} distinct "
                                  f"device buffers (layers); a step runs the 3 ops through all {L} layers",
                       "l2": f"flushed before every timed step (256 MiB memset), outside the timed events; "
                             f"{L} layers x 75.5 MB of weights per step also exceed L2",
                       "gemm_tflops_per_shape": {f"{k}x{n}": 2.0 * M_TOKENS * n * k / (t / 1e3) / 1e12
                                                 for (k, n), t in zip(SHAPES, per_shape_ms)},
                       "plans": plans},
            "f16_config0": {"workload": "BASELINE configs[0]: F16 MUL_MAT N=K=4096, M=512, one launch, L2 flushed",
                            "us": f16_us, "tflops": 2.0 * M_TOKENS * 4096 * 4096 / (f16_us / 1e6) / 1e12
                            if f16_us else None},
            "check": {"max_rel_err_kernels": err_dev, "max_rel_err_plugin": err_e2e, "tolerance": 1e-2,
                      "ok": err_dev <= 1e-2 and err_e2e <= 1e-2,
                      "sample": "16 output rows per shape against the fp64 oracle, after the timed region"},
            "e2e": {"value": step_flops() * world / (e2e_ms / 1e3) / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms,
                    "path": "ggml_backend_b200_graph_compute on one graph of the 3 MUL_MAT nodes (one layer), "
                            "activations and dst in pinned host memory from the backend's host buffer type, "
                            "copied in and out inside every call on copy streams overlapped with the other "
                            "nodes' kernels; weights pageable host tensors cached on the device by name and "
                            "content; wall-clock time of the synchronous call",
                    "pageable_value": step_flops() / e2e_pg_s / 1e12 if e2e_pg_s else None},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": profile_traffic(),
                         "traffic_launch": "DRAM bytes of the (K=4096, N=14336) launch, one ncu capture "
                                           "(profiles/gemm_q4k_m512_cluster_split.md)",
                         "kernel": "gemm_kernel<BT,Q4_K> (tcgen05, fused Q4_K dequant)",
                         "peak_source": f"{peak_src} bf16_tflops (burst)",
                         "algorithmic": "2*M*N*K FLOP per launch; per shape the mean CUDA-event time of its "
                                        "launch over layers and steps, summed over the 3 shapes"},
            "cpu_baseline": {"value": cpu_val, "unit": "TFLOP/s", "cores": os.cpu_count(), "kind": "port",
                             "sample": f"{CPU_SAMPLE_ROWS} token rows x 3 shapes per rep, median of 5 reps (the "
                                       f"host CPU's quantized MUL_MAT path restated, oracle/cpu_path.c: activations "
                                       f"to 8-bit blocks of 256, integer Q4_K block dots, AVX2, OpenMP over all "
                                       f"cores -- the stand-in for ggml's CPU backend, which is not on the box)",
                             "fp64_oracle": {"value": f64_val, "unit": "TFLOP/s",
                                             "what": "the reference's rocket_cpu_matmul_slice restated (fp64 "
                                                     "accumulation over ggml-decoded weights), same sample"}},
            "clocks": clocks,
            "gpu_launches": launches_per_step * args.steps,
        }
        if multi:
            line["multi_gpu"] = multi
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


# ------------------------------------------------------------------------------------------------
# secondary workloads (not the headline): MoE layer and flash attention
# ------------------------------------------------------------------------------------------------

MOE = dict(E=128, top=8, hidden=2048, ffn=768, tokens=2048, wtype=12)


def moe_flops_per_rank():
    m = MOE
    return 3 * 2.0 * m["tokens"] * m["top"] * m["hidden"] * m["ffn"]


def run_moe(args, world_override=None, inside=False):
    """The MoE layer of configs[3]. inside: called from the headline arm of an N-GPU run (the process
    group exists; return the timing instead of printing a line); world_override=1: this rank alone runs
    the single-GPU layer (all experts), the N = 1 reference of the expert-parallel numbers."""
    import numpy as np
    import torch
    import ggml_b200 as g
    from ggml_b200 import quants
    world, rank, local = dist_env()
    if world_override is not None:
        world = world_override
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1 and not inside:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    g.lib()
    E, top, H, F, T, wt = (MOE[k] for k in ("E", "top", "hidden", "ffn", "tokens", "wtype"))
    e_loc = E // world
    rng = np.random.default_rng(0xB200)                 # the same expert stacks on every rank

    def stack(K, N):
        # 16 distinct quantized experts repeated to 128 (the host quantizer is the slow part;
        # the device work does not depend on the values)
        pool = 16
        w = (rng.standard_normal((pool * N, K), dtype=np.float32) * np.float32(0.02))
        nat = np.tile(quants.quantize(wt, w).reshape(pool, N, -1), (E // pool, 1, 1)).reshape(E * N, -1)
        rows = nat[rank * e_loc * N:(rank + 1) * e_loc * N] if world > 1 else nat
        raw = torch.from_numpy(np.ascontiguousarray(rows).reshape(-1)).to(dev)
        out = torch.empty(g.weight_packed_size(wt, rows.shape[0], K), dtype=torch.uint8, device=dev)
        g.weight_pack(wt, raw, rows.shape[0], K, out)
        return out

    w_gate, w_up, w_down = stack(H, F), stack(H, F), stack(F, H)
    rng = np.random.default_rng(0xB200 + 17 * rank)     # this rank's tokens
    x = torch.from_numpy(rng.standard_normal((T, 1, H), dtype=np.float32)).to(dev)
    h = torch.empty((T, top, F), dtype=torch.float32, device=dev)     # swiglu(gate, up)
    logits = torch.from_numpy(rng.standard_normal((T, E), dtype=np.float32))
    ids = torch.topk(torch.softmax(logits, -1), top, dim=-1).indices.to(torch.int32).to(dev)
    y_gate = torch.empty((T, top, F), device=dev)
    y_up = torch.empty((T, top, F), device=dev)
    y_down = torch.empty((T, top, H), device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    if world > 1 and args.ep == "nccl":
        from ggml_b200.ep import DeviceOps, ExpertParallelMulMatId
        ep = ExpertParallelMulMatId(ops=DeviceOps(err))

        def layer():
            ep(wt, w_gate, H, F, E, x, 1, ids, y_gate)
            ep(wt, w_up, H, F, E, x, 1, ids, y_up)
            g.check(g.swiglu(y_gate, y_up, h), "swiglu")
            ep(wt, w_down, F, H, E, h, top, ids, y_down)
    elif world > 1:
        from ggml_b200.ep import DeviceOps, PeerExpertParallelMulMatId
        ep = PeerExpertParallelMulMatId(T, top, H, H, ops=DeviceOps(err), n_members_max=1)

        def layer():
            # the expert FFN where the experts are: x is pushed once, gate, up, swiglu and down run
            # on the owner, and only the down projection's rows come back (the result is a view of
            # the exchange's return buffer, [T, top, H])
            ep.ffn(wt, w_gate, w_up, wt, w_down, H, F, E, x, ids)
    else:
        ws = torch.empty(max(g.mul_mat_id_workspace_size(H, F, E, top, T), g.mul_mat_id_workspace_size(F, H, E, top, T),
                             g.mul_mat_id_ffn_workspace_size(H, F, E, top, T)), dtype=torch.uint8, device=dev)

        def one(wst, K, N, b, ne11, y):
            rc = g.mul_mat_id(wt, wst, K, N, E, b, K * 4, ne11 * K * 4, ne11, ids, 4, top * 4, top, T, y, N * 4,
                              top * N * 4, ws, err)
            g.check(rc, "mul_mat_id")

        def layer_chain():
            # the ops one by one, as graph_compute runs them when the chain cannot fuse: gate and
            # up as one group (one route and gather-pack), SWIGLU, down
            rc = g.mul_mat_id_group(wt, [w_gate, w_up], [F, F], H, E, x, H * 4, H * 4, 1, ids, 4, top * 4, top, T,
                                    [y_gate, y_up], [F * 4, F * 4], [top * F * 4, top * F * 4], ws, err)
            g.check(rc, "mul_mat_id_group")
            g.check(g.swiglu(y_gate, y_up, h), "swiglu")
            one(w_down, F, H, h, top, y_down)

        def layer():
            # the fused expert FFN graph_compute forms from the four nodes: one route for the
            # three projections, SWIGLU fused into the down projection's packing
            g.check(g.mul_mat_id_ffn(wt, w_gate, w_up, wt, w_down, H, F, E, x, H * 4, H * 4, 1, ids, 4, top * 4, top,
                                     T, y_down, H * 4, top * H * 4, ws, err), "mul_mat_id_ffn")

    stream = torch.cuda.current_stream()

    def timed(fn):
        for _ in range(args.warmup):
            flush.zero_()
            fn()
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        times = []
        for _ in range(args.steps):
            flush.zero_()
            torch.cuda._sleep(400000)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
        if int(err.item()) != 0:
            raise SystemExit(f"device error {int(err.item())}")
        return sorted(times)[len(times) // 2]

    ms_local = timed(layer)
    chain_ms = timed(layer_chain) if world == 1 and not inside else None
    t = torch.tensor([ms_local], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = float(t.item())
    if inside:
        return {"ms": ms, "tokens_per_s": T * world / (ms / 1e3),
                "tflops": moe_flops_per_rank() * world / (ms / 1e3) / 1e12}
    if rank == 0:
        peaks, src = measured_peaks()
        tf = moe_flops_per_rank() * world / (ms / 1e3) / 1e12
        line = {"metric": "MoE MUL_MAT_ID layer prompt tokens/sec (expert FFN: gate+up, swiglu, down; Q4_K, 128 experts top-8)",
                "value": T * world / (ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f16 (fp32 accumulate)", "data": "synthetic",
                "config": {"workload": "BASELINE configs[3] MoE layer, 2048 tokens per rank, experts split "
                                       f"{E}/{world} per rank" +
                                       ((" (NCCL all-to-all)" if args.ep == "nccl" else
                                         " (exchanges by kernel stores into NVLink peer memory)") if world > 1 else ""),
                           "weights": "16 distinct N(0,0.02) Q4_K experts per stack, repeated to 128",
                           "median_of_steps": True},
                "tflops": tf,
                "op_chain_ms_per_layer": chain_ms,
                "roofline": {"bound": "tensor", "achieved": tf / world, "peak": float(peaks["bf16_tflops"]),
                             "unit": "TFLOP/s", "frac": tf / world / float(peaks["bf16_tflops"]),
                             "peak_source": f"{src} bf16_tflops (burst)"}}
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


def run_fa(args):
    import numpy as np
    import torch
    import ggml_b200 as g
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    g.lib()
    D, T, Hq, HK = 128, 512, 32, 8
    res = {}
    for KV in (1024, 4096, 16384):
        gen = torch.Generator(device="cpu").manual_seed(KV)
        q = torch.randn((Hq, T, D), generator=gen).to(dev)
        k = torch.randn((HK, KV, D), generator=gen).to(torch.float16).to(dev)
        v = torch.randn((HK, KV, D), generator=gen).to(torch.float16).to(dev)
        pos = torch.arange(KV - T, KV).view(T, 1)
        m = torch.where(torch.arange(KV).view(1, KV) <= pos, 0.0, float("-inf")).to(torch.float16).to(dev)
        dst = torch.empty((T, Hq, D), device=dev)
        ws = torch.empty(g.flash_attn_workspace_size(D, D, T, Hq, KV, HK), dtype=torch.uint8, device=dev)
        err = torch.zeros(1, dtype=torch.int32, device=dev)

        def call():
            g.flash_attn_ext(q, D * 4, T * D * 4, k, D * 2, KV * D * 2, v, D * 2, KV * D * 2, m, KV * 2, dst, D, D,
                             T, Hq, KV, HK, 1.0 / np.sqrt(D), 0.0, ws, err)

        for _ in range(args.warmup):
            call()
        torch.cuda.synchronize()
        ts = []
        for _ in range(args.steps):
            torch.cuda._sleep(200000)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            call()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        if int(err.item()) != 0:
            raise SystemExit(f"device error {int(err.item())}")
        ms = sorted(ts)[len(ts) // 2]
        causal = 4.0 * Hq * D * (T * (KV - T) + T * (T + 1) / 2)    # causal-effective FLOPs
        res[KV] = {"ms": ms, "tflops_causal": causal / (ms / 1e3) / 1e12,
                   "tflops_dense": 4.0 * Hq * T * KV * D / (ms / 1e3) / 1e12}
    if rank == 0:
        peaks, src = measured_peaks()
        best = res[16384]["tflops_causal"]
        line = {"metric": "FLASH_ATTN_EXT prefill TFLOP/s (causal-effective), 32/8 heads, D 128, n_q 512",
                "value": best, "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": res[16384]["ms"], "higher_is_better": True, "scaling": "replicas only",
                "vs_baseline": None, "dtype": "f16 (fp32 softmax/accumulate)", "data": "synthetic",
                "config": {"workload": "BASELINE configs[2], value at n_kv=16384", "per_n_kv": res},
                "roofline": {"bound": "tensor", "achieved": best, "peak": float(peaks["bf16_tflops"]),
                             "unit": "TFLOP/s", "frac": best / float(peaks["bf16_tflops"]),
                             "peak_source": f"{src} bf16_tflops (burst)"}}
        print(json.dumps(line), flush=True)
    return 0


def run_gemv(args):
    """Decode-size MUL_MAT (b200_mul_mat_vec): the three weights of the headline sweep, quantized to
    --decode-type, against M = --decode-m token rows, L2 flushed before every step. value = weight
    bytes streamed per second (the kernel's roofline is HBM: each weight byte is read once); the
    per-shape times (activation prep + weight-streaming kernel, CUDA events) are in config."""
    import numpy as np
    import torch
    import ggml_b200 as g
    from ggml_b200 import quants
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    g.lib()
    M = args.decode_m
    wtype = {"q4_k": g.Q4_K, "q6_k": g.Q6_K, "q8_0": g.Q8_0}[args.decode_type]
    tname = args.decode_type.upper()
    rng = np.random.default_rng(0xB200)
    packed, acts, outs, wss, sizes = [], [], [], [], []
    wbytes = 0
    for (k, n) in SHAPES:
        w = (rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02))
        raw = torch.from_numpy(quants.quantize(wtype, w).reshape(-1)).to(dev)
        p = torch.empty(g.weight_packed_size(wtype, n, k), dtype=torch.uint8, device=dev)
        g.weight_pack(wtype, raw, n, k, p)
        packed.append(p)
        sizes.append(p.numel())
        wbytes += p.numel()
        acts.append(torch.from_numpy(rng.standard_normal((M, k)).astype(np.float32)).to(dev))
        outs.append(torch.empty((M, n), dtype=torch.float32, device=dev))
        wss.append(torch.empty(max(256, g.lib().b200_mul_mat_vec_workspace_size(M, n, k)), dtype=torch.uint8, device=dev))
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step(evs=None):
        for i, (k, n) in enumerate(SHAPES):
            if evs:
                evs[i].record(stream)
            g.check(g.mul_mat_vec(wtype, packed[i], n, k, acts[i], M, outs[i], wss[i], err, stream=stream),
                    "mul_mat_vec")
        if evs:
            evs[len(SHAPES)].record(stream)

    for _ in range(args.warmup):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
    ts = []
    for _ in range(args.steps):
        flush.zero_()
        torch.cuda._sleep(1000000)
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(len(SHAPES) + 1)]
        step(evs)
        ts.append(evs)
    torch.cuda.synchronize()
    clocks = sampler.stop() if sampler else None
    if int(err.item()) != 0:
        raise SystemExit(f"device error {int(err.item())}")
    ms = statistics.median(evs[0].elapsed_time(evs[-1]) for evs in ts)
    per = {}
    for i, (k, n) in enumerate(SHAPES):
        us = statistics.median(evs[i].elapsed_time(evs[i + 1]) for evs in ts) * 1e3
        per[f"{k}x{n}"] = {"us": us, "GB/s": sizes[i] / (us / 1e6) / 1e9}
    if rank == 0:
        peaks, src = measured_peaks()
        gbs = wbytes / (ms / 1e3) / 1e9
        peak = float(peaks.get("hbm_gbs", 6650.0))
        line = {"metric": f"decode MUL_MAT GB/s of {tname} weight streamed (b200_mul_mat_vec)", "value": gbs,
                "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                "higher_is_better": True, "scaling": "replicas only", "vs_baseline": None,
                "dtype": f"f16 activations x {tname} weights, fp32 accumulate", "data": "synthetic",
                "config": {"workload": f"the weights of BASELINE configs[1] as {tname} at M={M} token rows, one op "
                                       "per shape per step", "weight_bytes_per_step": wbytes,
                           "tokens_per_s": M / (ms / 1e3), "per_shape": per,
                           "l2": "flushed before every timed step (256 MiB memset), outside the timed events",
                           "median_of_steps": True},
                "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                             "peak_source": f"{src} hbm_gbs"},
                "clocks": clocks, "gpu_launches": 2 * len(SHAPES) * args.steps}
        print(json.dumps(line), flush=True)
    return 0


def time_sweep_1gpu(args, m_tokens):
    """One GPU's time for one layer of the sweep at m_tokens (b200_mul_mat per shape, whole
    weights), measured the way run_gemm_sharded measures the sharded op: L2 flushed and a GPU
    delay before every step, CUDA events around it; the reference for its strong scaling."""
    import numpy as np
    import torch
    import ggml_b200 as g
    from ggml_b200 import quants
    dev = torch.device("cuda", torch.cuda.current_device())
    rng = np.random.default_rng(0xB200)
    ws, acts, outs, wss = [], [], [], []
    for (k, n) in SHAPES:
        w = (rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02))
        raw = torch.from_numpy(quants.quantize(WTYPE, w).reshape(-1)).to(dev)
        packed = torch.empty(g.weight_packed_size(WTYPE, n, k), dtype=torch.uint8, device=dev)
        g.weight_pack(WTYPE, raw, n, k, packed)
        ws.append(packed)
        acts.append(torch.from_numpy(rng.standard_normal((m_tokens, k)).astype(np.float32)).to(dev))
        outs.append(torch.empty((m_tokens, n), dtype=torch.float32, device=dev))
        wss.append(torch.empty(max(256, g.mul_mat_workspace_size(m_tokens, n, k, WTYPE)), dtype=torch.uint8,
                               device=dev))
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    evs = []
    for it in range(args.warmup + args.steps):
        flush.zero_()
        torch.cuda._sleep(1000000)
        e = [torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)]
        e[0].record(stream)
        for i, (k, n) in enumerate(SHAPES):
            g.mul_mat(WTYPE, ws[i], n, k, acts[i], m_tokens, outs[i], wss[i], err, stream=stream)
        e[1].record(stream)
        if it >= args.warmup:
            evs.append(e)
    torch.cuda.synchronize()
    if int(err.item()) != 0:
        raise SystemExit(f"device error {int(err.item())} in the one-GPU sweep")
    return sum(e[0].elapsed_time(e[1]) for e in evs) / len(evs)


def run_gemm_sharded(args, inside=False, m_tokens=M_TOKENS):
    """The headline sweep with every weight's rows split across the ranks (ggml_b200.tp): each
    rank packs its row block of each shape's weight, runs the N-sharded MUL_MAT on the shared
    activation, and ends holding the full dst. value = the sweep's FLOPs / max-over-ranks time.
    inside: called from the headline arm (the process group exists; return the timing).
    m_tokens: the token count (the sweep's M; 512 for the headline)."""
    import numpy as np
    import torch
    import ggml_b200 as g
    from ggml_b200 import quants
    from ggml_b200.tp import PeerShardedMulMat, shard_rows
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if inside:
        pass
    elif world > 1:
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=dev)
    else:
        torch.distributed.init_process_group("gloo", init_method="tcp://127.0.0.1:29581", rank=0, world_size=1)
    g.lib()
    rng = np.random.default_rng(0xB200)
    shards, acts = [], []
    for (k, n) in SHAPES:
        w = (rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02))
        lo, hi = shard_rows(n, world, rank)
        raw = torch.from_numpy(quants.quantize(WTYPE, w[lo:hi]).reshape(-1)).to(dev)
        packed = torch.empty(g.weight_packed_size(WTYPE, hi - lo, k), dtype=torch.uint8, device=dev)
        g.weight_pack(WTYPE, raw, hi - lo, k, packed)
        shards.append(packed)
        acts.append(torch.from_numpy(rng.standard_normal((m_tokens, k)).astype(np.float32)).to(dev))
    tp = PeerShardedMulMat(m_tokens, max(n for (_, n) in SHAPES))
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)

    def step():
        for i, (k, n) in enumerate(SHAPES):
            tp(WTYPE, shards[i], n, k, acts[i], m_tokens, stream=stream)

    for _ in range(args.warmup):
        flush.zero_()
        torch.cuda._sleep(1000000)
        step()
    torch.cuda.synchronize()
    if int(tp.err.item()) != 0:
        raise SystemExit(f"device error {int(tp.err.item())} during warm-up")
    sampler = ClockSampler(local) if rank == 0 else None
    torch.distributed.barrier()
    torch.cuda.synchronize()
    if sampler:
        sampler.start()
    evs = []
    for _ in range(args.steps):
        flush.zero_()
        torch.cuda._sleep(1000000)
        e = [torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)]
        e[0].record(stream)
        step()
        e[1].record(stream)
        evs.append(e)
    torch.cuda.synchronize()
    torch.distributed.barrier()
    clocks = sampler.stop() if sampler else None
    if int(tp.err.item()) != 0:
        raise SystemExit(f"device error {int(tp.err.item())} in the timed region")
    ms_local = sum(e[0].elapsed_time(e[1]) for e in evs) / len(evs)
    vals = torch.tensor([ms_local], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(vals, op=torch.distributed.ReduceOp.MAX)
    ms = float(vals.item())
    tp.close()
    if inside:
        return {"ms": ms, "tflops": step_flops(m_tokens) / (ms / 1e3) / 1e12}
    if rank == 0:
        flops = step_flops()
        line = {"metric": METRIC, "value": flops / (ms / 1e3) / 1e12, "unit": "TFLOP/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "f16 (fp32 accumulate)", "data": "synthetic",
                "config": {"workload": WORKLOAD + "; every weight's rows split across the ranks, the output "
                                                  "all-gathered by the GEMM epilogue's stores into peer memory",
                           "weight_type": "Q4_K", "global_batch": M_TOKENS, "seq_len": M_TOKENS,
                           "parallelism": f"N-sharded x{world}",
                           "l2": "flushed before every timed step (256 MiB memset), outside the timed events",
                           "tokens_per_s": M_TOKENS / (ms / 1e3)},
                "clocks": clocks, "gpu_launches": 4 * len(SHAPES) * args.steps}
        print(json.dumps(line), flush=True)
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()
    return 0


def _ne_nb(t):
    """ggml ne[4] / nb[4] (bytes) of a torch tensor whose dims are listed outermost first."""
    import ctypes
    ne = list(reversed(t.shape)) + [1] * (4 - t.dim())
    nb = [st * t.element_size() for st in reversed(t.stride())]
    last = nb[-1] * ne[t.dim() - 1]
    nb = nb + [last] * (4 - t.dim())
    return (ctypes.c_int64 * 4)(*ne), (ctypes.c_size_t * 4)(*nb)


def run_glue(args):
    """The glue ops of a Llama-8B-shaped layer at a 512-token ubatch (hidden 4096, FFN 14336, 32
    query / 8 KV heads of 128) and the MoE router of configs[3] (128 experts, 2048 tokens), each
    through its C-ABI entry point on device tensors, L2 flushed before every step. value = the
    ops' algorithmic bytes (one read of every input element, one write of every output element)
    per second of their summed CUDA-event time; per-op figures in config."""
    import ctypes
    import torch
    import ggml_b200 as g
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    lib = g.lib()
    stream = torch.cuda.current_stream(dev)
    sp = ctypes.c_void_p(stream.cuda_stream)
    gen = torch.Generator(device=dev).manual_seed(0xB200)
    T, E, F, H, HK, D = 512, 4096, 14336, 32, 8, 128

    def rnd(*shape, dtype=torch.float32):
        return torch.randn(*shape, generator=gen, device=dev, dtype=torch.float32).to(dtype)

    x, res, wn = rnd(T, E), rnd(T, E), rnd(E)
    q, k = rnd(T, H, D), rnd(T, HK, D)
    pos = torch.arange(T, device=dev, dtype=torch.int32)
    gate, up = rnd(T, F), rnd(T, F)
    table = rnd(32000, E, dtype=torch.float16)
    ids = torch.randint(0, 32000, (T,), generator=gen, device=dev, dtype=torch.int32)
    logits = rnd(2048, 128)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    o_e = torch.empty(T, E, device=dev)
    o_q, o_k = torch.empty_like(q), torch.empty_like(k)
    o_f = torch.empty(T, F, device=dev)
    o_kh = torch.empty(T, HK, D, device=dev, dtype=torch.float16)
    o_rows = torch.empty(T, E, device=dev)
    o_p = torch.empty_like(logits)
    o_ids = torch.empty(2048, 128, device=dev, dtype=torch.int32)
    P = lambda t: ctypes.c_void_p(t.data_ptr())   # noqa: E731
    sh = {n: _ne_nb(t) for n, t in (("x", x), ("wn", wn), ("q", q), ("k", k), ("f", gate), ("tab", table),
                                     ("ids", ids.view(1, T)), ("lg", logits), ("kh", o_kh))}
    ops = [
        # RMS_NORM and the MUL by the norm weight, fused as graph_compute runs them
        ("rms_norm_mul", 8 * T * E + 4 * E,
         lambda: lib.b200_rms_norm_mul(P(x), *sh["x"], 1e-5, P(wn), None, P(o_e), sp)),
        ("rope_q", 8 * T * H * D, lambda: lib.b200_rope(P(q), *sh["q"], P(pos), D, 2, 500000.0, 1.0, 1.0, P(o_q), sp)),
        ("rope_k", 8 * T * HK * D,
         lambda: lib.b200_rope(P(k), *sh["k"], P(pos), D, 2, 500000.0, 1.0, 1.0, P(o_k), sp)),
        ("cpy_k_f16", 6 * T * HK * D, lambda: lib.b200_cpy(0, P(o_k), *sh["k"], 1, P(o_kh), *sh["kh"], sp)),
        ("swiglu", 12 * T * F,
         lambda: lib.b200_swiglu(P(gate), sh["f"][1], P(up), sh["f"][1], sh["f"][0], P(o_f), sp)),
        ("add_residual", 12 * T * E, lambda: lib.b200_binary(0, P(x), *sh["x"], P(res), *sh["x"], P(o_e), sp)),
        ("get_rows_f16", 6 * T * E + 4 * T,
         lambda: lib.b200_get_rows(1, P(table), *sh["tab"], P(ids), *sh["ids"], P(o_rows), P(err), sp)),
        ("router_soft_max", 8 * 2048 * 128, lambda: lib.b200_soft_max(P(logits), *sh["lg"], 1.0, P(o_p), sp)),
        ("router_argsort", 8 * 2048 * 128, lambda: lib.b200_argsort(P(o_p), *sh["lg"], 1, P(o_ids), sp)),
    ]
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)

    def step(evs=None):
        for i, (_, _, fn) in enumerate(ops):
            if evs:
                evs[i][0].record(stream)
            rc = fn()
            if rc != 0:
                raise SystemExit(f"glue op {ops[i][0]} failed: {rc}")
            if evs:
                evs[i][1].record(stream)

    for _ in range(max(3, args.warmup)):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
    per = [[] for _ in ops]
    steps = []
    for _ in range(args.steps):
        flush.zero_()
        torch.cuda._sleep(1000000)
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in ops]
        step(evs)
        steps.append(evs)
    torch.cuda.synchronize()
    clocks = sampler.stop() if sampler else None
    if int(err.item()) != 0:
        raise SystemExit(f"device error {int(err.item())}")
    for evs in steps:
        for i, (e0, e1) in enumerate(evs):
            per[i].append(e0.elapsed_time(e1))
    med = [statistics.median(v) for v in per]
    total_bytes = sum(b for _, b, _ in ops)
    total_ms = sum(med)
    if rank == 0:
        peaks, src = measured_peaks()
        peak = float(peaks.get("hbm_gbs", 6650.0))
        gbs = total_bytes / (total_ms / 1e3) / 1e9
        table_out = {name: {"us": m * 1e3, "GB/s": b / (m / 1e3) / 1e9, "frac": b / (m / 1e3) / 1e9 / peak}
                     for (name, b, _), m in zip(ops, med)}
        line = {"metric": "glue-op GB/s (algorithmic bytes) at Llama-8B prefill shapes, T=512, and the configs[3] "
                          "MoE router", "value": gbs, "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": total_ms, "higher_is_better": True,
                "scaling": "replicas only", "vs_baseline": None, "dtype": "f32 (f16 table / KV cache)",
                "data": "synthetic",
                "config": {"workload": "RMS_NORM*MUL (fused), ROPE q/k, CPY k->f16, SWIGLU, ADD, GET_ROWS, SOFT_MAX, "
                                       "ARGSORT via their C-ABI entry points", "ops": table_out,
                           "l2": "flushed before every timed step (256 MiB memset), outside the timed events",
                           "median_of_steps": True},
                "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                             "peak_source": f"{src} hbm_gbs"},
                "clocks": clocks, "gpu_launches": len(ops) * args.steps}
        print(json.dumps(line), flush=True)
    return 0


LAYER_DIMS = dict(E=4096, F=14336, H=32, HK=8, D=128, vocab=128256, layers=32, prompt=4096, ubatch=512)


def run_layer(args):
    """BASELINE configs[4]'s prefill, layer by layer: one Llama-3-8B-architecture layer (hidden 4096,
    FFN 14336, 32 query / 8 KV heads of 128, RoPE theta 500000, Q4_K weights) as llama.cpp builds its
    graph (ggml_b200.graph.llama_layer), every node claimed (B200_GLUE=1) and computed by
    graph_compute on tensors in the backend's device buffer. The 4096-token prompt runs as 8 ubatches
    of 512; ubatch i attends to 512 (i + 1) keys. Each ubatch's layer is timed (wall clock of the
    synchronous graph_compute call, L2 flushed before each); prompt tokens/s = 4096 / (32 layers x the
    sum over the 8 ubatches). Not included: the token embedding lookup, the final norm and the output
    head (llama.cpp computes logits for the last token only by default)."""
    os.environ.setdefault("B200_GLUE", "1")
    os.environ.setdefault("B200_FLASH_ATTN_MIN_KV", "512")   # the first ubatch attends to 512 keys
    import numpy as np
    import torch
    import ggml_b200 as g
    from ggml_b200 import quants
    from ggml_b200.graph import llama_layer
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    g.lib()
    d = LAYER_DIMS
    E, F, H, HK, D, T = d["E"], d["F"], d["H"], d["HK"], d["D"], d["ubatch"]
    n_ub = d["prompt"] // T
    rng = np.random.default_rng(0xB200)
    # N(0, 0.02) Q4_K weights: one [F, E] block (q, k, v, o are slices of its rows) and one [E, F]
    big = quants.quantize(g.Q4_K, rng.standard_normal((F, E), dtype=np.float32) * np.float32(0.02))
    down = quants.quantize(g.Q4_K, rng.standard_normal((E, F), dtype=np.float32) * np.float32(0.02))
    wsrc = {"attn_q": big[:E], "attn_k": big[E:E + D * HK], "attn_v": big[E + D * HK:E + 2 * D * HK],
            "attn_output": big[F - E:], "ffn_gate": big, "ffn_up": big, "ffn_down": down}
    be = g.Backend()
    graphs = []
    for i in range(n_ub):
        n_kv = T * (i + 1)
        # size a buffer for this graph: a dry run of the allocator
        sizes = []

        def count(n):
            sizes.append(n)
            return 0, True
        llama_layer(T, E=E, F=F, H=H, HK=HK, D=D, n_kv=n_kv, wtype=g.Q4_K, rope_base=500000.0, il=i, alloc=count)
        size = sum((n + 255) // 256 * 256 for n in sizes) + (1 << 20)
        buf = g.DeviceBuffer(be, size)
        top = [0]

        def alloc(n, buf=buf, top=top):
            off = top[0]
            top[0] += (n + 255) // 256 * 256
            return buf.base + off, True
        L = llama_layer(T, E=E, F=F, H=H, HK=HK, D=D, n_kv=n_kv, wtype=g.Q4_K, rope_base=500000.0, il=i, alloc=alloc)
        off = lambda t: t.data - buf.base   # noqa: E731
        buf.set(off(L.inputs["x"]), rng.standard_normal((T, E), dtype=np.float32))
        buf.set(off(L.inputs["pos"]), np.arange(n_kv - T, n_kv, dtype=np.int32))
        Tp = L.inputs["mask"].ne[1]
        mask = np.full((Tp, n_kv), -np.inf, np.float32)
        for t in range(T):
            mask[t, :n_kv - T + t + 1] = 0.0
        buf.set(off(L.inputs["mask"]), mask.astype(np.float16).view(np.uint16))
        for c in L.caches.values():
            buf.set(off(c), (rng.standard_normal(c.ne[0] * c.ne[1], dtype=np.float32)).astype(np.float16).view(np.uint16))
        for name, t in L.weights.items():
            if t.type == g.F32:
                buf.set(off(t), np.ones(t.ne[0], np.float32))
            else:
                buf.set(off(t), np.ascontiguousarray(wsrc[name]))
        for nd in L.nodes:
            if not g.supports_op(nd):
                raise SystemExit(f"node {nd.name.decode()} not claimed")
        graphs.append((n_kv, L, buf))
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    sampler = ClockSampler(local)
    per = {}
    for n_kv, L, buf in graphs:
        for _ in range(max(3, args.warmup)):
            if be.graph_compute(L.nodes) != g.STATUS_SUCCESS:
                raise SystemExit("graph_compute failed")
    sampler.start()
    for n_kv, L, buf in graphs:
        ts = []
        for _ in range(args.steps):
            flush.zero_()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            if be.graph_compute(L.nodes) != g.STATUS_SUCCESS:
                raise SystemExit("graph_compute failed")
            ts.append(time.perf_counter() - t0)
        per[n_kv] = statistics.median(ts)
    clocks = sampler.stop()
    layer_s = sum(per.values())
    prefill_s = layer_s * d["layers"]
    tps = d["prompt"] / prefill_s
    # algorithmic FLOPs of one layer at ubatch T with n_kv keys: projections + causal attention
    proj = 2.0 * T * E * (E + 2 * D * HK + E + 3 * F)
    attn = lambda n_kv: 4.0 * H * D * (T * (n_kv - T) + T * (T + 1) / 2)   # noqa: E731
    flops = sum(proj + attn(n) for n in per)
    assert be.cpu_fallbacks() == 0 and be.device_errors() == 0
    line = {"metric": "prompt tokens/sec, Llama-3-8B-architecture prefill (32 layers x one measured layer), "
                      "4096-token prompt in 512-token ubatches", "value": tps, "unit": "tokens/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": layer_s * 1e3, "higher_is_better": True,
            "scaling": "replicas only", "vs_baseline": None, "dtype": "f16 x Q4_K (fp32 accumulate)",
            "data": "synthetic",
            "config": {"workload": "BASELINE configs[4]: one layer per ubatch through graph_compute on device "
                                   "buffers (B200_GLUE=1), all 8 ubatches of a 4096-token prompt",
                       "layer_ms_per_ubatch_n_kv": {str(k): v * 1e3 for k, v in per.items()},
                       "layer_tflops": flops / layer_s / 1e12,
                       "excluded": "token embedding, final norm, output head (last-token logits only)",
                       "timing": "wall clock of the synchronous graph_compute call, median of steps, L2 flushed",
                       "routes": {r: be.route_ops(r) for r in ("q4_K", "fused", "fa", "glue")}},
            "clocks": clocks}
    print(json.dumps(line), flush=True)
    for _, _, buf in graphs:
        buf.free()
    be.close()
    return 0


def run_crossover(args):
    """Where a claimed MUL_MAT stops paying: graph_compute on one MUL_MAT node with HOST tensors (the
    reference's setting: the host keeps activations in its CPU buffers and the backend claims the op,
    ggml-rocket.cpp:846-894) against the host CPU computing the same product, per M, for F16 and Q4_K
    weights of two Llama-8B shapes. The device arm copies the activations in and the output out inside
    the call (pageable memory, what an ACCEL device's host gets, and pinned memory from this backend's
    host buffer type); its weight is already cached on the device, as it is after a model's first
    ubatch. The CPU arm is torch's fp32 matmul over the dequantized weight on every host core (an
    optimized BLAS standing in for ggml's CPU backend, which is absent here). M* is the smallest M
    whose device time beats the CPU's."""
    os.environ.setdefault("B200_MIN_M", "4")
    os.environ.setdefault("B200_MIN_M_QUANT", "4")
    import numpy as np
    import torch
    import ggml_b200 as g
    from ggml_b200 import quants
    world, rank, local = dist_env()
    if rank != 0:
        return 0
    torch.cuda.set_device(local)
    g.lib()
    torch.set_num_threads(os.cpu_count())
    rng = np.random.default_rng(0xC805)
    Ms = (4, 8, 16, 32, 64, 128, 256, 512)
    be = g.Backend()
    res = {}
    reps = max(3, min(args.steps, 10))
    for wtype in (g.F16, g.Q4_K):
        for (k, n) in ((4096, 4096), (4096, 14336)):
            w = rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)
            if wtype == g.F16:
                nat = w.astype(np.float16).view(np.uint8).reshape(n, -1)
                wf = torch.from_numpy(w.astype(np.float16).astype(np.float32))
            else:
                nat = quants.quantize(wtype, w)
                import oracle
                oracle.build()
                wf = torch.from_numpy(oracle.dequantize(wtype, nat, k))
            rows = {}
            for M in Ms:
                a = rng.standard_normal((M, k), dtype=np.float32)
                out = {}
                for pinned in (False, True):
                    if pinned:
                        a_h, a_ptr = _pinned_array(g, a.nbytes, np.float32, a.shape)
                        o_h, o_ptr = _pinned_array(g, M * n * 4, np.float32, (M, n))
                    else:
                        a_h, o_h = np.empty_like(a), np.empty((M, n), np.float32)
                        a_ptr, o_ptr = a_h.ctypes.data, o_h.ctypes.data
                    a_h[:] = a
                    wt = g.make_tensor(wtype, [k, n], data=nat, name=f"xover.{wtype}.{k}x{n}.weight")
                    at = g.make_tensor(g.F32, [k, M], data=a_ptr, name="x")
                    dt = g.make_tensor(g.F32, [n, M], data=o_ptr, op=g.OP_MUL_MAT, srcs=[wt, at], name="y")
                    if not g.supports_op(dt):
                        raise SystemExit(f"MUL_MAT M={M} not claimed")
                    for _ in range(2):
                        be.graph_compute([dt])
                    ts = []
                    for _ in range(reps):
                        t0 = time.perf_counter()
                        if be.graph_compute([dt]) != g.STATUS_SUCCESS:
                            raise SystemExit("graph_compute failed")
                        ts.append(time.perf_counter() - t0)
                    out["pinned" if pinned else "pageable"] = statistics.median(ts) * 1e6
                    if pinned:
                        g.lib().ggml_backend_b200_host_free(a_ptr)
                        g.lib().ggml_backend_b200_host_free(o_ptr)
                at_ = torch.from_numpy(a)
                torch.matmul(at_, wf.T)
                ts = []
                for _ in range(reps):
                    t0 = time.perf_counter()
                    torch.matmul(at_, wf.T)
                    ts.append(time.perf_counter() - t0)
                out["cpu"] = statistics.median(ts) * 1e6
                rows[M] = {kk: round(v, 1) for kk, v in out.items()}
            xo = {arm: next((M for M in Ms if rows[M][arm] < rows[M]["cpu"]), None) for arm in ("pageable", "pinned")}
            res[f"{g.TYPE_NAMES[wtype]} K={k} N={n}"] = {"us_by_M": rows, "crossover_M": xo}
    be.close()
    worst = max((v["crossover_M"]["pageable"] or 10 ** 9) for v in res.values())
    line = {"metric": "MUL_MAT claim crossover: smallest M at which graph_compute (host tensors) beats the host CPU",
            "value": worst, "unit": "rows", "n_gpus": 1, "steps": reps, "warmup": 2, "higher_is_better": False,
            "scaling": "replicas only", "vs_baseline": None, "dtype": "f16 / Q4_K (fp32 accumulate)",
            "data": "synthetic",
            "config": {"workload": "one MUL_MAT node per graph_compute call, weights cached on the device, "
                                   "activations and output in host memory",
                       "cpu_arm": f"torch fp32 matmul over the dequantized weight, {os.cpu_count()} threads",
                       "timing": "wall clock per synchronous call, median", "shapes": res}}
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "moe":
        return run_moe(args)
    if args.workload == "fa":
        return run_fa(args)
    if args.workload == "gemv":
        return run_gemv(args)
    if args.workload == "glue":
        return run_glue(args)
    if args.workload == "layer":
        return run_layer(args)
    if args.workload == "crossover":
        return run_crossover(args)
    if args.shard:
        return run_gemm_sharded(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
