"""Benchmark of the B200 GGUF dequant-matmul path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: the seven linear weights of a Llama-3-8B layer
in Q4_K -- q (4096x4096), k, v (1024x4096), o (4096x4096), gate, up
(14336x4096), down (4096x14336) -- as batch-1 decode GEMVs with fp32
activations.  One step = one pass over 8 distinct layer copies (56 GEMVs,
982 MB of blocks, about 7.8x the 126 MB L2, so every step streams from HBM).
Inputs are seeded synthetic tensors with the config's distributions.

* value     -- GB/s of weight blocks (algorithmic bytes: blocks + x + y)
               with everything resident in HBM; CUDA graph of the step,
               CUDA events on the launching stream.
* e2e       -- the same pass through the reference-facing C ABI
               (ftc_backend_matmul, the ft::IBackend::matmul equivalent):
               host x in, host y out, per call, the step's calls issued by
               a native loop as the engine's C++ decode loop issues them
               (e2e_python: the same calls from a Python loop); weights
               resident (uploaded once, as at Engine::load).
* roofline  -- the dominant kernel (gate/up shape 14336x4096) timed alone.
* cpu_baseline -- the CPU port of the reference's CpuBackend::matmul on a
               bounded sample (N=1, rank 0).
For N>1 every rank runs the same workload on its own GPU (replicas; the
decode GEMV does not shard): value = sum over ranks, time = max over ranks.
"""
import argparse
import atexit
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from xwfes_b200 import formats as F, synth as S  # noqa: E402

METRIC = "Q4_K dequant-GEMV HBM GB/s (% of peak) & prefill dequant-GEMM TFLOPS"
LAYER = [("q", 4096, 4096), ("k", 1024, 4096), ("v", 1024, 4096), ("o", 4096, 4096),
         ("gate", 14336, 4096), ("up", 14336, 4096), ("down", 4096, 14336)]
N_LAYERS = 8
# the workload both arms report (the reference arm times a bounded sample of it)
CONFIG = {
    "workload": "config 2: Q4_K decode GEMV, Llama-3-8B layer shapes (q,k,v,o 4096/1024x4096; "
                "gate,up 14336x4096; down 4096x14336), batch 1, fp32 activations",
    "l2": "inputs larger than L2: each GPU step streams 8 distinct layer copies (982 MB)",
}
# activation vector each GEMV reads (q/k/v share one, gate/up share one)
X_OF = {"q": "attn_in", "k": "attn_in", "v": "attn_in", "o": "attn_out", "gate": "ffn_in",
        "up": "ffn_in", "down": "ffn_mid"}
# launches of one decode layer: matrices that read the same activations go
# in one grouped launch, as a decode step issues them (o and down each wait
# for the attention / SiLU result in a real model)
GROUPS = [("qkv", ("q", "k", "v")), ("o", ("o",)), ("gate_up", ("gate", "up")), ("down", ("down",))]
SHAPE = {name: (n, k) for name, n, k in LAYER}
X_LEN = {"attn_in": 4096, "attn_out": 4096, "ffn_in": 4096, "ffn_mid": 14336}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


def peaks_sustained():
    """MEASURED_PEAKS.json's sustained bf16 GEMM rate (TFLOP/s), or None."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return json.load(open(p)).get("bf16_tflops_sustained")
    return None


def layer_bytes():
    w = sum(F.row_bytes(F.Q4_K, k) * n for _, n, k in LAYER)
    xy = sum(4 * (n + k) for _, n, k in LAYER)
    return w, xy


def make_weights(seed=0):
    return [{name: S.weight(F.Q4_K, n, k, seed=seed, name=f"L{li}.{name}")
             for name, n, k in LAYER} for li in range(N_LAYERS)]


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi samples (every 100 ms) of one GPU's clocks, power, load and
    throttle reasons, each stamped with the host time it arrived; the GPU is
    picked by its PCI bus id (nvidia-smi's domain:bus:device.function form).
    The timed region of a step (K x ~0.3 ms) is shorter than the sampling
    period, so the caller replays the same step graph back to back for a
    couple of seconds right after it and marks that window; the summary
    keeps the samples inside the window (the whole run without one) taken
    at >= 50 % utilization."""
    Q = ("pci.bus_id,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, bus_id):
        self.bus = (bus_id or "").lower()
        self.lines = []
        self.proc = None
        self.window = None

    @staticmethod
    def bus_id_of(props):
        """nvidia-smi's bus id string of a torch device (e.g. 00000000:1b:00.0)."""
        dom = getattr(props, "pci_domain_id", None)
        bus = getattr(props, "pci_bus_id", None)
        devn = getattr(props, "pci_device_id", None)
        if bus is None or devn is None:
            return ""
        return f"{dom or 0:08x}:{bus:02x}:{devn:02x}.0"

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def load_window(self, replay, seconds=2.0):
        """Run replay() (one batch of back-to-back step replays, synchronised)
        until `seconds` have passed and mark that span as the window."""
        t0 = time.time()
        while time.time() - t0 < seconds:
            replay()
        self.window = (t0, time.time())

    def __exit__(self, *a):
        proc, self.proc = self.proc, None
        if proc:
            proc.terminate()
            try:
                proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                proc.kill()
            self.t.join(timeout=5)

    def summary(self):
        sm, mx, pw, reasons, n_all = [], None, [], set(), 0
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        w = self.window
        rows = [[v.strip() for v in ln.split(",")] for t, ln in self.lines
                if w is None or w[0] + 0.15 <= t <= w[1]]
        rows = [f for f in rows if len(f) >= 9]
        mine = [f for f in rows if self.bus and f[0].lower().endswith(self.bus[-12:])]
        matched = bool(mine)
        if not mine and rows:  # bus id unknown: the first GPU listed
            first = rows[0][0]
            mine = [f for f in rows if f[0] == first]
        for f in mine:
            try:
                clk, mxc, p, util = float(f[1]), float(f[2]), float(f[3]), float(f[4])
            except ValueError:
                continue
            n_all += 1
            mx = mxc
            if util < 50:  # idle moments (host work) inside the window too
                continue
            sm.append(clk)
            pw.append(p)
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "power_w_median": statistics.median(pw) if pw else None,
                "reasons": sorted(reasons), "samples": len(sm), "samples_all": n_all,
                "gpu": self.bus if matched else "unmatched (first GPU listed)",
                "window": (f"{w[1] - w[0]:.1f} s of back-to-back replays of the timed step graph, "
                           "right after the timed region" if w else
                           "whole run (set-up excluded), samples with utilization >= 50 %")}


# ------------------------------------------------------------- our path

def side_measurement(name, fn, on_error):
    """A single-GPU measurement beside the headline one: a Python-level
    failure in it is reported in the JSON line (and on stderr) instead of
    costing the whole line.  Not used around collectives, which every rank
    must enter alike."""
    try:
        return fn()
    except Exception as e:  # noqa: BLE001 - reported, not hidden
        import traceback
        traceback.print_exc()
        err = f"{name}: {type(e).__name__}: {e}"
        if isinstance(on_error, dict):
            return {k: {"error": err} for k in on_error}
        return {"error": err}


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from xwfes_b200 import ftc

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    be = ftc.CudaBackend(local_rank)
    clk = ClockSampler(ClockSampler.bus_id_of(torch.cuda.get_device_properties(dev)))

    t0 = time.time()
    layers = make_weights(seed=0)
    hosts = {}
    for li, L in enumerate(layers):
        for name, n, k in LAYER:
            T = ftc.HostTensor(L[name], F.Q4_K, (k, n), name=f"L{li}.{name}")
            be.upload(T)
            hosts[(li, name)] = T
    xs_host = {nm: S.activations_f32(1, ln, seed=0, name=nm) for nm, ln in X_LEN.items()}
    xs = {nm: torch.from_numpy(a).to(dev) for nm, a in xs_host.items()}
    ys = {name: torch.empty((1, n), dtype=torch.float32, device=dev) for name, n, _ in LAYER}
    setup_s = time.time() - t0

    # device views of the cached blocks (the same HBM copies the C ABI uses)
    dptr = {key: be.device_ptr(T) for key, T in hosts.items()}

    stream = torch.cuda.Stream(device=dev)
    L = ftc.lib()

    import ctypes as C
    group_args = {}
    for li in range(N_LAYERS):
        for gname, members in GROUPS:
            P = len(members)
            k = SHAPE[members[0]][1]
            group_args[(li, gname)] = (
                P, (C.c_void_p * P)(*[dptr[(li, m)] for m in members]),
                (C.c_int64 * P)(*[SHAPE[m][0] for m in members]), k,
                xs[X_OF[members[0]]].data_ptr(),
                (C.c_void_p * P)(*[ys[m].data_ptr() for m in members]))

    # prefetch hints: the weight regions of the launch that follows
    hint_args = {}
    for li in range(N_LAYERS):
        for gname, members in GROUPS:
            P = len(members)
            hint_args[(li, gname)] = (
                P, (C.c_void_p * P)(*[dptr[(li, m)] for m in members]),
                (C.c_int64 * P)(*[SHAPE[m][0] * F.row_bytes(F.Q4_K, SHAPE[m][1]) for m in members]))

    def launch(li, gname, s, nxt=None):
        P, wa, na, k, xp, ya = group_args[(li, gname)]
        nn, nw, nb = hint_args[nxt] if nxt else (0, None, None)
        rc = L.ftc_mul_mat_vec_multi_hint(F.Q4_K, P, wa, na, k, F.row_bytes(F.Q4_K, k), xp, 1, ya,
                                          nn, nw, nb, s)
        if rc:
            raise ftc.FtcError("ftc_mul_mat_vec_multi_hint", rc, ftc.last_error())

    order = [(li, g) for li in range(N_LAYERS) for g, _ in GROUPS]

    def step(s):
        for i, key in enumerate(order):
            launch(*key, s, nxt=order[(i + 1) % len(order)])

    sp = stream.cuda_stream
    clk.__enter__()
    atexit.register(clk.__exit__, None, None, None)  # also on an error path
    with torch.cuda.stream(stream):
        step(sp)  # eager warm-up outside capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step(sp)
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            graph.replay()
    torch.cuda.synchronize()

    wbytes, xybytes = layer_bytes()
    step_bytes = N_LAYERS * (wbytes + xybytes)
    launches_per_step = N_LAYERS * len(GROUPS)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        ev0.record(stream)
        for _ in range(args.steps):
            graph.replay()  # replays on the current stream == `stream`
        ev1.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms = ev0.elapsed_time(ev1) / args.steps

    # clocks under this load: the same step graph back to back, untimed
    def replay_batch():
        with torch.cuda.stream(stream):
            for _ in range(100):
                graph.replay()
        torch.cuda.synchronize()

    clk.load_window(replay_batch)

    # dominant kernel alone: the gate/up launch over the 8 layer copies, graph-replayed
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g2, stream=stream):
        for li in range(N_LAYERS):
            launch(li, "gate_up", sp, nxt=((li + 1) % N_LAYERS, "gate_up"))
    reps = 200
    with torch.cuda.stream(stream):
        for _ in range(3):
            g2.replay()
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(reps):
            g2.replay()
        ev1.record(stream)
        torch.cuda.synchronize()
    k_ms = ev0.elapsed_time(ev1) / (reps * N_LAYERS)
    k_bytes = 2 * F.row_bytes(F.Q4_K, 4096) * 14336 + 4 * (4096 + 2 * 14336)

    # every launch group alone (8 launches per graph), for the per-group breakdown
    per_group = {}
    for gname, members in GROUPS:
        gg = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gg, stream=stream):
            for li in range(N_LAYERS):
                launch(li, gname, sp, nxt=((li + 1) % N_LAYERS, gname))
        with torch.cuda.stream(stream):
            for _ in range(3):
                gg.replay()
            torch.cuda.synchronize()
            ev0.record(stream)
            for _ in range(50):
                gg.replay()
            ev1.record(stream)
            torch.cuda.synchronize()
        us = ev0.elapsed_time(ev1) * 1e3 / (50 * N_LAYERS)
        gbytes = sum(F.row_bytes(F.Q4_K, SHAPE[m][1]) * SHAPE[m][0] for m in members)
        per_group[gname] = {"us": round(us, 2), "MB": round(gbytes / 1e6, 1),
                            "GBps": round(gbytes / (us * 1e-6) / 1e9, 0)}
        del gg

    decode_extras = side_measurement(
        "decode_extras", lambda: time_decode_extras(dev, dptr, stream),
        {"q8_0_config1": None, "batched": None, "q6_k_head": None})

    # e2e through the C ABI: host x in, host y out, per ftc_backend_matmul call
    ext = torch.cuda.ExternalStream(be.stream(), device=dev)
    yh = {name: np.empty((1, n), dtype=np.float32) for name, n, _ in LAYER}

    # the step's 56 calls in engine order, issued from native code (the
    # reference's engine is a C++ loop over IBackend::matmul)
    seq = be.matmul_sequence([(xs_host[X_OF[name]], 1, k, hosts[(li, name)], yh[name])
                              for li in range(N_LAYERS) for name, n, k in LAYER])
    seq.run(3)
    e2e_steps = max(20, min(args.steps, 200))
    barrier()
    torch.cuda.synchronize()
    ev0.record(ext)
    seq.run(e2e_steps)
    ev1.record(ext)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = ev0.elapsed_time(ev1) / e2e_steps

    # the same calls one by one from Python (CudaBackend.matmul per call)
    def e2e_step():
        for li in range(N_LAYERS):
            for name, n, k in LAYER:
                be.matmul(xs_host[X_OF[name]], 1, k, hosts[(li, name)], yh[name])

    for _ in range(3):
        e2e_step()
    barrier()
    torch.cuda.synchronize()
    ev0.record(ext)
    for _ in range(e2e_steps):
        e2e_step()
    ev1.record(ext)
    torch.cuda.synchronize()
    barrier()
    e2e_py_ms = ev0.elapsed_time(ev1) / e2e_steps
    h2d = N_LAYERS * sum(4 * k for _, _, k in LAYER)
    d2h = N_LAYERS * sum(4 * n for _, n, _ in LAYER)
    e2e_direct = side_measurement(
        "e2e_no_graphs",
        lambda: time_e2e_direct(dev, local_rank, hosts, xs_host, e2e_steps, step_bytes), None)

    prefill = side_measurement("prefill", lambda: time_prefill(dev), None)
    gemm_sustained = side_measurement("gemm_sustained",
                                      lambda: time_gemm_sustained(dev, clk.bus), None)
    gemm_status = ftc.device_status()
    tp_block = time_tp(dev, world, rank)
    moe = side_measurement("moe", lambda: time_moe(dev), None) if world == 1 else None
    attn = side_measurement("attention", lambda: time_attention(dev), None)
    ep_layer = time_ep(dev, world, rank)
    clk.__exit__(None, None, None)

    # max over ranks
    t = torch.tensor([ms, e2e_ms, k_ms, e2e_py_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms, k_ms, e2e_py_ms = t.tolist()

    del graph, g2
    be.close()
    if rank != 0:
        return None
    hbm, _, peak_kind = peaks()
    prefill_sum = prefill_summary(prefill, gemm_status)
    gbs = step_bytes * world / (ms * 1e-3) / 1e9
    k_gbs = k_bytes / (k_ms * 1e-3) / 1e9
    line = {
        "metric": METRIC,
        "value": round(gbs, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded Q4_K blocks and N(0,1) fp32 activations, config 2 distributions)",
        "config": CONFIG,
        "step": {
            "layers_per_step": N_LAYERS,
            "bytes_per_step": step_bytes,
            "parallelism": f"replicas x{world}",
            "graph": "CUDA graph of the step: 8 layers x 4 launches (q/k/v grouped, o, "
                     "gate/up grouped, down), programmatic dependent launch between them; "
                     "each launch prefetches the first 24 MB of the next one's weights into L2 "
                     "(ftc_mul_mat_vec_multi_hint)",
        },
        "pct_of_peak": round(100 * gbs / world / hbm, 1),
        "tokens_per_s": round(world * 1e3 / (ms / N_LAYERS * 32), 1),
        "tokens_per_s_note": "per-GPU decode rate of a 32-layer Llama-3-8B linear stack "
                             "at this layer time x world (attention and head excluded)",
        "roofline": {
            "bound": "hbm",
            "kernel": "gemv_q4k_dp4a, grouped gate+up (2 x 14336x4096), batch 1",
            "achieved": round(k_gbs, 1),
            "peak": hbm,
            "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs burst)",
            "unit": "GB/s",
            "frac": round(k_gbs / hbm, 3),
            "traffic": traffic_from_profiles(),
            "bytes_per_launch": k_bytes,
            "per_group": per_group,
            "us_per_launch": round(k_ms * 1e3, 3),
            "prefill_gemm": gemm_roofline(prefill_sum, short=True),
        },
        "roofline_gemm": gemm_roofline(prefill_sum, sustained_run=gemm_sustained),
        "e2e": {
            "value": round(step_bytes / (e2e_ms * 1e-3) / 1e9 * world, 2),
            "unit": "GB/s",
            "ms_per_step": round(e2e_ms, 4),
            "steps": e2e_steps,
            "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
            "api": "ftc_backend_matmul (ft::IBackend::matmul) called 56 times per step, in "
                   "engine order, from a native loop (MatmulSequence, host/call_loop.c): host x "
                   "copied into pinned staging, one cached CUDA graph per (weight, shape) "
                   "replayed per call (copy kernel in, GEMV storing y into pinned memory), sync "
                   "per call",
        },
        "e2e_python": {
            "value": round(step_bytes / (e2e_py_ms * 1e-3) / 1e9 * world, 2),
            "unit": "GB/s",
            "ms_per_step": round(e2e_py_ms, 4),
            "api": "the same 56 calls one by one from Python (CudaBackend.matmul, ctypes)",
        },
        "decode_batched": decode_extras["batched"],
        "q6_k_head": decode_extras["q6_k_head"],
        "q8_0_config1": decode_extras["q8_0_config1"],
        "e2e_no_graphs": e2e_direct,
        "prefill_dequant_gemm": prefill_sum,
        "tp_block": tp_block,
        "moe": moe,
        "attention": attn,
        "ep_moe": ep_layer,
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk.summary(),
        "setup_s": round(setup_s, 1),
    }
    return line


def time_e2e_direct(dev, local_rank, hosts, xs_host, steps, step_bytes):
    """The e2e pass through a second backend created with
    FTC_BACKEND_GRAPHS=0 (each ftc_backend_matmul issues its copy-in, GEMV and
    copy-out directly instead of replaying a cached graph): same calls, same
    host buffers, weights uploaded to its own cache first."""
    import torch
    from xwfes_b200 import ftc
    old = os.environ.get("FTC_BACKEND_GRAPHS")
    os.environ["FTC_BACKEND_GRAPHS"] = "0"
    try:
        be = ftc.CudaBackend(local_rank)
    finally:
        if old is None:
            os.environ.pop("FTC_BACKEND_GRAPHS", None)
        else:
            os.environ["FTC_BACKEND_GRAPHS"] = old
    try:
        for T in hosts.values():
            be.upload(T)
        yh = {name: np.empty((1, n), dtype=np.float32) for name, n, _ in LAYER}
        seq = be.matmul_sequence([(xs_host[X_OF[name]], 1, k, hosts[(li, name)], yh[name])
                                  for li in range(N_LAYERS) for name, n, k in LAYER])
        seq.run(3)
        ext = torch.cuda.ExternalStream(be.stream(), device=dev)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        ev0.record(ext)
        seq.run(steps)
        ev1.record(ext)
        torch.cuda.synchronize()
        ms = ev0.elapsed_time(ev1) / steps
        return {"value": round(step_bytes / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(ms, 4), "steps": steps,
                "api": "ftc_backend_matmul with FTC_BACKEND_GRAPHS=0 (copy kernel, GEMV and "
                       "any copy issued per call), pinned staging, sync per call; the 56 calls "
                       "from the native loop, as e2e"}
    finally:
        be.close()


def time_decode_extras(dev, dptr, stream, reps=20):
    """Config 2's other cases: the same 8 layer copies at batch 4 and 8 (one
    ftc_mul_mat_vec_multi launch per group of matrices sharing activations --
    q/k/v, o, gate/up, down -- graph-replayed), and the Q6_K output head
    (128256 x 4096, 431 MB, larger than L2) at batch 1."""
    import ctypes as C
    import torch
    from xwfes_b200 import ftc
    L = ftc.lib()
    hbm, _, _ = peaks()
    sp = stream.cuda_stream
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    wbytes, _ = layer_bytes()
    batched = {}
    for m in (4, 8):
        xm = {nm: torch.from_numpy(S.activations_f32(m, ln, seed=0, name=nm)).to(dev)
              for nm, ln in X_LEN.items()}
        ym = {name: torch.empty((m, n), dtype=torch.float32, device=dev) for name, n, _ in LAYER}

        gargs = []
        for li in range(N_LAYERS):
            for _, members in GROUPS:
                P = len(members)
                k = SHAPE[members[0]][1]
                gargs.append((P, (C.c_void_p * P)(*[dptr[(li, mm)] for mm in members]),
                              (C.c_int64 * P)(*[SHAPE[mm][0] for mm in members]), k,
                              xm[X_OF[members[0]]].data_ptr(),
                              (C.c_void_p * P)(*[ym[mm].data_ptr() for mm in members])))

        def bstep():
            for P, wa, na, k, xp, ya in gargs:
                rc = L.ftc_mul_mat_vec_multi(F.Q4_K, P, wa, na, k, F.row_bytes(F.Q4_K, k), xp, m,
                                             ya, sp)
                if rc:
                    raise ftc.FtcError("ftc_mul_mat_vec_multi", rc, ftc.last_error())

        with torch.cuda.stream(stream):
            bstep()  # eager warm-up outside capture
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            bstep()
        with torch.cuda.stream(stream):
            for _ in range(3):
                g.replay()
            torch.cuda.synchronize()
            ev0.record(stream)
            for _ in range(reps):
                g.replay()
            ev1.record(stream)
            torch.cuda.synchronize()
        us = ev0.elapsed_time(ev1) * 1e3 / reps / N_LAYERS  # per layer
        gbs = wbytes / (us * 1e-6) / 1e9
        batched[str(m)] = {"us_per_layer": round(us, 2), "weight_GBps": round(gbs, 1),
                           "frac_of_hbm": round(gbs / hbm, 3),
                           "tokens_per_s": round(m / (32 * us * 1e-6), 1)}
        del g
    n, k = 128256, 4096
    # 8 repeats of 16032 seeded rows: the bytes differ in address, not content
    w = torch.from_numpy(np.tile(S.weight(F.Q6_K, n // 8, k, seed=0, name="head"), (8, 1))).to(dev)
    x = torch.from_numpy(S.activations_f32(1, k, seed=0, name="head")).to(dev)
    y = torch.empty((1, n), dtype=torch.float32, device=dev)
    with torch.cuda.stream(stream):
        for _ in range(3):
            ftc.mul_mat_vec(w, F.Q6_K, n, k, x, y=y, stream=stream)
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(reps):
            ftc.mul_mat_vec(w, F.Q6_K, n, k, x, y=y, stream=stream)
        ev1.record(stream)
        torch.cuda.synchronize()
    us = ev0.elapsed_time(ev1) * 1e3 / reps
    hb = n * F.row_bytes(F.Q6_K, k)
    head = {"us": round(us, 1), "weight_GBps": round(hb / (us * 1e-6) / 1e9, 1),
            "frac_of_hbm": round(hb / (us * 1e-6) / 1e9 / hbm, 3), "bytes": hb,
            "l2": "weight 431 MB > L2: every launch streams from HBM"}
    del w
    # config 1 (Q8_0 4096 x 4096, 17.8 MB): 8 copies per graph so the launches stream from HBM
    n1 = k1 = 4096
    w1 = [torch.from_numpy(S.weight(F.Q8_0, n1, k1, seed=c, name="c1")).to(dev) for c in range(8)]
    x1 = torch.from_numpy(S.activations_f32(1, k1, seed=0, name="c1")).to(dev)
    y1 = torch.empty((1, n1), dtype=torch.float32, device=dev)
    with torch.cuda.stream(stream):
        for wc in w1:
            ftc.mul_mat_vec(wc, F.Q8_0, n1, k1, x1, y=y1, stream=stream)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for wc in w1:
                ftc.mul_mat_vec(wc, F.Q8_0, n1, k1, x1, y=y1, stream=stream)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(reps):
            g.replay()
        ev1.record(stream)
        torch.cuda.synchronize()
    us = ev0.elapsed_time(ev1) * 1e3 / reps / len(w1)
    b1 = n1 * F.row_bytes(F.Q8_0, k1)
    q8 = {"workload": "config 1: Q8_0 GEMV 4096x4096, batch 1 (8 weight copies per graph)",
          "us": round(us, 2), "weight_GBps": round(b1 / (us * 1e-6) / 1e9, 1),
          "frac_of_hbm": round(b1 / (us * 1e-6) / 1e9 / hbm, 3), "bytes": b1}
    del g, w1
    return {"q8_0_config1": q8,
            "batched": {"workload": "config 2 layer x 8 copies, fp32 activations, batch 4 and 8 "
                                    "(gemv_q4k_imma: integer tensor path, one launch per group "
                                    "of matrices sharing activations)",
                        "per_batch": batched},
            "q6_k_head": {"workload": "config 2 Q6_K output head 128256x4096, batch 1", **head}}


TP_M = [1, 16, 1024]
L2_BYTES = 126 * 2**20


TP_PEER_M = 16


def time_tp(dev, world, rank, seed=0):
    """Config 4: the Llama-3-70B-shaped Q4_K block (q, k, v, o, gate, up,
    down), tensor-parallel over the `world` GPUs (strong scaling: the block's
    work is split).  Each rank holds its shards (rank_shards); enough weight
    copies rotate through the timed passes that each pass streams its shards
    from HBM.  Each pass is a CUDA graph of the forward (NCCL allreduces
    included).  Time per pass = max over ranks (CUDA events, barrier before)."""
    import torch
    import torch.distributed as dist
    from xwfes_b200 import tp
    from xwfes_b200 import ftc
    d = tp.DIMS_70B
    hbm, bf16, _ = peaks()
    ops = tp.CudaOps(dev)
    shard_b = tp.weight_bytes(d) // world
    copies = min(4, max(1, -(-2 * L2_BYTES // shard_b)))
    # partials of up to TP_PEER_M tokens go through the NVLink peer allreduce
    peer, peer_note = None, None
    if world > 1:
        try:
            peer = ftc.PeerAllreduce(TP_PEER_M * d["n_embd"])
        except RuntimeError as e:  # raised on every rank alike: all fall back to NCCL
            peer_note = f"peer allreduce unavailable, NCCL for every M ({e})"
    blocks = [tp.TPBlock.build(d, world, rank, ops, tp.rank_shards(d, world, rank, seed=seed + c),
                               peer=peer)
              for c in range(copies)]
    out = {}
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st = torch.cuda.current_stream()
    cs = torch.cuda.Stream(device=dev)
    for M in TP_M:
        # config 4's bf16 N(0,1) activations, carried as fp32 (every value bf16-exact)
        x = torch.from_numpy(S.bf16_bits_to_f32(
            S.activations_bf16(M, d["n_embd"], seed=seed, name=f"tp.x{M}"))).to(dev)
        reps = 60 if M <= 16 else 12
        with torch.cuda.stream(cs):
            for i in range(3 * copies):  # eager warm-up (NCCL, kernel attributes) before capture
                blocks[i % copies].forward(x)
        torch.cuda.synchronize()
        # one CUDA graph per weight copy: the forward's launches and both
        # allreduces replay without host work in between
        graphs = []
        for b in blocks:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cs):
                b.forward(x)
            graphs.append(g)
        with torch.cuda.stream(cs):
            for i in range(3 * copies):
                graphs[i % copies].replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier(device_ids=[dev.index])
        st = cs
        ev0.record(st)
        with torch.cuda.stream(cs):
            for i in range(reps):
                graphs[i % copies].replay()
        ev1.record(st)
        torch.cuda.synchronize()
        del graphs
        t = torch.tensor([ev0.elapsed_time(ev1) / reps], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        us = t.item() * 1e3
        gbs = tp.weight_bytes(d) / (us * 1e-6) / 1e9
        tfl = tp.flops(d, M) / (us * 1e-6) / 1e12
        out[str(M)] = {"us": round(us, 1), "tokens_per_s": round(M / (us * 1e-6), 1),
                       "weight_GBps": round(gbs, 1), "tflops": round(tfl, 2),
                       # fractions of the world's aggregate measured peaks
                       "frac_of_hbm": round(gbs / (world * hbm), 3),
                       "frac_of_bf16": round(tfl / (world * bf16), 3),
                       "bound": "hbm" if M <= 16 else "tensor"}
    del blocks
    if peer is not None:
        dist.barrier(device_ids=[dev.index])  # no rank still writes into a peer's buffer
        peer.close()
    return {"workload": "config 4: Llama-3-70B-shaped Q4_K block (q 8192x8192, k/v 1024x8192, "
                        "o 8192x8192, gate/up 28672x8192, down 8192x28672), bf16 N(0,1) activations "
                        "carried as fp32",
            "parallelism": f"tp{world} (column-parallel q/k/v/gate/up, row-parallel o/down, "
                           f"allreduce of fp32 partials after o and down: one-shot over NVLink "
                           f"peer memory (ftc_peer_ar) for M <= {TP_PEER_M}, NCCL above)",
            "scaling": "strong (the whole block's work is split over the GPUs)",
            "weight_bytes": tp.weight_bytes(d), "weight_copies_rotated": copies,
            "kernels": "M<=8: decode GEMV (fp32); M>8: tcgen05 GEMM on row-scaled fp16",
            "limits": {"1": "per-launch start-up of the rank's decode GEMVs (~3-4 us each, "
                            "activation planes built after the dependency wait) and the "
                            "allreduce waits fused into the o and down GEMVs",
                       "16": "the small-M tcgen05 GEMM on the rank's shards (dequant-bound, "
                             "cut tiles) and the one-shot peer allreduces",
                       "1024": "two fp32 NCCL allreduces of 33.5 MB and mid-sized rank GEMMs"},
            **({"note": peer_note} if peer_note else {}),
            "per_M": out}


ATTN_CTX = [512, 4096, 32768]


def time_attention(dev, reps=50):
    """The engine's attention on the device (ftc_attention, ft/src/engine.cpp:
    137-177) at Llama-3-8B's heads (32 query heads, 8 KV heads, head_dim
    128): one decode row over a context of n positions, fp32 KV rows as
    ft::KvCache keeps them.  Enough layer copies are rotated (about 512 MB)
    that every call reads its K and V from HBM.  Beside it, the reference's
    own CPU attention (Engine::Impl::attn) on this host's cores at 4096."""
    import torch
    from xwfes_b200 import ftc
    nh, nkv, hd = 32, 8, 128
    dk = nkv * hd
    hbm, _, _ = peaks()
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    out = {}
    st = torch.cuda.Stream(device=dev)
    for n in ATTN_CTX:
        base = n - 1
        row_bytes = n * dk * 4
        copies = max(2, (512 << 20) // (2 * row_bytes))
        ks = [torch.randn((n, dk), device=dev, generator=g) for _ in range(copies)]
        vs = [torch.randn((n, dk), device=dev, generator=g) for _ in range(copies)]
        q = torch.randn((1, nh * hd), device=dev, generator=g)
        o = torch.empty((1, nh * hd), device=dev)
        need = int(ftc.lib().ftc_attention_workspace_bytes(1, nh, nkv, hd, base))
        ws = torch.empty(max(need, 16), dtype=torch.uint8, device=dev)
        with torch.cuda.stream(st):
            def call(i):
                k, v = ks[i % copies], vs[i % copies]
                ftc.attention(q, nh, nkv, hd, k[base:], v[base:], base=base, k_cache=k,
                              v_cache=v, out=o, ws=ws, stream=st)
            for i in range(copies):
                call(i)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=st):
                for i in range(copies):
                    call(i)
            for _ in range(3):
                graph.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            r = max(1, reps // copies)
            e0.record(st)
            for _ in range(r):
                graph.replay()
            e1.record(st)
            e1.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (r * copies)
        kv_bytes = 2 * row_bytes
        gbs = kv_bytes / (us * 1e-6) / 1e9
        out[str(n)] = {"us": round(us, 2), "kv_bytes": kv_bytes, "GBps": round(gbs, 1),
                       "frac_of_hbm": round(gbs / hbm, 3),
                       "layer_copies": copies}
        del graph, ks, vs
    ref = None
    try:
        from oracle import oracle as O
        R = O.ref_engine()
        if R is not None:
            n, threads = 4096, os.cpu_count() or 1
            rng = np.random.default_rng(0)
            qh = rng.standard_normal((1, nh * hd), dtype=np.float32)
            kh = rng.standard_normal((n, dk), dtype=np.float32)
            vh = rng.standard_normal((n, dk), dtype=np.float32)
            oh = np.empty_like(qh)
            p = lambda a: a.ctypes.data_as(O._p)  # noqa: E731
            ts = []
            for _ in range(5):
                t0 = time.perf_counter()
                R.ftref_attn(p(qh), 1, nh, nkv, hd, p(kh), p(vh), n - 1, p(kh[n - 1:]),
                             p(vh[n - 1:]), p(oh), threads)
                ts.append(time.perf_counter() - t0)
            ref = {"ctx": n, "us": round(statistics.median(ts) * 1e6, 1), "cores": threads,
                   "kind": "reference (Engine::Impl::attn compiled from its sources)"}
    except Exception as e:  # the checker library is optional on a box
        ref = {"error": str(e)[:200]}
    traffic = None
    prof = os.path.join(ROOT, "profiles", "attention_decode_32k.md")
    if os.path.exists(prof):
        for ln in open(prof):
            if ln.startswith("traffic_bytes_per_launch:"):
                traffic = int(ln.split(":", 1)[1].strip())
    if "32768" in out:
        out["32768"]["traffic"] = traffic  # ncu dram bytes of one split launch at this size
    return {"workload": "Llama-3-8B attention heads (32 q, 8 kv, head_dim 128), one decode row, "
                        "fp32 KV cache",
            "api": "ftc_attention (split positions, cp.async K/V staging, split combine)",
            "per_ctx": out, "reference_cpu_4096": ref, "status": ftc.device_status()}


MOE_T = [1, 64, 1024]


def time_moe(dev):
    """Config 5: Mixtral-8x7B-shaped MoE layer (8 experts, top-2) through
    ftc_moe_ffn, graph-replayed; L2 flushed (256 MB write) before every timed
    replay."""
    import torch
    from xwfes_b200 import ftc
    E, U, K, FF = 8, 2, 4096, 14336
    hbm, bf16, _ = peaks()
    mk = lambda nm, n, k: torch.from_numpy(
        S.expert_weights(F.Q4_K, E, n, k, seed=0, name=f"moe.{nm}")).to(dev)
    layer = ftc.MoeLayer(mk("gate", FF, K), mk("up", FF, K), mk("down", K, FF), n_experts=E,
                         top_k=U, n_embd=K, n_ff=FF)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    per_expert = 3 * FF * F.row_bytes(F.Q4_K, K)
    out = {}
    st = torch.cuda.Stream(device=dev)
    for T in MOE_T:
        logits = torch.from_numpy(S.router_logits(T, E, seed=0)).to(dev)
        x = torch.from_numpy(S.activations_bf16(T, K, seed=0, name="moe.x").view(np.int16)).to(
            dev).view(torch.bfloat16)
        with torch.cuda.stream(st):
            y = layer(logits, x, stream=st)
            for _ in range(3):
                layer(logits, x, out=y, stream=st)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=st):
                layer(logits, x, out=y, stream=st)
            ts = []
            for _ in range(15):
                flush.add_(1)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(st)
                g.replay()
                e1.record(st)
                e1.synchronize()
                ts.append(e0.elapsed_time(e1) * 1e3)
        used = int((layer.routing(T)[2] > 0).sum().item())
        us = statistics.median(ts)
        gbs = used * per_expert / (us * 1e-6) / 1e9
        tfl = 2.0 * T * U * 3 * FF * K / (us * 1e-6) / 1e12
        out[str(T)] = {"us": round(us, 1), "tokens_per_s": round(T / (us * 1e-6), 1),
                       "experts_used": used,
                       "weight_GBps": round(gbs, 1), "tflops": round(tfl, 2),
                       "frac_of_hbm": round(gbs / hbm, 3), "frac_of_bf16": round(tfl / bf16, 3),
                       "path": "decode GEMVs" if 2 * T * U <= 8 else "grouped tcgen05 GEMMs"}
        del g
    return {"workload": "config 5: 8 experts x Q4_K gate/up 14336x4096 + down 4096x14336, "
                        "top-2 softmax routing of N(0,1) fp32 logits, bf16 N(0,1) tokens",
            "api": "ftc_moe_ffn (routing, grouping, expert FFNs, combine on the device)",
            "per_T": out, "status": ftc.device_status()}


EP_T = [64, 1024]


def time_ep(dev, world, rank):
    """Config 5 expert-parallel: each rank holds 8/world experts (full
    Mixtral-8x7B expert shapes) and T/world of the tokens; one forward =
    routing, packing into fixed-capacity send buffers, count and row
    all-to-alls with equal splits, device regrouping, local grouped expert
    GEMMs, reverse all-to-all, combine.  No host synchronisation inside a
    forward, so it is captured and replayed as a CUDA graph (NCCL included);
    time = max over ranks, CUDA events, barrier before."""
    import torch
    import torch.distributed as dist
    from xwfes_b200 import ep
    d = ep.DIMS_MIXTRAL
    hbm, bf16, _ = peaks()
    E, U, K, FF = d["n_experts"], d["top_k"], d["n_embd"], d["n_ff"]
    e0, e1 = ep.expert_range(E, world, rank)
    mk = lambda nm, n, k: torch.from_numpy(np.stack(
        [S.weight(F.Q4_K, n, k, seed=0, name=f"moe.{nm}.{e}") for e in range(e0, e1)])).to(dev)
    ops = ep.CudaEPOps(dev, mk("gate", FF, K), mk("up", FF, K), mk("down", K, FF), e1 - e0, U, K,
                       FF)
    per_expert = 3 * FF * F.row_bytes(F.Q4_K, K)
    out = {}
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cs = torch.cuda.Stream(device=dev)
    for T in EP_T:
        t0, t1 = ep.token_range(T, world, rank)
        layer = ep.EPMoE(E, U, K, world, rank, ops, max_tokens=-(-T // world))
        logits = torch.from_numpy(S.router_logits(T, E, seed=0)[t0:t1]).to(dev)
        x = torch.from_numpy(S.activations_bf16(T, K, seed=0, name="moe.x")[t0:t1].view(
            np.int16)).to(dev).view(torch.bfloat16)
        with torch.cuda.stream(cs):
            for _ in range(3):  # eager warm-up (NCCL, workspaces, GEMM partial-sum scratch)
                layer.forward(logits, x)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=cs):
            layer.forward(logits, x)
        with torch.cuda.stream(cs):
            for _ in range(3):
                g.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier(device_ids=[dev.index])
        reps = 10
        ev0.record(cs)
        with torch.cuda.stream(cs):
            for _ in range(reps):
                g.replay()
        ev1.record(cs)
        torch.cuda.synchronize()
        del g
        t = torch.tensor([ev0.elapsed_time(ev1) / reps], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        us = t.item() * 1e3
        gbs = E * per_expert / (us * 1e-6) / 1e9
        tfl = 2.0 * T * U * 3 * FF * K / (us * 1e-6) / 1e12
        out[str(T)] = {"us": round(us, 1), "tokens_per_s": round(T / (us * 1e-6), 1),
                       "weight_GBps": round(gbs, 1), "tflops": round(tfl, 2),
                       "frac_of_hbm": round(gbs / (world * hbm), 3),
                       "frac_of_bf16": round(tfl / (world * bf16), 3)}
    return {"workload": "config 5: Mixtral-8x7B-shaped MoE layer, expert-parallel, T tokens "
                        "split over the ranks",
            "parallelism": f"ep{world} ({E // world} experts per GPU; equal-split NCCL "
                           "all-to-alls of counts, token rows (bf16) and expert outputs (fp32) "
                           "with a fixed capacity per rank; CUDA graph per forward)",
            "scaling": "strong (T and the 8 experts are split over the GPUs)",
            "per_T": out}


PREFILL_SHAPES = [(14336, 4096), (4096, 14336)]
PREFILL_M = [128, 512, 2048, 8192]


def time_prefill(dev, reps=20, copies=4):
    """Config 3: Q4_K dequant-GEMM (tcgen05) at every (N, K) x M, bf16
    activations, bf16 output.  Each timed launch uses the next of `copies`
    weight copies and a distinct activation tensor per M, so consecutive
    launches do not find their tiles in L2 (4 x 33 MB + activations)."""
    import torch
    from xwfes_b200 import ftc
    out = {}
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st = torch.cuda.current_stream()
    for n, k in PREFILL_SHAPES:
        ws = [torch.from_numpy(S.weight(F.Q4_K, n, k, seed=c, name=f"p.{n}x{k}")).to(dev)
              for c in range(copies)]
        for m in PREFILL_M:
            x = torch.from_numpy(S.activations_bf16(m, k, seed=0, name=f"p.{m}")).to(dev).view(
                torch.bfloat16)
            y = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
            for i in range(3):
                ftc.gemm(ws[i % copies], F.Q4_K, n, k, x, y=y, y_dtype=F.BF16)
            torch.cuda.synchronize()
            ev0.record(st)
            for i in range(reps):
                ftc.gemm(ws[i % copies], F.Q4_K, n, k, x, y=y, y_dtype=F.BF16)
            ev1.record(st)
            torch.cuda.synchronize()
            us = ev0.elapsed_time(ev1) * 1e3 / reps
            out[f"{n}x{k}_m{m}"] = {"us": round(us, 2),
                                    "tflops": round(2.0 * m * n * k / (us * 1e-6) / 1e12, 1)}
        del ws
    return out


def time_gemm_sustained(dev, bus, seconds=2.0, copies=4):
    """Config 3 at M = 8192 (14336 x 4096) back to back for ~2 s with the
    clocks sampled meanwhile: the GEMM's rate once the 1 kW power cap holds
    the clocks down, next to the cuBLAS GEMM's sustained figure."""
    import torch
    from xwfes_b200 import ftc
    n, k, m = 14336, 4096, 8192
    ws = [torch.from_numpy(S.weight(F.Q4_K, n, k, seed=c, name=f"p.{n}x{k}")).to(dev)
          for c in range(copies)]
    x = torch.from_numpy(S.activations_bf16(m, k, seed=0, name=f"p.{m}")).to(dev).view(
        torch.bfloat16)
    y = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    for c in range(copies):
        ftc.gemm(ws[c], F.Q4_K, n, k, x, y=y, y_dtype=F.BF16)
    torch.cuda.synchronize()
    clk = ClockSampler(bus)
    clk.__enter__()
    launches = 0
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def batch():
        nonlocal launches
        for c in range(copies * 4):
            ftc.gemm(ws[c % copies], F.Q4_K, n, k, x, y=y, y_dtype=F.BF16)
        launches += copies * 4
        torch.cuda.synchronize()

    try:
        ev0.record()
        clk.load_window(batch, seconds)
        ev1.record()
        torch.cuda.synchronize()
    finally:
        clk.__exit__(None, None, None)
    us = ev0.elapsed_time(ev1) * 1e3 / launches
    c = clk.summary()
    return {"tflops": round(2.0 * m * n * k / (us * 1e-6) / 1e12, 1), "us_per_launch": round(us, 1),
            "launches": launches, "sm_mhz": c["sm_mhz"], "power_w_median": c["power_w_median"],
            "reasons": c["reasons"], "clock_samples": c["samples"]}


def prefill_summary(prefill, status):
    if "error" in prefill:
        return {**prefill, "device_status": status}
    _, bf16_peak, kind = peaks()
    big = [v["tflops"] for kk, v in prefill.items() if kk.endswith("_m8192")]
    best = max(v["tflops"] for v in prefill.values())
    head = sum(big) / len(big)
    return {"metric": "Q4_K prefill dequant-GEMM TFLOPS (config 3, M=8192, mean of both shapes)",
            "value": round(head, 1), "unit": "TFLOP/s",
            "frac_of_peak": round(head / bf16_peak, 3),
            "peak": bf16_peak, "peak_kind": f"{kind} bf16 dense (MEASURED_PEAKS.json bf16_tflops)",
            "best": best, "per_shape": prefill, "device_status": status,
            "dtype": "bf16 x bf16(dequantized Q4_K) -> fp32 accumulate -> bf16"}


def gemm_roofline(prefill_sum, short=False, sustained_run=None):
    """The metric's second half as a roofline object: config 3's dequant-GEMM
    (gemm_q4k_tc) at M = 8192, mean of both shapes, against the measured
    dense bf16 peak; per-M figures beside it."""
    if not prefill_sum or "value" not in prefill_sum:
        return prefill_sum
    per = prefill_sum["per_shape"]
    per_m = {}
    for m in PREFILL_M:
        v = [r["tflops"] for kk, r in per.items() if kk.endswith(f"_m{m}")]
        per_m[str(m)] = round(sum(v) / len(v), 1)
    out = {"bound": "tensor", "kernel": "gemm_q4k_tc (tcgen05, TMEM accumulator), config 3",
           "achieved": prefill_sum["value"], "peak": prefill_sum["peak"], "unit": "TFLOP/s",
           "frac": prefill_sum["frac_of_peak"], "tflops_per_M": per_m}
    if not short:
        sustained = peaks_sustained()
        if sustained:
            # the same number against the cuBLAS GEMM measured back to back for
            # seconds (power-capped clocks), for context; `frac` stays on burst
            out["frac_of_sustained"] = round(prefill_sum["value"] / sustained, 3)
            out["peak_sustained"] = sustained
        if sustained_run:
            out["sustained_2s"] = sustained_run
        out.update({"peak_kind": prefill_sum["peak_kind"], "traffic": gemm_traffic_from_profiles(),
                    "traffic_case": "14336x4096, M=8192 (one ncu capture, profiles/gemm_q4k_prefill.md)",
                    "flops_per_launch": "2*M*N*K (M=8192: 962.1 GFLOP per shape)",
                    "device_status": prefill_sum.get("device_status")})
    return out


def gemm_traffic_from_profiles():
    """dram bytes per launch of the config-3 GEMM from profiles/gemm_q4k_prefill.md
    (line 'traffic_bytes_per_launch: N'), or None."""
    p = os.path.join(ROOT, "profiles", "gemm_q4k_prefill.md")
    if not os.path.exists(p):
        return None
    for ln in open(p):
        if ln.startswith("traffic_bytes_per_launch:"):
            try:
                return int(ln.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


def traffic_from_profiles():
    """dram bytes per launch of the dominant kernel from the committed ncu
    summary (profiles/gemv_q4k_decode.md, line 'traffic_bytes_per_launch: N')."""
    p = os.path.join(ROOT, "profiles", "gemv_q4k_decode.md")
    if not os.path.exists(p):
        return None
    for ln in open(p):
        if ln.startswith("traffic_bytes_per_launch:"):
            try:
                return int(ln.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


def run_ncu_probe():
    """Five grouped gate+up launches (2 x 14336x4096 Q4_K, 66 MB), the bench's
    dominant kernel, on one layer copy: the small case for ncu captures."""
    import torch
    from xwfes_b200 import ftc
    dev = torch.device("cuda", 0)
    ws = [torch.from_numpy(S.weight(F.Q4_K, 14336, 4096, seed=0, name=f"L0.{m}")).to(dev)
          for m in ("gate", "up")]
    x = torch.from_numpy(S.activations_f32(1, 4096, seed=0, name="ffn_in")).to(dev)
    for _ in range(5):
        ys = ftc.mul_mat_vec_multi(ws, F.Q4_K, [14336, 14336], 4096, x)
    torch.cuda.synchronize()
    print(json.dumps({"probe": "gemv_q4k_dp4a gate+up 2x14336x4096 x5", "y0": float(ys[0][0, 0])}))
    return 0


def run_ncu_imma_probe():
    """Three batch-4 grouped gate+up launches (2 x 14336x4096 Q4_K, 66 MB, 4
    tokens): the small case for ncu captures of the integer tensor-core GEMV
    (gemv_q4k_imma)."""
    import torch
    from xwfes_b200 import ftc
    dev = torch.device("cuda", 0)
    ws = [torch.from_numpy(S.weight(F.Q4_K, 14336, 4096, seed=0, name=f"L0.{m}")).to(dev)
          for m in ("gate", "up")]
    x = torch.from_numpy(S.activations_f32(4, 4096, seed=0, name="ffn_in")).to(dev)
    for _ in range(3):
        ys = ftc.mul_mat_vec_multi(ws, F.Q4_K, [14336, 14336], 4096, x)
    torch.cuda.synchronize()
    print(json.dumps({"probe": "gemv_q4k_imma gate+up 2x14336x4096 M=4 x3", "y0": float(ys[0][0, 0]),
                      "status": ftc.device_status()}))
    return 0


def run_ncu_gemm_probe():
    """Three config-3 dequant-GEMM launches at the roofline's M = 8192 (W 33 MB,
    X 67 MB, Y 235 MB on the device, ~0.9 ms each): the case for ncu captures
    of the tensor-core kernel."""
    import torch
    from xwfes_b200 import ftc
    dev = torch.device("cuda", 0)
    n, k, m = 14336, 4096, 8192
    w = torch.from_numpy(S.weight(F.Q4_K, n, k, seed=0, name=f"p.{n}x{k}")).to(dev)
    x = torch.from_numpy(S.activations_bf16(m, k, seed=0, name=f"p.{m}")).to(dev).view(
        torch.bfloat16)
    y = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    for _ in range(3):
        ftc.gemm(w, F.Q4_K, n, k, x, y=y, y_dtype=F.BF16)
    torch.cuda.synchronize()
    print(json.dumps({"probe": "gemm_q4k_tc 14336x4096 M=8192 x3", "status": ftc.device_status()}))
    return 0


def run_ncu_q6k_probe():
    """Three batch-1 GEMVs of config 2's Q6_K output head (128256 x 4096,
    431 MB on the device, larger than L2): the case for ncu captures of the
    dp4a kernel on Q6_K rows."""
    import torch
    from xwfes_b200 import ftc
    dev = torch.device("cuda", 0)
    n, k = 128256, 4096
    w = torch.from_numpy(S.weight(F.Q6_K, n, k, seed=0, name="q6k.head")).to(dev)
    x = torch.from_numpy(S.activations_f32(1, k, seed=0, name="q6k.x")).to(dev)
    y = torch.empty((1, n), dtype=torch.float32, device=dev)
    for _ in range(3):
        ftc.mul_mat_vec(w, F.Q6_K, n, k, x, y=y)
    torch.cuda.synchronize()
    print(json.dumps({"probe": "gemv_q4k_dp4a on Q6_K 128256x4096 x3", "status": ftc.device_status()}))
    return 0


def run_ncu_attention_probe():
    """Three ftc_attention launches (split kernel + combine each): one decode
    row of Llama-3-8B heads over 32768 positions, K and V 134 MB each on the
    device: the case for ncu captures of attn_split."""
    import torch
    from xwfes_b200 import ftc
    dev = torch.device("cuda", 0)
    nh, nkv, hd, n = 32, 8, 128, 32768
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    k = torch.randn((n, nkv * hd), device=dev, generator=g)
    v = torch.randn((n, nkv * hd), device=dev, generator=g)
    q = torch.randn((1, nh * hd), device=dev, generator=g)
    for _ in range(3):
        ftc.attention(q, nh, nkv, hd, k[n - 1:], v[n - 1:], base=n - 1, k_cache=k, v_cache=v)
    torch.cuda.synchronize()
    print(json.dumps({"probe": "attn_split 32 q / 8 kv heads x 128, 32768 positions x3",
                      "status": ftc.device_status()}))
    return 0


def run_ncu_gemm_split_probe():
    """Three dequant-GEMM launches on a tensor-parallel rank's shape (the
    stacked q/k/v shard of config 4 at 8 GPUs: 1280 x 8192 Q4_K, 16 tokens,
    fp16 row-scaled operands): 10 output tiles, so each tile's K range is cut
    into pieces on several SMs and the partials are summed by the last piece
    of each tile."""
    import torch
    from xwfes_b200 import ftc
    dev = torch.device("cuda", 0)
    n, k, m = 1280, 8192, 16
    w = torch.from_numpy(S.weight(F.Q4_K, n, k, seed=0, name=f"p.{n}x{k}")).to(dev)
    x = torch.from_numpy(S.activations_f32(m, k, seed=0, name=f"p.s{m}")).to(dev)
    x16, e = ftc.rows_to_f16(x)
    y = torch.empty((m, n), dtype=torch.float32, device=dev)
    for _ in range(3):
        ftc.gemm_rowscaled(w, F.Q4_K, n, k, x16, e, y=y)
    torch.cuda.synchronize()
    print(json.dumps({"probe": "gemm_q4k_tc cut tiles 1280x8192 M=16 x3",
                      "status": ftc.device_status()}))
    return 0


def run_down_axpy(reps=50):
    """The engine's neuron-major down projection (ftc_matmul_down_axpy) on the
    Llama-3-8B dense down shape, n_ff = 14336 rows of 4096 Q4_K weights, at 1
    and 8 tokens: 4 weight copies rotated (132 MB > L2), CUDA events.  Prints
    one JSON line; also the small case for an ncu capture (-k regex:rows_axpy)."""
    import torch
    from xwfes_b200 import ftc
    dev = torch.device("cuda", 0)
    n_in, n = 14336, 4096
    ws = [torch.from_numpy(S.weight(F.Q4_K, n_in, n, seed=c, name="axpy")).to(dev)
          for c in range(4)]
    hbm, _, kind = peaks()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    out = {}
    for m in (1, 8):
        x = torch.from_numpy(S.activations_f32(m, n_in, seed=0, name="axpy.x")).to(dev)
        y = torch.zeros((m, n), dtype=torch.float32, device=dev)
        need = ftc.lib().ftc_matmul_down_axpy_workspace_bytes(F.Q4_K, n_in, n, m)
        scratch = torch.empty(max(need, 1), dtype=torch.uint8, device=dev)
        for i in range(3):
            ftc.matmul_down_axpy(ws[i % 4], F.Q4_K, n_in, n, x, y, ws=scratch)
        torch.cuda.synchronize()
        ev0.record()
        for i in range(reps):
            ftc.matmul_down_axpy(ws[i % 4], F.Q4_K, n_in, n, x, y, ws=scratch)
        ev1.record()
        torch.cuda.synchronize()
        us = ev0.elapsed_time(ev1) * 1e3 / reps
        b = n_in * F.row_bytes(F.Q4_K, n) + 4 * m * (n_in + 2 * n)
        out[str(m)] = {"us": round(us, 2), "GBps": round(b / (us * 1e-6) / 1e9, 1),
                       "frac": round(b / (us * 1e-6) / 1e9 / hbm, 3), "bytes": b,
                       "workspace_bytes": need}
    print(json.dumps({"probe": "ftc_matmul_down_axpy 14336 rows x 4096 Q4_K", "peak": hbm,
                      "peak_kind": kind, "per_M": out, "status": ftc.device_status()}))
    return 0


# ----------------------------------------------------------- CPU baselines

def cpu_port_run(threads, warmup, steps=None, budget_s=15.0, max_s=150.0):
    """The CPU port of CpuBackend::matmul (oracle) on config 2 with ``threads``
    host threads.  One step = the seven GEMVs of one Llama-3-8B Q4_K layer, or,
    when ``steps`` layers would take longer than ``max_s``, one of the seven
    (in rotation) so the run stays bounded.  ``steps`` None: as many layer
    steps as fit in about ``budget_s``.  Per-step times are taken one by one;
    the rate uses their median (host noise shows in min / max)."""
    from oracle import oracle as O
    L = make_weights(seed=0)[0]
    xs = {nm: S.activations_f32(1, ln, seed=0, name=nm) for nm, ln in X_LEN.items()}
    gemv_bytes = {name: F.row_bytes(F.Q4_K, k) * n + 4 * (n + k) for name, n, k in LAYER}

    def gemv(name, k):
        O.matmul(xs[X_OF[name]], L[name], F.Q4_K, k, threads=threads)

    def layer():
        for name, _, k in LAYER:
            gemv(name, k)
        return sum(gemv_bytes.values())

    for _ in range(max(1, warmup)):
        layer()
    t = time.perf_counter()
    layer()
    t1 = time.perf_counter() - t
    if steps is None:
        steps = max(3, int(budget_s / max(t1, 1e-3)))
    per_gemv = steps * t1 > max_s
    times, nbytes = [], []
    for i in range(steps):
        t = time.perf_counter()
        if per_gemv:
            name, _, k = LAYER[i % len(LAYER)]
            gemv(name, k)
            nbytes.append(gemv_bytes[name])
        else:
            nbytes.append(layer())
        times.append(time.perf_counter() - t)
    rates = sorted(b / t / 1e9 for b, t in zip(nbytes, times))
    return {"gbs": statistics.median(rates), "gbs_min": rates[0], "gbs_max": rates[-1],
            "steps": steps, "ms_per_step": 1e3 * statistics.median(times),
            "step": "one GEMV of the layer, in rotation" if per_gemv else
                    "one Llama-3-8B Q4_K layer (7 GEMVs)"}


def reference_q8_0_config1(threads):
    """The reference's own CpuBackend::matmul (oracle/_ref) on config 1, with
    all host threads and with one."""
    from oracle import oracle as O
    if not O.have_ref():
        return None
    w = S.weight(F.Q8_0, 4096, 4096, seed=0, name="c1")
    x = S.activations_f32(1, 4096, seed=0, name="c1")
    out = {}
    for th in sorted({threads, 1}, reverse=True):
        O.ref_matmul(x, w, F.Q8_0, 4096, threads=th)
        reps = 20
        t = time.perf_counter()
        for _ in range(reps):
            O.ref_matmul(x, w, F.Q8_0, 4096, threads=th)
        dt = (time.perf_counter() - t) / reps
        out[th] = w.nbytes / dt / 1e9
    return {"value": round(out[threads], 3), "unit": "GB/s", "cores": threads,
            "value_1_thread": round(out[1], 3), "kind": "reference",
            "sample": "config 1: Q8_0 4096x4096 GEMV, 20 calls per thread count"}


def reference_expert_chunk_q8_0(threads):
    """The reference's own CpuBackend::run_expert_chunk (oracle/_ref) on the
    Q8_0 variant of config 5 (the reference has no Q4_K decoder): one window
    of 1280 neurons -- the window ExpertStreamer::auto_chunk picks for the
    16 MiB staging budget, ft/include/ft/chunker.h:81-89 -- of one expert
    (4096 x 14336 shapes) with 16 tokens (T = 64, top-2, 8 experts: 16 rows
    per expert on average); all host threads and one."""
    from oracle import oracle as O
    if not O.have_ref():
        return None
    K, IC, M = 4096, 1280, 16
    g, u, d = (S.weight(F.Q8_0, IC, K, seed=0, name=f"c5q8.{nm}") for nm in ("gate", "up", "down"))
    x = S.activations_f32(M, K, seed=0, name="c5q8.x")
    wb = g.nbytes + u.nbytes + d.nbytes
    per = {}
    for th in sorted({threads, 1}, reverse=True):
        out = np.zeros((M, K), dtype=np.float32)
        O.ref_expert_chunk(x, out, g, u, d, F.Q8_0, K, IC, threads=th)
        reps = 3
        t = time.perf_counter()
        for _ in range(reps):
            O.ref_expert_chunk(x, out, g, u, d, F.Q8_0, K, IC, threads=th)
        per[th] = (time.perf_counter() - t) / reps
    windows = 8 * -(-14336 // IC)  # every expert holds tokens at T = 64
    return {"s_per_window": round(per[threads], 4), "s_per_window_1_thread": round(per[1], 4),
            "weight_GBps": round(wb / per[threads] / 1e9, 3), "cores": threads,
            "layer_s_at_T64": round(windows * per[threads], 2),
            "tokens_per_s_at_T64": round(64 / (windows * per[threads]), 2),
            "kind": "reference",
            "sample": f"one run_expert_chunk window: Q8_0, K=4096, IC={IC}, M={M}, 3 calls per "
                      "thread count; layer time = 8 experts x 12 windows of it"}


def run_reference(args):
    """--impl reference: the reference's CPU path on this host's cores.  The
    reference cannot run Q4_K (no decoder), so the timed arm is the port of
    its CpuBackend::matmul (same row split, dot_row_f32 arithmetic) over the
    same Q4_K layer; its own Q8_0 number is reported beside it."""
    threads = os.cpu_count() or 1
    r = cpu_port_run(threads, args.warmup, steps=args.steps)
    gbs = r["gbs"]
    steps = args.steps
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": round(gbs, 3),
        "unit": "GB/s",
        "n_gpus": args.gpus,
        "steps": steps,
        "warmup": args.warmup,
        "ms_per_step": round(r["ms_per_step"], 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded Q4_K blocks and N(0,1) fp32 activations, config 2 distributions)",
        "config": CONFIG,
        "step": {"parallelism": f"{threads} host threads", "sample": r["step"]},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "gbs_min": round(r["gbs_min"], 3), "gbs_max": round(r["gbs_max"], 3),
                         "sample": f"{r['step']} per step, median of per-step rates; the "
                                   "reference has no Q4_K decoder, so this is the oracle port "
                                   "of its CpuBackend::matmul"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "reference_q8_0_config1": reference_q8_0_config1(threads),
        "reference_expert_chunk_q8_0_config5": reference_expert_chunk_q8_0(threads),
    }


# ------------------------------------------------------------------- main

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=4000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ncu", action="store_true",
                    help="profiling mode: a few launches of the dominant kernel "
                         "(grouped gate+up Q4_K GEMV) on one layer copy, no timing")
    ap.add_argument("--ncu-imma", action="store_true",
                    help="profiling mode: three batch-4 grouped gate+up launches of the integer "
                         "tensor-core GEMV (2 x 14336x4096), no timing")
    ap.add_argument("--ncu-gemm-split", action="store_true",
                    help="profiling mode: three dequant-GEMM launches with cut tiles on a TP rank's "
                         "q/k/v shard (1280x8192, M=16), no timing")
    ap.add_argument("--ncu-gemm", action="store_true",
                    help="profiling mode: three launches of the config-3 dequant-GEMM "
                         "(14336x4096, M=8192, bf16), no timing")
    ap.add_argument("--ncu-q6k", action="store_true",
                    help="profiling mode: three batch-1 GEMVs of config 2's Q6_K output head "
                         "(128256x4096, 431 MB), no timing")
    ap.add_argument("--ncu-attention", action="store_true",
                    help="profiling mode: three ftc_attention launches, one decode row over a "
                         "32768-position fp32 KV cache (Llama-3-8B heads), no timing")
    ap.add_argument("--down-axpy", action="store_true",
                    help="time the neuron-major down projection (ftc_matmul_down_axpy) alone "
                         "and print one JSON line; also the case for ncu captures of rows_axpy")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.ncu:
        return run_ncu_probe()
    if args.ncu_imma:
        return run_ncu_imma_probe()
    if args.ncu_gemm:
        return run_ncu_gemm_probe()
    if args.ncu_gemm_split:
        return run_ncu_gemm_split_probe()
    if args.ncu_attention:
        return run_ncu_attention_probe()
    if args.ncu_q6k:
        return run_ncu_q6k_probe()
    if args.down_axpy:
        return run_down_axpy()

    if args.impl == "reference":
        if rank != 0:
            return 0
        print(json.dumps(run_reference(args)), flush=True)
        return 0

    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    line = run_ours(args, rank, world, local_rank)
    if rank == 0 and line is not None:
        if world == 1 and not args.no_cpu_baseline:
            threads = os.cpu_count() or 1
            r = cpu_port_run(threads, warmup=2)
            line["cpu_baseline"] = {
                "value": round(r["gbs"], 3), "unit": "GB/s", "cores": threads, "kind": "port",
                "gbs_min": round(r["gbs_min"], 3), "gbs_max": round(r["gbs_max"], 3),
                "sample": f"{r['step']} x {r['steps']} steps, median {r['ms_per_step']:.1f} ms; "
                          "the reference has no Q4_K decoder, so this is the oracle port of "
                          "its CpuBackend::matmul"}
            ref = reference_q8_0_config1(threads)
            if ref:
                line["reference_q8_0_config1"] = ref
            ref = reference_expert_chunk_q8_0(threads)
            if ref:
                line["reference_expert_chunk_q8_0_config5"] = ref
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
