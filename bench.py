"""Benchmark of the B200 MoE hot path (BASELINE.json metric: MoE-layer tokens/s, achieved HBM GB/s and %
of roofline).

Default workload: one decode step = T=1 token through all 58 DeepSeek-R1 MoE layers on
one B200, every layer's 256 IQ2_XXS experts + shared expert + router resident in HBM (58 distinct layers,
~170 GB; a step streams ~6.35 GB of weights, far above the 126 MB L2, so no flush is needed between steps).
Each layer takes its own seeded N(0,1) fp32 input row and residual; layers run back to back on one stream,
captured as one CUDA graph per step.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload decode|prefill|imbalance] [--impl ours|reference]

N > 1 (torchrun): expert parallelism: rank r holds experts [r*256/N, (r+1)*256/N) of
every layer (plus router and shared expert), and each rank decodes its own token (weak scaling: T=1 per
GPU); per layer the rows go to the expert owners and the partial sums come back through two all-to-alls
(the library's NCCL communicator, captured in the step's CUDA graph).  value = tokens of all ranks /
max-over-ranks time.  `--parallelism replicas` runs N independent single-GPU replicas instead.
`--workload prefill --tokens 4096` at N > 1 is BASELINE config 3 (expert-parallel batch, T global).
--impl reference times the CPU oracle (the restatement of the reference's CPU path) on the host cores on a
bounded sample.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

N_LAYERS = 58
SEED = 0x10C1
HIDDEN, INTER, NE = 7168, 2048, 256
MAT = INTER * (HIDDEN // 256) * 66                       # 3 784 704 bytes per expert matrix
ROUTER_BYTES = NE * HIDDEN * 4
DOWN_FMTS = {"iq2": (4, 66), "q2k": (5, 84), "q3k": (6, 110)}   # --down-fmt: format id, bytes per 256-weight block


def down_bytes(args):
    """Bytes of one expert's down matrix in the decode workload's down format."""
    return HIDDEN * (INTER // 256) * DOWN_FMTS[args.down_fmt][1]


FMT_Q5K = 3                                              # --shared-fmt q5k: Q5_K gate/up + Q6_K down (the real model's)
SH_MODEL_BYTES = 2 * INTER * (HIDDEN // 256) * 176 + HIDDEN * (INTER // 256) * 210   # 32 227 328


def shared_bytes(args):
    """Bytes of the shared expert's three matrices in the decode workload."""
    return SH_MODEL_BYTES if args.shared_fmt == "q5k" else 2 * MAT + down_bytes(args)


# DeepSeek-R1 routing (inherited by configs 1-4): 8 groups of 32 experts, top 4 groups
N_GROUP, TOPK_GROUP = 8, 4


NOMINAL_HBM_GBS = 7700.0     # HBM3e nominal (HGX B200); frac is against the measured copy bandwidth


def measured_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


def ncu_traffic(kernel, workload):
    """Per-launch DRAM bytes of `kernel` from the committed ncu summary (profiles/ncu_traffic.txt), or None."""
    p = os.path.join(REPO, "profiles", "ncu_traffic.txt")
    if not os.path.exists(p):
        return None
    for line in open(p):
        f = line.split()
        if len(f) >= 3 and not line.startswith("#") and f[0] == kernel and f[1] == workload:
            return float(f[2])
    return None


class DriverEvents:
    """Timing events created through the CUDA driver API: the library records them on its launch stream
    (also inside graph capture), and elapsed times are read with cuEventElapsedTime."""

    def __init__(self, n):
        import ctypes
        self.ct = ctypes
        self.cu = ctypes.CDLL("libcuda.so.1")
        self.ev = [ctypes.c_void_p() for _ in range(n)]
        for e in self.ev:
            rc = self.cu.cuEventCreate(ctypes.byref(e), 0)
            if rc != 0:
                raise RuntimeError("cuEventCreate failed: %d" % rc)

    def elapsed(self, a, b):
        ms = self.ct.c_float()
        rc = self.cu.cuEventElapsedTime(self.ct.byref(ms), self.ev[a], self.ev[b])
        if rc != 0:
            raise RuntimeError("cuEventElapsedTime failed: %d" % rc)
        return ms.value


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu):
        self.gpu, self.proc, self.lines = gpu, None, []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.Q, "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1])); mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ distributed plumbing
def dist_setup(args):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def dist_init(ws, local):
    import torch
    import torch.distributed as dist
    if ws > 1 and not dist.is_initialized():
        from datetime import timedelta
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
    return dist if ws > 1 else None


def barrier(dist):
    import torch
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(dist, v):
    import torch
    if dist is None:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------ CPU baseline (oracle)
def cpu_layer(O, L, keep=8, seed=SEED):
    """Layer L of the CPU decode workload, set up outside any timed region (the GPU arm's weights are resident
    too): its seeded input row, residual, router weights and bias, and the IQ2_XXS weights of the experts its
    token selects plus the shared expert."""
    rng = np.random.default_rng(seed + L)
    x = rng.standard_normal((1, HIDDEN)).astype(np.float32)
    r = rng.standard_normal((1, HIDDEN)).astype(np.float32)
    W = (rng.standard_normal((NE, HIDDEN)) * 0.02).astype(np.float32)
    bias = (rng.standard_normal(NE) * 0.01).astype(np.float32)
    cfg = O.route_cfg(8, keep, 1, N_GROUP, TOPK_GROUP)
    _, sel, _ = O.router(x, W, bias, cfg)
    used = sorted(set(int(e) for e in sel[0]))
    remap = {e: i for i, e in enumerate(used)}
    ids = np.array([[remap[int(e)] for e in sel[0]]], np.int32)
    gate = np.concatenate([O.gen_iq2(seed, L, 0, e, INTER, HIDDEN) for e in used])
    up = np.concatenate([O.gen_iq2(seed, L, 1, e, INTER, HIDDEN) for e in used])
    down = np.concatenate([O.gen_iq2(seed, L, 2, e, HIDDEN, INTER) for e in used])
    sh = [O.gen_iq2(seed, L, m, 256, *((INTER, HIDDEN) if m < 2 else (HIDDEN, INTER))) for m in range(3)]
    return dict(x=x, r=r, W=W, bias=bias, cfg=cfg, ids=ids, gate=gate, up=up, down=down, sh=sh)


def cpu_layer_forward(O, lay):
    """One T=1 layer on the CPU oracle: router (sigmoid, grouped top-8, weights) + experts + combine."""
    _, _, w = O.router(lay["x"], lay["W"], lay["bias"], lay["cfg"])
    O.moe_layer(lay["x"], lay["r"], lay["gate"], lay["up"], lay["down"], MAT, lay["ids"], w, *lay["sh"])


def cpu_cores():
    return int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))


def cpu_decode_sample(n_layers, keep=8, seed=SEED):
    """Time the CPU oracle on T=1 decode for n_layers layers (router + experts + combine); returns
    (seconds per layer, cores).  Weights for the selected experts are generated before the clock starts."""
    from oracle import oracle as O
    O.build()
    times = []
    for L in range(n_layers):
        lay = cpu_layer(O, L, keep, seed)
        t0 = time.perf_counter()
        cpu_layer_forward(O, lay)
        times.append(time.perf_counter() - t0)
    return float(np.mean(times)), cpu_cores()


# ------------------------------------------------------------------ decode workload (config 1)
def decode_config(args, ws, distinct, fmt=4, model_sh=False, layer_bytes=None):
    """The config object of the decode line (both arms)."""
    if layer_bytes is None:
        layer_bytes = args.keep * (2 * MAT + down_bytes(args)) + shared_bytes(args) + ROUTER_BYTES + 3 * 4 * HIDDEN
    return {"workload": ("config1_decode_T1_58layers" if fmt == 4 else "decode_T1_58layers_%s_down" % args.down_fmt) +
                        ("_q5k_q6k_shared" if model_sh else ""),
            "model": ("DeepSeek-R1 MoE layer (IQ2_XXS, 256 experts + shared)" if fmt == 4 else
                      "DeepSeek-R1 MoE layer (IQ2_XXS gate/up, %s down as in the real model, 256 experts + shared)" % args.down_fmt) +
                     ("; shared expert Q5_K gate/up + Q6_K down as in the real model" if model_sh else ""),
            "global_batch": ws, "seq_len": 1, "layers": args.layers, "distinct_layers_resident": distinct,
            "top_k": 8, "n_group": N_GROUP, "topk_group": TOPK_GROUP, "keep": args.keep,
            "parallelism": "replicas" if ws > 1 else "single",
            "l2": "no flush: a step streams %.2f GB of distinct weights (> 126 MB L2)" % (args.layers * layer_bytes / 1e9)}


def build_decode(dev, n_layers, keep, fmt=4, ds=MAT, sh_fmt=4, sh_bytes=None):
    import torch
    from loki_b200 import moe as M
    free, total = torch.cuda.mem_get_info(dev)
    per_layer = 2 * NE * MAT + NE * ds + (2 * MAT + ds if sh_bytes is None else sh_bytes) + ROUTER_BYTES
    fit = int((free - (6 << 30)) // per_layer)
    distinct = max(1, min(n_layers, fit))
    layers = [M.LayerWeights(dev, SEED, L, down_fmt=fmt, sh_fmt=sh_fmt) for L in range(distinct)]
    torch.cuda.synchronize(dev)
    return layers, distinct


def run_decode(args, ws, rank, local, dist):
    import torch
    import ctypes
    from loki_b200 import moe as M
    from loki_b200 import native as N
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    fmt, DS = DOWN_FMTS[args.down_fmt][0], down_bytes(args)
    model_sh = args.shared_fmt == "q5k"
    SHB = shared_bytes(args)
    layers, distinct = build_decode(dev, args.layers, args.keep, fmt, DS, FMT_Q5K if model_sh else 4, SHB)
    layer_of = [L % distinct for L in range(args.layers)]
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    xs = torch.randn(args.layers, 1, HIDDEN, device=dev, generator=g)
    rs = torch.randn(args.layers, 1, HIDDEN, device=dev, generator=g)
    hs = torch.empty(args.layers, 1, HIDDEN, device=dev)
    mos = torch.empty(args.layers, 1, HIDDEN, device=dev)
    ctx = M.MoeLayer(local, keep=args.keep, max_tokens=1, n_group=N_GROUP, topk_group=TOPK_GROUP)
    structs = [l.struct() for l in layers]
    L = N.lib()
    stream = torch.cuda.Stream(dev)

    def step(events=None):
        s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        for i in range(args.layers):
            if events is not None:
                arr = (ctypes.c_void_p * 4)(*[events.ev[4 * i + j].value for j in range(4)])
                L.lk_moe_set_events(ctx.ctx, arr)
            rc = L.lk_moe_forward(ctx.ctx, ctypes.byref(structs[layer_of[i]]), ctypes.c_void_p(xs[i].data_ptr()),
                                  ctypes.c_void_p(rs[i].data_ptr()), 1, None, ctypes.c_void_p(hs[i].data_ptr()),
                                  ctypes.c_void_p(mos[i].data_ptr()), None, None, s)
            N.check(rc, ctx.ctx)
        if events is not None:
            L.lk_moe_set_events(ctx.ctx, None)

    # warm-up eager (sets kernel attributes, first-touch), then capture one step as a graph
    with torch.cuda.stream(stream):
        step()
    torch.cuda.synchronize(dev)
    ctx.device_error()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    ev = DriverEvents(4 * args.layers)
    graph_ev = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph_ev, stream=stream):
        step(ev)
    torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        graph.replay()
    barrier(dist)
    clocks = ClockSampler(local) if rank == 0 else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    barrier(dist)
    with torch.cuda.stream(stream):
        t0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        t1.record(stream)
    barrier(dist)
    ms = t0.elapsed_time(t1)
    # per-kernel pass: the same step with events around each layer's gate/up, down and combine launches
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.steps // 4)):
            graph_ev.replay()
    torch.cuda.synchronize(dev)
    cl = clocks.stop() if clocks else None
    ctx.device_error()
    gu = np.array([ev.elapsed(4 * i, 4 * i + 1) for i in range(args.layers)])
    dn = np.array([ev.elapsed(4 * i + 1, 4 * i + 2) for i in range(args.layers)])
    cb = np.array([ev.elapsed(4 * i + 2, 4 * i + 3) for i in range(args.layers)])
    ms_max = max_over_ranks(dist, ms)
    tokens = args.steps * ws
    value = tokens / (ms_max / 1e3)
    hbm, bf16, peak_kind = measured_peaks()
    n_slots = args.keep + (0 if model_sh else 1)                     # the model-format shared expert has own launches
    gu_bytes = n_slots * 2 * MAT + 4 * HIDDEN                       # routed (+ IQ2_XXS shared) gate/up rows, x in
    dn_bytes = n_slots * DS + n_slots * (INTER + INTER // 32 * 4) + n_slots * HIDDEN * 4
    layer_bytes = args.keep * (2 * MAT + DS) + SHB + ROUTER_BYTES + 3 * 4 * HIDDEN
    gu_ms = float(gu.mean())
    achieved = gu_bytes / (gu_ms / 1e3) / 1e9
    traffic = ncu_traffic("k_gate_up", "decode_T1")
    out = {
        "metric": "MoE-layer tokens/s (T=1 decode through 58 layers)", "value": round(value, 2), "unit": "tokens/s",
        "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": ("iq2_xxs x q8 (int8 dp4a, fp32 accumulate)" if fmt == 4 else
                  "iq2_xxs gate/up, %s down x q8 (int8 dp4a, fp32 accumulate)" % args.down_fmt) +
                 ("; shared expert q5_k/q6_k x q8" if model_sh else ""),
        "data": "synthetic: seeded IQ2_XXS experts (BASELINE config 0 generator), router W N(0,0.02), bias N(0,0.01), x/resid N(0,1) fp32",
        "config": decode_config(args, ws, distinct, fmt, model_sh, layer_bytes),
        "layer": {"ms_per_layer": round(ms_max / args.steps / args.layers * 1e3, 3), "unit_ms_per_layer": "us",
                  "bytes_per_layer": layer_bytes,
                  "achieved_gbs": round(layer_bytes * args.layers * args.steps / (ms_max / 1e3) / 1e9, 1),
                  "frac_of_hbm": round(layer_bytes * args.layers * args.steps / (ms_max / 1e3) / 1e9 / hbm, 4),
                  # per-kernel times come from a second capture with event nodes between the kernels, which
                  # serialise them; in the timed graph each kernel's prologue overlaps its predecessor
                  # (programmatic dependent launch), so "rest" (layer minus the two) can be negative.  With the
                  # model-format shared expert its two launches (before the routed ones) fall into "rest".
                  "kernel_us_event_graph": {"gate_up": round(gu_ms * 1e3, 2), "down_combine": round(float(dn.mean()) * 1e3, 2),
                                            "rest": round(ms_max / args.steps / args.layers * 1e3 - gu_ms * 1e3 - float(dn.mean()) * 1e3, 2)}},
        "roofline": {"kernel": "k_gate_up<1> (routed + shared gate/up + SwiGLU + q8)" if not model_sh else
                               "k_gate_up<1> (routed gate/up + SwiGLU + q8)", "bound": "hbm",
                     "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 4),
                     "traffic": traffic, "algorithmic_bytes_per_launch": gu_bytes, "peak_source": peak_kind,
                     "frac_of_nominal_7700": round(achieved / NOMINAL_HBM_GBS, 4),
                     "down_kernel_frac": round(dn_bytes / (float(dn.mean()) / 1e3) / 1e9 / hbm, 4)},
        # per layer: router (+top-k), gate/up, down, combine (+ the model-format shared expert's gate/up and down)
        "gpu_launches": args.steps * args.layers * (6 if model_sh else 4),
    }
    if cl:
        out["clocks"] = cl
    return out, layers, ctx, structs, xs, rs


def _min_over_ranks(dist, v):
    import torch
    if dist is None:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return float(t.item())


def _ep_setup(args, ws, rank, local, dist, max_local_tokens, layers_wanted, p2p_cap=0):
    import torch
    from loki_b200 import moe as M
    from loki_b200.ep import EpMoeLayer, NativeEpOps, NativeComm, P2PExchange
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    E = NE // ws
    free, _ = torch.cuda.mem_get_info(dev)
    per_layer = (3 * E + 3) * MAT + ROUTER_BYTES
    distinct = int(_min_over_ranks(dist, max(1, min(layers_wanted, int((free - (10 << 30)) // per_layer)))))
    shards = [M.LayerWeights(dev, SEED, L, n_experts=E, expert0=rank * E) for L in range(distinct)]
    comm = NativeComm(local)
    ops = NativeEpOps(local, ws, max_local_tokens, keep=args.keep, n_group=N_GROUP, topk_group=TOPK_GROUP)
    p2p = P2PExchange(local, p2p_cap) if p2p_cap else None
    torch.cuda.synchronize(dev)
    return dev, shards, distinct, comm, ops, EpMoeLayer(comm, ops, p2p=p2p)


def run_ep_decode(args, ws, rank, local, dist):
    """Expert-parallel decode: T=1 token per rank through the layers, experts sharded 256/N per GPU."""
    import torch
    import ctypes
    from loki_b200 import native as N
    dev, shards, distinct, comm, ops, layer = _ep_setup(args, ws, rank, local, dist, 1, args.layers,
                                                        p2p_cap=1 if args.exchange == "p2p" else 0)
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    xs = torch.randn(args.layers, 1, HIDDEN, device=dev, generator=g)
    rs = torch.randn(args.layers, 1, HIDDEN, device=dev, generator=g)
    outs = [None] * args.layers
    L = N.lib()
    ev = DriverEvents(4 * args.layers)

    def step(events=False):
        for i in range(args.layers):
            if events:
                L.lk_moe_set_events(ops.expert.ctx, (ctypes.c_void_p * 4)(*[ev.ev[4 * i + j].value for j in range(4)]))
            outs[i] = layer.forward(shards[i % distinct], xs[i], rs[i])
        if events:
            L.lk_moe_set_events(ops.expert.ctx, None)

    stream = torch.cuda.Stream(dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(stream):
        step()                                     # eager: kernel attributes, NCCL peer connections
    torch.cuda.synchronize(dev)
    ops.device_error()
    graph, graph_ev = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph_ev, stream=stream):
        step(events=True)
    with torch.cuda.graph(graph, stream=stream):       # captured last: `outs` are this graph's outputs
        step()
    torch.cuda.synchronize(dev)
    for _ in range(args.warmup):
        graph.replay()
    barrier(dist)
    clocks = ClockSampler(local) if rank == 0 else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(dist)
    with torch.cuda.stream(stream):
        t0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        t1.record(stream)
    barrier(dist)
    ms = t0.elapsed_time(t1)
    with torch.cuda.stream(stream):
        for _ in range(3):
            graph_ev.replay()
    torch.cuda.synchronize(dev)
    barrier(dist)
    # end to end: pinned host inputs in, every layer's h out, inside the timed region
    hx = torch.empty(args.layers, 2, 1, HIDDEN, pin_memory=True)
    hx.copy_(torch.stack([xs, rs], 1).cpu())
    hout = torch.empty(args.layers, 1, HIDDEN, pin_memory=True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_e2e = max(2, args.steps // 2)
    barrier(dist)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(n_e2e):
            xs.copy_(hx[:, 0], non_blocking=True)
            rs.copy_(hx[:, 1], non_blocking=True)
            graph.replay()
            for i in range(args.layers):
                hout[i].copy_(outs[i][0], non_blocking=True)
        e1.record(stream)
    barrier(dist)
    e2e_ms = max_over_ranks(dist, e0.elapsed_time(e1))
    cl = clocks.stop() if clocks else None
    ops.device_error()
    gu = np.array([ev.elapsed(4 * i, 4 * i + 1) for i in range(args.layers)])
    dn = np.array([ev.elapsed(4 * i + 1, 4 * i + 2) for i in range(args.layers)])
    # distinct local experts each layer's expert stage streamed (all ranks' selections)
    sel = torch.stack([outs[i][2][0] for i in range(args.layers)])              # [layers][keep] this rank's token
    if dist is not None:
        allsel = [torch.empty_like(sel) for _ in range(ws)]
        dist.all_gather(allsel, sel)
        allsel = torch.stack(allsel, 1)                                         # [layers][ws][keep]
    else:
        allsel = sel[:, None]
    E = NE // ws
    loc = [(allsel[i][(allsel[i] // E) == rank]).unique().numel() for i in range(args.layers)]
    gu_bytes = np.array([2 * MAT * n + 4 * HIDDEN * ws for n in loc], np.float64)
    achieved = float(np.mean(gu_bytes / (gu / 1e3))) / 1e9
    ach_all = max_over_ranks(dist, -achieved)
    achieved_min = -ach_all
    ms_max = max_over_ranks(dist, ms)
    value = args.steps * ws / (ms_max / 1e3)
    hbm, bf16, peak_kind = measured_peaks()
    graph.reset()
    graph_ev.reset()
    if layer.p2p is not None:
        layer.p2p.close()
    comm.close()
    out = {
        "metric": "MoE-layer tokens/s (T=1 decode through 58 layers)", "value": round(value, 2), "unit": "tokens/s",
        "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "iq2_xxs x q8 (int8 dp4a, fp32 accumulate)",
        "data": "synthetic: seeded IQ2_XXS experts (BASELINE config 0 generator), router W N(0,0.02), bias N(0,0.01), x/resid N(0,1) fp32",
        "config": {"workload": "config1_decode_T1_58layers_ep", "model": "DeepSeek-R1 MoE layer (IQ2_XXS, 256 experts + shared)",
                   "global_batch": ws, "seq_len": 1, "layers": args.layers, "distinct_layers_resident": distinct,
                   "top_k": 8, "n_group": N_GROUP, "topk_group": TOPK_GROUP, "keep": args.keep, "parallelism": "ep%d" % ws, "experts_per_gpu": E,
                   "exchange": ("peer-memory mailboxes over NVLink (CUDA IPC, flag + bounded wait), in the step's CUDA graph"
                                if args.exchange == "p2p" else
                                "2 all-to-alls per layer (library NCCL communicator, grouped send/recv, in the step's CUDA graph)"),
                   "l2": "no flush: a step streams the selected experts of %d distinct layers (> 126 MB L2)" % distinct},
        "layer": {"ms_per_layer": round(ms_max / args.steps / args.layers * 1e3, 3), "unit_ms_per_layer": "us",
                  "expert_stage_us": {"gate_up": round(float(gu.mean()) * 1e3, 2), "down_combine": round(float(dn.mean()) * 1e3, 2)},
                  "local_experts_per_layer": round(float(np.mean(loc)), 2)},
        "roofline": {"kernel": "k_gate_up (expert-rank gate/up + SwiGLU + q8 on received rows)", "bound": "hbm",
                     "achieved": round(achieved_min, 1), "peak": hbm, "unit": "GB/s", "frac": round(achieved_min / hbm, 4),
                     "traffic": None, "algorithmic_bytes_per_launch": float(np.mean(gu_bytes)), "peak_source": peak_kind,
                     "frac_of_nominal_7700": round(achieved_min / NOMINAL_HBM_GBS, 4),
                     "note": "min over ranks of the mean per-layer achieved bandwidth"},
        "e2e": {"value": round(n_e2e * ws / (e2e_ms / 1e3), 2), "unit": "tokens/s",
                "h2d_bytes_per_step": args.layers * 2 * HIDDEN * 4, "d2h_bytes_per_step": args.layers * HIDDEN * 4,
                "path": "pinned host x/resid -> CUDA-graph step of EpMoeLayer.forward x58 -> pinned host h (stream events)"},
        # per layer (p2p): router + send (one launch), gate/up (with the rows wait + slot tables), down (storing
        # each entry's row in its home mailbox), the combine (publishing the return flags, then waiting for every
        # owner's); with NCCL: router, pack, unpack, gate/up, down, combine, return unpack and the home combine
        # around the library's all-to-alls
        "gpu_launches": args.steps * args.layers * (4 if args.exchange == "p2p" else 8),
    }
    if cl:
        out["clocks"] = cl
    return out


def run_ep_prefill(args, ws, rank, local, dist):
    """expert-parallel batch, T tokens per step in total (T/N per rank), top-8 routing by
    the router (bf16 N(0,1) hidden states), experts sharded 256/N per GPU; compact row exchange (one count
    exchange and host read per step); strong scaling."""
    import torch
    T = args.tokens
    assert T % ws == 0
    Tl = T // ws
    dev, shards, distinct, comm, ops, layer = _ep_setup(args, ws, rank, local, dist, Tl, 1)
    W = shards[0]
    g = torch.Generator(device=dev).manual_seed(4321 + rank)
    x = torch.randn(Tl, HIDDEN, device=dev, generator=g).to(torch.bfloat16).float()
    r = torch.randn(Tl, HIDDEN, device=dev, generator=g).to(torch.bfloat16).float()
    stream = torch.cuda.Stream(dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            out = layer.forward(W, x, r)
    torch.cuda.synchronize(dev)
    ops.device_error()
    barrier(dist)
    clocks = ClockSampler(local) if rank == 0 else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(dist)
    with torch.cuda.stream(stream):
        t0.record(stream)
        for _ in range(args.steps):
            out = layer.forward(W, x, r)
        t1.record(stream)
    barrier(dist)
    ms = t0.elapsed_time(t1)
    cl = clocks.stop() if clocks else None
    ops.device_error()
    ms_max = max_over_ranks(dist, ms)
    sent, got = layer.last_counts
    value = T * args.steps / (ms_max / 1e3)
    hbm, bf16, peak_kind = measured_peaks()
    flops = 2.0 * T * (args.keep + 1) * 3 * HIDDEN * INTER + 2.0 * T * HIDDEN * NE
    comm.close()
    o = {
        "metric": "MoE-layer tokens/s (T=%d expert-parallel batch, one layer)" % T, "value": round(value, 1), "unit": "tokens/s",
        "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "iq2_xxs x q8 activations: gate/up tcgen05 kind::f16 with exact integer weights and hi/lo fp16 activations "
                 "(the reference's group sums), h re-quantised to q8; down tcgen05 fp16; fp32 accumulate; rows exchanged as q8",
        "data": "synthetic: seeded IQ2_XXS experts, router W N(0,0.02), bias N(0,0.01), bf16 N(0,1) hidden states",
        "config": {"workload": "config3_ep_batch_T%d" % T, "global_batch": T, "seq_len": T, "layers": 1, "top_k": 8, "n_group": N_GROUP, "topk_group": TOPK_GROUP,
                   "keep": args.keep, "parallelism": "ep%d" % ws, "experts_per_gpu": NE // ws, "rows_sent": sent,
                   "rows_received": got, "l2": "no flush: each rank streams its %.2f GB shard" % ((3 * NE // ws + 3) * MAT / 1e9)},
        "layer": {"flops": flops, "achieved_tflops": round(flops / (ms_max / args.steps / 1e3) / 1e12, 1),
                  "tensor_frac_of_bf16_peak": round(flops / (ms_max / args.steps / 1e3) / 1e12 / (bf16 * ws), 4)},
        "gpu_launches": args.steps * 12,
    }
    if cl:
        o["clocks"] = cl
    return o


def run_imbalance(args, ws, rank, local, dist):
    """one MoE layer, keep 2 of the top-8 (the reference's --experts 2 mode), T in
    {1, 8, 64, 512}; the router bias makes expert popularity Zipf(1.2)-like with the hottest expert at ~10x
    the mean entry count (lam calibrated by loki_b200.synthetic).  Each step runs on a different seeded layer
    (4 resident) and L2 is flushed (a 256 MB write) between steps outside the timed windows.  N > 1: expert
    parallel, T tokens per rank (weak scaling)."""
    import torch
    from loki_b200 import moe as M
    from loki_b200 import synthetic as S
    from loki_b200.ep import EpMoeLayer, NativeEpOps, NativeComm
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    lam = S.calibrate_zipf_lambda(n_group=N_GROUP, topk_group=TOPK_GROUP)
    bias = torch.from_numpy(S.zipf_bias(lam)).to(dev)
    E = NE // ws
    nl = 4
    layers = [M.LayerWeights(dev, SEED, 100 + L, n_experts=E, expert0=rank * E, router_bias=bias) for L in range(nl)]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    comm = NativeComm(local) if ws > 1 else None
    sweep = {}
    hbm, bf16, peak_kind = measured_peaks()
    for T in (1, 8, 64, 512):
        g = torch.Generator(device=dev).manual_seed(9000 + T + 17 * rank)
        xs = [torch.randn(T, HIDDEN, device=dev, generator=g) for _ in range(nl)]
        rs = [torch.randn(T, HIDDEN, device=dev, generator=g) for _ in range(nl)]
        if ws > 1:
            ops = NativeEpOps(local, ws, T, keep=2, n_group=N_GROUP, topk_group=TOPK_GROUP)
            layer = EpMoeLayer(comm, ops)
            fwd = lambda i: layer.forward(layers[i % nl], xs[i % nl], rs[i % nl])
        else:
            ctx = M.MoeLayer(local, keep=2, max_tokens=T, n_group=N_GROUP, topk_group=TOPK_GROUP)
            fwd = lambda i: ctx.forward(layers[i % nl], xs[i % nl], rs[i % nl])
        for i in range(args.warmup):
            fwd(i)
        torch.cuda.synchronize(dev)
        times, sels = [], []
        for i in range(args.steps):
            flush.fill_(i & 0xFF)
            barrier(dist)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            out = fwd(i)
            b.record()
            torch.cuda.synchronize(dev)
            times.append(a.elapsed_time(b))
            sels.append(out[2].reshape(-1))
        ms = float(np.mean([max_over_ranks(dist, t) for t in times]))
        sel = torch.cat(sels)
        if dist is not None:
            alls = [torch.empty_like(sel) for _ in range(ws)]
            dist.all_gather(alls, sel)
            sel = torch.cat(alls)
        cnt = torch.bincount(sel.long(), minlength=NE).float() / args.steps
        sweep[str(T)] = {"tokens_per_s": round(T * ws / (ms / 1e3), 1), "ms_per_step": round(ms, 4),
                         "hottest_over_mean": round(float(cnt.max() / cnt.mean()), 2),
                         "experts_used": int((cnt > 0).sum()),
                         "path": "tcgen05 GEMM" if T >= 192 else ("mma.sync register-fed" if T >= 48 else "dp4a matvec")}
    if comm is not None:
        comm.close()
    out = {
        "metric": "MoE-layer tokens/s (load-imbalance sweep: keep 2, Zipf-biased router, T=512 headline)",
        "value": sweep["512"]["tokens_per_s"], "unit": "tokens/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": sweep["512"]["ms_per_step"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "iq2_xxs x q8 (dp4a) / fp16 mma.sync / fp16 tcgen05", "data": "synthetic: seeded IQ2_XXS experts, x N(0,1) fp32, Zipf router bias",
        "config": {"workload": "config4_imbalance", "keep": 2, "top_k": 8, "n_group": N_GROUP, "topk_group": TOPK_GROUP, "zipf_s": 1.2, "lambda": round(lam, 5),
                   "parallelism": "ep%d" % ws if ws > 1 else "single", "l2": "flushed (256 MB write) between steps"},
        "sweep": sweep,
    }
    return out


def e2e_decode(args, layers, distinct, keep):
    """Decode through the engine-facing fl_* ABI with host buffers, driven from C++ the way the engine drives
    it (libloki_replay.so lkr_decode): per layer fl_moe_prepare (H2D x/resid, router, shared expert) ->
    fl_moe_auto (keep pass on the device, experts, combine, D2H h/moe).  The engine's unchanged sequence
    (fl_fetch -> host keep pass -> fl_moe) is timed beside it.  Wall clock; every copy and host
    synchronisation is inside the timed region."""
    from loki_b200 import fused as F
    rng = np.random.default_rng(77)
    xs = rng.standard_normal((args.layers, 1, HIDDEN)).astype(np.float32)
    rs = rng.standard_normal((args.layers, 1, HIDDEN)).astype(np.float32)
    per_layer = [layers[i % distinct] for i in range(args.layers)]
    n = max(1, args.steps // 2)
    out = {}
    for device_keep in (True, False):
        fc = F.FusedCtx()
        try:
            sec, _ = F.replay_decode(fc, per_layer, xs, rs, keep, max(1, args.warmup), n, down_fmt=DOWN_FMTS[args.down_fmt][0],
                                     device_keep=device_keep)
            out[device_keep] = (round(n / sec, 2), fc.error())
        finally:
            fc.close()
    h2d = args.layers * (2 * HIDDEN * 4)
    d2h = args.layers * (2 * HIDDEN * 4 + keep * 8)
    return {"value": out[True][0], "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "path": "C++ engine replay (libloki_replay.so): fl_moe_prepare -> fl_moe_auto per layer (pinned host mirrors, "
                    "wall clock)",
            "engine_sequence": {"value": out[False][0], "unit": "tokens/s",
                                "path": "fl_moe_prepare -> fl_fetch -> host keep pass -> fl_moe per layer (the engine's calls "
                                        "unchanged)",
                                "h2d_bytes_per_step": args.layers * (2 * HIDDEN * 4 + keep * 8),
                                "d2h_bytes_per_step": args.layers * (8 * 8 + 2 * HIDDEN * 4 + 2 * HIDDEN * 4)},
            "steps": n, "error": out[True][1] | out[False][1]}


def run_prefill(args, ws, rank, local, dist, W=None, T=None, steps=None, warmup=None):
    """BASELINE config 2 (T=512) and config 3's single-GPU shape (T=4096): one MoE layer, bf16 N(0,1) hidden
    states (fed as fp32), top-8 of 256 experts chosen from uniform-random router logits (the router GEMV still
    runs), the batch regime's kernels (q8 gate/up on tcgen05, IQ2_XXS down on tcgen05), combine with the shared
    expert.  A step = one layer forward.  W: resident layer weights to reuse (default: layer 0 is built)."""
    import torch
    import ctypes
    from loki_b200 import moe as M
    from loki_b200 import native as N
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    T = T or args.tokens
    steps = steps or args.steps
    warmup = max(3, warmup or args.warmup)
    fmt, DS = DOWN_FMTS[args.down_fmt][0], down_bytes(args)
    model_fmt = fmt != 4 or args.shared_fmt == "q5k"
    if W is None:
        W = M.LayerWeights(dev, SEED, 0, down_fmt=fmt, sh_fmt=FMT_Q5K if args.shared_fmt == "q5k" else 4)
    g = torch.Generator(device=dev).manual_seed(4321 + rank)
    x = torch.randn(T, HIDDEN, device=dev, generator=g).to(torch.bfloat16).float()
    r = torch.randn(T, HIDDEN, device=dev, generator=g).to(torch.bfloat16).float()
    logits = torch.rand(T, NE, device=dev, generator=g) * 2 - 1
    h = torch.empty(T, HIDDEN, device=dev)
    mo = torch.empty(T, HIDDEN, device=dev)
    ctx = M.MoeLayer(local, keep=args.keep, max_tokens=T, n_group=N_GROUP, topk_group=TOPK_GROUP)
    st = W.struct()
    L = N.lib()
    stream = torch.cuda.Stream(dev)
    ev = DriverEvents(4)

    def step(events=False):
        s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        if events:
            L.lk_moe_set_events(ctx.ctx, (ctypes.c_void_p * 4)(*[e.value for e in ev.ev]))
        N.check(L.lk_moe_forward(ctx.ctx, ctypes.byref(st), ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(r.data_ptr()), T,
                                 ctypes.c_void_p(logits.data_ptr()), ctypes.c_void_p(h.data_ptr()), ctypes.c_void_p(mo.data_ptr()),
                                 None, None, s), ctx.ctx)
        if events:
            L.lk_moe_set_events(ctx.ctx, None)

    with torch.cuda.stream(stream):
        for _ in range(warmup):
            step()
    torch.cuda.synchronize(dev)
    ctx.device_error()
    barrier(dist)
    clocks = ClockSampler(local) if rank == 0 else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(dist)
    with torch.cuda.stream(stream):
        t0.record(stream)
        for _ in range(steps):
            step()
        t1.record(stream)
    barrier(dist)
    ms = t0.elapsed_time(t1)
    gu_ms, dn_ms = [], []
    with torch.cuda.stream(stream):
        for _ in range(3):
            step(events=True)
            torch.cuda.synchronize(dev)
            gu_ms.append(ev.elapsed(0, 1))
            dn_ms.append(ev.elapsed(1, 2))
    cl = clocks.stop() if clocks else None
    ctx.device_error()
    ms_max = max_over_ranks(dist, ms)
    value = T * steps * ws / (ms_max / 1e3)
    hbm, bf16, peak_kind = measured_peaks()
    # routing statistics of the step (distinct experts, tokens per expert)
    sel = torch.topk(torch.sigmoid(logits) + W.router_bias, 8, dim=1).indices
    distinct = int(torch.unique(sel).numel())
    sh_iq2 = args.shared_fmt != "q5k"
    # algorithmic bytes and flops per launch: each distinct expert's matrices read once, the activations in and out
    gu_bytes = (distinct + sh_iq2) * 2 * MAT + T * HIDDEN * 4 + T * (args.keep + 1) * INTER * 2
    dn_bytes = (distinct + sh_iq2) * DS + T * (args.keep + 1) * (INTER * 2 + HIDDEN * 4)
    entries = T * (args.keep + sh_iq2)
    gu_flops, dn_flops = 2.0 * entries * 2 * HIDDEN * INTER, 2.0 * entries * HIDDEN * INTER
    layer_bytes = distinct * (2 * MAT + DS) + shared_bytes(args) + ROUTER_BYTES + T * HIDDEN * 4 * 4
    flops = 2.0 * T * (args.keep + 1) * 3 * HIDDEN * INTER + 2.0 * T * HIDDEN * NE
    g_ms, d_ms = float(np.median(gu_ms)), float(np.median(dn_ms))
    # HBM-bound where the weights' bytes at peak take longer than the flops at the bf16 peak (T=512); else tensor
    tensor_bound = gu_flops / (bf16 * 1e12) > gu_bytes / (hbm * 1e9)
    gu_gbs, gu_tf = gu_bytes / (g_ms / 1e3) / 1e9, gu_flops / (g_ms / 1e3) / 1e12
    dn_gbs, dn_tf = dn_bytes / (d_ms / 1e3) / 1e9, dn_flops / (d_ms / 1e3) / 1e12
    wl = "prefill_T%d" % T
    out = {
        "metric": "MoE-layer tokens/s (T=%d %s, one layer)" % (T, "prefill" if T <= 512 else "batch"),
        "value": round(value, 1), "unit": "tokens/s",
        "n_gpus": ws, "steps": steps, "warmup": warmup, "ms_per_step": round(ms_max / steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "iq2_xxs x q8 activations: gate/up tcgen05 kind::f16 with exact integer weights and hi/lo fp16 activations "
                 "(the reference's group sums), h re-quantised to q8; down tcgen05 fp16; fp32 accumulate" if not model_fmt else
                 "the real model's formats (%s down, %s shared): IQ2_XXS q8 gate/up on tcgen05 (h re-quantised to q8), K-quant "
                 "down mma.sync fp16; Q5_K/Q6_K shared on tcgen05 (fp16 hi/lo gate/up operands, q8 h); fp32 accumulate" % (args.down_fmt, args.shared_fmt),
        "data": "synthetic: seeded IQ2_XXS experts, uniform-random router logits U(-1,1), bf16 N(0,1) hidden states",
        "config": {"workload": ("config2_prefill_T%d" % T if T == 512 else "config3_batch_T%d_1gpu" % T if T == 4096 else wl) +
                               ("" if not model_fmt else "_%s_down_%s_shared" % (args.down_fmt, args.shared_fmt)),
                   "global_batch": T * ws, "seq_len": T, "layers": 1, "top_k": 8, "n_group": N_GROUP, "topk_group": TOPK_GROUP,
                   "keep": args.keep, "distinct_experts": distinct, "parallelism": "replicas" if ws > 1 else "single",
                   "l2": "no flush: a step streams %.2f GB of distinct weights (> 126 MB L2)" % (layer_bytes / 1e9)},
        "layer": {"bytes": layer_bytes, "flops": flops, "achieved_gbs": round(layer_bytes / (ms_max / steps / 1e3) / 1e9, 1),
                  "achieved_tflops": round(flops / (ms_max / steps / 1e3) / 1e12, 1),
                  "frac_of_hbm": round(layer_bytes / (ms_max / steps / 1e3) / 1e9 / hbm, 4),
                  "frac_of_bf16": round(flops / (ms_max / steps / 1e3) / 1e12 / bf16, 4),
                  "kernel_ms_event": {"gate_up": round(g_ms, 4), "down": round(d_ms, 4),
                                      "rest": round(ms_max / steps - g_ms - d_ms, 4)}},
        "roofline": {"kernel": "k_gate_up_q8 (+ its activation-tile pre-pass): q8 gate/up + SwiGLU + q8 of h",
                     "bound": "tensor" if tensor_bound else "hbm",
                     "achieved": round(gu_tf if tensor_bound else gu_gbs, 1), "peak": bf16 if tensor_bound else hbm,
                     "unit": "TFLOP/s" if tensor_bound else "GB/s",
                     "frac": round(gu_tf / bf16 if tensor_bound else gu_gbs / hbm, 4),
                     "traffic": ncu_traffic("k_gate_up_q8", wl), "algorithmic_bytes_per_launch": gu_bytes,
                     "algorithmic_flops_per_launch": gu_flops, "peak_source": peak_kind,
                     "hbm_gbs": round(gu_gbs, 1), "hbm_frac": round(gu_gbs / hbm, 4),
                     "tensor_tflops": round(gu_tf, 1), "tensor_frac": round(gu_tf / bf16, 4),
                     "frac_of_nominal_7700": round(gu_gbs / NOMINAL_HBM_GBS, 4),
                     "down": {"kernel": "k_prefill_down" if fmt == 4 else "k_kq_mma_down", "ms": round(d_ms, 4),
                              "hbm_gbs": round(dn_gbs, 1), "hbm_frac": round(dn_gbs / hbm, 4),
                              "tensor_tflops": round(dn_tf, 1), "tensor_frac": round(dn_tf / bf16, 4),
                              "traffic": ncu_traffic("k_prefill_down" if fmt == 4 else "k_kq_mma_down", wl)}},
        # this library's kernels per step: router, slot build, gate/up activation tiles, gate/up GEMM, down GEMM,
        # combine; K-quant downs add a second slot build and take k_kq_mma_down for the down; a Q5_K/Q6_K shared
        # expert adds its 6 dense-path kernels (3 dequantisations, the q8 of x, the gate/up and down GEMMs)
        "gpu_launches": steps * ((6 if fmt == 4 else 7) + (6 if args.shared_fmt == "q5k" else 0)),
    }
    if cl:
        out["clocks"] = cl
    del ctx
    return out


def reference_arm(args, ws, rank):
    """--impl reference: the CPU oracle (the restatement of the reference's path) on the host cores, timed on the
    same workload as the GPU arm's line: each step is T=1 through the 58 distinct layers (router, experts,
    combine), every layer's weights set up before the clock starts."""
    if rank != 0:
        return None
    from oracle import oracle as O
    O.build()
    layers = [cpu_layer(O, L, args.keep) for L in range(args.layers)]
    per_step = []
    for s in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        for lay in layers:
            cpu_layer_forward(O, lay)
        if s >= args.warmup:
            per_step.append(time.perf_counter() - t0)
    t_step = float(np.mean(per_step))
    value = 1.0 / t_step
    cores = cpu_cores()
    sample = "every step: T=1 through %d distinct layers (router, 8 routed + shared IQ2_XXS experts, combine)" % args.layers
    return {"impl": "reference", "metric": "MoE-layer tokens/s (T=1 decode through 58 layers)", "value": round(value, 4),
            "unit": "tokens/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t_step * 1e3, 2), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "iq2_xxs x q8 (int32 dot, fp64 accumulate)",
            "data": "synthetic: seeded IQ2_XXS experts (BASELINE config 0 generator), router W N(0,0.02), bias N(0,0.01), x/resid N(0,1) fp32",
            "config": decode_config(args, 1, args.layers),
            "cpu_baseline": {"value": round(value, 4), "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": round(value, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode", choices=["decode", "prefill", "imbalance"])
    ap.add_argument("--tokens", type=int, default=512, help="prefill workload: tokens per step")
    ap.add_argument("--layers", type=int, default=N_LAYERS)
    ap.add_argument("--keep", type=int, default=8)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--down-fmt", default="iq2", choices=sorted(DOWN_FMTS),
                    help="decode workload: format of the down matrices (q2k / q3k: the real model's; no e2e or CPU leg)")
    ap.add_argument("--shared-fmt", default="iq2", choices=["iq2", "q5k"],
                    help="decode workload: the shared expert's formats (q5k: the real model's Q5_K gate/up + Q6_K down)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU-baseline sample (profiling runs)")
    ap.add_argument("--no-batch", action="store_true", help="decode workload: skip the T=512 / T=4096 sub-measurements")
    ap.add_argument("--cpu-layers", type=int, default=2, help="layers in the CPU-baseline sample")
    ap.add_argument("--parallelism", default="ep", choices=["ep", "replicas"], help="N > 1: expert parallel or replicas")
    ap.add_argument("--exchange", default="p2p", choices=["p2p", "nccl"], help="EP decode row exchange")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    ws, rank, local = dist_setup(args)
    if args.impl == "reference":
        out = reference_arm(args, ws, rank)
        if out is not None:
            print(json.dumps(out), flush=True)
        return
    import torch
    dist = dist_init(ws, local)
    if args.workload == "imbalance":
        out = run_imbalance(args, ws, rank, local, dist)
        if rank == 0:
            print(json.dumps(out), flush=True)
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return
    if ws > 1 and args.parallelism == "ep":
        out = run_ep_prefill(args, ws, rank, local, dist) if args.workload == "prefill" else run_ep_decode(args, ws, rank, local, dist)
        if rank == 0:
            print(json.dumps(out), flush=True)
        dist.barrier()
        dist.destroy_process_group()
        return
    if args.workload == "prefill":
        out = run_prefill(args, ws, rank, local, dist)
        if rank == 0:
            print(json.dumps(out), flush=True)
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return
    out, layers, ctx, structs, xs, rs = run_decode(args, ws, rank, local, dist)
    if args.down_fmt != "iq2" or args.shared_fmt != "iq2":
        args.no_cpu = True                          # the CPU sample is the IQ2_XXS layer
    if args.down_fmt != "iq2" and args.shared_fmt == "iq2":
        args.no_e2e = True                          # fl_moe_prepare's IQ2_XXS shared expert has IQ2_XXS downs
    if not args.no_e2e:
        e2e = e2e_decode(args, layers, len(layers), args.keep)
        e2e_v = max_over_ranks(dist, 1.0 / e2e["value"])
        e2e["value"] = round(ws / e2e_v, 2)
        out["e2e"] = e2e
    if rank == 0 and ws == 1 and not args.no_cpu:
        t_layer, cores = cpu_decode_sample(args.cpu_layers, keep=args.keep)
        out["cpu_baseline"] = {"value": round(1.0 / (t_layer * args.layers), 4), "unit": "tokens/s", "cores": cores,
                               "kind": "port", "sample": "%d layers of T=1 decode through the C++ oracle, scaled to %d layers"
                               % (args.cpu_layers, args.layers)}
    if ws == 1 and not args.no_batch and args.down_fmt == "iq2" and args.shared_fmt == "iq2":
        # the metric's other two token counts on the same GPU, reusing resident layer 0: BASELINE config 2 (T=512)
        # and config 3's shape on one GPU (T=4096)
        del ctx, structs, xs, rs
        W0 = layers[0]
        del layers[1:]
        torch.cuda.empty_cache()
        out["prefill_T512"] = run_prefill(args, ws, rank, local, dist, W=W0, T=512, steps=10, warmup=3)
        torch.cuda.empty_cache()
        out["batch_T4096"] = run_prefill(args, ws, rank, local, dist, W=W0, T=4096, steps=5, warmup=3)
    if rank == 0:
        print(json.dumps(out), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
