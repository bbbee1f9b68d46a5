#!/usr/bin/env python
"""Memory-layer forward benchmark (B200).

One step = one forward of the memory-layer block of KumarDev7/model
(model.py:108-120 around memory.py:119-227) over T = 8192 tokens per GPU at
the single-layer configuration: d_model 256, H 4, d_key 256,
n_sub_keys 512 (262,144 slots), top_k 16, d_value 256, float32 values.
Inputs are synthetic and seeded: hidden ~ N(0,1), Glorot-uniform router /
gate / output kernels, sub_keys ~ N(0, 1/128), values ~ N(0, 0.02).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

With N > 1 (torchrun, one process per GPU) the value table is row-sharded
over the ranks (--pool sharded, the default: slot s on rank s % N) and each
rank routes its own 8192 tokens, so the work per GPU is fixed (weak
scaling); --pool replicated runs N independent replicas instead.

Prints one JSON line (rank 0).  ``value`` is whole-job tokens/s from CUDA
events around each step (inputs resident in HBM; L2 flushed before every
step), max over ranks; ``e2e`` is the same through the C ABI with the hidden
states copied in from pinned host memory and the layer output copied back
inside the timed region.  ``--impl reference`` times the CPU oracle (a
float32 restatement of the reference layer) on the host's cores.
"""

from __future__ import annotations

import argparse
import ctypes as C
import json
import math
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOAD = dict(name="cfg0_layer_forward", tokens_per_gpu=8192, d_model=256, heads=4, d_key=256, n_sub_keys=512,
                top_k=16, d_value=256, values_dtype="f32", seed=0)
FLUSH_BYTES = 256 << 20          # > 126 MB L2
FALLBACK_HBM_GBS = 6650.0
NOMINAL_HBM_GBS = 8000.0         # B200 HBM3e as NVIDIA quotes it (DGX; 7700 on HGX), for context
NOMINAL_TF32_TFLOPS = 1100.0     # dense tf32 tensor peak as NVIDIA quotes it, for context


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--values-dtype", choices=["f32", "f16", "bf16"], default="f32")
    ap.add_argument("--tokens", type=int, default=WORKLOAD["tokens_per_gpu"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--inflight", type=int, default=6,
                    help="host-buffer calls in flight (on as many streams) in the e2e measurement")
    ap.add_argument("--host-chunks", type=int, default=1,
                    help="chunks of the host-buffer pipeline timed as e2e (memlayer_layer_forward_host)")
    ap.add_argument("--workload", choices=["cfg0", "cfg1", "cfg2", "cfg3", "cfg4", "host"], default="cfg0",
                    help="cfg0 (default, the driver's line): configs[0] layer forward; cfg2: configs[2] decode "
                         "latency on a 67M-slot fp16 table; cfg3: configs[3] billion-slot bf16 table "
                         "row-sharded over >= 4 GPUs; cfg4: configs[4] forward + fetched-row Adagrad; host: configs[2] "
                         "shapes with the table in page-locked host memory")
    ap.add_argument("--split", action="store_true",
                    help="N>1: one call per step with the exchange in two overlapped token halves "
                         "(MEMLAYER_PHASE_SPLIT); default: the three phases one after another")
    ap.add_argument("--emulate-ranks", type=int, default=0,
                    help="time the row-sharded phases of P ranks driven from one process on one GPU "
                         "(all ROUTE, then all GATHER, then all REDUCE); for profiling without NVLink")
    ap.add_argument("--exchange", choices=["p2p", "nccl"], default="p2p",
                    help="row-sharded pool (N > 1): partial rows stored into the token owners' memory by the "
                         "gather kernel (p2p), or the staged baseline: NCCL all-gather of the routing entries "
                         "and reduce-scatter of the partial rows between the library's phases (nccl)")
    ap.add_argument("--no-parity", action="store_true",
                    help="N > 1: skip the check of the sharded result against the single-GPU layer")
    ap.add_argument("--pool", choices=["sharded", "replicated"], default="sharded",
                    help="N>1: row-shard the value table over the ranks (default) or replicate it")
    return ap.parse_args()


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """Polls NVML (SM clock, max clock, clock-event reasons) on a thread."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, index: int, period: float = 0.005):
        self.samples, self.reasons, self.ok = [], set(), False
        self.period, self._stop = period, threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # noqa: BLE001 - clocks are reported as unavailable
            self.err = str(e)
        self.t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:  # noqa: BLE001
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self.t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.ok:
            self.t.join()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": "NVML unavailable"}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons - {"gpu_idle"}), "samples": len(self.samples), "source": "nvml"}


# ---------------------------------------------------------------- inputs
def make_inputs(torch, device, W, values_dtype, seed, value_rows=None):
    """Seeded synthetic inputs; ``value_rows`` < n^2 draws only this rank's
    rows of a row-sharded table (same distribution)."""
    g = torch.Generator(device=device).manual_seed(seed)
    T, dm, H, dk, n, d = (W[k] for k in ("tokens_per_gpu", "d_model", "heads", "d_key", "n_sub_keys", "d_value"))

    def glorot(fi, fo):
        lim = math.sqrt(6.0 / (fi + fo))
        return (torch.rand(fi, fo, device=device, generator=g) * 2 - 1) * lim

    vdt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[values_dtype]
    x = {
        "h": torch.randn(T, dm, device=device, generator=g),
        "w_router": glorot(dm, H * dk), "b_router": torch.zeros(H * dk, device=device),
        "sub_keys": torch.randn(H, 2, n, dk // 2, device=device, generator=g) * math.sqrt(1 / 128),
        "log_t": torch.full((1,), math.log(10.0), device=device),
        # drawn in the table's own dtype (no float32 copy of a large table)
        "values": torch.randn(n * n if value_rows is None else value_rows, d, device=device, generator=g,
                              dtype=vdt).mul_(0.02),
        "w_gate": glorot(dm, d), "b_gate": torch.zeros(d, device=device),
        "w_out": glorot(d, dm), "b_out": torch.zeros(dm, device=device),
    }
    return x


def clustered_hidden(torch, device, T, dm, seed, centers=64, sigma=0.3, zipf_a=1.1):
    """configs[3] / [4] hidden states: 64 Gaussian centres ~ N(0, I) with
    Zipf(1.1) cluster weights (p_r ~ r^-1.1), plus sigma * N(0, I)."""
    g = torch.Generator(device=device).manual_seed(seed)
    c = torch.randn(centers, dm, device=device, generator=g)
    p = torch.arange(1, centers + 1, device=device, dtype=torch.float64) ** -zipf_a
    idx = torch.multinomial((p / p.sum()).float(), T, replacement=True, generator=g)
    return c[idx] + sigma * torch.randn(T, dm, device=device, generator=g)


class LayerCall:
    """Pre-built C-ABI call of memlayer_layer_forward on resident buffers."""

    def __init__(self, torch, L, W, x, device, values_dtype):
        T, H, k, d, dm = (W[k] for k in ("tokens_per_gpu", "heads", "top_k", "d_value", "d_model"))
        dt = {"f32": L.F32, "f16": L.F16, "bf16": L.BF16}[values_dtype]
        self.L, self.torch = L, torch
        self.cfg = L.MemlayerConfig(tokens=T, heads=H, n_sub_keys=W["n_sub_keys"], d_key=W["d_key"], d_value=d,
                                    top_k=k, d_model=dm, values_dtype=dt, routing_noise=1.0, min_temperature=10.0,
                                    max_temperature=100.0, query_scale=0, balance_temperature_grad=0)
        self.y = torch.empty(T, dm, device=device)
        self.slots = torch.empty(T, H, k, dtype=torch.int32, device=device)
        self.weights = torch.empty(T, H, k, device=device)
        self.top1 = torch.empty(1, device=device)
        self.temp = torch.empty(1, device=device)
        self.events = L.MemlayerStageEvents()
        pool = L.MemlayerPoolArgs(sub_keys=x["sub_keys"].data_ptr(), log_temperature=x["log_t"].data_ptr(),
                                  values=x["values"].data_ptr(), slots=self.slots.data_ptr(),
                                  weights=self.weights.data_ptr(), top1_weight=self.top1.data_ptr(),
                                  temperature=self.temp.data_ptr(), stage_events=C.pointer(self.events))
        self.args = L.MemlayerLayerArgs(h=x["h"].data_ptr(), w_router=x["w_router"].data_ptr(),
                                        b_router=x["b_router"].data_ptr(), w_gate=x["w_gate"].data_ptr(),
                                        b_gate=x["b_gate"].data_ptr(), w_out=x["w_out"].data_ptr(),
                                        b_out=x["b_out"].data_ptr(), y=self.y.data_ptr(), mem=None, pool=pool)
        nb = C.c_size_t()
        L.check(L.lib().memlayer_layer_workspace_size(C.byref(self.cfg), C.byref(nb)), "workspace_size")
        self.ws = torch.empty(nb.value, dtype=torch.uint8, device=device)
        self.ws_bytes = nb.value

    def __call__(self, stream, events=None):
        for i in range(self.L.STAGE_EVENTS):
            self.events.events[i] = None if events is None else events[i].cuda_event
        self.L.check(self.L.lib().memlayer_layer_forward(C.byref(self.cfg), C.byref(self.args),
                                                         self.ws.data_ptr(), self.ws_bytes, stream.cuda_stream),
                     "memlayer_layer_forward")


class ShardedLayerCall(LayerCall):
    """memlayer_layer_forward_sharded on resident buffers: this rank's local
    rows of the row-sharded table, the three phases issued back to back on
    one stream (events between them time the owner-side gather)."""

    def __init__(self, torch, L, W, x, device, values_dtype):
        from model_b200.shard import connect
        super().__init__(torch, L, W, x, device, values_dtype)
        self.comm = connect(self.cfg)                   # collective over the default group
        self.world = self.comm.world
        nb = C.c_size_t()
        L.check(L.lib().memlayer_shard_workspace_size(C.byref(self.cfg), self.world, 1, C.byref(nb)),
                "shard_workspace_size")
        self.ws = torch.empty(nb.value, dtype=torch.uint8, device=device)
        self.ws_bytes = nb.value

    def set_io(self, h, y):
        self.args.h, self.args.y = h.data_ptr(), y.data_ptr()

    def __call__(self, stream, events=None, phase_events=None, split=False):
        """phase_events None: one call (``split``: the two token halves
        overlapped); else the three phases one after another with events
        between them (times the owner-side gather alone)."""
        for i in range(self.L.STAGE_EVENTS):
            self.events.events[i] = None if events is None else events[i].cuda_event
        f = self.L.lib().memlayer_layer_forward_sharded
        if phase_events is None:
            self.L.check(f(C.byref(self.cfg), C.byref(self.args), self.comm.handle,
                           self.L.PHASE_ALL | (self.L.PHASE_SPLIT if split else 0), self.ws.data_ptr(),
                           self.ws_bytes, stream.cuda_stream), "memlayer_layer_forward_sharded")
            return
        for j, ph in enumerate((self.L.PHASE_ROUTE, self.L.PHASE_GATHER, self.L.PHASE_REDUCE)):
            self.L.check(f(C.byref(self.cfg), C.byref(self.args), self.comm.handle, ph, self.ws.data_ptr(),
                           self.ws_bytes, stream.cuda_stream), "memlayer_layer_forward_sharded")
            if phase_events is not None and j < 2:
                phase_events[j].record(stream)


class StagedLayerCall(LayerCall):
    """The row-sharded layer with the NCCL exchange (the baseline the fused
    peer-store gather is measured against): memlayer_layer_forward_staged's
    ROUTE, an NCCL all-gather of every rank's packed (slot, weight) entries,
    GATHER of this rank's rows for every rank's tokens, an NCCL
    reduce-scatter of the partial rows, REDUCE (gate and output projection),
    all on one stream."""

    def __init__(self, torch, L, W, x, device, values_dtype, rank, world):
        super().__init__(torch, L, W, x, device, values_dtype)
        T, H, k, d = (W[q] for q in ("tokens_per_gpu", "heads", "top_k", "d_value"))
        self.rank, self.world = rank, world
        self.route = torch.empty(world, 2, T * H * k, dtype=torch.int32, device=device)
        mine = self.route[rank]
        self.slots = mine[0].view(T, H, k)
        self.weights = mine[1].view(torch.float32).view(T, H, k)
        self.args.pool.slots, self.args.pool.weights = self.slots.data_ptr(), self.weights.data_ptr()
        self.partials = torch.empty(world, T, d, device=device)
        self.mem_in = torch.empty(T, d, device=device)
        self.sargs = L.MemlayerStagedArgs(all_slots=self.route.data_ptr(), all_weights=self.route[0, 1].data_ptr(),
                                          route_stride=2 * T * H * k, partials=self.partials.data_ptr(),
                                          mem=self.mem_in.data_ptr(), rank=rank, world=world)

    def set_io(self, h, y):
        self.args.h, self.args.y = h.data_ptr(), y.data_ptr()

    def _phase(self, ph, stream):
        self.L.check(self.L.lib().memlayer_layer_forward_staged(C.byref(self.cfg), C.byref(self.args),
                                                                C.byref(self.sargs), ph, self.ws.data_ptr(),
                                                                self.ws_bytes, stream.cuda_stream),
                     "memlayer_layer_forward_staged")

    def __call__(self, stream, events=None, phase_events=None, split=False):
        """events: the route's stage events (0-4) and the end (5);
        phase_events: after the all-gather, after the gather, after the
        reduce-scatter."""
        import torch.distributed as dist
        for i in range(self.L.STAGE_EVENTS):
            self.events.events[i] = None if events is None or i == 5 else events[i].cuda_event
        with self.torch.cuda.stream(stream):
            self._phase(self.L.PHASE_ROUTE, stream)
            dist.all_gather_into_tensor(self.route.view(-1), self.route[self.rank].view(-1))
            if phase_events is not None:
                phase_events[0].record(stream)
            self._phase(self.L.PHASE_GATHER, stream)
            if phase_events is not None:
                phase_events[1].record(stream)
            dist.reduce_scatter_tensor(self.mem_in.view(-1), self.partials.view(-1))
            if phase_events is not None:
                phase_events[2].record(stream)
            self._phase(self.L.PHASE_REDUCE, stream)
            if events is not None:
                events[5].record(stream)


def staged_gather_bytes(W, values_dtype, world):
    """Algorithmic bytes of one staged gather launch on one rank: its share
    of all ranks' value rows, every rank's packed routing entries, and the
    partial rows it writes (one per token of every rank)."""
    T, H, k, d = W["tokens_per_gpu"], W["heads"], W["top_k"], W["d_value"]
    es = {"f32": 4, "f16": 2, "bf16": 2}[values_dtype]
    rows = T * H * k * d * es
    return rows, rows + world * T * H * k * 8 + world * T * d * 4


def shard_gather_bytes(W, values_dtype, world):
    """Algorithmic bytes of one owner-side gather launch on one rank, for the
    expected even spread of slots over ranks: the rank's share of all ranks'
    value rows, its inbox entries, and the partial rows it stores (local
    and over NVLink); plus the partial bytes that cross NVLink."""
    T, H, k, d = W["tokens_per_gpu"], W["heads"], W["top_k"], W["d_value"]
    es = {"f32": 4, "f16": 2, "bf16": 2}[values_dtype]
    rows = T * H * k * d * es                       # world * T tokens' fetches / world owners
    entries = T * H * k * 8 + world * T * 4
    partials = world * T * d * 4
    return rows, rows + entries + partials, (world - 1) * T * d * 4


def gather_bytes(W, values_dtype):
    """Algorithmic bytes of one combine+gather launch (the dominant HBM
    kernel): value rows + stage-1 lists + gate in + gated output + slots/weights."""
    T, H, k, d = W["tokens_per_gpu"], W["heads"], W["top_k"], W["d_value"]
    es = {"f32": 4, "f16": 2, "bf16": 2}[values_dtype]
    rows = T * H * k * d * es
    io = T * H * 2 * k * 12 + T * d * 4 * 2 + T * H * k * 8 + T * H * 4
    return rows, rows + io


def tensor_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def score_gemm_flops(W):
    """Algorithmic FLOPs of the score contraction (memory.py:149):
    2 * tokens * heads * 2 halves * n_sub_keys * (d_key / 2)."""
    return 2 * W["tokens_per_gpu"] * W["heads"] * 2 * W["n_sub_keys"] * (W["d_key"] // 2)


def load_traffic(kernel):
    p = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        return json.load(f).get(kernel)


# ---------------------------------------------------------------- CPU oracle timing
def cpu_oracle_rate(W, tokens, repeats=3, threads=None):
    """tokens/s of the CPU oracle layer forward on `tokens` tokens of the
    workload, token chunks spread over a thread pool of all host cores."""
    import concurrent.futures as cf

    import numpy as np

    from oracle import memlayer_ref as ref
    threads = threads or os.cpu_count() or 1
    rng = np.random.default_rng(W["seed"])
    H, dk, n, d, dm, k = (W[x] for x in ("heads", "d_key", "n_sub_keys", "d_value", "d_model", "top_k"))
    values = rng.standard_normal((n * n, d), dtype=np.float32) * np.float32(0.02)
    sk = rng.standard_normal((H, 2, n, dk // 2), dtype=np.float32) * np.float32(math.sqrt(1 / 128))

    def glorot(fi, fo):
        lim = math.sqrt(6.0 / (fi + fo))
        return rng.uniform(-lim, lim, (fi, fo)).astype(np.float32)
    wr, wg, wo = glorot(dm, H * dk), glorot(dm, d), glorot(d, dm)
    h = rng.standard_normal((tokens, dm), dtype=np.float32)
    cfg = ref.PoolConfig(n_sub_keys=n, heads=H, d_key=dk, d_value=d, top_k=k)
    z = lambda m: np.zeros(m, np.float32)  # noqa: E731
    log_t = np.log(np.float32(10.0))
    chunk = max(64, tokens // threads)

    def one(s):
        return ref.layer_forward(cfg, h[s:s + chunk], wr, z(H * dk), sk, log_t, values, wg, z(d), wo, z(dm))[0]

    with cf.ThreadPoolExecutor(threads) as ex:
        list(ex.map(one, range(0, min(tokens, chunk * threads), chunk)))   # warm-up
        times = []
        for _ in range(repeats):
            t0 = time.perf_counter()
            list(ex.map(one, range(0, tokens, chunk)))
            times.append(time.perf_counter() - t0)
    return tokens / statistics.median(times), threads, f"{tokens} tokens x {repeats} runs (median), " \
        f"{chunk}-token chunks over {threads} threads, numpy float32"


# ---------------------------------------------------------------- arms
def run_reference(args, W, rank):
    if rank != 0:
        return None
    # every step is one forward of the full token batch on all host cores
    tokens = args.tokens
    steps = max(5, min(args.steps, 20))
    rate, cores, sample = cpu_oracle_rate(W, tokens, repeats=steps)
    line = {"impl": "reference", "metric": "memory-layer tokens/s", "value": rate, "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": steps, "warmup": 1, "ms_per_step": 1000.0 * tokens / rate,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": W["name"], **{k: W[k] for k in W if k != "name"}},
            "cpu_baseline": {"value": rate, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": rate, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    return line


def run_ours(args, W, rank, world):
    import torch

    from model_b200 import _lib as L
    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(device)
    lib = L.lib()
    sharded = world > 1 and args.pool == "sharded"
    staged = sharded and args.exchange == "nccl"
    T, dm = W["tokens_per_gpu"], W["d_model"]
    full_values = None
    if sharded:
        # one model on every rank: the same parameters and table (each rank
        # keeps its rows s % world == rank), each rank's own tokens
        x = make_inputs(torch, device, W, args.values_dtype, W["seed"])
        full_values = x["values"]
        x["values"] = full_values[rank::world].contiguous()
        if args.no_parity:
            full_values = None
        g = torch.Generator(device=device).manual_seed(W["seed"] + 1 + rank)
        x["h"] = torch.randn(T, dm, device=device, generator=g)
        torch.cuda.empty_cache()
    else:
        x = make_inputs(torch, device, W, args.values_dtype, W["seed"] + rank)
    if staged:
        call = StagedLayerCall(torch, L, W, x, device, args.values_dtype, rank, world)
    else:
        call = (ShardedLayerCall if sharded else LayerCall)(torch, L, W, x, device, args.values_dtype)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    overlapped = sharded and args.split and not staged

    def step(events=None, phase_events=None):
        if sharded:
            call(stream, events, phase_events, split=overlapped and phase_events is None)
        else:
            call(stream, events)

    for _ in range(args.warmup):
        flush.zero_()
        step()
    torch.cuda.synchronize()

    K = args.steps
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(L.STAGE_EVENTS)] for _ in range(K)]
    pev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(K)] if sharded else None
    for row in ev:                 # create the driver events before handing them to the library
        for e in row:
            e.record(stream)
    torch.cuda.synchronize()
    launches0 = lib.memlayer_kernel_launch_count()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    with ClockSampler(device.index) as clk:
        for i in range(K):
            flush.zero_()
            if staged:
                step(ev[i], pev[i])     # the phases and the collectives, events between them
            else:
                step(ev[i])             # one call per step (single GPU, or the row-sharded call)
        torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    launches = (lib.memlayer_kernel_launch_count() - launches0) // K
    step_ms = [ev[i][0].elapsed_time(ev[i][5]) for i in range(K)]
    stage = lambda a, b: statistics.mean(ev[i][a].elapsed_time(ev[i][b]) for i in range(K))  # noqa: E731
    pstage = lambda f: statistics.mean(f(i) for i in range(K))  # noqa: E731
    stages = {"projections": stage(0, 1), "prep": stage(1, 2), "score_topk": stage(2, 3),
              "combine_gather": stage(3, 4), "finalize_out": stage(4, 5)}
    if not sharded:
        # the library overlaps the second token half's score with the first
        # half's gather inside each call; the kernels' own times for the
        # roofline come from a pass with that overlap off (MEMLAYER_OVERLAP=0)
        G = min(K, 20)
        gev = [[torch.cuda.Event(enable_timing=True) for _ in range(L.STAGE_EVENTS)] for _ in range(G)]
        for row in gev:
            for e in row:
                e.record(stream)
        torch.cuda.synchronize()
        os.environ["MEMLAYER_OVERLAP"] = "0"
        for i in range(G):
            flush.zero_()
            call(stream, gev[i])
        torch.cuda.synchronize()
        del os.environ["MEMLAYER_OVERLAP"]
        gst = lambda a, b: statistics.mean(gev[i][a].elapsed_time(gev[i][b]) for i in range(G))  # noqa: E731
        stages = {"projections": stage(0, 1), "prep": stage(1, 2),
                  "score_and_first_half_gather": stage(2, 3), "second_half_gather": stage(3, 4),
                  "finalize_out": stage(4, 5),
                  "score_topk": gst(2, 3), "combine_gather": gst(3, 4), "unoverlapped_step": gst(0, 5)}
    elif staged:
        stages = {"projections": stage(0, 1), "prep": stage(1, 2), "score_topk": stage(2, 3),
                  "combine": stage(3, 4),
                  "finalize_allgather": pstage(lambda i: ev[i][4].elapsed_time(pev[i][0])),
                  "staged_gather_alone": pstage(lambda i: pev[i][0].elapsed_time(pev[i][1])),
                  "reduce_scatter": pstage(lambda i: pev[i][1].elapsed_time(pev[i][2])),
                  "reduce_out": pstage(lambda i: pev[i][2].elapsed_time(ev[i][5]))}
    else:
        # row-sharded: one call per timed step (issuing the three phases as
        # separate calls costs enough host time per step that a rank whose
        # host falls behind idles its GPU, and every other rank then waits
        # for it in the exchange); the phases' own times come from a separate
        # phased pass below, untimed in the step figure
        stages = {"projections": stage(0, 1), "prep": stage(1, 2), "score_topk": stage(2, 3),
                  "combine_scatter": stage(3, 4), "finalize_exchange_reduce_out": stage(4, 5)}
        # the owner-side gather alone: the three phases one after another,
        # untimed in the step figure, for the gather kernel's roofline
        G = min(K, 20)
        gev = [[torch.cuda.Event(enable_timing=True) for _ in range(L.STAGE_EVENTS)] for _ in range(G)]
        for row in gev:
            for e in row:
                e.record(stream)
        torch.cuda.synchronize()
        torch.distributed.barrier()
        for i in range(G):
            flush.zero_()
            call(stream, gev[i], pev[i])
        torch.cuda.synchronize()
        torch.distributed.barrier()
        stages["shard_gather_alone"] = statistics.mean(pev[i][0].elapsed_time(pev[i][1]) for i in range(G))
        stages["phased_reduce_out"] = statistics.mean(pev[i][1].elapsed_time(gev[i][5]) for i in range(G))
        stages["phased_step"] = statistics.mean(gev[i][0].elapsed_time(gev[i][5]) for i in range(G))
    ms = statistics.mean(step_ms)

    # ---- e2e through the C ABI with host buffers ----
    # Every step copies its hidden state in from pinned host memory and its
    # output back; e2e = K steps of tokens over the device time of all K.
    # One GPU: --inflight calls in flight on as many streams (separate host /
    # staging buffers per call), as a server runs requests: one call's
    # host-to-device copy overlaps another's layer, and the calls' kernels
    # overlap on the GPU (an ALU-bound score kernel beside an HBM-bound
    # gather).  Sharded (every rank in lockstep on its default stream): the
    # calls run one after another; hidden states and outputs are double
    # buffered so that the next step's copy in and the previous step's copy
    # out run on copy streams during the current step.  `e2e_serial` is one
    # call at a time with its copies around it.
    NF = max(1, args.inflight)
    streams = [stream] + [torch.cuda.Stream(device) for _ in range(NF - 1)]
    nbuf = 2 if sharded else NF
    h_hosts = [x["h"].cpu().pin_memory() for _ in range(nbuf)]
    y_hosts = [torch.empty_like(call.y, device="cpu").pin_memory() for _ in range(nbuf)]
    host_issue = []
    if sharded:
        h_dev = [x["h"], torch.empty_like(x["h"])]
        y_dev = [call.y, torch.empty_like(call.y)]
        cin, cout = torch.cuda.Stream(device), torch.cuda.Stream(device)
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_call = [torch.cuda.Event() for _ in range(2)]
        ev_out = [torch.cuda.Event() for _ in range(2)]
        inflight = 1
        e2e_api = ("memlayer_layer_forward_staged with NCCL all-gather / reduce-scatter" if staged
                   else "memlayer_layer_forward_sharded") + \
            ", host copies double-buffered on two copy streams"

        def e2e_run(pipelined, steps):
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            torch.distributed.barrier()
            start.record(stream)
            cin.wait_event(start)
            cout.wait_event(start)
            t0 = time.perf_counter()
            for i in range(steps):
                b = i % 2 if pipelined else 0
                with torch.cuda.stream(cin):
                    if i >= 2 or not pipelined:
                        cin.wait_event(ev_call[b])      # the call that last read h_dev[b] is done
                    h_dev[b].copy_(h_hosts[b], non_blocking=True)
                    ev_in[b].record(cin)
                stream.wait_event(ev_in[b])
                if i >= 2 or not pipelined:
                    stream.wait_event(ev_out[b])        # y_dev[b] of an earlier step is copied out
                call.set_io(h_dev[b], y_dev[b])
                step()
                ev_call[b].record(stream)
                with torch.cuda.stream(cout):
                    cout.wait_event(ev_call[b])
                    y_hosts[b].copy_(y_dev[b], non_blocking=True)
                    ev_out[b].record(cout)
                if not pipelined:
                    stream.wait_event(ev_out[b])
            host_issue.append((time.perf_counter() - t0) * 1e3 / steps)
            stream.wait_stream(cout)
            end.record(stream)
            torch.cuda.synchronize()
            call.set_io(h_dev[0], y_dev[0])
            return start.elapsed_time(end) / steps

        for e in ev_call + ev_out:
            e.record(stream)
        for _ in range(max(1, args.warmup // 2)):
            e2e_run(True, 2)
        e2e_ms = e2e_run(True, K)
        e2e_host_issue_ms = host_issue[-1]
        e2e_serial_ms = e2e_run(False, max(1, K // 2))
    else:
        hnb = C.c_size_t()
        L.check(lib.memlayer_layer_host_workspace_size(C.byref(call.cfg), args.host_chunks, C.byref(hnb)), "host ws")
        hws = [torch.empty(hnb.value, dtype=torch.uint8, device=device) for _ in range(NF)]
        hargs, hargs_keep = [], []
        for j in range(NF):
            a_ = L.MemlayerLayerArgs.from_buffer_copy(call.args)
            a_.h, a_.y = h_hosts[j].data_ptr(), y_hosts[j].data_ptr()
            a_.pool.top1_weight = None
            a_.pool.stage_events = None
            if j:   # every other call in flight writes its own routing outputs
                extra = [torch.empty_like(call.slots), torch.empty_like(call.weights), torch.empty_like(call.temp)]
                a_.pool.slots, a_.pool.weights, a_.pool.temperature = (t.data_ptr() for t in extra)
                hargs_keep.append(extra)
            hargs.append(a_)

        def host_step(j):
            L.check(lib.memlayer_layer_forward_host(C.byref(call.cfg), C.byref(hargs[j]), args.host_chunks,
                                                    hws[j].data_ptr(), hnb.value, streams[j].cuda_stream),
                    "memlayer_layer_forward_host")
        inflight = NF
        e2e_api = (f"memlayer_layer_forward_host ({args.host_chunks} chunk(s), pinned host h / y), "
                   f"{NF} calls in flight on {NF} streams")

        def e2e_run(n_inflight, steps):
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            start.record(stream)
            for st in streams[1:n_inflight]:
                st.wait_event(start)
            t0 = time.perf_counter()
            for i in range(steps):
                with torch.cuda.stream(streams[i % n_inflight]):
                    host_step(i % n_inflight)
            host_issue.append((time.perf_counter() - t0) * 1e3 / steps)   # host time to issue one call
            for st in streams[1:n_inflight]:
                stream.wait_stream(st)
            end.record(stream)
            torch.cuda.synchronize()
            return start.elapsed_time(end) / steps

        for _ in range(max(1, args.warmup // 2)):
            e2e_run(inflight, 2)
        e2e_ms = e2e_run(inflight, K)
        e2e_host_issue_ms = host_issue[-1]
        e2e_serial_ms = e2e_run(1, max(1, K // 2))

    # ---- parity of the sharded step (N > 1): the same tokens through the
    # single-GPU layer with the whole table, on this rank's GPU ----
    parity = None
    if sharded and full_values is not None:
        flush.zero_()
        call.set_io(x["h"], call.y)
        step()
        torch.cuda.synchronize()
        y_sh, slots_sh, w_sh = call.y.clone(), call.slots.clone(), call.weights.clone()
        if staged:
            mem_sh = call.mem_in.clone()
        single = LayerCall(torch, L, W, dict(x, values=full_values), device, args.values_dtype)
        single(stream)
        torch.cuda.synchronize()
        y1 = single.y
        same_slots = bool(torch.equal(slots_sh, single.slots))
        same_w = bool(torch.equal(w_sh, single.weights))
        err = (y_sh.double() - y1.double()).abs()
        ref_abs = y1.double().abs()
        max_rel_y = float(err.max() / ref_abs.max().clamp_min(1e-30))
        floor = 1e-3 * float(ref_abs.max())
        max_elem_rel_y = float((err / (ref_abs + floor)).max())
        pvec = torch.tensor([0.0 if same_slots else 1.0, 0.0 if same_w else 1.0, max_rel_y, max_elem_rel_y,
                             float(not torch.isfinite(y_sh).all())], dtype=torch.float64, device=device)
        torch.distributed.all_reduce(pvec, op=torch.distributed.ReduceOp.MAX)
        parity = {"tokens": T * world, "checked_against": "memlayer_layer_forward on the whole table, "
                  "same tokens, same GPU (every rank, max over ranks)",
                  "slots_equal": pvec[0].item() == 0.0, "weights_equal": pvec[1].item() == 0.0,
                  "max_rel_y": pvec[2].item(),
                  "max_elem_rel_y": pvec[3].item(),
                  "elem_rel_floor": "1e-3 x max|y| added to |y| per element",
                  "tolerance": 1e-5 if args.values_dtype == "f32" else 2e-2,
                  "nonfinite": pvec[4].item() != 0.0}
        parity["ok"] = (parity["slots_equal"] and parity["weights_equal"] and not parity["nonfinite"]
                        and parity["max_rel_y"] <= parity["tolerance"])
        del single, full_values
        torch.cuda.empty_cache()

    gather_stage = (stages["staged_gather_alone"] if staged else stages["shard_gather_alone"] if sharded
                    else stages["combine_gather"])
    stats = torch.tensor([ms, e2e_ms, gather_stage, stages["score_topk"], e2e_serial_ms], dtype=torch.float64,
                         device=device)
    rank_stages = None
    if world > 1:
        torch.distributed.all_reduce(stats, op=torch.distributed.ReduceOp.MAX)
        # every rank's own step and stages (the step figure is their max)
        names = sorted(stages)
        mine = torch.tensor([statistics.mean(step_ms)] + [stages[k] for k in names], dtype=torch.float64,
                            device=device)
        allr = [torch.empty_like(mine) for _ in range(world)]
        torch.distributed.all_gather(allr, mine)
        rank_stages = [dict(zip(["step"] + names, t.tolist())) for t in allr]
    ms, e2e_ms, gather_ms, score_ms, e2e_serial_ms = stats.tolist()
    if sharded and not staged:     # every rank's kernels are done before the peers are unmapped
        torch.cuda.synchronize()
        torch.distributed.barrier()
        call.comm.close()
    if rank != 0:
        return None

    hbm, src = peaks()
    bf16, _ = tensor_peak()
    gname = "staged_gather_kernel" if staged else "shard_gather_kernel" if sharded else "combine_gather_kernel"
    if staged:
        rows_b, alg_b = staged_gather_bytes(W, args.values_dtype, world)
        nvlink_b = 0
    elif sharded:
        rows_b, alg_b, nvlink_b = shard_gather_bytes(W, args.values_dtype, world)
    else:
        (rows_b, alg_b), nvlink_b = gather_bytes(W, args.values_dtype), 0
    achieved = alg_b / (gather_ms * 1e-3) / 1e9
    traffic = load_traffic(gname)
    traffic_src = None
    if traffic is not None:
        traffic_src = traffic.get("source", "ncu capture")
        if sharded and traffic.get("world") not in (None, world):
            traffic_src = f"{traffic_src} (captured at {traffic.get('world')} ranks, not at {world})"
    score_flops = score_gemm_flops(W)
    score_tf = score_flops / (score_ms * 1e-3) / 1e12
    kernels = {
        gname: {"bound": "hbm", "ms": gather_ms, "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": achieved / hbm, "peak_nominal": NOMINAL_HBM_GBS, "frac_nominal": achieved / NOMINAL_HBM_GBS,
                "algorithmic_bytes_per_launch": alg_b,
                "traffic": None if traffic is None else traffic.get("bytes_per_launch"),
                "traffic_source": traffic_src},
        "score_topk_tc_kernel": {"bound": "tensor", "ms": score_ms, "achieved": score_tf, "peak": bf16,
                                 "unit": "TFLOP/s", "frac": score_tf / bf16, "algorithmic_flops_per_launch": score_flops,
                                 "issued_tf32_tflops": 3 * score_tf,
                                 "frac_nominal_tf32": 3 * score_tf / NOMINAL_TF32_TFLOPS,
                                 "note": "float32-faithful score GEMM issued as 3 tf32 MMAs per product; "
                                         "peak is the measured dense bf16 figure",
                                 "traffic": None if load_traffic("score_topk_tc_kernel") is None
                                 else load_traffic("score_topk_tc_kernel").get("bytes_per_launch")},
    }
    dominant = max(kernels, key=lambda k: kernels[k]["ms"])
    line = {
        "metric": "memory-layer tokens/s", "value": T * world / (ms * 1e-3), "unit": "tokens/s",
        "n_gpus": world, "steps": K, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded: hidden N(0,1), Glorot kernels, sub_keys N(0,1/128), values N(0,0.02))",
        "config": {"workload": W["name"], **{k: W[k] for k in W if k != "name"},
                   "values_dtype": args.values_dtype,
                   "l2": "flushed before every step (256 MiB write, outside the step events)",
                   "parallelism": (f"pool-row-shard{world}" + ("-nccl-staged" if staged else "-p2p")
                                   + ("-split" if overlapped else "") if sharded
                                   else f"replicas{world}") if world > 1
                   else "single"},
        "roofline": {"kernel": dominant, "peak_source": src,
                     **{k: v for k, v in kernels[dominant].items() if k != "ms"}},
        "roofline_kernels": kernels,
        "gather_gbs": rows_b / (gather_ms * 1e-3) / 1e9,
        **({"nvlink_partial_gbs_per_gpu": nvlink_b / (gather_ms * 1e-3) / 1e9} if sharded and not staged else {}),
        "stages_ms": stages,
        **({"stages_ms_per_rank": rank_stages} if rank_stages else {}),
        **({"parity": parity} if parity is not None else {}),
        "e2e": {"value": T * world / (e2e_ms * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": h_hosts[0].numel() * 4, "d2h_bytes_per_step": y_hosts[0].numel() * 4,
                "api": e2e_api, "ms_per_step": e2e_ms, "calls_in_flight": inflight,
                "host_issue_ms_per_call": e2e_host_issue_ms,
                "note": ("copies of one step overlap the neighbouring steps' layer calls" if sharded else
                         "calls in flight overlap on the GPU, so e2e can exceed the one-call-at-a-time value"),
                "l2": "not flushed: every step reads the 268 MB value table, larger than L2"},
        "e2e_serial": {"value": T * world / (e2e_serial_ms * 1e-3), "unit": "tokens/s",
                       "ms_per_step": e2e_serial_ms, "calls_in_flight": 1},
        "gpu_launches": int(launches) * K,
        "gpu_launches_per_step": int(launches),
        "clocks": clk.summary(),
    }
    if world == 1 and not args.no_cpu_baseline:
        rate, cores, sample = cpu_oracle_rate(W, W["tokens_per_gpu"])
        line["cpu_baseline"] = {"value": rate, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample}
    return line


# ---------------------------------------------------------------- other configs
def _events(torch, n):
    return [torch.cuda.Event(enable_timing=True) for _ in range(n)]


def _common_line(W, world, steps, warmup, ms, value, unit, dtype, extra):
    line = {"metric": "memory-layer tokens/s", "value": value, "unit": unit, "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": ms, "higher_is_better": True, "vs_baseline": None, "dtype": dtype,
            "data": "synthetic (seeded)", "config": {"workload": W["name"], **{k: W[k] for k in W if k != "name"}}}
    line.update(extra)
    return line


def _model_params(torch, device, mc, values, sub_keys, seed=0):
    """Seeded random-init parameters of a MemoryPoolLM (the reference's
    shapes) created on the device, around an existing pool table."""
    g = torch.Generator(device=device).manual_seed(seed)
    dm, H = mc.d_model, mc.n_heads
    dh = dm // H

    def r(*shape, std=1.0):
        return torch.randn(*shape, device=device, generator=g) * std

    def dense(fi, fo):
        return {"kernel": r(fi, fo, std=fi ** -0.5), "bias": torch.zeros(fo, device=device)}

    def ln():
        return {"scale": torch.ones(dm, device=device), "bias": torch.zeros(dm, device=device)}

    p = {"embed": {"embedding": r(mc.vocab_size, dm)}, "pos_embed": r(mc.max_len, dm, std=0.02)}
    for i in range(mc.n_layers):
        p[f"ln_attn_{i}"] = ln()
        p[f"attn_{i}"] = {n: {"kernel": r(dm, H, dh, std=dm ** -0.5), "bias": torch.zeros(H, dh, device=device)}
                          for n in ("query", "key", "value")}
        p[f"attn_{i}"]["out"] = {"kernel": r(H, dh, dm, std=dm ** -0.5), "bias": torch.zeros(dm, device=device)}
        p[f"ln_ffn_{i}"] = ln()
        if i not in mc.memory_layers or mc.memory_ffn:
            p[f"ffn_in_{i}"] = dense(dm, dm * mc.ffn_mult)
            p[f"ffn_out_{i}"] = dense(dm * mc.ffn_mult, dm)
        if i in mc.memory_layers:
            p[f"router_{i}"] = dense(dm, mc.pool_heads * mc.d_key)
            p[f"mem_gate_{i}"] = dense(dm, mc.d_value)
            p[f"mem_out_{i}"] = dense(mc.d_value, dm)
    p["pool"] = {"sub_keys": sub_keys, "values": values,
                 "log_temperature": torch.tensor(math.log(10.0), device=device)}
    p["ln_final"] = ln()
    return p


def run_cfg1(args):
    """configs[1], the full model forward: byte-BPE vocabulary 16,384, d_model
    256, 4 layers, 4 attention heads, FFN x4, seq 256, batch 32, memory
    layers 1 and 3 sharing one pool of 262,144 x 256 fp16 rows (H 4, top_k
    16, d_key 128, the reference run's setting); random-init weights, tokens
    uniform over the vocabulary.  A step is one memlayer_model_forward
    (embeddings -> 4 layers -> tied logits [8192, 16384]); the two memory
    layers' own time is measured separately (their calls alone)."""
    import torch

    from model_b200 import MemoryPoolLM, ModelConfig
    from model_b200 import _lib as L
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    W = dict(WORKLOAD, name="cfg1_model_forward", d_key=128, values_dtype="f16")
    B, T = 32, 256
    mc = ModelConfig(vocab_size=16384, max_len=T, d_model=256, n_layers=4, n_heads=4, ffn_mult=4,
                     memory_layers=(1, 3), n_sub_keys=512, pool_heads=4, d_key=128, d_value=256, top_k=16)
    x = make_inputs(torch, device, W, "f16", W["seed"])
    model = MemoryPoolLM(mc)
    prep = model.prepare(_model_params(torch, device, mc, x["values"], x["sub_keys"], W["seed"]))
    g = torch.Generator(device=device).manual_seed(W["seed"] + 7)
    tokens = torch.randint(0, mc.vocab_size, (B, T), device=device, generator=g, dtype=torch.int32)
    stream = torch.cuda.current_stream(device)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=device)
    launches0 = L.lib().memlayer_kernel_launch_count()
    prep.forward(tokens, check=True)
    launches = L.lib().memlayer_kernel_launch_count() - launches0
    for _ in range(args.warmup):
        flush.zero_()
        prep.forward(tokens)
    torch.cuda.synchronize()
    K = args.steps
    e = [_events(torch, 2) for _ in range(K)]
    with ClockSampler(device.index) as clk:
        for i in range(K):
            flush.zero_()
            e[i][0].record(stream)
            logits = prep.forward(tokens)
            e[i][1].record(stream)
        torch.cuda.synchronize()
    ms = statistics.mean(a.elapsed_time(b) for a, b in e)
    # the two memory layers' calls alone, on the same hidden-state size
    xs = [x, make_inputs(torch, device, W, "f16", W["seed"] + 1)]
    xs[1]["values"], xs[1]["sub_keys"] = x["values"], x["sub_keys"]
    calls = [LayerCall(torch, L, W, xx, device, "f16") for xx in xs]
    me = [_events(torch, 2) for _ in range(K)]
    for i in range(K):
        flush.zero_()
        me[i][0].record(stream)
        for c in calls:
            c(stream)
        me[i][1].record(stream)
    torch.cuda.synchronize()
    mem_ms = statistics.mean(a.elapsed_time(b) for a, b in me)
    # e2e: tokens in from pinned host memory, the logits' argmax back (the step's result)
    tok_host = tokens.cpu().pin_memory()
    tok_dev = torch.empty_like(tokens)
    out_host = torch.empty(B, T, dtype=torch.int64).pin_memory()
    ee = _events(torch, 2)
    torch.cuda.synchronize()
    ee[0].record(stream)
    for i in range(K):
        tok_dev.copy_(tok_host, non_blocking=True)
        lg = prep.forward(tok_dev)
        out_host.copy_(lg.argmax(-1), non_blocking=True)
    ee[1].record(stream)
    torch.cuda.synchronize()
    e2e_ms = ee[0].elapsed_time(ee[1]) / K
    dm, F, V = 256, 1024, mc.vocab_size
    dense_per_token = 2 * (4 * 4 * dm * dm + 2 * 2 * dm * F + dm * V)   # qkv + out in 4 layers, 2 FFNs, logits
    attn_per_token = 4 * 2 * 2 * (T // 2) * dm                          # QK^T and PV over half the keys
    line = _common_line(W, 1, K, args.warmup, ms, B * T / (ms * 1e-3), "tokens/s", "f32", {
        "metric": "model forward tokens/s", "scaling": "n/a",
        "backbone_flops_per_token": dense_per_token + attn_per_token, "stages_ms": {"model_forward": ms, "memory_layers_alone": mem_ms},
        "config": {"workload": "cfg1_model_forward", "vocab": mc.vocab_size, "d_model": 256, "layers": 4,
                   "heads": 4, "ffn_mult": 4, "seq": T, "batch": B, "memory_layers": [1, 3],
                   "pool": "262144 x 256 fp16, H 4, top_k 16, d_key 128", "values_dtype": "f16",
                   "l2": "flushed before every step"},
        "gpu_launches_per_step": int(launches),
        "e2e": {"value": B * T / (e2e_ms * 1e-3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": tok_host.numel() * 4, "d2h_bytes_per_step": out_host.numel() * 8,
                "api": "MemoryPoolLM (memlayer_model_forward), tokens copied in, argmax of the logits copied out"},
        "clocks": clk.summary(),
        "data": "synthetic: random-init weights, tokens uniform over the vocabulary",
        "note": "float32 backbone on the tensor cores (3xTF32 Dense layers), float32 SIMT attention"})
    del logits
    return line


def run_cfg4(args, rank=0, world=1):
    """configs[0] shapes, f32 values, 8192 Zipf-clustered tokens
    per GPU; step = layer forward with routing statistics + backward through
    the router (balance term included; the read-output gradient feeds the row
    update) + fetched-row gradients + global-norm clip + row-wise Adagrad on
    the touched rows + key_diversity_loss with its gradient.
    revive_dead_keys (every revive_every steps in the reference) is timed
    once beside it (rank 0).  The upstream gradient of the layer's output is
    drawn (the backbone is not built).  With N > 1 the table is row-sharded:
    the sharded forward, then the owner-sharded row update (each rank's
    merged rows pushed to their owners over NVLink) with a drawn probe
    gradient (the layer backward is single-GPU); times are the max over
    ranks."""
    import torch

    from model_b200 import _lib as L
    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)) if world > 1 else 0)
    torch.cuda.set_device(device)
    W = dict(WORKLOAD, name="cfg4_sparse_update", values_dtype="f32")
    N = W["n_sub_keys"] ** 2
    T, d, H, k = W["tokens_per_gpu"], W["d_value"], W["heads"], W["top_k"]
    if world > 1:
        from model_b200.shard import connect, shard_rows
        rows = shard_rows(N, rank, world)
        x = make_inputs(torch, device, W, "f32", W["seed"], rows)
        x["h"] = clustered_hidden(torch, device, T, W["d_model"], W["seed"] + 1 + rank)
        call = ShardedLayerCall(torch, L, W, x, device, "f32")
    else:
        rows = N
        x = make_inputs(torch, device, W, "f32", W["seed"])
        x["h"] = clustered_hidden(torch, device, T, W["d_model"], W["seed"] + 1)
        call = LayerCall(torch, L, W, x, device, "f32")
        # a training forward keeps its read output for the backward (as MemoryLayer.apply_train does)
        mem_keep = torch.empty(T, W["d_value"], device=device)
        call.args.mem = mem_keep.data_ptr()
    cnt_slot = torch.empty(N, device=device)
    cnt_sub = torch.empty(H, 2, W["n_sub_keys"], device=device)
    bal = torch.empty(1, device=device)
    call.args.pool.slot_counts, call.args.pool.subkey_counts = cnt_slot.data_ptr(), cnt_sub.data_ptr()
    call.args.pool.balance_loss = bal.data_ptr()
    accum = torch.zeros(rows, device=device)
    lib = L.lib()
    # the backward through the router (memlayer_layer_backward, single GPU): the
    # upstream gradient dy of the layer's output is drawn (no backbone); its
    # read-output gradient is the probe gradient the row update consumes
    # (model.py:114-115).  Row-sharded (N > 1): no backward yet, the probe
    # gradient is drawn.
    dm = W["d_model"]
    dy = torch.randn(T, dm, device=device, generator=torch.Generator(device=device).manual_seed(13 + rank)) * 1e-3
    g = torch.randn(T, d, device=device, generator=torch.Generator(device=device).manual_seed(7 + rank)) * 1e-3
    if world == 1:
        gb = {n_: torch.empty(*sh, device=device) for n_, sh in (
            ("dh", (T, dm)), ("dw_router", (dm, H * W["d_key"])), ("db_router", (H * W["d_key"],)),
            ("dsub_keys", tuple(x["sub_keys"].shape)), ("dlog_temperature", (1,)), ("dw_gate", (dm, d)),
            ("db_gate", (d,)), ("dw_out", (d, dm)), ("db_out", (dm,)))}
        ga = L.MemlayerLayerGrads(dy=dy.data_ptr(), balance_coef=0.01, route_through_pool=0,
                                  forward_workspace=call.ws.data_ptr(), probe=g.data_ptr(),
                                  **{n_: t.data_ptr() for n_, t in gb.items()})
        bnb = C.c_size_t()
        L.check(lib.memlayer_layer_backward_workspace_size(C.byref(call.cfg), 1, C.byref(bnb)), "backward ws")
        bws = torch.empty(bnb.value, dtype=torch.uint8, device=device)

    def backward():
        if world == 1:
            L.check(lib.memlayer_layer_backward(C.byref(call.cfg), C.byref(call.args), C.byref(ga), bws.data_ptr(),
                                                bnb.value, stream.cuda_stream), "memlayer_layer_backward")
    rest = torch.tensor([0.5], device=device)
    scale = torch.empty(1, device=device)
    n_u = torch.empty(1, dtype=torch.int32, device=device)
    # the C call of memlayer_row_adagrad (train.py:378-383, 396-399), or of
    # memlayer_row_adagrad_sharded on the row-sharded table, built once
    reads = (L.MemlayerRead * 1)(L.MemlayerRead(slots=call.slots.data_ptr(), weights=call.weights.data_ptr(),
                                                grad=g.data_ptr(), tokens=T))
    ada = L.MemlayerAdagradArgs(values=x["values"].data_ptr(), accum=accum.data_ptr(), lr=0.01, grad_clip=1.0,
                                rest_sq_norm=rest.data_ptr(), clip_scale=scale.data_ptr(), n_unique=n_u.data_ptr())
    rb = C.c_size_t()
    if world > 1:
        rcomm = connect(call.cfg, n_reads=1)
        L.check(lib.memlayer_shard_rowgrad_workspace_size(rcomm.handle, T * H * k, C.byref(rb)), "rowgrad ws")
    else:
        L.check(lib.memlayer_rowgrad_workspace_size(C.byref(call.cfg), T * H * k, C.byref(rb)), "rowgrad ws")
    rws = torch.empty(rb.value, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=device)

    def update():
        if world > 1:
            L.check(lib.memlayer_row_adagrad_sharded(C.byref(call.cfg), reads, 1, C.byref(ada), rcomm.handle,
                                                     L.PHASE_ALL, rws.data_ptr(), rb.value, stream.cuda_stream),
                    "memlayer_row_adagrad_sharded")
        else:
            L.check(lib.memlayer_row_adagrad(C.byref(call.cfg), reads, 1, C.byref(ada), rws.data_ptr(), rb.value,
                                             stream.cuda_stream), "memlayer_row_adagrad")
    # key_diversity_loss and its gradient, scaled by key_diversity_coef (train.py:327-329)
    kd_loss = torch.empty(1, device=device)
    kd_grad = torch.empty_like(x["sub_keys"])
    kb = C.c_size_t()
    L.check(lib.memlayer_key_diversity_workspace_size(C.byref(call.cfg), C.byref(kb)), "key diversity ws")
    kws = torch.empty(max(kb.value, 256), dtype=torch.uint8, device=device)

    def diversity():
        L.check(lib.memlayer_key_diversity(C.byref(call.cfg), x["sub_keys"].data_ptr(), kd_loss.data_ptr(),
                                           kd_grad.data_ptr(), 0.01, kws.data_ptr(), kb.value, stream.cuda_stream),
                "memlayer_key_diversity")
    for _ in range(args.warmup):
        flush.zero_()
        call(stream)
        backward()
        update()
        diversity()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    K = args.steps
    e0, e1, e2, e3, eb = (_events(torch, K) for _ in range(5))
    for i in range(K):
        flush.zero_()
        e0[i].record(stream)
        call(stream)
        e1[i].record(stream)
        backward()
        eb[i].record(stream)
        update()
        e2[i].record(stream)
        diversity()
        e3[i].record(stream)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    step = statistics.mean(e0[i].elapsed_time(e3[i]) for i in range(K))
    fwd = statistics.mean(e0[i].elapsed_time(e1[i]) for i in range(K))
    bwd = statistics.mean(e1[i].elapsed_time(eb[i]) for i in range(K))
    upd = statistics.mean(eb[i].elapsed_time(e2[i]) for i in range(K))
    div = statistics.mean(e2[i].elapsed_time(e3[i]) for i in range(K))
    # the same forward with the training-time selection noise (memory.py:155-159: a
    # standard Gumbel sample scaled by routing_noise * noise_scale), which takes the
    # score kernel's general top-k path
    gum = -torch.log(-torch.log(torch.rand(T, H, 2, W["n_sub_keys"], device=device,
                                           generator=torch.Generator(device=device).manual_seed(11))
                                .clamp_(min=torch.finfo(torch.float32).tiny)))
    call.args.pool.train, call.args.pool.noise_scale, call.args.pool.gumbel = 1, 1.0, gum.data_ptr()
    for _ in range(args.warmup):
        flush.zero_()
        call(stream)
    torch.cuda.synchronize()
    n0, n1 = _events(torch, K), _events(torch, K)
    for i in range(K):
        flush.zero_()
        n0[i].record(stream)
        call(stream)
        n1[i].record(stream)
    torch.cuda.synchronize()
    fwd_noisy = statistics.mean(n0[i].elapsed_time(n1[i]) for i in range(K))
    call.args.pool.train, call.args.pool.gumbel = 0, None
    U = int(n_u.item())
    if world > 1:
        t = torch.tensor([step, fwd, bwd, upd, div, fwd_noisy], dtype=torch.float64, device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        u_all = torch.tensor([U], dtype=torch.int64, device=device)
        torch.distributed.all_reduce(u_all)
        torch.cuda.synchronize()
        torch.distributed.barrier()
        rcomm.close()
        call.comm.close()
        if rank != 0:
            return None
        step, fwd, bwd, upd, div, fwd_noisy = t.tolist()
        U = int(u_all.item())
    # revive_dead_keys (every revive_every steps in the reference trainer), timed on its own on copies
    from model_b200 import keys as KM
    q_sample = torch.nn.functional.normalize(torch.randn(4096, H, 2, W["d_key"] // 2, device=device), dim=-1)
    usage = torch.distributions.Dirichlet(torch.full((W["n_sub_keys"],), 0.3)).sample((H, 2)).to(device)
    rv0, rv1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(3):
        KM.revive_dead_keys(x["sub_keys"], usage, q_sample, 0.5, generator=torch.Generator(device).manual_seed(1))
    pick = torch.randint(0, 4096, (H, 2, W["n_sub_keys"]), device=device)
    normal = torch.randn_like(x["sub_keys"])
    rv0.record(stream)
    _, _, rdead = KM.revive_dead_keys(x["sub_keys"], usage, q_sample, 0.5, pick=pick, normal=normal)
    rv1.record(stream)
    torch.cuda.synchronize()
    revive_ms = rv0.elapsed_time(rv1)
    F = T * H * k
    hbm, src = peaks()
    upd_bytes = F * 8 + T * d * 4 + U * (2 * d * 4 + 8) // world
    return _common_line(W, world, K, args.warmup, step, world * T / (step * 1e-3), "tokens/s", "f32", {
        "scaling": "weak", "stages_ms": {"forward": fwd, "backward": bwd, "row_grad_adagrad": upd,
                                         "key_diversity": div},
        "forward_with_selection_noise_ms": fwd_noisy,
        "stage_note": "max over ranks of each stage" if world > 1 else "per-stage means",
        "revive_dead_keys_ms": revive_ms, "revived": int(rdead.sum().item()),
        "unique_rows": U, "fetches": F * world, "clip_scale": float(scale.item()),
        "row_update": {"algorithmic_bytes": upd_bytes, "achieved_gbs": upd_bytes / (upd * 1e-3) / 1e9,
                       "peak": hbm, "peak_source": src, "frac": upd_bytes / (upd * 1e-3) / 1e9 / hbm,
                       "bytes_note": "per rank: slots+weights of every fetch, one read of every probe-gradient row, "
                                     "read+write of its share of the touched value rows and accumulators"},
        "note": ("upstream gradient dy drawn (no backbone); backward through the router with the balance "
                 "term (coef 0.01) gives the row update's probe gradient; L2 flushed before every step")
                if world == 1 else
                ("table row-sharded, owner-sharded row update over NVLink; the layer backward is single-GPU, "
                 "so the probe gradient is drawn here; L2 flushed before every step")})


def run_host(args):
    """configs[2] shapes (H 4, top_k 16, d_key 128, d_value 256 fp16) with the
    value table in page-locked host memory (the reference's host tier,
    memory.py:180-183): n_sub_keys 4096 (16.8 M slots x 512 B = 8.6 GB
    pinned; smaller when the host has less than 4x that available).  Per call
    latency at batch 1, 8 and 64 and the 8192-token throughput; host-link
    bytes = distinct rows x 512 B (each crosses once per call)."""
    import torch

    from model_b200 import _lib as L
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    n_sub, H, k, dk, d = 4096, 4, 16, 128, 256
    avail = 0
    with open("/proc/meminfo") as f:
        for line in f:
            if line.startswith("MemAvailable:"):
                avail = int(line.split()[1]) * 1024
    while n_sub > 512 and 4 * n_sub * n_sub * d * 2 > avail:
        n_sub //= 2
    N = n_sub * n_sub
    table = torch.empty(N, d, dtype=torch.float16, pin_memory=True)
    g = torch.Generator(device=device).manual_seed(0)
    step = 1 << 20
    for s0 in range(0, N, step):     # filled from the GPU: fast and seeded
        s1 = min(s0 + step, N)
        table[s0:s1].copy_((torch.randn(s1 - s0, d, device=device, generator=g) * 0.02).half())
    torch.cuda.synchronize()
    sub_keys = torch.randn(H, 2, n_sub, dk // 2, device=device, generator=g) * (1 / 128) ** 0.5
    log_t = torch.tensor([math.log(10.0)], device=device)
    stream = torch.cuda.current_stream(device)
    res = {}
    for M in (1, 8, 64, 8192):
        cfg = L.MemlayerConfig(tokens=M, heads=H, n_sub_keys=n_sub, d_key=dk, d_value=d, top_k=k, d_model=256,
                               values_dtype=L.F16, routing_noise=1.0, min_temperature=10.0, max_temperature=100.0)
        q = torch.randn(M, H, dk, device=device, generator=g)
        out = torch.empty(M, d, device=device)
        sl = torch.empty(M, H, k, dtype=torch.int32, device=device)
        w = torch.empty(M, H, k, device=device)
        a = L.MemlayerPoolArgs(queries=q.data_ptr(), sub_keys=sub_keys.data_ptr(), log_temperature=log_t.data_ptr(),
                               values=table.data_ptr(), out=out.data_ptr(), slots=sl.data_ptr(), weights=w.data_ptr())
        nb = C.c_size_t()
        L.check(L.lib().memlayer_host_table_workspace_size(C.byref(cfg), C.byref(nb)), "host table ws")
        ws = torch.empty(nb.value, dtype=torch.uint8, device=device)
        f = L.lib().memlayer_pool_forward_host_table
        for _ in range(args.warmup):
            L.check(f(C.byref(cfg), C.byref(a), ws.data_ptr(), nb.value, stream.cuda_stream), "host table fwd")
        torch.cuda.synchronize()
        reps = max(args.steps, 20) if M < 8192 else args.steps
        e0, e1 = _events(torch, 2)
        e0.record(stream)
        for _ in range(reps):
            L.check(f(C.byref(cfg), C.byref(a), ws.data_ptr(), nb.value, stream.cuda_stream), "host table fwd")
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        U = int(torch.unique(sl).numel())
        res[str(M)] = {"ms_per_call": ms, "tokens_per_s": M / (ms * 1e-3), "distinct_rows": U,
                       "fetches": M * H * k, "host_link_gbs": U * d * 2 / (ms * 1e-3) / 1e9}
    big = res["8192"]
    W = dict(WORKLOAD, name="host_table_cfg2_shapes", n_sub_keys=n_sub, d_key=dk, values_dtype="f16",
             tokens_per_gpu=8192)
    return _common_line(W, 1, args.steps, args.warmup, big["ms_per_call"], big["tokens_per_s"], "tokens/s", "f16", {
        "scaling": "weak", "per_batch": res, "table_bytes_pinned_host": N * d * 2,
        "note": "value table in page-locked host memory; each distinct row crosses the host link once per call; "
                "no L2 flush (the host table is not cached in HBM)"})


def run_cfg2(args):
    """configs[2] decode: n_sub_keys 8192 (67,108,864 slots x 256 fp16 =
    34.4 GB, HBM-resident), H 4, top_k 16, d_key 128, d_model 256; one call
    per decode step at batch 1, 8 and 64; per-step device latency."""
    import torch

    from model_b200 import _lib as L
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    res = {}
    W = dict(WORKLOAD, name="cfg2_decode", n_sub_keys=8192, d_key=128, values_dtype="f16")
    x = None
    for B in (1, 8, 64):
        Wb = dict(W, tokens_per_gpu=B)
        if x is None:
            x = make_inputs(torch, device, Wb, "f16", W["seed"])
        else:
            x["h"] = torch.randn(B, W["d_model"], device=device)
        call = LayerCall(torch, L, Wb, x, device, "f16")
        stream = torch.cuda.current_stream(device)
        for _ in range(args.warmup):
            call(stream)
        torch.cuda.synchronize()
        ev = [_events(torch, L.STAGE_EVENTS) for _ in range(args.steps)]
        for row in ev:
            for e in row:
                e.record(stream)
        torch.cuda.synchronize()
        for i in range(args.steps):
            call(stream, ev[i])
        torch.cuda.synchronize()
        t = sorted(e[0].elapsed_time(e[5]) * 1000 for e in ev)
        st = lambda a, b: statistics.median(e[a].elapsed_time(e[b]) * 1000 for e in ev)  # noqa: E731
        res[B] = {"p50_us": t[len(t) // 2], "p90_us": t[int(len(t) * 0.9)], "tokens_per_s": B / (t[len(t) // 2] * 1e-6),
                  "stages_us": {"prep_projections": st(0, 2), "score_topk": st(2, 3), "combine_gather": st(3, 4),
                                "finalize_out": st(4, 5)}}
        # the same layer call as one CUDA graph per decode step (model_b200.generate.LayerDecodeStep);
        # host-observed rate: each step issued, run and waited for, as a token-by-token loop does
        from model_b200 import MemoryLayer, MemoryPool
        from model_b200.generate import LayerDecodeStep, decode_steps_per_second
        pool = MemoryPool(n_sub_keys=W["n_sub_keys"], heads=W["heads"], d_key=W["d_key"], d_value=W["d_value"],
                          top_k=W["top_k"])
        layer = MemoryLayer(pool, d_model=W["d_model"], layer=1)
        lp = {"router_1": {"kernel": x["w_router"], "bias": x["b_router"]},
              "mem_gate_1": {"kernel": x["w_gate"], "bias": x["b_gate"]},
              "mem_out_1": {"kernel": x["w_out"], "bias": x["b_out"]},
              "pool": {"sub_keys": x["sub_keys"], "values": x["values"], "log_temperature": x["log_t"]}}
        gstep = LayerDecodeStep(layer, lp, B)
        estep = LayerDecodeStep(layer, lp, B, graph=False)
        for _ in range(args.warmup):
            gstep.step(x["h"])
            estep.step(x["h"])
        ge = _events(torch, 2 * args.steps)
        for i in range(args.steps):
            ge[2 * i].record(stream)
            gstep.step(x["h"], stream)
            ge[2 * i + 1].record(stream)
        torch.cuda.synchronize()
        gt = sorted(ge[2 * i].elapsed_time(ge[2 * i + 1]) * 1000 for i in range(args.steps))
        res[B]["graph_p50_us"] = gt[len(gt) // 2]
        res[B]["host_steps_per_s"] = {"eager": decode_steps_per_second(estep, 200),
                                      "graph": decode_steps_per_second(gstep, 200)}
    # the whole model's decode step around the same pool (4 layers, d_model 256, 4 heads, FFN x4,
    # memory layers 1 and 3, 16,384-token vocabulary): MemoryPoolLM's Generator, one CUDA graph per step
    from model_b200 import Generator, MemoryPoolLM, ModelConfig
    mc = ModelConfig(vocab_size=16384, max_len=256, d_model=256, n_layers=4, n_heads=4, ffn_mult=4,
                     memory_layers=(1, 3), n_sub_keys=W["n_sub_keys"], pool_heads=4, d_key=128, d_value=256, top_k=16)
    prep = MemoryPoolLM(mc).prepare(_model_params(torch, device, mc, x["values"], x["sub_keys"], W["seed"]))
    model_res = {}
    for B in (1, 8, 64):
        gen = Generator(MemoryPoolLM(mc), prep, batch_size=B)
        tok = torch.randint(0, mc.vocab_size, (B,), device=device, dtype=torch.int32)
        for i in range(args.warmup):
            gen.step(tok, i)
        gs = gen.stream
        ge = _events(torch, 2 * args.steps)
        for i in range(args.steps):
            ge[2 * i].record(gs)
            gen.step(tok, (args.warmup + i) % mc.max_len)
            ge[2 * i + 1].record(gs)
        torch.cuda.synchronize()
        if gen.status():
            raise RuntimeError(f"model decode step status {gen.status()}")
        gt = sorted(ge[2 * i].elapsed_time(ge[2 * i + 1]) * 1000 for i in range(args.steps))
        t0 = time.perf_counter()
        n = 100
        for i in range(n):
            gen.step(tok, i % mc.max_len)
            gs.synchronize()
        host = n / (time.perf_counter() - t0)
        model_res[B] = {"graph_p50_us": gt[len(gt) // 2], "graph_p90_us": gt[int(len(gt) * 0.9)],
                        "tokens_per_s": B / (gt[len(gt) // 2] * 1e-6), "host_steps_per_s": host}
        del gen
    return _common_line(W, 1, args.steps, args.warmup, res[64]["p50_us"] / 1000, res[64]["tokens_per_s"],
                        "tokens/s", "f16", {"scaling": "n/a", "decode": res, "model_decode": model_res,
                                            "note": "value = batch 64; per-step device time, L2 not flushed "
                                                    "(decode steps run back to back); graph_p50_us: the same "
                                                    "call replayed as a CUDA graph; host_steps_per_s: steps "
                                                    "issued and waited for one at a time; model_decode: the "
                                                    "whole model's decode step (backbone + both memory layers "
                                                    "+ 16,384-way logits) around the same 34 GB pool"})


def run_cfg3(args, rank, world):
    """n_sub_keys 32768 (2^30 slots x 256 bf16 = 550 GB)
    row-sharded over the ranks, H 8, top_k 32, d_key 256, d_model 256;
    65,536 Zipf-clustered tokens in total (65,536 / N per rank)."""
    import torch

    from model_b200 import _lib as L
    from model_b200.shard import shard_rows
    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(device)
    W = dict(WORKLOAD, name="cfg3_billion_slot_prefill", n_sub_keys=32768, heads=8, top_k=32, d_key=256,
             values_dtype="bf16", tokens_per_gpu=65536 // world)
    rows = shard_rows(W["n_sub_keys"] ** 2, rank, world)
    x = make_inputs(torch, device, W, "bf16", W["seed"], rows)
    x["h"] = clustered_hidden(torch, device, W["tokens_per_gpu"], W["d_model"], W["seed"] + 1 + rank)
    call = ShardedLayerCall(torch, L, W, x, device, "bf16")
    stream = torch.cuda.current_stream(device)
    for _ in range(args.warmup):
        call(stream)
    torch.cuda.synchronize()
    K = args.steps
    ev = [_events(torch, L.STAGE_EVENTS) for _ in range(K)]
    pev = [_events(torch, 2) for _ in range(K)]
    for row in ev:
        for e in row:
            e.record(stream)
    torch.cuda.synchronize()
    torch.distributed.barrier()
    for i in range(K):
        call(stream, ev[i], pev[i])
    torch.cuda.synchronize()
    torch.distributed.barrier()
    ms = statistics.mean(ev[i][0].elapsed_time(ev[i][5]) for i in range(K))
    st = lambda a, b: statistics.mean(ev[i][a].elapsed_time(ev[i][b]) for i in range(K))  # noqa: E731
    stages = {"projections": st(0, 1), "score_topk": st(2, 3), "combine_push": st(3, 4),
              "shard_gather": statistics.mean(pev[i][0].elapsed_time(pev[i][1]) for i in range(K)),
              "reduce_out": statistics.mean(pev[i][1].elapsed_time(ev[i][5]) for i in range(K))}
    t = torch.tensor([ms] + list(stages.values()), dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    torch.cuda.synchronize()
    torch.distributed.barrier()
    call.comm.close()
    if rank != 0:
        return None
    ms = float(t[0])
    stages = dict(zip(stages, t[1:].tolist()))
    score_flops = 2 * 65536 * W["heads"] * 2 * W["n_sub_keys"] * (W["d_key"] // 2)
    tp, _ = tensor_peak()
    return _common_line(W, world, K, args.warmup, ms, 65536 / (ms * 1e-3), "tokens/s", "bf16", {
        "scaling": "strong", "stages_ms_max_over_ranks": stages,
        "score_tflops_per_gpu": score_flops / world / (stages["score_topk"] * 1e-3) / 1e12,
        "tensor_peak": tp, "note": "no L2 flush (the 68.7 GB/GPU table and 1.1 TFLOP/GPU score GEMM dwarf L2)"})


def run_emulated(args):
    """configs[0] shapes on P communicators of one process and one GPU: each
    phase is launched for every rank before the next phase, so no kernel
    waits on a later launch.  Reports per-phase device time per rank."""
    import torch

    from model_b200 import MemoryLayer, MemoryPool
    from model_b200 import _lib as L
    from model_b200.shard import ShardedCall, emulated_comms, shard_values
    world = args.emulate_ranks
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    W = dict(WORKLOAD, tokens_per_gpu=args.tokens)
    pool = MemoryPool(n_sub_keys=W["n_sub_keys"], heads=W["heads"], d_key=W["d_key"], d_value=W["d_value"],
                      top_k=W["top_k"])
    layer = MemoryLayer(pool, d_model=W["d_model"], layer=1)
    params = layer.init(W["seed"])
    T = W["tokens_per_gpu"]
    comms = emulated_comms(pool.config(T, torch.float32, W["d_model"]), world)
    calls = []
    for r in range(world):
        p = dict(params, pool=dict(params["pool"], values=shard_values(params["pool"]["values"], r, world)))
        h = torch.randn(T, W["d_model"], device=device, generator=torch.Generator(device=device).manual_seed(r))
        calls.append(ShardedCall(layer, comms[r], p, h))
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    res = {ph: [] for ph in ("route", "gather", "reduce")}
    for it in range(args.warmup + args.steps):
        for ph, code in (("route", L.PHASE_ROUTE), ("gather", L.PHASE_GATHER), ("reduce", L.PHASE_REDUCE)):
            ev = []
            for c in calls:
                flush.zero_()
                e0, e1 = _events(torch, 2)
                e0.record(stream)
                c.run(code)
                e1.record(stream)
                ev.append((e0, e1))
            torch.cuda.synchronize()
            if it >= args.warmup:
                res[ph] += [a.elapsed_time(b) for a, b in ev]
    for c in calls:
        c.check()
        c.comm.close()
    ms = {k: statistics.median(v) for k, v in res.items()}
    return {"metric": "row-sharded phase time per rank (emulated ranks, one GPU)", "value": sum(ms.values()),
            "unit": "ms", "n_gpus": 1, "emulated_ranks": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": False, "phases_ms": ms, "config": {"workload": "cfg0_layer_forward_sharded_emulated",
                                                                   "tokens_per_rank": T},
            "note": "partial rows and inbox entries stay in this GPU's memory: no NVLink traffic"}


def main():
    args = parse()
    W = dict(WORKLOAD, values_dtype=args.values_dtype, tokens_per_gpu=args.tokens)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1 and args.impl == "ours":
        import datetime

        import torch
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    if args.impl == "reference":
        line = run_reference(args, W, rank)
    elif args.emulate_ranks:
        line = run_emulated(args)
    elif args.workload == "cfg4":
        line = run_cfg4(args, rank, world)
    elif args.workload == "cfg1":
        line = run_cfg1(args)
    elif args.workload == "cfg2":
        line = run_cfg2(args)
    elif args.workload == "host":
        line = run_host(args)
    elif args.workload == "cfg3":
        line = run_cfg3(args, rank, world)
    else:
        line = run_ours(args, W, rank, world)
    if line is not None:
        print(json.dumps(line), flush=True)
    if world > 1 and args.impl == "ours":
        import torch
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
