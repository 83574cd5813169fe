"""Benchmark of the two-stage block-sparse attention forward on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 3]
                    [--impl ours|reference] [--scaling weak|strong]

A *step* is one forward pass (pool -> score/select -> fine) over one batch of
synthetic inputs of the chosen workload (default: B1 H8 N32768 D64, bf16,
block_size 64, top_k 16, causal -- the shape the reference's headline numbers
are quoted on).  Rank 0 prints one JSON line.

* ``value``: effective TFLOP/s (FLOPs of the reference's benchmark/flops.py
  model, summed over every unit all ranks processed, divided by the max over
  ranks of the CUDA-event time of K steps), inputs resident in HBM, L2
  flushed before every step.  Each timed step replays a CUDA graph of one
  whole forward (captured once after the warm-up: every kernel and memset
  of the step runs every step; ``--no-graph`` launches them directly).
  With N GPUs the workload's (batch, head) units
  are split over the ranks (``--scaling strong``, the default; ``weak`` runs
  the whole workload on every rank); ``with_gather`` then times the forward
  plus the NCCL all-gather that assembles the whole output on every rank.
* ``stages`` / ``roofline_path``: per-stage and whole-path algorithmic bytes
  and FLOPs against the measured HBM and bf16 peaks.
* ``e2e``: the same metric through the public host-memory entry point
  (``attention_from_host``) with pinned host buffers: the host->device copies
  of Q, K, V and the device->host copy of O are inside the timed region
  (overlapped with the forward, chunk by chunk of units).
* ``roofline``: the fine-stage kernel, FLOPs per launch / its event time
  against the measured bf16 dense peak.
* ``cpu_baseline``: the numpy restatement of the reference's block_indexer
  timed on this host's cores on a bounded sample (rank 0, N=1 only).

``--impl reference`` times the reference algorithm on the host cores (the
oracle port of attention/block_indexer.py) on the same workload -- every
unit and every query row per step -- and prints the same line with
``"impl": "reference"``.

``--mode decode`` measures decode-time reuse instead (its own JSON line):
one step appends one token per (batch, head) unit to a KV cache of the
workload's shape that is nearly full, re-pools the block it lands in and
attends the new row over the cache, all in one launch
(``bsa_decode_step``); ``value`` is milliseconds per step, with the roofline
of the step's HBM bytes and the decode oracle timed on the host beside it.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "block-sparse attn fwd ms + effective TFLOPS & HBM GB/s at N=32k, 1/2/4/8 B200"

WORKLOADS = {
    1: dict(B=1, H=8, N=1024, D=64, block_size=64, top_k=16, causal=True, dist="normal"),
    2: dict(B=1, H=8, N=8192, D=64, block_size=64, top_k=16, causal=False, dist="normal"),
    3: dict(B=1, H=8, N=32768, D=64, block_size=64, top_k=16, causal=True, dist="normal"),
    4: dict(B=2, H=32, N=32768, D=128, block_size=64, top_k=32, causal=True, dist="clustered"),
    5: dict(B=1, H=16, N=131072, D=64, block_size=128, top_k=16, causal=True, dist="block_scaled"),
}
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_FLUSH_BYTES = 256 << 20
STAGES = ["pool", "select", "bucket", "fine", "combine"]


def workload_name(cfg):
    return (f"block-sparse attention fwd B{cfg['B']} H{cfg['H']} N{cfg['N']} D{cfg['D']} "
            f"bs{cfg['block_size']} k{cfg['top_k']} {'causal' if cfg['causal'] else 'non-causal'} "
            f"{cfg['dist']}")


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    except (OSError, ValueError):
        return dict(FALLBACK_PEAKS), "fallback"


def per_query_flops(cfg):
    from flash_vs_sparse_attention_b200.flops import compute_flops
    return compute_flops(1, 1, cfg["N"], cfg["D"], "block_indexer_b200", cfg["block_size"],
                         cfg["top_k"]) // cfg["N"]


# --------------------------------------------------------------------------
# Clock sampling during the timed region.
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        import tempfile
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.25)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary(self):
        rows = []
        try:
            for line in open(self.path):
                f = [x.strip() for x in line.split(",")]
                if len(f) >= 9 and f[1].replace(".", "").isdigit():
                    rows.append(f)
        except OSError:
            pass
        finally:
            if self.path:
                try:
                    os.unlink(self.path)
                except OSError:
                    pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm = [float(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]),
                "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit()),
                "samples": len(rows), "reasons": reasons}


# --------------------------------------------------------------------------
def gpu_inputs(cfg, n_units, seed, device):
    """Synthetic (1, n_units, N, D) bf16 inputs generated on the device with the
    workload's value distribution."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    N, D, bs = cfg["N"], cfg["D"], cfg["block_size"]
    shape = (1, n_units, N, D)

    def randn(*s):
        return torch.randn(*s, generator=g, device=device, dtype=torch.float32)

    if cfg["dist"] == "normal":
        out = [randn(*shape) for _ in range(3)]
    elif cfg["dist"] == "block_scaled":
        nb = N // bs
        out = []
        for _ in range(3):
            sc = torch.rand(1, n_units, nb, 1, 1, generator=g, device=device) * 1.5 + 0.5
            out.append((randn(1, n_units, nb, bs, D) * sc).reshape(shape))
    elif cfg["dist"] == "clustered":
        nb = N // bs
        centres = randn(1, n_units, 64, D)
        ck = torch.randint(0, 64, (1, n_units, nb), generator=g, device=device)
        cq = torch.randint(0, 64, (1, n_units, nb), generator=g, device=device)

        def blocks(ids):
            c = torch.gather(centres, 2, ids[..., None].expand(-1, -1, -1, D))
            return c[:, :, :, None, :].expand(-1, -1, -1, bs, -1).reshape(shape)

        kc = blocks(ck)
        out = [blocks(cq) + 0.1 * randn(*shape), kc + 0.1 * randn(*shape), kc + 0.1 * randn(*shape)]
    else:
        raise ValueError(cfg["dist"])
    return [t.to(torch.bfloat16).contiguous() for t in out]


def run_ours(args, cfg):
    import torch
    import torch.distributed as dist

    from flash_vs_sparse_attention_b200 import _lib
    from flash_vs_sparse_attention_b200 import block_indexer_b200 as bi
    from flash_vs_sparse_attention_b200 import flops as F
    from flash_vs_sparse_attention_b200.sharding import unit_range

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    U = cfg["B"] * cfg["H"] if not args.units else args.units
    if args.scaling is None:
        args.scaling = "strong"   # one problem's (batch, head) units split over the ranks
    if args.scaling == "weak":
        my_units = U
        total_units = U * world
    else:
        a, b = unit_range(U, world, rank)
        my_units = b - a
        total_units = U
    if my_units == 0:
        raise SystemExit("strong scaling with more ranks than units")
    Q, K, V = gpu_inputs(cfg, my_units, seed=1000 + rank, device=dev)
    O = torch.empty_like(Q)
    L = _lib.lib()
    p = bi.problem(1, my_units, cfg["N"], cfg["D"], cfg["causal"], cfg["block_size"], cfg["top_k"])
    ws_bytes = bi.workspace_bytes(p)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    sp = ctypes.c_void_p(stream.cuda_stream)
    n_launch = ctypes.c_int(0)
    ev_arr = (ctypes.c_void_p * len(STAGES))()

    def forward(stage_events=None, stream_handle=None):
        if stage_events is not None:
            for i, e in enumerate(stage_events):
                ev_arr[i] = ctypes.c_void_p(e.cuda_event)
            evp = ev_arr
        else:
            evp = None
        st = L.bsa_forward_ex(ctypes.byref(p), ctypes.c_void_p(Q.data_ptr()),
                              ctypes.c_void_p(K.data_ptr()), ctypes.c_void_p(V.data_ptr()),
                              ctypes.c_void_p(O.data_ptr()), ctypes.c_void_p(ws.data_ptr()),
                              ctypes.c_size_t(ws_bytes), stream_handle or sp, evp,
                              len(STAGES) if evp else 0, ctypes.byref(n_launch))
        _lib.check(st, "bsa_forward_ex")

    for _ in range(args.warmup):
        flush.zero_()
        forward()
    torch.cuda.synchronize()

    # The timed steps replay a CUDA graph of one forward (every kernel and
    # memset of the step, captured once with the same buffers), which removes
    # the per-launch gaps the host call leaves between kernels; the stage
    # times come from a second, directly launched pass with stage events.
    graph = None
    if not args.no_graph:
        gs = torch.cuda.Stream(dev)
        gs.wait_stream(stream)
        with torch.cuda.stream(gs):
            forward(stream_handle=ctypes.c_void_p(gs.cuda_stream))
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=gs):
            forward(stream_handle=ctypes.c_void_p(gs.cuda_stream))
        torch.cuda.synchronize()
        graph_launches = n_launch.value
        for _ in range(2):
            flush.zero_()
            graph.replay()
        torch.cuda.synchronize()

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    stage_ev = [[torch.cuda.Event(enable_timing=True) for _ in STAGES] for _ in range(args.steps)]
    # torch creates the CUDA event on its first record; create them all now so
    # the C ABI can record them by handle inside the timed region.
    for evs in stage_ev:
        for e in evs:
            e.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches = 0
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            flush.zero_()
            starts[i].record(stream)
            if graph is not None:
                graph.replay()
                launches += graph_launches
            else:
                forward(stage_ev[i])
                launches += n_launch.value
            ends[i].record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    stage_starts = starts
    if graph is not None:
        # Stage times: the same steps launched directly with stage events.
        stage_starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        for i in range(args.steps):
            flush.zero_()
            stage_starts[i].record(stream)
            forward(stage_ev[i])
        torch.cuda.synchronize()
    stage_ms = {name: [] for name in STAGES}
    for i in range(args.steps):
        prev = stage_starts[i]
        for name, e in zip(STAGES, stage_ev[i]):
            stage_ms[name].append(prev.elapsed_time(e))
            prev = e
    total = torch.tensor([sum(step_ms)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(total, op=dist.ReduceOp.MAX)
    total_ms = total.item()
    ms_per_step = total_ms / args.steps
    flops_step = F.compute_flops(1, total_units, cfg["N"], cfg["D"], "block_indexer_b200",
                                 cfg["block_size"], cfg["top_k"])
    value = flops_step * args.steps / (total_ms * 1e-3) / 1e12
    hbm_bytes = F.min_hbm_bytes(1, total_units, cfg["N"], cfg["D"])

    # ---- end to end through the public API with pinned host buffers ----
    e2e = None
    if not args.no_e2e:
        Qh, Kh, Vh = (t.cpu().pin_memory() for t in (Q, K, V))
        Oh = torch.empty(Q.shape, dtype=Q.dtype).pin_memory()

        def e2e_step():
            # Host buffers in, host buffer out: the public host-memory entry
            # point overlaps the PCIe copies of one chunk of units with the
            # forward of the previous one, and returns when O is on the host.
            bi.attention_from_host(Qh, Kh, Vh, causal=cfg["causal"],
                                   block_size=cfg["block_size"], top_k=cfg["top_k"], out=Oh)

        for _ in range(max(1, args.warmup)):
            e2e_step()
        torch.cuda.synchronize()
        es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        es.record(stream)
        for _ in range(args.steps):
            e2e_step()
        ee.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([es.elapsed_time(ee)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = t.item()
        e2e = {"value": round(flops_step * args.steps / (e2e_ms * 1e-3) / 1e12, 4),
               "unit": "TFLOP/s", "ms_per_step": round(e2e_ms / args.steps, 4),
               "h2d_bytes_per_step": 3 * Q.numel() * Q.element_size(),
               "d2h_bytes_per_step": O.numel() * O.element_size()}
        del Qh, Kh, Vh, Oh

    # ---- the head-sharded output gathered on every rank (N > 1) ----
    # The same forward followed by the all-gather of every rank's units
    # (sharding.gather_units: one all_gather_into_tensor over NCCL), timed as
    # its own region: the latency a caller that wants the whole output sees.
    with_gather = None
    if world > 1 and args.scaling == "strong":
        from flash_vs_sparse_attention_b200.sharding import gather_units
        for _ in range(args.warmup):
            flush.zero_()
            forward()
            gather_units(O, U)
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        gs, ge = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g_ms = 0.0
        for _ in range(args.steps):
            flush.zero_()
            gs.record(stream)
            forward()
            gather_units(O, U)
            ge.record(stream)
            torch.cuda.synchronize()
            g_ms += gs.elapsed_time(ge)
        t = torch.tensor([g_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        per = -(-U // world)
        shard_bytes = per * cfg["N"] * cfg["D"] * 2
        with_gather = {"ms_per_step": round(t.item() / args.steps, 4),
                       "value": round(flops_step * args.steps / (t.item() * 1e-3) / 1e12, 4),
                       "unit": "TFLOP/s",
                       "collective": "all_gather_into_tensor (NCCL) of the (batch, head) shards",
                       "bytes_per_rank": shard_bytes, "bytes_total": shard_bytes * world}

    # ---- roofline of the fine-stage kernel ----
    # The stage events cover the first pass of the forward; a workload whose
    # units do not fit one workspace runs in passes of `pass_units` (the
    # forward halves the unit count until the pass fits the workspace).
    pass_units = my_units
    while pass_units > 1 and L.bsa_workspace_bytes(ctypes.byref(p), pass_units) > ws_bytes:
        pass_units = (pass_units + 1) // 2
    peaks, peak_kind = load_peaks()
    fine_ms = statistics.mean(stage_ms["fine"])
    fine_flops = F.fine_matmul_flops(1, pass_units, cfg["N"], cfg["D"], cfg["block_size"],
                                     cfg["top_k"])
    achieved = fine_flops / (fine_ms * 1e-3) / 1e12 if fine_ms > 0 else None
    peak = float(peaks["bf16_tflops"])
    # DRAM traffic of the fine kernel per (batch, head) unit, from a one-launch
    # ncu capture of a smaller case (profiles/traffic.json), scaled by the
    # units of this launch (the traffic grows in proportion to the units).
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tpath):
        try:
            per_unit = json.load(open(tpath)).get(f"config{args.config}", {}).get("fine_per_unit")
            traffic = int(per_unit * pass_units) if per_unit else None
        except (OSError, ValueError, TypeError):
            traffic = None
    stages = stage_model(cfg, pass_units, {k: statistics.mean(v) for k, v in stage_ms.items()},
                         peaks, peak_kind)
    path_flops = F.compute_flops(1, my_units, cfg["N"], cfg["D"], "block_indexer_b200",
                                 cfg["block_size"], cfg["top_k"])
    path_tflops = path_flops * args.steps / (total_ms * 1e-3) / 1e12
    roofline_path = {
        "tflops": round(path_tflops, 2),
        "tensor_frac": round(path_tflops / float(peaks["bf16_tflops"]), 4),
        "hbm_gbs": round(F.min_hbm_bytes(1, my_units, cfg["N"], cfg["D"]) * args.steps
                         / (total_ms * 1e-3) / 1e9, 2),
        "hbm_frac": round(F.min_hbm_bytes(1, my_units, cfg["N"], cfg["D"]) * args.steps
                          / (total_ms * 1e-3) / 1e9 / float(peaks["hbm_gbs"]), 4),
        "note": "per rank: flops.py FLOPs and compulsory bytes (Q, K, V in, O out) over the "
                "step time, against the measured bf16 GEMM and copy peaks"}
    roofline = {"kernel": "fine (tensor-core, key-block-stationary)", "bound": "tensor",
                "achieved": round(achieved, 2) if achieved else None, "peak": peak,
                "unit": "TFLOP/s", "frac": round(achieved / peak, 4) if achieved else None,
                "peak_source": f"{peak_kind} bf16_tflops (burst)",
                "traffic": traffic,
                "traffic_unit": "bytes per launch (ncu per-unit figure in profiles/traffic.json x units)",
                "traffic_gbs": round(traffic / (fine_ms * 1e-3) / 1e9, 1) if traffic and fine_ms > 0 else None,
                "flops_per_launch": fine_flops, "units_per_launch": pass_units,
                "launch_ms": round(fine_ms, 4)}

    if world > 1:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 4), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": workload_name(cfg) + (
                           f" (only {U} of {cfg['B'] * cfg['H']} units)" if args.units else ""),
                       "units_per_gpu": my_units,
                       "total_units": total_units, "global_batch": cfg["B"] * (world if args.scaling == "weak" else 1),
                       "heads": cfg["H"], "seq_len": cfg["N"], "head_dim": cfg["D"],
                       "block_size": cfg["block_size"], "top_k": cfg["top_k"],
                       "causal": cfg["causal"], "parallelism": f"head-sharded x{world}",
                       "l2": f"flushed before every step ({L2_FLUSH_BYTES >> 20} MiB write, outside the events)",
                       "launch": ("one CUDA graph of a whole forward (all its kernels and memsets), "
                                  "captured once and replayed every step; stage times from a "
                                  "direct pass") if graph is not None else "direct launches"},
            "hbm_gbs": round(hbm_bytes * args.steps / (total_ms * 1e-3) / 1e9, 2),
            "hbm_gbs_note": "compulsory bytes (read Q,K,V + write O) / step time",
            "stages_ms": {k: round(statistics.mean(v), 4) for k, v in stage_ms.items()},
            "stages_units": pass_units,
            "stages": stages,
            "roofline_path": roofline_path,
            "with_gather": with_gather,
            "roofline": roofline, "clocks": clk.summary(), "e2e": e2e,
            "gpu_launches": launches,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(cfg, args)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def stage_model(cfg, units, stage_ms, peaks, peak_kind):
    """Per stage of one pass of ``units`` units: its algorithmic HBM bytes (and
    FLOPs), what bounds it, and the achieved fraction of that bound from the
    stage's CUDA-event time.  Bytes per unit (N rows, D, k, nb blocks):
      pool    K in, block means out (fp32 + bf16 hi/lo)    N D 2 + nb D 8
      select  Q and the hi/lo means in, idx out            N D 2 + nb D 4 + N k 4
              (+ 2 * 2 N nb D FLOP on tensor cores, half with causal skipping)
      bucket  idx in twice, V in (block max), lists and
              (query, slot) map out                         4 N k 4 + N D 2
      fine    Q, K, V in, partials out (fp16 O + m, l)     3 N D 2 + N k (2 D + 8)
              (+ 4 N k bs D FLOP: the flops.py fine-matmul term)
      combine partials and map in, O out                   N k (2 D + 8) + N k 4 + N D 2
    """
    from flash_vs_sparse_attention_b200 import flops as F
    N, D, k, bs = cfg["N"], cfg["D"], cfg["top_k"], cfg["block_size"]
    nb = N // bs
    u = units
    part = N * k * (2 * D + 8)
    model = {
        "pool": (u * (N * D * 2 + nb * D * 8), 0),
        "select": (u * (N * D * 2 + nb * D * 4 + N * k * 4),
                   u * 2 * 2 * N * nb * D // (2 if cfg["causal"] else 1)),
        "bucket": (u * (4 * N * k * 4 + N * D * 2), 0),
        "fine": (u * (3 * N * D * 2 + part), F.fine_matmul_flops(1, u, N, D, bs, k)),
        "combine": (u * (part + N * k * 4 + N * D * 2), 0),
    }
    hbm, tc = float(peaks["hbm_gbs"]), float(peaks["bf16_tflops"])
    out = {}
    for name, (nbytes, nflop) in model.items():
        ms = stage_ms.get(name, 0.0)
        if ms <= 0:
            continue
        gbs = nbytes / (ms * 1e-3) / 1e9
        d = {"ms": round(ms, 4), "bytes": nbytes, "gbs": round(gbs, 1), "hbm_frac": round(gbs / hbm, 4)}
        if nflop:
            tf = nflop / (ms * 1e-3) / 1e12
            d.update({"flops": nflop, "tflops": round(tf, 2), "tensor_frac": round(tf / tc, 4)})
        d["bound"] = "tensor" if name == "fine" else "hbm"
        out[name] = d
    out["peaks"] = f"{peak_kind} hbm_gbs {hbm}, bf16_tflops {tc} (burst)"
    return out


# --------------------------------------------------------------------------
def cpu_sample(cfg, n_rows, seed=0):
    """Bounded CPU sample: ``n_rows`` query rows of unit 0, in whole 512-row
    chunks spread evenly over the sequence (causal rows late in the sequence
    see more blocks, early ones fewer)."""
    from oracle import unit_inputs
    q, k, v = unit_inputs(cfg, 0, seed)
    N = cfg["N"]
    chunks = max(1, n_rows // 512)
    starts = sorted({int(round(x)) * 512 for x in
                     [i * (N // 512 - 1) / max(1, chunks - 1) for i in range(chunks)]})
    rows = [list(range(s, min(N, s + 512))) for s in starts]
    return q, k, v, rows


def time_oracle(cfg, q, k, v, rows_list, threads):
    """Run the oracle's attention on each row chunk with ``threads`` workers."""
    import concurrent.futures as cf
    import numpy as np
    from oracle import attention_unit
    from oracle.block_indexer_np import _limit_blas_threads

    def one(rows):
        attention_unit(q, k, v, cfg["causal"], cfg["block_size"], cfg["top_k"],
                       rows=np.asarray(rows))

    t0 = time.perf_counter()
    with _limit_blas_threads(1), cf.ThreadPoolExecutor(threads) as ex:
        list(ex.map(one, rows_list))
    return time.perf_counter() - t0


def cpu_baseline(cfg, args):
    threads = os.cpu_count() or 1
    q, k, v, rows = cpu_sample(cfg, args.cpu_rows or cfg["N"])
    n = sum(len(r) for r in rows)
    time_oracle(cfg, q, k, v, rows[:1], threads)  # warm-up
    secs = time_oracle(cfg, q, k, v, rows, threads)
    fl = per_query_flops(cfg) * n
    return {"value": round(fl / secs / 1e12, 6), "unit": "TFLOP/s", "cores": threads,
            "kind": "port", "seconds": round(secs, 3),
            "sample": f"{n} query rows of unit 0 ({len(rows)} chunks of 512 spread over N) through "
                      f"the numpy restatement of attention/block_indexer.py, {threads} threads"}


def run_reference(args, cfg):
    """The reference algorithm (the oracle port of attention/block_indexer.py)
    on the host cores, on the same workload as our arm: every (batch, head)
    unit and every query row per timed step (``--cpu-rows R`` instead times R
    rows of unit 0).  Warm-up steps run one 512-row chunk each."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np
    from oracle import unit_inputs
    threads = os.cpu_count() or 1
    U, N = cfg["B"] * cfg["H"], cfg["N"]
    if args.cpu_rows:
        q, k, v, rows = cpu_sample(cfg, args.cpu_rows)
        units = [(q, k, v, rows)]
        sample = (f"{sum(len(r) for r in rows)} query rows of unit 0 per step, numpy restatement "
                  f"of attention/block_indexer.py, {threads} host threads")
    else:
        units = []
        for u in range(U):
            q, k, v = unit_inputs(cfg, u, 0)
            units.append((q, k, v, [list(range(s0, min(N, s0 + 512))) for s0 in range(0, N, 512)]))
        sample = (f"the whole workload per step: all {U} units x {N} query rows, numpy "
                  f"restatement of attention/block_indexer.py, {threads} host threads")
    n = sum(len(r) for (_, _, _, rs) in units for r in rs)
    fl = per_query_flops(cfg) * n
    q0, k0, v0, r0 = units[0]
    for _ in range(args.warmup):
        time_oracle(cfg, q0, k0, v0, r0[:1], threads)
    times = []
    for _ in range(args.steps):
        times.append(sum(time_oracle(cfg, q, k, v, rs, threads) for (q, k, v, rs) in units))
    total = sum(times)
    value = fl * args.steps / total / 1e12
    world = int(os.environ.get("WORLD_SIZE", "1"))
    line = {
        "metric": METRIC, "value": round(value, 6), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": args.scaling or "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": {"workload": workload_name(cfg), "total_units": U, "global_batch": cfg["B"],
                   "heads": cfg["H"], "seq_len": N, "head_dim": cfg["D"],
                   "block_size": cfg["block_size"], "top_k": cfg["top_k"], "causal": cfg["causal"],
                   "rows_per_step": n, "parallelism": f"{threads} host threads of rank 0"},
        "cpu_baseline": {"value": round(value, 6), "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------
DECODE_METRIC = "block-sparse decode step ms (1 new token per head, KV cache N=32k)"


def run_decode(args, cfg):
    """One step = append one token per unit to a cache of N keys (the step's K
    and V rows written in), re-pool the block it lands in, attend the new row
    over the cache: one bsa_decode_step launch.  L2 is flushed before every
    step, outside the events."""
    import numpy as np
    import torch

    from flash_vs_sparse_attention_b200 import _lib
    from flash_vs_sparse_attention_b200 import block_indexer_b200 as bi

    if int(os.environ.get("WORLD_SIZE", "1")) != 1:
        raise SystemExit("--mode decode runs on one GPU")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    U, N, D, bs, k = cfg["B"] * cfg["H"], cfg["N"], cfg["D"], cfg["block_size"], cfg["top_k"]
    n_new = args.warmup + args.steps
    Q, K, V = gpu_inputs(cfg, U, seed=7, device=dev)       # positions [0, N)
    start = N - n_new                                      # cache length before the first step
    L = _lib.lib()
    p = bi.problem(1, U, N, D, True, bs, k)
    K_repr = torch.zeros(1, U, N // bs, D, dtype=torch.float32, device=dev)
    Kc, Vc = torch.zeros_like(K), torch.zeros_like(V)
    Kc[:, :, :start], Vc[:, :, :start] = K[:, :, :start], V[:, :, :start]
    bi.pool_k_blocks(Kc, K_repr, 0, -(-start // bs), start, bs)
    O = torch.empty(1, U, 1, D, dtype=torch.bfloat16, device=dev)
    rows = [[t_[:, :, t:t + 1].contiguous() for t in range(start, N)] for t_ in (Q, K, V)]
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    sp = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)

    def step(i):
        _lib.check(L.bsa_decode_step(ctypes.byref(p), bi._ptr(rows[0][i]), bi._ptr(rows[1][i]),
                                     bi._ptr(rows[2][i]), start + i, bi._ptr(Kc), bi._ptr(Vc),
                                     bi._ptr(K_repr), bi._ptr(O), sp), "bsa_decode_step")

    for i in range(args.warmup):
        flush.zero_()
        step(i)
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(0) as clk:
        for j in range(args.steps):
            flush.zero_()
            starts[j].record()
            step(args.warmup + j)
            ends[j].record()
        torch.cuda.synchronize()
    ms = [a.elapsed_time(b) for a, b in zip(starts, ends)]
    ms_step = sum(ms) / len(ms)
    # The floor of this timing pattern: the same flush and event pair around
    # a one-element fill (one tiny kernel, no memory traffic to speak of).
    tiny = torch.zeros(1, device=dev)
    floor = []
    for j in range(args.steps):
        flush.zero_()
        starts[j].record()
        tiny.fill_(1.0)
        ends[j].record()
    torch.cuda.synchronize()
    floor = sorted(a.elapsed_time(b) for a, b in zip(starts, ends))
    floor_ms = floor[len(floor) // 2]
    # HBM bytes a step must move: the visible block means (fp32), the top_k
    # selected blocks' K and V, the new row's Q, K, V in and O out, and the
    # re-pooled block (its keys in, its mean out).
    nbv = N // bs
    step_bytes = U * (nbv * D * 4 + k * bs * D * 2 * 2 + 4 * D * 2 + bs * D * 2 + D * 4)
    peaks, peak_kind = load_peaks()
    achieved = step_bytes / (ms_step * 1e-3) / 1e9
    # The decode oracle on the host for one step (all units, 1 thread).
    from oracle import decode_rows
    Qn, Kn, Vn = (t[0].float().cpu().numpy() for t in (Q, K, V))
    t_last = N - 1
    t0 = time.perf_counter()
    for u in range(U):
        decode_rows(Qn[u, t_last:t_last + 1], t_last, Kn[u], Vn[u], True, bs, k)
    cpu_ms = (time.perf_counter() - t0) * 1e3
    line = {
        "metric": DECODE_METRIC, "value": round(ms_step, 5), "unit": "ms", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": f"decode step {workload_name(cfg)}: 1 new row per unit, cache of "
                               f"{start}..{N - 1} keys", "units": U,
                   "l2": f"flushed before every step ({L2_FLUSH_BYTES >> 20} MiB write, outside the events)"},
        "tokens_per_s": round(U / (ms_step * 1e-3), 1),
        "roofline": {"kernel": "decode step (append, re-pool, select, attend: one launch)", "bound": "hbm",
                     "achieved": round(achieved, 2), "peak": float(peaks["hbm_gbs"]), "unit": "GB/s",
                     "frac": round(achieved / float(peaks["hbm_gbs"]), 5),
                     "peak_source": f"{peak_kind} hbm_gbs", "traffic": None,
                     "bytes_per_step": step_bytes,
                     "note": "one launch per step, a cluster of 8 CTAs per unit; at a few MB the step is "
                             "bound by dependent memory round trips and the launch",
                     "event_floor_ms": round(floor_ms, 5),
                     "event_floor_note": "median of the same flush + event pair around a one-element "
                                         "fill: launch and event overhead, not step work"},
        "clocks": clk.summary(), "gpu_launches": args.steps,
        "cpu_baseline": {"value": round(cpu_ms, 3), "unit": "ms", "cores": 1, "kind": "port",
                         "sample": f"one decode step of all {U} units (the last position) through the "
                                   "numpy decode oracle, 1 thread"},
    }
    print(json.dumps(line), flush=True)


BACKWARD_METRIC = "block-sparse attn bwd ms (fine-stage dQ, dK, dV; selection fixed)"


def run_backward(args, cfg):
    """One step = the backward pass of the workload's fine stage (bsa_backward:
    the per-row log-sum-exp, the bucket lists, the per-block kernel, the dQ
    sum) for a fixed selection, forward output and output gradient.  L2 is flushed before every step, outside
    the events.  Algorithmic work: the five products of an attention backward
    over the selected keys (scores, dP, dQ, dK, dV), 10 N k bs D FLOP a unit."""
    import torch

    from flash_vs_sparse_attention_b200 import block_indexer_b200 as bi

    if int(os.environ.get("WORLD_SIZE", "1")) != 1:
        raise SystemExit("--mode backward runs on one GPU")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    U = args.units or cfg["B"] * cfg["H"]
    N, D, bs, k, causal = cfg["N"], cfg["D"], cfg["block_size"], cfg["top_k"], cfg["causal"]
    Q, K, V = gpu_inputs(cfg, U, seed=9, device=dev)
    dO = torch.randn(Q.shape, generator=torch.Generator(device=dev).manual_seed(10),
                     device=dev).to(torch.bfloat16)
    idx = bi.select_blocks(Q, K, causal=causal, block_size=bs, top_k=k)
    O = bi.fine(Q, K, V, idx, causal=causal, block_size=bs)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    for _ in range(args.warmup):
        flush.zero_()
        bi.backward(Q, K, V, O, dO, idx, causal, bs)
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(0) as clk:
        for j in range(args.steps):
            flush.zero_()
            starts[j].record()
            bi.backward(Q, K, V, O, dO, idx, causal, bs)
            ends[j].record()
        torch.cuda.synchronize()
    ms_step = sum(a.elapsed_time(b) for a, b in zip(starts, ends)) / args.steps
    flop = 10 * U * N * k * bs * D
    peaks, peak_kind = load_peaks()
    tflops = flop / (ms_step * 1e-3) / 1e12
    # The oracle's backward on the host for a sample: the first rows of unit
    # 0 (causal rows see only earlier keys, so a prefix is their whole work).
    from oracle.backward_np import backward_unit
    rows = min(N, 2048)
    q, kk, v, g = (t[0, 0, :rows].float().cpu().numpy() for t in (Q, K, V, dO))
    t0 = time.perf_counter()
    backward_unit(q, kk, v, g, causal, bs, min(k, rows // bs))
    cpu_ms = (time.perf_counter() - t0) * 1e3
    line = {
        "metric": BACKWARD_METRIC, "value": round(ms_step, 4), "unit": "ms", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": f"backward {workload_name(cfg)}", "units": U,
                   "l2": f"flushed before every step ({L2_FLUSH_BYTES >> 20} MiB write, outside the events)"},
        "tflops": round(tflops, 2),
        "roofline": {"kernel": "backward (CUDA cores: per-block dK, dV and dQ shares)", "bound": "tensor",
                     "achieved": round(tflops, 2), "peak": float(peaks["bf16_tflops"]),
                     "unit": "TFLOP/s", "frac": round(tflops / float(peaks["bf16_tflops"]), 5),
                     "peak_source": f"{peak_kind} bf16_tflops", "traffic": None,
                     "flops_per_step": flop,
                     "note": "CUDA-core kernels measured against the tensor-core peak"},
        "clocks": clk.summary(), "gpu_launches": 6 * args.steps,
        "cpu_baseline": {"value": round(cpu_ms, 3), "unit": "ms", "cores": 1, "kind": "port",
                         "sample": f"rows 0..{rows - 1} of unit 0 through the numpy backward "
                                   "oracle, 1 thread (a causal prefix is the rows' whole work)"},
    }
    print(json.dumps(line), flush=True)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=3, choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--scaling", default=None, choices=["weak", "strong"],
                    help="strong (default): the workload's (batch, head) units are split over "
                         "the GPUs; weak: every GPU runs all of them")
    ap.add_argument("--cpu-rows", type=int, default=0,
                    help="query rows of unit 0 in the CPU timings (0: one whole unit for the "
                         "cpu_baseline key, the whole workload for --impl reference)")
    ap.add_argument("--units", type=int, default=0,
                    help="run only this many (batch, head) units of the workload (0: all); "
                         "for small profiling captures, not for bench lines")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-graph", action="store_true",
                    help="launch the timed steps directly instead of replaying a CUDA graph")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--mode", default="forward", choices=["forward", "decode", "backward"],
                    help="decode: one-token decode steps over a KV cache; backward: the fine "
                         "stage's gradients (each its own JSON line)")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        raise SystemExit("--warmup must be at least 3")
    cfg = WORKLOADS[args.config]
    if args.mode == "decode":
        run_decode(args, cfg)
    elif args.mode == "backward":
        run_backward(args, cfg)
    elif args.impl == "reference":
        run_reference(args, cfg)
    else:
        run_ours(args, cfg)


if __name__ == "__main__":
    main()
