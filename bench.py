"""Benchmark of the MoE-layer hot path (one JSON line on rank 0).

Workload: one MoE layer (hidden 2048, 256 routed experts of intermediate 512
in GGUF IQ4_XS, top-8 + a sigmoid-gated shared expert, f32 router) over a 512-token prefill
with a Zipf(1.1) per-expert router bias; seeded synthetic weights and tokens.  A step is one
``moe_forward`` (router, top-8, bucketing, grouped experts, combine) over 512 tokens.  The same
line carries the decode (M=1, config 0) figures under "decode".

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

--impl reference times the reference's algorithm on the host cores (the C restatement in
oracle/, f32 accumulation, all threads), on a bounded sample of the same workload.
With N > 1 (torchrun), the prefill is expert parallel: rank r holds experts [r*256/N, (r+1)*256/N)
and 512 tokens of its own; tokens travel to the ranks owning their experts and partial rows come
back through NCCL all-to-all (weak scaling, 512 tokens per GPU).  "config3" times 8192 tokens in
total over the N GPUs (strong scaling).  Decode runs on every GPU independently.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
PKG_DIR = ROOT / "moe-680m_b200"

METRIC = "MoE-layer tok/s at M=1 and 512-tok prefill; % of HBM / tensor-core roofline"
SEED = 20240601
PREFILL_M = 512
ZIPF = 1.1
CPU_SAMPLE_TOKENS = 512
PREFILL_LAYERS = 4  # independently seeded config-1 layers, cycled step by step (no L2 reuse)
WORKLOAD = ("config1: prefill 512 tok per GPU, Zipf(1.1) router bias, 1 MoE layer "
            "(H=2048, I=512, E=256, top-8 + gated shared, IQ4_XS)")
CONFIG3_M = 8192
CONFIG2_LAYERS = 40
CONFIG2_STEPS = 256
CONFIG4_M = 64
VOCAB, VOCAB_HIDDEN = 248320, 2048  # the LM head (token_embd) of the reference model
VOCAB_BYTES = VOCAB * VOCAB_HIDDEN // 256 * 136


def load_pkg():
    if "moe680m_b200" in sys.modules:
        return sys.modules["moe680m_b200"]
    spec = importlib.util.spec_from_file_location("moe680m_b200", PKG_DIR / "__init__.py",
                                                  submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["moe680m_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def ncu_traffic(kernel_stage: str):
    """DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) of a stage's kernel
    from the committed ncu summaries: a line ``ncu_dram_bytes[<stage>]: <bytes> (<file note>)``."""
    import re
    for f in sorted((ROOT / "profiles").glob("*.md")):
        for line in f.read_text().splitlines():
            m = re.match(r"\s*ncu_dram_bytes\[(\w+)\]:\s*(\d+)", line)
            if m and m.group(1) == kernel_stage:
                return int(m.group(2)), f"profiles/{f.name}"
    return None, None


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, dev_id: str | None):
        self.p = None
        self.dev = dev_id

    def __enter__(self):
        try:
            cmd = ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "200"]
            if self.dev:
                cmd += ["-i", self.dev]
            self.p = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.p = None
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.p:
            time.sleep(0.25)
            self.p.terminate()
            try:
                self.out, _ = self.p.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()

    def summary(self):
        rows = [r.split(", ") for r in (self.out or "").strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def distinct_experts(routed: np.ndarray) -> int:
    return len(np.unique(routed))


NVLINK_GBS = 770.0  # measured peer-copy bandwidth per direction per GPU on this pool's B200s


def ep_exchange_bytes(routed_all: np.ndarray, world: int, m: int, epr: int, hidden: int, k: int,
                      transport: str = "peer", capacity: int | None = None) -> np.ndarray:
    """Bytes each rank moves over NVLink in one expert-parallel step, [world][2] (out, in).

    routed_all: [world*m, k] expert ids, rank r's tokens at rows r*m..(r+1)*m.  A token visits
    the ranks owning its experts; the visits to other ranks cross NVLink twice: the row and its
    record (hidden*4 + (k+1)*8 bytes) to the expert rank, the partial row (hidden*4 bytes) back."""
    n = world * m
    owner = np.repeat(np.arange(world), m)
    visits = np.zeros((n, world), bool)
    visits[np.arange(n)[:, None], routed_all.astype(np.int64) // epr] = True
    visits[np.arange(n), owner] = False
    sent = np.array([visits[owner == r].sum() for r in range(world)], np.int64)  # rows r dispatches
    recv = visits.sum(axis=0).astype(np.int64)                                     # rows r serves
    row_in, row_back = hidden * 4 + (k + 1) * 8, hidden * 4
    if transport != "peer":
        # the NCCL all-to-alls move whole fixed-capacity blocks to and from every other rank,
        # used rows or not
        cap = capacity if capacity is not None else m
        blk = (world - 1) * cap * (row_in + row_back)
        return np.full((world, 2), blk, np.int64)
    out = sent * row_in + recv * row_back
    inn = recv * row_in + sent * row_back
    return np.stack([out, inn], axis=1)


def cpu_baseline(shapes, x: np.ndarray, min_seconds: float = 10.0, threads: int = 0):
    """C restatement of the reference's MoE layer (f32 accumulation) on the host cores: whole
    512-token prefills repeated until ``min_seconds`` of CPU time have passed."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import coracle
    layer = host_layer(shapes)
    xs = np.ascontiguousarray(x)
    coracle.moe_forward(layer, xs[:4], xs[:4], acc64=False, nthreads=threads)  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        coracle.moe_forward(layer, xs, xs, acc64=False, nthreads=threads)
        n += xs.shape[0]
        dt = time.perf_counter() - t0
        if dt >= min_seconds:
            break
    return layer, n / dt, dt, n


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    pkg = load_pkg()
    from moe680m_b200 import synth
    sys.path.insert(0, str(ROOT / "oracle"))
    import coracle
    sh = synth.LayerShapes()
    layer = coracle.synthetic_layer(SEED, 0, sh, ZIPF)
    x = synth.tokens(SEED, 0, PREFILL_M, sh.hidden)
    # every host thread, explicitly: torchrun exports OMP_NUM_THREADS=1, which the OpenMP
    # default of the C restatement would otherwise honour
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    n = CPU_SAMPLE_TOKENS
    for i in range(args.warmup):
        coracle.moe_forward(layer, x[:n], x[:n], acc64=False, nthreads=cores)
    times = []
    for i in range(args.steps):
        xs = np.ascontiguousarray(np.roll(x, -n * i, axis=0)[:n])
        t0 = time.perf_counter()
        coracle.moe_forward(layer, xs, xs, acc64=False, nthreads=cores)
        times.append(time.perf_counter() - t0)
    ms = 1e3 * sum(times) / len(times)
    v = n / (ms / 1e3)
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
            "config": {"workload": WORKLOAD, "sample_tokens_per_step": n,
                       "omp_threads": cores},
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": "port",
                             "sample": f"{n} of the 512 prefill tokens per step; the reference "
                                       "(Rust+Vulkan) cannot be built here, so its algorithm runs "
                                       f"as the C restatement in oracle/ (f32 accumulation, OpenMP, "
                                       f"{cores} threads)"},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


_HOST_LAYER = {}


def host_layer(shapes):
    """Host copy of config-1 layer 0 for the C restatement (built once)."""
    if "l" not in _HOST_LAYER:
        sys.path.insert(0, str(ROOT / "oracle"))
        import coracle
        _HOST_LAYER["l"] = coracle.synthetic_layer(SEED, 0, shapes, ZIPF)
    return _HOST_LAYER["l"]


def oracle_rows_check(shapes, x: np.ndarray, got: np.ndarray, n_rows: int = 48) -> dict:
    """Sampled rows of a timed step's output against the f64 C oracle (the checker only)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import coracle
    rows = np.random.default_rng(7).choice(x.shape[0], size=min(n_rows, x.shape[0]), replace=False)
    rows.sort()
    xr = np.ascontiguousarray(x[rows])
    ref = coracle.moe_forward(host_layer(shapes), xr, xr, acc64=True, nthreads=os.cpu_count() or 0)["out64"]
    g = got[rows].astype(np.float64)
    return {"rows": int(len(rows)), "rel_l2": float(np.linalg.norm(g - ref) / np.linalg.norm(ref)),
            "max_rel": float(np.abs(g - ref).max() / np.abs(ref).max())}


def _max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _gather_floats(v: float, world: int) -> list:
    if world == 1:
        return [v]
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], device="cuda", dtype=torch.float64)
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [float(o.item()) for o in out]


def _barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def lm_head_leg(ctx, synth, stream, hbm, rank):
    """LM head: the 248,320 x 2048 IQ4_XS projection + greedy argmax (moe_vocab_logits), M = 1
    and 8, 50 timed launches each with CUDA events on the library's stream (the 270 MB weight
    exceeds the L2, so every launch reads it from HBM)."""
    import torch
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    wv = ctx.alloc(VOCAB_BYTES)
    ctx.synth_iq4xs(wv, synth.tensor_key(SEED, 90, 0, 0), 0, VOCAB_BYTES // 136)
    out = {"vocab": VOCAB, "hidden": VOCAB_HIDDEN, "alg_bytes_per_launch": VOCAB_BYTES,
           "l2": "270 MB weight exceeds the 126 MB L2"}
    for mv in (1, 8):
        xv = [ctx.put(synth.tokens(SEED + 17, rank * 1000 + i, mv, VOCAB_HIDDEN)) for i in range(4)]
        lv, iv = ctx.alloc(mv * VOCAB * 4), ctx.alloc(256)
        for i in range(3):
            ctx.vocab_logits(wv, VOCAB, VOCAB_HIDDEN, xv[i % 4], mv, lv, iv)
        torch.cuda.synchronize()
        kv = 50
        ev0.record(stream)
        for i in range(kv):
            ctx.vocab_logits(wv, VOCAB, VOCAB_HIDDEN, xv[i % 4], mv, lv, iv)
        ev1.record(stream)
        torch.cuda.synchronize()
        ctx.sync()
        usv = ev0.elapsed_time(ev1) / kv * 1e3
        gbs = VOCAB_BYTES / (usv / 1e6) / 1e9
        out[f"m{mv}"] = {"us_per_launch": usv, "hbm_gbs": gbs, "hbm_frac": gbs / hbm,
                         "outputs": "f32 logits + argmax ids"}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-check", action="store_true", help="skip the parity check of the timed step")
    ap.add_argument("--only", default="all", choices=["all", "prefill", "lm_head"],
                    help="prefill: skip the decode, config-3, end-to-end and CPU legs; lm_head: only "
                         "the LM-head leg, 0.3 GB on the device (profiling runs)")
    ap.add_argument("--ep", default="peer", choices=["peer", "nccl", "torch"],
                    help="expert-parallel exchange at N>1: peer = moe_forward_ep over NVLink peer memory "
                         "(default), nccl = moe_forward_ep over NCCL all-to-all, torch = ep.py over "
                         "torch.distributed")
    ap.add_argument("--path", type=int, default=0,
                    help="expert kernels: 0 auto, 1 CUDA-core GEMV, 2 tcgen05 (A in smem), 3 tcgen05 (A in TMEM)")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)

    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    load_pkg()
    from moe680m_b200 import ep, host, synth

    if args.only == "lm_head":  # the LM-head leg alone, on each rank's GPU
        arena = torch.empty(VOCAB_BYTES + (64 << 20), dtype=torch.uint8, device=torch.device("cuda", local))
        ctx = host.Context(local, arena.numel(), external_ptr=arena.data_ptr())
        stream = torch.cuda.Stream()
        torch.cuda.set_stream(stream)
        ctx.set_stream(stream.cuda_stream)
        res = lm_head_leg(ctx, synth, stream, peaks()[0], rank)
        if rank == 0:
            print(json.dumps({"lm_head": res}), flush=True)
        ctx.close()
        if world > 1:
            dist.destroy_process_group()
        return

    sh = synth.LayerShapes()
    E, H = sh.n_experts, sh.hidden
    ep_mode = world > 1
    epr = E // world
    my_experts = range(rank * epr, (rank + 1) * epr) if ep_mode else None
    only_prefill = args.only == "prefill"
    # decode layers: the 40-layer stack of config 2 (17 GB); the single-layer decode leg cycles
    # through them (no L2 hits)
    n_dec_layers = 0 if only_prefill else CONFIG2_LAYERS
    c3_tokens = CONFIG3_M // world
    n_full_check = 1 if (ep_mode and rank == 0) else 0  # rank 0's full layer for the EP parity check
    arena_bytes = ((n_dec_layers + PREFILL_LAYERS + n_full_check) * sh.expert_bytes * (E + 1)
                   + (0 if only_prefill else 2 * sh.expert_bytes * (E + 1))
                   + (0 if only_prefill else VOCAB_BYTES)
                   + (3 << 30))
    arena = torch.empty(arena_bytes, dtype=torch.uint8, device=torch.device("cuda", local))
    ctx = host.Context(local, arena_bytes, external_ptr=arena.data_ptr())
    stream = torch.cuda.Stream()  # a real stream: torch events, NCCL and the library share it
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream.cuda_stream)
    ctx.set_path(args.path)
    c_ep = ep_mode and args.ep != "torch"
    if c_ep:  # the library's own expert-parallel group (NCCL id from rank 0)
        uid = [host.Context.ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        ctx.ep_set_transport(host.MOE_EP_TRANSPORT_PEER if args.ep == "peer" else host.MOE_EP_TRANSPORT_NCCL)
        ctx.ep_init(uid[0], world, rank)
    pre_ids = host.build_synthetic_model(ctx, SEED, PREFILL_LAYERS, sh, ZIPF, experts=my_experts)[2]
    pre = pre_ids[0]
    dec_ids = host.build_synthetic_model(ctx, SEED + 1, n_dec_layers, sh, None)[2] if n_dec_layers else []
    K, W = args.steps, args.warmup
    n_x = K + W
    xs = [synth.tokens(SEED, rank * 1000 + i, PREFILL_M, H) for i in range(n_x)]
    x_offs = [ctx.put(x) for x in xs]
    out_off = ctx.alloc(PREFILL_M * H * 4)

    ep_graphs, ep_caps = [], []

    def make_step(lid, m, out):
        if c_ep:
            xin_ep = ctx.alloc(m * H * 4)  # the captured step's fixed input rows
            nb = m * H * 4
            arena[xin_ep:xin_ep + nb].zero_()
            ctx.forward_ep(lid, xin_ep, xin_ep, out, m, m)  # eager first step: buffers, workspace
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            try:
                with torch.cuda.graph(g, stream=stream):
                    ctx.forward_ep(lid, xin_ep, xin_ep, out, m, m)
                ok = 1
            except Exception as e:  # noqa: BLE001 - reported in the JSON line
                ok, why = 0, type(e).__name__
            flag = torch.tensor([ok], device=arena.device)
            dist.all_reduce(flag, op=dist.ReduceOp.MIN)
            captured = bool(int(flag.item()))
            if captured:
                ep_caps.append(g)
            ep_graphs.append(("captured" if captured else "eager" + ("" if ok else f" ({why})"))
                             + ", transport " + {0: "nccl", 1: "peer"}.get(ctx.ep_transport(), "?"))

            def step(x_off):
                if x_off != xin_ep:
                    arena[xin_ep:xin_ep + nb].copy_(arena[x_off:x_off + nb])
                if captured:
                    g.replay()
                else:
                    ctx.forward_ep(lid, xin_ep, xin_ep, out, m, m)

            def eager(x_off):
                arena[xin_ep:xin_ep + nb].copy_(arena[x_off:x_off + nb])
                ctx.forward_ep(lid, xin_ep, xin_ep, out, m, m)
            step.eager = eager
        elif ep_mode:
            xin_ep = ctx.alloc(m * H * 4)  # the captured step's fixed input rows
            ops = ep.LibraryEpOps(ctx, arena, lid, ep.EpShape(H, E, sh.top_k, world, m), rank,
                                  xin_ep, xin_ep, out)
            nb = m * H * 4
            arena[xin_ep:xin_ep + nb].zero_()
            ep.exchange_forward(ops, None, m, 1.0)  # eager first step: caches, workspace
            try:
                ep_caps.append(ep.CapturedExchange(ops, None, m, 1.0))
                ok = 1
            except Exception as e:  # noqa: BLE001 - reported in the JSON line
                ok, why = 0, type(e).__name__
            # every rank replays a graph or none does (collectives must match)
            flag = torch.tensor([ok], device=arena.device)
            dist.all_reduce(flag, op=dist.ReduceOp.MIN)
            if int(flag.item()):
                ci = len(ep_caps) - 1
                ep_graphs.append("captured")
            else:
                if ok:
                    ep_caps.pop()
                ci = None
                ep_graphs.append("eager" + ("" if ok else f" ({why})"))

            def step(x_off):
                if x_off != xin_ep:
                    arena[xin_ep:xin_ep + nb].copy_(arena[x_off:x_off + nb])
                if ci is not None:
                    ep_caps[ci].replay()
                else:
                    ep.exchange_forward(ops, None, m, 1.0)

            def eager(x_off):
                arena[xin_ep:xin_ep + nb].copy_(arena[x_off:x_off + nb])
                ep.exchange_forward(ops, None, m, 1.0)
            step.eager = eager
        else:
            ctx.reserve(lid, m)

            def step(x_off):
                ctx.forward(lid, x_off, x_off, out, m)
        return step

    # one step per layer; timed step i runs layer i mod PREFILL_LAYERS, so consecutive steps
    # stream different weights (4 layers x ~82 touched experts x 1.67 MB = 0.55 GB > the 126 MB L2)
    layer_steps = [make_step(lid, PREFILL_M, out_off) for lid in pre_ids]

    def step(x_off, i=0):
        layer_steps[i % PREFILL_LAYERS](x_off)
    step.eager = lambda x_off, i=0: getattr(layer_steps[i % PREFILL_LAYERS], "eager",
                                            layer_steps[i % PREFILL_LAYERS])(x_off)
    torch.cuda.synchronize()

    # ---- prefill: inputs resident in HBM ----------------------------------------------------
    for i in range(W):
        step(x_offs[i], i)
    ctx.sync()
    dev_uuid = None
    try:
        dev_uuid = str(torch.cuda.get_device_properties(local).uuid)
        dev_uuid = dev_uuid if dev_uuid.startswith("GPU-") else "GPU-" + dev_uuid
    except Exception:
        pass
    l0 = ctx.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(dev_uuid) as clk:
        ev0.record(stream)
        for i in range(K):
            step(x_offs[W + i], i)
        ev1.record(stream)
        torch.cuda.synchronize()
    launches = ctx.launch_count() - l0
    if ep_caps:  # graph replays do not pass through the library's launch counter
        l1 = ctx.launch_count()
        step.eager(x_offs[W], 0)
        torch.cuda.synchronize()
        launches = (ctx.launch_count() - l1) * K
    my_ms = ev0.elapsed_time(ev1) / K
    ms = _max_over_ranks(my_ms, world)
    _barrier(world)
    value = world * PREFILL_M / (ms / 1e3)
    rank_ms = _gather_floats(my_ms, world)

    # ---- parity of the timed step: the output of step 0's layer on fixed tokens ------------
    parity = None
    if not args.no_check:
        step(x_offs[W], 0)
        torch.cuda.synchronize()
        nb = PREFILL_M * H * 4
        got_t = arena[out_off:out_off + nb].view(torch.float32).view(PREFILL_M, H).clone()
        x_t = arena[x_offs[W]:x_offs[W] + nb].view(torch.float32).view(PREFILL_M, H).clone()
        if ep_mode:
            gx = [torch.empty_like(x_t) for _ in range(world)]
            gy = [torch.empty_like(got_t) for _ in range(world)]
            dist.all_gather(gx, x_t)
            dist.all_gather(gy, got_t)
            if rank == 0:
                # the same tokens through the single-GPU layer (all 256 experts) on rank 0
                full = host.build_synthetic_model(ctx, SEED, 1, sh, ZIPF)[2][0]
                mt = world * PREFILL_M
                xa = torch.cat(gx).cpu().numpy()
                ya = torch.cat(gy).cpu().numpy()
                xo_all, yo_all = ctx.put(xa), ctx.alloc(mt * H * 4)
                ctx.forward(full, xo_all, xo_all, yo_all, mt)
                ctx.sync()
                ref = ctx.download(yo_all, (mt, H)).astype(np.float64)
                parity = {"ep_parity": {"tokens": mt, "vs": "single-GPU moe_forward of the same tokens",
                                        "rel_l2": float(np.linalg.norm(ya - ref) / np.linalg.norm(ref)),
                                        "max_rel": float(np.abs(ya - ref).max() / np.abs(ref).max())},
                          "oracle": oracle_rows_check(sh, xa, ya)}
        else:
            parity = {"oracle": oracle_rows_check(sh, x_t.cpu().numpy(), got_t.cpu().numpy())}

    # ---- per-stage device times (profiling pass, not the timed run) -------------------------
    ctx.profile(True)
    for i in range(K):
        step.eager(x_offs[W + i], i)
    stages = ctx.profile_read()
    ctx.profile(False)
    # distinct experts whose weights this GPU streams (all ranks' tokens reach a rank's experts)
    routed = np.concatenate([ctx.do_route(pre_ids[i % PREFILL_LAYERS], x_offs[W + i], PREFILL_M,
                                          sh.top_k)[0][None] for i in range(K)])  # [K, M, k]
    if ep_mode:
        t = torch.from_numpy(routed.astype(np.int64)).cuda()
        allr = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(allr, t)
        routed = np.concatenate([a.cpu().numpy() for a in allr], axis=1)
    distinct = [len([e for e in np.unique(routed[i]) if my_experts is None or e in my_experts])
                for i in range(K)]
    n_mats = statistics.mean(distinct) + 1  # + shared expert
    hbm, tfl, peak_kind = peaks()
    stage_ms = {k: v[1] / max(v[0], 1) for k, v in stages.items()}
    # the tensor-core launches on the timed stream carry the routed experts only when the library
    # runs the shared expert as its own concurrent pass (batches of 64+ tokens, the default)
    tc_mats = n_mats - (1 if os.environ.get("MOE_B200_SHARED_SPLIT", "1") != "0" and not ep_mode else 0)
    alg_bytes = {"gemv13": n_mats * 2 * sh.w13_bytes, "gemv2": n_mats * sh.w2_bytes,
                 "tc13": tc_mats * 2 * sh.w13_bytes, "tc2": tc_mats * sh.w2_bytes,
                 "router": E * H * 4 + H * 4 + PREFILL_M * H * 4}
    dom = max(stage_ms, key=stage_ms.get)
    layer_bytes = n_mats * sh.expert_bytes
    ach = alg_bytes.get(dom, 0.0) / (stage_ms[dom] / 1e3) / 1e9 if dom in alg_bytes else None
    traffic, traffic_src = ncu_traffic(dom)
    roofline = {"bound": "hbm", "kernel": dom, "achieved": ach, "peak": hbm, "unit": "GB/s",
                "frac": ach / hbm if ach else None, "traffic": traffic, "traffic_source": traffic_src,
                "peak_kind": peak_kind,
                "alg_bytes_per_launch": alg_bytes.get(dom),
                "layer_achieved_gbs": layer_bytes / (ms / 1e3) / 1e9,
                "layer_frac": layer_bytes / (ms / 1e3) / 1e9 / hbm,
                "stage_ms": {k: round(v, 4) for k, v in stage_ms.items()}}
    if ep_mode:
        # the expert-parallel step against its two floors: this GPU's expert weights from HBM and
        # the rows crossing NVLink (the larger direction of the busiest GPU, at the measured
        # peer bandwidth)
        try:
            tr = {0: "nccl", 1: "peer"}.get(ctx.ep_transport(), "nccl") if c_ep else "torch"
            nv = max(float(ep_exchange_bytes(routed[i], world, PREFILL_M, epr, H, sh.top_k, tr,
                                             PREFILL_M).max()) for i in range(K))
            t_nv, t_hbm = nv / (NVLINK_GBS * 1e3), layer_bytes / (hbm * 1e3)
            roofline["ep_step"] = {"nvlink_bytes_max": nv, "nvlink_us": t_nv, "hbm_us": t_hbm,
                                   "target_us": max(t_nv, t_hbm), "step_us": ms * 1e3,
                                   "frac": max(t_nv, t_hbm) / (ms * 1e3), "nvlink_gbs": NVLINK_GBS,
                                   "transport": tr}
        except Exception as e:  # noqa: BLE001 - reported, never fatal to the bench
            roofline["ep_step"] = {"error": repr(e)}

    e2e, decode, cpu, config3, config2, config4, lm_head = None, None, None, None, None, None, None
    if not only_prefill:
        # ---- end to end through the public API: pinned host buffers, copies inside --------------
        hx = [torch.from_numpy(x).pin_memory() for x in xs[:4]]
        hout = torch.empty((PREFILL_M, H), dtype=torch.float32).pin_memory()
        xin = ctx.alloc(PREFILL_M * H * 4)
        nbytes = PREFILL_M * H * 4

        hout2 = [hout, torch.empty((PREFILL_M, H), dtype=torch.float32).pin_memory()]

        if ep_mode:
            # expert parallel: upload, the exchange step, blocking read-back of the result
            def e2e_step(i):
                ctx.upload_ptr(xin, hx[i % 4].data_ptr(), nbytes)
                step(xin, i)
                ctx.download_ptr(out_off, hout.data_ptr(), nbytes)
        else:
            # moe_forward_host: each step's rows go up on a copy stream, the layer runs, the result
            # comes back on another copy stream; successive steps overlap (the serving pattern)
            def e2e_step(i):
                ctx.forward_host(pre_ids[i % PREFILL_LAYERS], hx[i % 4].data_ptr(), hout2[i % 2].data_ptr(),
                                 PREFILL_M)
        # steady state of the serving pipeline: at least 100 steps (a few ms), after 5 warm-up steps
        k_e2e = max(K, 100)
        for i in range(5):
            e2e_step(i)
        ctx.sync()
        torch.cuda.synchronize()
        _barrier(world)
        t0 = time.perf_counter()
        for i in range(k_e2e):
            e2e_step(i)
        ctx.sync()
        e2e_s = _max_over_ranks((time.perf_counter() - t0) / k_e2e, world)
        e2e = {"value": world * PREFILL_M / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": nbytes,
               "d2h_bytes_per_step": nbytes, "steps": k_e2e,
               "api": "moe_arena_upload + moe_forward_ep + moe_arena_download per step" if ep_mode else
                      "moe_forward_host per step (pinned host rows in and out), one moe_sync after the timed steps"}

        # ---- config 3: 8192 tokens in total over the N GPUs (strong scaling), uniform router
        # logits and the config-1 Zipf skew ------------------------------------------------------
        config3 = {"tokens_total": CONFIG3_M, "tokens_per_gpu": c3_tokens,
                   "parallelism": f"ep{world}" if ep_mode else "single GPU"}
        for name, zipf in (("uniform", None), ("zipf1.1", ZIPF)):
            lid = host.build_synthetic_model(ctx, SEED + 3, 1, sh, zipf, experts=my_experts)[2][0]
            xc = [ctx.put(synth.tokens(SEED + 3, rank * 1000 + i, c3_tokens, H)) for i in range(4)]
            oc = ctx.alloc(c3_tokens * H * 4)
            step3 = make_step(lid, c3_tokens, oc)
            for i in range(3):
                step3(xc[i % 4])
            torch.cuda.synchronize()
            _barrier(world)
            k3 = max(5, K // 2)
            ev0.record(stream)
            for i in range(k3):
                step3(xc[i % 4])
            ev1.record(stream)
            torch.cuda.synchronize()
            my3 = ev0.elapsed_time(ev1) / k3
            ms3 = _max_over_ranks(my3, world)
            flops = CONFIG3_M * (sh.top_k + 1) * 6 * sh.inter * H
            config3[name] = {"ms_per_step": ms3, "tok_s": CONFIG3_M / (ms3 / 1e3),
                             "rank_ms": [round(v, 4) for v in _gather_floats(my3, world)],
                             "tensor_tflops_per_gpu": flops / (ms3 / 1e3) / 1e12 / world,
                             "tensor_frac": flops / (ms3 / 1e3) / 1e12 / world / tfl}

        # ---- decode (config 0): M=1, cycling through 16 layers ----------------------------------
        kd = max(K, 64)
        xd = [ctx.put(synth.tokens(SEED + 7, rank * 1000 + i, 1, H)) for i in range(kd)]
        od = ctx.alloc(H * 4)
        for i in range(2 * n_dec_layers):  # capture every layer's graph before timing
            ctx.forward(dec_ids[i % n_dec_layers], xd[i % kd], xd[i % kd], od, 1)
        torch.cuda.synchronize()
        ev0.record(stream)
        for i in range(kd):
            ctx.forward(dec_ids[i % n_dec_layers], xd[i], xd[i], od, 1)
        ev1.record(stream)
        torch.cuda.synchronize()
        eager_ms = ev0.elapsed_time(ev1) / kd  # one host call per token: bounded by the host
        # device time: the same kd single-token layers (fresh token, next layer each) captured as
        # one CUDA graph and replayed, as a decoding engine runs them
        gd = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gd, stream=stream):
            for i in range(kd):
                ctx.forward(dec_ids[i % n_dec_layers], xd[i], xd[i], od, 1)
        gd.replay()
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(3):
            gd.replay()
        ev1.record(stream)
        torch.cuda.synchronize()
        dms = ev0.elapsed_time(ev1) / (3 * kd)
        del gd
        ctx.profile(True)
        for i in range(kd):
            ctx.forward(dec_ids[i % n_dec_layers], xd[i], xd[i], od, 1)
        dstages = {k: v[1] / max(v[0], 1) for k, v in ctx.profile_read().items()}
        ctx.profile(False)
        dec_bytes = (sh.top_k + 1) * sh.expert_bytes
        decode = {"tok_s": 1e3 / dms, "us_per_token": dms * 1e3, "eager_us_per_token": eager_ms * 1e3,
                  "timing": f"CUDA graph of {kd} single-token layer launches, replayed 3 times",
                  "layer_achieved_gbs": dec_bytes / (dms / 1e3) / 1e9,
                  "layer_frac": dec_bytes / (dms / 1e3) / 1e9 / hbm,
                  "alg_bytes_per_token": dec_bytes, "stage_us": {k: round(v * 1e3, 2) for k, v in dstages.items()},
                  "l2": f"{n_dec_layers} layers ({n_dec_layers * sh.expert_bytes * (E + 1) / 1e9:.1f} GB) cycled, a fresh token per step",
                  "parallelism": "one GPU per replica" if world > 1 else "single GPU"}

        # ---- config 2: 40-layer stack, x <- x + MoE(RMSNorm(x)) per layer, one token per step,
        # 256 steps; one token step (40 x (RMSNorm + fused decode layer)) is a captured CUDA graph
        x2, xb2 = ctx.alloc(H * 4), ctx.alloc(H * 4)
        xt = [ctx.put(synth.tokens(SEED + 11, rank * 1000 + i, 1, H)) for i in range(CONFIG2_STEPS)]

        for li, lid in enumerate(dec_ids):  # layer l prefetches layer l+1's fixed weights
            ctx.layer_set_next(lid, dec_ids[(li + 1) % len(dec_ids)])

        def token_step():  # moe_forward_norm: RMSNorm + layer + residual in one launch per layer
            for li, lid in enumerate(dec_ids):
                src, dst = (x2, xb2) if li % 2 == 0 else (xb2, x2)
                ctx.forward_norm(lid, src, dst, 1, 1e-6)
        arena[x2:x2 + H * 4].copy_(arena[xt[0]:xt[0] + H * 4])
        token_step()  # eager first step (workspace)
        torch.cuda.synchronize()
        g2 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g2, stream=stream):
            token_step()
        torch.cuda.synchronize()
        ev0.record(stream)
        for i in range(CONFIG2_STEPS):
            arena[x2:x2 + H * 4].copy_(arena[xt[i]:xt[i] + H * 4])
            g2.replay()
        ev1.record(stream)
        torch.cuda.synchronize()
        us2 = ev0.elapsed_time(ev1) / CONFIG2_STEPS * 1e3
        step_bytes = n_dec_layers * dec_bytes
        config2 = {"layers": n_dec_layers, "steps": CONFIG2_STEPS, "tok_s": 1e6 / us2, "us_per_token": us2,
                   "hbm_gbs": step_bytes / (us2 / 1e6) / 1e9, "hbm_frac": step_bytes / (us2 / 1e6) / 1e9 / hbm,
                   "expert_bytes_resident_gb": n_dec_layers * sh.expert_bytes * (E + 1) / 1e9,
                   "step": "CUDA graph of 40 fused (RMSNorm + decode layer + residual) launches; fresh token copied in per step"}
        del g2

        # ---- config 4: batched decode, 64 independent tokens, both expert kernels ----------------
        m4 = CONFIG4_M
        x4 = [ctx.put(synth.tokens(SEED + 13, rank * 1000 + i, m4, H)) for i in range(4)]
        o4 = ctx.alloc(m4 * H * 4)
        lid4 = dec_ids[0]
        routed4 = ctx.do_route(lid4, x4[0], m4, sh.top_k)[0]
        d4 = len(np.unique(routed4)) + 1
        ctx.set_path(0)  # what the library picks by itself at M=64: read from its stage names
        ctx.profile(True)
        ctx.forward(lid4, x4[0], x4[0], o4, m4)
        auto_st = ctx.profile_read()
        ctx.profile(False)
        auto = "tcgen05" if "tc13" in auto_st else "gemv" if "gemv13" in auto_st else "?"
        config4 = {"tokens": m4, "distinct_experts_plus_shared": d4,
                   "auto_choice": auto, "auto_stages": sorted(auto_st)}
        for name, path in (("gemv", 1), ("tcgen05", 3)):
            ctx.set_path(path)
            for i in range(3):
                ctx.forward(lid4, x4[i % 4], x4[i % 4], o4, m4)
            torch.cuda.synchronize()
            k4 = 20
            ev0.record(stream)
            for i in range(k4):
                ctx.forward(lid4, x4[i % 4], x4[i % 4], o4, m4)
            ev1.record(stream)
            torch.cuda.synchronize()
            ms4 = ev0.elapsed_time(ev1) / k4
            b4 = d4 * sh.expert_bytes
            config4[name] = {"ms_per_step": ms4, "tok_s": m4 / (ms4 / 1e3), "hbm_gbs": b4 / (ms4 / 1e3) / 1e9,
                             "hbm_frac": b4 / (ms4 / 1e3) / 1e9 / hbm}
        ctx.set_path(args.path)

        lm_head = lm_head_leg(ctx, synth, stream, hbm, rank)

        # ---- CPU baseline (rank 0, N=1 only) ------------------------------------------------------
        if rank == 0 and world == 1 and not args.no_cpu:
            ncpu = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
            _, v, dt, n = cpu_baseline(sh, xs[0], threads=ncpu)
            cpu = {"value": v, "unit": "tok/s", "cores": ncpu, "kind": "port",
                   "sample": f"{n} tokens = repeated config-1 512-token prefills ({dt:.1f} s), C "
                             "restatement of the reference MoE layer (oracle/, f32, OpenMP all cores)"}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": K,
                "warmup": W, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32" if args.path == 1 else "f16 (f32 accumulate)",
                "data": "synthetic (seeded IQ4_XS weights generated on device, N(0,1) tokens)",
                "config": {"workload": WORKLOAD,
                           "tokens_per_step": PREFILL_M * world,
                           "parallelism": (f"ep{world}: {epr} experts per GPU, " + {
                               "peer": "dispatch stores / combine loads over NVLink peer memory (moe_forward_ep)",
                               "nccl": "NCCL all-to-all inside moe_forward_ep",
                               "torch": "torch.distributed all-to-all (ep.py)"}[args.ep]) if ep_mode else "single GPU",
                           "expert_kernels": {0: "auto (tcgen05, A in TMEM)", 1: "CUDA-core GEMV",
                                              2: "tcgen05, A in smem", 3: "tcgen05, A in TMEM"}[args.path],
                           "distinct_experts_per_gpu": round(statistics.mean(distinct), 1),
                           "ep_step": ep_graphs[0] if ep_graphs else None,
                           "l2": (f"{PREFILL_LAYERS} independently seeded layers cycled step by step "
                                  f"(~{n_mats * sh.expert_bytes / 1e6:.0f} MB of touched weights per step, "
                                  f"{PREFILL_LAYERS * n_mats * sh.expert_bytes / 1e6:.0f} MB per cycle vs the "
                                  "126 MB L2); fresh tokens per step; no L2 flush"),
                           "rank_ms": [round(v, 4) for v in rank_ms]},
                "parity": parity, "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches,
                "clocks": clk.summary(), "decode": decode, "config2": config2, "config3": config3,
                "config4": config4, "lm_head": lm_head}
        print(json.dumps(line), flush=True)
    torch.cuda.synchronize()
    ep_caps.clear()  # captured NCCL work must be released before the process group
    _barrier(world)
    ctx.close()
    del arena
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
