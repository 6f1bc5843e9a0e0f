"""Benchmark: block-sparse attention TFLOP/s (executed FLOPs) on 1..8 B200.

Default workload (the one the metric is quoted on at
1/2/4/8 GPUs): a head-sharded full-stack step — 30 attention layers of the
Matrix-Game shape (24 heads, head_dim 128, 30x52 latent, 4-frame query chunk,
64-frame memory, 3D blocks (4,4,8), keep 25%, cosine selection), QKV/O
projections of hidden 3072 (random-init bf16), Ulysses all-to-all before and
after each attention when N > 1 (NVLink peer pushes by default, checked bit for
bit against NCCL before timing; ``--exchange nccl`` for NCCL itself). ``--workload mg_layer`` runs
BASELINE config 3 instead (single MG-shaped layer with the pruned-memory gather).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference] [--workload W]

One JSON line on rank 0. ``value`` = executed sparse-attention FLOPs of every
layer on every rank / device time of the K timed steps (max over ranks).
``e2e`` = the same metric with each step's input hidden states copied from
pinned host memory and its output copied back inside the timed region.
``--impl reference`` times the reference's CPU path (the oracle port: its
block-mask logic + dense masked torch attention) on the host cores.
"""

from __future__ import annotations

import argparse
import dataclasses
import json
import math
import os
import re
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "sparse-attn fwd ms/call & TFLOP/s (executed FLOPs) at 1/2/4/8 B200 vs roofline"
UNIT = "TFLOP/s"


def _peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("bf16_tflops"), d.get("bf16_tflops_sustained"), "measured"
    return 1590.0, 1400.0, "fallback"


def _hbm_peak():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    return json.load(open(p)).get("hbm_gbs", 6650.0) if os.path.exists(p) else 6650.0


def _profile_traffic(kernel_tag):
    """Per-launch DRAM bytes of the attention kernel from the committed ncu summary
    (a line ``traffic_bytes_per_launch: <int>`` in profiles/<kernel_tag>*.md)."""
    import glob
    for path in sorted(glob.glob(os.path.join(REPO, "profiles", kernel_tag + "*.md"))):
        m = re.search(r"traffic_bytes_per_launch:\s*([0-9]+)", open(path).read())
        if m:
            return int(m.group(1)), os.path.basename(path)
    return None, None


class ClockSampler:
    """Samples SM clocks and clock-event (throttle) reasons while the timed region
    runs: NVML reads every 20 ms (read-only queries), else nvidia-smi at 100 ms."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, local_rank):
        self.local_rank = local_rank
        self.proc = None
        self.stop = threading.Event()
        self.samples = []      # (sm_mhz, max_mhz, set of reason names)
        self.nvml = None

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        try:
            uuid = str(torch.cuda.get_device_properties(self.local_rank).uuid)
            return pynvml, pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.local_rank)

    def _poll_nvml(self):
        nv, h = self.nvml
        mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        while not self.stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                active = {name for name, const in self.REASONS if bits & getattr(nv, const)}
                self.samples.append((float(sm), float(mx), active))
            except Exception:
                pass
            self.stop.wait(0.02)

    def __enter__(self):
        try:
            self.nvml = self._nvml_handle()
            self.t = threading.Thread(target=self._poll_nvml, daemon=True)
            self.t.start()
            return self
        except Exception:
            self.nvml = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.local_rank}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read_smi, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read_smi(self):
        names = [n for n, _ in self.REASONS]
        for ln in self.proc.stdout:
            parts = [x.strip() for x in ln.strip().split(",")]
            if len(parts) < 9:
                continue
            try:
                self.samples.append((float(parts[1]), float(parts[2]),
                                     {n for n, v in zip(names, parts[5:9]) if v.lower().startswith("active")}))
            except ValueError:
                continue

    def __exit__(self, *exc):
        self.stop.set()
        if self.nvml is not None:
            self.t.join(timeout=2)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        mx = self.samples[-1][1]
        sm = [x[0] for x in self.samples]
        loaded = [x for x in sm if x > 0.5 * (mx or max(sm))] or sm
        reasons = set().union(*(x[2] for x in self.samples))
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvml" if self.nvml is not None else "nvidia-smi"}


# ---------------------------------------------------------------------------
# CPU reference path (oracle port) — cpu_baseline and --impl reference
# ---------------------------------------------------------------------------
def cpu_reference_sample(cfg, heads=1, seed=3):
    """One bounded sample of the workload on the host: pooled-score selection
    (reference rules) + dense masked torch attention for ``heads`` heads of one
    layer. Returns (seconds, executed sparse FLOPs of the sample, threads)."""
    from oracle import li_oracle as O
    threads = torch.get_num_threads()
    LH, LW = cfg.latent_hw
    tile = cfg.tile
    bs = tile[0] * tile[1] * tile[2]
    g = torch.Generator().manual_seed(seed)
    D = cfg.head_dim
    q = torch.randn(1, heads, cfg.q_tokens, D, generator=g).to(torch.bfloat16).float().numpy()
    k = torch.randn(1, heads, cfg.kv_frames * cfg.frame_tokens, D, generator=g).to(torch.bfloat16).float().numpy()
    v = torch.randn(1, heads, cfg.kv_frames * cfg.frame_tokens, D, generator=g).to(torch.bfloat16).float().numpy()
    t0 = time.perf_counter()
    qt, qp = O.tile_pool(q, cfg.query_frames, LH, LW, tile, "bf16")
    kt, kp = O.tile_pool(k, cfg.kv_frames, LH, LW, tile, "bf16")
    vt = O.tile_raster(v, cfg.kv_frames, LH, LW, tile)
    gk = O.grid_dims(cfg.kv_frames, LH, LW, tile)
    nq, nk = cfg.blocks()
    idx, cnt = O.generate_prefill_indices(qp, kp, 0, gk, dict(tile_size=tile, topk_ratio=cfg.keep_ratio,
                                                              sim_metric=cfg.metric), "bf16", q_offset=nk - nq)
    qtt, ktt, vtt = (torch.from_numpy(np.ascontiguousarray(a)) for a in (qt, kt, vt))
    kflat = ktt.reshape(1, heads, nk * bs, D)
    vflat = vtt.reshape(1, heads, nk * bs, D)
    for h in range(heads):
        for i in range(nq):
            mask = torch.zeros(nk, dtype=torch.bool)
            mask[torch.from_numpy(idx[0, h, i, :cnt[0, h, i]].astype(np.int64))] = True
            m = mask.repeat_interleave(bs)[None, :].expand(bs, -1)
            torch.nn.functional.scaled_dot_product_attention(qtt[0, h, i][None], kflat[0, h][None],
                                                             vflat[0, h][None], attn_mask=m[None])
    dt = time.perf_counter() - t0
    return dt, cfg.attention_flops(heads), threads


def run_reference(args, cfg, rank, world):
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    for _ in range(max(0, args.warmup_ref)):
        cpu_reference_sample(cfg)
    times, flops = [], 0.0
    for s in range(args.steps):
        dt, fl, threads = cpu_reference_sample(cfg, seed=10 + s)
        times.append(dt)
        flops += fl
    value = flops / sum(times) / 1e12
    sample = (f"1 head of 1 layer per step ({cfg.query_frames}-frame query chunk vs {cfg.kv_frames}-frame K/V, "
              f"{cfg.blocks()[0]} query blocks x {cfg.budget()} selected blocks): block-mask logic + dense masked "
              f"SDPA in fp32 on bf16-valued inputs")
    line = {"metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * sum(times) / len(times),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": dict(workload_config(cfg, args, world), exchange=None, cuda_graph=False),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def workload_config(cfg, args, world):
    nq, nk = cfg.blocks()
    name = "config5_head_sharded_stack" if cfg.heads == 24 and cfg.layers == 30 else \
        f"stack_{cfg.layers}layers_{cfg.heads}heads"
    return {"workload": name if args.workload == "stack" else "config3_mg_layer",
            "layers": cfg.layers, "heads": cfg.heads, "head_dim": cfg.head_dim, "hidden": cfg.hidden,
            "latent_hw": list(cfg.latent_hw), "query_frames": cfg.query_frames,
            "memory_frames": cfg.memory_frames, "tile": list(cfg.tile), "keep_ratio": cfg.keep_ratio,
            "sim_metric": cfg.metric, "q_blocks": nq, "k_blocks": nk, "selected_blocks": cfg.budget(),
            "attn_tflop_per_call": cfg.attention_flops() / 1e12,
            "parallelism": f"ulysses_heads{world}", "l2": "inputs larger than L2 (resident K/V >> 126 MB)",
            "exchange": cfg.exchange if world > 1 else None,
            "cuda_graph": bool(getattr(args, "graph", False)) and args.workload == "stack"}


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def exchange_check(stack, x, group):
    """Layer 0's two exchanges through the NVLink peer path (li_a2a_push: q into the
    receive buffer, k and v into the owners' resident K/V buffers; the output rows)
    and through NCCL all_to_all_single on the same inputs; True when every rank's
    results agree bit for bit (one collective vote)."""
    from light_interaction_project_b200.ulysses import head_to_seq
    cfg, world, rank, hl = stack.cfg, stack.world, stack.rank, stack.hl
    B, s, _ = x.shape
    D, S = cfg.head_dim, s * world
    q = stack.qkv_exchange(0, x)                                                   # peer path
    got_q = q.permute(0, 2, 1, 3).reshape(S, hl * D).clone()
    got_kv = stack.kv_buf[0][stack.kv_buf[0].shape[0] - S:].reshape(S, 2 * hl * D).clone()
    send = torch.matmul(x.reshape(B * s, cfg.hidden), stack.w_qkv_rank[0])          # [P, s, 3*hl*D]
    want = torch.empty_like(send)
    dist.all_to_all_single(want, send, group=group)
    want = want.view(S, 3 * hl * D)
    ok = torch.equal(got_q, want[:, : hl * D]) and torch.equal(got_kv, want[:, hl * D:])
    g = torch.Generator(device=x.device)
    g.manual_seed(99 + rank)
    o_tok = torch.randn(B, S, hl, D, generator=g, device=x.device).to(torch.bfloat16)
    row = hl * D * o_tok.element_size()
    got = stack.ex_out.push(o_tok, s, row, s * row, row, rank * row, cfg.heads * row // hl)
    got = got[: s * cfg.heads * D].view(B, s, cfg.heads, D).clone()
    ok = ok and torch.equal(got, head_to_seq(o_tok.permute(0, 2, 1, 3), world, group))
    vote = torch.tensor([1 if ok else 0], device=x.device, dtype=torch.int32)
    dist.all_reduce(vote, op=dist.ReduceOp.MIN, group=group)
    torch.cuda.synchronize()
    return bool(vote.item())


def run_gpu(args, cfg, rank, world, local_rank):
    from light_interaction_project_b200 import _lib as L
    from light_interaction_project_b200 import kernels as K
    from light_interaction_project_b200.ulysses import HeadShardedStack

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    L.load()
    # The attention kernel's own duration: events on the launching stream (torch's
    # current stream, which the library is handed) around each attention call.
    attn_timing = {"on": False, "events": []}
    attn_call = K.sparse_attn_raster

    def timed_attn(*a, **kw):
        if not attn_timing["on"]:
            return attn_call(*a, **kw)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        out = attn_call(*a, **kw)
        e.record()
        attn_timing["events"].append((s, e))
        return out
    K.sparse_attn_raster = timed_attn
    group = dist.group.WORLD if world > 1 else None
    stack = HeadShardedStack(cfg, rank, world, dev, group=group)
    x0 = stack.make_input()
    # N > 1 with the peer exchange: check it bit for bit against NCCL on this box
    # before anything is timed; on a mismatch every rank falls back to NCCL. The
    # stack is rebuilt for that, since its resident K/V buffers are the IPC-shared
    # ones the closed exchange owned.
    exch = None
    if world > 1:
        exch = {"transport": cfg.exchange, "check": None}
        if stack.ex_qkv is not None:
            ok = exchange_check(stack, x0, group)
            exch["check"] = ok
            if not ok:
                torch.cuda.synchronize()
                dist.barrier()
                stack.close()
                del x0
                stack = HeadShardedStack(dataclasses.replace(cfg, exchange="nccl"), rank, world, dev, group=group)
                x0 = stack.make_input()
                exch["transport"] = "nccl (peer exchange failed its check)"

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # Warm-up.
    for _ in range(args.warmup):
        stack.step(x0)
    barrier()
    K.raise_device_errors(dev)
    # With --graph (the default) the whole 30-layer step is one CUDA graph: x0 is
    # its static input, refilled in place for the end-to-end leg. Every kernel and
    # exchange of every layer still runs on each replay.
    if args.graph:
        stack.capture(x0)
        per_step_launches = stack.graph_launches
        barrier()
        run_step = lambda: stack.replay()  # noqa: E731
    else:
        run_step = lambda: stack.step(x0)  # noqa: E731
    run_step()
    barrier()

    # Device-resident timing.
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    launches0 = L.kernel_launches()
    with ClockSampler(local_rank) as clk:
        start.record()
        for s in range(args.steps):
            attn_timing["on"] = not args.graph and s == args.steps - 1
            run_step()
        end.record()
        barrier()
    attn_timing["on"] = False
    n_launch = per_step_launches * args.steps if args.graph else L.kernel_launches() - launches0
    ms = start.elapsed_time(end)
    # One eager step after the timed region (same kernels, same inputs) gives the
    # per-layer phase breakdown of this rank and, with --graph, the attention
    # kernel's events.
    marks = []
    attn_timing["on"] = args.graph
    stack.step(x0, marks=marks)
    attn_timing["on"] = False
    barrier()
    attn_ms = [a.elapsed_time(b) for a, b in attn_timing["events"]]
    breakdown = {}
    prev = None
    for name, ev in marks:
        if name != "start":
            breakdown[name] = breakdown.get(name, 0.0) + prev.elapsed_time(ev) / cfg.layers
        prev = ev
    if attn_ms:
        a_ms = sum(attn_ms) / len(attn_ms)
        breakdown["selection"] = breakdown.pop("selection_and_attention") - a_ms
        breakdown["attention_kernel_and_combine"] = a_ms
    breakdown = {k: round(v, 4) for k, v in breakdown.items()}
    # End-to-end: host input -> device, step, device output -> host, all on the
    # step's stream; the copies also get their own events.
    x_host = x0.cpu().pin_memory()
    y_host = torch.empty_like(x_host).pin_memory()
    barrier()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    copy_ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    s2.record()
    for i in range(args.steps):
        ev = copy_ev[i]
        ev[0].record()
        if args.graph:
            x0.copy_(x_host, non_blocking=True)
            ev[1].record()
            y = stack.replay()
        else:
            xd = x_host.to(dev, non_blocking=True)
            ev[1].record()
            y = stack.step(xd)
        ev[2].record()
        y_host.copy_(y, non_blocking=True)
        ev[3].record()
    e2.record()
    barrier()
    ms_e2e = s2.elapsed_time(e2)
    h2d_ms = sum(ev[0].elapsed_time(ev[1]) for ev in copy_ev) / args.steps
    d2h_ms = sum(ev[2].elapsed_time(ev[3]) for ev in copy_ev) / args.steps
    K.raise_device_errors(dev)

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    stack.close()
    # The host-side reference sample (rank 0, N=1 only, on every host core) runs
    # before the last collective, so every rank leaves the process group together.
    cpu = None
    if rank == 0 and world == 1:
        prev = torch.get_num_threads()
        torch.set_num_threads(os.cpu_count() or 1)
        cpu = cpu_reference_sample(cfg)
        torch.set_num_threads(prev)
    t = torch.tensor([ms, ms_e2e, sum(attn_ms) / len(attn_ms), h2d_ms, d2h_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, ms_e2e, attn_call_ms, h2d_ms, d2h_ms = t.tolist()
    if rank != 0:
        return
    total_flops = cfg.attention_flops() * cfg.layers * args.steps
    value = total_flops / (ms * 1e-3) / 1e12
    e2e_value = total_flops / (ms_e2e * 1e-3) / 1e12
    burst, sustained, kind = _peaks()
    per_launch_flops = cfg.attention_flops(cfg.heads // world)
    achieved = per_launch_flops / (attn_call_ms * 1e-3) / 1e12
    traffic, tfile = _profile_traffic("attn_fwd_config5")
    if traffic is not None and world != 1:
        traffic = traffic // world
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "attn_kernel_ms": attn_call_ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) hidden states, random-init bf16 weights, random resident K/V memory)",
        "config": workload_config(cfg, args, world),
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": sustained, "unit": "TFLOP/s",
                     "frac": achieved / sustained, "traffic": traffic,
                     "peak_kind": f"{kind} bf16 sustained (burst {burst})",
                     "traffic_source": tfile},
        "e2e": {"value": e2e_value, "unit": UNIT, "ms_per_step": ms_e2e / args.steps,
                "h2d_bytes_per_step": int(x_host.numel() * x_host.element_size() * world),
                "d2h_bytes_per_step": int(y_host.numel() * y_host.element_size() * world),
                "h2d_ms_per_step": h2d_ms, "d2h_ms_per_step": d2h_ms},
        "gpu_launches": int(n_launch * world),
        "clocks": clk.summary(),
        # Rank 0's mean ms per layer by phase, from one eager step (exchanges include
        # waiting for the other ranks).
        "layer_breakdown_ms": breakdown,
    }
    if exch is not None:
        line["exchange_check"] = exch["check"]
        line["config"]["exchange"] = exch["transport"]
    if cpu is not None:
        cpu_s, cpu_fl, threads = cpu
        line["cpu_baseline"] = {"value": cpu_fl / cpu_s / 1e12, "unit": UNIT, "cores": threads, "kind": "port",
                                "sample": "1 head of 1 layer: block-mask logic + dense masked SDPA (fp32) on the host"}
    print(json.dumps(line), flush=True)


def run_gpu_layer(args, rank, world, local_rank):
    """one Matrix-Game-shaped layer. K/V of 16 retained frames
    (drawn without replacement from a 64-frame seeded pool) are gathered behind
    the resident current chunk, then pooling, selection (query-chunk rows of the
    bidirectional selection) and the sparse attention run through the public
    ``run_sparse_attention``. Heads are split across ranks (no collective)."""
    from light_interaction_project_b200 import bi_sparse_operation as mg
    from light_interaction_project_b200 import kernels as K
    from light_interaction_project_b200.ulysses import StackConfig

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    cfg = StackConfig(layers=1, memory_frames=16, keep_ratio=0.30)
    H = cfg.heads // world
    LH, LW = cfg.latent_hw
    HW = LH * LW
    g = torch.Generator(device=dev).manual_seed(1 + rank)
    pool_frames = 64
    k_pool = torch.randn(1, H, pool_frames * HW, 128, generator=g, device=dev).to(torch.bfloat16)
    v_pool = torch.randn(1, H, pool_frames * HW, 128, generator=g, device=dev).to(torch.bfloat16)
    rng = np.random.default_rng(1234)
    ids = torch.from_numpy(rng.choice(pool_frames, 16, replace=False).astype(np.int32)).to(dev)
    kv_tokens = cfg.kv_frames * HW
    k_buf = torch.randn(1, H, kv_tokens, 128, generator=g, device=dev).to(torch.bfloat16)
    v_buf = torch.randn(1, H, kv_tokens, 128, generator=g, device=dev).to(torch.bfloat16)
    q = torch.randn(1, H, cfg.q_tokens, 128, generator=g, device=dev).to(torch.bfloat16)
    nq, nk = cfg.blocks()
    params = {"tile_size": cfg.tile, "topk_ratio": cfg.keep_ratio, "sim_metric": cfg.metric}

    def step():
        K.gather_frames(k_pool, ids, HW, out=k_buf[:, :, :16 * HW])
        K.gather_frames(v_pool, ids, HW, out=v_buf[:, :, :16 * HW])
        return mg.run_sparse_attention(q, k_buf, v_buf, 0, 0, cfg.latent_hw, params, q_block_offset=nk - nq)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        s.record()
        for _ in range(args.steps):
            step()
        e.record()
        torch.cuda.synchronize()
    ms = s.elapsed_time(e) / args.steps
    # The retained-frame gather alone (K and V: 16 frames x 24 heads each), against
    # the HBM copy peak: algorithmic bytes = read + write of the gathered rows.
    s.record()
    for _ in range(args.steps):
        K.gather_frames(k_pool, ids, HW, out=k_buf[:, :, :16 * HW])
        K.gather_frames(v_pool, ids, HW, out=v_buf[:, :, :16 * HW])
    e.record()
    torch.cuda.synchronize()
    gather_ms = s.elapsed_time(e) / args.steps
    gather_bytes = 2 * 2 * 16 * HW * H * 128 * 2      # (K, V) x (read, write)
    # Attention kernel alone.
    qp = K.pool_blocks(q, cfg.query_frames, LH, LW, cfg.tile)
    kp = K.pool_blocks(k_buf, cfg.kv_frames, LH, LW, cfg.tile)
    gq = K.grid_blocks(cfg.query_frames, LH, LW, cfg.tile)
    gk = K.grid_blocks(cfg.kv_frames, LH, LW, cfg.tile)
    from light_interaction_project_b200 import _lib as L
    p = K.select_params(L.SELECT_BIDIR, cfg.metric, cfg.tile, gk, gk, 0, 0, cfg.keep_ratio, 7, nk - nq)
    idx, cnt = K.select_blocks(qp, kp, p)
    gq3, gk3 = L.grid3d(cfg.query_frames, LH, LW, cfg.tile), L.grid3d(cfg.kv_frames, LH, LW, cfg.tile)
    for _ in range(3):
        K.sparse_attn_raster(q, gq3, None, None, k_buf, v_buf, gk3, idx, cnt)
    s.record()
    for _ in range(args.steps):
        K.sparse_attn_raster(q, gq3, None, None, k_buf, v_buf, gk3, idx, cnt)
    e.record()
    torch.cuda.synchronize()
    attn_ms = s.elapsed_time(e) / args.steps
    K.raise_device_errors(dev)
    if rank == 0:
        fl = cfg.attention_flops(H)
        burst, sustained, kind = _peaks()
        print(json.dumps({"metric": METRIC, "workload": "config3_mg_layer", "n_gpus": world,
                          "value": fl * world / (ms * 1e-3) / 1e12, "unit": UNIT, "ms_per_call": ms,
                          "attn_kernel_ms": attn_ms, "attn_kernel_tflops": fl / (attn_ms * 1e-3) / 1e12,
                          "frac_of_burst": fl / (attn_ms * 1e-3) / 1e12 / burst, "peak_kind": kind,
                          "gather_ms": gather_ms, "gather_bytes": gather_bytes,
                          "gather_gbs": gather_bytes / (gather_ms * 1e-3) / 1e9,
                          "gather_frac_of_hbm": gather_bytes / (gather_ms * 1e-3) / 1e9 / _hbm_peak(),
                          "q_blocks": nq, "k_blocks": nk, "selected": cfg.budget(), "clocks": clk.summary()}),
              flush=True)


def run_configs(args):
    """``--workload configs``: BASELINE configs 1-4 through the public operators on
    one GPU (ms/call, executed TFLOP/s) beside the oracle's CPU path on a one-head
    sample scaled to all heads. One JSON line per case. Synthetic seeded inputs
    (no RoPE; the timing does not depend on the values).

    The last case is the HY prefill / KV-recompute call at full context: q, k
    and v cover the same 16 frames, B = 2 (the plain and ProPE streams), 256 text
    tokens, and q handed over as ``query.transpose(1, 2)`` of a [B, S, H, D]
    tensor, as the patched HY attention does."""
    from light_interaction_project_b200 import bi_sparse_operation_for_KV_cache as hyp
    from oracle import li_oracle as O
    from light_interaction_project_b200 import ar_sparse_operation as ar
    from light_interaction_project_b200 import bi_sparse_operation as mg
    from light_interaction_project_b200 import kernels as K
    from light_interaction_project_b200.pipeline import sparse_forward
    from light_interaction_project_b200 import _lib as L
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    L.load()
    burst, _, kind = _peaks()
    torch.set_num_threads(os.cpu_count() or 1)
    hy = lambda tile, ratio, rp: dict(tile_size=tile, topk_ratio=ratio, recent_protect=rp,  # noqa: E731
                                      sim_metric="scaled_dot_product")
    cases = [("config1_toy", "hy", torch.float32, 4, 64, 8, 8, 2, 6, hy((2, 4, 8), 0.5, 2), False),
             ("config2_hy", "hy", torch.bfloat16, 16, 128, 30, 52, 4, 16, hy((1, 8, 16), 0.25, 4), False),
             ("config3_mg", "mg", torch.bfloat16, 24, 128, 30, 52, 4, 20,
              dict(tile_size=(4, 4, 8), topk_ratio=0.30, sim_metric="cosine"), False)]
    for mem in (8, 16, 32, 64):
        for keep in (0.10, 0.25, 0.50, 1.00):
            cases.append((f"config4_mem{mem}_keep{int(keep * 100)}", "hy", torch.bfloat16, 16, 128, 30, 52, 4, mem,
                          hy((1, 8, 16), keep, 4), True))
    cases.append(("f2_hy_prefill_b2_full_context", "hy_prefill", torch.bfloat16, 16, 128, 30, 52, 16, 16,
                  dict(tile_size=(4, 8, 4), topk_ratio=0.3, sim_metric="scaled_dot_product"), False))
    if args.cases:
        cases = [c for c in cases if re.search(args.cases, c[0])]
    for name, mode, dt, H, D, LH, LW, Fq, Fk, params, bias in cases:
        HW = LH * LW
        B, ntok_txt = (2, 256) if mode == "hy_prefill" else (1, 0)
        g = torch.Generator(device=dev).manual_seed(5)
        if mode == "hy_prefill":
            q = torch.randn(B, Fq * HW, H, D, generator=g, device=dev).to(dt).transpose(1, 2)
        else:
            q = torch.randn(B, H, Fq * HW, D, generator=g, device=dev).to(dt)
        k = torch.randn(B, H, Fk * HW, D, generator=g, device=dev).to(dt)
        v = torch.randn(B, H, Fk * HW, D, generator=g, device=dev).to(dt)
        kt = torch.randn(B, H, ntok_txt, D, generator=g, device=dev).to(dt)
        vt = torch.randn(B, H, ntok_txt, D, generator=g, device=dev).to(dt)
        tile = params["tile_size"]
        gq, gk = K.grid_blocks(Fq, LH, LW, tile), K.grid_blocks(Fk, LH, LW, tile)
        nq, nk = int(np.prod(gq)), int(np.prod(gk))
        bs = tile[0] * tile[1] * tile[2]
        empty = q[:, :, :0]
        sb = None
        if bias:
            rng = np.random.default_rng(7 + Fk)
            sb = torch.from_numpy((0.01 * rng.lognormal(0.0, 1.0, size=(1, 1, 1, nk))).astype(np.float32)).to(dev)
        smode = L.SELECT_DECODE if mode == "hy" else L.SELECT_BIDIR
        sp = K.select_params(smode, params["sim_metric"], tile, gq if mode == "hy" else gk, gk, ntok_txt,
                             params.get("recent_protect", 0), params["topk_ratio"], 7, nk - nq if mode == "mg" else 0)
        ntxt_blk, sel = K.select_budget(sp, nq, nk)   # the library's own budget rule
        sel += ntxt_blk
        if mode == "hy_prefill":
            def call():
                hyp.get_infer_state().current_chunk_index = 3
                return hyp.run_sparse_prefill_attention(q, kt, vt, k, v, 0, (LH, LW), params)
        elif mode == "mg":
            call = lambda: mg.run_sparse_attention(q, k, v, 0, 0, (LH, LW), params, q_block_offset=nk - nq)  # noqa
        elif bias:
            call = lambda: sparse_forward(q, empty, empty, k, v, (LH, LW), params, L.SELECT_DECODE, tile,  # noqa
                                          score_bias=sb)
        else:
            call = lambda: ar.run_sparse_attention(q, empty, empty, k, v, 0, (LH, LW), params)  # noqa
        for _ in range(3):
            call()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(10):
            call()
        b.record()
        torch.cuda.synchronize()
        K.raise_device_errors(dev)
        ms = a.elapsed_time(b) / 10
        fl = 4.0 * B * H * nq * bs * sel * bs * D
        # CPU: the oracle's path (selection + dense masked SDPA) on batch 0, head 0,
        # scaled to B * H heads.
        qn, kn, vn, ktn, vtn = (x[:1, :1].float().cpu().numpy() for x in (q, k, v, kt, vt))
        odt = "fp32" if dt == torch.float32 else "bf16"
        t0 = time.perf_counter()
        if mode == "mg":
            O.run_sparse_attention_mg(qn, kn, vn, 0, (LH, LW), params, odt, q_offset=nk - nq)
        elif mode == "hy_prefill":
            O.run_sparse_prefill_attention_hy(qn, ktn, vtn, kn, vn, (LH, LW), params, odt)
        else:
            O.run_sparse_attention_hy(qn, ktn, vtn, kn, vn, (LH, LW), params, odt)
        cpu_ms = (time.perf_counter() - t0) * 1e3 * B * H
        print(json.dumps({"workload": "configs", "case": name, "gpu_ms_per_call": round(ms, 4),
                          "executed_tflop": fl / 1e12, "tflops": round(fl / (ms * 1e-3) / 1e12, 1),
                          "frac_of_burst": round(fl / (ms * 1e-3) / 1e12 / burst, 3), "peak_kind": kind,
                          "selected_per_q_block": sel, "q_blocks": nq, "k_blocks": nk, "heads": H, "batch": B,
                          "text_tokens": ntok_txt,
                          "cpu_ms_per_call": round(cpu_ms, 1), "cpu_sample": "batch 0 head 0, scaled to B*H",
                          "cpu_threads": torch.get_num_threads(), "cpu_count": os.cpu_count(),
                          "score_bias": "lognormal(0,1)*0.01 per key block" if bias else None}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="stack", choices=["stack", "mg_layer", "configs"])
    ap.add_argument("--layers", type=int, default=30)
    ap.add_argument("--heads", type=int, default=24,
                    help="attention heads of the stack (24 = config 5; 3 on one GPU is the per-rank shape at N = 8)")
    ap.add_argument("--warmup-ref", type=int, default=0)
    ap.add_argument("--cases", default="", help="--workload configs: regex selecting case names")
    ap.add_argument("--graph", action=argparse.BooleanOptionalAction, default=True,
                    help="stack: run each step as one captured CUDA graph (--no-graph: eager launches)")
    ap.add_argument("--exchange", default="peer", choices=["peer", "nccl"],
                    help="stack, N > 1: all-to-all over NVLink peer memory (li_a2a_push) or NCCL")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    from light_interaction_project_b200.ulysses import StackConfig
    cfg = StackConfig(layers=args.layers, heads=args.heads, exchange=args.exchange)
    if args.impl == "reference":
        run_reference(args, cfg, rank, world)
        return
    if args.workload == "mg_layer":
        run_gpu_layer(args, rank, world, local_rank)
        return
    if args.workload == "configs":
        if rank == 0:
            run_configs(args)
        return
    if world > 1:
        import datetime
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_gpu(args, cfg, rank, world, local_rank)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
