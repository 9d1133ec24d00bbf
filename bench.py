#!/usr/bin/env python
"""Benchmark of the routed block-sparse attention layer.

One step = one pass of the hot path over one CFG batch of the Wan2.1-14B 720p
self-attention layer: Morton pack of Q/K/V (1x16 microtiles), block-sparse
attention over the per-(branch, head, query-block) CSR routes whose output
store writes each row back to its raster token (the unpack folded into the
epilogue).  57,600 tokens, CFG batch 2, 40 heads, head_dim 128, bf16, routes from
the seeded Gaussian-blob procedure (top-mass 0.95, keep cap 0.625, 29 sink
blocks).  Inputs (3 x 1.18 GB) are larger than L2, so no flush is needed.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl bsa|reference]

N > 1 runs under torchrun: CFG branches on two rank groups, heads split inside
a group with a sequence<->head all-to-all (NCCL); value is the whole-job rate
at fixed total work ("strong").  ``--impl reference`` times the reference's CPU
algorithm (the oracle port) on rank 0 with all host cores.
Prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

REPO = Path(__file__).resolve().parent
METRIC = "Wan-14B 57.6k-token sparse attn layer ms & eff. TFLOPS; 5-step forward sec"
UNIT = "TFLOPS"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# dram__bytes_read.sum + dram__bytes_write.sum of one attention launch per
# (branch, head) it processes: ncu capture of the 4-head config-4 case (2 branches,
# 387.8 MB read + 105.8 MB written) divided by 8; traffic grows with the heads
# processed, so a launch's traffic is this times its branches x heads.
ATTENTION_TRAFFIC_PER_BRANCH_HEAD = (387.8e6 + 105.8e6) / 8


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=("bsa", "reference"), default="bsa")
    p.add_argument("--workload", choices=("layer", "forward5"), default="layer",
                   help="layer: config-4 attention layer (default); forward5: config-5 "
                        "five-step Wan2.1-14B forward")
    p.add_argument("--layers", type=int, default=0,
                   help="forward5 only: fewer transformer layers (0 = the model's 40)")
    p.add_argument("--heads", type=int, default=40, help="heads (40 = config 4; fewer for profiling)")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cfg-split", action="store_true",
                   help="one rank group for both CFG branches (every rank exchanges heads)")
    p.add_argument("--pull-chunks", default=None,
                   help="N > 2 with --exchange peer: head counts of the pull chunks, "
                        "comma-separated (default: a fifth of the rank's heads, then the rest)")
    p.add_argument("--exchange", choices=("peer", "nccl"), default="peer",
                   help="N > 2: head exchange over peer memory (inputs pulled from the ranks' "
                        "shards, outputs stored by the attention into them), or by NCCL "
                        "all-to-alls")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-route-stage", action="store_true")
    p.add_argument("--no-gpu-comparator", action="store_true",
                   help="skip timing the reference's own GPU path (compiled FlexAttention)")
    p.add_argument("--cpu-seconds", type=float, default=12.0,
                   help="target CPU time of the cpu_baseline sample")
    return p.parse_args(argv)


def load_peaks():
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return {k: float(d[k]) for k in FALLBACK_PEAKS}, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# ----------------------------------------------------------------------------
# workload
# ----------------------------------------------------------------------------

def layer_config(heads):
    from dit_sparse_atten_b200 import synthetic
    c = synthetic.CONFIG4
    return synthetic.LayerConfig(c.name, c.grid, c.batch, heads, c.head_dim, c.block,
                                 c.mass_target, c.keep)


def blob_scores(cfg):
    """Per-branch blob block scores [B, H, Qb, Kb] (CPU, seeds 100 + branch)."""
    from dit_sparse_atten_b200 import synthetic
    full = synthetic.CONFIG4.heads
    return torch.stack([synthetic.blob_scores(full, cfg.blocks, seed=100 + b)[:cfg.heads]
                        for b in range(cfg.batch)])


def kept_flops(route, tokens, block, dim):
    """Algorithmic FLOPs of QK^T + PV over kept blocks: sum 4 * q_valid * k_valid * D."""
    blocks = route.shape[-1]
    sizes = torch.clamp(tokens - torch.arange(blocks, dtype=torch.float64) * block, max=block)
    per = (sizes[:, None] * sizes[None, :]).to(route.device)
    return float(4.0 * dim * (route.to(torch.float64) * per).sum())


# ----------------------------------------------------------------------------
# clocks during the timed region
# ----------------------------------------------------------------------------

class ClockSampler:
    """SM clocks and clock-event reasons of one GPU during the timed region.

    Read-only NVML queries from a background thread every 20 ms, plus one
    sample on entry and one on exit so that short regions are covered;
    ``nvidia-smi -lms`` is the fallback when NVML is unavailable.
    """
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.nvml = None
        self.samples = []            # (sm_mhz, max_mhz, set of reason names)
        try:
            import pynvml
            pynvml.nvmlInit()
            props = torch.cuda.get_device_properties(index)
            bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
            try:
                self.handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except pynvml.NVMLError:
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.bits = {"hw_slowdown": pynvml.nvmlClocksEventReasonHwSlowdown,
                         "hw_thermal_slowdown": pynvml.nvmlClocksEventReasonHwThermalSlowdown,
                         "sw_thermal_slowdown": pynvml.nvmlClocksEventReasonSwThermalSlowdown,
                         "sw_power_cap": pynvml.nvmlClocksEventReasonSwPowerCap}
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.handle,
                                                                  pynvml.NVML_CLOCK_SM))
            self.nvml = pynvml
        except Exception:
            self.nvml = None

    def _sample(self):
        n = self.nvml
        sm = float(n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM))
        mask = n.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
        self.samples.append((sm, self.max_mhz,
                             {name for name, bit in self.bits.items() if mask & bit}))

    def _loop(self):
        while not self._stop.wait(0.02):
            self._sample()

    def __enter__(self):
        if self.nvml is not None:
            import threading
            self._sample()
            self._stop = threading.Event()
            self._thread = threading.Thread(target=self._loop, daemon=True)
            self._thread.start()
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.nvml is not None:
            self._stop.set()
            self._thread.join()
            self._sample()
            return
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            for line in out.splitlines():
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 7:
                    continue
                try:
                    sm, mx = float(parts[0]), float(parts[1])
                except ValueError:
                    continue
                self.samples.append((sm, mx, {name for name, val in zip(self.NAMES, parts[3:7])
                                              if val.lower() == "active"}))

    def summary(self):
        sm = [s[0] for s in self.samples]
        reasons = set().union(*(s[2] for s in self.samples)) if self.samples else set()
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": self.samples[-1][1] if self.samples else None,
                "samples": len(sm), "reasons": sorted(reasons),
                "source": "nvml" if self.nvml is not None else "nvidia-smi"}


# ----------------------------------------------------------------------------
# CPU baseline: the reference's own CPU code (baseline/_ref), else the oracle port
# ----------------------------------------------------------------------------

def reference_root():
    """Directory that holds the reference's ``attention_backends`` package:
    ``$BSA_REFERENCE`` if set, else ``baseline/_ref`` (the reference installed
    unmodified with pip), else None."""
    candidates = []
    if os.environ.get("BSA_REFERENCE"):
        candidates.append(Path(os.environ["BSA_REFERENCE"]))
    candidates.append(REPO / "baseline" / "_ref")
    for root in candidates:
        if (root / "attention_backends" / "flex.py").exists():
            return root
    return None


def load_reference():
    """``(modules, None)`` with the reference's flex / sparse / spatial /
    layout_ops modules, or ``(None, reason)`` when it is not installed."""
    root = reference_root()
    if root is None:
        return None, "reference package not installed (no baseline/_ref, no $BSA_REFERENCE)"
    if str(root) not in sys.path:
        sys.path.insert(0, str(root))
    try:
        from attention_backends import flex, layout_ops, sparse, spatial
    except Exception as exc:  # a broken install is reported, not fatal
        return None, f"reference import failed: {exc!r}"
    return SimpleNamespace(flex=flex, sparse=sparse, spatial=spatial, layout_ops=layout_ops,
                           root=str(root)), None


def cpu_model():
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_threads():
    return os.cpu_count() or 1


def reference_routes(ref, cfg, heads):
    """Config-4 routes of the first ``heads`` heads per branch, made by the
    reference's own rule: ``_top_mass_route`` on the blob scores, then the
    first-frame sink (``flex.py:83-94,550-566``)."""
    scores = blob_scores(cfg)
    routes = []
    for b in range(cfg.batch):
        r = ref.flex._top_mass_route(scores[b, :heads], cfg.mass_target, cfg.keep)
        r[..., :cfg.sink_blocks] = True
        routes.append(r)
    return routes


class RefCpuAttention:
    """The reference's CPU sparse attention, ``sparse_chunk(use_triton=False)``
    (``sparse.py:670-751``), on (branch, query-block) rows of config 4 over a
    subset of heads (its route statistics included, as the reference computes
    them).  Each call takes the next query blocks, branches alternating."""

    kind = "reference"

    def __init__(self, ref, cfg, heads=8):
        self.ref, self.cfg, self.heads = ref, cfg, heads
        self.routes = reference_routes(ref, cfg, heads)
        g = torch.Generator().manual_seed(41)
        shape = (1, cfg.tokens, heads, cfg.head_dim)
        self.qkv = [torch.randn(shape, generator=g).to(torch.bfloat16).float() for _ in range(3)]
        self.stats = ref.sparse._empty_route_stats(heads, cfg.blocks, "cpu")
        self.cursor = 0

    def describe(self, rows, seconds):
        return (f"{rows} (branch, query-block) rows x {self.heads} heads of config 4 through the "
                f"reference's sparse_chunk(use_triton=False), float32 ({seconds:.1f} s)")

    def run(self, rows):
        cfg, q, k, v = self.cfg, *self.qkv
        flops = 0.0
        for _ in range(rows):
            idx = self.cursor % (cfg.batch * cfg.blocks)
            self.cursor += 1
            b, qb = idx % cfg.batch, (idx // cfg.batch * 37) % cfg.blocks
            route = self.routes[b]
            self.ref.sparse.sparse_chunk(q, k, v, route, cfg.block, qb * cfg.block,
                                         (qb + 1) * cfg.block, cfg.head_dim ** -0.5, self.stats,
                                         use_triton=False)
            flops += 4.0 * cfg.block ** 2 * cfg.head_dim * float(route[:, qb].sum())
        return flops


class PortCpuAttention:
    """Fallback when the reference is not installed: the oracle port of the
    same CPU path (gather the kept key blocks of one (head, query block),
    masked softmax, PV, float32)."""

    kind = "port"

    def __init__(self, cfg):
        from oracle import route as oroute
        scores = blob_scores(cfg).numpy()
        self.routes = oroute.add_first_frame_sink(
            oroute.top_mass_route(scores, cfg.mass_target, cfg.keep), cfg.grid, cfg.block)
        self.cfg = cfg
        g = torch.Generator().manual_seed(41)
        shape = (cfg.tokens, 128)
        self.qkv = [torch.randn(shape, generator=g).to(torch.bfloat16).float().numpy()
                    for _ in range(3)]
        self.cursor = 0

    def describe(self, rows, seconds):
        return (f"{rows} (branch, head, query-block) rows of config 4 through the numpy "
                f"oracle port (float32, {seconds:.1f} s)")

    def run(self, rows):
        from oracle import attention as oatt
        cfg = self.cfg
        q, k, v = self.qkv
        flops = 0.0
        for _ in range(rows):
            idx = self.cursor % (cfg.batch * cfg.heads * cfg.blocks)
            self.cursor += 1
            b, rest = divmod(idx, cfg.heads * cfg.blocks)
            h, qb = divmod(rest, cfg.blocks)
            route = self.routes[b, h][None]
            oatt.block_sparse_attention(q[:, None], k[:, None], v[:, None], route, cfg.block,
                                        query_blocks=[qb], dtype=np.float32)
            flops += 4.0 * 128 * 128 * 128 * float(route[0, qb].sum())
        return flops


def cpu_attention_sample(cfg):
    ref, _why = load_reference()
    return RefCpuAttention(ref, cfg) if ref is not None else PortCpuAttention(cfg)


def reference_cpu_stages(ref, cfg, heads=4):
    """The reference's route decision and spatial reorder on the host, on
    ``heads`` of the 40 heads, scaled to one config-4 layer (2 branches x 40
    heads): sampled mass S = 16 -> persistence prior -> ``_top_mass_route`` ->
    sink -> ``pack_boolean_rows`` (``flex.py:205-251,535-541,83-94``,
    ``layout_ops.py:128-151``), and ``reorder_qkv`` + ``restore``
    (``spatial.py:86-93``, CPU ``index_select``)."""
    scale_to_layer = cfg.batch * cfg.heads / heads
    g = torch.Generator().manual_seed(5)
    shape = (1, cfg.tokens, heads, cfg.head_dim)
    q, k, v = (torch.randn(shape, generator=g).to(torch.bfloat16) for _ in range(3))
    prev = reference_routes(ref, cfg, heads)[1]
    t0 = time.perf_counter()
    mass = ref.flex._sampled_block_mass(q, k, cfg.block, samples=16)
    t1 = time.perf_counter()
    mass = mass + 0.5 * mass.mean(-1, keepdim=True) * prev.float()
    route = ref.flex._top_mass_route(mass, cfg.mass_target, cfg.keep)
    route[..., :cfg.sink_blocks] = True
    ref.layout_ops.pack_boolean_rows(route)
    t2 = time.perf_counter()
    layout = ref.spatial.build_spatial_layout(cfg.grid, cfg.block)
    t3 = time.perf_counter()
    qp, kp, vp = layout.reorder_qkv(q, k, v)
    layout.restore(vp)
    t4 = time.perf_counter()
    return {"route_mass_s_per_layer": (t1 - t0) * scale_to_layer,
            "route_select_pack_s_per_layer": (t2 - t1) * scale_to_layer,
            "reorder_restore_s_per_layer": (t4 - t3) * scale_to_layer,
            "spatial_layout_build_s": t3 - t2,
            "sample": f"{heads} of {cfg.heads} heads of one branch, scaled x{scale_to_layer:g} "
                      "to a config-4 layer (2 branches x 40 heads)"}


def run_cpu_baseline(cfg, seconds):
    torch.set_num_threads(cpu_threads())
    sample = cpu_attention_sample(cfg)
    sample.run(1)  # warm-up
    flops, t0, rows = 0.0, time.perf_counter(), 0
    while time.perf_counter() - t0 < seconds or rows < 4:
        flops += sample.run(2)
        rows += 2
    dt = time.perf_counter() - t0
    line = {"value": flops / dt / 1e12, "unit": UNIT, "cores": cpu_threads(), "kind": sample.kind,
            "cpu_model": cpu_model(), "sample": sample.describe(rows, dt)}
    if sample.kind == "reference":
        line["stages"] = reference_cpu_stages(sample.ref, cfg)
    return line


def run_reference_arm(args):
    """``--impl reference``: the reference's CPU implementation, rank 0 only."""
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    cfg = layer_config(40)
    torch.set_num_threads(cpu_threads())
    sample = cpu_attention_sample(cfg)
    per_step = 1
    for _ in range(max(1, args.warmup)):
        sample.run(per_step)
    flops, t0 = 0.0, time.perf_counter()
    for _ in range(args.steps):
        flops += sample.run(per_step)
    dt = time.perf_counter() - t0
    value = flops / dt / 1e12
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "impl": "reference",
        "data": "synthetic (seeded N(0,1) bf16-valued Q/K/V; blob routes of config 4)",
        "config": {"workload": "config4_wan14b_720p: 57,600 tokens, CFG batch 2, 40 heads, "
                               "head_dim 128, keep cap 0.625, sink 29",
                   "step_sample": sample.describe(per_step, dt / args.steps)},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cpu_threads(),
                         "kind": sample.kind, "cpu_model": cpu_model(),
                         "sample": sample.describe(per_step * args.steps, dt)},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


# ----------------------------------------------------------------------------
# GPU arm
# ----------------------------------------------------------------------------

def main(argv=None):
    args = parse_args(argv)
    if args.impl == "reference":
        return run_reference_arm(args)
    if args.workload == "forward5":
        return run_forward5(args)

    import torch.distributed as dist

    from dit_sparse_atten_b200 import _native, kernels, parallel, synthetic
    from dit_sparse_atten_b200.spatial import build_spatial_layout

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    _native.load_library()

    cfg = layer_config(args.heads)
    plan = parallel.make_plan(world, rank, cfg.heads, batch=cfg.batch,
                              split_cfg=not args.no_cfg_split)
    group = parallel.new_groups(plan) if world > 1 else None
    branches = plan.branches(cfg.batch)
    hs = plan.head_slice
    P = plan.group_size

    # routes: blob scores -> GPU selection (bit-identical to the reference's rule)
    scores = blob_scores(cfg)
    sel = kernels.route_select(scores.to(device), target=cfg.mass_target, keep=cfg.keep,
                               sink_blocks=cfg.sink_blocks)
    route_all = sel.route.bool()                                   # [B, H, Qb, Kb]
    total_flops = kept_flops(route_all, cfg.tokens, cfg.block, cfg.head_dim)
    keep_fraction = float(route_all.float().mean())
    local_route = route_all[branches][:, hs].contiguous()
    counts, indices = kernels.pack_boolean_rows(local_route)

    layout = build_spatial_layout(cfg.grid, cfg.block)
    q, k, v = synthetic.wan_qkv(cfg, seed=41, device=device)
    q, k, v = (x[branches].contiguous() for x in (q, k, v))
    t_local = cfg.tokens // P
    seq = slice(plan.group_rank * t_local, (plan.group_rank + 1) * t_local)
    if P > 1:
        q, k, v = (x[:, seq].contiguous() for x in (q, k, v))
    torch.cuda.synchronize()

    stream = torch.cuda.current_stream(device)
    attn_events = []
    pipe = None
    if P > 1:
        # chunked exchange overlapped with the attention of earlier chunks,
        # one pipelined call per CFG branch of this rank's group
        pipe = parallel.PipelinedHeadParallel(group, P, cfg.heads, t_local,
                                              perm=layout.permutation_cpu,
                                              inverse=layout.inverse_cpu,
                                              peer_out=args.exchange == "peer",
                                              peer_in=args.exchange == "peer",
                                              pull_chunks=([int(x) for x in
                                                            args.pull_chunks.split(",")]
                                                           if args.pull_chunks else None))
        if pipe.peer_in and len(branches) == 1:
            # the step's inputs live in this rank's mapped input shard (as a
            # caller that produces them there would have them): no copy
            bufs = pipe.input_buffers(device, q.dtype, cfg.head_dim)
            for dst_t, src_t in zip(bufs, (q, k, v)):
                dst_t.copy_(src_t)
            q, k, v = bufs
        csr_cache = {}

        def chunk_csr(bi, c):
            # the CSR rows of chunk c's heads (the chunk plan of the exchange
            # in effect), cut once per branch and chunk
            hs = pipe.chunk_slices()[c]
            key = (bi, hs.start, hs.stop)
            if key not in csr_cache:
                csr_cache[key] = (counts[bi, hs].contiguous(), indices[bi, hs].contiguous())
            return csr_cache[key]
        branch_now = [0]

        chunk_events = []

        def attend_chunk(qp, kp, vp, c, out, out_rows, peers=None):
            # the output store writes token order straight into the ranks'
            # output shards over peer memory (or into the send buffer of the
            # output all-to-all): the unpack and the exchange folded in
            cur = torch.cuda.current_stream(device)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(cur)
            csr = chunk_csr(branch_now[0], c)
            if peers is not None:
                kernels.block_sparse_attention_peers(qp, kp, vp, *csr, peers, block=cfg.block,
                                                     out_rows=out_rows)
            else:
                kernels.block_sparse_attention(qp, kp, vp, *csr, block=cfg.block, out=out,
                                               out_rows=out_rows)
            e1.record(cur)
            chunk_events.append((e0, e1))
            if c == len(pipe.chunk_slices()) - 1:
                # attention time of the step: first chunk start to last chunk end
                attn_events.append((chunk_events[0][0], [e for _, e in chunk_events]))
                chunk_events.clear()
            return None

    perm_dev = layout.permutation(device)

    def attend(qh, kh, vh):
        # pack, then attention whose output store writes raster order (the
        # unpack folded into the epilogue)
        qp, kp, vp = layout.reorder_qkv(qh, kh, vh)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        out = kernels.block_sparse_attention(qp, kp, vp, counts, indices, block=cfg.block,
                                             out_rows=perm_dev)
        e1.record(stream)
        attn_events.append((e0, e1))
        return out

    def step():
        if pipe is not None:
            outs = []
            for bi in range(len(branches)):
                branch_now[0] = bi
                outs.append(pipe(q[bi:bi + 1], k[bi:bi + 1], v[bi:bi + 1], attend_chunk))
            return outs
        return attend(q, k, v)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    _native.check_device_errors()
    attn_events.clear()
    barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            out = step()
        end.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms = start.elapsed_time(end) / args.steps
    attn_ms = sum(max(a.elapsed_time(e) for e in b) if isinstance(b, list) else a.elapsed_time(b)
                  for a, b in attn_events) / args.steps
    _native.check_device_errors()
    rank_ms = None
    if world > 1:
        # Per-rank step and attention times (max over ranks is the reported
        # figure; the spread shows load imbalance between head shards).
        mine = torch.tensor([ms, attn_ms], device=device, dtype=torch.float64)
        every = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(every, mine)
        rank_ms = {"step": [round(float(e[0]), 3) for e in every],
                   "attention": [round(float(e[1]), 3) for e in every],
                   # step time not covered by this rank's attention span: the
                   # exchange (and its row moves) left exposed
                   "exposed": [round(float(e[0] - e[1]), 3) for e in every]}
        ms = max(float(e[0]) for e in every)
        attn_ms = max(float(e[1]) for e in every)

    # per-stage breakdown (one extra step, rank-local)
    stages = {}
    comparator = None
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    qh, kh, vh = (q, k, v) if P == 1 else (None, None, None)
    if P == 1:
        ev[0].record(stream)
        qp, kp, vp = layout.reorder_qkv(q, k, v)
        ev[1].record(stream)
        out_p = kernels.block_sparse_attention(qp, kp, vp, counts, indices, block=cfg.block,
                                               out_rows=perm_dev)
        ev[2].record(stream)
        # the standalone unpack kernel (not part of the step: its store is
        # folded into the attention), timed for the reorder's roofline
        layout.restore(out_p)
        ev[3].record(stream)
        torch.cuda.synchronize()
        elem = q.numel() * q.element_size()
        pack_ms, unpack_ms = ev[0].elapsed_time(ev[1]), ev[2].elapsed_time(ev[3])
        stages = {"pack_ms": pack_ms, "attention_ms": ev[1].elapsed_time(ev[2]),
                  "unpack_ms_standalone": unpack_ms,
                  "pack_hbm_gbs": 6 * elem / pack_ms / 1e6,
                  "unpack_hbm_gbs": 2 * elem / unpack_ms / 1e6}
        if not args.no_route_stage:
            stages.update(route_stage(cfg, qp, kp, local_route, kernels, device, stream,
                                      layout.neighbors(device)))
            stages.update(bootstrap_stage(cfg, qp, kp, vp, kernels, stream))
            stages.update(prologue_stage(cfg, layout, kernels, device, stream))
        if not args.no_gpu_comparator:
            try:
                comparator = gpu_comparator(cfg, q, k, v, qp, kp, vp, local_route, counts,
                                            indices, stages, kernels)
            except Exception as exc:   # the reference's own code failed: report, go on
                comparator = {"unavailable": f"reference GPU path raised {exc!r}"[:400]}
            torch.cuda.synchronize()

    peaks, peak_src = load_peaks()
    local_flops = kept_flops(local_route, cfg.tokens, cfg.block, cfg.head_dim)
    achieved = local_flops / (attn_ms * 1e-3) / 1e12
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops_sustained"],
                "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops_sustained"],
                "traffic": ATTENTION_TRAFFIC_PER_BRANCH_HEAD * local_route.shape[0] * local_route.shape[1],
                "traffic_source": "ncu dram bytes of the 4-head case, scaled by branches x heads",
                "peak_source": f"bf16_tflops_sustained ({peak_src})",
                "frac_of_burst": achieved / peaks["bf16_tflops"],
                "kernel": "bsa_attention_kernel<128>", "kernel_ms": attn_ms,
                "flops_per_launch": local_flops}

    value = total_flops / (ms * 1e-3) / 1e12
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded Wan-like RMS-normed + 3D-RoPE Q/K, N(0,1) V; blob routes)",
        "config": {
            "workload": "config4_wan14b_720p: one self-attention layer, CFG batch 2",
            "tokens": cfg.tokens, "heads": cfg.heads, "head_dim": cfg.head_dim,
            "cfg_batch": cfg.batch, "block": cfg.block, "grid": list(cfg.grid),
            "microtile": list(layout.microtile_shape), "keep_fraction": keep_fraction,
            "kept_flops": total_flops,
            "dense_equivalent_tflops": 4.0 * cfg.tokens ** 2 * cfg.heads * cfg.head_dim
            * cfg.batch / (ms * 1e-3) / 1e12,
            "parallelism": ("single GPU" if world == 1 else
                            f"{plan.cfg_groups} CFG group(s) x {P}-way head parallel "
                            + (f"({len(pipe.chunk_slices())} head chunks "
                               f"({[sl.stop - sl.start for sl in pipe.chunk_slices()]} heads) "
                               "overlapped with attention; "
                               + ("inputs pulled from the ranks' shards and outputs stored by "
                                  "the attention into them, over peer memory)"
                                  if pipe.peer_in else
                                  "NCCL input and output all-to-alls)")
                               if pipe is not None else "(NCCL)")),
            "l2": "inputs (3 x 1.18 GB) exceed L2; no flush"},
        "stages": stages,
        **({"gpu_comparator": comparator} if comparator is not None else {}),
        "roofline": roofline,
        # pack + attention per step (unpack folded into the store); the chunked
        # exchange runs send gather, packed gather, attention and output
        # scatter per chunk
        # per rank and branch: C send-row scatters, C receive gathers, C
        # attentions (+ C output scatters with the NCCL output all-to-all)
        "gpu_launches": args.steps * world * (
            len(branches) * len(pipe.chunk_slices())
            * (2 if pipe.peer_in else 3 if pipe.peer_out else 4)
            if pipe is not None else 2),
        **({"rank_ms": rank_ms} if rank_ms is not None else {}),
        "clocks": clocks.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = run_cpu_baseline(cfg, args.cpu_seconds)
    if not args.no_e2e:
        line["e2e"] = run_e2e(args, cfg, plan, group, branches, local_route, layout, device,
                              total_flops)
    if world > 1:
        dist.barrier()
    if rank == 0:
        print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()
    return 0


# ----------------------------------------------------------------------------
# config 5: 5-step Wan2.1-14B forward
# ----------------------------------------------------------------------------

FORWARD5_FLEX = dict(bootstrap_mode="sampled", prefetch_sampled_bootstrap=True,
                     sampled_update_interval=2, prefetch_sampled_update=False, route_samples=16,
                     route_persistence=0.5, mass_target=0.95, keep=0.625,
                     dense_route_threshold=0.58, spatial_reorder=True, total_steps=5)


def run_forward5(args):
    """Config 5: five denoising steps of a random-init Wan2.1-14B (40 layers,
    dim 5120, 57,600 tokens, text 512 x 4096), CFG on, through the repo's
    frontend (``wan_model``) on 1-8 GPUs: CFG branches on two rank groups,
    tokens sequence-parallel inside a group, self-attention head-parallel.
    Three runs of the same generation: dense SDPA attention; the
    ``flex_reuse`` backend with the reference's recommended flags
    (``README.md:46-54``: sampled bootstrap, sampled update every 2 steps,
    dense dispatch at keep >= 0.58); and the same backend with the dense
    threshold off, so every route after layer 0 / step 0 runs sparse.  Each is
    warmed up with three steps (first use of every collective included), then
    timed from the first transformer call to the last scheduler update with
    CUDA events (max over ranks)."""
    import torch.distributed as dist

    from dit_sparse_atten_b200 import _native, parallel, wan_model
    from dit_sparse_atten_b200.context import reset_runtime_state
    from dit_sparse_atten_b200.dense import DenseBackend
    from dit_sparse_atten_b200.flex import FlexReuseBackend, FlexReuseConfig

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    _native.load_library()
    cfg = wan_model.WanConfig(layers=args.layers) if args.layers else wan_model.WAN_14B
    grid = (16, 45, 80)
    plan = parallel.make_plan(world, rank, cfg.heads, batch=2)
    group = parallel.new_groups(plan) if world > 1 else None
    pair = (wan_model.pair_groups(world, plan.group_size)
            if world > 1 and plan.cfg_groups == 2 else None)
    P = plan.group_size
    shard = wan_model.SequenceShard(group if P > 1 else None, P, plan.group_rank)
    weights = wan_model.WanWeights(cfg, device, seed=0)
    model = wan_model.WanTransformer(weights, grid, shard, wan_model.fused_prologue(cfg.heads,
                                                                                   cfg.eps))
    g = torch.Generator(device=device)
    g.manual_seed(1)
    latent = torch.randn((cfg.in_channels, grid[0], 2 * grid[1], 2 * grid[2]), generator=g,
                         device=device)
    text = [torch.randn((1, cfg.text_tokens, cfg.text_dim), generator=g, device=device,
                        dtype=torch.bfloat16) for _ in range(2)]
    rows = wan_model.patchify(latent, cfg)[model.rows].contiguous()
    branches = plan.branches(2)
    contexts = {b: model.context(text[b]) for b in branches}
    combine = wan_model.CfgCombine(5.0, pair_group=pair)

    def timed(make_backend, steps):
        backend = make_backend()
        reset_runtime_state()

        def attention(q, k, v):
            if isinstance(backend, FlexReuseBackend):
                return backend.head_parallel(q, k, v, shard.group, P)
            return parallel.head_parallel_attention(q, k, v, lambda a, b, c: backend(a, b, c),
                                                    shard.group, P)
        step_ms = []
        marks = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        marks[0].record()
        out = wan_model.denoise(model, rows, contexts, attention, combine, steps=steps,
                                on_step=lambda i: marks[i + 1].record())
        torch.cuda.synchronize()
        _native.check_device_errors()
        step_ms = [marks[i].elapsed_time(marks[i + 1]) for i in range(steps)]
        total = torch.tensor([sum(step_ms)], device=device, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(total, op=dist.ReduceOp.MAX)
        summary = backend.profile_summary() if hasattr(backend, "profile_summary") else None
        return float(total[0]) / 1e3, step_ms, summary, bool(torch.isfinite(out).all())

    variants = {
        "dense": lambda: DenseBackend(),
        "flex_reuse": lambda: FlexReuseBackend(FlexReuseConfig(**FORWARD5_FLEX),
                                               process_group=group),
        "flex_reuse_all_sparse": lambda: FlexReuseBackend(
            FlexReuseConfig(**{**FORWARD5_FLEX, "dense_route_threshold": None}),
            process_group=group),
    }
    results = {}
    with ClockSampler(local) as clocks:
        for name, make in variants.items():
            # warm-up: three steps with a fresh state, so the route bootstrap,
            # its adoption (the keep all-reduce) and an update have all run once
            timed(make, 3)
            seconds, step_ms, summary, finite = timed(make, 5)
            results[name] = {"forward_5step_s": seconds,
                             "step_ms_rank0": [round(x, 1) for x in step_ms],
                             "finite": finite}
            if summary is not None:
                results[name]["routes"] = {k: summary[k] for k in
                                           ("phase_counts", "mean_route_keep",
                                            "dense_dispatched_routes", "released_routes")}
    line = {
        "metric": METRIC, "value": results["flex_reuse"]["forward_5step_s"], "unit": "s",
        "n_gpus": world, "steps": 5, "warmup": 3, "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init Wan2.1-14B weights, seeded latent and text)",
        "config": {"workload": "config5_wan14b_5step_forward: 57,600 tokens, CFG on, "
                               f"{cfg.layers} layers, dim {cfg.dim}, FFN {cfg.ffn}, "
                               f"{cfg.heads} heads, text {cfg.text_tokens} x {cfg.text_dim}",
                   "parallelism": f"{plan.cfg_groups} CFG group(s) x {P}-way sequence/head "
                                  "parallel (Ulysses all-to-all, NCCL)",
                   "params": weights.parameter_count(),
                   "flex_reuse_flags": FORWARD5_FLEX},
        "variants": results,
        "speedup_vs_dense": {k: results["dense"]["forward_5step_s"] / v["forward_5step_s"]
                             for k, v in results.items() if k != "dense"},
        "clocks": clocks.summary(),
    }
    if rank == 0:
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def route_stage(cfg, qp, kp, route, kernels, device, stream, neighbors):
    """Route decision on this layer: sampled mass (S=16) + prior + top-mass + sink + CSR,
    and the directional frontier update of the same route (flex.py:517-534)."""
    prev = route
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    for _ in range(2):
        mass = kernels.sampled_block_mass(qp, kp, cfg.block, 16)
        kernels.route_select(mass, prev, 0.5, cfg.mass_target, cfg.keep, cfg.sink_blocks)
    ev[0].record(stream)
    mass = kernels.sampled_block_mass(qp, kp, cfg.block, 16)
    ev[1].record(stream)
    kernels.route_select(mass, prev, 0.5, cfg.mass_target, cfg.keep, cfg.sink_blocks)
    ev[2].record(stream)
    torch.cuda.synchronize()
    mass_ms, select_ms = ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2])
    front = kernels.frontier_mask(prev, neighbors)
    dev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    for i in range(3):
        if i == 2:
            dev[0].record(stream)
        kernels.directional_update(mass, prev, neighbors, keep=cfg.keep, persistence=0.5,
                                   previous_frontier=front, sink_blocks=cfg.sink_blocks)
    dev[1].record(stream)
    torch.cuda.synchronize()
    directional_ms = dev[0].elapsed_time(dev[1])
    from dit_sparse_atten_b200 import _native
    _native.check_device_errors()   # a timed-out wait must not pass as a timing
    B, H, Qb = mass.shape[0], mass.shape[1], mass.shape[2]
    # mass 4 + previous 1 + frontier 1 + candidates 3 (clear, scatter, final)
    # + route/frontier/exploration/dropped/added 5 + CSR ids 4 bytes per cell
    directional_bytes = B * H * Qb * Qb * 18 + B * H * Qb * 4
    sampled = 2 * B * H * Qb * 16 * cfg.head_dim * 2
    select_bytes = B * H * Qb * Qb * (4 + 1 + 1 + 4) + B * H * Qb * 4
    return {"route_mass_ms": mass_ms, "route_select_ms": select_ms,
            # algorithmic: one Q_s K_s^T product (the kernel streams the keys once)
            "route_mass_tflops": 2 * B * H * (Qb * 16) ** 2 * cfg.head_dim / mass_ms / 1e9,
            "route_select_hbm_gbs": select_bytes / select_ms / 1e6,
            "directional_update_ms": directional_ms,
            "directional_update_hbm_gbs": directional_bytes / directional_ms / 1e6,
            "route_mass_hbm_gbs": (sampled + B * H * Qb * Qb * 4) / mass_ms / 1e6}


def bootstrap_stage(cfg, qp, kp, vp, kernels, stream):
    """Exact bootstrap of this layer (flex.py:254-272): dense attention that
    also yields its exact block mass (one pass over the keys)."""
    from dit_sparse_atten_b200 import _native
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    kernels.dense_attention_block_mass(qp, kp, vp)
    ev[0].record(stream)
    kernels.dense_attention_block_mass(qp, kp, vp)
    ev[1].record(stream)
    torch.cuda.synchronize()
    _native.check_device_errors()
    ms = ev[0].elapsed_time(ev[1])
    B, T, H, D = qp.shape
    return {"bootstrap_dense_and_mass_ms": ms,
            "bootstrap_dense_tflops": 4.0 * B * H * T * T * D / ms / 1e9}


def gpu_comparator(cfg, q, k, v, qp, kp, vp, route_all, counts, indices, stages, kernels,
                   reps=5):
    """The reference's own GPU path on this GPU, on the same config-4 inputs and
    routes, stage by stage as its stage profiler does (``profiles/flex_route.py:53-127``):
    compiled FlexAttention over ``_build_block_mask`` of the same boolean route,
    ``_sampled_block_mass`` (S = 16), prior + ``_top_mass_route`` + sink +
    ``_build_block_mask``, the Triton ``reorder_qkv`` and ``restore``, the
    exact bootstrap (dense FlexAttention with LSE + ``_block_attention_mass``)
    and dense SDPA.  Each CFG branch is one batch-1 call, as the reference
    runs them.  Times are CUDA-event medians; this repo's figures for the same
    stages come from ``stages`` and the ratios are reference ms / this ms."""
    ref, why = load_reference()
    if ref is None:
        return {"unavailable": why}
    import torch.nn.functional as F

    B, T, H, D = qp.shape
    scale = D ** -0.5
    block = cfg.block

    def timed(fn, n=reps):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        times = []
        for _ in range(n):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            e1.synchronize()
            times.append(e0.elapsed_time(e1))
        return statistics.median(times)

    where = os.path.relpath(ref.root, REPO) if ref.root.startswith(str(REPO)) else "$BSA_REFERENCE"
    res = {"reference": f"{where}: the reference's attention_backends, unmodified "
                        f"(torch {torch.__version__}, FlexAttention compiled by Inductor)",
           "errors": {}}
    t0 = time.perf_counter()

    def stage(name, fn):
        # one failing stage of the reference (e.g. a Triton kernel that does
        # not compile here) is reported and the others still run
        try:
            fn()
        except Exception as exc:
            res["errors"][name] = repr(exc)[:300]
        torch.cuda.synchronize()

    masks = [ref.flex._build_block_mask(route_all[b], T, block) for b in range(B)]

    def flex_sparse():
        return [ref.flex._flex_output(qp[b:b + 1], kp[b:b + 1], vp[b:b + 1], masks[b], block,
                                      True, scale=scale) for b in range(B)]

    def flex_stage():
        theirs = flex_sparse()
        torch.cuda.synchronize()
        res["compile_s"] = time.perf_counter() - t0
        # same inputs, same routes: the reference's output against this repo's kernel
        mine = kernels.block_sparse_attention(qp, kp, vp, counts, indices, block=block)
        diff = torch.cat([(theirs[b][0].float() - mine[b].float()).abs().flatten()
                          for b in range(B)])
        res["flex_vs_bsa_max_abs"] = float(diff.max())
        res["flex_vs_bsa_mean_abs"] = float(diff.mean())
        del theirs, mine, diff
        res["flex_sparse_ms"] = timed(flex_sparse)

    stage("flex_sparse", flex_stage)

    def sampled():
        return [ref.flex._sampled_block_mass(qp[b:b + 1], kp[b:b + 1], block, samples=16,
                                             scale=scale) for b in range(B)]

    masses = []

    def sampled_stage():
        masses.extend(sampled())
        res["sampled_mass_ms"] = timed(sampled)

    stage("sampled_mass", sampled_stage)

    def select_and_mask():
        for b in range(B):
            m = masses[b] + 0.5 * masses[b].mean(-1, keepdim=True) * route_all[b].float()
            r = ref.flex._top_mass_route(m, cfg.mass_target, cfg.keep)
            r[..., :cfg.sink_blocks] = True
            ref.flex._build_block_mask(r, T, block)

    if masses:
        stage("select_and_mask",
              lambda: res.__setitem__("select_and_mask_ms", timed(select_and_mask)))
    del masses, masks

    layout = ref.spatial.build_spatial_layout(cfg.grid, block)
    stage("reorder", lambda: res.__setitem__("reorder_ms",
                                             timed(lambda: layout.reorder_qkv(q, k, v))))
    stage("restore", lambda: res.__setitem__("restore_ms", timed(lambda: layout.restore(q))))
    stage("sdpa_dense", lambda: res.__setitem__("sdpa_dense_ms", timed(
        lambda: F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2),
                                               v.transpose(1, 2), scale=scale), n=3)))

    dense_flex = ref.flex._flex_kernel(True)

    def dense_lse():
        return [dense_flex(qp[b:b + 1].transpose(1, 2), kp[b:b + 1].transpose(1, 2),
                           vp[b:b + 1].transpose(1, 2), scale=scale, return_lse=True)
                for b in range(B)]

    def exact_bootstrap():
        for b, (_o, lse) in enumerate(dense_lse()):
            ref.flex._block_attention_mass(qp[b:b + 1], kp[b:b + 1], lse, block, scale=scale)

    stage("dense_flex_lse", lambda: res.__setitem__("dense_flex_lse_ms", timed(dense_lse, n=3)))
    stage("exact_bootstrap", lambda: res.__setitem__("exact_bootstrap_ms",
                                                     timed(exact_bootstrap, n=3)))
    res["total_s"] = time.perf_counter() - t0

    pairs = {"attention": ("flex_sparse_ms", "attention_ms"),
             "sampled_mass": ("sampled_mass_ms", "route_mass_ms"),
             "select": ("select_and_mask_ms", "route_select_ms"),
             "reorder": ("reorder_ms", "pack_ms"),
             "exact_bootstrap": ("exact_bootstrap_ms", "bootstrap_dense_and_mass_ms")}
    res["speedup"] = {name: res[a] / stages[b] for name, (a, b) in pairs.items()
                      if stages.get(b) and res.get(a)}
    if stages.get("attention_ms") and stages.get("pack_ms") and res.get("flex_sparse_ms"):
        # the layer as the reference runs it (pack, sparse attention, restore)
        # against this repo's step (pack, attention with the unpack in its store)
        theirs_layer = res["reorder_ms"] + res["flex_sparse_ms"] + res["restore_ms"]
        res["layer_ms"] = theirs_layer
        res["speedup"]["layer"] = theirs_layer / (stages["pack_ms"] + stages["attention_ms"])
    return res


def prologue_stage(cfg, layout, kernels, device, stream):
    """The processor's prologue for this layer (both branches): Q/K RMSNorm,
    RoPE and the reorder into route-block order in one pass (HBM-bound)."""
    from dit_sparse_atten_b200 import _native, synthetic
    proj, weights, rotary = synthetic.prologue_inputs(cfg.batch, cfg.grid, cfg.heads, seed=9)
    proj = [p.to(device) for p in proj]
    wq, wk = (w.float().to(device) for w in weights)
    cos, sin = rotary.real.float().to(device), rotary.imag.float().to(device)
    perm = layout.permutation_cpu.to(device)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    kernels.qkv_prologue(*proj, cfg.heads, wq, wk, 1e-6, cos, sin, perm=perm)
    ev[0].record(stream)
    kernels.qkv_prologue(*proj, cfg.heads, wq, wk, 1e-6, cos, sin, perm=perm)
    ev[1].record(stream)
    torch.cuda.synchronize()
    _native.check_device_errors()
    ms = ev[0].elapsed_time(ev[1])
    # read and write Q, K, V once, plus the rotary tables
    algorithmic = 6 * proj[0].numel() * 2 + 2 * cos.numel() * 4
    return {"prologue_ms": ms, "prologue_hbm_gbs": algorithmic / ms / 1e6}


def run_e2e(args, cfg, plan, group, branches, local_route, layout, device, total_flops):
    """Same step through the public backend API, pinned host buffers in and out."""
    import torch.distributed as dist

    from dit_sparse_atten_b200 import parallel, synthetic
    from dit_sparse_atten_b200.context import set_routing_context
    from dit_sparse_atten_b200.flex import FlexReuseBackend, FlexReuseConfig

    world = plan.world
    P = plan.group_size
    backend = FlexReuseBackend(FlexReuseConfig(spatial_reorder=True, bootstrap_mode="sampled",
                                               keep=cfg.keep, mass_target=cfg.mass_target))
    heads_local = plan.heads_per_rank
    for i, b in enumerate(branches):
        backend.install_route(local_route[i], attention_id=1, branch=b, tokens=cfg.tokens,
                              heads=heads_local, head_dim=cfg.head_dim, device=device,
                              grid=cfg.grid)
    t_local = cfg.tokens // P
    g = torch.Generator().manual_seed(77)
    nb = len(branches)
    host = [torch.randn((nb, t_local, cfg.heads, cfg.head_dim), generator=g)
            .to(torch.bfloat16).pin_memory() for _ in range(3)]
    out_host = torch.empty_like(host[0]).pin_memory()
    stream = torch.cuda.current_stream(device)
    # Copies overlap compute: inputs of (step, branch) go up on h2d, results
    # come back on d2h, compute stays on the current stream; device input
    # buffers alternate by step parity.  Every step still copies its own
    # inputs from pinned host memory and reads its result back.
    h2d = torch.cuda.Stream(device)
    d2h = torch.cuda.Stream(device)
    dev_in = [[[torch.empty_like(host[t][b], device=device) for t in range(3)] for b in range(nb)]
              for _ in range(2)]
    slot_free = [[None] * nb for _ in range(2)]

    def step(i):
        slot = i % 2
        for bi, b in enumerate(branches):
            bufs = dev_in[slot][bi]
            with torch.cuda.stream(h2d):
                if slot_free[slot][bi] is not None:
                    h2d.wait_event(slot_free[slot][bi])
                for t in range(3):
                    bufs[t].copy_(host[t][bi], non_blocking=True)
                ready = torch.cuda.Event()
                ready.record(h2d)
            stream.wait_event(ready)
            set_routing_context(attention_id=1, step=1, branch=b, grid=cfg.grid)
            qi, ki, vi = (x.unsqueeze(0) for x in bufs)
            out = backend.head_parallel(qi, ki, vi, group, P)
            done = torch.cuda.Event()
            done.record(stream)
            slot_free[slot][bi] = done
            with torch.cuda.stream(d2h):
                d2h.wait_event(done)
                out_host[bi].copy_(out[0], non_blocking=True)
                out.record_stream(d2h)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    h2d.wait_event(start)
    d2h.wait_event(start)
    for i in range(args.steps):
        step(args.warmup + i)
    stream.wait_stream(d2h)
    stream.wait_stream(h2d)
    end.record(stream)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t[0])
    per_rank_in = sum(h.numel() * h.element_size() for h in host)
    return {"value": total_flops / (ms * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": ms,
            "h2d_bytes_per_step": per_rank_in * world,
            "d2h_bytes_per_step": out_host.numel() * out_host.element_size() * world,
            "api": "FlexReuseBackend.head_parallel (reuse phase, spatial reorder; head chunks "
                   "overlapped with the exchange for P > 1) per CFG branch; "
                   "H2D/D2H on side streams overlapping compute (every step copies its own "
                   "inputs in and its output out)"}


if __name__ == "__main__":
    sys.exit(main())
