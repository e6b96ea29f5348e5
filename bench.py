"""Benchmark of the VQ-MoE expert layer on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c1|c2|c3|c4]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N \
        --master-addr 127.0.0.1 --master-port P bench.py --gpus N ...

Metric: VQ-MoE layer tokens/s, with the dominant kernel's
HBM GB/s as a fraction of the measured roofline.

A step is one call of the Qwen3.5-MoE sparse block (router, fused VQ
gate/up + SwiGLU, VQ down, shared expert, combine) over one batch of
synthetic tokens, configuration c2 (H 2048, 128 experts top-8, I 768 +
shared 768, 64 tokens = 16 sequences x (1 + 3 MTP drafts)) at every N, so
that the scaling run compares like with like. By default the N GPUs run N
independent replicas of the layer, each on its own 64 tokens (tokens are
independent: no collective on the data path; weak scaling). `--tp S`
tensor-splits the layer S ways instead (gate/up cut on I, down on I,
float32 partials all-reduced over NCCL), as far as the reference's cut
rules allow -- c2's I = 768 allows 2 and 4 -- with N / S replicas of the
split. `--workload c4` (H 4096, 256 experts top-8, I 1536, 256 tokens) is
the tensor-split block the baseline names for 2/4/8 GPUs.

Inputs larger than L2: the timed loop cycles over several independently
seeded copies of the layer (> 3x the 126 MB L2 in total), so every step
streams its experts from HBM, as consecutive layers of a model do.
`value` times CUDA-graph replays of the block with the input resident in
HBM; `e2e` times the public captured call (`CapturedBlock`) with the input
copied from pinned host memory and the output read back every step.

--impl reference times the CPU restatement of the reference semantics
(`oracle/`, the reference's own MLX code cannot run here) on all host
threads; each step is a bounded sample (a rotating subset of the routed
experts, rescaled by its share of the layer's expert work).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "VQ-MoE layer tokens/s"
UNIT = "tokens/s"
EXPERT_KERNEL = "expert_kernel<true,true>"
# kernels of one block call: router logits, top-k + routing sort, shared
# gate/up, shared down, routed experts (both stages), combine
LAUNCHES_PER_STEP = 6


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--tp", type=int, default=1,
                    help="tensor split of the layer (N / tp independent replicas)")
    return ap.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return world, rank, local


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], "measured"
    return 6650.0, "fallback"


def tensor_peak():
    """Dense bf16 TFLOP/s: the burst figure (a kernel timed alone)."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text())["bf16_tflops"], "measured"
    return 1590.0, "fallback"


def traffic_from_profiles(kernel_key: str, workload: str):
    """DRAM bytes per launch of `kernel_key` from the committed ncu summary
    (a line `dram_bytes_per_launch <workload> <kernel> <bytes>`)."""
    for f in sorted((ROOT / "profiles").glob("*.md")) + sorted((ROOT / "profiles").glob("*.txt")):
        for line in f.read_text().splitlines():
            m = re.match(r"\s*dram_bytes_per_launch\s+(\S+)\s+(\S+)\s+([0-9.eE+]+)", line)
            if m and m.group(1) == workload and m.group(2) == kernel_key:
                return float(m.group(3))
    return None


# ---------------------------------------------------------------- clocks

REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
           0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
           0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
           0x100: "display_clock_setting"}


class ClockSampler:
    """NVML samples of SM clock and clock-event reasons in a thread."""

    def __init__(self, local_rank: int, period_s: float = 0.005):
        self.samples, self.reasons, self.period = [], 0, period_s
        self.ok = False
        self.max_mhz = None
        try:
            import pynvml as N
            N.nvmlInit()
            self.N = N
            import torch
            props = torch.cuda.get_device_properties(local_rank)
            h = None
            try:
                bus = "%08x:%02x:%02x.0" % (props.pci_domain_id, props.pci_bus_id, props.pci_device_id)
                h = N.nvmlDeviceGetHandleByPciBusId(bus.encode())
            except Exception:
                vis = os.environ.get("CUDA_VISIBLE_DEVICES")
                idx = int(vis.split(",")[local_rank]) if vis else local_rank
                h = N.nvmlDeviceGetHandleByIndex(idx)
            self.h = h
            self.max_mhz = N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # no NVML: report no clock record
            self.err = str(e)
        self._stop = threading.Event()

    def _run(self):
        N = self.N
        while not self._stop.is_set():
            try:
                self.samples.append(N.nvmlDeviceGetClockInfo(self.h, N.NVML_CLOCK_SM))
                self.reasons |= N.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception:
                pass
            time.sleep(self.period)

    def start(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()

    def stop(self):
        if self.ok:
            self._stop.set()
            self._t.join()

    def record(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [],
                    "samples": 0}
        r = [n for b, n in REASONS.items() if self.reasons & b and b != 0x1]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": r, "samples": len(self.samples)}


# ------------------------------------------------------------- our arm

def run_ours(args, world, rank, local):
    import torch
    import torch.distributed as dist
    from knurlogic_b200 import CapturedBlock, _lib, synth, tensor_split

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    workload = args.workload or "c2"
    cfg = synth.CONFIGS[workload]
    T = cfg.tokens
    tp, dp = split_plan(cfg, world, args.tp)
    # tensor-split groups of tp consecutive ranks; each group (a data-parallel
    # replica) runs the layer on its own batch of tokens
    group = None
    if tp > 1:
        groups = [dist.new_group(list(range(g * tp, (g + 1) * tp))) for g in range(dp)]
        group = groups[rank // tp]
    tp_rank, replica = rank % tp, rank // tp

    # copies of the layer: > 3x L2 of weights streamed per cycle
    per_layer = synth.algorithmic_bytes(cfg, cfg.experts) / tp
    L = max(2, min(16, math.ceil(3 * 126e6 / per_layer) + 1))
    blocks = []
    for i in range(L):
        w = synth.make_weights(cfg, seed=100 + i, device=dev, scales="ones")
        blocks.append(tensor_split.build_block(w, cfg.top_k, rank=tp_rank, n=tp, group=group))
        del w
    x = synth.make_input(cfg, seed=7 + replica, device=dev)
    # one graph per layer copy: block (+ all-reduce under a split)
    outs = [torch.empty(T, cfg.hidden, dtype=torch.bfloat16, device=dev) for _ in range(L)]
    parts = [torch.empty(T, cfg.hidden, dtype=torch.float32, device=dev) for _ in range(L)]

    def step(i):
        b = blocks[i]
        if tp == 1:
            b.forward_into(x, outs[i])
        else:
            b.forward_into(x, parts[i])
            dist.all_reduce(parts[i], group=group)
            outs[i].copy_(parts[i])

    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for i in range(L):
            step(i)
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize(dev)
    graphs = []
    for i in range(L):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step(i)
        graphs.append(g)
    torch.cuda.synchronize(dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    # ---- warm-up, then exactly K timed steps
    for i in range(args.warmup):
        graphs[i % L].replay()
    clocks = ClockSampler(local)
    barrier()
    torch.cuda.synchronize(dev)
    clocks.start()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record()
    for i in range(args.steps):
        graphs[i % L].replay()
    ev1.record()
    torch.cuda.synchronize(dev)
    clocks.stop()
    barrier()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / args.steps
    value = T * dp * args.steps / (ms / 1e3)

    # ---- stage times of the block (events between its kernels), rank 0
    stage = None
    inds_count = None
    if rank == 0 and T <= 2048:      # the timed entry point takes one launch of tokens
        stage, inds_count = stage_profile(blocks, x, cfg, dev, args, tp)

    # ---- end to end through the public captured call, host buffers
    xh = x.cpu().pin_memory()
    yh = torch.empty(T, cfg.hidden, dtype=torch.bfloat16).pin_memory()
    cap = [CapturedBlock(b, T) for b in blocks]
    for i in range(max(3, args.warmup)):
        cap[i % L](xh, out=yh)
    barrier()
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        cap[i % L](xh, out=yh)
    e1.record()
    torch.cuda.synchronize(dev)
    barrier()
    ems = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ems], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ems = float(t.item())
    e2e = {"value": T * dp * args.steps / (ems / 1e3), "unit": UNIT,
           "h2d_bytes_per_step": xh.numel() * xh.element_size(),
           "d2h_bytes_per_step": yh.numel() * yh.element_size()}
    del cap
    # graphs holding NCCL calls go before the process group does
    del graphs
    torch.cuda.synchronize(dev)

    if rank != 0:
        return None
    peak, peak_kind = peaks()
    roof = None
    if T >= 1024:
        # prefill: a contraction; the layer's algorithmic flops over the step
        tpk, tpk_kind = tensor_peak()
        fl = synth.algorithmic_flops(cfg) / tp
        achieved = fl / (ms_per_step / 1e3) / 1e12
        roof = {"bound": "tensor", "kernel": "whole layer (router, experts, shared expert, combine)",
                "achieved": round(achieved, 2), "peak": tpk, "unit": "TFLOP/s",
                "frac": round(achieved / tpk, 4), "peak_source": tpk_kind,
                "algorithmic_flops_per_step": int(fl), "traffic": None}
    elif stage:
        ex_bytes = stage["experts_bytes"]
        achieved = ex_bytes / (stage["experts_ms"] / 1e3) / 1e9
        traffic = traffic_from_profiles(EXPERT_KERNEL, workload)
        roof = {"bound": "hbm",
                "kernel": "routed experts: VQ gate/up + SwiGLU, then VQ down x routing weight",
                "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "kernel_name": EXPERT_KERNEL,
                "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                "algorithmic_bytes_per_launch": int(ex_bytes),
                "traffic": traffic,
                "layer_achieved_gbs": round(stage["layer_bytes"] / (stage["layer_ms"] / 1e3) / 1e9, 1),
                "layer_frac": round(stage["layer_bytes"] / (stage["layer_ms"] / 1e3) / 1e9 / peak, 4)}
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(cfg, workload)
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
        "higher_is_better": True, "scaling": "weak" if dp > 1 or world == 1 else "strong",
        "vs_baseline": None, "dtype": "vq-u8 codes / fp16 dequant / bf16 io",
        "data": "synthetic (seeded; uniform codes, N(0,0.02) codebooks, N(0,1) tokens)",
        "config": {"workload": workload, "tokens": T, "hidden": cfg.hidden,
                   "experts": cfg.experts, "top_k": cfg.top_k, "inter": cfg.inter,
                   "shared_inter": cfg.shared_inter, "codebook": f"{cfg.codebook_size}x{cfg.dim} fp16",
                   "group": cfg.group, "tensor_parallel": tp, "replicas": dp,
                   "parallelism": f"tp{tp}" + (f"xdp{dp}" if dp > 1 else ""), "layer_copies": L,
                   "l2": "inputs larger than L2 (layer copies cycled)",
                   "distinct_experts": inds_count},
        "roofline": roof,
        "stages_ms": stage and {k: round(v, 5) for k, v in stage.items() if k.endswith("_ms")},
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": LAUNCHES_PER_STEP * args.steps,
        "clocks": clocks.record(),
    }
    return line


def split_plan(cfg, world, tp=1):
    """(tensor split, replicas) for `world` GPUs: the requested split of the
    layer (at most the largest power-of-two split that the reference's cut
    rules allow), times independent replicas of that split, each on its own
    tokens."""
    from knurlogic_b200 import tensor_split
    shapes = {"mlp.switch_mlp.gate_proj.codes": (cfg.experts, cfg.inter, cfg.hidden // 4),
              "mlp.switch_mlp.up_proj.codes": (cfg.experts, cfg.inter, cfg.hidden // 4),
              "mlp.switch_mlp.down_proj.codes": (cfg.experts, cfg.hidden, cfg.inter // 4),
              "mlp.switch_mlp.down_proj.vq_scales": (cfg.experts, cfg.hidden, cfg.inter // cfg.group)}
    if cfg.shared_inter:
        shapes["mlp.shared_expert.gate_proj.weight"] = (cfg.shared_inter, cfg.hidden)
        shapes["mlp.shared_expert.down_proj.weight"] = (cfg.hidden, cfg.shared_inter)
    tp = max(1, min(tp, world))
    while tp > 1 and (world % tp or tensor_split.refusals(shapes, tp)):
        tp //= 2
    return tp, world // tp


def stage_profile(blocks, x, cfg, dev, args, world):
    """Per-stage device times (CUDA events between the block's kernels,
    on its stream) averaged over min(K, 500) steps, and the algorithmic
    bytes of the gate/up launch and of the whole layer."""
    import ctypes

    import torch

    from knurlogic_b200 import _lib, synth
    T = x.shape[0]
    L = len(blocks)
    n = min(args.steps, 500)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(n)]
    out = torch.empty(T, cfg.hidden, dtype=torch.float32 if world > 1 else torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream(dev)
    for row in evs:                      # create the events
        for e in row:
            e.record(stream)
    torch.cuda.synchronize(dev)
    descs = [b._desc() for b in blocks]
    wss = [b.workspace(T, dev) for b in blocks]
    odt = _lib.OUT_F32 if world > 1 else _lib.OUT_BF16
    for i in range(n):
        b = i % L
        arr = (ctypes.c_void_p * 5)(*[e.cuda_event for e in evs[i]])
        _lib.call("vqmoe_sparse_moe_block_timed", ctypes.byref(descs[b]), x.data_ptr(), T,
                  out.data_ptr(), odt, wss[b].data_ptr(), wss[b].numel(), stream.cuda_stream,
                  arr, 5)
    torch.cuda.synchronize(dev)
    # events: start | router + routing sort | routed experts (both stages) |
    # join of the shared expert's side stream | combine
    names = ["router_ms", "experts_ms", "shared_wait_ms", "combine_ms"]
    acc = {k: 0.0 for k in names}
    lay = 0.0
    for row in evs[min(10, n - 1):]:
        for j, k in enumerate(names):
            acc[k] += row[j].elapsed_time(row[j + 1])
        lay += row[0].elapsed_time(row[4])
    m = len(evs[min(10, n - 1):])
    st = {k: v / m for k, v in acc.items()}
    st["layer_ms"] = lay / m
    # distinct experts touched: copy 0's routing (every copy has its own
    # router, all drawn from the same distribution)
    inds = routed_experts(blocks[0], x, dev)
    D = len(set(inds))
    H, I, k = cfg.hidden, cfg.inter // world, cfg.top_k
    per = 2 * (I * H // cfg.dim + 2 * I * H // cfg.group)
    # routed-expert launch: codes + scales of the D experts touched (gate,
    # up and down), the three codebooks, x (its fp16 copy) in, the weighted
    # expert outputs [T*k, H] out (the SwiGLU activations between the two
    # stages stay in L2)
    st["experts_bytes"] = (D * per * 3 // 2 + 3 * cfg.codebook_size * cfg.dim * 2 + T * H * 2
                           + T * k * H * 2)
    c2 = synth.MoEConfig("x", cfg.experts, cfg.top_k, H, I, cfg.shared_inter // world, T)
    st["layer_bytes"] = synth.algorithmic_bytes(c2, D)
    return st, D


def routed_experts(block, x, dev):
    import torch

    from knurlogic_b200 import _lib
    T = x.shape[0]
    k = block.top_k
    inds = torch.empty(T, k, dtype=torch.int32, device=dev)
    sc = torch.empty(T, k, dtype=torch.float32, device=dev)
    n = _lib.lib().vqmoe_router_workspace_size(T, block.num_experts)
    ws = torch.empty(n, dtype=torch.uint8, device=dev)
    _lib.call("vqmoe_router", x.data_ptr(), block.gate.weight.data_ptr(), None, T, block.hidden,
              block.num_experts, k, inds.data_ptr(), sc.data_ptr(), None, ws.data_ptr(), n,
              torch.cuda.current_stream(dev).cuda_stream)
    return inds.flatten().tolist()


# ------------------------------------------------------- CPU baselines

def _oracle_inputs(cfg, seed=100):
    import numpy as np

    from knurlogic_b200 import synth
    from oracle import moe_ref as R
    w = synth.make_weights(cfg, seed=seed, device="cpu", scales="ones")
    x = synth.make_input(cfg, seed=7, device="cpu")

    def n(t):
        return t.float().numpy() if t.dtype in (__import__("torch").bfloat16,
                                                  __import__("torch").float16) else t.numpy()
    p = {"router": n(w["mlp.gate.weight"])}
    for name, key in (("gate_proj", "gate"), ("up_proj", "up"), ("down_proj", "down")):
        q = f"mlp.switch_mlp.{name}."
        p[key] = R.LazyVQ(n(w[q + "codes"]), n(w[q + "codebook"]), n(w[q + "vq_scales"]), cfg.group)
    if cfg.shared_inter:
        p["shared_gate"] = n(w["mlp.shared_expert.gate_proj.weight"])
        p["shared_up"] = n(w["mlp.shared_expert.up_proj.weight"])
        p["shared_down"] = n(w["mlp.shared_expert.down_proj.weight"])
        p["shared_expert_gate"] = n(w["mlp.shared_expert_gate.weight"])
    return n(x), p


def cpu_baseline(cfg, workload):
    """The oracle on this host: one full block call (a bounded sample)."""
    from oracle import cpu_baseline as C
    x, p = _oracle_inputs(cfg)
    sec, n = C.time_block(x, p, cfg.top_k, vq=True)
    return {"value": round(x.shape[0] / sec, 2), "unit": UNIT, "cores": n, "kind": "port",
            "sample": f"one full {workload} block call ({x.shape[0]} tokens), numpy oracle, "
                      f"experts on {n} threads ({sec:.2f} s)"}


def run_reference(args, world, rank):
    """The reference arm: the oracle port on all host threads, K steps."""
    from concurrent.futures import ThreadPoolExecutor

    import numpy as np

    from knurlogic_b200 import synth
    from oracle import cpu_baseline as C
    workload = args.workload or "c2"
    cfg = synth.CONFIGS[workload]
    tp, dp = split_plan(cfg, world, args.tp)
    x, p = _oracle_inputs(cfg)
    n = C.threads()
    from oracle import moe_ref as R
    inds, _, _ = R.router(x, p["router"], cfg.top_k)
    routed = np.unique(inds)
    D = len(routed)
    budget = 120.0 / max(1, args.steps + args.warmup)     # seconds per step
    with ThreadPoolExecutor(n) as pool:
        # calibrate: seconds per expert with n experts in flight
        t0 = time.perf_counter()
        C.block(x, p, cfg.top_k, True, pool, experts=routed[:n])
        per_expert = (time.perf_counter() - t0) / n
        m = int(max(1, min(D, budget / max(per_expert, 1e-6))))
        cursor = 0
        done_tokens, secs = 0.0, 0.0
        for i in range(args.warmup + args.steps):
            sel = np.take(routed, np.arange(cursor, cursor + m) % D)
            cursor = (cursor + m) % D
            t0 = time.perf_counter()
            got, _ = C.block(x, p, cfg.top_k, True, pool, experts=sel)
            dt = time.perf_counter() - t0
            if i >= args.warmup:
                secs += dt
                done_tokens += x.shape[0] * got / D
    value = done_tokens / secs
    sample = (f"per step {m} of the {D} routed experts of one {workload} block call "
              f"({x.shape[0]} tokens; router included), rescaled by its share of the "
              f"layer's expert work; numpy oracle on {n} threads")
    return {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "impl": "reference",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1e3 * secs / args.steps, 3), "higher_is_better": True,
            "scaling": "weak" if dp > 1 or world == 1 else "strong", "vs_baseline": None,
            "dtype": "vq-u8 codes / fp16 dequant / bf16 io", "data": "synthetic (seeded)",
            "config": {"workload": workload, "tokens": cfg.tokens, "tensor_parallel": tp, "replicas": dp},
            "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": n, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def main():
    args = parse()
    world, rank, local = dist_env()
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args, world, rank)), flush=True)
        return 0
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    try:
        line = run_ours(args, world, rank, local)
    finally:
        if world > 1:
            dist.destroy_process_group()
    if rank == 0 and line is not None:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
