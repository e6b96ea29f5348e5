"""Benchmark of the VQ-MoE expert layer on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c1|c2|c3|c4] [--tp S]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N \
        --master-addr 127.0.0.1 --master-port P bench.py --gpus N ...

Metric: VQ-MoE layer tokens/s, with the dominant kernel's
HBM GB/s as a fraction of the measured roofline.

A step is one call of the Qwen3.5-MoE sparse block (router, fused VQ
gate/up + SwiGLU, VQ down, shared expert, combine) over one batch of
synthetic tokens.
* One GPU: configuration c2 (H 2048, 128 experts top-8, I 768 + shared 768,
  64 tokens = 16 sequences x (1 + 3 MTP drafts)), the configuration the
  decode metric is quoted on. The line also carries secondary figures: the
  c3 prefill step (4096 tokens, Zipf 1.1) with the tcgen05 grouped GEMM's
  own duration and tensor roofline, and c4 unsplit on one GPU.
* N GPUs: the tensor-split block the baseline names for 2/4/8 B200 (c4:
  H 4096, 256 experts top-8, I 1536, 256 tokens), split N ways -- gate/up
  cut on I, down on I, float32 partials all-reduced over NCCL and rounded
  once (strong scaling: the same 256 tokens at every N). The line carries
  the all-reduce's share of the step and, as a secondary figure, N
  independent c2 replicas. `--workload` / `--tp` pick any other plan.

Inputs larger than L2: the timed loop cycles over several independently
seeded copies of the layer (> 3x the 126 MB L2 in total), so every step
streams its experts from HBM, as consecutive layers of a model do.
`value` times CUDA-graph replays of the block with the input resident in
HBM; `e2e` times the public captured call (`CapturedBlock`) with the input
copied from pinned host memory and the output read back every step.

--impl reference times the CPU restatement of the reference semantics
(`oracle/`; the reference's own MLX code cannot run here) on all host
threads, on the same workload; every step is one whole block call.
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


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", default=None,
                    help="c1..c4 (default: c2 on one GPU, c4 split N ways on N GPUs)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decoder", action="store_true",
                    help="skip the C5 decoder figure (build, two 8192-token prefills of 32 sequences)")
    ap.add_argument("--decoder-tokens", type=int, default=17,
                    help="generated tokens timed per sequence in the C5 decoder figure")
    ap.add_argument("--no-secondary", action="store_true",
                    help="skip the secondary figures (prefill c3, c4 unsplit, c2 replicas)")
    ap.add_argument("--tp", type=int, default=None,
                    help="tensor split of the layer (N / tp independent replicas)")
    ap.add_argument("--tp-reduce", choices=("p2p", "nccl"), default="p2p",
                    help="the split's reduction: the combine + float32 sum in one kernel over NVLink peer "
                         "memory (default), or a float32 NCCL all-reduce after the combine")
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

def launches_per_call(cfg, T):
    """Our kernels per block call: router logits + routing (one kernel up
    to 512 tokens, a top-k and a sort kernel beyond), the shared expert's
    two matmuls, the input permute of the prefill path, the routed experts
    (one launch), the combine -- per 2048-token chunk."""
    from knurlogic_b200.synth import MoEConfig  # noqa: F401
    n = 0
    for t0 in range(0, T, 2048):
        t = min(2048, T - t0)
        n += 2 + (1 if t > 512 else 0) + (2 if cfg.shared_inter else 0) + 1 + 1
        if t * cfg.top_k >= 32 * cfg.experts:
            n += 1
    return n


def build_copies(cfg, tp, tp_rank, group, dev, seed0=100, tp_reduce="p2p"):
    """Independently seeded copies of the layer (this rank's cut of each),
    more than 3x the 126 MB L2 of weights in total."""
    from knurlogic_b200 import synth, tensor_split
    per_layer = synth.algorithmic_bytes(cfg, cfg.experts) / tp
    L = max(2, min(16, math.ceil(3 * 126e6 / per_layer) + 1))
    blocks = []
    for i in range(L):
        w = synth.make_weights(cfg, seed=seed0 + i, device=dev, scales="ones")
        blocks.append(tensor_split.build_block(w, cfg.top_k, rank=tp_rank, n=tp, group=group,
                                               tp_reduce=tp_reduce))
        del w
    return blocks


class Graphs:
    """One CUDA graph per layer copy: the block, with under a split its
    reduction -- the peer-memory kernel inside the block call, or the float32
    NCCL all-reduce of the partials and the bf16 rounding."""

    def __init__(self, blocks, x, tp, group, dev):
        import torch
        import torch.distributed as dist
        T, H = x.shape
        self.L = len(blocks)
        self.outs = [torch.empty(T, H, dtype=torch.bfloat16, device=dev) for _ in blocks]
        self.parts = [torch.empty(T, H, dtype=torch.float32, device=dev) for _ in blocks]

        def step(i):
            b = blocks[i]
            if tp == 1 or b.tp_reduce == "p2p":
                b.forward_into(x, self.outs[i])
            else:
                b.forward_into(x, self.parts[i])
                dist.all_reduce(self.parts[i], group=group)
                self.outs[i].copy_(self.parts[i])
        self.step = step
        for b in blocks:                         # collectives of the split, before any capture
            if tp > 1 and b.tp_reduce == "p2p":
                b.tp_buffers(x.shape[0], dev)
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for i in range(self.L):
                step(i)
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        self.graphs = []
        for i in range(self.L):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                step(i)
            self.graphs.append(g)
        torch.cuda.synchronize(dev)

    def replay(self, i):
        self.graphs[i % self.L].replay()


def timed(fn, steps, warmup, world, local, dev, clocks=None):
    """ms for exactly `steps` calls of fn(i) after `warmup` untimed ones:
    CUDA events on the current stream, a barrier and a synchronize on both
    sides, the max over ranks."""
    import torch
    import torch.distributed as dist

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
    for i in range(warmup):
        fn(i)
    barrier()
    torch.cuda.synchronize(dev)
    if clocks:
        clocks.start()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        fn(i)
    e1.record()
    torch.cuda.synchronize(dev)
    if clocks:
        clocks.stop()
    barrier()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def default_plan(args, world):
    """(workload, requested tensor split): c2 on one GPU (the configuration
    the decode metric is quoted on); on N GPUs the tensor-split block the
    baseline names for 2/4/8 B200 (c4, split N ways)."""
    workload = args.workload or ("c4" if world > 1 else "c2")
    tp = args.tp if args.tp is not None else (world if world > 1 and workload == "c4" else 1)
    return workload, tp


def split_groups(world, tp, rank):
    import torch.distributed as dist
    if tp == 1:
        return None
    dp = world // tp
    groups = [dist.new_group(list(range(g * tp, (g + 1) * tp))) for g in range(dp)]
    return groups[rank // tp]


def tp_share(blocks, x, group, world, local, dev, n):
    """The NCCL reduction's share of a tensor-split step: per step, the
    block (float32 partial) and the float32 all-reduce replayed as separate
    graphs with CUDA events between them, averaged over n steps, max over
    ranks. (The peer-memory path has no separate reduction to time: its
    combine and reduction are one kernel, timed by `tp_reduce_share`.)"""
    import torch
    import torch.distributed as dist
    T, H = x.shape
    part = torch.empty(T, H, dtype=torch.float32, device=dev)
    L = len(blocks)
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for b in blocks:
            b.forward_into(x, part)
        dist.all_reduce(part, group=group)
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize(dev)
    gb = []
    for b in blocks:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            b.forward_into(x, part)
        gb.append(g)
    ga = torch.cuda.CUDAGraph()
    with torch.cuda.graph(ga):
        dist.all_reduce(part, group=group)
    torch.cuda.synchronize(dev)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(n)]
    dist.barrier(device_ids=[local])
    for i in range(n):
        evs[i][0].record()
        gb[i % L].replay()
        evs[i][1].record()
        ga.replay()
        evs[i][2].record()
    torch.cuda.synchronize(dev)
    rows = evs[min(10, n - 1):]
    blk = sum(r[0].elapsed_time(r[1]) for r in rows) / len(rows)
    ar = sum(r[1].elapsed_time(r[2]) for r in rows) / len(rows)
    t = torch.tensor([blk, ar], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    blk, ar = (float(v) for v in t.tolist())
    del ga, gb
    torch.cuda.synchronize(dev)
    return {"block_ms": round(blk, 5), "allreduce_ms": round(ar, 5),
            "allreduce_share": round(ar / (blk + ar), 4), "allreduce_bytes": T * H * 4,
            "note": "block and float32 all-reduce replayed as separate graphs, CUDA events between them; "
                    "the all-reduce time includes waiting for the slowest rank's block"}


def tp_reduce_share(blocks, x, tp, local, dev, n):
    """The split block's stages and the reduction's share. Per step the same
    layer copy runs twice: the unsplit entry into bf16 (the whole router,
    its combine kernel, no reduction) and the split entry with events
    between its stages (router on T/n tokens + routing exchange + sort,
    routed experts, side-stream join, the fused combine + float32 reduction
    over NVLink peer memory). Averages over n steps, max over ranks (every
    rank makes the same calls)."""
    import ctypes

    import torch
    import torch.distributed as dist

    from knurlogic_b200 import _lib
    T = x.shape[0]
    L = len(blocks)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(7)] for _ in range(n)]
    stream = torch.cuda.current_stream(dev)
    for row in evs:
        for e in row:
            e.record(stream)
    torch.cuda.synchronize(dev)
    out = torch.empty(T, x.shape[1], dtype=torch.bfloat16, device=dev)
    descs = [b._desc() for b in blocks]
    wss = [b.workspace(T, dev) for b in blocks]
    tps = [b.tp_buffers(T, dev) for b in blocks]
    dist.barrier(device_ids=[local])
    for i in range(n):
        b = i % L
        evs[i][0].record(stream)
        _lib.call("vqmoe_sparse_moe_block", ctypes.byref(descs[b]), x.data_ptr(), T, out.data_ptr(),
                  _lib.OUT_BF16, wss[b].data_ptr(), wss[b].numel(), stream.cuda_stream)
        arr = (ctypes.c_void_p * 5)(*[e.cuda_event for e in evs[i][1:6]])
        _lib.call("vqmoe_sparse_moe_block_tp_timed", ctypes.byref(descs[b]), ctypes.byref(tps[b]), x.data_ptr(), T,
                  out.data_ptr(), wss[b].data_ptr(), wss[b].numel(), stream.cuda_stream, arr, 5)
    torch.cuda.synchronize(dev)
    rows = evs[min(10, n - 1):]

    def mean(a, b):
        return sum(r[a].elapsed_time(r[b]) for r in rows) / len(rows)

    vals = [mean(0, 1), mean(1, 5), mean(1, 2), mean(2, 3), mean(3, 4), mean(4, 5)]
    t = torch.tensor(vals, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    plain, call, router, experts, wait, reduce = (float(v) for v in t.tolist())
    return {"block_ms": round(plain, 5), "split_call_ms": round(call, 5),
            "split_stages_ms": {"router_exchange_sort_ms": round(router, 5), "experts_ms": round(experts, 5),
                                "shared_wait_ms": round(wait, 5), "fused_reduce_ms": round(reduce, 5)},
            "reduce_share": round(reduce / call, 4),
            "nvlink_bytes_per_rank": 2 * T * x.shape[1] * 2 * (tp - 1) // tp,
            "note": "unsplit entry (whole router, combine kernel, no reduction) against the split entry's stages; "
                    "the fused reduce includes waiting for the slowest rank"}


def decoder_profile(dev, gen, batch=32, prompt=8192, k=3):
    """The baseline's C5 decoder (48 layers, hidden 4096, GQA 32/4 x 128,
    256 VQ experts top-8 + a shared expert, vocab 151936, a one-layer MTP
    head drafting 3) with random-init weights on ONE B200: 32 sequences of
    8192 uniform random prompt tokens, then the first `gen` generated tokens
    by plain greedy decoding and by MTP drafting, each decode step a CUDA
    graph replay; device times by CUDA events. Random weights make the
    head's drafts unrelated to the trunk's choices (acceptance near 0), so
    the MTP figure is the cost of a verify step, not a speed-up."""
    import torch

    from knurlogic_b200 import decoder
    cfg = decoder.CONFIGS["c5"]
    torch.cuda.empty_cache()
    model = decoder.build(cfg, seed=1, device=dev)
    g = torch.Generator(device=dev).manual_seed(2)
    prompts = torch.randint(0, cfg.vocab, (batch, prompt), generator=g, device=dev)
    decoder.generate_greedy(model, prompts[:, :64], 4, graphs=True)          # warm-up
    decoder.generate_mtp(model, prompts[:, :64], 4, k=k, graphs=True)
    sg = {}
    plain = decoder.generate_greedy(model, prompts, gen, graphs=True, stats=sg)
    toks, sm = decoder.generate_mtp(model, prompts, gen, k=k, graphs=True)
    r = {"workload": "c5", "layers": cfg.layers, "hidden": cfg.hidden, "heads": f"{cfg.heads}/{cfg.kv_heads}x{cfg.head_dim}",
         "experts": f"{cfg.moe.experts} top-{cfg.moe.top_k}, I {cfg.moe.inter}, shared {cfg.moe.shared_inter}",
         "vocab": cfg.vocab, "sequences": batch, "prompt_tokens": prompt, "generated_tokens_timed": gen,
         "n_gpus": 1, "weights_gb": round(torch.cuda.memory_allocated(dev) / 1e9, 1),
         "prefill_ms": round(sg["prefill_ms"], 1),
         "prefill_tokens_per_s": round(batch * prompt / (sg["prefill_ms"] / 1e3), 1),
         "greedy_ms_per_step": round(sg["decode_ms"] / (gen - 1), 3),
         "greedy_tokens_per_s": round(batch * (gen - 1) / (sg["decode_ms"] / 1e3), 1),
         "mtp_steps": sm["steps"], "mtp_ms_per_step": round(sm["decode_ms"] / max(sm["steps"], 1), 3),
         "mtp_tokens_per_s": round(batch * (gen - 1) / (sm["decode_ms"] / 1e3), 1),
         "mtp_acceptance": round(sm["accepted"] / max(sm["drafted"], 1), 4),
         "mtp_tokens_equal_greedy": bool(torch.equal(plain, toks)),
         "note": "one B200 (the baseline's C5 names 8 at TP=8); the first tokens of the 512; random-init weights"}
    del model, prompts
    torch.cuda.empty_cache()
    return r


def quick_value(workload, tp, rank, world, local, dev, steps, warmup):
    """tokens/s of `workload` split tp ways (world / tp replicas), graph
    replays over layer copies: a secondary figure beside the headline."""
    from knurlogic_b200 import synth
    cfg = synth.CONFIGS[workload]
    tp, dp = split_plan(cfg, world, tp)
    group = split_groups(world, tp, rank)
    blocks = build_copies(cfg, tp, rank % tp, group, dev, seed0=300)
    x = synth.make_input(cfg, seed=11 + rank // tp, device=dev)
    G = Graphs(blocks, x, tp, group, dev)
    ms = timed(G.replay, steps, warmup, world, local, dev)
    del G, blocks
    return {"workload": workload, "tokens": cfg.tokens, "tensor_parallel": tp, "replicas": dp,
            "value": round(cfg.tokens * dp * steps / (ms / 1e3), 1), "unit": UNIT,
            "ms_per_step": round(ms / steps, 5), "steps": steps}


def quick_value_ep(workload, rank, world, local, dev, steps, warmup):
    """tokens/s of `workload` with its experts split by id over all `world`
    ranks (`expert_split`: whole experts, every rank routes every token, the
    combine over peer memory), graph replays over layer copies: the
    alternative to the tensor split, beside the headline."""
    import math

    import torch.distributed as dist

    from knurlogic_b200 import expert_split, synth
    cfg = synth.CONFIGS[workload]
    shapes = {"mlp.switch_mlp.gate_proj.codes": (cfg.experts, cfg.inter, cfg.hidden // 4),
              "mlp.switch_mlp.gate_proj.codebook": (cfg.codebook_size, cfg.dim),
              "mlp.gate.weight": (cfg.experts, cfg.hidden)}
    why = expert_split.refusals(shapes, world)
    if why:
        return {"workload": workload, "refused": "; ".join(why)}
    per_layer = synth.algorithmic_bytes(cfg, cfg.experts) / world
    L = max(2, min(16, math.ceil(3 * 126e6 / per_layer) + 1))
    blocks = []
    for i in range(L):
        w = synth.make_weights(cfg, seed=300 + i, device=dev, scales="ones")
        blocks.append(expert_split.build_block(w, cfg.top_k, rank, world, dist.group.WORLD))
        del w
    x = synth.make_input(cfg, seed=11, device=dev)
    G = Graphs(blocks, x, world, dist.group.WORLD, dev)
    ms = timed(G.replay, steps, warmup, world, local, dev)
    del G, blocks
    return {"workload": workload, "tokens": cfg.tokens, "expert_parallel": world, "replicas": 1,
            "value": round(cfg.tokens * steps / (ms / 1e3), 1), "unit": UNIT,
            "ms_per_step": round(ms / steps, 5), "steps": steps}


def prefill_profile(dev, steps=100, warmup=5):
    """c3 (4096 prefill tokens, Zipf 1.1) on this GPU: the step time of the
    whole block (graph replays over layer copies, so weights stream from
    HBM), and the tcgen05 grouped GEMM's own duration per 2048-token launch
    (CUDA events around it inside the block, through the timed entry), with
    its tensor roofline against the burst bf16 peak."""
    import ctypes

    import torch

    from knurlogic_b200 import _lib, synth
    cfg = synth.CONFIGS["c3"]
    blocks = build_copies(cfg, 1, 0, None, dev, seed0=200)
    x = synth.make_input(cfg, seed=9, device=dev)
    G = Graphs(blocks, x, 1, None, dev)
    ms = timed(G.replay, steps, warmup, 1, 0, dev)
    del G
    step_ms = ms / steps
    # the grouped GEMM alone, on the first 2048-token launch of the step
    Tc = 2048
    xc = x[:Tc].contiguous()
    n = 60
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(6)] for _ in range(n)]
    out = torch.empty(Tc, cfg.hidden, dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream(dev)
    for row in evs:                      # torch creates an event at its first record
        for e in row:
            e.record(stream)
    torch.cuda.synchronize(dev)
    descs = [b._desc() for b in blocks]
    wss = [b.workspace(Tc, dev) for b in blocks]
    for i in range(n):
        b = i % len(blocks)
        arr = (ctypes.c_void_p * 6)(*[e.cuda_event for e in evs[i]])
        _lib.call("vqmoe_sparse_moe_block_timed", ctypes.byref(descs[b]), xc.data_ptr(), Tc,
                  out.data_ptr(), _lib.OUT_BF16, wss[b].data_ptr(), wss[b].numel(),
                  stream.cuda_stream, arr, 6)
    torch.cuda.synchronize(dev)
    rows = evs[10:]
    k_ms = sum(r[5].elapsed_time(r[2]) for r in rows) / len(rows)
    perm_ms = sum(r[1].elapsed_time(r[5]) for r in rows) / len(rows)
    router_ms = sum(r[0].elapsed_time(r[1]) for r in rows) / len(rows)
    k_flops = 2 * Tc * cfg.top_k * 3 * cfg.inter * cfg.hidden
    tpk, kind = tensor_peak()
    layer_fl = synth.algorithmic_flops(cfg)
    del blocks
    torch.cuda.synchronize(dev)
    return {"workload": "c3", "tokens": cfg.tokens, "steps": steps,
            "ms_per_step": round(step_ms, 5), "value": round(cfg.tokens / (step_ms / 1e3), 1), "unit": UNIT,
            "layer_tflops": round(layer_fl / (step_ms / 1e3) / 1e12, 2),
            "layer_frac": round(layer_fl / (step_ms / 1e3) / 1e12 / tpk, 4),
            "kernel": "expert_prefill_kernel", "kernel_ms": round(k_ms, 5),
            "kernel_flops_per_launch": k_flops,
            "kernel_tflops": round(k_flops / (k_ms / 1e3) / 1e12, 2),
            "kernel_frac": round(k_flops / (k_ms / 1e3) / 1e12 / tpk, 4),
            "peak_tflops": tpk, "peak_source": kind + " (burst)",
            "router_ms_per_launch": round(router_ms, 5), "permute_ms_per_launch": round(perm_ms, 5)}


def run_ours(args, world, rank, local):
    import torch
    import torch.distributed as dist

    from knurlogic_b200 import CapturedBlock, synth

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    workload, tp_req = default_plan(args, world)
    cfg = synth.CONFIGS[workload]
    T = cfg.tokens
    tp, dp = split_plan(cfg, world, tp_req)
    # tensor-split groups of tp consecutive ranks; each group (a data-parallel
    # replica) runs the layer on its own batch of tokens
    group = split_groups(world, tp, rank)
    replica = rank // tp
    blocks = build_copies(cfg, tp, rank % tp, group, dev, tp_reduce=args.tp_reduce)
    L = len(blocks)
    x = synth.make_input(cfg, seed=7 + replica, device=dev)

    # ---- the headline: exactly K graph replays after W warm-up
    G = Graphs(blocks, x, tp, group, dev)
    clocks = ClockSampler(local)
    ms = timed(G.replay, args.steps, args.warmup, world, local, dev, clocks)
    ms_per_step = ms / args.steps
    value = T * dp * args.steps / (ms / 1e3)
    del G
    torch.cuda.synchronize(dev)

    comm = None
    if tp > 1:
        comm = (tp_reduce_share(blocks, x, tp, local, dev, min(args.steps, 200)) if args.tp_reduce == "p2p"
                else tp_share(blocks, x, group, world, local, dev, min(args.steps, 200)))
        comm["reduce"] = args.tp_reduce

    # ---- stage times of the block (events between its kernels), rank 0
    stage, distinct = None, None
    if rank == 0 and T <= 2048:      # the timed entry point takes one launch of tokens
        stage, distinct = stage_profile(blocks, x, cfg, dev, args, tp)
    if world > 1:
        dist.barrier(device_ids=[local])

    # ---- end to end through the public captured call, host buffers
    xh = x.cpu().pin_memory()
    yh = torch.empty(T, cfg.hidden, dtype=torch.bfloat16).pin_memory()
    cap = [CapturedBlock(b, T) for b in blocks]
    ems = timed(lambda i: cap[i % L](xh, out=yh), args.steps, max(3, args.warmup), world, local, dev)
    cap[0].check_status()
    e2e = {"value": T * dp * args.steps / (ems / 1e3), "unit": UNIT,
           "h2d_bytes_per_step": xh.numel() * xh.element_size(),
           "d2h_bytes_per_step": yh.numel() * yh.element_size()}
    # graphs holding NCCL calls go before the process group does
    del cap, blocks
    torch.cuda.synchronize(dev)

    # ---- secondary figures beside the headline
    secondary = {}
    if not args.no_secondary:
        if world == 1 and workload == "c2":
            secondary["prefill"] = prefill_profile(dev)
            secondary["c4_tp1"] = quick_value("c4", 1, rank, world, local, dev, 100, 5)
            if not args.no_decoder:
                secondary["decoder_c5"] = decoder_profile(dev, args.decoder_tokens)
        elif world > 1 and tp > 1:
            secondary["c2_replicas"] = quick_value("c2", 1, rank, world, local, dev, 200, 10)
            if workload == "c4" and tp == world:
                secondary["c4_expert_split"] = quick_value_ep("c4", rank, world, local, dev, 200, 10)

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
        "higher_is_better": True, "scaling": "weak" if tp == 1 else "strong",
        "vs_baseline": None, "dtype": "vq-u8 codes / fp16 dequant / bf16 io",
        "data": "synthetic (seeded; uniform codes, N(0,0.02) codebooks, N(0,1) tokens)",
        "config": {"workload": workload, "tokens": T, "hidden": cfg.hidden,
                   "experts": cfg.experts, "top_k": cfg.top_k, "inter": cfg.inter,
                   "shared_inter": cfg.shared_inter, "codebook": f"{cfg.codebook_size}x{cfg.dim} fp16",
                   "group": cfg.group, "tensor_parallel": tp, "replicas": dp,
                   "parallelism": f"tp{tp}" + (f"xdp{dp}" if dp > 1 else ""), "layer_copies": L,
                   "l2": "inputs larger than L2 (layer copies cycled)",
                   "distinct_experts": distinct},
        "roofline": roof,
        "stages_ms": stage and {k: round(v, 5) for k, v in stage.items() if k.endswith("_ms")},
        "tensor_split": comm,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": launches_per_call(cfg, T) * args.steps,
        "clocks": clocks.record(),
        "secondary": secondary or None,
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
    """The oracle on this host: two whole block calls, the second timed."""
    from oracle import cpu_baseline as C
    x, p = _oracle_inputs(cfg)
    C.time_block(x, p, cfg.top_k, vq=True)
    sec, n = C.time_block(x, p, cfg.top_k, vq=True)
    return {"value": round(x.shape[0] / sec, 2), "unit": UNIT, "cores": n, "kind": "port",
            "sample": f"one whole {workload} block call ({x.shape[0]} tokens: router, every routed expert, "
                      f"combine, shared expert), numpy oracle, experts on {n} worker threads, BLAS held "
                      f"to one thread each ({sec:.2f} s)"}


def run_reference(args, world, rank):
    """The reference arm: the oracle port (the CPU restatement of the
    reference's block) on all host threads. Every step is one whole block
    call on the arm's workload -- router, every routed expert, combine and
    shared expert. When K + W such calls would not finish within about two
    minutes, only the first steps that fit are timed (at least 3; warm-up
    cut to one call), and the line says how many."""
    from knurlogic_b200 import synth
    from oracle import cpu_baseline as C
    workload, tp_req = default_plan(args, world)
    cfg = synth.CONFIGS[workload]
    tp, dp = split_plan(cfg, world, tp_req)
    x, p = _oracle_inputs(cfg)
    n = C.threads()
    budget = 120.0
    with C.pool_of(n) as pool:
        t0 = time.perf_counter()
        C.block(x, p, cfg.top_k, True, pool)          # first warm-up call, also the estimate
        est = time.perf_counter() - t0
        fit = int(budget / max(est, 1e-6))
        if args.warmup + args.steps <= fit:
            warm, steps = args.warmup, args.steps
        else:
            warm, steps = min(args.warmup, 1), max(3, min(args.steps, fit))
        for _ in range(max(0, warm - 1)):
            C.block(x, p, cfg.top_k, True, pool)
        t0 = time.perf_counter()
        for _ in range(steps):
            C.block(x, p, cfg.top_k, True, pool)
        secs = time.perf_counter() - t0
    T = x.shape[0]
    value = T * steps / secs
    sample = (f"every step one whole {workload} block call ({T} tokens: router, every routed expert, "
              f"combine{', shared expert' if cfg.shared_inter else ''}), numpy oracle, experts on {n} "
              f"worker threads, BLAS held to one thread each; {steps} of the {args.steps} steps timed")
    return {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "impl": "reference",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1e3 * secs / steps, 3), "higher_is_better": True,
            "scaling": "weak" if tp == 1 else "strong", "vs_baseline": None,
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
