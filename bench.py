#!/usr/bin/env python
"""PopKV decode-step benchmark on B200 (the benchmark configuration's config 1 by default).

A step is one single-layer PopKV decode step of the retrieval path: query
encode + popcount score over the whole context + top-k with the current slot
reserved + 256-token split attention + merge (the reference's decode branch,
popkv.py:1076-1115).  Default workload: batch 1, 32 query / 8 KV heads,
head_dim 128, context 32768, budget 4096, PopKV-Q preset (token group 128,
dim group 16), bf16 K/V/Q, seeded synthetic inputs (popkv_b200.workloads).

With N GPUs (torchrun) the KV heads -- cache, metadata, query heads -- are
sharded across ranks and each step ends with the merge fused with the
all-gather over NVLink peer memory (``--gather nccl``: an NCCL all-gather);
the total work is fixed: strong scaling.

Timing: W warm-up steps, then exactly K steps between a barrier +
synchronize.  The steps run as the layers of one decoded token do in the
decoder's per-token graph: ``--chain`` (8) consecutive steps, each on the next
layer copy, captured in one CUDA graph; each replay is bracketed by CUDA
events on the launching stream, the device times are summed over K steps and
the max over ranks is reported.  ``single_step_graph`` repeats the
measurement with one graph launch per step.  L2: steps cycle over enough
copies of the layer (cache + metadata) that the working set of consecutive
steps exceeds the 126 MB L2.

``--impl reference`` times the reference's CPU implementation of the path
(the C restatement in oracle/, OpenMP over all host cores) on the same
workload; the other ranks of a multi-GPU launch exit without work.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

METRIC = "decode ms/token (score+top-k+sparse attn), one layer"
UNIT = "ms"
# The reference's published PG19 decode breakdown (PopKV-Q at 32K, budget
# 4096, per token over its 30 sparse layers; score_comparison.csv and
# report.md of its five-methods run): score 1.365 + top-k 1.814 + partial
# 3.600 + merge 0.143 = 6.922 ms -> per layer.
PUBLISHED_MS_PER_LAYER = (1.365 + 1.814 + 3.600 + 0.143) / 30.0

# DRAM traffic per launch (dram__bytes_read.sum + dram__bytes_write.sum) of the
# step's kernels at the default workload, taken from one ncu capture of each
# kernel at config 1 (not measured by this script, which runs without ncu).
NCU_TRAFFIC_CONFIG1 = {
    "score_fused": 16_829_952,
    "attn_partial": 55_847_680 + 448_768,
    "topk": 2_134_016,
    "prepack": 67_169_024 + 4_106_752,
}
DEFAULT_WORKLOAD = {"context": 32768, "budget": 4096, "batch": 1, "preset": "popkv-q"}
L2_BYTES = 126 * 1024 * 1024


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10000)
    p.add_argument("--warmup", type=int, default=50)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--context", type=int, default=32768)
    p.add_argument("--budget", type=int, default=4096)
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--preset", choices=("popkv-q", "popkv-s", "popkv-normal"), default="popkv-q")
    p.add_argument("--no-graph", action="store_true", help="launch eagerly instead of a CUDA graph")
    p.add_argument("--select", choices=("auto", "hist", "radix"), default="radix",
                   help="top-k path of the step (hist: score kernel builds the first radix histogram)")
    p.add_argument("--gather", choices=("peer", "nccl"), default="peer",
                   help="N>1: merge fused with the all-gather over NVLink peer memory, or NCCL all-gather")
    p.add_argument("--split", type=int, default=256, help="selected slots per attention partial")
    p.add_argument("--chunks", type=int, default=1,
                   help="KV-head chunks pipelined on forked streams inside the step graph")
    p.add_argument("--chain", type=int, default=8,
                   help="layer steps per captured CUDA graph in the timed loop, each on the next layer copy "
                        "(as the layers of one decoded token run in the decoder's graph); 1: one graph "
                        "launch per step")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU baseline sample budget")
    p.add_argument("--stage-reps", type=int, default=50)
    p.add_argument("--mlp-parallel", choices=("replicated", "tensor"), default="replicated",
                   help="--model on several GPUs: replicated o_proj/MLP (one all-gather per layer) or "
                        "tensor-parallel (two all-reduces per layer)")
    p.add_argument("--all-reduce", choices=("peer", "nccl"), default="peer",
                   help="--mlp-parallel tensor: sum the partial products with popkv_peer_sum over NVLink peer "
                        "memory or with an NCCL all-reduce")
    p.add_argument("--no-model", action="store_true",
                   help="skip the full-model decode measurement that a 1-GPU default run adds")
    p.add_argument("--model", action="store_true",
                   help="full 32-layer Llama-3.1-8B-shaped greedy decode (config 2) instead of one layer")
    p.add_argument("--model-method", choices=("popkv-s", "popkv-q", "popkv-normal", "full"), default="popkv-s")
    p.add_argument("--gen-steps", type=int, default=256, help="timed greedy decode steps (--model)")
    p.add_argument("--prefill", choices=("model", "synthetic"), default="model",
                   help="--model: run the prefix through the model, or fill the caches with the synthetic "
                        "key/value distributions (config 4 sizes)")
    p.add_argument("--products", action="store_true",
                   help="time the decode step's weight-streaming products against cuBLAS at the model's shapes")
    p.add_argument("--product-shape", default=None,
                   help="ROWSxK: one product shape only, 3 launches each (for an ncu capture)")
    return p.parse_args(argv)


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------

def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def init_dist(world: int, local: int):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return dist if world > 1 else None


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------

class ClockSampler:
    """Samples nvidia-smi SM clocks and throttle reasons every 100 ms in the background."""

    FIELDS = ("clocks.sm", "clocks.max.sm", "power.draw", "clocks_event_reasons.active",
              "clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
              "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.samples: list[tuple[float, list[str]]] = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu_index), f"--query-gpu={','.join(self.FIELDS)}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return self
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) == len(self.FIELDS):
                self.samples.append((time.time(), parts))

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)

    def summary(self, t0: float, t1: float) -> dict:
        inside = [s for t, s in self.samples if t0 <= t <= t1]
        window = "timed"
        if not inside:
            inside = [s for t, s in self.samples if t <= t1][-3:]
            window = "nearest"
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        mhz = [float(s[0]) for s in inside if s[0].replace(".", "").isdigit()]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for s in inside for n, v in zip(names, s[4:8]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(mhz) if mhz else None,
                "sm_max_mhz": float(inside[0][1]) if inside[0][1].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(inside), "window": window}


def physical_gpu_index(local: int) -> int:
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    if visible:
        items = [x.strip() for x in visible.split(",") if x.strip()]
        if local < len(items) and items[local].isdigit():
            return int(items[local])
    return local


# ---------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------

def make_layer(args, world, rank, device):
    """One layer's shard for this rank: cache/metadata/query heads of its KV heads."""
    import numpy as np
    import torch
    from popkv_b200 import popkv as P
    from popkv_b200.workloads import decode_inputs, to_bf16_bits

    q_heads, kv_heads = 32, 8
    if kv_heads % world:
        raise SystemExit(f"--gpus {world} must divide the 8 KV heads")
    kv_local, q_local = kv_heads // world, q_heads // world
    x = decode_inputs(batch=args.batch, context=args.context, seed=0, dtype="bf16")
    ks, qs = slice(rank * kv_local, (rank + 1) * kv_local), slice(rank * q_local, (rank + 1) * q_local)

    def dev(a):
        bits = to_bf16_bits(np.ascontiguousarray(a))
        return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).to(device)

    layer = {
        "keys": dev(x.keys[:, ks]), "values": dev(x.values[:, ks]), "queries": dev(x.queries[:, qs]),
        "cur_k": dev(x.current_keys[:, ks]), "cur_v": dev(x.current_values[:, ks]),
        "mapping": torch.arange(q_local, device=device, dtype=torch.int64) // (q_heads // kv_heads),
        "q_local": q_local, "kv_local": kv_local, "host": x, "kv_slice": ks, "q_slice": qs,
    }
    tg, g = P.POPKV_PRESETS[args.preset]
    layer["tg"], layer["g"] = tg, g
    return layer


def fold_batch(layer, batch: int):
    """Independent sequences as extra heads: [B, KVH, ...] -> [1, B*KVH, ...].

    Each sequence has its own cache and metadata (config 3's batch); the step
    then runs as batch 1 over B times the heads, with the consecutive GQA
    mapping of every sequence's query heads onto its own KV heads.
    """
    import torch
    out = dict(layer)
    kvl, ql = layer["kv_local"], layer["q_local"]
    out["keys"] = layer["keys"].reshape(1, batch * kvl, *layer["keys"].shape[2:])
    out["values"] = layer["values"].reshape(1, batch * kvl, *layer["values"].shape[2:])
    out["queries"] = layer["queries"].reshape(1, batch * ql, 128)
    out["cur_k"] = layer["cur_k"].reshape(1, batch * kvl, 128)
    out["cur_v"] = layer["cur_v"].reshape(1, batch * kvl, 128)
    out["mapping"] = torch.arange(batch * ql, device=layer["mapping"].device, dtype=torch.int64) // (ql // kvl)
    out["q_local"], out["kv_local"] = batch * ql, batch * kvl
    return out


def build_steps(args, layer, copies: int, gather=None):
    """`copies` independent layer instances (own cache + metadata), each a captured step."""
    import torch
    from popkv_b200 import popkv as P
    from popkv_b200.decode import SparseAttentionStep
    steps = []
    for _ in range(copies):
        keys = layer["keys"].clone()
        values = layer["values"].clone()
        B = args.batch
        # One cache per step: a batch of independent sequences arrives folded into heads.
        caches = []
        for b in range(B):
            caches.append(P.build_popkv_cache(keys[b], group_size=layer["tg"], dim_group_size=layer["g"],
                                              reserve_tokens=0))
        step = SparseAttentionStep(caches[0], keys, values, layer["mapping"], budget=args.budget,
                                   q_dtype=torch.bfloat16, batch=B, use_graph=not args.no_graph,
                                   select=args.select, chunks=args.chunks, gather=gather,
                                   split_tokens=args.split)
        step.queries.copy_(layer["queries"])
        step.current_keys.copy_(layer["cur_k"])
        step.current_values.copy_(layer["cur_v"])
        steps.append(step)
    return steps


def layer_bytes(args, layer) -> int:
    T, D = args.context, 128
    kv = layer["kv_local"]
    reps = 128 // layer["g"]
    return args.batch * kv * T * (2 * D * 2 + 32 + 4 * reps)


def union_rows(step) -> int:
    """Distinct cached rows the step's query heads selected, summed over (batch, KV head).

    The query heads of one KV head read the union of their selections from
    HBM once (L2 serves the repeats), so the attention's algorithmic bytes
    count each distinct row once.  The current token's slot is not a cached row.
    """
    import torch
    idx = step.indices
    B, QH, _ = idx.shape
    group = QH // step.kv_heads
    rows = 0
    for b in range(B):
        for h in range(step.kv_heads):
            sel = idx[b, h * group:(h + 1) * group].reshape(-1)
            rows += int(torch.unique(sel[sel < step.prefix_tokens]).numel())
    return rows


def algorithmic_bytes(args, layer, rows: int) -> dict:
    """Bytes each stage must move once (no re-reads), per step of this rank.

    `rows` = distinct selected cached rows (union over each KV head's query heads).
    """
    T, D, B = args.context, 128, args.batch
    kv, qh = layer["kv_local"], layer["q_local"]
    reps = 128 // layer["g"]
    k = min(args.budget - 1, T)
    sel = k + 1
    splits = math.ceil(sel / args.split)
    meta = B * kv * T * (32 + 4 * reps)
    scores = B * qh * T * 2
    idx = B * qh * sel * 8
    gathered = (rows + B * kv) * 2 * D * 2  # distinct K and V rows + the current token's
    partials = B * qh * splits * (D + 2) * 4
    qio = B * qh * D * 2
    return {
        "query_encode": qio + B * qh * (32 + 8 * reps),
        "score": meta + scores + B * qh * (32 + 8 * reps),
        "score_fused": meta + scores + qio,
        "score_tc": meta + scores + qio,
        "score_popcount": meta + scores + qio,
        "score_topk_hist": meta + 2 * scores + qio + idx + 2 * B * qh * 2048 * 4,
        "score_topk_radix": meta + 2 * scores + qio + idx,
        "topk": scores + idx,
        "attn_partial": gathered + idx + partials + qio,
        "attn_merge": partials + qio,
        "attn_fused": gathered + idx + 2 * partials + 2 * qio,
        # Per-step algorithmic bytes: metadata + distinct gathered rows + int32
        # indices + q/out (scores and partials are intermediates).
        "step": meta + gathered + B * qh * sel * 4 + 2 * qio,
        # The same with every query head's selection counted separately.
        "step_upper_bound": meta + B * qh * sel * 2 * D * 2 + B * qh * sel * 4 + 2 * qio,
    }


# ---------------------------------------------------------------------------
# our implementation
# ---------------------------------------------------------------------------

def run_ours(args, world, rank, local):
    import torch
    dist = init_dist(world, local)
    device = torch.device("cuda", local)
    from popkv_b200 import _lib
    _lib.lib()
    layer = make_layer(args, world, rank, device)
    batch = args.batch
    if batch > 1:  # independent sequences, folded into heads; everything below runs as batch 1
        if world > 1:
            raise SystemExit("batch > 1 runs on one GPU")
        layer = fold_batch(layer, batch)
        args = argparse.Namespace(**{**vars(args), "batch": 1, "no_cpu_baseline": True})
    copies = max(2, math.ceil(3 * L2_BYTES / max(1, layer_bytes(args, layer))))
    copies = min(copies, 16)
    q_local = layer["q_local"]
    peer = None
    if dist is not None and args.gather == "peer":
        from popkv_b200.sharding import PeerGather
        peer = PeerGather(args.batch * q_local, torch.bfloat16, device)
    steps = build_steps(args, layer, copies, gather=peer)
    gathered = torch.empty((world * q_local, 128), device=device, dtype=torch.bfloat16) if dist else None

    def one_step(i):
        out = steps[i % copies].replay()
        if dist is not None and peer is None:
            dist.all_gather_into_tensor(gathered, out.view(q_local, 128))
        return out

    stream = torch.cuda.current_stream(device)
    for i in range(args.warmup):
        one_step(i)
    torch.cuda.synchronize(device)

    # Chains: `chain` consecutive layer steps (each on the next layer copy)
    # captured into one CUDA graph, as the layers of a decoded token are; the
    # timed loop replays them so that exactly K steps run.
    chain = max(1, min(args.chain, args.steps))
    if args.no_graph or (dist is not None and peer is None) or args.chunks != 1:
        chain = 1  # eager steps, or an NCCL all-gather after each replay

    def capture_chain(n, offset):
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(device)
        side.wait_stream(stream)
        with torch.cuda.graph(g, stream=side):
            for j in range(n):
                steps[(offset + j) % copies]._launch(side)
        stream.wait_stream(side)
        return g

    full, rem = divmod(args.steps, chain)
    if chain > 1:
        chains = [capture_chain(chain, 0)] + ([capture_chain(rem, full * chain)] if rem else [])
        plan = [(chains[0], chain)] * full + ([(chains[1], rem)] if rem else [])
        for _ in range(max(1, math.ceil(args.warmup / chain))):
            chains[0].replay()
    else:
        plan = [(None, 1)] * args.steps
    torch.cuda.synchronize(device)
    sampler = ClockSampler(physical_gpu_index(local)).start()
    time.sleep(0.25)
    # Keep the GPU busy while the sampler warms up, then time exactly K steps.
    for i in range(args.warmup):
        one_step(i)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(device)
    starts = [torch.cuda.Event(enable_timing=True) for _ in plan]
    ends = [torch.cuda.Event(enable_timing=True) for _ in plan]
    t0 = time.time()
    for i, (g, _) in enumerate(plan):
        starts[i].record(stream)
        if g is None:
            one_step(i)
        else:
            g.replay()
        ends[i].record(stream)
    torch.cuda.synchronize(device)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(device)
    t1 = time.time()
    sampler.stop()
    total_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    # The same steps with one graph launch per step (per-step events), for comparison.
    single_n = min(args.steps, 400)
    s_starts = [torch.cuda.Event(enable_timing=True) for _ in range(single_n)]
    s_ends = [torch.cuda.Event(enable_timing=True) for _ in range(single_n)]
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(device)
    for i in range(single_n):
        s_starts[i].record(stream)
        one_step(i)
        s_ends[i].record(stream)
    torch.cuda.synchronize(device)
    single_ms = sum(s.elapsed_time(e) for s, e in zip(s_starts, s_ends))
    total = torch.tensor([total_ms, single_ms], device=device, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(total, op=dist.ReduceOp.MAX)
    ms_per_step = float(total[0].item()) / args.steps
    single_ms_per_step = float(total[1].item()) / single_n
    chains = plan = None

    stages = stage_breakdown(args, layer, steps, device)
    e2e = end_to_end(args, layer, steps, device, dist, gathered, world, peer)
    clocks = sampler.summary(t0, t1)

    if dist is not None:
        # Per-stage and e2e maxima over ranks.
        vec = torch.tensor([stages[k]["us"] for k in sorted(stages)] + [e2e["value"]],
                           device=device, dtype=torch.float64)
        dist.all_reduce(vec, op=dist.ReduceOp.MAX)
        for j, k in enumerate(sorted(stages)):
            stages[k]["us"] = float(vec[j].item())
        e2e["value"] = float(vec[-1].item())
    # The published per-layer figure and the ncu traffic are for config 1 itself.
    default_workload = all({**vars(args), "batch": batch}.get(k) == v for k, v in DEFAULT_WORKLOAD.items())
    if rank == 0:
        rows = union_rows(steps[0])
        abytes = algorithmic_bytes(args, layer, rows)
        peaks = measured_peaks()
        for name, st in stages.items():
            if name in abytes and st["us"] > 0:
                gbs = abytes[name] / (st["us"] * 1e-6) / 1e9
                st["algorithmic_bytes"] = abytes[name]
                st["achieved_gbs"] = round(gbs, 1)
                st["frac_of_hbm"] = round(gbs / peaks["hbm_gbs"], 4)
        # The step's own kernels; a histogram top-k is only timed with its score kernel.
        names = {"score": "score_fused", "topk": "topk", "score_hist": "score_topk_hist",
                 "topk_hist": "score_topk_hist", "attn_partial": "attn_partial",
                 "attn_merge": "attn_merge", "retrieve": "retrieve"}
        timed = {names[k]: stages[names[k]] for k in steps[0].kernels if names[k] in stages}
        dominant = max(timed, key=lambda k: timed[k]["us"])
        dom = stages[dominant]
        step_bytes = abytes["step"]
        result = {
            "metric": METRIC, "value": round(ms_per_step, 5), "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 5), "higher_is_better": False,
            "scaling": "strong",
            "vs_baseline": round(ms_per_step / PUBLISHED_MS_PER_LAYER, 4) if default_workload else None,
            "dtype": "bf16", "data": "synthetic (seeded N(0,1) keys x lognormal channel factors + RoPE)",
            "config": {
                "workload": (f"config {1 if batch == 1 else 3}: single-layer decode step, {args.preset}, "
                             f"batch {batch}, 32 q / 8 kv heads, head_dim 128, context {args.context}, "
                             f"budget {args.budget}"),
                "preset": args.preset, "token_group": layer["tg"], "dim_group": layer["g"],
                "batch": batch, "context": args.context, "budget": args.budget,
                "parallelism": f"kv-head shard x{world}" + ("" if world == 1 else (
                    " + merge fused with the all-gather over NVLink peer memory" if peer is not None
                    else " + NCCL all-gather")),
                "l2": f"steps cycle over {copies} layer copies ({copies * layer_bytes(args, layer) / 2**20:.0f} MiB) > L2",
                "launch": ("eager" if args.no_graph else
                           "CUDA graph per layer step" if chain == 1 else
                           f"{chain} layer steps per CUDA graph (each on the next layer copy, as the layers "
                           f"of one decoded token), replays timed with CUDA events"),
            },
            "single_step_graph": {"ms_per_step": round(single_ms_per_step, 5), "steps": single_n,
                                  "timing": "one graph launch per step, CUDA events around each"},
            "roofline": {
                "bound": "hbm", "kernel": dominant,
                "achieved": dom.get("achieved_gbs"), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": dom.get("frac_of_hbm"),
                "traffic": (NCU_TRAFFIC_CONFIG1.get(dominant) if world == 1 and default_workload else None),
                "traffic_source": "ncu capture of this kernel at config 1 (a constant here, not this run)",
                "algorithmic_bytes": dom.get("algorithmic_bytes"),
                "peak_source": peaks["source"],
                # The whole step against the same peak: its algorithmic bytes (metadata,
                # distinct gathered K/V rows, indices, q/out) over the step time.
                "step": {"algorithmic_bytes": step_bytes,
                         "achieved": round(step_bytes / (ms_per_step * 1e-3) / 1e9, 1),
                         "frac": round(step_bytes / (ms_per_step * 1e-3) / 1e9 / peaks["hbm_gbs"], 4)},
            },
            "step_roofline": {
                "algorithmic_bytes": step_bytes,
                "distinct_rows": rows,
                "upper_bound_bytes": abytes["step_upper_bound"],
                "achieved_gbs": round(step_bytes / (ms_per_step * 1e-3) / 1e9, 1),
                "frac": round(step_bytes / (ms_per_step * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
            },
            "stages_us": {k: v for k, v in stages.items()},
            "e2e": e2e,
            "gpu_launches": 4 * args.steps,
            "clocks": clocks,
        }
        if not args.no_cpu_baseline and world == 1:
            result["cpu_baseline"] = cpu_baseline(args, layer, max_seconds=args.cpu_seconds)
    if world == 1 and not args.no_model:
        # The metric's second half: full-model decode ms/token (config 2), one GPU.
        model_args = argparse.Namespace(**{**vars(args), "context": 32768, "budget": 4096, "batch": 1,
                                           "prefill": "model"})
        model = measure_model(model_args, 1, 0, device, None, warmup=3)
        result["full_model"] = {k: model[k] for k in ("metric", "value", "unit", "vs_baseline", "data", "config",
                                                     "roofline", "e2e", "gpu_launches", "clocks")}
    if rank == 0:
        print(json.dumps(result), flush=True)
    for st in steps:
        st.graph = None
    if dist is not None:
        if peer is not None:
            if peer.error():
                print(f"rank {rank}: a peer-gather wait gave up", file=sys.stderr, flush=True)
            peer.close()
        dist.barrier()
        dist.destroy_process_group()


def time_events(fn, reps, device):
    """Device time of one call (us): `reps` calls captured in a CUDA graph and replayed.

    Launching through the graph keeps host overhead (Python, ctypes) out of the
    measurement, as in the captured decode step; each call still pays its
    in-graph launch gap.
    """
    import torch
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        for _ in range(3):
            fn()
    torch.cuda.current_stream(device).wait_stream(side)
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        for _ in range(reps):
            fn()
    graph.replay()
    torch.cuda.synchronize(device)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream(device)
    a.record(stream)
    for _ in range(5):
        graph.replay()
    b.record(stream)
    torch.cuda.synchronize(device)
    del graph
    return a.elapsed_time(b) / (5 * reps) * 1e3


def stage_breakdown(args, layer, steps, device):
    """Per-kernel device time (median over reps, each on a cold layer copy)."""
    import torch
    from popkv_b200 import _lib
    from popkv_b200 import popkv_cuda as C
    lib, check, ptr = _lib.lib(), _lib.check, _lib.ptr
    n = len(steps)

    class _CurrentStream:  # resolves to the capturing stream at launch time
        @property
        def _as_parameter_(self):
            return _lib.stream_of(device)
    s = _CurrentStream()
    reps = args.stage_reps
    out = {}
    ctr = {"i": 0}

    def cold():
        ctr["i"] += 1
        return steps[ctr["i"] % n]

    def run(name, launch):
        def fn():
            launch(cold())
        out[name] = {"us": round(time_events(fn, reps, device), 2)}

    B = args.batch
    run("query_encode", lambda st: check(lib.popkv_query_encode(
        ptr(st.queries), _lib.BF16, B * st.q_heads, 128, st.g, ptr(st.q_sign), ptr(st.q_mag),
        ptr(st.q_low), ptr(st.q_delta), s)))
    run("score", lambda st: check(lib.popkv_score_encoded(
        ptr(st.q_sign), ptr(st.q_mag), ptr(st.q_low), ptr(st.q_delta), B, st.q_heads,
        *(ptr(t) for t in st.cache.packed), st.kv_heads, int(st.cache.packed[0].shape[1]),
        ptr(st.head_to_kv), st.prefix_tokens, st.g, ptr(st.scores), s)))
    run("score_fused", lambda st: check(lib.popkv_score(
        ptr(st.queries), _lib.BF16, B, st.q_heads, 128, *(ptr(t) for t in st.cache.packed),
        st.kv_heads, int(st.cache.packed[0].shape[1]), ptr(st.head_to_kv), st.prefix_tokens, st.g,
        ptr(st.scores), _lib.F16, s)))
    run("score_popcount", lambda st: check(lib.popkv_score_popcount(
        ptr(st.queries), _lib.BF16, B, st.q_heads, 128, *(ptr(t) for t in st.cache.packed),
        st.kv_heads, int(st.cache.packed[0].shape[1]), ptr(st.head_to_kv), st.prefix_tokens, st.g,
        ptr(st.scores), _lib.F16, s)))
    run("score_tc", lambda st: check(lib.popkv_score_tc(
        ptr(st.queries), _lib.BF16, B, st.q_heads, 128, *(ptr(t) for t in st.cache.packed),
        st.kv_heads, int(st.cache.packed[0].shape[1]), ptr(st.head_to_kv), st.prefix_tokens, st.g,
        ptr(st.scores), _lib.F16, s)))
    # popkv_topk_hist consumes (and re-zeroes) the histogram popkv_score_hist
    # builds, so the two are only timed as a pair.
    def score_topk_hist(st):
        check(lib.popkv_score_hist(
            ptr(st.queries), _lib.BF16, B, st.q_heads, *(ptr(t) for t in st.cache.packed), st.kv_heads,
            int(st.cache.packed[0].shape[1]), ptr(st.head_to_kv), st.prefix_tokens, st.g, ptr(st.scores),
            ptr(st.hist), s))
        check(lib.popkv_topk_hist(
            ptr(st.scores), ptr(st.hist), B * st.q_heads, st.prefix_tokens, st.prefix_tokens, st.k,
            st.prefix_tokens, ptr(st.indices), st.selected, s))
    if args.context <= 65536:  # the histogram top-k takes rows of at most 65536 scores
        run("score_topk_hist", score_topk_hist)

    def score_topk_radix(st):
        check(lib.popkv_score(
            ptr(st.queries), _lib.BF16, B, st.q_heads, 128, *(ptr(t) for t in st.cache.packed),
            st.kv_heads, int(st.cache.packed[0].shape[1]), ptr(st.head_to_kv), st.prefix_tokens, st.g,
            ptr(st.scores), _lib.F16, s))
        check(lib.popkv_topk(
            ptr(st.scores), _lib.F16, B * st.q_heads, st.prefix_tokens, st.prefix_tokens, st.k,
            st.prefix_tokens, ptr(st.indices), st.selected, s))
    run("score_topk_radix", score_topk_radix)
    run("topk", lambda st: check(lib.popkv_topk(
        ptr(st.scores), _lib.F16, B * st.q_heads, st.prefix_tokens, st.prefix_tokens, st.k,
        st.prefix_tokens, ptr(st.indices), st.selected, s)))

    def partial(st):
        pk, pv = st.prefix_keys, st.prefix_values
        check(lib.popkv_attn_partial(
            ptr(st.queries), _lib.BF16, B, st.q_heads, 128, ptr(pk), ptr(pv), _lib.BF16, st.kv_heads,
            st.prefix_tokens, pk.stride(0), pk.stride(1), pk.stride(2), pv.stride(0), pv.stride(1),
            pv.stride(2), ptr(st.current_keys), ptr(st.current_values), ptr(st.indices), st.selected,
            None, ptr(st.head_to_kv), st.split_tokens, ptr(st.partials), s))
    run("attn_partial", partial)
    if steps[0].gather is not None:
        run("attn_merge_gather", lambda st: st.gather.launch(st.partials, st.splits, s))
    run("attn_merge", lambda st: check(lib.popkv_attn_merge(
        ptr(st.partials), B * st.q_heads, st.splits, 128, ptr(st.output), _lib.BF16, s)))

    def fused(st):
        pk, pv = st.prefix_keys, st.prefix_values
        check(lib.popkv_attn_partial_merge(
            ptr(st.queries), _lib.BF16, B, st.q_heads, 128, ptr(pk), ptr(pv), _lib.BF16, st.kv_heads,
            st.prefix_tokens, pk.stride(0), pk.stride(1), pk.stride(2), pv.stride(0), pv.stride(1),
            pv.stride(2), ptr(st.current_keys), ptr(st.current_values), ptr(st.indices), st.selected,
            None, ptr(st.head_to_kv), st.split_tokens, ptr(st.partials), ptr(st.counters),
            ptr(st.output), _lib.BF16, s))
    run("attn_fused", fused)
    # The step's own graph: replayed back to back (one host call per step).
    stream = torch.cuda.current_stream(device)
    for _ in range(3):
        cold().replay()
    torch.cuda.synchronize(device)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(reps):
        cold().replay()
    b.record(stream)
    torch.cuda.synchronize(device)
    out["step_graph"] = {"us": round(a.elapsed_time(b) / reps * 1e3, 2)}

    # Prepack of the whole context and a mid-group append (not part of the step),
    # launched through the C ABI so host-side validation stays outside the events.
    keys0 = layer["keys"][0]
    tg, g = layer["tg"], layer["g"]
    planes = C.pack_keys(keys0, token_group_size=tg, dim_group_size=g)
    kvh, T = int(keys0.shape[0]), int(keys0.shape[1])
    cap = int(planes[0].shape[1])

    def pack(src, tokens):
        check(lib.popkv_pack(ptr(src), _lib.BF16, kvh, tokens, 128, src.stride(0), src.stride(1),
                             *(ptr(t) for t in planes), cap, 0, tg, g, s))
    out["prepack"] = {"us": round(time_events(lambda: pack(keys0, T), max(5, reps // 5), device), 2)}
    occ = max(1, tg // 2)
    out["append"] = {"us": round(time_events(lambda: pack(keys0, occ), reps, device), 2),
                     "occupancy": occ}
    # The decoded token's KV append fused with the re-encode of its open group
    # (row occ - 1 of a group starting at 0), on a scratch copy of the caches.
    if tg <= 128:
        kc, vc = keys0.clone(), layer["values"][0].clone()
        nk, nv = keys0[:, occ - 1].contiguous(), layer["values"][0][:, occ - 1].contiguous()

        def append_kv():
            check(lib.popkv_append_kv(ptr(nk), ptr(nv), _lib.BF16, kvh, 128, ptr(kc), ptr(vc), kc.stride(0),
                                      kc.stride(1), vc.stride(0), vc.stride(1), occ - 1,
                                      *(ptr(t) for t in planes), cap, 0, tg, g, s))
        out["append_kv"] = {"us": round(time_events(append_kv, reps, device), 2), "occupancy": occ}
    return out


def end_to_end(args, layer, steps, device, dist, gathered, world, peer=None):
    """Same step through the public API with pinned host inputs and a host read of the output.

    One GPU, or several with the peer-memory gather: SparseAttentionStep with
    host_io, whose graph carries the host-to-device copy of q | k | v and the
    device-to-host copy of the (gathered) output.  Several GPUs with NCCL: the
    step, then the all-gather, then the device-to-host copy.
    """
    import torch
    from popkv_b200.decode import SparseAttentionStep
    st = steps[0]
    stream = torch.cuda.current_stream(device)
    if dist is None or peer is not None:
        # One host_io step per layer copy, cycled like the device-timed steps (> L2).
        hsteps = []
        for src in steps:
            step = SparseAttentionStep(src.cache, src.prefix_keys, src.prefix_values, src.head_to_kv,
                                       budget=args.budget, q_dtype=torch.bfloat16, batch=args.batch,
                                       use_graph=not args.no_graph, select=args.select, host_io=True,
                                       gather=peer, split_tokens=args.split)
            step.host_queries.copy_(layer["queries"].cpu())
            step.host_current_keys.copy_(layer["cur_k"].cpu())
            step.host_current_values.copy_(layer["cur_v"].cpu())
            hsteps.append(step)

        def e2e_step(i):
            step = hsteps[i % len(hsteps)]
            step(step.host_queries, step.host_current_keys, step.host_current_values)
        h2d = hsteps[0]._in_bytes
        d2h = hsteps[0].host_output.numel() * hsteps[0].host_output.element_size()
        api = "popkv_b200.decode.SparseAttentionStep(host_io=True).__call__ (pinned host in/out)"
        if peer is not None:
            api = api.replace("host_io=True", "host_io=True, gather=PeerGather")
    else:
        q_host = layer["queries"].cpu().pin_memory()
        k_host = layer["cur_k"].cpu().pin_memory()
        v_host = layer["cur_v"].cpu().pin_memory()
        out_host = torch.empty((world * st.q_heads, 128), dtype=st.output.dtype).pin_memory()

        def e2e_step(i):
            s2 = steps[i % len(steps)]
            out = s2(q_host, k_host, v_host)
            dist.all_gather_into_tensor(gathered, out.view(s2.q_heads, 128))
            out_host.copy_(gathered, non_blocking=True)
        h2d = (q_host.numel() + k_host.numel() + v_host.numel()) * 2
        d2h = out_host.numel() * 2
        api = "popkv_b200.decode.SparseAttentionStep.__call__ + all_gather (pinned host in/out)"

    for i in range(min(args.warmup, 20)):
        e2e_step(i)
    torch.cuda.synchronize(device)
    n = max(20, min(args.steps, 500))
    # Host-visible latency: each call is timed on the host clock from the call
    # until the result is readable on the host (the stream synchronised).
    total = 0.0
    for i in range(n):
        t0 = time.perf_counter()
        e2e_step(i)
        stream.synchronize()
        total += time.perf_counter() - t0
    ms = total * 1e3 / n
    # Back-to-back calls without a host wait per call (device-timed), for context.
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for i in range(n):
        e2e_step(i)
    b.record(stream)
    torch.cuda.synchronize(device)
    pipelined = a.elapsed_time(b) / n
    return {"value": round(ms, 5), "unit": UNIT, "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "api": api,
            "timing": "host clock per call, call to host-readable result (stream synchronised)",
            "pipelined_ms": round(pipelined, 5)}


def measured_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        data = json.loads(path.read_text())
        return {"hbm_gbs": float(data["hbm_gbs"]), "source": "MEASURED_PEAKS.json (measured)"}
    except Exception:
        return {"hbm_gbs": 6650.0, "source": "fallback 6.65 TB/s"}


# ---------------------------------------------------------------------------
# CPU baseline: the oracle port on the host cores
# ---------------------------------------------------------------------------

def cpu_step_fn(args, x, tg, g):
    """Prepare the oracle inputs once; return a callable running one decode step on the CPU."""
    import numpy as np
    import oracle
    from popkv_b200.workloads import to_bf16_bits, head_to_kv
    kbits = to_bf16_bits(x.keys[0])
    vbits = to_bf16_bits(x.values[0])
    qbits = to_bf16_bits(x.queries)
    ck, cv = to_bf16_bits(x.current_keys[0]), to_bf16_bits(x.current_values[0])
    mapping = head_to_kv(32, 8)
    planes = oracle.pack(kbits, "bf16", token_group_size=tg, dim_group_size=g)
    T = args.context

    def step():
        enc = oracle.query_encode(qbits, "bf16", dim_group_size=g)
        _, s16 = oracle.score(enc, planes, head_to_kv=mapping, tokens=T, dim_group_size=g, head_dim=128)
        idx = oracle.select_with_current(s16, args.budget, T)[0]
        return oracle.attention(qbits[0], "bf16", kbits, vbits, "bf16", ck, cv, idx, mapping)
    return step


def cpu_baseline(args, layer, max_seconds: float) -> dict:
    import oracle
    step = cpu_step_fn(args, layer["host"], layer["tg"], layer["g"])
    step()  # warm-up
    times = []
    start = time.perf_counter()
    while time.perf_counter() - start < max_seconds and len(times) < 200:
        t = time.perf_counter()
        step()
        times.append((time.perf_counter() - t) * 1e3)
    return {"value": round(statistics.median(times), 3), "unit": UNIT, "cores": oracle.num_threads(),
            "kind": "port",
            "sample": f"{len(times)} full decode steps (encode+score over {args.context} tokens, "
                      f"top-k, attention over {args.budget} slots x 32 heads), median; "
                      f"C oracle with OpenMP on {os.cpu_count()} host cores"}


def run_reference(args, world, rank):
    if rank != 0:
        return
    import oracle
    from popkv_b200 import popkv as P
    from popkv_b200.workloads import decode_inputs
    tg, g = P.POPKV_PRESETS[args.preset]
    x = decode_inputs(batch=1, context=args.context, seed=0, dtype="bf16")
    step = cpu_step_fn(args, x, tg, g)
    for _ in range(max(1, min(args.warmup, 3))):
        step()
    steps = max(1, min(args.steps, 40))
    start = time.perf_counter()
    times = []
    for _ in range(steps):
        t = time.perf_counter()
        step()
        times.append((time.perf_counter() - t) * 1e3)
        if time.perf_counter() - start > 60:
            break
    ms = sum(times) / len(times)
    result = {
        "impl": "reference", "metric": METRIC, "value": round(ms, 3), "unit": UNIT,
        "n_gpus": world, "steps": len(times), "warmup": args.warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) keys x lognormal channel factors + RoPE)",
        "config": {"workload": f"config 1: single-layer decode step, {args.preset}, batch 1, 32 q / 8 kv "
                               f"heads, head_dim 128, context {args.context}, budget {args.budget}",
                   "preset": args.preset, "context": args.context, "budget": args.budget},
        "cpu_baseline": {"value": round(ms, 3), "unit": UNIT, "cores": oracle.num_threads(),
                         "kind": "port",
                         "sample": f"{len(times)} full decode steps on the C restatement of the "
                                   "reference's kernels (the reference's own CPU path is PyTorch "
                                   "source that cannot travel to this host)"},
        "e2e": {"value": round(ms, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    result["reference_gpu"] = reference_gpu_stages(args)
    print(json.dumps(result), flush=True)


def reference_gpu_stages(args) -> dict:
    """The reference's own CUDA kernels on this GPU, beside this package's, timed the same way.

    The reference's extension (csrc/popkv_ext.cu, compiled from its sources by
    oracle/build_ref.py with its own flags) runs the decode branch's GPU
    stages as the reference launches them (popkv.py:1078-1099): eager calls,
    device time from CUDA events over back-to-back calls, cycling over 8 copies
    of the keys and planes (more than L2).  The split attention is Triton
    source (sparse_kernels.py:237-318) that does not travel to the GPU host.
    """
    try:
        import torch
        from oracle.build_ref import load_reference_extension
        if not torch.cuda.is_available():
            return {"unavailable": "no CUDA device"}
        ref = load_reference_extension()
    except Exception as exc:  # noqa: BLE001  (a missing or stale build is reported, not fatal)
        return {"unavailable": f"reference extension failed to load: {exc}"}
    if ref is None:
        return {"unavailable": "reference extension not built (the package was built without a reference checkout)"}
    from popkv_b200 import popkv as P
    from popkv_b200 import popkv_cuda as C
    from popkv_b200.workloads import decode_inputs, head_to_kv
    dev = torch.device("cuda", 0)
    tg, g = P.POPKV_PRESETS[args.preset]
    T, k, copies = args.context, min(args.budget - 1, args.context), 8
    x = decode_inputs(batch=1, context=T, seed=0, dtype="bf16")
    keys = [torch.from_numpy(x.keys[0]).to(torch.bfloat16).to(dev).contiguous() for _ in range(copies)]
    q = torch.from_numpy(x.queries).to(torch.bfloat16).to(dev).contiguous()
    mapping = torch.from_numpy(head_to_kv(32, 8)).to(dev)
    pack = (lambda kk: ref.pack(kk, T, tg)) if g == 32 else (lambda kk: ref.pack_dim(kk, T, g, tg))
    r_planes = [pack(kk) for kk in keys]
    r_enc = (torch.empty((1, 32, 4), dtype=torch.int32, device=dev), torch.empty((1, 32, 4), dtype=torch.int32, device=dev),
             torch.empty((1, 32, 128 // g), device=dev), torch.empty((1, 32, 128 // g), device=dev))
    ref.query_encode_out(q, *r_enc, g)
    r_scores = [ref.score_encoded(*r_enc, *pl, mapping, T, g) for pl in r_planes]
    o_planes = [C.pack_keys(kk, token_capacity=T, token_group_size=tg, dim_group_size=g) for kk in keys]
    o_enc = C.query_encode(q, dim_group_size=g)
    o_scores = [C.score_encoded(o_enc, pl, head_to_kv=mapping, tokens=T, dim_group_size=g) for pl in o_planes]
    torch.cuda.synchronize(dev)

    def timed(fn, reps=60):
        for i in range(5):
            fn(i)
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for i in range(reps):
            fn(i)
        b.record()
        torch.cuda.synchronize(dev)
        return round(a.elapsed_time(b) * 1e3 / reps, 2)

    def r_chain(i):
        ref.query_encode_out(q, *r_enc, g)
        sc = ref.score_encoded(*r_enc, *r_planes[i % copies], mapping, T, g)
        torch.topk(sc, k, dim=-1, sorted=False)

    def o_chain(i):
        enc = C.query_encode(q, dim_group_size=g)
        sc = C.score_encoded(enc, o_planes[i % copies], head_to_kv=mapping, tokens=T, dim_group_size=g)
        P.topk(sc, k)

    def graph_timed(fn, reps=20, replays=10):
        """Device time per call with `reps` calls captured in one CUDA graph (no host gaps)."""
        for i in range(3):
            fn(i)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(reps):
                fn(i)
        graph.replay()
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(replays):
            graph.replay()
        b.record()
        torch.cuda.synchronize(dev)
        return round(a.elapsed_time(b) * 1e3 / (replays * reps), 2)

    reference_graph = {
        "query_encode": graph_timed(lambda i: ref.query_encode_out(q, *r_enc, g)),
        "score_encoded": graph_timed(lambda i: ref.score_encoded(*r_enc, *r_planes[i % copies], mapping, T, g)),
        "topk": graph_timed(lambda i: torch.topk(r_scores[i % copies], k, dim=-1, sorted=False)),
        "encode_score_topk": graph_timed(r_chain),
    }
    ours_graph = {
        "query_encode": graph_timed(lambda i: C.query_encode(q, dim_group_size=g)),
        "score_encoded": graph_timed(lambda i: C.score_encoded(o_enc, o_planes[i % copies], head_to_kv=mapping,
                                                               tokens=T, dim_group_size=g)),
        "topk": graph_timed(lambda i: P.topk(o_scores[i % copies], k)),
        "encode_score_topk": graph_timed(o_chain),
    }
    reference = {
        "prepack": timed(lambda i: pack(keys[i % copies]), reps=20),
        "query_encode": timed(lambda i: ref.query_encode_out(q, *r_enc, g)),
        "score_encoded": timed(lambda i: ref.score_encoded(*r_enc, *r_planes[i % copies], mapping, T, g)),
        "topk": timed(lambda i: torch.topk(r_scores[i % copies], k, dim=-1, sorted=False)),
        "encode_score_topk": timed(r_chain),
    }
    ours = {
        "prepack": timed(lambda i: C.pack_keys(keys[i % copies], token_capacity=T, token_group_size=tg,
                                               dim_group_size=g), reps=20),
        "query_encode": timed(lambda i: C.query_encode(q, dim_group_size=g)),
        "score_encoded": timed(lambda i: C.score_encoded(o_enc, o_planes[i % copies], head_to_kv=mapping, tokens=T,
                                                         dim_group_size=g)),
        "topk": timed(lambda i: P.topk(o_scores[i % copies], k)),
        "encode_score_topk": timed(o_chain),
    }
    return {"unit": "us per call (CUDA events, 8 copies > L2)", "preset": args.preset, "context": T,
            "budget": args.budget, "reference_eager": reference, "ours_eager": ours,
            "reference_graph": reference_graph, "ours_graph": ours_graph,
            "timing": "eager: back-to-back calls as the reference launches them (host overhead included when the "
                      "GPU waits for it); graph: the same calls captured in a CUDA graph (device time)",
            "attention": "unavailable: the reference's split attention is Triton source (sparse_kernels.py:237-318) "
                         "that does not travel to the GPU host",
            "build": "oracle/build_ref.py: csrc/popkv_ext.cu + popkv_ext.cpp, -O3 --use_fast_math, sm_100a"}


# ---------------------------------------------------------------------------
# full-model decode (config 2)
# ---------------------------------------------------------------------------

MODEL_METRIC = "full-model decode ms/token (32-layer Llama-3.1-8B shape, greedy)"
# The reference's published full-model generation ms/token (decode + selection
# + update) at 32K, batch 1, budget 4096 (README.md:60-61 of the reference).
PUBLISHED_MODEL_MS = {"popkv-s": 43.011, "popkv-q": 43.888}


def model_bytes_per_step(dec, weights, position: int) -> dict:
    """Algorithmic HBM bytes of one decode step: weights, dense-layer K/V, sparse metadata + gathered rows.

    The sparse gather is the per-head upper bound (every query head's budget of
    distinct K and V rows); the step's real union is smaller when query heads
    of a group share tokens.
    """
    B, kvh, qh = dec.batch, dec.kvh, dec.qh
    L = dec.cfg.num_hidden_layers
    dense = L - len(dec.sparse_layers)
    w = dec.weight_bytes_per_step()  # this rank's q/k/v rows (and MLP slice in tensor mode)
    kv_dense = dense * B * kvh * (position + 1) * 128 * 2 * 2
    reps = 128 // dec.g
    meta = len(dec.sparse_layers) * B * kvh * position * (32 + 4 * reps)
    gather = len(dec.sparse_layers) * B * qh * min(dec.budget, position + 1) * 128 * 2 * 2
    return {"weights": w, "dense_kv": kv_dense, "sparse_metadata": meta, "sparse_gather_upper": gather,
            "total": w + kv_dense + meta + gather}


def run_model(args, world, rank, local):
    import torch
    dist = init_dist(world, local)
    device = torch.device("cuda", local)
    result = measure_model(args, world, rank, device, dist)
    if rank == 0:
        print(json.dumps(result), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def measure_model(args, world, rank, device, dist, warmup=None):
    """Time the full-model greedy decode (config 2 by default); the JSON object on rank 0, None elsewhere."""
    import torch
    from popkv_b200 import _lib
    from popkv_b200.decoder import LLAMA31_8B, LlamaSparseDecoder, LlamaWeights
    from popkv_b200.popkv import POPKV_PRESETS, RetrievalConfig
    _lib.lib()
    cfg = LLAMA31_8B
    method = args.model_method
    tg, g = POPKV_PRESETS.get(method, (32, 32))
    retrieval = RetrievalConfig(budget=args.budget, group_size=tg, dim_group_size=g)
    weights = LlamaWeights.random(cfg, device=device, seed=0)
    T, W, K = args.context, (args.warmup if warmup is None else warmup), args.gen_steps
    dec = LlamaSparseDecoder(weights, method=method, retrieval=retrieval, batch=args.batch,
                             max_context=T + W + 2 * K + 2, rank=rank, world=world,
                             group=None, mlp_parallel=args.mlp_parallel,
                             all_reduce=args.all_reduce)
    gen = torch.Generator().manual_seed(0)
    ids = torch.randint(0, cfg.vocab_size, (args.batch, T), generator=gen)
    torch.cuda.synchronize(device)
    t_prefill = time.time()
    if args.prefill == "model":
        dec.prefill(ids)
    else:
        dec.prefill_synthetic(T, seed=rank)
    prefill_s = time.time() - t_prefill
    stream = torch.cuda.current_stream(device)
    for _ in range(W):
        dec.step()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(device)
    position0 = int(dec.position.item())
    sampler = ClockSampler(physical_gpu_index(device.index or 0)).start()
    time.sleep(0.25)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.time()
    torch.cuda.nvtx.range_push("decode_steps")  # the launch-list capture filters on this range
    start.record(stream)
    for _ in range(K):
        dec.step()
    end.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize(device)
    t1 = time.time()
    sampler.stop()
    total = torch.tensor([start.elapsed_time(end)], device=device, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(total, op=dist.ReduceOp.MAX)
    ms = float(total.item()) / K
    # End to end through the public API: each step takes its token id from the
    # host (pinned) and returns the greedy next id to the host.
    host_tok = torch.empty((args.batch,), dtype=torch.int64).pin_memory()
    host_next = torch.empty_like(host_tok)
    host_tok.copy_(dec.token.cpu())
    e2e_steps = min(K, 64)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        dec.token.copy_(host_tok, non_blocking=True)
        dec.step()
        host_next.copy_(dec.token, non_blocking=True)
        stream.synchronize()
        host_tok.copy_(host_next)
    e1.record(stream)
    torch.cuda.synchronize(device)
    e2e = torch.tensor([e0.elapsed_time(e1)], device=device, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(e2e, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e.item()) / e2e_steps
    if rank == 0:
        peaks = measured_peaks()
        mid = position0 + K // 2
        abytes = model_bytes_per_step(dec, weights, mid)
        gbs = abytes["total"] / (ms * 1e-3) / 1e9
        dense = cfg.num_hidden_layers - len(dec.sparse_layers)
        # Our kernels per step: dense layer 6 (2 norms, RoPE/append, partial, merge,
        # SiLU), sparse layer 9 (+ score, top-k, append re-encode), final norm 1.
        ours_per_step = dense * 6 + len(dec.sparse_layers) * 9 + 1
        if dec._peer_sum is not None:
            ours_per_step += 2 * cfg.num_hidden_layers  # the peer all-reduces
        workload = ("config 2: 32-layer Llama-3.1-8B-shaped decoder" if args.batch == 1 and T <= 65536
                    else "config 4 shape: 32-layer Llama-3.1-8B-shaped decoder")
        result = {
            "metric": MODEL_METRIC, "value": round(ms, 4), "unit": "ms", "n_gpus": world,
            "steps": K, "warmup": W, "ms_per_step": round(ms, 4), "higher_is_better": False,
            "scaling": "strong",
            "vs_baseline": (round(ms / PUBLISHED_MODEL_MS[method], 4) if method in PUBLISHED_MODEL_MS
                            and args.context == 32768 and args.batch == 1 else None),
            "dtype": "bf16",
            "data": ("synthetic (random-init weights N(0, 0.02), uniform random prefix ids)" if args.prefill == "model"
                     else "synthetic (random-init weights N(0, 0.02); prefix K/V drawn from the seeded key/value "
                          "distributions, no model prefill)"),
            "config": {
                "workload": f"{workload}, {method} "
                            f"(layers 0-1 dense), batch {args.batch}, prefix {T}, budget {args.budget}, "
                            f"{K} greedy steps after {W} warm-up steps",
                "method": method, "batch": args.batch, "prefix": T, "budget": args.budget,
                "prefill": args.prefill,
                "context_at_timed_steps": [position0, position0 + K - 1],
                "parallelism": f"kv-head shard x{world}" + (
                    "" if world == 1 else " + NCCL all-gather per layer, replicated MLP"
                    if args.mlp_parallel == "replicated" else
                    " + tensor-parallel o_proj/MLP, two NCCL all-reduces per layer"
                    if args.all_reduce == "nccl" else
                    " + tensor-parallel o_proj/MLP, two peer-memory all-reduces (popkv_peer_sum) per layer"),
                "l2": "each step streams ~16 GB of weights > L2",
                "launch": "one CUDA graph per token (device-resident position), replayed",
            },
            "roofline": {
                "bound": "hbm", "kernel": "whole step", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 4), "traffic": None,
                "algorithmic_bytes": abytes, "peak_source": peaks["source"],
            },
            "prefill_s": round(prefill_s, 2),
            "e2e": {"value": round(e2e_ms, 4), "unit": "ms", "h2d_bytes_per_step": 8 * args.batch,
                    "d2h_bytes_per_step": 8 * args.batch, "steps": e2e_steps,
                    "api": "popkv_b200.decoder.LlamaSparseDecoder.step (token id in from pinned host, "
                           "greedy id back, synchronised per step)"},
            "gpu_launches": ours_per_step * K,
            "clocks": sampler.summary(t0, t1),
        }
    else:
        result = None
    dec.close()
    del dec, weights
    torch.cuda.empty_cache()
    return result


# ---------------------------------------------------------------------------
# weight-streaming products vs cuBLAS (the model step's dominant kernels)
# ---------------------------------------------------------------------------

MODEL_PRODUCTS = {"qkv": (6144, 4096), "o_proj": (4096, 4096), "gate_up": (28672, 4096),
                  "down": (4096, 14336), "lm_head": (128256, 4096)}


def run_products(args):
    """popkv_linear against torch.mm (cuBLAS) at batch 1, each timed as a CUDA graph
    of back-to-back launches cycling over weight copies larger than L2."""
    import torch
    from popkv_b200 import _lib
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    lib, check, ptr = _lib.lib(), _lib.check, _lib.ptr
    peaks = measured_peaks()
    shapes = MODEL_PRODUCTS
    reps = 20
    if args.product_shape:
        n, k = (int(v) for v in args.product_shape.lower().split("x"))
        shapes, reps = {args.product_shape: (n, k)}, 3
    results = {}
    for name, (n, k) in shapes.items():
        copies = max(2, int(3 * L2_BYTES // (n * k * 2)) + 1)
        gen = torch.Generator(device=device)
        gen.manual_seed(0)
        ws = [torch.empty(n, k, device=device, dtype=torch.bfloat16).normal_(generator=gen) for _ in range(copies)]
        x = torch.empty(1, k, device=device, dtype=torch.bfloat16).normal_(generator=gen)
        out = torch.empty(1, n, device=device, dtype=torch.bfloat16)

        def ours(i):
            check(lib.popkv_linear(ptr(ws[i % copies]), n, k, ptr(x), 1, ptr(out), n, _lib.stream_of(device)))

        def cublas(i):
            torch.mm(x, ws[i % copies].t(), out=out)

        entry = {}
        for label, fn in (("ours", ours), ("cublas", cublas)):
            if args.product_shape:  # plain launches, for a profiler
                for i in range(reps):
                    fn(i)
                torch.cuda.synchronize(device)
                continue
            us = time_graph(fn, reps, device)
            gbs = n * k * 2 / (us * 1e-6) / 1e9
            entry[label] = {"us": round(us, 2), "gbs": round(gbs, 1), "frac_of_hbm": round(gbs / peaks["hbm_gbs"], 4)}
        results[name] = {"rows": n, "k": k, **entry}
        del ws
    if not args.product_shape:
        print(json.dumps({"metric": "weight-streaming product time, batch 1 (graph-timed, weights > L2)",
                          "unit": "us", "peak_gbs": peaks["hbm_gbs"], "peak_source": peaks["source"],
                          "products": results}), flush=True)


def time_graph(fn, reps, device) -> float:
    """Mean device time of fn(i) over `reps` launches captured back to back in one CUDA graph."""
    import torch
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        fn(0)
        fn(1)
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        for i in range(reps):
            fn(i)
    graph.replay()
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(3):
        graph.replay()
    end.record()
    torch.cuda.synchronize(device)
    return start.elapsed_time(end) * 1000.0 / (3 * reps)


def main(argv=None):
    args = parse_args(argv)
    world, rank, local = dist_env()
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    if args.model:
        run_model(args, world, rank, local)
        return
    if args.products:
        run_products(args)
        return
    run_ours(args, world, rank, local)


if __name__ == "__main__":
    main()
