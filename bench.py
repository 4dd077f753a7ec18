"""Benchmark of the paged-KV rollout hot path (append + paged GQA decode attention).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 4] [--impl ours|reference]

One step = one decode step of every sequence through all layers: per layer,
append one K/V token per (sequence, kv head) and attend over the sequence's
pages (BASELINE metric: KV-read HBM GB/s and seq-steps/s). Inputs are seeded
synthetic tensors of the BASELINE config shapes (no dataset is involved) and
stay resident in HBM; the KV pool (~130 GB per GPU for config 4) is far larger
than the 126 MB L2, so no L2 flush is needed between steps.

Multi-GPU: one process per GPU (torchrun). Sequences are independent, so the
job is partitioned — each rank owns a seeded shard of whole sequences
(LPT-balanced by context length), its own page pool and block tables — and no
collective runs inside the timed region; only the start barrier and the
max-over-ranks time reduction cross ranks. `--scaling strong` (the default)
shards the config's own sequence count over the N GPUs, as BASELINE states the
configs (config 4: 1024 sequences over 1/2/4/8 GPUs); `--scaling weak` gives
every GPU the full count.

Rank 0 prints ONE JSON line. `--impl reference` times the CPU restatement of
the reference algorithm (oracle/, the reference itself is Python/Triton and
has no CPU implementation of its own) on the host cores instead.
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

import numpy as np
import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "paged KV decode: KV-read HBM GB/s and seq-steps/s at 1/2/4/8 B200"

# DRAM bytes (read + write) per algorithmic byte of one decode launch, per
# config, from one-launch ncu captures of decode_tc_kernel on a reduced case of
# that config's geometry (dram__bytes_read.sum + dram__bytes_write.sum over the
# launch's algorithmic bytes). Traffic grows with the pages read, so
# roofline.traffic scales the ratio to the full launch.
# config 3 counts every sequence's reads of its group's shared prompt pages in
# its algorithmic bytes, but those pages come from L2 after the first reader:
# its traffic is 1.012x the unique K/V bytes.
DECODE_DRAM_TRAFFIC_RATIO = {3: 0.4254, 4: 1.0017, 5: 1.0023}
UNIT = "seq-steps/s"


# ----------------------------------------------------------------------------- workloads
CONFIGS = {
    3: dict(name="config3: 16 prompts x group 8, shared 512-token prompt pages + U{1..512} private tokens",
            seqs=128, hq=12, hkv=2, d=128, bs=16, layers=28),
    4: dict(name="config4: 1024 seqs, ctx U[1024,8192], 12q/2kv, D128, bf16, bs16, 28 layers",
            seqs=1024, hq=12, hkv=2, d=128, bs=16, layers=28),
    5: dict(name="config5: Qwen2.5-7B geometry, 64 seqs, ctx log-U[4096,32768], 28q/4kv, D128, bf16, bs16, 28 layers",
            seqs=64, hq=28, hkv=4, d=128, bs=16, layers=28),
}


def global_lengths(config: int, n_total: int, seed: int = 1234) -> np.ndarray:
    """Post-append context length of every sequence of the whole job."""
    rs = np.random.RandomState(seed)
    if config == 4:
        return rs.randint(1024, 8193, size=n_total)
    if config == 5:
        return np.exp(rs.uniform(np.log(4096), np.log(32768), size=n_total)).astype(np.int64)
    if config == 3:
        return 512 + rs.randint(1, 513, size=n_total)
    raise ValueError(config)


def shard_indices(config: int, lens: np.ndarray, rank: int, world: int) -> list[int]:
    """Sequences of `rank`: LPT by context length (config 3: whole GRPO groups of 8,
    so a group's shared prompt pages stay on one GPU)."""
    if config == 3:
        group = 8
        n_groups = len(lens) // group
        costs = [lens[g * group:(g + 1) * group].sum() for g in range(n_groups)]
        groups = lpt_assign(costs, world)[rank]
        return [g * group + j for g in groups for j in range(group)]
    return lpt_assign(lens.tolist(), world)[rank]


def workload_config(args, world: int) -> dict:
    """The `config` object of the JSON line: the workload only (both arms print the same one)."""
    c = dict(CONFIGS[args.config])
    strong = args.scaling == "strong"
    if args.seqs:
        c["seqs"] = args.seqs
        c["name"] += f" [reduced to {args.seqs} seqs" + (" in all]" if strong else "/GPU]")
    n_total = c["seqs"] if strong else c["seqs"] * world
    lens = global_lengths(args.config, n_total)
    mine = shard_indices(args.config, lens, 0, world)
    layers = args.layers or c["layers"]
    pages = sum((int(lens[i]) + c["bs"] - 1) // c["bs"] for i in mine)
    if args.config == 3:  # each group's 32 prompt pages are stored once
        pages -= (len(mine) // 8) * 7 * (512 // c["bs"])
    pool_gb = 2 * layers * pages * c["hkv"] * c["bs"] * c["d"] * 2 / 1e9
    return {
        "workload": c["name"],
        "seqs_total": n_total,
        "seqs_per_gpu": len(mine),
        "layers": layers,
        "q_heads": c["hq"],
        "kv_heads": c["hkv"],
        "head_dim": c["d"],
        "block_size": c["bs"],
        "step": "per layer: append 1 token per sequence and kv head, then paged decode attention over ctx",
        "l2": "no flush: KV pool of rank 0 %.1f GB >> 126 MB L2" % pool_gb,
        "parallelism": f"dp{world} (sequence shards, LPT by context length, no collective)",
        "sharding": (f"strong: the config's {n_total} sequences split over {world} GPU(s)" if strong else
                     f"weak: {c['seqs']} sequences per GPU ({n_total} in all)"),
    }


class Workload:
    """One rank's shard: page pool, block tables, per-layer q/k_new/v_new, context lengths."""

    def __init__(self, config: int, rank: int, world: int, layers: int | None, device, seqs: int | None = None,
                 strong: bool = True):
        c = dict(CONFIGS[config])
        if seqs:
            c["seqs"] = seqs
            c["name"] += f" [reduced to {seqs} seqs" + (" in all]" if strong else "/GPU]")
        self.config, self.cfg = config, c
        self.layers = layers or c["layers"]
        hq, hkv, d, bs = c["hq"], c["hkv"], c["d"], c["bs"]
        n_total = c["seqs"] if strong else c["seqs"] * world
        self.n_total = n_total
        lens = global_lengths(config, n_total)
        mine = shard_indices(config, lens, rank, world)
        self.ctx_post = torch.tensor([int(lens[i]) for i in mine], dtype=torch.int32)
        B = len(mine)
        self.B, self.hq, self.hkv, self.d, self.bs = B, hq, hkv, d, bs
        g = torch.Generator(device="cpu").manual_seed(1000 + rank)
        pages = [(int(n) + bs - 1) // bs for n in self.ctx_post]
        if config == 3:
            # each group of 8 shares its 32 full prompt pages (refcounted in a real pool)
            prompt_pages = 512 // bs
            tables, nxt = [], 0
            for gi in range(B // 8):
                shared = list(range(nxt, nxt + prompt_pages))
                nxt += prompt_pages
                for j in range(8):
                    own = pages[gi * 8 + j] - prompt_pages
                    tables.append(shared + list(range(nxt, nxt + own)))
                    nxt += own
            num_blocks = nxt
            perm = torch.randperm(num_blocks, generator=g)
            tables = [[int(perm[p]) for p in t] for t in tables]
            self.unique_tokens = sum(512 for _ in range(B // 8)) + sum(int(n) - 512 for n in self.ctx_post)
        else:
            num_blocks = sum(pages)
            perm = torch.randperm(num_blocks, generator=g).tolist()
            tables, off = [], 0
            for p in pages:
                tables.append(perm[off:off + p])
                off += p
            self.unique_tokens = int(self.ctx_post.sum())
        self.max_blocks = max(len(t) for t in tables)
        bt = np.zeros((B, self.max_blocks), dtype=np.int32)
        for i, t in enumerate(tables):
            bt[i, : len(t)] = t
        self.num_blocks = num_blocks
        self.block_tables_cpu = torch.from_numpy(bt)
        self.device = device
        self.block_tables = self.block_tables_cpu.to(device)
        self.ctx_pre = (self.ctx_post - 1).to(device)
        self.ctx = self.ctx_post.to(device)
        # the pool: [layers, pages, hkv, bs, d] bf16, N(0,1)
        shape = (self.layers, num_blocks, hkv, bs, d)
        self.k_pool = torch.empty(shape, dtype=torch.bfloat16, device=device)
        self.v_pool = torch.empty(shape, dtype=torch.bfloat16, device=device)
        gd = torch.Generator(device=device).manual_seed(77 + rank)
        for t in (self.k_pool, self.v_pool):
            for layer in range(self.layers):  # per layer keeps the fp32 temporaries small
                t[layer].normal_(generator=gd)
        self.q = torch.randn(self.layers, B, hq, d, device=device, generator=gd).to(torch.bfloat16)
        self.k_new = torch.randn(self.layers, B, hkv, d, device=device, generator=gd).to(torch.bfloat16)
        self.v_new = torch.randn(self.layers, B, hkv, d, device=device, generator=gd).to(torch.bfloat16)
        self.out = torch.empty(self.layers, B, hq, d, dtype=torch.float32, device=device)

    # algorithmic bytes (one layer), the roofline numerator
    def kv_read_bytes_layer(self) -> int:
        return int(self.ctx_post.sum()) * self.hkv * self.d * 2 * 2

    def decode_bytes_layer(self) -> int:
        pages = int(((self.ctx_post + self.bs - 1) // self.bs).sum())
        return (self.kv_read_bytes_layer() + self.B * self.hq * self.d * (2 + 4) + pages * 4 + self.B * 4)

    def append_bytes_layer(self) -> int:
        return self.B * self.hkv * self.d * 2 * 2 * 2  # read new K,V + write into pages


def lpt_assign(costs, world):
    """sharding.lpt_assign, loaded from its file: importing the package would
    load libpkv.so, which the reference arm must not map."""
    import importlib.util

    spec = importlib.util.spec_from_file_location("_pkv_sharding", REPO / "grpo_training_engine_b200" / "sharding.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.lpt_assign(costs, world)


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self._t:
            self._t.join(timeout=2)
        sm, smax, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(smax) if smax else None,
            "power_w_max": max(power) if power else None,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


# ----------------------------------------------------------------------------- helpers
def measured_peaks() -> tuple[float, str]:
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
        except (KeyError, ValueError):
            pass
    return 6650.0, "fallback"


def physical_gpu(local: int) -> int:
    """nvidia-smi index of this process's GPU (CUDA_VISIBLE_DEVICES may remap it)."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        try:
            return int(vis.split(",")[local])
        except (ValueError, IndexError):
            return local
    return local


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and args.impl == "ours":
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


# ----------------------------------------------------------------------------- our arm
def run_ours(args, rank, world, local):
    import grpo_training_engine_b200 as pkv
    from grpo_training_engine_b200 import ops

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    shard_world = args.shard_of or world  # --shard-of N: rank 0's shard of an N-GPU job, on this GPU alone
    wl = Workload(args.config, rank, shard_world, args.layers, device, args.seqs, strong=args.scaling == "strong")
    L, B = wl.layers, wl.B
    stream = torch.cuda.current_stream(device)

    ws = {"buf": None}  # one plan workspace, reused by every step

    def step(ev_pairs=None):
        plan = ops.plan_decode(wl.ctx, wl.hq, wl.hkv, wl.d, wl.bs, wl.max_blocks,
                               pages_per_split=args.pages_per_split, workspace=ws["buf"])
        ws["buf"] = plan.workspace
        for layer in range(L):
            kc, vc = wl.k_pool[layer], wl.v_pool[layer]
            # one event pair per step, around all L layers after the plan: an
            # event node between two layers would keep the second launch from
            # starting early (programmatic dependent launch), so the per-layer
            # time is the bracket / L
            if ev_pairs is not None and layer == 0:
                ev_pairs[0][0].record()
            if args.separate_append:
                pkv.paged_kv_append(wl.k_new[layer], wl.v_new[layer], kc, vc, wl.block_tables, wl.ctx_pre)
            if args.separate_append:
                pkv.paged_attention_decode(wl.q[layer], kc, vc, wl.block_tables, wl.ctx, out=wl.out[layer],
                                           plan=plan, exact=args.exact)
            else:  # one launch: append the token at ctx - 1 and attend over ctx; every layer after the
                # first follows the previous layer's decode launch and may schedule its pages before it ends
                pkv.paged_attention_decode(wl.q[layer], kc, vc, wl.block_tables, wl.ctx, out=wl.out[layer],
                                           plan=plan, exact=args.exact, k_new=wl.k_new[layer],
                                           v_new=wl.v_new[layer], early_start=layer > 0)
            if ev_pairs is not None and layer == L - 1:
                ev_pairs[0][1].record()
        return plan

    step()
    torch.cuda.synchronize()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    # external events: inside a CUDA graph they become event-record nodes
    ev_all = [[[torch.cuda.Event(enable_timing=True, external=args.graph) for _ in range(2)]]
              for _ in range(args.steps)]  # one pair per step, around the L layers
    graph = None
    if args.graph:
        graph = capture_steps(lambda: [step(ev_all[s]) for s in range(args.steps)])
        graph.replay()  # untimed: the first launch also uploads the graph
        torch.cuda.synchronize()

    clocks = ClockSampler(physical_gpu(local))
    clocks.start()
    time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    if graph is not None:
        graph.replay()
    else:
        for s in range(args.steps):
            step(ev_all[s])
    t1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    ms_local = t0.elapsed_time(t1)
    ms = max_over_ranks(ms_local, world)
    layers_ms = [pairs[0][0].elapsed_time(pairs[0][1]) for pairs in ev_all]
    decode_avg_ms = sum(layers_ms) / len(layers_ms) / L  # mean launch (one layer) of the step
    rank_avg = [decode_avg_ms]
    if world > 1:  # per-rank step-time spread: every rank's mean layer time
        import torch.distributed as dist

        t = torch.zeros(world, dtype=torch.float64, device=device)
        t[rank] = ms_local / args.steps
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        rank_avg = [round(float(x), 4) for x in t.tolist()]

    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([float(B), float(wl.kv_read_bytes_layer() * L)], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        total_seqs, total_kv = int(t[0].item()), float(t[1].item())
    else:
        total_seqs, total_kv = B, float(wl.kv_read_bytes_layer() * L)
    ms_per_step = ms / args.steps
    value = total_seqs / (ms_per_step / 1e3)
    kv_gbs = total_kv / (ms_per_step / 1e3) / 1e9

    peak, peak_kind = measured_peaks()
    dec_bytes = wl.decode_bytes_layer() + (0 if args.separate_append else wl.append_bytes_layer())
    achieved = dec_bytes / (decode_avg_ms / 1e3) / 1e9
    chosen_pps = plan_pps(wl, args)  # the split length the plan kernel picked
    merges = 1 if wl.max_blocks > split_floor(wl, args) else 0  # split-K merge launch per layer
    traffic_ratio = DECODE_DRAM_TRAFFIC_RATIO.get(wl.config)
    launches = args.steps * (1 + ((2 if args.separate_append else 1) + merges) * L)

    # ---- end-to-end through the public ops with pinned host buffers
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, wl, world, device)

    # ---- CPU baseline (rank 0, N=1 only)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(wl, args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True,
            "scaling": args.scaling,
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic: seeded N(0,1) q/K/V/new tokens, seeded context lengths and random page permutations",
            "config": workload_config(args, world),
            "shard_of": args.shard_of or None,
            "run": {
                "pages_per_split": chosen_pps,
                "step": ("1 plan per step, then per layer one launch that appends the token and decodes (layers "
                         "after the first with early start: pages scheduled before the previous launch ends)"
                         if not args.separate_append else "1 plan per step, then per layer append + decode launches"),
                "launch": (f"the {args.steps} timed steps captured as one CUDA graph, replayed once (after "
                           f"{args.warmup} eager warm-up steps and one untimed replay)" if args.graph else
                           "eager launches from Python"),
                "softmax_weights": "16-bit hi+lo (exact)" if args.exact else "bf16",
            },
            "step_ms_per_rank": rank_avg if world > 1 else None,
            "kv_read_GBps": round(kv_gbs, 1),
            "kv_read_GBps_per_gpu": round(kv_gbs / world, 1),
            "roofline": {
                "kernel": ("decode_tc_kernel (one launch = one layer of all sequences"
                           + (")" if args.separate_append else ", append included)")),
                "bound": "hbm",
                "achieved": round(achieved, 1),
                "peak": peak,
                "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else peak_kind,
                "unit": "GB/s",
                "frac": round(achieved / peak, 4),
                "traffic": (args.traffic_bytes if args.traffic_bytes is not None else
                            (int(traffic_ratio * dec_bytes) if traffic_ratio else None)),
                "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of a one-launch "
                                   "capture of a reduced case of this config, scaled by pages read"
                                   if traffic_ratio else None),
                "algorithmic_bytes_per_launch": dec_bytes,
                "avg_launch_ms": round(decode_avg_ms, 4),
                "timing": (f"CUDA events around the {L} layers of every timed step (after its plan), "
                           f"divided by {L}" + (", split-K merge launches included" if merges else "")),
            },
            "gpu_launches": launches,
            "clocks": clk,
        }
        if wl.config == 3:
            line["unique_kv_GBps"] = round(kv_gbs * wl.unique_tokens / float(wl.ctx_post.sum()), 1)
        if e2e is not None:
            line["e2e"] = e2e
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)


def capture_steps(fn):
    """Capture the launches fn() makes on the current device into one CUDA graph.

    The library's entry points only enqueue kernels on torch's current stream
    (no allocation, no synchronisation when the plan workspace and outputs are
    passed in), so a decode step captures as-is."""
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    return graph


def plan_pps(wl, args) -> int:
    """Split length the plan kernel chose for this workload (read back from a plan)."""
    from grpo_training_engine_b200 import ops

    return ops.plan_decode(wl.ctx, wl.hq, wl.hkv, wl.d, wl.bs, wl.max_blocks,
                           pages_per_split=args.pages_per_split).chosen_pages_per_split()


def split_floor(wl, args) -> int:
    """Shortest split the plan may choose: the merge launch runs whenever a
    sequence can be longer than that (the workspace is sized for it)."""
    from grpo_training_engine_b200 import _lib

    lib = _lib.load()
    ws = lib.pkv_decode_workspace_size(wl.B, wl.hq, wl.hkv, wl.d, wl.max_blocks, args.pages_per_split)
    for p in range(8, 513, 8):  # the smallest length whose workspace equals the library's
        if lib.pkv_decode_workspace_size(wl.B, wl.hq, wl.hkv, wl.d, wl.max_blocks, p) == ws:
            return p
    return int(lib.pkv_decode_pages_per_split(wl.B, wl.hq, wl.hkv, wl.d, wl.max_blocks, args.pages_per_split))


def run_e2e(args, wl, world, device):
    """Same step through the public ops, with per-step inputs copied from pinned host
    memory (q, k_new, v_new of every layer, context lengths) and outputs copied back
    (fp32 attention output of every layer), inside the timed region."""
    import grpo_training_engine_b200 as pkv
    from grpo_training_engine_b200 import ops

    L = wl.layers
    # a layer's inputs (q, k_new, v_new) sit back to back in pinned host memory
    # and in device memory, so each layer's inputs cross PCIe in one copy
    qb, kb = wl.q[0].numel() * wl.q.element_size(), wl.k_new[0].numel() * wl.k_new.element_size()
    per = qb + 2 * kb
    in_h = torch.empty(L, per, dtype=torch.uint8).pin_memory()
    in_h[:, :qb] = wl.q.cpu().reshape(L, -1).view(torch.uint8)
    in_h[:, qb:qb + kb] = wl.k_new.cpu().reshape(L, -1).view(torch.uint8)
    in_h[:, qb + kb:] = wl.v_new.cpu().reshape(L, -1).view(torch.uint8)
    ctx_h = wl.ctx_post.clone().pin_memory()
    out_h = torch.empty(wl.out.shape, dtype=torch.float32).pin_memory()
    in_d = torch.empty(L, per, dtype=torch.uint8, device=device)
    q_d = [in_d[l, :qb].view(wl.q.dtype).view(wl.q.shape[1:]) for l in range(L)]
    kn_d = [in_d[l, qb:qb + kb].view(wl.k_new.dtype).view(wl.k_new.shape[1:]) for l in range(L)]
    vn_d = [in_d[l, qb + kb:].view(wl.v_new.dtype).view(wl.v_new.shape[1:]) for l in range(L)]
    ctx_d = [torch.empty_like(wl.ctx) for _ in range(2)]  # double-buffered across steps
    out_d = torch.empty_like(wl.out)
    copy = torch.cuda.Stream(device)  # host -> device
    back = torch.cuda.Stream(device)  # device -> host (the other PCIe direction, concurrently)
    h2d = [torch.cuda.Event() for _ in range(L)]
    done = [torch.cuda.Event() for _ in range(L)]
    d2h = [torch.cuda.Event() for _ in range(L)]
    ctx_ready = [torch.cuda.Event() for _ in range(2)]
    ctx_free = [torch.cuda.Event() for _ in range(2)]
    state = {"step": 0, "ws": None}

    def step(first: bool):
        comp = torch.cuda.current_stream(device)
        s = state["step"]
        state["step"] += 1
        buf = s % 2
        with torch.cuda.stream(copy):
            if s >= 2:
                copy.wait_event(ctx_free[buf])  # step s-2 finished reading this buffer
            ctx_d[buf].copy_(ctx_h, non_blocking=True)
            ctx_ready[buf].record(copy)
            for layer in range(L):
                if not first:
                    copy.wait_event(done[layer])  # previous step consumed this layer's inputs
                in_d[layer].copy_(in_h[layer], non_blocking=True)
                h2d[layer].record(copy)
        comp.wait_event(ctx_ready[buf])
        ctx = ctx_d[buf]
        ctx_pre = ctx - 1 if args.separate_append else None
        plan = ops.plan_decode(ctx, wl.hq, wl.hkv, wl.d, wl.bs, wl.max_blocks, pages_per_split=args.pages_per_split,
                               workspace=state["ws"])
        state["ws"] = plan.workspace
        for layer in range(L):
            comp.wait_event(h2d[layer])
            if not first:
                comp.wait_event(d2h[layer])  # previous step's output left the device
            kc, vc = wl.k_pool[layer], wl.v_pool[layer]
            if args.separate_append:
                pkv.paged_kv_append(kn_d[layer], vn_d[layer], kc, vc, wl.block_tables, ctx_pre)
                pkv.paged_attention_decode(q_d[layer], kc, vc, wl.block_tables, ctx, out=out_d[layer], plan=plan,
                                           exact=args.exact)
            else:
                pkv.paged_attention_decode(q_d[layer], kc, vc, wl.block_tables, ctx, out=out_d[layer], plan=plan,
                                           exact=args.exact, k_new=kn_d[layer], v_new=vn_d[layer],
                                           early_start=layer > 0)
            done[layer].record(comp)
            with torch.cuda.stream(back):
                back.wait_event(done[layer])
                out_h[layer].copy_(out_d[layer], non_blocking=True)
                d2h[layer].record(back)
        ctx_free[buf].record(comp)

    step(True)
    torch.cuda.synchronize()
    for _ in range(max(1, args.warmup)):
        step(False)
    torch.cuda.synchronize()
    graph = None
    if args.graph:
        state["step"] = 0

        def body():
            cap = torch.cuda.current_stream(device)
            copy.wait_stream(cap)  # fork the copy streams into the capture
            back.wait_stream(cap)
            for i in range(args.steps):
                step(i == 0)  # a replay starts after the previous one has finished
            cap.wait_stream(copy)  # and join them back
            cap.wait_stream(back)

        graph = capture_steps(body)
        graph.replay()
        torch.cuda.synchronize()
    comp = torch.cuda.current_stream(device)
    barrier(world)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(comp)
    if graph is not None:
        graph.replay()
    else:
        for _ in range(args.steps):
            step(False)
    comp.wait_stream(copy)
    comp.wait_stream(back)
    t1.record(comp)
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(t0.elapsed_time(t1), world) / args.steps
    ok = torch.allclose(out_h[0], wl.out[0].cpu())
    total = wl.n_total
    h2d_bytes = in_h.numel() + ctx_h.numel() * 4
    return {
        "value": round(total / (ms / 1e3), 2),
        "unit": UNIT,
        "h2d_bytes_per_step": int(h2d_bytes),
        "d2h_bytes_per_step": int(out_h.numel() * 4),
        "ms_per_step": round(ms, 4),
        "api": ("grpo_training_engine_b200.paged_kv_append + paged_attention_decode (C ABI pkv_append / "
                "pkv_decode_run)" if args.separate_append else
                "grpo_training_engine_b200.paged_attention_decode(k_new=, v_new=) (C ABI pkv_append_decode_run)"),
        "launch": ("the timed steps' copies and calls captured as one CUDA graph on three streams "
                   "(compute, host->device, device->host)" if graph is not None else
                   "eager launches from Python on three streams (compute, host->device, device->host)"),
        "output_matches_device_run": bool(ok),
    }


# ----------------------------------------------------------------------------- CPU baseline
def _cpu_sample(wl, n_seqs: int, seed: int = 0):
    """A bounded CPU copy of n_seqs sequences of one layer (pages copied into a small pool)."""
    rs = np.random.RandomState(seed)
    idx = rs.choice(wl.B, size=min(n_seqs, wl.B), replace=False)
    bt = wl.block_tables_cpu[idx]
    pages = torch.unique(bt)
    remap = torch.full((wl.num_blocks,), -1, dtype=torch.int32)
    remap[pages.long()] = torch.arange(len(pages), dtype=torch.int32)
    k = wl.k_pool[0, pages.to(wl.device).long()].cpu()
    v = wl.v_pool[0, pages.to(wl.device).long()].cpu()
    ctx = wl.ctx_post[idx]
    bt_small = remap[bt.long()]
    bt_small[bt_small < 0] = 0
    q = wl.q[0, idx.tolist()].cpu()
    kn = wl.k_new[0, idx.tolist()].cpu()
    vn = wl.v_new[0, idx.tolist()].cpu()
    return q, k, v, bt_small, ctx, kn, vn


def cpu_baseline(wl, seconds: float, nthreads: int = 0) -> dict:
    """Time the oracle (CPU restatement of the reference kernels) on a bounded sample
    of this workload: n sequences of one layer, append + 3-pass decode; scaled to
    seq-steps/s over all layers."""
    from oracle import oracle

    oracle.build()
    threads = nthreads or oracle.max_threads()
    n = 4
    while True:
        q, k, v, bt, ctx, kn, vn = _cpu_sample(wl, n)
        t = time.perf_counter()
        oracle.append(kn, vn, k, v, bt, ctx - 1)
        oracle.decode(q, k, v, bt, ctx, nthreads=threads)
        dt = time.perf_counter() - t
        if dt * 2 > seconds or n >= wl.B:
            break
        n = min(wl.B, max(n * 2, int(n * seconds / max(dt, 1e-3) * 0.5)))
    per_layer = dt / len(ctx)
    value = 1.0 / (per_layer * wl.layers)
    return {
        "value": round(value, 4),
        "unit": UNIT,
        "cores": threads,
        "kind": "port",
        "sample": f"{len(ctx)} of {wl.B} sequences x 1 of {wl.layers} layers (append + 3-pass decode, "
                  f"{dt:.1f} s), scaled linearly to all layers",
        "cpu": _cpu_name(),
    }


def _cpu_name() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ----------------------------------------------------------------------------- model-level rollout
def _profile_rollout_kernels(pkv, model, ids, kw, short=4, long_=24):
    """Kernel time per rollout step by kernel name: CUDA activity of rollouts of
    `short` and `long_` tokens under the torch profiler, difference / (long_ - short)."""
    import collections

    from torch.profiler import ProfilerActivity, profile

    mask = torch.ones_like(ids)
    pkv.paged_kv_decode(model, ids, mask, max_new_tokens=short, **kw)
    torch.cuda.synchronize()

    def kernel_times(n):
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            pkv.paged_kv_decode(model, ids, mask, max_new_tokens=n, **kw)
            torch.cuda.synchronize()
        tot, cnt = collections.Counter(), collections.Counter()
        for e in prof.events():
            if e.device_type == torch.autograd.DeviceType.CUDA:
                tot[e.name[:90]] += e.device_time_total
                cnt[e.name[:90]] += 1
        return tot, cnt

    t_s, c_s = kernel_times(short)
    t_l, c_l = kernel_times(long_)
    steps = long_ - short
    per = {k: (t_l[k] - t_s.get(k, 0)) / steps for k in t_l}
    total = sum(v for v in per.values() if v > 0)
    top = sorted(per.items(), key=lambda kv: -kv[1])[:16]
    return {"per_step_us": round(total, 1),
            "top": [{"kernel": k, "calls_per_step": (c_l[k] - c_s.get(k, 0)) / steps, "us_per_step": round(v, 1),
                     "share": round(v / total, 4)} for k, v in top]}


def run_rollout(args):
    """Model-level decode steps of paged_kv_decode (the trainer's rollout call) on the
    DeepSeek-R1-Distill-Qwen-1.5B geometry with random bf16 weights: eager steps vs
    steps replayed as one CUDA graph. Per-step time = difference of two rollouts of
    different lengths (the prefill and setup cancel), CUDA events, 1 GPU."""
    import grpo_training_engine_b200 as pkv
    from transformers import Qwen2Config, Qwen2ForCausalLM

    device = torch.device("cuda", 0)
    cfg = Qwen2Config(hidden_size=1536, intermediate_size=8960, num_hidden_layers=28, num_attention_heads=12,
                      num_key_value_heads=2, vocab_size=151936, max_position_embeddings=4096,
                      rope_theta=10000.0, tie_word_embeddings=True, attn_implementation="sdpa")
    torch.manual_seed(0)
    with torch.device(device):
        model = Qwen2ForCausalLM(cfg).to(torch.bfloat16).eval()
    batch, prompt = 128, 512
    ids = torch.randint(0, cfg.vocab_size, (batch, prompt), device=device)
    mask = torch.ones_like(ids)
    # long enough that the per-call graph capture (tens of ms) is small next to the steps
    short, long_ = 4, 4 + max(args.steps, 128)
    kw = dict(do_sample=True, temperature=0.7, top_p=0.9, seed=7, pad_token_id=0)

    def timed(n, graph, x=ids, share=True):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        pkv.paged_kv_decode(model, x, torch.ones_like(x), max_new_tokens=n, use_cuda_graph=graph,
                            share_prompt_pages=share, **kw)
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1)

    def per_step(graph, x=ids, share=True):
        # both lengths once untimed (allocator pools of both sizes, kernels loaded), then
        # five calls of each. The HF prefill of distinct prompts varies by up to ~0.3 s from
        # call to call, always upward (as much as 128 steps take), so each length's fastest
        # call is the one without that delay: the difference of the minima
        timed(short, graph, x, share)
        timed(long_, graph, x, share)
        pairs = [(timed(short, graph, x, share), timed(long_, graph, x, share)) for _ in range(5)]
        t_s = min(t for t, _ in pairs)
        ms = (min(t for _, t in pairs) - t_s) / (long_ - short)
        setup = t_s - short * ms
        return {"ms_per_step": round(ms, 3), "seq_steps_per_s": round(batch / ms * 1e3, 1),
                "setup_prefill_ms": round(setup, 2)}

    if args.profile_kernels:
        print(json.dumps(_profile_rollout_kernels(pkv, model, ids, kw)), flush=True)
        return
    res = {"graph" if graph else "eager": per_step(graph) for graph in (False, True)}
    # GRPO groups: 16 prompts x 8 responses (the trainer's expanded prompt per group):
    # one prefill per prompt and shared prompt pages, against every row prefilled
    # into private pages
    group = 8
    gids = torch.randint(0, cfg.vocab_size, (batch // group, prompt), device=device).repeat_interleave(group, 0)
    grouped = {"shared" if share else "private": per_step(True, gids, share) for share in (False, True)}
    print(json.dumps({
        "metric": "model-level rollout decode step (paged_kv_decode), seq-steps/s",
        "unit": "seq-steps/s",
        "n_gpus": 1,
        "data": "synthetic: random bf16 weights of the 1.5B geometry, random prompt ids",
        "config": {"model": "DeepSeek-R1-Distill-Qwen-1.5B geometry (28 L, hidden 1536, 12q/2kv, D 128, "
                            "vocab 151936), random weights", "batch": batch, "prompt_len": prompt,
                   "sampling": "temperature 0.7, top-p 0.9", "steps_timed": long_ - short},
        "eager": res["eager"], "graph": res["graph"],
        "speedup": round(res["eager"]["ms_per_step"] / res["graph"]["ms_per_step"], 3),
        "grpo_groups": {"prompts": batch // group, "group": group, **grouped},
    }), flush=True)


# ----------------------------------------------------------------------------- projection GEMM
def run_linear(args):
    """The projections of one layer of the 1.5B rollout step plus its LM head (128 rows, bf16) on
    pkv_linear against cuBLAS. Per shape, one call on each of n copies of the weights (n >= 4, the
    copies together > 3 x L2, so every call streams its weights from HBM) is captured as one CUDA
    graph and replayed back to back; time per call = the fastest of three replays / n (CUDA events),
    after --warmup eager calls. pkv_linear runs with PKV_LINEAR_WEIGHTS_STATIC, as in the rollout step; cuBLAS multiplies
    by an input-major copy (what the model path passes it), and the SiLU gate adds pkv_silu_mul."""
    from grpo_training_engine_b200 import ops

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    hid, inter, vocab, rows = 1536, 8960, 151936, 128
    shapes = [("qkv_bias", 2048, hid, True, False), ("o_proj", hid, hid, False, False),
              ("gate_up_silu", inter, hid, False, True), ("down", hid, inter, False, False),
              ("lm_head", vocab, hid, False, False)]
    out = []
    for name, n, k, with_bias, silu in shapes:
        wrows = 2 * n if silu else n
        wbytes = wrows * k * 2
        calls = max(4, math.ceil(3 * 126e6 / wbytes))  # copies together > 3 x L2
        ws = [(torch.randn(wrows, k, device=dev, generator=g) / k ** 0.5).to(torch.bfloat16) for _ in range(calls)]
        wts = [w.t().contiguous() for w in ws]
        x = torch.randn(rows, k, device=dev, generator=g).to(torch.bfloat16)
        b = torch.randn(n, device=dev, generator=g).to(torch.bfloat16) if with_bias else None
        o_ours = torch.empty(rows, n, dtype=torch.bfloat16, device=dev)

        def ours(i):
            ops.linear(x, ws[i], b, silu_gate=silu, out=o_ours, weights_static=True)

        def cublas(i):
            wt = wts[i]
            if silu:
                gu = x @ wt
                ops.silu_mul(gu[:, :n], gu[:, n:])
            elif b is not None:
                torch.addmm(b, x, wt)
            else:
                x @ wt

        times = {}
        for label, fn in (("ours", ours), ("cublas", cublas)):
            for i in range(args.warmup):
                fn(i)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for i in range(calls):
                    fn(i)
            best = float("inf")
            for _ in range(3):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                graph.replay()
                e1.record()
                torch.cuda.synchronize()
                best = min(best, e0.elapsed_time(e1) * 1e3 / calls)
            times[label] = best
            del graph
        out.append({"name": name, "n": n, "k": k, "weight_bytes": wbytes, "calls_per_replay": calls,
                    "ours_us": round(times["ours"], 2), "cublas_us": round(times["cublas"], 2),
                    "ours_GBps": round(wbytes / times["ours"] / 1e3, 1),
                    "cublas_GBps": round(wbytes / times["cublas"] / 1e3, 1)})
        del ws, wts
        torch.cuda.empty_cache()
    print(json.dumps({"metric": "projection GEMMs of the 1.5B rollout step (128 rows, bf16): us per call",
                      "unit": "us", "timing": "calls on distinct weight copies replayed back to back as one CUDA "
                      "graph; fastest of 3 replays / calls", "shapes": out}), flush=True)


# ----------------------------------------------------------------------------- sampling
def run_sample(args):
    """ops.sample_top_p on 128 rows of the 151,936-token vocabulary (temperature 0.7, top-p 0.9),
    bf16 and fp32 logits of three kinds (N(0, 9), N(0, 1), one peaked block over a low bulk): the
    default kernel path against the radix-select path (PKV_SAMPLE_FORCE_RADIX), CUDA events around
    one call (the draw of the uniforms included), median of --steps calls after --warmup; the two
    paths must give the same tokens."""
    from grpo_training_engine_b200 import ops

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    rows, vocab = 128, 151936
    kinds = {"normal_sd3": torch.randn(rows, vocab, device=dev, generator=g) * 3,
             "normal_sd1": torch.randn(rows, vocab, device=dev, generator=g),
             "peaked": torch.randn(rows, vocab, device=dev, generator=g) * 2 - 10}
    kinds["peaked"][:, :50] += torch.randn(rows, 50, device=dev, generator=g) * 3 + 20

    def median_us(fn, n):
        ts = []
        for i in range(args.warmup + n):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            if i >= args.warmup:
                ts.append(e0.elapsed_time(e1) * 1e3)
        return statistics.median(ts)

    out = []
    for name, x in kinds.items():
        for dt in (torch.bfloat16, torch.float32):
            logits = x.to(dt)
            fast = median_us(lambda: ops.sample_top_p(logits, 0.7, 0.9), args.steps)
            radix = median_us(lambda: ops.sample_top_p(logits, 0.7, 0.9, force_radix=True), max(3, args.steps // 4))
            a = ops.sample_top_p(logits, 0.7, 0.9, generator=torch.Generator(device=dev).manual_seed(2))
            b = ops.sample_top_p(logits, 0.7, 0.9, generator=torch.Generator(device=dev).manual_seed(2),
                                 force_radix=True)
            out.append({"logits": name, "dtype": str(dt).split(".")[1], "us": round(fast, 1),
                        "radix_us": round(radix, 1), "same_tokens": bool(torch.equal(a, b))})
    print(json.dumps({"metric": "top-p sampling of 128 x 151,936 logits (T 0.7, top-p 0.9): us per call",
                      "unit": "us", "timing": "CUDA events around one ops.sample_top_p call, median",
                      "results": out}), flush=True)


# ----------------------------------------------------------------------------- host cost of eager calls
def run_host(args):
    """Host-to-host cost of eager calls through the public API on a launch-bound case (8 sequences of
    64 tokens, 12q/2kv, D 128, bf16 cache, block size 16), where the GPU work of a call is a few µs:
    wall-clock time (time.perf_counter) around --steps x 100 back-to-back calls with one synchronize
    at the end, after --warmup x 100 calls; median of 5 such runs. Cases: the fused append + decode
    with a plan made once, the same with the plan made by the call, the decode alone, one step of the
    reference-facing low-level driver paged_kv_decode (fused append + decode, greedy pick, its per-step
    finished check; projections and logits precomputed), and a torch.add of two 8-element tensors for
    the scale of one torch launch."""
    from grpo_training_engine_b200 import paged_attention_decode, plan_decode
    from grpo_training_engine_b200.paged_kv import paged_kv_decode  # the low-level driver

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    b, hq, hkv, d, bs, ctx_len, new = 8, 12, 2, 128, 16, 64, 32
    max_blocks = (ctx_len + new) // bs + 1
    nblk = b * max_blocks
    kc = torch.randn(nblk, hkv, bs, d, device=dev, generator=g).to(torch.bfloat16)
    vc = torch.randn(nblk, hkv, bs, d, device=dev, generator=g).to(torch.bfloat16)
    bt = torch.arange(nblk, device=dev, dtype=torch.int32).reshape(b, max_blocks)
    ctx = torch.full((b,), ctx_len, dtype=torch.int32, device=dev)
    q = torch.randn(b, hq, d, device=dev, generator=g).to(torch.bfloat16)
    kn = torch.randn(b, hkv, d, device=dev, generator=g).to(torch.bfloat16)
    vn = torch.randn(b, hkv, d, device=dev, generator=g).to(torch.bfloat16)
    out = torch.empty(b, hq, d, device=dev)
    plan = plan_decode(ctx, hq, hkv, d, bs, max_blocks)
    logits = torch.randn(b, 1000, device=dev, generator=g)
    ids = torch.randint(0, 1000, (b, 1), device=dev, generator=g)
    s8 = torch.ones(8, device=dev)
    s8o = torch.empty(8, device=dev)

    def driver_step():
        paged_kv_decode(ids, kc, vc, bt, ctx, lambda t: (q, kn, vn), lambda a: logits, max_new_tokens=new,
                        do_sample=False)

    cases = [
        ("append_decode_plan_reused", 1, lambda: paged_attention_decode(q, kc, vc, bt, ctx, out=out, plan=plan,
                                                                         k_new=kn, v_new=vn)),
        ("append_decode_plan_per_call", 1, lambda: paged_attention_decode(q, kc, vc, bt, ctx, out=out,
                                                                           k_new=kn, v_new=vn)),
        ("decode_plan_reused", 1, lambda: paged_attention_decode(q, kc, vc, bt, ctx, out=out, plan=plan)),
        ("paged_kv_decode_step", new, driver_step),
        ("torch_add_8", 1, lambda: torch.add(s8, s8, out=s8o)),
    ]
    res = {}
    for name, per_call, fn in cases:
        calls = max(1, 100 // per_call)
        for _ in range(args.warmup * calls):
            fn()
        torch.cuda.synchronize()
        runs = []
        for _ in range(5):
            t0 = time.perf_counter()
            for _ in range(args.steps * calls):
                fn()
            torch.cuda.synchronize()
            runs.append((time.perf_counter() - t0) * 1e6 / (args.steps * calls * per_call))
        res[name] = round(statistics.median(runs), 2)
    print(json.dumps({"metric": "host-to-host time per eager call (launch-bound case), us", "unit": "us",
                      "case": f"{b} seqs x {ctx_len} tokens, {hq}q/{hkv}kv, D {d}, bf16, bs {bs}",
                      "timing": "perf_counter around back-to-back calls, one synchronize, median of 5",
                      "results": res}), flush=True)


# ----------------------------------------------------------------------------- reference arm
def run_reference(args, rank, world):
    """CPU restatement of the reference algorithm on the host cores (the reference is
    Python/Triton and has no CPU implementation; its kernels only run in Triton's
    interpreter, which needs the reference checkout and takes ~12 s per config-1 call)."""
    if rank != 0:
        return
    from oracle import oracle

    oracle.build()
    threads = oracle.max_threads()
    c = dict(CONFIGS[args.config])
    if args.seqs:
        c["seqs"] = args.seqs
    # the rank-0 shard's lengths of the same workload, on the CPU without a GPU pool
    world = max(world, 1)
    lens = global_lengths(args.config, c["seqs"] if args.scaling == "strong" else c["seqs"] * world)
    mine = shard_indices(args.config, lens, 0, world)
    layers = args.layers or c["layers"]
    hq, hkv, d, bs = c["hq"], c["hkv"], c["d"], c["bs"]
    rs = np.random.RandomState(5)

    def sample(n):
        idx = rs.choice(len(mine), size=min(n, len(mine)), replace=False)
        ctx = torch.tensor([int(lens[mine[i]]) for i in idx], dtype=torch.int32)
        pages = [(int(x) + bs - 1) // bs for x in ctx]
        nb = sum(pages)
        perm = torch.randperm(nb, generator=torch.Generator().manual_seed(int(rs.randint(1 << 30))))
        mb = max(pages)
        bt = torch.zeros(len(idx), mb, dtype=torch.int32)
        off = 0
        for i, p in enumerate(pages):
            bt[i, :p] = perm[off:off + p].int()
            off += p
        g = torch.Generator().manual_seed(int(rs.randint(1 << 30)))
        k = torch.randn(nb, hkv, bs, d, generator=g).to(torch.bfloat16)
        v = torch.randn(nb, hkv, bs, d, generator=g).to(torch.bfloat16)
        q = torch.randn(len(idx), hq, d, generator=g).to(torch.bfloat16)
        kn = torch.randn(len(idx), hkv, d, generator=g).to(torch.bfloat16)
        vn = torch.randn(len(idx), hkv, d, generator=g).to(torch.bfloat16)
        return q, k, v, bt, ctx, kn, vn

    def run(s):
        q, k, v, bt, ctx, kn, vn = s
        t = time.perf_counter()
        oracle.append(kn, vn, k, v, bt, ctx - 1)
        oracle.decode(q, k, v, bt, ctx, nthreads=threads)
        return time.perf_counter() - t

    # size one step's sample to ~target seconds of CPU work, build it once,
    # then time every step on it (the data does not change the work)
    n = max(1, threads // 2)
    while True:
        smp = sample(n)
        dt = run(smp)
        if dt >= args.ref_step_seconds * 0.5 or n >= len(mine):
            break
        n = min(len(mine), max(n + 1, int(n * args.ref_step_seconds / max(dt, 1e-3))))
    for _ in range(args.warmup):
        run(smp)
    times, seqs = [], 0
    for _ in range(args.steps):
        times.append(run(smp))
        seqs += len(smp[4])
    total = sum(times)
    value = seqs / (total * layers)
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 4),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(1e3 * total / args.steps, 3),
        "higher_is_better": True,
        "scaling": args.scaling,
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: seeded N(0,1) q/K/V/new tokens, seeded context lengths and random page permutations",
        "config": workload_config(args, world),
        "cpu_baseline": {
            "value": round(value, 4),
            "unit": UNIT,
            "cores": threads,
            "kind": "port",
            "sample": f"each step: {n} sequences of the rank-0 shard x 1 layer (append + 3-pass decode), "
                      f"seq-steps/s scaled to {layers} layers",
            "cpu": _cpu_name(),
        },
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=4, choices=sorted(CONFIGS))
    ap.add_argument("--layers", type=int, default=None, help="override the layer count (diagnostics only)")
    ap.add_argument("--seqs", type=int, default=None,
                    help="override the sequence count (in all with strong scaling, per GPU with weak; diagnostics)")
    ap.add_argument("--shard-of", type=int, default=0,
                    help="diagnostics on one GPU: run rank 0's shard of an N-GPU job (the JSON line then "
                         "describes that shard, not a whole job)")
    ap.add_argument("--scaling", choices=["strong", "weak"], default="strong",
                    help="strong: the config's sequences split over the GPUs (BASELINE's statement of the configs); "
                         "weak: every GPU gets the config's full sequence count")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--pages-per-split", type=int, default=0)
    ap.add_argument("--exact", action="store_true", help="decode with PKV_DECODE_EXACT_P")
    ap.add_argument("--no-graph", dest="graph", action="store_false",
                    help="launch every kernel from Python instead of replaying a CUDA graph of the timed steps")
    ap.add_argument("--separate-append", action="store_true",
                    help="append with its own launch (pkv_append) instead of inside the decode launch")
    ap.add_argument("--profile-kernels", action="store_true",
                    help="with --rollout: per-kernel time of one graph-replayed step (torch profiler)")
    ap.add_argument("--rollout", action="store_true",
                    help="time the model-level rollout step (eager vs CUDA graph) instead of the decode path")
    ap.add_argument("--linear", action="store_true",
                    help="time the projection GEMM (pkv_linear) against cuBLAS on the rollout step's shapes")
    ap.add_argument("--sample", action="store_true",
                    help="time the top-p sampling kernels (bf16 and fp32 logits) against the radix path")
    ap.add_argument("--host", action="store_true",
                    help="host-to-host time per eager call of the decode API on a launch-bound case")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--ref-step-seconds", type=float, default=1.0)
    ap.add_argument("--traffic-bytes", type=float, default=None,
                    help="DRAM bytes per decode launch from an ncu capture, reported as roofline.traffic")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.rollout:
        run_rollout(args)
        return
    if args.linear:
        run_linear(args)
        return
    if args.sample:
        run_sample(args)
        return
    if args.host:
        run_host(args)
        return
    rank, world, local = dist_setup(args)
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    try:
        run_ours(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
