#!/usr/bin/env python
"""Benchmark of the MoE verification path on B200.

Default workload: a 48-layer Qwen3-30B-A3B-shaped
target with random-init bf16 N(0, 0.02) weights, a 512-token context of
uniform random token ids, and one verify pass per step over a seeded 64-node
draft tree (depth 6, branching <= 4) with its ancestor attention mask; 24
expert-cache slots per layer backed by a page-locked host copy of all
experts.  One step = one verify forward pass (65 query rows) + greedy
acceptance + KV-cache rollback to the context.

Reported (one JSON line, rank 0):
  value      committed tokens/s with the step inputs already on the device
             (committed = accepted path + 1; random weights accept nothing,
             so one token per verify pass), summed over ranks: device-managed
             expert caches (misses planned and filled on the GPU), the verify
             pass replayed from one CUDA graph, expert-id-ascending execution;
  e2e        the same with the step's inputs copied from pinned host memory
             into the graph's buffers and the argmax read back;
  other_policy / host_managed  the resident-first policy, and the
             reference's host-managed protocol (eager, copy-engine fills);
  resident   the same pass with 128 slots per layer (every expert resident);
  moe_block  the MoE verify block of layer 0 alone, one CUDA graph per block,
             L2 flushed between replays;
  roofline   the grouped SwiGLU kernel against the measured HBM copy peak,
             and (``h2d``) the headline's fill bytes per step against the
             pinned-copy peak measured in the same run;
  config1 / config3 / config4 / config5_anchor  the other BASELINE
             configurations (fp32 0-slot block; slot sweep; end-to-end
             speculative decoding; configuration 5's workload on one GPU);
  cpu_baseline  a bounded sample of the reference's CPU path (stock Hugging
             Face Qwen3-MoE on the host cores; ``--impl reference`` times the
             whole 48-layer model).

Multi-GPU (torchrun, N > 1): configuration 5, expert-parallel over the ranks
(``ep_arm``, "scaling": strong); ``--impl reference`` times the reference's
CPU path on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

EXPERT_BYTES = 3 * 2048 * 768 * 2  # one packed bf16 expert slot
# DRAM bytes (read + write) per active expert of one grouped SwiGLU call
# (both phases), from an ncu capture of that kernel at 65 token rows over 127
# active experts: 801.3 + 5.7 + 400.4 + 5.9 MB.  The roofline's `traffic`
# scales it by the experts a launch processes, and only at the captured row
# count (the activation bytes per expert change with the rows).
SWIGLU_CAPTURE_ROWS = 65
SWIGLU_DRAM_BYTES_PER_EXPERT = (801.3e6 + 5.7e6 + 400.4e6 + 5.9e6) / 127


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=("b200", "reference"), default="b200")
    p.add_argument("--slots", type=int, default=24)
    p.add_argument("--policy", choices=("expert_id_ascending", "resident_first"),
                   default="expert_id_ascending",
                   help="expert execution policy of the headline passes (the other one is also timed)")
    p.add_argument("--layers", type=int, default=48)
    p.add_argument("--ctx", type=int, default=512)
    p.add_argument("--nodes", type=int, default=64)
    p.add_argument("--depth", type=int, default=6)
    p.add_argument("--branch", type=int, default=4)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--no-resident", action="store_true", help="skip the 128-slot variant")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-extras", action="store_true",
                   help="skip the configuration 1, 3 and 4 measurements of the default line")
    p.add_argument("--cpu-layers", type=int, default=1, help="decoder layers timed on the CPU")
    p.add_argument("--mode", choices=("auto", "verify", "ep", "decode", "block", "graph", "sweep",
                                      "kernels"),
                   default="auto",
                   help="auto: verify on one GPU, ep under torchrun with N > 1; verify: BASELINE "
                        "config 2; ep: config 5 (8 requests, experts sharded over the ranks); "
                        "decode: config 4 (end-to-end speculative decoding with a drafter stand-in "
                        "and SpecFit selection); "
                        "block: the MoE verify block alone on one resident layer; graph: only the "
                        "resident (128-slot) verify pass replayed from a CUDA graph; sweep: config 3 "
                        "(12/24/48/128 slots, cold and warm, Zipf routes, a 128-node tree); kernels: each "
                        "hot kernel alone at the configurations' sizes, L2 cold and warm")
    p.add_argument("--requests", type=int, default=8, help="--mode ep: concurrent requests in total")
    p.add_argument("--ep-ctx", type=int, default=4096, help="--mode ep: context tokens per request")
    p.add_argument("--decode-ctx", type=int, default=2048, help="--mode decode: context tokens")
    p.add_argument("--new-tokens", type=int, default=256, help="--mode decode: tokens to generate")
    p.add_argument("--hf-forward", action="store_true",
                   help="run the Hugging Face layer forward instead of the lean fused forward")
    p.add_argument("--eager-decode", action="store_true",
                   help="--mode decode: verify passes without CUDA graphs")
    p.add_argument("--sweep-slots", default="12,24,48,128", help="--mode sweep: slots per layer")
    p.add_argument("--sweep-nodes", type=int, default=128, help="--mode sweep: tree nodes")
    p.add_argument("--sweep-depth", type=int, default=8, help="--mode sweep: tree depth")
    p.add_argument("--tokens", type=int, default=65, help="rows per MoE block in --mode block")
    p.add_argument("--routes", choices=("router", "zipf", "uniform"), default="router",
                   help="--mode block: routes from the router, Zipf(1.1) or uniform top-8")
    p.add_argument("--fused-gather", action="store_true",
                   help="resident expert path: token rows read inside the grouped SwiGLU (TMA gather4)")
    p.add_argument("--kernel", default="",
                   help="--mode kernels: comma-separated kernel names to run (default: all)")
    p.add_argument("--kernel-rows", default="7,65,512",
                   help="--mode kernels: the row counts of the per-token cases (router ... grouped_swiglu)")
    return p.parse_args(argv)


# ----------------------------------------------------------------- helpers


def dist_info():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def measured_peaks() -> dict:
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": float(data["hbm_gbs"]), "bf16_tflops": float(data["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def pinned_h2d_peak(pool, device, slots: int = 48, reps: int = 3) -> dict:
    """Host-to-device copy rate of this box for the cache's fill pattern:
    ``slots`` back-to-back copies of one packed expert (9,437,184 B) from the
    page-locked expert pool into a device buffer on a side stream, CUDA
    events, best of ``reps``."""
    src = pool.data[0]
    n = min(slots, src.shape[0])
    dst = torch.empty(n, src.shape[1], dtype=src.dtype, device=device)
    stream = torch.cuda.Stream(device)
    best = None
    with torch.cuda.stream(stream):
        for _ in range(reps + 1):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for i in range(n):
                dst[i].copy_(src[i], non_blocking=True)
            b.record(stream)
            b.synchronize()
            ms = a.elapsed_time(b)
            best = ms if best is None else min(best, ms)
    nbytes = n * src.shape[1] * src.element_size()
    del dst
    return {"GBps": round(nbytes / (best * 1e-3) / 1e9, 2), "bytes": nbytes,
            "how": f"{n} copies of one packed expert from the page-locked pool, best of {reps}"}


def h2d_roofline_of(per_step: dict, ms_per_step: float, peak: dict) -> dict:
    """H2D roofline of a cache-bound step: expert fill bytes per step (H2D
    submissions x 9,437,184 B) over the step time, against the pinned-copy
    rate measured in the same run."""
    nbytes = per_step["h2d_submissions"] * EXPERT_BYTES
    achieved = nbytes / (ms_per_step * 1e-3) / 1e9
    return {"bound": "h2d", "fills_per_step": per_step["h2d_submissions"],
            "bytes_per_step": int(nbytes), "achieved": round(achieved, 2), "peak": peak["GBps"],
            "unit": "GB/s", "frac": round(achieved / peak["GBps"], 4),
            "floor_ms": round(nbytes / (peak["GBps"] * 1e9) * 1e3, 3), "peak_source": peak["how"]}


class ClockSampler:
    """nvidia-smi clock/throttle samples while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        if self.proc is None or self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.file.flush()
        rows = [r.split(",") for r in Path(self.file.name).read_text().splitlines() if r.strip()]
        os.unlink(self.file.name)
        sm, smax, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            try:
                sm.append(float(r[1]))
                smax.append(float(r[2]))
            except (ValueError, IndexError):
                continue
            for name, val in zip(names, r[5:9]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "samples": len(sm), "reasons": sorted(reasons)}


def workload_tree(nodes, depth, branch, seed, vocab):
    """The benchmark's seeded draft tree, shared by both arms: parents precede
    children (1-based ids, 0 = the pending seed), depth <= ``depth``, at most
    ``branch`` children per node, distinct sibling tokens, later nodes
    preferred as parents so the tree reaches its depth.  Returns
    ``(token_ids, parent_ids, depths)``; equals
    ``specfit_b200.synthetic.random_tree`` (checked by a CPU test) but lives
    here so the reference arm imports nothing from the package."""
    rng = np.random.default_rng(seed)
    parents, depths, tokens = [], [], []
    child_count, node_depth, siblings = {0: 0}, {0: 0}, {0: set()}
    while len(parents) < nodes:
        cands = [n for n in range(len(parents) + 1) if node_depth[n] < depth and child_count[n] < branch]
        if not cands:
            raise ValueError("tree shape cannot hold that many nodes")
        w = np.array([1.0 + n for n in cands], dtype=np.float64)
        parent = int(rng.choice(cands, p=w / w.sum()))
        node = len(parents) + 1
        tok = int(rng.integers(0, vocab))
        while tok in siblings[parent]:
            tok = int(rng.integers(0, vocab))
        siblings[parent].add(tok)
        parents.append(parent)
        depths.append(node_depth[parent] + 1)
        tokens.append(tok)
        child_count[parent] += 1
        child_count[node] = 0
        node_depth[node] = node_depth[parent] + 1
        siblings[node] = set()
    return tuple(tokens), tuple(parents), tuple(depths)


def make_tree(nodes, depth, branch, seed, vocab):
    from specfit_b200.runtime.eagle3_types import Eagle3DraftTree

    tok, par, dep = workload_tree(nodes, depth, branch, seed, vocab)
    rng = np.random.default_rng(seed)
    cond, cum = [], []
    for p in par:
        c = float(rng.uniform(0.05, 1.0))
        cond.append(c)
        cum.append((0.0 if p == 0 else cum[p - 1]) + math.log(c))
    return Eagle3DraftTree(tok, par, dep, tuple(cond), tuple(cum))


def reference_config(layers: int):
    """Qwen3-30B-A3B shape built from transformers alone (48 layers, hidden
    2048, 128 experts top-8, moe_intermediate 768, 32/4 heads of 128, vocab
    151,936, RoPE theta 1e6, RMSNorm eps 1e-6); the B200 arm's
    ``qwen3_moe_config`` gives the same values (checked by a CPU test)."""
    from transformers import Qwen3MoeConfig

    return Qwen3MoeConfig(
        vocab_size=151936, hidden_size=2048, intermediate_size=6144, num_hidden_layers=layers,
        num_attention_heads=32, num_key_value_heads=4, head_dim=128, max_position_embeddings=40960,
        rms_norm_eps=1e-6, rope_parameters={"rope_type": "default", "rope_theta": 1000000.0},
        tie_word_embeddings=False, moe_intermediate_size=768, num_experts=128, num_experts_per_tok=8,
        norm_topk_prob=True, decoder_sparse_step=1, mlp_only_layers=[], attention_bias=False)


def headline_config(args) -> dict:
    """The workload description both arms print (identical by construction)."""
    return {
        "workload": (f"BASELINE config 2: {args.layers}-layer Qwen3-30B-A3B-shaped verify pass over a "
                     f"{args.nodes}-node tree (depth {args.depth}, branching <= {args.branch}), "
                     f"{args.ctx}-token context, {args.slots} expert-cache slots per layer"),
        "verify_tokens_per_step": 1 + args.nodes,
        "slots_per_layer": args.slots,
        "parallelism": "single GPU",
        "l2_flush": "not needed: each step streams > 57 GB of expert weights (>> 126 MB L2)",
    }


# --------------------------------------------------------------- B200 arm


def make_forward(model, hf: bool):
    """The target forward the runners call: the lean fused forward by
    default, the stock Hugging Face forward with ``--hf-forward``."""
    if hf:
        return model
    from specfit_b200.runtime.lean_forward import LeanQwen3Forward

    return LeanQwen3Forward(model)


def apply_kernel_options(loaded, args) -> None:
    """``--fused-gather``: every layer's resident expert path reads its token
    rows inside the grouped SwiGLU (TMA gather4) instead of gathering them
    first."""
    if getattr(args, "fused_gather", False):
        for layer in loaded.model.model.layers:
            layer.mlp.experts.fused_gather = True


class VerifyRunner:
    def __init__(self, loaded, ctx_ids, tree, seed_tok, device, fwd=None):
        from specfit_b200.runtime.kv_cache import ReservedCache

        self.loaded = loaded
        self.model = loaded.model
        self.fwd = fwd if fwd is not None else self.model
        self.tree = tree
        self.device = device
        self.ctx = ctx_ids.shape[1]
        self.cache = ReservedCache(config=self.model.config, capacity=self.ctx + 1 + tree.draft_node_count)
        with torch.no_grad():
            self.fwd(input_ids=ctx_ids, past_key_values=self.cache, use_cache=True)
        seed = torch.tensor([[seed_tok]])
        self.h_ids = tree.verification_token_ids(seed).pin_memory()
        self.h_mask = tree.verification_attention_mask(base_kv_length=self.ctx, device="cpu").pin_memory()
        self.h_pos = tree.verification_position_ids(base_kv_length=self.ctx, device="cpu").pin_memory()
        self.d_ids = self.h_ids.to(device)
        self.d_mask = self.h_mask.to(device)
        self.d_pos = self.h_pos.to(device)

    def step_device(self):
        """Inputs already on the device; returns the device argmax."""
        with torch.no_grad():
            out = self.fwd(input_ids=self.d_ids, attention_mask=self.d_mask, position_ids=self.d_pos,
                           past_key_values=self.cache, use_cache=True)
            am = out.logits[0].argmax(-1)
        self.cache.crop(self.ctx)
        return am

    def step_e2e(self) -> int:
        """Host inputs in, accepted path out; returns committed tokens."""
        ids = self.h_ids.to(self.device, non_blocking=True)
        mask = self.h_mask.to(self.device, non_blocking=True)
        pos = self.h_pos.to(self.device, non_blocking=True)
        with torch.no_grad():
            out = self.fwd(input_ids=ids, attention_mask=mask, position_ids=pos,
                           past_key_values=self.cache, use_cache=True)
            am = out.logits[0].argmax(-1).cpu().unsqueeze(0)
        self.cache.crop(self.ctx)
        return len(self.tree.accepted_path(am)) + 1

    @property
    def h2d_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.h_ids, self.h_mask, self.h_pos))

    @property
    def d2h_bytes(self) -> int:
        return self.h_ids.numel() * 8


def timed_steps(fn, steps, warmup, world, device, on_start=None, label: str = "timed"):
    """W untimed then K timed calls of ``fn`` between barriers and device
    synchronisations, CUDA events on the current stream; ``on_start`` (if
    given) runs after the warm-up, outside the timed region.  Returns the
    max over ranks of the timed milliseconds and ``fn``'s results."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(device)
    barrier(world)
    if on_start is not None:
        on_start()
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    results = []
    torch.cuda.nvtx.range_push(label)
    start.record()
    for _ in range(steps):
        results.append(fn())
    end.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize(device)
    barrier(world)
    ms = start.elapsed_time(end)
    return max_over_ranks(ms, world, device), results


def moe_block_profile(runner, layers_to_time=None):
    """Per-layer MoE block time (CUDA events around every layer.mlp) over one
    verify pass, and the distinct experts each layer touched."""
    model = runner.model
    starts, ends, active = {}, {}, {}
    hooks = []
    for i, layer in enumerate(model.model.layers):
        def pre(mod, args, i=i):
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            starts[i] = e

        def post(mod, args, out, i=i):
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            ends[i] = e

        def gate_hook(mod, args, out, i=i):
            active[i] = out[2]

        hooks += [layer.mlp.register_forward_pre_hook(pre), layer.mlp.register_forward_hook(post),
                  layer.mlp.gate.register_forward_hook(gate_hook)]
    try:
        runner.step_device()
        torch.cuda.synchronize()
    finally:
        for h in hooks:
            h.remove()
    times = [starts[i].elapsed_time(ends[i]) for i in sorted(starts)]
    uniq = [int(torch.unique(active[i]).numel()) for i in sorted(active)]
    return times, uniq


def swiglu_roofline(loaded, device, tokens, peaks, iters=20):
    """Time the grouped SwiGLU kernel alone on layer 0's resident slots."""
    from specfit_b200 import ops

    layer = loaded.model.model.layers[0]
    experts = layer.mlp.experts
    cache = experts.cache
    table = cache.device_slot_table(experts._keys)
    if table is None:
        return None
    g = torch.Generator(device=device).manual_seed(5)
    x = (torch.randn(tokens, 2048, generator=g, device=device)).to(torch.bfloat16)
    _, w, idx = layer.mlp.gate(x)
    d = ops.moe_dispatch(idx, experts.num_experts)
    xs, ws = ops.moe_gather(x, w, d)
    storage = cache.storage.view(cache.slot_count, -1)
    act = torch.empty(xs.shape[0], 768, dtype=torch.bfloat16, device=device)
    ys = torch.empty(xs.shape[0], 2048, dtype=torch.bfloat16, device=device)
    run = lambda: ops.grouped_swiglu(xs, ws, d, table, storage, 2048, 768, act_workspace=act, out=ys)
    for _ in range(3):
        run()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        run()
    e.record()
    torch.cuda.synchronize()
    us = s.elapsed_time(e) * 1e3 / iters
    uniq = int(d.num_active.item())
    rows = xs.shape[0]
    algo = uniq * EXPERT_BYTES + rows * 2048 * 2 * 2 + rows * 768 * 2 * 2 + rows * 4
    achieved = algo / (us * 1e-6) / 1e9
    return {"bound": "hbm", "kernel": "swiglu_tc_kernel (phase 1 + 2)", "achieved": round(achieved, 1),
            "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
            "traffic": (round(SWIGLU_DRAM_BYTES_PER_EXPERT * uniq) if tokens == SWIGLU_CAPTURE_ROWS
                        else None),
            "traffic_source": ("estimated, not measured in this run: ncu dram__bytes_read+write per "
                               "expert of a capture at 65 rows x 127 experts, times this launch's "
                               "experts" if tokens == SWIGLU_CAPTURE_ROWS else
                               f"null: the ncu capture was taken at {SWIGLU_CAPTURE_ROWS} rows, not {tokens}"),
            "launch_us": round(us, 2), "experts": uniq, "tokens": tokens,
            "algorithmic_bytes": algo, "peak_source": peaks["source"] + " hbm_gbs (burst copy)"}


def moe_block_graph(loaded, device, tokens, peaks, reps=20, warmup=3):
    """The MoE verify block of layer 0 on the device alone: router, dispatch,
    gather, grouped SwiGLU over the layer's resident slots and combine,
    captured as one CUDA graph and timed by CUDA events around each replay,
    with L2 flushed (a 256 MB write, outside the events) before every replay.
    The rows are N(0,1), which the random router spreads over nearly every
    expert -- the full-coverage case of the per-expert byte count.
    Algorithmic bytes = distinct experts x one packed slot + the router
    weight + the input rows read + the output rows written."""
    from specfit_b200 import ops

    layer = loaded.model.model.layers[0]
    experts = layer.mlp.experts
    gate = layer.mlp.gate
    cache = experts.cache
    table = cache.device_slot_table(experts._keys)
    if table is None:
        return None
    hidden, inter, num_experts = experts.hidden_size, experts.intermediate_size, experts.num_experts
    g = torch.Generator(device=device).manual_seed(7)
    x = torch.randn(tokens, hidden, generator=g, device=device).to(torch.bfloat16)
    storage = cache.storage.view(cache.slot_count, -1)

    def block():
        _, w, idx = ops.router_topk(x, gate.weight, gate.top_k, gate.norm_topk_prob)
        d = ops.moe_dispatch(idx, num_experts)
        xs, ws = ops.moe_gather(x, w, d)
        ys = ops.grouped_swiglu(xs, ws, d, table, storage, hidden, inter)
        return ops.moe_combine(ys, d, idx), d

    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        for _ in range(2):
            block()
    torch.cuda.current_stream(device).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        _, d = block()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    pairs = []
    for r in range(warmup + reps):
        flush.fill_(r & 0xFF)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        graph.replay()
        b.record(stream)
        if r >= warmup:
            pairs.append((a, b))
    torch.cuda.synchronize(device)
    us = [a.elapsed_time(b) * 1e3 for a, b in pairs]
    uniq = int(d.num_active.item())
    del graph
    med = statistics.median(us)
    algo = uniq * EXPERT_BYTES + num_experts * hidden * 2 + 2 * tokens * hidden * 2
    achieved = algo / (med * 1e-6) / 1e9
    return {"us_per_block_median": round(med, 2), "us_per_block_min": round(min(us), 2),
            "replays": reps, "tokens": tokens, "experts": uniq, "algorithmic_bytes": algo,
            "achieved_GBps": round(achieved, 1), "peak_GBps": peaks["hbm_gbs"],
            "frac_of_hbm_peak": round(achieved / peaks["hbm_gbs"], 4),
            "peak_source": peaks["source"] + " hbm_gbs (burst copy)",
            "launch": "one CUDA graph per block (router, dispatch, gather, grouped SwiGLU, combine)",
            "l2": "flushed before each replay (256 MB write outside the timed events)"}


def reference_model(cfg, seed: int, std: float = 0.02):
    """Stock Hugging Face ``Qwen3MoeForCausalLM`` on the host, bf16, every
    linear weight N(0, std) and every norm weight 1 (the B200 arm's
    initialisation; the draws differ, the distribution is the same).  Built
    on the meta device and allocated in bf16 so no fp32 copy of the model is
    ever held; weights are drawn in fp32 chunks of at most 64 Mi elements."""
    from transformers import Qwen3MoeForCausalLM

    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device("meta"):
            model = Qwen3MoeForCausalLM(cfg)
    finally:
        torch.set_default_dtype(prev)
    model.to_empty(device="cpu")
    gen = torch.Generator().manual_seed(seed)
    chunk = 1 << 26
    with torch.no_grad():
        for name, p in model.named_parameters():
            flat = p.data.view(-1)
            if "norm" in name:
                flat.fill_(1.0)
                continue
            for i in range(0, flat.numel(), chunk):
                part = flat[i:i + chunk]
                part.copy_(torch.randn(part.numel(), generator=gen).mul_(std))
    model.model.rotary_emb = type(model.model.rotary_emb)(config=cfg)  # fp32 frequencies
    model.requires_grad_(False)
    return model.eval()


def reference_model_bytes(layers: int) -> int:
    """bf16 bytes of ``reference_model`` at the Qwen3-30B-A3B shape."""
    per_layer = (128 * 3 * 2048 * 768 + 128 * 2048 + (32 + 2 * 4) * 128 * 2048 + 2048 * 32 * 128
                 + 2 * 128 + 2 * 2048)
    return 2 * (layers * per_layer + 2 * 151936 * 2048 + 2048)


def config1_block(device, h2d_peak_gbps=None, reps: int = 5, cpu_reps: int = 3) -> dict:
    """BASELINE configuration 1 on the GPU: one fp32 MoE block (router +
    experts + combine), 32 tokens, the seed-0 draw of
    ``synthetic.config1_inputs``, with "0 slots": the cache's contents are
    invalidated before every block (``GpuExpertCache.invalidate_contents``,
    the reference's ``discard_completed_experts``), so every selected expert
    is streamed from page-locked host memory on every call.  Host-managed
    (copy-engine fills) and device-managed (kernel fills, no host round
    trip) blocks are timed with CUDA events; the output is compared with the
    reference-generated golden of the same input.  The CPU baseline is the
    stock Hugging Face ``Qwen3MoeSparseMoeBlock`` in fp32 with the same
    weights on all host cores."""
    from transformers import Qwen3MoeConfig
    from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeSparseMoeBlock

    from specfit_b200 import ops, synthetic
    from specfit_b200.runtime import ExpertKey, GpuExpertCache, Qwen3OffloadedExperts
    from specfit_b200.runtime.qwen3_verifier import ExpertHostPool

    weights, x = synthetic.config1_inputs(seed=0, tokens=32)
    E, H, I = weights.router.shape[0], weights.router.shape[1], weights.down.shape[2]
    pool = ExpertHostPool(1, E, 3 * H * I, dtype=torch.float32)
    for e in range(E):
        pool.data[0, e].copy_(weights.packed(e))
    cache = GpuExpertCache({ExpertKey(0, e): pool.data[0, e] for e in range(E)}, slot_count=E, device=device,
                           adopt_pinned_sources=True)
    experts = Qwen3OffloadedExperts(layer_id=0, cache=cache, hidden_size=H, intermediate_size=I)
    xd, wr = x.to(device), weights.router.to(device)

    def block():
        _, w, idx = ops.router_topk(xd, wr, 8, True)
        return experts(xd, idx, w)

    rows = {}
    out = None
    for mode in ("host", "device"):
        times, fills = [], []
        for i in range(reps + 1):
            torch.cuda.synchronize()
            if cache.device_managed:
                cache.leave_device_mode()
            cache.invalidate_contents()
            if mode == "device":
                cache.enter_device_mode()
            before = cache.stats().h2d_submissions
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            out = block()
            b.record()
            b.synchronize()
            if i:
                times.append(a.elapsed_time(b))
                fills.append(cache.stats().h2d_submissions - before)
        ms = statistics.median(times)
        nbytes = statistics.median(fills) * 3 * H * I * 4
        rows[mode] = {"block_ms": round(ms, 3), "fills_per_block": statistics.median(fills),
                      "h2d_bytes": int(nbytes), "h2d_GBps": round(nbytes / (ms * 1e-3) / 1e9, 2)}
        if h2d_peak_gbps:
            rows[mode]["h2d_frac"] = round(nbytes / (ms * 1e-3) / 1e9 / h2d_peak_gbps, 4)
    cache.leave_device_mode()
    golden = np.load(REPO / "tests" / "golden" / "moe_cfg1_f32.npz")
    err = float(np.abs(out.float().cpu().numpy() - golden["out_specfit"]).max())
    cache.close()
    pool.close()

    torch.set_num_threads(os.cpu_count() or 1)
    cfg = Qwen3MoeConfig(hidden_size=H, num_experts=E, num_experts_per_tok=8, moe_intermediate_size=I,
                         norm_topk_prob=True)
    ref = Qwen3MoeSparseMoeBlock(cfg).eval()
    with torch.no_grad():
        ref.gate.weight.copy_(weights.router)
        ref.experts.gate_up_proj.copy_(weights.gate_up)
        ref.experts.down_proj.copy_(weights.down)
        ref(x[None])
        t0 = time.perf_counter()
        for _ in range(cpu_reps):
            ref(x[None])
        cpu_ms = (time.perf_counter() - t0) / cpu_reps * 1e3
    return {"workload": "BASELINE config 1: one fp32 MoE block, 32 tokens, hidden 2048, 128 experts top-8, "
                        "moe_intermediate 768, 0 cache slots (contents invalidated before every block)",
            "host_managed": rows["host"], "device_managed": rows["device"],
            "h2d_peak_GBps": h2d_peak_gbps, "max_abs_err_vs_reference_golden": err,
            "cpu_baseline": {"block_ms": round(cpu_ms, 2), "cores": torch.get_num_threads(), "kind": "reference",
                             "sample": "stock HF Qwen3MoeSparseMoeBlock, fp32, same weights and input"}}


def cpu_reference_run(args, model_layers: int, steps: int, warmup: int):
    """The reference's CPU path: a stock Hugging Face Qwen3-MoE target on the
    host cores (all threads) — embedding, ``model_layers`` decoder layers
    (SDPA under the 4-D ancestor mask, stock sparse-MoE block), final norm and
    lm_head — verifying the benchmark's tree over a ``args.ctx``-token cache
    (prefilled outside the timer), then the greedy accepted path and the
    rollback to the context (``eagle3_tree.py:1202-1340``).  The tree mask,
    positions and accepted path come from the CPU restatement in
    ``oracle/tree_oracle.py`` (``eagle3_types.py:429-502``); nothing is
    imported from ``specfit_b200``.  Returns (seconds per pass over the
    timed steps, committed tokens per pass, threads)."""
    from transformers import DynamicCache

    from oracle import tree_oracle

    torch.set_num_threads(os.cpu_count() or 1)
    cfg = reference_config(model_layers)
    cfg._attn_implementation = "sdpa"
    tok, par, dep = workload_tree(args.nodes, args.depth, args.branch, seed=2, vocab=cfg.vocab_size)
    model = reference_model(cfg, seed=args.seed)
    gen = torch.Generator().manual_seed(1)
    ctx_ids = torch.randint(0, cfg.vocab_size, (1, args.ctx), generator=gen)
    seed_tok = int(torch.randint(0, cfg.vocab_size, (1,), generator=gen))
    ids = torch.tensor([[seed_tok, *tok]])
    mask = torch.from_numpy(tree_oracle.verification_attention_mask(par, args.ctx))[None, None]
    pos = torch.from_numpy(tree_oracle.verification_position_ids(dep, args.ctx)).reshape(1, -1)
    committed = []
    with torch.no_grad():
        cache = DynamicCache(config=cfg)
        model(input_ids=ctx_ids, past_key_values=cache, use_cache=True)

        def step():
            out = model(input_ids=ids, attention_mask=mask, position_ids=pos, past_key_values=cache,
                        use_cache=True)
            am = out.logits[0].argmax(-1).tolist()
            cache.crop(args.ctx)
            return len(tree_oracle.accepted_path(par, tok, am)) + 1

        for _ in range(warmup):
            step()
        t0 = time.perf_counter()
        for _ in range(steps):
            committed.append(step())
        elapsed = time.perf_counter() - t0
    del model, cache
    return elapsed / steps, sum(committed) / steps, torch.get_num_threads()


def cpu_reference_sample(args, layers=1):
    """Bounded sample of the reference's CPU path for the B200 arm's
    ``cpu_baseline``: a ``layers``-layer model (two timed passes after one
    warm-up) with the decoder-layer time scaled to ``args.layers`` layers; the
    embedding + lm_head share is timed in the same way on a 0-layer model."""
    t_n, _, cores = cpu_reference_run(args, layers, steps=2, warmup=1)
    t_0, _, _ = cpu_reference_run(args, 0, steps=2, warmup=1)
    per_pass = t_0 + (t_n - t_0) * args.layers / max(layers, 1)
    desc = (f"stock HF Qwen3-MoE on the host cores, {layers} decoder layer(s) timed and scaled to "
            f"{args.layers}, + embedding/norm/lm_head timed; T={1 + args.nodes}, ctx={args.ctx}, bf16")
    return per_pass, desc, cores


def b200_arm(args):
    rank, world, local = dist_info()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=device)
    from specfit_b200 import ops, synthetic
    from specfit_b200.runtime.qwen3_verifier import (ExpertHostPool, build_random_offloaded_qwen3,
                                                     qwen3_moe_config)

    peaks = measured_peaks()
    cfg = qwen3_moe_config(args.layers)
    elems = 3 * cfg.hidden_size * cfg.moe_intermediate_size
    shm = None
    if world > 1:
        shm = f"/dev/shm/specfit_b200_pool_{os.environ.get('MASTER_PORT', '0')}"
        if local == 0:
            pool = ExpertHostPool(cfg.num_hidden_layers, cfg.num_experts, elems, shm_path=shm)
            pool.fill_random(args.seed, device)
        barrier(world)
        if local != 0:
            pool = ExpertHostPool(cfg.num_hidden_layers, cfg.num_experts, elems, shm_path=shm)
    else:
        pool = ExpertHostPool(cfg.num_hidden_layers, cfg.num_experts, elems)
        pool.fill_random(args.seed, device)
    t_build = time.perf_counter()
    loaded = build_random_offloaded_qwen3(device=device, slots_per_layer=args.slots, config=cfg,
                                          seed=args.seed, pool=pool)
    apply_kernel_options(loaded, args)
    gen = torch.Generator().manual_seed(1)
    ctx_ids = torch.randint(0, cfg.vocab_size, (1, args.ctx), generator=gen).to(device)
    tree = make_tree(args.nodes, args.depth, args.branch, seed=2, vocab=cfg.vocab_size)
    seed_tok = int(torch.randint(0, cfg.vocab_size, (1,), generator=gen))
    runner = VerifyRunner(loaded, ctx_ids, tree, seed_tok, device,
                          fwd=make_forward(loaded.model, args.hf_forward))
    build_s = time.perf_counter() - t_build

    from specfit_b200.runtime import ExpertExecutionPolicy

    h2d_peak = pinned_h2d_peak(pool, device)
    policy = ExpertExecutionPolicy(args.policy)
    other = (ExpertExecutionPolicy.EXPERT_ID_ASCENDING if policy is ExpertExecutionPolicy.RESIDENT_FIRST
             else ExpertExecutionPolicy.RESIDENT_FIRST)

    def timed_with_stats(fn, pol, clocks_out=None):
        """K timed steps of ``fn`` under policy ``pol``: (ms, results, cache
        counters per timed step, launches of ours in the timed region).  With
        ``clocks_out`` (the headline) the clocks are sampled and the timed
        region is the NVTX range "headline"."""
        loaded.set_expert_execution_policy(pol)
        before: dict = {}
        start = lambda: before.update(loaded.cache_stats(), launches=ops.LAUNCHES[0])
        if clocks_out is not None:
            with ClockSampler(device.index) as clk:
                t_ms, res = timed_steps(fn, args.steps, args.warmup, world, device, on_start=start,
                                        label="headline")
            clocks_out.update(clk.summary())
        else:
            t_ms, res = timed_steps(fn, args.steps, args.warmup, world, device, on_start=start)
        launched = ops.LAUNCHES[0] - before["launches"]
        after = loaded.cache_stats()
        return t_ms, res, {k: (after[k] - before[k]) / args.steps for k in after}, launched

    def committed_of(argmaxes) -> int:
        return sum(len(tree.accepted_path(a.cpu().unsqueeze(0))) + 1 for a in argmaxes)

    # Host-managed caches (the reference's protocol: routes read back per
    # layer, leases, copy-engine fills), eager, both execution policies.
    host = {}
    for pol in (policy, other):
        t_ms, ams, per_step, _ = timed_with_stats(runner.step_device, pol)
        host[pol] = (t_ms, ams, per_step)
    assert all(torch.equal(a, host[policy][1][0]) for a in host[other][1]), \
        "execution policies gave different argmaxes"
    loaded.set_expert_execution_policy(policy)
    h_e2e_ms, h_e2e = timed_steps(runner.step_e2e, args.steps, 1, world, device)
    host_managed = {
        pol.value: {"value": round(committed_of(host[pol][1]) / (host[pol][0] / 1e3), 4), "unit": "tokens/s",
                    "ms_per_step": round(host[pol][0] / args.steps, 3), "cache_per_step": host[pol][2],
                    "h2d": h2d_roofline_of(host[pol][2], host[pol][0] / args.steps, h2d_peak)}
        for pol in (policy, other)}
    host_managed["e2e"] = {"value": round(sum(h_e2e) / (h_e2e_ms / 1e3), 4), "unit": "tokens/s",
                           "ms_per_step": round(h_e2e_ms / args.steps, 3), "execution_policy": policy.value}
    host_managed["note"] = ("eager passes; each layer reads its routed experts back, leases them on the host "
                            "and fills misses with the copy engine")

    # Device-managed caches: the same cache decisions taken on the device,
    # misses filled by a kernel from page-locked host memory, and the whole
    # verify pass replayed from one CUDA graph (the headline).
    from specfit_b200.runtime.verify_graph import VerifyGraph

    torch.cuda.synchronize()
    loaded.enter_device_managed_caches()
    dev_runs = {}
    clock_summary: dict = {}
    vg = None
    for pol in (other, policy):  # the headline policy last, with the clocks sampled
        # The policy is an argument of the captured plan kernels: one graph per policy.
        del vg
        torch.cuda.synchronize()
        loaded.set_expert_execution_policy(pol)
        vg = VerifyGraph(loaded.model, runner.cache, q_len=1 + args.nodes, device=device, forward=runner.fwd)
        launched0 = ops.LAUNCHES[0]
        vg.capture(runner.d_ids, runner.d_mask, runner.d_pos, warmup=2)
        launches_per_pass = (ops.LAUNCHES[0] - launched0) // 3  # two warm-up passes + the captured one
        t_ms, ams, per_step, _ = timed_with_stats(lambda: vg.replay().clone(), pol,
                                                  clock_summary if pol is policy else None)
        dev_runs[pol] = (t_ms, ams, per_step)
    assert all(torch.equal(a, host[policy][1][0]) for r in dev_runs.values() for a in r[1]), \
        "device-managed caches gave different argmaxes"
    ms, ams, timed_stats = dev_runs[policy]
    # The capture counted every wave; a layer whose experts fit its slots
    # skips its later waves (3 launches each) through the conditional node,
    # and each layer with later waves adds one join kernel.  The inputs are
    # the same every step, so the last pass's plans hold for every step.
    for c in loaded.caches:
        dr = c.directory
        if dr is not None and dr.waves > 1:
            if int(dr.wave_count[1:].sum()) == 0:
                launches_per_pass -= 3 * (dr.waves - 1)
            launches_per_pass += 1
    launches = launches_per_pass * args.steps
    value = sum_over_ranks(committed_of(ams), world, device) / (ms / 1e3)
    h2d_roofline = h2d_roofline_of(timed_stats, ms / args.steps, h2d_peak)
    other_policy = {"execution_policy": other.value,
                    "value": round(committed_of(dev_runs[other][1]) / (dev_runs[other][0] / 1e3), 4),
                    "unit": "tokens/s", "ms_per_step": round(dev_runs[other][0] / args.steps, 3),
                    "cache_per_step": dev_runs[other][2],
                    "h2d": h2d_roofline_of(dev_runs[other][2], dev_runs[other][0] / args.steps, h2d_peak)}
    loaded.set_expert_execution_policy(policy)

    def device_e2e():
        vg.load(runner.h_ids, runner.h_mask, runner.h_pos)
        return len(tree.accepted_path(vg.replay().cpu().unsqueeze(0))) + 1

    e2e_ms, e2e_comm = timed_steps(device_e2e, args.steps, 1, world, device)
    e2e_total = sum_over_ranks(sum(e2e_comm), world, device)
    del vg
    torch.cuda.synchronize()
    loaded.leave_device_managed_caches()
    stats24 = loaded.cache_stats()

    # The same passes under predicted cross-layer prefetch (the reference
    # runner's Qwen3ExpertPrefetch: lookahead 1, 2 copies in flight), each
    # pass predicted from the routes of the previous one.
    routes: dict = {}
    hooks = [layer.mlp.gate.register_forward_hook(
        lambda mod, a, out, l=l: routes.__setitem__(l, out[2])) for l, layer in
        enumerate(loaded.model.model.layers)]
    runner.step_device()
    for h in hooks:
        h.remove()
    preds = {l: tuple(sorted(set(r.reshape(-1).tolist()))) for l, r in routes.items()}

    def step_prefetch():
        with loaded.prefetch_experts(preds, lookahead_layers=1, max_inflight=2):
            return runner.step_device()

    pf_ms, pf_ams = timed_steps(step_prefetch, args.steps, args.warmup, world, device)
    pf_committed = sum(len(tree.accepted_path(a.cpu().unsqueeze(0))) + 1 for a in pf_ams)
    pf_value = sum_over_ranks(pf_committed, world, device) / (pf_ms / 1e3)

    result = {
        "metric": "committed tokens/s (Qwen3-30B-A3B shape, bs1)",
        "value": round(value, 4),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (random-init bf16 N(0,0.02) weights, uniform random context tokens, seeded 64-node tree)",
        "config": headline_config(args),
        "forward": ("Hugging Face decoder layers" if args.hf_forward else
                    "lean fused layer forward (runtime/lean_forward.py)"),
        "cache_mode": ("device-managed caches (misses planned and filled on the device), the verify pass "
                       "replayed from one CUDA graph"),
        "execution_policy": policy.value,
        "cache_per_step": timed_stats,
        "other_policy": other_policy,
        "host_managed": host_managed,
        "predicted_prefetch": {"value": round(pf_value, 4), "unit": "tokens/s",
                               "ms_per_step": round(pf_ms / args.steps, 3),
                               "predictions": "routes of the previous verify pass",
                               "lookahead_layers": 1, "max_inflight": 2},
        "gpu_launches": int(launches),
        "e2e": {"value": round(e2e_total / (e2e_ms / 1e3), 4), "unit": "tokens/s",
                "h2d_bytes_per_step": runner.h2d_bytes, "d2h_bytes_per_step": runner.d2h_bytes,
                "ms_per_step": round(e2e_ms / args.steps, 3)},
        "clocks": clock_summary,
        "setup_s": round(build_s, 1),
        "roofline": {"h2d": h2d_roofline},
    }

    if not args.no_resident and args.slots < cfg.num_experts:
        # Same model, caches rebuilt with one slot per expert and warmed.
        from specfit_b200.runtime import GpuExpertCache

        torch.cuda.synchronize()
        new = []
        for l, layer in enumerate(loaded.model.model.layers):
            old = layer.mlp.experts.cache
            old.close()
            c = GpuExpertCache(pool.sources(l), slot_count=cfg.num_experts, device=device,
                               adopt_pinned_sources=True)
            layer.mlp.experts.cache = c
            new.append(c)
        loaded.caches = tuple(new)
        torch.cuda.empty_cache()
        t0 = time.perf_counter()
        loaded.warm_all_caches()
        warm_s = time.perf_counter() - t0
        rsteps = max(args.steps, 10)
        # Eager resident pass (host-launched ops), then the CUDA-graph pass.
        eager_ms, _ = timed_steps(runner.step_device, rsteps, args.warmup, world, device)
        from specfit_b200.runtime.verify_graph import VerifyGraph

        vg = VerifyGraph(loaded.model, runner.cache, q_len=1 + args.nodes, device=device,
                         forward=runner.fwd)
        before = ops.LAUNCHES[0]
        vg.capture(runner.d_ids, runner.d_mask, runner.d_pos, warmup=2)
        graph_launches = (ops.LAUNCHES[0] - before) // 3  # two warm-up passes + the captured one
        with ClockSampler(device.index) as rclocks:
            rms, rams = timed_steps(lambda: vg.replay().clone(), rsteps, args.warmup, world, device)
        rcommitted = sum(len(tree.accepted_path(a.cpu().unsqueeze(0))) + 1 for a in rams)
        rvalue = sum_over_ranks(rcommitted, world, device) / (rms / 1e3)

        def graph_e2e():
            vg.load(runner.h_ids, runner.h_mask, runner.h_pos)
            am = vg.replay().cpu().unsqueeze(0)
            return len(tree.accepted_path(am)) + 1

        re2e_ms, re2e_comm = timed_steps(graph_e2e, rsteps, 1, world, device)
        times, uniq = moe_block_profile(runner)
        block_us = statistics.median(times) * 1e3
        block_bytes = statistics.median(uniq) * EXPERT_BYTES
        result["resident"] = {
            "slots_per_layer": cfg.num_experts,
            "value": round(rvalue, 3), "unit": "tokens/s",
            "ms_per_step": round(rms / rsteps, 3),
            "launch": "CUDA graph of the verify forward (runtime/verify_graph.py)",
            "gpu_launches_per_step": int(graph_launches),
            "eager_ms_per_step": round(eager_ms / rsteps, 3),
            "e2e": {"value": round(sum_over_ranks(sum(re2e_comm), world, device) / (re2e_ms / 1e3), 3),
                    "unit": "tokens/s", "ms_per_step": round(re2e_ms / rsteps, 3),
                    "h2d_bytes_per_step": runner.h2d_bytes, "d2h_bytes_per_step": runner.d2h_bytes},
            "warm_fill_s": round(warm_s, 2),
            "warm_fill_GBps": round(pool.nbytes / warm_s / 1e9, 1),
            "clocks": rclocks.summary(),
        }
        eager_block = {
            "us_per_layer_median": round(block_us, 1),
            "us_per_layer_min": round(min(times) * 1e3, 1),
            "experts_per_layer_median": statistics.median(uniq),
            "algorithmic_GBps": round(block_bytes / (block_us * 1e-6) / 1e9, 1),
            "note": ("CUDA events around each layer.mlp in one eager, host-launched resident verify "
                     "pass (T=65): includes the host gaps between launches"),
        }
        try:
            block = moe_block_graph(loaded, device, 1 + args.nodes, peaks)
        except Exception as err:  # reported, never fatal to the headline line
            block = {"error": f"{type(err).__name__}: {err}"}
        result["moe_block"] = dict(block or {"error": "layer 0 slots not all resident"},
                                   eager_in_model=eager_block)
        result["roofline"] = dict(swiglu_roofline(loaded, device, 1 + args.nodes, peaks) or {},
                                  h2d=h2d_roofline)

    if world == 1 and not args.no_extras and not args.no_resident and args.slots < cfg.num_experts:
        # The other BASELINE configurations that run on this target and pool,
        # each reported under its own key and never fatal to the headline.
        try:  # configuration 4 on the resident (128-slot, warm) caches left by the resident variant
            dec, spec = decode_measure(loaded, cfg, args, device, cpu=not args.no_cpu_baseline)
            spec.release_graphs()
            keep = ("metric", "value", "unit", "ms_per_step", "e2e", "cycle", "cpu_baseline", "config",
                    "reference_cost_model", "gpu_launches", "clocks")
            result["config4"] = {k: dec[k] for k in keep if k in dec}
        except Exception as err:
            result["config4"] = {"error": f"{type(err).__name__}: {err}"}
        try:
            result["config3"] = sweep_measure(loaded, pool, cfg, args, device)
        except Exception as err:
            result["config3"] = {"error": f"{type(err).__name__}: {err}"}
        try:
            result["config1"] = config1_block(device, h2d_peak["GBps"])
        except Exception as err:
            result["config1"] = {"error": f"{type(err).__name__}: {err}"}

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        per_pass, desc, cores = cpu_reference_sample(args, layers=args.cpu_layers)
        result["cpu_baseline"] = {"value": round(1.0 / per_pass, 5), "unit": "tokens/s", "cores": cores,
                                  "kind": "reference", "sample": desc,
                                  "seconds_per_verify_pass": round(per_pass, 3),
                                  "note": ("a bounded sample: layer 0 routes uncollapsed random hidden states "
                                           "to ~120 experts, so scaling it to 48 layers overstates the CPU "
                                           "pass; bench.py --impl reference times all 48 layers")}
    if world == 1 and not args.no_extras:
        # Configuration 5's workload on this one GPU (all 128 experts local):
        # the N = 1 point of the expert-parallel scaling series, whose N > 1
        # lines (torchrun) run the same workload sharded over the ranks.
        torch.cuda.synchronize()
        loaded.close()
        pool.close()
        import gc

        gc.collect()
        torch.cuda.empty_cache()
        try:
            ep = ep_measure(args, 0, 1, device)
            result["config5_anchor"] = {k: ep[k] for k in ("metric", "value", "unit", "ms_per_step", "e2e",
                                                           "config", "exchange_variants_ms_per_step",
                                                           "phases_us_per_layer_max_over_ranks", "roofline")}
        except Exception as err:
            result["config5_anchor"] = {"error": f"{type(err).__name__}: {err}"}
    if world > 1:
        import torch.distributed as dist

        barrier(world)
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)
    pool.close()
    if shm and local == 0:
        try:
            os.unlink(shm)
        except FileNotFoundError:
            pass


class EpRunner:
    """BASELINE configuration 5 on one rank: ``requests / world`` requests
    with ``ep_ctx``-token contexts, each verifying the same 64-node tree in
    one batched forward; per-layer routes replaced by seeded Zipf(1.1)
    routes over the global (request, token) order."""

    def __init__(self, args, loaded, cfg, device, rank, world):
        from specfit_b200 import synthetic
        from specfit_b200.runtime.kv_cache import ReservedCache

        self.model = loaded.model
        self.fwd = make_forward(loaded.model, args.hf_forward)
        self.device = device
        self.batch = args.requests // world
        self.ctx = args.ep_ctx
        self.tree = make_tree(args.nodes, args.depth, args.branch, seed=2, vocab=cfg.vocab_size)
        q = 1 + self.tree.draft_node_count
        gen = torch.Generator().manual_seed(1)
        ctx_all = torch.randint(0, cfg.vocab_size, (args.requests, self.ctx), generator=gen)
        seeds = torch.randint(0, cfg.vocab_size, (args.requests,), generator=gen)
        lo, hi = rank * self.batch, (rank + 1) * self.batch
        self.cache = ReservedCache(config=cfg, capacity=self.ctx + q)
        with torch.no_grad():
            self.fwd(input_ids=ctx_all[lo:hi].to(device), past_key_values=self.cache, use_cache=True,
                     logits_to_keep=1)
        torch.cuda.synchronize(device)
        self.h_ids = torch.cat([self.tree.verification_token_ids(seeds[b].view(1, 1))
                                for b in range(lo, hi)]).pin_memory()
        mask = self.tree.verification_attention_mask(base_kv_length=self.ctx, device="cpu")
        self.h_mask = mask.expand(self.batch, -1, -1, -1).contiguous().pin_memory()
        pos = self.tree.verification_position_ids(base_kv_length=self.ctx, device="cpu")
        self.h_pos = pos.expand(self.batch, -1).contiguous().pin_memory()
        self.d_ids, self.d_mask, self.d_pos = (t.to(device) for t in (self.h_ids, self.h_mask, self.h_pos))
        # Zipf routes of every layer for the global verify tokens; this rank's rows.
        self.routes = [torch.from_numpy(synthetic.zipf_routes(args.requests * q, l, args.seed)
                                        [lo * q:hi * q]).to(device)
                       for l in range(cfg.num_hidden_layers)]
        self.override = False
        self.hooks = [layer.mlp.gate.register_forward_hook(self._route_hook(l))
                      for l, layer in enumerate(self.model.model.layers)]

    def _route_hook(self, l):
        def hook(mod, args, out):
            if self.override:
                return out[0], out[1], self.routes[l]
            return None
        return hook

    def _forward(self, ids, mask, pos):
        self.override = True
        try:
            with torch.no_grad():
                out = self.fwd(input_ids=ids, attention_mask=mask, position_ids=pos,
                               past_key_values=self.cache, use_cache=True)
                am = out.logits.argmax(-1)
        finally:
            self.override = False
        self.cache.crop(self.ctx)
        return am

    def committed(self, am_host) -> int:
        return sum(len(self.tree.accepted_path(am_host[b:b + 1])) + 1 for b in range(self.batch))

    def step_device(self):
        return self._forward(self.d_ids, self.d_mask, self.d_pos)

    def step_e2e(self) -> int:
        ids = self.h_ids.to(self.device, non_blocking=True)
        mask = self.h_mask.to(self.device, non_blocking=True)
        pos = self.h_pos.to(self.device, non_blocking=True)
        return self.committed(self._forward(ids, mask, pos).cpu())

    @property
    def h2d_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.h_ids, self.h_mask, self.h_pos))

    @property
    def d2h_bytes(self) -> int:
        return self.h_ids.numel() * 8


def ep_swiglu_roofline(runner, moe, rank, world, device, peaks, iters=20):
    """The grouped SwiGLU on this rank's experts over the rows it receives in
    layer 0 of a verify pass (all ranks' tokens routed by the Zipf routes)."""
    from specfit_b200 import ops
    from specfit_b200.synthetic import zipf_routes

    q = runner.h_ids.shape[1]
    T = q * runner.batch * world
    idx = torch.from_numpy(zipf_routes(T, 0, 0)).to(device)
    g = torch.Generator(device=device).manual_seed(5)
    x = torch.randn(T, moe.hidden, generator=g, device=device).to(torch.bfloat16)
    w = torch.rand(T, idx.shape[1], generator=g, device=device)
    send = ops.ep_send_pack(x, idx, w, moe.num_experts, world)
    counts = send.counts.cpu().tolist()
    lo = sum(c[0] for c in counts[:rank])
    pairs, routes = counts[rank]
    rows = send.rows[lo:lo + pairs]
    d, _ = ops.ep_recv_group(rows, pairs, moe.hidden, moe.top_k, moe.local_experts, torch.bfloat16)
    xs, ws = ops.ep_recv_gather(rows, d, moe.hidden, torch.bfloat16, routes)
    act = torch.empty(max(routes, 1), moe.inter, dtype=torch.bfloat16, device=device)
    ys = torch.empty(max(routes, 1), moe.hidden, dtype=torch.bfloat16, device=device)
    run = lambda: ops.grouped_swiglu(xs, ws, d, moe.slot, moe.storage, moe.hidden, moe.inter,
                                     act_workspace=act, out=ys[:routes])
    for _ in range(3):
        run()
    torch.cuda.synchronize(device)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        run()
    e.record()
    torch.cuda.synchronize(device)
    us = s.elapsed_time(e) * 1e3 / iters
    uniq = int(d.num_active.item())
    algo = uniq * EXPERT_BYTES + routes * moe.hidden * 2 * 2 + routes * moe.inter * 2 * 2 + routes * 4
    achieved = algo / (us * 1e-6) / 1e9
    return {"bound": "hbm", "kernel": "swiglu_tc_kernel (phase 1 + 2)", "achieved": round(achieved, 1),
            "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
            "traffic": None, "launch_us": round(us, 2), "experts": uniq, "rows": routes,
            "algorithmic_bytes": algo, "peak_source": peaks["source"] + " hbm_gbs (burst copy)",
            "rank": rank}


def ep_arm(args):
    """expert-parallel verify over the ranks
    (``ep_measure``), one process per GPU."""
    rank, world, local = dist_info()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if args.requests % world:
        raise SystemExit("--requests must be a multiple of the number of GPUs")
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=device)
    result = ep_measure(args, rank, world, device)
    if world > 1:
        import torch.distributed as dist

        barrier(world)
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


def ep_measure(args, rank: int, world: int, device) -> dict:
    """Configuration 5 on this rank: the prefill and a reference timing use
    the NCCL exchange; the headline runs the verify pass with the
    peer-memory exchange, captured as one CUDA graph per rank (no host
    synchronisation inside a pass).  One eager peer pass is also timed phase
    by phase (CUDA events around send / receive / grouped SwiGLU / return /
    combine of every layer; medians over layers, max over ranks)."""
    from specfit_b200 import ops
    from specfit_b200.runtime.ep_verifier import build_random_ep_qwen3
    from specfit_b200.runtime.qwen3_verifier import qwen3_moe_config
    from specfit_b200.runtime.verify_graph import VerifyGraph

    peaks = measured_peaks()
    cfg = qwen3_moe_config(args.layers)
    t0 = time.perf_counter()
    loaded = build_random_ep_qwen3(device=device, rank=rank, world=world, config=cfg, seed=args.seed)
    runner = EpRunner(args, loaded, cfg, device, rank, world)
    q = 1 + runner.tree.draft_node_count
    setup_s = time.perf_counter() - t0

    # Reference point: the NCCL exchange, eager (one host sync per layer).
    nccl_ms, _ = timed_steps(runner.step_device, args.steps, 2, world, device)
    moes = loaded.moes()
    plans = [m.last_plan for m in moes]

    # Peer-memory exchange: eager, then one CUDA graph per verify pass.
    peer = loaded.attach_peer_exchange(max_tokens=runner.batch * q)
    loaded.use_peer(True)
    peer_eager_ms, _ = timed_steps(runner.step_device, args.steps, 2, world, device)
    peer.phase_events = []
    runner.step_device()
    phases = peer.phase_times_us()
    peer.phase_events = None
    phases = {k: round(max_over_ranks(v, world, device), 2) for k, v in phases.items()}
    times, _ = moe_block_profile(runner)
    vg = VerifyGraph(loaded.model, runner.cache, q_len=q, device=device, batch=runner.batch,
                     forward=runner.fwd)
    barrier(world)
    runner.override = True
    try:
        before = ops.LAUNCHES[0]
        vg.capture(runner.d_ids, runner.d_mask, runner.d_pos, warmup=2)
        graph_launches = (ops.LAUNCHES[0] - before) // 3  # two warm-up passes + the captured one
    finally:
        runner.override = False
    barrier(world)
    with ClockSampler(device.index) as clocks:
        ms, ams = timed_steps(lambda: vg.replay().clone(), args.steps, args.warmup, world, device)
    committed = sum(runner.committed(a.cpu()) for a in ams)
    value = sum_over_ranks(committed, world, device) / (ms / 1e3)

    def graph_e2e():
        vg.load(runner.h_ids, runner.h_mask, runner.h_pos)
        return runner.committed(vg.replay().cpu())

    e2e_ms, e2e_comm = timed_steps(graph_e2e, args.steps, 1, world, device)
    e2e_value = sum_over_ranks(sum(e2e_comm), world, device) / (e2e_ms / 1e3)
    peer.check()

    row_bytes = ops.ep_row_bytes(torch.bfloat16, cfg.hidden_size, cfg.num_experts_per_tok)
    sent = [sum(p.send_pairs) * row_bytes + sum(p.send_routes) * cfg.hidden_size * 2 for p in plans]
    local_rows = statistics.median([sum(p.recv_routes) for p in plans])
    block_us = statistics.median(times) * 1e3
    block_us_max = max_over_ranks(block_us, world, device)
    result = {
        "metric": "committed tokens/s (Qwen3-30B-A3B shape, 8 requests, expert-parallel)",
        "value": round(value, 3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (random-init bf16 N(0,0.02) weights, uniform random context tokens, seeded "
                "64-node tree, seeded Zipf(1.1) routes per layer)",
        "config": {
            "workload": (f"BASELINE config 5: {args.layers}-layer Qwen3-30B-A3B-shaped verify over "
                         f"{args.requests} concurrent requests x {args.nodes}-node tree ({args.requests * q} "
                         f"verify tokens per step), {args.ep_ctx}-token context each, Zipf(1.1) routes, "
                         f"{cfg.num_experts} experts sharded over {world} GPU(s) "
                         f"({cfg.num_experts // world} resident per GPU per layer), dispatch/return "
                         "through peer memory over NVLink, one CUDA graph per verify pass"),
            "requests_per_gpu": runner.batch,
            "verify_tokens_per_step": args.requests * q,
            "parallelism": f"ep{world}, attention data-parallel over requests",
            "forward": ("Hugging Face decoder layers" if args.hf_forward else
                        "lean fused layer forward (runtime/lean_forward.py)"),
            "l2_flush": (f"not needed: each step reads {args.layers * cfg.num_experts // world} resident "
                         f"experts ({args.layers * cfg.num_experts // world * EXPERT_BYTES / 1e9:.1f} GB) "
                         "per GPU, >> 126 MB L2"),
        },
        "gpu_launches": int(graph_launches) * args.steps,
        "e2e": {"value": round(e2e_value, 3), "unit": "tokens/s",
                "h2d_bytes_per_step": runner.h2d_bytes, "d2h_bytes_per_step": runner.d2h_bytes,
                "ms_per_step": round(e2e_ms / args.steps, 3)},
        "clocks": clocks.summary(),
        "exchange_variants_ms_per_step": {
            "nccl_all_to_all_eager": round(nccl_ms / args.steps, 3),
            "peer_memory_eager": round(peer_eager_ms / args.steps, 3),
            "peer_memory_cuda_graph": round(ms / args.steps, 3),
        },
        "moe_block": {
            "us_per_layer_median_max_over_ranks": round(block_us_max, 1),
            "rows_per_rank_median": local_rows,
            "nvlink_bytes_sent_per_layer_rank0": int(statistics.median(sent)),
            "note": "CUDA events around each layer.mlp in an eager peer-memory pass (router, send "
                    "plan + push, receive wait + grouping + gather, grouped SwiGLU, return, combine)",
        },
        "phases_us_per_layer_max_over_ranks": phases,
        "roofline": ep_swiglu_roofline(runner, moes[0], rank, world, device, peaks),
        "setup_s": round(setup_s, 1),
    }
    del vg
    torch.cuda.synchronize(device)
    loaded.close()
    return result


def cpu_decode_sample(cfg, verify_tokens: int, ctx: int, rows_per_level: int, levels: int):
    """Host-core time of one speculative-decoding cycle of the reference's
    CPU path: the Hugging Face decoder layer (SDPA under the tree mask over a
    ``ctx``-token cache, stock sparse-MoE block) for ``verify_tokens`` rows,
    scaled to all layers, plus the target lm_head, plus the drafter's GEMMs
    (its decoder layer and lm_head over ``rows_per_level`` rows, ``levels``
    times).  Returns (seconds per cycle, description, threads)."""
    from transformers import DynamicCache
    from transformers.models.qwen3_moe.modeling_qwen3_moe import (Qwen3MoeDecoderLayer,
                                                                   Qwen3MoeRotaryEmbedding)

    torch.set_num_threads(os.cpu_count() or 1)
    cfgc = type(cfg).from_dict(cfg.to_dict())
    cfgc._attn_implementation = "sdpa"
    gen = torch.Generator().manual_seed(11)
    layer = Qwen3MoeDecoderLayer(cfgc, 0).to(torch.bfloat16).eval()
    H, V = cfgc.hidden_size, cfgc.vocab_size
    bf = dict(dtype=torch.bfloat16)
    with torch.no_grad():
        for p in layer.parameters():
            p.normal_(0.0, 0.02, generator=gen)
        rope = Qwen3MoeRotaryEmbedding(cfgc)
        head = torch.randn(V, H, generator=gen).mul_(0.02).to(**bf)
        kv = DynamicCache(config=cfgc)
        ch = torch.randn(1, ctx, H, generator=gen).to(**bf)
        cpos = torch.arange(ctx).unsqueeze(0)
        layer(ch, attention_mask=None, position_ids=cpos, past_key_values=kv, use_cache=True,
              position_embeddings=rope(ch, cpos))
        x = torch.randn(1, verify_tokens, H, generator=gen).to(**bf)
        mask = torch.ones(1, 1, verify_tokens, ctx + verify_tokens, dtype=torch.bool)
        mask[..., ctx:] = torch.tril(torch.ones(verify_tokens, verify_tokens, dtype=torch.bool))
        pos = torch.arange(ctx, ctx + verify_tokens).unsqueeze(0)
        pe = rope(x, pos)

        def one_layer():
            layer(x, attention_mask=mask, position_ids=pos, past_key_values=kv, use_cache=True,
                  position_embeddings=pe)
            kv.crop(ctx)

        one_layer()
        t0 = time.perf_counter()
        one_layer()
        layer_s = time.perf_counter() - t0
        t0 = time.perf_counter()
        torch.nn.functional.linear(x, head).argmax(-1)
        head_s = time.perf_counter() - t0
        # Drafter per level: q/k/v from [rows, 2H], o_proj, gate/up/down (6144), lm_head + top-k.
        r = torch.randn(rows_per_level, 2 * H, generator=gen).to(**bf)
        w_qkv = torch.randn(4096 + 2 * 512, 2 * H, generator=gen).to(**bf)
        w_o = torch.randn(H, 4096, generator=gen).to(**bf)
        w_gu = torch.randn(2 * 6144, H, generator=gen).to(**bf)
        w_d = torch.randn(H, 6144, generator=gen).to(**bf)
        hq = torch.randn(rows_per_level, H, generator=gen).to(**bf)
        a_o = torch.randn(rows_per_level, 4096, generator=gen).to(**bf)
        a_d = torch.randn(rows_per_level, 6144, generator=gen).to(**bf)
        t0 = time.perf_counter()
        torch.nn.functional.linear(r, w_qkv)
        torch.nn.functional.linear(a_o, w_o)
        torch.nn.functional.linear(hq, w_gu)
        torch.nn.functional.linear(a_d, w_d)
        torch.log_softmax(torch.nn.functional.linear(hq, head).float(), -1).topk(4)
        level_s = time.perf_counter() - t0
    cycle = layer_s * cfgc.num_hidden_layers + head_s + level_s * levels
    desc = (f"HF Qwen3MoeDecoderLayer (sdpa, stock MoE) x1 on CPU at {verify_tokens} verify rows over a "
            f"{ctx}-token cache, scaled to {cfgc.num_hidden_layers} layers, + lm_head, + drafter GEMMs "
            f"({levels} levels x {rows_per_level} rows incl. the 151,936-way lm_head); bf16")
    return cycle, desc, torch.get_num_threads()


def decode_mode(args):
    """BASELINE configuration 4 alone (``decode_measure``) on a freshly built target."""
    from specfit_b200.runtime.qwen3_verifier import build_random_offloaded_qwen3, qwen3_moe_config

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    cfg = qwen3_moe_config(args.layers)
    t0 = time.perf_counter()
    loaded = build_random_offloaded_qwen3(device=device, slots_per_layer=cfg.num_experts, config=cfg,
                                          seed=args.seed)
    apply_kernel_options(loaded, args)
    loaded.warm_all_caches()
    result, spec = decode_measure(loaded, cfg, args, device, setup_s=time.perf_counter() - t0)
    print(json.dumps(result), flush=True)
    spec.release_graphs()
    loaded.close()


def decode_measure(loaded, cfg, args, device, setup_s: float = 0.0, cpu: bool | None = None):
    """end-to-end speculative decoding on one B200
    over ``loaded`` (every expert resident).  Returns the result line and the
    speculator (whose graphs the caller releases)."""
    from specfit_b200 import ops, synthetic
    from specfit_b200.runtime.eagle3_drafter import build_random_drafter
    from specfit_b200.runtime.speculator import B200TreeSpeculator, BernoulliAcceptance
    from specfit_b200.selection import SelectionCostModel

    t0 = time.perf_counter()
    L = cfg.num_hidden_layers
    aux = (1, 23, 44) if L == 48 else tuple(sorted({1 % L, (L * 23) // 48, (L * 44) // 48}))
    drafter = build_random_drafter(loaded.model, seed=args.seed + 1000, aux_layers=aux)
    cost = SelectionCostModel(synthetic.SELECTION_SIZE_MEAN_NS, synthetic.SELECTION_INTERCEPT_NS,
                              synthetic.SELECTION_EXPERT_NS)
    gen = torch.Generator().manual_seed(1)
    ctx_host = torch.randint(0, cfg.vocab_size, (1, args.decode_ctx), generator=gen).pin_memory()
    spec = B200TreeSpeculator(loaded, drafter, cost_model=cost, acceptance=BernoulliAcceptance(0),
                              route_seed=args.seed, graphs=not args.eager_decode,
                              reserve_tokens=args.decode_ctx + args.new_tokens + 16,
                              lean=not args.hf_forward)
    setup_s += time.perf_counter() - t0

    def run(new_tokens, acceptance_seed):
        spec.acceptance = BernoulliAcceptance(acceptance_seed)
        t = time.perf_counter()
        ids = ctx_host.to(device, non_blocking=True)
        res = spec.generate(ids, new_tokens)
        return res, time.perf_counter() - t

    for w in range(max(args.warmup, 1)):
        run(32, 100 + w)
    # The reference's frozen A100 coefficients (expert transfers over PCIe)
    # price a drafted node above its reward here; SpecFit's own procedure fits
    # the model to the machine, so the headline uses one fitted on this B200.
    ref_res, _ = run(args.new_tokens, 7)
    peaks = measured_peaks()
    calibrated = verify_fit = None
    if not args.eager_decode:
        expert_ns = EXPERT_BYTES / peaks["hbm_gbs"]
        verify_fit = spec.calibrate_cost_model(expert_ns=expert_ns)
        spec.acceptance = BernoulliAcceptance(98)
        calibrated = spec.calibrate_cycle_cost_model(ctx_host.to(device, non_blocking=True),
                                                     expert_ns=expert_ns)
        spec.cost_model = calibrated
        run(32, 99)
    launches0 = ops.LAUNCHES[0]
    with ClockSampler(device.index) as clocks:
        res, wall = run(args.new_tokens, 7)
    launches = ops.LAUNCHES[0] - launches0
    cyc = res.cycles
    value = res.committed / res.decode_s
    mean = lambda xs: float(statistics.mean(xs)) if xs else 0.0
    per_cycle = res.committed / max(len(cyc), 1)
    result = {
        "metric": "committed tokens/s (Qwen3-30B-A3B shape, EAGLE-3 drafting, bs1)",
        "value": round(value, 3),
        "unit": "tokens/s",
        "n_gpus": 1,
        "steps": len(cyc),
        "warmup": args.warmup,
        "ms_per_step": round(res.decode_s * 1e3 / max(len(cyc), 1), 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (random-init bf16 N(0,0.02) target and drafter, uniform random context; "
                "per-token Zipf(1.1) routes; acceptance Bernoulli(p_depth), p_depth ~ Beta(4,2))",
        "config": {
            "workload": (f"BASELINE config 4: end-to-end speculative decoding, {args.layers}-layer "
                         f"Qwen3-30B-A3B-shaped target (all 128 experts resident), EAGLE-3-shaped drafter "
                         f"stand-in (1 layer, fc over target layers {list(aux)}, 151,936 vocab) drafting "
                         f"60-node pools of depth <= 8, SpecFit exact selection (<= 7 nodes, the "
                         f"reference's natural/legacy cost model), {args.decode_ctx}-token context, "
                         f"{args.new_tokens} generated tokens"),
            "step": "one speculative cycle (draft, select, verify, commit)",
            "verify": "eager" if args.eager_decode else "one CUDA graph per tree size (1-8 rows)",
            "forward": ("Hugging Face decoder layers" if args.hf_forward else
                        "lean fused layer forward (runtime/lean_forward.py)"),
            "l2_flush": "not needed: each verify pass reads the routed experts of every layer (GBs)",
        },
        "gpu_launches": int(launches),
        "e2e": {"value": round(res.committed / wall, 3), "unit": "tokens/s",
                "h2d_bytes_per_step": int(ctx_host.numel() * 8 / max(len(cyc), 1)),
                "d2h_bytes_per_step": 8 * int(round(per_cycle)),
                "includes": "context H2D, prefill of the context, every cycle, token read-back"},
        "clocks": clocks.summary(),
        "cycle": {"committed_per_cycle": round(per_cycle, 3),
                  "selected_nodes_mean": round(mean([c.selected for c in cyc]), 3),
                  "accepted_mean": round(mean([c.accepted for c in cyc]), 3),
                  "pool_nodes_mean": round(mean([c.pool_nodes for c in cyc]), 2),
                  "host_ms": {"draft": round(mean([c.draft_ms for c in cyc]), 3),
                              "select": round(mean([c.select_ms for c in cyc]), 3),
                              "verify": round(mean([c.verify_ms for c in cyc]), 3),
                              "commit": round(mean([c.commit_ms for c in cyc]), 3),
                              "draft_split": ({k: round(mean([t[k] for t in res.draft_split]), 3)
                                               for k in res.draft_split[0]} if res.draft_split else {})},
                  "prefill_s": round(res.prefill_s, 3)},
        "cost_model": ({"kind": "SelectionCostModel fitted on this B200 the reference's way: whole "
                                "decode cycles timed per forced tree size; slope = one packed expert "
                                "over the measured HBM bandwidth",
                        "size_intercept_ns": [round(x) for x in calibrated.size_intercept_ns],
                        "size_mean_ns": [round(x) for x in calibrated.size_mean_ns],
                        "expert_ns": round(calibrated.expert_ns, 1),
                        "verify_only_intercept_ns": [round(x) for x in verify_fit.size_intercept_ns]}
                       if calibrated is not None else {"kind": "reference natural/legacy coefficients"}),
        "reference_cost_model": {
            "value": round(ref_res.committed / ref_res.decode_s, 3), "unit": "tokens/s",
            "committed_per_cycle": round(ref_res.committed / max(len(ref_res.cycles), 1), 3),
            "selected_nodes_mean": round(mean([c.selected for c in ref_res.cycles]), 3),
            "note": "same run with the reference's frozen A100 natural/legacy coefficients "
                    "(210.7 us per distinct (layer, expert)): no drafted node pays for itself"},
        "setup_s": round(setup_s, 1),
    }
    try:  # the grouped SwiGLU at the mean verify size, on layer 0's resident slots
        result["roofline"] = swiglu_roofline(loaded, device, 1 + int(round(mean([c.selected for c in cyc]))),
                                             peaks)
    except Exception as err:  # reported, never fatal to the line
        result["roofline"] = {"error": f"{type(err).__name__}: {err}"}
    if (not args.no_cpu_baseline) if cpu is None else cpu:
        vt = 1 + int(round(mean([c.selected for c in cyc])))
        cycle_s, desc, cores = cpu_decode_sample(cfg, vt, args.decode_ctx, 8, 8)
        result["cpu_baseline"] = {"value": round(per_cycle / cycle_s, 5), "unit": "tokens/s",
                                  "cores": cores, "kind": "reference",
                                  "sample": desc + f"; {per_cycle:.3f} committed tokens per cycle as "
                                            "measured on the GPU run (same seeds)",
                                  "seconds_per_cycle": round(cycle_s, 3)}
    return result, spec


def reference_arm(args):
    """``--impl reference``: the reference's CPU path (``cpu_reference_run``)
    on the B200 arm's workload.  The whole ``args.layers``-layer model is
    materialised when the host has the memory for it (61 GB at 48 layers);
    otherwise the largest layer count that fits is timed and scaled, and the
    line says so."""
    rank, world, local = dist_info()
    if rank != 0:
        return
    import psutil

    need = reference_model_bytes(args.layers)
    avail = psutil.virtual_memory().available
    if need * 1.15 + (8 << 30) <= avail:
        per_pass, per_commit, cores = cpu_reference_run(args, args.layers, args.steps, args.warmup)
        sample = (f"stock HF Qwen3-MoE, all {args.layers} decoder layers materialised on the host "
                  f"({need / 1e9:.1f} GB bf16); every timed step is a full verify pass")
        value = per_commit / per_pass
    else:
        fit = max(1, int((avail - (8 << 30)) / 1.15 - reference_model_bytes(0)) //
                  (reference_model_bytes(1) - reference_model_bytes(0)))
        fit = min(fit, args.layers, 8)
        per_pass, sample, cores = cpu_reference_sample(args, layers=fit)
        sample += f" (host has {avail / 1e9:.0f} GB available, the full model needs {need / 1e9:.0f} GB)"
        value = 1.0 / per_pass
    print(json.dumps({
        "impl": "reference",
        "metric": "committed tokens/s (Qwen3-30B-A3B shape, bs1)",
        "value": round(value, 5), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(per_pass * 1e3, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init bf16 N(0,0.02) weights, uniform random context tokens, seeded 64-node tree)",
        "config": headline_config(args),
        "cpu_baseline": {"value": round(value, 5), "unit": "tokens/s", "cores": cores, "kind": "reference",
                         "sample": sample},
        "e2e": {"value": round(value, 5), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def block_mode(args):
    """The MoE verify block alone (router, dispatch, gather, grouped SwiGLU,
    combine) on one layer whose 128 experts are resident in HBM; bf16
    N(0,0.02) weights drawn on the GPU.  One step = one block call."""
    from specfit_b200 import ops, synthetic

    device = torch.device("cuda", 0)
    peaks = measured_peaks()
    g = torch.Generator(device=device).manual_seed(args.seed)
    e, h, i = synthetic.NUM_EXPERTS, synthetic.HIDDEN, synthetic.MOE_INTER
    storage = (torch.randn(e, 3 * h * i, generator=g, device=device) * 0.02).to(torch.bfloat16)
    router = (torch.randn(e, h, generator=g, device=device) * 0.02).to(torch.bfloat16)
    x = torch.randn(args.tokens, h, generator=g, device=device).to(torch.bfloat16)
    slot = torch.arange(e, dtype=torch.int32, device=device)
    zipf = None
    if args.routes == "zipf":
        zipf = torch.from_numpy(synthetic.zipf_routes(args.tokens, layer=0, seed=args.seed)).to(device)
    elif args.routes == "uniform":
        rng = np.random.default_rng(args.seed)
        zipf = torch.from_numpy(np.stack([rng.permutation(e)[:8] for _ in range(args.tokens)])).to(device)

    def block():
        _, w, idx = ops.router_topk(x, router, 8, True)
        if zipf is not None:
            idx = zipf
        d = ops.moe_dispatch(idx, e)
        xs, ws = ops.moe_gather(x, w, d)
        ys = ops.grouped_swiglu(xs, ws, d, slot, storage, h, i)
        return ops.moe_combine(ys, d, idx), d

    ms, outs = timed_steps(block, args.steps, args.warmup, 1, device)
    uniq = int(outs[-1][1].num_active.item())
    us = ms * 1e3 / args.steps

    # Per-op device time of one more block (events between the launches).
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
    ev[0].record()
    _, w, idx = ops.router_topk(x, router, 8, True)
    if zipf is not None:
        idx = zipf
    ev[1].record()
    d = ops.moe_dispatch(idx, e)
    ev[2].record()
    xs, ws = ops.moe_gather(x, w, d)
    ev[3].record()
    ys = ops.grouped_swiglu(xs, ws, d, slot, storage, h, i)
    ev[4].record()
    ops.moe_combine(ys, d, idx)
    ev[5].record()
    torch.cuda.synchronize()
    names = ("router", "dispatch", "gather", "grouped_swiglu", "combine")
    per_op = {n: round(ev[j].elapsed_time(ev[j + 1]) * 1e3, 2) for j, n in enumerate(names)}
    algo = uniq * EXPERT_BYTES + e * h * 2
    print(json.dumps({"mode": "block", "tokens": args.tokens, "routes": args.routes, "experts": uniq,
                      "us_per_block": round(us, 2), "per_op_us": per_op,
                      "algorithmic_GBps": round(algo / us / 1e3, 1),
                      "frac_of_hbm_peak": round(algo / us / 1e3 / peaks["hbm_gbs"], 4)}), flush=True)


def graph_mode(args):
    """Resident verify pass only: every expert in HBM (128 slots per layer),
    one CUDA graph per pass, ``--steps`` replays inside the NVTX range
    "timed" (kernel profiling of the verify pass)."""
    from specfit_b200.runtime.qwen3_verifier import build_random_offloaded_qwen3, qwen3_moe_config
    from specfit_b200.runtime.verify_graph import VerifyGraph

    device = torch.device("cuda", 0)
    cfg = qwen3_moe_config(args.layers)
    loaded = build_random_offloaded_qwen3(device=device, slots_per_layer=cfg.num_experts, config=cfg,
                                          seed=args.seed)
    apply_kernel_options(loaded, args)
    loaded.warm_all_caches()
    gen = torch.Generator().manual_seed(1)
    ctx_ids = torch.randint(0, cfg.vocab_size, (1, args.ctx), generator=gen).to(device)
    tree = make_tree(args.nodes, args.depth, args.branch, seed=2, vocab=cfg.vocab_size)
    seed_tok = int(torch.randint(0, cfg.vocab_size, (1,), generator=gen))
    runner = VerifyRunner(loaded, ctx_ids, tree, seed_tok, device,
                          fwd=make_forward(loaded.model, args.hf_forward))
    vg = VerifyGraph(loaded.model, runner.cache, q_len=1 + args.nodes, device=device, forward=runner.fwd)
    vg.capture(runner.d_ids, runner.d_mask, runner.d_pos)
    ms, _ = timed_steps(vg.replay, args.steps, args.warmup, 1, device)
    print(json.dumps({"mode": "graph", "layers": args.layers, "ms_per_pass": round(ms / args.steps, 3),
                      "verify_tokens": 1 + args.nodes}), flush=True)
    loaded.close()


def sweep_measure(loaded, pool, cfg, args, device) -> dict:
    """BASELINE configuration 3, the expert-cache sweep, on an already built
    target: every layer's routes are replaced by seeded per-layer Zipf(1.1)
    top-8 routes (``synthetic.zipf_routes``) for the 129 verify rows of a
    128-node tree, and the caches are rebuilt at each slot count over the
    shared page-locked pool.  Per slot count: the cold pass (fresh caches,
    host-managed, eager) and warm passes with device-managed caches replayed
    from one CUDA graph (each pass starts from the state the previous one
    left), with CUDA-event times and fills per pass.  Derived: the warm
    pass's H2D GB/s, the fill time it exposes beyond the resident (128-slot)
    pass, overlap = 1 - exposed / (fill bytes at the pinned-copy rate), and
    the grouped SwiGLU's phase-1 tiles per SM (148 persistent CTAs)."""
    from specfit_b200 import synthetic
    from specfit_b200.runtime import GpuExpertCache
    from specfit_b200.runtime.verify_graph import VerifyGraph

    L, E = cfg.num_hidden_layers, cfg.num_experts
    nodes = args.sweep_nodes
    T = 1 + nodes
    routes = [torch.from_numpy(synthetic.zipf_routes(T, l, seed=args.seed + 3)).to(device) for l in range(L)]
    layers = loaded.model.model.layers
    hooks = [layer.mlp.gate.register_forward_hook(
        lambda mod, a, out, l=l: (out[0], out[1], routes[l]) if out[2].shape[0] == T else None)
        for l, layer in enumerate(layers)]
    gen = torch.Generator().manual_seed(1)
    ctx_ids = torch.randint(0, cfg.vocab_size, (1, args.ctx), generator=gen).to(device)
    tree = make_tree(nodes, args.sweep_depth, args.branch, seed=2, vocab=cfg.vocab_size)
    seed_tok = int(torch.randint(0, cfg.vocab_size, (1,), generator=gen))
    peak = pinned_h2d_peak(pool, device)

    def set_slots(slots: int) -> None:
        torch.cuda.synchronize()
        new = []
        for l, layer in enumerate(layers):
            layer.mlp.experts.cache.close()
            c = GpuExpertCache(pool.sources(l), slot_count=slots, device=device, adopt_pinned_sources=True)
            layer.mlp.experts.cache = c
            new.append(c)
        loaded.caches = tuple(new)
        torch.cuda.empty_cache()

    def timed(fn):
        before = loaded.cache_stats()["h2d_submissions"]
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        return a.elapsed_time(b), loaded.cache_stats()["h2d_submissions"] - before

    try:
        set_slots(E)
        loaded.warm_all_caches()
        runner = VerifyRunner(loaded, ctx_ids, tree, seed_tok, device, fwd=make_forward(loaded.model, False))
        timed(runner.step_device)
        resident_ms = statistics.median(timed(runner.step_device)[0] for _ in range(3))
        active = [len(set(r.reshape(-1).tolist())) for r in routes]
        tiles = statistics.mean(a * (cfg.moe_intermediate_size // 64) for a in active)
        from specfit_b200.runtime import ExpertExecutionPolicy

        rows = []
        for slots in [int(x) for x in args.sweep_slots.split(",")]:
            set_slots(slots)
            loaded.set_expert_execution_policy(ExpertExecutionPolicy.EXPERT_ID_ASCENDING)
            cold_ms, cold_fills = timed(runner.step_device)
            row = {"slots": slots, "cold_ms": round(cold_ms, 2), "cold_fills": cold_fills}
            loaded.enter_device_managed_caches()
            for pol in (ExpertExecutionPolicy.EXPERT_ID_ASCENDING, ExpertExecutionPolicy.RESIDENT_FIRST):
                loaded.set_expert_execution_policy(pol)  # captured into the plan kernels: one graph each
                vg = VerifyGraph(loaded.model, runner.cache, q_len=T, device=device, forward=runner.fwd)
                vg.capture(runner.d_ids, runner.d_mask, runner.d_pos, warmup=2)
                warm = [timed(vg.replay) for _ in range(max(args.steps, 3))]
                del vg
                torch.cuda.synchronize()
                warm_ms = statistics.median(w[0] for w in warm)
                warm_fills = warm[-1][1]
                fill_bytes = warm_fills * EXPERT_BYTES
                exposed = max(warm_ms - resident_ms, 0.0)
                busy = fill_bytes / (peak["GBps"] * 1e9) * 1e3
                key = "warm" if pol is ExpertExecutionPolicy.EXPERT_ID_ASCENDING else "warm_resident_first"
                row[key] = {"ms": round(warm_ms, 2), "fills": warm_fills,
                            "h2d_GBps": round(fill_bytes / (warm_ms * 1e-3) / 1e9, 1),
                            "exposed_fill_ms": round(exposed, 2),
                            "overlap": round(1.0 - exposed / busy, 3) if busy > 0 else 1.0}
            loaded.leave_device_managed_caches()
            loaded.set_expert_execution_policy(ExpertExecutionPolicy.EXPERT_ID_ASCENDING)
            rows.append(row)
    finally:
        for h in hooks:
            h.remove()
    return {"workload": (f"BASELINE config 3: {L}-layer target, {T} verify rows ({nodes}-node tree), "
                         f"{args.ctx}-token context, per-layer Zipf(1.1) top-8 routes, slots {args.sweep_slots}; "
                         "cold = fresh host-managed caches, warm = device-managed caches, one CUDA graph per pass"),
            "rows": rows, "resident_ms": round(resident_ms, 2), "h2d_peak": peak,
            "experts_per_layer_mean": round(statistics.mean(active), 1),
            "swiglu_phase1_tiles_per_sm": round(tiles / num_sms_of(device), 2)}


def sweep_mode(args):
    """``--mode sweep``: configuration 3 alone (``sweep_measure``)."""
    from specfit_b200.runtime.qwen3_verifier import (ExpertHostPool, build_random_offloaded_qwen3,
                                                     qwen3_moe_config)

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    cfg = qwen3_moe_config(args.layers)
    pool = ExpertHostPool(cfg.num_hidden_layers, cfg.num_experts, 3 * cfg.hidden_size * cfg.moe_intermediate_size)
    pool.fill_random(args.seed, device)
    loaded = build_random_offloaded_qwen3(device=device, slots_per_layer=cfg.num_experts, config=cfg,
                                          seed=args.seed, pool=pool)
    apply_kernel_options(loaded, args)
    with ClockSampler(device.index) as clocks:
        sweep = sweep_measure(loaded, pool, cfg, args, device)
    head = next((r for r in sweep["rows"] if r["slots"] == args.slots), sweep["rows"][0])
    result = {
        "metric": "verify passes/s (config 3 sweep, warm cache)",
        "value": round(1e3 / head["warm"]["ms"], 3), "unit": "passes/s", "n_gpus": 1,
        "steps": max(args.steps, 3), "warmup": 2, "ms_per_step": head["warm"]["ms"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init bf16 weights; per-layer Zipf(1.1) top-8 routes replace the router)",
        "config": {"workload": sweep["workload"], "headline_slots": head["slots"]},
        **{k: v for k, v in sweep.items() if k != "workload"},
        "clocks": clocks.summary(),
    }
    loaded.close()
    pool.close()
    print(json.dumps(result), flush=True)


def kernel_cases(device, only=(), rows=(7, 65, 512)):
    """(name, case, launch, algorithmic bytes) for every hot kernel at the
    sizes the configurations run it at: 7 rows (a decode verify pass), 65
    (configuration 2), 512 (configuration 5's step); bf16 inputs drawn on the
    device; routes Zipf(1.1) (configurations 3 and 5) or uniform."""
    from specfit_b200 import _native as N
    from specfit_b200 import ops, synthetic

    H, E, K, I = synthetic.HIDDEN, synthetic.NUM_EXPERTS, synthetic.TOP_K, synthetic.MOE_INTER
    HQ, HKV, D, V = synthetic.NUM_HEADS, synthetic.NUM_KV_HEADS, synthetic.HEAD_DIM, synthetic.VOCAB
    g = torch.Generator(device=device).manual_seed(11)
    bf = dict(dtype=torch.bfloat16, device=device)

    def randn(*shape, std=1.0):
        return (torch.randn(*shape, generator=g, device=device) * std).to(torch.bfloat16)

    want = lambda name: not only or name in only
    cur = lambda: torch.cuda.current_stream(device).cuda_stream  # the stream at call time (graph capture)
    cases = []
    storage = slot = router = None
    if want("router") or want("grouped_swiglu") or "grouped_swiglu_gathered" in only:
        router = randn(E, H, std=0.02)
    if want("grouped_swiglu") or "grouped_swiglu_gathered" in only:
        storage = randn(E, 3 * H * I, std=0.02)
        slot = torch.arange(E, dtype=torch.int32, device=device)
    for t in rows:
        x = randn(t, H)
        idx = torch.from_numpy(synthetic.zipf_routes(t, layer=0, seed=3)).to(device)
        w = torch.softmax(torch.randn(t, K, generator=g, device=device), -1)
        d = ops.moe_dispatch(idx, E)
        xs, ws = ops.moe_gather(x, w, d)
        if want("router"):
            cases.append(("router", f"T={t}", lambda x=x: ops.router_topk(x, router, K, True),
                          t * H * 2 + E * H * 2 + t * E * 4 + t * K * 12))
        if want("dispatch"):
            cases.append(("dispatch", f"T={t} zipf", lambda idx=idx: ops.moe_dispatch(idx, E),
                          t * K * 8 + 2 * t * K * 4 + 3 * E * 4))
        if want("gather"):
            cases.append(("gather", f"T={t}", lambda x=x, w=w, d=d: ops.moe_gather(x, w, d),
                          t * H * 2 + t * K * 4 + t * K * (H * 2 + 4)))
        if want("combine"):
            ys = randn(t * K, H)
            cases.append(("combine", f"T={t}", lambda ys=ys, d=d, idx=idx: ops.moe_combine(ys, d, idx),
                          t * K * H * 2 + t * H * 2 + t * K * 12))
        if want("combine_add_rmsnorm"):
            ys, res, hn = randn(t * K, H), randn(t, H), torch.empty(t, H, **bf)
            nw = torch.ones(H, **bf)
            cases.append(("combine_add_rmsnorm", f"T={t}",
                          lambda ys=ys, d=d, idx=idx, res=res, nw=nw, hn=hn:
                          ops.moe_combine_add_rmsnorm(ys, d, idx, res, nw, 1e-6, out=hn),
                          t * K * H * 2 + 3 * t * H * 2 + t * K * 12 + H * 2))
        if want("add_rmsnorm"):
            xa, res, hn = randn(t, H), randn(t, H), torch.empty(t, H, **bf)
            nw = torch.ones(H, **bf)
            cases.append(("add_rmsnorm", f"T={t}",
                          lambda xa=xa, res=res, nw=nw, hn=hn, t=t: N.check(N.lib.sf_add_rmsnorm(
                              xa.data_ptr(), res.data_ptr(), res.data_ptr(), nw.data_ptr(), 1e-6, t, H,
                              hn.data_ptr(), cur()), "sf_add_rmsnorm"),
                          4 * t * H * 2 + H * 2))
        if want("grouped_swiglu") or "grouped_swiglu_gathered" in only:
            for kind in ("zipf", "uniform"):
                if kind == "uniform":
                    rng = np.random.default_rng(t)
                    uidx = torch.from_numpy(np.stack([rng.permutation(E)[:K] for _ in range(t)])).to(device)
                    ud = ops.moe_dispatch(uidx, E)
                    uxs, uws = ops.moe_gather(x, w, ud)
                else:
                    ud, uxs, uws = d, xs, ws
                torch.cuda.synchronize(device)
                n_act = int(ud.num_active.item())
                if want("grouped_swiglu"):
                    cases.append(("grouped_swiglu", f"T={t} {kind} ({n_act} experts)",
                                  lambda a=uxs, b=uws, c=ud: ops.grouped_swiglu(a, b, c, slot, storage, H, I),
                                  n_act * EXPERT_BYTES + t * K * (H * 2 * 2 + 4)))
                if "grouped_swiglu_gathered" in only:  # the gathered variant, only when named
                    cases.append(("grouped_swiglu_gathered", f"T={t} {kind} ({n_act} experts)",
                                  lambda c=ud, x=x, w=w: ops.grouped_swiglu_gathered(x, w, c, slot, storage, H, I),
                                  n_act * EXPERT_BYTES + t * H * 2 + t * K * (H * 2 + 4)))
    # tree_attention_tc (the tcgen05 kernel) runs only when named explicitly.
    for name, impl in (("tree_attention", N.SF_ATTN_AUTO), ("tree_attention_tc", N.SF_ATTN_TCGEN05)):
        if (name == "tree_attention" and not want(name)) or (name == "tree_attention_tc" and name not in only):
            continue
        for t, ctx in ((7, 2048), (65, 512), (65, 4096)):
            q = randn(HQ, t, D)
            kv = randn(2, HKV, ctx + t, D)
            bits = ops.tree_bits_from_parents([max(0, i - 2) for i in range(1, t)], device)
            cases.append((name, f"T={t} ctx={ctx}",
                          lambda q=q, kv=kv, bits=bits, ctx=ctx, impl=impl:
                          ops.tree_attention(q, kv[0], kv[1], bits, ctx, impl=impl),
                          (ctx + t) * HKV * D * 2 * 2 + 2 * t * HQ * D * 2))
    if want("tree_attention_batched"):
        # Configuration 5's attention: 8 requests x 65 rows x 32 heads over
        # 4,161 keys each, one batched launch against one launch per request.
        B5, T5, C5 = 8, 65, 4096
        q5 = randn(B5, HQ, T5, D)
        kv5 = [randn(B5, HKV, C5 + T5 + 31, D) for _ in range(2)]
        par5 = synthetic.random_tree(T5 - 1, max_depth=6, max_branch=4, seed=5)[1]
        bits5 = ops.tree_bits_from_parents(par5, device).unsqueeze(0).expand(B5, -1, -1).contiguous()
        out5 = torch.empty(B5, T5, HQ, D, **bf)
        k5, v5 = kv5[0][:, :, :C5 + T5], kv5[1][:, :, :C5 + T5]
        nbytes = B5 * ((C5 + T5) * HKV * D * 2 * 2 + 2 * T5 * HQ * D * 2)
        cases.append(("tree_attention_batched", f"B={B5} T={T5} ctx={C5} one launch",
                      lambda: ops.tree_attention_batched(q5, k5, v5, bits5, C5, out=out5), nbytes))
        cases.append(("tree_attention_batched", f"B={B5} T={T5} ctx={C5} one launch per request",
                      lambda: [ops.tree_attention(q5[b], k5[b], v5[b], bits5[b], C5, out=out5[b])
                               for b in range(B5)], nbytes))
    if want("dir_plan") or want("dir_fill"):
        # The device-managed cache's plan and fill kernels at configuration 2's
        # shape: 24 slots per layer, 40 routed experts, misses from a
        # page-locked pool of 8 experts.
        from specfit_b200.runtime import ExpertKey, GpuExpertCache
        from specfit_b200.runtime.qwen3_verifier import ExpertHostPool

        hp = ExpertHostPool(1, 8, 3 * H * I)
        hp.data.zero_()
        srcs = {ExpertKey(0, e): hp.data[0, e % 8] for e in range(E)}
        cache = GpuExpertCache(srcs, slot_count=24, device=device, adopt_pinned_sources=True)
        directory = cache.enter_device_mode()
        idx = torch.from_numpy(np.stack([np.random.default_rng(r).permutation(40)[:K] for r in range(65)])).to(device)
        d = ops.moe_dispatch(idx, E)
        stream = torch.cuda.current_stream(device).cuda_stream
        directory.plan(d, False, stream)
        store = cache.storage.view(24, -1)
        if want("dir_plan"):
            cases.append(("dir_plan", "E=128 S=24, 40 experts",
                          lambda: directory.plan(d, False, cur()), 24 * 16 + 128 * 4 + 6 * (128 * 8 + 24 * 8)))
        if want("dir_fill"):
            torch.cuda.synchronize(device)
            n = int(directory.fill_count[0].item())
            cases.append(("dir_fill", f"{n} experts of 9.44 MB from page-locked host memory (bytes over PCIe)",
                          lambda: directory.fill(0, store, cur()), n * EXPERT_BYTES))
        kernel_cases.keep = (hp, cache)  # alive while the cases run
    if want("logsoftmax_topk"):
        for rows in (1, 8):
            logits = randn(rows, V)
            cases.append(("logsoftmax_topk", f"rows={rows} vocab={V}",
                          lambda logits=logits: ops.logsoftmax_topk(logits, 8, 4.5), rows * V * 2))
    if want("lm_head"):
        head = randn(V, H, std=0.02)
        for rows in (7, 65):
            xr = randn(rows, H)
            cases.append(("lm_head", f"rows={rows} fused argmax (ours)",
                          lambda xr=xr: ops.linear_argmax(xr, head), V * H * 2 + rows * V * 2))
            cases.append(("lm_head", f"rows={rows} library GEMM + torch argmax",
                          lambda xr=xr: torch.nn.functional.linear(xr, head).argmax(-1), V * H * 2 + rows * V * 2))
    if want("qkv"):
        wq = randn((HQ + 2 * HKV) * D, H, std=0.02)
        xq = randn(65, H)
        yq = torch.empty(65, wq.shape[0], **bf)
        cases.append(("qkv", "rows=65 2048->5120 (ours)",
                      lambda: N.check(N.lib.sf_linear_bf16(xq.data_ptr(), 65, H, wq.data_ptr(), wq.shape[0],
                                                           yq.data_ptr(), cur()), "sf_linear_bf16"),
                      wq.numel() * 2 + 65 * (H + wq.shape[0]) * 2))
        cases.append(("qkv", "rows=65 2048->5120 library GEMM", lambda: torch.nn.functional.linear(xq, wq),
                      wq.numel() * 2 + 65 * (H + wq.shape[0]) * 2))
    if want("linear"):
        for rows, n_in, n_out in ((7, HQ * D, H), (8, 3 * H, H)):
            xw = randn(rows, n_in)
            wt = randn(n_out, n_in, std=0.02)
            cases.append(("linear", f"rows={rows} {n_in}->{n_out}",
                          lambda xw=xw, wt=wt: ops.linear(xw, wt), n_out * n_in * 2 + rows * (n_in + n_out) * 2))
    return cases


def kernels_mode(args):
    """Each hot kernel alone (``kernel_cases``): per launch, CUDA events
    around it with L2 flushed before it (a 256 MB write outside the events:
    "cold"), the mean of back-to-back launches ("warm", the in-pass case
    where the producer's output is still in L2), and the mean of the same
    back-to-back launches replayed from one CUDA graph ("graph": no host
    launch cost between them, as inside the verify pass; null where the case
    cannot be captured).  One JSON line per case: us, algorithmic bytes,
    GB/s and the fraction of the measured HBM copy peak (cold).  Small
    enough to run whole under a profiler with -k/-c."""
    device = torch.device("cuda", 0)
    peaks = measured_peaks()
    only = tuple(k for k in args.kernel.split(",") if k)
    cases = kernel_cases(device, only, tuple(int(r) for r in args.kernel_rows.split(",") if r))
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    iters = max(args.steps, 3)
    for name, case, fn, algo in cases:
        for _ in range(max(args.warmup, 3)):
            fn()
        pairs = []
        for r in range(iters):
            flush.fill_(r & 0xFF)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn()
            b.record(stream)
            pairs.append((a, b))
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(iters):
            fn()
        b.record(stream)
        torch.cuda.synchronize(device)
        cold = statistics.median(x.elapsed_time(y) * 1e3 for x, y in pairs)
        warm = a.elapsed_time(b) * 1e3 / iters
        graph_us = None
        try:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for _ in range(iters):
                    fn()
            graph.replay()
            ga, gb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ga.record(stream)
            graph.replay()
            gb.record(stream)
            torch.cuda.synchronize(device)
            graph_us = round(ga.elapsed_time(gb) * 1e3 / iters, 2)
            del graph
        except RuntimeError:
            torch.cuda.synchronize(device)
        print(json.dumps({"mode": "kernels", "kernel": name, "case": case, "us_cold": round(cold, 2),
                          "us_warm": round(warm, 2), "us_graph": graph_us, "algorithmic_bytes": int(algo),
                          "GBps_cold": round(algo / cold / 1e3, 1),
                          "frac_of_hbm_peak_cold": round(algo / cold / 1e3 / peaks["hbm_gbs"], 4),
                          "us_at_peak": round(algo / peaks["hbm_gbs"] / 1e3, 2),
                          "peak_source": peaks["source"] + " hbm_gbs"}), flush=True)


def num_sms_of(device) -> int:
    return torch.cuda.get_device_properties(device).multi_processor_count


def main(argv=None):
    args = parse_args(argv)
    if args.impl == "reference":
        reference_arm(args)
    elif args.mode == "block":
        block_mode(args)
    elif args.mode == "graph":
        graph_mode(args)
    elif args.mode == "decode":
        decode_mode(args)
    elif args.mode == "sweep":
        sweep_mode(args)
    elif args.mode == "kernels":
        kernels_mode(args)
    elif args.mode == "ep" or (args.mode == "auto" and dist_info()[1] > 1):
        ep_arm(args)
    else:
        b200_arm(args)


if __name__ == "__main__":
    main()
