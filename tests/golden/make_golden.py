"""Generate the golden fixtures under ``tests/golden/`` from the SpecFit
reference itself.

Run in a container where the reference source tree is available:

    python tests/golden/make_golden.py --reference /path/to/SpecFit

The reference is imported through ``reference_shim`` (its two absent
third-party packages are import-only stubs) and executed on the CPU:

* the router and sparse-MoE block are Hugging Face ``transformers``'
  ``Qwen3MoeTopKRouter`` / ``Qwen3MoeSparseMoeBlock`` (the reference's target
  model, ``src/specfit/runtime/qwen3_offloaded_model.py:741-747``);
* the expert block is the reference's own ``Qwen3OffloadedExperts.forward``
  (``src/specfit/runtime/qwen3_offloaded_experts.py:98-164``), driven through
  a CPU stand-in for ``GpuExpertCache`` that hands out the packed expert
  tensors (the cache needs CUDA; the arithmetic does not);
* dispatch fixtures are the reference's grouping ops
  (``qwen3_offloaded_experts.py:173-178``);
* tree fixtures are ``Eagle3DraftTree`` (``runtime/eagle3_types.py:429-502``).

The fixtures store outputs only; inputs are regenerated from the seeds with
``specfit_b200.synthetic`` (the same torch CPU generator draws), so the files
stay small.  bf16 tensors are stored as their uint16 bit patterns.
"""
from __future__ import annotations

import argparse
import math
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(HERE))

from specfit_b200 import synthetic  # noqa: E402


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16)


class _CpuLease:
    def __init__(self, tensor):
        self._tensor = tensor

    def wait(self, stream=None):
        return self._tensor

    def release(self):
        pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.release()


class _CpuCache:
    """Minimal stand-in for GpuExpertCache on the CPU (no eviction)."""

    def __init__(self, sources):
        self.device = torch.device("cpu")
        self._sources = dict(sources)

    def acquire(self, key):
        return _CpuLease(self._sources[key])

    def _prefetch(self, key):
        return _CpuLease(self._sources[key])

    def resident_expert_ids(self):
        return ()


def reference_experts(ref, weights: synthetic.MoeLayerWeights, hidden, idx, topw, *, order=None,
                      reduction="canonical"):
    from specfit.state import ExpertKey

    inter = weights.down.shape[2]
    sources = {ExpertKey(0, e): weights.packed(e) for e in range(weights.router.shape[0])}
    module = ref.Qwen3OffloadedExperts(
        layer_id=0,
        cache=_CpuCache(sources),
        hidden_size=weights.router.shape[1],
        intermediate_size=inter,
        reduction_mode=reduction,
    )
    with torch.no_grad():
        return module(hidden, idx, topw, execution_order=order)


def hf_block(weights: synthetic.MoeLayerWeights, dtype, top_k=8):
    from transformers import Qwen3MoeConfig
    from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeSparseMoeBlock

    experts, hidden = weights.router.shape
    config = Qwen3MoeConfig(
        hidden_size=hidden,
        moe_intermediate_size=weights.down.shape[2],
        num_experts=experts,
        num_experts_per_tok=top_k,
        norm_topk_prob=True,
        hidden_act="silu",
    )
    block = Qwen3MoeSparseMoeBlock(config).to(dtype)
    with torch.no_grad():
        block.gate.weight.copy_(weights.router)
        block.experts.gate_up_proj.copy_(weights.gate_up)
        block.experts.down_proj.copy_(weights.down)
    return block.eval()


def make_cfg1(ref, out: Path):
    weights, x = synthetic.config1_inputs(seed=0, tokens=32)
    block = hf_block(weights, torch.float32)
    with torch.no_grad():
        probs, topw, idx = block.gate(x)
        out_hf = block(x.unsqueeze(0))[0]
        out_sf = reference_experts(ref, weights, x, idx, topw)
        logits = torch.nn.functional.linear(x, weights.router)
    np.savez_compressed(
        out / "moe_cfg1_f32.npz",
        idx=idx.numpy(),
        weights=topw.numpy(),
        probs=probs.numpy(),
        logits=logits.numpy(),
        out_hf=out_hf.numpy(),
        out_specfit=out_sf.numpy(),
    )
    print("cfg1: unique experts", len(torch.unique(idx)))


def make_bf16_layer(ref, out: Path, seed: int, tokens: int, name: str):
    weights, x = synthetic.bf16_layer_inputs(seed=seed, tokens=tokens)
    block = hf_block(weights, torch.bfloat16)
    with torch.no_grad():
        logits = torch.nn.functional.linear(x, weights.router)
        probs, topw, idx = block.gate(x)
        out_sf = reference_experts(ref, weights, x, idx, topw)
        out_hf = block(x.unsqueeze(0))[0]
    np.savez_compressed(
        out / f"{name}.npz",
        logits_bits=bf16_bits(logits),
        probs=probs.float().numpy(),
        weights=topw.float().numpy(),
        idx=idx.numpy(),
        out_specfit_bits=bf16_bits(out_sf),
        out_hf_bits=bf16_bits(out_hf),
    )
    print(name, "unique experts", len(torch.unique(idx)))


def make_dispatch(out: Path):
    """The reference grouping: stable sort, unique_consecutive, route tokens
    (qwen3_offloaded_experts.py:173-178) and per-expert torch.where (:120)."""
    cases = {}
    rng = np.random.default_rng(5)
    shapes = {
        "t65_uniform": rng.integers(0, 128, size=(65, 8)),
        "t1": rng.permutation(128)[:8].reshape(1, 8),
        "t512_zipf": synthetic.zipf_routes(512, layer=3, seed=7),
        "t129_zipf": synthetic.zipf_routes(129, layer=0, seed=1),
        "t7_k3_e5": rng.integers(0, 5, size=(7, 3)),
        "t4_one_expert": np.full((4, 8), 17),
    }
    for name, idx in shapes.items():
        idx_t = torch.as_tensor(np.asarray(idx), dtype=torch.long)
        sorted_ids, positions = torch.sort(idx_t.reshape(-1), stable=True)
        unique, counts = torch.unique_consecutive(sorted_ids, return_counts=True)
        route_tokens = torch.div(positions, idx_t.shape[1], rounding_mode="floor")
        where_tokens = []
        for e in unique.tolist():
            tok, _ = torch.where(idx_t == e)
            where_tokens.append(tok.numpy())
        cases[f"{name}__idx"] = idx_t.numpy()
        cases[f"{name}__positions"] = positions.numpy()
        cases[f"{name}__unique"] = unique.numpy()
        cases[f"{name}__counts"] = counts.numpy()
        cases[f"{name}__route_tokens"] = route_tokens.numpy()
        cases[f"{name}__where_tokens"] = (
            np.concatenate(where_tokens) if where_tokens else np.zeros(0, np.int64)
        )
    np.savez_compressed(out / "dispatch.npz", **cases)


def make_expert_kats(ref, out: Path):
    """Small cases of tests/gpu/test_qwen3_offloaded_experts.py run on CPU."""
    import torch.nn.functional as F

    res = {}
    # (a) :60-156 canonical output invariant to execution order, H=4, I=3.
    hidden, inter = 4, 3
    g = torch.Generator().manual_seed(29)
    gate_up = torch.randn(3, 2 * inter, hidden, dtype=torch.bfloat16, generator=g)
    down = torch.randn(3, hidden, inter, dtype=torch.bfloat16, generator=g)
    x = torch.randn(2, hidden, dtype=torch.bfloat16, generator=g)
    idx = torch.tensor([[0, 1, 2], [2, 0, 1]], dtype=torch.long)
    w = torch.tensor([[0.50, 0.30, 0.20], [0.45, 0.35, 0.20]], dtype=torch.bfloat16)
    weights = synthetic.MoeLayerWeights(torch.zeros(3, hidden), gate_up, down)
    res["small_gate_up_bits"] = bf16_bits(gate_up)
    res["small_down_bits"] = bf16_bits(down)
    res["small_x_bits"] = bf16_bits(x)
    res["small_idx"] = idx.numpy()
    res["small_w_bits"] = bf16_bits(w)
    res["small_out_012_bits"] = bf16_bits(reference_experts(ref, weights, x, idx, w, order=(0, 1, 2)))
    res["small_out_210_bits"] = bf16_bits(reference_experts(ref, weights, x, idx, w, order=(2, 1, 0)))
    # (b) :379-458 bf16 reduction order matters: 1, 2**-8, -1.
    silu_one = F.silu(torch.tensor(1.0, dtype=torch.bfloat16)).item()
    desired = (1.0, 2.0 ** -8, -1.0)
    gu = torch.ones(3, 2, 1, dtype=torch.bfloat16)
    dn = torch.tensor([[[v / silu_one]] for v in desired], dtype=torch.bfloat16)
    kat = synthetic.MoeLayerWeights(torch.zeros(3, 1), gu, dn)
    xk = torch.ones(1, 1, dtype=torch.bfloat16)
    ik = torch.tensor([[0, 1, 2]], dtype=torch.long)
    wk = torch.ones(1, 3, dtype=torch.bfloat16)
    res["kat_down_bits"] = bf16_bits(dn)
    res["kat_arrival_012"] = reference_experts(
        ref, kat, xk, ik, wk, order=(0, 1, 2), reduction="arrival_order").float().numpy()
    res["kat_arrival_021"] = reference_experts(
        ref, kat, xk, ik, wk, order=(0, 2, 1), reduction="arrival_order").float().numpy()
    res["kat_canonical_021"] = reference_experts(
        ref, kat, xk, ik, wk, order=(0, 2, 1), reduction="canonical").float().numpy()
    np.savez_compressed(out / "expert_kats.npz", **res)
    print("kat arrival 012/021:", res["kat_arrival_012"], res["kat_arrival_021"])


def make_tree(out: Path):
    from specfit.runtime.eagle3_types import Eagle3DraftTree

    def tree_from(tokens, parents, depths, seed):
        rng = np.random.default_rng(seed)
        cond = tuple(float(p) for p in rng.uniform(0.05, 1.0, size=len(tokens)))
        cum = []
        for i, parent in enumerate(parents):
            base = 0.0 if parent == 0 else cum[parent - 1]
            cum.append(base + math.log(cond[i]))
        return Eagle3DraftTree(token_ids=tuple(tokens), parent_ids=tuple(parents), depths=tuple(depths),
                               conditional_probabilities=cond, cumulative_log_probabilities=tuple(cum))

    res = {}
    cases = {
        "kat5": ((7, 2, 6, 3), (0, 0, 1, 2), (1, 1, 2, 2), 2, [2, 0, 3, 0, 4]),
    }
    t64 = synthetic.random_tree(64, max_depth=6, max_branch=4, seed=2)
    t128 = synthetic.random_tree(128, max_depth=8, max_branch=4, seed=3)
    t60 = synthetic.random_tree(60, max_depth=8, max_branch=4, seed=4)
    for name, (tok, par, dep) in (("t64", t64), ("t128", t128), ("t60", t60)):
        # Verifier predictions that walk down a deep path then stop.
        rng = np.random.default_rng(len(tok))
        verifier = rng.integers(0, synthetic.VOCAB, size=1 + len(tok))
        node = 0
        for _ in range(4):
            kids = [i for i, p in enumerate(par, start=1) if p == node]
            if not kids:
                break
            pick = kids[-1]
            verifier[node] = tok[pick - 1]
            node = pick
        cases[name] = (tok, par, dep, 512, verifier.tolist())
    for name, (tok, par, dep, base, verifier) in cases.items():
        tree = tree_from(tok, par, dep, seed=len(tok))
        mask = tree.verification_attention_mask(base_kv_length=base, device=torch.device("cpu"))
        pos = tree.verification_position_ids(base_kv_length=base, device=torch.device("cpu"))
        acc = tree.accepted_path(torch.tensor([verifier]))
        res[f"{name}__tokens"] = np.array(tok, dtype=np.int64)
        res[f"{name}__parents"] = np.array(par, dtype=np.int64)
        res[f"{name}__depths"] = np.array(dep, dtype=np.int64)
        res[f"{name}__base"] = np.array(base)
        res[f"{name}__verifier"] = np.array(verifier, dtype=np.int64)
        res[f"{name}__mask_tree"] = mask[0, 0, :, base:].numpy()
        res[f"{name}__prefix_all"] = np.array(bool(mask[0, 0, :, :base].all()))
        res[f"{name}__positions"] = pos[0].numpy()
        res[f"{name}__accepted"] = np.array(acc, dtype=np.int64)
    np.savez_compressed(out / "tree.npz", **res)


def make_selection(out: Path):
    """SpecFit exact selection (src/specfit/specfit_exact.py:58-94) and the
    adaptive-depth rule of LevelSpecFit (src/specfit/main_comparison.py:63-103)
    on seeded pools; inputs are regenerated from the stored parameters by
    specfit_b200.synthetic.selection_case."""
    import json
    from types import SimpleNamespace

    from specfit.main_comparison import LevelSpecFit
    from specfit.selection_methods import SelectionCostModel, probability_ids
    from specfit.selection_refinement import CacheCostModel
    from specfit.specfit_exact import exact_specfit_selection

    def objects(case):
        n = len(case.parents)
        nodes = [SimpleNamespace(raw_id=i + 1, parent_raw_id=case.parents[i], depth=case.depths[i],
                                 generation_ordinal=i,
                                 cumulative_log_probability=case.cum_logp[i]) for i in range(n)]
        pool = SimpleNamespace(nodes=nodes)
        atlas = SimpleNamespace(position_to_raw=tuple(range(n + 1)), expert_ids_by_raw_layer=tuple(
            (raw, layer, tuple(int(e) for e in case.routes[raw, layer]))
            for raw in range(n + 1) for layer in range(48)))
        atlas48 = [tuple(tuple(int(e) for e in case.routes[raw, layer]) for raw in range(n + 1))
                   for layer in range(48)]
        resident = 0
        for layer in range(48):
            for e in np.nonzero(case.resident[layer])[0]:
                resident |= 1 << (128 * layer + int(e))
        return pool, atlas, atlas48, resident

    B, beta = synthetic.SELECTION_INTERCEPT_NS, synthetic.SELECTION_EXPERT_NS
    models = {
        "natural": dict(kind="selection", intercept=list(B), expert_ns=beta, missing_ns=0.0),
        "cache": dict(kind="cache", intercept=list(B), expert_ns=beta, missing_ns=0.9 * beta),
        "flat": dict(kind="selection", intercept=[1.0] * 8, expert_ns=1.0, missing_ns=0.0),
        "steep": dict(kind="selection", intercept=[1.0] + [1e12] * 7, expert_ns=1.0, missing_ns=0.0),
    }

    def build(m):
        if m["kind"] == "cache":
            return CacheCostModel(tuple(m["intercept"]), m["expert_ns"], m["missing_ns"])
        return SelectionCostModel(tuple(m["intercept"]), tuple(m["intercept"]), m["expert_ns"])

    cases = []
    for n in (2, 6, 10, 14, 18):
        for seed in range(8):
            for name in ("natural", "cache"):
                cases.append(dict(seed=seed, n=n, shared=False, level_prob=None, model=models[name],
                                  resident=name == "cache"))
    for seed in range(3):
        for name in ("natural", "flat", "steep", "cache"):
            cases.append(dict(seed=100 + seed, n=18, shared=True, level_prob=None, model=models[name],
                              resident=name == "cache"))
    # The reference's compensated-summation tie case (tests/unit/
    # test_selection_refinement.py:65-78): equal footprints, intercepts equal
    # to the probability-ranked rewards.
    kat = synthetic.selection_case(7, 18, shared_routes=True,
                                   level_prob=(0.47454250539060727, 0.35255387827663837))
    kpool, _, _, _ = objects(kat)
    probs = {nd.raw_id: math.exp(nd.cumulative_log_probability) for nd in kpool.nodes}
    offsets = [1.0 + sum((probs[i] for i in probability_ids(kpool, k)), start=0.0) for k in range(8)]
    cases.append(dict(seed=7, n=18, shared=True, level_prob=[0.47454250539060727, 0.35255387827663837],
                      model=dict(kind="selection", intercept=offsets, expert_ns=0.0, missing_ns=0.0),
                      resident=False))
    for c in cases:
        case = synthetic.selection_case(c["seed"], c["n"], shared_routes=c["shared"],
                                        level_prob=c["level_prob"])
        pool, atlas, atlas48, resident = objects(case)
        model = build(c["model"])
        c["selected"] = list(exact_specfit_selection(pool, atlas, model,
                                                     resident if c["resident"] else 0))
        if c["model"]["kind"] == "selection":
            level = LevelSpecFit(model, atlas48)
            stops = []
            for prefix in range(2, c["n"] + 1, 4):
                stop, ids = level.stop(pool.nodes[:prefix])
                stops.append([prefix, bool(stop), list(ids)])
            c["stops"] = stops
    (out / "selection.json").write_text(json.dumps(cases))
    print("selection cases", len(cases), "kat selection", cases[-1]["selected"])


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", default=os.environ.get("SPECFIT_REFERENCE", ""),
                        help="root of the SpecFit reference checkout")
    parser.add_argument("--only", default="")
    args = parser.parse_args()
    if not args.reference:
        parser.error("--reference is required")
    import reference_shim

    reference_shim.install(str(Path(args.reference) / "src"))
    torch.set_num_threads(os.cpu_count() or 1)
    from specfit.runtime import qwen3_offloaded_experts as ref

    out = HERE
    jobs = {
        "cfg1": lambda: make_cfg1(ref, out),
        "bf16": lambda: make_bf16_layer(ref, out, seed=11, tokens=65, name="moe_bf16_t65"),
        "dispatch": lambda: make_dispatch(out),
        "kats": lambda: make_expert_kats(ref, out),
        "tree": lambda: make_tree(out),
        "selection": lambda: make_selection(out),
    }
    for name, job in jobs.items():
        if args.only and name not in args.only.split(","):
            continue
        job()


if __name__ == "__main__":
    main()
