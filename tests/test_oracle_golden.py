"""Pin the CPU oracle against golden vectors produced by the reference itself
(``tests/golden/make_golden.py``).  CPU only."""
import numpy as np
import pytest
import torch

from oracle import moe_oracle as mo
from oracle import tree_oracle as to
from specfit_b200 import synthetic


def bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def test_bf16_round_matches_torch():
    rng = np.random.default_rng(0)
    vals = np.concatenate([rng.standard_normal(100000).astype(np.float32) * 10,
                           np.array([0.0, -0.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, 65504.0], np.float32)])
    ref = torch.from_numpy(vals).to(torch.bfloat16).float().numpy()
    assert np.array_equal(mo.bf16_round(vals), ref)


def test_f64_to_bf16_single_rounding():
    rng = np.random.default_rng(1)
    vals = rng.standard_normal(100000) * 3
    got = mo.f64_to_bf16(vals).astype(np.float64)
    # Correct rounding: no other bf16 value is closer.
    ulp = np.ldexp(1.0, np.frexp(got)[1] - 8)
    assert np.all(np.abs(got - vals) <= ulp / 2 + 1e-300)
    # Through torch (double -> bf16) agrees except where double rounding bites.
    via_torch = torch.from_numpy(vals).to(torch.bfloat16).double().numpy()
    assert np.mean(via_torch == got) > 0.999


def test_router_cfg1_f32_indices_bit_exact(golden_dir):
    g = np.load(golden_dir / "moe_cfg1_f32.npz")
    weights, x = synthetic.config1_inputs(seed=0, tokens=32)
    probs, w, idx, logits = mo.router_topk(x.numpy(), weights.router.numpy(), 8, True, "f32")
    assert np.array_equal(idx, g["idx"])
    np.testing.assert_allclose(w, g["weights"], rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(probs, g["probs"], rtol=1e-5, atol=1e-8)
    np.testing.assert_allclose(logits, g["logits"], rtol=1e-5, atol=1e-5)


def test_router_bf16_t65_indices(golden_dir):
    """bf16 logits: equal to the reference's own wherever its fp32-accumulated
    GEMM rounds like the exact sum; every index difference is explained by a
    one-ulp logit difference or an exact tie at the top-k cut."""
    g = np.load(golden_dir / "moe_bf16_t65.npz")
    weights, x = synthetic.bf16_layer_inputs(seed=11, tokens=65)
    xf = x.float().numpy()
    wf = weights.router.float().numpy()
    probs, w, idx, logits = mo.router_topk(xf, wf, 8, True, "bf16")
    ref_logits = bits_to_f32(g["logits_bits"])
    differ = logits != ref_logits
    assert differ.mean() < 0.01
    # Same logits -> the same expert SET per token (ties at the cut aside).
    _, _, idx_on_ref, _ = mo.router_topk(xf, wf, 8, True, "bf16")
    ref_idx = g["idx"]
    ties = mo.boundary_ties(ref_logits, 8)
    for t in range(idx.shape[0]):
        mine = set(mo.topk_lowest_id(ref_logits[t:t + 1], 8)[0].tolist())
        theirs = set(ref_idx[t].tolist())
        if not ties[t]:
            assert mine == theirs, t
        else:
            # The reference picked among equal values at the cut.
            cut = np.sort(ref_logits[t])[::-1][7]
            assert {e for e in mine ^ theirs} <= set(np.nonzero(ref_logits[t] == cut)[0].tolist())
    assert idx_on_ref.shape == ref_idx.shape


def test_moe_cfg1_f32_block(golden_dir):
    g = np.load(golden_dir / "moe_cfg1_f32.npz")
    weights, x = synthetic.config1_inputs(seed=0, tokens=32)
    packed = {e: weights.packed(e).numpy() for e in np.unique(g["idx"])}
    out = mo.moe_experts(x.numpy(), g["idx"], g["weights"], packed, 2048, 768, "f32")
    np.testing.assert_allclose(out, g["out_specfit"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(g["out_hf"], g["out_specfit"], rtol=1e-5, atol=1e-6)


def test_moe_bf16_t65_block(golden_dir):
    g = np.load(golden_dir / "moe_bf16_t65.npz")
    weights, x = synthetic.bf16_layer_inputs(seed=11, tokens=65)
    idx = g["idx"]
    packed = {e: weights.packed(e).float().numpy() for e in np.unique(idx)}
    out = mo.moe_experts(x.float().numpy(), idx, g["weights"], packed, 2048, 768, "bf16")
    ref = bits_to_f32(g["out_specfit_bits"])
    err = np.abs(out - ref).max()
    cos = float((out * ref).sum() / np.linalg.norm(out) / np.linalg.norm(ref))
    assert err <= 2e-2 and cos >= 0.999, (err, cos)


@pytest.mark.parametrize("case", ["t65_uniform", "t1", "t512_zipf", "t129_zipf", "t7_k3_e5", "t4_one_expert"])
def test_dispatch_bit_exact(golden_dir, case):
    g = np.load(golden_dir / "dispatch.npz")
    idx = g[f"{case}__idx"]
    num_experts = 5 if case == "t7_k3_e5" else 128
    counts, offsets, sorted_pos, inv_pos, active, n_active = mo.dispatch(idx, num_experts)
    assert np.array_equal(sorted_pos, g[f"{case}__positions"])
    assert np.array_equal(active[:n_active], g[f"{case}__unique"])
    assert np.array_equal(counts[active[:n_active]], g[f"{case}__counts"])
    assert np.array_equal(sorted_pos // idx.shape[1], g[f"{case}__route_tokens"])
    assert np.array_equal(sorted_pos // idx.shape[1], g[f"{case}__where_tokens"])
    assert np.array_equal(np.argsort(inv_pos), sorted_pos)


def test_expert_kats(golden_dir):
    g = np.load(golden_dir / "expert_kats.npz")
    gate_up = bits_to_f32(g["small_gate_up_bits"])
    down = bits_to_f32(g["small_down_bits"])
    packed = {e: np.concatenate([gate_up[e, :3].ravel(), gate_up[e, 3:].ravel(), down[e].ravel()])
              for e in range(3)}
    x = bits_to_f32(g["small_x_bits"])
    w = bits_to_f32(g["small_w_bits"])
    out = mo.moe_experts(x, g["small_idx"], w, packed, 4, 3, "bf16")
    ref = bits_to_f32(g["small_out_012_bits"])
    assert np.array_equal(bits_to_f32(g["small_out_210_bits"]), ref)
    np.testing.assert_allclose(out, ref, atol=1.6e-2, rtol=1.6e-2)
    # Reduction-order KAT: arrival (0,1,2) rounds 2**-8 away, (0,2,1) keeps it.
    kat_down = bits_to_f32(g["kat_down_bits"])
    kat = {e: np.array([1.0, 1.0, kat_down[e, 0, 0]], np.float32) for e in range(3)}
    ones = np.ones((1, 1), np.float32)
    idx = np.array([[0, 1, 2]])
    wk = np.ones((1, 3), np.float32)
    a012 = mo.moe_experts(ones, idx, wk, kat, 1, 1, "bf16", order=(0, 1, 2))
    a021 = mo.moe_experts(ones, idx, wk, kat, 1, 1, "bf16", order=(0, 2, 1))
    assert a012[0, 0] == g["kat_arrival_012"][0, 0] == 0.0
    assert a021[0, 0] == g["kat_arrival_021"][0, 0] == 2.0 ** -8
    assert g["kat_canonical_021"][0, 0] == 0.0


@pytest.mark.parametrize("case", ["kat5", "t64", "t128", "t60"])
def test_tree_helpers(golden_dir, case):
    g = np.load(golden_dir / "tree.npz")
    parents = tuple(int(p) for p in g[f"{case}__parents"])
    tokens = tuple(int(t) for t in g[f"{case}__tokens"])
    depths = tuple(int(d) for d in g[f"{case}__depths"])
    base = int(g[f"{case}__base"])
    mask = to.verification_attention_mask(parents, base)
    assert np.array_equal(mask[:, base:], g[f"{case}__mask_tree"])
    assert bool(g[f"{case}__prefix_all"]) and mask[:, :base].all()
    assert np.array_equal(to.verification_position_ids(depths, base), g[f"{case}__positions"])
    assert to.accepted_path(parents, tokens, g[f"{case}__verifier"]) == tuple(g[f"{case}__accepted"].tolist())
    bits = to.ancestor_bits(parents)
    q = 1 + len(parents)
    unpacked = np.array([[(bits[i, j // 32] >> (j % 32)) & 1 for j in range(q)] for i in range(q)], bool)
    assert np.array_equal(unpacked, g[f"{case}__mask_tree"])


def test_synthetic_tree_shape():
    tok, par, dep = synthetic.random_tree(64, max_depth=6, max_branch=4, seed=2)
    assert len(tok) == 64 and max(dep) == 6
    assert all(sum(1 for p in par if p == n) <= 4 for n in range(65))
