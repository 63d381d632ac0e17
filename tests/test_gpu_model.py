"""Verify pass of a small Qwen3-MoE target on the B200 path.

* Logits of a tree verify pass match the stock Hugging Face model (SDPA,
  stock sparse-MoE block) holding the same weights.
* Each tree node's logits equal those of an independent causal pass over the
  node's own path (the property of the reference's
  tests/gpu/test_eagle3_tree.py:1435 and test_eagle3_equivalence.py:18).
"""
import math

import numpy as np
import pytest
import torch

from specfit_b200 import synthetic

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def small_config():
    from specfit_b200.runtime.qwen3_verifier import qwen3_moe_config

    return qwen3_moe_config(2, hidden=256, experts=16, top_k=4, moe_inter=128, heads=8, kv_heads=2,
                            head_dim=128, vocab=512)


@pytest.fixture(scope="module")
def loaded():
    from specfit_b200.runtime.qwen3_verifier import build_random_offloaded_qwen3

    cfg = small_config()
    m = build_random_offloaded_qwen3(device=DEV, slots_per_layer=16, config=cfg, seed=3, std=0.05)
    yield m
    m.close()


def hf_twin(loaded):
    """Stock HF model with the same weights (SDPA attention, stock MoE)."""
    from transformers import Qwen3MoeForCausalLM

    cfg = small_config()
    cfg._attn_implementation = "sdpa"
    ref = Qwen3MoeForCausalLM(cfg).to(DEV, torch.bfloat16).eval()
    src = dict(loaded.model.named_parameters())
    pool = loaded.pool.data
    inter, hid = cfg.moe_intermediate_size, cfg.hidden_size
    with torch.no_grad():
        for name, p in ref.named_parameters():
            if ".mlp.experts." in name:
                layer = int(name.split(".")[2])
                w = pool[layer].to(DEV)
                if name.endswith("gate_up_proj"):
                    p.copy_(w[:, : 2 * inter * hid].reshape(-1, 2 * inter, hid))
                else:
                    p.copy_(w[:, 2 * inter * hid:].reshape(-1, hid, inter))
            else:
                p.copy_(src[name])
    return ref


def make_tree(nodes=12, depth=4, seed=1):
    from specfit_b200.runtime.eagle3_types import Eagle3DraftTree

    tok, par, dep = synthetic.random_tree(nodes, max_depth=depth, max_branch=3, seed=seed, vocab=512)
    cond, cum = [], []
    rng = np.random.default_rng(seed)
    for i, p in enumerate(par):
        c = float(rng.uniform(0.1, 1.0))
        cond.append(c)
        cum.append((0.0 if p == 0 else cum[p - 1]) + math.log(c))
    return Eagle3DraftTree(tok, par, dep, tuple(cond), tuple(cum))


def verify_logits(model, ctx_ids, tree, seed_tok):
    from transformers import DynamicCache

    cache = DynamicCache(config=model.config)
    with torch.no_grad():
        model(input_ids=ctx_ids, past_key_values=cache, use_cache=True)
        base = ctx_ids.shape[1]
        ids = tree.verification_token_ids(torch.tensor([[seed_tok]], device=DEV))
        mask = tree.verification_attention_mask(base_kv_length=base, device=DEV)
        pos = tree.verification_position_ids(base_kv_length=base, device=DEV)
        out = model(input_ids=ids, attention_mask=mask, position_ids=pos, past_key_values=cache,
                    use_cache=True)
    return out.logits[0].float()


def test_verify_pass_matches_stock_hf(loaded):
    ref = hf_twin(loaded)
    ctx = torch.randint(0, 512, (1, 40), generator=torch.Generator().manual_seed(0)).to(DEV)
    tree = make_tree()
    mine = verify_logits(loaded.model, ctx, tree, 7)
    theirs = verify_logits(ref, ctx, tree, 7)
    cos = torch.nn.functional.cosine_similarity(mine, theirs, dim=-1)
    assert cos.min().item() >= 0.99, cos
    agree = (mine.argmax(-1) == theirs.argmax(-1)).float().mean().item()
    assert agree >= 0.9, agree


def test_tree_nodes_equal_causal_paths(loaded):
    from transformers import DynamicCache

    model = loaded.model
    ctx = torch.randint(0, 512, (1, 33), generator=torch.Generator().manual_seed(1)).to(DEV)
    tree = make_tree(nodes=10, depth=5, seed=4)
    tree_logits = verify_logits(model, ctx, tree, 11)
    for node in (0, 3, 7, 10):
        path = []
        n = node
        while n:
            path.append(tree.token_ids[n - 1])
            n = tree.parent_ids[n - 1]
        ids = torch.tensor([[11] + path[::-1]], device=DEV)
        cache = DynamicCache(config=model.config)
        with torch.no_grad():
            model(input_ids=ctx, past_key_values=cache, use_cache=True)
            out = model(input_ids=ids, past_key_values=cache, use_cache=True).logits[0, -1].float()
        cos = torch.nn.functional.cosine_similarity(out, tree_logits[node], dim=0).item()
        assert cos >= 0.999, (node, cos)
        assert out.argmax().item() == tree_logits[node].argmax().item()


def test_pool_is_page_locked(loaded):
    assert loaded.pool.data[0, 0].is_pinned()
    assert all(c.sources_are_pinned for c in loaded.caches)


@pytest.mark.parametrize("reserved", [False, True])
def test_verify_graph_replay_equals_eager(reserved):
    """A captured verify pass (every expert resident) replays bit for bit,
    over a DynamicCache or an in-place ReservedCache; the eager reference
    always uses Hugging Face's DynamicCache."""
    from transformers import DynamicCache

    from specfit_b200.runtime.kv_cache import ReservedCache
    from specfit_b200.runtime.qwen3_verifier import build_random_offloaded_qwen3
    from specfit_b200.runtime.verify_graph import VerifyGraph

    m = build_random_offloaded_qwen3(device=DEV, slots_per_layer=16, config=small_config(), seed=5,
                                     std=0.05)
    try:
        m.warm_all_caches()
        model = m.model
        ctx = torch.randint(0, 512, (1, 37), generator=torch.Generator().manual_seed(2)).to(DEV)
        cache = DynamicCache(config=model.config)
        with torch.no_grad():
            model(input_ids=ctx, past_key_values=cache, use_cache=True)
        trees = [make_tree(nodes=9, depth=4, seed=s) for s in (1, 2)]
        inputs = []
        for tree in trees:
            ids = tree.verification_token_ids(torch.tensor([[5]], device=DEV))
            mask = tree.verification_attention_mask(base_kv_length=37, device=DEV)
            pos = tree.verification_position_ids(base_kv_length=37, device=DEV)
            inputs.append((ids, mask, pos))
        eager = []
        for ids, mask, pos in inputs:
            with torch.no_grad():
                out = model(input_ids=ids, attention_mask=mask, position_ids=pos, past_key_values=cache,
                            use_cache=True)
            eager.append(out.logits[0].clone())
            cache.crop(37)
        if reserved:
            cache = ReservedCache(config=model.config, capacity=47)
            with torch.no_grad():
                model(input_ids=ctx, past_key_values=cache, use_cache=True)
            for (ids, mask, pos), ref in zip(inputs, eager):  # eager passes over the reserved cache
                with torch.no_grad():
                    out = model(input_ids=ids, attention_mask=mask, position_ids=pos,
                                past_key_values=cache, use_cache=True)
                assert torch.equal(out.logits[0], ref)
                cache.crop(37)
        vg = VerifyGraph(model, cache, q_len=10, device=DEV)
        vg.capture(*inputs[0])
        hits_before = m.caches[0].stats().resident_hits
        for (ids, mask, pos), ref in zip(inputs, eager):
            vg.load(ids, mask, pos)
            vg.replay()
            torch.cuda.synchronize()
            assert torch.equal(vg.logits[0], ref)
        assert cache.get_seq_length() == 37
        assert m.caches[0].stats().resident_hits > hits_before  # replays count hits
    finally:
        m.close()


def test_lean_forward_matches_hf_forward():
    """The lean forward (fused norms, q/k norm + rotary + cache write, fused
    q|k|v GEMM) gives the Hugging Face forward's logits within bf16
    tolerance, for a prefill and a tree-masked verify pass, and leaves the
    same cache rows."""
    from specfit_b200.runtime.kv_cache import ReservedCache
    from specfit_b200.runtime.lean_forward import LeanQwen3Forward
    from specfit_b200.runtime.qwen3_verifier import build_random_offloaded_qwen3

    m = build_random_offloaded_qwen3(device=DEV, slots_per_layer=16, config=small_config(), seed=5,
                                     std=0.05)
    try:
        m.warm_all_caches()
        model = m.model
        lean = LeanQwen3Forward(model)
        ctx = torch.randint(0, 512, (1, 37), generator=torch.Generator().manual_seed(2)).to(DEV)
        tree = make_tree(nodes=9, depth=4, seed=1)
        ids = tree.verification_token_ids(torch.tensor([[5]], device=DEV))
        mask = tree.verification_attention_mask(base_kv_length=37, device=DEV)
        pos = tree.verification_position_ids(base_kv_length=37, device=DEV)
        outs = []
        caches = []
        for fwd in (model, lean):
            cache = ReservedCache(config=model.config, capacity=64)
            with torch.no_grad():
                pre = fwd(input_ids=ctx, past_key_values=cache, use_cache=True).logits
                ver = fwd(input_ids=ids, attention_mask=mask, position_ids=pos, past_key_values=cache,
                          use_cache=True).logits
            outs.append((pre.float(), ver.float()))
            caches.append(cache)
        for a, b in zip(outs[0], outs[1]):
            cos = torch.nn.functional.cosine_similarity(a.reshape(-1, a.shape[-1]), b.reshape(-1, b.shape[-1]), dim=-1)
            assert cos.min().item() >= 0.999
            assert (a - b).abs().max().item() <= 5e-2
        for la, lb in zip(caches[0].layers, caches[1].layers):
            assert la.get_seq_length() == lb.get_seq_length() == 47
            assert torch.allclose(la.keys.float(), lb.keys.float(), atol=2e-2, rtol=0)
            assert torch.allclose(la.values.float(), lb.values.float(), atol=2e-2, rtol=0)
    finally:
        m.close()
