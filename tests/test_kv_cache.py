"""ReservedCache (in-place KV writes) against Hugging Face's DynamicCache on
CPU: same keys/values after prefill, verify-sized updates, crops and
regrowth past the reserved capacity."""
import torch

from specfit_b200.runtime.kv_cache import ReservedCache, ReservedLayer
from specfit_b200.runtime.qwen3_verifier import qwen3_moe_config


def test_reserved_cache_matches_dynamic_cache():
    from transformers import DynamicCache

    cfg = qwen3_moe_config(2)
    ref = DynamicCache(config=cfg)
    res = ReservedCache(config=cfg, capacity=40)
    assert all(isinstance(l, ReservedLayer) for l in res.layers)
    g = torch.Generator().manual_seed(0)
    steps = [(0, 24), (None, 9), ("crop", 24), (None, 9), ("crop", 24), (None, 30), ("crop", 30), (None, 5)]
    for op, n in steps:
        if op == "crop":
            ref.crop(n)
            res.crop(n)
        else:
            for layer in range(2):
                k = torch.randn(2, 4, n, 8, generator=g)
                v = torch.randn(2, 4, n, 8, generator=g)
                a = ref.update(k, v, layer)
                b = res.update(k, v, layer)
                assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
        assert ref.get_seq_length() == res.get_seq_length()
    assert res.layers[0].capacity >= 59  # grew past the reservation
