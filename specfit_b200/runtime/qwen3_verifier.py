"""A Qwen3-MoE target with offloaded experts on the B200 path.

``build_random_offloaded_qwen3`` is the random-init counterpart of the
reference loader ``load_offloaded_qwen3`` (``src/specfit/runtime/
qwen3_offloaded_model.py:667-840``): it builds the Hugging Face
``Qwen3MoeForCausalLM`` on the meta device, replaces every ``layer.mlp`` with
``Qwen3B200SparseMoeBlock`` (router + offloaded experts behind one
``GpuExpertCache`` per layer, as :280-310 and :597-606 do), materialises the
non-expert weights on the GPU and routes attention through the tree-attention
kernel.  The result is the same ``(model, caches)`` pairing as the reference's
``LoadedOffloadedQwen3``, so verify passes run through the model's normal
``forward(input_ids, attention_mask=<4-D tree mask>, position_ids,
past_key_values)``.

Expert weights live in an ``ExpertHostPool``: one page-locked host array
``[layers, experts, 3*H*I]`` (packed ``gate | up | down`` rows, the packed-v1
layout of ``adapters/qwen3_packed_checkpoint.py:20-23``), registered with
``cudaHostRegister`` so its exact size is pinned (no allocator rounding) and
the caches adopt slices of it without copying.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import synthetic
from .gpu_expert_cache import GpuExpertCache
from .moe_block import Qwen3B200SparseMoeBlock, Qwen3B200TopKRouter
from .qwen3_offloaded_experts import ExpertExecutionPolicy, Qwen3OffloadedExperts, ReductionMode
from .state import ExpertKey
from .tree_attention import install as install_tree_attention


def qwen3_moe_config(num_layers: int = synthetic.NUM_LAYERS, *, hidden: int = synthetic.HIDDEN,
                     experts: int = synthetic.NUM_EXPERTS, top_k: int = synthetic.TOP_K,
                     moe_inter: int = synthetic.MOE_INTER, heads: int = synthetic.NUM_HEADS,
                     kv_heads: int = synthetic.NUM_KV_HEADS, head_dim: int = synthetic.HEAD_DIM,
                     vocab: int = synthetic.VOCAB):
    """Qwen3-30B-A3B shape (48 layers, H 2048, 128 experts top-8, I 768,
    32/4 heads of 128, vocab 151936, RoPE theta 1e6, RMSNorm eps 1e-6)."""
    from transformers import Qwen3MoeConfig

    return Qwen3MoeConfig(
        vocab_size=vocab, hidden_size=hidden, intermediate_size=6144, num_hidden_layers=num_layers,
        num_attention_heads=heads, num_key_value_heads=kv_heads, head_dim=head_dim,
        max_position_embeddings=40960, rms_norm_eps=synthetic.RMS_EPS,
        rope_parameters={"rope_type": "default", "rope_theta": synthetic.ROPE_THETA},
        tie_word_embeddings=False, moe_intermediate_size=moe_inter, num_experts=experts,
        num_experts_per_tok=top_k, norm_topk_prob=True, decoder_sparse_step=1, mlp_only_layers=[],
        attention_bias=False)


class ExpertHostPool:
    """Page-locked host copy of every expert: ``[layers, experts, 3*H*I]``.

    With ``shm_path`` the array lives in a shared-memory file, so several
    processes on one node (one per GPU) map and pin the same physical pages
    instead of each holding a private copy."""

    def __init__(self, layers: int, experts: int, elems: int, dtype=torch.bfloat16, *,
                 shm_path: str | None = None) -> None:
        import os

        self.layers, self.experts, self.elems = layers, experts, elems
        self.shm_path = shm_path
        n = layers * experts * elems
        if shm_path is None:
            self.data = torch.empty(layers, experts, elems, dtype=dtype)
        else:
            nbytes = n * torch.empty((), dtype=dtype).element_size()
            fd = os.open(shm_path, os.O_RDWR | os.O_CREAT, 0o600)
            try:
                if os.fstat(fd).st_size < nbytes:
                    os.ftruncate(fd, nbytes)
            finally:
                os.close(fd)
            self.data = torch.from_file(shm_path, shared=True, size=n, dtype=dtype).view(
                layers, experts, elems)
        nbytes = self.data.numel() * self.data.element_size()
        # Portable | mapped: page-locked for every context and readable by
        # kernels (the device-managed cache fills slots with SM loads).
        rc = torch.cuda.cudart().cudaHostRegister(self.data.data_ptr(), nbytes, 0x01 | 0x02)
        if int(rc) != 0:
            import resource

            soft, hard = resource.getrlimit(resource.RLIMIT_MEMLOCK)
            raise RuntimeError(f"cudaHostRegister of the {nbytes / 1e9:.1f} GB expert pool failed "
                               f"({int(rc)}); RLIMIT_MEMLOCK soft={soft} hard={hard}")
        self._registered = True

    @property
    def nbytes(self) -> int:
        return self.data.numel() * self.data.element_size()

    def fill_random(self, seed: int, device, std: float = 0.02) -> None:
        """N(0, std) weights, drawn on the GPU per layer (seed + layer)."""
        for layer in range(self.layers):
            g = torch.Generator(device=device).manual_seed(seed + layer)
            block = torch.randn(self.experts, self.elems, generator=g, device=device,
                                dtype=torch.float32).mul_(std).to(self.data.dtype)
            self.data[layer].copy_(block, non_blocking=False)

    def sources(self, layer: int) -> dict:
        return {ExpertKey(layer, e): self.data[layer, e] for e in range(self.experts)}

    def close(self) -> None:
        if self._registered:
            torch.cuda.cudart().cudaHostUnregister(self.data.data_ptr())
            self._registered = False


@dataclass
class LoadedB200Qwen3:
    """The model and its per-layer caches (cf. ``LoadedOffloadedQwen3``,
    ``qwen3_offloaded_model.py:127-260``)."""

    model: torch.nn.Module
    caches: tuple
    pool: ExpertHostPool | None = None

    @property
    def expert_caches(self) -> tuple:
        """The reference's name for the per-layer caches."""
        return self.caches

    def _expert_modules(self) -> tuple:
        modules = tuple(layer.mlp.experts for layer in self.model.model.layers)
        if not all(isinstance(m, Qwen3OffloadedExperts) for m in modules):
            raise RuntimeError("every decoder layer must contain offloaded experts")
        return modules

    def cache_stats(self) -> dict:
        totals = dict(h2d_submissions=0, resident_hits=0, inflight_joins=0, evictions=0,
                      pending_use_guards=0)
        for c in self.caches:
            st = c.stats()
            for k in totals:
                totals[k] += getattr(st, k)
        return totals

    def cache_snapshots(self) -> tuple:
        return tuple(c.snapshot() for c in self.caches)

    def cold_reset_caches(self) -> None:
        torch.cuda.synchronize()
        for c in self.caches:
            c.cold_reset()

    cold_reset_expert_caches = cold_reset_caches

    def warm_all_caches(self) -> None:
        """Fill every slot that can hold an expert (all experts when the
        cache is as large as the layer)."""
        for c in self.caches:
            c.prefill_all()
        torch.cuda.synchronize()

    def enter_device_managed_caches(self) -> None:
        """Every layer's cache in device-managed mode (misses planned and
        filled on the device; a verify pass then needs no host round trip
        and can be captured in a CUDA graph)."""
        modules = self._expert_modules()
        if any(m._prediction_scheduler is not None for m in modules):
            raise RuntimeError("cannot switch cache mode during predicted prefetch")
        for m in modules:
            if m.reduction_mode is not ReductionMode.CANONICAL:
                raise ValueError("device-managed caches reduce canonically only")
        for c in self.caches:
            c.enter_device_mode()

    def leave_device_managed_caches(self) -> None:
        for c in self.caches:
            c.leave_device_mode()

    def set_expert_execution_policy(self, policy) -> None:
        policy = ExpertExecutionPolicy(policy)
        modules = self._expert_modules()
        if any(m._prediction_scheduler is not None for m in modules):
            raise RuntimeError("cannot switch execution policy during predicted prefetch")
        for m in modules:
            m.execution_policy = policy

    def set_expert_h2d_prefetch(self, enabled: bool) -> None:
        if type(enabled) is not bool:
            raise ValueError("h2d_prefetch must be a boolean")
        modules = self._expert_modules()
        if any(m._prediction_scheduler is not None for m in modules):
            raise RuntimeError("cannot switch H2D policy during predicted prefetch")
        if any(c.closed or c.active_lease_count for c in self.caches):
            raise RuntimeError("prefetch switching requires open caches without active leases")
        for m in modules:
            m.h2d_prefetch = enabled

    def prefetch_experts(self, predictions, *, lookahead_layers: int = 1, max_inflight: int = 2,
                         max_prefetch_per_layer: int | None = None, trace: bool = False,
                         prediction_probabilities=None, eviction_policy: str = "lru"):
        """A ``Qwen3ExpertPrefetch`` context for one forward
        (``qwen3_offloaded_model.py:217-227``)."""
        from .qwen3_expert_prefetch import Qwen3ExpertPrefetch

        return Qwen3ExpertPrefetch(self, predictions, lookahead_layers=lookahead_layers,
                                   max_inflight=max_inflight,
                                   max_prefetch_per_layer=max_prefetch_per_layer, trace=trace,
                                   prediction_probabilities=prediction_probabilities,
                                   eviction_policy=eviction_policy)

    def close(self) -> None:
        if any(getattr(layer.mlp.experts, "_prediction_scheduler", None) is not None
               for layer in self.model.model.layers):
            raise RuntimeError("cannot close the model during predicted prefetch")
        torch.cuda.synchronize()
        for c in self.caches:
            c.close()
        if self.pool is not None:
            self.pool.close()


LoadedOffloadedQwen3 = LoadedB200Qwen3  # the reference's name


def _init_layer_(module: torch.nn.Module, gen: torch.Generator, std: float) -> None:
    for name, p in sorted(module.named_parameters(), key=lambda kv: kv[0]):
        if name.endswith("norm.weight") or name.endswith("layernorm.weight"):
            p.data.fill_(1.0)
        else:
            p.data.normal_(0.0, std, generator=gen)


def materialize_random_(model, cfg, device, seed: int, std: float, dtype) -> None:
    """Allocate a meta-built model on ``device`` and draw its non-expert
    weights: layer l from a generator seeded ``seed + l``, embeddings and
    lm_head from ``seed + layers`` and ``seed + layers + 1``; norms are 1."""
    model.to_empty(device=device)
    with torch.no_grad():
        for l, layer in enumerate(model.model.layers):
            _init_layer_(layer, torch.Generator(device=device).manual_seed(seed + l), std)
        g = torch.Generator(device=device).manual_seed(seed + cfg.num_hidden_layers)
        model.model.embed_tokens.weight.normal_(0.0, std, generator=g)
        model.model.norm.weight.fill_(1.0)
        g = torch.Generator(device=device).manual_seed(seed + cfg.num_hidden_layers + 1)
        model.lm_head.weight.normal_(0.0, std, generator=g)
    model.to(dtype)
    # RoPE frequencies stay fp32 (rebuilt after the dtype cast), as a model
    # loaded in bf16 keeps them.
    model.model.rotary_emb = type(model.model.rotary_emb)(config=cfg, device=device)
    model.eval()


def build_random_offloaded_qwen3(*, device, slots_per_layer: int, num_layers: int = synthetic.NUM_LAYERS,
                                 seed: int = 0, dtype=torch.bfloat16, config=None,
                                 pool: ExpertHostPool | None = None,
                                 reduction_mode=ReductionMode.CANONICAL,
                                 expert_execution_policy=ExpertExecutionPolicy.EXPERT_ID_ASCENDING,
                                 cache_observer=None, std: float = 0.02) -> LoadedB200Qwen3:
    """Random-init bf16 N(0, std) target with ``slots_per_layer`` cache slots.

    Non-expert weights of layer l are drawn from a generator seeded with
    ``seed + l``; embeddings and lm_head from ``seed + num_layers`` and
    ``seed + num_layers + 1``; expert weights from the pool (``fill_random``
    with the same per-layer seeds when the pool is created here)."""
    from transformers import Qwen3MoeForCausalLM

    device = torch.device(device)
    cfg = config if config is not None else qwen3_moe_config(num_layers)
    cfg._attn_implementation = "sdpa"
    hidden, inter = cfg.hidden_size, cfg.moe_intermediate_size
    if pool is None:
        pool = ExpertHostPool(cfg.num_hidden_layers, cfg.num_experts, 3 * hidden * inter, dtype)
        pool.fill_random(seed, device, std)
    with torch.device("meta"):
        model = Qwen3MoeForCausalLM(cfg)
    caches = []
    for l, layer in enumerate(model.model.layers):
        cache = GpuExpertCache(pool.sources(l), slot_count=slots_per_layer, device=device,
                               adopt_pinned_sources=True, observer=cache_observer)
        experts = Qwen3OffloadedExperts(layer_id=l, cache=cache, hidden_size=hidden,
                                        intermediate_size=inter, reduction_mode=reduction_mode,
                                        execution_policy=expert_execution_policy)
        gate = Qwen3B200TopKRouter(cfg.num_experts, hidden, cfg.num_experts_per_tok,
                                   cfg.norm_topk_prob, device="meta")
        layer.mlp = Qwen3B200SparseMoeBlock(gate, experts)
        caches.append(cache)
    materialize_random_(model, cfg, device, seed, std, dtype)
    install_tree_attention(model)
    return LoadedB200Qwen3(model, tuple(caches), pool)
