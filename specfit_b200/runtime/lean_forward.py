"""Lean forward of a Qwen3-MoE target for prefill and verify passes.

The same computation as ``Qwen3MoeForCausalLM.forward`` with our MoE blocks
and tree attention (transformers/models/qwen3_moe/modeling_qwen3_moe.py:
decoder layer, attention, RMSNorm, rotary embedding), with the per-layer
chain of small torch kernels replaced by:

* ``sf_add_rmsnorm`` — each residual add fused with the next RMSNorm (input
  norm of the layer, post-attention norm, and the next layer's input norm or
  the final norm);
* one GEMM for the q|k|v projections (weights concatenated once); the
  projections run on the tcgen05 split-K kernel (``ops.linear``) for
  verify-sized row counts;
* ``sf_qk_norm_rope`` — q/k head norms, rotary embedding, and the cache
  update writing k and v rows straight into the ``ReservedCache`` buffers
  (at the host length, or at the device-side offset in static mode);
* the lm_head of verify-sized passes with the greedy argmax fused into it
  (``sf_linear_bf16_argmax``; the result carries ``argmax`` next to
  ``logits``);
* ``sf_tree_attention`` per request, the o projection, and the MoE block:
  its gate module (router hooks still fire) and, with every expert resident
  and no hooks on the block, the experts up to the combine, which is fused
  with the residual add and the next norm (``sf_moe_combine_add_rmsnorm``);
  otherwise the block module itself.

Hooks that the runtime relies on are honoured by hand: forward pre-hooks of
``self_attn`` (the prefetch scheduler's attention hook) run before each
layer's attention, and forward hooks of each decoder layer receive the
layer's output.  The model object stays the weight container; only
``ReservedCache`` caches are supported.
"""
from __future__ import annotations

from types import SimpleNamespace

import torch
import torch.nn.functional as F

from .. import _native as N
from .. import ops
from .kv_cache import ReservedLayer
from .moe_block import Qwen3B200SparseMoeBlock
from .qwen3_offloaded_experts import Qwen3OffloadedExperts
from .tree_attention import _causal_bits, _packed_bits


class LeanQwen3Forward:
    # Several requests' attention runs as one tcgen05 launch where a single
    # request would take that kernel too (sf_tree_attention's AUTO rule):
    # at least 256 packed query rows (query heads per KV head x rows) over
    # at least 2,048 keys.
    BATCHED_ATTENTION_MIN_KEYS = 2048
    BATCHED_ATTENTION_MIN_ROWS = 256

    def __init__(self, model, fused_head: bool = True) -> None:
        cfg = model.config
        self.model = model
        # Verify-sized passes (<= 128 rows) run the lm_head on the persistent
        # tcgen05 streaming kernel with the greedy argmax fused into its
        # epilogue (``out.argmax``); on a B200 that measured 128 vs 131 us at
        # 7 rows and 140 vs 145 us at 65 rows against the library GEMM plus
        # torch.argmax for the 151,936 x 2,048 head.  ``fused_head=False``
        # keeps ``ops.linear`` and leaves ``out.argmax`` None.
        self.fused_head = fused_head
        self.H = cfg.hidden_size
        self.hq, self.hkv, self.D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        if self.D != 128:
            raise ValueError("the lean forward needs head_dim 128")
        self.eps = float(cfg.rms_norm_eps)
        self.layers = []
        with torch.no_grad():
            for layer in model.model.layers:
                a = layer.self_attn
                self.layers.append(SimpleNamespace(
                    layer=layer,
                    wqkv=torch.cat((a.q_proj.weight, a.k_proj.weight, a.v_proj.weight), 0).contiguous(),
                    wo=a.o_proj.weight, qn=a.q_norm.weight.contiguous(),
                    kn=a.k_norm.weight.contiguous(), ln_in=layer.input_layernorm.weight.contiguous(),
                    ln_post=layer.post_attention_layernorm.weight.contiguous()))
        self.final = model.model.norm.weight.contiguous()

    def _norm(self, x, res_in, res_out, w, out, stream):
        N.check(N.lib.sf_add_rmsnorm(x.data_ptr(), None if res_in is None else res_in.data_ptr(),
                                     None if res_out is None else res_out.data_ptr(), w.data_ptr(),
                                     self.eps, x.shape[0], self.H, out.data_ptr(), stream),
                "sf_add_rmsnorm")
        ops._launched(1)

    @staticmethod
    def _moe_sorted(mlp, hn):
        """The MoE block up to its combine when the block and its experts
        carry no hooks and every expert is resident: (ys, dispatch, ids),
        else None.  The gate is still called as a module (its hooks fire)."""
        experts = getattr(mlp, "experts", None)
        if (not isinstance(mlp, Qwen3B200SparseMoeBlock) or not isinstance(experts, Qwen3OffloadedExperts)
                or mlp._forward_hooks or mlp._forward_pre_hooks or experts._forward_hooks
                or experts._forward_pre_hooks):
            return None
        _, weights, idx = mlp.gate(hn)
        out = experts.forward_sorted(hn, idx, weights)
        return None if out is None else (out[0], out[1], idx)

    @torch.no_grad()
    def __call__(self, input_ids, attention_mask=None, position_ids=None, past_key_values=None,
                 logits_to_keep: int = 0, use_cache: bool = True, attention_words=None):
        """``attention_words`` (int32 ``[B, T, words]``, e.g. from
        ``ops.tree_mask_words``) replaces ``attention_mask``: visibility bits
        over every cache row (prefix 0)."""
        cache = past_key_values
        if cache is None or not all(isinstance(l, ReservedLayer) for l in cache.layers):
            raise ValueError("the lean forward needs a ReservedCache")
        m = self.model.model
        B, T = input_ids.shape
        Nt = B * T
        dev = input_ids.device
        stream = torch.cuda.current_stream(dev).cuda_stream
        x = m.embed_tokens(input_ids).reshape(Nt, self.H)
        base = cache.get_seq_length()
        if position_ids is None:
            position_ids = torch.arange(base, base + T, device=dev).unsqueeze(0).expand(B, -1)
        cos, sin = m.rotary_emb(x.view(B, T, self.H), position_ids)
        cos = cos.reshape(Nt, self.D).contiguous()
        sin = sin.reshape(Nt, self.D).contiguous()
        res = torch.empty_like(x)
        hn = torch.empty_like(x)
        self._norm(x, None, res, self.layers[0].ln_in, hn, stream)
        static = cache.layers[0].static_offset is not None
        stacked_bits = None  # (kv_len, [B, T, words]) built once per pass for the batched attention
        for li, L in enumerate(self.layers):
            layer = L.layer
            for hook in tuple(layer.self_attn._forward_pre_hooks.values()):
                hook(layer.self_attn, (hn,))
            cl = cache.layers[li]
            if not cl.is_initialized:  # allocate the reserved buffers (shapes only matter)
                probe = torch.empty(B, self.hkv, T, self.D, dtype=x.dtype, device=dev)
                cl.lazy_initialization(probe, probe)
            if cl._kbuf.shape[0] != B or cl._kbuf.shape[1] != self.hkv:
                raise ValueError("batch or head count differs from the reserved cache")
            if static:
                row0, row0_dev = 0, cl.static_offset
                kv_len = cl.capacity
            else:
                row0, row0_dev = cl.length, None
                if row0 + T > cl.capacity:
                    cl._grow(row0 + T)
                kv_len = row0 + T
                cl.length = kv_len
                cl._publish()
            cap = cl.capacity
            qkv = ops.linear(hn, L.wqkv)
            q = torch.empty(B, self.hq, T, self.D, dtype=x.dtype, device=dev)
            N.check(N.lib.sf_qk_norm_rope(qkv.data_ptr(), B, T, self.hq, self.hkv, self.D,
                                          L.qn.data_ptr(), L.kn.data_ptr(), cos.data_ptr(),
                                          sin.data_ptr(), self.eps, q.data_ptr(),
                                          cl._kbuf.data_ptr(), cl._vbuf.data_ptr(),
                                          self.hkv * cap * self.D, cap * self.D, row0,
                                          None if row0_dev is None else row0_dev.data_ptr(), stream),
                    "sf_qk_norm_rope")
            ops._launched(1)
            if attention_words is not None:
                bits = [attention_words[b] for b in range(B)]
                prefix = 0
            elif attention_mask is None:
                bits = [_causal_bits(T, dev)] * B
                prefix = kv_len - T
            else:
                bits = _packed_bits(attention_mask, T, kv_len, B)
                prefix = 0
            attn = torch.empty(B, T, self.hq, self.D, dtype=x.dtype, device=dev)
            done = None
            if (B > 1 and kv_len >= self.BATCHED_ATTENTION_MIN_KEYS
                    and (self.hq // self.hkv) * T >= self.BATCHED_ATTENTION_MIN_ROWS):
                # Several requests: one launch of the tcgen05 kernel over all of them.
                if stacked_bits is None or stacked_bits[0] != kv_len:
                    stacked_bits = (kv_len, torch.stack([bb.reshape(T, -1) for bb in bits]))
                done = ops.tree_attention_batched(q, cl._kbuf[:, :, :kv_len], cl._vbuf[:, :, :kv_len],
                                                  stacked_bits[1], prefix, scale=self.D ** -0.5, out=attn)
            if done is None:
                for b in range(B):
                    ops.tree_attention(q[b], cl._kbuf[b, :, :kv_len], cl._vbuf[b, :, :kv_len], bits[b],
                                       prefix, scale=self.D ** -0.5, out=attn[b])
            o = ops.linear(attn.view(Nt, self.hq * self.D), L.wo)
            self._norm(o, res, res, L.ln_post, hn, stream)
            nxt = self.layers[li + 1].ln_in if li + 1 < len(self.layers) else self.final
            sorted_out = self._moe_sorted(layer.mlp, hn)
            if sorted_out is not None:  # combine + residual add + next norm in one launch
                ys, d, idx = sorted_out
                ops.moe_combine_add_rmsnorm(ys, d, idx, res, nxt, self.eps, out=hn)
            else:
                moe = layer.mlp(hn.view(B, T, self.H)).reshape(Nt, self.H)
                self._norm(moe, res, res, nxt, hn, stream)
            if layer._forward_hooks:
                out = res.view(B, T, self.H).clone()
                for hook in tuple(layer._forward_hooks.values()):
                    hook(layer, (), out)
        keep = T if not logits_to_keep else min(int(logits_to_keep), T)
        rows = hn.view(B, T, self.H)[:, T - keep:, :].contiguous()
        head = self.model.lm_head.weight
        if self.fused_head and B * keep <= 128 and head.dtype == torch.bfloat16 and self.H % 64 == 0:
            # lm_head and the greedy pick in one pass over the 151,936-row weight
            logits, argmax = ops.linear_argmax(rows, head)
            return SimpleNamespace(logits=logits, argmax=argmax)
        return SimpleNamespace(logits=ops.linear(rows, head), argmax=None)
