"""The allocation-free router entry point, called through the C ABI.

``sf_router_topk_noalloc`` serves callers that cannot allocate device memory
where they route: plugins of a serving engine that keeps the GPU's memory for
its own pools, hosts binding the library through a plain C FFI without a
device allocator, and paths that cannot take cudaMalloc's device-wide
synchronisation.  It runs the same kernels as the workspace entry point
``sf_router_topk`` with its scratch in an array built into the library, so
on consecutive calls that reuse that array its four outputs must equal the
workspace entry point's bit for bit; sizes beyond the array are refused.

This file is collected last on purpose: it runs after every other test of a
full run and also passes alone in a fresh process.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _native():
    from specfit_b200 import _native

    return _native


def _outputs(tokens, experts, top_k, dtype):
    return (torch.empty(tokens, experts, dtype=torch.float32, device=DEV),
            torch.empty(tokens, top_k, dtype=torch.float32, device=DEV),
            torch.empty(tokens, top_k, dtype=torch.int64, device=DEV),
            torch.empty(tokens, experts, dtype=dtype, device=DEV))


def _call_with_workspace(N, x, w, top_k):
    tokens, hidden = x.shape
    experts = w.shape[0]
    probs, tw, ti, logits = _outputs(tokens, experts, top_k, x.dtype)
    nbytes = N.lib.sf_router_topk_workspace_bytes(tokens, experts)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    code = N.SF_DTYPE_BF16 if x.dtype == torch.bfloat16 else N.SF_DTYPE_F32
    stream = torch.cuda.current_stream(DEV).cuda_stream
    rc = N.lib.sf_router_topk(x.data_ptr(), w.data_ptr(), code, tokens, hidden, experts, top_k, 1,
                              probs.data_ptr(), tw.data_ptr(), ti.data_ptr(), logits.data_ptr(),
                              ws.data_ptr(), nbytes, stream)
    N.check(rc, "sf_router_topk")
    return probs, tw, ti, logits


def _call_noalloc(N, x, w, top_k):
    tokens, hidden = x.shape
    experts = w.shape[0]
    probs, tw, ti, logits = _outputs(tokens, experts, top_k, x.dtype)
    code = N.SF_DTYPE_BF16 if x.dtype == torch.bfloat16 else N.SF_DTYPE_F32
    stream = torch.cuda.current_stream(DEV).cuda_stream
    rc = N.lib.sf_router_topk_noalloc(x.data_ptr(), w.data_ptr(), code, tokens, hidden, experts,
                                      top_k, 1, probs.data_ptr(), tw.data_ptr(), ti.data_ptr(),
                                      logits.data_ptr(), stream)
    N.check(rc, "sf_router_topk_noalloc")
    return probs, tw, ti, logits


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_noalloc_router_matches_workspace_router_on_consecutive_calls(dtype):
    N = _native()
    gen = torch.Generator().manual_seed(123)
    # Two calls in a row with different sizes: the second reuses the scratch
    # the first one left behind.
    for tokens in (65, 512):
        x = torch.randn(tokens, 2048, generator=gen).to(dtype).to(DEV)
        w = (torch.randn(128, 2048, generator=gen) * 0.02).to(dtype).to(DEV)
        ref = _call_with_workspace(N, x, w, 8)
        got = _call_noalloc(N, x, w, 8)
        torch.cuda.synchronize()
        for name, a, b in zip(("probs", "weights", "indices", "logits"), got, ref):
            assert torch.equal(a, b), f"{name} differ from sf_router_topk"
        if tokens == 65:
            # The indices also equal the CPU restatement of the router.
            from oracle import moe_oracle as mo

            _, _, idx, _ = mo.router_topk(x.float().cpu().numpy(), w.float().cpu().numpy(), 8, True,
                                          "bf16" if dtype == torch.bfloat16 else "f32")
            assert np.array_equal(got[2].cpu().numpy(), idx)


def test_noalloc_router_rejects_sizes_beyond_its_scratch():
    N = _native()
    limit = N.lib.sf_router_topk_noalloc_max_elems()
    assert limit == 1 << 19
    tokens = limit // 128 + 1
    dummy = torch.empty(1, dtype=torch.float32, device=DEV)
    p = dummy.data_ptr()
    rc = N.lib.sf_router_topk_noalloc(p, p, N.SF_DTYPE_BF16, tokens, 2048, 128, 8, 1, p, p, p, None,
                                      torch.cuda.current_stream(DEV).cuda_stream)
    assert rc == N.SF_ERR_WORKSPACE
    assert "built-in scratch" in N.last_error()
