"""The C-ABI library loads and exports every entry point the header declares.
CPU only: no kernel is launched."""
import ctypes

from specfit_b200 import _native


def test_library_exports_every_declared_symbol():
    declared = _native.declared_symbols()
    assert len(declared) >= 12
    lib = ctypes.CDLL(str(_native.LIB_PATH))
    missing = [name for name in declared if not hasattr(lib, name)]
    assert not missing, missing
    assert set(declared) == set(_native.SIGNATURES), "binding table out of sync with the header"


def test_host_only_queries():
    assert _native.lib.sf_abi_version() == 1
    assert _native.lib.sf_router_topk_workspace_bytes(65, 128) == 65 * 128 * 4
    assert _native.lib.sf_tree_attention_workspace_bytes(32, 65, 577) > 0
    assert _native.lib.sf_tree_attention_workspace_bytes(0, 65, 577) == 0


def test_argument_errors_are_reported_before_any_launch():
    # top_k = 0 is rejected during validation, before any CUDA call.
    rc = _native.lib.sf_router_topk(None, None, 1, 4, 8, 16, 0, 1, None, None, None, None, None, 0, None)
    assert rc == _native.SF_ERR_INVALID_ARGUMENT
    assert "top_k" in _native.last_error()
    try:
        _native.check(rc, "sf_router_topk")
    except ValueError as err:
        assert "top_k" in str(err)
    else:  # pragma: no cover
        raise AssertionError("ValueError expected")
    for head_dim in (130, 6, 0):  # above 128, not a multiple of 4, empty
        rc = _native.lib.sf_tree_attention(None, None, None, None, 0, 1, 1, 0, 32, 4, head_dim, 0, 0, 0,
                                           0, 1.0, None, None, 0, None)
        assert rc == _native.SF_ERR_INVALID_ARGUMENT and "head_dim" in _native.last_error()


def test_peer_layout_is_consistent():
    """Region layout of the peer exchange (host function, no GPU): sections in
    order, 256-byte aligned, sized for world x capacity rows."""
    import ctypes

    from specfit_b200 import _native as N

    d = N.EpPeer()
    d.world, d.top_k, d.hidden_size = 8, 8, 2048
    d.cap_pairs, d.cap_routes = 65, 520
    d.row_bytes, d.out_row_bytes = 4160, 4096
    total = N.lib.sf_ep_peer_layout(ctypes.byref(d))
    offs = [d.off_recv_rows, d.off_ret_rows, d.off_recv_counts, d.off_recv_arrive, d.off_ret_arrive]
    assert offs == sorted(offs) and all(o % 256 == 0 for o in offs)
    assert d.off_ret_rows - d.off_recv_rows >= 8 * 65 * 4160
    assert d.off_recv_counts - d.off_ret_rows >= 8 * 520 * 4096
    assert total >= d.off_ret_arrive + 8 * 8
    assert N.lib.sf_ep_row_bytes(N.SF_DTYPE_BF16, 2048, 8) == 4160
