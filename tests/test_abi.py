"""The C-ABI library loads and exports what include/flowmoe.h declares; host-side argument checks
(no GPU needed: every call here fails validation before any device work)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _declared():
    txt = (ROOT / "include" / "flowmoe.h").read_text()
    return sorted(set(re.findall(r"FM_API int (fm_\w+)\(", txt)))


def test_header_declares_entry_points():
    names = _declared()
    assert "fm_moe_block" in names and "fm_router_topk" in names and len(names) >= 10


def test_library_exports_every_declared_symbol():
    from flowmoe import _lib
    so = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in _declared() if not hasattr(so, n)]
    assert not missing, missing
    assert set(_declared()) == set(_lib.SIGNATURES), "ctypes signatures out of step with the header"


def test_version_and_error_buffer():
    from flowmoe import _lib
    buf = ctypes.create_string_buffer(64)
    assert _lib.lib.fm_version(buf, 64) == 0 and b"sm_100a" in buf.value


def _layer(**kw):
    from flowmoe._lib import FmLayer
    g = dict(hidden=2048, n_experts=128, top_k=8, ffn=768, shared_ffn=0, e_begin=0, e_local=128, flags=0)
    g.update(kw)
    return FmLayer(g["hidden"], g["n_experts"], g["top_k"], g["ffn"], g["shared_ffn"], g["e_begin"], g["e_local"],
                   g["flags"], None, None, None, None, None)


def test_workspace_size_grows_with_tokens():
    from flowmoe import _lib
    n1, n2 = ctypes.c_size_t(), ctypes.c_size_t()
    L = _layer()
    _lib.call("fm_workspace_size", ctypes.byref(L), 16, ctypes.byref(n1))
    _lib.call("fm_workspace_size", ctypes.byref(L), 8192, ctypes.byref(n2))
    assert 0 < n1.value < n2.value


@pytest.mark.parametrize("kw,code", [(dict(top_k=200), 1), (dict(hidden=100), 1), (dict(ffn=700), 1),
                                     (dict(e_begin=100, e_local=64), 1), (dict(n_experts=4096), 1)])
def test_bad_geometry_is_rejected(kw, code):
    from flowmoe import _lib
    n = ctypes.c_size_t()
    rc = _lib.lib.fm_workspace_size(ctypes.byref(_layer(**kw)), 16, ctypes.byref(n))
    assert rc == code
    assert _lib.last_error()


@pytest.mark.parametrize("flags,ok", [(0, True), (2, True), (3, True), (0x100, True), (0x102, True), (0x103, True),
                                      (1, False), (4, False), (0x101, False), (0x200, False), (0x302, False)])
def test_flags_checked(flags, ok):
    """fm_layer.flags: a kernel path (0 auto, 2 tcgen05, 3 GEMV) plus optionally FM_FIXED_ORDER (0x100)."""
    from flowmoe import _lib
    n = ctypes.c_size_t()
    rc = _lib.lib.fm_workspace_size(ctypes.byref(_layer(flags=flags)), 16, ctypes.byref(n))
    assert (rc == 0) == ok and (ok or rc == _lib.FM_EINVAL_SHAPE)


def test_fixed_order_workspace_holds_f32_rows():
    """The fixed-order mode's tcgen05 path keeps every y row in f32: T * (top_k + 1) * H * 4 bytes more."""
    from flowmoe import _lib
    a, b = ctypes.c_size_t(), ctypes.c_size_t()
    T, L = 4096, dict(shared_ffn=512)
    _lib.call("fm_workspace_size", ctypes.byref(_layer(**L)), T, ctypes.byref(a))
    _lib.call("fm_workspace_size", ctypes.byref(_layer(flags=0x100, **L)), T, ctypes.byref(b))
    assert b.value - a.value >= T * 9 * 2048 * 4


def test_topk_past_experts_raises_like_reference():
    from flowmoe import _lib
    with pytest.raises(_lib.FlowMoeError, match="topk"):
        _lib.call("fm_workspace_size", ctypes.byref(_layer(n_experts=4, top_k=5)), 1, ctypes.byref(ctypes.c_size_t()))


def test_small_workspace_is_rejected():
    from flowmoe import _lib
    rc = _lib.lib.fm_moe_block(ctypes.byref(_layer()), None, 0, None, None, None, None, 16, 16, None, None, 16, None)
    assert rc == _lib.FM_EWORKSPACE


def test_tile_geometry_checked():
    from flowmoe import _lib
    assert _lib.lib.fm_q4_1_to_tiles(None, 100, 2048, None, None) == _lib.FM_EINVAL_SHAPE


@pytest.mark.parametrize("n,k,rs,chunk", [(64, 200, 2, 5120), (48, 256, 2, 5120), (64, 256, 0, 5120), (64, 256, 2, 4096)])
def test_pool_import_bad_geometry_is_rejected(n, k, rs, chunk):
    """fm_pool_to_q4_1 checks k % 256, n % (32 rs) and the chunk size before any device work."""
    from flowmoe import _lib
    buf = (ctypes.c_uint8 * 16)()
    bad = (ctypes.c_int32 * 1)()
    rc = _lib.lib.fm_pool_to_q4_1(ctypes.cast(buf, ctypes.c_void_p), n, k, rs, chunk, ctypes.cast(buf, ctypes.c_void_p),
                                  ctypes.cast(bad, ctypes.c_void_p), None)
    assert rc == _lib.FM_EINVAL_SHAPE
    assert "fm_pool_to_q4_1" in _lib.last_error()


def test_empty_calls_are_no_ops():
    # T = 0 tokens: every entry point returns FM_OK before any device work, with no workspace at all
    from flowmoe import _lib
    L = ctypes.byref(_layer())
    assert _lib.lib.fm_router_topk(L, None, 0, 0, None, None, None, None, None, 0, None) == 0
    assert _lib.lib.fm_moe_block(L, None, 0, None, None, None, None, 0, 0, None, None, 0, None) == 0
    assert _lib.lib.fm_moe_layer(L, None, 0, None, 0, 0, None, None, None, None, 0, None) == 0
    assert _lib.lib.fm_moe_dispatch(L, None, 0, 0, None, None, None, None, None, 0, None) == 0


@pytest.mark.parametrize("T,t_real", [(16, 17), (16, -1), (-1, 0)])
def test_token_counts_outside_range_are_rejected(T, t_real):
    from flowmoe import _lib
    rc = _lib.lib.fm_moe_block(ctypes.byref(_layer()), None, 0, None, None, None, None, T, t_real, None, None, 0, None)
    assert rc == _lib.FM_EINVAL_SHAPE
    assert _lib.last_error()


@pytest.mark.parametrize("N,K,T,dt,ok", [(256, 512, 300, 0, True), (2560, 2560, 256, 1, True), (128, 64, 0, 1, True),
                                        (200, 512, 8, 1, False), (256, 500, 8, 1, False), (256, 512, -1, 1, False),
                                        (256, 512, 8, 7, False)])
def test_q4_gemm_shape_checks(N, K, T, dt, ok):
    """fm_q4_gemm: N a multiple of 128, K of 64, T >= 0, x f32 (0) or bf16 (1); the f32 input needs a bf16
    copy of x in the workspace."""
    from flowmoe import _lib
    n = ctypes.c_size_t()
    rc = _lib.lib.fm_q4_gemm_workspace_size(N, K, T, dt, ctypes.byref(n))
    assert (rc == 0) == ok and (ok or rc == _lib.FM_EINVAL_SHAPE)
    if ok and T > 0:
        m = ctypes.c_size_t()
        _lib.call("fm_q4_gemm_workspace_size", N, K, T, 1 - dt, ctypes.byref(m))
        assert (n.value - m.value if dt == 0 else m.value - n.value) >= T * K * 2


def test_q4_gemm_rejects_before_device_work():
    """Zero tokens is a no-op; a NULL pointer or a short workspace is refused on the host."""
    from flowmoe import _lib
    assert _lib.lib.fm_q4_gemm(None, 256, 512, None, 1, 0, None, None, 0, None) == 0
    assert _lib.lib.fm_q4_gemm(None, 256, 512, None, 1, 4, None, None, 0, None) == _lib.FM_EINVAL_SHAPE
    buf = (ctypes.c_uint8 * 64)()
    p = ctypes.addressof(buf) + (-ctypes.addressof(buf)) % 16
    rc = _lib.lib.fm_q4_gemm(p, 256, 512, p, 1, 4, p, p, 16, None)
    assert rc == _lib.FM_EWORKSPACE and "workspace" in _lib.last_error()
