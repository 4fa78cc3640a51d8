"""The C-ABI library loads, exports every declared symbol, and rejects bad
arguments with a status code and a message -- all without a GPU (the checks
run before any CUDA call)."""
import ctypes
import os
import re

import pytest

from whallm_b200 import _lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = []
    inc = os.path.join(ROOT, "include")
    for f in sorted(os.listdir(inc)):
        if f.endswith(".h"):
            src = open(os.path.join(inc, f)).read()
            names += re.findall(r"^WM_API\s+[\w\s\*]+?\b(\w+)\s*\(", src, re.M)
    return names


def test_header_declares_the_abi():
    names = declared_symbols()
    assert len(names) >= 15
    assert set(names) == set(L.SIGNATURES), "ctypes signatures and header differ"


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(L.LIB_PATH)
    for n in declared_symbols():
        assert hasattr(lib, n), n


def test_version_and_empty_error():
    assert L.lib().w_abi_version() == 1
    assert isinstance(L.last_error(), str)


def _expect(rc_name, *args, code=L.WM_ERR_INVALID, msg=None):
    rc = getattr(L.lib(), rc_name)(*args)
    assert rc == code, (rc_name, rc, L.last_error())
    if msg:
        assert msg in L.last_error()


def test_layer_rejects_bad_router_and_shared_expert_arguments():
    # checked before any CUDA call: the shared expert must be the last one (expert n_routed)
    f = "wmoe_mxfp4_moe_layer"
    _expect(f, None, 1, 256, 256, None, None, None, None, 8, 2, 0, -1.0, 1.0, None, None, None, None, 0, 0.0, 3,
            None, None, None, None, None, None, 0, None, msg="shared expert must be expert n_routed")
    _expect(f, None, 1, 256, 256, None, None, None, None, 8, 9, 0, -1.0, 1.0, None, None, None, None, 0, 0.0, -1,
            None, None, None, None, None, None, 0, None, msg="1 <= k <= min(32, n_routed)")
    _expect(f, None, 0, 256, 256, None, None, None, None, 8, 2, 0, -1.0, 1.0, None, None, None, None, 0, 0.0, 8,
            None, None, None, None, None, None, 0, None, code=L.WM_OK)


def test_mxfp4_rejects_partial_groups():
    _expect("wmxfp4_quantize", None, 1, 33, None, None, None, msg="complete BF16 rows")
    _expect("wmxfp4_dequantize", None, None, 1, 31, 0, None, None)


def test_kv_rejects_bad_format_and_width():
    _expect("wkv_quantize", None, 4, 576, 9, None, None, None, msg="unknown KV format")
    _expect("wkv_quantize", None, 4, 600, 0, None, None, None, msg="Invalid packed cache")
    _expect("wkv_dequantize", None, None, 4, 40, 1, None, None)


def test_router_rejects_bad_shapes():
    f = L.lib().wmoe_router_topk
    assert f(None, None, None, None, None, 4, 100, 16, 2, 0, -1.0, 1.0, None, None, None, None, None) == L.WM_ERR_INVALID
    assert "H % 8" in L.last_error()
    assert f(None, None, None, None, None, 4, 128, 2048, 2, 0, -1.0, 1.0, None, None, None, None, None) == L.WM_ERR_INVALID
    assert f(None, None, None, None, None, 4, 128, 16, 17, 0, -1.0, 1.0, None, None, None, None, None) == L.WM_ERR_INVALID
    assert f(None, None, None, None, None, 4, 128, 16, 2, 9, -1.0, 1.0, None, None, None, None, None) == L.WM_ERR_INVALID


def test_experts_reject_bad_arguments():
    f = L.lib().wmoe_mxfp4_moe_forward
    # gate/up order must be 0 or 1
    rc = f(None, None, None, 1, 8, 7168, 2048, 256, None, None, None, None, 7, 0.0, -1, None, None, None, 0, None)
    assert rc == L.WM_ERR_INVALID and "gate_up_order" in L.last_error()
    rc = f(None, None, None, 1, 8, 7160, 2048, 256, None, None, None, None, 0, 0.0, -1, None, None, None, 0, None)
    assert rc == L.WM_ERR_INVALID


def test_workspace_size_is_pure_host():
    n = L.lib().wmoe_workspace_size(16, 8, 7168, 2048, 257, 1)
    assert n > 16 * 9 * 7168 * 4
    assert L.lib().wmoe_workspace_size(-1, 8, 7168, 2048, 257, 1) == 0


def test_score_workspace_holds_split_partials():
    # a decode-size call over 40 row blocks splits K (f32 partials in the
    # workspace); a prefill-size call fills the GPU without splitting
    lib = L.lib()
    base = lib.wmx_linear_workspace_size(16, 5120, 128)
    assert lib.wmx_linear_workspace_size(16, 5120, 5120) >= base + 2 * 16 * 5120 * 4
    assert lib.wmx_linear_workspace_size(4096, 5120, 5120) == lib.wmx_linear_workspace_size(4096, 5120, 128)
    assert lib.wkv_scores_workspace_size(1, 1, 512, 0) == 0


def test_call_raises_valueerror_on_invalid():
    with pytest.raises(ValueError, match="complete BF16 rows"):
        L.call("wmxfp4_quantize", None, 1, 33, None, None, None)


def test_fp8_kv_entry_points_reject_other_formats():
    # checked before any CUDA call: block 64 goes with fp32 scales, block 32 with ue8m0
    for block, sf in ((32, 0), (64, 1), (16, 1)):
        with pytest.raises(L.NativeError, match="fp8 KV"):
            L.call("wkv_fp8_quantize", None, 4, 64, block, sf, None, None, None)
        with pytest.raises(L.NativeError, match="fp8 KV"):
            L.call("wkv_fp8_dequantize", None, None, 4, 64, block, sf, None, None)


def test_scores_and_linear_reject_bad_shapes():
    # host-side checks, before any device work: D (K) a multiple of 256, an MX format, B/Lq/L >= 1
    _expect("wmx_linear", None, 4, 5000, None, None, 64, L.WKV_MXFP8_B32, None, None, 0, None, msg="D % 256")
    _expect("wmx_linear", None, 4, 512, None, None, 64, L.WKV_FP8_F32_B64, None, None, 0, None, msg="fmt must be")
    _expect("wkv_mx_scores", None, 0, 1, 512, None, None, 64, L.WKV_MXFP8_B32, None, None, 0, None)
    _expect("wkv_mx_scores", None, 1, 1, 512, None, None, 64, L.WKV_MXFP4_B32, None, None, 0, None, msg="null buffer")
    _expect("wmx_linear", None, 0, 512, None, None, 64, L.WKV_MXFP8_B32, None, None, 0, None, code=L.WM_OK)


def test_peer_sum_rejects_misaligned_rows():
    # wep_sum_rows reads float4 partials and writes 8-byte bf16 groups: pointers off those boundaries are
    # rejected on the host (these addresses are never dereferenced)
    _expect("wep_sum_rows", ctypes.c_void_p(0x10004), 2, 3, 16, None, ctypes.c_void_p(0x20000), None,
            msg="16-byte")
    _expect("wep_sum_rows", ctypes.c_void_p(0x10000), 2, 3, 16, None, ctypes.c_void_p(0x20004), None,
            msg="8-byte")
