"""CPU tests of the C ABI: the library loads, exports every symbol that
include/b200lab.h declares, and rejects malformed calls before touching the
device (no compute is launched here)."""
import ctypes
import os
import re

import b200lab

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_functions():
    src = open(os.path.join(ROOT, "include", "b200lab.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    src = re.sub(r"^\s*#.*$", "", src, flags=re.M)
    return sorted(set(re.findall(r"^\s*(?:[A-Za-z_]\w*[\s*]+)+([A-Za-z_]\w*)\s*\(", src, flags=re.M)))


def test_header_symbols_exported():
    L = b200lab.lib()
    names = _declared_functions()
    assert set(names) == set(b200lab.EXPORTED), names
    for n in names:
        assert hasattr(L, n), n


def test_strerror_and_version():
    assert b200lab.strerror(0) == "ok"
    for code in (-1, -2, -3, -4, -5, -6):
        assert b200lab.strerror(code) != "unknown status"
    assert b200lab.strerror(12345) == "unknown status"
    assert b200lab.lib().b200lab_version() >= 100


def test_null_pointers_rejected_before_launch():
    L = b200lab.lib()
    n = ctypes.c_void_p(0)
    assert L.attn_fwd_sm100(n, n, n, n, 1, 1, 1, 16, 16, 128, 0.1, 0, 1, n, 0, n) == b200lab.ERR_INVALID
    assert L.gdn_decode_sm100(n, n, n, n, n, n, n, 1, 1, 1, 128, 128, 0, 0.1, 1, 1, n) == b200lab.ERR_INVALID
    assert L.gdn_prefill_sm100(n, n, n, n, n, n, n, 1, 8, 1, 1, 128, 128, 0, 0.1, 1, 1, n, 0, n) \
        in (b200lab.ERR_INVALID, b200lab.ERR_UNSUPPORTED)
    assert L.attn_fwd_sm100_host(n, n, n, n, n, n, n, n, 1, 1, 1, 16, 16, 128, 0.1, 0, 1, n) \
        == b200lab.ERR_INVALID
    p = ctypes.c_void_p(16)  # never dereferenced
    # packed GDN prefill: no cu_seqlens, or no tokens
    assert L.gdn_prefill_sm100_varlen(p, p, p, p, p, p, p, n, 64, 64, 1, 1, 1, 128, 128, 0, 0.1, 1, 1, p, 1 << 20, n) \
        == b200lab.ERR_INVALID
    assert L.gdn_prefill_sm100_varlen(p, p, p, p, p, p, p, p, 64, 0, 1, 1, 1, 128, 128, 0, 0.1, 1, 1, p, 1 << 20, n) \
        == b200lab.ERR_INVALID


def test_shape_rules_rejected_before_launch():
    L = b200lab.lib()
    p = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    n = ctypes.c_void_p(0)
    # Hq not a multiple of Hkv
    assert L.attn_fwd_sm100(p, p, p, p, 1, 3, 2, 16, 16, 128, 0.1, 0, 1, n, 0, n) == b200lab.ERR_INVALID
    # D = 96 is not built
    assert L.attn_fwd_sm100(p, p, p, p, 1, 2, 2, 16, 16, 96, 0.1, 0, 1, n, 0, n) == b200lab.ERR_UNSUPPORTED
    # bad dtype / causal flag / scale
    assert L.attn_fwd_sm100(p, p, p, p, 1, 2, 2, 16, 16, 128, 0.1, 0, 7, n, 0, n) == b200lab.ERR_INVALID
    assert L.attn_fwd_sm100(p, p, p, p, 1, 2, 2, 16, 16, 128, 0.1, 2, 1, n, 0, n) == b200lab.ERR_INVALID
    assert L.attn_fwd_sm100(p, p, p, p, 1, 2, 2, 16, 16, 128, -1.0, 0, 1, n, 0, n) == b200lab.ERR_INVALID
    # the host-buffer form applies the same rules before creating any stream
    assert L.attn_fwd_sm100_host(p, p, p, p, p, p, p, p, 1, 3, 2, 16, 16, 128, 0.1, 0, 1, n) == b200lab.ERR_INVALID
    assert L.attn_fwd_sm100_host(p, p, p, p, p, p, p, p, 1, 2, 2, 16, 16, 96, 0.1, 0, 1, n) \
        == b200lab.ERR_UNSUPPORTED
    assert L.attn_fwd_sm100_host(p, p, p, p, p, p, p, p, 1, 2, 2, 16, 16, 128, 0.1, 2, 1, n) == b200lab.ERR_INVALID
    assert L.attn_fwd_sm100_host(p, p, p, p, p, p, p, p, 1, 2, 2, 16, 16, 128, -1.0, 0, 1, n) \
        == b200lab.ERR_INVALID
    # decode: dk != 128, head_map 1 with Hv % Hqk != 0
    assert L.gdn_decode_sm100(p, p, p, p, p, p, p, 1, 1, 1, 64, 64, 0, 0.1, 1, 1, n) == b200lab.ERR_UNSUPPORTED
    assert L.gdn_decode_sm100(p, p, p, p, p, p, p, 1, 3, 4, 128, 128, 1, 0.1, 1, 1, n) == b200lab.ERR_INVALID


def test_state16_decode_rules_rejected_before_launch():
    L = b200lab.lib()
    p = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    n = ctypes.c_void_p(0)
    f = L.gdn_decode_sm100_state16
    # null pointers, an fp32 state dtype (that is gdn_decode_sm100), dk != 128
    assert f(n, n, n, n, n, n, b200lab.F16, n, 1, 1, 1, 128, 128, 0, 0.1, 1, 1, n) == b200lab.ERR_INVALID
    assert f(p, p, p, p, p, p, b200lab.F32, p, 1, 1, 1, 128, 128, 0, 0.1, 1, 1, n) == b200lab.ERR_INVALID
    assert f(p, p, p, p, p, p, b200lab.BF16, p, 1, 1, 1, 64, 64, 0, 0.1, 1, 1, n) == b200lab.ERR_UNSUPPORTED
    # state not 16-byte aligned
    odd = ctypes.c_void_p(24)
    assert f(p, p, p, p, p, odd, b200lab.F16, p, 1, 1, 1, 128, 128, 0, 0.1, 1, 1, n) == b200lab.ERR_INVALID


def test_prefill_segment_plan_in_workspace_sizes():
    """Host-side plan of the segmented chain, seen through the workspace queries (no GPU
    call: the SM count falls back to 148 without a device).  One GPU's share of C3 on 8 GPUs
    (Hv 4) is segmented; C3 itself (Hv 32, 128 state CTAs) and short sequences are not."""
    import b200lab
    L = b200lab.lib()
    full = lambda *a: L.gdn_prefill_sm100_workspace_ex(*a, 128, 128, b200lab.BF16)  # noqa: E731
    small = lambda *a: L.gdn_prefill_sm100_workspace_min(*a, 128, 128, b200lab.BF16)  # noqa: E731
    assert full(1, 4096, 16, 32) == small(1, 4096, 16, 32)
    assert full(1, 300, 2, 4) == small(1, 300, 2, 4)
    # 4 segments of 16 chunks, a head: end states 4 x 256 x 128 fp32, zero-state outputs
    # 4096 x 128 fp32, R 4096 x 128 bf16, segment starts 4 x 128 x 128 bf16
    extra = 4 * (4 * 256 * 128 * 4 + 4096 * 128 * 4 + 4096 * 128 * 2 + 4 * 128 * 128 * 2)
    assert full(1, 4096, 16, 4) == small(1, 4096, 16, 4) + extra
    assert L.gdn_prefill_sm100_workspace_ex(1, 4096, 16, 4, 128, 128, b200lab.F32) == \
        L.gdn_prefill_sm100_workspace_min(1, 4096, 16, 4, 128, 128, b200lab.F32) + extra
