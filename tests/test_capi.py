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
