"""Python binding of the B200-native attention / Gated DeltaNet library.

A thin ctypes layer over ``lib/libb200lab.so`` (C ABI in ``include/b200lab.h``)
that takes torch CUDA tensors.  torch is used only for device memory and
streams; every computation runs in the library's sm_100a kernels.  There is
no CPU fallback: if the shared library is missing or the device is not a
B200, calls raise.

Entry points (reference interface each replaces, cookys/turing-sm75):

* :func:`attn_fwd`     -- flash_attn_sm75_wmma / _ffma  (src/attn_sm75.cu:107-375)
* :func:`gdn_prefill`  -- gdn_wmma_kernel, gdn_prep/apply (src/gdn_sm75.cu:361-574, 896-1073)
* :func:`gdn_decode`   -- token-serial gdn_occ*_kernel at T=1 (src/gdn_sm75.cu:722-789)
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libb200lab.so")

OK = 0
ERR_INVALID = -1
ERR_UNSUPPORTED = -2
ERR_CUDA = -3
ERR_TIMEOUT = -4
ERR_WORKSPACE = -5
ERR_DEVICE = -6

F16, BF16, F32 = 0, 1, 2

# Every symbol include/b200lab.h declares (checked by tests/test_capi.py).
EXPORTED = (
    "attn_fwd_sm100", "attn_fwd_sm100_workspace", "attn_gated_fwd_sm100", "attn_fwd_sm100_varlen",
    "attn_fwd_sm100_host",
    "gdn_prefill_sm100", "gdn_prefill_sm100_workspace", "gdn_prefill_sm100_workspace_ex",
    "gdn_prefill_sm100_workspace_min",
    "gdn_prefill_sm100_noalloc",
    "gdn_prefill_sm100_fused", "gdn_prefill_sm100_varlen", "gdn_prefill_sm100_fused_varlen",
    "gdn_decode_sm100", "gdn_decode_sm100_state16", "gdn_decode_sm100_fused",
    "gdn_decode_sm100_slots",
    "b200lab_strerror", "b200lab_device_status", "b200lab_version", "b200lab_launch_count",
    "b200lab_watchdog_selftest",
)

_LIB = None


class B200LabError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {strerror(status)} (status {status})")


def build() -> None:
    """Compile the library in-tree (make -C turing-sm75_b200)."""
    import subprocess
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib() -> ctypes.CDLL:
    """Load lib/libb200lab.so (raises if it has not been built)."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(
                f"{LIB_PATH} is missing: build it with `make -C {_HERE}` "
                "(there is no fallback implementation)")
        L = ctypes.CDLL(LIB_PATH)
        vp, ci, cf, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
        L.attn_fwd_sm100.restype = ci
        L.attn_fwd_sm100.argtypes = [vp, vp, vp, vp] + [ci] * 6 + [cf, ci, ci, vp, sz, vp]
        L.attn_fwd_sm100_workspace.restype = sz
        L.attn_fwd_sm100_workspace.argtypes = [ci] * 7
        L.attn_fwd_sm100_host.restype = ci
        L.attn_fwd_sm100_host.argtypes = [vp] * 8 + [ci] * 6 + [cf, ci, ci, vp]
        L.attn_fwd_sm100_varlen.restype = ci
        L.attn_fwd_sm100_varlen.argtypes = [vp] * 6 + [ci] * 7 + [cf, ci, ci, vp]
        L.attn_gated_fwd_sm100.restype = ci
        L.attn_gated_fwd_sm100.argtypes = [vp] * 5 + [ci] * 6 + [cf, ci, ci, vp]
        L.gdn_prefill_sm100.restype = ci
        L.gdn_prefill_sm100.argtypes = [vp] * 7 + [ci] * 7 + [cf, ci, ci, vp, sz, vp]
        L.gdn_prefill_sm100_workspace.restype = sz
        L.gdn_prefill_sm100_workspace.argtypes = [ci] * 6
        L.gdn_prefill_sm100_workspace_ex.restype = sz
        L.gdn_prefill_sm100_workspace_ex.argtypes = [ci] * 7
        L.gdn_prefill_sm100_workspace_min.restype = sz
        L.gdn_prefill_sm100_workspace_min.argtypes = [ci] * 7
        L.gdn_prefill_sm100_noalloc.restype = ci
        L.gdn_prefill_sm100_noalloc.argtypes = [vp] * 7 + [ci] * 7 + [cf, ci, ci, vp]
        L.gdn_decode_sm100.restype = ci
        L.gdn_decode_sm100.argtypes = [vp] * 7 + [ci] * 6 + [cf, ci, ci, vp]
        L.gdn_prefill_sm100_fused.restype = ci
        L.gdn_prefill_sm100_varlen.restype = ci
        L.gdn_prefill_sm100_varlen.argtypes = [vp] * 8 + [ci] * 8 + [cf, ci, ci, vp, sz, vp]
        L.gdn_prefill_sm100_fused_varlen.restype = ci
        L.gdn_prefill_sm100_fused_varlen.argtypes = [vp] * 10 + [ci] * 8 + [cf, ci, ci, vp, sz, vp]
        L.gdn_prefill_sm100_fused.argtypes = [vp] * 9 + [ci] * 7 + [cf, ci, ci, vp, sz, vp]
        L.gdn_decode_sm100_slots.restype = ci
        L.gdn_decode_sm100_slots.argtypes = [vp] * 7 + [ci, vp] + [ci] * 6 + [cf, ci, ci, vp]
        L.gdn_decode_sm100_fused.restype = ci
        L.gdn_decode_sm100_fused.argtypes = [vp] * 9 + [ci] * 6 + [cf, ci, ci, vp]
        L.gdn_decode_sm100_state16.restype = ci
        L.gdn_decode_sm100_state16.argtypes = [vp] * 6 + [ci, vp] + [ci] * 6 + [cf, ci, ci, vp]
        L.b200lab_strerror.restype = ctypes.c_char_p
        L.b200lab_strerror.argtypes = [ci]
        L.b200lab_device_status.restype = ci
        L.b200lab_device_status.argtypes = [vp]
        L.b200lab_watchdog_selftest.restype = ci
        L.b200lab_watchdog_selftest.argtypes = [vp]
        L.b200lab_version.restype = ci
        L.b200lab_version.argtypes = []
        L.b200lab_launch_count.restype = ctypes.c_ulonglong
        L.b200lab_launch_count.argtypes = []
        _LIB = L
    return _LIB


def strerror(status: int) -> str:
    return lib().b200lab_strerror(int(status)).decode()


def _check(status: int, what: str) -> None:
    if status != OK:
        raise B200LabError(status, what)


# ----------------------------------------------------------------------------
# torch-facing wrappers
# ----------------------------------------------------------------------------
def _torch():
    import torch
    return torch


def _dtype_code(t) -> int:
    torch = _torch()
    if t.dtype == torch.float16:
        return F16
    if t.dtype == torch.bfloat16:
        return BF16
    if t.dtype == torch.float32:
        return F32
    raise TypeError(f"unsupported dtype {t.dtype}")


def _dev(t, name):
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (no CPU path)")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return ctypes.c_void_p(t.data_ptr())


def _stream(stream):
    torch = _torch()
    if stream is None:
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream)


def attn_fwd(Q, K, V, *, scale: float | None = None, causal: bool = False, out=None,
             workspace=None, stream=None):
    """Softmax attention forward.  Q [B,Hq,Sq,D], K/V [B,Hkv,Skv,D] (fp16/bf16) -> O like Q."""
    torch = _torch()
    B, Hq, Sq, D = Q.shape
    _, Hkv, Skv, _ = K.shape
    if K.shape != V.shape or K.shape[0] != B or K.shape[3] != D:
        raise ValueError("K/V shape mismatch")
    if K.dtype != Q.dtype or V.dtype != Q.dtype:
        raise TypeError("Q, K, V must share a dtype")
    if scale is None:
        scale = 1.0 / (D ** 0.5)
    if out is None:
        out = torch.empty_like(Q)
    need = lib().attn_fwd_sm100_workspace(B, Hq, Hkv, Sq, Skv, D, int(bool(causal)))
    ws_ptr, ws_bytes = ctypes.c_void_p(0), 0
    if need:
        if workspace is None:
            workspace = torch.empty(need, dtype=torch.uint8, device=Q.device)
        ws_ptr, ws_bytes = _dev(workspace, "workspace"), workspace.numel() * workspace.element_size()
    st = lib().attn_fwd_sm100(_dev(Q, "Q"), _dev(K, "K"), _dev(V, "V"), _dev(out, "out"),
                              B, Hq, Hkv, Sq, Skv, D, float(scale), int(bool(causal)),
                              _dtype_code(Q), ws_ptr, ws_bytes, _stream(stream))
    _check(st, "attn_fwd_sm100")
    return out


def attn_gated_fwd(Q, K, V, G=None, *, scale: float | None = None, causal: bool = False, out=None,
                   stream=None):
    """Gated softmax attention, head dim 256: softmax(scale Q K^T) V * sigmoid(G).
    Q, G [B,Hq,Sq,256], K/V [B,Hkv,Skv,256] (fp16/bf16); G None = no gate."""
    torch = _torch()
    B, Hq, Sq, D = Q.shape
    _, Hkv, Skv, _ = K.shape
    if K.shape != V.shape or K.shape[0] != B or K.shape[3] != D:
        raise ValueError("K/V shape mismatch")
    if G is not None and (G.shape != Q.shape or G.dtype != Q.dtype):
        raise ValueError("G must match Q")
    if scale is None:
        scale = 1.0 / (D ** 0.5)
    if out is None:
        out = torch.empty_like(Q)
    gp = _dev(G, "G") if G is not None else ctypes.c_void_p(0)
    st = lib().attn_gated_fwd_sm100(_dev(Q, "Q"), _dev(K, "K"), _dev(V, "V"), gp, _dev(out, "out"),
                                    B, Hq, Hkv, Sq, Skv, D, float(scale), int(bool(causal)),
                                    _dtype_code(Q), _stream(stream))
    _check(st, "attn_gated_fwd_sm100")
    return out


def attn_fwd_host(Qh, Kh, Vh, Oh, Qd, Kd, Vd, Od, *, scale: float | None = None, causal: bool = False,
                  stream=None):
    """attn_fwd from HOST tensors (pinned for overlap): copies in, computes and copies O back
    to Oh, pipelined over chunks of (batch, kv-head) units; Qd..Od are device tensors of the
    same shapes used as the staging buffers.  Oh is complete when `stream` reaches this point."""
    B, Hq, Sq, D = Qh.shape
    _, Hkv, Skv, _ = Kh.shape
    if Kh.shape != Vh.shape or Oh.shape != Qh.shape:
        raise ValueError("attn_fwd_host: K/V or O shape mismatch")
    for h, d, n in ((Qh, Qd, "Q"), (Kh, Kd, "K"), (Vh, Vd, "V"), (Oh, Od, "O")):
        if h.device.type != "cpu" or not h.is_contiguous():
            raise ValueError(f"attn_fwd_host: {n} host tensor must be contiguous CPU memory")
        if d.shape != h.shape or d.dtype != h.dtype:
            raise ValueError(f"attn_fwd_host: {n} device buffer must match the host tensor")
    if scale is None:
        scale = 1.0 / (D ** 0.5)
    st = lib().attn_fwd_sm100_host(ctypes.c_void_p(Qh.data_ptr()), ctypes.c_void_p(Kh.data_ptr()),
                                   ctypes.c_void_p(Vh.data_ptr()), ctypes.c_void_p(Oh.data_ptr()),
                                   _dev(Qd, "Qd"), _dev(Kd, "Kd"), _dev(Vd, "Vd"), _dev(Od, "Od"),
                                   B, Hq, Hkv, Sq, Skv, D, float(scale), int(bool(causal)), _dtype_code(Qh),
                                   _stream(stream))
    _check(st, "attn_fwd_sm100_host")
    return Oh


def attn_fwd_varlen(Q, K, V, cu_seqlens_q, cu_seqlens_k, max_seqlen_q: int, *, scale: float | None = None,
                    causal: bool = False, out=None, stream=None):
    """Packed sequences: Q [total_q,Hq,D], K/V [total_k,Hkv,D] (fp16/bf16), cu_seqlens int32 [B+1]
    on the device.  Returns O like Q."""
    torch = _torch()
    total_q, Hq, D = Q.shape
    total_k, Hkv, _ = K.shape
    B = cu_seqlens_q.numel() - 1
    if cu_seqlens_q.dtype != torch.int32 or cu_seqlens_k.dtype != torch.int32 or cu_seqlens_k.numel() != B + 1:
        raise ValueError("cu_seqlens must be int32 [B+1]")
    if scale is None:
        scale = 1.0 / (D ** 0.5)
    if out is None:
        out = torch.empty_like(Q)
    st = lib().attn_fwd_sm100_varlen(_dev(Q, "Q"), _dev(K, "K"), _dev(V, "V"), _dev(out, "out"),
                                     _dev(cu_seqlens_q, "cu_seqlens_q"), _dev(cu_seqlens_k, "cu_seqlens_k"),
                                     int(max_seqlen_q), total_q, total_k, B, Hq, Hkv, D, float(scale),
                                     int(bool(causal)), _dtype_code(Q), _stream(stream))
    _check(st, "attn_fwd_sm100_varlen")
    return out


def gdn_prefill_workspace_bytes(B, T, Hqk, Hv, dk=128, dv=128, in_dtype=BF16) -> int:
    """Workspace bytes of the prefill entries for inputs of type in_dtype (F16 / BF16 / F32),
    including the segmented chain's buffers when the shape uses it."""
    return int(lib().gdn_prefill_sm100_workspace_ex(B, T, Hqk, Hv, dk, dv, int(in_dtype)))


def gdn_prefill_workspace_min_bytes(B, T, Hqk, Hv, dk=128, dv=128, in_dtype=BF16) -> int:
    """The smallest workspace the prefill entries accept (the unsegmented chain)."""
    return int(lib().gdn_prefill_sm100_workspace_min(B, T, Hqk, Hv, dk, dv, int(in_dtype)))


def gdn_prefill(q, k, v, g_log, beta, state, *, scale: float | None = None, head_map: int = 0,
                out=None, out_dtype=None, workspace=None, stream=None):
    """Chunked Gated DeltaNet prefill.  q,k [B,T,Hqk,dk]; v [B,T,Hv,dv]; g_log,beta [B,T,Hv]
    fp32; state [B,Hv,dv,dk] fp32 (updated in place).  Returns o [B,T,Hv,dv]."""
    torch = _torch()
    B, T, Hqk, dk = q.shape
    Hv, dv = v.shape[2], v.shape[3]
    if scale is None:
        scale = 1.0 / (dk ** 0.5)
    if out is None:
        out = torch.empty((B, T, Hv, dv), dtype=out_dtype or q.dtype, device=q.device)
    need = gdn_prefill_workspace_bytes(B, T, Hqk, Hv, dk, dv, _dtype_code(q))
    ws_ptr, ws_bytes = ctypes.c_void_p(0), 0
    if need:
        if workspace is None:
            workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
        ws_ptr, ws_bytes = _dev(workspace, "workspace"), workspace.numel() * workspace.element_size()
    st = lib().gdn_prefill_sm100(_dev(q, "q"), _dev(k, "k"), _dev(v, "v"), _dev(g_log, "g_log"),
                                 _dev(beta, "beta"), _dev(state, "state"), _dev(out, "out"),
                                 B, T, Hqk, Hv, dk, dv, int(head_map), float(scale),
                                 _dtype_code(q), _dtype_code(out), ws_ptr, ws_bytes,
                                 _stream(stream))
    _check(st, "gdn_prefill_sm100")
    return out


def gdn_prefill_varlen(q, k, v, g_log, beta, state, cu_seqlens, max_seqlen: int, *, scale: float | None = None,
                       head_map: int = 0, out=None, out_dtype=None, workspace=None, stream=None):
    """Chunked prefill over packed sequences: q,k [total,Hqk,dk]; v [total,Hv,dv]; g_log,beta
    [total,Hv] fp32; cu_seqlens [B+1] int32 on the device; state [B,Hv,dv,dk] fp32 (in place).
    Returns o [total,Hv,dv]."""
    torch = _torch()
    total, Hqk, dk = q.shape
    Hv, dv = v.shape[1], v.shape[2]
    B = cu_seqlens.numel() - 1
    if cu_seqlens.dtype != torch.int32:
        raise TypeError("cu_seqlens must be int32")
    if scale is None:
        scale = 1.0 / (dk ** 0.5)
    if out is None:
        out = torch.empty((total, Hv, dv), dtype=out_dtype or q.dtype, device=q.device)
    need = gdn_prefill_workspace_bytes(B, max_seqlen, Hqk, Hv, dk, dv, _dtype_code(q))
    if workspace is None:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=q.device)
    st = lib().gdn_prefill_sm100_varlen(_dev(q, "q"), _dev(k, "k"), _dev(v, "v"), _dev(g_log, "g_log"),
                                        _dev(beta, "beta"), _dev(state, "state"), _dev(out, "out"),
                                        _dev(cu_seqlens, "cu_seqlens"), int(max_seqlen), int(total), B, Hqk, Hv,
                                        dk, dv, int(head_map), float(scale), _dtype_code(q), _dtype_code(out),
                                        _dev(workspace, "workspace"),
                                        workspace.numel() * workspace.element_size(), _stream(stream))
    _check(st, "gdn_prefill_sm100_varlen")
    return out


def gdn_prefill_fused_varlen(q, k, v, a, b, state, cu_seqlens, max_seqlen: int, *, A_log=None, dt_bias=None,
                             scale: float | None = None, head_map: int = 0, out=None, out_dtype=None,
                             workspace=None, stream=None):
    """gdn_prefill_fused over packed sequences: raw q,k [total,Hqk,dk]; v [total,Hv,dv]; logits
    a,b [total,Hv] fp32; cu_seqlens [B+1] int32 on the device; state [B,Hv,dv,dk] (in place)."""
    torch = _torch()
    total, Hqk, dk = q.shape
    Hv, dv = v.shape[1], v.shape[2]
    B = cu_seqlens.numel() - 1
    if cu_seqlens.dtype != torch.int32:
        raise TypeError("cu_seqlens must be int32")
    if scale is None:
        scale = 1.0 / (dk ** 0.5)
    if out is None:
        out = torch.empty((total, Hv, dv), dtype=out_dtype or q.dtype, device=q.device)
    need = gdn_prefill_workspace_bytes(B, max_seqlen, Hqk, Hv, dk, dv, _dtype_code(q))
    if workspace is None:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=q.device)
    opt = lambda t, n: _dev(t, n) if t is not None else ctypes.c_void_p(0)  # noqa: E731
    st = lib().gdn_prefill_sm100_fused_varlen(
        _dev(q, "q"), _dev(k, "k"), _dev(v, "v"), _dev(a, "a"), _dev(b, "b"), opt(A_log, "A_log"),
        opt(dt_bias, "dt_bias"), _dev(state, "state"), _dev(out, "out"), _dev(cu_seqlens, "cu_seqlens"),
        int(max_seqlen), int(total), B, Hqk, Hv, dk, dv, int(head_map), float(scale), _dtype_code(q),
        _dtype_code(out), _dev(workspace, "workspace"), workspace.numel() * workspace.element_size(),
        _stream(stream))
    _check(st, "gdn_prefill_sm100_fused_varlen")
    return out


def gdn_prefill_fused(q, k, v, a, b, state, *, A_log=None, dt_bias=None, scale: float | None = None,
                      head_map: int = 0, out=None, out_dtype=None, workspace=None, stream=None):
    """Chunked prefill with the pre-processing fused: raw q,k [B,T,Hqk,dk] (L2-normalised in the
    kernels); a, b [B,T,Hv] fp32 logits (g_log = -exp(A_log) softplus(a + dt_bias), beta =
    sigmoid(b)); A_log, dt_bias [Hv] fp32 or None; fp32 state in place."""
    torch = _torch()
    B, T, Hqk, dk = q.shape
    Hv, dv = v.shape[2], v.shape[3]
    if scale is None:
        scale = 1.0 / (dk ** 0.5)
    if out is None:
        out = torch.empty((B, T, Hv, dv), dtype=out_dtype or q.dtype, device=q.device)
    need = gdn_prefill_workspace_bytes(B, T, Hqk, Hv, dk, dv, _dtype_code(q))
    ws_ptr, ws_bytes = ctypes.c_void_p(0), 0
    if need:
        if workspace is None:
            workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
        ws_ptr, ws_bytes = _dev(workspace, "workspace"), workspace.numel() * workspace.element_size()
    opt = lambda t, n: _dev(t, n) if t is not None else ctypes.c_void_p(0)  # noqa: E731
    st = lib().gdn_prefill_sm100_fused(_dev(q, "q"), _dev(k, "k"), _dev(v, "v"), _dev(a, "a"), _dev(b, "b"),
                                       opt(A_log, "A_log"), opt(dt_bias, "dt_bias"), _dev(state, "state"),
                                       _dev(out, "out"), B, T, Hqk, Hv, dk, dv, int(head_map), float(scale),
                                       _dtype_code(q), _dtype_code(out), ws_ptr, ws_bytes, _stream(stream))
    _check(st, "gdn_prefill_sm100_fused")
    return out


def gdn_decode(q, k, v, g_log, beta, state, *, scale: float | None = None, head_map: int = 0,
               out=None, out_dtype=None, stream=None):
    """One Gated DeltaNet decode step.  q,k [B,Hqk,dk]; v [B,Hv,dv]; g_log,beta [B,Hv] fp32;
    state [B,Hv,dv,dk] fp32, or fp16/bf16 for the 16-bit-state entry (in place).
    Returns o [B,Hv,dv]."""
    torch = _torch()
    B, Hqk, dk = q.shape
    Hv, dv = v.shape[1], v.shape[2]
    if scale is None:
        scale = 1.0 / (dk ** 0.5)
    if out is None:
        out = torch.empty((B, Hv, dv), dtype=out_dtype or q.dtype, device=q.device)
    if state.dtype == torch.float32:
        st = lib().gdn_decode_sm100(_dev(q, "q"), _dev(k, "k"), _dev(v, "v"), _dev(g_log, "g_log"),
                                    _dev(beta, "beta"), _dev(state, "state"), _dev(out, "out"),
                                    B, Hqk, Hv, dk, dv, int(head_map), float(scale),
                                    _dtype_code(q), _dtype_code(out), _stream(stream))
        _check(st, "gdn_decode_sm100")
    else:
        # 16-bit state (fp16 / bf16): gdn_decode_sm100_state16
        st = lib().gdn_decode_sm100_state16(_dev(q, "q"), _dev(k, "k"), _dev(v, "v"),
                                            _dev(g_log, "g_log"), _dev(beta, "beta"),
                                            _dev(state, "state"), _dtype_code(state), _dev(out, "out"),
                                            B, Hqk, Hv, dk, dv, int(head_map), float(scale),
                                            _dtype_code(q), _dtype_code(out), _stream(stream))
        _check(st, "gdn_decode_sm100_state16")
    return out


def gdn_decode_fused(q, k, v, a, b, state, *, A_log=None, dt_bias=None, scale: float | None = None,
                     head_map: int = 0, out=None, out_dtype=None, stream=None):
    """Decode step with the pre-processing fused: raw q,k [B,Hqk,dk] (L2-normalised in the
    kernel); a, b [B,Hv] fp32 logits (g_log = -exp(A_log) softplus(a + dt_bias), beta =
    sigmoid(b)); A_log, dt_bias [Hv] fp32 or None; fp32 state [B,Hv,dv,dk] in place."""
    torch = _torch()
    B, Hqk, dk = q.shape
    Hv, dv = v.shape[1], v.shape[2]
    if scale is None:
        scale = 1.0 / (dk ** 0.5)
    if out is None:
        out = torch.empty((B, Hv, dv), dtype=out_dtype or q.dtype, device=q.device)
    opt = lambda t, n: _dev(t, n) if t is not None else ctypes.c_void_p(0)  # noqa: E731
    st = lib().gdn_decode_sm100_fused(_dev(q, "q"), _dev(k, "k"), _dev(v, "v"), _dev(a, "a"), _dev(b, "b"),
                                      opt(A_log, "A_log"), opt(dt_bias, "dt_bias"), _dev(state, "state"),
                                      _dev(out, "out"), B, Hqk, Hv, dk, dv, int(head_map), float(scale),
                                      _dtype_code(q), _dtype_code(out), _stream(stream))
    _check(st, "gdn_decode_sm100_fused")
    return out


def gdn_decode_slots(q, k, v, g_log, beta, state_pool, slots, *, scale: float | None = None,
                     head_map: int = 0, out=None, out_dtype=None, stream=None):
    """Decode step over a state pool: sequence b uses state_pool[slots[b]] (slots: int32 [B] on
    the device; < 0 = padding, skipped; >= n is reported as ERR_INVALID by device_status).
    state_pool [n,Hv,dv,dk] fp32 updated in place."""
    torch = _torch()
    B, Hqk, dk = q.shape
    Hv, dv = v.shape[1], v.shape[2]
    if slots.dtype != torch.int32 or slots.numel() != B:
        raise ValueError("slots must be int32 [B]")
    if scale is None:
        scale = 1.0 / (dk ** 0.5)
    if out is None:
        out = torch.zeros((B, Hv, dv), dtype=out_dtype or q.dtype, device=q.device)
    st = lib().gdn_decode_sm100_slots(_dev(q, "q"), _dev(k, "k"), _dev(v, "v"), _dev(g_log, "g_log"),
                                      _dev(beta, "beta"), _dev(state_pool, "state_pool"), _dev(slots, "slots"),
                                      int(state_pool.shape[0]), _dev(out, "out"), B, Hqk, Hv, dk, dv,
                                      int(head_map), float(scale), _dtype_code(q), _dtype_code(out),
                                      _stream(stream))
    _check(st, "gdn_decode_sm100_slots")
    return out


def launch_count() -> int:
    """Kernels this library has enqueued in this process so far."""
    return int(lib().b200lab_launch_count())


def device_status(stream=None) -> int:
    """Synchronise and return the library's device status (0 = no wait gave up)."""
    return int(lib().b200lab_device_status(_stream(stream)))


def watchdog_selftest(stream=None) -> None:
    """Enqueue the failure-path self-test: a kernel whose bounded wait never completes and
    gives up after the wait limit; the next device_status() returns ERR_TIMEOUT."""
    _check(lib().b200lab_watchdog_selftest(_stream(stream)), "b200lab_watchdog_selftest")
