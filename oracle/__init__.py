"""CPU oracle for the attention / Gated DeltaNet hot path.

TEST INFRASTRUCTURE ONLY.  This package is imported by ``tests/``, by
``__graft_entry__.smoke()`` and by ``bench.py``'s ``cpu_baseline`` and
``--impl reference`` legs, always as the checker or the timed CPU baseline.
The product library (``turing-sm75_b200/``) never imports it and has no CPU
fallback.

Two layers:

* ``build/liboracle.so`` -- an fp64 C restatement (``oracle.c``) of the
  reference's naive attention (src/attn_sm75.cu:55-94), serial GDN recurrence
  (src/gdn_sm75.cu:1078-1106) and chunked GDN algebra
  (src/gdn_sm75.cu:1109-1244).
* ``_ref/libref_gdn.so`` / ``_ref/libref_attn.so`` -- the reference's own
  functions compiled from its sources (``oracle/Makefile``), used to pin the
  restatement.  Absent when the reference was not available at build time.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_REF_GDN = None
_REF_ATTN = None

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")


def build() -> None:
    """Compile liboracle.so (and oracle/_ref when the reference is present)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "build", "liboracle.so")
        if not os.path.exists(path):
            build()
        L = ctypes.CDLL(path)
        L.orc_attn_fwd.restype = ctypes.c_int
        L.orc_attn_fwd.argtypes = [_f32p, _f32p, _f32p, _f64p] + [ctypes.c_int] * 6 + [
            ctypes.c_double, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
        gdn_args = [_f32p] * 5 + [_f64p, _f64p] + [ctypes.c_int] * 7 + [ctypes.c_double]
        L.orc_gdn_recurrent.restype = ctypes.c_int
        L.orc_gdn_recurrent.argtypes = gdn_args + [ctypes.c_int]
        L.orc_gdn_chunked.restype = ctypes.c_int
        L.orc_gdn_chunked.argtypes = gdn_args + [ctypes.c_int, ctypes.c_int]
        L.orc_gdn_chunked_refsolve.restype = ctypes.c_int
        L.orc_gdn_chunked_refsolve.argtypes = gdn_args + [ctypes.c_int, ctypes.c_int]
        L.orc_default_threads.restype = ctypes.c_int
        _LIB = L
    return _LIB


def default_threads() -> int:
    return int(lib().orc_default_threads())


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def attn_fwd(Q, K, V, scale: float, causal: bool, rows=None, nthreads: int = 0) -> np.ndarray:
    """fp64 softmax attention.  Q [B,Hq,Sq,D], K/V [B,Hkv,Skv,D] -> O [B,Hq,Sq|len(rows),D]."""
    Q, K, V = _f32(Q), _f32(K), _f32(V)
    B, Hq, Sq, D = Q.shape
    _, Hkv, Skv, _ = K.shape
    nrow = Sq if rows is None else len(rows)
    O = np.zeros((B, Hq, nrow, D), dtype=np.float64)
    rows_arr = None if rows is None else np.ascontiguousarray(np.asarray(rows, dtype=np.int32))
    rc = lib().orc_attn_fwd(Q, K, V, O, B, Hq, Hkv, Sq, Skv, D, float(scale), int(bool(causal)),
                            None if rows_arr is None else rows_arr.ctypes.data_as(ctypes.c_void_p),
                            0 if rows_arr is None else len(rows_arr), int(nthreads))
    if rc != 0:
        raise ValueError(f"orc_attn_fwd rejected its arguments (rc={rc})")
    return O


def _gdn_common(fn, q, k, v, g_log, beta, state, scale, head_map, extra, nthreads):
    q, k, v, g_log, beta = _f32(q), _f32(k), _f32(v), _f32(g_log), _f32(beta)
    B, T, Hqk, dk = q.shape
    Hv, dv = v.shape[2], v.shape[3]
    S = np.ascontiguousarray(np.array(state, dtype=np.float64, copy=True))
    out = np.zeros((B, T, Hv, dv), dtype=np.float64)
    rc = fn(q, k, v, g_log, beta, S, out, B, T, Hqk, Hv, dk, dv, int(head_map), float(scale),
            *extra, int(nthreads))
    if rc != 0:
        raise ValueError(f"oracle GDN call rejected its arguments (rc={rc})")
    return out, S


def gdn_recurrent(q, k, v, g_log, beta, state, scale, head_map=0, nthreads=0):
    """fp64 token-serial GDN.  Returns (out [B,T,Hv,dv], final state [B,Hv,dv,dk])."""
    return _gdn_common(lib().orc_gdn_recurrent, q, k, v, g_log, beta, state, scale, head_map,
                       (), nthreads)


def gdn_chunked(q, k, v, g_log, beta, state, scale, head_map=0, chunk=64, nthreads=0):
    return _gdn_common(lib().orc_gdn_chunked, q, k, v, g_log, beta, state, scale, head_map,
                       (int(chunk),), nthreads)


def gdn_chunked_refsolve(q, k, v, g_log, beta, state, scale, head_map=0, chunk=16, nthreads=0):
    return _gdn_common(lib().orc_gdn_chunked_refsolve, q, k, v, g_log, beta, state, scale,
                       head_map, (int(chunk),), nthreads)


# ----------------------------------------------------------------------------
# The reference's own code (oracle/_ref)
# ----------------------------------------------------------------------------
def ref_gdn_available() -> bool:
    return os.path.exists(os.path.join(_HERE, "_ref", "libref_gdn.so"))


def ref_gdn():
    """ctypes handle on the reference's gdn_cpu / gdn_chunked_cpu (fp32, Hq16 Hv48 Sv128)."""
    global _REF_GDN
    if _REF_GDN is None:
        L = ctypes.CDLL(os.path.join(_HERE, "_ref", "libref_gdn.so"))
        args = [_f32p] * 5 + [_f32p, _f32p, ctypes.c_int, ctypes.c_float]
        for name in ("ref_gdn_cpu", "ref_gdn_chunked_cpu"):
            getattr(L, name).restype = ctypes.c_int
            getattr(L, name).argtypes = args
        L.ref_gdn_shape.restype = ctypes.c_int
        L.ref_gdn_shape.argtypes = [ctypes.POINTER(ctypes.c_int)] * 4
        _REF_GDN = L
    return _REF_GDN


def ref_gdn_shape():
    vals = [ctypes.c_int() for _ in range(4)]
    ref_gdn().ref_gdn_shape(*[ctypes.byref(x) for x in vals])
    return tuple(x.value for x in vals)  # (Sv, Hq, Hv, CS)


def ref_gdn_run(q, k, v, g, b, state, T, scale, chunked=False):
    """Run the reference's fp32 CPU GDN on [T][Hq][Sv]-layout inputs (no batch)."""
    st = np.ascontiguousarray(np.array(state, dtype=np.float32, copy=True))
    Sv, Hq, Hv, _ = ref_gdn_shape()
    out = np.zeros((T, Hv, Sv), dtype=np.float32)
    fn = ref_gdn().ref_gdn_chunked_cpu if chunked else ref_gdn().ref_gdn_cpu
    rc = fn(_f32(q), _f32(k), _f32(v), _f32(g), _f32(b), st, out, int(T), float(scale))
    if rc != 0:
        raise ValueError("reference gdn rejected its arguments")
    return out, st


def ref_attn_available() -> bool:
    return os.path.exists(os.path.join(_HERE, "_ref", "libref_attn.so"))


def ref_attn():
    """ctypes handle on the reference's naive_attn_kernel launcher (GPU, fp16)."""
    global _REF_ATTN
    if _REF_ATTN is None:
        L = ctypes.CDLL(os.path.join(_HERE, "_ref", "libref_attn.so"))
        L.ref_naive_attn.restype = ctypes.c_int
        L.ref_naive_attn.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 3 + [
            ctypes.c_float, ctypes.c_int]
        _REF_ATTN = L
    return _REF_ATTN


# ----------------------------------------------------------------------------
# The reference's seeded input generators, restated (used to build inputs that
# are bit-identical to what the reference binaries feed their kernels).
# ----------------------------------------------------------------------------
def ref_lcg_gdn_inputs(T: int, Hq: int = 16, Hv: int = 48, Sv: int = 128):
    """LCG stream of src/gdn_sm75.cu:1270-1279: seed 1, x = x*1664525 + 1013904223,
    u = (x >> 8) / 2^24 - 0.5, drawn in the order q, k, v, g, beta."""
    n = [T * Hq * Sv, T * Hq * Sv, T * Hv * Sv, T * Hv, T * Hv]
    total = sum(n)
    seeds = np.empty(total, dtype=np.uint64)
    x = 1
    # Vectorised LCG: x_{i+1} = a x_i + c (mod 2^32); closed form via repeated squaring
    # is overkill for these sizes, a plain loop in chunks is fast enough.
    a, c = 1664525, 1013904223
    for i in range(total):
        x = (x * a + c) & 0xFFFFFFFF
        seeds[i] = x
    u = ((seeds >> np.uint64(8)).astype(np.float32) / np.float32(16777216.0)) - np.float32(0.5)
    u = u.astype(np.float32)
    off = 0
    parts = []
    for cnt in n:
        parts.append(u[off:off + cnt])
        off += cnt
    q = (parts[0] * np.float32(0.2)).reshape(T, Hq, Sv)
    k = (parts[1] * np.float32(0.2)).reshape(T, Hq, Sv)
    v = (parts[2] * np.float32(0.2)).reshape(T, Hv, Sv)
    g = (np.float32(-0.2) + parts[3] * np.float32(0.05)).reshape(T, Hv)
    b = (np.float32(0.4) + (parts[4] + np.float32(0.5)) * np.float32(0.4)).reshape(T, Hv)
    return q, k, v, g.astype(np.float32), b.astype(np.float32)
