"""CPU oracle for the laya_b200 parity tests.

TEST INFRASTRUCTURE ONLY: `tests/`, `__graft_entry__.smoke()` and `bench.py`'s cpu_baseline / reference arm are
the only callers.  The product package `laya_b200` never imports this.

`laya_oracle.c` restates the reference's CPU kernels (theolivenbaum/laya, C#) in plain C, in the reference's
floating-point order; `model.py` restates the reference's forward orchestration on top of them.  Parity of the
oracle itself is pinned against the reference's committed golden vectors in `tests/test_oracle.py`.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblaya_oracle.so")
SRC_PATH = os.path.join(HERE, "laya_oracle.c")

# x86-64-v3 (AVX2 + FMA) keeps the library portable to the GPU hosts; -ffp-contract=off keeps the
# reference's exact multiply/add/fma sequence.
CFLAGS = ["-O3", "-fPIC", "-shared", "-fopenmp", "-mavx2", "-mfma", "-ffp-contract=off", "-fno-math-errno",
          "-std=c11", "-Wall"]


# The AVX-512 restatements of the reference's panel kernels (laya_vnni.c), for the timed CPU baseline only.
VNNI_PATH = os.path.join(HERE, "liblaya_vnni.so")
VNNI_SRC = os.path.join(HERE, "laya_vnni.c")
VNNI_CFLAGS = ["-O3", "-fPIC", "-shared", "-fopenmp", "-mavx512f", "-mavx512bw", "-mavx512vnni", "-ffp-contract=off",
               "-std=c11", "-Wall"]


def build(force=False):
    """Compile laya_oracle.c into liblaya_oracle.so and laya_vnni.c into liblaya_vnni.so (gcc, a few seconds)."""
    for src, out, flags in ((SRC_PATH, LIB_PATH, CFLAGS), (VNNI_SRC, VNNI_PATH, VNNI_CFLAGS)):
        if not force and os.path.exists(out) and os.path.getmtime(out) >= os.path.getmtime(src):
            continue
        tmp = out + ".tmp"
        subprocess.check_call(["gcc", *flags, src, "-o", tmp, "-lm"])
        os.replace(tmp, out)
    return LIB_PATH


_vnni = None
_FAST = False
_packed = {}   # id(weight) -> (weight, packed): packed once, as the reference packs at load


def vnni_lib():
    """The AVX-512 VNNI kernels, or None when this CPU lacks them (or the library was not built)."""
    global _vnni
    if _vnni is None:
        if not os.path.exists(VNNI_PATH):
            build()
        L = ctypes.CDLL(VNNI_PATH)
        L.lv_supported.restype = ctypes.c_int
        L.lv_q8_packed_bytes.restype = ctypes.c_long
        L.lv_q8_packed_bytes.argtypes = [ctypes.c_int, ctypes.c_int]
        L.lv_q8_pack.argtypes = [_i8p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
        L.lv_q8_matmul.argtypes = [_i8p, _f32p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_void_p, _f32p, ctypes.c_int, ctypes.c_void_p]
        L.lv_f32_packed_floats.restype = ctypes.c_long
        L.lv_f32_packed_floats.argtypes = [ctypes.c_int, ctypes.c_int]
        L.lv_f32_pack.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, _f32p]
        L.lv_linear_f32.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, _f32p, ctypes.c_int, ctypes.c_int,
                                    ctypes.c_void_p, _f32p, ctypes.c_int]
        L.lv_attention.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, _i32p, _i32p, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_void_p, ctypes.c_void_p, _f32p]
        _vnni = L if L.lv_supported() else False
    return _vnni or None


def set_fast(enabled=True):
    """Route q8_matmul, linear_f32 and attention through the AVX-512 kernels (same bits; for timing the CPU
    baseline).
    Returns whether the fast path is in use (False when the CPU lacks AVX-512 VNNI)."""
    global _FAST
    _FAST = bool(enabled) and vnni_lib() is not None
    return _FAST


def _packed_q8(qw, dw):
    key = id(qw)
    hit = _packed.get(key)
    if hit is not None and hit[0] is qw:
        return hit[1]
    N, K = qw.shape
    buf = np.zeros(vnni_lib().lv_q8_packed_bytes(N, K), np.uint8)
    vnni_lib().lv_q8_pack(np.ascontiguousarray(qw), f32(dw), N, K, buf.ctypes.data)
    _packed[key] = (qw, buf)
    return buf


def _packed_f32(w):
    key = id(w)
    hit = _packed.get(key)
    if hit is not None and hit[0] is w:
        return hit[1]
    N, K = w.shape
    buf = np.zeros(vnni_lib().lv_f32_packed_floats(N, K), np.float32)
    vnni_lib().lv_f32_pack(f32(w), N, K, buf)
    _packed[key] = (w, buf)
    return buf


_lib = None

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(dtype=np.int8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_c = ctypes


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        sig = {
            "lo_num_threads": (_c.c_int, []),
            "lo_set_num_threads": (None, [_c.c_int]),
            "lo_fp16_round": (_c.c_float, [_c.c_float]),
            "lo_q8_quantize_weight_block": (_c.c_float, [_f32p, _i8p]),
            "lo_q8_quantize_weights": (None, [_f32p, _c.c_int, _c.c_int, _i8p, _f32p]),
            "lo_q8_quantize_activations": (None, [_f32p, _c.c_int, _c.c_int, _c.c_int, _i8p, _f32p]),
            "lo_q8_matmul": (None, [_i8p, _f32p, _c.c_int, _i8p, _f32p, _c.c_int, _c.c_int, _c.c_void_p, _f32p,
                                    _c.c_int]),
            "lo_q8_block_dots": (None, [_i8p, _c.c_int, _i8p, _c.c_int, _c.c_int, _i32p]),
            "lo_linear_f32": (None, [_f32p, _c.c_int, _c.c_int, _f32p, _c.c_int, _c.c_int, _c.c_void_p, _f32p,
                                     _c.c_int]),
            "lo_sum": (_c.c_float, [_f32p, _c.c_int]),
            "lo_dot": (_c.c_float, [_f32p, _f32p, _c.c_int]),
            "lo_layer_norm_rows": (None, [_f32p, _c.c_int, _c.c_int, _f32p, _c.c_void_p, _c.c_float, _f32p]),
            "lo_exp_vec": (_c.c_float, [_c.c_float]),
            "lo_erf_vec": (_c.c_float, [_c.c_float]),
            "lo_gelu1": (_c.c_float, [_c.c_float]),
            "lo_gelu": (None, [_f32p, _c.c_long]),
            "lo_relu": (None, [_f32p, _c.c_long]),
            "lo_softmax": (None, [_f32p, _c.c_int]),
            "lo_geglu": (None, [_f32p, _c.c_int, _c.c_int, _f32p]),
            "lo_rope_table": (None, [_c.c_int, _c.c_double, _c.c_int, _f32p, _f32p]),
            "lo_attention": (None, [_f32p, _c.c_int, _c.c_int, _i32p, _i32p, _c.c_int, _c.c_int, _c.c_void_p,
                                    _c.c_void_p, _f32p]),
            "lo_add": (None, [_f32p, _f32p, _c.c_long]),
            "lo_rms_norm_rows": (None, [_f32p, _c.c_int, _c.c_int, _f32p, _c.c_float, _f32p]),
            "lo_silu_vec": (None, [_f32p, _c.c_long]),
            "lo_silu_multiply": (None, [_f32p, _c.c_int, _c.c_int, _f32p]),
            "lo_multiply_sigmoid": (None, [_f32p, _f32p, _c.c_long]),
            "lo_l2_normalize": (None, [_f32p, _c.c_int, _c.c_float, _c.c_float]),
            "lo_rms_norm_gated": (None, [_f32p, _f32p, _f32p, _c.c_int, _c.c_float, _f32p]),
            "lo_delta_rule": (None, [_f32p, _c.c_int, _c.c_int, _c.c_int, _f32p, _f32p, _f32p, _c.c_int, _f32p,
                                     _f32p, _c.c_int, _f32p, _c.c_int]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


# ---------------------------------------------------------------------------------------------------------------
# Thin numpy-facing wrappers


def q8_quantize_weight_block(x):
    q = np.zeros(32, np.int8)
    d = lib().lo_q8_quantize_weight_block(f32(x), q)
    return np.float32(d), q


def q8_quantize_weights(w):
    w = f32(w)
    N, K = w.shape
    q = np.zeros((N, K), np.int8)
    d = np.zeros((N, K // 32), np.float32)
    lib().lo_q8_quantize_weights(w, N, K, q, d)
    return q, d


def q8_quantize_activations(x, features=None):
    """x [rows, stride] fp32 -> (q int8 [rows, K], d fp32 [rows, K/32]) with K = features (default stride)."""
    x = f32(x)
    rows, stride = x.shape
    K = stride if features is None else features
    q = np.zeros((rows, K), np.int8)
    d = np.zeros((rows, K // 32), np.float32)
    lib().lo_q8_quantize_activations(x, rows, stride, K, q, d)
    return q, d


def q8_matmul(qx, dx, qw, dw, bias=None):
    rows, K = qx.shape
    N = qw.shape[0]
    out = np.zeros((rows, N), np.float32)
    b = None if bias is None else f32(bias)
    if _FAST:
        scratch = np.empty(rows * K, np.uint8)
        vnni_lib().lv_q8_matmul(np.ascontiguousarray(qx), f32(dx), rows, _packed_q8(qw, dw).ctypes.data, N, K, _ptr(b),
                                out, N, scratch.ctypes.data)
        return out
    lib().lo_q8_matmul(np.ascontiguousarray(qx), f32(dx), rows, np.ascontiguousarray(qw), f32(dw), N, K, _ptr(b),
                       out, N)
    return out


def q8_linear(x, qw, dw, bias=None):
    qx, dx = q8_quantize_activations(x)
    return q8_matmul(qx, dx, qw, dw, bias)


def q8_block_dots(qx, qw):
    rows, K = qx.shape
    N = qw.shape[0]
    out = np.zeros((rows, N, K // 32), np.int32)
    lib().lo_q8_block_dots(np.ascontiguousarray(qx), rows, np.ascontiguousarray(qw), N, K, out)
    return out


def linear_f32(x, w, bias=None):
    x = f32(x)
    rows, K = x.shape
    N = w.shape[0]
    out = np.zeros((rows, N), np.float32)
    b = None if bias is None else f32(bias)
    if _FAST:
        vnni_lib().lv_linear_f32(x, rows, K, _packed_f32(w), N, K, _ptr(b), out, N)
        return out
    w = f32(w)
    lib().lo_linear_f32(x, rows, K, w, N, K, _ptr(b), out, N)
    return out


def layer_norm(x, w, b, eps):
    x = f32(x)
    rows, n = x.shape
    out = np.zeros_like(x)
    bb = None if b is None else f32(b)
    lib().lo_layer_norm_rows(x, rows, n, f32(w), _ptr(bb), np.float32(eps), out)
    return out


def gelu(x):
    y = f32(x).copy()
    lib().lo_gelu(y, y.size)
    return y


def relu(x):
    y = f32(x).copy()
    lib().lo_relu(y, y.size)
    return y


def softmax(x):
    y = f32(x).copy()
    lib().lo_softmax(y, y.size)
    return y


def geglu(wide):
    wide = f32(wide)
    rows, two_i = wide.shape
    out = np.zeros((rows, two_i // 2), np.float32)
    lib().lo_geglu(wide, rows, two_i // 2, out)
    return out


def rope_table(head_dim, theta, positions):
    c = np.zeros((positions, head_dim // 2), np.float32)
    s = np.zeros((positions, head_dim // 2), np.float32)
    lib().lo_rope_table(head_dim, float(theta), positions, c, s)
    return c, s


def attention(qkv, hidden, heads, seg_start, seg_len, window=-1, rope=None):
    qkv = f32(qkv)
    out = np.zeros((qkv.shape[0], hidden), np.float32)
    ss = np.ascontiguousarray(seg_start, dtype=np.int32)
    sl = np.ascontiguousarray(seg_len, dtype=np.int32)
    c = s = None
    if rope is not None:
        c, s = rope
    if _FAST and (hidden // heads) % 16 == 0:
        vnni_lib().lv_attention(qkv, hidden, heads, ss, sl, len(ss), int(window), _ptr(c), _ptr(s), out)
        return out
    lib().lo_attention(qkv, hidden, heads, ss, sl, len(ss), int(window), _ptr(c), _ptr(s), out)
    return out


def dot(a, b):
    return np.float32(lib().lo_dot(f32(a), f32(b), len(a)))
