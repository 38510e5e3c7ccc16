"""ctypes binding of the CPU oracle (liboracle.so built from oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() and by
the cpu-baseline leg of bench.py, always as the checker / the timed CPU
reference, never as a product path.  The functions take and return numpy
arrays and mirror the reference procedures cited in oracle.h.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_i64 = ctypes.c_int64
_int = ctypes.c_int

_lib = None


def build():
    """Compile liboracle.so with the Makefile beside this file."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        src = os.path.join(HERE, "oracle.c")
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
            build()
        L = ctypes.CDLL(LIB_PATH)
        sig = {
            "orc_quantize_int8": (None, [_f32p, _i64, _i8p, ctypes.POINTER(ctypes.c_float)]),
            "orc_dequantize_int8": (None, [_i8p, _i64, ctypes.c_float, _f32p]),
            "orc_quantize_int4_sym": (None, [_f32p, _i64, _u8p, ctypes.POINTER(ctypes.c_float)]),
            "orc_dequantize_int4_sym": (None, [_u8p, _i64, ctypes.c_float, _f32p]),
            "orc_quantize_int4_asym_tensor": (None, [_f32p, _i64, _u8p, ctypes.POINTER(ctypes.c_float),
                                                     ctypes.POINTER(ctypes.c_float)]),
            "orc_dequantize_int4_asym": (None, [_u8p, _f32p, _f32p, _i64, _i64, _i64, _i64, _f32p]),
            "orc_dequantize_transposed": (_int, [_int, _u8p, _f32p, _f32p, _i64, _i64, _i64, _i64, _f32p]),
            "orc_cf_fp32_to_packed": (ctypes.c_uint64, [ctypes.c_float, _int, _int]),
            "orc_cf_packed_to_fp32": (ctypes.c_float, [ctypes.c_uint64, _int, _int]),
            "orc_cf_encode_array": (_int, [_f32p, _i64, _int, _int, _u8p]),
            "orc_cf_decode_array": (_int, [_u8p, _i64, _int, _int, _f32p]),
            "orc_cf_required_exponent_bits": (_int, [_f32p, _i64, _int]),
            "orc_cf_required_mantissa_bits": (_int, [_f32p, _i64, ctypes.c_double, ctypes.c_void_p, _i64]),
            "orc_cpu_matmul": (None, [_f32p, _f32p, _i64, _i64, _i64, _f32p]),
            "orc_dequant_matmul_q4": (None, [_f32p, _u8p, _f32p, _f32p, _i64, _i64, _i64, _i64, _i64,
                                             _f32p, _f32p]),
            "orc_quantize_int4_asym_per_group": (None, [_f32p, _i64, _i64, _i64, _u8p, _f32p, _f32p]),
            "orc_quantize_int8_vectorized": (None, [_f32p, _i64, _i8p, ctypes.POINTER(ctypes.c_float)]),
            "orc_dequantize_gptq_linear": (None, [_i32p, _i32p, _u16p, _i32p, _i64, _i64, _i64, _f32p]),
            "orc_e4m3_ocp_to_float": (ctypes.c_float, [ctypes.c_uint8]),
            "orc_float_to_e4m3_ocp": (ctypes.c_uint8, [ctypes.c_float]),
            "orc_e2m1_to_float": (ctypes.c_float, [ctypes.c_uint8]),
            "orc_quantize_fp4_block16": (None, [_f32p, _i64, _i64, ctypes.c_float, _u8p, _u8p]),
            "orc_dequantize_fp4_block16": (None, [_u8p, _u8p, ctypes.c_float, _i64, _i64, _f32p]),
            "orc_gemv_f64": (None, [_f32p, _f32p, _i64, _i64, _i64, _f32p]),
            "orc_rmsnorm": (None, [_f32p, _f32p, _i64, _i64, ctypes.c_float, _f32p]),
            "orc_layernorm": (None, [_f32p, _f32p, _f32p, _i64, _i64, ctypes.c_float, _f32p]),
            "orc_embedding_lookup": (None, [_f32p, _i64, _i64, _i32p, _i64, _f32p]),
            "orc_greedy_sample": (None, [_f32p, _i64, _i64, _i32p, _i64, ctypes.c_float, _i32p]),
            "orc_swiglu": (None, [_f32p, _f32p, _i64, _f32p]),
            "orc_rope": (None, [_f32p, _i64, _i64, _i64, _i64, _i64, _f32p, _f32p]),
            "orc_attention_decode": (None, [_f32p, _f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64,
                                            _i64, _i64, ctypes.c_float, _f32p]),
            "orc_attention_prefill": (None, [_f32p, _f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64,
                                             _i64, _i64, _i64, ctypes.c_float, _f32p]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


# --------------------------------------------------------------- quant.nim
def quantize_int8(w):
    w = _c(w, np.float32).ravel()
    q = np.empty(w.size, np.int8)
    s = ctypes.c_float()
    lib().orc_quantize_int8(w, w.size, q, ctypes.byref(s))
    return q, np.float32(s.value)


def dequantize_int8(q, scale):
    q = _c(q, np.int8).ravel()
    out = np.empty(q.size, np.float32)
    lib().orc_dequantize_int8(q, q.size, float(scale), out)
    return out


def quantize_int4_sym(w):
    w = _c(w, np.float32).ravel()
    p = np.zeros((w.size + 1) // 2, np.uint8)
    s = ctypes.c_float()
    lib().orc_quantize_int4_sym(w, w.size, p, ctypes.byref(s))
    return p, np.float32(s.value)


def dequantize_int4_sym(packed, n, scale):
    out = np.empty(n, np.float32)
    lib().orc_dequantize_int4_sym(_c(packed, np.uint8), n, float(scale), out)
    return out


def quantize_int4_asym_tensor(w):
    w = _c(w, np.float32).ravel()
    p = np.zeros((w.size + 1) // 2, np.uint8)
    s, z = ctypes.c_float(), ctypes.c_float()
    lib().orc_quantize_int4_asym_tensor(w, w.size, p, ctypes.byref(s), ctypes.byref(z))
    return p, np.float32(s.value), np.float32(z.value)


def dequantize_int4_asym(data, scale, zero, rows, cols, group_size):
    scale = _c(np.atleast_1d(scale), np.float32)
    zero = _c(np.atleast_1d(zero), np.float32)
    out = np.empty(rows * cols, np.float32)
    lib().orc_dequantize_int4_asym(_c(data, np.uint8), scale, zero, scale.size, rows, cols,
                                   group_size, out)
    return out.reshape(rows, cols)


def dequantize_transposed(kind, data, scale, zero, rows, cols, group_size):
    scale = _c(np.atleast_1d(scale), np.float32)
    zero = _c(np.atleast_1d(zero), np.float32)
    out = np.empty(rows * cols, np.float32)
    rc = lib().orc_dequantize_transposed(kind, _c(data, np.uint8).view(np.uint8), scale, zero,
                                         scale.size, rows, cols, group_size, out)
    if rc != 0:
        raise ValueError("unsupported kind %d" % kind)
    return out.reshape(cols, rows)


# --------------------------------------------------------- customfloat.nim
def item_size(e, m):
    return (1 + e + m + 7) // 8


def cf_encode(x, e, m):
    x = _c(x, np.float32).ravel()
    out = np.zeros(x.size * item_size(e, m), np.uint8)
    if lib().orc_cf_encode_array(x, x.size, e, m, out) != 0:
        raise ValueError("encodeArray supports total_bits <= 64 only")
    return out


def cf_decode(buf, e, m):
    buf = _c(buf, np.uint8).ravel()
    isz = item_size(e, m)
    out = np.empty(buf.size // isz, np.float32)
    if lib().orc_cf_decode_array(buf, buf.size, e, m, out) != 0:
        raise ValueError("bad buffer length for itemSize %d" % isz)
    return out


def cf_pack(x, e, m):
    return int(lib().orc_cf_fp32_to_packed(float(x), e, m))


def cf_unpack(p, e, m):
    return np.float32(lib().orc_cf_packed_to_fp32(int(p), e, m))


def cf_required_exponent_bits(x, margin=1):
    x = _c(x, np.float32).ravel()
    return int(lib().orc_cf_required_exponent_bits(x, x.size, margin))


def cf_required_mantissa_bits(x, tol=1e-3, grad=None):
    x = _c(x, np.float32).ravel()
    if grad is None or np.size(grad) == 0:
        return int(lib().orc_cf_required_mantissa_bits(x, x.size, tol, None, 0))
    g = _c(grad, np.float32).ravel()
    return int(lib().orc_cf_required_mantissa_bits(x, x.size, tol, g.ctypes.data, g.size))


def cf_build_for_tensor(x, grad=None, tol=1e-3, margin=1):
    """customfloat.nim:200-206 buildCustomDtypeForTensor -> (e, m)."""
    return cf_required_exponent_bits(x, margin), cf_required_mantissa_bits(x, tol, grad)


# ---------------------------------------------------------- gpubackend.nim
def cpu_matmul(a, b, m, k, n):
    out = np.empty(m * n, np.float32)
    lib().orc_cpu_matmul(_c(a, np.float32).ravel(), _c(b, np.float32).ravel(), m, k, n, out)
    return out.reshape(m, n)


def dequant_matmul_q4(a, wq, scales, zeros, m, k, n, group_size, n_groups_per_row):
    wt = np.empty(k * n, np.float32)
    out = np.empty(m * n, np.float32)
    lib().orc_dequant_matmul_q4(_c(a, np.float32).ravel(), _c(wq, np.uint8).ravel(),
                                _c(scales, np.float32).ravel(), _c(zeros, np.float32).ravel(),
                                m, k, n, group_size, n_groups_per_row, wt, out)
    return out.reshape(m, n)


# ------------------------------------------------------- export_to_nimq.py
def quantize_int4_asym_per_group(w, group_size=128):
    w = _c(w, np.float32)
    rows, cols = w.shape
    ngr = (cols + group_size - 1) // group_size
    packed = np.zeros(rows * ((cols + 1) // 2), np.uint8)
    scales = np.empty(rows * ngr, np.float32)
    zeros = np.empty(rows * ngr, np.float32)
    lib().orc_quantize_int4_asym_per_group(w.ravel(), rows, cols, group_size, packed, scales, zeros)
    return packed, scales, zeros


def quantize_int8_vectorized(w):
    w = _c(w, np.float32).ravel()
    q = np.empty(w.size, np.int8)
    s = ctypes.c_float()
    lib().orc_quantize_int8_vectorized(w, w.size, q, ctypes.byref(s))
    return q, np.float32(s.value)


def dequantize_gptq_linear(qweight, qzeros, scales_f16, g_idx):
    qweight = _c(qweight, np.int32)
    kin = qweight.shape[0] * 8
    kout = qweight.shape[1]
    out = np.empty(kin * kout, np.float32)
    lib().orc_dequantize_gptq_linear(qweight.ravel(), _c(qzeros, np.int32).ravel(),
                                     _c(np.asarray(scales_f16, np.float16).view(np.uint16), np.uint16).ravel(),
                                     _c(g_idx, np.int32).ravel(), kin, kout,
                                     np.asarray(scales_f16).shape[0], out)
    return out.reshape(kout, kin)


# ------------------------------------------------------ FP4 (no reference)
def e4m3_ocp_to_float(v):
    return np.float32(lib().orc_e4m3_ocp_to_float(int(v)))


def float_to_e4m3_ocp(x):
    return int(lib().orc_float_to_e4m3_ocp(float(x)))


def quantize_fp4_block16(w, tensor_scale):
    w = _c(w, np.float32)
    rows, cols = w.shape
    packed = np.zeros(rows * ((cols + 1) // 2), np.uint8)
    bs = np.zeros(rows * ((cols + 15) // 16), np.uint8)
    lib().orc_quantize_fp4_block16(w.ravel(), rows, cols, float(tensor_scale), packed, bs)
    return packed, bs


def dequantize_fp4_block16(packed, block_scales, tensor_scale, rows, cols):
    out = np.empty(rows * cols, np.float32)
    lib().orc_dequantize_fp4_block16(_c(packed, np.uint8), _c(block_scales, np.uint8),
                                     float(tensor_scale), rows, cols, out)
    return out.reshape(rows, cols)


def gemv_f64(x, w):
    """y[m, n] = sum_k x[m, k] * w[n, k] accumulated in float64."""
    x = _c(x, np.float32)
    w = _c(w, np.float32)
    m, k = x.shape
    n = w.shape[0]
    y = np.empty(m * n, np.float32)
    lib().orc_gemv_f64(x.ravel(), w.ravel(), m, k, n, y)
    return y.reshape(m, n)


# ------------------------------------------------ nim_inference.nim decode glue
def rmsnorm(x, w, eps):
    x = _c(x, np.float32)
    rows, cols = x.shape
    y = np.empty(rows * cols, np.float32)
    lib().orc_rmsnorm(x.ravel(), _c(w, np.float32).ravel(), rows, cols, ctypes.c_float(eps), y)
    return y.reshape(rows, cols)


def layernorm(x, gamma, beta, eps):
    x = _c(x, np.float32)
    rows, cols = x.shape
    y = np.empty(rows * cols, np.float32)
    lib().orc_layernorm(x.ravel(), _c(gamma, np.float32).ravel(), _c(beta, np.float32).ravel(),
                        rows, cols, ctypes.c_float(eps), y)
    return y.reshape(rows, cols)


def embedding_lookup(table, ids):
    table = _c(table, np.float32)
    vocab, dim = table.shape
    ids = _c(ids, np.int32).ravel()
    out = np.empty(ids.size * dim, np.float32)
    lib().orc_embedding_lookup(table.ravel(), vocab, dim, ids, ids.size, out)
    return out.reshape(ids.size, dim)


def greedy_sample(logits, recent, penalty):
    """logits [rows][vocab]; recent [rows][n] int32 (n may be 0)."""
    logits = _c(logits, np.float32)
    rows, vocab = logits.shape
    recent = _c(recent, np.int32).reshape(rows, -1)
    n = recent.shape[1]
    out = np.empty(rows, np.int32)
    rec = recent.ravel() if recent.size else np.zeros(1, np.int32)
    lib().orc_greedy_sample(logits.ravel(), rows, vocab, rec, n, ctypes.c_float(penalty), out)
    return out


def swiglu(g, u):
    g = _c(g, np.float32).ravel()
    out = np.empty(g.size, np.float32)
    lib().orc_swiglu(g, _c(u, np.float32).ravel(), g.size, out)
    return out


def rope(data, B, T, H, D, pos_offset, cos_t, sin_t):
    d = np.array(data, np.float32).ravel()
    lib().orc_rope(d, B, T, H, D, pos_offset, _c(cos_t, np.float32).ravel(), _c(sin_t, np.float32).ravel())
    return d


def attention_prefill(q, k_new, v_new, k_cache, v_cache, T, H, HKV, D, max_seq, pos0, scale):
    """Returns (out[T*H*D], k_cache, v_cache) with rows pos0 .. pos0+T-1 appended."""
    kc = np.array(k_cache, np.float32).ravel()
    vc = np.array(v_cache, np.float32).ravel()
    out = np.empty(T * H * D, np.float32)
    lib().orc_attention_prefill(_c(q, np.float32).ravel(), _c(k_new, np.float32).ravel(),
                                _c(v_new, np.float32).ravel(), kc, vc, T, H, HKV, D, max_seq, pos0,
                                ctypes.c_float(scale), out)
    return out, kc, vc


def attention_decode(q, k_new, v_new, k_cache, v_cache, H, HKV, D, max_seq, pos, scale):
    """Returns (out[H*D], k_cache, v_cache) with row pos appended."""
    kc = np.array(k_cache, np.float32).ravel()
    vc = np.array(v_cache, np.float32).ravel()
    out = np.empty(H * D, np.float32)
    lib().orc_attention_decode(_c(q, np.float32).ravel(), _c(k_new, np.float32).ravel(),
                               _c(v_new, np.float32).ravel(), kc, vc, H, HKV, D, max_seq, pos,
                               ctypes.c_float(scale), out)
    return out, kc, vc
