"""Python binding of libnimf_cuda.so, mirroring Nimformer's backend.nim API.

The names, argument order and error behaviour follow backend.nim:87-186 and
customfloat.nim:8-43 so that code (and tests) written against the reference
read the same:

    ctx = newBackend()                       # backend.nim:66-70 (CUDA only)
    y = beMatmulQ4(ctx, a, wq, scales, zeros, M, K, N, groupSize, nGroupsPerRow)
    y = beMatmul(ctx, a, M, K, b, K2, N)
    y1, y2 = beMatmul2(ctx, a1, M1, K1, b1, K1b, N1, a2, M2, K2, b2, K2b, N2)
    buf = beCustomfloatEncode(ctx, arr, cf); arr = beCustomfloatDecode(ctx, buf, cf)
    data, cf = beApfCastForTraining(ctx, arr)

Failures raise CatchableError (the reference raises CatchableError from
cuda_runtime.nim:64-66 and never falls back to the CPU while
gForbidCpuFallback is true, gpubackend.nim:46-61).  There is no CPU path in
this module: if the CUDA library is missing the import of a be* call fails.

Beyond the drop-in procs, the Weight class exposes the device weight
registry (upload once, call many times) that the library adds.
"""
import ctypes
import os
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libnimf_cuda.so")

NIMF_OK = 0
ERR_NAMES = {-1: "ARG", -2: "SHAPE", -3: "CUDA", -4: "NCCL", -5: "TIMEOUT", -6: "UNSUPPORTED",
             -7: "STATE"}

KIND_F32, KIND_INT8, KIND_INT4_SYM, KIND_INT4_ASYM, KIND_CUSTOM_FLOAT, KIND_FP4 = 0, 1, 2, 3, 6, 100

# Every symbol include/nimf_cuda.h declares (checked by the ABI test).
EXPORTS = [
    "nimf_init", "nimf_shutdown", "nimf_last_error", "nimf_device_count", "nimf_sync",
    "nimf_alloc_count",
    "nimf_weight_register_q4g", "nimf_weight_register_i8", "nimf_weight_register_cf",
    "nimf_weight_register_fp4", "nimf_weight_register_f32", "nimf_weight_free",
    "nimf_weight_info", "nimf_matmul_w", "nimf_matmul_w_dev", "nimf_matmul_w_group_dev",
    "nimf_matmul_w_group", "nimf_matmul_q4",
    "nimf_weight_cache_clear", "nimf_q4_cache_set_check", "nimf_q4_cache_size",
    "nimf_matmul_f32", "nimf_matmul2_f32", "nimf_dequant_w",
    "nimf_cf_encode", "nimf_cf_decode", "nimf_cf_encode_dev", "nimf_cf_decode_dev",
    "nimf_cf_autoselect", "nimf_apf_cast", "nimf_cf_autoselect_dev_noalloc",
    "nimf_nimq_parse", "nimf_nimq_get", "nimf_nimq_register", "nimf_weight_register_gptq",
    "nimf_rmsnorm_dev", "nimf_layernorm_dev", "nimf_add_rmsnorm_dev", "nimf_add_dev", "nimf_swiglu_dev", "nimf_rope_dev",
    "nimf_attention_decode_dev", "nimf_embedding_lookup_dev", "nimf_greedy_sample_dev",
    "nimf_p2p_create", "nimf_p2p_connect", "nimf_p2p_allgather_dev", "nimf_p2p_destroy",
    "nimf_p2p_set_timeout_ms",
    "nimf_decode_create", "nimf_decode_step_dev", "nimf_decode_info", "nimf_decode_set_timeout_ms",
    "nimf_decode_destroy",
    "nimf_p2p_connect_comm", "nimf_comm_unique_id", "nimf_comm_init", "nimf_comm_info",
    "nimf_comm_allgather_dev", "nimf_comm_barrier", "nimf_comm_destroy", "nimf_shard_range",
    "nimf_matmul_w_allgather_dev", "nimf_decode_create_sharded",
    "nimf_gather_create", "nimf_matmul_w_group_gather_dev", "nimf_gather_set_timeout_ms",
    "nimf_gather_destroy", "nimf_attention_prefill_dev", "nimf_attention_decode_batch_dev",
    "nimf_q4_prefill_mode", "nimf_decode_timeline",
]


class CatchableError(Exception):
    """Raised for every non-zero status of the C library."""


_lib = None


def library_path():
    return LIB_PATH


def lib():
    """Loads libnimf_cuda.so (raises CatchableError if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise CatchableError("libnimf_cuda.so not found at %s: run __graft_entry__.build()" % LIB_PATH)
    L = ctypes.CDLL(LIB_PATH)
    i64, i32, vp, f32p = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p
    u64p = ctypes.POINTER(ctypes.c_uint64)
    sig = {
        "nimf_init": [i32],
        "nimf_shutdown": [],
        "nimf_device_count": [ctypes.POINTER(ctypes.c_int)],
        "nimf_sync": [],
        "nimf_alloc_count": [ctypes.POINTER(i64)],
        "nimf_weight_register_q4g": [vp, vp, vp, i64, i64, i64, i64, i64, i64, u64p],
        "nimf_weight_register_i8": [vp, vp, i64, i64, i64, i64, i64, u64p],
        "nimf_weight_register_cf": [vp, i32, i32, vp, i64, i64, i64, i64, u64p],
        "nimf_weight_register_fp4": [vp, vp, ctypes.c_float, i64, i64, i64, i64, u64p],
        "nimf_weight_register_f32": [vp, i64, i64, u64p],
        "nimf_weight_free": [ctypes.c_uint64],
        "nimf_weight_info": [ctypes.c_uint64, ctypes.POINTER(i64), ctypes.POINTER(i64),
                             ctypes.POINTER(ctypes.c_int), ctypes.POINTER(i64)],
        "nimf_matmul_w": [ctypes.c_uint64, vp, i64, vp],
        "nimf_matmul_w_dev": [ctypes.c_uint64, vp, i64, vp, vp],
        "nimf_matmul_w_group_dev": [vp, i32, vp, i64, vp, vp],
        "nimf_matmul_w_group": [vp, i32, vp, i64, vp],
        "nimf_matmul_q4": [vp, vp, vp, vp, i64, i64, i64, i64, i64, vp],
        "nimf_weight_cache_clear": [],
        "nimf_q4_cache_set_check": [i32],
        "nimf_q4_cache_size": [ctypes.POINTER(i64)],
        "nimf_matmul_f32": [vp, i64, i64, vp, i64, i64, vp],
        "nimf_matmul2_f32": [vp, i64, i64, vp, i64, i64, vp, i64, i64, vp, i64, i64, vp, vp],
        "nimf_dequant_w": [ctypes.c_uint64, vp],
        "nimf_cf_encode": [vp, i64, i32, i32, vp],
        "nimf_cf_decode": [vp, i64, i32, i32, vp],
        "nimf_cf_encode_dev": [vp, i64, i32, i32, vp, vp],
        "nimf_cf_decode_dev": [vp, i64, i32, i32, vp, vp],
        "nimf_cf_autoselect": [vp, i64, vp, i64, ctypes.c_double, i32,
                               ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)],
        "nimf_apf_cast": [vp, i64, vp, i64, ctypes.c_double, i32, ctypes.POINTER(ctypes.c_int),
                          ctypes.POINTER(ctypes.c_int), vp],
        "nimf_cf_autoselect_dev_noalloc": [vp, i64, vp, i64, ctypes.c_double, i32,
                                           ctypes.POINTER(ctypes.c_int),
                                           ctypes.POINTER(ctypes.c_int), vp],
        "nimf_nimq_parse": [vp, i64, vp, ctypes.POINTER(i64)],
        "nimf_nimq_get": [vp, i64, i64, ctypes.POINTER(NimqTensor)],
        "nimf_nimq_register": [vp, i64, i64, i64, i64, u64p],
        "nimf_weight_register_gptq": [vp, vp, vp, vp, i64, i64, i64, i64, i64, u64p],
        "nimf_rmsnorm_dev": [vp, vp, i64, i64, ctypes.c_float, vp, vp],
        "nimf_layernorm_dev": [vp, vp, vp, i64, i64, ctypes.c_float, vp, vp],
        "nimf_embedding_lookup_dev": [vp, i64, i64, vp, i64, vp, vp],
        "nimf_p2p_create": [i32, i32, i64, vp, ctypes.POINTER(i64)],
        "nimf_p2p_connect": [i64, vp],
        "nimf_p2p_allgather_dev": [i64, vp, i64, i64, i64, vp, i64, vp],
        "nimf_p2p_destroy": [i64],
        "nimf_p2p_set_timeout_ms": [i64],
        "nimf_decode_create": [ctypes.POINTER(DecodeDesc), ctypes.POINTER(i64)],
        "nimf_decode_create_sharded": [ctypes.POINTER(DecodeDesc), ctypes.POINTER(i64)],
        "nimf_decode_step_dev": [i64, vp, vp, vp, i32, vp, i64, ctypes.c_float, vp, vp],
        "nimf_decode_info": [i64, ctypes.POINTER(i64), ctypes.POINTER(i64), ctypes.POINTER(i64)],
        "nimf_decode_set_timeout_ms": [i64],
        "nimf_decode_destroy": [i64],
        "nimf_p2p_connect_comm": [i64],
        "nimf_comm_unique_id": [vp],
        "nimf_comm_init": [i32, i32, vp],
        "nimf_comm_info": [ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)],
        "nimf_comm_allgather_dev": [vp, i64, vp, vp],
        "nimf_comm_barrier": [],
        "nimf_comm_destroy": [],
        "nimf_shard_range": [i64, i32, i32, ctypes.POINTER(i64), ctypes.POINTER(i64)],
        "nimf_matmul_w_allgather_dev": [ctypes.c_uint64, vp, i64, vp, vp],
        "nimf_gather_create": [i64, ctypes.POINTER(i64), ctypes.POINTER(vp)],
        "nimf_matmul_w_group_gather_dev": [i64, vp, i32, vp, i64, vp, vp],
        "nimf_gather_set_timeout_ms": [i64],
        "nimf_gather_destroy": [i64],
        "nimf_q4_prefill_mode": [i32],
        "nimf_decode_timeline": [i64, vp, i64, i32],
        "nimf_attention_prefill_dev": [vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, i64,
                                       ctypes.c_float, vp, vp],
        "nimf_attention_decode_batch_dev": [vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, vp, vp,
                                            vp, ctypes.c_float, i32, vp, vp],
        "nimf_greedy_sample_dev": [vp, i64, i64, vp, i64, ctypes.c_float, vp, vp],
        "nimf_add_dev": [vp, vp, i64, vp, vp],
        "nimf_add_rmsnorm_dev": [vp, vp, vp, i64, i64, ctypes.c_float, vp, vp, vp],
        "nimf_swiglu_dev": [vp, vp, i64, vp, vp],
        "nimf_rope_dev": [vp, i64, i64, i64, i64, i64, vp, vp, i64, vp],
        "nimf_attention_decode_dev": [vp, vp, vp, vp, vp, i64, i64, i64, i64, i64,
                                      ctypes.c_float, vp, vp],
    }
    for name, args in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = ctypes.c_int
    L.nimf_last_error.argtypes = []
    L.nimf_last_error.restype = ctypes.c_char_p
    _lib = L
    return L


class DecodeLayerDesc(ctypes.Structure):
    """nimf_decode_layer_desc: one layer's weights (handles), norms and caches."""
    _fields_ = [("wq", ctypes.c_uint64), ("wk", ctypes.c_uint64), ("wv", ctypes.c_uint64),
                ("wo", ctypes.c_uint64), ("wgate", ctypes.c_uint64), ("wup", ctypes.c_uint64),
                ("wdown", ctypes.c_uint64), ("attn_norm", ctypes.c_void_p),
                ("ffn_norm", ctypes.c_void_p), ("k_cache", ctypes.c_void_p),
                ("v_cache", ctypes.c_void_p)]


class DecodeDesc(ctypes.Structure):
    """nimf_decode_desc: the stack's shape and its model-wide arrays."""
    _fields_ = [("n_layers", ctypes.c_int64), ("d_model", ctypes.c_int64),
                ("n_heads", ctypes.c_int64), ("n_kv_heads", ctypes.c_int64),
                ("head_dim", ctypes.c_int64), ("ffn_dim", ctypes.c_int64),
                ("vocab", ctypes.c_int64), ("max_seq", ctypes.c_int64),
                ("n_recent_max", ctypes.c_int64), ("norm_eps", ctypes.c_float),
                ("embedding", ctypes.c_void_p), ("final_norm", ctypes.c_void_p),
                ("lm_head", ctypes.c_uint64), ("rope_cos", ctypes.c_void_p),
                ("rope_sin", ctypes.c_void_p), ("layers", ctypes.POINTER(DecodeLayerDesc))]


class DecodePlan:
    """One whole decode step of a Llama-style int4-g128 stack as one launch
    (LlamaModelL.forwardStep with isPrefill = false, nim_inference.nim:887-921,
    plus the greedy branch of sampleTopP).  `layers` is a list of dicts with
    the keys of DecodeLayerDesc (weights as Weight objects or handles, arrays
    as device pointers); the other arrays are device pointers too.

    sharded=True builds the plan over the library communicator's GPUs
    (nimf_decode_create_sharded, collective): every weight is this rank's
    nimf.shard_rows rows, the caches hold this rank's n_kv_heads / world KV
    heads, and the step's outputs travel between the GPUs inside the launch."""

    def __init__(self, *, layers, embedding, final_norm, lm_head, rope_cos, rope_sin, d_model,
                 n_heads, n_kv_heads, head_dim, ffn_dim, vocab, max_seq, norm_eps=1e-6,
                 n_recent_max=64, sharded=False):
        h = lambda w: w.handle if isinstance(w, Weight) else int(w)
        arr = (DecodeLayerDesc * len(layers))()
        for i, l in enumerate(layers):
            arr[i] = DecodeLayerDesc(h(l["wq"]), h(l["wk"]), h(l["wv"]), h(l["wo"]),
                                     h(l["wgate"]), h(l["wup"]), h(l["wdown"]),
                                     l["attn_norm"], l["ffn_norm"], l["k_cache"], l["v_cache"])
        d = DecodeDesc(len(layers), d_model, n_heads, n_kv_heads, head_dim, ffn_dim, vocab, max_seq,
                       n_recent_max, norm_eps, embedding, final_norm, h(lm_head), rope_cos, rope_sin,
                       arr)
        pid = ctypes.c_int64()
        create = lib().nimf_decode_create_sharded if sharded else lib().nimf_decode_create
        check(create(ctypes.byref(d), ctypes.byref(pid)))
        self.plan = pid.value

    def step(self, token, next_token, pos, logits, recent=None, n_recent=0, penalty=1.0,
             advance_pos=False, stream=None):
        """Device pointers (ints); asynchronous on `stream`."""
        vp = ctypes.c_void_p
        check(lib().nimf_decode_step_dev(self.plan, vp(token), vp(next_token) if next_token else None,
                                         vp(pos), 1 if advance_pos else 0,
                                         vp(recent) if recent else None, n_recent,
                                         ctypes.c_float(penalty), vp(logits), vp(stream or 0)))

    def info(self):
        g, s, a = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
        check(lib().nimf_decode_info(self.plan, ctypes.byref(g), ctypes.byref(s), ctypes.byref(a)))
        return {"grid": g.value, "stages": s.value, "attn_splits": a.value}

    def destroy(self):
        if self.plan:
            check(lib().nimf_decode_destroy(self.plan))
            self.plan = 0


class NimqTensor(ctypes.Structure):
    """nimf_nimq_tensor: one record of a NIMQ2 stream (quant.nim:386-409)."""
    _fields_ = [("name", ctypes.c_void_p), ("name_len", ctypes.c_int64),
                ("kind", ctypes.c_int), ("ndims", ctypes.c_int),
                ("dims", ctypes.c_int64 * 8), ("n_scales", ctypes.c_int64),
                ("scales", ctypes.c_void_p), ("zeros", ctypes.c_void_p),
                ("group_size", ctypes.c_int64), ("exponent_bits", ctypes.c_int),
                ("mantissa_bits", ctypes.c_int), ("data", ctypes.c_void_p),
                ("data_len", ctypes.c_int64)]


def check(status):
    if status != NIMF_OK:
        msg = lib().nimf_last_error().decode(errors="replace")
        raise CatchableError("nimf error %s (%d): %s" % (ERR_NAMES.get(status, "?"), status, msg))


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _arr(a, dt):
    return np.ascontiguousarray(np.asarray(a, dtype=dt)).ravel()


# ----------------------------------------------------------- customfloat.nim
@dataclass
class CustomFloat:
    """customfloat.nim:8-13 (same fields, same derivation as newCustomFloat)."""
    exponentBits: int
    mantissaBits: int
    totalBits: int
    itemSize: int
    bias: int
    maxExp: int
    name: str
    usesUint64: bool


def newCustomFloat(exponentBits, mantissaBits, name=""):
    """customfloat.nim:15-31."""
    if exponentBits < 0 or mantissaBits < 0:
        raise CatchableError("newCustomFloat: negative bit count")
    total = 1 + exponentBits + mantissaBits
    if exponentBits > 0:
        bias, max_exp = (1 << (exponentBits - 1)) - 1, (1 << exponentBits) - 1
    else:
        bias, max_exp = 0, 0
    nm = name if name else "float%d_e%dm%d" % (total, exponentBits, mantissaBits)
    return CustomFloat(exponentBits, mantissaBits, total, (total + 7) // 8, bias, max_exp, nm,
                       total <= 64)


FP8_E4M3 = newCustomFloat(4, 3, "fp8_e4m3")
FP8_E5M2 = newCustomFloat(5, 2, "fp8_e5m2")
FP11 = newCustomFloat(5, 5, "fp11")
FP16C = newCustomFloat(5, 10, "float16_custom")
FP24 = newCustomFloat(8, 15, "float24")
FP32C = newCustomFloat(8, 23, "float32_custom")
FP40 = newCustomFloat(8, 31, "float40")
FP48 = newCustomFloat(8, 39, "float48")
FP64C = newCustomFloat(11, 52, "float64_custom")

APF_DEFAULT_REL_ERROR_TOL = 1e-3
APF_EXP_MARGIN_BITS = 1


# --------------------------------------------------------------- backend.nim
@dataclass
class Backend:
    """backend.nim:24-25; only the CUDA kind exists here."""
    kind: str = "cuda"
    device: int = 0


_initialised_device = None


def init(device=0):
    global _initialised_device
    check(lib().nimf_init(int(device)))
    _initialised_device = int(device)


def shutdown():
    global _initialised_device
    if _lib is not None:
        check(lib().nimf_shutdown())
    _initialised_device = None


def device_count():
    n = ctypes.c_int(0)
    check(lib().nimf_device_count(ctypes.byref(n)))
    return n.value


def newBackend(force="cuda", device=0):
    """backend.nim:66-70.  Only "cuda" (or "auto") is accepted: there is no
    CPU fallback (backend.nim:35-64 refuses one by default)."""
    if force not in ("cuda", "auto"):
        raise CatchableError("backend %r is not provided by libnimf_cuda" % force)
    init(device)
    return Backend("cuda", device)


def closeBackend(b):
    """backend.nim:72-73 (a no-op there as well)."""


def beMatmul(ctx, a, M, K, b, K2, N):
    """backend.nim:87-91: C[M,N] = A[M,K] . B[K2,N] (fp32)."""
    a = _arr(a, np.float32)
    b = _arr(b, np.float32)
    if a.size != M * K or b.size != K2 * N:
        raise CatchableError("beMatmul: array sizes do not match M,K,K2,N")
    out = np.empty(M * N, np.float32)
    check(lib().nimf_matmul_f32(_ptr(a), M, K, _ptr(b), K2, N, _ptr(out)))
    return out


def beMatmulQ4(ctx, a, wq, scales, zeros, M, K, N, groupSize, nGroupsPerRow):
    """backend.nim:93-110 (int4 asymmetric per-group weights, host arrays).
    The packed weight is uploaded once and cached, keyed by the three arrays'
    addresses and the shape and checked against a fingerprint of their
    contents on every call."""
    a = _arr(a, np.float32)
    wq = np.ascontiguousarray(wq, dtype=np.uint8).ravel()
    scales = _arr(scales, np.float32)
    zeros = _arr(zeros, np.float32)
    if a.size != M * K:
        raise CatchableError("beMatmulQ4: a has %d elements, expected M*K=%d" % (a.size, M * K))
    if wq.size < N * ((K + 1) // 2) or scales.size < N * nGroupsPerRow or zeros.size < N * nGroupsPerRow:
        raise CatchableError("beMatmulQ4: weight arrays too short")
    out = np.empty(M * N, np.float32)
    check(lib().nimf_matmul_q4(_ptr(a), _ptr(wq), _ptr(scales), _ptr(zeros), M, K, N, groupSize,
                               nGroupsPerRow, _ptr(out)))
    return out


def beMatmul2(ctx, a1, M1, K1, b1, K1b, N1, a2, M2, K2, b2, K2b, N2):
    """backend.nim:112-119."""
    a1, b1, a2, b2 = (_arr(v, np.float32) for v in (a1, b1, a2, b2))
    o1 = np.empty(M1 * N1, np.float32)
    o2 = np.empty(M2 * N2, np.float32)
    check(lib().nimf_matmul2_f32(_ptr(a1), M1, K1, _ptr(b1), K1b, N1, _ptr(a2), M2, K2, _ptr(b2),
                                 K2b, N2, _ptr(o1), _ptr(o2)))
    return o1, o2


def beCustomfloatEncode(ctx, arr, cf):
    """backend.nim:177-178 -> customfloat.nim:125-129."""
    if not cf.usesUint64:
        raise CatchableError("encodeArray supports total_bits <= 64 only")
    x = _arr(arr, np.float32)
    out = np.empty(x.size * cf.itemSize, np.uint8)
    if x.size:
        check(lib().nimf_cf_encode(_ptr(x), x.size, cf.exponentBits, cf.mantissaBits, _ptr(out)))
    return out


def beCustomfloatDecode(ctx, buf, cf):
    """backend.nim:180-181 -> customfloat.nim:131-136."""
    if not cf.usesUint64:
        raise CatchableError("decodeArray supports total_bits <= 64 only")
    b = np.ascontiguousarray(buf, dtype=np.uint8).ravel()
    if b.size % cf.itemSize:
        raise CatchableError("buffer length %d is not a multiple of itemSize %d" % (b.size, cf.itemSize))
    out = np.empty(b.size // cf.itemSize, np.float32)
    if b.size:
        check(lib().nimf_cf_decode(_ptr(b), b.size, cf.exponentBits, cf.mantissaBits, _ptr(out)))
    return out


def buildCustomDtypeForTensor(arr, gradArr=(), relErrorTol=APF_DEFAULT_REL_ERROR_TOL,
                              expMargin=APF_EXP_MARGIN_BITS):
    """customfloat.nim:200-206 (reductions on the device)."""
    x = _arr(arr, np.float32)
    g = _arr(gradArr, np.float32) if len(gradArr) else None
    e, m = ctypes.c_int(), ctypes.c_int()
    check(lib().nimf_cf_autoselect(_ptr(x), x.size, _ptr(g), 0 if g is None else g.size,
                                   float(relErrorTol), int(expMargin), ctypes.byref(e),
                                   ctypes.byref(m)))
    return newCustomFloat(e.value, m.value, "auto_e%dm%d" % (e.value, m.value))


def beApfCastForTraining(ctx, arr, gradArr=(), relErrorTol=APF_DEFAULT_REL_ERROR_TOL,
                         expMargin=APF_EXP_MARGIN_BITS):
    """backend.nim:183-186 -> customfloat.nim:208-213."""
    x = _arr(arr, np.float32)
    g = _arr(gradArr, np.float32) if len(gradArr) else None
    e, m = ctypes.c_int(), ctypes.c_int()
    out = np.empty(max(1, x.size * 8), np.uint8)
    check(lib().nimf_apf_cast(_ptr(x), x.size, _ptr(g), 0 if g is None else g.size,
                              float(relErrorTol), int(expMargin), ctypes.byref(e), ctypes.byref(m),
                              _ptr(out)))
    cf = newCustomFloat(e.value, m.value, "auto_e%dm%d" % (e.value, m.value))
    return out[: x.size * cf.itemSize].copy(), cf


# ------------------------------------------------------------ weight registry
class Weight:
    """A device-resident weight (upload once, matmul many times)."""

    def __init__(self, handle, rows, k, kind):
        self.handle, self.rows, self.k, self.kind = handle, rows, k, kind

    @staticmethod
    def _reg(fn, *args):
        h = ctypes.c_uint64(0)
        check(fn(*args, ctypes.byref(h)))
        rows, k = ctypes.c_int64(), ctypes.c_int64()
        kind = ctypes.c_int()
        check(lib().nimf_weight_info(h.value, ctypes.byref(rows), ctypes.byref(k), ctypes.byref(kind), None))
        return Weight(h.value, rows.value, k.value, kind.value)

    @classmethod
    def q4g(cls, wq, scales, zeros, N, K, groupSize, nGroupsPerRow=None, rows=None):
        """quant.nim int4 asymmetric per-group (QuantTensor layout)."""
        if nGroupsPerRow is None:
            nGroupsPerRow = (K + groupSize - 1) // groupSize if groupSize > 0 else 1
        r0, r1 = rows if rows is not None else (0, N)
        wq = np.ascontiguousarray(wq, dtype=np.uint8).ravel()
        scales, zeros = _arr(scales, np.float32), _arr(zeros, np.float32)
        return cls._reg(lib().nimf_weight_register_q4g, _ptr(wq), _ptr(scales), _ptr(zeros), N, K,
                        groupSize, nGroupsPerRow, r0, r1)

    @classmethod
    def i8(cls, q, scales, N, K, rows=None):
        r0, r1 = rows if rows is not None else (0, N)
        q = np.ascontiguousarray(q, dtype=np.int8).ravel()
        s = _arr(np.atleast_1d(scales), np.float32)
        return cls._reg(lib().nimf_weight_register_i8, _ptr(q), _ptr(s), s.size, N, K, r0, r1)

    @classmethod
    def cf(cls, data, cf, N, K, row_scales=None, rows=None):
        r0, r1 = rows if rows is not None else (0, N)
        d = np.ascontiguousarray(data, dtype=np.uint8).ravel()
        rs = None if row_scales is None else _arr(row_scales, np.float32)
        return cls._reg(lib().nimf_weight_register_cf, _ptr(d), cf.exponentBits, cf.mantissaBits,
                        _ptr(rs), N, K, r0, r1)

    @classmethod
    def fp4(cls, packed, block_scales, tensor_scale, N, K, rows=None):
        r0, r1 = rows if rows is not None else (0, N)
        p = np.ascontiguousarray(packed, dtype=np.uint8).ravel()
        b = np.ascontiguousarray(block_scales, dtype=np.uint8).ravel()
        return cls._reg(lib().nimf_weight_register_fp4, _ptr(p), _ptr(b), float(tensor_scale), N,
                        K, r0, r1)

    @classmethod
    def gptq(cls, qweight, qzeros, scales_f16, g_idx, rows=None):
        """GPTQ-native tensors (export_to_nimq.py:219-254 layout): qweight
        int32 [K/8][N], qzeros int32 [G][N/8], scales float16 [G][N], g_idx [K]."""
        qw = np.ascontiguousarray(qweight, dtype=np.int32)
        qz = np.ascontiguousarray(qzeros, dtype=np.int32)
        sc = np.ascontiguousarray(scales_f16, dtype=np.float16).view(np.uint16)
        gi = np.ascontiguousarray(g_idx, dtype=np.int32)
        K, N = qw.shape[0] * 8, qw.shape[1]
        r0, r1 = rows if rows is not None else (0, N)
        return cls._reg(lib().nimf_weight_register_gptq, _ptr(qw), _ptr(qz), _ptr(sc), _ptr(gi),
                        K, N, sc.shape[0], r0, r1)

    @classmethod
    def f32(cls, b_kn, K, N):
        b = _arr(b_kn, np.float32)
        return cls._reg(lib().nimf_weight_register_f32, _ptr(b), K, N)

    def matmul(self, x, M):
        """Host buffers in and out (blocking): y[M, rows]."""
        x = _arr(x, np.float32)
        if x.size != M * self.k:
            raise CatchableError("x has %d elements, expected %d" % (x.size, M * self.k))
        y = np.empty(M * self.rows, np.float32)
        check(lib().nimf_matmul_w(self.handle, _ptr(x), M, _ptr(y)))
        return y.reshape(M, self.rows)

    def matmul_dev(self, x_ptr, M, y_ptr, stream=None):
        """Device pointers (ints), asynchronous on `stream` (int handle or None)."""
        check(lib().nimf_matmul_w_dev(self.handle, ctypes.c_void_p(x_ptr), M,
                                      ctypes.c_void_p(y_ptr), ctypes.c_void_p(stream or 0)))

    @staticmethod
    def matmul_group(weights, x, M):
        """Weights sharing K applied to the same host x; returns a list of y."""
        x = _arr(x, np.float32)
        hs = (ctypes.c_uint64 * len(weights))(*[w.handle for w in weights])
        ys = [np.empty(M * w.rows, np.float32) for w in weights]
        yp = (ctypes.c_void_p * len(weights))(*[y.ctypes.data for y in ys])
        check(lib().nimf_matmul_w_group(hs, len(weights), _ptr(x), M, yp))
        return [y.reshape(M, w.rows) for y, w in zip(ys, weights)]

    @staticmethod
    def matmul_group_dev(weights, x_ptr, M, y_ptrs, stream=None):
        """Device-pointer form (ints), asynchronous on `stream`."""
        hs = (ctypes.c_uint64 * len(weights))(*[w.handle for w in weights])
        yp = (ctypes.c_void_p * len(weights))(*y_ptrs)
        check(lib().nimf_matmul_w_group_dev(hs, len(weights), ctypes.c_void_p(x_ptr), M, yp,
                                            ctypes.c_void_p(stream or 0)))

    def dequant(self):
        out = np.empty(self.rows * self.k, np.float32)
        check(lib().nimf_dequant_w(self.handle, _ptr(out)))
        return out.reshape(self.rows, self.k)

    def device_bytes(self):
        b = ctypes.c_int64()
        check(lib().nimf_weight_info(self.handle, None, None, None, ctypes.byref(b)))
        return b.value

    def free(self):
        if self.handle:
            check(lib().nimf_weight_free(self.handle))
            self.handle = 0


# ------------------------------------------------------------ N-sharding
# ------------------------------------------------------------ quant.nim I/O
class QuantStateDict:
    """A NIMQ2 state dict held in memory (quant.nim:429-448 loadQuantStateDict):
    `arch` (5 ints) and `tensors`, a list of (name, info) in file order where
    info has kind, shape, group_size, exponentBits, mantissaBits and numpy
    views of scales, zero_point and data.  `register(i, rows)` uploads tensor
    i as a device-resident Weight without a host dequantisation."""

    def __init__(self, raw):
        self.raw = np.frombuffer(bytes(raw), np.uint8)
        L = lib()
        arch = (ctypes.c_int32 * 5)()
        count = ctypes.c_int64()
        check(L.nimf_nimq_parse(_ptr(self.raw), self.raw.size, arch, ctypes.byref(count)))
        self.arch = list(arch)
        base = self.raw.ctypes.data
        self.tensors = []
        for i in range(count.value):
            t = NimqTensor()
            check(L.nimf_nimq_get(_ptr(self.raw), self.raw.size, i, ctypes.byref(t)))
            off = lambda p: (p or base) - base
            name = self.raw[off(t.name):off(t.name) + t.name_len].tobytes().decode()
            info = {"kind": t.kind, "shape": [t.dims[j] for j in range(t.ndims)],
                    "group_size": t.group_size, "exponentBits": t.exponent_bits,
                    "mantissaBits": t.mantissa_bits,
                    "scales": self.raw[off(t.scales):off(t.scales) + 4 * t.n_scales].view(np.float32),
                    "zero_point": self.raw[off(t.zeros):off(t.zeros) + 4 * t.n_scales].view(np.float32),
                    "data": self.raw[off(t.data):off(t.data) + t.data_len]}
            self.tensors.append((name, info))

    def index(self, name):
        for i, (nm, _) in enumerate(self.tensors):
            if nm == name:
                return i
        raise KeyError(name)

    def register(self, i, rows=None):
        _, info = self.tensors[i]
        n = info["shape"][0] if info["shape"] else 0
        r0, r1 = rows if rows is not None else (0, n)
        return Weight._reg(lib().nimf_nimq_register, _ptr(self.raw), self.raw.size, i, r0, r1)


def loadQuantStateDict(path_or_bytes):
    """quant.nim:429-448: (arch, [(name, info)]) plus the QuantStateDict."""
    raw = path_or_bytes
    if isinstance(path_or_bytes, (str, os.PathLike)):
        with open(path_or_bytes, "rb") as f:
            raw = f.read()
    sd = QuantStateDict(raw)
    return sd.arch, sd.tensors, sd


def shard_rows(n, world, rank, align=16):
    """Row range [r0, r1) of output channels held by `rank` of `world` GPUs.

    Rows are the reference's output channels (W[N][K], nimformer.nim:90), so a
    shard is a contiguous run of packed rows and of scale/zero rows; shards are
    whole 16-row tiles except the last, and sizes differ by at most one tile.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank %d of world %d" % (rank, world))
    tiles = (n + align - 1) // align
    t0, t1 = tiles * rank // world, tiles * (rank + 1) // world
    return min(n, t0 * align), min(n, t1 * align)


def gather_shards(parts, m):
    """Reassembles y[m][N] from the ranks' shard outputs y_r[m][n_r] (rank
    order), as an all-gather of the shards followed by a column concatenation."""
    return np.concatenate([np.asarray(p, np.float32).reshape(m, -1) for p in parts], axis=1)


# ------------------------------------------------------------ host quantiser
def quantize_int4_per_group(w, group_size=128):
    """export_to_nimq.py:363-395 quantize_int4_asymmetric_per_group, vectorised.

    Same numpy arithmetic as the exporter: per (row, group) min / max / range /
    scale / zero in float64, element arithmetic w / float32(scale) +
    float32(zero) in float32, np.round half-to-even, clip to [0, 15]; even
    columns in the low nibble.  Returns (packed uint8 [rows*ceil(K/2)],
    scales float32 [rows*ngr], zeros float32 [rows*ngr]).
    """
    w = np.ascontiguousarray(w, dtype=np.float32)
    if w.ndim != 2:
        raise CatchableError("quantize_int4_per_group expects a 2-D weight")
    rows, cols = w.shape
    gs = int(group_size)
    ngr = (cols + gs - 1) // gs
    full = cols // gs
    scales = np.zeros((rows, ngr), np.float32)
    zeros = np.zeros((rows, ngr), np.float32)
    q = np.zeros((rows, cols), np.uint8)

    def one(chunk):  # chunk [rows, g, n]
        mn = chunk.min(axis=2).astype(np.float64)
        mx = chunk.max(axis=2).astype(np.float64)
        rng = mx - mn
        ok = rng > 1e-12
        scale = np.where(ok, rng / 15.0, 1.0)
        zp = np.where(ok, -mn / np.where(ok, scale, 1.0), 0.0)
        sf, zf = scale.astype(np.float32), zp.astype(np.float32)
        t = chunk / sf[..., None]
        t = t + zf[..., None]
        return np.clip(np.round(t), 0, 15).astype(np.uint8), sf, zf

    if full:
        qq, sf, zf = one(w[:, :full * gs].reshape(rows, full, gs))
        q[:, :full * gs] = qq.reshape(rows, full * gs)
        scales[:, :full], zeros[:, :full] = sf, zf
    if ngr > full:
        qq, sf, zf = one(w[:, full * gs:].reshape(rows, 1, cols - full * gs))
        q[:, full * gs:] = qq.reshape(rows, -1)
        scales[:, full:], zeros[:, full:] = sf, zf
    bpr = (cols + 1) // 2
    packed = np.zeros((rows, bpr), np.uint8)
    packed[:, :(cols + 1) // 2] = q[:, 0::2]
    packed[:, :cols // 2] |= (q[:, 1::2] << 4)
    return packed.ravel(), scales.ravel(), zeros.ravel()
