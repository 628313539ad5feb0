"""CPU oracle for the Popcorn decode-step path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` import this package, and only as
the checker or the timed CPU baseline. The product (``popcorn_b200``) never
imports it.

The numerics live in ``popcorn_oracle.cpp`` (a C++ restatement of the
reference's Metal kernels, each function citing the file:line it follows);
this module is a numpy/ctypes front end. Arrays use numpy dtypes float32 and
float16; bf16 arrays are numpy uint16 holding the raw bf16 bits.
"""
import ctypes
import os

import numpy as np

from . import build as _build

DT = {"f32": 8, "f16": 9, "bf16": 10}
NP = {"f32": np.float32, "f16": np.float16, "bf16": np.uint16}

_lib = None


def lib():
    global _lib
    if _lib is None:
        path = _build.LIB
        if not os.path.exists(path):
            path = _build.build()
        _lib = ctypes.CDLL(path)
        _declare(_lib)
    return _lib


def _declare(L):
    P, I, L64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
    sig = {
        "or_convert": [P, I, P, I, L64],
        "or_kv_cache_write": [P, I, P, I, L64, L64, L64, L64, L64, L64],
        "or_rmsnorm": [P, I, P, P, I, L64, L64, F, I, I],
        "or_matvec_nk": [P, I, P, I, P, I, L64, L64],
        "or_matmul": [P, I, P, I, P, I, L64, L64, L64, I],
        "or_argmax": [P, I, L64, L64, P],
        "or_rope_build": [P, P, P, P, L64, L64, F],
        "or_rope_apply": [P, I, P, P, I, P, I, L64, L64, L64, L64],
        "or_gelu_tanh": [P, I, P, I, L64],
        "or_silu": [P, I, P, I, L64],
        "or_mul": [P, P, P, I, L64],
        "or_add": [P, P, P, I, L64],
        "or_flash_decoding": [P, I, P, P, I, P, I, L64, L64, L64, L64, L64, P, L64, L64, F, I,
                              ctypes.c_int32, P, P, P],
        "or_flash_attention": [P, I, P, P, I, P, I, L64, L64, L64, L64, L64, L64, F, I, ctypes.c_int32],
        "or_attention_exact": [P, I, P, P, I, P, L64, L64, L64, L64, L64, L64, P, L64, F, I,
                               ctypes.c_int32],
        "or_decode_layer": [P, I, P, P, P, P, P, P, P, P, P, L64, L64, L64, L64, L64, L64, L64, F, F,
                            I, P, P, P, I, I, P, P],
        "or_aq_matmul": [P, I, P, P, P, I, P, I, L64, L64, L64],
        "or_aq_matmul_exact": [P, I, P, P, P, I, P, L64, L64, L64],
        "or_embedding_gather": [P, P, I, P, I, L64, L64],
        "or_aq_embedding_gather": [P, P, P, P, I, P, I, L64, L64],
        "or_set_threads": [I],
    }
    for name, args in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = None
    L.or_threads.restype = I


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _c(a):
    return np.ascontiguousarray(a)


def set_threads(n):
    lib().or_set_threads(int(n))


def threads():
    return lib().or_threads()


# --- element conversions (PopcornDTypes.h:9-53) -----------------------------

def to_dtype(x, dt):
    """float32 array -> array holding `dt` elements (RNE; bf16 as uint16 bits)."""
    x = _c(np.asarray(x, dtype=np.float32))
    out = np.empty(x.shape, dtype=NP[dt])
    lib().or_convert(_p(x), DT["f32"], _p(out), DT[dt], x.size)
    return out


def to_f32(x, dt):
    x = _c(x)
    out = np.empty(x.shape, dtype=np.float32)
    lib().or_convert(_p(x), DT[dt], _p(out), DT["f32"], x.size)
    return out


# --- ops ---------------------------------------------------------------------

def kv_cache_write(src, sdt, cache, cdt, offset):
    """KVCacheWrite.metal:7-59. src [B,Nkv,Snew,Hd] into cache [B,Nkv,Smax,Hd] (in place)."""
    src = _c(src)
    B, Nkv, Snew, Hd = src.shape
    Smax = cache.shape[2]
    assert cache.flags.c_contiguous
    lib().or_kv_cache_write(_p(src), DT[sdt], _p(cache), DT[cdt], B, Nkv, Snew, Smax, Hd, offset)
    return cache


def rmsnorm(x, xdt, w, odt=None, eps=1e-6, add_one=False, width=0):
    """RMSNorm.metal:7-42 over the last axis; w is float32 [H] or None."""
    x = _c(x)
    odt = odt or xdt
    H = x.shape[-1]
    rows = x.size // H
    out = np.empty(x.shape, dtype=NP[odt])
    w = None if w is None else _c(np.asarray(w, dtype=np.float32))
    lib().or_rmsnorm(_p(x), DT[xdt], _p(w), _p(out), DT[odt], rows, H, eps, int(add_one), width)
    return out


def matvec_nk(x, xdt, w, wdt, odt):
    """Matvec.metal:56-127: y = W x with W [N,K]."""
    x, w = _c(x), _c(w)
    N, K = w.shape
    out = np.empty((N,), dtype=NP[odt])
    lib().or_matvec_nk(_p(x), DT[xdt], _p(w), DT[wdt], _p(out), DT[odt], K, N)
    return out


def matmul(a, adt, b, bdt, odt, transpose_b):
    """Matmul.metal:7-27: C = A B (or A B^T)."""
    a, b = _c(a), _c(b)
    M, K = a.shape
    N = b.shape[0] if transpose_b else b.shape[1]
    out = np.empty((M, N), dtype=NP[odt])
    lib().or_matmul(_p(a), DT[adt], _p(b), DT[bdt], _p(out), DT[odt], M, K, N, int(transpose_b))
    return out


def gelu_tanh(x, dt, odt=None):
    """GeluTanh.metal:6-35 (odt f32: the value before the store's rounding)."""
    x = _c(x)
    odt = odt or dt
    out = np.empty(x.shape, dtype=NP[odt])
    lib().or_gelu_tanh(_p(x), DT[dt], _p(out), DT[odt], x.size)
    return out


def silu(x, dt, odt=None):
    """silu(g) = g / (1 + exp(-g)) (odt f32: the value before rounding)."""
    x = _c(x)
    odt = odt or dt
    out = np.empty(x.shape, dtype=NP[odt])
    lib().or_silu(_p(x), DT[dt], _p(out), DT[odt], x.size)
    return out


def mul(a, b, dt):
    a, b = _c(a), _c(b)
    out = np.empty(a.shape, dtype=NP[dt])
    lib().or_mul(_p(a), _p(b), _p(out), DT[dt], a.size)
    return out


def add(a, b, dt):
    a, b = _c(a), _c(b)
    out = np.empty(a.shape, dtype=NP[dt])
    lib().or_add(_p(a), _p(b), _p(out), DT[dt], a.size)
    return out


def rope_build(positions, inv_freq, scaling=1.0):
    """RopeBuildCosSin.metal:5-21: fp32 cos / sin tables [T, Hd2]."""
    positions = _c(np.asarray(positions, np.int32))
    inv_freq = _c(np.asarray(inv_freq, np.float32))
    T, Hd2 = positions.size, inv_freq.size
    c = np.empty((T, Hd2), np.float32)
    s = np.empty((T, Hd2), np.float32)
    lib().or_rope_build(_p(positions), _p(inv_freq), _p(c), _p(s), T, Hd2, scaling)
    return c, s


def rope_apply(x, xdt, cos, sin, tdt, odt=None):
    """RopeApply.metal:6-49: x [B, T, Nh, Hd], tables [T, Hd/2]."""
    x, cos, sin = _c(x), _c(cos), _c(sin)
    odt = odt or xdt
    B, T, Nh, Hd = x.shape
    out = np.empty(x.shape, dtype=NP[odt])
    lib().or_rope_apply(_p(x), DT[xdt], _p(cos), _p(sin), DT[tdt], _p(out), DT[odt], B, T, Nh, Hd // 2)
    return out


def aq_quantize(w, group=64, sdt="bf16", bias=True):
    """MLX-style affine 4-bit quantisation of w [N, K] (float): per group of
    `group` values scale = (max - min) / 15, bias = min (scale and bias
    rounded to sdt first), q = clip(round((w - bias) / scale), 0, 15), packed
    8 per u32 word, lowest index in the lowest bits
    (AffineQuantizationFormat.swift:22-29). Without bias (the reference's
    nil-bias case): scale = max|w| / 15, q = clip(round(w / scale), 0, 15).
    This is test-data generation; the kernels only consume the format.
    Returns (packed u32 [N, K/8], scales [N, K/group], biases or None)."""
    w = np.asarray(w, np.float32)
    N, K = w.shape
    g = w.reshape(N, K // group, group)
    lo, hi = g.min(axis=2), g.max(axis=2)
    if bias:
        sc = np.maximum((hi - lo) / 15.0, 1e-8).astype(np.float32)
        scales = to_dtype(sc, sdt)
        biases = to_dtype(lo, sdt)
        s32, b32 = to_f32(scales, sdt) if sdt != "f32" else scales, to_f32(biases, sdt) if sdt != "f32" else biases
        q = np.clip(np.rint((g - b32[..., None]) / s32[..., None]), 0, 15)
    else:
        sc = np.maximum(np.abs(g).max(axis=2) / 15.0, 1e-8).astype(np.float32)
        scales = to_dtype(sc, sdt)
        biases = None
        s32 = to_f32(scales, sdt) if sdt != "f32" else scales
        q = np.clip(np.rint(g / s32[..., None]), 0, 15)
    q = q.astype(np.uint32).reshape(N, K // 8, 8)
    packed = np.zeros((N, K // 8), np.uint32)
    for i in range(8):
        packed |= q[:, :, i] << np.uint32(4 * i)
    return packed, scales, biases


def aq_dequantize(packed, scales, biases, sdt, K, group=64):
    """float32 [N, K] = q * scale + bias (fp32 arithmetic, as the kernels)."""
    N = packed.shape[0]
    q = np.stack([(packed >> np.uint32(4 * i)) & np.uint32(15) for i in range(8)], axis=-1).reshape(N, K)
    s = (to_f32(scales, sdt) if sdt != "f32" else scales).astype(np.float32)
    out = q.astype(np.float32) * np.repeat(s, group, axis=1)
    if biases is not None:
        b = (to_f32(biases, sdt) if sdt != "f32" else biases).astype(np.float32)
        out = out + np.repeat(b, group, axis=1)
    return out


def aq_matmul(x, xdt, packed, scales, biases, sdt, odt):
    """Affine-quantised Matmul (see or_aq_matmul): x [M, K] . dequant(W)^T."""
    x, packed, scales = _c(x), _c(np.asarray(packed, np.uint32)), _c(scales)
    biases = None if biases is None else _c(biases)
    M, K = x.shape
    N = packed.shape[0]
    out = np.empty((M, N), dtype=NP[odt])
    lib().or_aq_matmul(_p(x), DT[xdt], _p(packed), _p(scales), _p(biases), DT[sdt], _p(out), DT[odt], M, N, K)
    return out


def aq_matmul_exact(x, xdt, packed, scales, biases, sdt):
    x, packed, scales = _c(x), _c(np.asarray(packed, np.uint32)), _c(scales)
    biases = None if biases is None else _c(biases)
    M, K = x.shape
    N = packed.shape[0]
    out = np.empty((M, N), dtype=np.float64)
    lib().or_aq_matmul_exact(_p(x), DT[xdt], _p(packed), _p(scales), _p(biases), DT[sdt], _p(out), M, N, K)
    return out


def embedding_gather(ids, table, tdt, odt=None):
    """EmbeddingGather.metal: rows of table [V, H] at ids (int32)."""
    ids, table = _c(np.asarray(ids, np.int32)), _c(table)
    odt = odt or tdt
    T, H = ids.size, table.shape[1]
    out = np.empty((T, H), dtype=NP[odt])
    lib().or_embedding_gather(_p(ids), _p(table), DT[tdt], _p(out), DT[odt], T, H)
    return out


def aq_embedding_gather(ids, packed, scales, biases, sdt, odt, H):
    """AffineQuantizedEmbeddingGather.metal: dequantised rows at ids."""
    ids, packed, scales = _c(np.asarray(ids, np.int32)), _c(np.asarray(packed, np.uint32)), _c(scales)
    biases = None if biases is None else _c(biases)
    T = ids.size
    out = np.empty((T, H), dtype=NP[odt])
    lib().or_aq_embedding_gather(_p(ids), _p(packed), _p(scales), _p(biases), DT[sdt], _p(out), DT[odt], T, H)
    return out


def attention_mask(Sq, Sk, window=None):
    """AttentionMaskBuild.metal:5-21: f32 [Sq, Sk], 0 where query i (key
    position Sk - Sq + i) may see key j (j <= position, and position - j <
    window when a window is given), -inf elsewhere."""
    i = np.arange(Sq)[:, None]
    j = np.arange(Sk)[None, :]
    pos = Sk - Sq + i
    ok = j <= pos
    if window is not None and window >= 0:
        ok &= (pos - j) < window
    return np.where(ok, np.float32(0.0), np.float32(-np.inf)).astype(np.float32)


def argmax(x, dt):
    """Argmax.metal:5-76 over the last axis: int32 index per row (ties -> the
    lowest index; NaN never wins; a row of NaN gives 0x7fffffff for n >= 32)."""
    x = _c(x)
    N = x.shape[-1]
    rows = x.size // N
    out = np.empty(x.shape[:-1], dtype=np.int32)
    lib().or_argmax(_p(x), DT[dt], rows, N, _p(out))
    return out


MASK = {"causal": 0, "sliding": 1, "bidirectional": 2}


def flash_decoding(q, qdt, k, v, kvdt, odt, scale, mask="causal", window=-1, seq_lens=None,
                   partitions=8, return_partials=False):
    """FlashDecoding.metal:29-231. q [B,Nq,1,Hd]; k/v [B,Nkv,S,Hd].

    Without seq_lens every sequence has S keys (the reference). With seq_lens
    (int32 [B]) sequence b uses the first seq_lens[b] keys of a cache of
    length S (the ragged extension).
    """
    q, k, v = _c(q), _c(k), _c(v)
    B, Nq, Sq, Hd = q.shape
    assert Sq == 1
    _, Nkv, S, _ = k.shape
    lens = None if seq_lens is None else _c(np.asarray(seq_lens, dtype=np.int32))
    out = np.empty((B, Nq, 1, Hd), dtype=NP[odt])
    P = partitions
    pO = np.empty((B, Nq, P, Hd), np.float32) if return_partials else None
    pM = np.empty((B, Nq, P), np.float32) if return_partials else None
    pL = np.empty((B, Nq, P), np.float32) if return_partials else None
    lib().or_flash_decoding(_p(q), DT[qdt], _p(k), _p(v), DT[kvdt], _p(out), DT[odt], B, Nq, Nkv, S,
                            S, _p(lens), Hd, P, scale, MASK[mask], window, _p(pO), _p(pM), _p(pL))
    if return_partials:
        return out, (pO, pM, pL)
    return out


def flash_attention(q, qdt, k, v, kvdt, odt, scale, mask="causal", window=-1):
    """FlashAttention.metal:31-162 (prefill semantics, posQ = Sk - Sq + q)."""
    q, k, v = _c(q), _c(k), _c(v)
    B, Nq, Sq, Hd = q.shape
    _, Nkv, Sk, _ = k.shape
    out = np.empty((B, Nq, Sq, Hd), dtype=NP[odt])
    lib().or_flash_attention(_p(q), DT[qdt], _p(k), _p(v), DT[kvdt], _p(out), DT[odt], B, Nq, Nkv,
                             Sq, Sk, Hd, scale, MASK[mask], window)
    return out


def attention_exact(q, qdt, k, v, kvdt, scale, mask="causal", window=-1, seq_lens=None):
    """Float64 full-softmax attention (BidirectionalFATests.swift:9-53, generalised)."""
    q, k, v = _c(q), _c(k), _c(v)
    B, Nq, Sq, Hd = q.shape
    _, Nkv, S, _ = k.shape
    lens = None if seq_lens is None else _c(np.asarray(seq_lens, dtype=np.int32))
    out = np.empty((B, Nq, Sq, Hd), dtype=np.float64)
    lib().or_attention_exact(_p(q), DT[qdt], _p(k), _p(v), DT[kvdt], _p(out), B, Nq, Nkv, Sq, S, S,
                             _p(lens), Hd, scale, MASK[mask], window)
    return out


def decode_layer(x, dt, w_attn_norm, w_mlp_norm, w_qkv, w_o, w_gate, w_up, w_down, k_cache, v_cache,
                 Nq, Nkv, Hd, pos, eps=1e-6, attn_scale=1.0 / 16, act="gelu_tanh", q_norm=None, k_norm=None,
                 qk_norm=False, norm_v=False, rope_cos=None, rope_sin=None):
    """One batch-1 decode layer (see or_decode_layer). Caches [Nkv,Smax,Hd] updated in place.
    qk_norm: per-head RMSNorm of q / k (weights q_norm / k_norm, None = no
    weight) and, with norm_v, of v without weight; rope_cos / rope_sin: the
    step's table row (f32 [Hd/2]) for RoPE of q and k."""
    H = x.shape[-1]
    F = w_gate.shape[0]
    Smax = k_cache.shape[-2]
    out = np.empty((H,), dtype=NP[dt])
    args = [_c(a) for a in (x, w_attn_norm, w_mlp_norm, w_qkv, w_o, w_gate, w_up, w_down)]
    f32 = [None if a is None else _c(np.asarray(a, np.float32)) for a in (q_norm, k_norm, rope_cos, rope_sin)]
    lib().or_decode_layer(_p(args[0]), DT[dt], _p(args[1]), _p(args[2]), _p(args[3]), _p(args[4]),
                          _p(args[5]), _p(args[6]), _p(args[7]), _p(k_cache), _p(v_cache), H, Nq,
                          Nkv, Hd, F, Smax, pos, eps, attn_scale, 1 if act == "silu" else 0,
                          _p(out), _p(f32[0]), _p(f32[1]), int(qk_norm), int(norm_v), _p(f32[2]), _p(f32[3]))
    return out
