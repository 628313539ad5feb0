"""The CPU oracle pinned against the reference's own known-answer tests.

Every case here is a test of finnvoor/Popcorn (Tests/PopcornTests/...),
transcribed into tests/golden/reference_kats.json, run on the oracle.
"""
import os

import numpy as np
import pytest

import oracle
from tests.conftest import approx_equal
from tests.golden import make_golden


def test_kv_cache_write_kat(kats):
    c = kats["kv_cache_write"]
    src = np.array(c["src"], np.float32).reshape(c["B"], c["Nkv"], c["Snew"], c["Hd"])
    cache = np.array(c["cache_before"], np.float32).reshape(c["B"], c["Nkv"], c["Smax"], c["Hd"])
    oracle.kv_cache_write(src, "f32", cache, "f32", c["offset"])
    assert cache.ravel().tolist() == c["expected"]


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_kv_cache_write_bit_exact_16bit(dt):
    rng = np.random.default_rng(1)
    src = oracle.to_dtype(rng.standard_normal((2, 3, 5, 24)), dt)
    cache = np.zeros((2, 3, 9, 24), oracle.NP[dt])
    oracle.kv_cache_write(src, dt, cache, dt, 3)
    assert np.array_equal(cache[:, :, 3:8].view(np.uint16), src.view(np.uint16))
    assert not cache[:, :, :3].any() and not cache[:, :, 8:].any()


def test_kv_cache_write_f32_to_bf16_rne():
    x = np.array([1.0, 1.00390625, 1.01171875, -3.3e38, 3.4e38], np.float32).reshape(1, 1, 1, 5)
    cache = np.zeros((1, 1, 1, 5), np.uint16)
    oracle.kv_cache_write(x, "f32", cache, "bf16", 0)
    # RNE with no NaN special case (PopcornDTypes.h:29-34): ties to even.
    assert cache.ravel()[:3].tolist() == [0x3F80, 0x3F80, 0x3F82]


def test_rmsnorm_kats(kats):
    c = kats["rmsnorm_gemma_style"]
    x = np.array(c["x"], np.float32)
    out = oracle.rmsnorm(x, "f32", np.array(c["weight"], np.float32), eps=c["eps"], add_one=True)
    assert approx_equal(out, x / np.sqrt(np.float32(7.5)), c["eps_cmp"]).all()
    c = kats["rmsnorm_no_weight"]
    x = np.array(c["x"], np.float32).reshape(c["shape"])
    out = oracle.rmsnorm(x, "f32", None, eps=c["eps"])
    assert approx_equal(out, x / np.sqrt(np.float32(12.5)), c["eps_cmp"]).all()


@pytest.mark.parametrize("name", ["matmul_plain", "matmul_routes_vector_transposed_weights",
                                  "matmul_transposed_b"])
def test_matmul_kats(kats, name):
    c = kats[name]
    a = np.array(c["a"], np.float32).reshape(c["a_shape"])
    b = np.array(c["b"], np.float32).reshape(c["b_shape"])
    if a.shape[0] == 1 and c["transpose_b"]:
        out = oracle.matvec_nk(a[0], "f32", b, "f32", "f32")
    else:
        out = oracle.matmul(a, "f32", b, "f32", "f32", c["transpose_b"])
    assert out.ravel().tolist() == c["expected"]


def test_matmul_random_shapes(kats):
    rng = np.random.default_rng(7)
    for case in kats["matmul_random_shapes"]["cases"]:
        m, k, n, tb = case["m"], case["k"], case["n"], case["transpose_b"]
        a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        b = rng.uniform(-1, 1, (n, k) if tb else (k, n)).astype(np.float32)
        exp = a.astype(np.float64) @ (b.T if tb else b).astype(np.float64)
        if m == 1 and tb:
            got = oracle.matvec_nk(a[0], "f32", b, "f32", "f32")[None]
        else:
            got = oracle.matmul(a, "f32", b, "f32", "f32", tb)
        assert approx_equal(got, exp, 1e-3).all(), case["name"]


def test_gelu_mul_add_kats(kats):
    c = kats["gelu_tanh"]
    out = oracle.gelu_tanh(np.array(c["x"], np.float32), "f32")
    assert approx_equal(out, c["expected"], c["eps_cmp"]).all()
    c = kats["mul"]
    out = oracle.mul(np.array(c["a"], np.float32), np.array(c["b"], np.float32), "f32")
    assert out.tolist() == c["expected"]
    c = kats["add"]
    out = oracle.add(np.array(c["a"], np.float32), np.array(c["b"], np.float32), "f32")
    assert out.tolist() == c["expected"]


def test_gqa_head_mapping(kats):
    """KernelsTests.swift:510-547: both query heads read the single KV head."""
    c = kats["attention_gqa_mapping"]
    q = np.array(c["q"], np.float32).reshape(1, 2, 1, 2)
    k = np.array(c["k"], np.float32).reshape(1, 1, 2, 2)
    v = np.array(c["v"], np.float32).reshape(1, 1, 2, 2)
    # scale large enough that softmax is one-hot: the same peaked result
    # as the reference's AttentionOutput with one-hot scores.
    out = oracle.flash_decoding(q, "f32", k, v, "f32", "f32", scale=200.0)
    assert np.allclose(out.ravel(), c["output_with_onehot_probs_expected"], atol=1e-6)
    exact = oracle.attention_exact(q, "f32", k, v, "f32", scale=1.0)
    fd = oracle.flash_decoding(q, "f32", k, v, "f32", "f32", scale=1.0)
    assert approx_equal(fd, exact, 1e-5).all()


def test_bidirectional_fa_fixture(kats):
    """BidirectionalFATests.swift:90-150 against the committed fixture."""
    c = kats["bidirectional_fa"]
    q, k, v = make_golden.inputs()
    exp = np.load(os.path.join(os.path.dirname(make_golden.__file__), c["expected_file"]))
    scale = 1.0 / np.sqrt(64.0)
    got = oracle.flash_attention(q, "f32", k, v, "f32", "f32", scale, mask="bidirectional")
    assert np.abs(got - exp).max() < c["max_abs_delta"]
    ex = oracle.attention_exact(q, "f32", k, v, "f32", scale, mask="bidirectional")
    assert np.abs(ex - exp).max() < 1e-6
    causal = oracle.flash_attention(q, "f32", k, v, "f32", "f32", scale, mask="causal")
    assert not np.isnan(causal).any()
    # FlashDecoding pinned on the same fixture: the last query row attends to
    # all 96 keys under the causal mask, i.e. row 95 of the bidirectional output.
    fd = oracle.flash_decoding(q[:, :, 95:96], "f32", k, v, "f32", "f32", scale)
    assert np.abs(fd[:, :, 0] - exp[:, :, 95]).max() < c["max_abs_delta"]


def test_golden_fixture_regenerates():
    q, k, v = make_golden.inputs()
    exp = make_golden.reference_bidirectional_attention(q, k, v)
    saved = np.load(os.path.join(os.path.dirname(make_golden.__file__), "bidirectional_fa_expected.npy"))
    assert np.array_equal(exp, saved)


@pytest.mark.parametrize("mask,window", [("causal", -1), ("sliding", 40), ("bidirectional", -1)])
@pytest.mark.parametrize("dt", ["f32", "bf16", "f16"])
def test_flash_decoding_vs_exact(mask, window, dt):
    rng = np.random.default_rng(3)
    B, Nq, Nkv, S, Hd = 2, 8, 2, 300, 64
    q = oracle.to_dtype(rng.standard_normal((B, Nq, 1, Hd)), dt)
    k = oracle.to_dtype(rng.standard_normal((B, Nkv, S, Hd)), dt)
    v = oracle.to_dtype(rng.standard_normal((B, Nkv, S, Hd)), dt)
    got = oracle.flash_decoding(q, dt, k, v, dt, "f32", 0.125, mask=mask, window=window)
    ex = oracle.attention_exact(q, dt, k, v, dt, 0.125, mask=mask, window=window)
    assert np.abs(got - ex).max() < 1e-4


def test_flash_decoding_ragged_equals_per_sequence():
    """The ragged extension equals the reference run on each compact slice."""
    rng = np.random.default_rng(4)
    B, Nq, Nkv, S, Hd = 3, 4, 2, 200, 32
    q = rng.standard_normal((B, Nq, 1, Hd)).astype(np.float32)
    k = rng.standard_normal((B, Nkv, S, Hd)).astype(np.float32)
    v = rng.standard_normal((B, Nkv, S, Hd)).astype(np.float32)
    lens = np.array([200, 1, 77], np.int32)
    got = oracle.flash_decoding(q, "f32", k, v, "f32", "f32", 0.2, seq_lens=lens)
    for b in range(B):
        L = lens[b]
        ref = oracle.flash_decoding(q[b:b + 1], "f32", np.ascontiguousarray(k[b:b + 1, :, :L]),
                                    np.ascontiguousarray(v[b:b + 1, :, :L]), "f32", "f32", 0.2)
        assert np.array_equal(got[b:b + 1], ref)


def test_flash_decoding_partials_layout():
    """Empty partitions (past posQ) write m=-inf, l=0, O=0 (FlashDecoding.metal:78-87)."""
    q = np.ones((1, 1, 1, 4), np.float32)
    k = np.ones((1, 1, 3, 4), np.float32)
    v = np.ones((1, 1, 3, 4), np.float32)
    out, (pO, pM, pL) = oracle.flash_decoding(q, "f32", k, v, "f32", "f32", 1.0, return_partials=True)
    # per = ceil(3/8) = 1: partitions 0..2 hold one key each, 3..7 are empty.
    assert np.all(pL[0, 0, :3] == 1.0) and np.all(pL[0, 0, 3:] == 0.0)
    assert np.all(np.isneginf(pM[0, 0, 3:]))
    assert np.allclose(out, 1.0)


def test_argmax_kat(kats):
    k = kats["argmax"]
    x = np.array(k["x"], np.float32).reshape(k["shape"])
    assert oracle.argmax(x, "f32").tolist() == k["expected"]


def test_argmax_rules():
    """Argmax.metal:7-76: ties -> lowest index; NaN never wins; n >= 32 starts
    from (-inf, 0x7fffffff), n < 32 from element 0."""
    x = np.zeros((4, 40), np.float32)
    x[0, [3, 17, 30]] = 5.0                      # tie: lowest index
    x[1] = np.nan
    x[1, 22] = -np.inf                           # only non-NaN value
    x[2] = np.nan                                # nothing wins
    x[3] = -np.inf                               # all -inf: lowest index
    assert oracle.argmax(x, "f32").tolist() == [3, 22, 0x7fffffff, 0]
    y = np.array([[np.nan, 1.0, 2.0]], np.float32)  # n < 32: element 0 (NaN) is never beaten
    assert oracle.argmax(y, "f32").tolist() == [0]


def _rope_kat_expected(k):
    """The reference test's expected values (KernelsTests.swift:457-489)."""
    x = np.array(k["x"], np.float64).reshape(2, 4)
    pos = np.array(k["positions"], np.float64)
    inv = np.array(k["inv_freq"], np.float64)
    ang = pos[:, None] * inv[None, :]
    c, s = np.cos(ang), np.sin(ang)
    x1, x2 = x[:, :2], x[:, 2:]
    return c, s, np.concatenate([x1 * c - x2 * s, x1 * s + x2 * c], axis=1)


def test_rope_kat(kats):
    k = kats["rope"]
    ec, es, eout = _rope_kat_expected(k)
    c, s = oracle.rope_build(k["positions"], k["inv_freq"])
    assert approx_equal(c, ec).all() and approx_equal(s, es).all()
    x = np.array(k["x"], np.float32).reshape(k["x_shape"])
    out = oracle.rope_apply(x, "f32", c, s, "f32")
    assert approx_equal(out.reshape(2, 4), eout).all()
    assert np.array_equal(out[0, 0, 0], x[0, 0, 0])  # t = 0: unchanged


def test_rope_dtype_combinations():
    """RopeApply.swift:19-31 routes f32/f32, bf16/bf16 and bf16 x with f32
    tables; every combination agrees with a float64 rotation within the
    storage rounding."""
    rng = np.random.default_rng(3)
    T, Hd = 5, 16
    x = rng.standard_normal((2, T, 3, Hd)).astype(np.float32)
    inv = (10000.0 ** (-np.arange(Hd // 2) * 2.0 / Hd)).astype(np.float32)
    c, s = oracle.rope_build(np.arange(7, 7 + T), inv, scaling=0.5)
    xd = x.astype(np.float64)
    cd, sd = c.astype(np.float64)[None, :, None, :], s.astype(np.float64)[None, :, None, :]
    x1, x2 = xd[..., :Hd // 2], xd[..., Hd // 2:]
    exact = np.concatenate([x1 * cd - x2 * sd, x1 * sd + x2 * cd], axis=-1)
    for xdt, tdt, tol in [("f32", "f32", 1e-5), ("bf16", "bf16", 3e-2), ("bf16", "f32", 2e-2)]:
        out = oracle.to_f32(oracle.rope_apply(oracle.to_dtype(x, xdt), xdt, oracle.to_dtype(c, tdt),
                                              oracle.to_dtype(s, tdt), tdt), xdt)
        assert np.allclose(out, exact, rtol=tol, atol=tol), (xdt, tdt)


def test_aq_format_roundtrip():
    """4-bit little-endian packing (AffineQuantizationFormat.swift:22-29):
    value i sits in bits 4(i % 8) .. of word i / 8; dequantisation is
    q * scale + bias per group of 64 (AffineQuantizedTensor.swift:5-18)."""
    rng = np.random.default_rng(0)
    w = rng.standard_normal((3, 128)).astype(np.float32)
    packed, sc, bi = oracle.aq_quantize(w, sdt="f32")
    assert packed.shape == (3, 16) and sc.shape == (3, 2)
    q0 = packed[1, 5] >> np.uint32(4 * 3) & np.uint32(15)  # value 43 of row 1
    assert np.isclose(q0 * sc[1, 0] + bi[1, 0], oracle.aq_dequantize(packed, sc, bi, "f32", 128)[1, 43])
    deq = oracle.aq_dequantize(packed, sc, bi, "f32", 128)
    assert np.abs(deq - w).max() <= sc.max() / 2 + 1e-6


@pytest.mark.parametrize("M", [1, 3])
@pytest.mark.parametrize("bias", [True, False])
def test_aq_matmul_routes(M, bias):
    """m == 1 (aq_qmv_fast arithmetic) and m > 1 (aq_matvec_simd4
    arithmetic) both equal the float64 dequantised product within fp32
    accumulation error."""
    rng = np.random.default_rng(M)
    K, N = 640, 24
    w = rng.standard_normal((N, K)).astype(np.float32) * 0.05
    if not bias:
        w = np.abs(w)
    packed, sc, bi = oracle.aq_quantize(w, sdt="bf16", bias=bias)
    x = oracle.to_dtype(rng.standard_normal((M, K)), "bf16")
    got = oracle.aq_matmul(x, "bf16", packed, sc, bi, "bf16", "f32")
    exact = oracle.aq_matmul_exact(x, "bf16", packed, sc, bi, "bf16")
    assert np.allclose(got, exact, rtol=1e-4, atol=1e-4)


def test_embedding_gather():
    rng = np.random.default_rng(1)
    table = oracle.to_dtype(rng.standard_normal((50, 128)), "bf16")
    ids = np.array([3, 0, 49, 3], np.int32)
    assert np.array_equal(oracle.embedding_gather(ids, table, "bf16"), table[ids])
    packed, sc, bi = oracle.aq_quantize(oracle.to_f32(table, "bf16"), sdt="bf16")
    deq = oracle.aq_dequantize(packed, sc, bi, "bf16", 128)
    got = oracle.aq_embedding_gather(ids, packed, sc, bi, "bf16", "f32", 128)
    assert np.array_equal(got, deq[ids])


def test_embedding_gather_kat(kats):
    k = kats["embedding_gather"]
    table = np.array(k["table"], np.float32).reshape(k["shape"])
    assert oracle.embedding_gather(k["ids"], table, "f32").ravel().tolist() == k["expected"]


def test_attention_mask_kat(kats):
    """KernelsTests.swift:407-434 (causal, and a window of 2)."""
    k = kats["attention_mask"]
    c = k["causal"]
    m = oracle.attention_mask(c["Sq"], c["Sk"], c["window"])
    assert ((m == 0) == np.array(c["allowed"], bool)).all() and np.isinf(m[m != 0]).all()
    s = k["sliding"]
    m = oracle.attention_mask(s["Sq"], s["Sk"], s["window"])
    for r, row in enumerate(s["allowed_rows_0_to_2"]):
        for j, a in enumerate(row):
            if a is not None:
                assert (m[r, j] == 0) == bool(a), (r, j)
