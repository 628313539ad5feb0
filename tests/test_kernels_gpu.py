"""Parity of the CUDA kernels (through the C ABI) with the CPU oracle and the
reference's own known-answer tests. Every test here needs a B200."""
import os

import numpy as np
import pytest

import oracle
from tests.conftest import approx_equal
from tests.golden import make_golden
from tests.gpu_util import (assert_close, dot_tolerance, empty_dev, f32, from_dev, gated_candidates, rand,
                            residual_candidates, to_dev)

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def pc():
    import popcorn_b200
    return popcorn_b200


@pytest.fixture(scope="module")
def lib(pc):
    return pc.KernelLibrary(0)


@pytest.fixture()
def enc(pc, lib):
    return pc.KernelCommandEncoder(lib, scratch=pc.ScratchPool())


def run(enc, *kernels):
    enc.encode(*kernels)
    torch.cuda.synchronize()


# ---------------------------------------------------------------------------
# the reference's known-answer tests, through the CUDA path
# ---------------------------------------------------------------------------

def test_kat_kv_cache_write(pc, enc, kats):
    c = kats["kv_cache_write"]
    src = torch.tensor(c["src"], dtype=torch.float32, device="cuda").reshape(1, 1, 2, 2)
    cache = torch.zeros(1, 1, 4, 2, dtype=torch.float32, device="cuda")
    run(enc, pc.Kernels.KVCacheWrite(src, cache, offset=1, dims=(1, 1, 2, 4, 2)))
    assert cache.flatten().tolist() == c["expected"]
    cache.zero_()
    run(enc, pc.Kernels.KVCacheWrite(src, cache, offset=1))
    assert cache.flatten().tolist() == c["expected"]


def test_kat_rmsnorm(pc, enc, kats):
    c = kats["rmsnorm_gemma_style"]
    x = torch.tensor(c["x"], dtype=torch.float32, device="cuda")
    w = torch.tensor(c["weight"], dtype=torch.float32, device="cuda")
    out = torch.empty_like(x)
    run(enc, pc.Kernels.RMSNorm(x, w, into=out, dims=(1, 4), eps=c["eps"], add_one_to_weight=True))
    assert approx_equal(out.cpu().numpy(), np.array(c["x"]) / np.sqrt(7.5), c["eps_cmp"]).all()
    c = kats["rmsnorm_no_weight"]
    x = torch.tensor(c["x"], dtype=torch.float32, device="cuda").reshape(1, 2)
    out = torch.empty_like(x)
    run(enc, pc.Kernels.RMSNorm(x, into=out, eps=0.0))
    assert approx_equal(out.cpu().numpy().ravel(), np.array(c["x"]) / np.sqrt(12.5), c["eps_cmp"]).all()


@pytest.mark.parametrize("name", ["matmul_plain", "matmul_routes_vector_transposed_weights", "matmul_transposed_b"])
def test_kat_matmul(pc, enc, kats, name):
    c = kats[name]
    a = torch.tensor(c["a"], dtype=torch.float32, device="cuda").reshape(c["a_shape"])
    b = torch.tensor(c["b"], dtype=torch.float32, device="cuda").reshape(c["b_shape"])
    m = c["a_shape"][0]
    n = c["b_shape"][0] if c["transpose_b"] else c["b_shape"][1]
    out = torch.empty(m, n, dtype=torch.float32, device="cuda")
    run(enc, pc.Kernels.Matmul(a, b, into=out, transpose_b=c["transpose_b"]))
    assert out.flatten().tolist() == c["expected"]


def test_kat_matmul_random_shapes(pc, enc, kats):
    rng = np.random.default_rng(11)
    for case in kats["matmul_random_shapes"]["cases"]:
        m, k, n, tb = case["m"], case["k"], case["n"], case["transpose_b"]
        a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        b = rng.uniform(-1, 1, (n, k) if tb else (k, n)).astype(np.float32)
        out = torch.empty(m, n, dtype=torch.float32, device="cuda")
        run(enc, pc.Kernels.Matmul(to_dev(a, "f32"), to_dev(b, "f32"), into=out, transpose_b=tb, dims=(m, k, n)))
        exp = a.astype(np.float64) @ (b.T if tb else b).astype(np.float64)
        assert approx_equal(out.cpu().numpy(), exp, kats["matmul_random_shapes"]["eps_cmp"]).all(), case["name"]


def test_kat_gelu_mul_add(pc, enc, kats):
    c = kats["gelu_tanh"]
    x = torch.tensor(c["x"], dtype=torch.float32, device="cuda")
    out = torch.empty_like(x)
    run(enc, pc.Kernels.GeluTanh(x, into=out))
    assert approx_equal(out.cpu().numpy(), c["expected"], c["eps_cmp"]).all()
    c = kats["mul"]
    a = torch.tensor(c["a"], dtype=torch.float32, device="cuda")
    b = torch.tensor(c["b"], dtype=torch.float32, device="cuda")
    out = torch.empty_like(a)
    run(enc, pc.Kernels.Mul(a, b, into=out))
    assert out.tolist() == c["expected"]
    c = kats["add"]
    a = torch.tensor(c["a"], dtype=torch.float32, device="cuda")
    b = torch.tensor(c["b"], dtype=torch.float32, device="cuda")
    out = torch.empty_like(a)
    run(enc, pc.Kernels.Add(a, b, into=out))
    assert out.tolist() == c["expected"]


def test_kat_gqa_mapping(pc, enc, kats):
    c = kats["attention_gqa_mapping"]
    q = torch.tensor(c["q"], dtype=torch.float32, device="cuda").reshape(1, 2, 1, 2)
    k = torch.tensor(c["k"], dtype=torch.float32, device="cuda").reshape(1, 1, 2, 2)
    v = torch.tensor(c["v"], dtype=torch.float32, device="cuda").reshape(1, 1, 2, 2)
    out = torch.empty(1, 2, 1, 2, dtype=torch.float32, device="cuda")
    run(enc, pc.Kernels.FlashAttention(q, k, v, into=out, scale=200.0))
    assert np.allclose(out.flatten().cpu().numpy(), c["output_with_onehot_probs_expected"], atol=1e-6)


def test_kat_bidirectional_fa_fixture(pc, enc, kats):
    c = kats["bidirectional_fa"]
    q, k, v = make_golden.inputs()
    exp = np.load(os.path.join(os.path.dirname(make_golden.__file__), c["expected_file"]))
    scale = 1.0 / 8.0
    qd, kd, vd = to_dev(q, "f32"), to_dev(k, "f32"), to_dev(v, "f32")
    out = torch.empty_like(qd)
    run(enc, pc.Kernels.FlashAttention(qd, kd, vd, into=out, scale=scale, mask=pc.AttentionMask.bidirectional))
    got = out.cpu().numpy()
    assert not np.isnan(got).any()
    assert np.abs(got - exp).max() < c["max_abs_delta"]
    run(enc, pc.Kernels.FlashAttention(qd, kd, vd, into=out, scale=scale, mask=pc.AttentionMask.causal))
    assert not torch.isnan(out).any()
    # Decode path on the same fixture: the last row attends to all keys.
    qd1 = qd[:, :, 95:96].contiguous()
    o1 = torch.empty_like(qd1)
    run(enc, pc.Kernels.FlashAttention(qd1, kd, vd, into=o1, scale=scale))
    assert np.abs(o1.cpu().numpy()[:, :, 0] - exp[:, :, 95]).max() < c["max_abs_delta"]


# ---------------------------------------------------------------------------
# FlashDecoding parity
# ---------------------------------------------------------------------------

def _fd_case(pc, enc, B, Nq, Nkv, S, Hd, dt, odt, scale, mask="causal", window=-1, seed=0, kv_scale=1.0):
    rng = np.random.default_rng(seed)
    q = rand(rng, (B, Nq, 1, Hd), dt)
    k = rand(rng, (B, Nkv, S, Hd), dt, kv_scale)
    v = rand(rng, (B, Nkv, S, Hd), dt)
    exp = oracle.flash_decoding(q, dt, k, v, dt, odt, scale, mask=mask, window=window)
    pre = oracle.flash_decoding(q, dt, k, v, dt, "f32", scale, mask=mask, window=window)
    out = empty_dev((B, Nq, 1, Hd), odt)
    m = {"causal": pc.AttentionMask.causal, "bidirectional": pc.AttentionMask.bidirectional}.get(mask)
    if m is None:
        m = pc.AttentionMask.causal_sliding_window(window)
    kern = pc.Kernels.FlashAttention(to_dev(q, dt), to_dev(k, dt), to_dev(v, dt), into=out, scale=scale, mask=m)
    run(enc, kern)
    assert_close(from_dev(out, odt), exp, odt, what="FD B%d %d/%d S%d Hd%d %s->%s" % (B, Nq, Nkv, S, Hd, dt, odt),
                 pre=pre)
    return kern


def test_fd_config1_f16(pc, enc):
    """B1, 8Q/4KV, hd 256, ctx 1024, f16, scale 1/16."""
    k = _fd_case(pc, enc, 1, 8, 4, 1024, 256, "f16", "f16", 1.0 / 16, seed=1234)
    assert k.function_names[0] == "flash_decoding_partial_f16"


@pytest.mark.parametrize("dt,odt", [("bf16", "bf16"), ("bf16", "f32"), ("f32", "f32"), ("f16", "f32")])
@pytest.mark.parametrize("Hd", [64, 128, 256, 512])
def test_fd_dtypes_headdims(pc, enc, dt, odt, Hd):
    _fd_case(pc, enc, 2, 8, 2, 333, Hd, dt, odt, 1.0 / np.sqrt(Hd), seed=Hd)


@pytest.mark.parametrize("S", [1, 2, 31, 32, 33, 100, 4096])
def test_fd_lengths(pc, enc, S):
    _fd_case(pc, enc, 1, 16, 8, S, 256, "bf16", "bf16", 1.0 / 16, seed=S)


@pytest.mark.parametrize("Nq,Nkv", [(4, 4), (8, 1), (6, 2), (12, 4), (32, 4), (16, 8)])
def test_fd_gqa_groups(pc, enc, Nq, Nkv):
    _fd_case(pc, enc, 2, Nq, Nkv, 257, 128, "f16", "f16", 0.1, seed=Nq * 10 + Nkv)


@pytest.mark.parametrize("Hd", [40, 80, 96, 200])
def test_fd_generic_headdims(pc, enc, Hd):
    _fd_case(pc, enc, 2, 4, 2, 150, Hd, "bf16", "f32", 0.2, seed=Hd)


@pytest.mark.parametrize("mask,window", [("bidirectional", -1), ("sliding", 1), ("sliding", 100), ("sliding", 5000)])
def test_fd_masks(pc, enc, mask, window):
    _fd_case(pc, enc, 2, 8, 4, 1000, 256, "bf16", "f32", 1.0 / 16, mask=mask, window=window, seed=window + 7)


def test_fd_large_scores(pc, enc):
    """Peaked softmax (large logits) stays finite and matches."""
    _fd_case(pc, enc, 1, 8, 4, 2048, 256, "f16", "f32", 1.0, seed=5, kv_scale=4.0)


def test_fd_q_dtype_mismatch_rejected(pc):
    q = torch.zeros(1, 2, 1, 64, dtype=torch.float32, device="cuda")
    k = torch.zeros(1, 1, 8, 64, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(1, 2, 1, 64, dtype=torch.float32, device="cuda")
    with pytest.raises(pc.PopcornError) as e:
        pc.Kernels.FlashAttention(q, k, k, into=out, scale=1.0)
    assert e.value.code == pc.PopcornError.unsupportedDataTypeCombination


@pytest.mark.parametrize("B,ctx", [(1, 1024), (8, 4096), (4, 16384)])
def test_fd_ragged_sweep_shapes(pc, enc, B, ctx):
    """BASELINE config 3 shapes (16Q/8KV, hd 256, bf16) with ragged lengths
    U[ctx/2, ctx], checked against the oracle run per sequence."""
    rng = np.random.default_rng(B * 100003 + ctx)
    Nq, Nkv, Hd = 16, 8, 256
    lens = rng.integers(ctx // 2, ctx + 1, size=B).astype(np.int32)
    q = rand(rng, (B, Nq, 1, Hd), "bf16")
    k = rand(rng, (B, Nkv, ctx, Hd), "bf16")
    v = rand(rng, (B, Nkv, ctx, Hd), "bf16")
    exp = oracle.flash_decoding(q, "bf16", k, v, "bf16", "bf16", 1.0 / 16, seq_lens=lens)
    pre = oracle.flash_decoding(q, "bf16", k, v, "bf16", "f32", 1.0 / 16, seq_lens=lens)
    out = empty_dev((B, Nq, 1, Hd), "bf16")
    run(enc, pc.Kernels.FlashDecodingRagged(to_dev(q, "bf16"), to_dev(k, "bf16"), to_dev(v, "bf16"),
                                            to_dev(lens, "i32"), into=out, scale=1.0 / 16))
    assert_close(from_dev(out, "bf16"), exp, "bf16", what="ragged B%d ctx%d" % (B, ctx), pre=pre)


@pytest.mark.parametrize("B,ctx", [(32, 32768), (64, 16384)])
def test_fd_ragged_sweep_large(pc, enc, B, ctx):
    """The largest BASELINE config-3 points (16 Q / 8 KV heads, hd 256, bf16,
    ragged lengths U[ctx/2, ctx]), where the ragged split planner does its
    real work: the whole batch on the GPU (8.6 GB of K/V, generated there),
    four sampled sequences against the oracle run per sequence."""
    Nq, Nkv, Hd = 16, 8, 256
    gen = torch.Generator(device="cuda").manual_seed(B + ctx)
    lens = np.random.default_rng(B * 7 + ctx).integers(ctx // 2, ctx + 1, size=B).astype(np.int32)
    q = torch.randn(B, Nq, 1, Hd, device="cuda", generator=gen).to(torch.bfloat16)
    k = torch.randn(B, Nkv, ctx, Hd, device="cuda", generator=gen).to(torch.bfloat16)
    v = torch.randn(B, Nkv, ctx, Hd, device="cuda", generator=gen).to(torch.bfloat16)
    out = empty_dev((B, Nq, 1, Hd), "bf16")
    run(enc, pc.Kernels.FlashDecodingRagged(q, k, v, to_dev(lens, "i32"), into=out, scale=1.0 / 16))
    got = from_dev(out, "bf16")
    for b in (0, 1, B // 2, B - 1):
        L = int(lens[b])
        qs = from_dev(q[b:b + 1].contiguous(), "bf16")
        ks = from_dev(k[b:b + 1, :, :L].contiguous(), "bf16")
        vs = from_dev(v[b:b + 1, :, :L].contiguous(), "bf16")
        exp = oracle.flash_decoding(qs, "bf16", ks, vs, "bf16", "bf16", 1.0 / 16)
        pre = oracle.flash_decoding(qs, "bf16", ks, vs, "bf16", "f32", 1.0 / 16)
        assert_close(got[b:b + 1], exp, "bf16", what="ragged B%d ctx%d seq %d (len %d)" % (B, ctx, b, L), pre=pre)
    del k, v
    torch.cuda.empty_cache()


def test_fd_ragged_edges(pc, enc):
    """Lengths 0 (zeros out), 1 and Smax in one batch."""
    rng = np.random.default_rng(9)
    B, Nq, Nkv, S, Hd = 4, 4, 2, 300, 128
    lens = np.array([0, 1, 300, 77], np.int32)
    q = rand(rng, (B, Nq, 1, Hd), "f16")
    k = rand(rng, (B, Nkv, S, Hd), "f16")
    v = rand(rng, (B, Nkv, S, Hd), "f16")
    out = empty_dev((B, Nq, 1, Hd), "f32")
    run(enc, pc.Kernels.FlashDecodingRagged(to_dev(q, "f16"), to_dev(k, "f16"), to_dev(v, "f16"),
                                            to_dev(lens, "i32"), into=out, scale=0.1))
    got = from_dev(out, "f32")
    assert np.all(got[0] == 0)
    for b in range(1, B):
        L = int(lens[b])
        ref = oracle.flash_decoding(q[b:b + 1], "f16", np.ascontiguousarray(k[b:b + 1, :, :L]),
                                    np.ascontiguousarray(v[b:b + 1, :, :L]), "f16", "f32", 0.1)
        assert_close(got[b:b + 1], ref, "f32", what="ragged b%d" % b)


def test_fd_ragged_lengths_clamped(pc, enc):
    """seq_lens outside [0, Smax] (Smax = 1000, not a multiple of the 32-key
    tile) are clamped on the device: a length past the cache reads no row
    beyond it and equals length Smax; a negative length equals 0."""
    rng = np.random.default_rng(21)
    B, Nq, Nkv, S, Hd = 3, 8, 4, 1000, 256
    lens = np.array([S + 4000, S, -5], np.int32)
    q = rand(rng, (B, Nq, 1, Hd), "bf16")
    k = rand(rng, (B, Nkv, S, Hd), "bf16")
    v = rand(rng, (B, Nkv, S, Hd), "bf16")
    out = empty_dev((B, Nq, 1, Hd), "f32")
    run(enc, pc.Kernels.FlashDecodingRagged(to_dev(q, "bf16"), to_dev(k, "bf16"), to_dev(v, "bf16"),
                                            to_dev(lens, "i32"), into=out, scale=1.0 / 16))
    got = from_dev(out, "f32")
    exp = oracle.flash_decoding(q[:2], "bf16", k[:2], v[:2], "bf16", "f32", 1.0 / 16)
    assert_close(got[:2], exp, "f32", what="clamped lengths")
    assert np.all(got[2] == 0)


# ---------------------------------------------------------------------------
# KV write, RMSNorm, matvec, elementwise
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("sdt,cdt", [("f32", "f32"), ("bf16", "bf16"), ("f32", "bf16"), ("f16", "f16")])
@pytest.mark.parametrize("Hd", [256, 6])
def test_kv_cache_write_bit_exact(pc, enc, sdt, cdt, Hd):
    rng = np.random.default_rng(3)
    B, Nkv, Snew, Smax, off = 2, 3, 5, 17, 9
    src = rand(rng, (B, Nkv, Snew, Hd), sdt)
    cache = rand(rng, (B, Nkv, Smax, Hd), cdt)
    exp = cache.copy()
    oracle.kv_cache_write(src, sdt, exp, cdt, off)
    cd = to_dev(cache, cdt)
    run(enc, pc.Kernels.KVCacheWrite(to_dev(src, sdt), cd, offset=off))
    got = from_dev(cd, cdt)
    assert np.array_equal(got.view(np.uint8), exp.view(np.uint8))


def test_kv_cache_write_range_error(pc):
    src = torch.zeros(1, 1, 2, 4, device="cuda")
    cache = torch.zeros(1, 1, 4, 4, device="cuda")
    with pytest.raises(pc.PopcornError) as e:
        pc.Kernels.KVCacheWrite(src, cache, offset=3)
    assert e.value.code == pc.PopcornError.tensorShapeMismatch


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("rows,H", [(1, 2304), (3, 3584), (5, 17), (2, 9216)])
@pytest.mark.parametrize("weight,add_one", [(True, True), (True, False), (False, False)])
def test_rmsnorm(pc, enc, dt, rows, H, weight, add_one):
    rng = np.random.default_rng(rows * H)
    x = rand(rng, (rows, H), dt)
    w = (rng.standard_normal(H) * 0.1).astype(np.float32) if weight else None
    exp = oracle.rmsnorm(x, dt, w, eps=1e-6, add_one=add_one)
    pre = oracle.rmsnorm(x, dt, w, odt="f32", eps=1e-6, add_one=add_one)
    out = empty_dev((rows, H), dt)
    run(enc, pc.Kernels.RMSNorm(to_dev(x, dt), None if w is None else to_dev(w, "f32"), into=out, eps=1e-6,
                                add_one_to_weight=add_one))
    assert_close(from_dev(out, dt), exp, dt, what="rmsnorm", pre=pre)


@pytest.mark.parametrize("xdt,wdt,odt", [("f32", "f32", "f32"), ("f32", "bf16", "f32"), ("bf16", "bf16", "f32"),
                                         ("bf16", "bf16", "bf16"), ("f16", "f16", "f16"), ("f16", "f16", "f32"),
                                         ("f32", "f16", "f32")])
@pytest.mark.parametrize("K,N", [(2304, 4096), (9216, 2304), (131, 64), (256, 67), (2048, 2304), (8, 1)])
def test_matvec(pc, enc, xdt, wdt, odt, K, N):
    rng = np.random.default_rng(K + N)
    x = rand(rng, (1, K), xdt)
    w = rand(rng, (N, K), wdt, 0.02)
    exp = oracle.matvec_nk(x[0], xdt, w, wdt, odt)
    pre = oracle.matvec_nk(x[0], xdt, w, wdt, "f32")
    out = empty_dev((1, N), odt)
    kern = pc.Kernels.Matmul(to_dev(x, xdt), to_dev(w, wdt), into=out, transpose_b=True)
    assert kern.function_names[0].startswith("matvec_nk_")
    run(enc, kern)
    assert_close(from_dev(out, odt)[0], exp, odt, what="matvec %s.%s.%s K%d N%d" % (xdt, wdt, odt, K, N), pre=pre)


@pytest.mark.parametrize("adt,bdt,cdt", [("f32", "f32", "f32"), ("bf16", "bf16", "bf16"), ("f16", "f16", "f32"),
                                         ("f32", "bf16", "f32")])
@pytest.mark.parametrize("M,K,N,tb", [(70, 33, 50, False), (64, 64, 64, True), (3, 300, 130, True),
                                      (1, 64, 40, False)])
def test_matmul_general(pc, enc, adt, bdt, cdt, M, K, N, tb):
    rng = np.random.default_rng(M * K + N)
    a = rand(rng, (M, K), adt)
    b = rand(rng, (N, K) if tb else (K, N), bdt)
    exp = oracle.matmul(a, adt, b, bdt, cdt, tb)
    pre = oracle.matmul(a, adt, b, bdt, "f32", tb)
    out = empty_dev((M, N), cdt)
    run(enc, pc.Kernels.Matmul(to_dev(a, adt), to_dev(b, bdt), into=out, transpose_b=tb))
    assert_close(from_dev(out, cdt), exp, cdt, what="matmul", pre=pre)


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
def test_elementwise(pc, enc, dt):
    rng = np.random.default_rng(2)
    n = 9219
    a = rand(rng, (n,), dt, 3.0)
    b = rand(rng, (n,), dt)
    ad, bd = to_dev(a, dt), to_dev(b, dt)
    out = empty_dev((n,), dt)
    run(enc, pc.Kernels.GeluTanh(ad, into=out))
    assert_close(from_dev(out, dt), oracle.gelu_tanh(a, dt), dt, what="gelu", pre=oracle.gelu_tanh(a, dt, "f32"))
    run(enc, pc.Kernels.SiLU(ad, into=out))
    assert_close(from_dev(out, dt), oracle.silu(a, dt), dt, what="silu", pre=oracle.silu(a, dt, "f32"))
    run(enc, pc.Kernels.Mul(ad, bd, into=out))
    assert np.array_equal(from_dev(out, dt).view(np.uint8), oracle.mul(a, b, dt).view(np.uint8))
    run(enc, pc.Kernels.Add(ad, bd, into=out))
    assert np.array_equal(from_dev(out, dt).view(np.uint8), oracle.add(a, b, dt).view(np.uint8))


# ---------------------------------------------------------------------------
# fused decode ops == the reference op sequences
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_rmsnorm_matmul(pc, enc, dt):
    rng = np.random.default_rng(21)
    K, N = 2304, 4096
    x = rand(rng, (1, K), dt)
    nw = (rng.standard_normal(K) * 0.1).astype(np.float32)
    w = rand(rng, (N, K), dt, 0.02)
    xn = oracle.rmsnorm(x, dt, nw, eps=1e-6, add_one=True)
    exp = oracle.matvec_nk(xn[0], dt, w, dt, dt)
    pre = oracle.matvec_nk(xn[0], dt, w, dt, "f32")
    out = empty_dev((1, N), dt)
    run(enc, pc.Kernels.RMSNormMatmul(to_dev(x, dt), to_dev(nw, "f32"), to_dev(w, dt), into=out, eps=1e-6,
                                      add_one_to_weight=True))
    assert_close(from_dev(out, dt)[0], exp, dt, what="rmsnorm+matvec", pre=pre)


@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("act", [0, 1])
@pytest.mark.parametrize("norm", [True, False])
def test_gated_mlp(pc, enc, dt, act, norm):
    rng = np.random.default_rng(31 + act)
    K, F = 2304, 9216
    x = rand(rng, (1, K), dt)
    nw = (rng.standard_normal(K) * 0.1).astype(np.float32)
    wg = rand(rng, (F, K), dt, 0.02)
    wu = rand(rng, (F, K), dt, 0.02)
    xn = oracle.rmsnorm(x, dt, nw, eps=1e-6, add_one=True) if norm else x
    g = oracle.matvec_nk(xn[0], dt, wg, dt, dt)
    u = oracle.matvec_nk(xn[0], dt, wu, dt, dt)
    a = oracle.silu(g, dt) if act == 1 else oracle.gelu_tanh(g, dt)
    exp = oracle.mul(a, u, dt)
    cands = gated_candidates(oracle.matvec_nk(xn[0], dt, wg, dt, "f32"), oracle.matvec_nk(xn[0], dt, wu, dt, "f32"),
                             dt, act)
    out = empty_dev((1, F), dt)
    run(enc, pc.Kernels.GatedMLP(to_dev(x, dt), to_dev(wg, dt), to_dev(wu, dt), into=out,
                                 norm_weight=to_dev(nw, "f32") if norm else None, eps=1e-6, add_one_to_weight=True,
                                 activation=act))
    assert_close(from_dev(out, dt)[0], exp, dt, what="gated mlp", candidates=cands)


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_matmul_residual(pc, enc, dt):
    rng = np.random.default_rng(41)
    K, N = 9216, 2304
    a = rand(rng, (1, K), dt)
    w = rand(rng, (N, K), dt, 0.02)
    r = rand(rng, (1, N), dt)
    y = oracle.matvec_nk(a[0], dt, w, dt, dt)
    exp = oracle.add(r[0], y, dt)
    cands = residual_candidates(oracle.matvec_nk(a[0], dt, w, dt, "f32"), r[0], dt)
    out = empty_dev((1, N), dt)
    run(enc, pc.Kernels.MatmulResidual(to_dev(a, dt), to_dev(w, dt), to_dev(r, dt), into=out))
    assert_close(from_dev(out, dt)[0], exp, dt, what="matvec+add", candidates=cands)


@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("device_pos", [False, True])
def test_qkv_projection(pc, enc, dt, device_pos):
    rng = np.random.default_rng(51)
    H, Nq, Nkv, Hd, Smax, pos = 2304, 8, 4, 256, 64, 37
    x = rand(rng, (1, H), dt)
    nw = (rng.standard_normal(H) * 0.1).astype(np.float32)
    w = rand(rng, ((Nq + 2 * Nkv) * Hd, H), dt, 0.02)
    kc = rand(rng, (1, Nkv, Smax, Hd), dt)
    vc = rand(rng, (1, Nkv, Smax, Hd), dt)
    xn = oracle.rmsnorm(x, dt, nw, eps=1e-6, add_one=True)
    qkv = oracle.matvec_nk(xn[0], dt, w, dt, dt)
    qkv_pre = oracle.matvec_nk(xn[0], dt, w, dt, "f32")
    kd, vd = to_dev(kc, dt), to_dev(vc, dt)
    q_out = empty_dev((1, Nq, 1, Hd), dt)
    position = to_dev(np.array([pos], np.int32), "i32") if device_pos else None
    run(enc, pc.Kernels.QKVProjection(to_dev(x, dt), to_dev(nw, "f32"), to_dev(w, dt), q_out, kd, vd,
                                      offset=0 if device_pos else pos, position=position, eps=1e-6,
                                      add_one_to_weight=True))
    assert_close(from_dev(q_out, dt).ravel(), qkv[:Nq * Hd], dt, what="q", pre=qkv_pre[:Nq * Hd])
    gk, gv = from_dev(kd, dt), from_dev(vd, dt)
    assert_close(gk[0, :, pos].ravel(), qkv[Nq * Hd:(Nq + Nkv) * Hd], dt, what="k row",
                 pre=qkv_pre[Nq * Hd:(Nq + Nkv) * Hd])
    assert_close(gv[0, :, pos].ravel(), qkv[(Nq + Nkv) * Hd:], dt, what="v row", pre=qkv_pre[(Nq + Nkv) * Hd:])
    # every other cache row is untouched (bit-exact)
    mask = np.ones(Smax, bool)
    mask[pos] = False
    assert np.array_equal(gk[:, :, mask].view(np.uint16), kc[:, :, mask].view(np.uint16))
    assert np.array_equal(gv[:, :, mask].view(np.uint16), vc[:, :, mask].view(np.uint16))


# ---------------------------------------------------------------------------
# prefill FlashAttention
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("dt,odt", [("f32", "f32"), ("bf16", "bf16"), ("bf16", "f32"), ("f16", "f16")])
@pytest.mark.parametrize("mask,window", [("causal", -1), ("bidirectional", -1), ("sliding", 20)])
@pytest.mark.parametrize("B,Nq,Nkv,Sq,Sk,Hd", [(1, 4, 2, 40, 40, 64), (2, 2, 1, 7, 50, 128), (1, 8, 4, 130, 130, 256)])
def test_prefill_attention(pc, enc, dt, odt, mask, window, B, Nq, Nkv, Sq, Sk, Hd):
    rng = np.random.default_rng(Sq * 7 + Sk)
    q = rand(rng, (B, Nq, Sq, Hd), dt)
    k = rand(rng, (B, Nkv, Sk, Hd), dt)
    v = rand(rng, (B, Nkv, Sk, Hd), dt)
    scale = 1.0 / np.sqrt(Hd)
    exp = oracle.flash_attention(q, dt, k, v, dt, odt, scale, mask=mask, window=window)
    pre = oracle.flash_attention(q, dt, k, v, dt, "f32", scale, mask=mask, window=window)
    out = empty_dev((B, Nq, Sq, Hd), odt)
    m = {"causal": pc.AttentionMask.causal, "bidirectional": pc.AttentionMask.bidirectional}.get(mask)
    if m is None:
        m = pc.AttentionMask.causal_sliding_window(window)
    run(enc, pc.Kernels.FlashAttention(to_dev(q, dt), to_dev(k, dt), to_dev(v, dt), into=out, scale=scale, mask=m))
    assert_close(from_dev(out, odt), exp, odt, what="prefill FA", pre=pre)


@pytest.mark.parametrize("dt,odt", [("bf16", "bf16"), ("bf16", "f32"), ("f16", "f16")])
@pytest.mark.parametrize("mask,window", [("causal", -1), ("bidirectional", -1), ("sliding", 100)])
@pytest.mark.parametrize("B,Nq,Nkv,Sq,Sk,Hd", [(2, 4, 2, 300, 300, 128), (1, 2, 1, 64, 500, 256),
                                             (1, 3, 3, 200, 129, 128), (1, 2, 1, 256, 256, 256)])
def test_prefill_attention_tcgen05(pc, enc, dt, odt, mask, window, B, Nq, Nkv, Sq, Sk, Hd):
    """The tensor-core path (Sq >= 32, 16-bit, Hd 128/256): ragged query and key
    tiles, Sk > Sq and Sk < Sq (rows with no key give zeros), GQA 1/2/3."""
    rng = np.random.default_rng(Sq * 11 + Sk + Hd)
    q = rand(rng, (B, Nq, Sq, Hd), dt)
    k = rand(rng, (B, Nkv, Sk, Hd), dt)
    v = rand(rng, (B, Nkv, Sk, Hd), dt)
    scale = 1.0 / np.sqrt(Hd)
    exp = oracle.flash_attention(q, dt, k, v, dt, odt, scale, mask=mask, window=window)
    pre = oracle.flash_attention(q, dt, k, v, dt, "f32", scale, mask=mask, window=window)
    out = empty_dev((B, Nq, Sq, Hd), odt)
    m = {"causal": pc.AttentionMask.causal, "bidirectional": pc.AttentionMask.bidirectional}.get(mask)
    if m is None:
        m = pc.AttentionMask.causal_sliding_window(window)
    kern = pc.Kernels.FlashAttention(to_dev(q, dt), to_dev(k, dt), to_dev(v, dt), into=out, scale=scale, mask=m)
    assert kern.function_names == ["flash_attention_tc_bf16"]
    run(enc, kern)
    assert_close(from_dev(out, odt), exp, odt, what="tcgen05 prefill FA", pre=pre)
    assert pc.device_error_check(0) == 0


def test_prefill_attention_tcgen05_config4(pc, enc):
    """BASELINE config 4 attention (B 4, 8 Q / 4 KV heads, S 2048, Hd 256,
    bf16, causal) on the GPU; four (batch, head) planes checked against the
    oracle."""
    B, Nq, Nkv, S, Hd = 4, 8, 4, 2048, 256
    g = torch.Generator(device="cuda").manual_seed(44)
    q = torch.randn(B, Nq, S, Hd, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(B, Nkv, S, Hd, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(B, Nkv, S, Hd, device="cuda", generator=g).to(torch.bfloat16)
    out = torch.empty(B, Nq, S, Hd, device="cuda", dtype=torch.bfloat16)
    run(enc, pc.Kernels.FlashAttention(q, k, v, into=out, scale=1.0 / 16, mask=pc.AttentionMask.causal))
    for b, hq in ((0, 0), (1, 3), (2, 6), (3, 7)):
        hkv = hq * Nkv // Nq
        qs = from_dev(q[b:b + 1, hq:hq + 1].contiguous(), "bf16")
        ks = from_dev(k[b:b + 1, hkv:hkv + 1].contiguous(), "bf16")
        vs = from_dev(v[b:b + 1, hkv:hkv + 1].contiguous(), "bf16")
        exp = oracle.flash_attention(qs, "bf16", ks, vs, "bf16", "bf16", 1.0 / 16, mask="causal")
        pre = oracle.flash_attention(qs, "bf16", ks, vs, "bf16", "f32", 1.0 / 16, mask="causal")
        assert_close(from_dev(out[b:b + 1, hq:hq + 1].contiguous(), "bf16"), exp, "bf16",
                     what="config-4 FA b%d h%d" % (b, hq), pre=pre)


def test_no_device_errors_recorded(pc):
    assert pc.device_error_check(0) == 0


# ---------------------------------------------------------------------------
# tcgen05 tensor-core Matmul (m > 1, 16-bit inputs, transposeB)
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("M,K,N,dt,odt", [(128, 64, 256, "bf16", "f32"), (256, 2304, 512, "bf16", "bf16"),
                                          (300, 520, 200, "f16", "f32"), (32, 2304, 4096, "bf16", "bf16"),
                                          (64, 64, 64, "bf16", "bf16"), (17, 136, 40, "f16", "f16"),
                                          (1000, 1024, 1000, "bf16", "f32")])
def test_matmul_tcgen05(pc, enc, M, K, N, dt, odt):
    rng = np.random.default_rng(M + K + N)
    a = rand(rng, (M, K), dt)
    b = rand(rng, (N, K), dt, 0.05)
    out = empty_dev((M, N), odt)
    kern = pc.Kernels.Matmul(to_dev(a, dt), to_dev(b, dt), into=out, transpose_b=True)
    assert kern.function_names == ["matmul_tc_bf16_tb"]
    run(enc, kern)
    exp = oracle.matmul(a, dt, b, dt, odt, True)
    terms = np.abs(f32(a, dt).astype(np.float64)) @ np.abs(f32(b, dt).astype(np.float64)).T
    assert_close(from_dev(out, odt), exp, odt, what="tcgen05 matmul %dx%dx%d" % (M, K, N),
                 pre=oracle.matmul(a, dt, b, dt, "f32", True), pre_tol=dot_tolerance(terms))


@pytest.mark.parametrize("M,K,N,dt,odt", [(128, 64, 256, "bf16", "f32"), (256, 2304, 512, "bf16", "bf16"),
                                          (300, 520, 200, "f16", "f32"), (1000, 1024, 1000, "bf16", "f32"),
                                          (130, 72, 64, "f16", "f16")])
def test_matmul_tcgen05_b_not_transposed(pc, enc, M, K, N, dt, odt):
    """C = A . B with B stored [K, N]: MN-major B tiles on the tensor cores."""
    rng = np.random.default_rng(M * 3 + K + N)
    a = rand(rng, (M, K), dt)
    b = rand(rng, (K, N), dt, 0.05)
    out = empty_dev((M, N), odt)
    kern = pc.Kernels.Matmul(to_dev(a, dt), to_dev(b, dt), into=out, transpose_b=False)
    assert kern.function_names == ["matmul_tc_bf16_nn"]
    run(enc, kern)
    exp = oracle.matmul(a, dt, b, dt, odt, False)
    terms = np.abs(f32(a, dt).astype(np.float64)) @ np.abs(f32(b, dt).astype(np.float64))
    assert_close(from_dev(out, odt), exp, odt, what="tcgen05 matmul (B [K,N]) %dx%dx%d" % (M, K, N),
                 pre=oracle.matmul(a, dt, b, dt, "f32", False), pre_tol=dot_tolerance(terms))


def test_matmul_tcgen05_config4_rows(pc, enc):
    """BASELINE config 4 GEMM (8192 x 2304 x 9216, bf16, transposeB): the full
    product on the GPU, 24 sampled rows checked against the oracle."""
    M, K, N = 8192, 2304, 9216
    g = torch.Generator(device="cuda").manual_seed(4)
    a = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    b = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    run(enc, pc.Kernels.Matmul(a, b, into=out, transpose_b=True))
    rows = np.random.default_rng(0).choice(M, 24, replace=False)
    rows.sort()
    a_np = from_dev(a[torch.from_numpy(rows).cuda()].contiguous(), "bf16")
    b_np = from_dev(b, "bf16")
    exp = oracle.matmul(a_np, "bf16", b_np, "bf16", "bf16", True)
    got = from_dev(out, "bf16")[rows]
    terms = np.abs(f32(a_np, "bf16").astype(np.float64)) @ np.abs(f32(b_np, "bf16").astype(np.float64)).T
    assert_close(got, exp, "bf16", what="config-4 GEMM rows", pre=oracle.matmul(a_np, "bf16", b_np, "bf16", "f32", True),
                 pre_tol=dot_tolerance(terms))


def test_scalar_mul_kat(kats):
    """Kernels.ScalarMul (KernelsTests.swift:78-84): exact."""
    import popcorn_b200 as pc
    k = kats["scalar_mul"]
    x = torch.tensor(k["x"], dtype=torch.float32, device="cuda")
    out = torch.empty_like(x)
    pc.KernelCommandEncoder(pc.KernelLibrary(0)).encode(pc.Kernels.ScalarMul(x, by=k["scalar"], into=out))
    torch.cuda.synchronize()
    assert out.cpu().tolist() == k["expected"]


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_scalar_mul_16bit(dt):
    import popcorn_b200 as pc
    tdt = torch.float16 if dt == "f16" else torch.bfloat16
    x = torch.randn(1001, device="cuda").to(tdt)
    out = torch.empty_like(x)
    pc.KernelCommandEncoder(pc.KernelLibrary(0)).encode(pc.Kernels.ScalarMul(x, by=0.7071, into=out))
    torch.cuda.synchronize()
    # one fp32 product, one rounding to the storage type
    assert torch.equal(out, (x.float() * 0.7071).to(tdt))


@pytest.mark.parametrize("Sq,Sk,window", [(3, 3, None), (4, 4, 2), (1, 97, None), (33, 200, 17), (64, 64, 0)])
def test_attention_mask_build(Sq, Sk, window):
    """Kernels.AttentionMaskBuild against the oracle rule, exact."""
    import popcorn_b200 as pc
    mask = torch.full((Sq, Sk), 7.0, device="cuda")
    pc.KernelCommandEncoder(pc.KernelLibrary(0)).encode(pc.Kernels.AttentionMaskBuild(mask, sliding_window=window))
    torch.cuda.synchronize()
    assert np.array_equal(mask.cpu().numpy(), oracle.attention_mask(Sq, Sk, window))
