"""Matmul against an AffineQuantizedTensor (Matmul.swift:99-131, 279-351;
AffineQuantizedMatmul.metal) and the embedding gathers (EmbeddingGather
.metal, AffineQuantizedEmbeddingGather.metal) on the GPU against the oracle.

The reference has no test vectors for these kernels, so parity is pinned by
the oracle restatement (both reference routes: m == 1 aq_qmv_fast, m > 1
aq_matvec_simd4) and by the float64 dequantised product; the tolerance is
the fp32-accumulation one of every other GEMV (1e-3 abs + 2e-3 rel, one
bf16 ulp on bf16 outputs)."""
import numpy as np
import pytest

import oracle
from tests.gpu_util import assert_close, dot_tolerance, f32, from_dev, gated_candidates, residual_candidates, to_dev

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def pc():
    import popcorn_b200
    return popcorn_b200


def _enc(pc, scratch):
    return pc.KernelCommandEncoder(pc.KernelLibrary(0), scratch=pc.ScratchPool() if scratch else None)


def _qtensor(pc, rng, N, K, sdt, bias=True):
    w = rng.standard_normal((N, K)).astype(np.float32) * 0.02
    if not bias:
        w = np.abs(w)
    packed, sc, bi = oracle.aq_quantize(w, sdt=sdt, bias=bias)
    qt = pc.AffineQuantizedTensor(torch.from_numpy(packed.view(np.int32)).cuda(), to_dev(sc, sdt),
                                  to_dev(bi, sdt) if bi is not None else None, (N, K))
    return qt, packed, sc, bi


TDT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}

COMBOS = [("bf16", "bf16", "bf16"), ("bf16", "bf16", "f32"), ("f32", "bf16", "f32"), ("f16", "f16", "f16")]


@pytest.mark.parametrize("xdt,sdt,odt", COMBOS)
@pytest.mark.parametrize("M,N,K", [(1, 24, 64), (1, 2304, 2304), (1, 2304, 9216), (1, 9216, 2304), (3, 40, 640),
                                   (8, 2048, 2304), (13, 300, 1024), (1, 2304, 8256),
                                   (20, 64, 2304)])
@pytest.mark.parametrize("scratch", [False, True])
def test_aq_matmul(pc, xdt, sdt, odt, M, N, K, scratch):
    rng = np.random.default_rng(M * 1000 + N + K)
    qt, packed, sc, bi = _qtensor(pc, rng, N, K, sdt)
    x = oracle.to_dtype(rng.standard_normal((M, K)), xdt) if xdt != "f32" else \
        rng.standard_normal((M, K)).astype(np.float32)
    out = torch.empty(M, N, dtype={"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[odt],
                      device="cuda")
    enc = _enc(pc, scratch)
    enc.encode(pc.Kernels.Matmul(to_dev(x, xdt), qt, out))
    torch.cuda.synchronize()
    assert pc.device_error_check(0) == 0
    got = from_dev(out, odt)
    exp = oracle.aq_matmul(x, xdt, packed, sc, bi, sdt, odt)
    # the kernel folds each group's offset, (bias - 128 scale) * sum(x), so
    # its fp32 sum cancels differently from the oracle's: the flip allowance
    # is set by the magnitudes of the dequantised terms
    wq = oracle.aq_dequantize(packed, sc, bi, sdt, K)
    terms = np.abs(f32(x, xdt).astype(np.float64)) @ (np.abs(wq.astype(np.float64)) + 128 * np.abs(
        oracle.to_f32(np.repeat(sc, 64, axis=1), sdt).astype(np.float64))).T
    assert_close(got, exp, odt, what="aq matmul", pre=oracle.aq_matmul(x, xdt, packed, sc, bi, sdt, "f32"),
                 pre_tol=dot_tolerance(terms))
    if odt == "f32":
        exact = oracle.aq_matmul_exact(x, xdt, packed, sc, bi, sdt)
        assert np.allclose(got, exact, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("M", [1, 5])
def test_aq_matmul_without_bias(pc, M):
    """biases == nil (AffineQuantizedTensor.swift:63-65): w = q * scale."""
    rng = np.random.default_rng(M)
    qt, packed, sc, bi = _qtensor(pc, rng, 64, 512, "bf16", bias=False)
    assert bi is None and qt.biases is None
    x = oracle.to_dtype(rng.standard_normal((M, 512)), "bf16")
    out = torch.empty(M, 64, dtype=torch.float32, device="cuda")
    _enc(pc, True).encode(pc.Kernels.Matmul(to_dev(x, "bf16"), qt, out))
    torch.cuda.synchronize()
    assert_close(from_dev(out, "f32"), oracle.aq_matmul(x, "bf16", packed, sc, None, "bf16", "f32"), "f32")


def test_aq_matmul_repeated_split_k(pc):
    """Split-K counters are reset by every launch: repeated launches agree."""
    rng = np.random.default_rng(5)
    qt, packed, sc, bi = _qtensor(pc, rng, 2304, 9216, "bf16")
    x = to_dev(oracle.to_dtype(rng.standard_normal((1, 9216)), "bf16"), "bf16")
    enc = _enc(pc, True)
    outs = []
    for _ in range(3):
        out = torch.empty(1, 2304, dtype=torch.float32, device="cuda")
        enc.encode(pc.Kernels.Matmul(x, qt, out))
        outs.append(out)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])


def test_aq_matmul_rejects(pc):
    rng = np.random.default_rng(0)
    qt, *_ = _qtensor(pc, rng, 16, 128, "bf16")
    x = torch.zeros(1, 128, dtype=torch.float16, device="cuda")
    with pytest.raises(pc.PopcornError):  # f16 x with bf16 scales is not a served combination
        pc.Kernels.Matmul(x, qt, torch.zeros(1, 16, dtype=torch.float16, device="cuda"))
    with pytest.raises(pc.PopcornError):  # K mismatch
        pc.Kernels.Matmul(torch.zeros(1, 64, dtype=torch.bfloat16, device="cuda"), qt,
                          torch.zeros(1, 16, dtype=torch.bfloat16, device="cuda"))
    bad = pc.AffineQuantizedTensor(qt.packed_values, qt.scales, qt.biases, (16, 128), bits=8)
    with pytest.raises(pc.PopcornError):
        pc.Kernels.Matmul(torch.zeros(1, 128, dtype=torch.bfloat16, device="cuda"), bad,
                          torch.zeros(1, 16, dtype=torch.bfloat16, device="cuda"))


@pytest.mark.parametrize("tdt,odt", [("f32", "f32"), ("f16", "f16"), ("bf16", "bf16"), ("bf16", "f32")])
def test_embedding_gather(pc, tdt, odt):
    rng = np.random.default_rng(2)
    table = oracle.to_dtype(rng.standard_normal((1000, 2304)), tdt) if tdt != "f32" else \
        rng.standard_normal((1000, 2304)).astype(np.float32)
    ids = np.array([5, 999, 0, 5, 123], np.int32)
    out = torch.empty(5, 2304, dtype={"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[odt],
                      device="cuda")
    _enc(pc, False).encode(pc.Kernels.EmbeddingGather(to_dev(ids, "i32"), to_dev(table, tdt), out))
    torch.cuda.synchronize()
    exp = oracle.embedding_gather(ids, table, tdt, odt)
    assert np.array_equal(from_dev(out, odt).view(np.uint8), exp.view(np.uint8))


@pytest.mark.parametrize("sdt,odt", [("bf16", "bf16"), ("bf16", "f32"), ("f16", "f16")])
def test_aq_embedding_gather(pc, sdt, odt):
    rng = np.random.default_rng(3)
    V, H = 500, 2304
    qt, packed, sc, bi = _qtensor(pc, rng, V, H, sdt)
    ids = np.array([0, 499, 17, 17], np.int32)
    out = torch.empty(4, H, dtype={"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[odt],
                      device="cuda")
    _enc(pc, False).encode(pc.Kernels.EmbeddingGather(to_dev(ids, "i32"), qt, out))
    torch.cuda.synchronize()
    exp = oracle.aq_embedding_gather(ids, packed, sc, bi, sdt, odt, H)
    # one fp32 multiply-add and one rounding on both sides (an FMA may round once)
    assert_close(from_dev(out, odt), exp, odt, atol=1e-6, rtol=1e-6, what="aq gather")


def test_embedding_gather_bad_id_sets_error(pc):
    """An id outside the table: the row is skipped and bit 4 of the device
    error word is set (the reference does not check)."""
    table = torch.zeros(10, 64, dtype=torch.float32, device="cuda")
    out = torch.full((2, 64), 7.0, device="cuda")
    _enc(pc, False).encode(pc.Kernels.EmbeddingGather(to_dev(np.array([3, 10], np.int32), "i32"), table, out))
    torch.cuda.synchronize()
    assert pc.device_error_check(0) & 16
    assert torch.all(out[0] == 0) and torch.all(out[1] == 7.0)


def _f32(t):
    return t.detach().float().cpu().numpy()


@pytest.mark.parametrize("M", [1, 4])
@pytest.mark.parametrize("bf", ["bf16", "f16"])
def test_aq_fused_forms(pc, M, bf):
    """The fused 4-bit decode forms against their reference op sequences on
    the oracle: RMSNorm -> Matmul; Matmul -> Add; RMSNorm -> Matmul [gate;
    up] (8-row interleave) -> GeluTanh * up; RMSNorm -> Matmul -> q + KV write.
    bf16 x with bf16 scales (reference) and f16 / f16 (extension)."""
    rng = np.random.default_rng(M)
    K, N, eps = 2304, 512, 1e-6
    x = oracle.to_dtype(rng.standard_normal((M, K)), bf)
    nw = (0.1 * rng.standard_normal(K)).astype(np.float32)
    qt, packed, sc, bi = _qtensor(pc, rng, N, K, bf)
    enc = _enc(pc, False)
    xd = to_dev(x, bf)
    xn = oracle.rmsnorm(x, bf, nw, eps=eps, add_one=True)
    # RMSNorm -> Matmul
    out = torch.empty(M, N, dtype=TDT[bf], device="cuda")
    enc.encode(pc.Kernels.AqRMSNormMatmul(xd, to_dev(nw, "f32"), qt, out, eps=eps, add_one_to_weight=True))
    torch.cuda.synchronize()
    assert_close(from_dev(out, bf), oracle.aq_matmul(xn, bf, packed, sc, bi, bf, bf), bf, what="norm+matmul",
                 pre=oracle.aq_matmul(xn, bf, packed, sc, bi, bf, "f32"))
    # Matmul -> Add(residual)
    res = oracle.to_dtype(rng.standard_normal((M, N)), bf)
    out2 = torch.empty(M, N, dtype=TDT[bf], device="cuda")
    enc.encode(pc.Kernels.AqMatmulResidual(xd, qt, to_dev(res, bf), out2))
    torch.cuda.synchronize()
    exp2 = oracle.add(oracle.aq_matmul(x, bf, packed, sc, bi, bf, bf), res, bf)
    assert_close(from_dev(out2, bf), exp2, bf, what="matmul+residual",
                 candidates=residual_candidates(oracle.aq_matmul(x, bf, packed, sc, bi, bf, "f32"), res, bf))
    # gated: gate / up interleaved in blocks of 8
    F = N // 2
    qg, pg, sg, bg = _qtensor(pc, rng, F, K, bf)
    qu, pu, su, bu = _qtensor(pc, rng, F, K, bf)
    from popcorn_b200.decode import _interleave8
    out3 = torch.empty(M, F, dtype=TDT[bf], device="cuda")
    enc.encode(pc.Kernels.AqGatedMLP(xd, to_dev(nw, "f32"), _interleave8(qg, qu), out3, eps=eps,
                                     add_one_to_weight=True))
    torch.cuda.synchronize()
    g = oracle.aq_matmul(xn, bf, pg, sg, bg, bf, bf)
    u = oracle.aq_matmul(xn, bf, pu, su, bu, bf, bf)
    exp3 = oracle.mul(oracle.gelu_tanh(g, bf), u, bf)
    cands = gated_candidates(oracle.aq_matmul(xn, bf, pg, sg, bg, bf, "f32"), oracle.aq_matmul(xn, bf, pu, su, bu, bf, "f32"),
                             bf, 0)
    assert_close(from_dev(out3, bf), exp3, bf, what="gated", candidates=cands)
    # QKV: q [M, 2, 1, 128], caches [M, 1, 16, 128] written at position 5
    Nq, Nkv, Hd, Smax, pos = 2, 1, 128, 16, 5
    qk, pk, sk, bk = _qtensor(pc, rng, (Nq + 2 * Nkv) * Hd, K, bf)
    q = torch.zeros(M, Nq, 1, Hd, dtype=TDT[bf], device="cuda")
    kc = torch.zeros(M, Nkv, Smax, Hd, dtype=TDT[bf], device="cuda")
    vc = torch.zeros_like(kc)
    enc.encode(pc.Kernels.AqQKVProjection(xd, to_dev(nw, "f32"), qk, q, kc, vc,
                                          position=to_dev(np.array([pos], np.int32), "i32"), eps=eps,
                                          add_one_to_weight=True))
    torch.cuda.synchronize()
    qkv = oracle.aq_matmul(xn, bf, pk, sk, bk, bf, bf)
    qp = oracle.aq_matmul(xn, bf, pk, sk, bk, bf, "f32")
    assert_close(from_dev(q, bf).reshape(M, -1), qkv[:, :Nq * Hd], bf, what="q", pre=qp[:, :Nq * Hd])
    assert_close(from_dev(kc, bf)[:, 0, pos], qkv[:, Nq * Hd:(Nq + 1) * Hd], bf, what="k",
                 pre=qp[:, Nq * Hd:(Nq + 1) * Hd])
    assert_close(from_dev(vc, bf)[:, 0, pos], qkv[:, (Nq + 1) * Hd:], bf, what="v", pre=qp[:, (Nq + 1) * Hd:])
    assert torch.count_nonzero(kc[:, :, :pos]) == 0 and torch.count_nonzero(kc[:, :, pos + 1:]) == 0


def test_embedding_gather_kat(pc, kats):
    """KernelsTests.swift:121-138: exact."""
    k = kats["embedding_gather"]
    table = torch.tensor(k["table"], dtype=torch.float32, device="cuda").view(*k["shape"])
    out = torch.empty(len(k["ids"]), k["shape"][1], device="cuda")
    _enc(pc, False).encode(pc.Kernels.EmbeddingGather(torch.tensor(k["ids"], dtype=torch.int32, device="cuda"),
                                                      table, out))
    torch.cuda.synchronize()
    assert out.cpu().view(-1).tolist() == k["expected"]
