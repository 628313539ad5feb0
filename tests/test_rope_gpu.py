"""Kernels.RopeBuildCosSin / Kernels.RopeApply (RopeBuildCosSin.metal,
RopeApply.metal) and the fused per-head norm + RoPE of a decode step on the
GPU against the oracle: the reference's known answer, every routed dtype
combination, odd half-dims, and the fused form against the reference's op
sequence RMSNorm(q) -> RopeApply, RMSNorm(k) -> RopeApply, RMSNorm(v)
(Gemma4TextInference.swift:352-381)."""
import numpy as np
import pytest

import oracle
from tests.conftest import approx_equal
from tests.gpu_util import ATOL, RTOL, assert_chain_close, empty_dev, f32, from_dev, rand, to_dev

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def pc():
    import popcorn_b200
    return popcorn_b200


@pytest.fixture()
def enc(pc):
    return pc.KernelCommandEncoder(pc.KernelLibrary(0))


def _inv_freq(Hd, base=10000.0):
    return (base ** (-np.arange(Hd // 2) * 2.0 / Hd)).astype(np.float32)


def _tables(pc, enc, positions, inv, scaling=1.0):
    T, Hd2 = len(positions), len(inv)
    c, s = empty_dev((T, Hd2), "f32"), empty_dev((T, Hd2), "f32")
    enc.encode(pc.Kernels.RopeBuildCosSin(to_dev(np.asarray(positions, np.int32), "i32"), to_dev(inv, "f32"), c, s,
                                          scaling))
    torch.cuda.synchronize()
    return from_dev(c, "f32"), from_dev(s, "f32")


def test_rope_kat(pc, enc, kats):
    k = kats["rope"]
    c, s = _tables(pc, enc, k["positions"], np.array(k["inv_freq"], np.float32))
    oc, os_ = oracle.rope_build(k["positions"], k["inv_freq"])
    assert approx_equal(c, oc).all() and approx_equal(s, os_).all()
    x = np.array(k["x"], np.float32).reshape(k["x_shape"])
    out = empty_dev(x.shape, "f32")
    enc.encode(pc.Kernels.RopeApply(to_dev(x, "f32"), to_dev(c, "f32"), to_dev(s, "f32"), out))
    torch.cuda.synchronize()
    assert approx_equal(from_dev(out, "f32"), oracle.rope_apply(x, "f32", c, s, "f32")).all()


@pytest.mark.parametrize("T,Hd2,scaling", [(1, 64, 1.0), (37, 128, 0.7), (4096, 256, 1.0)])
def test_rope_build(pc, enc, T, Hd2, scaling):
    rng = np.random.default_rng(T)
    pos = rng.integers(0, 131072, size=T).astype(np.int32)
    inv = _inv_freq(2 * Hd2, 1e6)
    c, s = _tables(pc, enc, pos, inv, scaling)
    oc, os_ = oracle.rope_build(pos, inv, scaling)
    # cos / sin of arguments up to ~1.3e5 rad: both sides reduce the argument
    # exactly, so the tables agree to a few fp32 ulps
    assert np.allclose(c, oc, rtol=0, atol=2e-6) and np.allclose(s, os_, rtol=0, atol=2e-6)


@pytest.mark.parametrize("xdt,tdt", [("f32", "f32"), ("bf16", "bf16"), ("bf16", "f32"), ("f16", "f16"),
                                     ("f16", "f32")])
@pytest.mark.parametrize("shape", [(1, 1, 8, 256), (2, 7, 3, 6), (1, 33, 16, 128)])
def test_rope_apply(pc, enc, xdt, tdt, shape):
    rng = np.random.default_rng(sum(shape))
    B, T, Nh, Hd = shape
    x = rand(rng, shape, xdt)
    c, s = oracle.rope_build(rng.integers(0, 8192, size=T), _inv_freq(Hd))
    ct, st = oracle.to_dtype(c, tdt) if tdt != "f32" else c, oracle.to_dtype(s, tdt) if tdt != "f32" else s
    out = empty_dev(shape, xdt)
    enc.encode(pc.Kernels.RopeApply(to_dev(x, xdt), to_dev(ct, tdt), to_dev(st, tdt), out))
    torch.cuda.synchronize()
    g = f32(from_dev(out, xdt), xdt)
    e = f32(oracle.rope_apply(x, xdt, ct, st, tdt), xdt)
    assert np.allclose(g, e, rtol=RTOL, atol=ATOL)


def test_rope_apply_rejects(pc):
    with pytest.raises(pc.PopcornError):
        pc.Kernels.RopeApply(empty_dev((1, 2, 1, 5), "f32"), empty_dev((2, 2), "f32"), empty_dev((2, 2), "f32"),
                             empty_dev((1, 2, 1, 5), "f32"))
    with pytest.raises(pc.PopcornError):  # f32 x with bf16 tables is not routed (RopeApply.swift:27-28)
        pc.Kernels.RopeApply(empty_dev((1, 2, 1, 4), "f32"), empty_dev((2, 2), "bf16"), empty_dev((2, 2), "bf16"),
                             empty_dev((1, 2, 1, 4), "f32"))


def _reference_sequence(q, kc, vc, qn, kn, c, s, pos, dt, eps, norm_v):
    """RMSNorm(q) -> RopeApply; RMSNorm(k) -> RopeApply; RMSNorm(v), each
    stored in `dt` (Gemma4TextInference.swift:352-381), on the oracle."""
    B, Nq, _, Hd = q.shape
    Nkv = kc.shape[1]
    qo = oracle.rope_apply(oracle.rmsnorm(q, dt, qn, eps=eps).reshape(B, 1, Nq, Hd), dt, c, s, "f32")
    kr = np.ascontiguousarray(kc[:, :, pos, :]).reshape(B, 1, Nkv, Hd)
    ko = oracle.rope_apply(oracle.rmsnorm(kr, dt, kn, eps=eps), dt, c, s, "f32")
    vr = np.ascontiguousarray(vc[:, :, pos, :])
    vo = oracle.rmsnorm(vr, dt, None, eps=eps) if norm_v else vr
    return qo.reshape(q.shape), ko.reshape(B, Nkv, Hd), vo


@pytest.mark.parametrize("dt", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("B,Nq,Nkv,Hd,Smax,pos,device_pos,norm_v", [
    (1, 8, 1, 256, 64, 17, False, True),      # Gemma-style sliding layer, one sequence
    (4, 16, 8, 128, 300, 299, True, True),    # batched decode, position on the device, last slot
    (2, 4, 2, 512, 40, 0, False, False),      # global head dim, value rows left as they are
    (1, 3, 1, 6, 8, 5, False, True),          # odd half-dim
])
def test_qk_norm_rope(pc, enc, dt, B, Nq, Nkv, Hd, Smax, pos, device_pos, norm_v):
    rng = np.random.default_rng(B * 100 + Hd)
    eps = 1e-6
    q = rand(rng, (B, Nq, 1, Hd), dt, 2.0)
    kc = rand(rng, (B, Nkv, Smax, Hd), dt)
    vc = rand(rng, (B, Nkv, Smax, Hd), dt)
    qn = (1.0 + 0.1 * rng.standard_normal(Hd)).astype(np.float32)
    kn = (1.0 + 0.1 * rng.standard_normal(Hd)).astype(np.float32)
    # the step's one-row tables, as the reference builds them for t = 1
    c, s = oracle.rope_build([pos], _inv_freq(Hd))
    eq, ek, ev = _reference_sequence(q, kc, vc, qn, kn, c, s, pos, dt, eps, norm_v)
    qd, kd, vd = to_dev(q, dt), to_dev(kc, dt), to_dev(vc, dt)
    pos_t = to_dev(np.array([pos], np.int32), "i32") if device_pos else None
    enc.encode(pc.Kernels.QKNormRope(qd, kd, vd, to_dev(qn, "f32"), to_dev(kn, "f32"), to_dev(c, "f32"),
                                     to_dev(s, "f32"), offset=0 if device_pos else pos, position=pos_t, eps=eps,
                                     norm_v=norm_v))
    torch.cuda.synchronize()
    gk, gv = from_dev(kd, dt), from_dev(vd, dt)
    for g, e, what in [(from_dev(qd, dt), eq, "q"), (gk[:, :, pos, :], ek, "k"), (gv[:, :, pos, :], ev, "v")]:
        g, e = f32(np.ascontiguousarray(g), dt), f32(np.ascontiguousarray(e), dt)
        if dt == "f32":
            assert np.allclose(g, e, rtol=RTOL, atol=ATOL), what
        else:
            # two rounding points (norm, rope): at most a couple of ulps
            assert_chain_close(g, e, dt, what, ulps=2, rel=3e-3)
    # every other cache row is untouched
    mask = np.ones(Smax, bool)
    mask[pos] = False
    assert np.array_equal(gk[:, :, mask, :], kc[:, :, mask, :])
    assert np.array_equal(gv[:, :, mask, :], vc[:, :, mask, :])


def test_qk_norm_rope_table_row_by_position(pc, enc):
    """Tables covering every position: the kernel reads the position's row."""
    rng = np.random.default_rng(9)
    B, Nq, Nkv, Hd, Smax, pos = 1, 4, 2, 64, 32, 21
    dt = "bf16"
    q, kc, vc = rand(rng, (B, Nq, 1, Hd), dt), rand(rng, (B, Nkv, Smax, Hd), dt), rand(rng, (B, Nkv, Smax, Hd), dt)
    qn = np.ones(Hd, np.float32)
    kn = np.ones(Hd, np.float32)
    c, s = oracle.rope_build(np.arange(Smax), _inv_freq(Hd))
    eq, ek, ev = _reference_sequence(q, kc, vc, qn, kn, c[pos:pos + 1], s[pos:pos + 1], pos, dt, 1e-6, True)
    qd, kd, vd = to_dev(q, dt), to_dev(kc, dt), to_dev(vc, dt)
    enc.encode(pc.Kernels.QKNormRope(qd, kd, vd, to_dev(qn, "f32"), to_dev(kn, "f32"), to_dev(c, "f32"),
                                     to_dev(s, "f32"), offset=pos))
    torch.cuda.synchronize()
    assert_chain_close(f32(from_dev(qd, dt), dt), f32(eq, dt), dt, "q", ulps=2, rel=3e-3)
    assert_chain_close(f32(np.ascontiguousarray(from_dev(kd, dt)[:, :, pos]), dt), f32(ek, dt), dt, "k", ulps=2,
                       rel=3e-3)
