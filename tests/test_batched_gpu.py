"""Batched-decode helpers (QKVScatter, GatedActivation, AddRMSNorm) against
the oracle's composition of the reference ops, and the config-5 model
(popcorn_b200.tp.TPDecodeModel, one rank) against the oracle step."""
import numpy as np
import pytest

import oracle
from tests.gpu_util import (assert_chain_close, assert_close, empty_dev, f32, from_dev, gated_candidates, rand,
                            to_dev)

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def pc():
    import popcorn_b200
    return popcorn_b200


@pytest.fixture()
def enc(pc):
    return pc.KernelCommandEncoder(pc.KernelLibrary(0))


def run(enc, *ks):
    enc.encode(*ks)
    torch.cuda.synchronize()


@pytest.mark.parametrize("dt", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("device_pos", [False, True])
def test_qkv_scatter(pc, enc, dt, device_pos):
    rng = np.random.default_rng(3)
    B, Nq, Nkv, Hd, Smax, pos = 3, 4, 2, 128, 40, 17
    qkv = rand(rng, (B, (Nq + 2 * Nkv) * Hd), dt)
    kc = rand(rng, (B, Nkv, Smax, Hd), dt)
    vc = rand(rng, (B, Nkv, Smax, Hd), dt)
    q = empty_dev((B, Nq, 1, Hd), dt)
    kd, vd = to_dev(kc, dt), to_dev(vc, dt)
    position = torch.tensor([pos], dtype=torch.int32, device="cuda") if device_pos else None
    run(enc, pc.Kernels.QKVScatter(to_dev(qkv, dt), q, kd, vd, offset=0 if device_pos else pos, position=position))
    q_exp = qkv[:, :Nq * Hd].reshape(B, Nq, 1, Hd)
    k_new = np.ascontiguousarray(qkv[:, Nq * Hd:(Nq + Nkv) * Hd].reshape(B, Nkv, 1, Hd))
    v_new = np.ascontiguousarray(qkv[:, (Nq + Nkv) * Hd:].reshape(B, Nkv, 1, Hd))
    k_exp, v_exp = kc.copy(), vc.copy()
    oracle.kv_cache_write(k_new, dt, k_exp, dt, pos)
    oracle.kv_cache_write(v_new, dt, v_exp, dt, pos)
    # a bit-exact copy
    assert np.array_equal(from_dev(q, dt), q_exp)
    assert np.array_equal(from_dev(kd, dt), k_exp)
    assert np.array_equal(from_dev(vd, dt), v_exp)


def test_qkv_scatter_validation(pc):
    B, Nq, Nkv, Hd, Smax = 2, 4, 2, 128, 16
    qkv = torch.zeros(B, (Nq + 2 * Nkv) * Hd, device="cuda", dtype=torch.bfloat16)
    q = torch.zeros(B, Nq, 1, Hd, device="cuda", dtype=torch.bfloat16)
    kc = torch.zeros(B, Nkv, Smax, Hd, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(pc.PopcornError) as e:
        pc.Kernels.QKVScatter(qkv, q, kc, kc.clone(), offset=Smax)
    assert e.value.code == -1007
    with pytest.raises(pc.PopcornError):
        pc.Kernels.QKVScatter(qkv[:, :-Hd].contiguous(), q, kc, kc.clone(), offset=0)


@pytest.mark.parametrize("dt", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("act", [0, 1])
def test_gated_activation(pc, enc, dt, act):
    rng = np.random.default_rng(5 + act)
    rows, F = 5, 300
    gu = rand(rng, (rows, 2 * F), dt)
    out = empty_dev((rows, F), dt)
    run(enc, pc.Kernels.GatedActivation(to_dev(gu, dt), out, activation=act))
    g, u = np.ascontiguousarray(gu[:, :F]), np.ascontiguousarray(gu[:, F:])
    a = oracle.gelu_tanh(g, dt) if act == 0 else oracle.silu(g, dt)
    # g and u are stored inputs here: the rounding points are act's and the
    # product's, each proven by gated_candidates (exact inputs pass as pre)
    cands = gated_candidates(f32(g, dt), f32(u, dt), dt, act) if dt != "f32" else None
    assert_close(from_dev(out, dt), oracle.mul(a, u, dt), dt, what="gated activation", candidates=cands)


@pytest.mark.parametrize("dt", ["bf16", "f16", "f32"])
def test_add_rmsnorm(pc, enc, dt):
    rng = np.random.default_rng(9)
    rows, H = 4, 3584
    a, b = rand(rng, (rows, H), dt), rand(rng, (rows, H), dt)
    w = (rng.standard_normal(H) * 0.1).astype(np.float32)
    s_out, n_out = empty_dev((rows, H), dt), empty_dev((rows, H), dt)
    run(enc, pc.Kernels.AddRMSNorm(to_dev(a, dt), to_dev(b, dt), torch.from_numpy(w).cuda(), s_out, n_out,
                                   eps=1e-6, add_one_to_weight=True))
    s_exp = oracle.add(a, b, dt)
    assert np.array_equal(from_dev(s_out, dt), s_exp) or dt == "f32"
    assert_close(from_dev(s_out, dt), s_exp, dt, what="sum")
    assert_close(from_dev(n_out, dt), oracle.rmsnorm(s_exp, dt, w, eps=1e-6, add_one=True), dt, what="norm",
                 pre=oracle.rmsnorm(s_exp, dt, w, odt="f32", eps=1e-6, add_one=True))


def _oracle_step(m, host, dt):
    """The config-5 step on the host with the reference ops (same rounding
    points as TPDecodeModel's fused kernels)."""
    s = m.s
    nq, nkv, f, Hd, B = m.nq, m.nkv, m.f, s.Hd, s.B
    x = host["x"]
    xn = oracle.rmsnorm(x, dt, host["layers"][0]["attn_norm"], eps=s.eps, add_one=True)
    for i, w in enumerate(host["layers"]):
        nxt = host["layers"][i + 1]["attn_norm"] if i + 1 < len(host["layers"]) else host["final_norm"]
        qkv = oracle.matmul(xn, dt, w["w_qkv"], dt, dt, True)
        q = np.ascontiguousarray(qkv[:, :nq * Hd].reshape(B, nq, 1, Hd))
        kn = np.ascontiguousarray(qkv[:, nq * Hd:(nq + nkv) * Hd].reshape(B, nkv, 1, Hd))
        vn = np.ascontiguousarray(qkv[:, (nq + nkv) * Hd:].reshape(B, nkv, 1, Hd))
        kc, vc = w["k_cache"].copy(), w["v_cache"].copy()
        oracle.kv_cache_write(kn, dt, kc, dt, s.ctx - 1)
        oracle.kv_cache_write(vn, dt, vc, dt, s.ctx - 1)
        attn = oracle.flash_decoding(q, dt, kc, vc, dt, dt, s.scale)
        o = oracle.matmul(attn.reshape(B, nq * Hd), dt, w["w_o"], dt, dt, True)
        h = oracle.add(x, o, dt)
        hn = oracle.rmsnorm(h, dt, w["mlp_norm"], eps=s.eps, add_one=True)
        gu = oracle.matmul(hn, dt, w["w_gu"], dt, dt, True)
        act = oracle.mul(oracle.gelu_tanh(np.ascontiguousarray(gu[:, :f]), dt), np.ascontiguousarray(gu[:, f:]), dt)
        d = oracle.matmul(act, dt, w["w_down"], dt, dt, True)
        x = oracle.add(h, d, dt)
        xn = oracle.rmsnorm(x, dt, nxt, eps=s.eps, add_one=True)
    return oracle.matmul(xn, dt, host["lm_head"], dt, dt, True)


def test_tp_model_one_rank_matches_oracle(pc):
    """TPDecodeModel at TP 1 on a small 9B-like shape, one step: logits
    against the oracle's reference-op composition (chain bound over 2 layers)."""
    from popcorn_b200.tp import TPDecodeModel, TPShape
    dt = "bf16"
    shape = TPShape(hidden=512, q_heads=4, kv_heads=2, head_dim=128, ffn=1024, vocab=2048, layers=2, batch=4,
                    ctx=96, dtype=dt)
    m = TPDecodeModel(pc.KernelLibrary(0), shape, seed=3)
    m.x.normal_(generator=torch.Generator(device="cuda").manual_seed(1))
    host = {"x": from_dev(m.x, dt), "final_norm": m.final_norm.cpu().numpy(), "lm_head": from_dev(m.lm_head, dt),
            "layers": [{k: (v.cpu().numpy() if v.dtype == torch.float32 else from_dev(v, dt)) for k, v in w.items()}
                       for w in m.layers]}
    enc = m.encoder()
    m.step(enc, lambda t: None)
    torch.cuda.synchronize()
    exp = _oracle_step(m, host, dt)
    assert_chain_close(oracle.to_f32(from_dev(m.logits, dt), dt), oracle.to_f32(exp, dt), dt, what="logits",
                       ulps=16, rel=1e-2)
    assert pc.device_error_check(0) == 0


def _fill(pc, tensor, host):
    """Copies a host array into a raw library Tensor."""
    import ctypes
    from popcorn_b200 import _native as N
    a = np.ascontiguousarray(host)
    L = N.lib()
    assert L.pc_memcpy_htod_async(tensor.data_ptr, a.ctypes.data_as(ctypes.c_void_p), a.nbytes, None) == 0
    assert L.pc_stream_synchronize(None) == 0


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_peer_allreduce_world1(pc, enc, dt):
    """One rank: the all-reduce is the partial itself; then Add and RMSNorm.
    Repeated calls on both buffers check the epoch protocol."""
    rng = np.random.default_rng(12)
    rows, H = 4, 3584
    g = pc.PeerGroup(0, 1, 0, rows, H, dt, lambda b: [b])
    w = (rng.standard_normal(H) * 0.1).astype(np.float32)
    wd = torch.from_numpy(w).cuda()
    for it in range(3):
        for buf in (0, 1):
            part = rand(rng, (rows, H), dt)
            res = rand(rng, (rows, H), dt)
            _fill(pc, g.partial(buf), part)
            s_out, n_out = empty_dev((rows, H), dt), empty_dev((rows, H), dt)
            run(enc, pc.Kernels.AllReduceAddRMSNorm(g, buf, to_dev(res, dt), wd, s_out, n_out, eps=1e-6,
                                                    add_one_to_weight=True))
            s_exp = oracle.add(res, part, dt)
            assert np.array_equal(from_dev(s_out, dt), s_exp), (it, buf)
            assert_close(from_dev(n_out, dt), oracle.rmsnorm(s_exp, dt, w, eps=1e-6, add_one=True), dt, what="norm",
                         pre=oracle.rmsnorm(s_exp, dt, w, odt="f32", eps=1e-6, add_one=True))
    assert pc.device_error_check(0) == 0
    g.close()


@pytest.mark.parametrize("fuse_gemm", [False, True])
def test_tp_model_one_rank_peer_allreduce(pc, fuse_gemm):
    """The TP model with the peer all-reduce (one rank) against the oracle
    step, as test_tp_model_one_rank_matches_oracle: the all-reduce as its own
    kernel after the GEMM, or fused into the GEMM (one kernel)."""
    from popcorn_b200.tp import TPDecodeModel, TPShape
    dt = "bf16"
    shape = TPShape(hidden=512, q_heads=4, kv_heads=2, head_dim=128, ffn=1024, vocab=2048, layers=2, batch=4,
                    ctx=96, dtype=dt)
    m = TPDecodeModel(pc.KernelLibrary(0), shape, seed=3)
    m.use_peer_allreduce(lambda b: [b], fuse_gemm=fuse_gemm)
    m.x.normal_(generator=torch.Generator(device="cuda").manual_seed(1))
    host = {"x": from_dev(m.x, dt), "final_norm": m.final_norm.cpu().numpy(), "lm_head": from_dev(m.lm_head, dt),
            "layers": [{k: (v.cpu().numpy() if v.dtype == torch.float32 else from_dev(v, dt)) for k, v in w.items()}
                       for w in m.layers]}
    enc = m.encoder()
    names = [k.name for k in m.kernels() if k is not None]
    assert ("MatmulAllReduceAddRMSNorm" in names) == fuse_gemm
    m.step(enc, lambda t: pytest.fail("no collective on the peer path"))
    torch.cuda.synchronize()
    exp = _oracle_step(m, host, dt)
    assert_chain_close(oracle.to_f32(from_dev(m.logits, dt), dt), oracle.to_f32(exp, dt), dt, what="logits",
                       ulps=16, rel=1e-2)
    assert pc.device_error_check(0) == 0
