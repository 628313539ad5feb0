"""Tensor-parallel sharding plan of popcorn_b200.tp, checked on CPU: two
`gloo` ranks each compute one decode layer on their shard (with the oracle's
CPU ops) and all-reduce the o_proj / down_proj partial sums where the GPU
path does; the result must equal the unsharded layer."""
import os

import numpy as np
import pytest

import oracle
from popcorn_b200.tp import TPShape, shard_layer, shard_plan

SHAPE = dict(hidden=64, q_heads=4, kv_heads=2, head_dim=16, ffn=96, vocab=128, layers=1, batch=3, ctx=20,
             dtype="bf16")


def _full_layer(seed=0):
    s = TPShape(**SHAPE)
    rng = np.random.default_rng(seed)
    f = lambda *sh: (rng.standard_normal(sh) * 0.1).astype(np.float32)  # noqa: E731
    return s, {"w_q": f(s.Nq * s.Hd, s.H), "w_k": f(s.Nkv * s.Hd, s.H), "w_v": f(s.Nkv * s.Hd, s.H),
               "w_o": f(s.H, s.Nq * s.Hd), "w_gate": f(s.F, s.H), "w_up": f(s.F, s.H), "w_down": f(s.H, s.F),
               "attn_norm": f(s.H), "mlp_norm": f(s.H), "x": f(s.B, s.H) * 10,
               "k_cache": f(s.B, s.Nkv, s.ctx, s.Hd) * 10, "v_cache": f(s.B, s.Nkv, s.ctx, s.Hd) * 10}


def _layer(s, w, x, kc, vc, nq, nkv, all_reduce):
    """One decode layer in f32 on one shard (same op order as TPDecodeModel)."""
    B = x.shape[0]
    xn = oracle.rmsnorm(x, "f32", w["attn_norm"], eps=s.eps, add_one=True)
    q = oracle.matmul(xn, "f32", w["w_q"], "f32", "f32", True).reshape(B, nq, 1, s.Hd)
    k = oracle.matmul(xn, "f32", w["w_k"], "f32", "f32", True).reshape(B, nkv, 1, s.Hd)
    v = oracle.matmul(xn, "f32", w["w_v"], "f32", "f32", True).reshape(B, nkv, 1, s.Hd)
    kc, vc = kc.copy(), vc.copy()
    oracle.kv_cache_write(k, "f32", kc, "f32", s.ctx - 1)
    oracle.kv_cache_write(v, "f32", vc, "f32", s.ctx - 1)
    attn = oracle.flash_decoding(q, "f32", kc, vc, "f32", "f32", s.scale)
    o = all_reduce(oracle.matmul(attn.reshape(B, nq * s.Hd), "f32", w["w_o"], "f32", "f32", True))
    h = x + o
    hn = oracle.rmsnorm(h, "f32", w["mlp_norm"], eps=s.eps, add_one=True)
    g = oracle.matmul(hn, "f32", w["w_gate"], "f32", "f32", True)
    u = oracle.matmul(hn, "f32", w["w_up"], "f32", "f32", True)
    a = oracle.mul(oracle.gelu_tanh(g, "f32"), u, "f32")
    d = all_reduce(oracle.matmul(a, "f32", w["w_down"], "f32", "f32", True))
    return h + d


def _worker(rank, world, port, out_path):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    s, full = _full_layer()
    plan = shard_plan(s, rank, world)
    w = shard_layer(full, s, plan)
    k0, k1 = plan["kv_heads"]

    def all_reduce(a):
        t = torch.from_numpy(np.ascontiguousarray(a))
        dist.all_reduce(t)
        return t.numpy()

    y = _layer(s, w, full["x"], np.ascontiguousarray(full["k_cache"][:, k0:k1]),
               np.ascontiguousarray(full["v_cache"][:, k0:k1]), s.Nq // world, s.Nkv // world, all_reduce)
    if rank == 0:
        np.save(out_path, y)
    dist.destroy_process_group()


def test_shard_plan_covers_everything():
    s = TPShape()
    for world in (1, 2, 4, 8):
        plans = [shard_plan(s, r, world) for r in range(world)]
        for key, total in (("q_heads", 16), ("kv_heads", 8), ("ffn", 14336), ("vocab", 256000)):
            spans = [p[key] for p in plans]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        # each rank's query heads read only its own KV heads (GQA hkv = hq*Nkv/Nq)
        for p in plans:
            q0, q1 = p["q_heads"]
            k0, k1 = p["kv_heads"]
            assert all(k0 <= hq * s.Nkv // s.Nq < k1 for hq in range(q0, q1))
    with pytest.raises(ValueError):
        shard_plan(s, 0, 16)


def test_tp2_gloo_equals_unsharded(tmp_path):
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    out = str(tmp_path / "y.npy")
    mp.spawn(_worker, args=(2, port, out), nprocs=2, join=True)
    s, full = _full_layer()
    ref = _layer(s, full, full["x"], full["k_cache"], full["v_cache"], s.Nq, s.Nkv, lambda a: a)
    got = np.load(out)
    assert np.abs(got - ref).max() < 1e-4 * max(1.0, np.abs(ref).max())
