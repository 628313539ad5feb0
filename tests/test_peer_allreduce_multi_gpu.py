"""The one-shot peer-memory all-reduce (Kernels.AllReduceAddRMSNorm) across
2 GPUs, one process each (needs >= 2 GPUs; skipped otherwise):
  * the fused kernel against the exact sum of the ranks' partials, Add and
    RMSNorm, over several calls on both buffers;
  * the TP decode model's logits with the peer path against the same model
    with the NCCL all-reduce."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    import torch.distributed as dist
    import oracle
    import popcorn_b200 as pc
    from popcorn_b200 import _native as N
    from popcorn_b200.tp import TPDecodeModel, TPShape
    import ctypes
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))

    def all_gather(blob):
        out = [None] * world
        dist.all_gather_object(out, blob)
        return out

    # (1) the kernel against the exact sum
    rows, H, dt = 8, 3584, "bf16"
    g = pc.PeerGroup(rank, world, rank, rows, H, dt, all_gather)
    lib = pc.KernelLibrary(rank)
    enc = pc.KernelCommandEncoder(lib)
    w = (np.random.default_rng(1).standard_normal(H) * 0.1).astype(np.float32)
    wd = torch.from_numpy(w).cuda()
    res = torch.randn(rows, H, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16).cuda()
    errs = []
    for it in range(4):
        buf = it % 2
        parts = [torch.randn(rows, H, generator=torch.Generator().manual_seed(100 * it + r)).to(torch.bfloat16)
                 for r in range(world)]
        mine = parts[rank].contiguous()
        L = N.lib()
        assert L.pc_memcpy_htod_async(g.partial(buf).data_ptr, ctypes.c_void_p(mine.data_ptr()),
                                      mine.numel() * 2, None) == 0
        torch.cuda.synchronize()
        s_out = torch.empty(rows, H, dtype=torch.bfloat16, device="cuda")
        n_out = torch.empty_like(s_out)
        enc.encode(pc.Kernels.AllReduceAddRMSNorm(g, buf, res, wd, s_out, n_out, eps=1e-6, add_one_to_weight=True))
        torch.cuda.synchronize()
        total = sum(p.float() for p in parts).to(torch.bfloat16)  # fp32 sum in rank order, one rounding
        s_exp = (res.cpu().float() + total.float()).to(torch.bfloat16)
        errs.append(float((s_out.cpu().float() - s_exp.float()).abs().max()))
    flags = pc.device_error_check(rank)
    # (2) TP model: peer path vs NCCL path on the same weights
    shape = TPShape(hidden=512, q_heads=4, kv_heads=2, head_dim=128, ffn=1024, vocab=2048, layers=2, batch=4,
                    ctx=96, dtype="bf16")
    m = TPDecodeModel(lib, shape, rank=rank, world=world, seed=7, device=rank)
    x0 = torch.randn(shape.B, shape.H, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16).cuda()
    m.x.copy_(x0)
    enc2 = m.encoder()
    m.step(enc2, lambda t: dist.all_reduce(t))
    torch.cuda.synchronize()
    nccl_logits = m.logits.float().cpu().numpy()
    m.use_peer_allreduce(all_gather, fuse_gemm=True)
    m.x.copy_(x0)
    m.step(enc2, lambda t: None)
    torch.cuda.synchronize()
    peer_logits = m.logits.float().cpu().numpy()
    flags |= pc.device_error_check(rank)
    np.savez(os.path.join(out_dir, "r%d.npz" % rank), errs=np.array(errs), flags=flags, nccl=nccl_logits,
             peer=peer_logits)
    dist.barrier()
    g.close()
    m.peer.close()
    torch.cuda.synchronize()
    dist.barrier()
    os._exit(0)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_allreduce_two_gpus(tmp_path):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    from tests.gpu_util import assert_chain_close
    for r in range(2):
        d = np.load(tmp_path / ("r%d.npz" % r))
        assert int(d["flags"]) == 0
        # the sum is one bf16 rounding of the exact fp32 sum; the add one more
        assert float(d["errs"].max()) <= 0.0625, d["errs"]
        assert_chain_close(d["peer"], d["nccl"], "bf16", what="peer vs NCCL logits rank %d" % r, ulps=16, rel=1e-2)
