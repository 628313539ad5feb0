"""The peer all-reduce's bounded wait, on ONE GPU (no fault, no hang).

Kernels.AllReduceAddRMSNorm waits for every rank's published flag before it
reads that rank's partial sum over peer memory. A rank that never publishes
(it died, or never reached the call) must not hang the others: the wait
gives up after its iteration limit, sets bit 3 of the device error word,
skips the sum and lets the kernel finish. Here a world-2 group is built by
hand on one GPU whose second "rank" is plain local memory that nothing ever
writes: the first call must give up and report it, the context must stay
usable, and a call whose peer flag has been published must then succeed
with the exact sum."""
import ctypes
import time
import types

import numpy as np
import pytest

import oracle
from tests.gpu_util import assert_close, from_dev

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _group(parts, ctl):
    from popcorn_b200 import _native as N
    g = N.pc_peer_group()
    g.world, g.rank = 2, 0
    for r in range(2):
        g.partial[r][0] = parts[r][0].data_ptr()
        g.partial[r][1] = parts[r][1].data_ptr()
        g.control[r] = ctypes.cast(ctypes.c_void_p(ctl[r].data_ptr()), ctypes.POINTER(ctypes.c_uint32))
    return types.SimpleNamespace(c=g)


def test_allreduce_wait_gives_up_then_recovers():
    import popcorn_b200 as pc
    rows, H = 4, 1024
    gen = torch.Generator().manual_seed(3)
    parts = [torch.randn(2, rows, H, generator=gen).bfloat16().cuda() for _ in range(2)]
    # control blocks: flag[2], epoch[2], exit count, tile counts (uint32)
    ctl = [torch.zeros(16, dtype=torch.int32, device="cuda") for _ in range(2)]
    res = torch.randn(rows, H, generator=gen).bfloat16().cuda()
    w = (torch.randn(H, generator=gen) * 0.1).float().cuda()
    s_out = torch.empty(rows, H, dtype=torch.bfloat16, device="cuda")
    n_out = torch.empty_like(s_out)
    group = _group(parts, ctl)
    enc = pc.KernelCommandEncoder(pc.KernelLibrary(0))
    k = pc.Kernels.AllReduceAddRMSNorm(group, 0, res, w, s_out, n_out, eps=1e-6, add_one_to_weight=True)
    torch.cuda.synchronize()
    assert pc.device_error_check(0) == 0

    # (1) the peer never publishes: the wait gives up, the kernel finishes
    t0 = time.time()
    enc.encode(k)
    torch.cuda.synchronize()
    waited = time.time() - t0
    flags = pc.device_error_check(0)
    assert flags & 8, "bounded wait did not report a give-up (flags %#x)" % flags
    assert waited < 30.0, waited
    c0 = ctl[0].cpu().numpy()
    assert c0[0] == 1 and c0[2] == 1 and c0[4] == 0  # own flag published, epoch advanced, exit count reset

    # (2) the context is still usable: the peer now publishes epoch 2 for
    # buffer 0 (as if it had made both calls) and the next call completes
    ctl[1][0] = 2
    torch.cuda.synchronize()
    enc.encode(k)
    torch.cuda.synchronize()
    assert pc.device_error_check(0) == 0
    p0, p1 = parts[0][0].float(), parts[1][0].float()
    o = (p0 + p1).bfloat16().float()
    exp_sum = (res.float() + o).bfloat16()
    assert torch.equal(s_out, exp_sum)
    s_host = from_dev(exp_sum, "bf16")
    exp_norm = oracle.rmsnorm(s_host, "bf16", w.cpu().numpy(), eps=1e-6, add_one=True)
    assert_close(from_dev(n_out, "bf16"), exp_norm, "bf16", what="norm after recovery",
                 pre=oracle.rmsnorm(s_host, "bf16", w.cpu().numpy(), odt="f32", eps=1e-6, add_one=True))
