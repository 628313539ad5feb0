"""Decode attention with the early K/V copy (PC_HINT_KV_EARLY): the tiles
without a sequence's newest key are copied before the kernel waits for its
predecessor. The hint must never change results: it is checked against the
oracle of the reference's FlashDecoding (ragged lengths 0 / 1 / Smax,
sliding windows, splits whose first tile holds the newest key) and inside
the decode layer against the oracle layer."""
import numpy as np
import pytest

import __graft_entry__ as ge
import oracle
from tests.gpu_util import assert_chain_close, assert_close, empty_dev, from_dev, rand, to_dev

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def pc():
    import popcorn_b200
    return popcorn_b200


def test_hint_rejected_elsewhere(pc):
    a = torch.zeros(4, 64, dtype=torch.bfloat16, device="cuda")
    k = pc.Kernels.RMSNorm(a, None, into=a.clone())
    with pytest.raises(pc.PopcornError) as e:
        k.set_hint(k.HINT_KV_EARLY, 1)
    assert e.value.code == pc.PopcornError.kernelFunctionNotFound
    q = torch.zeros(1, 8, 1, 256, dtype=torch.float16, device="cuda")
    kv = torch.zeros(1, 4, 64, 256, dtype=torch.float16, device="cuda")
    fd = pc.Kernels.FlashAttention(q, kv, kv, into=q.clone(), scale=1.0)
    with pytest.raises(pc.PopcornError):
        fd.set_hint(99, 1)
    fd.set_hint(fd.HINT_KV_EARLY, 1)


@pytest.mark.parametrize("B,Nq,Nkv,S,Hd,dt,odt,lens,window", [
    (1, 8, 4, 4096, 256, "f16", "f16", [4096], None),          # config 2 attention
    (1, 8, 4, 1024, 256, "f16", "f16", None, None),            # config 1, no seq_lens
    (5, 16, 8, 1000, 256, "bf16", "f32", [0, 1, 33, 999, 1000], None),
    (2, 8, 4, 3000, 256, "bf16", "f32", [3000, 1777], 100),     # sliding window
    (2, 8, 2, 700, 128, "f16", "f32", [700, 129], None),
    (3, 4, 4, 500, 64, "bf16", "f32", [500, 64, 65], None),
])
def test_fd_kv_early_matches_oracle(pc, B, Nq, Nkv, S, Hd, dt, odt, lens, window):
    rng = np.random.default_rng(S + B)
    q = rand(rng, (B, Nq, 1, Hd), dt)
    k = rand(rng, (B, Nkv, S, Hd), dt)
    v = rand(rng, (B, Nkv, S, Hd), dt)
    mask = pc.AttentionMask.causal if window is None else pc.AttentionMask.causal_sliding_window(window)
    out = empty_dev((B, Nq, 1, Hd), odt)
    qd, kd, vd = to_dev(q, dt), to_dev(k, dt), to_dev(v, dt)
    if lens is None:
        kern = pc.Kernels.FlashAttention(qd, kd, vd, into=out, scale=1.0 / 16, mask=mask)
        exp = oracle.flash_decoding(q, dt, k, v, dt, odt, 1.0 / 16)
    else:
        ln = np.array(lens, np.int32)
        kern = pc.Kernels.FlashDecodingRagged(qd, kd, vd, to_dev(ln, "i32"), into=out, scale=1.0 / 16, mask=mask)
        exp = oracle.flash_decoding(q, dt, k, v, dt, odt, 1.0 / 16, mask="causal" if window is None else "sliding",
                                    window=-1 if window is None else window, seq_lens=ln)
    kern.set_hint(kern.HINT_KV_EARLY, 1)
    enc = pc.KernelCommandEncoder(pc.KernelLibrary(0), scratch=pc.ScratchPool())
    enc.encode(kern)
    torch.cuda.synchronize()
    assert pc.device_error_check(0) == 0
    assert_close(from_dev(out, odt), exp, odt, what="early-copy attention")


@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("ctx,pos", [(4096, 4095), (512, 300), (256, 0)])
def test_decode_layer_kv_early(dt, ctx, pos):
    """The five-kernel layer with the early K/V copy against the oracle layer;
    the rows other than the new one stay untouched."""
    from popcorn_b200.decode import LayerShape
    shape = LayerShape(max_ctx=ctx, dtype=dt)
    g, e, (kc, vc), ins = ge.smoke_layer(shape, pos=pos, seed=ctx + 3, kv_early=True)
    other = np.ones(ctx, bool)
    other[pos] = False
    assert np.array_equal(kc[:, other].view(np.uint16), ins["k_cache"][:, other].view(np.uint16))
    assert_chain_close(g, e, dt, what="layer output (early K/V copy)")
