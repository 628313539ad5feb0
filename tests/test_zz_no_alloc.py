"""The allocation-free decode attention entry point, called through the C ABI.

pc_flash_decoding_noalloc serves callers that cannot allocate device memory
(work enqueued during CUDA graph capture, allocation-free real-time loops,
hosts whose memory belongs to another framework): it keeps the split-KV
partials in a fixed array inside the library. Its output must equal the
encoder path's (pc_kernel_flash_attention / the ragged form, which borrow
the partials from a scratch allocator), call after call — the array keeps the
previous call's contents, so a stale read would show on the second call.
This file is collected last so that a failure here leaves every other test
already run.
"""
import ctypes

import numpy as np
import pytest

from tests.gpu_util import assert_close, empty_dev, from_dev, rand, to_dev

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _noalloc(q, k, v, out, lens, scale, mask):
    import popcorn_b200 as pc
    from popcorn_b200 import _native as N
    from popcorn_b200.api import _tc
    st = N.lib().pc_flash_decoding_noalloc(_tc(q), _tc(k), _tc(v), _tc(out), _tc(lens), ctypes.c_float(scale),
                                           mask.c(), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    if st != 0:
        raise pc.PopcornError(st, N.lib().pc_last_error_message().decode())


def _case(rng, B, Nq, Nkv, S, Hd, dt, odt, ragged):
    import popcorn_b200 as pc
    q = to_dev(rand(rng, (B, Nq, 1, Hd), dt), dt)
    k = to_dev(rand(rng, (B, Nkv, S, Hd), dt), dt)
    v = to_dev(rand(rng, (B, Nkv, S, Hd), dt), dt)
    lens = to_dev(rng.integers(S // 2, S + 1, size=B).astype(np.int32), "i32") if ragged else None
    scale = 1.0 / np.sqrt(Hd)
    ref = empty_dev((B, Nq, 1, Hd), odt)
    enc = pc.KernelCommandEncoder(pc.KernelLibrary(0), scratch=pc.ScratchPool())
    if ragged:
        enc.encode(pc.Kernels.FlashDecodingRagged(q, k, v, lens, into=ref, scale=scale))
    else:
        enc.encode(pc.Kernels.FlashAttention(q, k, v, into=ref, scale=scale))
    got = empty_dev((B, Nq, 1, Hd), odt)
    _noalloc(q, k, v, got, lens, scale, pc.AttentionMask.causal)
    torch.cuda.synchronize()
    return from_dev(got, odt), from_dev(ref, odt)


@pytest.mark.parametrize("B,Nq,Nkv,S,Hd,dt,odt,ragged", [
    (1, 8, 4, 1024, 256, "f16", "f16", False),
    (4, 16, 8, 4096, 256, "bf16", "bf16", True),  # config-3 shapes, ragged
    (2, 6, 2, 333, 96, "f32", "f32", False),      # generic head dim
])
def test_noalloc_matches_encoder_path_twice(B, Nq, Nkv, S, Hd, dt, odt, ragged):
    rng = np.random.default_rng(B * 1000 + S)
    for _ in range(2):  # two calls in a row, fresh inputs each time
        got, ref = _case(rng, B, Nq, Nkv, S, Hd, dt, odt, ragged)
        assert_close(got, ref, odt, what="no-alloc vs encoder path")


def test_noalloc_rejects_oversized_problem():
    import popcorn_b200 as pc
    from popcorn_b200 import _native as N
    cap = N.lib().pc_flash_decoding_noalloc_capacity()
    assert cap == 1 << 20
    # head_dim 512, 16 query heads on 2 KV heads, 32768 keys: the split plan
    # (37 splits on a 148-SM B200) needs 16 x 37 x 512 x 4 B of partial O
    # plus m and l, about 1.2 MB.
    B, Nq, Nkv, S, Hd = 1, 16, 2, 32768, 512
    q = torch.zeros(B, Nq, 1, Hd, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(B, Nkv, S, Hd, dtype=torch.bfloat16, device="cuda")
    out = torch.full_like(q, 7.0)
    with pytest.raises(pc.PopcornError) as e:
        _noalloc(q, k, k, out, None, 1.0, pc.AttentionMask.causal)
    assert e.value.code == pc.PopcornError.workspaceExhausted
    assert str(cap) in e.value.message
    torch.cuda.synchronize()
    assert torch.all(out == 7.0)  # nothing was launched
