"""The allocation-free decode attention entry point, called through the C ABI.

pc_flash_decoding_noalloc serves callers that cannot allocate device memory
(real-time decode loops that must never allocate, hosts whose device memory
belongs to another framework's pool): it keeps the split-KV partials in a
fixed array inside the library. It runs the encoder path's kernels with the
encoder path's split plan, so its output must equal that path's
(pc_kernel_flash_attention / the ragged form, which borrow the partials from
a scratch allocator) bit for bit, call after call. The array keeps the
previous call's contents: a larger problem followed by a smaller one leaves
stale slots behind that a wrong offset or split count would read. The
config-1 case is also checked against the oracle, so the test does not rest
on the encoder path alone. This file is collected last so that a failure
here leaves every other test already run.
"""
import ctypes

import numpy as np
import pytest

import oracle
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


def _mask(pc, window):
    return pc.AttentionMask.causal if window is None else pc.AttentionMask.causal_sliding_window(window)


def _case(rng, B, Nq, Nkv, S, Hd, dt, odt, ragged, window=None):
    """One problem through both entry points; returns (no-alloc, encoder,
    host inputs)."""
    import popcorn_b200 as pc
    qh = rand(rng, (B, Nq, 1, Hd), dt)
    kh = rand(rng, (B, Nkv, S, Hd), dt)
    vh = rand(rng, (B, Nkv, S, Hd), dt)
    q, k, v = to_dev(qh, dt), to_dev(kh, dt), to_dev(vh, dt)
    lens_h = rng.integers(S // 2, S + 1, size=B).astype(np.int32) if ragged else None
    lens = to_dev(lens_h, "i32") if ragged else None
    scale = 1.0 / np.sqrt(Hd)
    mask = _mask(pc, window)
    ref = empty_dev((B, Nq, 1, Hd), odt)
    enc = pc.KernelCommandEncoder(pc.KernelLibrary(0), scratch=pc.ScratchPool())
    if ragged:
        enc.encode(pc.Kernels.FlashDecodingRagged(q, k, v, lens, into=ref, scale=scale, mask=mask))
    else:
        enc.encode(pc.Kernels.FlashAttention(q, k, v, into=ref, scale=scale, mask=mask))
    got = empty_dev((B, Nq, 1, Hd), odt)
    _noalloc(q, k, v, got, lens, scale, mask)
    torch.cuda.synchronize()
    return from_dev(got, odt), from_dev(ref, odt), (qh, kh, vh, lens_h, scale)


# (B, Nq, Nkv, S, Hd, dt, odt, ragged, window). Each case runs twice: first
# at the given size, then at a smaller one, so the second call finds the
# first call's (larger) partials still in the shared array.
CASES = [
    (1, 8, 4, 1024, 256, "f16", "f16", False, None),
    (4, 16, 8, 4096, 256, "bf16", "bf16", True, None),  # config-3 shapes, ragged
    (2, 8, 4, 1000, 256, "bf16", "f32", False, 100),    # sliding window
    (2, 6, 2, 333, 96, "f32", "f32", False, None),      # generic head dim
]


@pytest.mark.parametrize("B,Nq,Nkv,S,Hd,dt,odt,ragged,window", CASES)
def test_noalloc_equals_encoder_path_twice(B, Nq, Nkv, S, Hd, dt, odt, ragged, window):
    rng = np.random.default_rng(B * 1000 + S)
    for S_call in (S, max(1, S // 3)):
        got, ref, _ = _case(rng, B, Nq, Nkv, S_call, Hd, dt, odt, ragged, window)
        assert np.array_equal(got, ref), "no-alloc output differs from the encoder path (S %d)" % S_call


def test_noalloc_config1_against_oracle():
    """BASELINE config 1 (B1, 8Q/4KV, hd 256, ctx 1024, f16) against the
    CPU oracle of the reference's FlashDecoding, on two calls in a row."""
    rng = np.random.default_rng(1234)
    for _ in range(2):
        got, _, (qh, kh, vh, _, scale) = _case(rng, 1, 8, 4, 1024, 256, "f16", "f16", False)
        exp = oracle.flash_decoding(qh, "f16", kh, vh, "f16", "f16", scale)
        assert_close(got, exp, "f16", what="no-alloc vs oracle (config 1)")


def test_noalloc_rejects_oversized_problem():
    import popcorn_b200 as pc
    from popcorn_b200 import _native as N
    cap = N.lib().pc_flash_decoding_noalloc_capacity()
    assert cap == 1 << 20
    # With per-sequence lengths the planner caps a split at 64 tiles of 32
    # keys, so 32768 keys need at least 16 splits on any GPU: the partial O
    # alone is then >= 4 x 16 x 16 x 512 x 4 B = 2 MiB, twice the capacity.
    B, Nq, Nkv, S, Hd = 4, 16, 2, 32768, 512
    q = torch.zeros(B, Nq, 1, Hd, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(B, Nkv, S, Hd, dtype=torch.bfloat16, device="cuda")
    lens = torch.full((B,), S, dtype=torch.int32, device="cuda")
    out = torch.full_like(q, 7.0)
    with pytest.raises(pc.PopcornError) as e:
        _noalloc(q, k, k, out, lens, 1.0, pc.AttentionMask.causal)
    assert e.value.code == pc.PopcornError.workspaceExhausted
    assert str(cap) in e.value.message
    torch.cuda.synchronize()
    assert torch.all(out == 7.0)  # nothing was launched
