"""The fused decode-step kernel (Kernels.DecodeStack, one persistent launch
for every layer of a step) against the five-kernel path on the same stack.

Both paths round at the same points; their fp32 dot products sum in
different orders, so outputs agree to the chain bound of a whole layer
(relative L2 < 5e-3, 8 ulps at the output's RMS scale) per layer passed.
Repeated launches check that the kernel leaves its arrival counters zeroed.
"""
import numpy as np
import pytest

from tests.gpu_util import assert_chain_close

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _pair(dt, layers, ctx, seed, act=0, kv_heads=4):
    import popcorn_b200 as pc
    from popcorn_b200.decode import DecodeStack, LayerShape
    lib = pc.KernelLibrary(0)
    shape = LayerShape(max_ctx=ctx, dtype=dt, activation=act, kv_heads=kv_heads)
    return [DecodeStack(lib, shape, layers, seed=seed, fused=f) for f in (False, True)]


def _host(t):
    return t.detach().float().cpu().numpy()


def _close(g, e, dt, what, depth):
    """Chain bound scaled by the number of layers the value passed through."""
    assert_chain_close(g, e, dt, what=what, ulps=8 * depth, rel=5e-3 * depth)


@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("layers,ctx,positions,kv_heads", [(3, 512, [300, 301, 302], 4),
                                                           (2, 4096, [4093, 4094, 4095], 4),
                                                           (2, 1000, [0, 31, 32, 999], 2),
                                                           (1, 256, [255], 8)])
def test_fused_stack_matches_five_kernel_path(dt, layers, ctx, positions, kv_heads):
    """GQA groups of 2 (config 2), 4 and 1; ragged last key tile; position 0."""
    import popcorn_b200 as pc
    plain, fused = _pair(dt, layers, ctx, seed=11, kv_heads=kv_heads)
    x0 = torch.randn(1, plain.shape.H, generator=torch.Generator().manual_seed(5)).to(plain.x.dtype)
    outs = []
    for st in (plain, fused):
        st.x.copy_(x0)
        enc = st.encoder()
        res = []
        for pos in positions:  # consecutive positions, each from the same input
            st.x.copy_(x0)
            st.set_position(pos)
            out = st.encode_step(enc)
            torch.cuda.synchronize()
            res.append((_host(out), [(_host(w.k_cache[0, :, pos]), _host(w.v_cache[0, :, pos])) for w in st.layers]))
        outs.append(res)
    assert pc.device_error_check(0) == 0
    for (gp, kvp), (gf, kvf) in zip(*outs):
        for i, ((kp, vp), (kf, vf)) in enumerate(zip(kvp, kvf)):
            _close(kf, kp, dt, "k row layer %d" % i, max(i, 1))
            _close(vf, vp, dt, "v row layer %d" % i, max(i, 1))
        _close(gf, gp, dt, "stack output", layers)


def test_fused_stack_rejects_unsupported_shape():
    import popcorn_b200 as pc
    from popcorn_b200.decode import DecodeStack, LayerShape
    shape = LayerShape(hidden=512, q_heads=4, kv_heads=2, head_dim=128, ffn=1024, max_ctx=64, dtype="f16")
    st = DecodeStack(pc.KernelLibrary(0), shape, 1, fused=True)
    with pytest.raises(pc.PopcornError):
        st.kernels()
