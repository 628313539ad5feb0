"""The decode layer over affine 4-bit weights (AqDecodeStack: the reference
layer, Gemma4TextInference.swift:312-436, with its Matmuls on
AffineQuantizedTensor weights, Matmul.swift:99-131) against the same op
sequence on the oracle: RMSNorm -> quantized Matmul (the m == 1 route) ->
KV write -> FlashDecoding -> quantized Matmul -> Add -> RMSNorm -> quantized
Matmul [gate; up] -> GeluTanh * up -> quantized Matmul -> Add, every
intermediate stored in bf16. A chain of ~12 rounding points: the chain
bound of the dense layer tests."""
import numpy as np
import pytest

import oracle
from tests.gpu_util import assert_chain_close

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _host16(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _q(qt):
    return (qt.packed_tensor.cpu().numpy().view(np.uint32), _host16(qt.scales), _host16(qt.biases))


def _oracle_layer(x, w, kc, vc, shape, pos):
    s = shape
    bf = "bf16"

    def mm(a, qt):
        packed, sc, bi = _q(qt)
        return oracle.aq_matmul(a.reshape(1, -1), bf, packed, sc, bi, bf, bf)[0]

    xn = oracle.rmsnorm(x, bf, w.attn_norm.cpu().numpy(), eps=s.eps, add_one=True)
    qkv = mm(xn, w.w_qkv)
    QN, KN = s.Nq * s.Hd, s.Nkv * s.Hd
    q = qkv[:QN].reshape(1, s.Nq, 1, s.Hd)
    kc[:, :, pos] = qkv[QN:QN + KN].reshape(1, s.Nkv, s.Hd)
    vc[:, :, pos] = qkv[QN + KN:].reshape(1, s.Nkv, s.Hd)
    attn = oracle.flash_decoding(q, bf, kc, vc, bf, bf, s.scale, seq_lens=[pos + 1])
    o = mm(attn.reshape(-1), w.w_o)
    h = oracle.add(x, o, bf)
    hn = oracle.rmsnorm(h, bf, w.mlp_norm.cpu().numpy(), eps=s.eps, add_one=True)
    act = oracle.mul(oracle.gelu_tanh(mm(hn, w.w_gate), bf), mm(hn, w.w_up), bf)
    d = mm(act, w.w_down)
    return oracle.add(h, d, bf)


@pytest.mark.parametrize("ctx,pos", [(512, 300), (4096, 4095)])
@pytest.mark.parametrize("ops", ["reference", "fused"])
def test_aq_decode_layer(ctx, pos, ops):
    """ops="reference": one kernel per reference op; ops="fused": the
    RMSNorm / residual / activation / KV-write folded into the 4-bit GEMVs."""
    import popcorn_b200 as pc
    from popcorn_b200.decode import AqDecodeStack, LayerShape
    shape = LayerShape(max_ctx=ctx, dtype="bf16")
    st = AqDecodeStack(pc.KernelLibrary(0), shape, 1, seed=ctx, ops=ops)
    st.set_position(pos)
    st.x.normal_(generator=torch.Generator(device="cuda").manual_seed(3))
    w = st.layers[0]
    x = _host16(st.x)[0]
    kc, vc = _host16(w.k_cache).copy(), _host16(w.v_cache).copy()
    out = st.encode_step(st.encoder())
    torch.cuda.synchronize()
    assert pc.device_error_check(0) == 0
    exp = _oracle_layer(x, w, kc, vc, shape, pos)
    got = _host16(out)[0]
    assert_chain_close(oracle.to_f32(got, "bf16"), oracle.to_f32(exp, "bf16"), "bf16", what="4-bit layer")
    # the new K/V rows reached the caches exactly as the projection stored them
    assert_chain_close(oracle.to_f32(_host16(w.k_cache)[:, :, pos], "bf16"), oracle.to_f32(kc[:, :, pos], "bf16"),
                       "bf16", what="k row", ulps=2)


@pytest.mark.parametrize("ops", ["reference", "fused"])
def test_aq_decode_stack_repeats(ops):
    """Two layers, repeated steps: identical results each time."""
    import popcorn_b200 as pc
    from popcorn_b200.decode import AqDecodeStack, LayerShape
    shape = LayerShape(max_ctx=256, dtype="bf16")
    st = AqDecodeStack(pc.KernelLibrary(0), shape, 2, seed=5, ops=ops)
    x0 = torch.randn(1, shape.H, device="cuda").bfloat16()
    enc = st.encoder()
    outs = []
    for _ in range(2):
        st.x.copy_(x0)
        st.set_position(100)
        outs.append(st.encode_step(enc).clone())
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])


def test_aq_decode_tail():
    """The 4-bit LM head with the final RMSNorm fused, then Argmax: logits
    against RMSNorm -> quantized Matmul on the oracle, the token against the
    reference Argmax of the GPU's logits."""
    import popcorn_b200 as pc
    from popcorn_b200.decode import AqDecodeStack, LayerShape
    shape = LayerShape(max_ctx=128, dtype="bf16")
    st = AqDecodeStack(pc.KernelLibrary(0), shape, 1, seed=9, vocab=4096)
    st.set_position(50)
    st.encode_step(st.encoder())
    torch.cuda.synchronize()
    h = _host16(st.out)[0]
    hn = oracle.rmsnorm(h, "bf16", st.final_norm.cpu().numpy(), eps=shape.eps, add_one=True)
    packed, sc, bi = _q(st.lm_head)
    exp = oracle.aq_matmul(hn.reshape(1, -1), "bf16", packed, sc, bi, "bf16", "bf16")
    got = _host16(st.logits)
    assert_chain_close(oracle.to_f32(got, "bf16"), oracle.to_f32(exp, "bf16"), "bf16", what="logits", ulps=3)
    assert st.token.item() == int(oracle.argmax(got, "bf16")[0])
