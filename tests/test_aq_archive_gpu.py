"""The input side end to end: an MLX-layout 4-bit safetensors archive
(Gemma4WeightLoader.swift / Gemma4Weights.swift names) read by
WeightLoader into AqDecodeStack.from_archive, one decode step with the
Gemma-4 attention prologue (q/k/v norms + RoPE) and plain-weight RMSNorm
(addOneToWeight false), against the same op sequence on the oracle fed from
the archive's arrays."""
import numpy as np
import pytest

import oracle
from tests.gpu_util import assert_chain_close

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

H, NQ, NKV, HD, F, CTX, POS = 512, 4, 2, 128, 1024, 64, 37
P = "language_model.model.layers.0"


def _write(path, rng):
    t, dense = {}, {}

    def q(name, n, k):
        w = (rng.standard_normal((n, k)) * 0.03).astype(np.float32)
        packed, sc, bi = oracle.aq_quantize(w, sdt="bf16")
        t[name + ".weight"], t[name + ".scales"], t[name + ".biases"] = (packed, "U32"), (sc, "BF16"), (bi, "BF16")
        dense[name] = (packed, sc, bi)

    def norm(name, n):
        v = oracle.to_dtype(1.0 + 0.1 * rng.standard_normal(n), "bf16")
        t[name + ".weight"] = (v, "BF16")
        dense[name] = oracle.to_f32(v, "bf16")

    norm(P + ".input_layernorm", H)
    norm(P + ".pre_feedforward_layernorm", H)
    norm(P + ".self_attn.q_norm", HD)
    norm(P + ".self_attn.k_norm", HD)
    q(P + ".self_attn.q_proj", NQ * HD, H)
    q(P + ".self_attn.k_proj", NKV * HD, H)
    q(P + ".self_attn.v_proj", NKV * HD, H)
    q(P + ".self_attn.o_proj", H, NQ * HD)
    q(P + ".mlp.gate_proj", F, H)
    q(P + ".mlp.up_proj", F, H)
    q(P + ".mlp.down_proj", H, F)
    from popcorn_b200 import safetensors as st
    st.save(path, t)
    return dense


def test_archive_to_decode_step(tmp_path):
    import popcorn_b200 as pc
    from popcorn_b200 import safetensors as st
    from popcorn_b200.decode import AqDecodeStack, LayerShape
    rng = np.random.default_rng(11)
    path = str(tmp_path / "model.safetensors")
    w = _write(path, rng)
    loader = st.WeightLoader(st.SafeTensors(path), st.Quantization(4, 64))
    shape = LayerShape(hidden=H, q_heads=NQ, kv_heads=NKV, head_dim=HD, ffn=F, max_ctx=CTX, dtype="bf16")
    stack = AqDecodeStack.from_archive(pc.KernelLibrary(0), shape, loader, 1, qk_norm_rope=True, norm_add_one=False)
    x = oracle.to_dtype(rng.standard_normal(H), "bf16")
    stack.x.copy_(torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).view(1, H))
    stack.set_position(POS)
    out = stack.encode_step(stack.encoder())
    torch.cuda.synchronize()
    assert pc.device_error_check(0) == 0

    bf = "bf16"

    def mm(a, name):
        packed, sc, bi = w[name]
        return oracle.aq_matmul(a.reshape(1, -1), bf, packed, sc, bi, bf, bf)[0]

    cos = stack.rope_cos[POS:POS + 1].cpu().numpy()
    sin = stack.rope_sin[POS:POS + 1].cpu().numpy()
    xn = oracle.rmsnorm(x, bf, w[P + ".input_layernorm"], eps=shape.eps)
    q = mm(xn, P + ".self_attn.q_proj").reshape(1, 1, NQ, HD)
    k = mm(xn, P + ".self_attn.k_proj").reshape(1, 1, NKV, HD)
    v = mm(xn, P + ".self_attn.v_proj").reshape(1, NKV, HD)
    q = oracle.rope_apply(oracle.rmsnorm(q, bf, w[P + ".self_attn.q_norm"], eps=shape.eps), bf, cos, sin, "f32")
    k = oracle.rope_apply(oracle.rmsnorm(k, bf, w[P + ".self_attn.k_norm"], eps=shape.eps), bf, cos, sin, "f32")
    v = oracle.rmsnorm(v, bf, None, eps=shape.eps)
    kc = np.zeros((1, NKV, CTX, HD), np.uint16)
    vc = np.zeros_like(kc)
    kc[:, :, POS] = k.reshape(1, NKV, HD)
    vc[:, :, POS] = v
    attn = oracle.flash_decoding(q.reshape(1, NQ, 1, HD), bf, kc, vc, bf, bf, shape.scale, seq_lens=[POS + 1])
    h = oracle.add(x, mm(attn.reshape(-1), P + ".self_attn.o_proj"), bf)
    hn = oracle.rmsnorm(h, bf, w[P + ".pre_feedforward_layernorm"], eps=shape.eps)
    act = oracle.mul(oracle.gelu_tanh(mm(hn, P + ".mlp.gate_proj"), bf), mm(hn, P + ".mlp.up_proj"), bf)
    exp = oracle.add(h, mm(act, P + ".mlp.down_proj"), bf)

    got = out.detach().cpu().view(torch.int16).numpy().view(np.uint16)[0]
    assert_chain_close(oracle.to_f32(got, bf), oracle.to_f32(exp, bf), bf, what="archive layer")
    kd = stack.layers[0].k_cache.cpu().view(torch.int16).numpy().view(np.uint16)
    assert_chain_close(oracle.to_f32(kd[:, :, POS], bf), oracle.to_f32(kc[:, :, POS], bf), bf, what="k row", ulps=3)
