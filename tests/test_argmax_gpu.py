"""Kernels.Argmax (Argmax.metal / Argmax.swift) on the GPU against the
oracle: the reference's known answer, ties, NaN and -inf rows, short rows
(`argmax`), one-CTA rows (`argmax_row`) and the two-pass form for an LM
head's vocabulary."""
import numpy as np
import pytest

import oracle
from tests.gpu_util import from_dev, to_dev

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def pc():
    import popcorn_b200
    return popcorn_b200


@pytest.fixture()
def enc(pc):
    return pc.KernelCommandEncoder(pc.KernelLibrary(0), scratch=pc.ScratchPool())


def _run(pc, enc, x, dt):
    xd = to_dev(x, dt)
    out = torch.empty(x.shape[:-1], dtype=torch.int32, device="cuda")
    enc.encode(pc.Kernels.Argmax(xd, out))
    torch.cuda.synchronize()
    return out.cpu().numpy()


def test_argmax_kat(pc, enc, kats):
    k = kats["argmax"]
    x = np.array(k["x"], np.float32).reshape(k["shape"])
    assert _run(pc, enc, x, "f32").tolist() == k["expected"]


@pytest.mark.parametrize("dt", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("rows,N", [(7, 5), (3, 31), (300, 100), (4, 4096), (1, 65537), (2, 256000), (33, 70000)])
def test_argmax_random(pc, enc, dt, rows, N):
    rng = np.random.default_rng(rows * 7 + N)
    x = rng.standard_normal((rows, N)).astype(np.float32)
    # ties at the maximum, NaN and -inf entries
    for r in range(rows):
        j = rng.choice(N, size=min(3, N), replace=False)
        x[r, j] = x[r].max() + 1.0
        if N > 40 and r % 3 == 1:
            x[r, rng.choice(N, size=5, replace=False)] = np.nan
    xo = oracle.to_dtype(x, dt)
    assert np.array_equal(_run(pc, enc, xo, dt), oracle.argmax(xo, dt))


@pytest.mark.parametrize("N", [20, 40, 100000])
def test_argmax_special_rows(pc, enc, N):
    x = np.zeros((3, N), np.float32)
    x[0] = np.nan            # N >= 32: nothing wins -> 0x7fffffff; N < 32: element 0
    x[1] = -np.inf           # all -inf: lowest index
    x[2] = np.nan
    x[2, N // 2] = -np.inf   # the only non-NaN value
    assert np.array_equal(_run(pc, enc, x, "f32"), oracle.argmax(x, "f32"))


def test_argmax_validation(pc):
    x = torch.zeros(4, 8, device="cuda")
    with pytest.raises(pc.PopcornError) as e:
        pc.Kernels.Argmax(x, torch.zeros(3, dtype=torch.int32, device="cuda"))
    assert e.value.code == -1007
    with pytest.raises(pc.PopcornError) as e:
        pc.Kernels.Argmax(x, torch.zeros(8, dtype=torch.int32, device="cuda"), axis=0)
    assert e.value.code == -1009


@pytest.mark.parametrize("fused", [False, True])
def test_decode_stack_lm_head_argmax(pc, fused):
    """The decode step's tail: final RMSNorm + LM head GEMV + Argmax. Logits
    against the oracle on the GPU's own hidden state; the token is the
    oracle's argmax of the GPU logits (bit-exact)."""
    from popcorn_b200.decode import DecodeStack, LayerShape
    from tests.gpu_util import assert_close
    dt = "f16"
    shape = LayerShape(max_ctx=256, dtype=dt)
    st = DecodeStack(pc.KernelLibrary(0), shape, 2, seed=5, fused=fused, vocab=50000)
    st.set_position(100)
    st.x.normal_(generator=torch.Generator(device="cuda").manual_seed(2))
    enc = st.encoder()
    st.encode_step(enc)
    torch.cuda.synchronize()
    h = from_dev(st.out, dt)
    hn = oracle.rmsnorm(h, dt, st.final_norm.cpu().numpy(), eps=shape.eps, add_one=True)[0]
    exp = oracle.matvec_nk(hn, dt, from_dev(st.lm_head, dt), dt, dt)
    logits = from_dev(st.logits, dt)[0]
    assert_close(logits, exp, dt, what="LM head logits", pre=oracle.matvec_nk(hn, dt, from_dev(st.lm_head, dt), dt, "f32"))
    assert int(st.token.item()) == int(oracle.argmax(logits[None, :], dt)[0])
    assert pc.device_error_check(0) == 0
