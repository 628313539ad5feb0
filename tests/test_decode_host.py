"""Host-side weight plumbing of the 4-bit stack, on CPU tensors: the 8-row
interleave the fused gated form reads, and row concatenation of affine
4-bit tensors (q/k/v into one QKV weight)."""
import numpy as np
import pytest

import oracle

torch = pytest.importorskip("torch")


def _qt(rng, n, k):
    from popcorn_b200.api import AffineQuantizedTensor
    w = rng.standard_normal((n, k)).astype(np.float32) * 0.02
    packed, sc, bi = oracle.aq_quantize(w, sdt="bf16")
    t = lambda a: torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)
    return AffineQuantizedTensor(torch.from_numpy(packed.view(np.int32).copy()), t(sc), t(bi), (n, k)), packed, sc, bi


def test_interleave8():
    from popcorn_b200.decode import _interleave8
    rng = np.random.default_rng(0)
    a, pa, sa, ba = _qt(rng, 24, 128)
    b, pb, sb, bb = _qt(rng, 24, 128)
    il = _interleave8(a, b)
    assert (il.out_features, il.in_features) == (48, 128)
    packed = il.packed_tensor.numpy().view(np.uint32)
    scales = il.scales.view(torch.int16).numpy().view(np.uint16)
    for i in range(3):  # rows 16i..16i+7 = a's 8i.., rows 16i+8.. = b's 8i..
        assert np.array_equal(packed[16 * i:16 * i + 8], pa[8 * i:8 * i + 8])
        assert np.array_equal(packed[16 * i + 8:16 * i + 16], pb[8 * i:8 * i + 8])
        assert np.array_equal(scales[16 * i + 8:16 * i + 16], sb[8 * i:8 * i + 8])


def test_concat_rows_dequantises_to_stacked_rows():
    from popcorn_b200.decode import _concat_rows
    rng = np.random.default_rng(1)
    parts = [_qt(rng, n, 256) for n in (32, 16, 16)]
    cat = _concat_rows([p[0] for p in parts])
    assert (cat.out_features, cat.in_features) == (64, 256)
    deq = oracle.aq_dequantize(cat.packed_tensor.numpy().view(np.uint32),
                               cat.scales.view(torch.int16).numpy().view(np.uint16),
                               cat.biases.view(torch.int16).numpy().view(np.uint16), "bf16", 256)
    exp = np.concatenate([oracle.aq_dequantize(p, s, b, "bf16", 256) for _, p, s, b in parts])
    assert np.array_equal(deq, exp)
