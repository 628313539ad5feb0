"""Helpers shared by the GPU parity tests: numpy <-> torch device tensors
and the tolerance rules the tests apply."""
import numpy as np

import oracle

# Parity tolerance for f16 / bf16 / f32 outputs (fp32 accumulation on both
# sides): |gpu - oracle| <= ATOL + RTOL * |oracle|.
ATOL = 1e-3
RTOL = 2e-3


def to_dev(a, dt):
    """numpy array in oracle layout (bf16 as uint16 bits) -> CUDA torch tensor."""
    import torch
    a = np.ascontiguousarray(a)
    if dt == "bf16":
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).cuda()
    if dt == "f16":
        return torch.from_numpy(a.astype(np.float16)).cuda()
    if dt == "f32":
        return torch.from_numpy(a.astype(np.float32)).cuda()
    if dt == "i32":
        return torch.from_numpy(a.astype(np.int32)).cuda()
    raise ValueError(dt)


def from_dev(t, dt):
    """CUDA torch tensor -> numpy array in oracle layout."""
    import torch
    t = t.detach().cpu().contiguous()
    if dt == "bf16":
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def empty_dev(shape, dt):
    import torch
    tdt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16, "i32": torch.int32}[dt]
    return torch.empty(shape, dtype=tdt, device="cuda")


def rand(rng, shape, dt, scale=1.0):
    """Seeded N(0, scale^2) values already rounded to `dt` (oracle layout)."""
    return oracle.to_dtype(rng.standard_normal(shape) * scale, dt)


def f32(a, dt):
    return oracle.to_f32(a, dt) if dt != "f32" else np.asarray(a, np.float32)


def bf16_ulp(x):
    """Spacing of bf16 numbers at |x| (8 significant bits)."""
    ax = np.maximum(np.abs(x).astype(np.float64), 1e-30)
    return 2.0 ** (np.floor(np.log2(ax)) - 7)


def f16_ulp(x):
    """Spacing of f16 numbers at |x| (11 significant bits, normal range)."""
    ax = np.maximum(np.abs(x).astype(np.float64), 2.0 ** -14)
    return 2.0 ** (np.floor(np.log2(ax)) - 10)


def assert_chain_close(g, e, dt, what="", ulps=8, rel=5e-3):
    """End-to-end bound for a chain of 10+ rounding points (a whole decode
    layer or stack): relative L2 below `rel`, and pointwise within the
    per-kernel tolerance or `ulps` ulps of the dtype at the output's RMS
    scale (outputs near zero come from h + d with |h|, |d| ~ 1). One
    intermediate that rounds one ulp apart moves later values by several
    ulps, so a chain cannot meet the per-kernel bound everywhere."""
    g = np.asarray(g, np.float64)
    e = np.asarray(e, np.float64)
    r = np.linalg.norm(g - e) / max(np.linalg.norm(e), 1e-30)
    assert r < rel, (what, r)
    scale = np.maximum(np.abs(e), np.sqrt(np.mean(e ** 2)))
    ulp = bf16_ulp(scale) if dt == "bf16" else f16_ulp(scale)
    bad = np.abs(g - e) > np.maximum(ATOL + RTOL * np.abs(e), ulps * ulp)
    assert not bad.any(), "%s: %d/%d outside the chain bound" % (what, int(bad.sum()), bad.size)


def assert_close(got, exp, dt, atol=ATOL, rtol=RTOL, what="", bf16_ulps=1):
    """north_star tolerance: within atol + rtol*|exp|. For bf16 outputs a
    difference of one bf16 ulp is also accepted: the tolerance is finer than
    bf16's spacing, so a last-bit rounding flip of two fp32 sums that agree
    to ~1e-6 would otherwise fail."""
    g = f32(got, dt).astype(np.float64)
    e = f32(exp, dt).astype(np.float64)
    assert g.shape == e.shape, (g.shape, e.shape)
    assert not np.isnan(g).any() or np.array_equal(np.isnan(g), np.isnan(e)), what + " NaN"
    err = np.abs(g - e)
    tol = atol + rtol * np.abs(e)
    if dt == "bf16":
        tol = np.maximum(tol, bf16_ulp(e) * bf16_ulps * 1.001)
    bad = err > tol
    if bad.any():
        i = np.argmax(err - tol)
        raise AssertionError("%s: %d/%d outside tolerance; worst at %d: got %r exp %r (tol %r)"
                             % (what, int(bad.sum()), bad.size, i, g.ravel()[i], e.ravel()[i], tol.ravel()[i]))
