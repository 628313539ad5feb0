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


def rounding_flips(got, exp, pre, dt, rel=1e-5, pre_tol=None):
    """Elements where got and exp are the two neighbours of the oracle's
    pre-rounding fp32 value `pre`, and `pre` lies within `rel` (relative) of
    the midpoint between them — or, for a dot product whose terms cancel,
    within `pre_tol` (absolute, per element: a few fp32 ulps of the sum of
    the terms' magnitudes, dot_tolerance): a last-bit round-to-nearest flip
    of two fp32 results that agree to their accumulation error, not an
    arithmetic difference."""
    g = np.asarray(got, np.float64)
    e = np.asarray(exp, np.float64)
    p = np.asarray(pre, np.float64)
    spacing = bf16_ulp(np.minimum(np.abs(g), np.abs(e))) if dt == "bf16" else f16_ulp(np.minimum(np.abs(g), np.abs(e)))
    adjacent = np.isclose(np.abs(g - e), spacing, rtol=1e-9, atol=0) & (np.sign(g) == np.sign(e))
    mid = 0.5 * (g + e)
    lim = rel * np.maximum(np.abs(mid), 1e-30)
    if pre_tol is not None:
        lim = np.maximum(lim, np.asarray(pre_tol, np.float64).reshape(lim.shape))
    near_mid = np.abs(p - mid) <= lim
    return adjacent & near_mid


def dot_tolerance(a_abs_dot_b_abs):
    """Accumulation error allowance of an fp32 dot product: 4 fp32 ulps
    (2^-22) of the sum of the terms' magnitudes sum_k |a_k b_k|. Two
    correct fp32 sums of the same terms in different orders (or on tensor
    cores) differ by about this much when the terms cancel."""
    return np.ldexp(np.asarray(a_abs_dot_b_abs, np.float64), -22)


def pre_add(a, b, dt):
    """fp32 sum of two stored values: Add's value before its rounding."""
    return (f32(a, dt).astype(np.float32) + f32(b, dt).astype(np.float32)).astype(np.float32)


def pre_mul(a, b, dt):
    """fp32 product of two stored values: Mul's value before its rounding."""
    return (f32(a, dt).astype(np.float32) * f32(b, dt).astype(np.float32)).astype(np.float32)


def _bf16_from_bits(bits):
    return (bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def _neighbours(pre, dt, rel=1e-5):
    """The stored value round(pre) and, where pre lies within `rel` of the
    midpoint between round(pre) and the dtype's next value on pre's side,
    that other neighbour too (else NaN)."""
    pre = np.asarray(pre, np.float32)
    p = pre.astype(np.float64)
    if dt == "bf16":
        rb = oracle.to_dtype(pre, "bf16").astype(np.uint16).astype(np.int64)
        r = _bf16_from_bits(rb.astype(np.uint16))
        toward_up = p > r
        # moving up means a larger magnitude for positive values
        step = np.where((r >= 0) == toward_up, 1, -1)
        ob = np.clip(rb + step, 0, 0xFFFF).astype(np.uint16)
        other = _bf16_from_bits(ob)
    else:
        r16 = pre.astype(np.float16)
        r = r16.astype(np.float64)
        other = np.where(p > r, np.nextafter(r16, np.float16(np.inf)),
                         np.nextafter(r16, np.float16(-np.inf))).astype(np.float64)
    mid = 0.5 * (r + other)
    near = (p != r) & (np.abs(p - mid) <= rel * np.maximum(np.abs(mid), 1e-30))
    return r, np.where(near, other, np.nan)


def residual_candidates(y_pre, r, dt):
    """Outputs of round(round(y_pre) + r) allowed by last-bit rounding flips
    at either rounding point (each flip only where the fp32 value lies within
    1e-5 of a midpoint): [n, 4] float64 (NaN = no candidate)."""
    y0, y1 = _neighbours(y_pre, dt)
    rf = f32(r, dt).astype(np.float32)
    cands = []
    for y in (y0, y1):
        s = (np.nan_to_num(y, nan=0.0).astype(np.float32) + rf).astype(np.float32)
        o0, o1 = _neighbours(s, dt)
        cands += [np.where(np.isnan(y), np.nan, o0), np.where(np.isnan(y), np.nan, o1)]
    return np.stack([c.ravel() for c in cands], 1)


def gated_candidates(g_pre, u_pre, dt, act):
    """Outputs of round(round(act(round(g_pre))) * round(u_pre)) allowed by
    last-bit rounding flips at any of its four rounding points (each flip
    only where the fp32 value lies within 1e-5 of a midpoint)."""
    fn = oracle.silu if act == 1 else oracle.gelu_tanh
    g0, g1 = _neighbours(g_pre, dt)
    u0, u1 = _neighbours(u_pre, dt)
    cands = []
    for g in (g0, g1):
        gv = np.nan_to_num(g, nan=0.0)
        a_pre = fn(oracle.to_dtype(gv, dt), dt, odt="f32")
        a0, a1 = _neighbours(a_pre, dt)
        for a in (a0, a1):
            for u in (u0, u1):
                ok = ~(np.isnan(g) | np.isnan(a) | np.isnan(u))
                p = (np.nan_to_num(a, nan=0.0).astype(np.float32) * np.nan_to_num(u, nan=0.0).astype(np.float32))
                o0, o1 = _neighbours(p.astype(np.float32), dt)
                cands += [np.where(ok, o0, np.nan), np.where(ok, o1, np.nan)]
    return np.stack([c.ravel() for c in cands], 1)


def assert_close(got, exp, dt, atol=ATOL, rtol=RTOL, what="", pre=None, candidates=None, pre_tol=None):
    """north_star tolerance: |got - exp| <= atol + rtol*|exp|, elementwise.
    For 16-bit outputs the tolerance is finer than the dtype's spacing, so
    two fp32 results that agree to ~1e-6 but sit on either side of a
    rounding midpoint store values one ulp apart. Such an element passes only
    with proof: `pre` (the oracle's fp32 value just before its final
    rounding) must lie within 1e-5 relative of the midpoint between the two
    stored neighbours (rounding_flips). For an output behind several
    rounding points, `candidates` lists the values that last-bit flips at
    those points (each proven the same way) can produce; an element equal to
    one of them passes. Without `pre` or `candidates` there is no slack."""
    g = f32(got, dt).astype(np.float64)
    e = f32(exp, dt).astype(np.float64)
    assert g.shape == e.shape, (g.shape, e.shape)
    assert not np.isnan(g).any() or np.array_equal(np.isnan(g), np.isnan(e)), what + " NaN"
    err = np.abs(g - e)
    tol = atol + rtol * np.abs(e)
    bad = err > tol
    if bad.any() and pre is not None and dt in ("bf16", "f16"):
        p = np.asarray(pre, np.float64).reshape(e.shape)
        bad &= ~rounding_flips(g, e, p, dt, pre_tol=pre_tol)
    if bad.any() and candidates is not None:
        # an element that equals one of the outputs a chain of last-bit
        # rounding flips allows (residual_candidates / gated_candidates)
        c = np.asarray(candidates, np.float64).reshape(g.size, -1)
        bad &= ~np.any(c == g.reshape(-1, 1), axis=1).reshape(g.shape)
    if bad.any():
        i = np.argmax(np.where(bad, err - tol, -np.inf))
        raise AssertionError("%s: %d/%d outside tolerance; worst at %d: got %r exp %r (tol %r)%s"
                             % (what, int(bad.sum()), bad.size, i, g.ravel()[i], e.ravel()[i], tol.ravel()[i],
                                "" if pre is None else " pre %r" % np.asarray(pre, np.float64).ravel()[i]))
