"""The decode layer (config-2 shapes) through the C ABI vs the oracle's
composition of the reference ops (oracle.decode_layer)."""
import numpy as np
import pytest

import __graft_entry__ as ge
import oracle
from tests.gpu_util import assert_close

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("act", [0, 1])
@pytest.mark.parametrize("ctx,pos", [(4096, 4095), (512, 300)])
def test_decode_layer_config2(dt, act, ctx, pos):
    from popcorn_b200.decode import LayerShape
    shape = LayerShape(max_ctx=ctx, dtype=dt, activation=act)
    g, e, (kc, vc), ins = ge.smoke_layer(shape, pos=pos, seed=ctx + act)
    gd = oracle.to_dtype(g, dt)
    assert_close(gd, oracle.to_dtype(e, dt), dt, what="layer output")
    # the new K/V rows equal what the oracle's KVCacheWrite stored
    assert_close(kc[:, pos], ins["k_cache"][:, pos], dt, what="k row")
    assert_close(vc[:, pos], ins["v_cache"][:, pos], dt, what="v row")
    # every other row is untouched
    other = np.ones(ctx, bool)
    other[pos] = False
    assert np.array_equal(kc[:, other].view(np.uint16), ins["k_cache"][:, other].view(np.uint16))


def test_smoke():
    ge.smoke()
