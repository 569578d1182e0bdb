"""The tensor-core decode GEMV math (gemv_mma.cuh: exact Q8_0 weights, the
activations as three int8 pieces per 32-block, s32 block sums on mma.sync)
against the oracle's exact-math matvec (f32 activations, double
accumulation).  The pieces represent each activation to 2^-22 of its
block's max |x|, so the products agree to f32 rounding: max relative error
below 1e-5 (the decode layer gate is 2e-3)."""
import numpy as np
import pytest

import vvq2_oracle as O
from fixtures_util import rel_err

pytestmark = pytest.mark.gpu

TOL = 1e-5


@pytest.mark.parametrize("n,k,m", [(1152, 896, 2), (896, 4864, 2), (4864, 896, 1), (37, 96, 2)])
def test_gemv_mma_matches_exact_matvec(vv, n, k, m):
    import synth
    rng = np.random.default_rng(n * 7 + k)
    raw, qt, ne0, ne1 = synth.q8_0_tensor(rng, n, k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    # blocks of very different scales, an all-zero block, tiny and large values
    x[0, :32] = 0.0
    x[-1, 32:64] *= 1e-6
    x[-1, 64:96] *= 3e4
    got = vv.debug_gemv_mma(raw, n, k, x)
    ref = np.stack([O.matvec(raw, qt, ne0, ne1, x[r], 0) for r in range(m)])
    e = rel_err(got, ref)
    print(f"gemv mma {n}x{k} rows {m}: max rel err {e:.2e}")
    assert e < TOL, e
