"""The dense tangent prior's oracle (oracle/tangent_prior.py) against the reference's own
_dense_tangent_prior_terms (inference/engine.py:15-158), recorded in
tests/golden/prior_tangent.npz by tests/golden/make_golden_prior.py."""
import os

import numpy as np
import pytest

from oracle.tangent_prior import synthetic_dense_maps, tangent_prior
from tests.golden.make_golden_prior import CASES
from tests.helpers import GOLDEN_DIR, rel_err


@pytest.mark.parametrize('name', sorted(CASES))
def test_prior_oracle_matches_reference(name):
    z = np.load(os.path.join(GOLDEN_DIR, 'prior_tangent.npz'))
    n, H, W, C, st, norm, z0, wt, seed = CASES[name]
    K, zc, maps, refs = synthetic_dense_maps(n, H, W, C, seed)
    loss, g, Hz = tangent_prior(np.zeros(n, np.int64), K, zc, maps, refs, wt, st, z0, norm)
    # float32 pieces (reference pointmap tangents, confidences) round differently from torch's
    assert abs(loss - float(z[f'{name}__loss'])) <= 1e-6 * abs(float(z[f'{name}__loss']))
    assert rel_err(g, z[f'{name}__g']) < 1e-6
    assert rel_err(Hz, z[f'{name}__H']) < 1e-6
