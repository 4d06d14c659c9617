"""The CPU reference arm of bench.py linearizes track shards in separate processes and sums
them: the summed shard systems (re-damped once) must equal the one-process system."""
import numpy as np
from scipy import sparse

import bench
from blast3r_b200.synthetic import make_scene
from oracle import ba_oracle as O
from tests.helpers import rel_err


def test_track_shards_sum_to_the_full_system():
    sc = make_scene(0, n_tracks=400, seed=3)
    d = dict(sc.lm_inputs())
    d['infos'] = d.pop('rigs')
    full = O.linearize(d, sc.options, dtype=np.float64, dense=False, residual_dtype=np.float32)
    bounds = np.linspace(0, sc.n_tracks, 4).astype(int)
    parts = [bench._ref_worker((bench._ref_shard(d, bounds[w], bounds[w + 1]), sc.options)) for w in range(3)]
    lam_parts = sum(p[3] for p in parts)
    S = sum(p[0] for p in parts) - sparse.diags(lam_parts)
    b = sum(p[1] for p in parts)
    dA = sum(p[2] for p in parts) - lam_parts
    lam = np.zeros_like(dA)
    for lo, sz, nblk in parts[0][4]:
        if sz * nblk:
            lam[lo:lo + sz * nblk] = 1e-12 * np.abs(dA[lo:lo + sz * nblk]).max()
    S = (S + sparse.diags(lam)).toarray()
    assert rel_err(S, full['S'].toarray()) < 1e-9
    assert rel_err(b, full['b']) < 1e-9
