"""Generate ``tests/golden/prior_tangent.npz`` from the REFERENCE's own dense tangent
prior (``_dense_tangent_prior_terms``, inference/engine.py:15-158), run on CPU in float64 (the
solver's production dtype) on seeded synthetic dense maps (``oracle.tangent_prior``).

Run in a container that has the naver/blast3r checkout (the tests only read the ``.npz``):

    B3R_REFERENCE=<path to blast3r checkout> python tests/golden/make_golden_prior.py
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import ref_ops                      # noqa: E402
from oracle.tangent_prior import synthetic_dense_maps  # noqa: E402

CASES = {
    # name: (n_imgs, H, W, C, stride, normalize_tangents, optim_Z0, weight_tan, seed)
    'norm_s4': (3, 41, 53, 5, 4, True, True, 0.7, 1),
    'norm_s3_noZ0': (2, 30, 37, 5, 3, True, False, 1.3, 2),
    'scaled_s4': (2, 44, 36, 5, 4, False, True, 0.5, 3),
    'two_channels': (2, 33, 29, 2, 2, True, True, 1.0, 4),
}


def main():
    ref = os.environ.get('B3R_REFERENCE')
    if not ref:
        raise SystemExit('set B3R_REFERENCE to the blast3r checkout')
    _, engine = ref_ops.install_into_reference(os.path.join(ref, 'src'))
    out = {}
    for name, (n, H, W, C, st, norm, z0, wt, seed) in CASES.items():
        K, zc, maps, refs = synthetic_dense_maps(n, H, W, C, seed)
        rigs = torch.stack([torch.arange(1, n + 1), torch.arange(n), torch.zeros(n, dtype=torch.int64)]).int()
        loss, g, Hz = engine._dense_tangent_prior_terms(
            rigs, torch.from_numpy(K), torch.from_numpy(zc), [torch.from_numpy(m) for m in maps],
            [torch.ones(H, W) for _ in maps], [torch.from_numpy(r) for r in refs], weight_tan=wt, tan_stride=st,
            optim_Z0=z0, dtype=torch.float64, compute_gn=True, normalize_tangents=norm)
        out[f'{name}__loss'] = np.float64(loss)
        out[f'{name}__g'] = g.numpy()
        out[f'{name}__H'] = Hz.numpy()
        print(name, float(loss), float(np.abs(g.numpy()).max()), float(np.abs(Hz.numpy()).max()))
    np.savez_compressed(os.path.join(HERE, 'prior_tangent.npz'), **out)


if __name__ == '__main__':
    main()
