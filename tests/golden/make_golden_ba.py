"""Generate ``tests/golden/refba_bundle_adjustment.npz`` from the REFERENCE's own phase loop.

Run in a container that has the naver/blast3r checkout (the tests only read the committed
``.npz``):

    B3R_REFERENCE=<path to blast3r checkout> python tests/golden/make_golden_ba.py

It builds a seeded configs[0] scene (20 images, 2,000 tracks), wraps it in the rig and track stand-ins of
``tests/helpers.py`` (the attributes of the reference's ``RigsData`` and ``ObservedTracks`` that
the loop uses; their own modules import the network stack) and runs the reference's
``bundle_adjustment`` (``inference/engine.py:405-503``) unchanged on the CPU, with the five CUDA
ops replaced by the CPU restatements of ``oracle/ref_ops.py``: two phases (pnorm 1 then 0.5,
depth coefficients 2 then 5, at most 3 and 2 LM iterations).  It stores the inputs and the
returned K, P_w2rig, z_coefs and points.
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from blast3r_b200.synthetic import make_scene   # noqa: E402
from oracle import ref_ops                      # noqa: E402
from tests.helpers import ba_objects            # noqa: E402

SCHEDULE = dict(pnorm=[1.0, 0.5], max_iters=[3, 2], n_zcfs=[2, 5])


def main():
    ref = os.environ.get('B3R_REFERENCE')
    if not ref:
        raise SystemExit('set B3R_REFERENCE to the blast3r checkout')
    _, engine = ref_ops.install_into_reference(os.path.join(ref, 'src'))
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    sc = make_scene(0, seed=31)
    rigs, tracks, pts3d = ba_objects(sc.lm_inputs(), 'cpu')
    out_rigs, pts = engine.bundle_adjustment(rigs, tracks, pts3d=pts3d, z_coefs=rigs.z_coefs.clone(),
                                             weight_z=sc.options['weight_z'], device='cpu', verbose=True, **SCHEDULE)
    np.savez_compressed(os.path.join(HERE, 'refba_bundle_adjustment.npz'),
                        **{f'in_{k}': v for k, v in sc.lm_inputs().items()}, in_weight_z=np.float64(sc.options['weight_z']),
                        **{f'sched_{k}': np.asarray(v) for k, v in SCHEDULE.items()},
                        out_K=out_rigs.K.numpy(), out_P_w2rig=out_rigs.P_w2rig.numpy(),
                        out_z_coefs=out_rigs.z_coefs.numpy(), out_pts3d=pts.numpy())
    print('obs', len(sc.pids), 'z_coefs out', tuple(out_rigs.z_coefs.shape))


if __name__ == '__main__':
    main()
