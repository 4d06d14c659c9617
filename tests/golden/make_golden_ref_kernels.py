"""Capture the REFERENCE CUDA kernels' outputs into ``tests/golden/refkern_*.npz``.

Runs on a GPU box.  It loads the reference's own extension, compiled from
``src/blast3r/extensions/cujac/sfm_jacobian_rigs.cu`` by ``oracle/build_ref.py`` into
``oracle/_ref/`` (built where the reference checkout exists; the built file travels), and
evaluates ``residuals_with_rigs`` and ``jacobians_with_rigs`` (float32 and float64) on the
inputs of every ``tests/golden/golden_*.npz`` case.  The committed outputs let the CPU test
suite check the oracle's restatement against the reference kernels themselves
(``tests/test_oracle_golden.py::test_oracle_matches_reference_kernels``).

    python tests/golden/make_golden_ref_kernels.py [--out DIR]
"""
import glob
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import build_ref          # noqa: E402
from tests.helpers import load_golden  # noqa: E402


def main():
    out_dir = sys.argv[sys.argv.index('--out') + 1] if '--out' in sys.argv else HERE
    os.makedirs(out_dir, exist_ok=True)
    ext = build_ref.load_built()
    if ext is None:
        raise SystemExit('oracle/_ref is not built: run python oracle/build_ref.py where the reference exists')
    for path in sorted(glob.glob(os.path.join(HERE, 'golden_*.npz'))):
        name = os.path.basename(path)[len('golden_'):-4]
        inp, opts, _ = load_golden(path)
        t = {k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in inp.items()}
        is_log = opts['depth_mode'] == 'log'
        res = ext.residuals_with_rigs(t['infos'], t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'],
                                      t['pids'], t['pix2d'], t['pix2d_std'], t['pix2d_dep'], is_log,
                                      opts['weight_z'], opts['pnorm'], opts['clip_pix_err'], opts['huber_delta'],
                                      1e-16)
        out = {'residuals9': res.contiguous().cpu().numpy()}
        for f64 in (False, True):
            J = ext.jacobians_with_rigs(t['infos'], t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'],
                                        t['pids'], t['pix2d_std'], t['pix2d_dep'], is_log, f64)
            tag = 'f64' if f64 else 'f32'
            out[f'J_cam_{tag}'], out[f'J_zcf_{tag}'], out[f'J_pts_{tag}'] = (j.cpu().numpy() for j in J)
        dst = os.path.join(out_dir, f'refkern_{name}.npz')
        np.savez_compressed(dst, **out)
        print(name, len(inp['pids']), 'observations ->', dst)


if __name__ == '__main__':
    main()
