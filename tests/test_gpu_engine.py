"""One full Levenberg-Marquardt iteration (``blast3r_b200.engine.lm_step``: residuals,
fused linearization, PCG on S, back-substitution, line search) against the reference's
own ``lm_step`` recorded in the golden fixtures (production float64 solver).

The fp32 linearization cannot be closer to the fp64 reference than conditioning allows.
The reference's own float32 solver lands a distance d32 from its float64 solver on each
case (weakly constrained depth coefficients at omega = 1e-4; focal/depth coupling with
per-frame focals); any other float32 solve of the same system lands within about d32 of
float64 too, in an unrelated direction.  The bound for each quantity is therefore 2e-3,
or 2.5 d32 when that is larger: "as close to float64 as the reference's float32 is"."""
import os

import numpy as np
import pytest
import torch

from blast3r_b200.engine import lm_step
from tests.helpers import golden_files, load_golden, rel_err, to_cuda

pytestmark = pytest.mark.gpu

CASES = [p for p in golden_files() if 'lm_K' in np.load(p).files]


@pytest.mark.parametrize('recompute', [True, False])
@pytest.mark.parametrize('path', CASES, ids=lambda p: p.split('golden_')[-1][:-4])
def test_lm_step_matches_reference(path, recompute):
    inp, opts, _ = load_golden(path)
    z = np.load(path)
    t = to_cuda(inp)

    def as_opt(v):
        return torch.from_numpy(v).cuda() if isinstance(v, np.ndarray) else v
    update, st = lm_step(t['infos'], t['pids'], t['pix2d'], t['pix2d_std'], t['pix2d_dep'], t['K'], t['P_rig2cam'],
                         t['P_w2rig'], t['z_coefs'], t['pts3d'], depth_mode=opts['depth_mode'], pnorm=opts['pnorm'],
                         clip_pix_err=opts['clip_pix_err'], huber_delta=opts['huber_delta'],
                         weight_z=opts['weight_z'], optim_K=as_opt(opts['optim_K']), optim_Z=as_opt(opts['optim_Z']),
                         optim_P=as_opt(opts['optim_P']), optim_X=as_opt(opts['optim_X']), optim_Z0=opts['optim_Z0'],
                         no_grad_f_from_rz=opts['no_grad_f_from_rz'], dtype=torch.float64,
                         recompute_residuals=recompute)
    assert abs(float(st.init_loss) - float(z['lm_init_loss'])) <= 1e-5 * abs(float(z['lm_init_loss']))
    loss_gap32 = abs(float(z['lm32_new_loss']) - float(z['lm_new_loss']))
    assert abs(float(st.new_loss) - float(z['lm_new_loss'])) <= max(1e-3 * abs(float(z['lm_init_loss'])),
                                                                    2.5 * loss_gap32)
    for key in ('pts3d', 'z_coefs', 'K', 'P_w2rig'):
        x0 = inp[key].astype(np.float64)
        step_ref = z['lm_' + key].astype(np.float64) - x0
        step = update[key].double().cpu().numpy() - x0
        if np.abs(step_ref).max() == 0:
            assert np.abs(step).max() == 0, key
            continue
        bound = max(2e-3, 2.5 * rel_err(z['lm32_' + key].astype(np.float64) - x0, step_ref))
        assert rel_err(step, step_ref) < bound, (key, rel_err(step, step_ref), bound)


def test_bundle_adjustment_matches_reference():
    """``engine.bundle_adjustment`` against the reference's own phase loop recorded in
    ``refba_bundle_adjustment.npz`` (configs[0], two phases: pnorm 1 then 0.5, depth coefficients
    2 then 5, at most 3 and 2 LM iterations): the same output shapes, the observation depth
    channels restored, a final objective (the last phase's loss, the quantity the loop
    minimises) within 25% of the reference's, and fx within the LM-step tolerance (2e-3).
    Where this loop ends varies from run to run (S is summed with atomics, and the scene has
    weakly determined directions: fy, the scale of the added depth channels): measured
    objectives 0.158 to 0.191 against the reference's 0.1758 (from 10.76 at the start), fy 530
    to 538 against its 538.2, fx within 3.5e-4."""
    from blast3r_b200.cujac import residual_loss
    from blast3r_b200.engine import bundle_adjustment
    from tests.helpers import GOLDEN_DIR, ba_objects
    z = np.load(os.path.join(GOLDEN_DIR, 'refba_bundle_adjustment.npz'))
    inp = {k[3:]: z[k] for k in z.files if k.startswith('in_') and k != 'in_weight_z'}
    sched = dict(pnorm=[float(v) for v in z['sched_pnorm']], max_iters=[int(v) for v in z['sched_max_iters']],
                 n_zcfs=[int(v) for v in z['sched_n_zcfs']])
    rigs, tracks, pts3d = ba_objects(inp, 'cuda')
    dep0 = tracks.pix2d_dep
    out, pts = bundle_adjustment(rigs, tracks, pts3d=pts3d, z_coefs=rigs.z_coefs.clone(), weight_z=float(z['in_weight_z']),
                                 device='cuda', verbose=False, **sched)
    assert tracks.pix2d_dep is dep0
    assert tuple(out.z_coefs.shape) == z['out_z_coefs'].shape and tuple(pts.shape) == z['out_pts3d'].shape
    t = to_cuda(inp)

    def loss(K, P_w2rig, z_coefs, pts):
        C = z_coefs.shape[1]
        v, _ = residual_loss(t['rigs'], K, t['P_rig2cam'], P_w2rig, z_coefs, pts, t['pids'], t['pix2d'],
                             t['pix2d_std'], t['pix2d_dep'][:, :C].contiguous(), True, float(z['in_weight_z']),
                             sched['pnorm'][-1], 100.0, 0.5)
        return float(v)
    ref = {k: torch.from_numpy(z['out_' + k]).cuda() for k in ('K', 'P_w2rig', 'z_coefs', 'pts3d')}
    l_ours = loss(out.K, out.P_w2rig, out.z_coefs, pts)
    l_ref = loss(ref['K'], ref['P_w2rig'], ref['z_coefs'], ref['pts3d'])
    print(f'bundle_adjustment: final objective {l_ours:.6f} (reference {l_ref:.6f}), focal '
          f'{float(out.K[0, 0, 0]):.3f} (reference {float(ref["K"][0, 0, 0]):.3f})')
    # where the loop ends depends on the rounding path (S is summed with atomics; phase 2 adds
    # three weakly weighted depth channels), so the objective is checked to the convergence
    # both reach (10.76 -> ~0.176, 60x) rather than to the rounding
    assert abs(l_ours - l_ref) <= 0.25 * l_ref, (l_ours, l_ref)
    assert rel_err(out.K[:, 0, 0].cpu().numpy(), z['out_K'][:, 0, 0]) < 2e-3
