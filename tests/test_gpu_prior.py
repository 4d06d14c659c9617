"""The dense tangent prior on the GPU (b3r_tangent_prior, b3r_lin_add_zprior) against its
oracle (oracle/tangent_prior.py, pinned to the reference's _dense_tangent_prior_terms), the
golden values recorded from the reference, and its place in the Schur system and lm_step."""
import os

import numpy as np
import pytest
import torch

from blast3r_b200.prior import dense_tangent_prior_terms
from blast3r_b200.synthetic import make_scene
from oracle.tangent_prior import synthetic_dense_maps, tangent_prior
from tests.golden.make_golden_prior import CASES
from tests.helpers import GOLDEN_DIR, TOL_ACC, rel_err, scene_inputs
from tests.test_gpu_schur import run_plan

pytestmark = pytest.mark.gpu

# the X side is double on both sides; the float32 reference-pointmap side rounds differently
TOL_PRIOR = 1e-5


def _gpu_terms(n, H, W, C, st, norm, z0, wt, seed, compute_gn=True, sizes=None):
    K, zc, maps, refs = synthetic_dense_maps(n, H, W, C, seed)
    if sizes is not None:                       # ragged images: crop each to its own size
        maps = [m[:h, :w].copy() for m, (h, w) in zip(maps, sizes)]
        refs = [r[:h, :w].copy() for r, (h, w) in zip(refs, sizes)]
    rigs = torch.stack([torch.arange(1, n + 1), torch.arange(n), torch.zeros(n, dtype=torch.int64)]).int().cuda()
    out = dense_tangent_prior_terms(rigs, torch.from_numpy(K).cuda(), torch.from_numpy(zc).cuda(),
                                    [torch.from_numpy(m).cuda() for m in maps], [torch.ones(1) for _ in maps],
                                    [torch.from_numpy(r).cuda() for r in refs], weight_tan=wt, tan_stride=st,
                                    optim_Z0=z0, dtype=torch.float64, compute_gn=compute_gn, normalize_tangents=norm)
    want = tangent_prior(np.zeros(n, np.int64), K, zc, maps, refs, wt, st, z0, norm)
    return out, want


@pytest.mark.parametrize('name', sorted(CASES))
def test_prior_kernel_matches_reference_values(name):
    z = np.load(os.path.join(GOLDEN_DIR, 'prior_tangent.npz'))
    (loss, g, Hz), _ = _gpu_terms(*CASES[name])
    assert abs(float(loss) - float(z[f'{name}__loss'])) <= TOL_PRIOR * abs(float(z[f'{name}__loss']))
    assert rel_err(g.cpu().numpy(), z[f'{name}__g']) < TOL_PRIOR
    assert rel_err(Hz.cpu().numpy(), z[f'{name}__H']) < TOL_PRIOR


@pytest.mark.parametrize('case', [
    (6, 96, 128, 5, 4, True, True, 0.3, 11, None),
    (5, 80, 100, 8, 3, True, True, 1.0, 12, [(80, 100), (33, 61), (7, 100), (80, 5), (2, 2)]),
    (4, 64, 64, 1, 4, True, True, 1.0, 13, None),
    (4, 70, 90, 3, 5, False, False, 2.0, 14, None),
], ids=['six-images', 'ragged-C8', 'one-channel', 'unnormalised'])
def test_prior_kernel_matches_oracle(case):
    (loss, g, Hz), (wl, wg, wH) = _gpu_terms(*case[:9], sizes=case[9])
    assert abs(float(loss) - wl) <= TOL_PRIOR * max(abs(wl), 1e-30)
    assert rel_err(g.cpu().numpy(), wg) < TOL_PRIOR
    assert rel_err(Hz.cpu().numpy(), wH) < TOL_PRIOR
    (l2, g2, H2), _ = _gpu_terms(*case[:9], compute_gn=False, sizes=case[9])
    assert g2 is None and H2 is None and abs(float(l2) - float(loss)) <= 1e-12 * abs(float(loss))


@pytest.mark.parametrize('optim_Z', [True, False])
def test_prior_enters_the_schur_system_before_damping(optim_Z):
    """S and b with z_prior = S and b without it, plus H_z on each image's depth-coefficient
    diagonal block and g_z on b (ba_solver.py:141-173); with the depth coefficients switched
    off the blocks hold the prior alone, adaptively damped."""
    sc = make_scene(0, n_imgs=10, n_tracks=500, seed=31)
    inp, opts = scene_inputs(sc), dict(sc.options)
    opts['optim_Z'] = optim_Z
    rng = np.random.default_rng(5)
    C = sc.n_zcf
    A = rng.normal(size=(sc.n_imgs, C, C))
    Hz = torch.from_numpy(np.einsum('ica,icb->iab', A, A) * 50.0).cuda()
    gz = torch.from_numpy(rng.normal(size=(sc.n_imgs, C)) * 3.0).cuda()
    plan, s0 = run_plan(inp, opts)
    S0, b0 = s0.to_dense().cpu().numpy(), s0.b.cpu().numpy()
    s1 = plan.linearize(s0.params, s0.opts, z_prior=(Hz, gz))
    torch.cuda.synchronize()
    S1, b1 = s1.to_dense().cpu().numpy(), s1.b.cpu().numpy()
    off = plan.info.off_Z
    D = np.zeros_like(S0)
    for i in range(sc.n_imgs):
        D[off + C * i:off + C * (i + 1), off + C * i:off + C * (i + 1)] = Hz[i].cpu().numpy()
    want = S0 + D
    if not optim_Z:       # the prior replaces the 1e-12 damping of a switched-off type by an adaptive one
        lam = 1e-12 * np.abs(np.diagonal(D)[off:]).max()
        idx = np.arange(off, S0.shape[0])
        want[idx, idx] += lam - 1e-12
    assert rel_err(S1, want) < TOL_ACC
    bw = b0.copy()
    bw[off:] += gz.cpu().numpy().reshape(-1)
    assert rel_err(b1, bw) < 1e-5


def test_lm_step_with_the_tangent_prior():
    from blast3r_b200.engine import lm_step
    sc = make_scene(0, n_imgs=8, n_tracks=400, seed=41)
    o = sc.options
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in sc.lm_inputs().items()}
    _, _, maps, refs = synthetic_dense_maps(sc.n_imgs, 48, 64, sc.n_zcf, 7)
    kw = dict(pnorm=o['pnorm'], clip_pix_err=o['clip_pix_err'], huber_delta=o['huber_delta'], weight_z=o['weight_z'],
              dtype=torch.float64)
    args = (t['rigs'], t['pids'], t['pix2d'], t['pix2d_std'], t['pix2d_dep'], t['K'], t['P_rig2cam'], t['P_w2rig'],
            t['z_coefs'], t['pts3d'])
    _, st0 = lm_step(*args, **kw)
    dense = dict(log_depth_maps=[torch.from_numpy(m).cuda() for m in maps], conf=[torch.ones(1)] * sc.n_imgs,
                 pts3d_ref=[torch.from_numpy(r).cuda() for r in refs])
    upd, st = lm_step(*args, weight_tan=0.5, **dense, **kw)
    torch.cuda.synchronize()
    prior0, _, _ = dense_tangent_prior_terms(t['rigs'], t['K'], t['z_coefs'], dense['log_depth_maps'], dense['conf'],
                                             dense['pts3d_ref'], weight_tan=0.5, compute_gn=False)
    # the objective carries the prior's loss, and the step is finite and lowers the loss
    assert abs(float(st.init_loss) - float(st0.init_loss) - float(prior0)) <= 1e-5 * float(st.init_loss)
    assert float(st.new_loss) <= float(st.init_loss) + 1e-4
    assert all(bool(torch.isfinite(v).all()) for v in upd.values())
