"""The CPU oracle against golden fixtures made by running the reference solver itself
(``tests/golden/make_golden.py``): S, b, the damped diag(A) preconditioner and the PCG
delta of the reference's ``GaussNewtonSolver`` (float64, the production precision)."""
import numpy as np
import pytest

from oracle import ba_oracle as O
from tests.helpers import golden_files, load_golden, rel_err

CASES = golden_files()


@pytest.mark.parametrize('path', CASES, ids=lambda p: p.split('golden_')[-1][:-4])
def test_oracle_matches_reference_solver(path):
    inp, opts, ref = load_golden(path)
    s = O.linearize(inp, opts, dtype=np.float64, residual_dtype=np.float32)
    # residual op (float32 in the reference)
    assert rel_err(s['residuals'], ref['f64_residuals9']) < 1e-6
    assert s['S'].shape == ref['f64_S'].shape
    assert rel_err(s['S'], ref['f64_S']) < 1e-7
    assert rel_err(s['b'], ref['f64_b']) < 1e-7
    assert rel_err(s['diagA'], ref['f64_diagA']) < 1e-7
    dc, it, conv = O.solve_delta(s)
    n = len(dc)
    assert rel_err(dc, ref['f64_delta'][:n]) < 1e-5


@pytest.mark.parametrize('path', CASES, ids=lambda p: p.split('golden_')[-1][:-4])
def test_oracle_pattern_covers_reference_nonzeros(path):
    """Every numerically non-zero block of the reference's dense S lies in the oracle's
    structural pattern, and every pattern block is non-zero somewhere."""
    inp, opts, ref = load_golden(path)
    lay = O.Layout(inp['infos'], inp['pids'], len(inp['K']), len(inp['P_w2rig']), len(inp['pts3d']),
                   inp['pix2d_dep'].shape[1], opts['optim_K'], opts['optim_P'], opts['optim_Z'], opts['optim_X'])
    pat = O.s_pattern(lay)
    S = ref['f64_S']
    inpat = np.zeros((lay.nb, lay.nb), bool)
    inpat[pat[:, 0], pat[:, 1]] = True
    for p in range(lay.nb):
        for q in range(p, lay.nb):
            r0, r1 = lay.block_off[p], lay.block_off[p] + lay.block_size[p]
            c0, c1 = lay.block_off[q], lay.block_off[q] + lay.block_size[q]
            nz = np.any(S[r0:r1, c0:c1] != 0)
            assert nz == inpat[p, q], (p, q, nz)


def test_chol3x3_restatement():
    rng = np.random.default_rng(0)
    A = rng.normal(size=(64, 3, 3))
    A = A @ A.transpose(0, 2, 1) + 0.1 * np.eye(3)
    b = rng.normal(size=(64, 3))
    x = O.chol3x3_solve(A, b, 1e-12)
    assert np.abs(np.einsum('nij,nj->ni', A, x) - b).max() < 1e-9


def test_jacobian_restatement_finite_differences():
    """J of the oracle against central differences of its own residual (point block)."""
    from blast3r_b200.synthetic import make_scene
    from tests.helpers import scene_inputs
    sc = make_scene(0, n_imgs=8, n_tracks=40, seed=7)
    d = scene_inputs(sc)
    args = lambda pts: (d['infos'], d['K'], d['P_rig2cam'], d['P_w2rig'], d['z_coefs'], pts, d['pids'])
    Jc, Jz, Jp = O.jacobians_with_rigs(*args(d['pts3d']), d['pix2d_std'], d['pix2d_dep'], True)
    eps = 1e-5
    for j in range(3):
        P1 = d['pts3d'].astype(np.float64).copy(); P1[:, j] += eps
        P0 = d['pts3d'].astype(np.float64).copy(); P0[:, j] -= eps
        r1 = O.residuals_with_rigs(*args(P1), d['pix2d'], d['pix2d_std'], d['pix2d_dep'], True)
        r0 = O.residuals_with_rigs(*args(P0), d['pix2d'], d['pix2d_std'], d['pix2d_dep'], True)
        fd = (r1 - r0) / (2 * eps)
        assert rel_err(Jp[:, :, j], fd) < 1e-6


REFKERN = {p.split('golden_')[-1][:-4]: p.replace('golden_', 'refkern_') for p in CASES}


@pytest.mark.parametrize('name', sorted(REFKERN))
def test_oracle_matches_reference_kernels(name):
    """The oracle's residual and Jacobian restatements against outputs of the reference's
    own CUDA kernels captured on a B200 (tests/golden/make_golden_ref_kernels.py)."""
    import os
    path = REFKERN[name]
    if not os.path.isfile(path):
        pytest.skip('reference-kernel fixtures not captured yet')
    inp, opts, _ = load_golden(path.replace('refkern_', 'golden_'))
    rk = np.load(path)
    is_log = opts['depth_mode'] == 'log'
    a = [inp[k] for k in ('infos', 'K', 'P_rig2cam', 'P_w2rig', 'z_coefs', 'pts3d', 'pids')]
    r = O.residuals_with_rigs(*a, inp['pix2d'], inp['pix2d_std'], inp['pix2d_dep'], is_log, opts['weight_z'],
                              opts['pnorm'], opts['clip_pix_err'], opts['huber_delta'])
    for j in range(3):
        assert rel_err(r[:, j], rk['residuals9'][:, j]) < 1e-5, j
    J = O.jacobians_with_rigs(*a, inp['pix2d_std'], inp['pix2d_dep'], is_log)
    for tag, tol in (('f64', 1e-9), ('f32', 1e-5)):
        for want, key in zip(J, ('J_cam', 'J_zcf', 'J_pts')):
            got = rk[f'{key}_{tag}']
            for rr in range(want.shape[1]):
                for cc in range(want.shape[2]):
                    if np.abs(want[:, rr, cc]).max() > 0:
                        assert rel_err(got[:, rr, cc], want[:, rr, cc]) < max(tol, 2e-7 if (rr == 2 and cc < 2) else tol)
