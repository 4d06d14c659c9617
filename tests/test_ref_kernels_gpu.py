"""Our reference-op mirrors against the reference's OWN CUDA extension, on the same B200.

``oracle/_ref/ba_with_rigs_cuda_kernels*.so`` is the reference's
``sfm_jacobian_rigs.cu`` compiled from its source by ``oracle/build_ref.py``; this test
calls both libraries on the same device tensors (golden-case inputs and seeded scenes).
"""
import numpy as np
import pytest
import torch

from blast3r_b200 import cujac
from blast3r_b200.synthetic import make_scene
from oracle import build_ref
from tests.helpers import TOL_OBS, golden_files, load_golden, rel_err, scene_inputs, to_cuda

pytestmark = pytest.mark.gpu

REF = None


def ref_ext():
    global REF
    if REF is None:
        REF = build_ref.load_built()
    if REF is None:
        pytest.skip('reference extension not built (oracle/_ref)')
    return REF


CASES = [('golden', p) for p in golden_files()] + [('scene', 0), ('scene', 3), ('scene', 1)]


def _inputs(case):
    if case[0] == 'golden':
        inp, opts, _ = load_golden(case[1])
        return inp, opts
    sc = make_scene(case[1], n_imgs=40 if case[1] == 1 else None, n_tracks=4000 if case[1] == 1 else None)
    return scene_inputs(sc), dict(sc.options)


def _ids(c):
    return c[1].split('golden_')[-1][:-4] if c[0] == 'golden' else f'cfg{c[1]}'


@pytest.mark.parametrize('case', CASES, ids=_ids)
def test_residuals_match_reference_kernel(case):
    ext = ref_ext()
    inp, opts = _inputs(case)
    t = to_cuda(inp)
    is_log = opts['depth_mode'] == 'log'
    args = (t['infos'], t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'], t['pids'], t['pix2d'],
            t['pix2d_std'], t['pix2d_dep'], is_log, opts['weight_z'], opts['pnorm'], opts['clip_pix_err'],
            opts['huber_delta'], 1e-16)
    want = ext.residuals_with_rigs(*args).cpu().numpy()
    got = cujac.residuals_with_rigs(*args).cpu().numpy()
    for j in range(9):
        assert rel_err(got[:, j], want[:, j]) < TOL_OBS, j


@pytest.mark.parametrize('f64', [False, True])
@pytest.mark.parametrize('case', CASES, ids=_ids)
def test_jacobians_match_reference_kernel(case, f64):
    ext = ref_ext()
    inp, opts = _inputs(case)
    t = to_cuda(inp)
    is_log = opts['depth_mode'] == 'log'
    args = (t['infos'], t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'], t['pids'], t['pix2d_std'],
            t['pix2d_dep'], is_log)
    want = ext.jacobians_with_rigs(*args, f64)
    got = cujac.jacobians_with_rigs(*args, float64=f64)
    tol = 1e-12 if f64 else TOL_OBS
    for g, w in zip(got, want):
        g, w = g.cpu().numpy(), w.cpu().numpy()
        for r in range(w.shape[1]):
            for c in range(w.shape[2]):
                if np.abs(w[:, r, c]).max() > 0:
                    assert rel_err(g[:, r, c], w[:, r, c]) < tol, (r, c)


def test_chol_bcoo_einsum_match_reference_kernels():
    ext = ref_ext()
    g = torch.Generator().manual_seed(5)
    A = torch.randn(512, 3, 3, generator=g, dtype=torch.float64)
    A = (A @ A.transpose(1, 2) + 0.3 * torch.eye(3, dtype=torch.float64)).cuda()
    b = torch.randn(512, 3, generator=g, dtype=torch.float64).cuda()
    assert rel_err(cujac.chol3x3_solve(A, b).cpu().numpy(), ext.chol3x3_solve(A, b, 1e-12).cpu().numpy()) < 1e-12
    blocks = torch.randn(200, 3, 6, generator=g, dtype=torch.float64).cuda()
    rows = torch.randint(0, 20, (200,), generator=g).cuda()
    cols = torch.randint(0, 30, (200,), generator=g).cuda()
    x = torch.randn(30 * 6, generator=g, dtype=torch.float64).cuda()
    assert rel_err(cujac.blockcoo_matvec(blocks, rows, cols, x, 20, 30).cpu().numpy(),
                   ext.blockcoo_matvec(blocks, rows, cols, x, 20, 30, False).cpu().numpy()) < 1e-12
    # (I, J, K) = (2, 6, 3): one of the reference's instantiated shapes (sfm_jacobian_rigs.cu:997-1004);
    # outside them the reference op throws, which ended the whole process here
    L = torch.randn(300, 3, 2, generator=g, dtype=torch.float64).cuda()
    R = torch.randn(300, 3, 6, generator=g, dtype=torch.float64).cuda()
    assert rel_err(cujac.fused_einsum_bki_bkj(L, R).cpu().numpy(), ext.fused_einsum_bki_bkj(L, R).cpu().numpy()) < 1e-12
