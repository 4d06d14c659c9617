"""Host-side logic of the GaussNewtonSolver mirror, without a GPU: planning through
compute_jacobians (host-only plan on CPU tensors), plan caching, column counts after
enabling, and unpack_delta_inplace (ba_solver.py:72-108, 228-248)."""
import numpy as np
import pytest
import torch

from blast3r_b200 import ba_solver as BS
from blast3r_b200.synthetic import make_scene


def _t(sc):
    return {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in sc.lm_inputs().items()}


def test_compute_jacobians_plans_and_caches():
    sc = make_scene(0, n_imgs=8, n_tracks=100)
    t = _t(sc)
    BS._PLAN_CACHE.clear()
    s = BS.GaussNewtonSolver(sc.n_cams, sc.n_nodes, sc.n_imgs, sc.n_tracks, 'cpu')
    J = s.compute_jacobians(t['rigs'], t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'], t['pids'],
                            t['pix2d_std'], t['pix2d_dep'], is_depth_log=True)
    assert J.plan.n_cam_params == 2 + 6 * 8 + 5 * 8
    assert J.shape == (3 * sc.n_obs, J.plan.n_cam_params + 3 * sc.n_tracks)
    s2 = BS.GaussNewtonSolver(sc.n_cams, sc.n_nodes, sc.n_imgs, sc.n_tracks, 'cpu')
    J2 = s2.compute_jacobians(t['rigs'], t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'],
                              t['pids'].clone(), t['pix2d_std'], t['pix2d_dep'], is_depth_log=True)
    assert J2.plan is J.plan                 # same structure (contents, not address) -> same plan
    sc3 = make_scene(0, n_imgs=8, n_tracks=100, seed=5)
    t3 = _t(sc3)
    J3 = s2.compute_jacobians(t3['rigs'], t3['K'], t3['P_rig2cam'], t3['P_w2rig'], t3['z_coefs'], t3['pts3d'],
                              t3['pids'], t3['pix2d_std'], t3['pix2d_dep'], is_depth_log=True)
    assert J3.plan is not J.plan


def test_masks_and_unpack_delta():
    sc = make_scene(3, n_imgs=8, n_tracks=150)
    t = _t(sc)
    mP = torch.ones(sc.n_nodes, dtype=torch.bool)
    mP[[0, 3]] = False
    s = BS.GaussNewtonSolver(sc.n_cams, sc.n_nodes, sc.n_imgs, sc.n_tracks, 'cpu')
    J = s.compute_jacobians(t['rigs'], t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'], t['pids'],
                            t['pix2d_std'], t['pix2d_dep'], is_depth_log=True, optim_P=mP, optim_X=False)
    assert s.nodes.n == 6 and list(s.nodes.true_idxs) == [1, 2, 4, 5, 6, 7]
    n = 2 * 8 + 6 * 6 + 5 * 8 + 3 * sc.n_tracks
    assert J.plan.n_cam_params + 3 * J.plan.info.n_points == n
    delta = torch.arange(n, dtype=torch.float32)
    dK, dP, dZ, dX = s.unpack_delta_inplace(delta)
    assert dK.shape == (8, 2) and dP.shape == (8, 6) and dZ.shape == (8, 5) and dX.shape == (sc.n_tracks, 3)
    assert (dP[0] == 0).all() and (dP[3] == 0).all() and dP[1, 0] == 16


def test_plan_cache_sees_a_reordering_of_pids():
    """Swapping two observations' track ids (positions 1,000,003 apart, which a weighted-sum
    fingerprint modulo 1,000,003 would not see) must give a new plan."""
    sc = make_scene(2, n_imgs=100, n_tracks=180000)
    assert sc.n_obs > 1000010
    t = _t(sc)
    BS._PLAN_CACHE.clear()
    s = BS.GaussNewtonSolver(sc.n_cams, sc.n_nodes, sc.n_imgs, sc.n_tracks, 'cpu')
    args = (t['rigs'], t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'])
    J = s.compute_jacobians(*args, t['pids'], t['pix2d_std'], t['pix2d_dep'], is_depth_log=True)
    pids = t['pids'].clone()
    i = int(np.nonzero(sc.pids[:-1000003] != sc.pids[1000003:])[0][0])
    pids[i], pids[i + 1000003] = t['pids'][i + 1000003], t['pids'][i]
    J2 = s.compute_jacobians(*args, pids, t['pix2d_std'], t['pix2d_dep'], is_depth_log=True)
    assert J2.plan is not J.plan
    J3 = s.compute_jacobians(*args, t['pids'].clone(), t['pix2d_std'], t['pix2d_dep'], is_depth_log=True)
    assert J3.plan is J.plan
    t['pids'][i] = t['pids'][i + 1000003]      # an in-place edit of the tensor the plan was built from
    J4 = s.compute_jacobians(*args, t['pids'], t['pix2d_std'], t['pix2d_dep'], is_depth_log=True)
    assert J4.plan is not J.plan


@pytest.mark.parametrize('scale', [0.0, 1e-7, 1e-4, 1e-3, 2e-3, 0.1, 1.0, 3.0])
def test_exp_se3_equals_matrix_exponential(scale):
    """cujac.exp_se3 (closed form) against the reference's torch.matrix_exp(hat_se3(xi))
    (extensions/cujac/__init__.py:56-58), float64, across the small-angle series threshold."""
    from blast3r_b200.cujac import exp_se3, hat_se3
    g = torch.Generator().manual_seed(7)
    xi = torch.randn(300, 6, dtype=torch.float64, generator=g) * scale
    want = torch.matrix_exp(hat_se3(xi))
    assert (exp_se3(xi) - want).abs().max().item() < 1e-13
    assert exp_se3(xi.float()).dtype == torch.float32


def test_plan_cache_sees_in_place_edits_of_the_same_tensor():
    """The same structure tensors, unmodified, reuse the plan without a comparison; an in-place
    edit of them (here two observations of an image swapped) gets a new plan, and so does an
    edit inside inference mode, whose tensors keep no modification counter."""
    sc = make_scene(0, n_imgs=8, n_tracks=100)
    orig = sc.pids.copy()
    t = _t(sc)                       # shares memory with sc's arrays
    BS._PLAN_CACHE.clear()
    try:
        p1 = BS.get_plan(t['rigs'], t['pids'], sc.n_cams, sc.n_nodes, sc.n_tracks, sc.n_zcf, device='cpu')
        assert BS.get_plan(t['rigs'], t['pids'], sc.n_cams, sc.n_nodes, sc.n_tracks, sc.n_zcf, device='cpu') is p1
        t['pids'][[0, 1]] = t['pids'][[1, 0]].clone()
        p2 = BS.get_plan(t['rigs'], t['pids'], sc.n_cams, sc.n_nodes, sc.n_tracks, sc.n_zcf, device='cpu')
        assert p2 is not p1
        with torch.inference_mode():
            pids = torch.from_numpy(orig.copy())
            p3 = BS.get_plan(t['rigs'], pids, sc.n_cams, sc.n_nodes, sc.n_tracks, sc.n_zcf, device='cpu')
            assert p3 is p1
            pids[[0, 1]] = pids[[1, 0]].clone()
            assert BS.get_plan(t['rigs'], pids, sc.n_cams, sc.n_nodes, sc.n_tracks, sc.n_zcf, device='cpu') is p2
    finally:
        BS._PLAN_CACHE.clear()
