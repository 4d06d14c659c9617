"""GPU: plans built incrementally for the online track merge (b3r_plan_append) linearize like
plans built from scratch and like the CPU oracle.

The online loop (inference/pipeline.py:196-224) merges every new frame's tracks into the
problem (``old | new``, inference/tracks.py:96-117) and runs BA on it.  Frame by frame, the
appended plan's S, b and preconditioner equal the fresh plan's up to summation order (old and
new tracks' pairs are visited in another order), and the oracle's within the accumulated
tolerance; one LM step per frame through the solver's plan cache, which appends by itself,
lands where the same step with fresh plans lands.
"""
import numpy as np
import pytest
import torch

from blast3r_b200 import ba_solver as BS
from blast3r_b200.engine import lm_step
from blast3r_b200.plan import BAPlan
from blast3r_b200.synthetic import OnlineSequence, make_scene
from oracle import ba_oracle as O
from tests.helpers import TOL_ACC, TOL_B, rel_err, scene_inputs, to_cuda

pytestmark = pytest.mark.gpu


def _linearize(plan, t, opts):
    lo = BAPlan.lin_opts(weight_z=opts['weight_z'], pnorm=opts['pnorm'], max_pix_err=opts['clip_pix_err'],
                         huber_delta=opts['huber_delta'])
    p = plan.params(t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'], t['pix2d_std'],
                    t['pix2d_dep'], pix2d=t['pix2d'])
    s = plan.linearize(p, lo)
    torch.cuda.synchronize()
    return s


@pytest.mark.parametrize('cfg,ni,nt,q0,q1', [(3, 32, 3000, 10, 18), (1, 40, 4000, 12, 16)])
def test_appended_plans_linearize_like_fresh_plans(cfg, ni, nt, q0, q1):
    seq = OnlineSequence(make_scene(cfg, n_imgs=ni, n_tracks=nt))
    prev = None
    for q in range(q0, q1):
        s = seq.frame(q)
        inp = scene_inputs(s)
        t = to_cuda(inp)
        app = BAPlan(t['infos'], t['pids'], s.n_cams, s.n_nodes, s.n_tracks, s.n_zcf, retain=True, base=prev)
        fresh = BAPlan(t['infos'], t['pids'], s.n_cams, s.n_nodes, s.n_tracks, s.n_zcf)
        a, b = _linearize(app, t, s.options), _linearize(fresh, t, s.options)
        Sa = a.to_dense().cpu().numpy()
        Sb = b.to_dense().cpu().numpy()
        assert rel_err(Sa, Sb) < TOL_ACC
        assert rel_err(a.b.cpu().numpy(), b.b.cpu().numpy()) < TOL_B
        assert rel_err(a.precond.cpu().numpy(), b.precond.cpu().numpy()) < TOL_ACC
        if q in (q0 + 1, q1 - 1):
            want = O.linearize(inp, s.options, dtype=np.float64, residual_dtype=np.float32)
            assert rel_err(Sa, want['S']) < TOL_ACC
            assert rel_err(a.b.cpu().numpy(), want['b']) < TOL_B
        # the point back-substitution of the appended plan (its own track order)
        dc = torch.linspace(-1e-3, 1e-3, app.n_cam_params, device='cuda')
        assert rel_err(a.backsub(dc).cpu().numpy(), b.backsub(dc).cpu().numpy()) < TOL_ACC
        prev = app


def _online_lm(seq, frames):
    out = []
    for q in frames:
        s = seq.frame(q)
        t = to_cuda(scene_inputs(s))
        o = s.options
        upd, st = lm_step(t['infos'], t['pids'], t['pix2d'], t['pix2d_std'], t['pix2d_dep'], t['K'], t['P_rig2cam'],
                          t['P_w2rig'], t['z_coefs'], t['pts3d'], pnorm=o['pnorm'], clip_pix_err=o['clip_pix_err'],
                          huber_delta=o['huber_delta'], weight_z=o['weight_z'], dtype=torch.float64)
        plan = BS._PLAN_CACHE[-1][2]
        out.append((float(st.init_loss), float(st.new_loss), upd['pts3d'].cpu().numpy(),
                    upd['P_w2rig'].cpu().numpy(), plan.appended))
    return out


def test_online_lm_steps_through_appended_plans():
    seq = OnlineSequence(make_scene(3, n_imgs=24, n_tracks=2000))
    frames = list(range(8, 13))
    keep = BS.INCREMENTAL_MAX_OBS
    try:
        BS._PLAN_CACHE.clear()
        inc = _online_lm(seq, frames)
        BS._PLAN_CACHE.clear()
        BS.INCREMENTAL_MAX_OBS = 0            # every plan from scratch
        ref = _online_lm(seq, frames)
    finally:
        BS.INCREMENTAL_MAX_OBS = keep
        BS._PLAN_CACHE.clear()
    assert [r[4] for r in inc] == [False] + [True] * (len(frames) - 1)
    assert not any(r[4] for r in ref)
    for a, b in zip(inc, ref):
        assert abs(a[0] - b[0]) <= 1e-5 * abs(b[0])
        assert abs(a[1] - b[1]) <= 1e-3 * abs(b[0])
        assert rel_err(a[2], b[2]) < 2e-3
        assert rel_err(a[3], b[3]) < 2e-3
