"""The allocation-free linearization entry point (b3r_linearize_schur_noalloc).

It exists for hosts that reach this library only through its C ABI and cannot allocate
device memory themselves, so they cannot provide the workspace b3r_linearize_schur asks
for; the library keeps a fixed 32 MiB workspace on each device for them.  These tests
call it through the C ABI and check it against the regular entry point, twice in a row
(the second time with moved points, so a stale workspace would show), and check that a
plan too large for the fixed workspace is refused.  This file is collected last on
purpose; it also passes when run alone in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from blast3r_b200 import _lib as L
from blast3r_b200.plan import BAPlan
from blast3r_b200.synthetic import make_scene
from tests.helpers import TOL_ACC, rel_err, scene_inputs, to_cuda

pytestmark = pytest.mark.gpu


def _plan(cfg, **kw):
    sc = make_scene(cfg, **kw)
    inp, opts = scene_inputs(sc), dict(sc.options)
    t = to_cuda(inp)
    plan = BAPlan(t['infos'], t['pids'], sc.n_cams, sc.n_nodes, sc.n_tracks, sc.n_zcf,
                  optim_K=opts['optim_K'], optim_P=opts['optim_P'])
    lo = BAPlan.lin_opts(weight_z=opts['weight_z'], pnorm=opts['pnorm'], max_pix_err=opts['clip_pix_err'],
                         huber_delta=opts['huber_delta'])
    return plan, t, lo


def _noalloc(plan, params, lo):
    S, b, dA, pc, hm = plan.new_outputs()
    out = L.Outputs(S_vals=S.data_ptr(), b=b.data_ptr(), diagA=dA.data_ptr(), precond=pc.data_ptr(),
                    hpp_max=hm.data_ptr())
    L.call('b3r_linearize_schur_noalloc', plan.handle, C.byref(params), C.byref(lo), C.byref(out),
           torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return S, b, dA, pc


def test_noalloc_matches_regular_entry_point_twice():
    plan, t, lo = _plan(3)                       # online SLAM window: fits the fixed workspace
    assert plan.info.workspace_bytes <= 32 << 20
    gen = torch.Generator(device='cuda').manual_seed(3)
    for call in range(2):
        pts = t['pts3d'] if call == 0 else (t['pts3d'] + 0.02 * torch.randn(t['pts3d'].shape, device='cuda',
                                                                           generator=gen)).contiguous()
        p = plan.params(t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], pts, t['pix2d_std'], t['pix2d_dep'],
                        pix2d=t['pix2d'])
        ref = plan.linearize(p, lo)              # regular entry point, caller-allocated workspace
        torch.cuda.synchronize()
        S, b, dA, pc = _noalloc(plan, p, lo)
        assert rel_err(S.cpu().numpy(), ref.S_vals.cpu().numpy()) < TOL_ACC
        assert rel_err(b.cpu().numpy(), ref.b.cpu().numpy()) < TOL_ACC
        assert rel_err(dA.cpu().numpy(), ref.diagA.cpu().numpy()) < TOL_ACC
        assert rel_err(pc.cpu().numpy(), ref.precond.cpu().numpy()) < TOL_ACC
        assert np.isfinite(S.cpu().numpy()).all()


def test_noalloc_refuses_plans_beyond_its_workspace():
    plan, t, lo = _plan(1)                       # ~0.5M observations: needs more than 32 MiB
    assert plan.info.workspace_bytes > 32 << 20
    p = plan.params(t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'], t['pix2d_std'],
                    t['pix2d_dep'], pix2d=t['pix2d'])
    with pytest.raises(L.B3RError, match='workspace'):
        _noalloc(plan, p, lo)
