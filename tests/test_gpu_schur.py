"""GPU parity of the fused linearization + Schur assembly (C ABI part 2).

* against the golden fixtures made by the reference's own solver (S, b, damped diag A);
* against the CPU oracle on seeded scenes of every configuration generator;
* the general path (residuals and weights passed in) against the recomputing path;
* point back-substitution against the oracle;
* at larger sizes, size-independent properties: S v against the implicit Schur operator
  A v - B D^-1 C v built from the explicit Jacobian op, and b against J^T W r.
"""
import numpy as np
import pytest
import torch

from blast3r_b200 import cujac
from blast3r_b200.plan import BAPlan
from blast3r_b200.synthetic import make_scene
from oracle import ba_oracle as O
from tests.helpers import TOL_ACC, TOL_B, TOL_OBS, golden_files, load_golden, rel_err, scene_inputs, to_cuda

pytestmark = pytest.mark.gpu


def run_plan(inp, opts, recompute=True):
    t = to_cuda(inp)
    plan = BAPlan(t['infos'], t['pids'], len(inp['K']), len(inp['P_w2rig']), len(inp['pts3d']),
                  inp['pix2d_dep'].shape[1], optim_K=opts.get('optim_K', True), optim_P=opts.get('optim_P', True),
                  optim_Z=opts.get('optim_Z', True), optim_X=opts.get('optim_X', True))
    is_log = opts.get('depth_mode', 'log') == 'log'
    lo = BAPlan.lin_opts(is_depth_log=is_log, weight_z=opts['weight_z'], pnorm=opts['pnorm'],
                         max_pix_err=opts['clip_pix_err'], huber_delta=opts['huber_delta'],
                         no_grad_f_from_rz=opts.get('no_grad_f_from_rz', False), optim_Z0=opts.get('optim_Z0', True),
                         optim_Z_1st_cam=opts.get('optim_Z_1st_cam', True))
    if recompute:
        p = plan.params(t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'], t['pix2d_std'],
                        t['pix2d_dep'], pix2d=t['pix2d'])
    else:
        res = cujac.residuals_with_rigs(t['infos'], t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'],
                                        t['pids'], t['pix2d'], t['pix2d_std'], t['pix2d_dep'], is_log,
                                        opts['weight_z'], opts['pnorm'], opts['clip_pix_err'], opts['huber_delta'])
        r, _, w = res.view(-1, 3, 3).unbind(dim=1)
        p = plan.params(t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'], t['pix2d_std'],
                        t['pix2d_dep'], residuals=r, w_pts=w)
    sys_ = plan.linearize(p, lo)
    torch.cuda.synchronize()
    return plan, sys_


@pytest.mark.parametrize('path', golden_files(), ids=lambda p: p.split('golden_')[-1][:-4])
def test_schur_matches_reference_solver(path):
    inp, opts, ref = load_golden(path)
    plan, s = run_plan(inp, opts)
    S = s.to_dense().cpu().numpy()
    assert S.shape == ref['f64_S'].shape
    assert rel_err(S, ref['f64_S']) < TOL_ACC
    assert rel_err(s.b.cpu().numpy(), ref['f64_b']) < TOL_B
    # reference preconditioner: damped diag(A) clamped at 1e-12 (ba_solver.py:191-192)
    assert rel_err(s.precond.cpu().numpy(), np.maximum(ref['f64_diagA'], 1e-12)) < TOL_ACC
    # the S pattern holds exactly the reference's non-zero blocks (the oracle test pins the
    # oracle pattern to them)
    lay = O.Layout(inp['infos'], inp['pids'], len(inp['K']), len(inp['P_w2rig']), len(inp['pts3d']),
                   inp['pix2d_dep'].shape[1], opts['optim_K'], opts['optim_P'], opts['optim_Z'], opts['optim_X'])
    rows, cols = plan.pattern()
    assert np.array_equal(np.stack([rows, cols], 1), O.s_pattern(lay))


@pytest.mark.parametrize('path', golden_files(), ids=lambda p: p.split('golden_')[-1][:-4])
def test_general_path_equals_recompute(path):
    """Residuals/weights handed in (the fixture's, from the reference) vs recomputed in-kernel.

    The in-kernel IRLS weight uses the exact power law (1/rr for pnorm 1) where the
    reference residual kernel calls powf, so the two agree to a few ulps, not bitwise:
    the bound is the float32 observation tolerance."""
    inp, opts, _ = load_golden(path)
    _, a = run_plan(inp, opts, recompute=True)
    _, b = run_plan(inp, opts, recompute=False)
    assert rel_err(b.S_vals.cpu().numpy(), a.S_vals.cpu().numpy()) < TOL_OBS
    assert rel_err(b.b.cpu().numpy(), a.b.cpu().numpy()) < TOL_OBS


SCENES = [(0, None, None), (3, None, None), (1, 60, 6000), (2, 80, 8000), (4, 60, 6000)]


@pytest.mark.parametrize('cfg,ni,nt', SCENES, ids=lambda v: str(v))
def test_schur_matches_oracle(cfg, ni, nt):
    sc = make_scene(cfg, n_imgs=ni, n_tracks=nt)
    inp, opts = scene_inputs(sc), dict(sc.options)
    want = O.linearize(inp, opts, dtype=np.float64, residual_dtype=np.float32)
    _, s = run_plan(inp, opts)
    assert rel_err(s.to_dense().cpu().numpy(), want['S']) < TOL_ACC
    assert rel_err(s.b.cpu().numpy(), want['b']) < TOL_B
    assert rel_err(s.diagA.cpu().numpy() + want['lam'], want['diagA']) < TOL_ACC


@pytest.mark.parametrize('cfg', [0, 3])
def test_backsub_matches_oracle(cfg):
    sc = make_scene(cfg)
    inp, opts = scene_inputs(sc), dict(sc.options)
    want = O.linearize(inp, opts, dtype=np.float64, residual_dtype=np.float32)
    plan, s = run_plan(inp, opts)
    rng = np.random.default_rng(cfg)
    dc = rng.normal(size=plan.n_cam_params) * 1e-3
    dp = s.backsub(torch.from_numpy(dc).float().cuda()).cpu().numpy().reshape(-1, 3)
    # oracle: delta_p = D^-1 (g_p - C dc), C = Hpc per observation summed per track
    lay = want['layout']
    Jc = O.camera_jacobian(want['J_cam'], want['J_zcf'], lay)
    W = np.clip(want['residuals'][:, 6:9].astype(np.float32), np.float32(1e-6), np.float32(1e6)).astype(np.float64)
    Hpc = np.einsum('nki,nk,nkj->nij', want['J_pts'], W, Jc)
    idx = want['idx']
    dco = np.where(idx >= 0, dc[np.maximum(idx, 0)], 0.0)
    Cdc = np.zeros((lay.nX, 3))
    np.add.at(Cdc, lay.tX, np.einsum('nij,nj->ni', Hpc, dco))
    ref = O.chol3x3_solve(want['Hpp'], want['g_p'] - Cdc)
    assert rel_err(dp, ref) < 1e-4


@pytest.mark.parametrize('cfg,ni,nt', [(1, None, None), (2, None, None), (4, 2000, 2_000_000)],
                         ids=['cfg1', 'cfg2', 'cfg4-2M-tracks'])
def test_schur_operator_property_full_size(cfg, ni, nt):
    """S v == A v - B D^-1 C v with A, B, C, D built from the explicit Jacobian op (fp64),
    and b == g_c - B D^-1 g_p, on the full configuration (size-independent check); for the
    depth-stitch configuration on 2M tracks (12M observations) of its generator."""
    sc = make_scene(cfg, n_imgs=ni, n_tracks=nt)
    inp, opts = scene_inputs(sc), dict(sc.options)
    plan, s = run_plan(inp, opts)
    t = to_cuda(inp)
    res = cujac.residuals_with_rigs(t['infos'], t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'],
                                    t['pids'], t['pix2d'], t['pix2d_std'], t['pix2d_dep'], True, opts['weight_z'],
                                    opts['pnorm'], opts['clip_pix_err'], opts['huber_delta'])
    r, _, w = [x.contiguous() for x in res.view(-1, 3, 3).unbind(dim=1)]
    Jc8, Jz, Jp = cujac.jacobians_with_rigs(t['infos'], t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'],
                                            t['pts3d'], t['pids'], t['pix2d_std'], t['pix2d_dep'], True, float64=True)
    n, C = Jz.shape[0], Jz.shape[2]
    W = w.clamp(1e-6, 1e6).double()
    Jc = torch.zeros(n, 3, 8 + C, dtype=torch.float64, device='cuda')
    Jc[:, :, :8] = Jc8
    Jc[:, 2, 8:] = Jz[:, 0]
    if not opts['optim_K']:                 # disabled types keep their columns with a zero J
        Jc[:, :, :2] = 0
    if not opts['optim_P']:
        Jc[:, :, 2:8] = 0
    img = torch.searchsorted(t['infos'][0].long(), torch.arange(n, device='cuda'), right=True)
    cam, node = t['infos'][2].long()[img], t['infos'][1].long()[img]
    nbK, nbP = plan.info.nb_K, plan.info.nb_P
    cols = torch.cat([2 * cam[:, None] + torch.arange(2, device='cuda'),
                      plan.info.off_P + 6 * node[:, None] + torch.arange(6, device='cuda'),
                      plan.info.off_Z + C * img[:, None] + torch.arange(C, device='cuda')], 1)
    pid = t['pids'].long()
    T = len(inp['pts3d'])
    Hpp = torch.zeros(T, 3, 3, dtype=torch.float64, device='cuda').index_add_(0, pid, torch.einsum('nki,nk,nkj->nij', Jp, W, Jp))
    lam_p = 1e-12 * torch.diagonal(Hpp, dim1=1, dim2=2).max()
    Hpp = Hpp + lam_p * torch.eye(3, dtype=torch.float64, device='cuda')
    Hpc = torch.einsum('nki,nk,nkj->nij', Jp, W, Jc)
    g = (W * r.double())
    g_c = torch.zeros(plan.n_cam_params, dtype=torch.float64, device='cuda').index_add_(0, cols.reshape(-1), torch.einsum('nkj,nk->nj', Jc, g).reshape(-1))
    g_p = torch.zeros(T, 3, dtype=torch.float64, device='cuda').index_add_(0, pid, torch.einsum('nkj,nk->nj', Jp, g))
    Dinv = torch.linalg.inv(Hpp)
    gen = torch.Generator(device='cuda').manual_seed(0)
    v = torch.randn(plan.n_cam_params, dtype=torch.float64, device='cuda', generator=gen)

    def schur_mv(v):
        Jv = torch.einsum('nkj,nj->nk', Jc, v[cols])
        Av = torch.zeros_like(v).index_add_(0, cols.reshape(-1), torch.einsum('nkj,nk->nj', Jc, W * Jv).reshape(-1))
        Cv = torch.zeros(T, 3, dtype=torch.float64, device='cuda').index_add_(0, pid, torch.einsum('nij,nj->ni', Hpc, v[cols]))
        DCv = torch.einsum('tij,tj->ti', Dinv, Cv)
        BDCv = torch.zeros_like(v).index_add_(0, cols.reshape(-1), torch.einsum('nij,ni->nj', Hpc, DCv[pid]).reshape(-1))
        return Av - BDCv

    lam = s.precond.double() - s.diagA.double()          # damping added to diag(S)
    want = schur_mv(v) + lam * v
    got = s.matvec(v)
    assert rel_err(got.cpu().numpy(), want.cpu().numpy()) < TOL_ACC
    Dg = torch.einsum('tij,tj->ti', Dinv, g_p)
    b_want = g_c - torch.zeros_like(g_c).index_add_(0, cols.reshape(-1), torch.einsum('nij,ni->nj', Hpc, Dg[pid]).reshape(-1))
    assert rel_err(s.b.cpu().numpy(), b_want.cpu().numpy()) < TOL_B


@pytest.mark.parametrize('C,z0', [(1, True), (2, False), (17, True)])
def test_schur_other_channel_counts(C, z0):
    """Depth-channel counts of the reference's phase schedules (n_zcfs 1 -> 2 channels with
    channel 0 frozen; 17 channels), each a separate kernel instantiation."""
    sc = make_scene(0, n_imgs=12, n_tracks=600, seed=21 + C)
    inp, opts = scene_inputs(sc), dict(sc.options)
    rng = np.random.default_rng(C)
    dep = inp['pix2d_dep']
    if C <= dep.shape[1]:
        dep = dep[:, :C]
    else:
        dep = np.concatenate([dep, rng.normal(0, 0.1, size=(len(dep), C - dep.shape[1])).astype(np.float32)], 1)
    inp['pix2d_dep'] = np.ascontiguousarray(dep)
    inp['z_coefs'] = np.ascontiguousarray(inp['z_coefs'][:, :1].repeat(C, 1) * (np.arange(C) == 0))
    opts['optim_Z0'] = z0
    want = O.linearize(inp, opts, dtype=np.float64, residual_dtype=np.float32)
    plan, s = run_plan(inp, opts)
    assert rel_err(s.to_dense().cpu().numpy(), want['S']) < TOL_ACC
    assert rel_err(s.b.cpu().numpy(), want['b']) < TOL_B


def test_depth_stitch_plan_matches_oracle_large():
    """The depth-stitch passes (focal and pose types off: only zcf blocks in S) on a
    configs[4]-structured scene with windows of 16 and loop-closure tracks."""
    sc = make_scene(4, n_imgs=300, n_tracks=60000)
    assert sc.meta['n_loop_tracks'] > 0
    inp, opts = scene_inputs(sc), dict(sc.options)
    want = O.linearize(inp, opts, dtype=np.float64, residual_dtype=np.float32)
    plan, s = run_plan(inp, opts)
    assert plan.info.depth_stitch == 1 and plan.info.record_floats == 8
    assert rel_err(s.to_dense().cpu().numpy(), want['S']) < TOL_ACC
    assert rel_err(s.b.cpu().numpy(), want['b']) < TOL_B
    assert rel_err(s.diagA.cpu().numpy() + want['lam'], want['diagA']) < TOL_ACC


@pytest.mark.parametrize('cfg', [1, 4])
def test_local_inputs_equal_global_inputs(cfg):
    """A shard plan fed only its own observations (obs_local) gives the same partial system
    and back-substitution as the same shard fed the global arrays."""
    sc = make_scene(cfg, n_imgs=60, n_tracks=6000)
    inp, opts = scene_inputs(sc), dict(sc.options)
    t = to_cuda(inp)
    lo = BAPlan.lin_opts(weight_z=opts['weight_z'], pnorm=opts['pnorm'], max_pix_err=opts['clip_pix_err'],
                         huber_delta=opts['huber_delta'])
    rng = (2000, 4500)
    res = []
    for local in (False, True):
        plan = BAPlan(t['infos'], t['pids'], sc.n_cams, sc.n_nodes, sc.n_tracks, sc.n_zcf, optim_K=opts['optim_K'],
                      optim_P=opts['optim_P'], track_range=rng, obs_local=local)
        rows = torch.from_numpy(plan.input_obs().astype(np.int64)).cuda()
        obs = {k: t[k][rows].contiguous() if local else t[k] for k in ('pix2d', 'pix2d_std', 'pix2d_dep')}
        p = plan.params(t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'], obs['pix2d_std'],
                        obs['pix2d_dep'], pix2d=obs['pix2d'])
        outs = plan.new_outputs()
        plan.lin_stage('points', p, lo, outs)
        plan.lin_stage('assemble', p, lo, outs)
        dp = plan.backsub(p, lo, plan.workspace(), torch.full((plan.n_cam_params,), 1e-3, device='cuda'))
        torch.cuda.synchronize()
        res.append([x.clone() for x in outs[:3]] + [outs[4].clone(), dp])
    # the same arithmetic per observation; only the order of the float atomics differs
    (S0, b0, d0, h0, p0), (S1, b1, d1, h1, p1) = res
    assert torch.equal(h0, h1)
    for a, b in ((S0, S1), (b0, b1), (d0, d1), (p0, p1)):
        assert rel_err(a.cpu().numpy(), b.cpu().numpy()) < 1e-6


@pytest.mark.parametrize('cfg,edit', [(0, None), (3, None), (4, None), (0, 'frozen-image')])
def test_linearization_objective_outputs(cfg, edit):
    """The linearization's residual and loss outputs equal the residual op's rows 0..2 and the
    sum of its Huber errors, for every observation (also those of an image whose blocks are
    all switched off, which the image-major passes do not visit)."""
    sc = make_scene(cfg, n_imgs=40 if cfg == 4 else None, n_tracks=3000 if cfg == 4 else None)
    inp, opts = scene_inputs(sc), dict(sc.options)
    t = to_cuda(inp)
    kw = {}
    if edit == 'frozen-image':          # image 3: focal shared (mono), pose and depth masked out
        mP = torch.ones(sc.n_nodes, dtype=torch.bool); mP[3] = False
        mZ = torch.ones(sc.n_imgs, dtype=torch.bool); mZ[3] = False
        kw = dict(optim_K=False, optim_P=mP, optim_Z=mZ)
    plan = BAPlan(t['infos'], t['pids'], len(inp['K']), len(inp['P_w2rig']), len(inp['pts3d']), sc.n_zcf,
                  optim_K=kw.get('optim_K', opts['optim_K']), optim_P=kw.get('optim_P', opts['optim_P']),
                  optim_Z=kw.get('optim_Z', True))
    p = plan.params(t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'], t['pix2d_std'],
                    t['pix2d_dep'], pix2d=t['pix2d'])
    lo = BAPlan.lin_opts(weight_z=opts['weight_z'], pnorm=opts['pnorm'], max_pix_err=opts['clip_pix_err'],
                         huber_delta=opts['huber_delta'])
    s = plan.linearize(p, lo, objective=True)
    full = cujac.residuals_with_rigs(t['infos'], t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'],
                                     t['pids'], t['pix2d'], t['pix2d_std'], t['pix2d_dep'], True, opts['weight_z'],
                                     opts['pnorm'], opts['clip_pix_err'], opts['huber_delta'])
    torch.cuda.synchronize()
    assert rel_err(s.residuals.cpu().numpy(), full[:, :3].t().cpu().numpy()) < TOL_OBS
    want = float(full[:, 3:6].double().sum())
    assert abs(float(s.loss_sum) - want) <= 1e-6 * abs(want)


def test_schur_entrywise_full_size_against_reference_jacobians():
    """configs[2] at full size (1,000 images, 1 M tracks, 5.84 M observations), S compared entry
    by entry (all 11,002 x 11,002 scalars) and b element by element with a float64 system built
    in torch from the reference's OWN compiled kernels: its residual/weight kernel and its
    float64 Jacobian kernel (oracle/_ref), then the Schur complement exactly as the reference
    solver forms it (ba_solver.py:123-188): W clamped, A = J_c^T W J_c, D = Hpp + lambda_p I,
    S = A - sum over same-track observation pairs Hpc_o^T D^-1 Hpc_o', b = g_c - Hpc^T D^-1 g_p.
    Nothing of this library's linearization is used on the reference side."""
    from oracle import build_ref
    ext = build_ref.load_built()
    if ext is None:
        pytest.skip('reference extension not built (oracle/_ref)')
    sc = make_scene(2)
    inp, opts = scene_inputs(sc), dict(sc.options)
    plan, s = run_plan(inp, opts)
    S_ours = s.to_dense()
    t = to_cuda(inp)
    del inp
    res = ext.residuals_with_rigs(t['infos'], t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'],
                                  t['pids'], t['pix2d'], t['pix2d_std'], t['pix2d_dep'], True, opts['weight_z'],
                                  opts['pnorm'], opts['clip_pix_err'], opts['huber_delta'], 1e-16)
    r, _, w = [x.contiguous() for x in res.view(-1, 3, 3).unbind(dim=1)]
    Jc8, Jz, Jp = ext.jacobians_with_rigs(t['infos'], t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'],
                                          t['pts3d'], t['pids'], t['pix2d_std'], t['pix2d_dep'], True, True)
    n, C = Jz.shape[0], Jz.shape[2]
    Wd = w.clamp(1e-6, 1e6).double()
    sW = Wd.sqrt()
    Jc = torch.zeros(n, 3, 8 + C, dtype=torch.float64, device='cuda')
    Jc[:, :, :8] = Jc8
    Jc[:, 2, 8:] = Jz[:, 0]
    Jcw = Jc * sW[:, :, None]
    Jpw = Jp * sW[:, :, None]
    del Jc, Jc8, Jz, Jp, res
    img = torch.searchsorted(t['infos'][0].long(), torch.arange(n, device='cuda'), right=True)
    cam, node = t['infos'][2].long()[img], t['infos'][1].long()[img]
    ncp = plan.n_cam_params
    cols = torch.cat([2 * cam[:, None] + torch.arange(2, device='cuda'),
                      plan.info.off_P + 6 * node[:, None] + torch.arange(6, device='cuda'),
                      plan.info.off_Z + C * img[:, None] + torch.arange(C, device='cuda')], 1)     # [n, 13]
    pid = t['pids'].long()
    T = sc.n_tracks
    Hpp = torch.zeros(T, 3, 3, dtype=torch.float64, device='cuda').index_add_(0, pid, torch.einsum('nki,nkj->nij', Jpw, Jpw))
    lam_p = 1e-12 * torch.diagonal(Hpp, dim1=1, dim2=2).max()
    Dinv = torch.linalg.inv(Hpp + lam_p * torch.eye(3, dtype=torch.float64, device='cuda'))
    del Hpp
    Hpc = torch.einsum('nki,nkj->nij', Jpw, Jcw)                                   # [n, 3, 13]
    sWr = sW * r.double()
    g_c = torch.zeros(ncp, dtype=torch.float64, device='cuda').index_add_(
        0, cols.reshape(-1), torch.einsum('nkj,nk->nj', Jcw, sWr).reshape(-1))
    g_p = torch.zeros(T, 3, dtype=torch.float64, device='cuda').index_add_(0, pid, torch.einsum('nkj,nk->nj', Jpw, sWr))
    Dg = torch.einsum('tij,tj->ti', Dinv, g_p)
    b_ref = g_c - torch.zeros_like(g_c).index_add_(0, cols.reshape(-1), torch.einsum('nij,ni->nj', Hpc, Dg[pid]).reshape(-1))
    err_b = rel_err(s.b.cpu().numpy(), b_ref.cpu().numpy())
    assert err_b < TOL_B, err_b
    del g_c, g_p, Dg, b_ref, Jpw
    S_ref = torch.zeros(ncp * ncp, dtype=torch.float64, device='cuda')
    W13 = cols.shape[1]

    def scatter(rows, colsb, vals):          # S_ref[rows_i, cols_j] += vals_ij (flattened)
        S_ref.index_add_(0, (rows[..., :, None] * ncp + colsb[..., None, :]).reshape(-1), vals.reshape(-1))
    for a in range(0, n, 1 << 20):         # A = sum_o J_c^T W J_c
        sl = slice(a, a + (1 << 20))
        scatter(cols[sl], cols[sl], torch.einsum('nki,nkj->nij', Jcw[sl], Jcw[sl]))
    del Jcw
    Z = torch.einsum('nij,njk->nik', Dinv[pid], Hpc)                                # D^-1 Hpc
    del Dinv
    order = torch.argsort(pid, stable=True)
    cnt = torch.bincount(pid, minlength=T)
    start = torch.cumsum(cnt, 0) - cnt
    for L in torch.unique(cnt).tolist():   # fill-in: every same-track pair (o, o'), o == o' included
        if L == 0:
            continue
        trk = torch.nonzero(cnt == L).squeeze(1)
        step = max(1, (1 << 26) // (L * L * W13 * W13))
        for c0 in range(0, len(trk), step):
            idx = order[start[trk[c0:c0 + step]][:, None] + torch.arange(L, device='cuda')]   # [m, L]
            P = torch.einsum('mari,mbrj->mabij', Hpc[idx], Z[idx])                          # [m, L, L, 13, 13]
            ci = cols[idx]
            S_ref.index_add_(0, (ci[:, :, None, :, None] * ncp + ci[:, None, :, None, :]).reshape(-1), -P.reshape(-1))
    S_ref = S_ref.view(ncp, ncp)
    S_ref += torch.diag(s.precond.double() - s.diagA.double())      # the per-type damping lambda on diag(S)
    err = float((S_ours - S_ref).abs().max() / S_ref.abs().max())
    print(f'configs[2] full size: S max|diff| / max|S| = {err:.2e}, b {err_b:.2e}')
    assert err < TOL_ACC, err
