"""Levenberg-Marquardt on the B200 solver: the reference's ``lm_step``
(inference/engine.py:206-334) with the same arguments, update rules, line search and return
values, running ``blast3r_b200.ba_solver`` and the library's residual op, and its phase loop
``bundle_adjustment`` (engine.py:405-503) on top of it, taking the reference's own rig and
track objects.

The dense tangent prior (``weight_tan > 0``, engine.py:15-158, 253-299) runs on the
library's ``b3r_tangent_prior`` kernel (``blast3r_b200.prior``).  With
``recompute_residuals`` (default) the linearization recomputes residuals and weights
in-kernel instead of reading the objective's tensors (same device function, same values).
"""
from collections import namedtuple

import torch

from . import _lib as L
from .ba_solver import GaussNewtonSolver
from .cujac import exp_se3, residual_loss, residuals_with_rigs as residual_func
from .prior import dense_tangent_prior_terms

BA_Status = namedtuple('BA_Status', 'init_loss, init_residuals, new_loss, new_residuals')


def shape_of(tensor, is_contiguous=True, finite=None):
    """Input checks of the reference (engine.py:340-344).  Given a list `finite`, the
    all-finite flag goes into it as a device tensor, for the caller to check for every input
    with one host synchronisation, instead of being checked here."""
    assert tensor.dtype in (torch.float32, torch.int32)
    if is_contiguous:
        assert tensor.is_contiguous()
    if finite is None:
        assert tensor.isfinite().all()
    else:
        finite.append(tensor.isfinite().all())
    return tensor.shape


def update_K(K0, delta_focal, min_f=100):
    """Focal update with the reference's clipping (engine.py:347-354)."""
    dfx, dfy = delta_focal.T
    K = K0.clone()
    K[:, 0, 0] -= dfx
    K[:, 1, 1] -= dfy
    K[:, 0, 0].clip_(min=min_f)
    K[:, 1, 1].clip_(min=min_f)
    return K


def reproj_score(res):
    """Mean of the best 80% reprojection errors ||res[i, :2]|| (engine.py:357-361), on the
    device without a sort: the library's exact radix select (b3r_reproj_score) finds the
    k-th smallest error and sums the ones below it.  `res` is an (n, >=2) float32 CUDA tensor
    of any strides (the residual op's output is a component-major view).  Returns a 0-d
    device tensor."""
    assert res.is_cuda and res.dtype == torch.float32 and res.dim() == 2, 'an (n, >=2) float32 CUDA tensor'
    n = res.shape[0]
    work = torch.empty(int(L.lib().b3r_reproj_score_work_bytes(n)) // 4 + 64, dtype=torch.float32, device=res.device)
    ptr = work.data_ptr()
    ptr += (-ptr) % 256
    out = torch.empty(1, dtype=torch.float32, device=res.device)
    L.call('b3r_reproj_score', res.data_ptr(), n, max(res.stride(0), 1), max(res.stride(1), 1), ptr,
           out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    return out[0]


def line_search(objective, K, P_w2rig, z_coefs, pts3d, delta, delta_K, delta_P, delta_zcf, delta_pts, init_loss,
                init_residuals, min_reproj=0.01, min_loss_delta=1e-4, verbose=False):
    """The reference's step-size search (engine.py:303-333): scales 1, 1/2, 1/4, 1/8, 1/64,
    1/512, 1/4096, 0 of `delta` (whose views are delta_K, delta_P, delta_zcf, delta_pts), the
    first that lowers the loss without collapsing the reprojection residual.  Returns
    (update, new_loss, new_residuals)."""
    update = dict()
    last_a = 1
    new_loss, new_residuals = init_loss, init_residuals
    for a in [0.5, 0.25, 0.125, 1 / 64, 1 / 512, 1 / 4096, 0]:
        update['K'] = update_K(K, delta_K)
        update['P_w2rig'] = (exp_se3(-delta_P) @ P_w2rig).contiguous()
        update['z_coefs'] = (z_coefs - delta_zcf).contiguous()
        update['pts3d'] = (pts3d - delta_pts).contiguous()
        new_loss, new_residuals, _ = objective(**update)
        # the reference's NaN fallback, loss margin and comparison, on the device, read back
        # with the score in one synchronisation
        # On a NaN loss the reference binds new_loss to the init_loss tensor itself, so its
        # in-place margin raises init_loss too and every later trial is compared with the
        # raised value (engine.py:316-318); the same here, in place on init_loss.
        isnan = new_loss.isnan()
        init_loss.add_(torch.where(isnan, min_loss_delta, 0.0).to(init_loss.dtype))
        new_loss = torch.where(isnan, init_loss, new_loss + min_loss_delta)
        was_nan, lower, new_reproj = torch.stack([isnan.float(), (new_loss < init_loss).float(),
                                                  reproj_score(new_residuals)]).tolist()
        if was_nan and verbose:
            print('Warning: loss is NaN')
        degenerate = new_reproj < min_reproj
        if degenerate and verbose:
            print(f'Rejecting step: reprojection residual collapsed to {new_reproj:.2e}')
        if lower and not degenerate:
            break
        delta *= a / last_a          # scales (delta_K, ..., delta_pts): they are views of delta
        last_a = a
    else:
        if verbose:
            print('Warning: loss is not decreasing')
    return update, new_loss, new_residuals


def lm_step(rigs, pids, pix2d, pix2d_std, pix2d_dep, K, P_rig2cam, P_w2rig, z_coefs, pts3d, depth_mode='log',
            pnorm=1, clip_pix_err=100, huber_delta=0.5, min_reproj=0.01, dampen=1e-12, min_loss_delta=1e-4,
            weight_z=1, log_depth_maps=None, conf=None, pts3d_ref=None, weight_tan=0.0, tan_stride=4,
            normalize_tangents=True, optim_K=True, optim_Z=True, optim_P=True, optim_X=True, optim_Z0=True,
            recompute_residuals=True, verbose=False, **ba_options):
    """One Levenberg-Marquardt step (engine.py:206-334): residuals, linearization + Schur
    solve, back-substitution, then the line search over step scales 1, 1/2, 1/4, 1/8,
    1/64, 1/512, 1/4096, 0 with the degenerate-geometry reject."""
    assert depth_mode in ('lin', 'log')
    is_depth_log = depth_mode == 'log'
    if weight_tan > 0:
        # implemented for log-depth combination only (engine.py:237-239)
        assert is_depth_log, 'tangent prior currently only implemented for depth_mode="log"'
    n_imgs = rigs.shape[1]
    fin = []                 # the inputs' all-finite flags, checked together below
    assert shape_of(rigs, finite=fin) == (3, n_imgs)
    n_cams = len(K)
    assert shape_of(K, finite=fin) == (n_cams, 3, 3)
    assert shape_of(P_rig2cam, is_contiguous=False, finite=fin) == (n_cams, 4, 4)
    n_nodes = len(P_w2rig)
    assert shape_of(P_w2rig, finite=fin) == (n_nodes, 4, 4)
    n_zcf = z_coefs.shape[1]
    assert shape_of(z_coefs, finite=fin) == (n_imgs, n_zcf)
    n_tracks = len(pts3d)
    assert shape_of(pts3d, finite=fin) == (n_tracks, 3)
    n_obs = len(pids)
    assert shape_of(pids, finite=fin) == (n_obs,)
    assert shape_of(pix2d, finite=fin) == (n_obs, 2)
    assert shape_of(pix2d_std, finite=fin) == (n_obs, 2)
    assert shape_of(pix2d_dep, finite=fin) == (n_obs, n_zcf)
    assert bool(torch.stack(fin).all()), 'non-finite input'
    assert 0 <= weight_z <= 10
    assert n_obs >= n_tracks, 'there must be more 2d kpts than tracks'
    assert huber_delta >= 0.1

    # the prior treats the intrinsics as constant within a step (engine.py:258-260)
    K_tan = K.detach()

    def objective(K, P_w2rig, pts3d, z_coefs, need_w=False):
        # the residual op's (n, 9) output is needed only for the IRLS weights that a
        # linearization without in-kernel recomputation reads; otherwise one fused pass gives
        # the loss and the residuals the line search scores (b3r_residual_loss)
        if need_w:
            residuals_, err_pts_, w_pts_ = residual_func(
                rigs, K, P_rig2cam, P_w2rig, z_coefs, pts3d, pids, pix2d, pix2d_std, pix2d_dep, is_depth_log,
                weight_z, pnorm, clip_pix_err, huber_delta).view(-1, 3, 3).unbind(dim=1)
            loss = err_pts_.mean()
        else:
            loss, residuals_ = residual_loss(rigs, K, P_rig2cam, P_w2rig, z_coefs, pts3d, pids, pix2d, pix2d_std,
                                             pix2d_dep, is_depth_log, weight_z, pnorm, clip_pix_err, huber_delta)
            w_pts_ = None
        if weight_tan > 0:
            tan_loss, _, _ = dense_tangent_prior_terms(
                rigs, K_tan, z_coefs, log_depth_maps, conf, pts3d_ref, weight_tan=float(weight_tan),
                tan_stride=int(tan_stride), optim_Z0=optim_Z0, dtype=loss.dtype, compute_gn=False,
                normalize_tangents=bool(normalize_tangents))
            loss = loss + tan_loss
        return loss, residuals_, w_pts_

    jac = GaussNewtonSolver(n_cams, n_nodes, n_imgs, n_tracks, pts3d.device, dampen=dampen, **ba_options)
    z_prior = tan_loss0 = None
    if weight_tan > 0:                 # adds only to the depth-coefficient normal equations
        tan_loss0, g_z, H_z = dense_tangent_prior_terms(
            rigs, K_tan, z_coefs, log_depth_maps, conf, pts3d_ref, weight_tan=float(weight_tan),
            tan_stride=int(tan_stride), optim_Z0=optim_Z0, dtype=jac.dtype, compute_gn=True,
            normalize_tangents=bool(normalize_tangents))
        z_prior = (H_z, g_z)
    J = jac.compute_jacobians(rigs, K, P_rig2cam, P_w2rig, z_coefs, pts3d, pids, pix2d_std, pix2d_dep,
                              optim_K=optim_K, optim_Z=optim_Z, optim_Z0=optim_Z0, optim_P=optim_P,
                              optim_X=optim_X, is_depth_log=is_depth_log,
                              pix2d=pix2d if recompute_residuals else None)
    lin_kw = dict(weight_z=weight_z, pnorm=pnorm, max_pix_err=clip_pix_err, huber_delta=huber_delta)
    # The solve is queued without reading its status back, so that the back-substitution and
    # the first line-search trial are queued while the PCG kernel runs; its status is checked
    # once the line search has synchronised anyway.
    if recompute_residuals:
        # the objective at the current parameters comes out of the linearization's own passes
        # (the same residuals and Huber errors the residual op computes)
        delta, init_loss, init_residuals = jac.solve_with_objective(J, z_prior=z_prior, lin_kw=lin_kw, wait=False)
        if tan_loss0 is not None:
            init_loss = init_loss + tan_loss0.to(init_loss.dtype)
    else:
        init_loss, init_residuals, w_pts = objective(K, P_w2rig, pts3d, z_coefs, need_w=True)
        delta = jac.solve_delta(J, init_residuals, w_pts, z_prior=z_prior, lin_kw=lin_kw, wait=False)
    delta_K, delta_P, delta_zcf, delta_pts = jac.unpack_delta_inplace(delta)

    update, new_loss, new_residuals = line_search(objective, K, P_w2rig, z_coefs, pts3d, delta, delta_K, delta_P,
                                                  delta_zcf, delta_pts, init_loss, init_residuals, min_reproj,
                                                  min_loss_delta, verbose)
    jac.check_solve()
    return update, BA_Status(init_loss, init_residuals, new_loss, new_residuals)


def iter_on(*iterators):
    """The reference's phase schedule (engine.py:364-383): every argument is a scalar or a list;
    lists of length one are broadcast, the others must share one length; yields one tuple of
    values per phase."""
    iterable = lambda it: isinstance(it, (tuple, list))   # noqa: E731
    max_len = max([len(it) for it in iterators if iterable(it)] + [1])
    its = []
    for it in iterators:
        if iterable(it):
            assert len(it) in (1, max_len), f'missing {max_len - len(it)} values for parameter={it}'
            its.append(it[0] if len(it) == 1 else it)
        else:
            its.append(it)
    for step in range(max_len):
        yield tuple(it[step] if iterable(it) else it for it in its)


def _todevice(x, device):
    if x is None:
        return None
    if isinstance(x, (list, tuple)):
        return type(x)(_todevice(v, device) for v in x)
    return x.to(device) if isinstance(x, torch.Tensor) else x


def bundle_adjustment(rigs_data, track_data, pts3d=None, z_coefs=None, max_iters=1000, pnorm=0.5, optim_P=True,
                      optim_Z=True, optim_Z0=True, optim_K=True, optim_X=True, weight_z=0.1, dense_depth=None,
                      dense_conf=None, dense_pts3d_ref=None, tangent_reg=0.0, tan_stride=4, normalize_tangents=True,
                      n_zcfs=None, no_Jfz=False, max_n_phases=-1, device='cuda', verbose=True, **other_lm_kwargs):
    """The reference's main bundle-adjustment loop (engine.py:405-503) on this library's
    ``lm_step``: the same arguments, phase schedule (scalars or per-phase lists, ``iter_on``),
    per-phase depth-channel changes (``n_zcfs``: coefficients dropped or zero-padded, the first
    log-depth channel kept and frozen unless 2 or all channels are used), the same stopping
    rule (each phase iterates until a step does not lower the loss or ``max_iters``) and the
    same return value (``rigs_data.update(K, P_rig2cam, P_w2rig, z_coefs)``, ``pts3d``).

    ``rigs_data`` and ``track_data`` are the reference's ``RigsData`` and ``ObservedTracks``
    (any objects with their attributes: ``to``, ``infos``, ``K``, ``P_rig2cam``, ``P_w2rig``,
    ``depth_mode``, ``n_imgs``, ``update``, ``z_coefs_from_scale``; ``pids``, ``pix2d``,
    ``pix2d_std``, ``pix2d_dep``).  Each phase's LM iterations run in float64 solves with
    adaptive damping 1e-12, as in the reference."""
    trk = track_data.to(device)
    rig = rigs_data.to(device)
    dense_depth = _todevice(dense_depth, device)
    dense_conf = _todevice(dense_conf, device)
    dense_pts3d_ref = _todevice(dense_pts3d_ref, device)
    if z_coefs is None:
        z_coefs = rig.z_coefs_from_scale(trk)
    original_pix2d_dep = trk.pix2d_dep
    pts3d = _todevice(pts3d, device)
    assert pts3d is not None, 'the 3D points must be initialized before bundle adjustment'
    variables = dict(K=rig.K, P_rig2cam=rig.P_rig2cam, P_w2rig=rig.P_w2rig, z_coefs=z_coefs, pts3d=pts3d)
    phase_num = 0
    for pnorm, max_iters, optim_K, optim_P, optim_Z, optim_X, weight_z, n_zcfs, tangent_reg in \
            iter_on(pnorm, max_iters, optim_K, optim_P, optim_Z, optim_X, weight_z, n_zcfs, tangent_reg):
        phase_num += 1
        if phase_num > (max_n_phases % 1000):
            break
        dense_depth_use = dense_depth
        if n_zcfs is not None:               # remove or add depth coefficients for this phase
            z_coefs = variables['z_coefs']
            optim_Z0 = True
            if rig.depth_mode[:3] == 'log':
                optim_Z0 = (n_zcfs == 2) or (n_zcfs == original_pix2d_dep.shape[1])
                n_zcfs += not optim_Z0       # the first channel stays in, unoptimized
            trk.pix2d_dep = original_pix2d_dep[:, :n_zcfs].contiguous()
            if dense_depth is not None:
                assert len(dense_depth) == rig.n_imgs, 'log_depth_maps must be n_imgs x (H, W, C)'
                assert all(d.shape[-1] >= n_zcfs for d in dense_depth), \
                    'not enough dense depth channels for the requested n_zcfs'
                dense_depth_use = [d[..., :n_zcfs] for d in dense_depth]
            if n_zcfs < z_coefs.shape[1]:
                assert n_zcfs >= 1
                variables['z_coefs'] = z_coefs[:, :n_zcfs].contiguous()
            elif n_zcfs > z_coefs.shape[1]:
                assert trk.pix2d_dep.shape[1] == n_zcfs, 'not enough multi-depthmaps in the original data'
                variables['z_coefs'] = torch.cat((z_coefs, z_coefs.new_zeros((len(z_coefs), n_zcfs - z_coefs.shape[1]))),
                                                 dim=1).contiguous()
        if verbose:
            print(f"Starting phase {phase_num}, with {variables['z_coefs'].shape[1]} z-coefs.")
        it = 0
        while it < max_iters:
            update, status = lm_step(rig.infos(trk), trk.pids, trk.pix2d, trk.pix2d_std, trk.pix2d_dep, **variables,
                                     log_depth_maps=dense_depth_use, conf=dense_conf, pts3d_ref=dense_pts3d_ref,
                                     weight_tan=tangent_reg, tan_stride=tan_stride,
                                     normalize_tangents=normalize_tangents, optim_K=optim_K, optim_Z=optim_Z,
                                     optim_P=optim_P, optim_X=optim_X, optim_Z0=optim_Z0, pnorm=pnorm,
                                     weight_z=weight_z, no_grad_f_from_rz=no_Jfz, depth_mode=rig.depth_mode,
                                     dampen=1e-12, adaptive_dampen=True, dtype=torch.float64, **other_lm_kwargs)
            if verbose:
                before, after = float(reproj_score(status.init_residuals)), float(reproj_score(status.new_residuals))
                avg_focal = float((update['K'][:, 0, 0].mean() + update['K'][:, 1, 1].mean()) / 2)
                print(f'Loss at iter={it}: {float(status.init_loss):.3f} --> {float(status.new_loss):.3f}, '
                      f'reproj_score: {before:.3f} --> {after:.3f}, avg_focal={avg_focal:.2f}')
            if status.new_loss >= status.init_loss:
                break
            variables.update(update)
            it += 1
    trk.pix2d_dep = original_pix2d_dep       # restore
    pts3d = variables.pop('pts3d')
    return rigs_data.update(**variables), pts3d
