"""Drop-in for the reference's ``GaussNewtonSolver`` (inference/ba_solver.py:20-248).

Same constructor, ``compute_jacobians``, ``solve_delta`` and ``unpack_delta_inplace``
signatures and results.  Instead of wrapping explicit Jacobians in block matrices and
running a matrix-free PCG on the implicit Schur complement (ba_solver.py:184-206), it

1. ``compute_jacobians`` returns a lazy ``Linearization`` handle (the structure is planned
   once per phase and cached: ``BAPlan``);
2. ``solve_delta`` runs the fused B200 linearization (residual, Jacobians, IRLS weights,
   per-track Hpp inversion, Schur assembly into the block-sparse S and b, per-type
   adaptive damping), then the reference's PCG on the explicit S (one cooperative device
   kernel, same iteration and stopping rule), then the point back-substitution
   delta_p = D^-1 (g_p - C delta_c).

``compute_jacobians`` accepts one extra keyword, ``pix2d``: with it the kernels recompute
residuals and weights in-kernel (identical values: one shared device function); without
it they read the ``residuals`` / ``w_pts`` handed to ``solve_delta``, as the reference does.
"""
import weakref

import torch

from . import _lib as L
from .plan import BAPlan

N_FOC = 2
N_TAU = 6


class Param:
    def __init__(self, n):
        self.n = self.true_n = n
        self.true_idxs = None


class Linearization:
    """Everything solve_delta needs to linearize at the current parameters."""

    def __init__(self, plan, tensors, flags):
        self.plan, self.tensors, self.flags = plan, tensors, flags
        self.system = None
        n = plan.n_obs
        self.shape = (3 * n, plan.n_cam_params + 3 * plan.info.n_points)


_PLAN_CACHE = []        # (key, structure tensors, plan), most recent last
# The online loop (inference/pipeline.py:212-224) runs a global BA every gba_step = 8 frames and
# a frozen single-frame BA on the others: 16 plans keep the last global BA's plans (one per
# phase) in the cache for the next global BA to extend.
_PLAN_CACHE_MAX = 16
# Plans of at most this many observations keep their host-side lists, so that the next
# structure of an online loop (the merge old | new of inference/pipeline.py:196-224) is planned
# incrementally (b3r_plan_append); the host memory they hold is about 40 B per observation plus
# 8 B per observation pair.
INCREMENTAL_MAX_OBS = 1 << 22


def _structure(rigs, pids, modes):
    """The tensors that define a plan's structure (device copies are kept for comparison)."""
    return [rigs, pids] + [m for m in modes if isinstance(m, torch.Tensor)]


def _same(a, b):
    return a.shape == b.shape and a.dtype == b.dtype and a.device == b.device and torch.equal(a, b)


def _version(t):
    """The tensor's in-place modification counter (None for inference tensors, which keep none)."""
    try:
        return t._version
    except RuntimeError:
        return None


def _saved(cur):
    """What the cache keeps of a plan's structure tensors: a copy of each, a weak reference to
    the caller's tensor and its modification counter."""
    return [(t.detach().clone(), weakref.ref(t), _version(t)) for t in cur]


def _matches(cur, saved):
    """The structure tensors hold the saved values: each is the very tensor the plan was built
    from, not modified in place since (its counter unchanged: no device comparison, no
    synchronisation), or equal element by element to the saved copy."""
    if len(cur) != len(saved):
        return False
    for a, (copy, ref, ver) in zip(cur, saved):
        if ver is not None and ref() is a and _version(a) == ver:
            continue
        if not _same(a, copy):
            return False
    return True


def _append_candidate(key, n_imgs, n_obs, n_cams, n_nodes, n_tracks, C):
    """The most recently used cached plan that kept its host state and that the new structure
    may extend (sizes only grow, same C and enable flags; b3r_plan_append checks the rest).
    The whole cache is searched: in the online loop the plans of the frozen single-frame BAs
    come between two global BAs."""
    def kinds(k):           # bool masks grow with the problem: compare flag kinds (the library
        return tuple(m if isinstance(m, bool) else 'mask' for m in k[6])   # checks each old status)
    for k, _, plan in reversed(_PLAN_CACHE):
        if not getattr(plan, 'retained', False) or k[5] != C or kinds(k) != kinds(key):
            continue
        if (plan.n_imgs <= n_imgs and plan.n_obs <= n_obs and plan.n_cams <= n_cams and plan.n_nodes <= n_nodes
                and plan.n_tracks <= n_tracks and plan.n_obs > 0):
            return plan
    return None


def get_plan(rigs, pids, n_cams, n_nodes, n_tracks, C, optim_K=True, optim_P=True, optim_Z=True,
             optim_X=True, device=None):
    """Plan for this structure, reused while the structure tensors hold the same values.

    A cached plan is returned only when ``rigs``, ``pids`` and every bool mask are the tensors
    it was built from, unmodified since, or equal element by element to the copies taken then
    (one device comparison), so a reordering or an in-place edit of the structure always gets a
    new plan.  A
    structure that extends a cached plan's the way the online loop merges tracks gets its plan
    by b3r_plan_append (incremental: only the new tracks are planned)."""
    modes = (optim_K, optim_P, optim_Z, optim_X)
    key = (tuple(rigs.shape), tuple(pids.shape), n_cams, n_nodes, n_tracks, C,
           tuple(m if isinstance(m, bool) else ('mask', tuple(m.shape)) for m in modes))
    cur = _structure(rigs, pids, modes)
    for j, (k, saved, plan) in enumerate(_PLAN_CACHE):
        if k == key and _matches(cur, saved):
            _PLAN_CACHE.append(_PLAN_CACHE.pop(j))
            return plan
    retain = len(pids) <= INCREMENTAL_MAX_OBS
    plan = None
    base = _append_candidate(key, rigs.shape[1], len(pids), n_cams, n_nodes, n_tracks, C) if retain else None
    if base is not None:
        try:
            plan = BAPlan(rigs, pids, n_cams, n_nodes, n_tracks, C, optim_K=optim_K, optim_P=optim_P,
                          optim_Z=optim_Z, optim_X=optim_X, device=device, retain=True, base=base)
        except L.B3RError:     # not an extension of that plan (tracks removed, reordered...)
            plan = None
    if plan is None:
        plan = BAPlan(rigs, pids, n_cams, n_nodes, n_tracks, C, optim_K=optim_K, optim_P=optim_P,
                      optim_Z=optim_Z, optim_X=optim_X, device=device, retain=retain)
    if len(_PLAN_CACHE) >= _PLAN_CACHE_MAX:
        _PLAN_CACHE.pop(0)
    _PLAN_CACHE.append((key, _saved(cur), plan))
    return plan


class GaussNewtonSolver:
    """Bundle-adjustment solver for a problem with existing depth estimates."""

    def __init__(self, n_cams, n_nodes, n_imgs, n_tracks, device, no_grad_f_from_rz=False, dampen=1e-12,
                 adaptive_dampen=True, dtype=torch.float32):
        self.cams = Param(n_cams)
        self.nodes = Param(n_nodes)
        self.imgs = Param(n_imgs)
        self.tracks = Param(n_tracks)
        self.device = torch.device(device)
        self.dtype = dtype
        self.dampen = dampen
        self.adaptive_dampen = adaptive_dampen
        self.no_grad_f_from_rz = no_grad_f_from_rz
        self._pcg_result = None

    def compute_jacobians(self, rigs, K, P_rig2cam, P_w2rig, z_coefs, pts3d, pids, pix2d_std, pix2d_dep,
                          is_depth_log, optim_Z_1st_cam=True, optim_Z0=True, optim_K=True, optim_Z=True,
                          optim_P=True, optim_X=True, pix2d=None):
        assert rigs.shape == (3, self.imgs.n)
        C = pix2d_dep.shape[1]
        self.n_kpts, self.n_zcf = len(pids), C
        plan = get_plan(rigs, pids, self.cams.n, self.nodes.n, self.tracks.n, C, optim_K, optim_P,
                        optim_Z, optim_X, device=self.device)
        # column counts after enabling (ba_solver.py:72-108)
        for prm, status in ((self.cams, optim_K), (self.nodes, optim_P), (self.imgs, optim_Z),
                            (self.tracks, optim_X)):
            if isinstance(status, torch.Tensor):
                idxs = status.nonzero().squeeze(-1)
                if len(idxs):
                    prm.n = len(idxs)
                    prm.true_idxs = idxs.to(self.device)
        flags = dict(is_depth_log=bool(is_depth_log), optim_Z_1st_cam=bool(optim_Z_1st_cam),
                     optim_Z0=bool(optim_Z0))
        tensors = dict(K=K, P_rig2cam=P_rig2cam, P_w2rig=P_w2rig, z_coefs=z_coefs, pts3d=pts3d,
                       pix2d_std=pix2d_std, pix2d_dep=pix2d_dep, pix2d=pix2d)
        return Linearization(plan, tensors, flags)

    def linearize(self, J, residuals=None, w_pts=None, clamp_w=(1e-6, 1e6), lin_kw=None, z_prior=None,
                  objective=False):
        """Run the fused linearization; returns the SchurSystem (S, b, diag A, preconditioner)."""
        t, f = J.tensors, J.flags
        kw = dict(lin_kw or {})
        opts = BAPlan.lin_opts(is_depth_log=f['is_depth_log'], clamp_w=clamp_w, dampen=self.dampen,
                               adaptive_dampen=self.adaptive_dampen, no_grad_f_from_rz=self.no_grad_f_from_rz,
                               optim_Z0=f['optim_Z0'], optim_Z_1st_cam=f['optim_Z_1st_cam'], **kw)
        # the plan's track-sorted copy of the observation arrays is refreshed for every
        # linearization: the caller may have edited them in place, or new arrays may sit at
        # the addresses of old ones
        J.plan.stage_obs(t['pix2d'], t['pix2d_std'], t['pix2d_dep'])
        if t['pix2d'] is not None:
            p = J.plan.params(t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'], t['pix2d_std'],
                              t['pix2d_dep'], pix2d=t['pix2d'])
        else:
            p = J.plan.params(t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'], t['pix2d_std'],
                              t['pix2d_dep'], residuals=residuals, w_pts=w_pts)
        J.system = J.plan.linearize(p, opts, z_prior=z_prior, objective=objective)
        return J.system

    @property
    def last_solve(self):
        """Iterations and convergence of the last solve: dict(iters, converged)."""
        return self.check_solve()

    def check_solve(self):
        """Reads the last solve's PCG status (one synchronisation when the solve was queued
        with ``wait=False``); raises if a grid-barrier wait of the PCG kernel ran out."""
        if self._pcg_result is None:
            return {}
        it, conv = BAPlan.pcg_status(self._pcg_result)
        return dict(iters=it, converged=conv)

    def solve_delta(self, J, residuals, w_pts, clamp_w=(1e-6, 1e6), z_prior=None, lin_kw=None, wait=True):
        """delta = [delta_c, delta_p] solving (J^T W J + damping) delta = J^T W r through the
        Schur complement (ba_solver.py:110-182); float32 like the reference."""
        assert residuals.shape == (self.n_kpts, 3)
        # without the weights the linearization must recompute them in-kernel (pix2d given)
        assert (w_pts is None and J.tensors['pix2d'] is not None) or w_pts.shape in ((self.n_kpts, 1),
                                                                                   (self.n_kpts, 3))
        zp = None
        if z_prior is not None:
            H_z, g_z = z_prior
            if H_z is not None and g_z is not None:
                # the reference's checks (ba_solver.py:149-157): one C x C block per enabled image
                assert g_z.shape == (self.imgs.n, self.n_zcf), \
                    f"bad g_z shape {g_z.shape}, expected {(self.imgs.n, self.n_zcf)}"
                assert H_z.shape == (self.imgs.n, self.n_zcf, self.n_zcf), \
                    f"bad H_z shape {H_z.shape}, expected {(self.imgs.n, self.n_zcf, self.n_zcf)}"
                if self.imgs.true_idxs is not None and self.imgs.n != self.imgs.true_n:
                    raise TypeError('z_prior with a partial depth-coefficient mask is not supported')
                zp = (H_z, g_z)
        s = self.linearize(J, residuals, w_pts, clamp_w, lin_kw, z_prior=zp)
        return self._solve(s, wait)

    def solve_with_objective(self, J, clamp_w=(1e-6, 1e6), z_prior=None, lin_kw=None, wait=True):
        """solve_delta for a linearization that recomputes residuals in-kernel (compute_jacobians
        given pix2d), which also returns the objective at the linearization point from the same
        passes: (delta, loss, residuals) with loss the mean Huber error over the (n_obs, 3)
        errors (0-d float32, what lm_step's objective computes, engine.py:263-281) and residuals
        an (n_obs, 3) view.  ``wait=False`` (also for solve_delta) returns without reading the
        PCG's status back: the caller queues more work and calls ``check_solve`` later."""
        assert J.tensors['pix2d'] is not None, 'the objective needs in-kernel residuals (pix2d)'
        s = self.linearize(J, None, None, clamp_w, lin_kw, z_prior=z_prior, objective=True)
        loss = (s.loss_sum[0] / max(3 * self.n_kpts, 1)).to(torch.float32)
        return self._solve(s, wait), loss, s.residuals.transpose(0, 1)

    def _solve(self, s, wait=True):
        dt = torch.float64 if self.dtype == torch.float64 else torch.float32
        # the reference's PCG (ba_solver.py:202, 1197-1238) as one device kernel on the explicit S
        delta_c, self._pcg_result = s.plan.pcg(s.S_vals, s.precond, s.b.to(dt), tol=1e-6, maxiter=300, wait=False)
        if wait:
            self.check_solve()
        delta_p = s.backsub(delta_c.to(torch.float32))
        return torch.cat([delta_c.to(torch.float32), delta_p])

    def unpack_delta_inplace(self, delta):
        """(dK, dP, dZ, dX), re-expanded over disabled columns (ba_solver.py:228-248)."""
        sizes = [self.cams.n * N_FOC, self.nodes.n * N_TAU, self.imgs.n * self.n_zcf, self.tracks.n * 3]
        cum = torch.tensor(sizes).cumsum(0)
        assert delta.shape == (int(cum[-1]),)
        dK, dP, dZ, dX = delta.tensor_split(cum[:-1].tolist())

        def expand(d, prm, k):
            d = d.view(prm.n, k)
            if prm.true_idxs is not None:
                d2 = d.new_zeros((prm.true_n, k))
                d2[prm.true_idxs] = d
                return d2
            return d
        return (expand(dK, self.cams, N_FOC), expand(dP, self.nodes, N_TAU), expand(dZ, self.imgs, self.n_zcf),
                expand(dX, self.tracks, 3))
