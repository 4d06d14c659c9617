"""Python wrapper of the fused linearization plan (C ABI part 2 of ``include/b3r.h``).

``BAPlan`` holds the static structure of one BA phase (built once on the host from the
image-sorted ``infos``/``pids`` of ``RigsData.infos`` / ``ObservedTracks``, then kept on
the GPU).  ``BAPlan.linearize`` runs residual -> Jacobians -> IRLS weights -> per-track
point elimination -> Schur assembly and returns a ``SchurSystem`` whose S lives in the
plan's block-sparse pattern (upper block triangle, diagonal blocks in full).
"""
import ctypes as C

import numpy as np
import torch

from . import _lib as L


def _enable_mode(status, n):
    """(mode, host mask) for one parameter type, mirroring GaussNewtonSolver.enable
    (inference/ba_solver.py:72-108)."""
    if status is True or status is None:
        return L.ENABLE_ALL, None
    if status is False:
        return L.ENABLE_ZERO, None
    m = status.detach().cpu().numpy() if isinstance(status, torch.Tensor) else np.asarray(status)
    if m.dtype != np.bool_ or m.shape != (n,):
        raise ValueError(f'bad enable status (expected bool mask of shape ({n},)): {status!r}')
    return L.ENABLE_MASK, np.ascontiguousarray(m.astype(np.uint8))


class SchurSystem:
    """Output of one linearization: S (block values), b, diag(A), preconditioner."""

    def __init__(self, plan, S_vals, b, diagA, precond, hpp_max, workspace, params, opts):
        self.plan, self.S_vals, self.b, self.diagA, self.precond = plan, S_vals, b, diagA, precond
        self.hpp_max, self.workspace, self.params, self.opts = hpp_max, workspace, params, opts
        self.residuals = self.loss_sum = None

    def matvec(self, x):
        """y = S x (float32 or float64 x)."""
        return self.plan.spmv(self.S_vals, x)

    def to_dense(self):
        return self.plan.dense(self.S_vals)

    def backsub(self, delta_c):
        """Point update delta_p = Hpp^-1 (g_p - Hpc delta_c) of this plan's tracks."""
        return self.plan.backsub(self.params, self.opts, self.workspace, delta_c)


class BAPlan:
    def __init__(self, infos, pids, n_cams, n_nodes, n_tracks, n_zcf, optim_K=True, optim_P=True,
                 optim_Z=True, optim_X=True, track_range=None, device=None, obs_local=False, track_owner=None,
                 rank=0, retain=False, base=None):
        """Plan one BA phase's structure.

        ``retain`` keeps the host-side track, segment and pair lists so that a later plan can
        be appended to this one.  ``base``: an earlier plan built with ``retain`` whose problem
        this one extends the way the online loop merges tracks (``old | new``,
        inference/tracks.py:96-117; images, tracks, cameras and nodes only added, every old
        image's observations first in its range): the plan is then built incrementally by
        ``b3r_plan_append`` (``B3RError`` if the structure does not extend ``base``)."""
        infos_h = np.ascontiguousarray(torch.as_tensor(infos).detach().cpu().numpy().astype(np.int32))
        pids_h = np.ascontiguousarray(torch.as_tensor(pids).detach().cpu().numpy().astype(np.int32))
        n_imgs = infos_h.shape[1]
        if device is None:
            device = torch.device('cuda', torch.cuda.current_device())
        device = torch.device(device)
        self.device = device
        self.n_imgs, self.n_cams, self.n_nodes, self.n_tracks, self.C = n_imgs, n_cams, n_nodes, n_tracks, n_zcf
        self.n_obs = len(pids_h)
        modes = [_enable_mode(s, n) for s, n in ((optim_K, n_cams), (optim_P, n_nodes),
                                                  (optim_Z, n_imgs), (optim_X, n_tracks))]
        self._keep = [infos_h, pids_h] + [m for _, m in modes if m is not None]
        u8 = C.POINTER(C.c_uint8)
        t0, t1 = track_range if track_range is not None else (0, n_tracks)
        owner = None
        if track_owner is not None:                 # tracks t with track_owner[t] == rank
            owner = np.ascontiguousarray(np.asarray(track_owner, np.int32))
            if owner.shape != (n_tracks,):
                raise ValueError(f'track_owner must have shape ({n_tracks},)')
            self._keep.append(owner)
            self.own_tracks = np.flatnonzero(owner == rank)
        else:
            self.own_tracks = np.arange(t0, t1)
        desc = L.PlanDesc(n_imgs=n_imgs, n_cams=n_cams, n_nodes=n_nodes, n_tracks=n_tracks, n_obs=self.n_obs,
                          C=n_zcf, infos=infos_h.ctypes.data_as(C.POINTER(C.c_int32)),
                          pids=pids_h.ctypes.data_as(C.POINTER(C.c_int32)),
                          mode_K=modes[0][0], mode_P=modes[1][0], mode_Z=modes[2][0], mode_X=modes[3][0],
                          mask_K=modes[0][1].ctypes.data_as(u8) if modes[0][1] is not None else None,
                          mask_P=modes[1][1].ctypes.data_as(u8) if modes[1][1] is not None else None,
                          mask_Z=modes[2][1].ctypes.data_as(u8) if modes[2][1] is not None else None,
                          mask_X=modes[3][1].ctypes.data_as(u8) if modes[3][1] is not None else None,
                          track_begin=t0, track_end=t1,
                          device=device.index if device.type == 'cuda' else -1, obs_local=int(bool(obs_local)),
                          track_owner=owner.ctypes.data_as(C.POINTER(C.c_int32)) if owner is not None else None,
                          rank=int(rank), retain=int(bool(retain)))
        self._h = C.c_void_p()
        if base is None:
            L.call('b3r_plan_create', C.byref(self._h), C.byref(desc))
        else:
            L.call('b3r_plan_append', C.byref(self._h), base.handle, C.byref(desc))
        self.retained = bool(retain)
        self.appended = base is not None
        self.info = L.PlanInfo()
        L.call('b3r_plan_get_info', self._h, C.byref(self.info))
        i = self.info
        rp = np.zeros(i.n_blocks + 1, np.int32)
        ci = np.zeros(i.nnzb, np.int32)
        vo = np.zeros(i.nnzb, np.int64)
        bs = np.zeros(i.n_blocks, np.int32)
        bo = np.zeros(i.n_blocks, np.int32)
        L.call('b3r_plan_get_pattern', self._h, rp.ctypes.data, ci.ctypes.data, vo.ctypes.data, bs.ctypes.data,
               bo.ctypes.data)
        self.row_ptr, self.col_idx, self.val_off, self.block_size, self.block_off = rp, ci, vo, bs, bo
        self.n_cam_params = i.n_cam_params
        self._ws = None

    def input_obs(self):
        """Global image-sorted index of every row of the per-observation arrays this plan's
        linearization reads (all observations, or with ``obs_local`` only this rank's)."""
        out = np.empty(int(self.info.n_obs_input), np.int32)
        L.call('b3r_plan_get_input_obs', self._h, out.ctypes.data)
        return out

    def __del__(self):
        h = getattr(self, '_h', None)
        if h is not None and h.value:
            try:
                L.lib().b3r_plan_destroy(h)
            except Exception:
                pass
            self._h = None

    @property
    def handle(self):
        return self._h

    def pattern(self):
        """(block rows, block cols) of the stored blocks, both int64 numpy arrays."""
        rows = np.repeat(np.arange(self.info.n_blocks), np.diff(self.row_ptr))
        return rows, self.col_idx.astype(np.int64)

    def workspace(self):
        if self._ws is None:
            nbytes = int(self.info.workspace_bytes)
            self._ws = torch.empty(nbytes + 256, dtype=torch.uint8, device=self.device)
        ptr = self._ws.data_ptr()
        return ptr + ((-ptr) % 256)

    def new_outputs(self):
        f = dict(dtype=torch.float32, device=self.device)
        return (torch.empty(int(self.info.nnz), **f), torch.empty(self.n_cam_params, **f),
                torch.empty(self.n_cam_params, **f), torch.empty(self.n_cam_params, **f), torch.empty(1, **f))

    # ------------------------------------------------------------------ linearization
    @staticmethod
    def lin_opts(is_depth_log=True, weight_z=1.0, pnorm=1.0, max_pix_err=100.0, huber_delta=0.5,
                 w_pts_nul=1e-16, clamp_w=(1e-6, 1e6), dampen=1e-12, adaptive_dampen=True,
                 no_grad_f_from_rz=False, optim_Z0=True, optim_Z_1st_cam=True):
        return L.LinOpts(is_depth_log=int(bool(is_depth_log)), weight_z=weight_z, pnorm=pnorm,
                         max_pix_err=max_pix_err, huber_delta=huber_delta, w_pts_nul=w_pts_nul,
                         clamp_w_lo=clamp_w[0], clamp_w_hi=clamp_w[1], dampen=dampen,
                         adaptive_dampen=int(bool(adaptive_dampen)),
                         no_grad_f_from_rz=int(bool(no_grad_f_from_rz)), optim_Z0=int(bool(optim_Z0)),
                         optim_Z_1st_cam=int(bool(optim_Z_1st_cam)))

    def params(self, K, P_rig2cam, P_w2rig, z_coefs, pts3d, pix2d_std, pix2d_dep, pix2d=None,
               residuals=None, w_pts=None):
        """C-ABI parameter struct (keeps the tensors alive in ``self._live``)."""
        for t, n in ((K, 'K'), (P_w2rig, 'P_w2rig'), (z_coefs, 'z_coefs'), (pts3d, 'pts3d'),
                     (pix2d_std, 'pix2d_std'), (pix2d_dep, 'pix2d_dep')):
            if t.dtype != torch.float32 or not t.is_contiguous() or t.device != self.device:
                raise RuntimeError(f'{n} must be a contiguous float32 tensor on {self.device}')
        if not (P_rig2cam.stride(1) == 4 and P_rig2cam.stride(2) == 1):
            raise RuntimeError('P_rig2c should be (N,4,4) and contiguous inside 4x4 blocks')
        p = L.Params(K=K.data_ptr(), P_rig2c=P_rig2cam.data_ptr(), P_rig2c_stride=P_rig2cam.stride(0),
                     P_w2rig=P_w2rig.data_ptr(), z_coefs=z_coefs.data_ptr(), pts3d=pts3d.data_ptr(),
                     pix2d=pix2d.data_ptr() if pix2d is not None else None,
                     pix2d_std=pix2d_std.data_ptr(), pix2d_dep=pix2d_dep.data_ptr())
        live = [K, P_rig2cam, P_w2rig, z_coefs, pts3d, pix2d_std, pix2d_dep, pix2d]
        if pix2d is None:
            if residuals is None or w_pts is None:
                raise RuntimeError('residuals and w_pts are required when pix2d is not given')
            p.residuals, p.res_stride_n, p.res_stride_c = residuals.data_ptr(), residuals.stride(0), residuals.stride(1)
            p.w_pts, p.w_stride_n, p.w_stride_c = w_pts.data_ptr(), w_pts.stride(0), w_pts.stride(1)
            p.w_cols = w_pts.shape[1]
            live += [residuals, w_pts]
        self._live = live
        return p

    def linearize(self, params, opts, outputs=None, stream=None, z_prior=None, objective=False):
        """Full single-GPU linearization; returns a SchurSystem.  ``z_prior`` = (H_z, g_z), the
        dense tangent prior's terms ([n_imgs, C, C], [n_imgs, C]), is added to the system before
        its damping (solve_delta's z_prior, ba_solver.py:141-173).  With ``objective`` the
        system also carries the objective at the linearization point, evaluated by the same
        passes: ``residuals`` [3, n_obs_input] and ``loss_sum`` (double, the sum of the Huber
        errors)."""
        S, b, dA, pc, hm = outputs if outputs is not None else self.new_outputs()
        res = loss = None
        if objective:
            res = torch.empty((3, int(self.info.n_obs_input)), dtype=torch.float32, device=self.device)
            loss = torch.empty(1, dtype=torch.float64, device=self.device)
        out = L.Outputs(S_vals=S.data_ptr(), b=b.data_ptr(), diagA=dA.data_ptr(), precond=pc.data_ptr(),
                        hpp_max=hm.data_ptr(), residuals=res.data_ptr() if res is not None else None,
                        loss=loss.data_ptr() if loss is not None else None)
        ws = self.workspace()
        s = stream if stream is not None else torch.cuda.current_stream().cuda_stream
        if z_prior is None:
            L.call('b3r_linearize_schur', self._h, C.byref(params), C.byref(opts), ws, C.byref(out), s)
        else:
            Hz, gz = (t.to(device=self.device, dtype=torch.float64).contiguous() for t in z_prior)
            assert Hz.shape == (self.n_imgs, self.C, self.C) and gz.shape == (self.n_imgs, self.C)
            L.call('b3r_lin_points', self._h, C.byref(params), C.byref(opts), ws, C.byref(out), s)
            L.call('b3r_lin_assemble', self._h, C.byref(params), C.byref(opts), ws, C.byref(out), s)
            L.call('b3r_lin_add_zprior', self._h, Hz.data_ptr(), gz.data_ptr(), ws, C.byref(out), s)
            L.call('b3r_lin_finalize', self._h, C.byref(opts), ws, C.byref(out), s)
            self._live_prior = (Hz, gz)
        sysm = SchurSystem(self, S, b, dA, pc, hm, ws, params, opts)
        sysm.residuals, sysm.loss_sum = res, loss
        return sysm

    def capture(self, params, opts, outputs=None):
        """CUDA graph of one full linearization on fixed buffers (the tensors `params` points
        at and the outputs): each replay relinearizes at those tensors' current values with one
        launch from the host.  For latency-bound problems (online windows), where the seven
        kernel launches and three clears cost as much as the work.  Returns (graph, system)."""
        outs = outputs if outputs is not None else self.new_outputs()
        side = torch.cuda.Stream(device=self.device)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            self.linearize(params, opts, outs)     # one-time setup (attributes, staging) outside the graph
        torch.cuda.current_stream().wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            system = self.linearize(params, opts, outs)
        return g, system

    def lin_stage(self, name, params, opts, outputs, stream=None):
        """One stage ('points', 'assemble', 'finalize') of a sharded linearization."""
        S, b, dA, pc, hm = outputs
        out = L.Outputs(S_vals=S.data_ptr(), b=b.data_ptr(), diagA=dA.data_ptr(),
                        precond=pc.data_ptr() if pc is not None else None, hpp_max=hm.data_ptr())
        s = stream if stream is not None else torch.cuda.current_stream().cuda_stream
        ws = self.workspace()
        if name == 'finalize':
            L.call('b3r_lin_finalize', self._h, C.byref(opts), ws, C.byref(out), s)
        else:
            L.call('b3r_lin_' + name, self._h, C.byref(params), C.byref(opts), ws, C.byref(out), s)

    def spmv(self, S_vals, x):
        y = torch.empty_like(x)
        s = torch.cuda.current_stream().cuda_stream
        name = 'b3r_schur_spmv_f64' if x.dtype == torch.float64 else 'b3r_schur_spmv'
        L.call(name, self._h, S_vals.data_ptr(), x.contiguous().data_ptr(), y.data_ptr(), s)
        return y

    def pcg(self, S_vals, precond, b, tol=1e-6, maxiter=300, barrier_spin_limit=0, flags=0, raw=False, wait=True):
        """Solve S x = b on the device (b3r_pcg_ex): the reference's PCG iteration and
        stopping rule, one cooperative kernel.  Returns (x, iterations, converged); raises if a
        grid-barrier wait ran out (with ``raw``, returns (x, iterations, converged, error)
        instead).  ``barrier_spin_limit`` bounds every barrier wait (0: the library's default).
        With ``wait=False`` nothing is read back: returns (x, result), result the device int32
        [iterations, converged, error, replacements] that ``pcg_status`` reads later, so that
        the host can queue the work that follows while the solve runs."""
        assert b.dtype in (torch.float32, torch.float64)
        b = b.contiguous()
        x = torch.empty_like(b)
        work = torch.empty(int(L.lib().b3r_pcg_work_bytes(self._h)) // 8 + 32, dtype=torch.float64, device=b.device)
        res = torch.zeros(4, dtype=torch.int32, device=b.device)
        dt = L.B3R_F64 if b.dtype == torch.float64 else L.B3R_F32
        L.call('b3r_pcg_ex', self._h, S_vals.data_ptr(), precond.contiguous().data_ptr(), b.data_ptr(), x.data_ptr(),
               dt, float(tol), int(maxiter), int(barrier_spin_limit), int(flags), work.data_ptr(), res.data_ptr(),
               torch.cuda.current_stream().cuda_stream)
        if not wait:
            return x, res
        it, conv, err = res[:3].tolist()
        if raw:
            return x, int(it), bool(conv), int(err)
        if err:
            raise L.B3RError('b3r_pcg: a grid barrier of the PCG kernel gave up')
        return x, int(it), bool(conv)

    @staticmethod
    def pcg_status(res):
        """(iterations, converged) of a ``pcg(..., wait=False)`` result; raises if a grid-barrier
        wait of that solve ran out."""
        it, conv, err = res[:3].tolist()
        if err:
            raise L.B3RError('b3r_pcg: a grid barrier of the PCG kernel gave up')
        return int(it), bool(conv)

    def backsub(self, params, opts, workspace_ptr, delta_c, delta_p=None):
        if delta_p is None:
            delta_p = torch.zeros(3 * self.info.n_points, dtype=torch.float32, device=self.device)
        dc = delta_c.to(torch.float32).contiguous()
        L.call('b3r_backsub', self._h, C.byref(params), C.byref(opts), workspace_ptr, dc.data_ptr(),
               delta_p.data_ptr(), torch.cuda.current_stream().cuda_stream)
        return delta_p

    def dense(self, S_vals):
        """Dense symmetric S (float64, on S_vals' device) from the block values."""
        n = self.n_cam_params
        Sv = S_vals.detach().to(torch.float64).cpu().numpy()
        D = np.zeros((n, n))
        rows, cols = self.pattern()
        for j in range(len(cols)):
            p, q = rows[j], cols[j]
            bp, bq = self.block_size[p], self.block_size[q]
            blk = Sv[self.val_off[j]:self.val_off[j] + bp * bq].reshape(bp, bq)
            r0, c0 = self.block_off[p], self.block_off[q]
            D[r0:r0 + bp, c0:c0 + bq] = blk
            if p != q:
                D[c0:c0 + bq, r0:r0 + bp] = blk.T
        return torch.from_numpy(D).to(S_vals.device)

    def lin_pass(self, pass_id, params, opts, outputs, stream=None):
        """One pass (b3r_lin_pass): PASS_PREP/POINTS/FACTOR/DIAG/PAIRS of _lib, in that order."""
        S, b, dA, pc, hm = outputs
        out = L.Outputs(S_vals=S.data_ptr(), b=b.data_ptr(), diagA=dA.data_ptr(),
                        precond=pc.data_ptr() if pc is not None else None, hpp_max=hm.data_ptr())
        s = stream if stream is not None else torch.cuda.current_stream().cuda_stream
        L.call('b3r_lin_pass', self._h, C.byref(params), C.byref(opts), self.workspace(), C.byref(out),
               int(pass_id), s)

    def stage_obs(self, pix2d, pix2d_std, pix2d_dep, stream=None):
        """Re-gather the static observation arrays into the plan's track-sorted copy."""
        s = stream if stream is not None else torch.cuda.current_stream().cuda_stream
        L.call('b3r_plan_stage_obs', self._h, pix2d.data_ptr() if pix2d is not None else None,
               pix2d_std.data_ptr(), pix2d_dep.data_ptr(), s)
