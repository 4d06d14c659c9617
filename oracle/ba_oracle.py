"""CPU oracle for the BA linearization + Schur assembly path (TEST INFRASTRUCTURE ONLY).

This module restates, in numpy, the reference algorithm of naver/blast3r's
bundle-adjustment hot path.  It is the parity checker of the CUDA product path:
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import it.  The product never calls it and has no CPU fallback.

Reference pieces restated here (paths relative to the reference project root):

* observation -> image search ........ ``extensions/cujac/sfm_jacobian_rigs.cu:72-88``
* residual + Huber/IRLS weights ...... ``sfm_jacobian_rigs.cu:129-259`` (wrapper ``:1048-1101``)
* Jacobians .......................... ``sfm_jacobian_rigs.cu:323-509`` (wrapper ``:1105-1148``)
* batched 3x3 Cholesky solve ......... ``sfm_jacobian_rigs.cu:560-634``
* J masking / column enabling ........ ``inference/ba_solver.py:34-108``
* weights, gradient, J *= sqrt(W) .... ``ba_solver.py:123-132``
* Gram blocks (A, B, C, D) ........... ``ba_solver.py:854-924, 1063-1071``
* per-type adaptive damping .......... ``ba_solver.py:510-517, 572-582, 1188-1191``
* reduced rhs b = g_c - B D^-1 g_p ... ``ba_solver.py:184-188``
* implicit Schur matvec .............. ``ba_solver.py:196-200``
* PCG ................................ ``ba_solver.py:1197-1238``
* delta unpacking .................... ``ba_solver.py:228-248``

Parity status: the algebra (Gram blocks, damping, S, b) is pinned to the reference's
own ``ba_solver.py`` run on CPU (``tests/golden/make_golden.py`` -> ``tests/golden/*.npz``);
the residual and Jacobian restatements are pinned to the reference CUDA kernels'
outputs captured on a B200 (``tests/golden/make_golden_ref_kernels.py``).

All math runs in ``dtype`` (float64 by default: the oracle is the accurate truth the
fp32 CUDA path is compared against, with the tolerances written in the tests).
"""
import numpy as np

N_FOC, N_TAU = 2, 6


# --------------------------------------------------------------------------------------
# per-observation kernels
# --------------------------------------------------------------------------------------

def obs_to_image(infos, n_obs):
    """Image id of every observation: the reference's binary search over the end
    offsets ``infos[0]`` (``sfm_jacobian_rigs.cu:72-88``); equivalently the solver's
    ``bincount(cum)[:-1].cumsum()`` (``ba_solver.py:51``)."""
    cum = np.asarray(infos[0], np.int64)
    return np.searchsorted(cum, np.arange(n_obs), side='right')


def _geometry(infos, K, P_rig2c, P_w2rig, pts3d, pids, dt):
    n = len(pids)
    img = obs_to_image(infos, n)
    node = np.asarray(infos[1], np.int64)[img]
    cam = np.asarray(infos[2], np.int64)[img]
    X = pts3d.astype(dt)[np.asarray(pids, np.int64)]
    Kc = K.astype(dt)[cam]
    fx, cx, fy, cy = Kc[:, 0, 0], Kc[:, 0, 2], Kc[:, 1, 1], Kc[:, 1, 2]
    Prw = P_w2rig.astype(dt)[node]
    Pcr = P_rig2c.astype(dt)[cam]
    R_rw, t_rw = Prw[:, :3, :3], Prw[:, :3, 3]
    R_cr, t_cr = Pcr[:, :3, :3], Pcr[:, :3, 3]
    X_r = np.einsum('nij,nj->ni', R_rw, X) + t_rw           # .cu:200-203
    X_c = np.einsum('nij,nj->ni', R_cr, X_r) + t_cr         # .cu:205-208
    return dict(img=img, node=node, cam=cam, fx=fx, cx=cx, fy=fy, cy=cy,
                R_rw=R_rw, R_cr=R_cr, X_r=X_r, X_c=X_c)


def residuals_with_rigs(infos, K, P_rig2c, P_w2rig, z_coefs, pts3d, pids, pix2d, pix2d_std,
                        pix2d_dep, is_depth_log, weight_z=1.0, pnorm=-1.0, max_pix_err=100.0,
                        huber_delta=0.5, w_pts_nul=1e-16, dtype=np.float64):
    """Residual op (``sfm_jacobian_rigs.cu:129-259``, wrapper ``:1048-1101``).

    Returns (n, 9) = [residual(3), err(3), w(3)] when ``pnorm > 0`` else (n, 3); rows of
    observations with camera depth z <= 1e-3 stay zero (``.cu:212``, outputs start from
    ``torch::zeros`` at ``.cu:1073``).
    """
    dt = dtype
    g = _geometry(infos, K, P_rig2c, P_w2rig, pts3d, pids, dt)
    n = len(pids)
    X_c, img = g['X_c'], g['img']
    z = X_c[:, 2]
    valid = z > 1e-3
    zs = np.where(valid, z, 1.0)
    kpt = pix2d.astype(dt)
    std = pix2d_std.astype(dt)
    out = np.zeros((n, 9 if pnorm > 0 else 3), dt)
    p0 = (g['fx'] * X_c[:, 0] + g['cx'] * X_c[:, 2]) / zs     # .cu:217-218
    p1 = (g['fy'] * X_c[:, 1] + g['cy'] * X_c[:, 2]) / zs
    res = np.zeros((n, 3), dt)
    res[:, 0] = (p0 - kpt[:, 0]) / std[:, 0]                  # .cu:226-228
    res[:, 1] = (p1 - kpt[:, 1]) / std[:, 1]
    guid = np.einsum('nc,nc->n', z_coefs.astype(dt)[img], pix2d_dep.astype(dt))   # .cu:231-233
    fbar = 0.5 * (g['fx'] + g['fy'])
    if is_depth_log:
        res[:, 2] = fbar * (guid - np.log(zs))                # .cu:235-236
    else:
        with np.errstate(divide='ignore', invalid='ignore'):
            res[:, 2] = fbar * np.log(guid / zs)              # .cu:237-238
    out[:, :3] = res
    if pnorm > 0:                                             # .cu:240-258
        a = 0.5 * pnorm * huber_delta ** (pnorm - 2)
        b = huber_delta ** pnorm - a * huber_delta * huber_delta
        wz = np.array([1.0, 1.0, weight_z], dt)
        r = np.abs(res)
        r = np.where(r > max_pix_err, max_pix_err, r)
        with np.errstate(divide='ignore', invalid='ignore'):
            out[:, 3:6] = wz * np.where(r <= huber_delta, a * r * r, r ** pnorm - b)
            r = np.where(r < huber_delta, huber_delta, r)
            out[:, 6:9] = np.where(r == max_pix_err, w_pts_nul, wz * r ** (pnorm - 2))
    out[~valid] = 0
    return out


def jacobians_with_rigs(infos, K, P_rig2c, P_w2rig, z_coefs, pts3d, pids, pix2d_std, pix2d_dep,
                        is_depth_log, dtype=np.float64):
    """Jacobian op (``sfm_jacobian_rigs.cu:323-509``, wrapper ``:1105-1148``).

    Returns J_cam (n,3,8) = [d/dfx, d/dfy, d/dtau(6)], J_zcf (n,1,C) (depth row only) and
    J_pts (n,3,3); rows of observations with z <= 1e-3 stay zero (``.cu:408``).
    The focal derivative of the depth row is rounded to float32, as the reference
    stores it in a ``float`` local even for float64 output (``.cu:481-487``).
    """
    dt = dtype
    g = _geometry(infos, K, P_rig2c, P_w2rig, pts3d, pids, dt)
    n = len(pids)
    C = pix2d_dep.shape[1]
    X_c, X_r, img = g['X_c'], g['X_r'], g['img']
    fx, cx, fy, cy = g['fx'], g['cx'], g['fy'], g['cy']
    z = X_c[:, 2]
    valid = z > 1e-3
    zs = np.where(valid, z, 1.0)
    inv_z = 1.0 / zs
    inv_z2 = inv_z * inv_z
    fbar = 0.5 * (fx + fy)
    p0 = fx * X_c[:, 0] + cx * X_c[:, 2]                      # not divided by z (.cu:401-402)
    p1 = fy * X_c[:, 1] + cy * X_c[:, 2]
    std = pix2d_std.astype(dt)
    Jp = np.zeros((n, 3, 3), dt)                              # .cu:414-435
    Jp[:, 0, 0] = fx * inv_z / std[:, 0]
    Jp[:, 0, 2] = (cx * inv_z - p0 * inv_z2) / std[:, 0]
    Jp[:, 1, 1] = fy * inv_z / std[:, 1]
    Jp[:, 1, 2] = (cy * inv_z - p1 * inv_z2) / std[:, 1]
    Jp[:, 2, 2] = -fbar * inv_z
    J_proj_rig = Jp @ g['R_cr']                               # .cu:439-441
    Jrt = np.zeros((n, 3, 6), dt)                             # .cu:444-453
    Jrt[:, 0, 1], Jrt[:, 0, 2], Jrt[:, 0, 3] = X_r[:, 2], -X_r[:, 1], 1
    Jrt[:, 1, 0], Jrt[:, 1, 2], Jrt[:, 1, 4] = -X_r[:, 2], X_r[:, 0], 1
    Jrt[:, 2, 0], Jrt[:, 2, 1], Jrt[:, 2, 5] = X_r[:, 1], -X_r[:, 0], 1
    J_tau = J_proj_rig @ Jrt                                  # .cu:457-458
    J_pts = J_proj_rig @ g['R_rw']                            # .cu:461-463
    guid = np.einsum('nc,nc->n', z_coefs.astype(dt)[img], pix2d_dep.astype(dt))
    J_cam = np.zeros((n, 3, 8), dt)
    J_cam[:, 0, 0] = X_c[:, 0] * inv_z / std[:, 0]           # .cu:473
    J_cam[:, 1, 1] = X_c[:, 1] * inv_z / std[:, 1]           # .cu:477
    with np.errstate(divide='ignore', invalid='ignore'):
        if is_depth_log:
            jkf = 0.5 * (guid + np.log(inv_z))
        else:
            jkf = 0.5 * np.log(guid * inv_z)
    jkf = np.where(guid > 0, jkf, 0.0).astype(np.float32).astype(dt)
    J_cam[:, 2, 0] = jkf
    J_cam[:, 2, 1] = jkf
    J_cam[:, :, 2:] = J_tau
    dep = pix2d_dep.astype(dt)
    if is_depth_log:
        J_zcf = (fbar[:, None] * dep)[:, None, :]             # .cu:496-501
    else:
        with np.errstate(divide='ignore', invalid='ignore'):
            s = np.where(guid != 0, fbar / np.where(guid != 0, guid, 1.0), 0.0)
        J_zcf = (s[:, None] * dep)[:, None, :]
    J_cam[~valid] = 0
    J_zcf = np.where(valid[:, None, None], J_zcf, 0.0)
    J_pts[~valid] = 0
    return J_cam, J_zcf.astype(dt), J_pts


def chol3x3_solve(blocks, rhs, jitter=1e-12):
    """Batched guarded 3x3 SPD solve (``sfm_jacobian_rigs.cu:560-634``): symmetrise,
    add ``jitter`` to the diagonal, Cholesky with non-positive pivots bumped by
    ``jitter``, forward and back substitution.  ``rhs`` is (N,3) or (N,3,k)."""
    A = np.asarray(blocks, np.float64)
    b = np.asarray(rhs, np.float64)
    vec = b.ndim == 2
    if vec:
        b = b[..., None]
    a00 = A[:, 0, 0] + jitter
    a11 = A[:, 1, 1] + jitter
    a22 = A[:, 2, 2] + jitter
    a01 = (A[:, 0, 1] + A[:, 1, 0]) * 0.5
    a02 = (A[:, 0, 2] + A[:, 2, 0]) * 0.5
    a12 = (A[:, 1, 2] + A[:, 2, 1]) * 0.5
    a00 = np.where(a00 > 0, a00, a00 + jitter)
    l00 = np.sqrt(a00)
    l10 = a01 / l00
    l20 = a02 / l00
    t11 = a11 - l10 * l10
    t11 = np.where(t11 > 0, t11, t11 + jitter)
    l11 = np.sqrt(t11)
    l21 = (a12 - l10 * l20) / l11
    t22 = a22 - l20 * l20 - l21 * l21
    t22 = np.where(t22 > 0, t22, t22 + jitter)
    l22 = np.sqrt(t22)
    l00, l10, l20, l11, l21, l22 = (v[:, None] for v in (l00, l10, l20, l11, l21, l22))
    z0 = b[:, 0] / l00
    z1 = (b[:, 1] - l10 * z0) / l11
    z2 = (b[:, 2] - l20 * z0 - l21 * z1) / l22
    x2 = z2 / l22
    x1 = (z1 - l21 * x2) / l11
    x0 = (z0 - l10 * x1 - l20 * x2) / l00
    x = np.stack([x0, x1, x2], axis=1)
    return x[..., 0] if vec else x


# --------------------------------------------------------------------------------------
# parameter enabling (ba_solver.py:34-108) and typed parameter blocks
# --------------------------------------------------------------------------------------

def _enable(status, n_true, per_obs_block):
    """Column map of one parameter type after ``GaussNewtonSolver.enable``.

    Returns (n_cols, col_of_block (n_true,) with -1 for removed blocks, obs_active (n,),
    zeroed).  ``True``: all blocks kept; ``False``: columns kept but the whole J block
    is zero (``ZerosMat``, damped to exactly 1e-12*I at ``ba_solver.py:510-517``); a bool
    mask: disabled columns are removed and observations of disabled blocks get zero J
    blocks (``ba_solver.py:76-104``)."""
    if status is True or status is None:
        return n_true, np.arange(n_true), np.ones(len(per_obs_block), bool), False
    if status is False:
        return n_true, np.arange(n_true), np.zeros(len(per_obs_block), bool), True
    m = np.asarray(status, bool)
    assert m.shape == (n_true,)
    idx = np.nonzero(m)[0]
    if len(idx) == 0:
        return n_true, np.arange(n_true), np.zeros(len(per_obs_block), bool), True
    col = np.full(n_true, -1)
    col[idx] = np.arange(len(idx))
    return len(idx), col, m[per_obs_block], False


class Layout:
    """Reduced camera-side parameter vector [foc | tau | zcf] and the point vector,
    in the reference's order (``ba_solver.py:119, 229``), with typed parameter blocks
    numbered foc (size 2), tau (size 6), zcf (size C) in that order."""

    def __init__(self, infos, pids, n_cams, n_nodes, n_tracks, C, optim_K=True, optim_P=True,
                 optim_Z=True, optim_X=True):
        n = len(pids)
        self.n_obs, self.C = n, C
        self.img = obs_to_image(infos, n)
        self.cam = np.asarray(infos[2], np.int64)[self.img]
        self.node = np.asarray(infos[1], np.int64)[self.img]
        self.trk = np.asarray(pids, np.int64)
        n_imgs = infos.shape[1]
        self.n_true = dict(K=n_cams, P=n_nodes, Z=n_imgs, X=n_tracks)
        self.nK, self.colK, self.actK, self.zeroK = _enable(optim_K, n_cams, self.cam)
        self.nP, self.colP, self.actP, self.zeroP = _enable(optim_P, n_nodes, self.node)
        self.nZ, self.colZ, self.actZ, self.zeroZ = _enable(optim_Z, n_imgs, self.img)
        self.nX, self.colX, self.actX, self.zeroX = _enable(optim_X, n_tracks, self.trk)
        self.off_P = N_FOC * self.nK
        self.off_Z = self.off_P + N_TAU * self.nP
        self.n_cam_params = self.off_Z + C * self.nZ
        self.n_params = self.n_cam_params + 3 * self.nX
        # typed blocks
        self.nb = self.nK + self.nP + self.nZ
        self.block_size = np.concatenate([np.full(self.nK, N_FOC), np.full(self.nP, N_TAU),
                                          np.full(self.nZ, C)]).astype(np.int64)
        self.block_off = np.concatenate([[0], np.cumsum(self.block_size)[:-1]]).astype(np.int64)
        self.block_type = np.concatenate([np.zeros(self.nK, int), np.ones(self.nP, int),
                                          np.full(self.nZ, 2)])
        # per-observation typed block ids (-1: inactive / zero)
        self.bK = np.where(self.actK & (not self.zeroK), self.colK[self.cam], -1)
        self.bP = np.where(self.actP & (not self.zeroP), self.nK + self.colP[self.node], -1)
        self.bZ = np.where(self.actZ & (not self.zeroZ), self.nK + self.nP + self.colZ[self.img], -1)
        self.tX = np.where(self.actX & (not self.zeroX), self.colX[self.trk], -1)

    def obs_blocks(self):
        return np.stack([self.bK, self.bP, self.bZ], axis=1)


def camera_jacobian(J_cam, J_zcf, layout, no_grad_f_from_rz=False, optim_Z_1st_cam=True,
                    optim_Z0=True):
    """Per-observation camera-side Jacobian (n, 3, 2+6+C) with the reference's masking
    (``ba_solver.py:38-39, 59-60, 76-104``); inactive blocks are zeroed."""
    n = J_cam.shape[0]
    C = J_zcf.shape[2]
    Jc = np.zeros((n, 3, N_FOC + N_TAU + C), J_cam.dtype)
    Jc[:, :, :8] = J_cam
    jz = J_zcf[:, 0, :].copy()
    if not optim_Z_1st_cam:
        jz[0, 0] = 0
    if not optim_Z0:
        jz[:, 0] = 0
    Jc[:, 2, 8:] = jz
    if no_grad_f_from_rz:
        Jc[:, 2, :2] = 0
    Jc[layout.bK < 0, :, 0:2] = 0
    Jc[layout.bP < 0, :, 2:8] = 0
    Jc[layout.bZ < 0, :, 8:] = 0
    return Jc


# --------------------------------------------------------------------------------------
# Schur system
# --------------------------------------------------------------------------------------

def s_pattern(layout):
    """Typed-block pattern of S (upper triangle, p <= q), sorted row-major.

    Blocks (p, q) appear iff p == q (every block: damping puts a diagonal block on each,
    ``ba_solver.py:510-517, 572-582``), or p and q are both touched by one observation
    (A = J_c^T W J_c), or by two observations of one eliminated track (B D^-1 C fill-in,
    ``ba_solver.py:196-200``)."""
    ob = layout.obs_blocks()
    keys = [np.arange(layout.nb, dtype=np.int64) * (layout.nb + 1)]
    nb = layout.nb

    def add_pairs(bi, bj):
        m = (bi >= 0) & (bj >= 0)
        lo = np.minimum(bi[m], bj[m])
        hi = np.maximum(bi[m], bj[m])
        keys.append(lo * nb + hi)

    for a in range(3):
        for b in range(3):
            add_pairs(ob[:, a], ob[:, b])
    # fill-in through eliminated tracks: all observation pairs of a track
    t = layout.tX
    sel = np.nonzero(t >= 0)[0]
    if len(sel):
        order = sel[np.argsort(t[sel], kind='stable')]
        ts = t[order]
        starts = np.concatenate([[0], np.nonzero(np.diff(ts))[0] + 1])
        lens = np.diff(np.concatenate([starts, [len(ts)]]))
        # pairs (i, j) inside each track segment
        for L in np.unique(lens):
            segs = starts[lens == L]
            ii, jj = np.meshgrid(np.arange(L), np.arange(L), indexing='ij')
            oi = order[segs[:, None] + ii.ravel()[None]].ravel()
            oj = order[segs[:, None] + jj.ravel()[None]].ravel()
            for a in range(3):
                for b in range(3):
                    add_pairs(ob[oi, a], ob[oj, b])
    k = np.unique(np.concatenate(keys))
    return np.stack([k // nb, k % nb], axis=1)


def schur_system(J_cam, J_zcf, J_pts, residuals, w_pts, layout, clamp_w=(1e-6, 1e6),
                 dampen=1e-12, adaptive_dampen=True, no_grad_f_from_rz=False,
                 optim_Z_1st_cam=True, optim_Z0=True, dense=True, dtype=np.float64, obs_mask=None):
    """The reduced system of ``GaussNewtonSolver.solve_delta`` before its PCG.

    Follows ``ba_solver.py:123-188``: W = clamp(w), g = J^T (W r), J *= sqrt(W), the Gram
    blocks A (camera/depth), B = C^T (camera x point) and D (per-track 3x3), per-type
    adaptive damping (1e-12 x max |diag| of each block type, exactly 1e-12 for disabled
    types), and the Schur complement S = A - B D^-1 C with D^-1 applied through the
    guarded 3x3 Cholesky (``sfm_jacobian_rigs.cu:560-634``); b = g_c - B D^-1 g_p.

    Returns a dict with S (dense, reduced camera-side size) or S blocks, b, g, diagA (the
    damped diagonal of A, i.e. the reference's PCG preconditioner before its clamp),
    and per-track quantities for back-substitution.  ``obs_mask`` (bool per observation)
    keeps only those observations' contributions: the partial system of one shard.
    """
    dt = dtype
    n = J_cam.shape[0]
    C = J_zcf.shape[2]
    w = 2 + 6 + C
    Jc = camera_jacobian(J_cam, J_zcf, layout, no_grad_f_from_rz, optim_Z_1st_cam, optim_Z0).astype(dt)
    Jp = J_pts.astype(dt).copy()
    Jp[layout.tX < 0] = 0
    # weights in float32 like the reference (w_pts is float32)
    W32 = np.clip(np.asarray(w_pts, np.float32), np.float32(clamp_w[0]), np.float32(clamp_w[1]))
    if W32.shape[1] == 1:
        W32 = np.repeat(W32, 3, axis=1)
    if obs_mask is not None:
        W32 = np.where(np.asarray(obs_mask, bool)[:, None], W32, np.float32(0))
    Wr = (W32 * np.asarray(residuals, np.float32)).astype(dt)        # ba_solver.py:128
    sW = np.sqrt(W32).astype(dt)                                      # ba_solver.py:132
    Jcw = Jc * sW[:, :, None]
    Jpw = Jp * sW[:, :, None]

    # scalar indices of every observation's camera-side columns
    idx = np.full((n, w), -1, np.int64)
    ob = layout.obs_blocks()
    for a, (lo, sz) in enumerate([(0, 2), (2, 6), (8, C)]):
        bid = ob[:, a]
        m = bid >= 0
        idx[m, lo:lo + sz] = layout.block_off[bid[m]][:, None] + np.arange(sz)[None]
    nc = layout.n_cam_params

    # gradient
    gc_obs = np.einsum('nkj,nk->nj', Jc, Wr)
    g_c = np.zeros(nc, dt)
    m = idx >= 0
    np.add.at(g_c, idx[m], gc_obs[m])
    T = layout.nX
    trk = layout.tX
    gp_obs = np.einsum('nkj,nk->nj', Jp, Wr)
    g_p = np.zeros((max(T, 1), 3), dt)
    mt = trk >= 0
    np.add.at(g_p, trk[mt], gp_obs[mt])

    # A (undamped) diagonal and per-type damping
    Hcc = np.einsum('nki,nkj->nij', Jcw, Jcw)
    diagA = np.zeros(nc, dt)
    dmask = idx >= 0
    np.add.at(diagA, idx[dmask], np.einsum('nii->ni', Hcc)[dmask])
    lam = np.zeros(nc, dt)
    for tcode, (nblk, zero, lo, sz) in enumerate([(layout.nK, layout.zeroK, 0, 2),
                                                   (layout.nP, layout.zeroP, layout.off_P, 6),
                                                   (layout.nZ, layout.zeroZ, layout.off_Z, C)]):
        if nblk == 0:
            continue
        sl = slice(lo, lo + sz * nblk)
        if zero:
            lam[sl] = dampen
        else:
            lam[sl] = dampen * (np.abs(diagA[sl]).max() if adaptive_dampen else 1.0)
    # Hpp (per track) and its damping
    Hpp = np.zeros((max(T, 1), 3, 3), dt)
    np.add.at(Hpp, trk[mt], np.einsum('nki,nkj->nij', Jpw, Jpw)[mt])
    if layout.zeroX:
        lam_p = dampen
    else:
        lam_p = dampen * (np.abs(np.einsum('tii->ti', Hpp[:T])).max() if (adaptive_dampen and T) else 1.0)
    Hpp_d = Hpp + lam_p * np.eye(3)[None]
    # Hpc per observation, D^-1 applied per track through the guarded Cholesky
    Hpc = np.einsum('nki,nkj->nij', Jpw, Jcw)                 # (n, 3, w)
    out = dict(g_c=g_c, g_p=g_p[:T], diagA=diagA + lam, lam=lam, lam_p=lam_p, Hpp=Hpp_d[:T],
               n_cam_params=nc, idx=idx)
    DinvHpc = np.zeros_like(Hpc)
    if T:
        DinvHpc[mt] = chol3x3_solve(Hpp_d[trk[mt]], Hpc[mt])
    Dinv_gp = chol3x3_solve(Hpp_d[:T], g_p[:T]) if T else np.zeros((0, 3))
    # b = g_c - B D^-1 g_p
    bq = np.zeros((n, w), dt)
    bq[mt] = np.einsum('nki,nk->ni', Hpc[mt], Dinv_gp[trk[mt]])
    b = g_c.copy()
    np.add.at(b, idx[m], -bq[m])
    out['b'] = b
    out['Dinv_gp'] = Dinv_gp

    # S = A - B D^-1 C ; pairs of observations inside each track
    pairs_i, pairs_j = _track_pairs(trk)
    if dense:
        S = np.zeros((nc, nc), dt)
        _scatter_sym(S, idx, Hcc, np.arange(n), np.arange(n), sign=1.0)
        if len(pairs_i):
            for s in range(0, len(pairs_i), 1 << 18):
                pi, pj = pairs_i[s:s + (1 << 18)], pairs_j[s:s + (1 << 18)]
                P = np.einsum('nki,nkj->nij', Hpc[pi], DinvHpc[pj])
                _scatter_sym(S, idx, P, pi, pj, sign=-1.0)
        S[np.arange(nc), np.arange(nc)] += lam
        out['S'] = S
    else:
        # same sums, accumulated as a sparse matrix in chunks (large problems)
        import scipy.sparse as sp
        S = _sparse_sum(idx, Hcc, np.arange(n), np.arange(n), nc, 1.0)
        for s in range(0, len(pairs_i), 1 << 17):
            pi, pj = pairs_i[s:s + (1 << 17)], pairs_j[s:s + (1 << 17)]
            P = np.einsum('nki,nkj->nij', Hpc[pi], DinvHpc[pj])
            S = S + _sparse_sum(idx, P, pi, pj, nc, -1.0)
        out['S'] = (S + sp.diags(lam)).tocsr()
    return out


def _sparse_sum(idx, P, pi, pj, nc, sign):
    import scipy.sparse as sp
    ri = np.broadcast_to(idx[pi][:, :, None], P.shape)
    cj = np.broadcast_to(idx[pj][:, None, :], P.shape)
    m = (ri >= 0) & (cj >= 0)
    return sp.coo_matrix((sign * P[m], (ri[m], cj[m])), shape=(nc, nc)).tocsr()


def _track_pairs(trk):
    """All ordered observation pairs (i, j) of each eliminated track (incl. i == j)."""
    sel = np.nonzero(trk >= 0)[0]
    if len(sel) == 0:
        return np.zeros(0, np.int64), np.zeros(0, np.int64)
    order = sel[np.argsort(trk[sel], kind='stable')]
    ts = trk[order]
    starts = np.concatenate([[0], np.nonzero(np.diff(ts))[0] + 1])
    lens = np.diff(np.concatenate([starts, [len(ts)]]))
    PI, PJ = [], []
    for L in np.unique(lens):
        segs = starts[lens == L]
        ii, jj = np.meshgrid(np.arange(L), np.arange(L), indexing='ij')
        PI.append(order[segs[:, None] + ii.ravel()[None]].ravel())
        PJ.append(order[segs[:, None] + jj.ravel()[None]].ravel())
    return np.concatenate(PI), np.concatenate(PJ)


def _scatter_sym(S, idx, P, pi, pj, sign):
    ri = idx[pi]            # (m, w)
    cj = idx[pj]
    mr = ri >= 0
    mc = cj >= 0
    rr = np.broadcast_to(ri[:, :, None], P.shape)
    cc = np.broadcast_to(cj[:, None, :], P.shape)
    mm = mr[:, :, None] & mc[:, None, :]
    np.add.at(S, (rr[mm], cc[mm]), sign * P[mm])


def dense_to_blocks(S, layout, pattern):
    """Cut a dense reduced S into the typed blocks of ``pattern`` (list of (p, q))."""
    out = []
    for p, q in pattern:
        r0, r1 = layout.block_off[p], layout.block_off[p] + layout.block_size[p]
        c0, c1 = layout.block_off[q], layout.block_off[q] + layout.block_size[q]
        out.append(S[r0:r1, c0:c1])
    return out


# --------------------------------------------------------------------------------------
# one full linearization from raw inputs
# --------------------------------------------------------------------------------------

def linearize(scene_inputs, options, dtype=np.float64, dense=True, residual_dtype=None, obs_mask=None):
    """Residual -> Jacobians -> Schur system for one LM iteration, from raw inputs.

    ``scene_inputs``: dict with infos, pids, pix2d, pix2d_std, pix2d_dep, K, P_rig2cam,
    P_w2rig, z_coefs, pts3d (numpy); ``options``: pnorm, huber_delta, clip_pix_err,
    weight_z, depth_mode, optim_K/P/Z/X/Z0, no_grad_f_from_rz, optim_Z_1st_cam.
    """
    d = scene_inputs
    o = dict(pnorm=1.0, huber_delta=0.5, clip_pix_err=100.0, weight_z=1.0, depth_mode='log',
             optim_K=True, optim_P=True, optim_Z=True, optim_X=True, optim_Z0=True,
             no_grad_f_from_rz=False, optim_Z_1st_cam=True)
    o.update(options)
    is_log = o['depth_mode'] == 'log'
    rdt = residual_dtype or dtype
    res = residuals_with_rigs(d['infos'], d['K'], d['P_rig2cam'], d['P_w2rig'], d['z_coefs'],
                              d['pts3d'], d['pids'], d['pix2d'], d['pix2d_std'], d['pix2d_dep'],
                              is_log, o['weight_z'], o['pnorm'], o['clip_pix_err'],
                              o['huber_delta'], 1e-16, dtype=rdt)
    J_cam, J_zcf, J_pts = jacobians_with_rigs(d['infos'], d['K'], d['P_rig2cam'], d['P_w2rig'],
                                              d['z_coefs'], d['pts3d'], d['pids'], d['pix2d_std'],
                                              d['pix2d_dep'], is_log, dtype=dtype)
    lay = Layout(d['infos'], d['pids'], len(d['K']), len(d['P_w2rig']), len(d['pts3d']),
                 d['pix2d_dep'].shape[1], o['optim_K'], o['optim_P'], o['optim_Z'], o['optim_X'])
    sys_ = schur_system(J_cam, J_zcf, J_pts, res[:, :3].astype(np.float32), res[:, 6:9].astype(np.float32),
                        lay, no_grad_f_from_rz=o['no_grad_f_from_rz'],
                        optim_Z_1st_cam=o['optim_Z_1st_cam'], optim_Z0=o['optim_Z0'],
                        dense=dense, dtype=dtype, obs_mask=obs_mask)
    sys_.update(residuals=res, J_cam=J_cam, J_zcf=J_zcf, J_pts=J_pts, layout=lay)
    return sys_


# --------------------------------------------------------------------------------------
# solve (reference semantics) -- used to check the end-to-end delta
# --------------------------------------------------------------------------------------

def pcg(A_mv, b, M_mv=None, tol=1e-6, maxiter=300):
    """Preconditioned CG with the reference's stopping rule and best-so-far return
    (``ba_solver.py:1197-1238``)."""
    x = np.zeros_like(b)
    r = b - A_mv(x)
    z = M_mv(r) if M_mv is not None else r
    p = z.copy()
    rz_old = r @ z
    best = (np.inf, x, 0)
    bnorm = max(np.linalg.norm(b), 1e-12)
    for k in range(1, maxiter + 1):
        Ap = A_mv(p)
        denom = max(p @ Ap, 1e-32)
        alpha = rz_old / denom
        x = x + alpha * p
        r = r - alpha * Ap
        rn = np.linalg.norm(r)
        if rn < best[0]:
            best = (rn, x, k)
        if rn <= tol * bnorm:
            return x, k, True
        z = M_mv(r) if M_mv is not None else r
        rz_new = r @ z
        if not np.isfinite(rz_new):
            break
        beta = rz_new / max(rz_old, 1e-32)
        p = z + beta * p
        rz_old = rz_new
    return best[1], best[2], False


def solve_delta(sys_, tol=1e-6, maxiter=300):
    """delta = [delta_c, delta_p] from an oracle system with a dense S
    (``ba_solver.py:184-206``): PCG on S with the diag(A) Jacobi preconditioner, then
    delta_p = D^-1 (g_p - C delta_c)."""
    S, b = sys_['S'], sys_['b']
    dA = np.maximum(sys_['diagA'], 1e-12)
    dc, it, conv = pcg(lambda v: S @ v, b, lambda v: v / dA, tol=tol, maxiter=maxiter)
    return dc, it, conv
