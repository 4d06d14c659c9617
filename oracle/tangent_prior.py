"""CPU oracle of the dense tangent prior (TEST INFRASTRUCTURE ONLY).

A numpy restatement of the reference's ``_dense_tangent_prior_terms`` and
``confident_in_planar_regions`` (naver/blast3r ``src/blast3r/inference/engine.py:15-179``),
with ``depthmap_to_pts3d`` (``src/blast3r/utils/geometry.py:137-153``): the checker of the
B200 kernel ``b3r_tangent_prior``.  Pinned to the reference function itself through
``tests/golden/prior_tangent.npz`` (``tests/golden/make_golden_prior.py``).

Precision follows the reference's tensors: the combined depth, its points and derivatives
in float64 (the solver's production dtype), the reference pointmap, its tangents and the
planarity confidence in float32 (float32 reductions may round differently from torch's:
the recorded reference values agree to about 1e-7).
"""
import numpy as np


def planar_confidence(D0, alpha=1e4):
    """confident_in_planar_regions (engine.py:161-179), in the dtype of D0."""
    D0 = np.asarray(D0)
    dt = D0.dtype.type
    lx = dt(2) * D0
    lx[:, 1:] -= D0[:, :-1]
    lx[:, :-1] -= D0[:, 1:]
    ly = dt(2) * D0
    ly[1:, :] -= D0[:-1, :]
    ly[:-1, :] -= D0[1:, :]
    H, W = D0.shape
    pad = np.full((H + 2, W + 2), np.inf, D0.dtype)
    pad[1:-1, 1:-1] = D0
    mn = np.min(np.stack([pad[i:i + H, j:j + W] for i in range(3) for j in range(3)]), axis=0)
    mn = np.maximum(mn, dt(1e-12))
    lx = lx / mn
    ly = ly / mn
    return np.exp(dt(-alpha) * (lx * lx + ly * ly)).astype(D0.dtype)


def _rays(H, W, K):
    """depthmap_to_pts3d(ones, K): K^-1 (u + 1/2, v + 1/2, 1) on an H x W grid (float64)."""
    Ki = np.linalg.inv(K)
    u, v = np.meshgrid(np.arange(W) + 0.5, np.arange(H) + 0.5, indexing='xy')
    pix = np.stack([u, v, np.ones_like(u)], -1)
    return pix @ Ki.T


def tangent_prior(cam_ids, K, z_coefs, log_depth_maps, pts3d_ref, weight_tan, tan_stride=4, optim_Z0=True,
                  normalize_tangents=True, eps=1e-4):
    """(tan_loss, g_z [n_imgs, C], H_z [n_imgs, C, C]) in float64 (engine.py:15-158)."""
    n_imgs, C = z_coefs.shape
    g_z = np.zeros((n_imgs, C))
    H_z = np.zeros((n_imgs, C, C))
    loss = 0.0
    if weight_tan <= 0:
        return loss, g_z, H_z
    o = tan_stride // 2
    for i in range(n_imgs):
        Ki = np.asarray(K[cam_ids[i]], np.float64).copy()
        Ki[:2, 2] -= o
        Ki[:2] /= tan_stride
        L = np.asarray(log_depth_maps[i], np.float32)[o::tan_stride, o::tan_stride].astype(np.float64)
        if min(L.shape[1:]) < 2:                              # engine.py:82-83
            continue
        a = np.asarray(z_coefs[i], np.float64)
        D = np.exp(np.minimum(np.einsum('c,hwc->hw', a, L), 80))
        B = _rays(L.shape[0], L.shape[1], Ki)
        X = B * D[..., None]
        X0 = np.asarray(pts3d_ref[i], np.float32)[o::tan_stride, o::tan_stride]
        if not normalize_tangents:                            # engine.py:96-101
            z0 = X0[..., 2]
            m = z0 > 1e-6
            if m.any():
                r = np.sort((D[m] / z0[m]).ravel())
                scale = r[(len(r) - 1) // 2]                    # torch.median: the lower median
            else:
                scale = 1.0
            X0 = np.float32(scale) * X0      # a 0-d float64 tensor times a float32 one stays float32
        tx, ty = X[1:] - X[:-1], X[:, 1:] - X[:, :-1]
        tx0, ty0 = X0[1:] - X0[:-1], X0[:, 1:] - X0[:, :-1]
        inv_sx0 = 1.0 / np.maximum(np.linalg.norm(tx0, axis=-1, keepdims=True), np.asarray(eps, tx0.dtype))
        inv_sy0 = 1.0 / np.maximum(np.linalg.norm(ty0, axis=-1, keepdims=True), np.asarray(eps, ty0.dtype))
        tx0_hat, ty0_hat = tx0 * inv_sx0, ty0 * inv_sy0
        if normalize_tangents:
            inv_sx = 1.0 / np.maximum(np.linalg.norm(tx, axis=-1, keepdims=True), eps)
            inv_sy = 1.0 / np.maximum(np.linalg.norm(ty, axis=-1, keepdims=True), eps)
        else:
            inv_sx, inv_sy = inv_sx0, inv_sy0
        tx_hat, ty_hat = tx * inv_sx, ty * inv_sy
        rx, ry = tx_hat - tx0_hat, ty_hat - ty0_hat
        Cw = planar_confidence(X0[:, :, 2])
        wx = np.sqrt(np.maximum(Cw[1:, :] * Cw[:-1, :], 0)).astype(np.float64)
        wy = np.sqrt(np.maximum(Cw[:, 1:] * Cw[:, :-1], 0)).astype(np.float64)
        if rx.size:
            loss += weight_tan * (wx[..., None] * rx * rx).mean()
        if ry.size:
            loss += weight_tan * (wy[..., None] * ry * ry).mean()
        S = D[None] * L.transpose(2, 0, 1)                     # dD/da_c = D L_c
        dX = S[..., None] * B[None]
        dtx = dX[:, 1:] - dX[:, :-1]
        dty = dX[:, :, 1:] - dX[:, :, :-1]
        if normalize_tangents:
            dtx = (dtx - tx_hat[None] * (dtx * tx_hat[None]).sum(-1, keepdims=True)) * inv_sx[None]
            dty = (dty - ty_hat[None] * (dty * ty_hat[None]).sum(-1, keepdims=True)) * inv_sy[None]
        else:
            dtx = dtx * inv_sx[None]
            dty = dty * inv_sy[None]
        for w, r, dt in ((wx, rx, dtx), (wy, ry, dty)):
            if not r.size:
                continue
            s = weight_tan / r.size
            wf, rf, df = w.reshape(-1), r.reshape(-1, 3), dt.reshape(C, -1, 3)
            g_z[i] += s * np.einsum('n,cnk,nk->c', wf, df, rf)
            H_z[i] += s * np.einsum('n,cnk,dnk->cd', wf, df, df)
    if not optim_Z0:                                           # engine.py:153-156
        g_z[:, 0] = 0
        H_z[:, 0, :] = 0
        H_z[:, :, 0] = 0
    return float(loss), g_z, H_z


def synthetic_dense_maps(n_imgs, H, W, C, seed, K=None):
    """Seeded smooth log-depth channels [log z, 1, small smooth fields...] and a reference
    pointmap from a perturbed main depth, for tests (a tilted plane with bumps and a step)."""
    rng = np.random.default_rng(seed)
    if K is None:
        K = np.array([[1.2 * W, 0, W / 2], [0, 1.2 * W, H / 2], [0, 0, 1]], np.float32)[None]
    v, u = np.meshgrid(np.arange(H), np.arange(W), indexing='ij')
    maps, refs = [], []
    for i in range(n_imgs):
        z = 2.0 + 0.3 * (u / W) + 0.2 * np.sin(3 * v / H + i) + 0.5 * (u > W * (0.4 + 0.1 * i))
        ch = [np.log(z)]
        if C > 1:
            ch.append(np.ones_like(z))
        for c in range(2, C):
            ch.append(0.1 * np.cos((c + 1) * u / W + rng.normal()) * np.sin((c + 2) * v / H))
        L = np.stack(ch, -1).astype(np.float32)
        zr = z * (1 + 0.01 * rng.normal(size=z.shape))
        Ki = np.linalg.inv(K[0].astype(np.float64))
        pix = np.stack([u + 0.5, v + 0.5, np.ones_like(u, dtype=np.float64)], -1)
        refs.append(((pix @ Ki.T) * zr[..., None]).astype(np.float32))
        maps.append(L)
    z_coefs = np.zeros((n_imgs, C), np.float32)
    z_coefs[:, 0] = 1.0 + 0.02 * rng.normal(size=n_imgs)
    if C > 1:
        z_coefs[:, 1] = 0.05 * rng.normal(size=n_imgs)
    return np.asarray(K, np.float32), z_coefs, maps, refs
