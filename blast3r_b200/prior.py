"""Dense tangent prior on the depth coefficients, on the B200 kernel ``b3r_tangent_prior``.

``dense_tangent_prior_terms`` has the signature, defaults, checks and results of the
reference's ``_dense_tangent_prior_terms`` (inference/engine.py:15-158): the prior's loss and,
with ``compute_gn``, its Gauss-Newton terms (g_z [n_imgs, C], H_z [n_imgs, C, C]) on the
depth coefficients, for every image in one launch instead of a per-image loop.
"""
import ctypes as C

import numpy as np
import torch

from . import _lib as L


class DenseMap(C.Structure):
    _fields_ = [('log_depth', C.c_void_p), ('pts3d_ref', C.c_void_p), ('H', C.c_int32), ('W', C.c_int32),
                ('channel_stride', C.c_int32), ('reserved', C.c_int32)]


def _median_scales(z_coefs, log_depth_maps, pts3d_ref, tan_stride, dtype):
    """Per image, the reference's scale of the reference pointmap when the tangents are not
    normalised: the median of D / z0 over the grid cells with z0 > 1e-6 (engine.py:96-101)."""
    sub = slice(tan_stride // 2, None, tan_stride)
    out = []
    for i in range(len(log_depth_maps)):
        Lm = log_depth_maps[i][sub, sub].to(dtype)
        D = torch.exp(torch.einsum('c,hwc->hw', z_coefs[i].to(dtype), Lm).clamp(max=80))
        z0 = pts3d_ref[i][sub, sub][..., 2]
        m = z0 > 1e-6
        out.append(torch.median(D[m] / z0[m]).to(torch.float64) if m.any() else D.new_tensor(1.0, dtype=torch.float64))
    return torch.stack(out)


def dense_tangent_prior_terms(rigs, K, z_coefs, log_depth_maps, conf, pts3d_ref, *, weight_tan=0.0, tan_stride=4,
                              optim_Z0=True, dtype=torch.float32, compute_gn=True, normalize_tangents=True,
                              eps=1e-4):
    """(tan_loss, g_z, H_z) of the dense tangent prior, in ``dtype``; g_z and H_z are None
    when ``compute_gn`` is False.  ``conf`` is checked for presence only, like the reference
    (the weights come from the reference pointmap's planarity)."""
    n_imgs, Cz = z_coefs.shape
    if weight_tan <= 0:
        return (z_coefs.new_zeros((), dtype=dtype),
                None if not compute_gn else z_coefs.new_zeros((n_imgs, Cz), dtype=dtype),
                None if not compute_gn else z_coefs.new_zeros((n_imgs, Cz, Cz), dtype=dtype))
    assert tan_stride >= 1
    assert None not in (log_depth_maps, conf, pts3d_ref)
    assert len(log_depth_maps) == len(conf) == len(pts3d_ref) == n_imgs
    dev = z_coefs.device
    if dev.type != 'cuda':
        raise RuntimeError('dense_tangent_prior_terms runs on the GPU: pass CUDA tensors')
    keep = []
    maps = (DenseMap * n_imgs)()
    cells = 1
    o = tan_stride // 2
    for i in range(n_imgs):
        Lm, X0 = log_depth_maps[i], pts3d_ref[i]
        assert Lm.ndim == 3 and Lm.shape[2] == Cz, \
            f'expected log_depth_maps n_imgs x (H,W,C), got {tuple(Lm.shape)}'
        assert X0.shape[:2] == Lm.shape[:2] and X0.shape[2] == 3, 'pts3d_ref must be n_imgs x (H,W,3)'
        Lm = Lm.to(device=dev, dtype=torch.float32)
        if not (Lm.stride(2) == 1 and Lm.stride(0) == Lm.shape[1] * Lm.stride(1)):
            Lm = Lm.contiguous()
        X0 = X0.to(device=dev, dtype=torch.float32).contiguous()
        keep += [Lm, X0]
        H, W = Lm.shape[:2]
        maps[i] = DenseMap(Lm.data_ptr(), X0.data_ptr(), H, W, Lm.stride(1), 0)
        cells = max(cells, max(0, (H - o + tan_stride - 1) // tan_stride) * max(0, (W - o + tan_stride - 1) // tan_stride))
    raw = np.frombuffer(bytes(maps), dtype=np.uint8)
    maps_d = torch.from_numpy(raw.copy()).to(dev)
    cam_ids = rigs.to(dev)[2].to(torch.int32).contiguous()
    Kf = K.detach().to(device=dev, dtype=torch.float32).contiguous()
    zc = z_coefs.detach().to(device=dev, dtype=torch.float32).contiguous()
    scale = None
    if not normalize_tangents:
        scale = _median_scales(zc, log_depth_maps, pts3d_ref, tan_stride, dtype).to(dev).contiguous()
    loss = torch.empty(1, dtype=torch.float64, device=dev)
    g = torch.empty(n_imgs, Cz, dtype=torch.float64, device=dev) if compute_gn else None
    Hz = torch.empty(n_imgs, Cz, Cz, dtype=torch.float64, device=dev) if compute_gn else None
    L.call('b3r_tangent_prior', maps_d.data_ptr(), n_imgs, int(cells), Kf.data_ptr(), cam_ids.data_ptr(),
           zc.data_ptr(), Cz, scale.data_ptr() if scale is not None else None, int(tan_stride), float(weight_tan),
           float(eps), int(bool(optim_Z0)), int(bool(normalize_tangents)), loss.data_ptr(),
           g.data_ptr() if g is not None else None, Hz.data_ptr() if Hz is not None else None,
           torch.cuda.current_stream().cuda_stream)
    return (loss[0].to(dtype), g.to(dtype) if g is not None else None, Hz.to(dtype) if Hz is not None else None)
