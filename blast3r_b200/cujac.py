"""Drop-in for the reference's ``blast3r.extensions.cujac`` module, on the B200 library.

Same function names, argument order, defaults, output shapes and dtypes as the
reference's pybind module (``extensions/cujac/sfm_jacobian_rigs.cu:1254-1275``) and
its Python shim (``extensions/cujac/__init__.py:18-58``).  Every op runs on the CUDA
stream current in torch and calls ``libb3r.so`` through its C ABI; there is no CPU
fallback (CPU tensors raise, like the reference extension).
"""
import torch

from . import _lib as L


def _cuda(t, name, dtype=None):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise RuntimeError(f'{name} is not on CUDA device')
    if dtype is not None and t.dtype != dtype:
        raise RuntimeError(f'{name} must be {dtype}, got {t.dtype}')
    return t


def _cont(t, name, ndim, last=None, dtype=torch.float32):
    _cuda(t, name, dtype)
    if not t.is_contiguous():
        raise RuntimeError(f'{name} is not memory-contiguous')
    if t.dim() != ndim:
        raise RuntimeError(f'{name}.ndim should be == {ndim}, not {t.dim()}')
    if last is not None and t.shape[-1] != last:
        raise RuntimeError(f'{name}.shape[-1] should be == {last}, not {t.shape[-1]}')
    return t


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _check_inputs(infos, K, P_rig2c, P_w2rig, z_coefs, pts3d, pids, pix2d, pix2d_std, pix2d_dep):
    """Mirror of check_inputs (sfm_jacobian_rigs.cu:1013-1044)."""
    _cont(infos, 'infos', 2, dtype=torch.int32)
    _cont(K, 'K', 3, 3)
    _cuda(P_rig2c, 'P_rig2c', torch.float32)
    if not (P_rig2c.dim() == 3 and P_rig2c.stride(1) == 4 and P_rig2c.stride(2) == 1):
        raise RuntimeError('P_rig2c should be (N,4,4) and contiguous inside 4x4 blocks')
    _cont(P_w2rig, 'P_w2rig', 3, 4)
    _cont(z_coefs, 'z_coefs', 2)
    _cont(pts3d, 'pts3d', 2, 3)
    _cont(pids, 'pids', 1, dtype=torch.int32)
    _cont(pix2d, 'pix2d', 2, 2)
    _cont(pix2d_std, 'pix2d_std', 2, 2)
    _cont(pix2d_dep, 'pix2d_dep', 2)
    if infos.shape[0] != 3:
        raise RuntimeError('infos should have 3 rows = [nkpt_cum, node_ids, cam_ids]')
    C = pix2d_dep.shape[1]
    if C != z_coefs.shape[1]:
        raise RuntimeError('Number of Z coefs is not consistent')
    return infos.shape[1], pids.shape[0], C


def residuals_with_rigs(infos, K, P_rig2c, P_w2rig, z_coefs, pts3d, pids, pix2d, pix2d_std, pix2d_dep,
                        is_depth_log, weight_z=1.0, pnorm=-1.0, max_pix_err=100.0, huber_delta=0.5,
                        w_pts_nul=1e-16):
    """(n_obs, 9) = [residual, err, weight] per observation ((n_obs, 3) if pnorm <= 0),
    a transposed view of a [n_out, n_obs] buffer like the reference
    (``sfm_jacobian_rigs.cu:1048-1101``)."""
    n_imgs, n_obs, C = _check_inputs(infos, K, P_rig2c, P_w2rig, z_coefs, pts3d, pids, pix2d, pix2d_std,
                                     pix2d_dep)
    if not (pnorm == -1 or 0 < pnorm <= 2):
        raise RuntimeError('pnorm must be in {-1} U ]0,2]')
    n_out = 9 if pnorm > 0 else 3
    out = torch.empty((n_out, n_obs), dtype=torch.float32, device=pix2d.device)
    L.call('b3r_residuals_with_rigs', infos.data_ptr(), n_imgs, K.data_ptr(), len(K), P_rig2c.data_ptr(),
           P_rig2c.stride(0), P_w2rig.data_ptr(), len(P_w2rig), z_coefs.data_ptr(), C, pts3d.data_ptr(),
           len(pts3d), pids.data_ptr(), n_obs, pix2d.data_ptr(), pix2d_std.data_ptr(), pix2d_dep.data_ptr(),
           int(bool(is_depth_log)), float(weight_z), float(pnorm), float(max_pix_err), float(huber_delta),
           float(w_pts_nul), out.data_ptr(), _stream())
    return out.transpose(0, 1)


def residual_loss(infos, K, P_rig2c, P_w2rig, z_coefs, pts3d, pids, pix2d, pix2d_std, pix2d_dep, is_depth_log,
                  weight_z=1.0, pnorm=1.0, max_pix_err=100.0, huber_delta=0.5, residuals=True):
    """The objective of ``lm_step`` in one pass (b3r_residual_loss): (loss, residuals) with loss =
    the mean Huber error (the reference's ``err.mean()`` over the (n_obs, 3) errors, a 0-d float32
    tensor) and residuals the (n_obs, 3) residuals (a transposed view of a [3, n_obs] buffer), or
    None when ``residuals`` is False."""
    n_imgs, n_obs, C = _check_inputs(infos, K, P_rig2c, P_w2rig, z_coefs, pts3d, pids, pix2d, pix2d_std,
                                     pix2d_dep)
    dev = pix2d.device
    loss = torch.empty(1, dtype=torch.float64, device=dev)
    res = torch.empty((3, n_obs), dtype=torch.float32, device=dev) if residuals else None
    L.call('b3r_residual_loss', infos.data_ptr(), n_imgs, K.data_ptr(), len(K), P_rig2c.data_ptr(),
           P_rig2c.stride(0), P_w2rig.data_ptr(), len(P_w2rig), z_coefs.data_ptr(), C, pts3d.data_ptr(),
           len(pts3d), pids.data_ptr(), n_obs, pix2d.data_ptr(), pix2d_std.data_ptr(), pix2d_dep.data_ptr(),
           int(bool(is_depth_log)), float(weight_z), float(pnorm), float(max_pix_err), float(huber_delta),
           loss.data_ptr(), res.data_ptr() if res is not None else None, _stream())
    mean = (loss[0] / max(3 * n_obs, 1)).to(torch.float32)
    return mean, (res.transpose(0, 1) if res is not None else None)


def jacobians_with_rigs(infos, K, P_rig2c, P_w2rig, z_coefs, pts3d, pids, pix2d_std, pix2d_dep,
                        is_depth_log, float64=False):
    """[J_cam (n,3,8), J_zcf (n,1,C), J_pts (n,3,3)] (``sfm_jacobian_rigs.cu:1105-1148``)."""
    n_imgs, n_obs, C = _check_inputs(infos, K, P_rig2c, P_w2rig, z_coefs, pts3d, pids, pix2d_std,
                                     pix2d_std, pix2d_dep)
    dt = torch.float64 if float64 else torch.float32
    dev = pix2d_std.device
    J_cam = torch.empty((n_obs, 3, 8), dtype=dt, device=dev)
    J_zcf = torch.empty((n_obs, 1, C), dtype=dt, device=dev)
    J_pts = torch.empty((n_obs, 3, 3), dtype=dt, device=dev)
    L.call('b3r_jacobians_with_rigs', infos.data_ptr(), n_imgs, K.data_ptr(), len(K), P_rig2c.data_ptr(),
           P_rig2c.stride(0), P_w2rig.data_ptr(), len(P_w2rig), z_coefs.data_ptr(), C, pts3d.data_ptr(),
           len(pts3d), pids.data_ptr(), n_obs, pix2d_std.data_ptr(), pix2d_dep.data_ptr(),
           int(bool(is_depth_log)), int(bool(float64)), J_cam.data_ptr(), J_zcf.data_ptr(), J_pts.data_ptr(),
           _stream())
    return [J_cam, J_zcf, J_pts]


def _dtype_code(t):
    if t.dtype == torch.float32:
        return L.B3R_F32
    if t.dtype == torch.float64:
        return L.B3R_F64
    raise RuntimeError('Only float32/float64 supported')


def chol3x3_solve(blocks, rhs, jitter=1e-12):
    """Batched 3x3 SPD solve (``sfm_jacobian_rigs.cu:1151-1169``)."""
    _cuda(blocks, 'blocks')
    _cuda(rhs, 'rhs')
    if not (blocks.is_contiguous() and rhs.is_contiguous()):
        raise RuntimeError('blocks and rhs must be contiguous')
    if not (blocks.dim() == 3 and blocks.shape[1:] == (3, 3)):
        raise RuntimeError('blocks must have shape [N,3,3]')
    if not (rhs.dim() == 2 and rhs.shape[1] == 3 and rhs.shape[0] == blocks.shape[0]):
        raise RuntimeError('rhs must have shape [N,3]')
    if blocks.dtype != rhs.dtype:
        raise RuntimeError('dtype mismatch between blocks and rhs')
    out = torch.empty_like(rhs)
    L.call('b3r_chol3x3_solve', blocks.data_ptr(), rhs.data_ptr(), out.data_ptr(), blocks.shape[0],
           float(jitter), _dtype_code(blocks), _stream())
    return out


def blockcoo_matvec(blocks, row_indices, col_indices, x, HB1, WB1, transpose_blocks=False):
    """y = A x or A^T x for a block-COO A (``sfm_jacobian_rigs.cu:1171-1219``)."""
    _cuda(blocks, 'blocks')
    _cuda(x, 'x')
    _cuda(row_indices, 'row_indices')
    _cuda(col_indices, 'col_indices')
    if not blocks.is_contiguous() or blocks.dim() != 3:
        raise RuntimeError('blocks must be contiguous [N,bh,bw]')
    if not x.is_contiguous():
        raise RuntimeError('x must be contiguous')
    if blocks.dtype != x.dtype:
        raise RuntimeError('dtype mismatch')
    if row_indices.dtype != col_indices.dtype or row_indices.dtype not in (torch.int32, torch.int64):
        raise RuntimeError('indices must both be int32 or int64')
    row_indices = row_indices.contiguous()
    col_indices = col_indices.contiguous()
    N, bh, bw = blocks.shape
    in_len = HB1 * bh if transpose_blocks else WB1 * bw
    out_len = WB1 * bw if transpose_blocks else HB1 * bh
    if x.numel() != in_len:
        raise RuntimeError('x has wrong length for the provided shapes')
    y = torch.empty(out_len, dtype=blocks.dtype, device=blocks.device)
    L.call('b3r_blockcoo_matvec', blocks.data_ptr(), bh, bw, row_indices.data_ptr(), col_indices.data_ptr(),
           int(row_indices.dtype == torch.int64), N, x.data_ptr(), y.data_ptr(), HB1, WB1,
           int(bool(transpose_blocks)), _dtype_code(blocks), _stream())
    return y


def fused_einsum_bki_bkj(left, right):
    """einsum('bki,bkj->bij') with strided batches (``sfm_jacobian_rigs.cu:1222-1250``)."""
    _cuda(left, 'left')
    _cuda(right, 'right')
    if left.dim() != 3 or right.dim() != 3:
        raise RuntimeError('expected [B,K,I] and [B,K,J]')
    if left.shape[0] != right.shape[0] or left.shape[1] != right.shape[1]:
        raise RuntimeError('B or K mismatch')
    if left.dtype != right.dtype:
        raise RuntimeError('dtype mismatch')
    if left.stride(2) != 1 or right.stride(2) != 1:
        raise RuntimeError('inner stride must be 1')
    B, K, I = left.shape
    J = right.shape[2]
    out = torch.empty((B, I, J), dtype=left.dtype, device=left.device)
    L.call('b3r_fused_einsum_bki_bkj', left.data_ptr(), left.stride(0), left.stride(1), right.data_ptr(),
           right.stride(0), right.stride(1), out.data_ptr(), B, K, I, J, _dtype_code(left), _stream())
    return out


# reference names (extensions/cujac/__init__.py:18-22)
compute_residuals_with_rigs = residuals_with_rigs
compute_jacobians_with_rigs = jacobians_with_rigs


# Lie-algebra update of SE(3) (extensions/cujac/__init__.py:27-58): the step after the path
def skew_symmetric(w, device):
    wx, wy, wz = w.T
    res = w.new_zeros((len(w), 3, 3), device=device)
    res[:, 2, 1], res[:, 1, 2] = wx, -wx
    res[:, 2, 0], res[:, 0, 2] = -wy, wy
    res[:, 0, 1], res[:, 1, 0] = -wz, wz
    return res


def hat_se3(xi):
    hat = xi.new_zeros((len(xi), 4, 4))
    hat[:, :3, :3] = skew_symmetric(xi[:, :3], device=xi.device)
    hat[:, :3, 3] = xi[:, 3:]
    return hat


def exp_se3(xi):
    """exp(hat_se3(xi)), the matrix exponential the reference takes with torch.matrix_exp, in
    closed form: with w = xi[:, :3] (angle th = |w|, W = [w]x) and v = xi[:, 3:],
    R = I + A W + B W^2 and t = (I + B W + C W^2) v, A = sin(th)/th, B = (1 - cos th)/th^2,
    C = (th - sin th)/th^3 (Rodrigues' formula and the left Jacobian of SE(3); Barfoot,
    "State Estimation for Robotics", 2017, sec. 7.1.3), Taylor series below th = 1e-3, in
    float64.  Batched torch.matrix_exp reads its squaring counts back to the host; this form
    keeps the line search free of that synchronisation."""
    x = xi.to(torch.float64)
    w, v = x[:, :3], x[:, 3:]
    th2 = (w * w).sum(-1)
    small = th2 < 1e-6
    th = torch.where(small, torch.ones_like(th2), th2).sqrt()
    s, c = torch.sin(th), torch.cos(th)
    A = torch.where(small, 1 - th2 / 6 + th2 * th2 / 120, s / th)
    B = torch.where(small, 0.5 - th2 / 24 + th2 * th2 / 720, (1 - c) / (th * th))
    Cc = torch.where(small, 1 / 6 - th2 / 120 + th2 * th2 / 5040, (th - s) / (th * th * th))
    W = skew_symmetric(w, device=xi.device)
    W2 = W @ W
    eye = torch.eye(3, dtype=torch.float64, device=xi.device)
    out = x.new_zeros((len(x), 4, 4))
    out[:, :3, :3] = eye + A[:, None, None] * W + B[:, None, None] * W2
    out[:, :3, 3] = ((eye + B[:, None, None] * W + Cc[:, None, None] * W2) @ v[:, :, None])[:, :, 0]
    out[:, 3, 3] = 1
    return out.to(xi.dtype)
