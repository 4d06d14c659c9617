"""CPU stand-ins for the reference's five CUDA ops (TEST INFRASTRUCTURE ONLY).

The reference's Python solver (``inference/ba_solver.py``) binds its native ops through
``extensions/cujac/__init__.py:7-22``.  To run that solver unchanged on a machine without
a GPU, ``install_into_reference()`` registers a module named
``blast3r.extensions.cujac.ba_with_rigs_cuda_kernels`` whose functions restate the
reference kernels on CPU tensors:

* ``residuals_with_rigs``  -> ``sfm_jacobian_rigs.cu:129-259, 1048-1101``
* ``jacobians_with_rigs``  -> ``sfm_jacobian_rigs.cu:323-509, 1105-1148``
* ``chol3x3_solve``        -> ``sfm_jacobian_rigs.cu:560-634, 1151-1169``
* ``blockcoo_matvec``      -> ``sfm_jacobian_rigs.cu:760-803, 1171-1219``
* ``fused_einsum_bki_bkj`` -> ``sfm_jacobian_rigs.cu:880-941, 1222-1250``

Used only by ``tests/golden/make_golden.py`` (fixture generation in a container that
has the reference checkout) and the oracle self-tests.
"""
import sys
import types

import numpy as np
import torch

from . import ba_oracle as O


def residuals_with_rigs(infos, K, P_rig2c, P_w2rig, z_coefs, pts3d, pids, pix2d, pix2d_std,
                        pix2d_dep, is_depth_log, weight_z=1.0, pnorm=-1.0, max_pix_err=100.0,
                        huber_delta=0.5, w_pts_nul=1e-16):
    out = O.residuals_with_rigs(*(t.numpy() for t in (infos, K, P_rig2c, P_w2rig, z_coefs, pts3d,
                                                        pids, pix2d, pix2d_std, pix2d_dep)),
                                is_depth_log, weight_z, pnorm, max_pix_err, huber_delta, w_pts_nul,
                                dtype=np.float32)
    # the reference returns a [n_out, n] buffer transposed to (n, n_out)
    return torch.from_numpy(np.ascontiguousarray(out.T)).transpose(0, 1)


def jacobians_with_rigs(infos, K, P_rig2c, P_w2rig, z_coefs, pts3d, pids, pix2d_std, pix2d_dep,
                        is_depth_log, float64=False):
    dt = np.float64 if float64 else np.float32
    J = O.jacobians_with_rigs(*(t.numpy() for t in (infos, K, P_rig2c, P_w2rig, z_coefs, pts3d,
                                                      pids, pix2d_std, pix2d_dep)),
                              is_depth_log, dtype=dt)
    return [torch.from_numpy(np.ascontiguousarray(j.astype(dt))) for j in J]


def chol3x3_solve(blocks, rhs, jitter=1e-12):
    x = O.chol3x3_solve(blocks.numpy(), rhs.numpy(), jitter)
    return torch.from_numpy(x.astype(blocks.numpy().dtype))


def blockcoo_matvec(blocks, row_indices, col_indices, x, HB1, WB1, transpose_blocks=False):
    N, bh, bw = blocks.shape
    r = row_indices.long()
    c = col_indices.long()
    if not transpose_blocks:
        xs = x.view(WB1, bw)[c]                                  # (N, bw)
        contrib = torch.einsum('nij,nj->ni', blocks, xs)
        y = torch.zeros(HB1, bh, dtype=blocks.dtype)
        y.index_add_(0, r, contrib)
    else:
        xs = x.view(HB1, bh)[r]
        contrib = torch.einsum('nij,ni->nj', blocks, xs)
        y = torch.zeros(WB1, bw, dtype=blocks.dtype)
        y.index_add_(0, c, contrib)
    return y.ravel()


def fused_einsum_bki_bkj(left, right):
    return torch.einsum('bki,bkj->bij', left, right).contiguous()


def make_module():
    m = types.ModuleType('blast3r.extensions.cujac.ba_with_rigs_cuda_kernels')
    for f in (residuals_with_rigs, jacobians_with_rigs, chol3x3_solve, blockcoo_matvec,
              fused_einsum_bki_bkj):
        setattr(m, f.__name__, f)
    return m


def install_into_reference(reference_src):
    """Put the reference's ``src`` dir on ``sys.path`` and register the CPU ops module
    before ``blast3r.extensions.cujac`` is first imported."""
    if reference_src not in sys.path:
        sys.path.insert(0, reference_src)
    sys.modules['blast3r.extensions.cujac.ba_with_rigs_cuda_kernels'] = make_module()
    import blast3r.extensions.cujac as cujac          # noqa: F401  (binds the module above)
    import blast3r.inference.ba_solver as ba_solver
    import blast3r.inference.engine as engine
    return ba_solver, engine
