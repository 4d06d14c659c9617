"""The reference's own solver, run for the benchmark's baselines (TEST AND BENCHMARK
INFRASTRUCTURE ONLY: the product never imports this module).

``bench.py`` times, beside the B200 path, the reference's own code on the same synthetic
inputs, from its installed copy in ``baseline/_ref`` (an offline ``pip install`` of the
reference checkout, which builds its CUDA extensions with its own ``setup.py``):

* on the GPU: ``GaussNewtonSolver.compute_jacobians`` -> ``solve_delta``
  (``inference/ba_solver.py:34-206``) with the reference's compiled CUDA ops;
* on the host cores: the same unmodified Python algebra with the five CUDA ops replaced by
  the CPU restatements of ``oracle/ref_ops.py`` (the reference has no CPU ops of its own:
  ``extensions/cujac/__init__.py:7-8`` falls back to a module that raises).

The two bind different modules under the same name, so each runs in a process of its own.
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
REF_DIR = os.path.join(ROOT, 'baseline', '_ref')


def available():
    """True when the installed reference copy is present."""
    return os.path.isfile(os.path.join(REF_DIR, 'blast3r', 'inference', 'ba_solver.py'))


def import_reference(cpu_ops):
    """(ba_solver, engine) modules of the installed reference; with ``cpu_ops`` its native
    ops module is the CPU restatement (registered before the package is first imported)."""
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    if cpu_ops:
        from oracle import ref_ops
        sys.modules['blast3r.extensions.cujac.ba_with_rigs_cuda_kernels'] = ref_ops.make_module()
    else:
        # the reference's CUDA ops as compiled from its source by oracle/build_ref.py (the
        # build the GPU tests already load); the installed package's own build otherwise
        from oracle import build_ref
        mod = build_ref.load_built()
        if mod is not None:
            sys.modules['blast3r.extensions.cujac.ba_with_rigs_cuda_kernels'] = mod
    import blast3r.extensions.cujac  # noqa: F401
    import blast3r.inference.ba_solver as ba_solver
    import blast3r.inference.engine as engine
    return ba_solver, engine


def tensors(scene_inputs, device):
    return {k: torch.from_numpy(np.ascontiguousarray(v)).to(device) for k, v in scene_inputs.items()}


def linearize(ba_solver, engine, t, opts, dtype, solve=False):
    """One reference linearization on the tensors ``t`` (cpu or cuda), as ``lm_step`` runs
    it (``engine.py:263-302``): the residual op, ``GaussNewtonSolver.compute_jacobians`` and
    ``solve_delta``.  With ``solve=False`` the solve stops where the PCG would start: its
    ``_solver`` is replaced by the reduced right-hand side b = g_c - B D^-1 g_p exactly as
    ``_solve_CG`` forms it (``ba_solver.py:184-188``) and returns a zero step, so what is
    timed is the work the fused B200 linearization replaces.  Returns (delta, b or None)."""
    is_log = opts.get('depth_mode', 'log') == 'log'
    res = engine.residual_func(t['rigs'], t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'],
                               t['pids'], t['pix2d'], t['pix2d_std'], t['pix2d_dep'], is_log, opts['weight_z'],
                               opts['pnorm'], opts['clip_pix_err'], opts['huber_delta'])
    residuals, _, w_pts = res.view(-1, 3, 3).unbind(dim=1)
    n_imgs = t['rigs'].shape[1]
    solver = ba_solver.GaussNewtonSolver(len(t['K']), len(t['P_w2rig']), n_imgs, len(t['pts3d']),
                                         t['pts3d'].device, dampen=1e-12, adaptive_dampen=True, dtype=dtype)
    out = {}
    if not solve:
        def rhs_only(JTJ, JTr):
            g_c, g_p = JTr.tensor_split((JTJ.A.shape[0],))
            out['b'] = g_c - (JTJ.B @ JTJ.D.solve(g_p)).to_dense().ravel()
            return torch.zeros_like(JTr)
        solver._solver = rhs_only
    J = solver.compute_jacobians(t['rigs'], t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'],
                                 t['pids'], t['pix2d_std'], t['pix2d_dep'], is_depth_log=is_log,
                                 optim_K=opts['optim_K'], optim_P=opts['optim_P'], optim_Z=opts['optim_Z'],
                                 optim_X=opts['optim_X'], optim_Z0=opts.get('optim_Z0', True))
    delta = solver.solve_delta(J, residuals, w_pts)
    return delta, out.get('b')
