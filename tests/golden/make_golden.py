"""Generate the golden fixtures ``tests/golden/golden_*.npz`` from the REFERENCE solver.

Run in a container that has the naver/blast3r checkout (it is NOT needed on the GPU box
or by the tests, which only read the committed ``.npz`` files):

    B3R_REFERENCE=<path to blast3r checkout> python tests/golden/make_golden.py

For every case it builds a small seeded scene (``blast3r_b200.synthetic``), then runs the
reference's own ``inference/ba_solver.py`` unchanged, with the reference's five CUDA ops
replaced by the CPU restatements in ``oracle/ref_ops.py``:

* ``GaussNewtonSolver.compute_jacobians`` (``ba_solver.py:34-108``),
* ``GaussNewtonSolver.solve_delta`` (``ba_solver.py:110-182``), with ``_solver``
  wrapped to capture the damped ``SchurMatrix`` and ``J^T W r`` right before the PCG,
* ``S = A - B inv(D) C`` densified from the reference's own block matrices,
  ``b = g_c - B D^-1 g_p`` exactly as ``_solve_CG`` forms it (``ba_solver.py:184-188``),
  the damped diag(A) preconditioner (``ba_solver.py:191-192``), and the final delta.

Both the production float64 solver (``engine.py:490``) and the float32 default are run.
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from blast3r_b200.synthetic import make_scene   # noqa: E402
from oracle import ref_ops                      # noqa: E402

CASES = {
    # name: (config, n_imgs, n_tracks, seed, option overrides, edits)
    'mono_log': (0, 8, 120, 100, dict(), ('behind', 'outlier')),
    'multicam_log': (3, 8, 150, 101, dict(), ()),
    'mono_lin_flags': (0, 8, 120, 102, dict(depth_mode='lin', optim_Z0=False, no_grad_f_from_rz=True,
                                          optim_Z_1st_cam=False), ('lin',)),
    'depth_stitch': (0, 8, 120, 103, dict(optim_K=False, optim_P=False, weight_z=1.0), ()),
    'frozen_points': (0, 8, 120, 104, dict(optim_X=False), ()),
    'masked_nodes': (3, 8, 150, 105, dict(optim_P='mask:0,3', optim_Z='mask:5'), ()),
}


def _mask(spec, n):
    if isinstance(spec, str) and spec.startswith('mask:'):
        m = np.ones(n, bool)
        m[[int(v) for v in spec[5:].split(',')]] = False
        return m
    return spec


def build_case(name):
    cfg, n_imgs, n_tracks, seed, over, edits = CASES[name]
    sc = make_scene(cfg, seed=seed, n_imgs=n_imgs, n_tracks=n_tracks)
    opts = dict(sc.options)
    opts.update(no_grad_f_from_rz=False, optim_Z_1st_cam=True)
    opts.update(over)
    d = {k: np.array(v) for k, v in sc.lm_inputs().items()}
    if 'lin' in edits:
        d['pix2d_dep'][:, 0] = np.exp(d['pix2d_dep'][:, 0])     # linear-depth channel
    if 'behind' in edits:
        # move one track behind the first camera that sees it: its observation there has z <= 1e-3
        t = int(d['pids'][0])
        P = d['P_w2rig'][0]
        c = -P[:3, :3].T @ P[:3, 3]
        d['pts3d'][t] = (c - 0.5 * P[2, :3]).astype(np.float32)
    if 'outlier' in edits:
        d['pix2d'][7] += np.float32(450.0)                      # |r| clipped at 100 -> null weight
    opts['optim_P'] = _mask(opts['optim_P'], sc.n_nodes)
    opts['optim_Z'] = _mask(opts['optim_Z'], sc.n_imgs)
    return sc, d, opts


def run_reference(ba_solver, engine, d, opts, dtype):
    t = {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in d.items()}
    is_log = opts['depth_mode'] == 'log'
    res = engine.residual_func(t['rigs'], t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'],
                               t['pids'], t['pix2d'], t['pix2d_std'], t['pix2d_dep'], is_log,
                               opts['weight_z'], opts['pnorm'], opts['clip_pix_err'], opts['huber_delta'])
    residuals, err, w_pts = res.reshape(-1, 3, 3).unbind(dim=1)
    n_imgs = t['rigs'].shape[1]
    solver = ba_solver.GaussNewtonSolver(len(t['K']), len(t['P_w2rig']), n_imgs, len(t['pts3d']), 'cpu',
                                         no_grad_f_from_rz=opts['no_grad_f_from_rz'], dampen=1e-12,
                                         adaptive_dampen=True, dtype=dtype)

    def as_opt(v):
        return torch.from_numpy(v) if isinstance(v, np.ndarray) else v

    J = solver.compute_jacobians(t['rigs'], t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'],
                                 t['pids'], t['pix2d_std'], t['pix2d_dep'], is_depth_log=is_log,
                                 optim_Z_1st_cam=opts['optim_Z_1st_cam'], optim_Z0=opts['optim_Z0'],
                                 optim_K=as_opt(opts['optim_K']), optim_Z=as_opt(opts['optim_Z']),
                                 optim_P=as_opt(opts['optim_P']), optim_X=as_opt(opts['optim_X']))
    cap = {}
    orig = solver._solver

    def capture(JTJ, JTr):
        cap['JTr'] = JTr.clone()
        A = JTJ.A.to_dense()
        B = JTJ.B.to_dense()
        Cm = JTJ.C.to_dense()
        D = JTJ.D.to_dense()
        cap['S'] = A - B @ torch.linalg.inv(D) @ Cm
        g_c, g_p = JTr.tensor_split((JTJ.A.shape[0],))
        cap['b'] = g_c - (JTJ.B @ JTJ.D.solve(g_p)).to_dense().ravel()
        cap['diagA'] = JTJ.A.diag()
        cap['Dblocks'] = JTJ.D.blocks.clone() if hasattr(JTJ.D, 'blocks') else D
        out = orig(JTJ, JTr)
        cap['delta_full'] = out.clone()
        return out

    solver._solver = capture
    delta = solver.solve_delta(J, residuals, w_pts)
    dK, dP, dZ, dX = solver.unpack_delta_inplace(delta.clone())
    return dict(residuals9=res.contiguous().numpy(), S=cap['S'].numpy(), b=cap['b'].numpy(),
                JTr=cap['JTr'].numpy(), diagA=cap['diagA'].numpy(), delta=delta.numpy(),
                dK=dK.numpy(), dP=dP.numpy(), dZ=dZ.numpy(), dX=dX.numpy(),
                n_cam_params=np.int64(cap['S'].shape[0]))


def run_reference_lm_step(engine, d, opts, dtype=torch.float64, prefix='lm'):
    """One reference lm_step (engine.py:206-334), production float64 solver by default."""
    t = {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in d.items()}

    def as_opt(v):
        return torch.from_numpy(v) if isinstance(v, np.ndarray) else v
    update, st = engine.lm_step(t['rigs'], t['pids'], t['pix2d'], t['pix2d_std'], t['pix2d_dep'], t['K'],
                                t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'], depth_mode=opts['depth_mode'],
                                pnorm=opts['pnorm'], clip_pix_err=opts['clip_pix_err'],
                                huber_delta=opts['huber_delta'], weight_z=opts['weight_z'],
                                optim_K=as_opt(opts['optim_K']), optim_Z=as_opt(opts['optim_Z']),
                                optim_P=as_opt(opts['optim_P']), optim_X=as_opt(opts['optim_X']),
                                optim_Z0=opts['optim_Z0'], no_grad_f_from_rz=opts['no_grad_f_from_rz'],
                                dampen=1e-12, adaptive_dampen=True, dtype=dtype)
    return {f'{prefix}_K': update['K'].numpy(), f'{prefix}_P_w2rig': update['P_w2rig'].numpy(),
            f'{prefix}_z_coefs': update['z_coefs'].numpy(), f'{prefix}_pts3d': update['pts3d'].numpy(),
            f'{prefix}_init_loss': np.float64(st.init_loss), f'{prefix}_new_loss': np.float64(st.new_loss)}


def main():
    ref = os.environ.get('B3R_REFERENCE')
    if not ref:
        raise SystemExit('set B3R_REFERENCE to the blast3r checkout')
    ba_solver, engine = ref_ops.install_into_reference(os.path.join(ref, 'src'))
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    for name in CASES:
        sc, d, opts = build_case(name)
        out = {}
        for dt, tag in ((torch.float64, 'f64'), (torch.float32, 'f32')):
            r = run_reference(ba_solver, engine, d, opts, dt)
            for k, v in r.items():
                out[f'{tag}_{k}'] = v
        if opts['optim_Z_1st_cam']:          # lm_step has no optim_Z_1st_cam argument
            out.update(run_reference_lm_step(engine, d, opts))
            out.update(run_reference_lm_step(engine, d, opts, torch.float32, 'lm32'))
        meta = {k: (np.asarray(v) if not isinstance(v, str) else np.array(v)) for k, v in opts.items()}
        np.savez_compressed(os.path.join(HERE, f'golden_{name}.npz'),
                            **{f'in_{k}': v for k, v in d.items()},
                            **{f'opt_{k}': v for k, v in meta.items()}, **out)
        print(name, 'obs', len(d['pids']), 'cam params', out['f64_n_cam_params'],
              'max|S|', np.abs(out['f64_S']).max())


if __name__ == '__main__':
    main()
