"""Shared test helpers: golden-fixture loading, scene -> tensors, tolerances."""
import glob
import os

import numpy as np
import torch

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden')

# Parity tolerances (fp32 CUDA path vs the fp64 oracle / reference):
TOL_OBS = 1e-5      # per-observation quantities (residuals, J): max|a-b| / max|b| per component
TOL_ACC = 1e-4      # accumulated blocks (S, diag A): max|a-b| / max|b|
TOL_B = 1e-5        # the reduced gradient b (north-star tolerance for b): max|a-b| / max|b|


def golden_files():
    return sorted(glob.glob(os.path.join(GOLDEN_DIR, 'golden_*.npz')))


def load_golden(path):
    z = np.load(path, allow_pickle=False)
    d = {k[3:]: z[k] for k in z.files if k.startswith('in_')}
    opts = {}
    for k in z.files:
        if k.startswith('opt_'):
            v = z[k]
            if v.ndim == 0:
                v = v.item()
                if isinstance(v, (bool, np.bool_)):
                    v = bool(v)
            else:
                v = v.astype(bool)
            opts[k[4:]] = v
    inp = dict(infos=d['rigs'], pids=d['pids'], pix2d=d['pix2d'], pix2d_std=d['pix2d_std'],
               pix2d_dep=d['pix2d_dep'], K=d['K'], P_rig2cam=d['P_rig2cam'], P_w2rig=d['P_w2rig'],
               z_coefs=d['z_coefs'], pts3d=d['pts3d'])
    ref = {k: z[k] for k in z.files if k.startswith('f64_') or k.startswith('f32_')}
    return inp, opts, ref


def scene_inputs(sc):
    d = dict(sc.lm_inputs())
    d['infos'] = d.pop('rigs')
    return d


def to_cuda(inp, device='cuda'):
    return {k: torch.from_numpy(np.ascontiguousarray(v)).to(device) for k, v in inp.items()}


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.abs(b).max() if b.size else 1.0
    return float(np.abs(a - b).max() / max(den, 1e-300)) if b.size else 0.0
