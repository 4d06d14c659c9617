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


class BARigs:
    """Stand-in for the reference's ``RigsData`` (inference/rigs.py:16-96) with the attributes and
    methods its ``bundle_adjustment`` uses: cameras, nodes, per-image depth coefficients, ``to``,
    ``infos`` (cumulative keypoints per image, node ids, camera ids as int32) and ``update``."""

    def __init__(self, K, P_rig2cam, P_w2rig, z_coefs, cam_ids, nod_ids, depth_mode='log'):
        self.K, self.P_rig2cam, self.P_w2rig, self.z_coefs = K, P_rig2cam, P_w2rig, z_coefs
        self.cam_ids, self.nod_ids, self.depth_mode = cam_ids, nod_ids, depth_mode

    @property
    def n_imgs(self):
        return len(self.cam_ids)

    def to(self, device):
        return BARigs(*(t.to(device) for t in (self.K, self.P_rig2cam, self.P_w2rig, self.z_coefs, self.cam_ids,
                                                 self.nod_ids)), self.depth_mode)

    def infos(self, tracks):
        return torch.stack((torch.cumsum(tracks.nppi, dim=-1), self.nod_ids, self.cam_ids)).to(torch.int32)

    def update(self, **u):
        d = dict(K=self.K, P_rig2cam=self.P_rig2cam, P_w2rig=self.P_w2rig, z_coefs=self.z_coefs)
        d.update(u)
        return BARigs(d['K'], d['P_rig2cam'], d['P_w2rig'], d['z_coefs'], self.cam_ids, self.nod_ids, self.depth_mode)


class BATracks:
    """Stand-in for the reference's ``ObservedTracks`` (inference/tracks.py:20-60): keypoints
    per image, track ids, 2-D observations, their std and multi-depth values, and ``to``."""

    def __init__(self, nppi, pids, pix2d, pix2d_std, pix2d_dep):
        self.nppi, self.pids, self.pix2d, self.pix2d_std, self.pix2d_dep = nppi, pids, pix2d, pix2d_std, pix2d_dep

    def to(self, device):
        return BATracks(*(t.to(device) for t in (self.nppi, self.pids, self.pix2d, self.pix2d_std, self.pix2d_dep)))


def ba_objects(inp, device):
    """(BARigs, BATracks, pts3d) of a scene's lm_step inputs (dict of numpy arrays)."""
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(device) for k, v in inp.items()}
    infos = t['rigs'].long()
    nppi = torch.diff(torch.cat([infos[0].new_zeros(1), infos[0]]))
    rigs = BARigs(t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], infos[2], infos[1])
    return rigs, BATracks(nppi, t['pids'], t['pix2d'], t['pix2d_std'], t['pix2d_dep']), t['pts3d']
