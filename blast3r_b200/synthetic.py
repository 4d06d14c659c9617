"""Seeded synthetic bundle-adjustment scenes in the reference's data layout.

The reference feeds its BA hot path from ``ObservedTracks`` / ``RigsData``
(``inference/tracks.py:20-31``, ``inference/rigs.py:15-31``):

* observations are **image-sorted**; ``nppi[i]`` observations belong to image ``i``
  and inside an image they are ordered by track id (``tracks.py:853-860``);
* ``infos = int32 stack(cumsum(nppi), node_ids, cam_ids)`` (``rigs.py:50-51``);
* ``pix2d_std`` is all ones (``tracks.py:862``);
* the multi-depth channels are ``[F0, 1, F1, F2, F3]``: the constant-ones channel
  (the beta coefficient) sits at index 1 (``multidepth.py:54``).

No public dataset is used.  The five configurations below follow the shapes, sizes
and value distributions of the benchmark configurations of this build (cameras on a
circle / spherical figure-eight / forward trajectory looking at the scene, windows of
trajectory neighbours, loop-closure camera pairs, geometric track lengths, N(0,1 px)
pixel noise, 2 deg / 0.05 pose perturbation, N(0,0.05) point perturbation, focal x1.05).
Everything is drawn from ``numpy.random.default_rng(seed)``.
"""
from dataclasses import dataclass, field
import numpy as np

IMG_W, IMG_H = 512, 384
FOCAL = 600.0


@dataclass
class Scene:
    """One BA problem instance (numpy arrays, reference dtypes and layout)."""
    name: str
    n_imgs: int
    n_cams: int
    n_nodes: int
    n_tracks: int
    infos: np.ndarray        # (3, n_imgs) int32: cumsum(nppi), node_ids, cam_ids
    pids: np.ndarray         # (n_obs,) int32, image-sorted
    pix2d: np.ndarray        # (n_obs, 2) float32
    pix2d_std: np.ndarray    # (n_obs, 2) float32
    pix2d_dep: np.ndarray    # (n_obs, C) float32
    K: np.ndarray            # (n_cams, 3, 3) float32   (initial, perturbed)
    P_rig2cam: np.ndarray    # (n_cams, 4, 4) float32   (identity: no rigs)
    P_w2rig: np.ndarray      # (n_nodes, 4, 4) float32  (initial, perturbed)
    z_coefs: np.ndarray      # (n_imgs, C) float32      (initial)
    pts3d: np.ndarray        # (n_tracks, 3) float32    (initial, perturbed)
    options: dict = field(default_factory=dict)   # solver settings of the config
    truth: dict = field(default_factory=dict)     # ground-truth parameters
    meta: dict = field(default_factory=dict)

    @property
    def n_obs(self):
        return len(self.pids)

    @property
    def n_zcf(self):
        return self.pix2d_dep.shape[1]

    def lm_inputs(self):
        """Positional inputs of ``lm_step`` / the residual op, in reference order."""
        return dict(rigs=self.infos, pids=self.pids, pix2d=self.pix2d, pix2d_std=self.pix2d_std,
                    pix2d_dep=self.pix2d_dep, K=self.K, P_rig2cam=self.P_rig2cam,
                    P_w2rig=self.P_w2rig, z_coefs=self.z_coefs, pts3d=self.pts3d)


CONFIGS = {
    0: dict(name='cfg0-tiny', n_imgs=20, traj='circle', n_tracks=2_000, length=('uniform', 2, 6),
            window=8, loops=0, mono=True, weight_z=1e-4, optim_K=True, optim_P=True),
    1: dict(name='cfg1-mid', n_imgs=200, traj='figure8', n_tracks=100_000, length=('geometric', 5),
            window=8, loops=10, mono=True, weight_z=1e-4, optim_K=True, optim_P=True),
    2: dict(name='cfg2-large', n_imgs=1_000, traj='figure8', n_tracks=1_000_000, length=('geometric', 6),
            window=16, loops=20, mono=True, weight_z=1e-4, optim_K=True, optim_P=True),
    3: dict(name='cfg3-slam-window', n_imgs=64, traj='forward', n_tracks=30_000, length=('uniform', 2, 8),
            window=None, loops=0, mono=False, weight_z=1e-4, optim_K=True, optim_P=True),
    4: dict(name='cfg4-depth-stitch', n_imgs=10_000, traj='figure8', n_tracks=10_000_000,
            length=('geometric', 6), window=16, loops=200, mono=True, weight_z=1.0,
            optim_K=False, optim_P=False),
}


def _rodrigues(axis, angle):
    """Rotation matrices for unit axes (N,3) and angles (N,) [radians]."""
    axis = np.asarray(axis, np.float64)
    k = axis / np.linalg.norm(axis, axis=-1, keepdims=True)
    K = np.zeros(k.shape[:-1] + (3, 3))
    K[..., 0, 1], K[..., 0, 2] = -k[..., 2], k[..., 1]
    K[..., 1, 0], K[..., 1, 2] = k[..., 2], -k[..., 0]
    K[..., 2, 0], K[..., 2, 1] = -k[..., 1], k[..., 0]
    a = np.asarray(angle, np.float64)[..., None, None]
    return np.eye(3) + np.sin(a) * K + (1 - np.cos(a)) * (K @ K)


def _look_at(centers, target=np.zeros(3), up=np.array([0.0, 0.0, 1.0])):
    """World-to-camera rotations (x right, y down, z forward) and translations."""
    z = target[None] - centers
    z /= np.linalg.norm(z, axis=1, keepdims=True)
    x = np.cross(z, up[None])
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    y = np.cross(z, x)
    R = np.stack([x, y, z], axis=1)
    t = -np.einsum('nij,nj->ni', R, centers)
    return R, t


def _trajectory(kind, n, rng):
    if kind == 'circle':
        th = 2 * np.pi * np.arange(n) / n
        c = np.stack([3 * np.cos(th), 3 * np.sin(th), np.zeros(n)], 1)
        return _look_at(c)
    if kind == 'figure8':
        # spherical figure-eight of radius 3: azimuth A sin t, elevation B sin 2t
        t = 2 * np.pi * np.arange(n) / n
        az, el = np.deg2rad(60) * np.sin(t), np.deg2rad(20) * np.sin(2 * t)
        c = 3 * np.stack([np.cos(el) * np.cos(az), np.cos(el) * np.sin(az), np.sin(el)], 1)
        return _look_at(c)
    if kind == 'forward':
        c = np.stack([np.zeros(n), np.zeros(n), 0.1 * np.arange(n)], 1)
        R = np.repeat(np.eye(3)[None], n, 0)
        return R, -c
    raise ValueError(kind)


def _track_lengths(spec, n_tracks, max_len, rng):
    if spec[0] == 'uniform':
        L = rng.integers(spec[1], spec[2] + 1, size=n_tracks)
    else:
        L = rng.geometric(1.0 / spec[1], size=n_tracks)
    return np.clip(L, 2, np.minimum(30, max_len)).astype(np.int64)


def _sample_windows(n_imgs, window, loops, L, rng, chunk=1 << 21):
    """Per track: the L distinct camera ids it is observed in (ragged, flattened).

    A track's candidates are a window of ``window`` consecutive trajectory neighbours, or for
    a loop-closure track the union of the windows around the two images of a loop pair; its
    L cameras are the first L candidates in a random order.  The random orders come from a
    table of 4096 random permutations (one table lookup per track instead of a sort), so
    every subset of each length stays reachable."""
    T = len(L)
    is_loop = np.zeros(T, bool)
    pairs = None
    if loops > 0:
        u = rng.integers(0, n_imgs, size=loops)
        v = (u + n_imgs // 2 + rng.integers(-n_imgs // 8, n_imgs // 8 + 1, size=loops)) % n_imgs
        pairs = np.stack([u, v], 1)
        is_loop = rng.random(T) < loops / n_imgs
    W2 = 2 * window
    perm1 = rng.permuted(np.tile(np.arange(window, dtype=np.int16), (4096, 1)), axis=1)
    perm2 = rng.permuted(np.tile(np.arange(W2, dtype=np.int16), (4096, 1)), axis=1)
    L = np.minimum(L, np.where(is_loop, W2, window))
    ptr = np.concatenate([[0], np.cumsum(L)])
    cams = np.empty(int(ptr[-1]), np.int64)
    for s in range(0, T, chunk):
        e = min(T, s + chunk)
        n = e - s
        start = rng.integers(0, n_imgs, size=n)
        lp = is_loop[s:e]
        order = np.empty((n, W2), np.int16)
        order[:, :window] = perm1[rng.integers(0, 4096, size=n)]
        nl = int(lp.sum())
        if nl:
            order[lp] = perm2[rng.integers(0, 4096, size=nl)]
        offs = order.astype(np.int64)
        cand = (start[:, None] + offs[:, :window]) % n_imgs if not nl else None
        if nl:
            cand = np.empty((n, W2), np.int64)
            cand[~lp, :window] = (start[~lp, None] + offs[~lp, :window]) % n_imgs
            k = rng.integers(0, loops, size=nl)
            o = offs[lp]
            side = o >= window                     # candidate from the second window
            base = np.where(side, pairs[k, 1, None], pairs[k, 0, None]) - window // 2
            cand[lp] = (base + np.where(side, o - window, o)) % n_imgs
        m = np.arange(cand.shape[1])[None] < L[s:e, None]
        cams[ptr[s]:ptr[e]] = cand[m]
    return cams, ptr, is_loop


def make_scene(cfg, seed=None, n_tracks=None, n_imgs=None, dtype_check=True):
    """Generate configuration ``cfg`` (0..4); ``seed`` defaults to the config index.

    ``n_tracks`` / ``n_imgs`` override the sizes (for reduced test cases with the same
    generator).
    """
    c = dict(CONFIGS[cfg])
    if n_tracks is not None:
        c['n_tracks'] = n_tracks
    if n_imgs is not None:
        c['n_imgs'] = n_imgs
    rng = np.random.default_rng(cfg if seed is None else seed)
    I, T = c['n_imgs'], c['n_tracks']
    C = 5
    R, t = _trajectory(c['traj'], I, rng)

    # ---- track visibility ----
    if c['traj'] == 'forward':
        L = _track_lengths(c['length'], T, I, rng)
        start = rng.integers(0, I - L + 1)
        ptr = np.concatenate([[0], np.cumsum(L)])
        tid = np.repeat(np.arange(T), L)
        cams = start[tid] + (np.arange(ptr[-1]) - ptr[tid])
        is_loop = np.zeros(T, bool)
        # points ahead of the last frame that sees them, depth >= 1 in every frame
        last_z = 0.1 * (start + L - 1)
        depth = 1.0 + rng.random(T) * 4.0
        pts = np.stack([rng.uniform(-1.5, 1.5, T) * (depth / 3 + 0.3),
                        rng.uniform(-1.0, 1.0, T) * (depth / 3 + 0.3),
                        last_z + depth], 1)
    else:
        L = _track_lengths(c['length'], T, c['window'], rng)
        cams, ptr, is_loop = _sample_windows(I, c['window'], c['loops'], L, rng)
        L = np.diff(ptr)
        tid = np.repeat(np.arange(T), L)
        pts = rng.uniform(-1, 1, size=(T, 3))

    # ---- intrinsics ----
    if c['mono']:
        Cm = 1
        cam_ids = np.zeros(I, np.int32)
        f = np.full(1, FOCAL)
    else:
        Cm = I
        cam_ids = np.arange(I, dtype=np.int32)
        f = FOCAL * rng.uniform(0.95, 1.05, size=I)
    K_true = np.zeros((Cm, 3, 3))
    K_true[:, 0, 0] = K_true[:, 1, 1] = f
    K_true[:, 0, 2], K_true[:, 1, 2], K_true[:, 2, 2] = IMG_W / 2, IMG_H / 2, 1.0

    # ---- observations (track-major), then image-sorted ----
    Xc = np.einsum('nij,nj->ni', R[cams], pts[tid]) + t[cams]
    z = Xc[:, 2]
    fo = f[cam_ids[cams]]
    u = fo * Xc[:, 0] / z + IMG_W / 2 + rng.normal(0, 1, len(z))
    v = fo * Xc[:, 1] / z + IMG_H / 2 + rng.normal(0, 1, len(z))
    dep = np.empty((len(z), C), np.float32)
    dep[:, 0] = np.log(z)
    dep[:, 1] = 1.0
    dep[:, 2:] = rng.normal(0, 0.1, size=(len(z), C - 2))
    order = np.argsort(cams, kind='stable')      # stable: track order inside each image
    pids = tid[order].astype(np.int32)
    pix2d = np.stack([u, v], 1)[order].astype(np.float32)
    pix2d_dep = dep[order]
    nppi = np.bincount(cams, minlength=I)
    infos = np.stack([np.cumsum(nppi), np.arange(I), cam_ids]).astype(np.int32)

    # ---- initial (perturbed) parameters ----
    axis = rng.normal(size=(I, 3))
    Rp = _rodrigues(axis, np.full(I, np.deg2rad(2.0)))
    dt = rng.normal(size=(I, 3))
    dt *= 0.05 / np.linalg.norm(dt, axis=1, keepdims=True)
    P_true = np.tile(np.eye(4), (I, 1, 1))
    P_true[:, :3, :3], P_true[:, :3, 3] = R, t
    P0 = np.tile(np.eye(4), (I, 1, 1))
    P0[:, :3, :3] = Rp @ R
    P0[:, :3, 3] = np.einsum('nij,nj->ni', Rp, t) + dt
    K0 = K_true.copy()
    K0[:, 0, 0] *= 1.05
    K0[:, 1, 1] *= 1.05
    pts0 = pts + rng.normal(0, 0.05, size=pts.shape)
    z0 = np.zeros((I, C), np.float32)
    z0[:, 0] = 1.0

    options = dict(pnorm=1.0, huber_delta=1.0, clip_pix_err=100.0, weight_z=c['weight_z'],
                   depth_mode='log', optim_K=c['optim_K'], optim_P=c['optim_P'],
                   optim_Z=True, optim_X=True, optim_Z0=True)
    meta = dict(config=cfg, seed=cfg if seed is None else seed, mean_track_length=float(L.mean()),
                max_track_length=int(L.max()), n_loop_tracks=int(is_loop.sum()))
    return Scene(name=c['name'], n_imgs=I, n_cams=Cm, n_nodes=I, n_tracks=T, infos=infos,
                 pids=pids, pix2d=pix2d, pix2d_std=np.ones_like(pix2d), pix2d_dep=pix2d_dep,
                 K=K0.astype(np.float32), P_rig2cam=np.tile(np.eye(4, dtype=np.float32), (Cm, 1, 1)),
                 P_w2rig=P0.astype(np.float32), z_coefs=z0, pts3d=pts0.astype(np.float32),
                 options=options,
                 truth=dict(K=K_true.astype(np.float32), P_w2rig=P_true.astype(np.float32),
                            pts3d=pts.astype(np.float32)),
                 meta=meta)


class OnlineSequence:
    """A scene as the online loop grows it, one frame at a time (inference/pipeline.py:196-224).

    After frame q the problem holds images 0..q and every track whose last observation is in
    an image <= q.  Each frame's tracks are appended after the earlier ones with the next ids
    and, inside every image, their observations follow the earlier tracks' observations: the
    layout ``ObservedTracks.__or__`` gives the merge ``old | new`` (inference/tracks.py:96-117).
    ``frame(q)`` returns that problem as a ``Scene`` (initial parameters of the full scene).
    """

    def __init__(self, sc):
        I, T = sc.n_imgs, sc.n_tracks
        img = np.repeat(np.arange(I), np.diff(np.concatenate([[0], sc.infos[0]])))
        last = np.full(T, -1)
        np.maximum.at(last, sc.pids, img)
        t_order = np.lexsort((np.arange(T), last))          # tracks by (last image, id)
        new_id = np.empty(T, np.int64)
        new_id[t_order] = np.arange(T)
        pids = new_id[sc.pids]
        self.rows = np.lexsort((pids, img))                  # image-major, then new track id
        self.pids = pids[self.rows].astype(np.int32)
        self.img = img[self.rows]
        self.t_order = t_order
        self.n_upto = np.searchsorted(last[t_order], np.arange(I), side='right')
        self.sc = sc

    def frame(self, q):
        sc = self.sc
        nt = int(self.n_upto[q])
        keep = (self.img <= q) & (self.pids < nt)
        rows = self.rows[keep]
        nppi = np.bincount(self.img[keep], minlength=q + 1)
        cam_ids = sc.infos[2, :q + 1]
        n_cams = int(cam_ids.max()) + 1
        infos = np.stack([np.cumsum(nppi), np.arange(q + 1), cam_ids]).astype(np.int32)
        return Scene(name=f'{sc.name}-frame{q}', n_imgs=q + 1, n_cams=n_cams, n_nodes=q + 1, n_tracks=nt,
                     infos=infos, pids=np.ascontiguousarray(self.pids[keep]),
                     pix2d=sc.pix2d[rows], pix2d_std=sc.pix2d_std[rows], pix2d_dep=sc.pix2d_dep[rows],
                     K=sc.K[:n_cams], P_rig2cam=sc.P_rig2cam[:n_cams], P_w2rig=sc.P_w2rig[:q + 1],
                     z_coefs=sc.z_coefs[:q + 1], pts3d=sc.pts3d[self.t_order[:nt]],
                     options=dict(sc.options), meta=dict(sc.meta, frame=q))
