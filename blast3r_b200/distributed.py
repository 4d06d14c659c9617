"""Track-sharded linearization across GPUs (one process per GPU, torch.distributed).

Every Hpp, Hpc and Schur term belongs to one track, so tracks shard by id: each rank
eliminates its own points and accumulates a partial S, b and diag(A) in the one S
pattern every rank shares (the plan builds it from all tracks).  Per linearization:

1. ``b3r_lin_points`` on every rank, then an all-reduce (MAX) of the point-damping
   maximum, which must be global before any Hpp is inverted (ba_solver.py:579-581);
2. ``b3r_lin_assemble`` on every rank;
3. one reduce (SUM) of the contiguous S | b | diag(A) buffer to the solving rank;
4. ``b3r_lin_finalize`` there: per-type damping from the reduced diag(A)
   (ba_solver.py:572-582) and the preconditioner.

Only the reduce moves bulk data (S is ~10 MB for configs[2]); it goes over NCCL.
"""
import numpy as np
import torch
import torch.distributed as dist


def shard_tracks(pids, n_tracks, world, rank):
    """Contiguous track-id range [t0, t1) of ``rank``, balanced by observation count.
    Returns (t0, t1, observations of the range)."""
    pids = np.asarray(pids)
    cnt = np.bincount(pids, minlength=n_tracks)
    cum = np.concatenate([[0], np.cumsum(cnt)])
    total = cum[-1]
    bounds = [int(np.searchsorted(cum, total * r / world, side='left')) for r in range(world + 1)]
    bounds[0], bounds[-1] = 0, n_tracks
    return bounds[rank], bounds[rank + 1], int(cum[bounds[rank + 1]] - cum[bounds[rank]])


def shard_tracks_by_image(infos, pids, n_tracks, world):
    """Owner rank of every track: tracks ordered by their first image (then id) and cut into
    ``world`` contiguous runs of about equal observation counts, so that each rank's tracks
    share a range of images.  A rank then meets about 1/world of the image pairs (segments)
    instead of a thin slice of all of them: its pair tasks stay long and its partial S
    touches few block rows.  Returns (owner int32 [n_tracks], observations per rank)."""
    infos = np.asarray(infos)
    pids = np.asarray(pids).astype(np.int64)
    cum = np.asarray(infos[0], np.int64)
    img = np.repeat(np.arange(len(cum)), np.diff(np.concatenate([[0], cum])))
    first = np.full(n_tracks, len(cum), np.int64)
    np.minimum.at(first, pids, img)                   # first image of every track
    cnt = np.bincount(pids, minlength=n_tracks)
    order = np.lexsort((np.arange(n_tracks), first))
    cum_obs = np.cumsum(cnt[order])
    total = int(cum_obs[-1]) if n_tracks else 0
    cuts = np.searchsorted(cum_obs, [total * r / world for r in range(1, world)], side='left')
    rank_of_pos = np.zeros(n_tracks, np.int32)
    for c in cuts:
        rank_of_pos[c + 1:] += 1
    owner = np.empty(n_tracks, np.int32)
    owner[order] = rank_of_pos
    per_rank = np.bincount(owner, weights=cnt, minlength=world).astype(np.int64)
    return owner, per_rank


class ShardedSchur:
    """Runs the sharded linearization for one rank's ``BAPlan`` (built with its
    ``track_range``).  The reduced S, b, diag(A) and preconditioner are valid on ``root``."""

    def __init__(self, plan, root=0, group=None):
        self.plan, self.root, self.group = plan, root, group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        dev = plan.device
        ncp, nnz = plan.n_cam_params, int(plan.info.nnz)
        self.red = torch.empty(nnz + 2 * ncp, dtype=torch.float32, device=dev)   # S | b | diag(A)
        self.S, self.b, self.diagA = self.red[:nnz], self.red[nnz:nnz + ncp], self.red[nnz + ncp:]
        self.precond = torch.empty(ncp, dtype=torch.float32, device=dev)
        self.hpp_max = torch.empty(1, dtype=torch.float32, device=dev)
        self.outputs = (self.S, self.b, self.diagA, self.precond, self.hpp_max)
        self._own = self._order = None
        if self.world > 1:                      # every rank's track list, once (for the point exchange)
            own = torch.from_numpy(np.ascontiguousarray(plan.own_tracks, np.int64)).to(dev)
            cnt = torch.tensor([own.numel()], dtype=torch.int64, device=dev)
            cnts = [torch.empty_like(cnt) for _ in range(self.world)]
            dist.all_gather(cnts, cnt, group=self.group)
            self._counts = [int(c) for c in cnts]
            self._cap = max(max(self._counts), 1)
            padded = torch.zeros(self._cap, dtype=torch.int64, device=dev)
            padded[:own.numel()] = own
            lists = torch.empty(self.world * self._cap, dtype=torch.int64, device=dev)
            dist.all_gather_into_tensor(lists, padded, group=self.group)
            self._own = own
            self._order = torch.cat([lists[r * self._cap:r * self._cap + c] for r, c in enumerate(self._counts)])
            self._valid = torch.cat([torch.arange(r * self._cap, r * self._cap + c, device=dev)
                                     for r, c in enumerate(self._counts)])

    def gather_points(self, dp):
        """The point update of every rank's tracks on every rank: each rank sends the 3-vectors
        of its own tracks only (an all-gather of about 1/world of delta_p each), not a SUM
        all-reduce of the whole, mostly zero, vector."""
        if self.world == 1:
            return dp
        v = dp.view(-1, 3)
        send = torch.zeros(self._cap, 3, dtype=dp.dtype, device=dp.device)
        send[:self._own.numel()] = v[self._own]
        recv = torch.empty(self.world * self._cap, 3, dtype=dp.dtype, device=dp.device)
        dist.all_gather_into_tensor(recv, send, group=self.group)
        out = torch.zeros_like(v)
        out[self._order] = recv[self._valid]
        return out.view(-1)

    def linearize(self, params, opts):
        if self.world == 1:
            self.plan.linearize(params, opts, self.outputs)
            return self
        self.plan.lin_stage('points', params, opts, self.outputs)
        dist.all_reduce(self.hpp_max, op=dist.ReduceOp.MAX, group=self.group)
        self.plan.lin_stage('assemble', params, opts, self.outputs)
        dist.reduce(self.red, dst=self.root, group=self.group)
        if self.rank == self.root:
            self.plan.lin_stage('finalize', params, opts, self.outputs)
        return self


def sharded_lm_step(sharded, rigs, pids, pix2d, pix2d_std, pix2d_dep, K, P_rig2cam, P_w2rig, z_coefs, pts3d,
                    depth_mode='log', pnorm=1, clip_pix_err=100, huber_delta=0.5, min_reproj=0.01, dampen=1e-12,
                    min_loss_delta=1e-4, weight_z=1, dtype=torch.float32, verbose=False):
    """One Levenberg-Marquardt step (engine.py:206-334) over track-sharded ranks.

    Every rank holds all inputs.  The linearization is sharded (``ShardedSchur``); the root
    solves S delta_c = b with the device PCG and broadcasts delta_c; each rank back-substitutes
    its own tracks' points and an all-gather of those assembles delta_p; the objective (the
    residual op over all observations, cheap next to the linearization) is evaluated on every
    rank, so the line search takes the same decisions everywhere and every rank ends with the
    same parameters.  The plan must enable whole parameter types (bool optim flags, the
    reference's default), not masks.  Returns (update, BA_Status) like ``engine.lm_step``.
    """
    from .cujac import residual_loss
    from .engine import BA_Status, line_search
    from .plan import BAPlan
    plan = sharded.plan
    is_log = depth_mode == 'log'

    def objective(K, P_w2rig, pts3d, z_coefs):
        loss, res = residual_loss(rigs, K, P_rig2cam, P_w2rig, z_coefs, pts3d, pids, pix2d, pix2d_std, pix2d_dep,
                                  is_log, weight_z, pnorm, clip_pix_err, huber_delta)
        return loss, res, None

    init_loss, init_residuals, _ = objective(K, P_w2rig, pts3d, z_coefs)
    lo = BAPlan.lin_opts(is_depth_log=is_log, weight_z=weight_z, pnorm=pnorm, max_pix_err=clip_pix_err,
                         huber_delta=huber_delta, dampen=dampen)
    p = plan.params(K, P_rig2cam, P_w2rig, z_coefs, pts3d, pix2d_std, pix2d_dep, pix2d=pix2d)
    plan.stage_obs(pix2d, pix2d_std, pix2d_dep)          # the observation arrays may have changed
    sharded.linearize(p, lo)
    dt = torch.float64 if dtype == torch.float64 else torch.float32
    if sharded.rank == sharded.root:
        dc, _, _ = plan.pcg(sharded.S, sharded.precond, sharded.b.to(dt), tol=1e-6, maxiter=300)
    else:
        dc = torch.empty(plan.n_cam_params, dtype=dt, device=plan.device)
    if sharded.world > 1:
        dist.broadcast(dc, src=sharded.root, group=sharded.group)
    dp = sharded.gather_points(plan.backsub(p, lo, plan.workspace(), dc))   # own tracks, then all
    delta = torch.cat([dc.to(torch.float32), dp])
    i = plan.info
    n_cams, n_nodes, n_imgs, n_pts, C = i.nb_K, i.nb_P, i.nb_Z, i.n_points, plan.C
    sizes = [2 * n_cams, 6 * n_nodes, C * n_imgs, 3 * n_pts]
    assert delta.numel() == sum(sizes)
    dK, dP, dZ, dX = delta.split(sizes)
    update, new_loss, new_res = line_search(objective, K, P_w2rig, z_coefs, pts3d, delta, dK.view(n_cams, 2),
                                            dP.view(n_nodes, 6), dZ.view(n_imgs, C), dX.view(n_pts, 3), init_loss,
                                            init_residuals, min_reproj, min_loss_delta, verbose)
    return update, BA_Status(init_loss, init_residuals, new_loss, new_res)
