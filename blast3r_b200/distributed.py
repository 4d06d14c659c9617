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
