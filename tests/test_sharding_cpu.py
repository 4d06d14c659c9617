"""Host logic of the track-sharded linearization, on CPU.

* per-rank host-only plans (``device = -1``) built with the shard ranges of
  ``blast3r_b200.distributed.shard_tracks`` share one S pattern and partition the tracks and
  observation pairs;
* two ``gloo`` ranks each compute the partial system of their tracks with the oracle,
  all-reduce S, b and diag(A) (the SUM the NCCL path does), apply the per-type damping
  from the reduced diag(A) once, and must equal the single-process system.
"""
import ctypes as C
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from blast3r_b200 import _lib as L
from blast3r_b200.distributed import shard_tracks, shard_tracks_by_image
from blast3r_b200.synthetic import make_scene
from oracle import ba_oracle as O
from tests.helpers import rel_err, scene_inputs


def _host_plan(sc, t0, t1, owner=None, rank=0):
    infos = np.ascontiguousarray(sc.infos, np.int32)
    pids = np.ascontiguousarray(sc.pids, np.int32)
    own = np.ascontiguousarray(owner, np.int32) if owner is not None else None
    d = L.PlanDesc(n_imgs=sc.n_imgs, n_cams=sc.n_cams, n_nodes=sc.n_nodes, n_tracks=sc.n_tracks, n_obs=sc.n_obs,
                   C=sc.n_zcf, infos=infos.ctypes.data_as(C.POINTER(C.c_int32)),
                   pids=pids.ctypes.data_as(C.POINTER(C.c_int32)), track_begin=t0, track_end=t1, device=-1,
                   track_owner=own.ctypes.data_as(C.POINTER(C.c_int32)) if own is not None else None, rank=rank)
    h = C.c_void_p()
    L.call('b3r_plan_create', C.byref(h), C.byref(d))
    info = L.PlanInfo()
    L.call('b3r_plan_get_info', h, C.byref(info))
    rp = np.zeros(info.n_blocks + 1, np.int32)
    ci = np.zeros(info.nnzb, np.int32)
    vo = np.zeros(info.nnzb, np.int64)
    L.call('b3r_plan_get_pattern', h, rp.ctypes.data, ci.ctypes.data, vo.ctypes.data, None, None)
    L.call('b3r_plan_destroy', h)
    return info, (rp, ci, vo)


@pytest.mark.parametrize('world', [2, 3, 8])
def test_shard_plans_share_pattern_and_partition_work(world):
    sc = make_scene(1, n_imgs=40, n_tracks=4000)
    full, pat = _host_plan(sc, 0, sc.n_tracks)
    ranges = [shard_tracks(sc.pids, sc.n_tracks, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == sc.n_tracks
    assert all(ranges[r][1] == ranges[r + 1][0] for r in range(world - 1))
    assert sum(r[2] for r in ranges) == sc.n_obs
    pairs = tracks = obs = 0
    for t0, t1, n_loc in ranges:
        info, p = _host_plan(sc, t0, t1)
        assert all(np.array_equal(a, b) for a, b in zip(p, pat))      # one S layout on every rank
        assert info.nnz == full.nnz and info.n_segments == full.n_segments
        pairs += info.n_pairs
        tracks += info.n_tracks_local
        obs += info.n_obs_local
        assert info.n_obs_local == n_loc
    assert (pairs, tracks, obs) == (full.n_pairs, full.n_tracks_local, full.n_obs_local)
    # balanced by observations (each rank within 5% of the mean)
    per = [r[2] for r in ranges]
    assert max(per) < 1.05 * sc.n_obs / world + 30


@pytest.mark.parametrize('world', [2, 4, 8])
def test_image_sharding_partitions_work_on_fewer_segments(world):
    """Tracks sharded by first image: the ranks partition tracks, observations and pairs,
    share one S layout, stay balanced by observations, and each meets far fewer image-pair
    segments (longer pair tasks) than with id-range sharding."""
    sc = make_scene(2, n_imgs=200, n_tracks=40000)
    full, pat = _host_plan(sc, 0, sc.n_tracks)
    owner, per_rank = shard_tracks_by_image(sc.infos, sc.pids, sc.n_tracks, world)
    assert owner.shape == (sc.n_tracks,) and set(np.unique(owner)) == set(range(world))
    assert per_rank.sum() == sc.n_obs and per_rank.max() < 1.05 * sc.n_obs / world + 40
    pairs = tracks = obs = tasks_img = tasks_id = 0
    for r in range(world):
        info, p = _host_plan(sc, 0, 0, owner=owner, rank=r)
        assert all(np.array_equal(a, b) for a, b in zip(p, pat))
        pairs += info.n_pairs
        tracks += info.n_tracks_local
        obs += info.n_obs_local
        tasks_img += info.n_pair_tasks
        t0, t1, _ = shard_tracks(sc.pids, sc.n_tracks, world, r)
        tasks_id += _host_plan(sc, t0, t1)[0].n_pair_tasks
    assert (pairs, tracks, obs) == (full.n_pairs, full.n_tracks_local, full.n_obs_local)
    assert tasks_img < (0.8 if world == 2 else 0.5) * tasks_id, (tasks_img, tasks_id)


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, result_path, by_image):
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        sc = make_scene(0, n_imgs=10, n_tracks=300, seed=9)
        inp, opts = scene_inputs(sc), dict(sc.options)
        if by_image:
            owner, _ = shard_tracks_by_image(sc.infos, sc.pids, sc.n_tracks, world)
            mask = owner[sc.pids] == rank
        else:
            t0, t1, _ = shard_tracks(sc.pids, sc.n_tracks, world, rank)
            mask = (sc.pids >= t0) & (sc.pids < t1)
        part = O.linearize(inp, opts, obs_mask=mask)
        lam = part['lam']
        S_part = torch.from_numpy(part['S'] - np.diag(lam))         # undamped partial S
        b_part = torch.from_numpy(part['b'].copy())
        dA_part = torch.from_numpy(part['diagA'] - lam)
        for x in (S_part, b_part, dA_part):
            dist.all_reduce(x)                                       # SUM, as the NCCL reduce
        if rank == 0:
            full = O.linearize(inp, opts)
            lay = full['layout']
            dA = dA_part.numpy()
            lam_red = np.zeros_like(dA)
            for lo, sz, nblk in ((0, 2, lay.nK), (lay.off_P, 6, lay.nP), (lay.off_Z, lay.C, lay.nZ)):
                sl = slice(lo, lo + sz * nblk)
                lam_red[sl] = 1e-12 * np.abs(dA[sl]).max()
            S = S_part.numpy() + np.diag(lam_red)
            errs = [rel_err(S, full['S']), rel_err(b_part.numpy(), full['b']),
                    rel_err(dA + lam_red, full['diagA'])]
            np.save(result_path, np.array(errs))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize('by_image', [False, True], ids=['id-ranges', 'by-image'])
def test_gloo_two_ranks_partial_systems_sum_to_full(tmp_path, by_image):
    out = str(tmp_path / 'errs.npy')
    mp.spawn(_rank_main, args=(2, _free_port(), out, by_image), nprocs=2, join=True)
    errs = np.load(out)
    assert (errs < 1e-9).all(), errs


def _gather_main(rank, world, port, result_path):
    """Each rank holds the point update of its own tracks (zeros elsewhere), as the
    back-substitution leaves it; ShardedSchur.gather_points must give every rank the full
    update."""
    from types import SimpleNamespace
    from blast3r_b200.distributed import ShardedSchur
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        sc = make_scene(0, n_imgs=10, n_tracks=300, seed=9)
        owner, _ = shard_tracks_by_image(sc.infos, sc.pids, sc.n_tracks, world)
        own = np.flatnonzero(owner == rank)
        plan = SimpleNamespace(device=torch.device('cpu'), n_cam_params=4, info=SimpleNamespace(nnz=8),
                               own_tracks=own)
        full = torch.from_numpy(np.random.default_rng(3).normal(size=(sc.n_tracks, 3)).astype(np.float32))
        mine = torch.zeros_like(full)
        mine[own] = full[own]
        got = ShardedSchur(plan).gather_points(mine.view(-1))
        np.save(result_path + f'.{rank}.npy', np.array([float((got.view(-1, 3) - full).abs().max())]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize('world', [2, 3])
def test_gloo_point_update_gathered_on_every_rank(tmp_path, world):
    out = str(tmp_path / 'gather')
    mp.spawn(_gather_main, args=(world, _free_port(), out), nprocs=world, join=True)
    for r in range(world):
        assert np.load(out + f'.{r}.npy')[0] == 0.0
