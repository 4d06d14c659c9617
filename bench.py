#!/usr/bin/env python
"""Benchmark of the BA linearization + Schur assembly hot path (one JSON line on rank 0).

A step is one linearization of the whole problem: residual, Jacobians, IRLS weights,
per-track 3x3 point elimination and assembly of the Schur-reduced camera/depth system S
and its gradient b (on several GPUs also the all-reduce of the point-damping maximum and
the NCCL reduce of the partial S, b and diag(A) to rank 0, which then damps S).

Workloads (seeded synthetic data of the benchmark configurations, tracks sharded by id
across ranks; strong scaling: the total problem is fixed):
  headline   configs[2]: 1,000 cameras, 1M tracks, ~5.8M observations, mono focal, K=4
  configs4   configs[4]: the depth-stitch phase, 10,000 cameras, 10M tracks, ~58M
             observations, focal and poses fixed, omega = 1 (only depth-coefficient blocks)
The observation arrays are larger than the 126 MB L2, so no flush is needed between steps.

On one GPU the line also carries: one full LM iteration on configs[2], ten LM iterations of
configs[1], configs[3]'s relinearization latency (direct and CUDA graph), the reference's own
GPU path on the same B200 and its CPU path on the host cores.  On N GPUs every workload
carries a parity record against a single-GPU linearization of the same problem.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
"""
import argparse
import datetime
import hashlib
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = 'observations linearized+Schur-assembled/sec'
UNIT = 'observations/s'


def parse_args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=20)
    ap.add_argument('--warmup', type=int, default=5)
    ap.add_argument('--impl', default='b200', choices=['b200', 'reference'])
    ap.add_argument('--config', type=int, default=2)
    ap.add_argument('--tracks', type=int, default=None,
                    help='override the headline configuration\'s track count (same generator; profiling cases)')
    ap.add_argument('--no-configs4', action='store_true', help='skip the configs[4] sub-record')
    ap.add_argument('--configs4-tracks', type=int, default=None, help='configs[4] track count (default: full)')
    ap.add_argument('--configs4-steps', type=int, default=10)
    ap.add_argument('--no-extras', action='store_true',
                    help='headline step only (no LM iterations, latency records or reference timings)')
    ap.add_argument('--cpu-sample-tracks', type=int, default=200000,
                    help='tracks of the bounded CPU-baseline sample (same generator)')
    ap.add_argument('--ref-step-tracks', type=int, default=200000,
                    help='tracks per step of the reference (CPU) arm')
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--e2e-steps', type=int, default=8)
    ap.add_argument('--channels', type=int, default=None,
                    help='keep the first C depth channels of the scene (C = 2: one log-depth channel and beta)')
    ap.add_argument('--no-reference-gpu', action='store_true', help='skip timing the reference\'s GPU path')
    ap.add_argument('--internal', default=None, help=argparse.SUPPRESS)
    return ap.parse_args(argv)


def dist_env():
    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    return world, rank, local


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""
    FIELDS = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
              'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
              'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.f = tempfile.NamedTemporaryFile('w+', suffix='.csv', delete=False)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(['nvidia-smi', f'--id={self.gpu}', f'--query-gpu={self.FIELDS}',
                                          '--format=csv,noheader,nounits', '-lms', '200'],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except (OSError, ValueError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        self.f.flush()
        self.f.seek(0)
        sm, mx, reasons = [], [], set()
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        for line in self.f.read().strip().splitlines():
            parts = [p.strip() for p in line.split(',')]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == 'active':
                    reasons.add(nm)
        os.unlink(self.f.name)
        if not sm:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': ['unavailable'], 'samples': 0}
        return {'sm_mhz': float(np.median(sm)), 'sm_max_mhz': float(max(mx)), 'reasons': sorted(reasons),
                'samples': len(sm)}


def measured_peaks():
    path = os.path.join(ROOT, 'MEASURED_PEAKS.json')
    if os.path.isfile(path):
        with open(path) as f:
            p = json.load(f)
        return float(p['hbm_gbs']), 'measured'
    return 6650.0, 'fallback'


# ------------------------------------------------------------------------------------------
# synthetic scenes, shared by the ranks of a job through a file cache
# ------------------------------------------------------------------------------------------
_SCENE_ARRAYS = ('infos', 'pids', 'pix2d', 'pix2d_std', 'pix2d_dep', 'K', 'P_rig2cam', 'P_w2rig', 'z_coefs',
                 'pts3d')


def cached_scene(cfg, n_tracks=None, seed=None):
    """``make_scene(cfg, ...)`` through a file cache: the first process that asks for a scene
    generates and saves it, the others (the other ranks of this job, later runs on the same
    machine) load it.  The key includes the generator's source, so a changed generator never
    reads an old scene."""
    import fcntl
    from blast3r_b200 import synthetic
    with open(synthetic.__file__, 'rb') as f:
        key = hashlib.sha1(f.read() + repr((cfg, n_tracks, seed)).encode()).hexdigest()[:16]
    d = os.environ.get('B3R_SCENE_CACHE', os.path.join(tempfile.gettempdir(), 'b3r_scene_cache'))
    try:
        os.makedirs(d, exist_ok=True)
        lock = open(os.path.join(d, f'cfg{cfg}_{key}.lock'), 'w')
    except OSError:
        return synthetic.make_scene(cfg, seed=seed, n_tracks=n_tracks)
    path = os.path.join(d, f'cfg{cfg}_{key}.npz')
    with lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        if os.path.isfile(path):
            z = np.load(path, allow_pickle=False)
            meta = json.loads(str(z['meta_json']))
            return synthetic.Scene(name=meta['name'], n_imgs=meta['n_imgs'], n_cams=meta['n_cams'],
                                   n_nodes=meta['n_nodes'], n_tracks=meta['n_tracks'],
                                   **{k: z[k] for k in _SCENE_ARRAYS}, options=meta['options'],
                                   meta=meta['meta'])
        sc = synthetic.make_scene(cfg, seed=seed, n_tracks=n_tracks)
        meta = dict(name=sc.name, n_imgs=sc.n_imgs, n_cams=sc.n_cams, n_nodes=sc.n_nodes, n_tracks=sc.n_tracks,
                    options=sc.options, meta=sc.meta)
        tmp = path + f'.{os.getpid()}.tmp.npz'
        try:
            np.savez(tmp, meta_json=np.array(json.dumps(meta)), **{k: getattr(sc, k) for k in _SCENE_ARRAYS})
            os.replace(tmp, path)
        except OSError:
            try:
                os.unlink(tmp)
            except OSError:
                pass
        return sc


def channel_subset(sc, C):
    """The scene with its first C depth channels (and coefficients) only.  The generator's
    channel 0 is the log-depth and channel 1 the constant 1 (beta), so C = 2 is the
    one-channel depth model alpha F + beta of the reference's first BA phase."""
    if C is None or C == sc.n_zcf:
        return sc
    import dataclasses
    return dataclasses.replace(sc, pix2d_dep=np.ascontiguousarray(sc.pix2d_dep[:, :C]),
                               z_coefs=np.ascontiguousarray(sc.z_coefs[:, :C]))


# ------------------------------------------------------------------------------------------
# roofline bookkeeping: compulsory fp32 bytes of one linearization
# ------------------------------------------------------------------------------------------
def algorithmic_bytes(n_obs, n_tracks, plan_info, block_size):
    """Compulsory bytes of one linearization (fp32): per observation pix2d 8 + std 8 +
    depth channels 4C + image id 4 + residual write 12 = 52 B (C = 5); per track point 12 +
    track offset 4 = 16 B; S (upper-triangle scalars) and b written once."""
    bs = np.asarray(block_size, np.int64)
    nnz_upper = int(plan_info.nnz) - int((bs * (bs - 1) // 2).sum())
    C = 5
    per_obs = 8 + 8 + 4 * C + 4 + 12
    return per_obs * n_obs + 16 * n_tracks + 4 * (nnz_upper + int(plan_info.n_cam_params)), nnz_upper


def kernel_source_sha():
    """Hash of the kernel and planner sources: a committed ncu summary is used only when it
    was captured from these exact sources."""
    h = hashlib.sha1()
    for f in ('b3r_schur.cu', 'b3r_common.cuh', 'b3r_plan.cpp', 'b3r_plan.h'):
        with open(os.path.join(ROOT, 'blast3r_b200', 'csrc', f), 'rb') as fh:
            h.update(fh.read())
    return h.hexdigest()[:16]


def profile_traffic(name, units):
    """DRAM bytes per launch of each pass for this rank's workload, from the committed ncu
    summary profiles/traffic_<name>.txt (a reduced case of the same generator): each pass's
    captured bytes scaled by the units it processes (observations for points and diag, tracks
    for factor, pairs for pairs).  Used only when the summary's source_sha equals the hash of
    the current kernel and planner sources; otherwise (None, why): a capture of other sources
    is never used."""
    path = os.path.join(ROOT, 'profiles', f'traffic_{name}.txt')
    if not os.path.isfile(path):
        return None, 'no capture'
    vals = {}
    with open(path) as f:
        for line in f:
            if ':' in line:
                k, v = line.split(':', 1)
                vals[k.strip()] = v.strip()
    if vals.get('source_sha') != kernel_source_sha():
        return None, 'capture is of other sources'
    n_obs, n_tracks, n_pairs = units
    scale = {'points': n_obs / float(vals['units_obs']), 'diag': n_obs / float(vals['units_obs']),
             'factor': n_tracks / float(vals['units_tracks']), 'pairs': n_pairs / float(vals['units_pairs'])}
    out = {p: (float(vals[f'{p}_dram_read']) + float(vals[f'{p}_dram_write'])) * scale[p] for p in scale}
    return out, f'{os.path.relpath(path, ROOT)} (reduced case scaled by units)'


# ------------------------------------------------------------------------------------------
# one workload on this rank
# ------------------------------------------------------------------------------------------
class Workload:
    PASSES = ['prep', 'points', 'factor', 'diag', 'pairs', 'finalize']

    def __init__(self, cfg, n_tracks, world, rank, dev, obs_local):
        import torch
        from blast3r_b200.distributed import ShardedSchur, shard_tracks_by_image
        from blast3r_b200.plan import BAPlan
        self.cfg, self.world, self.rank, self.dev = cfg, world, rank, dev
        tg = time.perf_counter()
        sc = self.sc = cached_scene(cfg, n_tracks=n_tracks)
        self.scene_s = time.perf_counter() - tg
        # tracks sharded by first image (each rank's tracks share a range of images)
        owner, per_rank = shard_tracks_by_image(sc.infos, sc.pids, sc.n_tracks, world)
        self.n_local = int(per_rank[rank])
        self.tracks_local = int((owner == rank).sum())
        o = sc.options
        tp = time.perf_counter()
        plan = self.plan = BAPlan(sc.infos, sc.pids, sc.n_cams, sc.n_nodes, sc.n_tracks, sc.n_zcf,
                                  optim_K=o['optim_K'], optim_P=o['optim_P'], optim_Z=o['optim_Z'],
                                  optim_X=o['optim_X'], track_owner=owner, rank=rank, device=dev,
                                  obs_local=obs_local)
        torch.cuda.synchronize(dev)
        self.plan_s = time.perf_counter() - tp
        rows = plan.input_obs()
        self.obs_local = obs_local
        # host arrays this rank reads: its observations (all of them on one GPU) and the
        # parameters
        self.host_obs = {k: np.ascontiguousarray(getattr(sc, k)[rows] if obs_local else getattr(sc, k))
                         for k in ('pix2d', 'pix2d_std', 'pix2d_dep')}
        self.host_par = {k: np.ascontiguousarray(getattr(sc, k)) for k in ('K', 'P_rig2cam', 'P_w2rig', 'z_coefs',
                                                                          'pts3d')}
        self.t = {k: torch.from_numpy(v).to(dev) for k, v in {**self.host_obs, **self.host_par}.items()}
        self.p = self.params(self.t)
        self.lo = BAPlan.lin_opts(weight_z=o['weight_z'], pnorm=o['pnorm'], max_pix_err=o['clip_pix_err'],
                                  huber_delta=o['huber_delta'])
        self.sharded = ShardedSchur(plan)

    def params(self, t):
        return self.plan.params(t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'], t['pix2d_std'],
                                t['pix2d_dep'], pix2d=t['pix2d'])

    def step(self):
        self.sharded.linearize(self.p, self.lo)

    def release(self):
        import torch
        for k in list(self.__dict__):
            if k not in ('cfg', 'world', 'rank', 'dev', 'scene_s', 'plan_s', 'n_local', 'tracks_local'):
                delattr(self, k)
        torch.cuda.empty_cache()


def timed(fn, steps, warmup, world, dev, clocks=None):
    """Device time of `steps` calls of fn after `warmup` untimed ones: CUDA events on the
    launching stream, barrier + synchronize on both sides, max over ranks.  Returns ms total."""
    import torch
    import torch.distributed as dist
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx = ClockSampler(dev.index) if clocks is not None else None
    if ctx is not None:
        ctx.__enter__()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    if ctx is not None:
        ctx.__exit__(None, None, None)
        clocks.update(ctx.summary())
    ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return float(ms.item())


def pass_times(wl, reps=5):
    """Device time of each pass on this rank (events between the launches, same inputs)."""
    import torch
    from blast3r_b200 import _lib as L
    S, b, dA, pc, hm = outs = wl.sharded.outputs
    acc = {k: 0.0 for k in Workload.PASSES}
    for _ in range(reps):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(Workload.PASSES) + 1)]
        S.zero_(); b.zero_(); dA.zero_(); hm.zero_()
        ev[0].record()
        for j, nm in enumerate(Workload.PASSES):
            if nm == 'finalize':
                wl.plan.lin_stage('finalize', wl.p, wl.lo, outs)
            else:
                pas = dict(prep=L.PASS_PREP, points=L.PASS_POINTS, factor=L.PASS_FACTOR, diag=L.PASS_DIAG,
                           pairs=L.PASS_PAIRS)[nm]
                wl.plan.lin_pass(pas, wl.p, wl.lo, outs)
            ev[j + 1].record()
        torch.cuda.synchronize()
        for j, nm in enumerate(Workload.PASSES):
            acc[nm] += ev[j].elapsed_time(ev[j + 1]) / reps
    tot = sum(acc.values())
    return {k: {'ms': round(v, 4), 'share': round(v / tot, 4)} for k, v in acc.items()}


def e2e_measure(wl, steps):
    """The same step through the public API from HOST buffers: every step copies this rank's
    inputs (its observation arrays, the camera parameters and the points) from
    pinned memory, re-stages the observations, linearizes (with the NCCL reduce on N GPUs),
    and rank 0 reads S and b back; all inside the timed region.  Two device input sets:
    step k+1's copies run on a copy stream while step k computes.  Returns (ms, h2d bytes,
    d2h bytes) of this rank."""
    import torch
    import torch.distributed as dist
    dev, world, rank = wl.dev, wl.world, wl.rank
    pin = {k: torch.from_numpy(v).pin_memory() for k, v in {**wl.host_obs, **wl.host_par}.items()}
    S, b = wl.sharded.S, wl.sharded.b
    S_h = torch.empty(S.numel(), dtype=torch.float32).pin_memory()
    b_h = torch.empty(b.numel(), dtype=torch.float32).pin_memory()
    h2d = sum(v.numel() * v.element_size() for v in pin.values())
    d2h = (S_h.numel() + b_h.numel()) * 4 if rank == 0 else 0
    sets = [wl.t, {k: torch.empty_like(v) for k, v in wl.t.items()}]
    psets = [wl.params(s_) for s_ in sets]
    cs = torch.cuda.Stream(device=dev)
    copied = [torch.cuda.Event(), torch.cuda.Event()]
    freed = [torch.cuda.Event(), torch.cuda.Event()]

    def issue_copy(k):
        with torch.cuda.stream(cs):
            if k >= 2:
                cs.wait_event(freed[k % 2])          # step k-2 is done with this set
            for key, src in pin.items():
                sets[k % 2][key].copy_(src, non_blocking=True)
            copied[k % 2].record(cs)

    def compute(k):
        cur = torch.cuda.current_stream()
        cur.wait_event(copied[k % 2])
        s_ = sets[k % 2]
        wl.plan.stage_obs(s_['pix2d'], s_['pix2d_std'], s_['pix2d_dep'])
        wl.sharded.linearize(psets[k % 2], wl.lo)
        freed[k % 2].record(cur)
        if rank == 0:
            S_h.copy_(S, non_blocking=True)
            b_h.copy_(b, non_blocking=True)

    def run(n):
        cs.wait_stream(torch.cuda.current_stream())   # copies start after the timing event
        issue_copy(0)
        for k in range(n):
            if k + 1 < n:
                issue_copy(k + 1)
            compute(k)

    run(2)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    run(steps)
    e1.record()
    torch.cuda.synchronize(dev)
    ms = torch.tensor([e0.elapsed_time(e1), h2d, d2h], dtype=torch.float64, device=dev)
    if world > 1:
        m = ms[:1].clone()
        dist.all_reduce(m, op=dist.ReduceOp.MAX)
        dist.all_reduce(ms, op=dist.ReduceOp.SUM)
        ms[0] = m[0]
    wl.plan.stage_obs(wl.t['pix2d'], wl.t['pix2d_std'], wl.t['pix2d_dep'])   # back to the first set
    return float(ms[0]), int(ms[1]), int(ms[2])


def parity_vs_single_gpu(wl):
    """N > 1: rank 0 linearizes the whole problem on its own GPU (one plan over all tracks,
    the global input arrays) and compares the reduced S, b and preconditioner of the timed
    run with it (max|a - b| / max|b|).  Outside the timed region."""
    import torch
    import torch.distributed as dist
    from blast3r_b200.plan import BAPlan
    torch.cuda.synchronize(wl.dev)
    dist.barrier()
    out = None
    if wl.rank == 0:
        sc, o = wl.sc, wl.sc.options
        full = BAPlan(sc.infos, sc.pids, sc.n_cams, sc.n_nodes, sc.n_tracks, sc.n_zcf, optim_K=o['optim_K'],
                      optim_P=o['optim_P'], optim_Z=o['optim_Z'], optim_X=o['optim_X'], device=wl.dev)
        t = {k: torch.from_numpy(np.ascontiguousarray(getattr(sc, k))).to(wl.dev)
             for k in ('pix2d', 'pix2d_std', 'pix2d_dep', 'K', 'P_rig2cam', 'P_w2rig', 'z_coefs', 'pts3d')}
        p = full.params(t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'], t['pix2d_std'],
                        t['pix2d_dep'], pix2d=t['pix2d'])
        s = full.linearize(p, wl.lo)
        torch.cuda.synchronize(wl.dev)

        def rel(a, b):
            a, b = a.double(), b.double()
            return float((a - b).abs().max() / b.abs().max().clamp_min(1e-300))
        out = {'vs': 'one-GPU linearization of the same problem (rank 0)',
               'rel_err_S': rel(wl.sharded.S, s.S_vals), 'rel_err_b': rel(wl.sharded.b, s.b),
               'rel_err_precond': rel(wl.sharded.precond, s.precond),
               'tolerance': {'S': 1e-4, 'b': 1e-5}}
        out['ok'] = out['rel_err_S'] < 1e-4 and out['rel_err_b'] < 1e-5
        del full, s, t, p
        torch.cuda.empty_cache()
    dist.barrier()
    return out


def measure_workload(wl, steps, warmup, peak, peak_kind, want_clocks, e2e_steps):
    """Timed steps, per-pass times, roofline, e2e and (N > 1) parity of one workload."""
    clocks = {} if want_clocks else None
    ms_total = timed(wl.step, steps, warmup, wl.world, wl.dev, clocks)
    ms_step = ms_total / steps
    sc, plan = wl.sc, wl.plan
    passes = pass_times(wl)
    dom = max((k for k in passes if k not in ('prep', 'finalize')), key=lambda k: passes[k]['ms'])
    # compulsory bytes of what this rank processes: its observations and tracks, and S, b
    B, nnz_upper = algorithmic_bytes(wl.n_local, wl.tracks_local, plan.info, plan.block_size)
    dom_ms = passes[dom]['ms']
    R = int(plan.info.record_floats)
    inter = {'elimination_records': 2 * 4 * R * int(plan.info.n_obs_local),
             'pair_lists': 8 * int(plan.info.n_pairs),
             'what': 'written by the diag pass and read by the pairs pass (records), read by the pairs pass '
                     '(pair lists): traffic of this design on top of the algorithmic bytes'}
    trafficv, tsrc = (profile_traffic(f'configs{wl.cfg}', (wl.n_local, wl.tracks_local, int(plan.info.n_pairs)))
                      if wl.world == 1 else (None, 'N > 1'))
    traffic = trafficv.get(dom) if trafficv else None
    roof = {'bound': 'hbm', 'kernel': f'{dom} pass ({passes[dom]["share"]:.2f} of the step)',
            'achieved': round(B / (dom_ms * 1e-3) / 1e9, 2), 'peak': peak, 'unit': 'GB/s',
            'frac': round(B / (dom_ms * 1e-3) / 1e9 / peak, 4), 'traffic': traffic,
            'traffic_source': tsrc, 'algorithmic_bytes': int(B), 'launch_ms': dom_ms,
            'peak_kind': f'of {peak_kind}',
            'bytes_rule': '52 B per observation + 16 B per track + 4 B per upper S scalar and per b entry '
                          '(this rank\'s observations and tracks)',
            'step': {'achieved': round(B / (ms_step * 1e-3) / 1e9, 2),
                     'frac': round(B / (ms_step * 1e-3) / 1e9 / peak, 4), 'ms': ms_step,
                     'traffic': sum(trafficv.values()) if trafficv else None},
            'intermediate_bytes': inter, 'passes': passes}
    rec = {'value': sc.n_obs * steps / (ms_total * 1e-3), 'unit': UNIT, 'ms_per_step': ms_step, 'steps': steps,
           'warmup': warmup, 'roofline': roof,
           'config': {'workload': f'configs[{wl.cfg}]', 'n_obs': sc.n_obs, 'n_tracks': sc.n_tracks,
                      'n_imgs': sc.n_imgs, 'mean_track_length': sc.meta['mean_track_length'],
                      'n_obs_pairs_rank0': int(plan.info.n_pairs), 'nnz_S': int(plan.info.nnz),
                      'depth_stitch_passes': bool(plan.info.depth_stitch),
                      'parallelism': f'track-sharded x{wl.world} (tracks by first image)' +
                                     (' + NCCL reduce of S, b' if wl.world > 1 else ''),
                      'l2': 'inputs larger than L2, no flush'},
           'setup_s': {'scene': round(wl.scene_s, 2), 'plan_rank0': round(wl.plan_s, 2)}}
    if clocks is not None:
        rec['clocks'] = clocks
    if e2e_steps:
        ms_e, h2d, d2h = e2e_measure(wl, e2e_steps)
        rec['e2e'] = {'value': sc.n_obs * e2e_steps / (ms_e * 1e-3), 'unit': UNIT, 'h2d_bytes_per_step': h2d,
                      'd2h_bytes_per_step': d2h}
    if wl.world > 1:
        rec['parity'] = parity_vs_single_gpu(wl)
    return rec


# ------------------------------------------------------------------------------------------
# LM iterations and latency (one GPU)
# ------------------------------------------------------------------------------------------
def lm_iterations(cfg, n_iter, warm, dev, n_tracks=None):
    """engine.lm_step repeated n_iter times from the configuration's initial parameters (each
    step's update feeds the next), after `warm` untimed steps from the same start.  Returns
    ms per iteration (CUDA events) and the loss before and after."""
    import torch
    from blast3r_b200.engine import lm_step
    sc = cached_scene(cfg, n_tracks=n_tracks)
    o = sc.options
    t0 = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in sc.lm_inputs().items()}

    def run(n):
        # the iteration loop of the reference's bundle_adjustment (engine.py:484-499): keep the
        # update while the loss decreases, stop at the first step that does not
        t = dict(t0)
        st, done = None, 0
        for _ in range(n):
            upd, st = lm_step(t['rigs'], t['pids'], t['pix2d'], t['pix2d_std'], t['pix2d_dep'], t['K'],
                              t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'], pnorm=o['pnorm'],
                              clip_pix_err=o['clip_pix_err'], huber_delta=o['huber_delta'],
                              weight_z=o['weight_z'], optim_K=o['optim_K'], optim_P=o['optim_P'],
                              dtype=torch.float64)
            done += 1
            if st.new_loss >= st.init_loss:
                break
            t.update(upd)
        return st, done
    first, _ = run(1)
    run(warm)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    tw = time.perf_counter()
    e0.record()
    last, done = run(n_iter)
    e1.record()
    torch.cuda.synchronize(dev)
    return {'ms': e0.elapsed_time(e1) / done, 'wall_ms': 1e3 * (time.perf_counter() - tw) / done,
            'plan_ms': plan_time_ms(sc, dev),
            'iterations': done, 'loss_first': [float(first.init_loss), float(first.new_loss)],
            'loss_last': float(last.new_loss),
            'what': 'engine.lm_step: residual op, fused linearization, PCG on S (tol 1e-6, <= 300 iterations), '
                    'back-substitution, line search; float64 solve like the reference\'s bundle_adjustment'}


def latency_record(cfg, dev, n=1000, online_planning=False):
    """One relinearization as an online caller sees it (host call to result, synchronised):
    direct calls and CUDA-graph replays, p50/p99 over n."""
    import torch
    from blast3r_b200.plan import BAPlan
    sc = cached_scene(cfg)
    o = sc.options
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in sc.lm_inputs().items()}
    plan_ms = plan_time_ms(sc, dev)
    plan = BAPlan(t['rigs'], t['pids'], sc.n_cams, sc.n_nodes, sc.n_tracks, sc.n_zcf, optim_K=o['optim_K'],
                  optim_P=o['optim_P'], device=dev)
    p = plan.params(t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'], t['pix2d_std'],
                    t['pix2d_dep'], pix2d=t['pix2d'])
    lo = BAPlan.lin_opts(weight_z=o['weight_z'], pnorm=o['pnorm'], max_pix_err=o['clip_pix_err'],
                         huber_delta=o['huber_delta'])
    outs = plan.new_outputs()

    def pct(v):
        v = np.asarray(v)
        return {'p50': round(float(np.percentile(v, 50)), 4), 'p99': round(float(np.percentile(v, 99)), 4)}

    def lat(fn):
        for _ in range(20):
            fn()
        torch.cuda.synchronize(dev)
        out = []
        for _ in range(n):
            ts = time.perf_counter()
            fn()
            torch.cuda.synchronize(dev)
            out.append(1e3 * (time.perf_counter() - ts))
        return out
    direct = lat(lambda: plan.linearize(p, lo, outs))
    graph, _ = plan.capture(p, lo, outs)
    replay = lat(graph.replay)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(100):
        graph.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    dev_ms = e0.elapsed_time(e1) / 100
    del graph
    return {'workload': f'configs[{cfg}]', 'n_obs': sc.n_obs, 'unit': 'ms', 'n': n, 'direct': pct(direct),
            'cuda_graph': pct(replay), 'device_ms_per_replay': round(dev_ms, 4),
            'plan_ms': plan_ms, 'online_planning': online_plan_record(cfg, dev) if online_planning else None}


def online_plan_record(cfg, dev):
    """Planning cost of the online loop's track merges (inference/pipeline.py:196-224) over the
    configuration's frames: each frame's problem (the earlier frames' tracks, then the new
    frame's, ObservedTracks.__or__ layout) planned from scratch (b3r_plan_create) and appended to
    the previous frame's plan (b3r_plan_append).  Each plan is timed from the device structure
    tensors to the uploaded plan, synchronised."""
    import torch
    from blast3r_b200.plan import BAPlan
    from blast3r_b200.synthetic import OnlineSequence
    seq = OnlineSequence(cached_scene(cfg))
    frames = []
    for q in range(1, seq.sc.n_imgs):
        s = seq.frame(q)
        frames.append((torch.from_numpy(np.ascontiguousarray(s.infos)).to(dev),
                       torch.from_numpy(np.ascontiguousarray(s.pids)).to(dev), s.n_cams, s.n_nodes, s.n_tracks,
                       s.n_zcf, s.n_obs))

    def run(incremental):
        prev, ts = None, []
        for infos, pids, nc, nn, nt, C, _ in frames:
            torch.cuda.synchronize(dev)
            t0 = time.perf_counter()
            plan = BAPlan(infos, pids, nc, nn, nt, C, device=dev, retain=incremental,
                          base=prev if incremental else None)
            torch.cuda.synchronize(dev)
            ts.append(1e3 * (time.perf_counter() - t0))
            prev = plan if incremental else None
        return ts
    run(True)
    # host timings on a shared machine are noisy: each frame's best of three passes per mode
    fulls, incs = [], []
    for _ in range(3):
        fulls.append(run(False))
        incs.append(run(True))
    full, inc = np.min(fulls, axis=0), np.min(incs, axis=0)
    return {'frames': len(frames), 'unit': 'ms', 'repeats': 3,
            'last_frame': {'n_obs': frames[-1][6], 'create_ms': round(float(full[-1]), 2),
                           'append_ms': round(float(inc[-1]), 2)},
            'all_frames': {'create_ms': round(float(full.sum()), 1), 'append_ms': round(float(inc.sum()), 1)},
            'what': 'plan of each online frame (old | new): b3r_plan_create from scratch vs b3r_plan_append to the '
                    'previous frame\'s plan, structure read back from the device, plan uploaded; per frame the best '
                    'of three passes'}


def plan_time_ms(sc, dev, reps=3):
    """Median time of a plan for the scene's structure (BAPlan: the structure read back from the
    device, b3r_plan_create's host planning and the upload of the plan), synchronised: what a
    change of the problem structure costs before the first linearization."""
    import torch
    from blast3r_b200.plan import BAPlan
    o = sc.options
    infos = torch.from_numpy(np.ascontiguousarray(sc.infos)).to(dev)     # device structure tensors, as the
    pids = torch.from_numpy(np.ascontiguousarray(sc.pids)).to(dev)       # reference's pipeline holds them
    ts = []
    for _ in range(reps):
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        plan = BAPlan(infos, pids, sc.n_cams, sc.n_nodes, sc.n_tracks, sc.n_zcf, optim_K=o['optim_K'],
                      optim_P=o['optim_P'], optim_Z=o['optim_Z'], optim_X=o['optim_X'], device=dev)
        torch.cuda.synchronize(dev)
        ts.append(1e3 * (time.perf_counter() - t0))
        del plan
    return round(float(np.median(ts)), 2)


# ------------------------------------------------------------------------------------------
# the reference's own code (subprocesses: its GPU path, its CPU path)
# ------------------------------------------------------------------------------------------
# The reference's GPU path cannot run this workload: its fused_einsum_bki_bkj dispatch
# (extensions/cujac/sfm_jacobian_rigs.cu:965-1006) has no (I, J, K) case for the blocks of 5
# depth coefficients against 6 pose columns, and on a B200 the call crashed the process
# (SIGSEGV in ba_solver.py:875, __matmul__obpc_obpr) instead of raising.  It is not run again.
REFERENCE_GPU_UNAVAILABLE = ('the reference\'s CUDA einsum has no kernel for the 5-coefficient x 6-pose blocks of '
                             'this configuration (sfm_jacobian_rigs.cu:965-1006); on a B200 its solver crashed with '
                             'SIGSEGV at ba_solver.py:875, so it is not run')


def internal_ref_gpu(args):
    """Child process: the reference's GaussNewtonSolver on this B200 with its own compiled
    CUDA ops, float64 (its production dtype) and float32; the linearization up to the PCG, and
    the full solve_delta (PCG and back-substitution)."""
    import faulthandler
    import torch
    from oracle import ref_runner as RR
    faulthandler.enable()
    ba_solver, engine = RR.import_reference(cpu_ops=False)
    sc = channel_subset(cached_scene(args.config, n_tracks=args.tracks), args.channels)
    t = RR.tensors(sc.lm_inputs(), 'cuda')
    out = {'n_obs': sc.n_obs, 'workload': f'configs[{args.config}]', 'depth_channels': sc.n_zcf}

    def run(dtype, solve, reps=3):
        RR.linearize(ba_solver, engine, t, sc.options, dtype, solve)     # warm-up
        torch.cuda.synchronize()
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            RR.linearize(ba_solver, engine, t, sc.options, dtype, solve)
            torch.cuda.synchronize()
            ts.append(time.perf_counter() - t0)
        return 1e3 * float(np.median(ts))
    for name, dt in (('f64', torch.float64), ('f32', torch.float32)):
        ms = run(dt, False)
        out[f'linearize_{name}_ms'] = round(ms, 2)
        out[f'linearize_{name}_obs_per_s'] = sc.n_obs / (ms * 1e-3)
    ms = run(torch.float64, True, reps=2)
    out['solve_f64_ms'] = round(ms, 2)
    out['peak_gpu_mem_gb'] = round(torch.cuda.max_memory_allocated() / 2**30, 2)
    print(json.dumps(out))


def b200_same_workload(cfg, n_tracks, channels, dev, reps=5):
    """This library on the reference-GPU workload: the fused linearization (host call to
    result, synchronised, median of reps) and the linearization + device PCG (float64
    vectors, the reference's tol and maxiter) + point back-substitution."""
    import torch
    from blast3r_b200.plan import BAPlan
    sc = channel_subset(cached_scene(cfg, n_tracks=n_tracks), channels)
    o = sc.options
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in sc.lm_inputs().items()}
    plan = BAPlan(t['rigs'], t['pids'], sc.n_cams, sc.n_nodes, sc.n_tracks, sc.n_zcf, optim_K=o['optim_K'],
                  optim_P=o['optim_P'], device=dev)
    p = plan.params(t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'], t['pix2d_std'],
                    t['pix2d_dep'], pix2d=t['pix2d'])
    lo = BAPlan.lin_opts(weight_z=o['weight_z'], pnorm=o['pnorm'], max_pix_err=o['clip_pix_err'],
                         huber_delta=o['huber_delta'])
    outs = plan.new_outputs()

    def lin():
        return plan.linearize(p, lo, outs)

    def solve():
        s_ = plan.linearize(p, lo, outs)
        x, _, _ = plan.pcg(s_.S_vals, s_.precond, s_.b.double())
        return s_.backsub(x.float())

    def wall(fn):
        fn()
        torch.cuda.synchronize(dev)
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            fn()
            torch.cuda.synchronize(dev)
            ts.append(time.perf_counter() - t0)
        return 1e3 * float(np.median(ts))
    out = {'linearize_ms': round(wall(lin), 3), 'solve_ms': round(wall(solve), 3)}
    out['linearize_obs_per_s'] = sc.n_obs / (out['linearize_ms'] * 1e-3)
    del plan, p, outs, t
    torch.cuda.empty_cache()
    return out


def reference_gpu_record(dev, channels=2, cfg=2):
    """The reference's own GaussNewtonSolver on this B200 (its compiled CUDA ops, a child
    process) beside this library on the same workload: configs[cfg]'s scene with its first
    `channels` depth channels, the depth model the reference's CUDA einsum dispatch covers
    (extensions/cujac/sfm_jacobian_rigs.cu:965-1006 has no 5-coefficient x 6-pose kernel,
    so the headline C = 5 workload does not run there)."""
    ref = run_child('ref-gpu', ['--config', str(cfg), '--channels', str(channels)])
    rec = {'workload': f'configs[{cfg}] scene, depth channels 0..{channels - 1} (alpha F + beta)',
           'reference': ref,
           'what': 'reference: residual_func + GaussNewtonSolver.compute_jacobians + solve_delta up to its PCG '
                   '(linearize_*) and the whole solve_delta (solve_f64); b200: the fused linearization and the '
                   'linearization + device PCG + back-substitution; host call to result, synchronised, median'}
    if 'unavailable' in ref:
        return rec
    ours = b200_same_workload(cfg, None, channels, dev)
    rec['b200'] = ours
    rec['speedup'] = {'linearize_vs_ref_f32': ref['linearize_f32_ms'] / ours['linearize_ms'],
                      'linearize_vs_ref_f64': ref['linearize_f64_ms'] / ours['linearize_ms'],
                      'solve_vs_ref_f64': ref['solve_f64_ms'] / ours['solve_ms']}
    return rec


def internal_ref_cpu(args):
    """Child process: the reference's own Python solver on the host cores (its five CUDA ops
    replaced by CPU restatements), float64, on a bounded sample of the workload."""
    import torch
    from oracle import ref_runner as RR
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    ba_solver, engine = RR.import_reference(cpu_ops=True)
    from blast3r_b200.synthetic import make_scene
    sc = make_scene(args.config, n_tracks=args.tracks, seed=1000)
    t = RR.tensors(sc.lm_inputs(), 'cpu')
    RR.linearize(ba_solver, engine, t, sc.options, torch.float64)        # warm-up
    ts = []
    t_all = time.perf_counter()
    while len(ts) < max(1, args.steps) or (time.perf_counter() - t_all < 10 and len(ts) < 20):
        t0 = time.perf_counter()
        RR.linearize(ba_solver, engine, t, sc.options, torch.float64)
        ts.append(time.perf_counter() - t0)
    print(json.dumps({'n_obs': sc.n_obs, 'n_tracks': sc.n_tracks, 'cores': cores, 'steps': len(ts),
                      'times_s': ts, 'value': sc.n_obs * len(ts) / sum(ts)}))


def run_child(mode, extra):
    cmd = [sys.executable, os.path.abspath(__file__), '--internal', mode] + extra
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=900, cwd=ROOT)
    lines = [ln for ln in r.stdout.strip().splitlines() if ln.startswith('{')]
    if r.returncode != 0 or not lines:
        tail = (r.stderr or r.stdout).strip().splitlines()[-12:] or ['no output']
        return {'unavailable': f'{mode} exited {r.returncode}', 'stderr_tail': [t[:300] for t in tail]}
    return json.loads(lines[-1])


def cpu_baseline(cfg, n_tracks):
    from oracle import ref_runner as RR
    if RR.available():
        r = run_child('ref-cpu', ['--config', str(cfg), '--tracks', str(n_tracks), '--steps', '3'])
        if 'unavailable' not in r:
            return {'value': r['value'], 'unit': UNIT, 'cores': r['cores'], 'kind': 'reference',
                    'sample': f'configs[{cfg}] generator with {n_tracks} tracks ({r["n_obs"]} observations), '
                              f'{r["steps"]} linearizations: the reference\'s own inference/ba_solver.py '
                              f'(compute_jacobians + solve_delta up to its PCG, float64) on the host cores '
                              f'(torch, {r["cores"]} threads), its five CUDA ops replaced by CPU restatements '
                              f'(oracle/ref_ops.py); {sum(r["times_s"]):.1f} s'}
    return cpu_baseline_port(cfg, min(n_tracks, 20000))


def cpu_baseline_port(cfg, n_tracks):
    """The oracle port on a bounded sample (single process): used when the reference's
    installed copy is absent."""
    from blast3r_b200.synthetic import make_scene
    from oracle import ba_oracle as O
    sc = make_scene(cfg, n_tracks=n_tracks)
    d = dict(sc.lm_inputs())
    d['infos'] = d.pop('rigs')
    t = time.perf_counter()
    O.linearize(d, sc.options, dtype=np.float64, dense=False, residual_dtype=np.float32)
    dt = time.perf_counter() - t
    return {'value': sc.n_obs / dt, 'unit': UNIT, 'cores': 1, 'kind': 'port',
            'sample': f'configs[{cfg}] generator with {n_tracks} tracks ({sc.n_obs} observations), '
                      f'oracle/ba_oracle.linearize (numpy float64, sparse S), {dt:.1f} s'}


# ------------------------------------------------------------------------------------------
# the reference arm: the reference's own CPU path
# ------------------------------------------------------------------------------------------
def _ref_shard(d, t0, t1):
    """The sub-problem of tracks [t0, t1): their observations only, the global parameter
    layout kept (image counts recounted, track ids unchanged)."""
    keep = (d['pids'] >= t0) & (d['pids'] < t1)
    cum = d['infos'][0]
    img = np.repeat(np.arange(len(cum)), np.diff(np.concatenate([[0], cum])))
    out = dict(d)
    out['infos'] = d['infos'].copy()
    out['infos'][0] = np.cumsum(np.bincount(img[keep], minlength=len(cum))).astype(d['infos'].dtype)
    for k in ('pids', 'pix2d', 'pix2d_std', 'pix2d_dep'):
        out[k] = np.ascontiguousarray(d[k][keep])
    return out


def _ref_worker(job):
    """One worker of the port arm: the oracle linearization of one track shard."""
    from oracle import ba_oracle as O
    d, opts = job
    s = O.linearize(d, opts, dtype=np.float64, dense=False, residual_dtype=np.float32)
    lay = s['layout']
    types = ((0, 2, lay.nK), (lay.off_P, 6, lay.nP), (lay.off_Z, lay.C, lay.nZ))
    return s['S'], s['b'], s['diagA'], s['lam'], types


def run_reference(args):
    """The reference's own CPU implementation of the path on the host cores: its
    inference/ba_solver.py (installed copy, torch on every host thread, float64 as in
    production) with the five CUDA ops restated on CPU, each step the linearization of a
    bounded sample of the workload (compute_jacobians + solve_delta up to its PCG).  Rank 0
    alone runs; the others exit."""
    world, rank, _ = dist_env()
    if rank != 0:
        return
    from oracle import ref_runner as RR
    if not RR.available():
        return run_reference_port(args)
    import torch
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    ba_solver, engine = RR.import_reference(cpu_ops=True)
    from blast3r_b200.synthetic import make_scene
    sc = make_scene(args.config, n_tracks=args.ref_step_tracks, seed=1000)
    t = RR.tensors(sc.lm_inputs(), 'cpu')
    times = []
    for step in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        RR.linearize(ba_solver, engine, t, sc.options, torch.float64)
        if step >= args.warmup:
            times.append(time.perf_counter() - t0)
    value = sc.n_obs * len(times) / float(np.sum(times))
    sample = (f'configs[{args.config}] generator, {args.ref_step_tracks} tracks ({sc.n_obs} observations) per step: '
              f'the reference\'s own inference/ba_solver.py (compute_jacobians + solve_delta up to its PCG, '
              f'float64) on {cores} host threads, its CUDA ops restated on CPU (oracle/ref_ops.py)')
    print(json.dumps({'impl': 'reference', 'metric': METRIC, 'value': value, 'unit': UNIT, 'n_gpus': args.gpus,
                      'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': 1e3 * float(np.mean(times)),
                      'higher_is_better': True, 'scaling': 'strong', 'vs_baseline': None, 'dtype': 'f64',
                      'data': 'synthetic', 'config': {'workload': f'configs[{args.config}] (bounded CPU sample)'},
                      'cpu_baseline': {'value': value, 'unit': UNIT, 'cores': cores, 'kind': 'reference',
                                       'sample': sample},
                      'e2e': {'value': value, 'unit': UNIT, 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}))


def run_reference_port(args):
    """Fallback reference arm when the installed reference copy is absent: the oracle port
    (numpy float64, sparse S) in one spawned process per host core, track shards summed."""
    import multiprocessing as mp
    from scipy import sparse
    from blast3r_b200.synthetic import make_scene
    n_workers = max(1, min(os.cpu_count() or 1, 64))
    for k in ('OMP_NUM_THREADS', 'MKL_NUM_THREADS', 'OPENBLAS_NUM_THREADS'):
        os.environ[k] = '1'
    tracks = min(4000 * n_workers, 400000)
    times = []
    sc = make_scene(args.config, n_tracks=tracks, seed=1000)
    d = dict(sc.lm_inputs())
    d['infos'] = d.pop('rigs')
    bounds = np.linspace(0, sc.n_tracks, n_workers + 1).astype(int)
    jobs = [(_ref_shard(d, bounds[w], bounds[w + 1]), sc.options) for w in range(n_workers)]
    with mp.get_context('spawn').Pool(n_workers) as pool:
        pool.map(_ref_worker, [])
        for step in range(args.warmup + args.steps):
            t = time.perf_counter()
            parts = pool.map(_ref_worker, jobs)
            lam_parts = sum(pt[3] for pt in parts)
            S = sum(pt[0] for pt in parts) - sparse.diags(lam_parts)
            dA = sum(pt[2] for pt in parts) - lam_parts
            lam = np.zeros_like(dA)
            for lo, sz, nblk in parts[0][4]:
                if sz * nblk:
                    lam[lo:lo + sz * nblk] = 1e-12 * np.abs(dA[lo:lo + sz * nblk]).max()
            (S + sparse.diags(lam)).tocsr()
            if step >= args.warmup:
                times.append(time.perf_counter() - t)
    value = sc.n_obs * len(times) / float(np.sum(times))
    sample = (f'configs[{args.config}] generator, {tracks} tracks ({sc.n_obs} observations) per step, oracle port '
              f'(numpy float64, sparse S) in {n_workers} processes by track range (installed reference absent)')
    print(json.dumps({'impl': 'reference', 'metric': METRIC, 'value': value, 'unit': UNIT, 'n_gpus': args.gpus,
                      'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': 1e3 * float(np.mean(times)),
                      'higher_is_better': True, 'scaling': 'strong', 'vs_baseline': None, 'dtype': 'f64',
                      'data': 'synthetic', 'config': {'workload': f'configs[{args.config}] (bounded CPU sample)'},
                      'cpu_baseline': {'value': value, 'unit': UNIT, 'cores': n_workers, 'kind': 'port',
                                       'sample': sample},
                      'e2e': {'value': value, 'unit': UNIT, 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}))


# ------------------------------------------------------------------------------------------
# the B200 arm
# ------------------------------------------------------------------------------------------
def run_b200(args):
    import torch
    import torch.distributed as dist

    world, rank, local = dist_env()
    # Libraries (NCCL) may print to the process's stdout; keep stdout for the one JSON line.
    json_fd = os.dup(1)
    os.dup2(2, 1)
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    if world > 1:
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=600), device_id=dev)
    peak, peak_kind = measured_peaks()

    wall = {}                     # wall-clock seconds of each part of this run
    t_run = time.perf_counter()

    def lap(name, t0):
        wall[name] = round(time.perf_counter() - t0, 1)
        return time.perf_counter()
    t0 = time.perf_counter()
    wl = Workload(args.config, args.tracks, world, rank, dev, obs_local=world > 1)
    head = measure_workload(wl, args.steps, args.warmup, peak, peak_kind, want_clocks=True,
                            e2e_steps=args.e2e_steps)
    t0 = lap('headline', t0)
    sc = wl.sc
    extras = {}
    if not args.no_extras:
        if world == 1:
            extras['latency_per_linearization'] = latency_record(args.config, dev, n=200)
            t0 = lap('latency', t0)
            extras['ms_per_lm_iteration'] = lm_iterations(args.config, 3, 3, dev, n_tracks=args.tracks)
        else:
            extras['ms_per_lm_iteration'] = sharded_lm_iteration(args, dev, world, rank)
        t0 = lap('lm_iterations', t0)
    wl.release()
    del wl
    if not args.no_configs4:
        wl4 = Workload(4, args.configs4_tracks, world, rank, dev, obs_local=world > 1)
        r4 = measure_workload(wl4, args.configs4_steps, 3, peak, peak_kind, want_clocks=False, e2e_steps=4)
        t0 = lap('configs4', t0)
        r4['note'] = ('the depth-stitch phase of configs[4] (scripts/xps/co3d_offline.sh:38 second phase): focal '
                      'and poses fixed, only depth-coefficient blocks in S; measured like the headline step')
        extras['configs4'] = r4
        wl4.release()
        del wl4
    if world == 1 and not args.no_extras:
        extras['configs3_latency'] = latency_record(3, dev, n=1000, online_planning=True)
        t0 = lap('configs3', t0)
        extras['configs1_lm_iterations'] = lm_iterations(1, 10, 2, dev)
        t0 = lap('configs1', t0)
        if not args.no_reference_gpu:
            extras['reference_gpu'] = reference_gpu_record(dev)
            extras['reference_gpu']['headline_workload'] = REFERENCE_GPU_UNAVAILABLE
            t0 = lap('reference_gpu', t0)

    if rank == 0:
        line = {'metric': METRIC, 'value': head['value'], 'unit': UNIT, 'n_gpus': world, 'steps': args.steps,
                'warmup': args.warmup, 'ms_per_step': head['ms_per_step'], 'higher_is_better': True,
                'scaling': 'strong', 'vs_baseline': None, 'dtype': 'f32',
                'data': 'synthetic (seeded generator of the configuration)',
                'config': dict(head['config'], workload=head['config']['workload'] +
                               (f' with {args.tracks} tracks' if args.tracks else '')),
                'roofline': head['roofline'], 'clocks': head.get('clocks'), 'e2e': head.get('e2e'),
                'gpu_launches': 7 * args.steps,   # prep, points, factor, diag, pairs, fin_max, fin_apply
                'setup_s': head['setup_s']}
        if 'parity' in head:
            line['parity'] = head['parity']
        line.update(extras)
        if world == 1 and not args.no_cpu_baseline:
            line['cpu_baseline'] = cpu_baseline(args.config, args.cpu_sample_tracks)
            t0 = lap('cpu_baseline', t0)
        wall['total'] = round(time.perf_counter() - t_run, 1)
        line['wall_s'] = wall
        sys.stdout.flush()
        os.write(json_fd, (json.dumps(line) + '\n').encode())
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def sharded_lm_iteration(args, dev, world, rank):
    """The sharded LM step on configs[2] (global inputs on every rank): sharded linearization,
    PCG on rank 0, delta_c broadcast, local back-substitution, delta_p gathered, line search on
    every rank; 3 timed after 3 untimed, max over ranks."""
    import torch
    import torch.distributed as dist
    from blast3r_b200.distributed import ShardedSchur, shard_tracks_by_image, sharded_lm_step
    from blast3r_b200.plan import BAPlan
    sc = cached_scene(args.config, n_tracks=args.tracks)
    o = sc.options
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in sc.lm_inputs().items()}
    owner, _ = shard_tracks_by_image(sc.infos, sc.pids, sc.n_tracks, world)
    plan = BAPlan(sc.infos, sc.pids, sc.n_cams, sc.n_nodes, sc.n_tracks, sc.n_zcf, optim_K=o['optim_K'],
                  optim_P=o['optim_P'], track_owner=owner, rank=rank, device=dev)
    sh = ShardedSchur(plan)
    last = {}

    def lm():
        _, st = sharded_lm_step(sh, t['rigs'], t['pids'], t['pix2d'], t['pix2d_std'], t['pix2d_dep'], t['K'],
                                t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'], pnorm=o['pnorm'],
                                clip_pix_err=o['clip_pix_err'], huber_delta=o['huber_delta'],
                                weight_z=o['weight_z'], dtype=torch.float64)
        last['st'] = st
    ms = timed(lm, 3, 3, world, dev) / 3
    out = {'ms': ms, 'loss': [float(last['st'].init_loss), float(last['st'].new_loss)],
           'what': 'distributed.sharded_lm_step: residual op, track-sharded linearization with the NCCL reduce, '
                   'PCG on S on rank 0, delta_c broadcast, local back-substitution, delta_p all-gather, line '
                   'search (max over ranks)'}
    del sh, plan, t
    torch.cuda.empty_cache()
    return out


def main():
    args = parse_args()
    if args.internal == 'ref-gpu':
        internal_ref_gpu(args)
    elif args.internal == 'ref-cpu':
        internal_ref_cpu(args)
    elif args.impl == 'reference':
        run_reference(args)
    else:
        run_b200(args)


if __name__ == '__main__':
    main()
