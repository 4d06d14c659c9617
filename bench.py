#!/usr/bin/env python
"""Benchmark of the BA linearization + Schur assembly hot path (one JSON line on rank 0).

A step is one linearization of the whole problem: residual, Jacobians, IRLS weights,
per-track 3x3 point elimination and assembly of the Schur-reduced camera/depth system S
and its gradient b (plus, on several GPUs, the all-reduce of the point-damping maximum and
the NCCL reduce of the partial S, b and diag(A) to rank 0, which then damps S).

Workload: configs[2] of the benchmark (1,000 cameras, 1M tracks, ~5.8M observations,
mono focal, K=4 depth channels), seeded synthetic data; tracks are sharded by id across
ranks (strong scaling: the total problem is fixed).  The observation arrays (~260 MB) are
larger than the 126 MB L2, so no explicit flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--config 2]
"""
import argparse
import datetime
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


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=20)
    ap.add_argument('--warmup', type=int, default=5)
    ap.add_argument('--impl', default='b200', choices=['b200', 'reference'])
    ap.add_argument('--config', type=int, default=2)
    ap.add_argument('--tracks', type=int, default=None,
                    help='override the configuration\'s track count (same generator; smaller profiling cases)')
    ap.add_argument('--cpu-sample-tracks', type=int, default=20000,
                    help='tracks in the bounded CPU-baseline sample (same generator)')
    ap.add_argument('--ref-step-tracks', type=int, default=4000,
                    help='tracks per step of the reference (CPU) arm')
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--e2e-steps', type=int, default=8)
    return ap.parse_args()


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


def algorithmic_bytes(n_obs, n_tracks, plan_info, block_size):
    """Compulsory bytes of one linearization (fp32): per observation pix2d 8 + std 8 +
    depth channels 4C + image id 4 + residual write 12 = 52 B (C = 5); per track point 12
    + track offset 4 = 16 B; S (upper-triangle scalars) and b written once."""
    bs = np.asarray(block_size, np.int64)
    nnz_upper = int(plan_info.nnz) - int((bs * (bs - 1) // 2).sum())
    return 52 * n_obs + 16 * n_tracks + 4 * (nnz_upper + int(plan_info.n_cam_params)), nnz_upper


def fp32_flops(L):
    """Useful fp32 FLOPs of one linearization with w = 13 camera-side columns:
    per observation ~300 + 3w(w+1) + 36w + 36, per observation pair 6 w^2."""
    w = 13
    L = np.asarray(L, np.int64)
    return float((L * (300 + 3 * w * (w + 1) + 36 * w + 36) + L * (L - 1) // 2 * 6 * w * w).sum())


def cpu_baseline(cfg, n_tracks, scene_kw=None):
    """Oracle port on a bounded sample of the same generator (single process)."""
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
    """One worker of the CPU reference arm: the oracle linearization of one track shard."""
    from oracle import ba_oracle as O
    d, opts = job
    s = O.linearize(d, opts, dtype=np.float64, dense=False, residual_dtype=np.float32)
    lay = s['layout']
    types = ((0, 2, lay.nK), (lay.off_P, 6, lay.nP), (lay.off_Z, lay.C, lay.nZ))
    return s['S'], s['b'], s['diagA'], s['lam'], types


def run_reference(args):
    """The reference's CPU path (the oracle restatement, numpy float64 with a sparse S) on
    every host core: each process linearizes the observations of one track range (tracks
    shard exactly: S, b and diag(A) are sums over tracks), the parent sums the partial
    systems and applies the per-type damping once.  Shipping the shards to the workers and
    the reduction are inside the timed region."""
    import multiprocessing as mp
    from scipy import sparse
    world, rank, _ = dist_env()
    if rank != 0:
        return
    from blast3r_b200.synthetic import make_scene
    n_workers = max(1, min(os.cpu_count() or 1, 64))
    for k in ('OMP_NUM_THREADS', 'MKL_NUM_THREADS', 'OPENBLAS_NUM_THREADS'):
        os.environ[k] = '1'                    # one thread per worker process
    tracks = min(args.ref_step_tracks * n_workers, 400000)
    times, nobs = [], []
    sc = make_scene(args.config, n_tracks=tracks, seed=1000)
    d = dict(sc.lm_inputs())
    d['infos'] = d.pop('rigs')
    bounds = np.linspace(0, sc.n_tracks, n_workers + 1).astype(int)
    jobs = [(_ref_shard(d, bounds[w], bounds[w + 1]), sc.options) for w in range(n_workers)]
    with mp.get_context('spawn').Pool(n_workers) as pool:
        pool.map(_ref_worker, [])              # start the workers before timing
        for step in range(args.warmup + args.steps):
            t = time.perf_counter()
            parts = pool.map(_ref_worker, jobs)
            # sum the undamped partial systems, then damp once from the summed diag(A)
            lam_parts = sum(pt[3] for pt in parts)
            S = sum(pt[0] for pt in parts) - sparse.diags(lam_parts)
            bvec = sum(pt[1] for pt in parts)
            dA = sum(pt[2] for pt in parts) - lam_parts
            lam = np.zeros_like(dA)
            for lo, sz, nblk in parts[0][4]:
                sl = slice(lo, lo + sz * nblk)
                if sz * nblk:
                    lam[sl] = 1e-12 * np.abs(dA[sl]).max()
            S = (S + sparse.diags(lam)).tocsr()
            if step >= args.warmup:
                times.append(time.perf_counter() - t)
                nobs.append(sc.n_obs)
    value = float(np.sum(nobs) / np.sum(times))
    sample = (f'configs[{args.config}] generator, {tracks} tracks (~{int(np.mean(nobs))} observations) per step, '
              f'oracle port (numpy float64, sparse S) in {n_workers} processes by track range, '
              f'partial systems summed')
    print(json.dumps({'impl': 'reference', 'metric': METRIC, 'value': value, 'unit': UNIT, 'n_gpus': args.gpus,
                      'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': 1e3 * float(np.mean(times)),
                      'higher_is_better': True, 'scaling': 'strong', 'vs_baseline': None, 'dtype': 'f64',
                      'data': 'synthetic', 'config': {'workload': f'configs[{args.config}] (bounded CPU sample)'},
                      'cpu_baseline': {'value': value, 'unit': UNIT, 'cores': n_workers, 'kind': 'port',
                                       'sample': sample},
                      'e2e': {'value': value, 'unit': UNIT, 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}))


def run_b200(args):
    import torch
    import torch.distributed as dist
    from blast3r_b200 import _lib as L
    from blast3r_b200.distributed import ShardedSchur, shard_tracks
    from blast3r_b200.plan import BAPlan
    from blast3r_b200.synthetic import make_scene

    world, rank, local = dist_env()
    # Libraries (NCCL) may print to the process's stdout; keep stdout for the one JSON line.
    json_fd = os.dup(1)
    os.dup2(2, 1)
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    if world > 1:
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=300), device_id=dev)
    sc = make_scene(args.config, n_tracks=args.tracks)
    t0, t1, n_local = shard_tracks(sc.pids, sc.n_tracks, world, rank)
    o = sc.options
    plan = BAPlan(sc.infos, sc.pids, sc.n_cams, sc.n_nodes, sc.n_tracks, sc.n_zcf, optim_K=o['optim_K'],
                  optim_P=o['optim_P'], optim_Z=o['optim_Z'], optim_X=o['optim_X'], track_range=(t0, t1), device=dev)
    host = {k: np.ascontiguousarray(v) for k, v in sc.lm_inputs().items()}
    t = {k: torch.from_numpy(v).to(dev) for k, v in host.items()}
    p = plan.params(t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'], t['pix2d_std'], t['pix2d_dep'],
                    pix2d=t['pix2d'])
    lo = BAPlan.lin_opts(weight_z=o['weight_z'], pnorm=o['pnorm'], max_pix_err=o['clip_pix_err'],
                         huber_delta=o['huber_delta'])
    ncp, nnz = plan.n_cam_params, int(plan.info.nnz)
    sharded = ShardedSchur(plan)
    S, b, dA, pc, hm = outs = sharded.outputs

    def step():
        sharded.linearize(p, lo)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms_total = float(ms.item())
    ms_step = ms_total / args.steps
    value = sc.n_obs * args.steps / (ms_total * 1e-3)
    clocks = clk.summary()

    # per-pass device time on this rank (same workload, events between the launches)
    names = ['prep', 'points', 'factor', 'diag', 'pairs', 'finalize']
    acc = {k: 0.0 for k in names}
    R = 5
    s = torch.cuda.current_stream().cuda_stream
    for _ in range(R):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(names) + 1)]
        S.zero_(); b.zero_(); dA.zero_(); hm.zero_()
        ev[0].record()
        for j, nm in enumerate(names):
            if nm == 'finalize':
                plan.lin_stage('finalize', p, lo, outs)
            else:
                pas = dict(prep=L.PASS_PREP, points=L.PASS_POINTS, factor=L.PASS_FACTOR, diag=L.PASS_DIAG,
                           pairs=L.PASS_PAIRS)[nm]
                plan.lin_pass(pas, p, lo, outs)
            ev[j + 1].record()
        torch.cuda.synchronize()
        for j, nm in enumerate(names):
            acc[nm] += ev[j].elapsed_time(ev[j + 1]) / R
    tot = sum(acc.values())
    passes = {k: {'ms': round(v, 4), 'share': round(v / tot, 4)} for k, v in acc.items()}

    # latency of one relinearization as an online caller sees it (host call to result on the
    # device, synchronised): direct calls and CUDA-graph replays (BAPlan.capture)
    latency = None
    if world == 1:
        def pct(v):
            v = np.sort(np.asarray(v))
            return {'p50': round(float(np.percentile(v, 50)), 4), 'p99': round(float(np.percentile(v, 99)), 4)}
        n_lat = 20
        lat_d = []
        for _ in range(n_lat + 3):
            torch.cuda.synchronize()
            t0_ = time.perf_counter()
            step()
            torch.cuda.synchronize()
            lat_d.append(1e3 * (time.perf_counter() - t0_))
        graph, _ = plan.capture(p, lo, outs)
        lat_g = []
        for _ in range(n_lat + 3):
            torch.cuda.synchronize()
            t0_ = time.perf_counter()
            graph.replay()
            torch.cuda.synchronize()
            lat_g.append(1e3 * (time.perf_counter() - t0_))
        latency = {'unit': 'ms', 'n': n_lat, 'direct': pct(lat_d[3:]), 'cuda_graph': pct(lat_g[3:])}
        del graph

    # end to end through the public API with host buffers
    pin = {k: torch.from_numpy(v).pin_memory() for k, v in host.items()}
    S_h = torch.empty(nnz, dtype=torch.float32).pin_memory()
    b_h = torch.empty(ncp, dtype=torch.float32).pin_memory()
    h2d = sum(v.numel() * v.element_size() for v in pin.values())
    d2h = (S_h.numel() + b_h.numel()) * 4

    # Two device input sets: step k+1's host->device copies run on a copy stream while step
    # k computes (the plan re-stages the observations of the set it is given each step).
    # Every step's copies and its S, b read-back are inside the timed region.
    sets = [t, {k: torch.empty_like(v) for k, v in t.items()}]
    psets = [plan.params(s_['K'], s_['P_rig2cam'], s_['P_w2rig'], s_['z_coefs'], s_['pts3d'], s_['pix2d_std'],
                         s_['pix2d_dep'], pix2d=s_['pix2d']) for s_ in sets]
    cs = torch.cuda.Stream(device=dev)
    copied = [torch.cuda.Event(), torch.cuda.Event()]
    freed = [torch.cuda.Event(), torch.cuda.Event()]

    def issue_copy(k):
        with torch.cuda.stream(cs):
            if k >= 2:
                cs.wait_event(freed[k % 2])          # step k-2 is done with this set
            for key in pin:
                sets[k % 2][key].copy_(pin[key], non_blocking=True)
            copied[k % 2].record(cs)

    def compute(k):
        cur = torch.cuda.current_stream()
        cur.wait_event(copied[k % 2])
        s_ = sets[k % 2]
        plan.stage_obs(s_['pix2d'], s_['pix2d_std'], s_['pix2d_dep'])
        sharded.linearize(psets[k % 2], lo)
        freed[k % 2].record(cur)
        if rank == 0:
            S_h.copy_(S, non_blocking=True)
            b_h.copy_(b, non_blocking=True)

    def e2e_run(n):
        cs.wait_stream(torch.cuda.current_stream())   # copies start after the timing event
        issue_copy(0)
        for k in range(n):
            if k + 1 < n:
                issue_copy(k + 1)
            compute(k)

    e2e_run(2)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0.record()
    e2e_run(args.e2e_steps)
    e1.record()
    torch.cuda.synchronize()
    ms_e = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ms_e, op=dist.ReduceOp.MAX)
    e2e_value = sc.n_obs * args.e2e_steps / (float(ms_e.item()) * 1e-3)

    # one full LM iteration through the public driver (N=1): residuals, fused linearization,
    # PCG on S, back-substitution and the line search of engine.lm_step
    lm_info = None
    if world == 1:
        from blast3r_b200.engine import lm_step
        from blast3r_b200 import ba_solver as BS
        last = {}

        def lm():
            _, st = lm_step(t['rigs'], t['pids'], t['pix2d'], t['pix2d_std'], t['pix2d_dep'], t['K'], t['P_rig2cam'],
                            t['P_w2rig'], t['z_coefs'], t['pts3d'], pnorm=o['pnorm'], clip_pix_err=o['clip_pix_err'],
                            huber_delta=o['huber_delta'], weight_z=o['weight_z'], optim_K=o['optim_K'],
                            optim_P=o['optim_P'], dtype=torch.float64)
            last['st'] = st
        for _ in range(3):                     # plans the structure once (cached per phase), then
            lm()                               # warms the allocator's pools for the step's buffers
        torch.cuda.synchronize()
        n_lm = 3
        t_lm = time.perf_counter()
        e0.record()
        for _ in range(n_lm):
            lm()
        e1.record()
        torch.cuda.synchronize()
        lm_info = {'ms': e0.elapsed_time(e1) / n_lm, 'wall_ms': 1e3 * (time.perf_counter() - t_lm) / n_lm,
                   'loss': [float(last['st'].init_loss), float(last['st'].new_loss)],
                   'what': 'engine.lm_step: residual op, fused linearization, PCG on S (tol 1e-6, <=300 it), '
                           'back-substitution, line search'}
    else:
        # the sharded step: sharded linearization, PCG on the root, delta_c broadcast, local
        # back-substitution, delta_p all-reduced, the line search on every rank
        from blast3r_b200.distributed import sharded_lm_step
        last = {}

        def lm():
            _, st = sharded_lm_step(sharded, t['rigs'], t['pids'], t['pix2d'], t['pix2d_std'], t['pix2d_dep'], t['K'],
                                    t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'], pnorm=o['pnorm'],
                                    clip_pix_err=o['clip_pix_err'], huber_delta=o['huber_delta'],
                                    weight_z=o['weight_z'], dtype=torch.float64)
            last['st'] = st
        plan.stage_obs(t['pix2d'], t['pix2d_std'], t['pix2d_dep'])
        for _ in range(3):
            lm()
        torch.cuda.synchronize()
        dist.barrier()
        n_lm = 3
        e0.record()
        for _ in range(n_lm):
            lm()
        e1.record()
        torch.cuda.synchronize()
        ms_lm = torch.tensor([e0.elapsed_time(e1) / n_lm], dtype=torch.float64, device=dev)
        dist.all_reduce(ms_lm, op=dist.ReduceOp.MAX)
        lm_info = {'ms': float(ms_lm.item()), 'loss': [float(last['st'].init_loss), float(last['st'].new_loss)],
                   'what': 'distributed.sharded_lm_step: residual op, track-sharded linearization with the NCCL '
                           'reduce, PCG on S on rank 0, delta_c broadcast, local back-substitution, delta_p '
                           'all-reduce, line search (max over ranks)'}

    if rank == 0:
        peak, peak_kind = measured_peaks()
        L_t = np.bincount(sc.pids, minlength=sc.n_tracks)[t0:t1]
        B, nnz_upper = algorithmic_bytes(n_local, t1 - t0, plan.info, plan.block_size)
        achieved = B / (ms_step * 1e-3) / 1e9
        flops = fp32_flops(L_t)
        sm_mhz = clocks['sm_mhz'] or 1965.0
        fp32_peak = 148 * 128 * 2 * sm_mhz * 1e6 / 1e12
        # dominant kernel: the pairs pass (segment-major pair products).  Its compulsory
        # bytes are every elimination record read once, the pair list, and the S values it
        # adds to; its time is the live CUDA-event time of the pass on the launch stream.
        R = int(plan.info.record_floats)
        pairs_B = 4 * R * int(plan.info.n_obs_local) + 8 * int(plan.info.n_pairs) + 4 * nnz_upper
        pairs_ms = passes['pairs']['ms']
        pairs_ach = pairs_B / (pairs_ms * 1e-3) / 1e9
        pairs_flops = 6.0 * 13 * 13 * int(plan.info.n_pairs)      # dense-equivalent Y_o^T Y_o' (w = 13)
        roof = {'bound': 'hbm', 'kernel': f"k_pairs (pairs pass, {passes['pairs']['share']:.2f} of the step)",
                'achieved': round(pairs_ach, 2), 'peak': peak, 'unit': 'GB/s', 'frac': round(pairs_ach / peak, 4),
                'traffic': read_traffic(args.config, world, 'pairs_dram_bytes_per_launch'),
                'algorithmic_bytes_per_launch': int(pairs_B), 'launch_ms': pairs_ms, 'peak_kind': f'of {peak_kind}',
                'fp32': {'flops_per_launch': pairs_flops,
                         'achieved_tflops': round(pairs_flops / (pairs_ms * 1e-3) / 1e12, 2),
                         'peak_tflops_at_median_clock': round(fp32_peak, 1),
                         'frac': round(pairs_flops / (pairs_ms * 1e-3) / 1e12 / fp32_peak, 4)},
                # the whole linearization step against HBM (bytes per observation x observations)
                'step': {'achieved': round(achieved, 2), 'frac': round(achieved / peak, 4),
                         'algorithmic_bytes': int(B),
                         'traffic': read_traffic(args.config, world, 'dram_bytes_per_step'),
                         'fp32_flops': flops, 'fp32_frac': round(flops / (ms_step * 1e-3) / 1e12 / fp32_peak, 4)},
                'passes': passes}
        line = {'metric': METRIC, 'value': value, 'unit': UNIT, 'n_gpus': world, 'steps': args.steps,
                'warmup': args.warmup, 'ms_per_step': ms_step, 'higher_is_better': True, 'scaling': 'strong',
                'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic (seeded generator of the configuration)',
                'config': {'workload': f'configs[{args.config}]' + (f' with {args.tracks} tracks' if args.tracks else ''), 'n_obs': sc.n_obs, 'n_tracks': sc.n_tracks,
                           'n_imgs': sc.n_imgs, 'mean_track_length': sc.meta['mean_track_length'],
                           'n_obs_pairs': int(plan.info.n_pairs), 'nnz_S': nnz,
                           'parallelism': f'track-sharded x{world}' + (' + NCCL reduce of S, b' if world > 1 else ''),
                           'l2': 'inputs larger than L2 (observation arrays ~260 MB), no flush'},
                'roofline': roof, 'clocks': clocks,
                'e2e': {'value': e2e_value, 'unit': UNIT, 'h2d_bytes_per_step': int(h2d), 'd2h_bytes_per_step': int(d2h)},
                'gpu_launches': 7 * args.steps}   # prep, points, factor, diag, pairs, fin_max, fin_apply (rank 0)
        if lm_info is not None:
            line['ms_per_lm_iteration'] = lm_info
        if latency is not None:
            line['latency_per_linearization'] = latency
        if world == 1 and not args.no_cpu_baseline:
            line['cpu_baseline'] = cpu_baseline(args.config, args.cpu_sample_tracks)
        sys.stdout.flush()
        os.write(json_fd, (json.dumps(line) + '\n').encode())
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def read_traffic(cfg, world, key):
    """DRAM bytes (`key`) from the committed ncu summary profiles/traffic_cfg<cfg>.txt, or None."""
    path = os.path.join(ROOT, 'profiles', f'traffic_cfg{cfg}.txt')   # measured DRAM bytes
    if world != 1 or not os.path.isfile(path):
        return None
    with open(path) as f:
        for line in f:
            if line.startswith(key + ':'):
                return float(line.split(':', 1)[1])
    return None


def main():
    args = parse_args()
    if args.impl == 'reference':
        run_reference(args)
    else:
        run_b200(args)


if __name__ == '__main__':
    main()
