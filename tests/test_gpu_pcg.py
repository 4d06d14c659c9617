"""The native PCG (b3r_pcg / b3r_pcg_f64, one cooperative kernel) against the step-by-step
PCG of ``tests/pcg_stepwise.py`` (the reference's iteration and stopping rule,
inference/ba_solver.py:1197-1238) on the same assembled S, b and preconditioner."""
import numpy as np
import pytest
import torch

from tests.pcg_stepwise import pcg as pcg_steps
from blast3r_b200.synthetic import make_scene
from tests.helpers import golden_files, load_golden, rel_err, scene_inputs
from tests.test_gpu_schur import run_plan

pytestmark = pytest.mark.gpu

# the resident kernel (rows of S in shared memory, where the plan's row groups fit, which they
# do for every case here) and the streaming kernel (rows of S read from L2)
KERNELS = pytest.mark.parametrize('kernel', ['resident', 'streaming'])


def _flags(kernel):
    from blast3r_b200 import _lib as L
    return {'resident': 0, 'streaming': L.PCG_STREAMING, 'global-tiles': L.PCG_TEST_GLOBAL_TILES}[kernel]


def _both(s, dtype, maxiter=300, kernel='resident'):
    b = s.b.to(dtype)
    M = s.precond.to(dtype)
    if kernel != 'streaming':
        assert s.plan.info.pcg_resident == 1
    x_n, it_n, conv_n = s.plan.pcg(s.S_vals, s.precond, b, tol=1e-6, maxiter=maxiter, flags=_flags(kernel))
    x_s, it_s, conv_s = pcg_steps(lambda v: s.matvec(v), b, M_mv=lambda v: v / M, tol=1e-6, maxiter=maxiter)
    return (x_n.double().cpu().numpy(), it_n, conv_n), (x_s.double().cpu().numpy(), it_s, conv_s)


def _check_close(s, xn, xs, itn, its, cn, cs, dist):
    """Same stopping decision and about the same iteration (the native kernel runs the
    pipelined form of the iteration, whose rounding differs), the native iterate's true
    residual within the stopping tolerance (or, unconverged, close to the stepwise one), and
    iterates within `dist`: two PCG runs that differ only in rounding drift apart by up to
    cond(S) times their residuals.  Unconverged iterates are compared in the S-norm (the
    error measure CG minimises): along the poorly determined directions of an ill-conditioned
    S the two runs' best-so-far iterates may differ more, without a difference in the step's
    quality."""
    assert cn == cs and abs(itn - its) <= max(2, 0.1 * its), (itn, its, cn, cs)
    b = s.b.double()
    xn_d, xs_d = torch.from_numpy(xn).cuda(), torch.from_numpy(xs).cuda()
    rn = float((s.matvec(xn_d) - b).norm() / b.norm())
    rs = float((s.matvec(xs_d) - b).norm() / b.norm())
    if cn:      # the stopping guarantee; where below it each run lands is arbitrary
        assert rn <= 1.05e-6, (rn, rs)
        assert rel_err(xn, xs) < dist
    else:       # best-so-far iterates after maxiter
        assert rn <= 1.5 * rs + 1e-7, (rn, rs)
        e = xn_d - xs_d
        assert float(torch.dot(e, s.matvec(e)).sqrt() / torch.dot(xs_d, s.matvec(xs_d)).sqrt()) < dist


@KERNELS
@pytest.mark.parametrize('path', golden_files(), ids=lambda p: p.split('golden_')[-1][:-4])
def test_native_pcg_equals_stepwise_f64(path, kernel):
    inp, opts, _ = load_golden(path)
    _, s = run_plan(inp, opts)
    (xn, itn, cn), (xs, its, cs) = _both(s, torch.float64, kernel=kernel)
    _check_close(s, xn, xs, itn, its, cn, cs, 1e-4)


@KERNELS
@pytest.mark.parametrize('path', golden_files(), ids=lambda p: p.split('golden_')[-1][:-4])
def test_native_pcg_equals_stepwise_f32(path, kernel):
    inp, opts, _ = load_golden(path)
    _, s = run_plan(inp, opts)
    (xn, itn, cn), (xs, its, cs) = _both(s, torch.float32, kernel=kernel)
    # the native kernel iterates in double for float32 vectors too: it converges whenever the
    # float32 step-by-step iteration does (and may where float32 stalls)
    assert cn or not cs
    # float32 iterates drift with the rounding order: compare true (float64) residuals, and
    # the distance to the float64 solution loosely
    b = s.b.double()
    rn = float((s.matvec(torch.from_numpy(xn).cuda()) - b).norm() / b.norm())
    rs = float((s.matvec(torch.from_numpy(xs).cuda()) - b).norm() / b.norm())
    assert rn <= 3.0 * rs + 1e-6, (rn, rs)
    ref = _both(s, torch.float64)[1][0]
    assert rel_err(xn, ref) < 1e-3


@pytest.mark.parametrize('kernel', ['resident', 'streaming', 'global-tiles'])
@pytest.mark.parametrize('cfg,ni,nt', [(1, 60, 6000), (3, None, None), (2, None, 100_000)])
def test_native_pcg_synthetic(cfg, ni, nt, kernel):
    """configs[3] (per-frame focals) is poorly conditioned: it does not reach 1e-6 in 300
    iterations and returns the best-so-far iterate.  The configs[2] case (1000 images, a mono
    camera whose focal row couples to every block) splits that row over helper blocks."""
    sc = make_scene(cfg, n_imgs=ni, n_tracks=nt)
    _, s = run_plan(scene_inputs(sc), dict(sc.options))
    (xn, itn, cn), (xs, its, cs) = _both(s, torch.float64, kernel=kernel)
    _check_close(s, xn, xs, itn, its, cn, cs, 1e-3)


@KERNELS
def test_native_pcg_best_so_far_when_not_converged(kernel):
    inp, opts, _ = load_golden(golden_files()[0])
    _, s = run_plan(inp, opts)
    (xn, itn, cn), (xs, its, cs) = _both(s, torch.float64, maxiter=3, kernel=kernel)
    assert not cn and not cs and itn == its
    assert rel_err(xn, xs) < 1e-9


def test_resident_and_streaming_kernels_agree():
    """The two kernels run the same iteration on the same row groups; only the order of the
    within-warp row sums differs."""
    sc = make_scene(1, n_imgs=60, n_tracks=6000)
    _, s = run_plan(scene_inputs(sc), dict(sc.options))
    b = s.b.double()
    x1, it1, c1 = s.plan.pcg(s.S_vals, s.precond, b, maxiter=40)
    x2, it2, c2 = s.plan.pcg(s.S_vals, s.precond, b, maxiter=40, flags=_flags('streaming'))
    assert c1 == c2 and abs(it1 - it2) <= 1
    assert rel_err(x1.cpu().numpy(), x2.cpu().numpy()) < 1e-6


@KERNELS
def test_pcg_barrier_wait_that_runs_out_returns_an_error(kernel):
    """The failure path of the kernel's grid barrier, without a fault: with a short wait limit
    and the test flag that makes the first barrier wait for an arrival no block makes, every
    block leaves, x is zeroed and result[2] reports it; the context stays usable and the next
    solve is normal."""
    from blast3r_b200 import _lib as L
    inp, opts, _ = load_golden(golden_files()[0])
    _, s = run_plan(inp, opts)
    b = s.b.double()
    f = _flags(kernel)
    x, it, conv, err = s.plan.pcg(s.S_vals, s.precond, b, barrier_spin_limit=2000,
                                  flags=L.PCG_TEST_UNREACHABLE_BARRIER | f, raw=True)
    torch.cuda.synchronize()
    assert err == 1 and not conv and float(x.abs().max()) == 0.0
    x2, it2, conv2 = s.plan.pcg(s.S_vals, s.precond, b, flags=f)
    x3, it3, conv3 = s.plan.pcg(s.S_vals, s.precond, b, barrier_spin_limit=1 << 20, flags=f)
    assert conv2 and conv3 and it2 == it3 and torch.equal(x2, x3)   # deterministic reductions
