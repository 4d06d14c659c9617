"""GPU parity of the reference-op mirrors (C ABI part 1) against the CPU oracle and
plain torch float64, through the C ABI."""
import numpy as np
import pytest
import torch

from blast3r_b200 import cujac
from blast3r_b200.synthetic import make_scene
from oracle import ba_oracle as O
from tests.helpers import TOL_OBS, golden_files, load_golden, rel_err, scene_inputs, to_cuda

pytestmark = pytest.mark.gpu

CASES = [('golden', p) for p in golden_files()] + [('scene', (0, None, None)), ('scene', (3, None, None)),
                                                     ('scene', (1, 40, 4000))]


def _inputs(case):
    kind, v = case
    if kind == 'golden':
        inp, opts, _ = load_golden(v)
        return inp, opts
    sc = make_scene(v[0], n_imgs=v[1], n_tracks=v[2])
    return scene_inputs(sc), dict(sc.options)


def _ids(c):
    return c[1].split('golden_')[-1][:-4] if c[0] == 'golden' else f'cfg{c[1][0]}'


@pytest.mark.parametrize('case', CASES, ids=_ids)
def test_residuals_with_rigs(case):
    inp, opts = _inputs(case)
    t = to_cuda(inp)
    is_log = opts.get('depth_mode', 'log') == 'log'
    args = (t['infos'], t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'], t['pids'], t['pix2d'],
            t['pix2d_std'], t['pix2d_dep'], is_log)
    out = cujac.residuals_with_rigs(*args, opts['weight_z'], opts['pnorm'], opts['clip_pix_err'],
                                    opts['huber_delta'])
    assert out.shape == (len(inp['pids']), 9) and out.stride() == (1, len(inp['pids']))
    ref = O.residuals_with_rigs(*(inp[k] for k in ('infos', 'K', 'P_rig2cam', 'P_w2rig', 'z_coefs', 'pts3d',
                                                   'pids', 'pix2d', 'pix2d_std', 'pix2d_dep')),
                                is_log, opts['weight_z'], opts['pnorm'], opts['clip_pix_err'], opts['huber_delta'])
    got = out.cpu().numpy()
    for j in range(3):
        assert rel_err(got[:, j], ref[:, j]) < TOL_OBS, j
    # Huber error and IRLS weight are exact functions of the residual: check them against
    # the reference formulas (sfm_jacobian_rigs.cu:240-258) applied to the GPU residuals,
    # so the check does not re-count the fp32 rounding of the residual itself.
    pn, hd, mx = opts['pnorm'], opts['huber_delta'], opts['clip_pix_err']
    a = 0.5 * pn * hd ** (pn - 2)
    bq = hd ** pn - a * hd * hd
    wz = np.array([1.0, 1.0, opts['weight_z']])
    rr = np.minimum(np.abs(got[:, :3].astype(np.float64)), mx)
    err = wz * np.where(rr <= hd, a * rr * rr, rr ** pn - bq)
    rw = np.maximum(rr, hd)
    w = np.where(rw == mx, 1e-16, wz * rw ** (pn - 2))
    valid = ref[:, 6:9].any(axis=1)
    assert rel_err(got[valid, 3:6], err[valid]) < 1e-6
    assert rel_err(got[valid, 6:9], w[valid]) < 1e-6
    assert not got[~valid].any()
    # pnorm = -1: residuals only
    r3 = cujac.residuals_with_rigs(*args)
    assert r3.shape == (len(inp['pids']), 3)
    assert rel_err(r3.cpu().numpy(), ref[:, :3]) < TOL_OBS


@pytest.mark.parametrize('float64', [False, True])
@pytest.mark.parametrize('case', CASES, ids=_ids)
def test_jacobians_with_rigs(case, float64):
    inp, opts = _inputs(case)
    t = to_cuda(inp)
    is_log = opts.get('depth_mode', 'log') == 'log'
    J = cujac.jacobians_with_rigs(t['infos'], t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'],
                                  t['pids'], t['pix2d_std'], t['pix2d_dep'], is_log, float64=float64)
    assert J[0].dtype == (torch.float64 if float64 else torch.float32)
    ref = O.jacobians_with_rigs(*(inp[k] for k in ('infos', 'K', 'P_rig2cam', 'P_w2rig', 'z_coefs', 'pts3d',
                                                   'pids', 'pix2d_std', 'pix2d_dep')), is_log)
    tol = 1e-9 if float64 else TOL_OBS
    for got, want in zip(J, ref):
        g = got.cpu().numpy()
        for r in range(want.shape[1]):
            for c in range(want.shape[2]):
                if np.abs(want[:, r, c]).max() > 0:
                    assert rel_err(g[:, r, c], want[:, r, c]) < max(tol, 2e-7 if r == 2 and c < 2 else tol)


def test_chol3x3_solve():
    g = torch.Generator().manual_seed(0)
    for dt in (torch.float32, torch.float64):
        A = torch.randn(1000, 3, 3, generator=g, dtype=torch.float64)
        A = A @ A.transpose(1, 2) + 0.5 * torch.eye(3, dtype=torch.float64)
        b = torch.randn(1000, 3, generator=g, dtype=torch.float64)
        x = cujac.chol3x3_solve(A.to(dt).cuda(), b.to(dt).cuda()).cpu().double()
        assert rel_err(x.numpy(), torch.linalg.solve(A, b).numpy()) < (1e-4 if dt == torch.float32 else 1e-10)


@pytest.mark.parametrize('bh,bw', [(3, 6), (6, 6), (2, 5), (17, 17), (3, 1)])
@pytest.mark.parametrize('transpose', [False, True])
def test_blockcoo_matvec(bh, bw, transpose):
    g = torch.Generator().manual_seed(bh * 31 + bw)
    HB, WB, N = 40, 30, 300
    blocks = torch.randn(N, bh, bw, generator=g, dtype=torch.float64)
    rows = torch.randint(0, HB, (N,), generator=g)
    cols = torch.randint(0, WB, (N,), generator=g)
    x = torch.randn((HB * bh) if transpose else (WB * bw), generator=g, dtype=torch.float64)
    D = torch.zeros(HB * bh, WB * bw, dtype=torch.float64)
    for n in range(N):
        D[rows[n] * bh:(rows[n] + 1) * bh, cols[n] * bw:(cols[n] + 1) * bw] += blocks[n]
    want = (D.T @ x) if transpose else (D @ x)
    for idt in (torch.int32, torch.int64):
        y = cujac.blockcoo_matvec(blocks.cuda(), rows.to(idt).cuda(), cols.to(idt).cuda(), x.cuda(), HB, WB,
                                  transpose)
        assert rel_err(y.cpu().numpy(), want.numpy()) < 1e-12


@pytest.mark.parametrize('K,I,J', [(3, 2, 6), (1, 5, 5), (3, 6, 6), (1, 17, 17), (3, 3, 9)])
def test_fused_einsum(K, I, J):
    g = torch.Generator().manual_seed(K * 100 + I * 10 + J)
    left = torch.randn(500, K, I + 2, generator=g, dtype=torch.float64)[:, :, 1:I + 1]   # strided batch view
    right = torch.randn(500, K, J, generator=g, dtype=torch.float64)
    got = cujac.fused_einsum_bki_bkj(left.cuda(), right.cuda()).cpu()
    assert rel_err(got.numpy(), torch.einsum('bki,bkj->bij', left, right).numpy()) < 1e-12


@pytest.mark.parametrize('cfg', [0, 3])
def test_residual_loss_equals_residual_op_mean(cfg):
    """b3r_residual_loss: the objective lm_step forms from the residual op (err.mean()) and
    the residuals the line search scores, in one pass."""
    from blast3r_b200.synthetic import make_scene
    sc = make_scene(cfg)
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in sc.lm_inputs().items()}
    o = sc.options
    args = (t['rigs'], t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'], t['pids'], t['pix2d'],
            t['pix2d_std'], t['pix2d_dep'], True, o['weight_z'], o['pnorm'], o['clip_pix_err'], o['huber_delta'])
    full = cujac.residuals_with_rigs(*args)
    res, err, _ = full.view(-1, 3, 3).unbind(dim=1)
    loss, r2 = cujac.residual_loss(*args)
    torch.cuda.synchronize()
    assert torch.equal(r2, res)
    assert abs(float(loss) - float(err.double().mean())) <= 1e-6 * abs(float(err.double().mean()))
