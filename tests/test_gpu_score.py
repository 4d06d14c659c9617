"""The line search's reprojection score on the device (b3r_reproj_score, an exact radix
select) against the reference's sort-based formula (engine.py:357-361)."""
import math

import numpy as np
import pytest
import torch

from blast3r_b200 import cujac
from blast3r_b200.engine import reproj_score
from blast3r_b200.synthetic import make_scene
from tests.helpers import scene_inputs, to_cuda

pytestmark = pytest.mark.gpu


def sort_score(res):
    e = res[:, :2].double().norm(dim=-1).sort().values
    n80 = len(e) * 80 // 100
    return float(e[:n80].mean())


@pytest.mark.parametrize('n,kind', [(1, 'gauss'), (2, 'gauss'), (5, 'gauss'), (1000, 'gauss'), (1000, 'ties'),
                                    (1000, 'zeros'), (1 << 20, 'gauss'), (1 << 20, 'ties'), (300001, 'wide'),
                                    (1000, 'fewnan'), (1000, 'mostnan')])
def test_score_matches_sort(n, kind):
    g = torch.Generator(device='cpu').manual_seed(n)
    if kind == 'gauss':
        r = torch.randn(n, 9, generator=g)
    elif kind == 'ties':           # a handful of distinct errors: the k-th value is tied many times
        r = torch.randint(0, 4, (n, 9), generator=g).float()
    elif kind == 'zeros':
        r = torch.zeros(n, 9)
    elif kind == 'wide':           # errors spread over many decades
        r = torch.randn(n, 9, generator=g) * torch.exp(8 * torch.randn(n, 1, generator=g))
    else:                          # NaN errors sort last: a few leave a finite score, many a NaN one
        r = torch.randn(n, 9, generator=g)
        r[torch.rand(n, generator=g) < (0.05 if kind == 'fewnan' else 0.5), 0] = float('nan')
    r = r.cuda()
    view = r.view(-1, 3, 3).unbind(dim=1)[0]           # the residual columns, row stride 9
    got = float(reproj_score(view))
    want = sort_score(view)
    if n * 80 // 100 == 0 or math.isnan(want):
        assert math.isnan(got) and math.isnan(want)
    else:
        assert abs(got - want) <= 1e-6 * max(abs(want), 1e-30), (got, want)


def test_score_on_the_residual_op_output():
    sc = make_scene(1, n_imgs=60, n_tracks=6000)
    inp, o = scene_inputs(sc), dict(sc.options)
    t = to_cuda(inp)
    res = cujac.residuals_with_rigs(t['infos'], t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'],
                                    t['pids'], t['pix2d'], t['pix2d_std'], t['pix2d_dep'], True, o['weight_z'],
                                    o['pnorm'], o['clip_pix_err'], o['huber_delta'])
    r = res.view(-1, 3, 3).unbind(dim=1)[0]
    got, want = float(reproj_score(r)), sort_score(r)
    assert abs(got - want) <= 1e-6 * abs(want), (got, want)
