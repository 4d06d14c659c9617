"""CUDA-graph replay of a linearization (BAPlan.capture) against direct calls: the same S and
b, and a replay after the parameters change in place linearizes at the new values."""
import numpy as np
import pytest
import torch

from blast3r_b200.plan import BAPlan
from blast3r_b200.synthetic import make_scene
from tests.helpers import rel_err

pytestmark = pytest.mark.gpu


def test_graph_replay_matches_direct_linearization():
    sc = make_scene(3)
    o = sc.options
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in sc.lm_inputs().items()}
    plan = BAPlan(t['rigs'], t['pids'], sc.n_cams, sc.n_nodes, sc.n_tracks, sc.n_zcf, optim_K=o['optim_K'],
                  optim_P=o['optim_P'], device=torch.device('cuda', 0))
    p = plan.params(t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'], t['pix2d_std'], t['pix2d_dep'],
                    pix2d=t['pix2d'])
    lo = BAPlan.lin_opts(weight_z=o['weight_z'], pnorm=o['pnorm'], max_pix_err=o['clip_pix_err'],
                         huber_delta=o['huber_delta'])
    graph, s_g = plan.capture(p, lo)
    for step in range(2):
        if step:
            t['pts3d'].add_(0.01 * torch.randn_like(t['pts3d']))      # new parameters, same buffers
        graph.replay()
        torch.cuda.synchronize()
        S_g, b_g = s_g.S_vals.clone(), s_g.b.clone()
        s_d = plan.linearize(p, lo)
        torch.cuda.synchronize()
        assert rel_err(S_g.cpu().numpy(), s_d.S_vals.cpu().numpy()) < 1e-4
        assert rel_err(b_g.cpu().numpy(), s_d.b.cpu().numpy()) < 1e-4
