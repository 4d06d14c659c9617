"""Incremental planning for the online track merge (b3r_plan_append), host-only plans on the CPU.

The online loop merges the tracks of every new frame into the problem (``old | new``,
inference/tracks.py:96-117, inference/pipeline.py:196-224) and runs BA on the result.  A plan
appended to the previous frame's plan must describe the merged problem exactly like a plan built
from scratch: the same S pattern and value offsets, the same observation pairs, segments,
tasks and workspace.  Structures that do not extend the old plan (track removal, reordering, an
old track seen in the new image) are refused with B3R_E_INVALID, and the solver's plan cache then
plans from scratch.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from blast3r_b200 import _lib as L
from blast3r_b200 import ba_solver as BS
from blast3r_b200.plan import BAPlan
from blast3r_b200.synthetic import OnlineSequence, make_scene

INFO_FIELDS = ['n_obs', 'n_obs_local', 'n_tracks_local', 'n_blocks', 'n_cam_params', 'n_points', 'nnzb', 'nnz',
               'n_pairs', 'n_segments', 'n_pair_tasks', 'n_diag_chunks', 'workspace_bytes', 'nb_K', 'nb_P',
               'nb_Z', 'off_P', 'off_Z', 'record_floats', 'n_obs_input', 'depth_stitch', 'pcg_row_groups',
               'pcg_resident']


def _desc(s, keep, retain=1, masks=None):
    infos = np.ascontiguousarray(s.infos, np.int32)
    pids = np.ascontiguousarray(s.pids, np.int32)
    keep += [infos, pids]
    kw = {}
    for name, m in (masks or {}).items():
        m = np.ascontiguousarray(m, np.uint8)
        keep.append(m)
        kw['mode_' + name] = L.ENABLE_MASK
        kw['mask_' + name] = m.ctypes.data_as(C.POINTER(C.c_uint8))
    return L.PlanDesc(n_imgs=s.n_imgs, n_cams=s.n_cams, n_nodes=s.n_nodes, n_tracks=s.n_tracks, n_obs=s.n_obs,
                      C=s.n_zcf, infos=infos.ctypes.data_as(C.POINTER(C.c_int32)),
                      pids=pids.ctypes.data_as(C.POINTER(C.c_int32)), track_begin=0, track_end=s.n_tracks,
                      device=-1, retain=retain, **kw)


def _create(s, retain=1, masks=None):
    keep = []
    h = C.c_void_p()
    L.call('b3r_plan_create', C.byref(h), C.byref(_desc(s, keep, retain, masks)))
    return h


def _append(base, s, retain=1, masks=None):
    keep = []
    h = C.c_void_p()
    L.call('b3r_plan_append', C.byref(h), base, C.byref(_desc(s, keep, retain, masks)))
    return h


def _summary(h):
    i = L.PlanInfo()
    L.call('b3r_plan_get_info', h, C.byref(i))
    rp = np.zeros(i.n_blocks + 1, np.int32)
    ci = np.zeros(i.nnzb, np.int32)
    vo = np.zeros(i.nnzb, np.int64)
    bs = np.zeros(i.n_blocks, np.int32)
    bo = np.zeros(i.n_blocks, np.int32)
    L.call('b3r_plan_get_pattern', h, rp.ctypes.data, ci.ctypes.data, vo.ctypes.data, bs.ctypes.data, bo.ctypes.data)
    return {f: getattr(i, f) for f in INFO_FIELDS}, (rp, ci, vo, bs, bo)


def _assert_same_plan(h_app, h_full):
    ia, pa = _summary(h_app)
    ib, pb = _summary(h_full)
    assert ia == ib
    for x, y in zip(pa, pb):
        assert np.array_equal(x, y)


def _frame_masks(s, q):
    # P: every fifth node's pose off; Z: images 1 and 4 without depth coefficients
    return dict(P=np.arange(s.n_nodes) % 5 != 2, Z=~np.isin(np.arange(s.n_imgs), [1, 4]))


@pytest.mark.parametrize('cfg,ni,nt,q0,masked', [(3, 64, 3000, 1, False), (3, 32, 2000, 3, True),
                                                 (0, 20, 2000, 2, False), (1, 40, 4000, 5, False),
                                                 (4, 40, 3000, 4, False)])
def test_append_chain_equals_full_plan(cfg, ni, nt, q0, masked):
    """Frame by frame, each plan appended to the previous one equals the plan built from scratch."""
    seq = OnlineSequence(make_scene(cfg, n_imgs=ni, n_tracks=nt))
    s = seq.frame(q0)
    opt = (lambda sc, q: _frame_masks(sc, q)) if masked else (lambda sc, q: None)
    if cfg == 4:                       # the depth-stitch phase: focal and poses off
        opt = lambda sc, q: None
    prev = _create(s, masks=opt(s, q0))
    try:
        for q in range(q0 + 1, ni):
            s = seq.frame(q)
            h_app = _append(prev, s, masks=opt(s, q))
            h_full = _create(s, retain=0, masks=opt(s, q))
            try:
                _assert_same_plan(h_app, h_full)
                L_t = np.bincount(s.pids, minlength=s.n_tracks)
                if not masked:
                    assert _summary(h_app)[0]['n_pairs'] == int((L_t * (L_t - 1) // 2).sum())
            finally:
                L.call('b3r_plan_destroy', h_full)
            L.call('b3r_plan_destroy', prev)
            prev = h_app
    finally:
        L.call('b3r_plan_destroy', prev)


def test_append_without_points_and_several_frames_at_once():
    """optim_X off (no elimination: no tracks, no pairs), and a merge of several frames."""
    seq = OnlineSequence(make_scene(3, n_imgs=24, n_tracks=1500))
    s5, s9 = seq.frame(5), seq.frame(9)
    keep = []
    d5 = _desc(s5, keep)
    d5.mode_X = L.ENABLE_ZERO
    h5 = C.c_void_p()
    L.call('b3r_plan_create', C.byref(h5), C.byref(d5))
    d9 = _desc(s9, keep)
    d9.mode_X = L.ENABLE_ZERO
    h9, hf = C.c_void_p(), C.c_void_p()
    L.call('b3r_plan_append', C.byref(h9), h5, C.byref(d9))
    L.call('b3r_plan_create', C.byref(hf), C.byref(d9))
    _assert_same_plan(h9, hf)
    assert _summary(h9)[0]['n_pairs'] == 0
    for h in (h5, h9, hf):
        L.call('b3r_plan_destroy', h)
    a, b = _create(s5), _create(s9, retain=0)
    c = _append(a, s9)
    _assert_same_plan(c, b)
    for h in (a, b, c):
        L.call('b3r_plan_destroy', h)


def _variant(s, **kw):
    d = dict(s.__dict__)
    d.update(kw)
    return type(s)(**d)


def test_append_refuses_structures_that_do_not_extend():
    seq = OnlineSequence(make_scene(3, n_imgs=16, n_tracks=800))
    s6, s7 = seq.frame(6), seq.frame(7)
    base = _create(s6)
    no_state = _create(s6, retain=0)
    try:
        with pytest.raises(L.B3RError, match='no host state'):
            _append(no_state, s7)
        # two observations of an old image swapped
        pids = s7.pids.copy()
        pids[[0, 1]] = pids[[1, 0]]
        with pytest.raises(L.B3RError, match='not an extension'):
            _append(base, _variant(s7, pids=pids))
        # an old track observed again in the new image
        pids = s7.pids.copy()
        pids[-1] = 0
        with pytest.raises(L.B3RError, match='not an extension'):
            _append(base, _variant(s7, pids=pids))
        # a track removed and the others renumbered (ObservedTracks.remove, tracks.py:130-141)
        keep_o = s7.pids != 3
        pids = s7.pids[keep_o]
        _, pids = np.unique(pids, return_inverse=True)
        img = np.repeat(np.arange(s7.n_imgs), np.diff(np.concatenate([[0], s7.infos[0]])))[keep_o]
        infos = s7.infos.copy()
        infos[0] = np.cumsum(np.bincount(img, minlength=s7.n_imgs))
        with pytest.raises(L.B3RError, match='not an extension'):
            _append(base, _variant(s7, pids=pids.astype(np.int32), infos=infos, n_tracks=s7.n_tracks - 1,
                                   pix2d=s7.pix2d[keep_o], pix2d_std=s7.pix2d_std[keep_o],
                                   pix2d_dep=s7.pix2d_dep[keep_o]))
        # another number of depth channels
        with pytest.raises(L.B3RError, match='not an extension'):
            _append(base, _variant(s7, pix2d_dep=s7.pix2d_dep[:, :4]))
        # the same structure is an extension by nothing: it gives the same plan
        same = _append(base, s6)
        full = _create(s6, retain=0)
        _assert_same_plan(same, full)
        L.call('b3r_plan_destroy', same)
        L.call('b3r_plan_destroy', full)
    finally:
        L.call('b3r_plan_destroy', base)
        L.call('b3r_plan_destroy', no_state)


def _frame_tensors(s):
    return {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in s.lm_inputs().items()}


def test_solver_plans_online_frames_incrementally():
    """GaussNewtonSolver.compute_jacobians through the plan cache: each new frame of the online
    loop gets an appended plan equal to a fresh one; a structure that does not extend the last
    plan (here: a frame dropped from the problem) is planned from scratch."""
    seq = OnlineSequence(make_scene(3, n_imgs=20, n_tracks=1200))
    BS._PLAN_CACHE.clear()
    plans = []
    for q in range(8, 12):
        s = seq.frame(q)
        t = _frame_tensors(s)
        solver = BS.GaussNewtonSolver(s.n_cams, s.n_nodes, s.n_imgs, s.n_tracks, 'cpu')
        J = solver.compute_jacobians(t['rigs'], t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'],
                                     t['pids'], t['pix2d_std'], t['pix2d_dep'], is_depth_log=True)
        plans.append(J.plan)
        assert J.plan.retained
        assert J.plan.appended == (q > 8)
        fresh = BAPlan(t['rigs'], t['pids'], s.n_cams, s.n_nodes, s.n_tracks, s.n_zcf, device='cpu')
        _assert_same_plan(J.plan.handle, fresh.handle)
    s = seq.frame(9)
    t = _frame_tensors(s)
    solver = BS.GaussNewtonSolver(s.n_cams, s.n_nodes, s.n_imgs, s.n_tracks, 'cpu')
    J = solver.compute_jacobians(t['rigs'], t['K'], t['P_rig2cam'], t['P_w2rig'], t['z_coefs'], t['pts3d'],
                                 t['pids'].clone(), t['pix2d_std'], t['pix2d_dep'], is_depth_log=True)
    assert J.plan is plans[1]            # the cached plan of that structure
    BS._PLAN_CACHE.clear()
    s9, s = seq.frame(9), seq.frame(10)
    t9, t = _frame_tensors(s9), _frame_tensors(s)
    assert not BS.get_plan(t9['rigs'], t9['pids'], s9.n_cams, s9.n_nodes, s9.n_tracks, s9.n_zcf,
                           device='cpu').appended
    pids = t['pids'].clone()
    pids[[0, 1]] = pids[[1, 0]]
    p = BS.get_plan(t['rigs'], pids, s.n_cams, s.n_nodes, s.n_tracks, s.n_zcf, device='cpu')
    assert p.retained and not p.appended
    BS._PLAN_CACHE.clear()


def test_solver_appends_with_growing_masks():
    """Bool-tensor enable masks grow with the problem (one entry per node / image): the cache
    still appends, and the plan equals a fresh one."""
    seq = OnlineSequence(make_scene(3, n_imgs=16, n_tracks=900))
    BS._PLAN_CACHE.clear()
    try:
        for q in range(6, 9):
            s = seq.frame(q)
            t = _frame_tensors(s)
            mP = torch.ones(s.n_nodes, dtype=torch.bool)
            mP[2] = False
            mZ = torch.ones(s.n_imgs, dtype=torch.bool)
            mZ[[1, 4]] = False
            p = BS.get_plan(t['rigs'], t['pids'], s.n_cams, s.n_nodes, s.n_tracks, s.n_zcf, optim_P=mP,
                            optim_Z=mZ, device='cpu')
            assert p.appended == (q > 6)
            fresh = BAPlan(t['rigs'], t['pids'], s.n_cams, s.n_nodes, s.n_tracks, s.n_zcf, optim_P=mP, optim_Z=mZ,
                           device='cpu')
            _assert_same_plan(p.handle, fresh.handle)
    finally:
        BS._PLAN_CACHE.clear()


def test_solver_appends_across_frozen_single_frame_plans():
    """The online loop's pattern (inference/pipeline.py:212-224): a global BA on the merged
    problem every few frames and, between them, frozen BAs of the new frame alone (one image,
    points fixed).  The next global BA's plan is appended to the last global one, not planned
    from scratch, although other plans were built in between; under inference mode, as the
    reference's online loop runs."""
    seq = OnlineSequence(make_scene(3, n_imgs=24, n_tracks=1500))
    BS._PLAN_CACHE.clear()
    try:
        with torch.inference_mode():
            for q in (12, 16, 20):
                s = seq.frame(q)
                t = _frame_tensors(s)
                p = BS.get_plan(t['rigs'], t['pids'], s.n_cams, s.n_nodes, s.n_tracks, s.n_zcf, device='cpu')
                assert p.appended == (q > 12)
                fresh = BAPlan(t['rigs'], t['pids'], s.n_cams, s.n_nodes, s.n_tracks, s.n_zcf, device='cpu')
                _assert_same_plan(p.handle, fresh.handle)
                for f in range(q + 1, q + 4):        # frozen BAs of the next frames alone
                    sf = seq.frame(f)
                    img = np.repeat(np.arange(sf.n_imgs), np.diff(np.concatenate([[0], sf.infos[0]])))
                    sel = img == f
                    pids = np.unique(sf.pids[sel], return_inverse=True)[1].astype(np.int32)
                    rigs = torch.tensor([[int(sel.sum())], [0], [0]], dtype=torch.int32)
                    BS.get_plan(rigs, torch.from_numpy(pids), 1, 1, int(pids.max()) + 1, s.n_zcf, optim_X=False,
                                device='cpu')
    finally:
        BS._PLAN_CACHE.clear()


def test_append_refuses_status_changes_of_old_images_and_tracks():
    """Old images keep their node, camera and active blocks, old tracks their point status:
    a change of any of them is refused (the old lists would no longer describe them)."""
    seq = OnlineSequence(make_scene(3, n_imgs=16, n_tracks=800))
    s6, s7 = seq.frame(6), seq.frame(7)
    base = _create(s6, masks=dict(Z=np.ones(s6.n_imgs, bool)))
    try:
        infos = s7.infos.copy()
        infos[2, 3] = 5                               # image 3 now uses camera 5
        with pytest.raises(L.B3RError, match='node or camera'):
            _append(base, _variant(s7, infos=infos), masks=dict(Z=np.ones(s7.n_imgs, bool)))
        mZ = np.ones(s7.n_imgs, bool)
        mZ[2] = False                                 # image 2's depth coefficients switched off ...
        keep = []
        d = _desc(s7, keep, masks=dict(Z=mZ))
        d.mode_K = d.mode_P = L.ENABLE_ZERO           # ... and its focal and pose too: image 2 has no block
        h = C.c_void_p()
        with pytest.raises(L.B3RError, match='active blocks'):
            L.call('b3r_plan_append', C.byref(h), base, C.byref(d))
        mX = np.ones(s7.n_tracks, bool)
        mX[0] = False                                 # track 0's point no longer optimised
        with pytest.raises(L.B3RError, match='point status'):
            _append(base, s7, masks=dict(Z=np.ones(s7.n_imgs, bool), X=mX))
        ok = _append(base, s7, masks=dict(Z=np.ones(s7.n_imgs, bool)))
        L.call('b3r_plan_destroy', ok)
    finally:
        L.call('b3r_plan_destroy', base)


def test_online_sequence_matches_the_reference_merge():
    """synthetic.OnlineSequence builds, frame by frame, exactly the problems the reference's own
    ObservedTracks.__or__ produces in its online loop (golden vectors from
    tests/golden/make_golden_merge.py: observations per image, track ids, keypoints)."""
    import os
    z = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden', 'refmerge_online.npz'))
    sc = make_scene(3, n_imgs=12, n_tracks=400, seed=301)
    assert np.array_equal(sc.pids, z['scene_pids']) and np.array_equal(sc.pix2d, z['scene_pix2d'])
    seq = OnlineSequence(sc)
    for q in range(sc.n_imgs):
        f = seq.frame(q)
        assert f.n_tracks == int(z[f'f{q}_n_tracks'])
        assert np.array_equal(np.diff(np.concatenate([[0], f.infos[0]])), z[f'f{q}_nppi'])
        assert np.array_equal(f.pids, z[f'f{q}_pids'])
        assert np.array_equal(f.pix2d, z[f'f{q}_pix2d'])


def test_append_edge_cases_empty_problems_and_empty_frames():
    """Appending to an empty problem (frame 0 holds no track yet), and a merge that adds an
    image without any observation (a frame whose tracks all continue later): both give the
    fresh plan."""
    seq = OnlineSequence(make_scene(3, n_imgs=10, n_tracks=500))
    s0, s1, s2 = seq.frame(0), seq.frame(1), seq.frame(2)
    assert s0.n_obs == 0 and s0.n_tracks == 0
    h0 = _create(s0)
    h1 = _append(h0, s1)
    f1 = _create(s1, retain=0)
    _assert_same_plan(h1, f1)
    h2 = _append(h1, s2)
    f2 = _create(s2, retain=0)
    _assert_same_plan(h2, f2)
    # one more image with no observation, same tracks
    infos = np.concatenate([s2.infos, np.array([[s2.infos[0, -1]], [s2.n_imgs], [s2.n_imgs]], np.int32)], 1)
    s3 = _variant(s2, infos=infos, n_imgs=s2.n_imgs + 1, n_nodes=s2.n_nodes + 1, n_cams=s2.n_cams + 1)
    h3 = _append(h2, s3)
    f3 = _create(s3, retain=0)
    _assert_same_plan(h3, f3)
    for h in (h0, h1, f1, h2, f2, h3, f3):
        L.call('b3r_plan_destroy', h)
