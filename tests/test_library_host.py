"""Host-side checks that need no GPU: the C-ABI library loads and exports every symbol
that ``include/b3r.h`` declares, and the host planner's S pattern equals the oracle's."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from blast3r_b200 import _lib as L
from blast3r_b200.synthetic import make_scene
from oracle import ba_oracle as O

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), 'include', 'b3r.h')


def header_symbols():
    txt = open(HEADER).read()
    return sorted(set(re.findall(r'^\s*(?:const\s+)?\w+\*?\s+\**(b3r_\w+)\s*\(', txt, re.M)))


def test_library_exports_every_header_symbol():
    lib = L.lib()
    syms = header_symbols()
    assert len(syms) >= 19
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) <= set(L.exported_symbols())
    assert lib.b3r_version().startswith(b'blast3r_b200')


def _host_plan(sc, **kw):
    infos = np.ascontiguousarray(sc.infos, np.int32)
    pids = np.ascontiguousarray(sc.pids, np.int32)
    d = L.PlanDesc(n_imgs=sc.n_imgs, n_cams=sc.n_cams, n_nodes=sc.n_nodes, n_tracks=sc.n_tracks,
                   n_obs=sc.n_obs, C=sc.n_zcf, infos=infos.ctypes.data_as(C.POINTER(C.c_int32)),
                   pids=pids.ctypes.data_as(C.POINTER(C.c_int32)), track_begin=0, track_end=sc.n_tracks,
                   device=-1, **kw)
    h = C.c_void_p()
    L.call('b3r_plan_create', C.byref(h), C.byref(d))
    info = L.PlanInfo()
    L.call('b3r_plan_get_info', h, C.byref(info))
    rp = np.zeros(info.n_blocks + 1, np.int32)
    ci = np.zeros(info.nnzb, np.int32)
    L.call('b3r_plan_get_pattern', h, rp.ctypes.data, ci.ctypes.data, None, None, None)
    L.call('b3r_plan_destroy', h)
    return info, np.stack([np.repeat(np.arange(info.n_blocks), np.diff(rp)), ci], 1)


@pytest.mark.parametrize('cfg,ni,nt', [(0, 8, 120), (3, 8, 150), (0, 20, 2000), (1, 40, 4000), (3, 64, 3000)])
def test_plan_pattern_equals_oracle(cfg, ni, nt):
    sc = make_scene(cfg, n_imgs=ni, n_tracks=nt)
    info, pat = _host_plan(sc)
    lay = O.Layout(sc.infos, sc.pids, sc.n_cams, sc.n_nodes, sc.n_tracks, sc.n_zcf)
    assert np.array_equal(pat, O.s_pattern(lay))
    assert info.n_cam_params == lay.n_cam_params
    # every cross-image observation pair of every track is planned exactly once
    L_t = np.bincount(sc.pids, minlength=sc.n_tracks)
    assert info.n_pairs == int((L_t * (L_t - 1) // 2).sum())


def test_plan_pattern_with_disabled_types():
    sc = make_scene(0, n_imgs=8, n_tracks=120)
    info, pat = _host_plan(sc, mode_K=L.ENABLE_ZERO, mode_P=L.ENABLE_ZERO)
    lay = O.Layout(sc.infos, sc.pids, sc.n_cams, sc.n_nodes, sc.n_tracks, sc.n_zcf, False, False)
    assert np.array_equal(pat, O.s_pattern(lay))


def test_plan_rejects_bad_inputs():
    sc = make_scene(0, n_imgs=8, n_tracks=50)
    bad = np.ascontiguousarray(sc.infos, np.int32).copy()
    bad[0, -1] += 1                       # cumulative count no longer matches n_obs
    pids = np.ascontiguousarray(sc.pids, np.int32)
    d = L.PlanDesc(n_imgs=sc.n_imgs, n_cams=sc.n_cams, n_nodes=sc.n_nodes, n_tracks=sc.n_tracks,
                   n_obs=sc.n_obs, C=sc.n_zcf, infos=bad.ctypes.data_as(C.POINTER(C.c_int32)),
                   pids=pids.ctypes.data_as(C.POINTER(C.c_int32)), track_begin=0, track_end=sc.n_tracks,
                   device=-1)
    h = C.c_void_p()
    with pytest.raises(L.B3RError, match='must equal n_obs'):
        L.call('b3r_plan_create', C.byref(h), C.byref(d))


def test_local_observation_input_rows():
    """With obs_local the input rows are this rank's observations in image order."""
    sc = make_scene(1, n_imgs=40, n_tracks=3000)
    t0, t1 = 1000, 2200
    infos = np.ascontiguousarray(sc.infos, np.int32)
    pids = np.ascontiguousarray(sc.pids, np.int32)
    for local in (0, 1):
        d = L.PlanDesc(n_imgs=sc.n_imgs, n_cams=sc.n_cams, n_nodes=sc.n_nodes, n_tracks=sc.n_tracks,
                       n_obs=sc.n_obs, C=sc.n_zcf, infos=infos.ctypes.data_as(C.POINTER(C.c_int32)),
                       pids=pids.ctypes.data_as(C.POINTER(C.c_int32)), track_begin=t0, track_end=t1,
                       device=-1, obs_local=local)
        h = C.c_void_p()
        L.call('b3r_plan_create', C.byref(h), C.byref(d))
        info = L.PlanInfo()
        L.call('b3r_plan_get_info', h, C.byref(info))
        rows = np.empty(info.n_obs_input, np.int32)
        L.call('b3r_plan_get_input_obs', h, rows.ctypes.data)
        L.lib().b3r_plan_destroy(h)
        want = np.nonzero((sc.pids >= t0) & (sc.pids < t1))[0] if local else np.arange(sc.n_obs)
        assert np.array_equal(rows, want)
