"""ctypes binding of the C-ABI library ``libb3r.so`` (declared in ``include/b3r.h``).

The library is built in-tree (``__graft_entry__.build()`` / ``make -C blast3r_b200/csrc``).
There is no fallback: every op of this package raises if the library is missing.
"""
import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, 'libb3r.so')

B3R_OK = 0
B3R_F32, B3R_F64 = 0, 1
ENABLE_ALL, ENABLE_ZERO, ENABLE_MASK = 0, 1, 2
PASS_PREP, PASS_POINTS, PASS_FACTOR, PASS_DIAG, PASS_PAIRS = 0, 1, 2, 3, 4
PASS_ELIMINATE = PASS_FACTOR   # former name
PCG_TEST_UNREACHABLE_BARRIER = 1
PCG_STREAMING = 2
PCG_TEST_GLOBAL_TILES = 4

_i32, _i64, _f32, _f64, _vp = C.c_int32, C.c_int64, C.c_float, C.c_double, C.c_void_p
_pi32 = C.POINTER(C.c_int32)
_pu8 = C.POINTER(C.c_uint8)


class PlanDesc(C.Structure):
    _fields_ = [('n_imgs', _i32), ('n_cams', _i32), ('n_nodes', _i32), ('n_tracks', _i32),
                ('n_obs', _i64), ('C', _i32), ('infos', _pi32), ('pids', _pi32),
                ('mode_K', _i32), ('mode_P', _i32), ('mode_Z', _i32), ('mode_X', _i32),
                ('mask_K', _pu8), ('mask_P', _pu8), ('mask_Z', _pu8), ('mask_X', _pu8),
                ('track_begin', _i32), ('track_end', _i32), ('device', _i32), ('obs_local', _i32),
                ('track_owner', _pi32), ('rank', _i32), ('retain', _i32)]


class PlanInfo(C.Structure):
    _fields_ = [('n_obs', _i64), ('n_obs_local', _i64), ('n_tracks_local', _i64),
                ('n_blocks', _i32), ('n_cam_params', _i32), ('n_points', _i32),
                ('nnzb', _i64), ('nnz', _i64), ('n_pairs', _i64), ('n_segments', _i64),
                ('n_pair_tasks', _i64), ('n_point_tasks', _i64), ('n_diag_chunks', _i64),
                ('workspace_bytes', _i64), ('nb_K', _i32), ('nb_P', _i32), ('nb_Z', _i32),
                ('off_P', _i32), ('off_Z', _i32), ('record_floats', _i32), ('n_obs_input', _i64),
                ('depth_stitch', _i32), ('pcg_row_groups', _i32),
                ('pcg_resident', _i32)]


class Params(C.Structure):
    _fields_ = [('K', _vp), ('P_rig2c', _vp), ('P_rig2c_stride', _i64), ('P_w2rig', _vp),
                ('z_coefs', _vp), ('pts3d', _vp), ('pix2d', _vp), ('pix2d_std', _vp),
                ('pix2d_dep', _vp), ('residuals', _vp), ('res_stride_n', _i64),
                ('res_stride_c', _i64), ('w_pts', _vp), ('w_stride_n', _i64),
                ('w_stride_c', _i64), ('w_cols', _i32)]


class LinOpts(C.Structure):
    _fields_ = [('is_depth_log', _i32), ('weight_z', _f32), ('pnorm', _f32), ('max_pix_err', _f32),
                ('huber_delta', _f32), ('w_pts_nul', _f32), ('clamp_w_lo', _f32), ('clamp_w_hi', _f32),
                ('dampen', _f64), ('adaptive_dampen', _i32), ('no_grad_f_from_rz', _i32),
                ('optim_Z0', _i32), ('optim_Z_1st_cam', _i32)]


class Outputs(C.Structure):
    _fields_ = [('S_vals', _vp), ('b', _vp), ('diagA', _vp), ('precond', _vp), ('hpp_max', _vp),
                ('residuals', _vp), ('loss', _vp)]


# name -> (restype, argtypes)
_SIGS = {
    'b3r_last_error': (C.c_char_p, []),
    'b3r_version': (C.c_char_p, []),
    'b3r_residuals_with_rigs': (C.c_int, [_vp, C.c_int, _vp, C.c_int, _vp, _i64, _vp, C.c_int, _vp,
                                          C.c_int, _vp, C.c_int, _vp, _i64, _vp, _vp, _vp, C.c_int,
                                          _f32, _f32, _f32, _f32, _f32, _vp, _vp]),
    'b3r_residual_loss': (C.c_int, [_vp, C.c_int, _vp, C.c_int, _vp, _i64, _vp, C.c_int, _vp, C.c_int, _vp,
                                    C.c_int, _vp, _i64, _vp, _vp, _vp, C.c_int, _f32, _f32, _f32, _f32, _vp, _vp,
                                    _vp]),
    'b3r_jacobians_with_rigs': (C.c_int, [_vp, C.c_int, _vp, C.c_int, _vp, _i64, _vp, C.c_int, _vp,
                                          C.c_int, _vp, C.c_int, _vp, _i64, _vp, _vp, C.c_int,
                                          C.c_int, _vp, _vp, _vp, _vp]),
    'b3r_chol3x3_solve': (C.c_int, [_vp, _vp, _vp, _i64, _f64, C.c_int, _vp]),
    'b3r_blockcoo_matvec': (C.c_int, [_vp, C.c_int, C.c_int, _vp, _vp, C.c_int, _i64, _vp, _vp,
                                      _i64, _i64, C.c_int, C.c_int, _vp]),
    'b3r_fused_einsum_bki_bkj': (C.c_int, [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, C.c_int,
                                           C.c_int, C.c_int, C.c_int, _vp]),
    'b3r_plan_create': (C.c_int, [C.POINTER(_vp), C.POINTER(PlanDesc)]),
    'b3r_plan_append': (C.c_int, [C.POINTER(_vp), _vp, C.POINTER(PlanDesc)]),
    'b3r_plan_destroy': (C.c_int, [_vp]),
    'b3r_plan_get_info': (C.c_int, [_vp, C.POINTER(PlanInfo)]),
    'b3r_plan_get_pattern': (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp]),
    'b3r_plan_stage_obs': (C.c_int, [_vp, _vp, _vp, _vp, _vp]),
    'b3r_plan_get_input_obs': (C.c_int, [_vp, _vp]),
    'b3r_linearize_schur': (C.c_int, [_vp, C.POINTER(Params), C.POINTER(LinOpts), _vp,
                                      C.POINTER(Outputs), _vp]),
    'b3r_linearize_schur_noalloc': (C.c_int, [_vp, C.POINTER(Params), C.POINTER(LinOpts), C.POINTER(Outputs), _vp]),
    'b3r_lin_points': (C.c_int, [_vp, C.POINTER(Params), C.POINTER(LinOpts), _vp, C.POINTER(Outputs), _vp]),
    'b3r_lin_assemble': (C.c_int, [_vp, C.POINTER(Params), C.POINTER(LinOpts), _vp, C.POINTER(Outputs), _vp]),
    'b3r_lin_pass': (C.c_int, [_vp, C.POINTER(Params), C.POINTER(LinOpts), _vp, C.POINTER(Outputs), C.c_int, _vp]),
    'b3r_lin_finalize': (C.c_int, [_vp, C.POINTER(LinOpts), _vp, C.POINTER(Outputs), _vp]),
    'b3r_schur_spmv': (C.c_int, [_vp, _vp, _vp, _vp, _vp]),
    'b3r_schur_spmv_f64': (C.c_int, [_vp, _vp, _vp, _vp, _vp]),
    'b3r_backsub': (C.c_int, [_vp, C.POINTER(Params), C.POINTER(LinOpts), _vp, _vp, _vp, _vp]),
    'b3r_pcg_work_bytes': (_i64, [_vp]),
    'b3r_reproj_score_work_bytes': (_i64, [_i64]),
    'b3r_reproj_score': (C.c_int, [_vp, _i64, _i64, _i64, _vp, _vp, _vp]),
    'b3r_pcg': (C.c_int, [_vp, _vp, _vp, _vp, _vp, _f64, C.c_int, _vp, _vp, _vp]),
    'b3r_pcg_f64': (C.c_int, [_vp, _vp, _vp, _vp, _vp, _f64, C.c_int, _vp, _vp, _vp]),
    'b3r_tangent_prior': (C.c_int, [_vp, _i32, _i32, _vp, _vp, _vp, _i32, _vp, _i32, _f64, _f64, _i32, _i32, _vp,
                                    _vp, _vp, _vp]),
    'b3r_lin_add_zprior': (C.c_int, [_vp, _vp, _vp, _vp, C.POINTER(Outputs), _vp]),
    'b3r_pcg_ex': (C.c_int, [_vp, _vp, _vp, _vp, _vp, C.c_int, _f64, C.c_int, _i64, C.c_int, _vp, _vp, _vp]),
}

_lib = None


def lib():
    """The loaded library (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.isfile(LIB_PATH):
            raise RuntimeError(f'{LIB_PATH} is missing: build it with __graft_entry__.build() '
                               f'or `make -C blast3r_b200/csrc`')
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def exported_symbols():
    return list(_SIGS)


class B3RError(RuntimeError):
    pass


def check(rc, what=''):
    if rc != B3R_OK:
        msg = lib().b3r_last_error().decode(errors='replace')
        raise B3RError(f'{what or "b3r call"} failed ({rc}): {msg}')
    return rc


def call(name, *args):
    return check(getattr(lib(), name)(*args), name)
