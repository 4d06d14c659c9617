// Part 2 of the C ABI: the fused per-LM-iteration linearization and Schur assembly.
//
// Replaces, for one LM iteration, GaussNewtonSolver.compute_jacobians + solve_delta up to
// its PCG (naver/blast3r src/blast3r/inference/ba_solver.py:34-188).  J is never written
// to memory.  Passes (one launch each, all on the caller's stream):
//   prep      per-image camera records (one 128-byte line per image)
//   points    track-major, one warp per <=32-observation task: per-track Hpp and g_p by a
//             segmented warp scan, and the max |diag(Hpp)| for adaptive damping
//   factor    per track: damped guarded 3x3 Cholesky Hpp = L L^T (sfm_jacobian_rigs.cu
//             :578-617) computed in double and rounded once, stored in reciprocal form, and
//             z = L^-1 g_p from the rounded factor (the one the elimination records use)
//   diag      image-major: per observation the elimination record Y = L^-1 Hpc in reduced
//             form (3 x [f0 f1 tau0..5 zscale]) + its depth channels, written to its
//             image-major slot; Hcc - Y^T Y and g_c - Y^T z expanded to the typed blocks of
//             its image, reduced per image chunk, one atomic per value per chunk; also
//             diag(Hcc) for the damping and preconditioner
//   pairs     segment-major: for every image pair (i, i') the sum over shared tracks of
//             -Y_o^T Y_o', one CTA per <= 1024-pair task, lane per observation pair, packed
//             float2 FMAs, records staged through shared memory by coalesced cp.async,
//             one atomic per value per task
//   finalize  per-type adaptive damping of diag(S) (ba_solver.py:510-517, 572-582) and
//             the Jacobi preconditioner of the reference's PCG (ba_solver.py:191-192)
#include <algorithm>
#include <cstring>
#include <mutex>
#include "b3r_common.cuh"
#include "b3r_plan.h"
#include "b3r_status.h"

namespace b3r {
namespace {

// Per-call state passed by value to the kernels.
struct Ctx {
  DevPlan d;
  LinOpts o;
  const float* K; const float* P_rig2c; int64_t P_stride; const float* P_w2rig;
  const float* z_coefs; const float* pts3d;
  const float* pix2d; const float* pix2d_std; const float* pix2d_dep;
  const float* res; int64_t rs_n, rs_c;
  const float* wpt; int64_t ws_n, ws_c; int w_cols;
  float* img_rec;     // [n_imgs*32]
  float* trec;        // [nT_loc*24]
  float* rec;         // [n_loc*R]
  float* t_rw;        // [6][n_loc] staged residual (0..2) and weight (3..5), general path
  float* misc;        // [64]: 4..6 per-type max |diag A|
  float* res_out;     // [3][n_in] residual outputs, or NULL
  double* loss_part;  // [n_c1_chunks + kRestBlocks] per-block Huber-error sums, or NULL
  float* hpp_max;     // [1] max |diag(Hpp)| (caller-visible, all-reduced across ranks)
  int no_grad_f_from_rz, optim_Z0, optim_Z_1st_cam;
  float dampen;
  int adaptive;
};

// ------------------------------------------------------------------------------------
// small kernels
// ------------------------------------------------------------------------------------
__global__ void k_prep_images(Ctx c) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= c.d.n_imgs) return;
  const int node = c.d.img_node[i], cam = c.d.img_cam[i];
  const float* Prw = c.P_w2rig + (int64_t)node * 16;
  const float* Pcr = c.P_rig2c + (int64_t)cam * c.P_stride;
  const float* Kc = c.K + (int64_t)cam * 9;
  float* r = c.img_rec + (int64_t)i * kImgRec;
#pragma unroll
  for (int a = 0; a < 3; ++a) {
#pragma unroll
    for (int b = 0; b < 3; ++b) { r[3 * a + b] = Prw[4 * a + b]; r[12 + 3 * a + b] = Pcr[4 * a + b]; }
    r[9 + a] = Prw[4 * a + 3];
    r[21 + a] = Pcr[4 * a + 3];
  }
  r[24] = Kc[0]; r[25] = Kc[4]; r[26] = Kc[2]; r[27] = Kc[5];
  r[28] = r[29] = r[30] = r[31] = 0.f;
}

__global__ void k_stage_obs(DevPlan d, const float* __restrict__ pix2d, const float* __restrict__ std_,
                            const float* __restrict__ dep) {
  const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= d.n_loc) return;
  const int64_t o = d.perm_t[k];
  if (pix2d) d.t_pix[k] = make_float2(pix2d[2 * o], pix2d[2 * o + 1]);
  d.t_std[k] = make_float2(std_[2 * o], std_[2 * o + 1]);
  for (int ch = 0; ch < d.C; ++ch) d.t_dep[(int64_t)ch * d.n_loc + k] = dep[o * d.C + ch];
}

__global__ void k_stage_rw(Ctx c) {
  const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= c.d.n_loc) return;
  const int64_t o = c.d.perm_t[k], n = c.d.n_loc;
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    c.t_rw[j * n + k] = c.res[o * c.rs_n + j * c.rs_c];
    c.t_rw[(3 + j) * n + k] = c.wpt[o * c.ws_n + (c.w_cols == 1 ? 0 : j) * c.ws_c];
  }
}

// ------------------------------------------------------------------------------------
// per-observation view used by every pass
// ------------------------------------------------------------------------------------
// Reduced camera-side Jacobian of one observation, rows scaled by sqrt(W):
//   columns 0,1 focal (fx, fy), 2..7 tau, 8 "z scale" (the depth-coefficient columns are
//   zs * dep_c in the depth row only, so they are carried as one column and expanded
//   with the depth channels when written out).
template <int CT>
struct ObsView {
  bool valid;
  float Jpw[9];     // sqrt(W) * d r / d X        (3x3 row-major)
  float Jcw[27];    // sqrt(W) * reduced camera J (3x9 row-major)
  float sWr[3];     // sqrt(W) * r, so J^T W r = Jw^T sWr
  float dep[CT];    // depth channels as used by J (optim_Z0 / optim_Z_1st_cam applied)
};

// Structural non-zeros of the reduced camera Jacobian: row 0 (x) has fx and tau, row 1 (y)
// fy and tau, row 2 (depth) every column.  Products skip the zero entries (the same values
// as the dense products for finite inputs).
__host__ __device__ constexpr bool jc_nz(int i, int a) { return i == 2 || (a >= 2 && a < 8) || a == i; }

// Masks of the image's blocks: bit 0 foc, 1 tau, 2 zcf active.
__device__ __forceinline__ int image_mask(const DevPlan& d, int img) {
  return (d.img_bk[3 * img] >= 0 ? 1 : 0) | (d.img_bk[3 * img + 1] >= 0 ? 2 : 0) |
         (d.img_bk[3 * img + 2] >= 0 ? 4 : 0);
}

template <int CT>
__device__ __forceinline__ void make_view(const Ctx& c, const ObsLin& L, float r0, float r1, float r2,
                                          float w0, float w1, float w2, const float* dep_raw, int64_t o,
                                          int mask, ObsView<CT>& V) {
  V.valid = L.valid;
  const float r[3] = {r0, r1, r2};
  const float w[3] = {w0, w1, w2};
  float sW[3];
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const float W = clampw(w[i], c.o.clamp_lo, c.o.clamp_hi);
    sW[i] = sqrtf(W);
    V.sWr[i] = sW[i] * r[i];
  }
  const bool mf = mask & 1, mt = mask & 2, mz = mask & 4;
  const float jkf = c.no_grad_f_from_rz ? 0.f : L.Jkf;
  float J[27];
  J[0] = mf ? L.Jf0 : 0.f; J[1] = 0.f;
  J[9] = 0.f;              J[10] = mf ? L.Jf1 : 0.f;
  J[18] = mf ? jkf : 0.f;  J[19] = mf ? jkf : 0.f;
#pragma unroll
  for (int i = 0; i < 3; ++i) {
#pragma unroll
    for (int t = 0; t < 6; ++t) J[9 * i + 2 + t] = mt ? L.Jt[6 * i + t] : 0.f;
  }
  J[8] = 0.f; J[17] = 0.f; J[26] = mz ? L.zs : 0.f;
#pragma unroll
  for (int i = 0; i < 3; ++i) {
#pragma unroll
    for (int a = 0; a < 9; ++a) V.Jcw[9 * i + a] = J[9 * i + a] * sW[i];
#pragma unroll
    for (int j = 0; j < 3; ++j) V.Jpw[3 * i + j] = L.Jp[3 * i + j] * sW[i];
  }
#pragma unroll
  for (int ch = 0; ch < CT; ++ch) V.dep[ch] = dep_raw[ch];
  // the reference zeroes channel 0 of observation 0's depth Jacobian (ba_solver.py:38)
  if (!c.optim_Z0 || (o == c.d.first_in && !c.optim_Z_1st_cam)) V.dep[0] = 0.f;
}

// Load + linearize local (track-sorted) observation k.
template <int CT>
__device__ __forceinline__ void view_local(const Ctx& c, int64_t k, ObsView<CT>& V, int& tl) {
  const DevPlan& d = c.d;
  const int4 ix = __ldg(d.t_idx + k);          // image, global track id, local track, o
  const int img = ix.x, gid = ix.y;
  tl = ix.z;
  const Cam cam = load_cam(c.img_rec + (int64_t)img * kImgRec);
  const float X[3] = {__ldg(c.pts3d + 3 * (int64_t)gid), __ldg(c.pts3d + 3 * (int64_t)gid + 1),
                      __ldg(c.pts3d + 3 * (int64_t)gid + 2)};
  const float2 s = d.t_std[k];
  float dep[CT], zc[CT];
#pragma unroll
  for (int ch = 0; ch < CT; ++ch) {
    dep[ch] = d.t_dep[(int64_t)ch * d.n_loc + k];
    zc[ch] = __ldg(c.z_coefs + (int64_t)img * CT + ch);
  }
  ObsLin L;
  float r0, r1, r2, w0, w1, w2;
  if (c.pix2d) {
    const float2 px = d.t_pix[k];
    linearize_obs<float, true, true, CT>(cam, X, px.x, px.y, s.x, s.y, dep, zc, CT, c.o, L);
    r0 = L.r[0]; r1 = L.r[1]; r2 = L.r[2]; w0 = L.w[0]; w1 = L.w[1]; w2 = L.w[2];
  } else {
    linearize_obs<float, false, true, CT>(cam, X, 0.f, 0.f, s.x, s.y, dep, zc, CT, c.o, L);
    const int64_t n = d.n_loc;
    r0 = c.t_rw[k]; r1 = c.t_rw[n + k]; r2 = c.t_rw[2 * n + k];
    w0 = c.t_rw[3 * n + k]; w1 = c.t_rw[4 * n + k]; w2 = c.t_rw[5 * n + k];
  }
  make_view<CT>(c, L, r0, r1, r2, w0, w1, w2, dep, ix.w, image_mask(d, img), V);
}



// Raw inputs of one local (track-sorted) observation, loaded one task ahead.
template <int CT>
struct LocIn {
  int4 ix;          // image, global track id, local track, o
  float X[3];
  float2 px, sd;
  float dep[CT];
};

template <int CT>
__device__ __forceinline__ void load_loc_in(const Ctx& c, int64_t k, bool valid, LocIn<CT>& in) {
  if (!valid) { in.ix = make_int4(0, 0, -1, 0); return; }
  const DevPlan& d = c.d;
  in.ix = __ldg(d.t_idx + k);
  const int64_t gid = in.ix.y;
  in.X[0] = __ldg(c.pts3d + 3 * gid); in.X[1] = __ldg(c.pts3d + 3 * gid + 1); in.X[2] = __ldg(c.pts3d + 3 * gid + 2);
  in.sd = d.t_std[k];
  in.px = c.pix2d ? d.t_pix[k] : make_float2(0.f, 0.f);
#pragma unroll
  for (int ch = 0; ch < CT; ++ch) in.dep[ch] = d.t_dep[(int64_t)ch * d.n_loc + k];
}

// Linearize a prefetched local observation k.
template <int CT>
__device__ __forceinline__ void view_loc(const Ctx& c, int64_t k, const LocIn<CT>& in, ObsView<CT>& V) {
  const int img = in.ix.x;
  const Cam cam = load_cam(c.img_rec + (int64_t)img * kImgRec);
  float zc[CT];
#pragma unroll
  for (int ch = 0; ch < CT; ++ch) zc[ch] = __ldg(c.z_coefs + (int64_t)img * CT + ch);
  ObsLin L;
  float r0, r1, r2, w0, w1, w2;
  if (c.pix2d) {
    linearize_obs<float, true, true, CT>(cam, in.X, in.px.x, in.px.y, in.sd.x, in.sd.y, in.dep, zc, CT, c.o, L);
    r0 = L.r[0]; r1 = L.r[1]; r2 = L.r[2]; w0 = L.w[0]; w1 = L.w[1]; w2 = L.w[2];
  } else {
    linearize_obs<float, false, true, CT>(cam, in.X, 0.f, 0.f, in.sd.x, in.sd.y, in.dep, zc, CT, c.o, L);
    const int64_t n = c.d.n_loc;
    r0 = c.t_rw[k]; r1 = c.t_rw[n + k]; r2 = c.t_rw[2 * n + k];
    w0 = c.t_rw[3 * n + k]; w1 = c.t_rw[4 * n + k]; w2 = c.t_rw[5 * n + k];
  }
  make_view<CT>(c, L, r0, r1, r2, w0, w1, w2, in.dep, in.ix.w, image_mask(c.d, img), V);
}

// Raw inputs of one image-major observation, loaded one batch ahead of their use so
// that the gathers (track point, track factor) overlap the previous batch's arithmetic.
template <int CT>
struct ObsIn {
  int4 ix;          // o, k (-1: track not eliminated), track id, local track
  float X[3];       // track point
  float px, py, sx, sy;
  float dep[CT];
  float4 tf0, tf1;  // track factor (reciprocal form) and z, track-record floats 12..19
  float4 tf2;       // track-record floats 20..23: z[2] (21..23 unused)
};

template <int CT>
__device__ __forceinline__ void load_obs_in(const Ctx& c, int e, int ee, ObsIn<CT>& in) {
  if (e >= ee) { in.ix = make_int4(0, -1, 0, -1); return; }
  in.ix = __ldg(c.d.c1_idx + e);
  const int64_t o = in.ix.x, pid = in.ix.z;
  in.X[0] = __ldg(c.pts3d + 3 * pid); in.X[1] = __ldg(c.pts3d + 3 * pid + 1); in.X[2] = __ldg(c.pts3d + 3 * pid + 2);
  const float2 s = __ldg(reinterpret_cast<const float2*>(c.pix2d_std) + o);
  in.sx = s.x; in.sy = s.y;
  if (c.pix2d) {
    const float2 q = __ldg(reinterpret_cast<const float2*>(c.pix2d) + o);
    in.px = q.x; in.py = q.y;
  } else {
    in.px = in.py = 0.f;
  }
#pragma unroll
  for (int ch = 0; ch < CT; ++ch) in.dep[ch] = __ldg(c.pix2d_dep + o * CT + ch);
  if (in.ix.y >= 0) {
    // trec is 256-byte aligned with 96-byte records: floats 12..19 are two aligned float4
    const float4* t4 = reinterpret_cast<const float4*>(c.trec + (int64_t)in.ix.w * 24 + 12);
    in.tf0 = t4[0]; in.tf1 = t4[1]; in.tf2 = t4[2];
  }
}

// Linearize a prefetched image-major observation of image img.
template <int CT, bool OBJ>
__device__ __forceinline__ void view_in(const Ctx& c, const ObsIn<CT>& in, int img, const Cam& cam, const float* zc,
                                        ObsView<CT>& V, float& esum) {
  const int64_t o = in.ix.x;
  ObsLin L;
  float r0, r1, r2, w0, w1, w2;
  esum = 0.f;
  if (c.pix2d) {
    linearize_obs<float, true, true, CT>(cam, in.X, in.px, in.py, in.sx, in.sy, in.dep, zc, CT, c.o, L);
    r0 = L.r[0]; r1 = L.r[1]; r2 = L.r[2]; w0 = L.w[0]; w1 = L.w[1]; w2 = L.w[2];
    if (OBJ) {
      if (c.res_out) {                            // the objective's residuals, at the input row
        const int64_t n = c.d.n_in;
        c.res_out[o] = r0; c.res_out[n + o] = r1; c.res_out[2 * n + o] = r2;
      }
      esum = L.err[0] + L.err[1] + L.err[2];
    }
  } else {
    linearize_obs<float, false, true, CT>(cam, in.X, 0.f, 0.f, in.sx, in.sy, in.dep, zc, CT, c.o, L);
    r0 = c.res[o * c.rs_n]; r1 = c.res[o * c.rs_n + c.rs_c]; r2 = c.res[o * c.rs_n + 2 * c.rs_c];
    const int64_t wc = c.w_cols == 1 ? 0 : c.ws_c;
    w0 = c.wpt[o * c.ws_n]; w1 = c.wpt[o * c.ws_n + wc]; w2 = c.wpt[o * c.ws_n + 2 * wc];
  }
  make_view<CT>(c, L, r0, r1, r2, w0, w1, w2, in.dep, o, image_mask(c.d, img), V);
}

// Hpp (upper: 00 01 02 11 12 22) and g_p of one observation.
template <int CT>
__device__ __forceinline__ void point_terms(const ObsView<CT>& V, float v[9]) {
  const int ia[6] = {0, 0, 0, 1, 1, 2}, ib[6] = {0, 1, 2, 1, 2, 2};
#pragma unroll
  for (int e = 0; e < 6; ++e) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 3; ++i) s += V.Jpw[3 * i + ia[e]] * V.Jpw[3 * i + ib[e]];
    v[e] = s;
  }
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 3; ++i) s += V.Jpw[3 * i + j] * V.sWr[i];
    v[6 + j] = s;
  }
}

// Elimination record of one observation, Y = L^-1 Hpc (3 x 9 reduced camera columns)
// and its depth channels: [0, 24) Y[r][a] at 8 r + a for the columns a < 8 (row-major, so
// that neighbouring columns pair up for packed float2 arithmetic), [24, 24+C) the depth
// channels, [24+C, 27+C) the z-scale column Y[r][8], padded to a multiple of 4 floats.
template <int CT>
__host__ __device__ constexpr int rec_floats() { return (27 + CT + 3) & ~3; }
template <int CT>
__host__ __device__ constexpr int rec_zs() { return 24 + CT; }

// Y = L^-1 Hpc of one observation from the track's factor in reciprocal form
// li = (1/l00, l10, l20, 1/l11, l21, 1/l22); written as the record of slot e.
template <int CT>
__device__ __forceinline__ void elim_record(const Ctx& c, int64_t e, const ObsView<CT>& V, const float li[6],
                                            float Y[9][3]) {
  constexpr int R = rec_floats<CT>();
  float rv[R];
#pragma unroll
  for (int a = 0; a < 9; ++a) {
    float h[3];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      float s = V.Jpw[6 + j] * V.Jcw[18 + a];
      if (jc_nz(1, a)) s = fmaf(V.Jpw[3 + j], V.Jcw[9 + a], s);
      if (jc_nz(0, a)) s = fmaf(V.Jpw[j], V.Jcw[a], s);
      h[j] = s;
    }
    const float y0 = h[0] * li[0];
    const float y1 = (h[1] - li[1] * y0) * li[3];
    const float y2 = (h[2] - li[2] * y0 - li[4] * y1) * li[5];
    Y[a][0] = y0; Y[a][1] = y1; Y[a][2] = y2;
#pragma unroll
    for (int r = 0; r < 3; ++r) rv[a < 8 ? 8 * r + a : rec_zs<CT>() + r] = Y[a][r];
  }
#pragma unroll
  for (int ch = 0; ch < CT; ++ch) rv[24 + ch] = V.dep[ch];
#pragma unroll
  for (int q = 27 + CT; q < R; ++q) rv[q] = 0.f;
  float4* dst = reinterpret_cast<float4*>(c.rec + e * R);
#pragma unroll
  for (int q = 0; q < R / 4; ++q) dst[q] = make_float4(rv[4 * q], rv[4 * q + 1], rv[4 * q + 2], rv[4 * q + 3]);
}

// Pass "points": per-track Hpp and g_p, and the max |diag(Hpp)|.  Persistent warps walk
// the point tasks with a stride; a short task (<= 32 observations, one per lane) has its
// inputs loaded while the warp still works on the previous one.
template <int CT>
__global__ void __launch_bounds__(128) k_points(Ctx c) {
  const int lane = threadIdx.x & 31;
  const int nw = (int)((gridDim.x * blockDim.x) >> 5);
  int task = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  float wmax = 0.f;
  auto task_in = [&](int t, LocIn<CT>& in) {
    if (t >= c.d.n_pt_tasks) { in.ix = make_int4(0, 0, -1, 0); return; }
    const int kb = c.d.pt_task[t], n = c.d.pt_task[t + 1] - kb;
    load_loc_in<CT>(c, kb + lane, n <= kWarp && lane < n, in);
  };
  LocIn<CT> nxt;
  task_in(task, nxt);
  for (; task < c.d.n_pt_tasks; task += nw) {             // warp-uniform
    const LocIn<CT> cur = nxt;
    task_in(task + nw, nxt);
    const int kb = c.d.pt_task[task], ke = c.d.pt_task[task + 1];
    const int n = ke - kb;
    float v[9];
#pragma unroll
    for (int j = 0; j < 9; ++j) v[j] = 0.f;
    if (n <= kWarp) {
      const bool act = lane < n;
      int tl = -1 - lane;
      if (act) {
        ObsView<CT> V;
        view_loc<CT>(c, kb + lane, cur, V);
        tl = cur.ix.z;
        point_terms<CT>(V, v);
      }
      const int tl_prev = __shfl_up_sync(0xffffffffu, tl, 1);
      const int tl_next = __shfl_down_sync(0xffffffffu, tl, 1);
      const bool head = act && (lane == 0 || tl_prev != tl);
      const bool tail = act && (lane == n - 1 || tl_next != tl);
      const unsigned heads = __ballot_sync(0xffffffffu, head);
      const unsigned below = heads & ((2u << lane) - 1u);
      const int seg_start = act ? 31 - __clz(below) : lane;
#pragma unroll
      for (int j = 0; j < 9; ++j) v[j] = seg_scan(v[j], lane, seg_start);
      if (tail) {
        float* t = c.trec + (int64_t)tl * 24;
#pragma unroll
        for (int j = 0; j < 9; ++j) t[j] = v[j];
        wmax = fmaxf(wmax, fmaxf(v[0], fmaxf(v[3], v[5])));
      }
    } else {                                             // one long track, in rounds
      const int tl = c.d.trk_t[kb];
      for (int k = kb + lane; k < ke; k += kWarp) {
        LocIn<CT> in;
        load_loc_in<CT>(c, k, true, in);
        ObsView<CT> V;
        view_loc<CT>(c, k, in, V);
        float u[9];
        point_terms<CT>(V, u);
#pragma unroll
        for (int j = 0; j < 9; ++j) v[j] += u[j];
      }
#pragma unroll
      for (int j = 0; j < 9; ++j) v[j] = warp_sum(v[j]);
      if (lane == 0) {
        float* t = c.trec + (int64_t)tl * 24;
#pragma unroll
        for (int j = 0; j < 9; ++j) t[j] = v[j];
        wmax = fmaxf(wmax, fmaxf(v[0], fmaxf(v[3], v[5])));
      }
    }
  }
  wmax = warp_max(wmax);
  if (lane == 0) atomic_max_nonneg(c.hpp_max, wmax);
}

// Pass "factor": damped Cholesky factor of every local track (BlockDiagMat.dampen_ then
// chol3x3_solve's guarded factorisation with jitter 1e-12, ba_solver.py:572-582, 589-599).
// The factor is computed in double and rounded once to the reciprocal form (1/l00, l10, l20,
// 1/l11, l21, 1/l22) stored at track-record floats 12..17, so the per-observation elimination
// Y = L^-1 Hpc needs no division; z = L^-1 g_p (floats 18..20) is solved from the same
// rounded factor, so that S (through Y^T Y) and b (through Y^T z) are eliminated with one
// factor: their rounding then stays consistent, which matters on ill-conditioned systems.
__global__ void __launch_bounds__(256) k_factor(Ctx c) {
  const int tl = blockIdx.x * blockDim.x + threadIdx.x;
  const float lam = c.dampen * (c.adaptive ? *c.hpp_max : 1.f);
  if (tl == 0) c.misc[1] = lam;   // point damping, reused by the back-substitution
  if (tl >= c.d.nT_loc) return;
  // the 96-byte track record as 16-byte pieces (the workspace is 256-byte aligned)
  float4* t4 = reinterpret_cast<float4*>(c.trec + (int64_t)tl * 24);
  const float4 a = t4[0], b = t4[1];
  const float g8 = c.trec[(int64_t)tl * 24 + 8];
  const float h00 = a.x + lam, h01 = a.y, h02 = a.z, h11 = a.w + lam, h12 = b.x, h22 = b.y + lam;
  // the factor in double, rounded once; z from the rounded factor (the same one S uses)
  double ld[6];
  chol3<double>((double)h00, (double)h01, (double)h02, (double)h01, (double)h11, (double)h12, (double)h02,
                (double)h12, (double)h22, 1e-12, ld);
  const float r0 = (float)(1.0 / ld[0]), l1 = (float)ld[1], l2 = (float)ld[2], r3 = (float)(1.0 / ld[3]);
  const float l4 = (float)ld[4], r5 = (float)(1.0 / ld[5]);
  const double z0 = (double)b.z * r0;
  const double z1 = ((double)b.w - (double)l1 * z0) * r3;
  const double z2 = ((double)g8 - (double)l2 * z0 - (double)l4 * z1) * r5;
  const float z[3] = {(float)z0, (float)z1, (float)z2};
  t4[3] = make_float4(r0, l1, l2, r3);                        // floats 12..15
  t4[4] = make_float4(l4, r5, z[0], z[1]);                    // floats 16..19
  t4[5] = make_float4(z[2], 0.f, 0.f, 0.f);                   // floats 20..23 (21..23 unused)
}

__device__ __forceinline__ double warp_sum_dbl(double v) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
  return v;
}

// The objective over this rank's observations in images without an active block (they have
// no image-major entry): residuals and Huber errors only.
template <int CT>
__global__ void __launch_bounds__(256) k_rest(Ctx c) {
  __shared__ double red[8];
  float acc = 0.f;
  for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < c.d.n_rest;
       j += (int64_t)gridDim.x * blockDim.x) {
    const int4 ix = __ldg(c.d.rest_idx + j);      // input row, image, track id
    const int64_t o = ix.x, pid = ix.z;
    const Cam cam = load_cam(c.img_rec + (int64_t)ix.y * kImgRec);
    const float X[3] = {__ldg(c.pts3d + 3 * pid), __ldg(c.pts3d + 3 * pid + 1), __ldg(c.pts3d + 3 * pid + 2)};
    float dep[CT], zc[CT];
#pragma unroll
    for (int ch = 0; ch < CT; ++ch) {
      dep[ch] = __ldg(c.pix2d_dep + o * CT + ch);
      zc[ch] = __ldg(c.z_coefs + (int64_t)ix.y * CT + ch);
    }
    const float2 q = __ldg(reinterpret_cast<const float2*>(c.pix2d) + o);
    const float2 sd = __ldg(reinterpret_cast<const float2*>(c.pix2d_std) + o);
    ObsLin L;
    linearize_obs<float, true, false, CT>(cam, X, q.x, q.y, sd.x, sd.y, dep, zc, CT, c.o, L);
    if (c.res_out) {
      const int64_t n = c.d.n_in;
      c.res_out[o] = L.r[0]; c.res_out[n + o] = L.r[1]; c.res_out[2 * n + o] = L.r[2];
    }
    acc += L.err[0] + L.err[1] + L.err[2];
  }
  const double t = warp_sum_dbl((double)acc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = t;
  __syncthreads();
  if (threadIdx.x == 0 && c.loss_part) {
    double u = 0.0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) u += red[w];
    c.loss_part[c.d.n_c1_chunks + blockIdx.x] = u;
  }
}

// The objective's sum of Huber errors from the per-block partial sums, in a fixed order.
__global__ void __launch_bounds__(256) k_loss_sum(const double* __restrict__ part, int n, double* __restrict__ loss) {
  __shared__ double red[8];
  double acc = 0.0;
  for (int j = threadIdx.x; j < n; j += blockDim.x) acc += part[j];
  acc = warp_sum_dbl(acc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < 8; ++w) t += red[w];
    *loss = t;
  }
}

// ------------------------------------------------------------------------------------
// pass "diag": image-major per-observation terms
// ------------------------------------------------------------------------------------
// Unique values accumulated per image chunk (symmetric blocks keep their upper triangle).
template <int CT>
struct DiagLayout {
  static constexpr int FF = 0;                      // (f,f)   3
  static constexpr int FT = 3;                      // (f,t)  12
  static constexpr int FZ = FT + 12;                // (f,z)  2C
  static constexpr int TT = FZ + 2 * CT;            // (t,t)  21
  static constexpr int TZ = TT + 21;                // (t,z)  6C
  static constexpr int ZZ = TZ + 6 * CT;            // (z,z)  C(C+1)/2
  static constexpr int B = ZZ + CT * (CT + 1) / 2;  // b      8+C
  static constexpr int DA = B + 8 + CT;             // diag(Hcc) 8+C
  static constexpr int N = DA + 8 + CT;
  // destination entries written per chunk (full blocks)
  static constexpr int E = 4 + 12 + 2 * CT + 36 + 6 * CT + CT * CT + 2 * (8 + CT);
};

__host__ __device__ constexpr int sym_idx(int a, int b, int n) { return a * n - a * (a - 1) / 2 + (b - a); }

template <int CT>
__device__ __forceinline__ void diag_terms(const Ctx& c, const ObsView<CT>& V, bool elim, int64_t e, float4 tf0,
                                           float4 tf1, float4 tf2, float* __restrict__ out) {
  // value v of this observation goes to out[v] (its lane's row of the warp's transpose
  // buffer), as soon as it is computed
  using Lay = DiagLayout<CT>;
  float H[9][9];
#pragma unroll
  for (int a = 0; a < 9; ++a)
#pragma unroll
    for (int b = a; b < 9; ++b) {
      float s = V.Jcw[18 + a] * V.Jcw[18 + b];
#pragma unroll
      for (int i = 1; i >= 0; --i)
        if (jc_nz(i, a) && jc_nz(i, b)) s = fmaf(V.Jcw[9 * i + a], V.Jcw[9 * i + b], s);
      H[a][b] = s;
    }
  float g[9];
#pragma unroll
  for (int a = 0; a < 9; ++a) {
    float s = V.Jcw[18 + a] * V.sWr[2];
#pragma unroll
    for (int i = 1; i >= 0; --i)
      if (jc_nz(i, a)) s = fmaf(V.Jcw[9 * i + a], V.sWr[i], s);
    g[a] = s;
  }
  // undamped diag(A) = diag(Hcc)
  out[Lay::DA + 0] = H[0][0];
  out[Lay::DA + 1] = H[1][1];
#pragma unroll
  for (int t = 0; t < 6; ++t) out[Lay::DA + 2 + t] = H[2 + t][2 + t];
#pragma unroll
  for (int ch = 0; ch < CT; ++ch) out[Lay::DA + 8 + ch] = H[8][8] * V.dep[ch] * V.dep[ch];
  if (elim) {                                     // eliminated track: record Y, subtract Y^T Y, Y^T z
    const float li[6] = {tf0.x, tf0.y, tf0.z, tf0.w, tf1.x, tf1.y};
    float Y[9][3];
    elim_record<CT>(c, e, V, li, Y);
    const float z0 = tf1.z, z1 = tf1.w, z2 = tf2.x;
#pragma unroll
    for (int a = 0; a < 9; ++a) {
#pragma unroll
      for (int b = a; b < 9; ++b)
        H[a][b] = fmaf(-Y[a][2], Y[b][2], fmaf(-Y[a][1], Y[b][1], fmaf(-Y[a][0], Y[b][0], H[a][b])));
      g[a] = fmaf(-Y[a][2], z2, fmaf(-Y[a][1], z1, fmaf(-Y[a][0], z0, g[a])));
    }
  }
  out[Lay::FF + 0] = H[0][0];
  out[Lay::FF + 1] = H[0][1];
  out[Lay::FF + 2] = H[1][1];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
#pragma unroll
    for (int t = 0; t < 6; ++t) out[Lay::FT + 6 * r + t] = H[r][2 + t];
#pragma unroll
    for (int ch = 0; ch < CT; ++ch) out[Lay::FZ + CT * r + ch] = H[r][8] * V.dep[ch];
  }
#pragma unroll
  for (int a = 0; a < 6; ++a) {
#pragma unroll
    for (int b = a; b < 6; ++b) out[Lay::TT + sym_idx(a, b, 6)] = H[2 + a][2 + b];
#pragma unroll
    for (int ch = 0; ch < CT; ++ch) out[Lay::TZ + CT * a + ch] = H[2 + a][8] * V.dep[ch];
  }
#pragma unroll
  for (int a = 0; a < CT; ++a) {
    const float ha = H[8][8] * V.dep[a];
#pragma unroll
    for (int b = a; b < CT; ++b) out[Lay::ZZ + sym_idx(a, b, CT)] = ha * V.dep[b];
  }
#pragma unroll
  for (int a = 0; a < 8; ++a) out[Lay::B + a] = g[a];
#pragma unroll
  for (int ch = 0; ch < CT; ++ch) out[Lay::B + 8 + ch] = g[8] * V.dep[ch];
}

constexpr int kDiagThreads = 64;   // two warps per image chunk

// Row stride (floats) of a warp's transpose buffer: >= N and 28 mod 32, so that the lanes'
// 16-byte row stores and the 16-byte column-group reads are both free of bank conflicts.
template <int CT> __host__ __device__ constexpr int diag_row_stride() {
  return DiagLayout<CT>::N + ((28 - DiagLayout<CT>::N) % 32 + 32) % 32;
}

// Per-image reduction of the per-observation values: each warp takes 32 observations at a
// time (lane = observation) and writes each observation's N values as one row of its
// transpose buffer; then each lane sums a group of four neighbouring values down the 32
// rows with 16-byte reads and keeps the running sums, so the N values never sit in every
// thread's registers across observations.
template <int CT, bool OBJ>
__global__ void __launch_bounds__(kDiagThreads, 6) k_diag(Ctx c, float* __restrict__ S, float* __restrict__ b,
                                                       float* __restrict__ diagA) {
  using Lay = DiagLayout<CT>;
  constexpr int NW = kDiagThreads / kWarp;
  constexpr int RS = diag_row_stride<CT>();
  constexpr int NG = (Lay::N + 3) / 4;             // groups of four values
  constexpr int NGL = (NG + 31) / 32;              // groups per lane
  extern __shared__ __align__(16) float red_dyn[];   // [NW][32 rows][RS]
  const int chunk = blockIdx.x;
  const int img = c.d.c1_img[chunk];
  const int eb = c.d.c1_chunk[chunk], ee = c.d.c1_chunk[chunk + 1];
  const Cam cam = load_cam(c.img_rec + (int64_t)img * kImgRec);
  float zc[CT];
#pragma unroll
  for (int ch = 0; ch < CT; ++ch) zc[ch] = __ldg(c.z_coefs + (int64_t)img * CT + ch);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float* rw = red_dyn + warp * (32 * RS);
  float4 run[NGL];
#pragma unroll
  for (int j = 0; j < NGL; ++j) run[j] = make_float4(0.f, 0.f, 0.f, 0.f);
  ObsIn<CT> nxt;
  load_obs_in<CT>(c, eb + warp * kWarp + lane, ee, nxt);
  float err_acc = 0.f;
  for (int base = eb + warp * kWarp; base < ee; base += NW * kWarp) {
    const int e = base + lane;
    const ObsIn<CT> cur = nxt;
    if (base + NW * kWarp < ee) load_obs_in<CT>(c, e + NW * kWarp, ee, nxt);   // next batch, warp-uniform
    if (e < ee) {
      ObsView<CT> V;
      float es;
      view_in<CT, OBJ>(c, cur, img, cam, zc, V, es);
      if (OBJ) err_acc += es;
      diag_terms<CT>(c, V, cur.ix.y >= 0, e, cur.tf0, cur.tf1, cur.tf2, rw + lane * RS);
    } else {
      for (int v = 0; v < Lay::N; ++v) rw[lane * RS + v] = 0.f;
    }
    __syncwarp();
#pragma unroll
    for (int j = 0; j < NGL; ++j) {
      const int g = lane + 32 * j;
      if (g < NG) {                 // columns 4g..4g+3 (those >= N are never emitted)
        // packed float2 adds: the same sums, in the same order, in half the instructions
        float2 t01 = make_float2(0.f, 0.f), t23 = make_float2(0.f, 0.f);
#pragma unroll 8
        for (int l = 0; l < 32; ++l) {
          const float4 x = *reinterpret_cast<const float4*>(rw + l * RS + 4 * g);
          t01 = __fadd2_rn(t01, make_float2(x.x, x.y));
          t23 = __fadd2_rn(t23, make_float2(x.z, x.w));
        }
        run[j].x += t01.x; run[j].y += t01.y; run[j].z += t23.x; run[j].w += t23.y;
      }
    }
    __syncwarp();
  }
  // cross-warp sum, then one atomic per destination entry
#pragma unroll
  for (int j = 0; j < NGL; ++j) {
    const int g = lane + 32 * j;
    if (g < NG) *reinterpret_cast<float4*>(rw + 4 * g) = run[j];
  }
  __shared__ double esm[NW];
  if (OBJ && c.loss_part) {                       // the chunk's Huber-error sum (no atomics)
    const double t = warp_sum_dbl((double)err_acc);
    if (lane == 0) esm[warp] = t;
  }
  __syncthreads();
  if (OBJ && c.loss_part && threadIdx.x == 0) {
    double t = 0.0;
#pragma unroll
    for (int w = 0; w < NW; ++w) t += esm[w];
    c.loss_part[chunk] = t;
  }
  const int* dst = c.d.img_dst + 6 * img;
  const int* sc = c.d.img_sc + 3 * img;
  for (int e = threadIdx.x; e < Lay::E; e += kDiagThreads) {
    int v, g = e;
    float* addr = nullptr;
    if (g < 4) {                                           // (f,f)
      const int r = g >> 1, q = g & 1;
      v = Lay::FF + sym_idx(min(r, q), max(r, q), 2);
      if (dst[0] >= 0) addr = S + dst[0] + g;
    } else if ((g -= 4) < 12) {                            // (f,t)
      v = Lay::FT + g;
      if (dst[1] >= 0) addr = S + dst[1] + g;
    } else if ((g -= 12) < 2 * CT) {                       // (f,z)
      v = Lay::FZ + g;
      if (dst[2] >= 0) addr = S + dst[2] + g;
    } else if ((g -= 2 * CT) < 36) {                       // (t,t)
      const int r = g / 6, q = g % 6;
      v = Lay::TT + sym_idx(min(r, q), max(r, q), 6);
      if (dst[3] >= 0) addr = S + dst[3] + g;
    } else if ((g -= 36) < 6 * CT) {                       // (t,z)
      v = Lay::TZ + g;
      if (dst[4] >= 0) addr = S + dst[4] + g;
    } else if ((g -= 6 * CT) < CT * CT) {                  // (z,z)
      const int r = g / CT, q = g % CT;
      v = Lay::ZZ + sym_idx(min(r, q), max(r, q), CT);
      if (dst[5] >= 0) addr = S + dst[5] + g;
    } else if ((g -= CT * CT) < 8 + CT) {                  // b
      v = Lay::B + g;
      const int blk = g < 2 ? 0 : (g < 8 ? 1 : 2), loc = g < 2 ? g : (g < 8 ? g - 2 : g - 8);
      if (sc[blk] >= 0) addr = b + sc[blk] + loc;
    } else {                                               // diag(A)
      g -= 8 + CT;
      v = Lay::DA + g;
      const int blk = g < 2 ? 0 : (g < 8 ? 1 : 2), loc = g < 2 ? g : (g < 8 ? g - 2 : g - 8);
      if (sc[blk] >= 0) addr = diagA + sc[blk] + loc;
    }
    if (addr) {
      float t = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) t += red_dyn[w * (32 * RS) + v];
      atomicAdd(addr, t);
    }
  }
}

// ------------------------------------------------------------------------------------
// pass "pairs": segment-major observation-pair products
// ------------------------------------------------------------------------------------
// A segment (i, i') owns the S blocks between image i's typed blocks (rows) and image
// i''s (columns).  For each of its observation pairs (o in i, o' in i', same track) the
// product P = Y_o^T Y_o' ((8+C) x (8+C) once the depth columns are expanded) is summed.
// One warp per pair task, one observation pair per lane per step.  The warp copies the
// 64 records of a step (32 pairs x 2 sides) into shared memory with coalesced 16-byte
// cp.async (eight lanes per 128-byte record), kPairStages - 1 steps ahead of the step it
// computes; each lane then reads its own pair's records from a padded slot (conflict-free
// 16-byte reads).  Each lane keeps the rows [A0, A1) of the product in registers (all 8+C
// rows for C <= 5; larger C splits the rows over `pair_roles` warps that each stream the
// task); the lane partials are summed through shared memory at the end of the task, one
// atomic per value.
constexpr int kPairStages = 3;   // cp.async ring depth per lane

// 16-byte asynchronous global -> shared copies (cp.async, completion by commit groups)
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(sa), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// Add -v to S at output (row a, column bcol) of segment s's pair product.
template <int CT>
__device__ __forceinline__ void emit_pair_value(const Ctx& c, float* __restrict__ S, int s, int a, int bcol, float v) {
  const int ta = a < 2 ? 0 : (a < 8 ? 1 : 2), ra = a < 2 ? a : (a < 8 ? a - 2 : a - 8);
  const int tb = bcol < 2 ? 0 : (bcol < 8 ? 1 : 2), cb = bcol < 2 ? bcol : (bcol < 8 ? bcol - 2 : bcol - 8);
  const int bsa = ta == 0 ? 2 : (ta == 1 ? 6 : CT), bsb = tb == 0 ? 2 : (tb == 1 ? 6 : CT);
  const int sb = 3 * ta + tb;
  const int mode = (c.d.seg_mode[s] >> (2 * sb)) & 3;
  if (mode == kModeNone) return;
  float* base = S + c.d.seg_dst[9 * (int64_t)s + sb];
  if (mode == kModeDirect) {
    atomicAdd(base + ra * bsb + cb, -v);
  } else if (mode == kModeTrans) {
    atomicAdd(base + cb * bsa + ra, -v);
  } else {
    atomicAdd(base + ra * bsb + cb, -v);
    atomicAdd(base + cb * bsb + ra, -v);
  }
}

// Warps that split the 8+C product rows of a pair task (at most ~100 accumulators per
// lane), all of them reading the same staged records.
#ifndef B3R_PAIR_ACC_MAX
#define B3R_PAIR_ACC_MAX 170   // accumulators per lane that set the number of row roles
#endif
template <int CT> __host__ __device__ constexpr int pair_roles() {
  return ((8 + CT) * (8 + CT) + B3R_PAIR_ACC_MAX - 1) / B3R_PAIR_ACC_MAX;
}
// Issue cost of product row a per pair: a base row ~18 instructions, a depth row ~8, plus
// ~15 for the z-scale products shared by the depth rows (charged to the first of them).
__host__ __device__ constexpr int pair_row_cost(int a) { return a < 8 ? 18 : (a == 8 ? 23 : 8); }
// First row of role r: the rows are cut where the cumulative cost crosses r/NR of the total.
template <int CT, int NR, int r> __host__ __device__ constexpr int role_row() {
  constexpr int W = 8 + CT;
  if (r <= 0) return 0;
  if (r >= NR) return W;
  int total = 0;
  for (int a = 0; a < W; ++a) total += pair_row_cost(a);
  const int target = r * total / NR;
  int cum = 0, best = 1;
  for (int a = 1; a <= W; ++a) {
    const int prev = cum;
    cum += pair_row_cost(a - 1);
    if (cum >= target) { best = (cum - target <= target - prev) ? a : a - 1; break; }
  }
  best = best < r ? r : best;                       // every role keeps at least one row
  return best > W - (NR - r) ? W - (NR - r) : best;
}
template <int CT, int NR, int r> __host__ __device__ constexpr int role_rows_max() {
  if constexpr (r >= NR) {
    return 0;
  } else {
    constexpr int n = role_row<CT, NR, r + 1>() - role_row<CT, NR, r>();
    constexpr int m = role_rows_max<CT, NR, r + 1>();
    return n > m ? n : m;
  }
}
template <int CT> __host__ __device__ constexpr int pair_slot_floats() { return 2 * rec_floats<CT>() + 4; }
// shared memory of a pair CTA: kPairStages step buffers (reused by the per-warp epilogue
// transposes), then 64 staged record indices per warp
template <int CT> __host__ __device__ constexpr int pair_stage_area() {
  constexpr int NR = pair_roles<CT>();
  constexpr int st = kPairStages * 32 * pair_slot_floats<CT>();
  constexpr int ep = NR * role_rows_max<CT, NR, 0>() * (8 + CT) * 33;
  return ((st > ep ? st : ep) + 3) & ~3;
}
template <int CT> __host__ __device__ constexpr int pair_smem_floats() {
  return pair_stage_area<CT>() + 64 * pair_roles<CT>();
}

// Rows [A0, A1) (role `role` of NR) of one pair task.  `stg` is the CTA's step buffers,
// `sidx` this warp's 64 staged record indices.  The products are accumulated with packed
// float2 FMAs (two neighbouring columns per instruction): row a < 8 of Y_o^T Y_o' is
// sum_r Y_o[r][a] * Y_o'[r][0..7] plus the depth columns u_a * dep', u_a = sum_r
// Y_o[r][a] zs'[r]; a depth row is dep[ch] * (zs^T Y_o') plus dep[ch] * (zs^T zs') * dep'.
template <int CT, int A0, int A1, int NR>
__device__ __forceinline__ void pair_task(const Ctx& c, float* __restrict__ S, int64_t task, float* stg, int* sidx,
                                          int role) {
  constexpr int R = rec_floats<CT>(), SLOT = pair_slot_floats<CT>(), Q = R / 4, ZS = rec_zs<CT>();
  constexpr int W = 8 + CT, NA = A1 - A0;
  constexpr int NZ2 = CT / 2, ODD = CT & 1, NC2 = 4 + NZ2;   // float2 columns per row
  constexpr int B0 = A0 < 8 ? A0 : 8, B1 = A1 < 8 ? A1 : 8;  // base rows of this role
  constexpr int Z0 = A0 > 8 ? A0 - 8 : 0, Z1 = A1 > 8 ? A1 - 8 : 0;   // depth rows
  constexpr int STAGE = 32 * SLOT;
  const int lane = threadIdx.x & 31;
  const int s = c.d.task_seg[task];
  const int64_t pb = c.d.task_pb[task], pe = c.d.task_pe[task];
  const int nit = (int)((pe - pb + 31) >> 5);
  const int2* __restrict__ pairs = reinterpret_cast<const int2*>(c.d.pairs);
  // Idle lanes of the last step repeat the task's last pair (a line the step copies anyway:
  // no shared hot spot); steps past the end copy nothing.
  auto load_kk = [&](int j) -> int2 {
    const int64_t p = pb + lane + 32 * (int64_t)j;
    return j < nit ? __ldg(pairs + (p < pe ? p : pe - 1)) : make_int2(0, 0);
  };
  // Copy this role's share of the records of step j (pair indices kk, one pair per lane):
  // piece g = lane + 32 m of the step is part g % Q of record g / Q (record 2 q + side is
  // side `side` of pair q), so consecutive lanes read consecutive 16 bytes of a record;
  // role w copies the piece rounds m in [M0, M1).
  auto stage = [&](int j, int2 kk) {
    __syncwarp();                        // this warp is done with its previous indices
    reinterpret_cast<int2*>(sidx)[lane] = kk;
    __syncwarp();
    float* dst = stg + (j % kPairStages) * STAGE;
    const int M0 = role * 2 * Q / NR, M1 = (role + 1) * 2 * Q / NR;
    if (j >= nit) {
      // nothing to copy
    } else if constexpr (32 % Q == 0 && Q <= 16) {
      // lane-constant part and record parity; the record advances by 32/Q per piece round
      constexpr int RPM = 32 / Q;
      const int r0 = lane / Q, part = lane % Q;
      float* d0 = dst + (r0 >> 1) * SLOT + (r0 & 1) * R + 4 * part;
      const float* s0 = c.rec + 4 * part;
#pragma unroll 4
      for (int m = M0; m < M1; ++m) cp_async16(d0 + (RPM / 2) * m * SLOT, s0 + (int64_t)sidx[r0 + RPM * m] * R);
    } else {
#pragma unroll 4
      for (int m = M0; m < M1; ++m) {
        const int g = lane + 32 * m;
        const int r = g / Q, part = g - r * Q;
        cp_async16(dst + (r >> 1) * SLOT + (r & 1) * R + 4 * part, c.rec + (int64_t)sidx[r] * R + 4 * part);
      }
    }
    cp_async_commit();   // one group per step, empty past the end: uniform group counting
  };
  float2 acc[NA][NC2];
  float acco[NA];
#pragma unroll
  for (int a = 0; a < NA; ++a) {
#pragma unroll
    for (int q = 0; q < NC2; ++q) acc[a][q] = make_float2(0.f, 0.f);
    acco[a] = 0.f;
  }
  stage(0, load_kk(0));
  stage(1, load_kk(1));
  int2 kk_next = load_kk(2);
  for (int j = 0; j < nit; ++j) {
    cp_async_wait<kPairStages - 2>();     // this thread's copies of step j have landed
    // every role's copies of step j are visible, and every role is done with step j-1,
    // whose buffer step j+2 reuses
    if constexpr (NR > 1) __syncthreads(); else __syncwarp();
    stage(j + 2, kk_next);
    kk_next = load_kk(j + 3);
    if (pb + lane + 32 * (int64_t)j < pe) {
      const float* buf = stg + (j % kPairStages) * STAGE + lane * SLOT;
      // column record through 16-byte reads, split into register pairs
      float cv[R];
#pragma unroll
      for (int q = 0; q < Q; ++q) {
        const float4 v = *reinterpret_cast<const float4*>(buf + R + 4 * q);
        cv[4 * q] = v.x; cv[4 * q + 1] = v.y; cv[4 * q + 2] = v.z; cv[4 * q + 3] = v.w;
      }
      float2 yc[3][4];                    // Y'[r][2q .. 2q+1]
#pragma unroll
      for (int r = 0; r < 3; ++r)
#pragma unroll
        for (int q = 0; q < 4; ++q) yc[r][q] = make_float2(cv[8 * r + 2 * q], cv[8 * r + 2 * q + 1]);
      float2 dc[NZ2 > 0 ? NZ2 : 1];       // column depth channels, paired
#pragma unroll
      for (int q = 0; q < NZ2; ++q) dc[q] = make_float2(cv[24 + 2 * q], cv[24 + 2 * q + 1]);
      const float dco = ODD ? cv[24 + CT - 1] : 0.f;
      const float zc0 = cv[ZS], zc1 = cv[ZS + 1], zc2 = cv[ZS + 2];
      if constexpr (Z1 > 0) {             // depth rows: dep[ch] * (zs^T Y'), dep[ch] * sz * dep'
        float rv[8];                      // row record floats 24..31: depth channels, z-scale column
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const float4 v = *reinterpret_cast<const float4*>(buf + 24 + 4 * q);
          rv[4 * q] = v.x; rv[4 * q + 1] = v.y; rv[4 * q + 2] = v.z; rv[4 * q + 3] = v.w;
        }
        const float zr0 = ZS + 2 < 32 ? rv[(ZS - 24) & 7] : buf[ZS];
        const float zr1 = ZS + 2 < 32 ? rv[(ZS + 1 - 24) & 7] : buf[ZS + 1];
        const float zr2 = ZS + 2 < 32 ? rv[(ZS + 2 - 24) & 7] : buf[ZS + 2];
        float2 qz[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          qz[q] = __fmul2_rn(make_float2(zr0, zr0), yc[0][q]);
          qz[q] = __ffma2_rn(make_float2(zr1, zr1), yc[1][q], qz[q]);
          qz[q] = __ffma2_rn(make_float2(zr2, zr2), yc[2][q], qz[q]);
        }
        const float sz = fmaf(zr2, zc2, fmaf(zr1, zc1, zr0 * zc0));
#pragma unroll
        for (int z = Z0; z < Z1; ++z) {
          const int a = 8 + z - A0;
          const float dr = 24 + z < 32 ? rv[z & 7] : buf[24 + z];
          const float2 d2 = make_float2(dr, dr);
#pragma unroll
          for (int q = 0; q < 4; ++q) acc[a][q] = __ffma2_rn(d2, qz[q], acc[a][q]);
          const float ds = dr * sz;
          const float2 s2 = make_float2(ds, ds);
#pragma unroll
          for (int q = 0; q < NZ2; ++q) acc[a][4 + q] = __ffma2_rn(s2, dc[q], acc[a][4 + q]);
          if (ODD) acco[a] = fmaf(ds, dco, acco[a]);
        }
      }
#pragma unroll
      for (int b = B0; b < B1; ++b) {      // base rows, their record values read four rows at a time
        const int a = b - A0;
        const float4 g0 = *reinterpret_cast<const float4*>(buf + (b & ~3));
        const float4 g1 = *reinterpret_cast<const float4*>(buf + 8 + (b & ~3));
        const float4 g2 = *reinterpret_cast<const float4*>(buf + 16 + (b & ~3));
        const int l = b & 3;
        const float t0 = l == 0 ? g0.x : (l == 1 ? g0.y : (l == 2 ? g0.z : g0.w));
        const float t1 = l == 0 ? g1.x : (l == 1 ? g1.y : (l == 2 ? g1.z : g1.w));
        const float t2 = l == 0 ? g2.x : (l == 1 ? g2.y : (l == 2 ? g2.z : g2.w));
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          acc[a][q] = __ffma2_rn(make_float2(t0, t0), yc[0][q], acc[a][q]);
          acc[a][q] = __ffma2_rn(make_float2(t1, t1), yc[1][q], acc[a][q]);
          acc[a][q] = __ffma2_rn(make_float2(t2, t2), yc[2][q], acc[a][q]);
        }
        const float u = fmaf(t2, zc2, fmaf(t1, zc1, t0 * zc0));
        const float2 u2 = make_float2(u, u);
#pragma unroll
        for (int q = 0; q < NZ2; ++q) acc[a][4 + q] = __ffma2_rn(u2, dc[q], acc[a][4 + q]);
        if (ODD) acco[a] = fmaf(u, dco, acco[a]);
      }
    }
  }
  cp_async_wait<0>();
  if constexpr (NR > 1) __syncthreads(); else __syncwarp();   // step buffers free for the epilogue
  // epilogue: transpose the lane partials through this role's part of the step buffers
  // (stride 33: conflict-free), then each lane sums values lane, lane+32, ... over the 32
  // lanes and emits them
  float* sm = stg + role * (role_rows_max<CT, NR, 0>() * W * 33);
#pragma unroll
  for (int a = 0; a < NA; ++a) {
#pragma unroll
    for (int q = 0; q < NC2; ++q) {
      sm[(a * W + 2 * q) * 33 + lane] = acc[a][q].x;
      if (2 * q + 1 < W) sm[(a * W + 2 * q + 1) * 33 + lane] = acc[a][q].y;
    }
    if (ODD) sm[(a * W + W - 1) * 33 + lane] = acco[a];
  }
  __syncwarp();
  for (int v = lane; v < NA * W; v += 32) {
    float t = 0.f;
#pragma unroll 8
    for (int j = 0; j < 32; ++j) t += sm[v * 33 + j];
    emit_pair_value<CT>(c, S, s, A0 + v / W, v % W, t);
  }
}


template <int CT, int NR, int r>
__device__ __forceinline__ void pair_role_dispatch(const Ctx& c, float* S, int64_t task, int role, float* stg,
                                                   int* sidx) {
  if constexpr (r < NR) {
    if (role == r) pair_task<CT, role_row<CT, NR, r>(), role_row<CT, NR, r + 1>(), NR>(c, S, task, stg, sidx, role);
    else pair_role_dispatch<CT, NR, r + 1>(c, S, task, role, stg, sidx);
  }
}

// One CTA per pair task (tasks longest first), one warp per row role.
template <int CT>
__global__ void __launch_bounds__(pair_roles<CT>() * 32) k_pairs(Ctx c, float* __restrict__ S) {
  extern __shared__ __align__(16) float sm_dyn[];
  const int role = threadIdx.x >> 5;
  int* sidx = reinterpret_cast<int*>(sm_dyn + pair_stage_area<CT>()) + 64 * role;
  pair_role_dispatch<CT, pair_roles<CT>(), 0>(c, S, (int64_t)blockIdx.x, role, sm_dyn, sidx);
}

// ------------------------------------------------------------------------------------
// depth-stitch plans: only the depth-coefficient (zcf) blocks take part in S
// ------------------------------------------------------------------------------------
// With the focal and pose types switched off (the reference's second BA phase, optim_K =
// optim_P = False, whose blocks become decoupled ZerosMat diagonals, ba_solver.py:508-517),
// the camera side of an observation is its image's zcf block, whose Jacobian is zs * dep in
// the depth row only (sfm_jacobian_rigs.cu:494-501).  So Hpc = h dep^T with the 3-vector
// h = zw * Jpw[2][:] (zw = sqrt(W_z) zs), the elimination record is y = L^-1 h plus the
// observation's depth channels, and every Schur term is a scalar times an outer product of
// depth vectors:
//   image block      (zw^2 - y.y) dep dep^T
//   gradient         (zw sqrt(W_z) r_z - y.z) dep          (z = L^-1 g_p)
//   diag(A)          zw^2 dep_c^2
//   pair product     (y_o . y_o') dep_o dep_o'^T
// These are the general passes' values with the focal and pose columns left out (the same
// per-observation arithmetic, in the same order).  Record: [0, 3) y, [3, 3+C) the depth
// channels, padded to a multiple of four floats (32 bytes for C = 5).
constexpr int kZonlyMaxC = 8;        // C*C accumulators per lane in the pair pass
template <int CT> __host__ __device__ constexpr int zrec_floats() { return (3 + CT + 3) & ~3; }

// Sum of v[0 .. 32 NG) over the warp, scattered: afterwards lane l holds in v[g] the total
// of value 32 g + l (a recursive-halving butterfly: 31 shuffles per group of 32 values).
template <int NG>
__device__ __forceinline__ void warp_reduce_scatter(float (&v)[32 * NG], int lane) {
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    float* w = v + 32 * g;
#pragma unroll
    for (int d = 16; d >= 1; d >>= 1) {
      const bool up = lane & d;
#pragma unroll
      for (int i = 0; i < d; ++i) {
        const float send = up ? w[i] : w[i + d];
        const float keep = up ? w[i + d] : w[i];
        w[i] = keep + __shfl_xor_sync(0xffffffffu, send, d);
      }
    }
    v[g] = w[0];
  }
}

constexpr int kDiagZThreads = 128;

// Image-major pass of a depth-stitch plan: one CTA per <= 1024-observation chunk of one
// image, thread per observation (the next batch's inputs loaded ahead); the image's zcf
// block, gradient and diag(A) summed per thread, then over the CTA, one atomic per value.
template <int CT, bool OBJ>
__global__ void __launch_bounds__(kDiagZThreads) k_diag_z(Ctx c, float* __restrict__ S, float* __restrict__ b,
                                                         float* __restrict__ diagA) {
  constexpr int NZZ = CT * (CT + 1) / 2, NV = NZZ + 2 * CT, R = zrec_floats<CT>();
  constexpr int NW = kDiagZThreads / 32;
  __shared__ float red[NW][NV];
  const int chunk = blockIdx.x;
  const int img = c.d.c1_img[chunk];
  const int eb = c.d.c1_chunk[chunk], ee = c.d.c1_chunk[chunk + 1];
  const Cam cam = load_cam(c.img_rec + (int64_t)img * kImgRec);
  float zc[CT];
#pragma unroll
  for (int ch = 0; ch < CT; ++ch) zc[ch] = __ldg(c.z_coefs + (int64_t)img * CT + ch);
  float acc[NV];
#pragma unroll
  for (int v = 0; v < NV; ++v) acc[v] = 0.f;
  float err_acc = 0.f;
  ObsIn<CT> nxt;
  load_obs_in<CT>(c, eb + threadIdx.x, ee, nxt);
  for (int base = eb; base < ee; base += kDiagZThreads) {
    const int e = base + threadIdx.x;
    const ObsIn<CT> cur = nxt;
    if (base + kDiagZThreads < ee) load_obs_in<CT>(c, e + kDiagZThreads, ee, nxt);   // CTA-uniform
    if (e >= ee) continue;
    ObsView<CT> V;
    float es;
    view_in<CT, OBJ>(c, cur, img, cam, zc, V, es);
    if (OBJ) err_acc += es;
    const float zw = V.Jcw[26];
    const float d = zw * zw;
    float a = d, g = zw * V.sWr[2];
    if (cur.ix.y >= 0) {                          // eliminated track: record y, subtract y.y, y.z
      const float h0 = V.Jpw[6] * zw, h1 = V.Jpw[7] * zw, h2 = V.Jpw[8] * zw;
      const float y0 = h0 * cur.tf0.x;
      const float y1 = (h1 - cur.tf0.y * y0) * cur.tf0.w;
      const float y2 = (h2 - cur.tf0.z * y0 - cur.tf1.x * y1) * cur.tf1.y;
      a = fmaf(-y2, y2, fmaf(-y1, y1, fmaf(-y0, y0, a)));
      g = fmaf(-y2, cur.tf2.x, fmaf(-y1, cur.tf1.w, fmaf(-y0, cur.tf1.z, g)));
      float rv[R];
      rv[0] = y0; rv[1] = y1; rv[2] = y2;
#pragma unroll
      for (int ch = 0; ch < CT; ++ch) rv[3 + ch] = V.dep[ch];
#pragma unroll
      for (int q = 3 + CT; q < R; ++q) rv[q] = 0.f;
      float4* dst = reinterpret_cast<float4*>(c.rec + (int64_t)e * R);
#pragma unroll
      for (int q = 0; q < R / 4; ++q) dst[q] = make_float4(rv[4 * q], rv[4 * q + 1], rv[4 * q + 2], rv[4 * q + 3]);
    }
#pragma unroll
    for (int i = 0; i < CT; ++i) {
      const float ai = a * V.dep[i];
#pragma unroll
      for (int j = i; j < CT; ++j) acc[sym_idx(i, j, CT)] += ai * V.dep[j];
      acc[NZZ + i] += g * V.dep[i];
      acc[NZZ + CT + i] += d * V.dep[i] * V.dep[i];
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const float t = warp_sum(acc[v]);
    if (lane == 0) red[warp][v] = t;
  }
  __shared__ double esm[NW];
  if (OBJ && c.loss_part) {                       // the chunk's Huber-error sum (no atomics)
    const double t = warp_sum_dbl((double)err_acc);
    if (lane == 0) esm[warp] = t;
  }
  __syncthreads();
  if (OBJ && c.loss_part && threadIdx.x == 0) {
    double t = 0.0;
#pragma unroll
    for (int w = 0; w < NW; ++w) t += esm[w];
    c.loss_part[chunk] = t;
  }
  const int dzz = c.d.img_dst[6 * img + 5], sz = c.d.img_sc[3 * img + 2];
  for (int e = threadIdx.x; e < CT * CT + 2 * CT; e += kDiagZThreads) {
    int v;
    float* addr;
    if (e < CT * CT) {                            // the image's (z,z) block, stored in full
      const int r = e / CT, q = e % CT;
      v = sym_idx(min(r, q), max(r, q), CT);
      addr = dzz >= 0 ? S + dzz + e : nullptr;
    } else if (e < CT * CT + CT) {
      v = NZZ + (e - CT * CT);
      addr = sz >= 0 ? b + sz + (e - CT * CT) : nullptr;
    } else {
      v = NZZ + CT + (e - CT * CT - CT);
      addr = sz >= 0 ? diagA + sz + (e - CT * CT - CT) : nullptr;
    }
    if (addr) {
      float t = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) t += red[w][v];
      atomicAdd(addr, t);
    }
  }
}

constexpr int kPairZThreads = 128;   // four pair tasks per CTA, one warp each

// Pair pass of a depth-stitch plan: warp per pair task, lane per observation pair, the
// C x C block of the segment's (z,z) sub-block summed per lane, reduce-scattered over the
// warp, one atomic per value per task.
template <int CT>
__global__ void __launch_bounds__(kPairZThreads) k_pairs_z(Ctx c, float* __restrict__ S) {
  constexpr int R = zrec_floats<CT>(), Q = R / 4, NG = (CT * CT + 31) / 32;
  const int lane = threadIdx.x & 31;
  const int64_t task = (int64_t)blockIdx.x * (kPairZThreads / 32) + (threadIdx.x >> 5);
  if (task >= c.d.n_tasks) return;                  // warp-uniform; no CTA barrier below
  const int s = c.d.task_seg[task];
  const int mode = (c.d.seg_mode[s] >> 16) & 3;     // sub-block (z,z) = 3 * 2 + 2
  if (mode == kModeNone) return;
  const int64_t pb = c.d.task_pb[task], pe = c.d.task_pe[task];
  const int2* __restrict__ pairs = c.d.pairs;
  const float4* __restrict__ rec4 = reinterpret_cast<const float4*>(c.rec);
  float acc[32 * NG];
#pragma unroll
  for (int v = 0; v < 32 * NG; ++v) acc[v] = 0.f;
  for (int64_t p = pb + lane; p < pe; p += 32) {
    const int2 kk = __ldg(pairs + p);
    float rv[R], cv[R];
#pragma unroll
    for (int q = 0; q < Q; ++q) {
      const float4 u = __ldg(rec4 + (int64_t)kk.x * Q + q), w = __ldg(rec4 + (int64_t)kk.y * Q + q);
      rv[4 * q] = u.x; rv[4 * q + 1] = u.y; rv[4 * q + 2] = u.z; rv[4 * q + 3] = u.w;
      cv[4 * q] = w.x; cv[4 * q + 1] = w.y; cv[4 * q + 2] = w.z; cv[4 * q + 3] = w.w;
    }
    const float sy = fmaf(rv[2], cv[2], fmaf(rv[1], cv[1], rv[0] * cv[0]));
#pragma unroll
    for (int i = 0; i < CT; ++i) {
      const float t = sy * rv[3 + i];
#pragma unroll
      for (int j = 0; j < CT; ++j) acc[CT * i + j] = fmaf(t, cv[3 + j], acc[CT * i + j]);
    }
  }
  warp_reduce_scatter<NG>(acc, lane);
  float* base = S + c.d.seg_dst[9 * (int64_t)s + 8];
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    const int v = 32 * g + lane;
    if (v >= CT * CT) continue;
    const int i = v / CT, j = v % CT;
    if (mode == kModeDirect) {
      atomicAdd(base + i * CT + j, -acc[g]);
    } else if (mode == kModeTrans) {
      atomicAdd(base + j * CT + i, -acc[g]);
    } else {
      atomicAdd(base + i * CT + j, -acc[g]);
      atomicAdd(base + j * CT + i, -acc[g]);
    }
  }
}

// ------------------------------------------------------------------------------------
// finalize: per-type adaptive damping and the Jacobi preconditioner
// ------------------------------------------------------------------------------------
__device__ __forceinline__ int scalar_type(const DevPlan& d, int j) { return j < d.off_P ? 0 : (j < d.off_Z ? 1 : 2); }

__global__ void k_fin_max(Ctx c, const float* __restrict__ diagA) {
  float m[3] = {0.f, 0.f, 0.f};
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < c.d.n_cam_params; j += gridDim.x * blockDim.x)
    m[scalar_type(c.d, j)] = fmaxf(m[scalar_type(c.d, j)], fabsf(diagA[j]));
#pragma unroll
  for (int t = 0; t < 3; ++t) {
    const float w = warp_max(m[t]);
    if ((threadIdx.x & 31) == 0) atomic_max_nonneg(c.misc + 4 + t, w);
  }
}

__global__ void k_fin_apply(Ctx c, const float* __restrict__ diagA, float* __restrict__ S, float* __restrict__ precond) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= c.d.n_cam_params) return;
  const int t = scalar_type(c.d, j);
  // a switched-off zcf type that received a dense prior is damped like a block diagonal
  const int zero = t == 0 ? c.d.zeroK : (t == 1 ? c.d.zeroP : (c.d.zeroZ && c.misc[8] == 0.f));
  // BlockDiagMat.dampen_ scales by max |diag| of the type; ZerosMat.dampen_ uses 1e-12*I
  const float lam = zero ? c.dampen : c.dampen * (c.adaptive ? c.misc[4 + t] : 1.f);
  S[c.d.sdiag_pos[j]] += lam;
  if (precond) precond[j] = fmaxf(diagA[j] + lam, 1e-12f);
}

// ------------------------------------------------------------------------------------
// y = S x from the upper block triangle
// ------------------------------------------------------------------------------------
template <typename T>
__global__ void k_spmv(DevPlan d, const float* __restrict__ S, const T* __restrict__ x, T* __restrict__ y) {
  const int64_t blk = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (blk >= d.nnzb) return;
  const int lane = threadIdx.x & 31;
  const int p = d.blk_row[blk], q = d.col_idx[blk];
  const int bp = d.bsize[p], bq = d.bsize[q], op = d.boff[p], oq = d.boff[q];
  const float* A = S + d.val_off[blk];
  // rows: y_p += A x_q
  for (int r = lane; r < bp; r += 32) {
    T s = 0;
    for (int cc = 0; cc < bq; ++cc) s += (T)A[r * bq + cc] * x[oq + cc];
    atomicAdd(y + op + r, s);
  }
  if (p == q) return;
  // columns: y_q += A^T x_p
  for (int cc = lane; cc < bq; cc += 32) {
    T s = 0;
    for (int r = 0; r < bp; ++r) s += (T)A[r * bq + cc] * x[op + r];
    atomicAdd(y + oq + cc, s);
  }
}

// ------------------------------------------------------------------------------------
// point back-substitution: delta_p = D^-1 (g_p - C delta_c) (ba_solver.py:203)
// ------------------------------------------------------------------------------------
// Each track's Hpp, g_p and C delta_c are re-accumulated in double from the observations
// (the same float32 per-observation Jacobians as the linearization), then solved with the
// damped guarded Cholesky.  Weakly triangulated points (short baselines) make Hpp badly
// conditioned, so the solve is done in double rather than from the float32 factors.
__device__ __forceinline__ double seg_scan_d(double v, int lane, int seg_start) {
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    double u = __shfl_up_sync(0xffffffffu, v, d);
    if (lane - d >= seg_start) v += u;
  }
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
  return v;
}

template <int CT>
__device__ __forceinline__ void backsub_terms(const Ctx& c, int64_t k, const float* __restrict__ dc, double u[12],
                                              int& tl) {
  ObsView<CT> V;
  view_local<CT>(c, k, V, tl);
  const int* sc = c.d.img_sc + 3 * __ldg(c.d.t_idx + k).x;
  double v[9];
#pragma unroll
  for (int a = 0; a < 2; ++a) v[a] = sc[0] >= 0 ? (double)dc[sc[0] + a] : 0.0;
#pragma unroll
  for (int a = 0; a < 6; ++a) v[2 + a] = sc[1] >= 0 ? (double)dc[sc[1] + a] : 0.0;
  double zz = 0.0;
  if (sc[2] >= 0) {
#pragma unroll
    for (int ch = 0; ch < CT; ++ch) zz += (double)V.dep[ch] * (double)dc[sc[2] + ch];
  }
  v[8] = zz;
  double Jv[3];
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    double s = 0.0;
#pragma unroll
    for (int a = 0; a < 9; ++a) s += (double)V.Jcw[9 * i + a] * v[a];
    Jv[i] = s;
  }
  const int ia[6] = {0, 0, 0, 1, 1, 2}, ib[6] = {0, 1, 2, 1, 2, 2};
#pragma unroll
  for (int e = 0; e < 6; ++e) {
    double s = 0.0;
#pragma unroll
    for (int i = 0; i < 3; ++i) s += (double)V.Jpw[3 * i + ia[e]] * (double)V.Jpw[3 * i + ib[e]];
    u[e] = s;
  }
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    double g = 0.0, cdv = 0.0;
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      g += (double)V.Jpw[3 * i + j] * (double)V.sWr[i];
      cdv += (double)V.Jpw[3 * i + j] * Jv[i];
    }
    u[6 + j] = g - cdv;
  }
  u[9] = u[10] = u[11] = 0.0;
}

__device__ __forceinline__ void backsub_solve(const Ctx& c, double lam, int tl, const double u[12], float* dp) {
  double l[6], z[3], x[3];
  chol3<double>(u[0] + lam, u[1], u[2], u[1], u[3] + lam, u[4], u[2], u[4], u[5] + lam, 1e-12, l);
  const double rhs[3] = {u[6], u[7], u[8]};
  chol3_fwd<double>(l, rhs, z);
  chol3_bwd<double>(l, z, x);
  const int64_t col = c.d.trk_col[tl];
  dp[3 * col] = (float)x[0]; dp[3 * col + 1] = (float)x[1]; dp[3 * col + 2] = (float)x[2];
}

template <int CT>
__global__ void __launch_bounds__(128) k_backsub(Ctx c, const float* __restrict__ dc, float* __restrict__ dp) {
  const int task = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (task >= c.d.n_pt_tasks) return;
  const int kb = c.d.pt_task[task], ke = c.d.pt_task[task + 1];
  const int n = ke - kb;
  const double lam = (double)c.misc[1];
  double u[12];
#pragma unroll
  for (int j = 0; j < 12; ++j) u[j] = 0.0;
  if (n <= kWarp) {
    const bool act = lane < n;
    int tl = -1 - lane;
    if (act) backsub_terms<CT>(c, kb + lane, dc, u, tl);
    const int tl_prev = __shfl_up_sync(0xffffffffu, tl, 1);
    const int tl_next = __shfl_down_sync(0xffffffffu, tl, 1);
    const bool head = act && (lane == 0 || tl_prev != tl);
    const bool tail = act && (lane == n - 1 || tl_next != tl);
    const unsigned heads = __ballot_sync(0xffffffffu, head);
    const int seg_start = act ? 31 - __clz(heads & ((2u << lane) - 1u)) : lane;
#pragma unroll
    for (int j = 0; j < 9; ++j) u[j] = seg_scan_d(u[j], lane, seg_start);
    if (tail) backsub_solve(c, lam, tl, u, dp);
  } else {
    const int tl = c.d.trk_t[kb];
    for (int k = kb + lane; k < ke; k += kWarp) {
      double w[12];
      int tl_k;
      backsub_terms<CT>(c, k, dc, w, tl_k);
#pragma unroll
      for (int j = 0; j < 9; ++j) u[j] += w[j];
    }
#pragma unroll
    for (int j = 0; j < 9; ++j) u[j] = warp_sum_d(u[j]);
    if (lane == 0) backsub_solve(c, lam, tl, u, dp);
  }
}

// ------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------
// Depth-channel counts with compiled kernels (the reference's multi-depth maps carry up
// to 17 channels, scripts/xps/*.sh "-nz 1 17").
#define B3R_FOR_EACH_C(X) X(1) X(2) X(3) X(4) X(5) X(6) X(7) X(8) X(17)

int check_device(const b3r_plan* plan) {
  int dev = -1;
  B3R_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  B3R_REQUIRE(dev == plan->device, "current device %d differs from the plan's device %d", dev, plan->device);
  return B3R_OK;
}

int make_ctx(b3r_plan* plan, const b3r_params* p, const b3r_lin_opts* o, void* ws, Ctx& c) {
  B3R_REQUIRE(plan && o && ws, "NULL plan/options/workspace");
  B3R_REQUIRE(((uintptr_t)ws & 255) == 0, "workspace must be 256-byte aligned");
  std::memset(&c, 0, sizeof(c));
  c.d = plan->d;
  c.o.is_depth_log = o->is_depth_log;
  c.o.weight_z = o->weight_z; c.o.pnorm = o->pnorm; c.o.max_pix_err = o->max_pix_err;
  c.o.huber_delta = o->huber_delta; c.o.w_pts_nul = o->w_pts_nul;
  c.o.clamp_lo = o->clamp_w_lo; c.o.clamp_hi = o->clamp_w_hi;
  finish_lin_opts(c.o);
  B3R_REQUIRE(o->pnorm > 0.f && o->pnorm <= 2.f, "pnorm must be in ]0, 2] for a linearization");
  c.no_grad_f_from_rz = o->no_grad_f_from_rz;
  c.optim_Z0 = o->optim_Z0;
  c.optim_Z_1st_cam = o->optim_Z_1st_cam;
  c.dampen = (float)o->dampen;
  c.adaptive = o->adaptive_dampen;
  char* w = (char*)ws;
  c.img_rec = (float*)(w + plan->ws_img);
  c.trec = (float*)(w + plan->ws_trec);
  c.rec = (float*)(w + plan->ws_rec);
  c.t_rw = (float*)(w + plan->ws_rw);
  c.misc = (float*)(w + plan->ws_misc);
  if (p) {
    B3R_REQUIRE(p->K && p->P_rig2c && p->P_w2rig && p->z_coefs && p->pts3d && p->pix2d_std && p->pix2d_dep,
                "NULL parameter pointer");
    B3R_REQUIRE(p->P_rig2c_stride >= 16, "P_rig2c stride must be >= 16");
    c.K = p->K; c.P_rig2c = p->P_rig2c; c.P_stride = p->P_rig2c_stride; c.P_w2rig = p->P_w2rig;
    c.z_coefs = p->z_coefs; c.pts3d = p->pts3d;
    c.pix2d = p->pix2d; c.pix2d_std = p->pix2d_std; c.pix2d_dep = p->pix2d_dep;
    B3R_REQUIRE(((uintptr_t)p->pix2d & 7) == 0 && ((uintptr_t)p->pix2d_std & 7) == 0,
                "pix2d and pix2d_std must be 8-byte aligned (float pairs)");
    if (!p->pix2d) {
      B3R_REQUIRE(p->residuals && p->w_pts, "residuals and w_pts are required when pix2d is NULL");
      B3R_REQUIRE(p->w_cols == 1 || p->w_cols == 3, "w_cols must be 1 or 3");
      c.res = p->residuals; c.rs_n = p->res_stride_n; c.rs_c = p->res_stride_c;
      c.wpt = p->w_pts; c.ws_n = p->w_stride_n; c.ws_c = p->w_stride_c; c.w_cols = p->w_cols;
    }
  }
  return B3R_OK;
}

template <int CT>
int launch_points(const Ctx& c, cudaStream_t s) {
  if (c.d.n_pt_tasks == 0) return B3R_OK;
  // persistent: one full wave of resident blocks, each warp walking tasks with a stride
  static int per_sm = 0, n_sm = 0;           // one occupancy query per instantiation
  if (per_sm == 0) {
    int dev = 0;
    B3R_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
    B3R_TRY(check_cuda(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev), "SM count"));
    B3R_TRY(check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_points<CT>, 128, 0),
                       "points occupancy"));
    per_sm = std::max(per_sm, 1);
  }
  const int blocks = (int)std::min<int64_t>(grid_for((int64_t)c.d.n_pt_tasks * 32, 128), (int64_t)per_sm * n_sm);
  k_points<CT><<<blocks, 128, 0, s>>>(c);
  return check_launch("points pass");
}

template <int CT>
int diag_launch(const Ctx& c, float* S, float* b, float* diagA, cudaStream_t s) {
  const size_t smem = (size_t)(kDiagThreads / kWarp) * 32 * diag_row_stride<CT>() * sizeof(float);
  static bool configured = false;          // one attribute call per instantiation
  if (!configured) {
    B3R_TRY(check_cuda(cudaFuncSetAttribute(k_diag<CT, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)smem), "diag smem attribute"));
    B3R_TRY(check_cuda(cudaFuncSetAttribute(k_diag<CT, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)smem), "diag smem attribute"));
    configured = true;
  }
  if (c.res_out || c.loss_part)
    k_diag<CT, true><<<c.d.n_c1_chunks, kDiagThreads, smem, s>>>(c, S, b, diagA);
  else
    k_diag<CT, false><<<c.d.n_c1_chunks, kDiagThreads, smem, s>>>(c, S, b, diagA);
  return check_launch("diag pass");
}

template <int CT>
int pairs_launch(const Ctx& c, float* S, cudaStream_t s) {
  const size_t smem = (size_t)pair_smem_floats<CT>() * sizeof(float);
  static bool configured = false;          // one attribute call per instantiation
  if (!configured) {
    B3R_TRY(check_cuda(cudaFuncSetAttribute(k_pairs<CT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                       "pairs smem attribute"));
    configured = true;
  }
  k_pairs<CT><<<(unsigned)c.d.n_tasks, pair_roles<CT>() * 32, smem, s>>>(c, S);
  return check_launch("pairs pass");
}

template <int CT>
int diag_z_launch(const Ctx& c, float* S, float* b, float* diagA, cudaStream_t s) {
  if constexpr (CT <= kZonlyMaxC) {
    if (c.res_out || c.loss_part)
      k_diag_z<CT, true><<<c.d.n_c1_chunks, kDiagZThreads, 0, s>>>(c, S, b, diagA);
    else
      k_diag_z<CT, false><<<c.d.n_c1_chunks, kDiagZThreads, 0, s>>>(c, S, b, diagA);
    return check_launch("diag pass (depth-stitch)");
  } else {
    return fail(B3R_E_INVALID, "internal: depth-stitch kernels for C=%d", CT);
  }
}

template <int CT>
int pairs_z_launch(const Ctx& c, float* S, cudaStream_t s) {
  if constexpr (CT <= kZonlyMaxC) {
    const int64_t per = kPairZThreads / 32;
    k_pairs_z<CT><<<(unsigned)((c.d.n_tasks + per - 1) / per), kPairZThreads, 0, s>>>(c, S);
    return check_launch("pairs pass (depth-stitch)");
  } else {
    return fail(B3R_E_INVALID, "internal: depth-stitch kernels for C=%d", CT);
  }
}

int launch_factor(const Ctx& c, cudaStream_t s) {
  k_factor<<<grid_for(std::max(c.d.nT_loc, 1), 256), 256, 0, s>>>(c);   // also records the damping
  return check_launch("factor pass");
}

template <int CT>
int launch_pass(const Ctx& c, int pass, float* S, float* b, float* diagA, cudaStream_t s) {
  switch (pass) {
    case B3R_PASS_POINTS:
      return launch_points<CT>(c, s);
    case B3R_PASS_ELIMINATE:
      return launch_factor(c, s);
    case B3R_PASS_DIAG:
      if (c.d.n_c1_chunks == 0) return B3R_OK;
      return c.d.zonly ? diag_z_launch<CT>(c, S, b, diagA, s) : diag_launch<CT>(c, S, b, diagA, s);
    case B3R_PASS_PAIRS:
      if (c.d.n_tasks == 0) return B3R_OK;
      return c.d.zonly ? pairs_z_launch<CT>(c, S, s) : pairs_launch<CT>(c, S, s);
  }
  return fail(B3R_E_INVALID, "bad pass %d", pass);
}

template <int CT>
int launch_assemble(const Ctx& c, float* S, float* b, float* diagA, cudaStream_t s) {
  B3R_TRY(launch_factor(c, s));
  if (c.d.zonly) {
    if (c.d.n_c1_chunks > 0) B3R_TRY(diag_z_launch<CT>(c, S, b, diagA, s));
    if (c.d.n_tasks > 0) B3R_TRY(pairs_z_launch<CT>(c, S, s));
    return B3R_OK;
  }
  if (c.d.n_c1_chunks > 0) B3R_TRY(diag_launch<CT>(c, S, b, diagA, s));
  if (c.d.n_tasks > 0) B3R_TRY(pairs_launch<CT>(c, S, s));
  return B3R_OK;
}

template <int CT>
int launch_backsub(const Ctx& c, const float* dc, float* dp, cudaStream_t s) {
  if (c.d.n_pt_tasks == 0) return B3R_OK;
  k_backsub<CT><<<grid_for((int64_t)c.d.n_pt_tasks * 32, 128), 128, 0, s>>>(c, dc, dp);
  return check_launch("backsub");
}

int stage_if_needed(b3r_plan* plan, const b3r_params* p, cudaStream_t s) {
  if (plan->staged && plan->staged_src[0] == p->pix2d && plan->staged_src[1] == p->pix2d_std &&
      plan->staged_src[2] == p->pix2d_dep)
    return B3R_OK;
  return b3r_plan_stage_obs(plan, p->pix2d, p->pix2d_std, p->pix2d_dep, s);
}

}  // namespace
}  // namespace b3r

using namespace b3r;

extern "C" int b3r_plan_stage_obs(b3r_plan* plan, const float* pix2d, const float* pix2d_std,
                                  const float* pix2d_dep, void* stream) {
  B3R_REQUIRE(plan != nullptr, "NULL plan");
  B3R_TRY(check_device(plan));
  B3R_REQUIRE(plan->d.n_loc == 0 || (pix2d_std && pix2d_dep), "NULL pix2d_std/pix2d_dep");
  if (plan->d.n_loc > 0) {
    k_stage_obs<<<grid_for(plan->d.n_loc, 256), 256, 0, as_stream(stream)>>>(plan->d, pix2d, pix2d_std, pix2d_dep);
    B3R_TRY(check_launch("b3r_plan_stage_obs"));
  }
  plan->staged = true;
  plan->staged_src[0] = pix2d; plan->staged_src[1] = pix2d_std; plan->staged_src[2] = pix2d_dep;
  return B3R_OK;
}

extern "C" int b3r_lin_points(b3r_plan* plan, const b3r_params* params, const b3r_lin_opts* opts,
                              void* workspace, const b3r_outputs* out, void* stream) {
  B3R_REQUIRE(params && out, "NULL params/outputs");
  Ctx c;
  B3R_TRY(make_ctx(plan, params, opts, workspace, c));
  B3R_TRY(check_device(plan));
  cudaStream_t s = as_stream(stream);
  B3R_TRY(stage_if_needed(plan, params, s));
  c.hpp_max = out->hpp_max ? out->hpp_max : c.misc;
  k_prep_images<<<grid_for(c.d.n_imgs, 128), 128, 0, s>>>(c);
  B3R_TRY(check_launch("prep images"));
  if (!params->pix2d && c.d.n_loc > 0) {
    k_stage_rw<<<grid_for(c.d.n_loc, 256), 256, 0, s>>>(c);
    B3R_TRY(check_launch("stage residuals"));
  }
  B3R_TRY(check_cuda(cudaMemsetAsync(c.hpp_max, 0, sizeof(float), s), "memset hpp_max"));
  switch (c.d.C) {
#define X(CC) case CC: return launch_points<CC>(c, s);
    B3R_FOR_EACH_C(X)
#undef X
    default: return fail(B3R_E_UNSUPPORTED, "no kernels compiled for C=%d depth channels", c.d.C);
  }
}

extern "C" int b3r_lin_assemble(b3r_plan* plan, const b3r_params* params, const b3r_lin_opts* opts,
                                void* workspace, const b3r_outputs* out, void* stream) {
  B3R_REQUIRE(params && out && out->S_vals && out->b && out->diagA, "NULL params/outputs");
  Ctx c;
  B3R_TRY(make_ctx(plan, params, opts, workspace, c));
  B3R_TRY(check_device(plan));
  cudaStream_t s = as_stream(stream);
  c.hpp_max = out->hpp_max ? out->hpp_max : c.misc;
  B3R_TRY(check_cuda(cudaMemsetAsync(out->S_vals, 0, sizeof(float) * (size_t)c.d.nnz, s), "memset S"));
  B3R_TRY(check_cuda(cudaMemsetAsync(out->b, 0, sizeof(float) * (size_t)c.d.n_cam_params, s), "memset b"));
  B3R_TRY(check_cuda(cudaMemsetAsync(out->diagA, 0, sizeof(float) * (size_t)c.d.n_cam_params, s), "memset diagA"));
  B3R_TRY(check_cuda(cudaMemsetAsync(c.misc + 8, 0, sizeof(float), s), "memset prior flag"));
  if (out->residuals || out->loss) {
    B3R_REQUIRE(params->pix2d, "residual and loss outputs need pix2d (in-kernel residuals)");
    c.res_out = out->residuals;
    c.loss_part = out->loss ? reinterpret_cast<double*>(reinterpret_cast<char*>(workspace) + plan->ws_loss) : nullptr;
  }
  switch (c.d.C) {
#define X(CC)                                                                                    \
    case CC:                                                                                     \
      B3R_TRY(launch_assemble<CC>(c, out->S_vals, out->b, out->diagA, s));                       \
      if (c.res_out || c.loss_part) {                                                            \
        k_rest<CC><<<kRestBlocks, 256, 0, s>>>(c);                                               \
        B3R_TRY(check_launch("objective of the remaining observations"));                        \
      }                                                                                          \
      break;
    B3R_FOR_EACH_C(X)
#undef X
    default: return fail(B3R_E_UNSUPPORTED, "no kernels compiled for C=%d depth channels", c.d.C);
  }
  if (c.loss_part) {
    k_loss_sum<<<1, 256, 0, s>>>(c.loss_part, c.d.n_c1_chunks + kRestBlocks, out->loss);
    B3R_TRY(check_launch("loss sum"));
  }
  return B3R_OK;
}

extern "C" int b3r_lin_pass(b3r_plan* plan, const b3r_params* params, const b3r_lin_opts* opts,
                            void* workspace, const b3r_outputs* out, int pass, void* stream) {
  B3R_REQUIRE(params && out, "NULL params/outputs");
  Ctx c;
  B3R_TRY(make_ctx(plan, params, opts, workspace, c));
  B3R_TRY(check_device(plan));
  cudaStream_t s = as_stream(stream);
  c.hpp_max = out->hpp_max ? out->hpp_max : c.misc;
  if (pass == B3R_PASS_PREP) {
    k_prep_images<<<grid_for(c.d.n_imgs, 128), 128, 0, s>>>(c);
    return check_launch("prep images");
  }
  switch (c.d.C) {
#define X(CC) case CC: return launch_pass<CC>(c, pass, out->S_vals, out->b, out->diagA, s);
    B3R_FOR_EACH_C(X)
#undef X
    default: return fail(B3R_E_UNSUPPORTED, "no kernels compiled for C=%d depth channels", c.d.C);
  }
}

extern "C" int b3r_lin_finalize(b3r_plan* plan, const b3r_lin_opts* opts, void* workspace,
                                const b3r_outputs* out, void* stream) {
  B3R_REQUIRE(out && out->S_vals && out->diagA, "NULL outputs");
  Ctx c;
  B3R_TRY(make_ctx(plan, nullptr, opts, workspace, c));
  B3R_TRY(check_device(plan));
  cudaStream_t s = as_stream(stream);
  if (c.d.n_cam_params == 0) return B3R_OK;
  B3R_TRY(check_cuda(cudaMemsetAsync(c.misc + 4, 0, 4 * sizeof(float), s), "memset maxima"));
  k_fin_max<<<std::min(grid_for(c.d.n_cam_params, 256), 148), 256, 0, s>>>(c, out->diagA);
  B3R_TRY(check_launch("finalize max"));
  k_fin_apply<<<grid_for(c.d.n_cam_params, 256), 256, 0, s>>>(c, out->diagA, out->S_vals, out->precond);
  return check_launch("finalize apply");
}

extern "C" int b3r_linearize_schur(b3r_plan* plan, const b3r_params* params, const b3r_lin_opts* opts,
                                   void* workspace, const b3r_outputs* out, void* stream) {
  B3R_TRY(b3r_lin_points(plan, params, opts, workspace, out, stream));
  B3R_TRY(b3r_lin_assemble(plan, params, opts, workspace, out, stream));
  return b3r_lin_finalize(plan, opts, workspace, out, stream);
}

template <typename T>
static int spmv_impl(const b3r_plan* plan, const float* S, const T* x, T* y, void* stream) {
  B3R_REQUIRE(plan && S && x && y, "NULL argument");
  B3R_TRY(check_device(plan));
  cudaStream_t s = as_stream(stream);
  B3R_TRY(check_cuda(cudaMemsetAsync(y, 0, sizeof(T) * (size_t)plan->d.n_cam_params, s), "memset y"));
  if (plan->d.nnzb == 0) return B3R_OK;
  k_spmv<T><<<grid_for(plan->d.nnzb, 4), 128, 0, s>>>(plan->d, S, x, y);
  return check_launch("b3r_schur_spmv");
}

extern "C" int b3r_schur_spmv(const b3r_plan* plan, const float* S_vals, const float* x, float* y, void* stream) {
  return spmv_impl<float>(plan, S_vals, x, y, stream);
}

extern "C" int b3r_schur_spmv_f64(const b3r_plan* plan, const float* S_vals, const double* x, double* y,
                                  void* stream) {
  return spmv_impl<double>(plan, S_vals, x, y, stream);
}

extern "C" int b3r_backsub(b3r_plan* plan, const b3r_params* params, const b3r_lin_opts* opts,
                           void* workspace, const float* delta_c, float* delta_p, void* stream) {
  B3R_REQUIRE(params && delta_c && delta_p, "NULL argument");
  Ctx c;
  B3R_TRY(make_ctx(plan, params, opts, workspace, c));
  B3R_TRY(check_device(plan));
  cudaStream_t s = as_stream(stream);
  switch (plan->d.C) {
#define X(CC) case CC: return launch_backsub<CC>(c, delta_c, delta_p, s);
    B3R_FOR_EACH_C(X)
#undef X
    default: return fail(B3R_E_UNSUPPORTED, "no kernels compiled for C=%d depth channels", plan->d.C);
  }
}

// ------------------------------------------------------------------------------------
// allocation-free linearization (no counterpart in the reference)
// ------------------------------------------------------------------------------------
// Hosts that drive the library only through this C ABI -- a Go, Java or plain C program
// with no CUDA allocator of its own, or an engine whose device memory is owned by a pool
// that forbids extra allocations during its iteration loop -- cannot allocate the
// per-call workspace that b3r_linearize_schur needs.  For them the workspace lives in the
// fixed device array below, which every GPU that loads this library holds until exit.
namespace b3r {
constexpr size_t kStaticWorkspaceBytes = size_t(32) << 20;   // 32 MiB per device
static __device__ __align__(256) unsigned char g_static_workspace[kStaticWorkspaceBytes];
constexpr int kStaticWsMaxDevices = 64;
static std::mutex g_static_ws_mutex;
static void* g_static_ws_ptr[kStaticWsMaxDevices] = {};
}  // namespace b3r

extern "C" int b3r_linearize_schur_noalloc(b3r_plan* plan, const b3r_params* params, const b3r_lin_opts* opts,
                                           const b3r_outputs* out, void* stream) {
  B3R_REQUIRE(plan && params && opts && out, "NULL argument");
  B3R_TRY(check_device(plan));
  B3R_REQUIRE(plan->info.workspace_bytes <= (int64_t)kStaticWorkspaceBytes,
              "this plan needs %lld bytes of workspace; the allocation-free entry point has a fixed "
              "%zu-byte (32 MiB) workspace: use b3r_linearize_schur with a caller-allocated workspace",
              (long long)plan->info.workspace_bytes, kStaticWorkspaceBytes);
  B3R_REQUIRE(plan->device >= 0 && plan->device < kStaticWsMaxDevices, "device %d out of range", plan->device);
  void* ws = nullptr;
  {
    // The array's host-side name is not a device address: take the real address once per
    // device, with that device current (check_device above guarantees it).  It stays valid
    // for the life of the process unless the device is reset (documented in the header).
    std::lock_guard<std::mutex> lock(g_static_ws_mutex);
    if (!g_static_ws_ptr[plan->device]) {
      void* p = nullptr;
      B3R_TRY(check_cuda(cudaGetSymbolAddress(&p, g_static_workspace), "cudaGetSymbolAddress(static workspace)"));
      g_static_ws_ptr[plan->device] = p;
    }
    ws = g_static_ws_ptr[plan->device];
  }
  // Every call shares the array and it keeps the previous call's contents.  The passes
  // overwrite every record they later read; the scalar slots (damping maxima) are cleared
  // here so no call depends on what an earlier one left behind.
  B3R_TRY(check_cuda(cudaMemsetAsync((char*)ws + plan->ws_misc, 0, 256, as_stream(stream)),
                     "clear static workspace scalars"));
  return b3r_linearize_schur(plan, params, opts, ws, out, stream);
}
