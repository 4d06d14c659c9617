// Device-side building blocks shared by every kernel of the library.
//
// The per-observation model restates the reference kernels of naver/blast3r
// (src/blast3r/extensions/cujac/sfm_jacobian_rigs.cu): the residual and Huber/IRLS
// weights of compute_residuals_rigs_cuda_kernel (:129-259) and the Jacobians of
// compute_jacobians_rigs_cuda_kernel (:323-509), in the same operation order so the
// float32 results stay within a few ulps of the reference's.  It is written once here
// and used by the residual op, the Jacobian op and every pass of the fused
// linearization, so all of them see identical residuals and weights.
#pragma once
#include <cmath>
#include <cstdint>
#include <cuda_runtime.h>

namespace b3r {

constexpr int kWarp = 32;

// ------------------------------------------------------------------------------------
// per-image camera record, precomputed once per linearization (k_prep_images)
// ------------------------------------------------------------------------------------
// [0..8] R_rw, [9..11] t_rw, [12..20] R_cr, [21..23] t_cr, [24] fx, [25] fy, [26] cx,
// [27] cy, [28..31] unused: 32 floats = one 128-byte line per image.
constexpr int kImgRec = 32;

template <typename T>
struct CamT {
  T R_rw[9], t_rw[3], R_cr[9], t_cr[3];
  T fx, fy, cx, cy;
};
using Cam = CamT<float>;

__device__ __forceinline__ Cam load_cam(const float* __restrict__ rec) {
  Cam c;
  const float4* r4 = reinterpret_cast<const float4*>(rec);
  float v[28];
#pragma unroll
  for (int i = 0; i < 7; ++i) {
    float4 q = __ldg(r4 + i);
    v[4 * i + 0] = q.x; v[4 * i + 1] = q.y; v[4 * i + 2] = q.z; v[4 * i + 3] = q.w;
  }
#pragma unroll
  for (int i = 0; i < 9; ++i) { c.R_rw[i] = v[i]; c.R_cr[i] = v[12 + i]; }
#pragma unroll
  for (int i = 0; i < 3; ++i) { c.t_rw[i] = v[9 + i]; c.t_cr[i] = v[21 + i]; }
  c.fx = v[24]; c.fy = v[25]; c.cx = v[26]; c.cy = v[27];
  return c;
}

// Camera of one observation straight from the reference arrays (reference ops path).
template <typename T>
__device__ __forceinline__ CamT<T> load_cam_ref(const float* __restrict__ K, const float* __restrict__ P_rig2c,
                                                int64_t P_rig2c_stride, const float* __restrict__ P_w2rig,
                                                int cam_idx, int node_idx) {
  CamT<T> c;
  const float* Prw = P_w2rig + (int64_t)node_idx * 16;
  const float* Pcr = P_rig2c + (int64_t)cam_idx * P_rig2c_stride;
#pragma unroll
  for (int r = 0; r < 3; ++r) {
#pragma unroll
    for (int k = 0; k < 3; ++k) { c.R_rw[3 * r + k] = Prw[4 * r + k]; c.R_cr[3 * r + k] = Pcr[4 * r + k]; }
    c.t_rw[r] = Prw[4 * r + 3];
    c.t_cr[r] = Pcr[4 * r + 3];
  }
  const float* Kc = K + (int64_t)cam_idx * 9;
  c.fx = Kc[0]; c.cx = Kc[2]; c.fy = Kc[4]; c.cy = Kc[5];
  return c;
}

// Image of observation `idx`: binary search over the cumulative counts infos[0]
// (sfm_jacobian_rigs.cu:72-88).
__device__ __forceinline__ int search_image(const int* __restrict__ cum, int n_img, int64_t idx) {
  int a = 0, b = n_img;
  while (b - a > 1) {
    int m = (a + b) / 2;
    if (idx < cum[m - 1]) b = m; else a = m;
  }
  return a;
}

// ------------------------------------------------------------------------------------
// per-observation linearization
// ------------------------------------------------------------------------------------
struct LinOpts {
  int is_depth_log;
  float weight_z, pnorm, max_pix_err, huber_delta, w_pts_nul;
  float clamp_lo, clamp_hi;
  // derived by finish_lin_opts: the Huber constants a = p/2 delta^(p-2) and
  // b = delta^p - a delta^2 (uniform per call, .cu:243-244), and which power law the
  // per-component terms follow (1: p == 1, rr^p = rr, rr^(p-2) = 1/rr; 2: p == 2,
  // rr^p = rr*rr, rr^(p-2) = 1; 0: general powf)
  float huber_a, huber_b;
  int pmode;
};

// Fill the derived fields of o (host side, once per call).
inline void finish_lin_opts(LinOpts& o) {
  o.pmode = o.pnorm == 1.f ? 1 : (o.pnorm == 2.f ? 2 : 0);
  o.huber_a = 0.f;
  o.huber_b = 0.f;
  if (o.pnorm > 0.f) {
    o.huber_a = 0.5f * o.pnorm * powf(o.huber_delta, o.pnorm - 2.f);
    o.huber_b = powf(o.huber_delta, o.pnorm) - o.huber_a * o.huber_delta * o.huber_delta;
  }
}

// Everything one observation contributes.
template <typename T>
struct ObsLinT {
  bool valid;        // camera depth z > 1e-3 (sfm_jacobian_rigs.cu:212, :408)
  T r[3];            // residual (x, y reprojection / std, focal-scaled log-depth)
  T err[3];          // Huber error
  T w[3];            // IRLS weight as the residual op outputs it (unclamped)
  T Jp[9];           // d r / d X_world, row-major 3x3
  T Jf0, Jf1;        // d r_x / d fx, d r_y / d fy
  float Jkf;         // d r_z / d fx = d r_z / d fy (a float even for double J, .cu:480)
  T Jt[18];          // d r / d tau, row-major 3x6 (rotation first)
  T zs;              // d r_z / d zcf_c = zs * dep_c
};
using ObsLin = ObsLinT<float>;

template <typename T> __device__ __forceinline__ T t_log(T x);
template <> __device__ __forceinline__ float t_log<float>(float x) { return logf(x); }
template <> __device__ __forceinline__ double t_log<double>(double x) { return log(x); }

// matmul<3,3,1> with bias, same summation order as the reference (.cu:91-114)
template <typename T>
__device__ __forceinline__ void mv3_bias(const T* A, const T* x, const T* b, T* y) {
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    T s = 0;
#pragma unroll
    for (int k = 0; k < 3; ++k) s += A[3 * r + k] * x[k];
    y[r] = s + b[r];
  }
}

// Residual + weights (+ Jacobians when WANT_J) of one observation.  `dep` holds the C raw
// depth channels, `zc` the image's C depth coefficients; CT > 0 fixes C at compile time.
// The residual is only computed for T = float (the reference residual kernel is float
// only, .cu:1074); the Jacobian follows the reference in T.
template <typename T, bool WANT_R, bool WANT_J, int CT>
__device__ __forceinline__ void linearize_obs(const CamT<T>& cam, const T X[3], float kx, float ky,
                                              float sx_, float sy_, const float* dep, const float* zc,
                                              int C_rt, const LinOpts& o, ObsLinT<T>& L) {
  const int C = CT > 0 ? CT : C_rt;
  T X_r[3], X_c[3];
  mv3_bias(cam.R_rw, X, cam.t_rw, X_r);
  mv3_bias(cam.R_cr, X_r, cam.t_cr, X_c);
  const T z = X_c[2];
  L.valid = !(z <= 1e-3);
  if (!L.valid) {
#pragma unroll
    for (int i = 0; i < 3; ++i) { L.r[i] = 0; L.err[i] = 0; L.w[i] = 0; }
    if (WANT_J) {
#pragma unroll
      for (int i = 0; i < 9; ++i) L.Jp[i] = 0;
#pragma unroll
      for (int i = 0; i < 18; ++i) L.Jt[i] = 0;
      L.Jf0 = L.Jf1 = 0; L.Jkf = 0.f; L.zs = 0;
    }
    return;
  }
  const T fx = cam.fx, fy = cam.fy, cx = cam.cx, cy = cam.cy;
  const T sx = sx_, sy = sy_;
  T guid = 0;
  if (CT > 0) {
#pragma unroll
    for (int c = 0; c < (CT > 0 ? CT : 1); ++c) guid += (T)zc[c] * (T)dep[c];
  } else {
    for (int c = 0; c < C; ++c) guid += (T)zc[c] * (T)dep[c];
  }
  const T fbar = T(0.5) * (fx + fy);
  if (WANT_R) {
    // projection and reprojection residual (.cu:217-228)
    // the quotients exactly as the reference forms them: p - k cancels, so the residual
    // keeps the reference's rounding of p
    const T p0 = (fx * X_c[0] + cx * X_c[2]) / z;
    const T p1 = (fy * X_c[1] + cy * X_c[2]) / z;
    L.r[0] = (p0 - (T)kx) / sx;
    L.r[1] = (p1 - (T)ky) / sy;
    // depth residual (.cu:235-238)
    if (o.is_depth_log) L.r[2] = fbar * (guid - t_log<T>(z));
    else                L.r[2] = fbar * t_log<T>(guid / z);
    // Huber error and IRLS weight per component (.cu:240-258)
    if (o.pnorm > 0.f) {
      const float a = o.huber_a, b = o.huber_b;
      const float wz[3] = {1.f, 1.f, o.weight_z};
#pragma unroll
      for (int i = 0; i < 3; ++i) {
        float rr = fabsf((float)L.r[i]);
        rr = (rr > o.max_pix_err) ? o.max_pix_err : rr;
        const float pw = o.pmode == 1 ? rr : (o.pmode == 2 ? rr * rr : powf(rr, o.pnorm));
        L.err[i] = wz[i] * ((rr <= o.huber_delta) ? a * rr * rr : pw - b);
        rr = (rr < o.huber_delta) ? o.huber_delta : rr;
        const float pw2 = o.pmode == 1 ? 1.f / rr : (o.pmode == 2 ? 1.f : powf(rr, o.pnorm - 2.f));
        L.w[i] = (rr == o.max_pix_err) ? o.w_pts_nul : wz[i] * pw2;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 3; ++i) { L.err[i] = 0; L.w[i] = 1; }
    }
  }
  if (!WANT_J) return;
  // Jacobians (.cu:410-508)
  // the Jacobian's divisions by z, sx, sy (.cu:410-480) become products with one
  // reciprocal each (within an ulp of the quotients; no cancellation follows them)
  const T inv_z = T(1.0f) / z, rsx = T(1.0f) / sx, rsy = T(1.0f) / sy;
  const T inv_z2 = inv_z * inv_z;
  const T P0 = fx * X_c[0] + cx * X_c[2];
  const T P1 = fy * X_c[1] + cy * X_c[2];
  T Jpc[9];
  Jpc[0] = fx * inv_z;             Jpc[1] = 0; Jpc[2] = cx * inv_z - P0 * inv_z2;
  Jpc[3] = 0; Jpc[4] = fy * inv_z; Jpc[5] = cy * inv_z - P1 * inv_z2;
  Jpc[6] = 0; Jpc[7] = 0;          Jpc[8] = -fbar * inv_z;
  Jpc[0] *= rsx; Jpc[2] *= rsx; Jpc[4] *= rsy; Jpc[5] *= rsy;
  // J_proj_rig = Jpc @ R_cr, skipping the structural zeros of Jpc (entries 1, 3, 6, 7):
  // the same value as the dense product (adding 0 or 0 * x changes no finite sum)
  T Jr[9];
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    Jr[c] = Jpc[0] * cam.R_cr[c] + Jpc[2] * cam.R_cr[6 + c];
    Jr[3 + c] = Jpc[4] * cam.R_cr[3 + c] + Jpc[5] * cam.R_cr[6 + c];
    Jr[6 + c] = Jpc[8] * cam.R_cr[6 + c];
  }
  // J_tau = Jr @ [-[X_r]x , I] (columns 0..2 rotation, 3..5 translation), written out
  // term by term without the zero and unit entries of the generator matrix
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    const T j0 = Jr[3 * r], j1 = Jr[3 * r + 1], j2 = Jr[3 * r + 2];
    L.Jt[6 * r + 0] = j1 * (-X_r[2]) + j2 * X_r[1];
    L.Jt[6 * r + 1] = j0 * X_r[2] + j2 * (-X_r[0]);
    L.Jt[6 * r + 2] = j0 * (-X_r[1]) + j1 * X_r[0];
    L.Jt[6 * r + 3] = j0;
    L.Jt[6 * r + 4] = j1;
    L.Jt[6 * r + 5] = j2;
  }
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      T s = 0;
#pragma unroll
      for (int k = 0; k < 3; ++k) s += Jr[3 * r + k] * cam.R_rw[3 * k + c];
      L.Jp[3 * r + c] = s;
    }
  L.Jf0 = X_c[0] * inv_z * rsx;
  L.Jf1 = X_c[1] * inv_z * rsy;
  float jkf = 0.f;
  if (guid > 0) jkf = o.is_depth_log ? (float)(0.5f * (guid + t_log<T>(inv_z))) : (float)(0.5f * t_log<T>(guid * inv_z));
  L.Jkf = jkf;
  L.zs = o.is_depth_log ? fbar : ((guid != 0) ? fbar / guid : T(0));
}

__device__ __forceinline__ float clampw(float w, float lo, float hi) {
  // torch.clamp(min=lo, max=hi)
  return fminf(fmaxf(w, lo), hi);
}

// ------------------------------------------------------------------------------------
// guarded 3x3 Cholesky (sfm_jacobian_rigs.cu:578-617): symmetrise, + jitter on the
// diagonal, non-positive pivots bumped by jitter.  Returns l00,l10,l20,l11,l21,l22.
// ------------------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ void chol3(T a00, T a01, T a02, T a10, T a11, T a12, T a20, T a21,
                                      T a22, T jitter, T l[6]) {
  a00 += jitter; a11 += jitter; a22 += jitter;
  const T a01s = (a01 + a10) * T(0.5);
  const T a02s = (a02 + a20) * T(0.5);
  const T a12s = (a12 + a21) * T(0.5);
  T l00sq = a00 > T(0) ? a00 : (a00 + jitter);
  const T l00 = sqrt(l00sq);
  const T l10 = a01s / l00;
  const T l20 = a02s / l00;
  T t11 = a11 - l10 * l10;
  t11 = t11 > T(0) ? t11 : (t11 + jitter);
  const T l11 = sqrt(t11);
  const T l21 = (a12s - l10 * l20) / l11;
  T t22 = a22 - l20 * l20 - l21 * l21;
  t22 = t22 > T(0) ? t22 : (t22 + jitter);
  const T l22 = sqrt(t22);
  l[0] = l00; l[1] = l10; l[2] = l20; l[3] = l11; l[4] = l21; l[5] = l22;
}

// forward solve L z = b
template <typename T>
__device__ __forceinline__ void chol3_fwd(const T l[6], const T b[3], T z[3]) {
  z[0] = b[0] / l[0];
  z[1] = (b[1] - l[1] * z[0]) / l[3];
  z[2] = (b[2] - l[2] * z[0] - l[4] * z[1]) / l[5];
}
// back solve L^T x = z
template <typename T>
__device__ __forceinline__ void chol3_bwd(const T l[6], const T z[3], T x[3]) {
  x[2] = z[2] / l[5];
  x[1] = (z[1] - l[4] * x[2]) / l[3];
  x[0] = (z[0] - l[1] * x[1] - l[2] * x[2]) / l[0];
}

// ------------------------------------------------------------------------------------
// warp helpers
// ------------------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, d));
  return v;
}
// Segmented inclusive scan (sum) over lanes; `seg_start` is the lane index of the first
// lane of the caller's segment.  The last lane of each segment ends with the total.
__device__ __forceinline__ float seg_scan(float v, int lane, int seg_start) {
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    float u = __shfl_up_sync(0xffffffffu, v, d);
    if (lane - d >= seg_start) v += u;
  }
  return v;
}

// atomic max for non-negative floats through their integer ordering
__device__ __forceinline__ void atomic_max_nonneg(float* addr, float v) {
  atomicMax(reinterpret_cast<int*>(addr), __float_as_int(fmaxf(v, 0.f)));
}

}  // namespace b3r
