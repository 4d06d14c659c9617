// Part 4 of the C ABI: the dense tangent prior on the depth coefficients.
//
// Restates the reference's _dense_tangent_prior_terms and confident_in_planar_regions
// (naver/blast3r src/blast3r/inference/engine.py:15-179) as one kernel over every image's
// subsampled grid instead of a per-image Python loop, and adds its Gauss-Newton terms to the
// assembled Schur system the way solve_delta adds z_prior (inference/ba_solver.py:141-173):
// g_z to the depth-coefficient gradient, H_z to the images' depth-coefficient diagonal
// blocks, both before the damping.
//
// Per image, on the grid subsampled by `stride` (first sample at stride / 2, intrinsics
// shifted and scaled to match), with log-depth channels L_c, coefficients a and rays
// B = K^-1 (u + 1/2, v + 1/2, 1):
//   D = exp(min(sum_c a_c L_c, 80)), X = D B, X0 the reference pointmap (times a per-image
//   scale when the tangents are not normalised);
//   forward differences t along rows (x) and columns (y) of X and X0, each normalised
//   (1 / max(|t|, eps)), residual r = t_hat - t0_hat, weight w = sqrt(max(C C', 0)) of the
//   planarity confidences C of the two end points (exp(-1e4 (lx^2 + ly^2)) of the reference
//   depth's Laplacians divided by its 3x3 minimum);
//   loss += weight_tan * mean(w r^2) per direction; with dX_c = D L_c B and its difference
//   dt_c (projected off t_hat and scaled by 1 / |t| when normalising),
//   g_c += s sum w dt_c . r and H_cd += s sum w dt_c . dt_d, s = weight_tan / (3 n_dir).
// The X side is computed in double (the solver's production dtype), the reference-pointmap
// side in float like the reference's float32 tensors.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include "b3r_common.cuh"
#include "b3r_plan.h"
#include "b3r_status.h"

namespace b3r {
namespace {

constexpr int kPriorThreads = 256;
constexpr int kPriorMaxC = 17;
constexpr float kPlanarAlpha = 1e4f;   // confident_in_planar_regions' alpha (engine.py:161)

struct PriorArgs {
  const b3r_dense_map* maps;
  int n_imgs, C, stride;
  const float* K;
  const int32_t* cam_ids;
  const float* z_coefs;
  const double* x0_scale;
  double weight, eps;
  int optim_Z0, normalize;
  double* loss;
  double* g;
  double* H;
};

struct ImgGeo {
  int Hs, Ws, cs;                 // subsampled grid, depth channel stride
  const float* L;                 // log-depth map (H, W, cs)
  const float* X0;                // reference pointmap (H, W, 3)
  int W, off, st;                 // full width, first sample, stride
  double Ki[9];                   // inverse of the subsampled intrinsics
  float s0;                       // reference pointmap scale
};

__device__ __forceinline__ int sub_len(int n, int off, int st) { return n > off ? (n - off + st - 1) / st : 0; }

// Position of (k, l), k <= l, in the row-major upper triangle of an n x n matrix.
__host__ __device__ constexpr int sym_off(int k, int l, int n) { return k * n - k * (k - 1) / 2 + (l - k); }

// Inverse of a 3x3 matrix by its adjugate (row-major).
__device__ __forceinline__ void inv3(const double m[9], double o[9]) {
  const double c00 = m[4] * m[8] - m[5] * m[7], c01 = m[5] * m[6] - m[3] * m[8], c02 = m[3] * m[7] - m[4] * m[6];
  const double det = m[0] * c00 + m[1] * c01 + m[2] * c02, id = 1.0 / det;
  o[0] = c00 * id; o[1] = (m[2] * m[7] - m[1] * m[8]) * id; o[2] = (m[1] * m[5] - m[2] * m[4]) * id;
  o[3] = c01 * id; o[4] = (m[0] * m[8] - m[2] * m[6]) * id; o[5] = (m[2] * m[3] - m[0] * m[5]) * id;
  o[6] = c02 * id; o[7] = (m[1] * m[6] - m[0] * m[7]) * id; o[8] = (m[0] * m[4] - m[1] * m[3]) * id;
}

__device__ __forceinline__ float ref_z(const ImgGeo& g, int v, int u) {
  const int64_t p = (int64_t)(g.off + v * g.st) * g.W + (g.off + u * g.st);
  return g.X0[3 * p + 2] * g.s0;
}

// Planarity confidence of grid cell (v, u) (confident_in_planar_regions, engine.py:161-179):
// Laplacians of the reference depth along columns and rows (missing neighbours count as
// zero), divided by the 3x3 minimum of the depth (clipped at 1e-12), exp(-alpha |.|^2).
__device__ __forceinline__ float planar_conf(const ImgGeo& g, int v, int u) {
  const float d = ref_z(g, v, u);
  float lx = 2.f * d, ly = 2.f * d;
  if (u >= 1) lx -= ref_z(g, v, u - 1);
  if (u <= g.Ws - 2) lx -= ref_z(g, v, u + 1);
  if (v >= 1) ly -= ref_z(g, v - 1, u);
  if (v <= g.Hs - 2) ly -= ref_z(g, v + 1, u);
  float mn = d;
  for (int dv = -1; dv <= 1; ++dv)
    for (int du = -1; du <= 1; ++du) {
      const int vv = v + dv, uu = u + du;
      if (vv >= 0 && vv < g.Hs && uu >= 0 && uu < g.Ws) mn = fminf(mn, ref_z(g, vv, uu));
    }
  const float nrm = fmaxf(mn, 1e-12f);
  lx /= nrm;
  ly /= nrm;
  return expf(-kPlanarAlpha * (lx * lx + ly * ly));
}

// The quantities of one grid cell that its edges need.
template <int CT>
struct Cell {
  double X[3], ray[3], D, L[CT];
  float X0[3], conf;
};

template <int CT>
__device__ __forceinline__ void load_cell(const ImgGeo& g, const double* a, int v, int u, Cell<CT>& c) {
  const int64_t p = (int64_t)(g.off + v * g.st) * g.W + (g.off + u * g.st);
  double lc = 0.0;
#pragma unroll
  for (int k = 0; k < CT; ++k) {
    c.L[k] = (double)g.L[p * g.cs + k];
    lc += a[k] * c.L[k];
  }
  c.D = exp(fmin(lc, 80.0));
  const double px = u + 0.5, py = v + 0.5;
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    c.ray[r] = g.Ki[3 * r] * px + g.Ki[3 * r + 1] * py + g.Ki[3 * r + 2];
    c.X[r] = c.ray[r] * c.D;
  }
#pragma unroll
  for (int r = 0; r < 3; ++r) c.X0[r] = g.X0[3 * p + r] * g.s0;
  c.conf = planar_conf(g, v, u);
}

// Contributions of the edge a -> b: loss, g (CT), H (upper triangle, CT (CT + 1) / 2),
// each already multiplied by the direction's scale.
template <int CT>
__device__ __forceinline__ void edge_terms(const Cell<CT>& A, const Cell<CT>& B, double scale, double eps,
                                           int normalize, int optim_Z0, double* acc) {
  constexpr int NH = CT * (CT + 1) / 2;
  float t0[3];
#pragma unroll
  for (int r = 0; r < 3; ++r) t0[r] = B.X0[r] - A.X0[r];
  const float n0 = sqrtf(t0[0] * t0[0] + t0[1] * t0[1] + t0[2] * t0[2]);
  const float inv0 = 1.0f / fmaxf(n0, (float)eps);
  double t[3];
#pragma unroll
  for (int r = 0; r < 3; ++r) t[r] = B.X[r] - A.X[r];
  const double inv = normalize ? 1.0 / fmax(sqrt(t[0] * t[0] + t[1] * t[1] + t[2] * t[2]), eps) : (double)inv0;
  double th[3], res[3];
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    th[r] = t[r] * inv;
    res[r] = th[r] - (double)(t0[r] * inv0);
  }
  const double w = (double)sqrtf(fmaxf(A.conf * B.conf, 0.f));
  acc[0] += scale * w * (res[0] * res[0] + res[1] * res[1] + res[2] * res[2]);
  double dt[CT][3];
#pragma unroll
  for (int k = 0; k < CT; ++k) {
    const double sa = A.D * A.L[k], sb = B.D * B.L[k];
    double d3[3];
#pragma unroll
    for (int r = 0; r < 3; ++r) d3[r] = sb * B.ray[r] - sa * A.ray[r];
    if (normalize) {
      const double dot = d3[0] * th[0] + d3[1] * th[1] + d3[2] * th[2];
#pragma unroll
      for (int r = 0; r < 3; ++r) d3[r] = (d3[r] - th[r] * dot) * inv;
    } else {
#pragma unroll
      for (int r = 0; r < 3; ++r) d3[r] *= inv;
    }
#pragma unroll
    for (int r = 0; r < 3; ++r) dt[k][r] = d3[r];
  }
  const double sw = scale * w;
#pragma unroll
  for (int k = 0; k < CT; ++k) {
    if (k == 0 && !optim_Z0) continue;                  // engine.py:153-156
    acc[1 + k] += sw * (dt[k][0] * res[0] + dt[k][1] * res[1] + dt[k][2] * res[2]);
#pragma unroll
    for (int l = k; l < CT; ++l)
      acc[1 + CT + sym_off(k, l, CT)] += sw * (dt[k][0] * dt[l][0] + dt[k][1] * dt[l][1] + dt[k][2] * dt[l][2]);
  }
  (void)NH;
}

template <int CT>
__global__ void __launch_bounds__(kPriorThreads) k_tangent_prior(PriorArgs P) {
  constexpr int NA = 1 + CT + CT * (CT + 1) / 2;
  __shared__ double red[kPriorThreads / 32][NA];
  const int img = blockIdx.y;
  const b3r_dense_map m = P.maps[img];
  ImgGeo g;
  g.st = P.stride;
  g.off = P.stride / 2;
  g.W = m.W;
  g.Hs = sub_len(m.H, g.off, g.st);
  g.Ws = sub_len(m.W, g.off, g.st);
  g.cs = m.channel_stride;
  g.L = m.log_depth;
  g.X0 = m.pts3d_ref;
  g.s0 = P.x0_scale ? (float)P.x0_scale[img] : 1.f;
  // the reference skips an image whose subsampled width or channel count is below 2
  // (min(L.shape[1:]) < 2, engine.py:82-83)
  const bool skip = g.Ws < 2 || CT < 2 || g.Hs < 1;
  {
    const float* Kc = P.K + 9 * (int64_t)P.cam_ids[img];
    double Kd[9];
#pragma unroll
    for (int q = 0; q < 9; ++q) Kd[q] = (double)Kc[q];
    Kd[2] -= g.off; Kd[5] -= g.off;                     // K[:2, 2] -= sub.start
#pragma unroll
    for (int q = 0; q < 6; ++q) Kd[q] /= g.st;          // K[:2] /= stride
    inv3(Kd, g.Ki);
  }
  double a[CT];
#pragma unroll
  for (int k = 0; k < CT; ++k) a[k] = (double)P.z_coefs[(int64_t)img * CT + k];
  const int nx = (g.Hs - 1) * g.Ws, ny = g.Hs * (g.Ws - 1);
  const double sx = nx > 0 ? P.weight / (3.0 * nx) : 0.0, sy = ny > 0 ? P.weight / (3.0 * ny) : 0.0;
  double acc[NA];
#pragma unroll
  for (int q = 0; q < NA; ++q) acc[q] = 0.0;
  const int cells = skip ? 0 : g.Hs * g.Ws;
  for (int cid = blockIdx.x * blockDim.x + threadIdx.x; cid < cells; cid += gridDim.x * blockDim.x) {
    const int v = cid / g.Ws, u = cid - v * g.Ws;
    Cell<CT> c0;
    load_cell<CT>(g, a, v, u, c0);
    if (v + 1 < g.Hs) {                                 // edge along the rows (tx)
      Cell<CT> c1;
      load_cell<CT>(g, a, v + 1, u, c1);
      edge_terms<CT>(c0, c1, sx, P.eps, P.normalize, P.optim_Z0, acc);
    }
    if (u + 1 < g.Ws) {                                 // edge along the columns (ty)
      Cell<CT> c1;
      load_cell<CT>(g, a, v, u + 1, c1);
      edge_terms<CT>(c0, c1, sy, P.eps, P.normalize, P.optim_Z0, acc);
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int q = 0; q < NA; ++q) {
    double t = acc[q];
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) t += __shfl_xor_sync(0xffffffffu, t, d);
    if (lane == 0) red[warp][q] = t;
  }
  __syncthreads();
  for (int q = threadIdx.x; q < NA; q += blockDim.x) {
    double t = 0.0;
    for (int w = 0; w < kPriorThreads / 32; ++w) t += red[w][q];
    if (t == 0.0) continue;
    if (q == 0) {
      atomicAdd(P.loss, t);
    } else if (q <= CT) {
      if (P.g) atomicAdd(P.g + (int64_t)img * CT + (q - 1), t);
    } else if (P.H) {
      int k = 0, r = q - 1 - CT;
      while (r >= CT - k) { r -= CT - k; ++k; }
      const int l = k + r;
      double* Hi = P.H + (int64_t)img * CT * CT;
      atomicAdd(Hi + k * CT + l, t);
      if (l != k) atomicAdd(Hi + l * CT + k, t);
    }
  }
}

// Adds H_z to the images' zcf diagonal blocks of S, g_z to b and diag(H_z) to diag(A)
// (before b3r_lin_finalize damps them).
__global__ void k_add_zprior(DevPlan d, const double* __restrict__ Hz, const double* __restrict__ gz,
                             float* __restrict__ S, float* __restrict__ b, float* __restrict__ diagA, float* misc) {
  const int i = blockIdx.x;
  const int C = d.C;
  const int dst = d.img_zdiag[i], sc = d.img_zsc[i];
  if (dst < 0) return;
  for (int e = threadIdx.x; e < C * C; e += blockDim.x) {
    S[dst + e] += (float)Hz[(int64_t)i * C * C + e];
    const int r = e / C, q = e - r * C;
    if (r == q) diagA[sc + r] += (float)Hz[(int64_t)i * C * C + e];
  }
  for (int c = threadIdx.x; c < C; c += blockDim.x) b[sc + c] += (float)gz[(int64_t)i * C + c];
  if (i == 0 && threadIdx.x == 0) misc[8] = 1.f;       // the zcf blocks now hold a prior
}

}  // namespace
}  // namespace b3r

using namespace b3r;

extern "C" int b3r_tangent_prior(const b3r_dense_map* maps, int32_t n_imgs, int32_t cells_hint, const float* K,
                                 const int32_t* cam_ids, const float* z_coefs, int32_t C, const double* x0_scale,
                                 int32_t stride, double weight_tan, double eps, int32_t optim_Z0, int32_t normalize,
                                 double* loss, double* g_z, double* H_z, void* stream) {
  B3R_REQUIRE(maps && K && cam_ids && z_coefs && loss, "NULL argument");
  B3R_REQUIRE(n_imgs >= 0 && stride >= 1, "bad n_imgs or stride");
  B3R_REQUIRE(C >= 1 && C <= kPriorMaxC, "C=%d out of range [1, %d]", C, kPriorMaxC);
  B3R_REQUIRE((g_z == nullptr) == (H_z == nullptr), "g_z and H_z are both given or both NULL");
  cudaStream_t s = as_stream(stream);
  B3R_TRY(check_cuda(cudaMemsetAsync(loss, 0, sizeof(double), s), "memset loss"));
  if (g_z) {
    B3R_TRY(check_cuda(cudaMemsetAsync(g_z, 0, sizeof(double) * (size_t)n_imgs * C, s), "memset g_z"));
    B3R_TRY(check_cuda(cudaMemsetAsync(H_z, 0, sizeof(double) * (size_t)n_imgs * C * C, s), "memset H_z"));
  }
  if (n_imgs == 0 || weight_tan <= 0.0) return B3R_OK;   // the reference returns zeros (engine.py:50-56)
  PriorArgs P{maps, n_imgs, C, stride, K, cam_ids, z_coefs, x0_scale, weight_tan, eps, optim_Z0, normalize,
              loss, g_z, H_z};
  const int bx = std::max(1, std::min((std::max(cells_hint, 1) + kPriorThreads - 1) / kPriorThreads, 64));
  const dim3 grid(bx, n_imgs);
  switch (C) {
#define X(CC) case CC: k_tangent_prior<CC><<<grid, kPriorThreads, 0, s>>>(P); break;
    X(1) X(2) X(3) X(4) X(5) X(6) X(7) X(8) X(17)
#undef X
    default: return fail(B3R_E_UNSUPPORTED, "no tangent-prior kernel for C=%d", C);
  }
  return check_launch("b3r_tangent_prior");
}

extern "C" int b3r_lin_add_zprior(b3r_plan* plan, const double* H_z, const double* g_z, void* workspace,
                                  const b3r_outputs* out, void* stream) {
  B3R_REQUIRE(plan && H_z && g_z && workspace && out && out->S_vals && out->b && out->diagA, "NULL argument");
  B3R_REQUIRE(((uintptr_t)workspace & 255) == 0, "workspace must be 256-byte aligned");
  int dev = -1;
  B3R_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  B3R_REQUIRE(dev == plan->device, "current device %d differs from the plan's device %d", dev, plan->device);
  if (plan->d.n_imgs == 0) return B3R_OK;
  float* misc = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + plan->ws_misc);
  k_add_zprior<<<plan->d.n_imgs, 64, 0, as_stream(stream)>>>(plan->d, H_z, g_z, out->S_vals, out->b, out->diagA, misc);
  return check_launch("b3r_lin_add_zprior");
}
