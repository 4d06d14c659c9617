// Part 1 of the C ABI: one-to-one mirrors of the reference's native ops
// (naver/blast3r src/blast3r/extensions/cujac/sfm_jacobian_rigs.cu, bindings :1254-1275),
// so the reference's Python solver can bind this library in place of its extension.
// Layouts, argument meaning and numerics follow the reference; outputs are written in
// full (the reference zero-fills them with torch::zeros before its kernels run).
#include <algorithm>
#include "b3r_common.cuh"
#include "b3r_status.h"

namespace b3r {

std::string& last_error_ref() {
  thread_local std::string s;
  return s;
}

namespace {
constexpr int kThreads = 128;   // one observation / item per thread, as the reference

// residuals_with_rigs (sfm_jacobian_rigs.cu:129-259): out is [n_out, n_obs]
__global__ void k_residuals(const int* __restrict__ infos, int n_imgs, const float* __restrict__ K,
                            const float* __restrict__ P_rig2c, int64_t P_stride,
                            const float* __restrict__ P_w2rig, const float* __restrict__ z_coefs,
                            int C, const float* __restrict__ pts3d, const int* __restrict__ pids,
                            int64_t n_obs, const float* __restrict__ pix2d,
                            const float* __restrict__ pix2d_std, const float* __restrict__ pix2d_dep,
                            LinOpts o, float* __restrict__ out) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n_obs) return;
  const int img = search_image(infos, n_imgs, idx);
  const int node = infos[n_imgs + img];
  const int cam = infos[2 * n_imgs + img];
  const int pt = pids[idx];
  const Cam c = load_cam_ref<float>(K, P_rig2c, P_stride, P_w2rig, cam, node);
  const float X[3] = {pts3d[3 * (int64_t)pt], pts3d[3 * (int64_t)pt + 1], pts3d[3 * (int64_t)pt + 2]};
  ObsLin L;
  linearize_obs<float, true, false, 0>(c, X, pix2d[2 * idx], pix2d[2 * idx + 1], pix2d_std[2 * idx],
                                       pix2d_std[2 * idx + 1], pix2d_dep + idx * C,
                                       z_coefs + (int64_t)img * C, C, o, L);
#pragma unroll
  for (int i = 0; i < 3; ++i) out[i * n_obs + idx] = L.r[i];
  if (o.pnorm > 0.f) {
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      out[(3 + i) * n_obs + idx] = L.err[i];
      out[(6 + i) * n_obs + idx] = L.w[i];
    }
  }
}

// The objective of lm_step (engine.py:263-281) without its [9, n_obs] buffer: every
// observation's residual and Huber error as the residual kernel forms them; the errors
// summed in double (one atomic per block), the residuals written component-major when
// asked for.
constexpr int kLossThreads = 256;
__global__ void __launch_bounds__(kLossThreads) k_residual_loss(
    const int* __restrict__ infos, int n_imgs, const float* __restrict__ K, const float* __restrict__ P_rig2c,
    int64_t P_stride, const float* __restrict__ P_w2rig, const float* __restrict__ z_coefs, int C,
    const float* __restrict__ pts3d, const int* __restrict__ pids, int64_t n_obs, const float* __restrict__ pix2d,
    const float* __restrict__ pix2d_std, const float* __restrict__ pix2d_dep, LinOpts o, double* __restrict__ loss,
    float* __restrict__ res) {
  __shared__ double red[kLossThreads / 32];
  double acc = 0.0;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < n_obs;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int img = search_image(infos, n_imgs, idx);
    const int node = infos[n_imgs + img];
    const int cam = infos[2 * n_imgs + img];
    const int pt = pids[idx];
    const Cam c = load_cam_ref<float>(K, P_rig2c, P_stride, P_w2rig, cam, node);
    const float X[3] = {pts3d[3 * (int64_t)pt], pts3d[3 * (int64_t)pt + 1], pts3d[3 * (int64_t)pt + 2]};
    ObsLin L;
    linearize_obs<float, true, false, 0>(c, X, pix2d[2 * idx], pix2d[2 * idx + 1], pix2d_std[2 * idx],
                                         pix2d_std[2 * idx + 1], pix2d_dep + idx * C,
                                         z_coefs + (int64_t)img * C, C, o, L);
    if (res) {
#pragma unroll
      for (int i = 0; i < 3; ++i) res[i * n_obs + idx] = L.r[i];
    }
    acc += (double)L.err[0] + (double)L.err[1] + (double)L.err[2];
  }
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, d);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < kLossThreads / 32; ++w) t += red[w];
    atomicAdd(loss, t);
  }
}

// jacobians_with_rigs (sfm_jacobian_rigs.cu:323-509)
template <typename T>
__global__ void k_jacobians(const int* __restrict__ infos, int n_imgs, const float* __restrict__ K,
                            const float* __restrict__ P_rig2c, int64_t P_stride,
                            const float* __restrict__ P_w2rig, const float* __restrict__ z_coefs,
                            int C, const float* __restrict__ pts3d, const int* __restrict__ pids,
                            int64_t n_obs, const float* __restrict__ pix2d_std,
                            const float* __restrict__ pix2d_dep, LinOpts o, T* __restrict__ J_cam,
                            T* __restrict__ J_zcf, T* __restrict__ J_pts) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n_obs) return;
  const int img = search_image(infos, n_imgs, idx);
  const int node = infos[n_imgs + img];
  const int cam = infos[2 * n_imgs + img];
  const int pt = pids[idx];
  const CamT<T> c = load_cam_ref<T>(K, P_rig2c, P_stride, P_w2rig, cam, node);
  const T X[3] = {(T)pts3d[3 * (int64_t)pt], (T)pts3d[3 * (int64_t)pt + 1], (T)pts3d[3 * (int64_t)pt + 2]};
  const float* dep = pix2d_dep + idx * C;
  ObsLinT<T> L;
  linearize_obs<T, false, true, 0>(c, X, 0.f, 0.f, pix2d_std[2 * idx], pix2d_std[2 * idx + 1], dep,
                                   z_coefs + (int64_t)img * C, C, o, L);
  T* jc = J_cam + idx * 24;
  // row 0: [dfx, 0, tau], row 1: [0, dfy, tau], row 2: [Jkf, Jkf, tau]
  jc[0] = L.Jf0; jc[1] = 0;
  jc[8] = 0;     jc[9] = L.Jf1;
  jc[16] = (T)L.Jkf; jc[17] = (T)L.Jkf;
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int i = 0; i < 6; ++i) jc[8 * r + 2 + i] = L.Jt[6 * r + i];
  T* jz = J_zcf + idx * C;
  for (int i = 0; i < C; ++i) jz[i] = L.zs * (T)dep[i];
  T* jp = J_pts + idx * 9;
#pragma unroll
  for (int i = 0; i < 9; ++i) jp[i] = L.Jp[i];
}

// chol3x3_solve (sfm_jacobian_rigs.cu:560-634)
template <typename T>
__global__ void k_chol3x3_solve(const T* __restrict__ blocks, const T* __restrict__ rhs,
                                T* __restrict__ out, int64_t N, T jitter) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N) return;
  const T* A = blocks + i * 9;
  T l[6];
  chol3<T>(A[0], A[1], A[2], A[3], A[4], A[5], A[6], A[7], A[8], jitter, l);
  const T b[3] = {rhs[3 * i], rhs[3 * i + 1], rhs[3 * i + 2]};
  T z[3], x[3];
  chol3_fwd<T>(l, b, z);
  chol3_bwd<T>(l, z, x);
  out[3 * i] = x[0]; out[3 * i + 1] = x[1]; out[3 * i + 2] = x[2];
}

// blockcoo_matvec (sfm_jacobian_rigs.cu:760-803): one thread per (block, output element)
template <typename T, typename I>
__global__ void k_bcoo_matvec(const T* __restrict__ blocks, int bh, int bw, const I* __restrict__ rows,
                              const I* __restrict__ cols, int64_t N, const T* __restrict__ x,
                              T* __restrict__ y, int transpose) {
  const int per = transpose ? bw : bh;
  const int64_t total = N * per;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (int64_t)blockDim.x * gridDim.x) {
    const int64_t bi = t / per;
    const int lo = (int)(t - bi * per);
    const int64_t rb = (int64_t)rows[bi], cb = (int64_t)cols[bi];
    const T* A = blocks + bi * (int64_t)(bh * bw);
    T acc = 0;
    if (!transpose) {
      for (int c = 0; c < bw; ++c) acc += A[lo * bw + c] * x[cb * bw + c];
      atomicAdd(y + rb * bh + lo, acc);
    } else {
      for (int r = 0; r < bh; ++r) acc += A[r * bw + lo] * x[rb * bh + r];
      atomicAdd(y + cb * bw + lo, acc);
    }
  }
}

// fused_einsum_bki_bkj (sfm_jacobian_rigs.cu:880-941): one thread per output element
template <typename T>
__global__ void k_einsum_bki_bkj(const T* __restrict__ left, int64_t l_bs, int64_t l_ks,
                                 const T* __restrict__ right, int64_t r_bs, int64_t r_ks,
                                 T* __restrict__ out, int64_t B, int K, int I, int J) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t per = (int64_t)I * J;
  if (t >= B * per) return;
  const int64_t b = t / per;
  const int ij = (int)(t - b * per);
  const int i = ij / J, j = ij - (ij / J) * J;
  const T* lb = left + b * l_bs;
  const T* rb = right + b * r_bs;
  T acc = 0;
  for (int k = 0; k < K; ++k) acc += lb[k * l_ks + i] * rb[k * r_ks + j];
  out[t] = acc;
}

LinOpts make_opts(int is_depth_log, float weight_z, float pnorm, float max_pix_err,
                  float huber_delta, float w_pts_nul) {
  LinOpts o;
  o.is_depth_log = is_depth_log;
  o.weight_z = weight_z; o.pnorm = pnorm; o.max_pix_err = max_pix_err;
  o.huber_delta = huber_delta; o.w_pts_nul = w_pts_nul;
  o.clamp_lo = 0.f; o.clamp_hi = 0.f;
  finish_lin_opts(o);
  return o;
}
}  // namespace
}  // namespace b3r

using namespace b3r;

extern "C" const char* b3r_last_error(void) { return last_error_ref().c_str(); }
extern "C" const char* b3r_version(void) { return "blast3r_b200 0.1 (sm_100a)"; }

static int check_common(const int32_t* infos, int n_imgs, const float* K, int n_cams,
                        const float* P_rig2c, int64_t P_rig2c_stride, const float* P_w2rig,
                        int n_nodes, const float* z_coefs, int C, const float* pts3d,
                        int n_tracks, const int32_t* pids, int64_t n_obs) {
  B3R_REQUIRE(n_obs >= 0 && n_imgs >= 1 && n_cams >= 1 && n_nodes >= 1 && n_tracks >= 0 && C >= 1,
              "bad sizes: n_obs=%lld n_imgs=%d n_cams=%d n_nodes=%d n_tracks=%d C=%d",
              (long long)n_obs, n_imgs, n_cams, n_nodes, n_tracks, C);
  B3R_REQUIRE(n_obs == 0 || (infos && K && P_rig2c && P_w2rig && z_coefs && pts3d && pids),
              "NULL input pointer");
  B3R_REQUIRE(P_rig2c_stride >= 16, "P_rig2c stride must be >= 16 floats (got %lld)",
              (long long)P_rig2c_stride);
  return B3R_OK;
}

extern "C" int b3r_residuals_with_rigs(const int32_t* infos, int n_imgs, const float* K, int n_cams,
                                       const float* P_rig2c, int64_t P_rig2c_stride,
                                       const float* P_w2rig, int n_nodes, const float* z_coefs,
                                       int C, const float* pts3d, int n_tracks,
                                       const int32_t* pids, int64_t n_obs, const float* pix2d,
                                       const float* pix2d_std, const float* pix2d_dep,
                                       int is_depth_log, float weight_z, float pnorm,
                                       float max_pix_err, float huber_delta, float w_pts_nul,
                                       float* out, void* stream) {
  B3R_TRY(check_common(infos, n_imgs, K, n_cams, P_rig2c, P_rig2c_stride, P_w2rig, n_nodes, z_coefs,
                       C, pts3d, n_tracks, pids, n_obs));
  B3R_REQUIRE(pnorm == -1.f || (pnorm > 0.f && pnorm <= 2.f), "pnorm must be in {-1} U ]0,2]");
  B3R_REQUIRE(n_obs == 0 || (pix2d && pix2d_std && pix2d_dep && out), "NULL observation/output pointer");
  if (n_obs == 0) return B3R_OK;
  LinOpts o = make_opts(is_depth_log, weight_z, pnorm, max_pix_err, huber_delta, w_pts_nul);
  k_residuals<<<grid_for(n_obs, kThreads), kThreads, 0, as_stream(stream)>>>(
      infos, n_imgs, K, P_rig2c, P_rig2c_stride, P_w2rig, z_coefs, C, pts3d, pids, n_obs, pix2d,
      pix2d_std, pix2d_dep, o, out);
  return check_launch("b3r_residuals_with_rigs");
}

extern "C" int b3r_residual_loss(const int32_t* infos, int n_imgs, const float* K, int n_cams, const float* P_rig2c,
                                 int64_t P_rig2c_stride, const float* P_w2rig, int n_nodes, const float* z_coefs,
                                 int C, const float* pts3d, int n_tracks, const int32_t* pids, int64_t n_obs,
                                 const float* pix2d, const float* pix2d_std, const float* pix2d_dep,
                                 int is_depth_log, float weight_z, float pnorm, float max_pix_err,
                                 float huber_delta, double* loss_sum, float* residuals, void* stream) {
  B3R_TRY(check_common(infos, n_imgs, K, n_cams, P_rig2c, P_rig2c_stride, P_w2rig, n_nodes, z_coefs,
                       C, pts3d, n_tracks, pids, n_obs));
  B3R_REQUIRE(pnorm > 0.f && pnorm <= 2.f, "pnorm must be in ]0,2] for a loss");
  B3R_REQUIRE(loss_sum != nullptr, "NULL loss_sum");
  B3R_REQUIRE(n_obs == 0 || (pix2d && pix2d_std && pix2d_dep), "NULL observation pointer");
  cudaStream_t s = as_stream(stream);
  B3R_TRY(check_cuda(cudaMemsetAsync(loss_sum, 0, sizeof(double), s), "b3r_residual_loss memset"));
  if (n_obs == 0) return B3R_OK;
  LinOpts o = make_opts(is_depth_log, weight_z, pnorm, max_pix_err, huber_delta, 1e-16f);
  const int g = (int)std::min<int64_t>(grid_for(n_obs, kLossThreads), 148 * 8);
  k_residual_loss<<<g, kLossThreads, 0, s>>>(infos, n_imgs, K, P_rig2c, P_rig2c_stride, P_w2rig, z_coefs, C, pts3d,
                                             pids, n_obs, pix2d, pix2d_std, pix2d_dep, o, loss_sum, residuals);
  return check_launch("b3r_residual_loss");
}

extern "C" int b3r_jacobians_with_rigs(const int32_t* infos, int n_imgs, const float* K, int n_cams,
                                       const float* P_rig2c, int64_t P_rig2c_stride,
                                       const float* P_w2rig, int n_nodes, const float* z_coefs,
                                       int C, const float* pts3d, int n_tracks,
                                       const int32_t* pids, int64_t n_obs, const float* pix2d_std,
                                       const float* pix2d_dep, int is_depth_log,
                                       int output_float64, void* J_cam, void* J_zcf, void* J_pts,
                                       void* stream) {
  B3R_TRY(check_common(infos, n_imgs, K, n_cams, P_rig2c, P_rig2c_stride, P_w2rig, n_nodes, z_coefs,
                       C, pts3d, n_tracks, pids, n_obs));
  B3R_REQUIRE(n_obs == 0 || (pix2d_std && pix2d_dep && J_cam && J_zcf && J_pts), "NULL pointer");
  if (n_obs == 0) return B3R_OK;
  LinOpts o = make_opts(is_depth_log, 1.f, -1.f, 100.f, 0.5f, 1e-16f);
  const int g = grid_for(n_obs, kThreads);
  if (output_float64)
    k_jacobians<double><<<g, kThreads, 0, as_stream(stream)>>>(
        infos, n_imgs, K, P_rig2c, P_rig2c_stride, P_w2rig, z_coefs, C, pts3d, pids, n_obs,
        pix2d_std, pix2d_dep, o, (double*)J_cam, (double*)J_zcf, (double*)J_pts);
  else
    k_jacobians<float><<<g, kThreads, 0, as_stream(stream)>>>(
        infos, n_imgs, K, P_rig2c, P_rig2c_stride, P_w2rig, z_coefs, C, pts3d, pids, n_obs,
        pix2d_std, pix2d_dep, o, (float*)J_cam, (float*)J_zcf, (float*)J_pts);
  return check_launch("b3r_jacobians_with_rigs");
}

extern "C" int b3r_chol3x3_solve(const void* blocks, const void* rhs, void* out, int64_t N,
                                 double jitter, int dtype, void* stream) {
  B3R_REQUIRE(N >= 0, "N must be >= 0");
  B3R_REQUIRE(dtype == B3R_F32 || dtype == B3R_F64, "dtype must be B3R_F32 or B3R_F64");
  if (N == 0) return B3R_OK;
  B3R_REQUIRE(blocks && rhs && out, "NULL pointer");
  const int g = grid_for(N, kThreads);
  if (dtype == B3R_F64)
    k_chol3x3_solve<double><<<g, kThreads, 0, as_stream(stream)>>>((const double*)blocks,
                                                                   (const double*)rhs, (double*)out, N, jitter);
  else
    k_chol3x3_solve<float><<<g, kThreads, 0, as_stream(stream)>>>((const float*)blocks, (const float*)rhs,
                                                                  (float*)out, N, (float)jitter);
  return check_launch("b3r_chol3x3_solve");
}

extern "C" int b3r_blockcoo_matvec(const void* blocks, int bh, int bw, const void* row_idx,
                                   const void* col_idx, int index_is_64, int64_t N, const void* x,
                                   void* y, int64_t HB1, int64_t WB1, int transpose, int dtype,
                                   void* stream) {
  B3R_REQUIRE(bh >= 1 && bh <= 32 && bw >= 1 && bw <= 32, "block shape (%d,%d) out of range", bh, bw);
  B3R_REQUIRE(N >= 0 && HB1 >= 0 && WB1 >= 0, "bad sizes");
  B3R_REQUIRE(dtype == B3R_F32 || dtype == B3R_F64, "dtype must be B3R_F32 or B3R_F64");
  const int64_t out_len = transpose ? WB1 * bw : HB1 * bh;
  const size_t es = dtype == B3R_F64 ? 8 : 4;
  cudaStream_t s = as_stream(stream);
  if (out_len > 0) {
    B3R_REQUIRE(y != nullptr, "NULL y");
    B3R_TRY(check_cuda(cudaMemsetAsync(y, 0, out_len * es, s), "b3r_blockcoo_matvec memset"));
  }
  if (N == 0) return B3R_OK;
  B3R_REQUIRE(blocks && row_idx && col_idx && x, "NULL pointer");
  const int64_t total = N * (transpose ? bw : bh);
  const int g = (int)std::min<int64_t>(grid_for(total, kThreads), 148 * 64);
#define B3R_BCOO(T, I)                                                                            \
  k_bcoo_matvec<T, I><<<g, kThreads, 0, s>>>((const T*)blocks, bh, bw, (const I*)row_idx,        \
                                             (const I*)col_idx, N, (const T*)x, (T*)y, transpose)
  if (dtype == B3R_F64) { if (index_is_64) B3R_BCOO(double, int64_t); else B3R_BCOO(double, int32_t); }
  else                  { if (index_is_64) B3R_BCOO(float, int64_t);  else B3R_BCOO(float, int32_t); }
#undef B3R_BCOO
  return check_launch("b3r_blockcoo_matvec");
}

extern "C" int b3r_fused_einsum_bki_bkj(const void* left, int64_t l_bs, int64_t l_ks,
                                        const void* right, int64_t r_bs, int64_t r_ks, void* out,
                                        int64_t B, int K, int I, int J, int dtype, void* stream) {
  B3R_REQUIRE(B >= 0 && K >= 1 && I >= 1 && J >= 1 && (int64_t)I * J <= 1024, "bad sizes");
  B3R_REQUIRE(dtype == B3R_F32 || dtype == B3R_F64, "dtype must be B3R_F32 or B3R_F64");
  if (B == 0) return B3R_OK;
  B3R_REQUIRE(left && right && out, "NULL pointer");
  const int g = grid_for(B * I * J, kThreads);
  if (dtype == B3R_F64)
    k_einsum_bki_bkj<double><<<g, kThreads, 0, as_stream(stream)>>>(
        (const double*)left, l_bs, l_ks, (const double*)right, r_bs, r_ks, (double*)out, B, K, I, J);
  else
    k_einsum_bki_bkj<float><<<g, kThreads, 0, as_stream(stream)>>>(
        (const float*)left, l_bs, l_ks, (const float*)right, r_bs, r_ks, (float*)out, B, K, I, J);
  return check_launch("b3r_fused_einsum_bki_bkj");
}
