// Part 3 of the C ABI: preconditioned conjugate gradient on the assembled Schur system.
//
// The reference solves S delta_c = b with a minimal PCG (naver/blast3r
// src/blast3r/inference/ba_solver.py:1197-1238, called at :202 with tol 1e-6 and maxiter
// 300): x0 = 0, Jacobi preconditioner, stop at the first iterate with ||r|| <= tol ||b||
// (returned), break on a non-finite r.z, else return the best-so-far iterate.  Each of its
// iterations is a dozen small launches with a host synchronisation.  Here the whole loop is
// ONE cooperative kernel: a grid-wide barrier (bounded spin, co-residency guaranteed by the
// cooperative launch) separates
//   phase A  the decisions on the previous iterate (best-so-far copy, convergence,
//            non-finite break, beta), p = z + beta p computed on the fly inside the matvec
//            Ap = S p (symmetric block rows cut into <= 64-entry warp tasks; a row of several
//            tasks adds its parts atomically) and the partial sums of p.Ap
//   phase B  x += alpha p, r -= alpha Ap, z = r / M and the partial sums of r.r and r.z
// so an iteration costs two barriers.  Vectors are float or double (the solver's dtype);
// reductions accumulate in double.
#include <algorithm>
#include <cstring>
#include "b3r_common.cuh"
#include "b3r_plan.h"
#include "b3r_status.h"

namespace b3r {
namespace {

constexpr int kPcgThreads = 256;
constexpr int kBarrierSpins = 1 << 24;   // polls before a grid barrier gives up

// Scalars and barrier words at the start of the work buffer (doubles).
struct PcgScalars {
  double pAp[2], rr[2], rz[2];   // partial-sum slots, by iteration parity
  double bb, rz0;                // ||b||^2 and r0.z0 of the prologue
  unsigned int bar_count, bar_gen, abort_flag, pad;
};

// Sense-counting grid barrier for a cooperative launch: the last block to arrive resets the
// count and bumps the generation; the others poll the generation, at most kBarrierSpins
// times.  Returns false (and raises abort_flag) if the poll gave up; every block checks
// abort_flag after each barrier, so all of them leave the loop together.
__device__ __forceinline__ bool grid_barrier(PcgScalars* sc, unsigned int& gen) {
  __shared__ int ok_s;
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 1;
    const unsigned int g = gen;
    __threadfence();
    const unsigned int arrived = atomicAdd(&sc->bar_count, 1u) + 1u;
    if (arrived == gridDim.x) {
      atomicExch(&sc->bar_count, 0u);
      __threadfence();
      atomicAdd(&sc->bar_gen, 1u);
    } else {
      volatile unsigned int* vg = &sc->bar_gen;
      int spins = 0;
      while (*vg == g) {
        if (++spins > kBarrierSpins) { ok = 0; atomicExch(&sc->abort_flag, 1u); break; }
        __nanosleep(64);
      }
    }
    __threadfence();
    gen = g + 1;
    ok_s = ok && (*(volatile unsigned int*)&sc->abort_flag == 0u);
  }
  __syncthreads();
  return ok_s != 0;
}

template <typename T>
__device__ __forceinline__ double block_sum(double v, double* red) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  double t = 0.0;
  if (threadIdx.x == 0)
    for (int i = 0; i < kPcgThreads / 32; ++i) t += red[i];
  return t;   // valid on thread 0
}

// The lanes of a warp compute the part of y_p = sum_q A_pq x_q over the symmetric entries
// [e0, e1) of block row p, with x_q = z_q + beta * pold_q formed on the fly (all of an
// entry's column values are loaded before its products); every lane returns the partial
// y_p[r] (r < bp) in yo.
template <typename T, int MAXB>
__device__ __forceinline__ void task_matvec(const DevPlan& d, const float* __restrict__ S, int bp, int e0, int e1,
                                            const T* __restrict__ z, const T* __restrict__ pold, T beta, int lane,
                                            T yo[MAXB]) {
  T y[MAXB];
#pragma unroll
  for (int r = 0; r < MAXB; ++r) y[r] = T(0);
  for (int e = e0 + lane; e < e1; e += 32) {
    const int4 en = __ldg(d.mv_ent + e);                 // value offset, column offset, bq, transposed
    const float* A = S + en.x;
    const int oq = en.y, bq = en.z;
    T xq[MAXB];
#pragma unroll
    for (int cc = 0; cc < MAXB; ++cc)                    // other blocks wrote z and pold: L2 reads
      xq[cc] = cc < bq ? __ldcg(z + oq + cc) + beta * __ldcg(pold + oq + cc) : T(0);
    if (en.w) {
#pragma unroll
      for (int cc = 0; cc < MAXB; ++cc)
#pragma unroll
        for (int r = 0; r < MAXB; ++r)
          if (cc < bq && r < bp) y[r] += (T)__ldg(A + cc * bp + r) * xq[cc];
    } else {
#pragma unroll
      for (int r = 0; r < MAXB; ++r)
#pragma unroll
        for (int cc = 0; cc < MAXB; ++cc)
          if (cc < bq && r < bp) y[r] += (T)__ldg(A + r * bq + cc) * xq[cc];
    }
  }
#pragma unroll
  for (int r = 0; r < MAXB; ++r) {
    T v = y[r];
#pragma unroll
    for (int dd = 16; dd > 0; dd >>= 1) v += __shfl_xor_sync(0xffffffffu, v, dd);
    yo[r] = v;
  }
}

template <typename T, int MAXB>
__global__ void __launch_bounds__(kPcgThreads) k_pcg(DevPlan d, const float* __restrict__ S,
                                                     const float* __restrict__ M, const T* __restrict__ b,
                                                     T* __restrict__ xo, double tol, int maxiter, T* vec,
                                                     PcgScalars* sc, int* result) {
  __shared__ double red[kPcgThreads / 32];
  const int n = d.n_cam_params;
  T* x = vec;                 // iterate (each element owned by one thread)
  T* r = vec + n;             // residual (owned)
  T* z = vec + 2 * (int64_t)n;        // preconditioned residual (owned; read by the matvec)
  T* Ap = vec + 3 * (int64_t)n;       // S p (written by the matvec warps)
  T* pbuf0 = vec + 4 * (int64_t)n;    // search direction, double-buffered by iteration parity
  T* pbuf1 = vec + 5 * (int64_t)n;
  T* bx = vec + 6 * (int64_t)n;       // best-so-far iterate (owned)
  const int tid = blockIdx.x * blockDim.x + threadIdx.x, nth = gridDim.x * blockDim.x;
  const int lane = threadIdx.x & 31;
  const int gw = tid >> 5, nwarps = nth >> 5;
  unsigned int gen = 0;
  if (threadIdx.x == 0) gen = *(volatile unsigned int*)&sc->bar_gen;

  // prologue: x0 = 0, r0 = b - S x0 = b, z0 = M^-1 r0, p = z0 (formed on the fly from p_old = 0)
  double s_rz = 0.0, s_bb = 0.0;
  for (int i = tid; i < n; i += nth) {
    const T bi = b[i], zi = bi / (T)M[i];
    x[i] = T(0); r[i] = bi; z[i] = zi; pbuf0[i] = T(0); pbuf1[i] = T(0); bx[i] = T(0); Ap[i] = T(0);
    s_rz += (double)bi * (double)zi;
    s_bb += (double)bi * (double)bi;
  }
  double t = block_sum<T>(s_rz, red);
  if (threadIdx.x == 0) atomicAdd(&sc->rz0, t);
  t = block_sum<T>(s_bb, red);
  if (threadIdx.x == 0) atomicAdd(&sc->bb, t);
  bool ok = grid_barrier(sc, gen);

  double rz_old = __ldcg(&sc->rz0);
  const double bnorm = fmax(sqrt(__ldcg(&sc->bb)), 1e-12);
  double best = __longlong_as_double(0x7ff0000000000000LL);   // +inf
  int best_k = 0, k_stop = 0;
  bool converged = false;
  for (int k = 1; ok && k <= maxiter + 1; ++k) {
    // ---- phase A: decisions on iterate k-1 (identical in every thread) ----
    double beta = 0.0;
    if (k > 1) {
      const double rn = sqrt(__ldcg(&sc->rr[(k - 1) & 1]));
      const double rz_new = __ldcg(&sc->rz[(k - 1) & 1]);
      if (rn < best) {                                   // best-so-far iterate
        best = rn;
        best_k = k - 1;
        for (int i = tid; i < n; i += nth) bx[i] = x[i];
      }
      if (rn <= tol * bnorm) { converged = true; k_stop = k - 1; break; }
      if (!isfinite(rz_new)) break;
      beta = rz_new / fmax(rz_old, 1e-32);
      rz_old = rz_new;
    }
    if (k > maxiter) break;
    const T* pold = (k & 1) ? pbuf0 : pbuf1;
    T* pnew = (k & 1) ? pbuf1 : pbuf0;
    const T tb = (T)beta;
    double s_pap = 0.0;
    for (int task = gw; task < d.n_mv_tasks; task += nwarps) {   // warp per matvec task
      const int4 tk = __ldg(d.mv_task + task);           // block row, entries [e0, e1), single
      const int p = tk.x, bp = d.bsize[p], op = d.boff[p];
      T yo[MAXB];
      task_matvec<T, MAXB>(d, S, bp, tk.y, tk.z, z, pold, tb, lane, yo);
      const bool first = tk.y == d.sym_ptr[p];
#pragma unroll
      for (int rr = 0; rr < MAXB; ++rr) {
        if (lane == rr && rr < bp) {
          const T pn = __ldcg(z + op + rr) + tb * __ldcg(pold + op + rr);
          if (tk.w) Ap[op + rr] = yo[rr];                // the row is one task
          else atomicAdd(Ap + op + rr, yo[rr]);          // zeroed by the previous phase B
          if (first) pnew[op + rr] = pn;
          s_pap += (double)pn * (double)yo[rr];          // p.Ap is linear in the row's tasks
        }
      }
    }
    t = block_sum<T>(s_pap, red);
    if (threadIdx.x == 0) atomicAdd(&sc->pAp[k & 1], t);
    if (!(ok = grid_barrier(sc, gen))) break;
    // ---- phase B: x, r, z and the partial sums of r.r, r.z ----
    const double alpha = rz_old / fmax(__ldcg(&sc->pAp[k & 1]), 1e-32);
    const T ta = (T)alpha;
    double s_rr = 0.0;
    s_rz = 0.0;
    for (int i = tid; i < n; i += nth) {
      const T xi = x[i] + ta * __ldcg(pnew + i);
      const T ri = r[i] - ta * __ldcg(Ap + i);
      Ap[i] = T(0);                                      // for the next matvec's atomics
      const T zi = ri / (T)M[i];
      x[i] = xi; r[i] = ri; z[i] = zi;
      s_rr += (double)ri * (double)ri;
      s_rz += (double)ri * (double)zi;
    }
    if (tid == 0) {            // the slots the next iteration accumulates into (last read before now)
      sc->pAp[(k + 1) & 1] = 0.0;
      sc->rr[(k + 1) & 1] = 0.0;
      sc->rz[(k + 1) & 1] = 0.0;
    }
    t = block_sum<T>(s_rr, red);
    if (threadIdx.x == 0) atomicAdd(&sc->rr[k & 1], t);
    t = block_sum<T>(s_rz, red);
    if (threadIdx.x == 0) atomicAdd(&sc->rz[k & 1], t);
    ok = grid_barrier(sc, gen);
  }
  // the converging iterate, else the best-so-far one (zeros if none improved)
  for (int i = tid; i < n; i += nth) xo[i] = ok ? (converged ? x[i] : bx[i]) : T(0);
  if (tid == 0) {
    result[0] = converged ? k_stop : best_k;
    result[1] = converged ? 1 : 0;
    result[2] = ok ? 0 : 1;     // 1: a grid barrier gave up
  }
}

template <typename T, int MAXB>
int pcg_launch(const b3r_plan* plan, const float* S, const float* M, const T* b, T* xo, double tol, int maxiter,
               void* work, int* result, cudaStream_t s) {
  const DevPlan& d = plan->d;
  static int per_sm = 0, n_sm = 0;         // one occupancy query per instantiation
  if (per_sm == 0) {
    int dev = 0;
    B3R_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
    B3R_TRY(check_cuda(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev), "SM count"));
    B3R_TRY(check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_pcg<T, MAXB>, kPcgThreads, 0),
                       "pcg occupancy"));
    B3R_REQUIRE(per_sm >= 1, "the PCG kernel does not fit on an SM");
  }
  const int want = (d.n_mv_tasks * 32 + kPcgThreads - 1) / kPcgThreads;   // one warp per matvec task
  const int grid = std::max(1, std::min(want, per_sm * n_sm));     // all co-resident
  PcgScalars* sc = reinterpret_cast<PcgScalars*>(work);
  T* vec = reinterpret_cast<T*>(reinterpret_cast<char*>(work) + 256);
  B3R_TRY(check_cuda(cudaMemsetAsync(sc, 0, sizeof(PcgScalars), s), "clear PCG scalars"));
  DevPlan dv = d;
  void* args[] = {&dv, &S, &M, &b, &xo, &tol, &maxiter, &vec, &sc, &result};
  B3R_TRY(check_cuda(cudaLaunchCooperativeKernel((const void*)k_pcg<T, MAXB>, dim3(grid), dim3(kPcgThreads), args,
                                                 0, s),
                     "pcg cooperative launch"));
  return B3R_OK;
}

template <typename T>
int pcg_impl(const b3r_plan* plan, const float* S, const float* M, const T* b, T* xo, double tol, int maxiter,
             void* work, int* result, void* stream) {
  B3R_REQUIRE(plan && S && M && b && xo && work && result, "NULL argument");
  B3R_REQUIRE(((uintptr_t)work & 255) == 0, "PCG work buffer must be 256-byte aligned");
  B3R_REQUIRE(maxiter >= 0, "maxiter must be >= 0");
  int dev = -1;
  B3R_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  B3R_REQUIRE(dev == plan->device, "current device %d differs from the plan's device %d", dev, plan->device);
  if (plan->d.n_cam_params == 0) return B3R_OK;
  int maxb = 0;
  for (int v : plan->pat.bsize) maxb = std::max(maxb, v);
  cudaStream_t s = as_stream(stream);
  if (maxb <= 8) return pcg_launch<T, 8>(plan, S, M, b, xo, tol, maxiter, work, result, s);
  B3R_REQUIRE(maxb <= 32, "block size %d > 32", maxb);
  return pcg_launch<T, 32>(plan, S, M, b, xo, tol, maxiter, work, result, s);
}

}  // namespace
}  // namespace b3r

using namespace b3r;

extern "C" int64_t b3r_pcg_work_bytes(const b3r_plan* plan) {
  if (!plan) return -1;
  return 256 + 7 * 8 * (int64_t)plan->d.n_cam_params;
}

extern "C" int b3r_pcg(const b3r_plan* plan, const float* S_vals, const float* precond, const float* b, float* x,
                       double tol, int maxiter, void* work, int* result, void* stream) {
  return pcg_impl<float>(plan, S_vals, precond, b, x, tol, maxiter, work, result, stream);
}

extern "C" int b3r_pcg_f64(const b3r_plan* plan, const float* S_vals, const float* precond, const double* b,
                           double* x, double tol, int maxiter, void* work, int* result, void* stream) {
  return pcg_impl<double>(plan, S_vals, precond, b, x, tol, maxiter, work, result, stream);
}
