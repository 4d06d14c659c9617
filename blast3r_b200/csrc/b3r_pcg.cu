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
//            Ap = S p (row panels of the symmetric S, built once per solve, cut into
//            <= 256-column warp tasks; a row of several tasks adds its parts atomically)
//            and the partial sums of p.Ap
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

// Work buffer layout: barrier words | per-block arrival flags | per-block partial sums |
// the seven vectors.  Same-address atomics from every block serialise at one L2 slice, so
// neither the barrier nor the reductions use them: each block writes its own flag and its
// own partial sums, and every block sums all partials in the same fixed order.
constexpr int kPcgMaxBlocks = 1024;
constexpr size_t kPcgFlagsOff = 256, kPcgPartOff = kPcgFlagsOff + 4 * kPcgMaxBlocks;
constexpr size_t kPcgVecOff = kPcgPartOff + 4 * 8 * kPcgMaxBlocks;
static_assert(kPcgMaxBlocks % kPcgThreads == 0, "barrier flags per polling thread");

inline size_t pcg_panel_off(const DevPlan& d) {        // panels after the seven vectors
  return (kPcgVecOff + 7 * 8 * (size_t)d.n_cam_params + 255) & ~size_t(255);
}

struct PcgWords {
  unsigned int bar_gen, unused;
};
// per-block partial sums: [0] p.Ap, [1] r.r, [2] r.z (prologue: b.b and r0.z0)
struct PcgPart {
  double v[4];
};

constexpr unsigned int kGenAbort = 0x80000000u;   // in bar_gen: the barrier was abandoned
constexpr unsigned int kFlagAbort = 0xFFFFFFFFu;  // a block's flag once it gave up waiting

__device__ __forceinline__ void st_release(unsigned int* p, unsigned int v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int ld_acquire(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid barrier for a cooperative launch: after a block-wide __syncthreads, thread 0 of every
// block publishes its arrival with a release store flags[block] = target; block 0's threads
// acquire-poll the flags, then thread 0 of block 0 release-stores bar_gen = target, which
// thread 0 of every other block acquire-polls before a block-wide __syncthreads (the
// release/acquire pair and the CTA barriers order every thread's writes before the barrier
// with every thread's reads after it).  Every poll is bounded (kBarrierSpins).  A block
// that gives up waiting for bar_gen leaves with false and sets its flag to kFlagAbort; block
// 0, seeing such a flag or giving up on one, publishes bar_gen with kGenAbort, and every
// block that reads it leaves with false, so all of them leave the loop at this barrier or
// the next one.
__device__ __forceinline__ bool grid_barrier(PcgWords* w, unsigned int* flags, unsigned int target) {
  __shared__ int ok_s;
  __syncthreads();                                       // the block's writes precede its arrival
  if (threadIdx.x == 0) {
    ok_s = 1;
    st_release(flags + blockIdx.x, target);
  }
  __syncthreads();
  if (blockIdx.x == 0) {
    // each thread polls its (up to kPcgMaxBlocks / kPcgThreads) flags with loads issued
    // together, so a thread's second flag costs no extra round trip
    constexpr int kPer = kPcgMaxBlocks / kPcgThreads;
    bool bad = false;
    for (int spins = 0;; ++spins) {
      unsigned int f[kPer];
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        const int b = threadIdx.x + j * kPcgThreads;
        f[j] = b < (int)gridDim.x ? ld_acquire(flags + b) : target;
      }
      bool all = true;
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        if (f[j] == kFlagAbort) bad = true;
        if (f[j] < target) all = false;
      }
      if (all) break;
      if (spins >= kBarrierSpins) { bad = true; break; }
      __nanosleep(32);
    }
    if (bad) ok_s = 0;
    __syncthreads();
    if (threadIdx.x == 0) st_release(&w->bar_gen, target | (ok_s ? 0u : kGenAbort));
  } else if (threadIdx.x == 0) {
    int spins = 0;
    unsigned int g;
    while (((g = ld_acquire(&w->bar_gen)) & ~kGenAbort) < target) {
      if (++spins > kBarrierSpins) break;
      __nanosleep(32);
    }
    if ((g & ~kGenAbort) < target || (g & kGenAbort)) {
      ok_s = 0;
      st_release(flags + blockIdx.x, kFlagAbort);
    }
  }
  __syncthreads();
  return ok_s != 0;
}

// Sum of v over the block (valid on thread 0).
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
  return t;
}

// Sum over blocks of partial field f, the same fixed order in every block; broadcast to
// every thread of the block.
__device__ __forceinline__ double grid_sum(const PcgPart* part, int f, double* red, double* bcast) {
  double v = 0.0;
  for (int b = threadIdx.x; b < (int)gridDim.x; b += blockDim.x) v += __ldcg(&part[b].v[f]);
  const double t = block_sum(v, red);
  if (threadIdx.x == 0) *bcast = t;
  __syncthreads();
  return *bcast;
}

// Sums of (u, v) over the block (valid on thread 0).
__device__ __forceinline__ double2 block_sum2(double u, double v, double2* red2) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) {
    u += __shfl_xor_sync(0xffffffffu, u, d);
    v += __shfl_xor_sync(0xffffffffu, v, d);
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red2[w] = make_double2(u, v);
  __syncthreads();
  double2 t = make_double2(0.0, 0.0);
  if (threadIdx.x == 0)
    for (int i = 0; i < kPcgThreads / 32; ++i) { t.x += red2[i].x; t.y += red2[i].y; }
  return t;
}

// Sums over blocks of partial fields f and f + 1 in one pass, the same fixed order in every
// block; broadcast to every thread of the block.
__device__ __forceinline__ double2 grid_sum2(const PcgPart* part, int f, double2* red2, double2* bcast) {
  double u = 0.0, v = 0.0;
  for (int b = threadIdx.x; b < (int)gridDim.x; b += blockDim.x) {
    u += __ldcg(&part[b].v[f]);
    v += __ldcg(&part[b].v[f + 1]);
  }
  const double2 t = block_sum2(u, v, red2);
  if (threadIdx.x == 0) *bcast = t;
  __syncthreads();
  return *bcast;
}

// Row panels of the symmetric S (once per solve, before the PCG kernel): warp per
// symmetric entry, copying its block (transposed when the entry is the transpose of the
// stored block) into its block row's panel.
__global__ void __launch_bounds__(256) k_build_panels(DevPlan d, const float* __restrict__ S, float* __restrict__ pan) {
  const int e = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  const int n_ent = d.sym_ptr[d.nb];
  if (e >= n_ent) return;
  const int4 en = d.mv_ent[e];                           // value offset, column offset, bq, transposed
  const int p = d.ent_row[e], bp = d.bsize[p], bq = en.z, W = d.pan_w[p];
  float* dst = pan + d.pan_off[p] + d.ent_col[e];
  for (int t = lane; t < bp * bq; t += 32) {
    const int r = t / bq, c = t - r * bq;
    dst[(int64_t)r * W + c] = S[en.x + (en.w ? c * bp + r : r * bq + c)];
  }
}

// The lanes of a warp compute the part of y_p = sum_c panel_p[r][c] x[col_c] over panel
// columns [c0, c1) of block row p (panel P of width W, column list cols) (at most kMvCols = 256, so at most eight per lane), with
// x = z + beta * pold formed on the fly.  The panel rows are read coalesced (consecutive
// lanes, consecutive columns) and so mostly are the x values (a block's columns are
// consecutive scalars).  Every lane returns the partial y_p[r] (r < bp) in yo.
template <typename T, int MAXB>
__device__ __forceinline__ void panel_matvec(const float* __restrict__ P, const int* __restrict__ cols, int W, int bp,
                                             int c0, int c1, const T* __restrict__ z, const T* __restrict__ pold,
                                             T beta, int lane, T yo[MAXB]) {
  constexpr int CPL = kMvCols / 32;                      // columns per lane
  T xc[CPL];
  bool has[CPL];
#pragma unroll
  for (int j = 0; j < CPL; ++j) {
    const int c = c0 + lane + 32 * j;
    has[j] = c < c1;
    const int col = has[j] ? __ldg(cols + c) : 0;
    xc[j] = has[j] ? __ldcg(z + col) + beta * __ldcg(pold + col) : T(0);   // other blocks wrote them
  }
  T y[MAXB];
#pragma unroll
  for (int r = 0; r < MAXB; ++r) y[r] = T(0);
#pragma unroll
  for (int j = 0; j < CPL; ++j) {
    if (!has[j]) continue;
    const int c = c0 + lane + 32 * j;
#pragma unroll
    for (int r = 0; r < MAXB; ++r)
      if (r < bp) y[r] += (T)__ldg(P + (int64_t)r * W + c) * xc[j];
  }
#pragma unroll
  for (int r = 0; r < MAXB; ++r) {
    T v = y[r];
#pragma unroll
    for (int dd = 16; dd > 0; dd >>= 1) v += __shfl_xor_sync(0xffffffffu, v, dd);
    yo[r] = v;
  }
}

// Three blocks per SM (<= 85 registers): more resident warps than matvec tasks leaves fewer
// warps with two tasks, and the slowest warp sets each iteration's pace (8.0 vs 9.8 ms for
// the cfg2 solve with two blocks per SM).
template <typename T, int MAXB>
__global__ void __launch_bounds__(kPcgThreads, 3) k_pcg(DevPlan d, const float* __restrict__ S,
                                                     const float* __restrict__ M, const T* __restrict__ b,
                                                     T* __restrict__ xo, double tol, int maxiter, char* work,
                                                     const float* __restrict__ pan, int* result) {
  __shared__ double red[kPcgThreads / 32];
  __shared__ double bc;
  __shared__ double2 red2[kPcgThreads / 32];
  __shared__ double2 bc2;
  PcgWords* w = reinterpret_cast<PcgWords*>(work);
  unsigned int* flags = reinterpret_cast<unsigned int*>(work + kPcgFlagsOff);
  PcgPart* part = reinterpret_cast<PcgPart*>(work + kPcgPartOff);
  T* vec = reinterpret_cast<T*>(work + kPcgVecOff);
  const int n = d.n_cam_params;
  T* x = vec;                          // iterate (each element owned by one thread)
  T* r = vec + n;                      // residual (owned)
  T* z = vec + 2 * (int64_t)n;         // preconditioned residual (owned; read by the matvec)
  T* Ap = vec + 3 * (int64_t)n;        // S p (written by the matvec warps)
  T* pbuf0 = vec + 4 * (int64_t)n;     // search direction, double-buffered by iteration parity
  T* pbuf1 = vec + 5 * (int64_t)n;
  T* bx = vec + 6 * (int64_t)n;        // best-so-far iterate (owned)
  const int tid = blockIdx.x * blockDim.x + threadIdx.x, nth = gridDim.x * blockDim.x;
  const int lane = threadIdx.x & 31;
  const int gw = tid >> 5, nwarps = nth >> 5;
  unsigned int target = 0;

  // prologue: x0 = 0, r0 = b - S x0 = b, z0 = M^-1 r0, p = z0 (formed on the fly from p_old = 0)
  double s_rz = 0.0, s_bb = 0.0;
  for (int i = tid; i < n; i += nth) {
    const T bi = b[i], zi = bi / (T)M[i];
    x[i] = T(0); r[i] = bi; z[i] = zi; pbuf0[i] = T(0); pbuf1[i] = T(0); bx[i] = T(0); Ap[i] = T(0);
    s_rz += (double)bi * (double)zi;
    s_bb += (double)bi * (double)bi;
  }
  double2 t2 = block_sum2(s_bb, s_rz, red2);
  if (threadIdx.x == 0) { part[blockIdx.x].v[1] = t2.x; part[blockIdx.x].v[2] = t2.y; }
  bool ok = grid_barrier(w, flags, ++target);
  t2 = grid_sum2(part, 1, red2, &bc2);
  const double bnorm = fmax(sqrt(t2.x), 1e-12);
  double rz_old = t2.y;
  double rn = 0.0, rz_new = 0.0;

  double best = __longlong_as_double(0x7ff0000000000000LL);   // +inf
  int best_k = 0, k_stop = 0;
  bool converged = false;
  for (int k = 1; ok && k <= maxiter + 1; ++k) {
    // ---- phase A: decisions on iterate k-1 (identical in every thread) ----
    double beta = 0.0;
    if (k > 1) {
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
      const int4 tk = __ldg(d.mv_task + task);           // block row, panel columns [c0, c1), flags
      const int4 rw = __ldg(d.mv_row + task);            // boff, W, panel offset / 4, column-list offset
      const int bp = tk.w >> 8, op = rw.x;
      const bool single = tk.w & 1, first = tk.w & 2;
      // this lane's scalar of the row (lane < bp): its new search direction, loaded early
      const T pn = lane < bp ? __ldcg(z + op + lane) + tb * __ldcg(pold + op + lane) : T(0);
      T yo[MAXB];
      panel_matvec<T, MAXB>(pan + 4 * (int64_t)rw.z, d.pan_col + rw.w, rw.y, bp, tk.y, tk.z, z, pold, tb, lane, yo);
#pragma unroll
      for (int rr = 0; rr < MAXB; ++rr) {
        if (lane == rr && rr < bp) {
          if (single) Ap[op + rr] = yo[rr];              // the row is one task
          else atomicAdd(Ap + op + rr, yo[rr]);          // zeroed by the previous phase B
          if (first) pnew[op + rr] = pn;
          s_pap += (double)pn * (double)yo[rr];          // p.Ap is linear in the row's tasks
        }
      }
    }
    const double t = block_sum(s_pap, red);
    if (threadIdx.x == 0) part[blockIdx.x].v[0] = t;
    if (!(ok = grid_barrier(w, flags, ++target))) break;
    // ---- phase B: x, r, z and the partial sums of r.r and r.z ----
    const double alpha = rz_old / fmax(grid_sum(part, 0, red, &bc), 1e-32);
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
    t2 = block_sum2(s_rr, s_rz, red2);
    if (threadIdx.x == 0) { part[blockIdx.x].v[1] = t2.x; part[blockIdx.x].v[2] = t2.y; }
    if (!(ok = grid_barrier(w, flags, ++target))) break;
    t2 = grid_sum2(part, 1, red2, &bc2);
    rn = sqrt(t2.x);
    rz_new = t2.y;
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
#ifndef B3R_PCG_BLOCKS_PER_SM
#define B3R_PCG_BLOCKS_PER_SM 0   // 0: as many as fit (more blocks make each grid barrier dearer)
#endif
  const int cap = B3R_PCG_BLOCKS_PER_SM > 0 ? std::min(per_sm, B3R_PCG_BLOCKS_PER_SM) : per_sm;
  const int grid = std::max(1, std::min(want, cap * n_sm));        // all co-resident
  B3R_REQUIRE(grid <= kPcgMaxBlocks, "internal: PCG grid %d > %d", grid, kPcgMaxBlocks);
  // barrier words and arrival flags start at zero (targets count up from 1 in every launch)
  B3R_TRY(check_cuda(cudaMemsetAsync(work, 0, kPcgPartOff, s), "clear PCG barrier words"));
  DevPlan dv = d;
  char* wk = reinterpret_cast<char*>(work);
  float* pan = reinterpret_cast<float*>(wk + pcg_panel_off(d));
  const int n_ent = (int)(2 * d.nnzb - d.nb);             // symmetric entries
  k_build_panels<<<grid_for((int64_t)n_ent * 32, 256), 256, 0, s>>>(dv, S, pan);
  B3R_TRY(check_launch("pcg panels"));
  const float* panc = pan;
  void* args[] = {&dv, &S, &M, &b, &xo, &tol, &maxiter, &wk, &panc, &result};
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
  return (int64_t)pcg_panel_off(plan->d) + 4 * plan->d.pan_floats;
}

extern "C" int b3r_pcg(const b3r_plan* plan, const float* S_vals, const float* precond, const float* b, float* x,
                       double tol, int maxiter, void* work, int* result, void* stream) {
  return pcg_impl<float>(plan, S_vals, precond, b, x, tol, maxiter, work, result, stream);
}

extern "C" int b3r_pcg_f64(const b3r_plan* plan, const float* S_vals, const float* precond, const double* b,
                           double* x, double tol, int maxiter, void* work, int* result, void* stream) {
  return pcg_impl<double>(plan, S_vals, precond, b, x, tol, maxiter, work, result, stream);
}
