// Part 3 of the C ABI: preconditioned conjugate gradient on the assembled Schur system.
//
// The reference solves S delta_c = b with a minimal PCG (naver/blast3r
// src/blast3r/inference/ba_solver.py:1197-1238, called at :202 with tol 1e-6 and maxiter
// 300): x0 = 0, Jacobi preconditioner, stop at the first iterate with ||r|| <= tol ||b||
// (returned), break on a non-finite r.z, else return the best-so-far iterate.  Each of its
// iterations is a dozen small launches with a host synchronisation.  Here the whole loop is
// ONE cooperative kernel running the pipelined form of the same iteration (Ghysels and
// Vanroose, "Hiding global synchronization latency in the preconditioned conjugate gradient
// algorithm", Parallel Computing 40, 2014, algorithm 4): with u = M^-1 r, w = S u,
// m = M^-1 w, n = S m and the recurrences z = n + beta z, q = m + beta q, s = w + beta s,
// p = u + beta p, x += alpha p, r -= alpha s, u -= alpha q, w -= alpha z, the iterate, its
// residual and the reference's r.z are those of the standard iteration, while the dot
// products (r.u, w.u, r.r) and the matvec n = S m of one iteration depend only on the
// previous iteration's vectors.  So one grid barrier per iteration suffices:
//   after the barrier every block sums the previous iteration's partial dot products in the
//   same fixed order, takes the reference's decisions (best-so-far copy, convergence,
//   non-finite break), forms alpha and beta, computes n = S m for its row group (row panels
//   of the symmetric S, built once per solve, cut into <= 256-column warp tasks whose partial
//   row sums go to fixed shared-memory slots, summed in task order: deterministic), updates
//   its rows of the eight vectors and publishes its partial dot products.
// Each block row belongs to one block's row group, so the update of a row never waits for
// another block; only m, which every block's matvec reads, is kept in two buffers by
// iteration parity.  Vectors are float or double (the solver's dtype); reductions
// accumulate in double.
#include <algorithm>
#include <cstring>
#include "b3r_common.cuh"
#include "b3r_plan.h"
#include "b3r_status.h"

namespace b3r {
namespace {

constexpr int kPcgThreads = 256;
// Polls (each followed by a 32 ns sleep) before a grid barrier gives up: about half a
// second, far beyond any barrier of a running solve; b3r_pcg_ex takes another limit.
constexpr long long kBarrierSpins = 1 << 24;
constexpr int kPcgVectors = 11;      // double vectors in the work buffer

// Work buffer layout: barrier words | per-block arrival flags | per-block partial sums |
// the vectors.  Same-address atomics from every block serialise at one L2 slice, so
// neither the barrier nor the reductions use them: each block writes its own flag and its
// own partial sums, and every block sums all partials in the same fixed order.
constexpr int kPcgMaxBlocks = 1024;
constexpr size_t kPcgFlagsOff = 256, kPcgPartOff = kPcgFlagsOff + 4 * kPcgMaxBlocks;
constexpr size_t kPcgHelpOff = kPcgPartOff + 4 * 8 * kPcgMaxBlocks;   // helper flags, then helper sums
constexpr int kPcgSrcMax = 3;        // source vectors of one matvec pass
static_assert(kPcgMaxBlocks % kPcgThreads == 0, "barrier flags per polling thread");
static_assert(kPcgThreads == 32 * kPcgWarps, "PCG block size");

__host__ __device__ inline size_t pcg_hsum_off(const DevPlan& d) {         // helper partial row sums [help][src][32]
  return (kPcgHelpOff + 4 * (size_t)d.n_pcg_help + 255) & ~size_t(255);
}
__host__ __device__ inline size_t pcg_vec_off(const DevPlan& d) {
  return (pcg_hsum_off(d) + 8 * (size_t)d.n_pcg_help * kPcgSrcMax * 32 + 255) & ~size_t(255);
}
__host__ __device__ inline size_t pcg_panel_off(const DevPlan& d) {        // panels after the vectors
  return (pcg_vec_off(d) + kPcgVectors * 8 * (size_t)d.n_cam_params + 255) & ~size_t(255);
}

struct PcgWords {
  unsigned int bar_gen, unused;
};
// per-block partial sums of the next iteration's r.u, w.u and r.r (prologue: r0.u0, w0.u0, b.b)
struct PcgPart {
  double v[4];
};

struct BarrierCfg {
  long long spins;     // polls before a wait gives up
  bool unreachable;    // test mode: block 0 waits for an arrival no block ever makes
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
// with every thread's reads after it).  Every poll is bounded (cfg.spins).  A block
// that gives up waiting for bar_gen leaves with false and sets its flag to kFlagAbort; block
// 0, seeing such a flag or giving up on one, publishes bar_gen with kGenAbort, and every
// block that reads it leaves with false, so all of them leave the loop at this barrier or
// the next one.
// With cfg.unreachable (a test of the failure path) block 0 waits for flag values one
// generation beyond what any block publishes, so its wait always runs out.
// A block arriving with ok == false (a helper wait ran out) arrives with kFlagAbort, so that
// every block leaves at this barrier.
__device__ __forceinline__ bool grid_barrier(PcgWords* w, unsigned int* flags, unsigned int target,
                                             const BarrierCfg& cfg, bool arrive_ok) {
  __shared__ int ok_s;
  __syncthreads();                                       // the block's writes precede its arrival
  if (threadIdx.x == 0) {
    ok_s = arrive_ok ? 1 : 0;
    st_release(flags + blockIdx.x, arrive_ok ? target : kFlagAbort);
  }
  __syncthreads();
  if (blockIdx.x == 0) {
    // each thread polls its (up to kPcgMaxBlocks / kPcgThreads, blockDim.x >= kPcgThreads)
    // flags with loads issued together, so a thread's second flag costs no extra round trip
    constexpr int kPer = kPcgMaxBlocks / kPcgThreads;
    bool bad = false;
    for (int spins = 0;; ++spins) {
      unsigned int f[kPer];
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        const int b = threadIdx.x + j * (int)blockDim.x;
        f[j] = b < (int)gridDim.x ? ld_acquire(flags + b) : target;
      }
      bool all = true;
      const unsigned int want = cfg.unreachable ? target + 1 : target;
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        if (f[j] == kFlagAbort) bad = true;
        if (f[j] < want) all = false;
      }
      if (all) break;
      if (spins >= cfg.spins) { bad = true; break; }
      __nanosleep(32);
    }
    if (bad) ok_s = 0;
    __syncthreads();
    if (threadIdx.x == 0) st_release(&w->bar_gen, target | (ok_s ? 0u : kGenAbort));
  } else if (threadIdx.x == 0) {
    int spins = 0;
    unsigned int g;
    while (((g = ld_acquire(&w->bar_gen)) & ~kGenAbort) < target) {
      if (++spins > cfg.spins) break;
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

// The lanes of a warp compute the part of y_p = sum_c panel_p[r][c] v[col_c] over panel
// columns [c0, c1) of block row p (panel P of width W, column list cols; at most kMvCols =
// 256, so at most eight per lane), in double, with v = src[col] (or src[col] / M[col] when
// DIV).  The panel rows are read coalesced (consecutive lanes, consecutive columns) and so
// mostly are the v values (a block's columns are consecutive scalars).  Every lane returns
// the partial y_p[r] (r < bp) in yo.
template <typename TS, int MAXB, bool DIV>
__device__ __forceinline__ void panel_matvec(const float* __restrict__ P, const int* __restrict__ cols, int W, int bp,
                                             int c0, int c1, const TS* __restrict__ src, const float* __restrict__ M,
                                             int lane, double yo[MAXB]) {
  constexpr int CPL = kMvCols / 32;                      // columns per lane
  double xc[CPL];
  bool has[CPL];
#pragma unroll
  for (int j = 0; j < CPL; ++j) {
    const int c = c0 + lane + 32 * j;
    has[j] = c < c1;
    const int col = has[j] ? __ldg(cols + c) : 0;
    if (DIV) xc[j] = has[j] ? (double)src[col] / (double)__ldg(M + col) : 0.0;
    else     xc[j] = has[j] ? (double)__ldcg(src + col) : 0.0;   // other blocks wrote it
  }
  double y[MAXB];
#pragma unroll
  for (int r = 0; r < MAXB; ++r) y[r] = 0.0;
#pragma unroll
  for (int j = 0; j < CPL; ++j) {
    if (!has[j]) continue;
    const int c = c0 + lane + 32 * j;
#pragma unroll
    for (int r = 0; r < MAXB; ++r)
      if (r < bp) y[r] += (double)__ldg(P + (int64_t)r * W + c) * xc[j];
  }
#pragma unroll
  for (int r = 0; r < MAXB; ++r) {
    double v = y[r];
#pragma unroll
    for (int dd = 16; dd > 0; dd >>= 1) v += __shfl_xor_sync(0xffffffffu, v, dd);
    yo[r] = v;
  }
}

// The matvec of one row group over NS source vectors at once (the panel values are loaded
// once): every task's partial row sums go to its shared-memory slots slots[s][.].
template <typename TS, int MAXB, int NS, bool DIV>
__device__ __forceinline__ void group_matvec(const DevPlan& d, const float* __restrict__ pan, int4 g,
                                             const TS* const (&src)[NS], const float* __restrict__ M,
                                             double (*slots)[kPcgSlots]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int task = g.x + warp; task < g.y; task += kPcgWarps) {
    const int4 tk = __ldg(d.mv_task + task);             // block row, panel columns [c0, c1), flags
    const int4 rw = __ldg(d.mv_row + task);              // boff, W, panel offset / 4, column-list offset
    const int bp = tk.w >> 8, slot = __ldg(d.mv_slot + task);
#pragma unroll
    for (int sv = 0; sv < NS; ++sv) {
      double yo[MAXB];
      panel_matvec<TS, MAXB, DIV>(pan + 4 * (int64_t)rw.z, d.pan_col + rw.w, rw.y, bp, tk.y, tk.z, src[sv], M, lane,
                                  yo);
#pragma unroll
      for (int rr = 0; rr < MAXB; ++rr)
        if (lane == rr && rr < bp) slots[sv][slot + rr] = yo[rr];
    }
  }
}

// (S v)_j of scalar j of the current row group: its row's task slots summed in task order.
__device__ __forceinline__ double slot_sum(const DevPlan& d, int j, const double* slots) {
  const int2 sc = __ldg(d.pcg_scl + j);
  const int nt = sc.y & 0xffff, stride = sc.y >> 16;
  double v = 0.0;
  for (int t = 0; t < nt; ++t) v += slots[sc.x + t * stride];
  return v;
}

struct HelpCfg {
  unsigned int* flags;    // [n_pcg_help] generation of the last partial sums published
  double* sums;           // [n_pcg_help][kPcgSrcMax][32]
  long long spins;
};

// One matvec pass of the PCG over this block's row groups: y = S v for NS source vectors, and
// for every scalar j the block owns, on_scalar(j, y_0..y_{NS-1}).  Helper groups of a split
// row go first in every block (they never wait): they publish their partial row sums with a
// release store of the pass's generation; the owner of the row adds them, in helper order,
// after an acquire poll (bounded; a poll that runs out clears ok).
template <typename TS, int MAXB, int NS, bool DIV, typename F>
__device__ __forceinline__ void matvec_pass(const DevPlan& d, const float* __restrict__ pan,
                                            const TS* const (&src)[NS], const float* __restrict__ M,
                                            double (*slots)[kPcgSlots], const HelpCfg& hc, unsigned int gen, bool& ok,
                                            F&& on_scalar) {
  __shared__ int wait_ok;
  for (int pass = 0; pass < 2; ++pass) {               // 0: helper groups, 1: the others
    for (int gi = blockIdx.x; gi < d.n_pcg_groups; gi += gridDim.x) {
      const int4 h = __ldg(d.pcg_grp2 + gi);
      const bool helper = h.z >= 0;
      if (helper != (pass == 0)) continue;
      const int4 g = __ldg(d.pcg_grp + gi);
      group_matvec<TS, MAXB, NS, DIV>(d, pan, g, src, M, slots);
      __syncthreads();
      if (helper) {
        const int bp = h.w, nt = h.x;
        for (int idx = threadIdx.x; idx < NS * bp; idx += blockDim.x) {
          const int sv = idx / bp, r = idx - sv * bp;
          double v = 0.0;
          for (int t = 0; t < nt; ++t) v += slots[sv][t * bp + r];
          hc.sums[((int64_t)h.z * kPcgSrcMax + sv) * 32 + r] = v;
        }
        __syncthreads();
        if (threadIdx.x == 0) st_release(hc.flags + h.z, gen);
      } else {
        if (h.y > 0) {                                  // the owner of a split row waits for its helpers
          if (threadIdx.x == 0) wait_ok = 1;
          __syncthreads();
          if (threadIdx.x < h.y) {
            long long spins = 0;
            while (ld_acquire(hc.flags + h.x + threadIdx.x) < gen) {
              if (++spins > hc.spins) { wait_ok = 0; break; }
              __nanosleep(32);
            }
          }
          __syncthreads();
          if (!wait_ok) ok = false;
        }
        for (int j = g.z + threadIdx.x; j < g.w; j += blockDim.x) {
          double y[NS];
#pragma unroll
          for (int sv = 0; sv < NS; ++sv) y[sv] = slot_sum(d, j, slots[sv]);
          if (h.y > 0) {
            const int r = j - g.z;
            for (int i = 0; i < h.y; ++i)
#pragma unroll
              for (int sv = 0; sv < NS; ++sv) y[sv] += __ldcg(hc.sums + ((int64_t)(h.x + i) * kPcgSrcMax + sv) * 32 + r);
          }
          on_scalar(j, y);
        }
      }
      __syncthreads();
    }
  }
}

// Sums of (u, v, w) over the block (valid on thread 0).
__device__ __forceinline__ double3 block_sum3(double u, double v, double w, double3* red3) {
#pragma unroll
  for (int dd = 16; dd > 0; dd >>= 1) {
    u += __shfl_xor_sync(0xffffffffu, u, dd);
    v += __shfl_xor_sync(0xffffffffu, v, dd);
    w += __shfl_xor_sync(0xffffffffu, w, dd);
  }
  const int wp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red3[wp] = make_double3(u, v, w);
  __syncthreads();
  double3 t = make_double3(0.0, 0.0, 0.0);
  if (threadIdx.x == 0)
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) { t.x += red3[i].x; t.y += red3[i].y; t.z += red3[i].z; }
  return t;
}

// Sums over blocks of partial fields 0..2, the same fixed order in every block; broadcast to
// every thread of the block.
__device__ __forceinline__ double3 grid_sum3(const PcgPart* part, double3* red3, double3* bcast) {
  double u = 0.0, v = 0.0, w = 0.0;
  for (int b = threadIdx.x; b < (int)gridDim.x; b += blockDim.x) {
    u += __ldcg(&part[b].v[0]);
    v += __ldcg(&part[b].v[1]);
    w += __ldcg(&part[b].v[2]);
  }
  const double3 t = block_sum3(u, v, w, red3);
  if (threadIdx.x == 0) *bcast = t;
  __syncthreads();
  return *bcast;
}

// Three blocks per SM (<= 85 registers); the planner sizes the row groups for that many.
// TI is the type of b and x (the solver's dtype); the iteration runs in double either way.
template <typename TI, int MAXB>
__global__ void __launch_bounds__(kPcgThreads, kPcgBlocksPerSm) k_pcg(
    DevPlan d, const float* __restrict__ M, const TI* __restrict__ b, TI* __restrict__ xo, double tol, int maxiter,
    char* work, const float* __restrict__ pan, int* result, long long spin_limit, int test_flags) {
  __shared__ double slots[kPcgSrcMax][kPcgSlots];
  __shared__ double3 red3[kResWarps];
  __shared__ double3 bc3;
  PcgWords* wd = reinterpret_cast<PcgWords*>(work);
  unsigned int* flags = reinterpret_cast<unsigned int*>(work + kPcgFlagsOff);
  PcgPart* part = reinterpret_cast<PcgPart*>(work + kPcgPartOff);
  const HelpCfg hc{reinterpret_cast<unsigned int*>(work + kPcgHelpOff),
                   reinterpret_cast<double*>(work + pcg_hsum_off(d)), spin_limit};
  double* vec = reinterpret_cast<double*>(work + pcg_vec_off(d));
  const int64_t n = d.n_cam_params;
  double* x = vec;                     // every vector element is owned by the block of its row group
  double* r = vec + n;
  double* u = vec + 2 * n;
  double* w = vec + 3 * n;
  double* z = vec + 4 * n;
  double* q = vec + 5 * n;
  double* s = vec + 6 * n;
  double* p = vec + 7 * n;
  double* bx = vec + 8 * n;            // best-so-far iterate
  double* mb[2] = {vec + 9 * n, vec + 10 * n};   // m = M^-1 w by iteration parity (read by every block)
  BarrierCfg bcfg{spin_limit, (test_flags & 1) != 0};
  unsigned int target = 0, gen = 0;
  bool ok = true;
  auto publish = [&](double a, double b2, double c) {
    const double3 t = block_sum3(a, b2, c, red3);
    if (threadIdx.x == 0) { part[blockIdx.x].v[0] = t.x; part[blockIdx.x].v[1] = t.y; part[blockIdx.x].v[2] = t.z; }
  };
  auto own_scalars = [&](auto&& fn) {                  // the scalars of this block's row groups
    for (int gi = blockIdx.x; gi < d.n_pcg_groups; gi += gridDim.x) {
      const int4 g = __ldg(d.pcg_grp + gi);
      for (int j = g.z + threadIdx.x; j < g.w; j += blockDim.x) fn(j);
    }
  };

  // prologue: x0 = 0, r0 = b, u0 = M^-1 b, w0 = S u0, m0 = M^-1 w0, and the partial sums of
  // r0.u0, w0.u0, b.b
  double s_g = 0.0, s_d = 0.0, s_bb = 0.0;
  {
    const TI* const src[1] = {b};
    matvec_pass<TI, MAXB, 1, true>(d, pan, src, M, slots, hc, ++gen, ok, [&](int j, const double* y) {
      const double bj = (double)b[j], Mj = (double)M[j];
      const double uj = bj / Mj, wj = y[0];
      x[j] = 0.0; r[j] = bj; u[j] = uj; w[j] = wj; mb[0][j] = wj / Mj;
      z[j] = 0.0; q[j] = 0.0; s[j] = 0.0; p[j] = 0.0; bx[j] = 0.0;
      s_g += bj * uj;
      s_d += wj * uj;
      s_bb += bj * bj;
    });
  }
  publish(s_g, s_d, s_bb);
  ok = grid_barrier(wd, flags, ++target, bcfg, ok);
  double3 t3 = grid_sum3(part, red3, &bc3);
  double gamma = t3.x, delta = t3.y;
  const double bnorm = fmax(sqrt(t3.z), 1e-12);
  double rn = sqrt(t3.z), gamma_old = 0.0, alpha_old = 1.0;

  double best = __longlong_as_double(0x7ff0000000000000LL);   // +inf
  int best_k = 0, k_stop = 0, replaced = 0;
  bool converged = false;
  for (int k = 1; ok && k <= maxiter + 1; ++k) {
    // ---- decisions on iterate k-1 (x_{k-1}, r_{k-1}; identical in every thread) ----
    if (k > 1) {
      if (rn <= tol * bnorm) {
        // The recurrences' residual may drift from b - S x: confirm with the true residual
        // before stopping.  If it is not below the tolerance, the iteration continues from
        // true values (residual replacement): r = b - S x, u = M^-1 r, w = S u, s = S p,
        // z = S q, m = M^-1 w.
        double s_rr = 0.0;
        {
          const double* const src[1] = {x};
          matvec_pass<double, MAXB, 1, false>(d, pan, src, M, slots, hc, ++gen, ok, [&](int j, const double* y) {
            const double rj = (double)b[j] - y[0];
            r[j] = rj;
            u[j] = rj / (double)M[j];
            s_rr += rj * rj;
          });
        }
        publish(0.0, 0.0, s_rr);
        if (!(ok = grid_barrier(wd, flags, ++target, bcfg, ok))) break;
        t3 = grid_sum3(part, red3, &bc3);
        rn = sqrt(t3.z);
        if (rn <= tol * bnorm) { converged = true; k_stop = k - 1; break; }
        ++replaced;
        s_g = 0.0; s_d = 0.0;
        double* mc = mb[(k - 1) & 1];
        {
          const double* const src[3] = {u, p, q};
          matvec_pass<double, MAXB, 3, false>(d, pan, src, M, slots, hc, ++gen, ok, [&](int j, const double* y) {
            w[j] = y[0];
            s[j] = y[1];
            z[j] = y[2];
            mc[j] = y[0] / (double)M[j];
            s_g += r[j] * u[j];
            s_d += y[0] * u[j];
          });
        }
        publish(s_g, s_d, 0.0);
        if (!(ok = grid_barrier(wd, flags, ++target, bcfg, ok))) break;
        t3 = grid_sum3(part, red3, &bc3);
        gamma = t3.x;
        delta = t3.y;
      }
      if (rn < best) {                                   // best-so-far iterate
        best = rn;
        best_k = k - 1;
        own_scalars([&](int j) { bx[j] = x[j]; });
      }
      if (!isfinite(gamma)) break;                       // the reference's r.z
    }
    if (k > maxiter) break;
    // ---- iteration k-1 of the pipelined recurrences ----
    const double beta = k > 1 ? gamma / fmax(gamma_old, 1e-32) : 0.0;
    const double den = k > 1 ? delta - beta * gamma / alpha_old : delta;   // = p.S p
    const double alpha = gamma / fmax(den, 1e-32);
    double* mn = mb[k & 1];
    double s_rr = 0.0;
    s_g = 0.0; s_d = 0.0;
    {
      const double* const src[1] = {mb[(k - 1) & 1]};
      matvec_pass<double, MAXB, 1, false>(d, pan, src, M, slots, hc, ++gen, ok, [&](int j, const double* y) {
        const double nj = y[0], mj = src[0][j], wj = w[j], uj = u[j];
        const double zj = nj + beta * z[j], qj = mj + beta * q[j], sj = wj + beta * s[j], pj = uj + beta * p[j];
        const double xj = x[j] + alpha * pj, rj = r[j] - alpha * sj, un = uj - alpha * qj, wn = wj - alpha * zj;
        z[j] = zj; q[j] = qj; s[j] = sj; p[j] = pj;
        x[j] = xj; r[j] = rj; u[j] = un; w[j] = wn;
        mn[j] = wn / (double)M[j];
        s_g += rj * un;
        s_d += wn * un;
        s_rr += rj * rj;
      });
    }
    publish(s_g, s_d, s_rr);
    if (!(ok = grid_barrier(wd, flags, ++target, bcfg, ok))) break;
    t3 = grid_sum3(part, red3, &bc3);
    gamma_old = gamma;
    alpha_old = alpha;
    gamma = t3.x;
    delta = t3.y;
    rn = sqrt(t3.z);
  }
  // the converging iterate, else the best-so-far one (zeros if none improved or a wait gave up)
  own_scalars([&](int j) { xo[j] = ok ? (TI)(converged ? x[j] : bx[j]) : TI(0); });
  if (!ok && threadIdx.x == 0) atomicOr(result + 2, 1);   // any block that gave up flags the solve
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    result[0] = converged ? k_stop : best_k;
    result[1] = converged ? 1 : 0;
    result[3] = replaced;
  }
}

// ---------------------------------------------------------------------------------------
// The resident kernel: the same iteration, row groups and stopping rule as k_pcg, laid out for
// latency.  One block of kResThreads threads per SM and one row group per block.  The group's
// panel tiles and column lists are copied into shared memory once per solve (tasks that do not
// fit read the panel in global memory), and scalar j of the group lives in registers of thread
// j - (first scalar), so the only global traffic of an iteration is the gather of the previous
// m = M^-1 w by the panel columns, this block's new m, its partial sums and the barrier.  x,
// u, p and q are written to global memory only when the true residual is checked (the
// verification matvec reads x, the replacement matvecs read u, p, q).

struct ResTask {
  long long pbase;   // global panel: float index of the task's row 0, column c0
  int W;             // global panel row stride
  int cbase;         // global column list: index of the task's column c0
  int soff;          // word offset of the tile (bp x len, row-major) and columns in shared memory, -1: global
  int len, bp, slot;
};

// Sum over the warp of eight per-lane values: a reduce-scatter in nine shuffles.  Lane l ends
// with the sum of y[((l >> 4) & 1) * 4 + ((l >> 3) & 1) * 2 + ((l >> 2) & 1)].
__device__ __forceinline__ double warp_rsum8(const double (&y)[8], int lane) {
  double a[4], b2[2];
  const bool h16 = lane & 16, h8 = lane & 8, h4 = lane & 4;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const double keep = h16 ? y[i + 4] : y[i], send = h16 ? y[i] : y[i + 4];
    a[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const double keep = h8 ? a[i + 2] : a[i], send = h8 ? a[i] : a[i + 2];
    b2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  double c = (h4 ? b2[1] : b2[0]) + __shfl_xor_sync(0xffffffffu, h4 ? b2[0] : b2[1], 4);
  c += __shfl_xor_sync(0xffffffffu, c, 2);
  c += __shfl_xor_sync(0xffffffffu, c, 1);
  return c;
}

// Source value of panel column col: v[col] (or v[col] / M[col] for the prologue's M^-1 b).
template <typename TS, bool DIV>
__device__ __forceinline__ double res_src(const TS* __restrict__ src, const float* __restrict__ M, int col) {
  return DIV ? (double)src[col] / (double)__ldg(M + col) : (double)__ldcg(src + col);
}

// The source values a lane needs for one task.  A task in shared memory has its columns
// padded to lenp = a multiple of 64 (padding: column 0 of the task, zero panel values); lane l
// takes columns 2l, 2l + 1 of each 64-column step (xc[2 step], xc[2 step + 1]).  A task read
// from the global panel: lane l takes columns l + 32 j (xc[j]).
template <typename TS, bool DIV>
__device__ __forceinline__ void res_gather(const ResTask& tk, const float* sm, const int* __restrict__ pan_col,
                                           const TS* __restrict__ src, const float* __restrict__ M, int lane,
                                           double (&xc)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) xc[j] = 0.0;
  if (tk.soff >= 0) {
    const int lenp = (tk.len + 63) & ~63;
    const int2* cols = reinterpret_cast<const int2*>(sm + tk.soff + tk.bp * lenp);
#pragma unroll
    for (int st = 0; st < 4; ++st) {
      if (st * 64 >= lenp) break;
      const int2 cc = cols[st * 32 + lane];
      xc[2 * st] = res_src<TS, DIV>(src, M, cc.x);
      xc[2 * st + 1] = res_src<TS, DIV>(src, M, cc.y);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = lane + 32 * j;
      if (c < tk.len) xc[j] = res_src<TS, DIV>(src, M, __ldg(pan_col + tk.cbase + c));
    }
  }
}

// The row sums of one task into its slots: a shared-memory tile (two columns per lane per
// step, 8-byte loads, no per-element bounds; the row count is warp-uniform), or a tile read
// from the global panel.
__device__ __forceinline__ void res_task(const ResTask& tk, const float* sm, const float* __restrict__ pan,
                                         double (&xc)[8], int lane, double* slots) {
  double y[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) y[r] = 0.0;
  if (tk.soff >= 0) {
    const int lenp = (tk.len + 63) & ~63;
    const float2* P = reinterpret_cast<const float2*>(sm + tk.soff) + lane;
#pragma unroll 1
    for (int st = 0; st < lenp; st += 64) {            // the step's values are xc[0], xc[1]
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        if (r >= tk.bp) break;
        const float2 pv = P[(r * lenp + st) >> 1];
        y[r] = fma((double)pv.x, xc[0], y[r]);
        y[r] = fma((double)pv.y, xc[1], y[r]);
      }
#pragma unroll
      for (int j = 0; j < 6; ++j) xc[j] = xc[j + 2];
    }
  } else {
    const float* P = pan + tk.pbase;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = lane + 32 * j;
      if (c >= tk.len) continue;
#pragma unroll
      for (int r = 0; r < 8; ++r)
        if (r < tk.bp) y[r] = fma((double)__ldg(P + (int64_t)r * tk.W + c), xc[j], y[r]);
    }
  }
  const double v = warp_rsum8(y, lane);
  const int row = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
  if ((lane & 3) == 0 && row < tk.bp) slots[tk.slot + row] = v;
}

// The group's matvec over one source vector: warp w takes tasks w, w + 16, ...; every task's
// partial row sums go to its shared-memory slots.
template <typename TS, bool DIV>
__device__ __forceinline__ void res_matvec(const ResTask* tasks, int ntask, const float* sm,
                                           const float* __restrict__ pan, const int* __restrict__ pan_col,
                                           const TS* __restrict__ src, const float* __restrict__ M, double* slots) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int t0 = warp; t0 < ntask; t0 += kResWarps) {
    double xa[8];
    const ResTask ta = tasks[t0];
    res_gather<TS, DIV>(ta, sm, pan_col, src, M, lane, xa);
    res_task(ta, sm, pan, xa, lane, slots);
  }
}

struct ResGroup {
  int4 g, h;          // pcg_grp, pcg_grp2 of the block's group
  int ntask;
  bool helper, own;   // a helper group; this thread owns scalar g.z + threadIdx.x
  int2 sc;            // the owned scalar's slot map
};

// One matvec pass of the resident kernel: (S v)_j for the scalar this thread owns (0 for the
// others).  Helper groups publish their row sums (source slot sv of their helper record) with a
// release store of gen; the owner of a split row adds them, in helper order, after a bounded
// acquire poll.
template <typename TS, bool DIV>
__device__ __forceinline__ double res_pass(const DevPlan& d, const ResGroup& rg, const ResTask* tasks, const float* sm,
                                           const float* __restrict__ pan, const TS* __restrict__ src,
                                           const float* __restrict__ M, double* slots, const HelpCfg& hc, int sv,
                                           unsigned int gen, bool& ok, int* wait_ok) {
  res_matvec<TS, DIV>(tasks, rg.ntask, sm, pan, d.pan_col, src, M, slots);
  __syncthreads();
  double y = 0.0;
  if (rg.helper) {
    const int bp = rg.h.w, nt = rg.h.x;
    if ((int)threadIdx.x < bp) {
      double v = 0.0;
      for (int t = 0; t < nt; ++t) v += slots[t * bp + threadIdx.x];
      hc.sums[((int64_t)rg.h.z * kPcgSrcMax + sv) * 32 + threadIdx.x] = v;
    }
    __syncthreads();
    if (threadIdx.x == 0) st_release(hc.flags + rg.h.z, gen);
  } else {
    if (rg.h.y > 0) {                                  // the owner of a split row waits for its helpers
      if (threadIdx.x == 0) *wait_ok = 1;
      __syncthreads();
      if ((int)threadIdx.x < rg.h.y) {
        long long spins = 0;
        while (ld_acquire(hc.flags + rg.h.x + threadIdx.x) < gen) {
          if (++spins > hc.spins) { *wait_ok = 0; break; }
          __nanosleep(32);
        }
      }
      __syncthreads();
      if (!*wait_ok) ok = false;
    }
    if (rg.own) {
      const int nt = rg.sc.y & 0xffff, stride = rg.sc.y >> 16;
      for (int t = 0; t < nt; ++t) y += slots[rg.sc.x + t * stride];
      for (int i = 0; i < rg.h.y; ++i)
        y += __ldcg(hc.sums + ((int64_t)(rg.h.x + i) * kPcgSrcMax + sv) * 32 + threadIdx.x);
    }
  }
  __syncthreads();                                     // the slots are reused by the next pass
  return y;
}

template <typename TI>
__global__ void __launch_bounds__(kResThreads, 1) k_pcg_res(
    DevPlan d, const float* __restrict__ M, const TI* __restrict__ b, TI* __restrict__ xo, double tol, int maxiter,
    char* work, const float* __restrict__ pan, int* result, long long spin_limit, int test_flags) {
  extern __shared__ __align__(16) float sm[];
  __shared__ double slots[kPcgSlots];
  __shared__ ResTask tasks[kPcgGroupTasks];
  __shared__ double3 red3[kResWarps];
  __shared__ double3 bc3;
  __shared__ int wait_ok;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  ResGroup rg;
  rg.g = __ldg(d.pcg_grp + blockIdx.x);
  rg.h = __ldg(d.pcg_grp2 + blockIdx.x);
  rg.ntask = rg.g.y - rg.g.x;
  rg.helper = rg.h.z >= 0;
  const int j = rg.g.z + threadIdx.x;                  // the scalar this thread owns
  rg.own = !rg.helper && j < rg.g.w;
  rg.sc = rg.own ? __ldg(d.pcg_scl + j) : make_int2(0, 0);
  // the group's task records, then its tiles and column lists
  for (int t = threadIdx.x; t < rg.ntask; t += blockDim.x) {
    const int4 tk = __ldg(d.mv_task + rg.g.x + t), rw = __ldg(d.mv_row + rg.g.x + t);
    ResTask r;
    r.pbase = 4LL * rw.z + tk.y;
    r.W = rw.y;
    r.cbase = rw.w + tk.y;
    r.soff = (test_flags & B3R_PCG_TEST_GLOBAL_TILES) ? -1 : __ldg(d.mv_soff + rg.g.x + t);
    r.len = tk.z - tk.y;
    r.bp = tk.w >> 8;
    r.slot = __ldg(d.mv_slot + rg.g.x + t);
    tasks[t] = r;
  }
  __syncthreads();
  for (int t = warp; t < rg.ntask; t += kResWarps) {
    const ResTask r = tasks[t];
    if (r.soff < 0) continue;
    const int lenp = (r.len + 63) & ~63;
    for (int rr = 0; rr < r.bp; ++rr)
      for (int c = lane; c < lenp; c += 32)
        sm[r.soff + rr * lenp + c] = c < r.len ? __ldg(pan + r.pbase + (int64_t)rr * r.W + c) : 0.f;
    int* cs = reinterpret_cast<int*>(sm + r.soff + r.bp * lenp);
    const int c0 = __ldg(d.pan_col + r.cbase);
    for (int c = lane; c < lenp; c += 32) cs[c] = c < r.len ? __ldg(d.pan_col + r.cbase + c) : c0;
  }
  __syncthreads();

  PcgWords* wd = reinterpret_cast<PcgWords*>(work);
  unsigned int* flags = reinterpret_cast<unsigned int*>(work + kPcgFlagsOff);
  PcgPart* part = reinterpret_cast<PcgPart*>(work + kPcgPartOff);
  const HelpCfg hc{reinterpret_cast<unsigned int*>(work + kPcgHelpOff),
                   reinterpret_cast<double*>(work + pcg_hsum_off(d)), spin_limit};
  double* vec = reinterpret_cast<double*>(work + pcg_vec_off(d));
  const int64_t n = d.n_cam_params;
  double* const mb0 = vec;             // m = M^-1 w by iteration parity (read by every block)
  double* const mb1 = vec + n;
  double* xg = vec + 2 * n;            // x, u, p, q published for the true-residual check
  double* ug = vec + 3 * n;
  double* pg = vec + 4 * n;
  double* qg = vec + 5 * n;
  BarrierCfg bcfg{spin_limit, (test_flags & B3R_PCG_TEST_UNREACHABLE_BARRIER) != 0};
  unsigned int target = 0, gen = 0;
  bool ok = true;
  auto publish = [&](double a, double b2, double c) {
    const double3 t = block_sum3(a, b2, c, red3);
    if (threadIdx.x == 0) { part[blockIdx.x].v[0] = t.x; part[blockIdx.x].v[1] = t.y; part[blockIdx.x].v[2] = t.z; }
  };
  // the owned scalar's elements of b, M and of the iteration's vectors
  const double bj = rg.own ? (double)b[j] : 0.0, Mj = rg.own ? (double)M[j] : 1.0;
  double xj = 0.0, rj = bj, uj = bj / Mj, wj = 0.0, zj = 0.0, qj = 0.0, sj = 0.0, pj = 0.0, bxj = 0.0, mj = 0.0;

  // prologue: w0 = S u0, m0 = M^-1 w0, and the partial sums of r0.u0, w0.u0, b.b
  double s_g = 0.0, s_d = 0.0, s_bb = 0.0;
  {
    const double y = res_pass<TI, true>(d, rg, tasks, sm, pan, b, M, slots, hc, 0, ++gen, ok, &wait_ok);
    if (rg.own) {
      wj = y;
      mj = wj / Mj;
      mb0[j] = mj;
      s_g = bj * uj;
      s_d = wj * uj;
      s_bb = bj * bj;
    }
  }
  publish(s_g, s_d, s_bb);
  ok = grid_barrier(wd, flags, ++target, bcfg, ok);
  double3 t3 = grid_sum3(part, red3, &bc3);
  double gamma = t3.x, delta = t3.y;
  const double bnorm = fmax(sqrt(t3.z), 1e-12);
  double rn = sqrt(t3.z), gamma_old = 0.0, alpha_old = 1.0;

  double best = __longlong_as_double(0x7ff0000000000000LL);   // +inf
  int best_k = 0, k_stop = 0, replaced = 0;
  bool converged = false;
  for (int k = 1; ok && k <= maxiter + 1; ++k) {
    // ---- decisions on iterate k-1 (identical in every thread) ----
    if (k > 1) {
      if (rn <= tol * bnorm) {
        // confirm with the true residual r = b - S x; if it misses the tolerance, continue
        // from true values: u = M^-1 r, w = S u, s = S p, z = S q, m = M^-1 w
        if (rg.own) xg[j] = xj;
        if (!(ok = grid_barrier(wd, flags, ++target, bcfg, ok))) break;
        double s_rr = 0.0;
        {
          const double y = res_pass<double, false>(d, rg, tasks, sm, pan, xg, M, slots, hc, 0, ++gen, ok, &wait_ok);
          if (rg.own) {
            rj = bj - y;
            uj = rj / Mj;
            s_rr = rj * rj;
            ug[j] = uj;
            pg[j] = pj;
            qg[j] = qj;
          }
        }
        publish(0.0, 0.0, s_rr);
        if (!(ok = grid_barrier(wd, flags, ++target, bcfg, ok))) break;
        t3 = grid_sum3(part, red3, &bc3);
        rn = sqrt(t3.z);
        if (rn <= tol * bnorm) { converged = true; k_stop = k - 1; break; }
        ++replaced;
        const double yu = res_pass<double, false>(d, rg, tasks, sm, pan, ug, M, slots, hc, 0, ++gen, ok, &wait_ok);
        const double yp = res_pass<double, false>(d, rg, tasks, sm, pan, pg, M, slots, hc, 1, ++gen, ok, &wait_ok);
        const double yq = res_pass<double, false>(d, rg, tasks, sm, pan, qg, M, slots, hc, 2, ++gen, ok, &wait_ok);
        s_g = 0.0; s_d = 0.0;
        if (rg.own) {
          wj = yu;
          sj = yp;
          zj = yq;
          mj = wj / Mj;
          ((k - 1) & 1 ? mb1 : mb0)[j] = mj;
          s_g = rj * uj;
          s_d = wj * uj;
        }
        publish(s_g, s_d, 0.0);
        if (!(ok = grid_barrier(wd, flags, ++target, bcfg, ok))) break;
        t3 = grid_sum3(part, red3, &bc3);
        gamma = t3.x;
        delta = t3.y;
      }
      if (rn < best) {                                   // best-so-far iterate
        best = rn;
        best_k = k - 1;
        bxj = xj;
      }
      if (!isfinite(gamma)) break;                       // the reference's r.z
    }
    if (k > maxiter) break;
    // ---- iteration k-1 of the pipelined recurrences ----
    const double beta = k > 1 ? gamma / fmax(gamma_old, 1e-32) : 0.0;
    const double den = k > 1 ? delta - beta * gamma / alpha_old : delta;   // = p.S p
    const double alpha = gamma / fmax(den, 1e-32);
    double s_rr = 0.0;
    s_g = 0.0; s_d = 0.0;
    {
      const double nj = res_pass<double, false>(d, rg, tasks, sm, pan, (k - 1) & 1 ? mb1 : mb0, M, slots, hc, 0, ++gen, ok,
                                                &wait_ok);
      if (rg.own) {
        zj = nj + beta * zj;
        qj = mj + beta * qj;
        sj = wj + beta * sj;
        pj = uj + beta * pj;
        xj += alpha * pj;
        rj -= alpha * sj;
        uj -= alpha * qj;
        wj -= alpha * zj;
        mj = wj / Mj;
        (k & 1 ? mb1 : mb0)[j] = mj;
        s_g = rj * uj;
        s_d = wj * uj;
        s_rr = rj * rj;
      }
    }
    publish(s_g, s_d, s_rr);
    if (!(ok = grid_barrier(wd, flags, ++target, bcfg, ok))) break;
    t3 = grid_sum3(part, red3, &bc3);
    gamma_old = gamma;
    alpha_old = alpha;
    gamma = t3.x;
    delta = t3.y;
    rn = sqrt(t3.z);
  }
  // the converging iterate, else the best-so-far one (zeros if none improved or a wait gave up)
  if (rg.own) xo[j] = ok ? (TI)(converged ? xj : bxj) : TI(0);
  if (!ok && threadIdx.x == 0) atomicOr(result + 2, 1);   // any block that gave up flags the solve
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    result[0] = converged ? k_stop : best_k;
    result[1] = converged ? 1 : 0;
    result[3] = replaced;
  }
}

template <typename T>
int pcg_res_launch(const b3r_plan* plan, const float* S, const float* M, const T* b, T* xo, double tol, int maxiter,
                   long long spin_limit, int test_flags, void* work, int* result, cudaStream_t s) {
  const DevPlan& d = plan->d;
  constexpr int kSmem = kResSmemWords * 4;
  static int per_sm = 0, n_sm = 0;         // one attribute set and occupancy query per instantiation
  if (per_sm == 0) {
    int dev = 0;
    B3R_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
    B3R_TRY(check_cuda(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev), "SM count"));
    B3R_TRY(check_cuda(cudaFuncSetAttribute((const void*)k_pcg_res<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            kSmem),
                       "resident PCG shared memory"));
    B3R_TRY(check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_pcg_res<T>, kResThreads, kSmem),
                       "resident PCG occupancy"));
    B3R_REQUIRE(per_sm >= 1, "the resident PCG kernel does not fit on an SM");
  }
  const int grid = d.n_pcg_groups;                          // one block per row group, all co-resident
  B3R_REQUIRE(grid >= 1 && grid <= per_sm * n_sm && grid <= kPcgMaxBlocks, "internal: resident PCG grid %d", grid);
  B3R_TRY(check_cuda(cudaMemsetAsync(work, 0, kPcgPartOff, s), "clear PCG barrier words"));
  if (d.n_pcg_help > 0)
    B3R_TRY(check_cuda(cudaMemsetAsync((char*)work + kPcgHelpOff, 0, 4 * (size_t)d.n_pcg_help, s),
                       "clear PCG helper flags"));
  B3R_TRY(check_cuda(cudaMemsetAsync(result, 0, 4 * sizeof(int), s), "clear PCG result"));
  DevPlan dv = d;
  char* wk = reinterpret_cast<char*>(work);
  float* pan = reinterpret_cast<float*>(wk + pcg_panel_off(d));
  const int n_ent = (int)(2 * d.nnzb - d.nb);
  k_build_panels<<<grid_for((int64_t)n_ent * 32, 256), 256, 0, s>>>(dv, S, pan);
  B3R_TRY(check_launch("pcg panels"));
  const float* panc = pan;
  void* args[] = {&dv, &M, &b, &xo, &tol, &maxiter, &wk, &panc, &result, &spin_limit, &test_flags};
  B3R_TRY(check_cuda(cudaLaunchCooperativeKernel((const void*)k_pcg_res<T>, dim3(grid), dim3(kResThreads), args,
                                                 kSmem, s),
                     "resident pcg cooperative launch"));
  return B3R_OK;
}

template <typename T, int MAXB>
int pcg_launch(const b3r_plan* plan, const float* S, const float* M, const T* b, T* xo, double tol, int maxiter,
               long long spin_limit, int test_flags, void* work, int* result, cudaStream_t s) {
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
  // one block per row group where they all fit at once (cooperative: all co-resident); the
  // blocks take the groups with a stride otherwise
  const int grid = std::max(1, std::min(d.n_pcg_groups, per_sm * n_sm));
  B3R_REQUIRE(grid <= kPcgMaxBlocks, "internal: PCG grid %d > %d", grid, kPcgMaxBlocks);
  // barrier words and arrival flags start at zero (targets count up from 1 in every launch);
  // result[2] is set by any block whose barrier wait runs out
  B3R_TRY(check_cuda(cudaMemsetAsync(work, 0, kPcgPartOff, s), "clear PCG barrier words"));
  if (d.n_pcg_help > 0)
    B3R_TRY(check_cuda(cudaMemsetAsync((char*)work + kPcgHelpOff, 0, 4 * (size_t)d.n_pcg_help, s),
                       "clear PCG helper flags"));
  B3R_TRY(check_cuda(cudaMemsetAsync(result, 0, 4 * sizeof(int), s), "clear PCG result"));
  DevPlan dv = d;
  char* wk = reinterpret_cast<char*>(work);
  float* pan = reinterpret_cast<float*>(wk + pcg_panel_off(d));
  const int n_ent = (int)(2 * d.nnzb - d.nb);             // symmetric entries
  k_build_panels<<<grid_for((int64_t)n_ent * 32, 256), 256, 0, s>>>(dv, S, pan);
  B3R_TRY(check_launch("pcg panels"));
  const float* panc = pan;
  void* args[] = {&dv, &M, &b, &xo, &tol, &maxiter, &wk, &panc, &result, &spin_limit, &test_flags};
  B3R_TRY(check_cuda(cudaLaunchCooperativeKernel((const void*)k_pcg<T, MAXB>, dim3(grid), dim3(kPcgThreads), args,
                                                 0, s),
                     "pcg cooperative launch"));
  return B3R_OK;
}

template <typename T>
int pcg_impl(const b3r_plan* plan, const float* S, const float* M, const T* b, T* xo, double tol, int maxiter,
             long long spin_limit, int flags, void* work, int* result, void* stream) {
  B3R_REQUIRE(plan && S && M && b && xo && work && result, "NULL argument");
  B3R_REQUIRE(((uintptr_t)work & 255) == 0, "PCG work buffer must be 256-byte aligned");
  B3R_REQUIRE(maxiter >= 0, "maxiter must be >= 0");
  B3R_REQUIRE(spin_limit >= 1, "the barrier spin limit must be >= 1");
  B3R_REQUIRE((flags & ~(B3R_PCG_TEST_UNREACHABLE_BARRIER | B3R_PCG_STREAMING | B3R_PCG_TEST_GLOBAL_TILES)) == 0,
              "unknown PCG flags %d", flags);
  int dev = -1;
  B3R_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  B3R_REQUIRE(dev == plan->device, "current device %d differs from the plan's device %d", dev, plan->device);
  if (plan->d.n_cam_params == 0) return B3R_OK;
  int maxb = 0;
  for (int v : plan->pat.bsize) maxb = std::max(maxb, v);
  cudaStream_t s = as_stream(stream);
  if (plan->d.pcg_resident && !(flags & B3R_PCG_STREAMING))
    return pcg_res_launch<T>(plan, S, M, b, xo, tol, maxiter, spin_limit, flags, work, result, s);
  if (maxb <= 8) return pcg_launch<T, 8>(plan, S, M, b, xo, tol, maxiter, spin_limit, flags, work, result, s);
  B3R_REQUIRE(maxb <= 32, "block size %d > 32", maxb);
  return pcg_launch<T, 32>(plan, S, M, b, xo, tol, maxiter, spin_limit, flags, work, result, s);
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
  return pcg_impl<float>(plan, S_vals, precond, b, x, tol, maxiter, kBarrierSpins, 0, work, result, stream);
}

extern "C" int b3r_pcg_f64(const b3r_plan* plan, const float* S_vals, const float* precond, const double* b,
                           double* x, double tol, int maxiter, void* work, int* result, void* stream) {
  return pcg_impl<double>(plan, S_vals, precond, b, x, tol, maxiter, kBarrierSpins, 0, work, result, stream);
}

extern "C" int b3r_pcg_ex(const b3r_plan* plan, const float* S_vals, const float* precond, const void* b, void* x,
                          int dtype, double tol, int maxiter, int64_t barrier_spin_limit, int flags, void* work,
                          int* result, void* stream) {
  const long long spins = barrier_spin_limit > 0 ? (long long)barrier_spin_limit : kBarrierSpins;
  if (dtype == B3R_F64)
    return pcg_impl<double>(plan, S_vals, precond, (const double*)b, (double*)x, tol, maxiter, spins, flags, work,
                            result, stream);
  B3R_REQUIRE(dtype == B3R_F32, "dtype must be B3R_F32 or B3R_F64");
  return pcg_impl<float>(plan, S_vals, precond, (const float*)b, (float*)x, tol, maxiter, spins, flags, work, result,
                         stream);
}
