// Part 4 of the C ABI: the line search's reprojection score without a sort.
//
// The reference's line search rejects a step whose reprojection residual collapsed
// (engine.py:308-333, reproj_score at :357-361): the mean of the smallest 80 % of the
// per-observation reprojection errors ||r[:2]||, computed by sorting all of them.  Here the
// k-th smallest error (k = floor(0.8 n)) is found exactly by a three-level radix select over
// the bit pattern of the non-negative float errors (11 + 11 + 9 bits: non-negative floats
// order like their bits), then one pass sums the errors below it; the k smallest are those
// plus (k - count below) copies of the k-th value, the same set a sort takes.
//
//   k_score_hist   level 0: compute each error (written once, compact) and histogram its top
//                  11 bits; levels 1, 2: histogram the next bits of the errors whose higher
//                  bits match the selected prefix (block-private shared-memory histograms)
//   k_score_pick   one block: find the bin holding the k-th error (block prefix sum over the
//                  bins), extend the prefix
//   k_score_sum    sum and count of the errors below the k-th; the last block writes the score
#include <algorithm>
#include "b3r_common.cuh"
#include "b3r_status.h"

namespace b3r {
namespace {

constexpr int kScoreThreads = 256;
constexpr int kBins = 2048;   // 11-bit digits (the last level uses 512 of them)

// Scalars of the select at the start of the work buffer.
struct ScoreState {
  unsigned int prefix;       // selected high bits so far
  unsigned long long rank;   // 1-based rank of the k-th error among those matching the prefix
  double sum;                // sum of the errors below the k-th
  unsigned long long below;  // how many errors are below the k-th
  unsigned int done_blocks;
  unsigned int pad;
  unsigned int hist[3][kBins];
};

__device__ __forceinline__ int digit_shift(int level) { return level == 0 ? 20 : (level == 1 ? 9 : 0); }
__device__ __forceinline__ int digit_bins(int level) { return level == 2 ? 512 : kBins; }

__global__ void __launch_bounds__(kScoreThreads) k_score_hist(const float* __restrict__ res, int64_t n,
                                                              int64_t so, int64_t sc, float* __restrict__ err,
                                                              ScoreState* st, int level) {
  __shared__ unsigned int h[kBins];
  for (int i = threadIdx.x; i < kBins; i += blockDim.x) h[i] = 0u;
  __syncthreads();
  const int sh = digit_shift(level), nb = digit_bins(level);
  const unsigned int prefix = level ? st->prefix : 0u;
  const int hs = level == 1 ? 20 : 9;   // bits already selected: those at and above hs
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float e;
    if (level == 0) {
      const float x = res[i * so], y = res[i * so + sc];
      e = sqrtf(x * x + y * y);
      err[i] = e;
    } else {
      e = err[i];
    }
    const unsigned int u = __float_as_uint(e) & 0x7FFFFFFFu;   // a NaN's sign bit aside, e >= 0
    if (level == 0 || (u >> hs) == prefix) atomicAdd(&h[(u >> sh) & (nb - 1)], 1u);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < nb; i += blockDim.x)
    if (h[i]) atomicAdd(&st->hist[level][i], h[i]);
}

// One block: the bin of this level that holds the rank-th error; rank becomes the rank
// within that bin and the prefix gains the bin's digit.  Each thread owns a run of
// consecutive bins (8 at 11-bit levels, 2 at the last); a block-wide prefix sum of the run
// totals tells the one thread whose run holds the rank-th error, which walks its run.  A
// rank beyond every count (errors that fell out of the prefix test) selects the last bin.
constexpr int kPickThreads = 256;
__global__ void __launch_bounds__(kPickThreads) k_score_pick(ScoreState* st, int level, int64_t k) {
  __shared__ unsigned long long wsum[kPickThreads / 32];
  const int nb = digit_bins(level), per = nb / kPickThreads, b0 = threadIdx.x * per;
  const unsigned long long r = level == 0 ? (unsigned long long)k : st->rank;
  unsigned long long c[kBins / kPickThreads], tot = 0;
#pragma unroll
  for (int j = 0; j < kBins / kPickThreads; ++j) {
    c[j] = j < per ? (unsigned long long)st->hist[level][b0 + j] : 0ull;
    tot += c[j];
  }
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  unsigned long long inc = tot;                          // inclusive scan within the warp
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const unsigned long long v = __shfl_up_sync(0xffffffffu, inc, d);
    if (lane >= d) inc += v;
  }
  if (lane == 31) wsum[w] = inc;
  __syncthreads();
  unsigned long long acc = inc - tot;                    // errors in the bins before this run
  for (int i = 0; i < w; ++i) acc += wsum[i];
  const bool last = threadIdx.x == kPickThreads - 1;
  if ((acc < r && r <= acc + tot) || (last && r > acc + tot)) {
    int bin = b0 + per - 1;
    for (int j = 0; j < per; ++j) {
      if (acc + c[j] >= r) { bin = b0 + j; break; }
      acc += c[j];
    }
    st->rank = r - acc;
    st->prefix = (level == 0 ? 0u : st->prefix << (level == 1 ? 11 : 9)) | (unsigned int)bin;
  }
}

__global__ void __launch_bounds__(kScoreThreads) k_score_sum(const float* __restrict__ err, int64_t n, int64_t k,
                                                             ScoreState* st, float* __restrict__ score) {
  __shared__ double ssum[kScoreThreads / 32];
  __shared__ unsigned long long scnt[kScoreThreads / 32];
  const float kth = __uint_as_float(st->prefix);   // all 31 value bits selected
  double s = 0.0;
  unsigned long long c = 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float e = err[i];
    if (e < kth) { s += e; ++c; }
  }
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, d);
    c += __shfl_xor_sync(0xffffffffu, c, d);
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) { ssum[w] = s; scnt[w] = c; }
  __syncthreads();
  if (threadIdx.x == 0) {
    double bs = 0.0;
    unsigned long long bc = 0;
    for (int i = 0; i < kScoreThreads / 32; ++i) { bs += ssum[i]; bc += scnt[i]; }
    atomicAdd(&st->sum, bs);
    atomicAdd(&st->below, bc);
    __threadfence();
    if (atomicAdd(&st->done_blocks, 1u) == gridDim.x - 1) {   // the last block has every sum
      __threadfence();
      const double tot = *(volatile double*)&st->sum;
      const unsigned long long nbl = *(volatile unsigned long long*)&st->below;
      *score = (float)((tot + (double)(k - (int64_t)nbl) * (double)kth) / (double)k);
    }
  }
}

}  // namespace
}  // namespace b3r

using namespace b3r;

extern "C" int64_t b3r_reproj_score_work_bytes(int64_t n_obs) {
  return (int64_t)((sizeof(ScoreState) + 255) & ~size_t(255)) + 4 * std::max<int64_t>(n_obs, 1);
}

extern "C" int b3r_reproj_score(const float* residuals, int64_t n_obs, int64_t stride_obs, int64_t stride_comp,
                                void* work, float* score, void* stream) {
  B3R_REQUIRE(residuals && work && score, "NULL argument");
  B3R_REQUIRE(n_obs >= 0 && stride_obs >= 1 && stride_comp >= 1, "bad sizes or strides");
  B3R_REQUIRE(((uintptr_t)work & 255) == 0, "work buffer must be 256-byte aligned");
  cudaStream_t s = as_stream(stream);
  const int64_t k = n_obs * 80 / 100;
  if (k == 0)     // the mean of no errors, as the reference's empty mean: NaN (all bits set)
    return check_cuda(cudaMemsetAsync(score, 0xFF, sizeof(float), s), "score");
  ScoreState* st = reinterpret_cast<ScoreState*>(work);
  float* err = reinterpret_cast<float*>(reinterpret_cast<char*>(work) + ((sizeof(ScoreState) + 255) & ~size_t(255)));
  B3R_TRY(check_cuda(cudaMemsetAsync(st, 0, sizeof(ScoreState), s), "clear score state"));
  const int grid = (int)std::min<int64_t>((n_obs + kScoreThreads - 1) / kScoreThreads, 148 * 8);
  for (int level = 0; level < 3; ++level) {
    k_score_hist<<<grid, kScoreThreads, 0, s>>>(residuals, n_obs, stride_obs, stride_comp, err, st, level);
    B3R_TRY(check_launch("score histogram"));
    k_score_pick<<<1, kPickThreads, 0, s>>>(st, level, k);
    B3R_TRY(check_launch("score pick"));
  }
  k_score_sum<<<grid, kScoreThreads, 0, s>>>(err, n_obs, k, st, score);
  return check_launch("score sum");
}
