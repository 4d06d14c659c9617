// Host planner: builds the static structure of one BA phase (b3r_plan_create).
//
// The reference rediscovers this structure on every LM iteration with torch.unique /
// index_add_ inside its block-matrix algebra (inference/ba_solver.py:854-924, 1063-1071);
// here it is computed once per phase, on the host, in O(n_obs * mean track length):
//   * image -> (foc, tau, zcf) typed blocks honouring the enable rules of
//     GaussNewtonSolver.enable (ba_solver.py:72-108);
//   * the local (this rank's) eliminated tracks, ordered by (first image, id), with their
//     observations grouped by track and packed into <=32-observation warp tasks;
//   * per-image observation chunks for the image-major diagonal pass;
//   * image-pair segments (from ALL tracks, so every rank shares one S pattern) and this
//     rank's observation-pair lists bucketed by segment, cut into pair tasks;
//   * the block-sparse pattern of S (upper block triangle) and every destination offset.
#include <algorithm>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <memory>
#include <mutex>
#include <numeric>
#include <pthread.h>
#include <new>
#include <thread>
#include "b3r_plan.h"
#include "b3r_status.h"

namespace b3r {
namespace {

struct TypeMap {
  int n_true = 0, n_cols = 0;
  bool zero = false;
  std::vector<int> col;   // -1: removed
};

int make_type(int mode, const uint8_t* mask, int n, const char* name, TypeMap& t) {
  t.n_true = n;
  t.col.assign(n, 0);
  if (mode == B3R_ENABLE_ALL || mode == B3R_ENABLE_ZERO) {
    std::iota(t.col.begin(), t.col.end(), 0);
    t.n_cols = n;
    t.zero = (mode == B3R_ENABLE_ZERO);
    return B3R_OK;
  }
  B3R_REQUIRE(mode == B3R_ENABLE_MASK, "bad enable mode %d for %s", mode, name);
  B3R_REQUIRE(mask != nullptr, "mask for %s is NULL", name);
  int c = 0;
  for (int j = 0; j < n; ++j) t.col[j] = mask[j] ? c++ : -1;
  if (c == 0) {   // every column removed: the reference falls back to ZerosMat (ba_solver.py:92-93)
    std::iota(t.col.begin(), t.col.end(), 0);
    t.n_cols = n;
    t.zero = true;
  } else {
    t.n_cols = c;
  }
  return B3R_OK;
}

inline int round4(int x) { return (x + 3) & ~3; }

// Host threads of the planner: $B3R_PLAN_THREADS, else the hardware's, at most 32.
int plan_threads() {
  if (const char* e = std::getenv("B3R_PLAN_THREADS")) {
    const int v = std::atoi(e);
    if (v >= 1) return std::min(v, 256);
  }
  const unsigned h = std::thread::hardware_concurrency();
  return (int)std::max(1u, std::min(h ? h : 1u, 32u));
}

// The planner's worker threads, started once and kept for the process: plan_threads() - 1
// workers plus the calling thread.  One parallel section at a time (plans built from several
// host threads take turns); a section runs task(t) for t in [0, nt) with t = 0 on the caller.
class PlanPool {
 public:
  // The pool is never destroyed (no join at exit).  A child process forked after the pool
  // started has none of its workers: the fork handler drops the pointer and the child starts
  // its own pool on first use.
  static PlanPool& get() {
    static std::once_flag once;
    std::call_once(once, [] { pthread_atfork(nullptr, nullptr, [] { instance() = nullptr; }); });
    static std::mutex mk;
    std::lock_guard<std::mutex> lk(mk);
    if (!instance()) instance() = new PlanPool(plan_threads() - 1);
    return *instance();
  }
  int size() const { return (int)workers_.size() + 1; }
  void run(int nt, const std::function<void(int)>& task) {
    nt = std::max(1, std::min(nt, size()));
    if (nt == 1) { task(0); return; }
    std::lock_guard<std::mutex> section(section_);
    {
      std::lock_guard<std::mutex> lk(m_);
      task_ = &task;
      n_active_ = nt;
      pending_ = nt - 1;
      ++gen_;
    }
    cv_.notify_all();
    task(0);
    std::unique_lock<std::mutex> lk(m_);
    done_.wait(lk, [&] { return pending_ == 0; });
    task_ = nullptr;
  }

 private:
  static PlanPool*& instance() {
    static PlanPool* p = nullptr;
    return p;
  }
  explicit PlanPool(int n) {
    for (int w = 0; w < n; ++w) workers_.emplace_back([this, w] { loop(w + 1); });
    for (auto& t : workers_) t.detach();
  }
  void loop(int id) {
    uint64_t seen = 0;
    for (;;) {
      const std::function<void(int)>* task;
      {
        std::unique_lock<std::mutex> lk(m_);
        cv_.wait(lk, [&] { return gen_ != seen; });
        seen = gen_;
        if (id >= n_active_) continue;
        task = task_;
      }
      (*task)(id);
      std::lock_guard<std::mutex> lk(m_);
      if (--pending_ == 0) done_.notify_one();
    }
  }
  std::vector<std::thread> workers_;
  std::mutex section_, m_;
  std::condition_variable cv_, done_;
  const std::function<void(int)>* task_ = nullptr;
  uint64_t gen_ = 0;
  int n_active_ = 0, pending_ = 0;
};

// fn(t, begin, end) over nt contiguous ranges of [0, n) on the planner's threads (the first
// range on the calling thread); at most one range per `grain` items, so that small plans (an
// online window) stay on few threads.
constexpr int64_t kPlanGrain = 1 << 14;
template <typename F>
void parallel_ranges(int64_t n, int nt, F&& fn, int64_t grain = kPlanGrain) {
  grain = std::max<int64_t>(grain, 1);
  nt = (int)std::max<int64_t>(1, std::min<int64_t>(nt, (n + grain - 1) / grain));
  nt = std::min(nt, PlanPool::get().size());
  const std::function<void(int)> task = [&](int t) { fn(t, n * t / nt, n * (t + 1) / nt); };
  PlanPool::get().run(nt, task);
}

}  // namespace

// Host-side intermediate of the planner (kept out of the public struct).
struct PlanBuild {
  const b3r_plan_desc* d;
  std::vector<int> img_of;                 // [n_obs]
  TypeMap K, P, Z, X;
  int nb = 0;
  std::vector<int> img_bk, img_sc, img_node, img_cam;
  std::vector<int> bsize, boff;
  // all eliminated tracks (global), grouped
  std::vector<int> all_ptr, all_obs;       // CSR over track id
  std::vector<char> elim;                  // [n_tracks]
  std::vector<char> owned;                 // [n_tracks] track belongs to this rank
  std::vector<char> obs_live;              // [n_obs] observation touches an active block
  // local side
  std::vector<int> loc_tracks, trk_col, perm_t, trk_t, img_t, pt_task, kof;
  std::vector<int> c1_obs, c1_k, c1_pid, c1_chunk, c1_img;
  // segments (global)
  std::vector<int> seg_row_ptr, seg_col;   // CSR over row image
  std::vector<int64_t> seg_cnt;
  std::vector<int2> pairs;
  std::vector<int64_t> task_pb, task_pe;
  std::vector<int> task_seg;
  // pattern
  std::vector<int> row_ptr, col_idx, val_off;
  std::vector<int> seg_dst, seg_mode, img_dst, sdiag_pos, blk_row, trk_ptr, img_zdiag, img_zsc;
  std::vector<int4> t_idx, c1_idx, rest_idx;
  std::vector<int> sym_ptr, sym_ent;
  std::vector<int4> mv_task, mv_row, mv_ent;
  std::vector<int4> pcg_grp, pcg_grp2;
  int n_pcg_help = 0;
  std::vector<int> mv_slot;
  std::vector<int2> pcg_scl;
  std::vector<int> mv_soff;
  int pcg_target_groups = 148;   // SMs of the plan's device (a B200's without one)
  int pcg_resident = 0;
  std::vector<int64_t> pan_off;
  std::vector<int> pan_w, col_off, pan_col, ent_col, ent_row;
  int64_t pan_floats = 0;
  int64_t nnz = 0;
};

static int build_maps(PlanBuild& B) {
  const b3r_plan_desc& d = *B.d;
  const int I = d.n_imgs;
  B3R_REQUIRE(I >= 1 && d.n_cams >= 1 && d.n_nodes >= 1 && d.n_tracks >= 0 && d.n_obs >= 0,
              "bad sizes");
  B3R_REQUIRE(d.C >= 1 && d.C <= 32, "C=%d out of range [1, 32]", d.C);
  B3R_REQUIRE(d.n_obs < (int64_t(1) << 31), "n_obs must be < 2^31 per plan");
  B3R_REQUIRE(d.infos != nullptr && (d.n_obs == 0 || d.pids != nullptr), "NULL infos/pids");
  B3R_REQUIRE(d.track_begin >= 0 && d.track_begin <= d.track_end && d.track_end <= d.n_tracks,
              "bad track range [%d, %d)", d.track_begin, d.track_end);
  B3R_REQUIRE(d.obs_local == 0 || d.obs_local == 1, "obs_local must be 0 or 1");
  B.owned.assign(d.n_tracks, 0);
  for (int t = 0; t < d.n_tracks; ++t)
    B.owned[t] = d.track_owner ? (d.track_owner[t] == d.rank) : (t >= d.track_begin && t < d.track_end);
  const int32_t* cum = d.infos;
  const int32_t* node = d.infos + I;
  const int32_t* cam = d.infos + 2 * I;
  int64_t prev = 0;
  for (int i = 0; i < I; ++i) {
    B3R_REQUIRE(cum[i] >= prev, "infos[0] must be non-decreasing (image %d)", i);
    B3R_REQUIRE(node[i] >= 0 && node[i] < d.n_nodes, "node id %d of image %d out of range", node[i], i);
    B3R_REQUIRE(cam[i] >= 0 && cam[i] < d.n_cams, "cam id %d of image %d out of range", cam[i], i);
    prev = cum[i];
  }
  B3R_REQUIRE(prev == d.n_obs, "infos[0][-1]=%lld must equal n_obs=%lld", (long long)prev,
              (long long)d.n_obs);
  B.img_of.resize(d.n_obs);
  int64_t o = 0;
  for (int i = 0; i < I; ++i)
    for (; o < cum[i]; ++o) B.img_of[o] = i;
  for (int64_t j = 0; j < d.n_obs; ++j)
    B3R_REQUIRE(d.pids[j] >= 0 && d.pids[j] < d.n_tracks, "pid %d of observation %lld out of range",
                d.pids[j], (long long)j);

  B3R_TRY(make_type(d.mode_K, d.mask_K, d.n_cams, "K", B.K));
  B3R_TRY(make_type(d.mode_P, d.mask_P, d.n_nodes, "P", B.P));
  B3R_TRY(make_type(d.mode_Z, d.mask_Z, d.n_imgs, "Z", B.Z));
  B3R_TRY(make_type(d.mode_X, d.mask_X, d.n_tracks, "X", B.X));
  const int nbK = B.K.n_cols, nbP = B.P.n_cols, nbZ = B.Z.n_cols;
  B.nb = nbK + nbP + nbZ;
  B.bsize.resize(B.nb);
  B.boff.resize(B.nb);
  int off = 0;
  for (int p = 0; p < B.nb; ++p) {
    B.bsize[p] = p < nbK ? 2 : (p < nbK + nbP ? 6 : d.C);
    B.boff[p] = off;
    off += B.bsize[p];
  }
  B.img_bk.assign(3 * I, -1);
  B.img_sc.assign(3 * I, -1);
  B.img_node.assign(node, node + I);
  B.img_cam.assign(cam, cam + I);
  for (int i = 0; i < I; ++i) {
    int bk = (!B.K.zero && B.K.col[cam[i]] >= 0) ? B.K.col[cam[i]] : -1;
    int bp = (!B.P.zero && B.P.col[node[i]] >= 0) ? nbK + B.P.col[node[i]] : -1;
    int bz = (!B.Z.zero && B.Z.col[i] >= 0) ? nbK + nbP + B.Z.col[i] : -1;
    B.img_bk[3 * i] = bk; B.img_bk[3 * i + 1] = bp; B.img_bk[3 * i + 2] = bz;
    B.img_sc[3 * i] = bk >= 0 ? B.boff[bk] : -1;
    B.img_sc[3 * i + 1] = bp >= 0 ? B.boff[bp] : -1;
    B.img_sc[3 * i + 2] = bz >= 0 ? B.boff[bz] : -1;
  }
  return B3R_OK;
}

static inline bool img_live(const PlanBuild& B, int i) {
  return B.img_bk[3 * i] >= 0 || B.img_bk[3 * i + 1] >= 0 || B.img_bk[3 * i + 2] >= 0;
}

static void build_image_major(PlanBuild& B);
static void pack_indices(PlanBuild& B);

// Eliminated tracks (point type enabled) and live observations (their image has an active
// block).
static void build_flags(PlanBuild& B) {
  const b3r_plan_desc& d = *B.d;
  const int nt = plan_threads();
  B.elim.assign(d.n_tracks, 0);
  if (!B.X.zero)
    parallel_ranges(d.n_tracks, nt, [&](int, int64_t a, int64_t b) {
      for (int64_t t = a; t < b; ++t) B.elim[t] = B.X.col[t] >= 0;
    });
  B.obs_live.resize(d.n_obs);
  parallel_ranges(d.n_obs, nt, [&](int, int64_t a, int64_t b) {
    for (int64_t o = a; o < b; ++o) B.obs_live[o] = img_live(B, B.img_of[o]);
  });
}

// Point tasks of local tracks [tl0, nT): whole tracks packed greedily into <= 32
// observations (one warp); a track longer than 32 gets a task of its own, which the kernels
// process in rounds.  Appends to pt_task, then its end sentinel.
static void pack_point_tasks(PlanBuild& B, int tl0) {
  const int nT = (int)B.loc_tracks.size();
  int cur = 0;          // observations in the open task
  bool open = false, open_long = false;
  for (int tl = tl0; tl < nT; ++tl) {
    const int L = B.trk_ptr[tl + 1] - B.trk_ptr[tl];
    if (open && (open_long || L > kPointTask || cur + L > kPointTask)) open = false;
    if (!open) {
      B.pt_task.push_back(B.trk_ptr[tl]);
      open = true;
      open_long = false;
      cur = 0;
    }
    cur += L;
    open_long = L > kPointTask;
  }
  if (nT > 0) B.pt_task.push_back(B.trk_ptr[nT]);
}

static int build_tracks(PlanBuild& B) {
  // Every O(n_obs) step runs on the planner's threads (plan_threads()); the results are the
  // same as one sequential pass: each track's observations end up in increasing o.
  const b3r_plan_desc& d = *B.d;
  const int T = d.n_tracks;
  const int64_t n = d.n_obs;
  const int nt = plan_threads();
  build_flags(B);
  // CSR of observations per eliminated track (all tracks): counts by relaxed atomic
  // increments, a prefix sum, an atomic fill, then each track's few observations sorted by o
  B.all_ptr.assign(T + 1, 0);
  int* cnt = B.all_ptr.data() + 1;
  parallel_ranges(n, nt, [&](int, int64_t a, int64_t b) {
    for (int64_t o = a; o < b; ++o) {
      const int t = d.pids[o];
      if (B.elim[t]) __atomic_fetch_add(cnt + t, 1, __ATOMIC_RELAXED);
    }
  });
  for (int t = 0; t < T; ++t) B.all_ptr[t + 1] += B.all_ptr[t];
  B.all_obs.resize(B.all_ptr[T]);
  {
    std::vector<int> fill(B.all_ptr.begin(), B.all_ptr.end() - 1);
    parallel_ranges(n, nt, [&](int, int64_t a, int64_t b) {
      for (int64_t o = a; o < b; ++o) {
        const int t = d.pids[o];
        if (B.elim[t]) B.all_obs[__atomic_fetch_add(&fill[t], 1, __ATOMIC_RELAXED)] = (int)o;
      }
    });
    parallel_ranges(T, nt, [&](int, int64_t a, int64_t b) {
      for (int64_t t = a; t < b; ++t) {
        int* x = B.all_obs.data() + B.all_ptr[t];
        const int L = B.all_ptr[t + 1] - B.all_ptr[t];
        for (int i = 1; i < L; ++i)            // insertion sort: tracks are short
          for (int j = i; j > 0 && x[j - 1] > x[j]; --j) std::swap(x[j - 1], x[j]);
      }
    });
  }
  // local tracks: eliminated, owned, non-empty; ordered by (first image, id)
  {
    // stable counting sort by first image (tracks in id order within an image)
    std::vector<int> first(T, -1);
    parallel_ranges(T, nt, [&](int, int64_t a, int64_t b) {
      for (int64_t t = a; t < b; ++t)
        if (B.owned[t] && B.elim[t] && B.all_ptr[t + 1] > B.all_ptr[t]) first[t] = B.img_of[B.all_obs[B.all_ptr[t]]];
    });
    std::vector<int> icnt(d.n_imgs + 1, 0);
    int64_t nloc = 0;
    for (int t = 0; t < T; ++t)
      if (first[t] >= 0) { icnt[first[t] + 1]++; ++nloc; }
    for (int i = 0; i < d.n_imgs; ++i) icnt[i + 1] += icnt[i];
    B.loc_tracks.resize(nloc);
    for (int t = 0; t < T; ++t)
      if (first[t] >= 0) B.loc_tracks[icnt[first[t]]++] = t;
  }
  const int nT = (int)B.loc_tracks.size();
  B.trk_col.resize(nT);
  B.trk_ptr.assign(nT + 1, 0);
  parallel_ranges(nT, nt, [&](int, int64_t a, int64_t b) {
    for (int64_t tl = a; tl < b; ++tl) {
      const int t = B.loc_tracks[tl];
      B.trk_col[tl] = B.X.col[t];
      B.trk_ptr[tl + 1] = B.all_ptr[t + 1] - B.all_ptr[t];
    }
  });
  for (int tl = 0; tl < nT; ++tl) B.trk_ptr[tl + 1] += B.trk_ptr[tl];
  const int64_t n_loc = nT ? B.trk_ptr[nT] : 0;
  B.perm_t.resize(n_loc);
  B.trk_t.resize(n_loc);
  B.img_t.resize(n_loc);
  B.kof.assign(n, -1);
  parallel_ranges(nT, nt, [&](int, int64_t a, int64_t b) {
    for (int64_t tl = a; tl < b; ++tl) {
      const int t = B.loc_tracks[tl];
      int64_t k = B.trk_ptr[tl];
      for (int j = B.all_ptr[t]; j < B.all_ptr[t + 1]; ++j, ++k) {
        const int o = B.all_obs[j];
        B.perm_t[k] = o;
        B.trk_t[k] = (int)tl;
        B.img_t[k] = B.img_of[o];
        B.kof[o] = (int)k;
      }
    }
  });
  pack_point_tasks(B, 0);
  build_image_major(B);
  pack_indices(B);
  return B3R_OK;
}

// Image-major chunks over the observations this rank owns (c1_*, rest_idx, c1_idx), from the
// track side's kof.  An observation's image decides whether it is live, so one count per image
// (owned observations; all of them when every track is this rank's) places every image's
// entries; the images are then filled in parallel, straight into the final arrays.
static void build_image_major(PlanBuild& B) {
  const b3r_plan_desc& d = *B.d;
  const int nt = plan_threads();
  const int I = d.n_imgs;
  const int32_t* cum = d.infos;
  const bool all_owned = !d.track_owner && d.track_begin == 0 && d.track_end == d.n_tracks;
  std::vector<int64_t> own(I, 0);
  parallel_ranges(I, nt, [&](int, int64_t i0, int64_t i1) {
    for (int64_t i = i0; i < i1; ++i) {
      const int64_t o0 = i ? cum[i - 1] : 0, o1 = cum[i];
      if (all_owned) {
        own[i] = o1 - o0;
      } else {
        int64_t c = 0;
        for (int64_t o = o0; o < o1; ++o) c += B.owned[d.pids[o]];
        own[i] = c;
      }
    }
  }, std::max<int64_t>(1, (int64_t)I * kPlanGrain / std::max<int64_t>(d.n_obs, 1)));
  std::vector<int64_t> e0(I + 1, 0), r0(I + 1, 0);
  std::vector<int> ch0(I + 1, 0);
  for (int i = 0; i < I; ++i) {
    const bool live = img_live(B, i);
    e0[i + 1] = e0[i] + (live ? own[i] : 0);
    r0[i + 1] = r0[i] + (live ? 0 : own[i]);
    ch0[i + 1] = ch0[i] + (live ? (int)((own[i] + kDiagChunk - 1) / kDiagChunk) : 0);
  }
  const int64_t n_c1 = e0[I];
  B.c1_obs.resize(n_c1); B.c1_k.resize(n_c1); B.c1_pid.resize(n_c1); B.c1_idx.resize(n_c1);
  B.c1_chunk.resize(ch0[I] + 1); B.c1_img.resize(ch0[I]);
  B.rest_idx.resize(r0[I]);
  parallel_ranges(I, nt, [&](int, int64_t i0, int64_t i1) {
    for (int64_t i = i0; i < i1; ++i) {
      const int64_t o0 = i ? cum[i - 1] : 0, o1 = cum[i];
      if (!img_live(B, (int)i)) {            // evaluated for the objective only
        int64_t r = r0[i];
        for (int64_t o = o0; o < o1; ++o) {
          const int t = d.pids[o];
          if (B.owned[t]) B.rest_idx[r++] = make_int4((int)o, (int)i, t, 0);
        }
        continue;
      }
      for (int c = ch0[i]; c < ch0[i + 1]; ++c) {
        B.c1_chunk[c] = (int)(e0[i] + (int64_t)(c - ch0[i]) * kDiagChunk);
        B.c1_img[c] = (int)i;
      }
      int64_t e = e0[i];
      for (int64_t o = o0; o < o1; ++o) {
        const int t = d.pids[o];
        if (!all_owned && !B.owned[t]) continue;
        const int kk = B.kof[o];
        B.c1_obs[e] = (int)o;
        B.c1_k[e] = kk;
        B.c1_pid[e] = t;
        B.c1_idx[e] = make_int4((int)o, kk, t, kk >= 0 ? B.trk_t[kk] : -1);
        ++e;
      }
    }
  }, std::max<int64_t>(1, (int64_t)I * kPlanGrain / std::max<int64_t>(d.n_obs, 1)));
  B.c1_chunk[ch0[I]] = (int)n_c1;
}

// Packed per-observation indices of the track side (one 16-byte load per observation in the
// kernels); the image-major side's (c1_idx) are written by build_image_major.
static void pack_indices(PlanBuild& B) {
  const int nt = plan_threads();
  B.t_idx.resize(B.perm_t.size());
  parallel_ranges((int64_t)B.perm_t.size(), nt, [&](int, int64_t a, int64_t b) {
    for (int64_t kk = a; kk < b; ++kk)
      B.t_idx[kk] = make_int4(B.img_t[kk], B.loc_tracks[B.trk_t[kk]], B.trk_t[kk], B.perm_t[kk]);
  });
}

}  // namespace b3r

namespace b3r {

// Segments: for each row image i, the sorted partner images i' >= i sharing an eliminated
// track (over ALL tracks).  For i' == i the segment only exists when a track has two
// live observations in image i.
static int build_segments(PlanBuild& B) {
  const b3r_plan_desc& d = *B.d;
  const int I = d.n_imgs;
  const int32_t* cum = d.infos;
  // each thread takes a contiguous range of row images; per image its partners, sorted
  const int nt = plan_threads();
  std::vector<std::vector<int>> part_col(nt), part_cnt(nt);
  const int64_t grain = std::max<int64_t>(1, (int64_t)I * 4096 / std::max<int64_t>(d.n_obs, 1));
  parallel_ranges(I, nt, [&](int t, int64_t i0, int64_t i1) {
    std::vector<int> stamp(I, -1), partners;
    std::vector<int>& col = part_col[t];
    std::vector<int>& cnt = part_cnt[t];
    for (int i = (int)i0; i < (int)i1; ++i) {
      partners.clear();
      const int64_t o0 = i ? cum[i - 1] : 0, o1 = cum[i];
      for (int64_t o = o0; o < o1; ++o) {
        const int tk = d.pids[o];
        if (!B.elim[tk] || !B.obs_live[o]) continue;
        for (int j = B.all_ptr[tk]; j < B.all_ptr[tk + 1]; ++j) {
          const int o2 = B.all_obs[j];
          if (o2 <= o || !B.obs_live[o2]) continue;   // o2 > o  =>  img(o2) >= i
          const int i2 = B.img_of[o2];
          if (stamp[i2] != i) { stamp[i2] = i; partners.push_back(i2); }
        }
      }
      std::sort(partners.begin(), partners.end());
      col.insert(col.end(), partners.begin(), partners.end());
      cnt.push_back((int)partners.size());
    }
  }, grain);
  B.seg_row_ptr.assign(I + 1, 0);
  B.seg_col.clear();
  int i = 0;
  for (int t = 0; t < nt; ++t) {
    B.seg_col.insert(B.seg_col.end(), part_col[t].begin(), part_col[t].end());
    for (int c : part_cnt[t]) { B.seg_row_ptr[i + 1] = B.seg_row_ptr[i] + c; ++i; }
  }
  B3R_REQUIRE(i == I, "internal: segment rows %d of %d", i, I);
  return B3R_OK;
}

static inline int64_t seg_lookup(const PlanBuild& B, int i, int i2) {
  const int* a = B.seg_col.data() + B.seg_row_ptr[i];
  const int* e = B.seg_col.data() + B.seg_row_ptr[i + 1];
  const int* p = std::lower_bound(a, e, i2);
  return (p != e && *p == i2) ? (int64_t)(p - B.seg_col.data()) : -1;
}

// This rank's observation pairs, bucketed by segment (stable in local track order), and
// the pair tasks.
// tracks per planner thread in the pair passes (a track's pairs grow with its length squared)
constexpr int64_t kPairGrain = 512;

static void build_tasks(PlanBuild& B);

static int build_pairs(PlanBuild& B) {
  const int64_t S = (int64_t)B.seg_col.size();
  const int64_t nT = (int64_t)B.loc_tracks.size();
  // Pairs (a < b) of every local track in local order, visited by track ranges: a two-pass
  // counting sort (count per thread and segment, then fill at per-thread offsets) keeps the
  // pairs of a segment in local track order, the same as one sequential pass.
  auto for_pairs = [&](int64_t tl0, int64_t tl1, auto&& fn) {
    for (int64_t tl = tl0; tl < tl1; ++tl) {
      const int64_t k0 = B.trk_ptr[tl];
      const int L = B.trk_ptr[tl + 1] - B.trk_ptr[tl];
      for (int a = 0; a < L; ++a) {
        const int ka = (int)(k0 + a);
        const int oa = B.perm_t[ka];
        if (!B.obs_live[oa]) continue;
        for (int b = a + 1; b < L; ++b) {
          const int kb = (int)(k0 + b);
          const int ob = B.perm_t[kb];
          if (!B.obs_live[ob]) continue;
          fn(seg_lookup(B, B.img_of[oa], B.img_of[ob]), ka, kb);
        }
      }
    }
  };
  const int nt = (int)std::max<int64_t>(1, std::min<int64_t>(plan_threads(), nT));
  std::vector<int64_t> cnt;
  try {
    cnt.assign((size_t)nt * (size_t)S, 0);
  } catch (const std::bad_alloc&) {
    return fail(B3R_E_NOMEM, "cannot allocate the planner's per-thread segment counts");
  }
  std::vector<int64_t> bad(nt, 0);
  parallel_ranges(nT, nt, [&](int t, int64_t a, int64_t b) {
    int64_t* c = cnt.data() + (size_t)t * S;
    for_pairs(a, b, [&](int64_t sg, int, int) { if (sg < 0) ++bad[t]; else c[sg]++; });
  }, kPairGrain);
  for (int t = 0; t < nt; ++t) B3R_REQUIRE(bad[t] == 0, "internal: %lld pairs without a segment", (long long)bad[t]);
  B.seg_cnt.assign(S + 1, 0);
  for (int64_t sg = 0; sg < S; ++sg) {
    int64_t run = 0;
    for (int t = 0; t < nt; ++t) run += cnt[(size_t)t * S + sg];
    B.seg_cnt[sg + 1] = B.seg_cnt[sg] + run;
  }
  for (int64_t sg = 0; sg < S; ++sg) {       // per-thread fill offsets
    int64_t run = B.seg_cnt[sg];
    for (int t = 0; t < nt; ++t) {
      const int64_t c = cnt[(size_t)t * S + sg];
      cnt[(size_t)t * S + sg] = run;
      run += c;
    }
  }
  const int64_t P = B.seg_cnt[S];
  try {
    B.pairs.resize(P);
  } catch (const std::bad_alloc&) {
    return fail(B3R_E_NOMEM, "cannot allocate %lld observation pairs", (long long)P);
  }
  // pairs name the elimination records by image-major slot e (the diag pass writes them)
  std::vector<int> e_of_k(B.perm_t.size(), -1);
  for (size_t e = 0; e < B.c1_k.size(); ++e)
    if (B.c1_k[e] >= 0) e_of_k[B.c1_k[e]] = (int)e;
  std::vector<int64_t> missing(nt, 0);
  parallel_ranges(nT, nt, [&](int t, int64_t a, int64_t b) {
    int64_t* fill = cnt.data() + (size_t)t * S;
    for_pairs(a, b, [&](int64_t sg, int ka, int kb) {
      const int2 pr = make_int2(e_of_k[ka], e_of_k[kb]);
      if (pr.x < 0 || pr.y < 0) ++missing[t];
      B.pairs[fill[sg]++] = pr;
    });
  }, kPairGrain);
  for (int t = 0; t < nt; ++t)
    B3R_REQUIRE(missing[t] == 0, "internal: pair observation without an image-major slot");
  build_tasks(B);
  return B3R_OK;
}

// Only the depth-coefficient type is active (focal and pose types off, C <= 8): the plan runs
// the depth-stitch passes with 3 + C float elimination records.
static bool plan_zonly(const PlanBuild& B) {
  bool any_kp = false, any_z = false;
  for (int i = 0; i < B.d->n_imgs; ++i) {
    any_kp = any_kp || B.img_bk[3 * i] >= 0 || B.img_bk[3 * i + 1] >= 0;
    any_z = any_z || B.img_bk[3 * i + 2] >= 0;
  }
  return !any_kp && any_z && B.d->C <= 8;
}
static int plan_record_floats(const PlanBuild& B) {
  return plan_zonly(B) ? round4(3 + B.d->C) : round4(27 + B.d->C);
}

// Pair-task order.  Each task reads the elimination records of its segment's two images from
// L2; within an order that keeps those records resident, the longest tasks go first so that
// the short ones fill in behind them (no long task left for the grid's tail).  Measured on
// configs[2] (the general pass, FP32-issue bound) and configs[4] (the depth-stitch pass, whose
// pair products are 28 FMA on 32-byte records, memory bound):
//   * general plans whose records fit in about twice the L2 (a rank's share on 4 or more GPUs):
//     one global longest-first order (pairs pass 0.240 against 0.279 ms for rank 0 of 4,
//     0.125 against 0.159 ms for rank 0 of 8);
//   * larger general plans: longest first within blocks of consecutive row images holding about
//     64 MB of records (one GPU: 0.832-0.837 ms for blocks of 50-100 images against 0.896 ms
//     row image by row image, 0.897 ms globally);
//   * depth-stitch plans: longest first within each row image (one GPU 2.49 ms, against 2.54 for
//     blocks of 100 images and 4.39 globally).
// The pair lists stay in segment order; a task is a (segment, range).
constexpr double kTaskGlobalBytes = 256e6;   // general plans with fewer record bytes: one order
constexpr double kTaskBlockBytes = 64e6;     // else blocks of row images with about this many
static void build_tasks(PlanBuild& B) {
  const int64_t S = (int64_t)B.seg_col.size();
  const int64_t P = B.seg_cnt[S];
  const int I = B.d->n_imgs;
  std::vector<std::pair<int64_t, int64_t>> cuts;   // (first pair, segment)
  for (int64_t s = 0; s < S; ++s)
    for (int64_t p = B.seg_cnt[s]; p < B.seg_cnt[s + 1]; p += kPairTask) cuts.emplace_back(p, s);
  std::vector<int64_t> ord(cuts.size());
  std::iota(ord.begin(), ord.end(), 0);
  auto len = [&](int64_t t) { return std::min<int64_t>(B.seg_cnt[cuts[t].second + 1] - cuts[t].first, kPairTask); };
  std::vector<int> row_of_seg(S);
  for (int i = 0; i + 1 < (int)B.seg_row_ptr.size(); ++i)
    for (int s2 = B.seg_row_ptr[i]; s2 < B.seg_row_ptr[i + 1]; ++s2) row_of_seg[s2] = i;
  // block of every row image
  std::vector<int> block(I, 0);
  if (plan_zonly(B)) {
    std::iota(block.begin(), block.end(), 0);
  } else {
    const double rec_bytes = 4.0 * plan_record_floats(B);
    std::vector<int64_t> n_img(I, 0);                 // image-major entries (records) per image
    for (size_t c = 0; c + 1 < B.c1_chunk.size(); ++c) n_img[B.c1_img[c]] += B.c1_chunk[c + 1] - B.c1_chunk[c];
    if (rec_bytes * (double)B.c1_obs.size() > kTaskGlobalBytes) {
      double acc = 0.0;
      int blk = 0;
      for (int i = 0; i < I; ++i) {
        if (acc > 0.0 && acc + rec_bytes * (double)n_img[i] > kTaskBlockBytes) { ++blk; acc = 0.0; }
        acc += rec_bytes * (double)n_img[i];
        block[i] = blk;
      }
    }
  }
  std::stable_sort(ord.begin(), ord.end(), [&](int64_t a, int64_t b) {
    const int ba = block[row_of_seg[cuts[a].second]], bb = block[row_of_seg[cuts[b].second]];
    return ba != bb ? ba < bb : len(a) > len(b);
  });
  B.task_pb.resize(cuts.size() + 1);
  B.task_pe.resize(cuts.size());
  B.task_seg.resize(cuts.size());
  for (size_t t = 0; t < ord.size(); ++t) {
    B.task_pb[t] = cuts[ord[t]].first;
    B.task_pe[t] = cuts[ord[t]].first + len(ord[t]);
    B.task_seg[t] = (int)cuts[ord[t]].second;
  }
  B.task_pb[cuts.size()] = P;
}

static inline int pat_lookup(const PlanBuild& B, int p, int q) {
  const int* a = B.col_idx.data() + B.row_ptr[p];
  const int* e = B.col_idx.data() + B.row_ptr[p + 1];
  const int* it = std::lower_bound(a, e, q);
  if (it == e || *it != q) return -1;
  return B.val_off[it - B.col_idx.data()];
}

static int build_pattern(PlanBuild& B) {
  const b3r_plan_desc& d = *B.d;
  const int I = d.n_imgs, nb = B.nb;
  std::vector<uint64_t> keys;
  keys.reserve((size_t)nb + 6 * I + 9 * B.seg_col.size());
  auto add = [&](int p, int q) {
    if (p < 0 || q < 0) return;
    if (p > q) std::swap(p, q);
    keys.push_back((uint64_t)p * (uint64_t)nb + (uint64_t)q);
  };
  for (int p = 0; p < nb; ++p) add(p, p);
  const int32_t* cum = d.infos;
  for (int i = 0; i < I; ++i) {
    const int64_t n_i = cum[i] - (i ? cum[i - 1] : 0);
    if (n_i == 0) continue;
    for (int a = 0; a < 3; ++a)
      for (int b = a; b < 3; ++b) add(B.img_bk[3 * i + a], B.img_bk[3 * i + b]);
  }
  for (int i = 0; i < I; ++i)
    for (int s = B.seg_row_ptr[i]; s < B.seg_row_ptr[i + 1]; ++s) {
      const int i2 = B.seg_col[s];
      for (int a = 0; a < 3; ++a)
        for (int b = 0; b < 3; ++b) add(B.img_bk[3 * i + a], B.img_bk[3 * i2 + b]);
    }
  std::sort(keys.begin(), keys.end());
  keys.erase(std::unique(keys.begin(), keys.end()), keys.end());
  B.row_ptr.assign(nb + 1, 0);
  B.col_idx.resize(keys.size());
  B.val_off.resize(keys.size());
  int64_t v = 0;
  for (size_t j = 0; j < keys.size(); ++j) {
    const int p = (int)(keys[j] / nb), q = (int)(keys[j] % nb);
    B.row_ptr[p + 1]++;
    B.col_idx[j] = q;
    B3R_REQUIRE(v < (int64_t(1) << 31), "S has more than 2^31 values");
    B.val_off[j] = (int)v;
    v += (int64_t)B.bsize[p] * B.bsize[q];
  }
  for (int p = 0; p < nb; ++p) B.row_ptr[p + 1] += B.row_ptr[p];
  B.nnz = v;
  B.blk_row.resize(keys.size());
  for (int p = 0; p < nb; ++p)
    for (int j = B.row_ptr[p]; j < B.row_ptr[p + 1]; ++j) B.blk_row[j] = p;
  // destinations of every segment's 9 sub-blocks
  const int64_t S = (int64_t)B.seg_col.size();
  B.seg_dst.assign(9 * S, -1);
  B.seg_mode.assign(S, 0);
  for (int i = 0; i < I; ++i)
    for (int s = B.seg_row_ptr[i]; s < B.seg_row_ptr[i + 1]; ++s) {
      const int i2 = B.seg_col[s];
      int mode = 0;
      for (int a = 0; a < 3; ++a)
        for (int b = 0; b < 3; ++b) {
          const int p = B.img_bk[3 * i + a], q = B.img_bk[3 * i2 + b];
          int m = kModeNone, off = -1;
          if (p >= 0 && q >= 0) {
            if (p < q) { m = kModeDirect; off = pat_lookup(B, p, q); }
            else if (p > q) { m = kModeTrans; off = pat_lookup(B, q, p); }
            else { m = kModeSym; off = pat_lookup(B, p, p); }
            B3R_REQUIRE(off >= 0, "internal: segment block (%d,%d) missing from pattern", p, q);
          }
          B.seg_dst[9 * s + 3 * a + b] = off;
          mode |= m << (2 * (3 * a + b));
        }
      B.seg_mode[s] = mode;
    }
  // each image's own diagonal-segment destinations: (f,f),(f,t),(f,z),(t,t),(t,z),(z,z)
  static const int AB[6][2] = {{0, 0}, {0, 1}, {0, 2}, {1, 1}, {1, 2}, {2, 2}};
  B.img_dst.assign(6 * I, -1);
  for (int i = 0; i < I; ++i)
    for (int j = 0; j < 6; ++j) {
      const int p = B.img_bk[3 * i + AB[j][0]], q = B.img_bk[3 * i + AB[j][1]];
      if (p >= 0 && q >= 0) B.img_dst[6 * i + j] = pat_lookup(B, p, q);
    }
  // symmetric block rows: row p holds its stored blocks (p, q >= p), then the transposes of
  // the stored blocks (q, p), q < p
  {
    const int64_t nnzb = (int64_t)B.col_idx.size();
    std::vector<int> cnt(nb + 1, 0);
    for (int pr = 0; pr < nb; ++pr)
      for (int j = B.row_ptr[pr]; j < B.row_ptr[pr + 1]; ++j) {
        cnt[pr + 1]++;
        if (B.col_idx[j] != pr) cnt[B.col_idx[j] + 1]++;
      }
    for (int pr = 0; pr < nb; ++pr) cnt[pr + 1] += cnt[pr];
    B.sym_ptr = cnt;
    B.sym_ent.assign(cnt[nb], 0);
    std::vector<int> fill(cnt.begin(), cnt.end() - 1);
    for (int pr = 0; pr < nb; ++pr)
      for (int j = B.row_ptr[pr]; j < B.row_ptr[pr + 1]; ++j) B.sym_ent[fill[pr]++] = 2 * j;
    for (int pr = 0; pr < nb; ++pr)
      for (int j = B.row_ptr[pr]; j < B.row_ptr[pr + 1]; ++j)
        if (B.col_idx[j] != pr) B.sym_ent[fill[B.col_idx[j]]++] = 2 * j + 1;
    B3R_REQUIRE((int64_t)B.sym_ent.size() == 2 * nnzb - nb || nb == 0, "internal: symmetric rows");
    B.mv_ent.resize(B.sym_ent.size());
    for (size_t e = 0; e < B.sym_ent.size(); ++e) {
      const int blk = B.sym_ent[e] >> 1, tr = B.sym_ent[e] & 1;
      const int q = tr ? B.blk_row[blk] : B.col_idx[blk];
      B.mv_ent[e] = make_int4(B.val_off[blk], B.boff[q], B.bsize[q], tr);
    }
    // row panels and matvec tasks (column chunks of <= kMvCols)
    B.pan_off.resize(nb); B.pan_w.resize(nb); B.col_off.resize(nb);
    B.ent_col.resize(B.sym_ent.size()); B.ent_row.resize(B.sym_ent.size());
    int64_t poff = 0;
    int coff = 0;
    for (int pr = 0; pr < nb; ++pr) {
      int w = 0;
      for (int e = B.sym_ptr[pr]; e < B.sym_ptr[pr + 1]; ++e) {
        B.ent_col[e] = w;
        B.ent_row[e] = pr;
        const int q = B.mv_ent[e].y;                      // column scalar offset
        for (int c2 = 0; c2 < B.mv_ent[e].z; ++c2) B.pan_col.push_back(q + c2);
        w += B.mv_ent[e].z;
      }
      B.pan_w[pr] = w;
      B.col_off[pr] = coff;
      B.pan_off[pr] = poff;
      coff += w;
      poff += ((int64_t)B.bsize[pr] * w + 3) & ~int64_t(3);   // 16-byte aligned panels
      const int single = w <= kMvCols ? 1 : 0;
      B3R_REQUIRE((B.pan_off[pr] >> 2) <= INT32_MAX, "PCG row panels beyond 2^33 floats");
      for (int c0 = 0; c0 < w; c0 += kMvCols) {
        B.mv_task.push_back(make_int4(pr, c0, std::min(c0 + kMvCols, w),
                                      single | (c0 == 0 ? 2 : 0) | (B.bsize[pr] << 8)));
        B.mv_row.push_back(make_int4(B.boff[pr], w, (int)(B.pan_off[pr] >> 2), B.col_off[pr]));
      }
    }
    B.pan_floats = poff;
    // PCG row groups, at most one per SM: the resident PCG kernel runs one block per SM,
    // holding its group's panel tiles in shared memory and its scalars in registers.  Rows are
    // packed into contiguous groups of at most X work ((bp + 1) W words: the panel and its
    // column list), kPcgGroupTasks tasks, kPcgSlots task-row sums and kResThreads scalars.  A
    // row above the cap (the focal row of a mono camera couples to every block) is split by
    // its tasks into an owner group and helper groups on other blocks: helpers publish their
    // partial row sums, the owner adds them (in helper order) before it updates the row.
    const int G = std::max(1, B.pcg_target_groups);
    int64_t total = 0;
    auto work_of = [&](int pr) { return (int64_t)(B.bsize[pr] + 1) * B.pan_w[pr]; };
    for (int pr = 0; pr < nb; ++pr) total += work_of(pr);
    auto n_tasks_of = [&](int pr) { return (B.pan_w[pr] + kMvCols - 1) / kMvCols; };
    // Greedy packing under a cap X on a group's work (optimal in the number of groups for
    // contiguous groups); a row above the cap is split into ceil(w / X) parts by its tasks.
    // The smallest cap that needs at most G groups is found by bisection.
    B.mv_slot.assign(B.mv_task.size(), 0);
    const int ncp_all = nb ? B.boff[nb - 1] + B.bsize[nb - 1] : 0;
    B.pcg_scl.assign(ncp_all, make_int2(0, 0));
    int task0 = 0, n_help = 0;
    int g_t0 = -1, g_slots = 0, g_sc0 = 0, g_sc1 = 0, n_groups = 0;
    int64_t g_work = 0;
    bool emit = false;
    auto close_group = [&]() {
      if (g_t0 < 0) return;
      ++n_groups;
      if (emit) {
        B.pcg_grp.push_back(make_int4(g_t0, task0, g_sc0, g_sc1));
        B.pcg_grp2.push_back(make_int4(0, 0, -1, 0));
      }
      g_t0 = -1;
      g_slots = 0;
      g_work = 0;
    };
    auto parts_of = [&](int pr, int64_t X) -> int {    // > 1: a split row
      const int nt = n_tasks_of(pr);
      const int64_t w = work_of(pr);
      const int by_caps = std::max((nt * B.bsize[pr] + kPcgSlots - 9) / (kPcgSlots - 8),   // ceil(nt / parts) tasks fit
                                   (nt + kPcgGroupTasks - 1) / kPcgGroupTasks);
      if (nt <= 1 || (w <= X && by_caps <= 1)) return 1;
      return (int)std::min<int64_t>(nt, std::max<int64_t>((w + X - 1) / X, by_caps));
    };
    auto pack = [&](int64_t X) {
      task0 = 0; n_help = 0; g_t0 = -1; g_slots = 0; g_work = 0; n_groups = 0;
      for (int pr = 0; pr < nb; ++pr) {
        const int nt0 = n_tasks_of(pr), bp0 = B.bsize[pr];
        const int parts = parts_of(pr, X);
        if (parts > 1) {
          close_group();
          const int first_help = n_help;
          for (int part = 0; part < parts; ++part) {
            const int tb = task0 + (int)((int64_t)nt0 * part / parts), te = task0 + (int)((int64_t)nt0 * (part + 1) / parts);
            ++n_groups;
            if (!emit) { if (part > 0) ++n_help; continue; }
            for (int t = tb; t < te; ++t) B.mv_slot[t] = (t - tb) * bp0;
            if (part == 0) {
              for (int r = 0; r < bp0; ++r) B.pcg_scl[B.boff[pr] + r] = make_int2(r, (te - tb) | (bp0 << 16));
              B.pcg_grp.push_back(make_int4(tb, te, B.boff[pr], B.boff[pr] + bp0));
              B.pcg_grp2.push_back(make_int4(first_help, parts - 1, -1, bp0));
            } else {
              B.pcg_grp.push_back(make_int4(tb, te, 0, 0));
              B.pcg_grp2.push_back(make_int4(te - tb, 0, n_help++, bp0));   // helper: its task count, slot
            }
          }
          task0 += nt0;
          continue;
        }
        const int64_t w = work_of(pr);
        if (g_t0 >= 0 && (g_work + w > X || (task0 - g_t0) + nt0 > kPcgGroupTasks || g_slots + nt0 * bp0 > kPcgSlots ||
                          B.boff[pr] + bp0 - g_sc0 > kResThreads))
          close_group();
        if (g_t0 < 0) { g_t0 = task0; g_sc0 = B.boff[pr]; }
        if (emit) {
          for (int t = 0; t < nt0; ++t) B.mv_slot[task0 + t] = g_slots + t * bp0;
          for (int r = 0; r < bp0; ++r) B.pcg_scl[B.boff[pr] + r] = make_int2(g_slots + r, nt0 | (bp0 << 16));
        }
        g_slots += nt0 * bp0;
        g_sc1 = B.boff[pr] + bp0;
        g_work += w;
        task0 += nt0;
      }
      close_group();
      return n_groups;
    };
    int64_t lo = std::max<int64_t>(1, (total + G - 1) / G), hi = std::max<int64_t>(lo, total);
    if (pack(hi) > G) {
      lo = hi;                                        // no cap gets down to G groups: the streaming kernel
    } else {
      while (lo < hi) {
        const int64_t mid = lo + (hi - lo) / 2;
        if (pack(mid) <= G) hi = mid; else lo = mid + 1;
      }
    }
    emit = true;
    pack(lo);
    B.n_pcg_help = n_help;
    B3R_REQUIRE(task0 == (int)B.mv_task.size(), "internal: PCG groups cover %d of %zu tasks", task0,
                B.mv_task.size());
    for (size_t gi = 0; gi < B.pcg_grp.size(); ++gi) {       // the kernels' shared-memory bounds
      const int4 g = B.pcg_grp[gi];
      for (int t = g.x; t < g.y; ++t)
        B3R_REQUIRE(B.mv_slot[t] + (B.mv_task[t].w >> 8) <= kPcgSlots, "internal: PCG group %zu needs more than %d slots",
                    gi, kPcgSlots);
    }
    // resident layout: each group's tasks take, in task order while they fit, (bp + 1) lenp
    // words of their block's shared memory, lenp = len rounded up to 64 (the tile bp x lenp,
    // row-major and zero-padded, then the columns)
    B.mv_soff.assign(B.mv_task.size(), -1);
    int maxb = 0;
    for (int pr = 0; pr < nb; ++pr) maxb = std::max(maxb, B.bsize[pr]);
    bool fits = (int)B.pcg_grp.size() <= G && maxb <= 8;
    for (size_t gi = 0; gi < B.pcg_grp.size(); ++gi) {
      const int4 g = B.pcg_grp[gi];
      if (g.w - g.z > kResThreads || g.y - g.x > kPcgGroupTasks) fits = false;
      int off = 0;
      for (int t = g.x; t < g.y; ++t) {
        const int4 tk = B.mv_task[t];
        const int words = ((tk.w >> 8) + 1) * ((tk.z - tk.y + 63) & ~63);
        if (off + words <= kResSmemWords) { B.mv_soff[t] = off; off += words; }
      }
    }
    B.pcg_resident = fits ? 1 : 0;
  }
  // every image's zcf diagonal block, also when the type is switched off (a dense prior can
  // still be added there)
  B.img_zdiag.assign(I, -1);
  B.img_zsc.assign(I, -1);
  for (int i = 0; i < I; ++i) {
    const int col = B.Z.col[i];
    if (col < 0) continue;
    const int p = B.K.n_cols + B.P.n_cols + col;
    B.img_zdiag[i] = pat_lookup(B, p, p);
    B.img_zsc[i] = B.boff[p];
  }
  // diagonal scalar positions
  const int ncp = nb ? B.boff[nb - 1] + B.bsize[nb - 1] : 0;
  B.sdiag_pos.resize(ncp);
  for (int p = 0; p < nb; ++p) {
    const int base = pat_lookup(B, p, p), bs = B.bsize[p];
    for (int r = 0; r < bs; ++r) B.sdiag_pos[B.boff[p] + r] = base + r * bs + r;
  }
  return B3R_OK;
}

}  // namespace b3r

namespace b3r {
namespace {

// Packs host arrays into one device allocation (256-byte aligned pieces).
struct Arena {
  struct Item { const void* src; size_t bytes; void** dst; size_t off; };
  std::vector<Item> items;
  size_t total = 0;
  template <typename T>
  void add(const std::vector<T>& v, const T** dst) { add_raw(v.data(), v.size() * sizeof(T), (void**)dst); }
  template <typename T>
  void add_mut(size_t count, T** dst) { add_raw(nullptr, count * sizeof(T), (void**)dst); }
  void add_raw(const void* src, size_t bytes, void** dst) { items.push_back({src, bytes, dst, 0}); }
  // Layout: the small constant pieces first, packed into one host image and copied at once (an
  // online plan has ~40 pieces of a few KB, whose separate synchronous copies cost more than
  // their bytes), then the large constant pieces (one copy each, no host staging), then the
  // pieces the kernels fill (nothing copied).
  static constexpr size_t kSmall = size_t(1) << 20;
  int upload(void** base) {
    auto pad = [](size_t b) { return (b + 255) & ~size_t(255); };
    total = 0;
    for (int pass = 0; pass < 3; ++pass)
      for (auto& it : items) {
        const int cls = !it.src ? 2 : (it.bytes < kSmall ? 0 : 1);
        if (cls != pass) continue;
        it.off = total;
        total += pad(it.bytes);
      }
    size_t small_end = 0;
    for (auto& it : items)
      if (it.src && it.bytes < kSmall) small_end = std::max(small_end, it.off + it.bytes);
    if (total == 0) total = 256;
    std::vector<char> img;
    try {
      img.assign(small_end, 0);
    } catch (const std::bad_alloc&) {
      return fail(B3R_E_NOMEM, "host allocation failed for the plan's upload image");
    }
    B3R_TRY(check_cuda(cudaMalloc(base, total), "plan cudaMalloc"));
    for (auto& it : items) {
      *it.dst = (char*)*base + it.off;
      if (!it.src || !it.bytes) continue;
      if (it.bytes < kSmall)
        std::memcpy(img.data() + it.off, it.src, it.bytes);
      else
        B3R_TRY(check_cuda(cudaMemcpy(*it.dst, it.src, it.bytes, cudaMemcpyHostToDevice), "plan upload"));
    }
    if (small_end)
      B3R_TRY(check_cuda(cudaMemcpy(*base, img.data(), small_end, cudaMemcpyHostToDevice), "plan upload"));
    return B3R_OK;
  }
};

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace
}  // namespace b3r

using namespace b3r;

namespace b3r {

// Host state a plan built with b3r_plan_desc.retain keeps for b3r_plan_append: the old
// problem's structure and the parts of its build that an appended problem reuses.
struct PlanState {
  b3r_plan_desc desc{};                   // the problem's sizes and modes (pointers cleared)
  std::vector<int32_t> infos, pids;       // copies of its structure arrays
  std::vector<char> elim, img_live;       // [n_tracks] eliminated, [n_imgs] has an active block
  std::vector<int> loc_tracks, trk_ptr, perm_t, trk_t, img_t, pt_task, kof;
  std::vector<int> seg_row_ptr, seg_col;
  std::vector<int64_t> seg_cnt;
  std::vector<int2> pairs;
};

}  // namespace b3r

// retain (and b3r_plan_append) cover single-rank plans: every track owned, global inputs.
static int check_retain(const b3r_plan_desc& d) {
  B3R_REQUIRE(d.retain == 0 || d.retain == 1, "retain must be 0 or 1");
  if (d.retain)
    B3R_REQUIRE(d.track_owner == nullptr && d.track_begin == 0 && d.track_end == d.n_tracks && !d.obs_local,
                "retain needs a single-rank plan (every track owned, obs_local 0)");
  return B3R_OK;
}

static int retain_state(PlanBuild& B, b3r_plan* P) {
  try {
    std::unique_ptr<PlanState> S(new PlanState());
    const b3r_plan_desc& d = *B.d;
    S->desc = d;
    S->desc.infos = S->desc.pids = S->desc.track_owner = nullptr;
    S->desc.mask_K = S->desc.mask_P = S->desc.mask_Z = S->desc.mask_X = nullptr;
    S->infos.assign(d.infos, d.infos + 3 * (size_t)d.n_imgs);
    S->pids.assign(d.pids, d.pids + d.n_obs);
    S->img_live.resize(d.n_imgs);
    for (int i = 0; i < d.n_imgs; ++i) S->img_live[i] = img_live(B, i);
    S->elim = std::move(B.elim);
    S->loc_tracks = std::move(B.loc_tracks); S->trk_ptr = std::move(B.trk_ptr);
    S->perm_t = std::move(B.perm_t); S->trk_t = std::move(B.trk_t); S->img_t = std::move(B.img_t);
    S->pt_task = std::move(B.pt_task); S->kof = std::move(B.kof);
    S->seg_row_ptr = std::move(B.seg_row_ptr); S->seg_col = std::move(B.seg_col);
    S->seg_cnt = std::move(B.seg_cnt); S->pairs = std::move(B.pairs);
    P->state = S.release();
    return B3R_OK;
  } catch (const std::bad_alloc&) {
    return fail(B3R_E_NOMEM, "host allocation failed while keeping the plan's host state");
  }
}

// The local track, image-major, segment and pair lists of the merged problem B.d (old | new,
// as ObservedTracks.__or__ builds it, inference/tracks.py:96-117) from the old plan's
// retained state.  Old tracks keep their local order, point tasks and pair lists (their
// observation indices and image-major slots shifted by the new observations inserted before
// them); the new tracks follow, ordered by (first image, id) among themselves.
constexpr int kPlanFromScratch = 1;   // build_appended: the extension is planned in full

static int build_appended(PlanBuild& B, const PlanState& O) {
  const b3r_plan_desc& d = *B.d;
  const b3r_plan_desc& d0 = O.desc;
  const int I = d.n_imgs, I0 = d0.n_imgs, T = d.n_tracks, T0 = d0.n_tracks;
  const int nt = plan_threads();
  B3R_REQUIRE(d.C == d0.C, "not an extension: C=%d, the old plan's %d", d.C, d0.C);
  B3R_REQUIRE(I >= I0 && T >= T0 && d.n_cams >= d0.n_cams && d.n_nodes >= d0.n_nodes,
              "not an extension: fewer images, tracks, cameras or nodes than the old plan");
  const int32_t* cum = d.infos;
  const int32_t* cum0 = O.infos.data();
  build_flags(B);
  for (int t = 0; t < T0; ++t)
    B3R_REQUIRE(B.elim[t] == O.elim[t], "not an extension: track %d changes its point status", t);
  // every old image's observations come first in its range, unchanged
  std::vector<int64_t> s_new(I + 1, 0), n_old(I, 0), add_o(I0, 0);
  for (int i = 0; i < I; ++i) s_new[i + 1] = cum[i];
  for (int i = 0; i < I0; ++i) {
    const int64_t s0 = i ? cum0[i - 1] : 0;
    n_old[i] = cum0[i] - s0;
    B3R_REQUIRE(cum[I + i] == cum0[I0 + i] && cum[2 * I + i] == cum0[2 * I0 + i],
                "not an extension: image %d changes its node or camera", i);
    B3R_REQUIRE(img_live(B, i) == (bool)O.img_live[i], "not an extension: image %d changes its active blocks", i);
    B3R_REQUIRE(s_new[i + 1] - s_new[i] >= n_old[i], "not an extension: image %d has fewer observations", i);
    B3R_REQUIRE(std::equal(d.pids + s_new[i], d.pids + s_new[i] + n_old[i], O.pids.data() + s0),
                "not an extension: image %d does not start with the old plan's observations", i);
    add_o[i] = s_new[i] - s0;
  }
  // observations after them belong to new tracks: their per-track lists, in increasing o
  const int nN = T - T0;
  std::vector<int> nptr(nN + 1, 0);
  for (int i = 0; i < I; ++i)
    for (int64_t o = s_new[i] + n_old[i]; o < s_new[i + 1]; ++o) {
      const int t = d.pids[o];
      B3R_REQUIRE(t >= T0, "not an extension: new observation %lld of image %d has old track %d", (long long)o, i, t);
      if (B.elim[t]) nptr[t - T0 + 1]++;
    }
  for (int j = 0; j < nN; ++j) nptr[j + 1] += nptr[j];
  // the new tracks are planned on one thread: a merge that adds more than a quarter of the
  // observations (many frames at once) is planned from scratch on all of them (the structure
  // is an extension all the same)
  if (4 * (d.n_obs - d0.n_obs) > d0.n_obs) return kPlanFromScratch;
  std::vector<int> nobs(nptr[nN]);
  {
    std::vector<int> fill(nptr.begin(), nptr.end() - 1);
    for (int i = 0; i < I; ++i)
      for (int64_t o = s_new[i] + n_old[i]; o < s_new[i + 1]; ++o) {
        const int t = d.pids[o];
        if (B.elim[t]) nobs[fill[t - T0]++] = (int)o;
      }
  }
  // new local tracks (eliminated, non-empty), ordered by (first image, id)
  std::vector<int> new_loc;
  {
    std::vector<int> icnt(I + 1, 0), first(nN, -1);
    for (int j = 0; j < nN; ++j)
      if (nptr[j + 1] > nptr[j]) { first[j] = B.img_of[nobs[nptr[j]]]; icnt[first[j] + 1]++; }
    for (int i = 0; i < I; ++i) icnt[i + 1] += icnt[i];
    new_loc.resize(icnt[I]);
    for (int j = 0; j < nN; ++j)
      if (first[j] >= 0) new_loc[icnt[first[j]]++] = T0 + j;
  }
  const int nT0 = (int)O.loc_tracks.size();
  const int64_t nloc0 = (int64_t)O.perm_t.size();
  const int nT = nT0 + (int)new_loc.size();
  B.loc_tracks.resize(nT);
  std::copy(O.loc_tracks.begin(), O.loc_tracks.end(), B.loc_tracks.begin());
  std::copy(new_loc.begin(), new_loc.end(), B.loc_tracks.begin() + nT0);
  B.trk_col.resize(nT);
  for (int tl = 0; tl < nT; ++tl) B.trk_col[tl] = B.X.col[B.loc_tracks[tl]];
  B.trk_ptr.assign(nT + 1, 0);
  std::copy(O.trk_ptr.begin(), O.trk_ptr.begin() + nT0 + 1, B.trk_ptr.begin());
  for (int j = 0; j < (int)new_loc.size(); ++j) {
    const int jn = new_loc[j] - T0;
    B.trk_ptr[nT0 + j + 1] = B.trk_ptr[nT0 + j] + (nptr[jn + 1] - nptr[jn]);
  }
  const int64_t n_loc = B.trk_ptr[nT];
  B.perm_t.resize(n_loc);
  B.trk_t.resize(n_loc);
  B.img_t.resize(n_loc);
  parallel_ranges(nloc0, nt, [&](int, int64_t a, int64_t b) {
    for (int64_t k = a; k < b; ++k) {
      B.perm_t[k] = (int)(O.perm_t[k] + add_o[O.img_t[k]]);
      B.trk_t[k] = O.trk_t[k];
      B.img_t[k] = O.img_t[k];
    }
  });
  B.kof.assign(d.n_obs, -1);
  for (int i = 0; i < I0; ++i)
    std::copy(O.kof.begin() + (s_new[i] - add_o[i]), O.kof.begin() + (s_new[i] - add_o[i] + n_old[i]),
              B.kof.begin() + s_new[i]);
  for (int j = 0; j < (int)new_loc.size(); ++j) {
    const int jn = new_loc[j] - T0;
    int64_t k = B.trk_ptr[nT0 + j];
    for (int q = nptr[jn]; q < nptr[jn + 1]; ++q, ++k) {
      const int o = nobs[q];
      B.perm_t[k] = o;
      B.trk_t[k] = nT0 + j;
      B.img_t[k] = B.img_of[o];
      B.kof[o] = (int)k;
    }
  }
  B.pt_task = O.pt_task;
  if (!B.pt_task.empty()) B.pt_task.pop_back();   // the old end sentinel
  pack_point_tasks(B, nT0);
  build_image_major(B);
  pack_indices(B);
  // image-major slot of each image's first observation (every observation of an image with an
  // active block has one, in o order: every track is this rank's), merged and old
  std::vector<int64_t> c1s(I + 1, 0), c1s0(I0 + 1, 0);
  for (int i = 0; i < I; ++i) c1s[i + 1] = c1s[i] + (img_live(B, i) ? s_new[i + 1] - s_new[i] : 0);
  for (int i = 0; i < I0; ++i) c1s0[i + 1] = c1s0[i] + (O.img_live[i] ? n_old[i] : 0);
  B3R_REQUIRE(c1s[I] == (int64_t)B.c1_obs.size(), "internal: image-major entries of the merged plan");
  // pairs (a < b) of live observations of the new local tracks
  auto for_new_pairs = [&](auto&& fn) {
    for (int tl = nT0; tl < nT; ++tl)
      for (int64_t ka = B.trk_ptr[tl]; ka < B.trk_ptr[tl + 1]; ++ka) {
        if (!B.obs_live[B.perm_t[ka]]) continue;
        for (int64_t kb = ka + 1; kb < B.trk_ptr[tl + 1]; ++kb)
          if (B.obs_live[B.perm_t[kb]]) fn(B.img_t[ka], B.img_t[kb], ka, kb);
      }
  };
  // segments: each row image's old partners merged with the new tracks' partners
  std::vector<uint64_t> keys;
  for_new_pairs([&](int ia, int ib, int64_t, int64_t) { keys.push_back((uint64_t)ia * (uint64_t)I + (uint64_t)ib); });
  std::sort(keys.begin(), keys.end());
  keys.erase(std::unique(keys.begin(), keys.end()), keys.end());
  B.seg_row_ptr.assign(I + 1, 0);
  B.seg_col.clear();
  std::vector<int64_t> old_seg;   // old segment of each merged segment, -1: new
  {
    size_t kk = 0;
    for (int i = 0; i < I; ++i) {
      const int ob = i < I0 ? O.seg_row_ptr[i] : 0, oe = i < I0 ? O.seg_row_ptr[i + 1] : 0;
      int ia = ob;
      for (;;) {
        const bool has_new = kk < keys.size() && keys[kk] / (uint64_t)I == (uint64_t)i;
        if (ia == oe && !has_new) break;
        const int ca = ia < oe ? O.seg_col[ia] : I;
        const int cb = has_new ? (int)(keys[kk] % (uint64_t)I) : I;
        if (ca <= cb) {
          B.seg_col.push_back(ca);
          old_seg.push_back(ia);
          ++ia;
          if (ca == cb) ++kk;
        } else {
          B.seg_col.push_back(cb);
          old_seg.push_back(-1);
          ++kk;
        }
      }
      B.seg_row_ptr[i + 1] = (int)B.seg_col.size();
    }
  }
  const int64_t S = (int64_t)B.seg_col.size();
  std::vector<int64_t> ncnt(S, 0);
  int64_t bad = 0;
  for_new_pairs([&](int ia, int ib, int64_t, int64_t) {
    const int64_t sg = seg_lookup(B, ia, ib);
    if (sg < 0) ++bad; else ncnt[sg]++;
  });
  B3R_REQUIRE(bad == 0, "internal: %lld new pairs without a segment", (long long)bad);
  B.seg_cnt.assign(S + 1, 0);
  std::vector<int> row_of_seg(S);
  for (int i = 0; i < I; ++i)
    for (int sg = B.seg_row_ptr[i]; sg < B.seg_row_ptr[i + 1]; ++sg) row_of_seg[sg] = i;
  auto old_cnt = [&](int64_t sg) { return old_seg[sg] < 0 ? 0 : O.seg_cnt[old_seg[sg] + 1] - O.seg_cnt[old_seg[sg]]; };
  for (int64_t sg = 0; sg < S; ++sg) B.seg_cnt[sg + 1] = B.seg_cnt[sg] + old_cnt(sg) + ncnt[sg];
  B.pairs.resize(B.seg_cnt[S]);
  // old pairs, their image-major slots shifted by the new entries before them
  parallel_ranges(S, nt, [&](int, int64_t a, int64_t b) {
    for (int64_t sg = a; sg < b; ++sg) {
      const int64_t os = old_seg[sg];
      if (os < 0) continue;
      const int i = row_of_seg[sg], i2 = B.seg_col[sg];
      const int ex = (int)(c1s[i] - c1s0[i]), ey = (int)(c1s[i2] - c1s0[i2]);
      int2* dst = B.pairs.data() + B.seg_cnt[sg];
      for (int64_t p = O.seg_cnt[os]; p < O.seg_cnt[os + 1]; ++p, ++dst)
        *dst = make_int2(O.pairs[p].x + ex, O.pairs[p].y + ey);
    }
  }, 256);
  // new pairs after them, in local track order
  std::vector<int> e_of_k(n_loc - nloc0, -1);
  for (int i = 0; i < I; ++i) {
    if (!img_live(B, i)) continue;
    for (int64_t o = s_new[i] + n_old[i]; o < s_new[i + 1]; ++o) {
      const int k = B.kof[o];
      const int64_t e = c1s[i] + (o - s_new[i]);
      B3R_REQUIRE(B.c1_obs[e] == (int)o, "internal: image-major slot of observation %lld", (long long)o);
      if (k >= nloc0) e_of_k[k - nloc0] = (int)e;
    }
  }
  std::vector<int64_t> fill(S);
  for (int64_t sg = 0; sg < S; ++sg) fill[sg] = B.seg_cnt[sg] + old_cnt(sg);
  for_new_pairs([&](int ia, int ib, int64_t ka, int64_t kb) {
    B.pairs[fill[seg_lookup(B, ia, ib)]++] = make_int2(e_of_k[ka - nloc0], e_of_k[kb - nloc0]);
  });
  build_tasks(B);
  return B3R_OK;
}

static void init_build(PlanBuild& B, const b3r_plan_desc* desc) {
  B.d = desc;
  if (desc->device >= 0) {
    int n_sm = 0;
    if (cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, desc->device) == cudaSuccess && n_sm > 0)
      B.pcg_target_groups = n_sm;
  }
}

static int finish_plan(PlanBuild& B, b3r_plan** out);

extern "C" int b3r_plan_append(b3r_plan** out, const b3r_plan* old, const b3r_plan_desc* desc) {
  B3R_REQUIRE(out != nullptr && old != nullptr && desc != nullptr, "NULL argument");
  *out = nullptr;
  B3R_REQUIRE(old->state != nullptr,
              "the old plan keeps no host state to append to (build it with b3r_plan_desc.retain = 1)");
  B3R_REQUIRE(desc->track_owner == nullptr && desc->track_begin == 0 && desc->track_end == desc->n_tracks &&
              !desc->obs_local, "b3r_plan_append builds single-rank plans (every track owned, obs_local 0)");
  B3R_TRY(check_retain(*desc));
  PlanBuild B;
  init_build(B, desc);
  try {
    B3R_TRY(build_maps(B));
    const int rc = build_appended(B, *old->state);
    if (rc == kPlanFromScratch) {
      B3R_TRY(build_tracks(B));
      B3R_TRY(build_segments(B));
      B3R_TRY(build_pairs(B));
    } else if (rc != B3R_OK) {
      return rc;
    }
    B3R_TRY(build_pattern(B));
    return finish_plan(B, out);
  } catch (const std::bad_alloc&) {
    return fail(B3R_E_NOMEM, "host allocation failed while planning");
  }
}

extern "C" int b3r_plan_create(b3r_plan** out, const b3r_plan_desc* desc) {
  B3R_REQUIRE(out != nullptr && desc != nullptr, "NULL argument");
  *out = nullptr;
  PlanBuild B;
  init_build(B, desc);
  B3R_TRY(check_retain(*desc));
  try {
    B3R_TRY(build_maps(B));
    B3R_TRY(build_tracks(B));
    B3R_TRY(build_segments(B));
    B3R_TRY(build_pairs(B));
    B3R_TRY(build_pattern(B));
    return finish_plan(B, out);
  } catch (const std::bad_alloc&) {
    return fail(B3R_E_NOMEM, "host allocation failed while planning");
  }
}

// Everything after the build_* steps: the device copy of the plan, the workspace layout and
// the info record; keeps the host state for b3r_plan_append when the desc asks for it.
static int finish_plan(PlanBuild& B, b3r_plan** out) {
  const b3r_plan_desc* desc = B.d;
  const bool host_only = desc->device < 0;   // planning only: pattern/info queries, no kernels
  int prev_dev = 0;
  if (!host_only) {
    B3R_TRY(check_cuda(cudaGetDevice(&prev_dev), "cudaGetDevice"));
    B3R_TRY(check_cuda(cudaSetDevice(desc->device), "cudaSetDevice"));
  }
  b3r_plan* P = new (std::nothrow) b3r_plan();
  if (!P) return fail(B3R_E_NOMEM, "plan allocation failed");
  P->device = desc->device;
  DevPlan& d = P->d;
  std::memset(&d, 0, sizeof(d));
  d.n_imgs = desc->n_imgs; d.n_cams = desc->n_cams; d.n_nodes = desc->n_nodes;
  d.n_tracks = desc->n_tracks; d.C = desc->C; d.n_obs = desc->n_obs;
  d.zonly = plan_zonly(B) ? 1 : 0;
  d.R = plan_record_floats(B);
  d.nbK = B.K.n_cols; d.nbP = B.P.n_cols; d.nbZ = B.Z.n_cols; d.nb = B.nb;
  d.off_P = 2 * d.nbK; d.off_Z = d.off_P + 6 * d.nbP;
  d.n_cam_params = d.off_Z + desc->C * d.nbZ;
  d.zeroK = B.K.zero; d.zeroP = B.P.zero; d.zeroZ = B.Z.zero; d.zeroX = B.X.zero;
  d.n_loc = (int64_t)B.perm_t.size();
  d.nT_loc = (int)B.loc_tracks.size();
  d.n_pt_tasks = B.pt_task.empty() ? 0 : (int)B.pt_task.size() - 1;
  d.n_c1 = (int64_t)B.c1_obs.size();
  d.n_c1_chunks = (int)B.c1_img.size();
  d.n_seg = (int64_t)B.seg_col.size();
  d.n_pairs = (int64_t)B.pairs.size();
  d.n_tasks = (int64_t)B.task_seg.size();
  d.nnzb = (int64_t)B.col_idx.size();
  d.nnz = B.nnz;

  // Input rows: the global observation index, or with obs_local the rank of the observation
  // among this rank's own (image-sorted) observations.  The kernels index the caller's
  // per-observation arrays by it; the planner's own structures keep global indices.
  std::vector<int> perm_dev;
  d.first_in = desc->n_obs > 0 ? 0 : -1;
  d.n_in = desc->n_obs;
  if (desc->obs_local) {
    std::vector<int> own(desc->n_obs, -1);
    for (int64_t o = 0; o < desc->n_obs; ++o) {
      const int t = desc->pids[o];
      if (B.owned[t]) {
        own[o] = (int)P->in_obs.size();
        P->in_obs.push_back((int)o);
      }
    }
    perm_dev.resize(B.perm_t.size());
    for (size_t k = 0; k < B.perm_t.size(); ++k) {
      perm_dev[k] = own[B.perm_t[k]];
      B.t_idx[k].w = own[B.t_idx[k].w];
    }
    for (auto& x : B.c1_idx) x.x = own[x.x];
    for (auto& x : B.rest_idx) x.x = own[x.x];
    d.first_in = desc->n_obs > 0 ? own[0] : -1;
    d.n_in = (int64_t)P->in_obs.size();
  }
  Arena A;
  A.add(B.img_bk, &d.img_bk); A.add(B.img_sc, &d.img_sc); A.add(B.img_dst, &d.img_dst);
  A.add(B.img_zdiag, &d.img_zdiag); A.add(B.img_zsc, &d.img_zsc);
  A.add(B.img_node, &d.img_node); A.add(B.img_cam, &d.img_cam);
  A.add(desc->obs_local ? perm_dev : B.perm_t, &d.perm_t); A.add(B.trk_t, &d.trk_t); A.add(B.img_t, &d.img_t);
  A.add(B.loc_tracks, &d.trk_gid); A.add(B.trk_col, &d.trk_col); A.add(B.pt_task, &d.pt_task);
  A.add_mut<float2>(d.n_loc, &d.t_pix); A.add_mut<float2>(d.n_loc, &d.t_std);
  A.add_mut<float>((size_t)d.n_loc * desc->C, &d.t_dep);
  A.add(B.c1_obs, &d.c1_obs); A.add(B.c1_k, &d.c1_k); A.add(B.c1_pid, &d.c1_pid); A.add(B.c1_chunk, &d.c1_chunk);
  A.add(B.c1_img, &d.c1_img);
  A.add(B.rest_idx, &d.rest_idx);
  d.n_rest = (int64_t)B.rest_idx.size();
  A.add(B.seg_dst, &d.seg_dst); A.add(B.seg_mode, &d.seg_mode);
  A.add(B.pairs, &d.pairs); A.add(B.task_pb, &d.task_pb); A.add(B.task_pe, &d.task_pe);
  A.add(B.task_seg, &d.task_seg);
  A.add(B.row_ptr, &d.row_ptr); A.add(B.col_idx, &d.col_idx); A.add(B.val_off, &d.val_off);
  A.add(B.bsize, &d.bsize); A.add(B.boff, &d.boff); A.add(B.sdiag_pos, &d.sdiag_pos);
  A.add(B.blk_row, &d.blk_row); A.add(B.trk_ptr, &d.trk_ptr);
  A.add(B.t_idx, &d.t_idx); A.add(B.c1_idx, &d.c1_idx);
  A.add(B.sym_ptr, &d.sym_ptr); A.add(B.sym_ent, &d.sym_ent);
  A.add(B.mv_task, &d.mv_task); A.add(B.mv_row, &d.mv_row); A.add(B.mv_ent, &d.mv_ent);
  d.n_mv_tasks = (int)B.mv_task.size();
  A.add(B.pcg_grp, &d.pcg_grp); A.add(B.pcg_grp2, &d.pcg_grp2);
  A.add(B.mv_slot, &d.mv_slot); A.add(B.pcg_scl, &d.pcg_scl); A.add(B.mv_soff, &d.mv_soff);
  d.pcg_resident = B.pcg_resident;
  d.n_pcg_groups = (int)B.pcg_grp.size();
  d.n_pcg_help = B.n_pcg_help;
  A.add(B.pan_off, &d.pan_off); A.add(B.pan_w, &d.pan_w); A.add(B.col_off, &d.col_off);
  A.add(B.pan_col, &d.pan_col); A.add(B.ent_col, &d.ent_col); A.add(B.ent_row, &d.ent_row);
  d.pan_floats = B.pan_floats;
  if (!host_only) {
    int rc = A.upload(&P->dev_mem);
    cudaSetDevice(prev_dev);
    if (rc != B3R_OK) { if (P->dev_mem) cudaFree(P->dev_mem); delete P; return rc; }
    P->dev_bytes = A.total;
  }

  // workspace layout: image records | track records | elimination records | staged r/w
  P->ws_img = 0;
  P->ws_trec = align256(P->ws_img + sizeof(float) * kImgRecFloats * (size_t)d.n_imgs);
  P->ws_rec = align256(P->ws_trec + sizeof(float) * 24 * (size_t)d.nT_loc);
  P->ws_rw = align256(P->ws_rec + sizeof(float) * (size_t)d.R * (size_t)d.n_c1);
  P->ws_loss = align256(P->ws_rw + sizeof(float) * 6 * (size_t)d.n_loc);
  P->ws_misc = align256(P->ws_loss + sizeof(double) * ((size_t)d.n_c1_chunks + kRestBlocks));
  const size_t ws_total = P->ws_misc + 256;

  P->pat.row_ptr = std::move(B.row_ptr); P->pat.col_idx = std::move(B.col_idx);
  P->pat.val_off = std::move(B.val_off); P->pat.bsize = std::move(B.bsize);
  P->pat.boff = std::move(B.boff);
  b3r_plan_info& I = P->info;
  std::memset(&I, 0, sizeof(I));
  I.n_obs = desc->n_obs; I.n_obs_local = d.n_loc; I.n_tracks_local = d.nT_loc;
  I.n_blocks = d.nb; I.n_cam_params = d.n_cam_params; I.n_points = B.X.n_cols;
  I.nnzb = d.nnzb; I.nnz = d.nnz; I.n_pairs = d.n_pairs; I.n_segments = d.n_seg;
  I.n_pair_tasks = d.n_tasks; I.n_point_tasks = d.n_pt_tasks; I.n_diag_chunks = d.n_c1_chunks;
  I.workspace_bytes = (int64_t)ws_total;
  I.nb_K = d.nbK; I.nb_P = d.nbP; I.nb_Z = d.nbZ; I.off_P = d.off_P; I.off_Z = d.off_Z;
  I.record_floats = d.R;
  I.n_obs_input = d.n_in;
  I.depth_stitch = d.zonly;
  I.pcg_row_groups = d.n_pcg_groups;
  I.pcg_resident = d.pcg_resident;
  if (desc->retain) {
    const int rc = retain_state(B, P);
    if (rc != B3R_OK) { b3r_plan_destroy(P); return rc; }
  }
  *out = P;
  return B3R_OK;
}

extern "C" int b3r_plan_destroy(b3r_plan* plan) {
  if (!plan) return B3R_OK;
  cudaError_t e = cudaSuccess;
  if (plan->dev_mem) {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(plan->device);
    e = cudaFree(plan->dev_mem);
    cudaSetDevice(prev);
  }
  delete plan->state;
  delete plan;
  return check_cuda(e, "b3r_plan_destroy");
}

extern "C" int b3r_plan_get_info(const b3r_plan* plan, b3r_plan_info* info) {
  B3R_REQUIRE(plan && info, "NULL argument");
  *info = plan->info;
  return B3R_OK;
}

extern "C" int b3r_plan_get_input_obs(const b3r_plan* plan, int32_t* obs) {
  B3R_REQUIRE(plan && obs, "NULL argument");
  if (plan->in_obs.empty()) {
    for (int64_t o = 0; o < plan->d.n_in; ++o) obs[o] = (int32_t)o;
  } else {
    std::copy(plan->in_obs.begin(), plan->in_obs.end(), obs);
  }
  return B3R_OK;
}

extern "C" int b3r_plan_get_pattern(const b3r_plan* plan, int32_t* row_ptr, int32_t* col_idx,
                                    int64_t* val_off, int32_t* block_size, int32_t* block_off) {
  B3R_REQUIRE(plan != nullptr, "NULL plan");
  const HostPattern& p = plan->pat;
  if (row_ptr) std::copy(p.row_ptr.begin(), p.row_ptr.end(), row_ptr);
  if (col_idx) std::copy(p.col_idx.begin(), p.col_idx.end(), col_idx);
  if (val_off) for (size_t j = 0; j < p.val_off.size(); ++j) val_off[j] = p.val_off[j];
  if (block_size) std::copy(p.bsize.begin(), p.bsize.end(), block_size);
  if (block_off) std::copy(p.boff.begin(), p.boff.end(), block_off);
  return B3R_OK;
}
