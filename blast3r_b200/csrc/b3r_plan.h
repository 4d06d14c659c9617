// Internal plan: the static structure of one BA phase, built on the host once
// (b3r_plan.cpp) and read by the fused linearization kernels (b3r_schur.cu).
//
// Index spaces
//   o  image-sorted observation index (the reference layout, tracks.py:853-860)
//   k  local observation index: observations of this rank's eliminated tracks, grouped
//      by track, tracks ordered by (first image, track id) so that tracks seen by the
//      same images are close in memory
//   tl local track index (0 .. nT_loc-1), in that order
//   p  typed parameter block: foc blocks [0, nbK), tau blocks [nbK, nbK+nbP), zcf blocks
//      [nbK+nbP, nb), the column order of the reference solver (ba_solver.py:119, 229)
//   s  segment: an ordered image pair (i <= i') that shares at least one eliminated track
#pragma once
#include <cstdint>
#include <vector>
#include <cuda_runtime.h>
#include "../../include/b3r.h"

namespace b3r {

constexpr int kPairTask = 1024;    // max observation pairs per pair task
constexpr int kDiagChunk = 1024;   // max observations per per-image diagonal chunk
constexpr int kPointTask = 32;     // max observations per point task (one warp)
constexpr int kImgRecFloats = 32;  // floats per per-image camera record
constexpr int kMvCols = 256;       // max panel columns per matvec task (8 per lane)
constexpr int kRestBlocks = 64;     // blocks of the objective pass over observations without an image-major entry
constexpr int kPcgSlots = 1024;    // per-task partial row sums one PCG row group keeps in shared memory
constexpr int kPcgBlocksPerSm = 3; // blocks per SM of the streaming PCG kernel
constexpr int kPcgWarps = 8;       // warps of a streaming PCG block
// The resident PCG kernel: one block of kResWarps warps per SM and one row group per block,
// the group's panel tiles and column lists in kResSmemWords words of shared memory, each of
// its scalars (at most kResThreads) in the registers of one thread.
constexpr int kResWarps = 16;
constexpr int kResThreads = 32 * kResWarps;
constexpr int kResSmemWords = 51200;   // 200 KiB
constexpr int kPcgGroupTasks = 128;    // matvec tasks of a PCG row group

// sub-block destination modes of a segment (2 bits each, 9 sub-blocks)
constexpr int kModeNone = 0, kModeDirect = 1, kModeTrans = 2, kModeSym = 3;

struct DevPlan {
  int n_imgs, n_cams, n_nodes, n_tracks, C, R;   // R = floats per elimination record
  int64_t n_obs;
  int nbK, nbP, nbZ, nb, n_cam_params, off_P, off_Z;
  int zeroK, zeroP, zeroZ, zeroX;
  int64_t first_in;       // input row of global observation 0 (-1: not in this plan's input)
  int64_t n_in;           // rows of the per-observation input arrays
  int zonly;              // only zcf blocks are active (focal and pose types off, C <= 8): the
                          // depth-stitch passes with 3 + C float records run instead

  const int* img_bk;      // [n_imgs*3] active block of (foc, tau, zcf) per image, -1 if none
  const int* img_sc;      // [n_imgs*3] scalar offset of those blocks, -1 if none
  const int* img_dst;     // [n_imgs*6] value offset of the image's own (f,f),(f,t),(f,z),(t,t),(t,z),(z,z)
  const int* img_zdiag;   // [n_imgs] value offset of the image's zcf diagonal block (any mode but
                          //  a masked-out image: -1)
  const int* img_zsc;     // [n_imgs] scalar offset of that block
  const int* img_node;    // [n_imgs]
  const int* img_cam;     // [n_imgs]

  // track-major side (eliminated tracks of this rank)
  int64_t n_loc;
  int nT_loc;
  const int* perm_t;      // [n_loc] input row of local observation k
  const int* trk_t;       // [n_loc] tl of local observation k
  const int* img_t;       // [n_loc] image of local observation k
  const int* trk_gid;     // [nT_loc] global track id
  const int* trk_col;     // [nT_loc] point column of the track in the delta vector
  int n_pt_tasks;
  const int* pt_task;     // [n_pt_tasks+1] first k of each point task
  float2* t_pix;          // [n_loc] staged pix2d
  float2* t_std;          // [n_loc] staged pix2d_std
  float* t_dep;           // [C][n_loc] staged pix2d_dep (channel-major)

  // image-major side (observations owned by this rank)
  int64_t n_c1;
  const int* c1_obs;      // [n_c1] o
  const int* c1_k;        // [n_c1] k, -1 if the track is not eliminated
  const int* c1_pid;      // [n_c1] track id (point index) of the observation
  int n_c1_chunks;
  const int* c1_chunk;    // [n_c1_chunks+1]
  // this rank's observations in images without an active block (no image-major entry): only
  // their residuals and losses are evaluated
  int64_t n_rest;
  const int4* rest_idx;   // [n_rest] (input row, image, track id, 0)
  const int* c1_img;      // [n_c1_chunks]

  // segments and their pair lists
  int64_t n_seg, n_pairs, n_tasks;
  const int* seg_dst;     // [n_seg*9] value offset of each (a,b) sub-block, -1 none
  const int* seg_mode;    // [n_seg] 2 bits per sub-block (a*3+b)
  const int2* pairs;      // [n_pairs] (e_row, e_col): image-major slots of the two observations
  const int64_t* task_pb; // [n_tasks] first pair of each task (tasks longest first)
  const int64_t* task_pe; // [n_tasks] end of each task
  const int* task_seg;    // [n_tasks]

  // S pattern
  int64_t nnzb, nnz;
  const int* row_ptr;     // [nb+1]
  const int* col_idx;     // [nnzb]
  const int* val_off;     // [nnzb]
  const int* bsize;       // [nb]
  const int* boff;        // [nb]
  const int* sdiag_pos;   // [n_cam_params] position of each diagonal scalar in S_vals
  const int* blk_row;     // [nnzb] block row of each stored block
  const int* trk_ptr;     // [nT_loc+1] first k of each local track
  const int4* t_idx;      // [n_loc] (image, global track id, tl, input row) of local observation k
  const int4* c1_idx;     // [n_c1] (input row, k or -1, track id, tl or -1) of image-major entry e
  // the full (symmetric) block rows of S for an atomic-free matvec: entries of block row p
  // are sym_ent[sym_ptr[p] .. sym_ptr[p+1]), each 2 * stored block + 1 if it is the
  // transpose of a stored block (q, p) with q < p
  const int* sym_ptr;     // [nb+1]
  const int* sym_ent;     // [2*nnzb - nb]
  // matvec work: row panels cut into tasks of <= kMvCols columns (a dense row,
  // e.g. the shared focal block of a mono-camera rig, spreads over many warps)
  int n_mv_tasks;
  const int4* mv_task;    // [n_mv_tasks] (block row, first panel column, end panel column,
                          //  1 if the row is one task | 2 if this is the row's first task |
                          //  the row's block size << 8)
  const int4* mv_row;     // [n_mv_tasks] the task's row fields, loaded beside mv_task so that no
                          //  load waits on another: (boff, W_p, pan_off / 4, col_off)
  const int4* mv_ent;     // [2*nnzb - nb] (value offset, column scalar offset, column block size,
                          //  1 if the entry is the transpose of the stored block)
  // row panels of the symmetric S for the PCG matvec: block row p is a dense bp x W_p
  // row-major panel (its entries' blocks side by side, transposes already flipped) at
  // float offset pan_off[p], with the W_p scalar columns at pan_col[col_off[p] ..]
  int64_t pan_floats;
  const int64_t* pan_off; // [nb]
  const int* pan_w;       // [nb] W_p
  const int* col_off;     // [nb]
  const int* pan_col;     // [sum W_p]
  const int* ent_col;     // [2*nnzb - nb] first panel column of each symmetric entry
  const int* ent_row;     // [2*nnzb - nb] block row of each symmetric entry
  // PCG row groups: contiguous block rows whose matvec tasks and vector updates one CTA does
  // (so the update of a row never waits for another CTA's matvec); about one group per
  // resident CTA, balanced by panel work
  int n_pcg_groups, n_pcg_help;
  const int4* pcg_grp;    // [n_pcg_groups] (first task, end task, first scalar, end scalar)
  const int4* pcg_grp2;   // [n_pcg_groups] owner of a split row: (first helper slot, helpers, -1,
                          //  block size); helper: (tasks, 0, its helper slot, block size);
                          //  others (0, 0, -1, 0)
  const int* mv_slot;     // [n_mv_tasks] first shared-memory slot of the task's row sums
  const int* mv_soff;     // [n_mv_tasks] resident kernel: word offset (a multiple of 64) of the
                          //  task's tile (bp x lenp, lenp = len rounded up to 64) and column list
                          //  in its block's shared memory, -1: read from the panel
  int pcg_resident;       // 1: the row groups fit the resident kernel (one per SM, <= kResThreads
                          //  scalars, block sizes <= 8)
  const int2* pcg_scl;    // [n_cam_params] (slot of the scalar's first task, the row's task
                          //  count | block size << 16): the scalar sums its tasks' slots in order
};

struct HostPattern {
  std::vector<int> row_ptr, col_idx, val_off, bsize, boff;
};

// Host state a plan keeps for b3r_plan_append (b3r_plan.cpp); null unless the plan was built
// with b3r_plan_desc.retain.
struct PlanState;

}  // namespace b3r

struct b3r_plan {
  b3r::DevPlan d;
  b3r::HostPattern pat;
  b3r_plan_info info;
  int device = 0;
  void* dev_mem = nullptr;
  size_t dev_bytes = 0;
  // workspace layout (byte offsets): image records | track records (24 floats: Hpp, g_p,
  // then the Cholesky factor in reciprocal form and L^-1 g_p) | elimination records (one
  // per image-major slot e) | staged r/w | misc scalars
  size_t ws_img = 0, ws_trec = 0, ws_rec = 0, ws_rw = 0, ws_loss = 0, ws_misc = 0;
  int64_t n_pairs_total = 0;
  std::vector<int> in_obs;   // global observation of each input row (empty: the identity)
  bool staged = false;
  const void* staged_src[3] = {nullptr, nullptr, nullptr};
  b3r::PlanState* state = nullptr;   // owned; freed by b3r_plan_destroy
};
