/*
 * b3r.h -- C ABI of the B200-native BLASt3R bundle-adjustment linearization library.
 *
 * Every entry point takes plain pointers and sizes (device pointers unless stated
 * otherwise), an opaque CUDA stream handle (`void* stream`, a cudaStream_t; NULL = the
 * legacy default stream) and returns an int status: B3R_OK (0) or a negative B3R_E_*
 * code, with a message available from b3r_last_error().  No C++ exception crosses the
 * ABI.  All work is enqueued asynchronously on `stream`; nothing synchronises the
 * device.  The library never allocates output buffers: callers pass them in.
 *
 * Part 1 mirrors, one to one, the native ops the reference binds through pybind
 * (naver/blast3r, src/blast3r/extensions/cujac/sfm_jacobian_rigs.cu:1254-1275, re-exported
 * by extensions/cujac/__init__.py:18-22), with the same argument meaning and layouts.
 *
 * Part 2 is the fused hot path that replaces the reference's per-LM-iteration
 * linearization (GaussNewtonSolver.compute_jacobians + solve_delta up to its PCG,
 * inference/ba_solver.py:34-188): residual, Jacobians, Huber/IRLS weights, per-track
 * 3x3 point-block inversion and the Schur-reduced camera/depth system
 * S = Hcc - Hcp Hpp^-1 Hpc with its gradient b, written into a precomputed
 * block-sparse pattern of S.
 */
#ifndef B3R_H
#define B3R_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B3R_OK 0
#define B3R_E_INVALID -1     /* bad argument (shape, size, flag, NULL pointer)        */
#define B3R_E_CUDA -2        /* a CUDA runtime call failed                            */
#define B3R_E_NOMEM -3       /* host or device allocation failed (plan creation only) */
#define B3R_E_UNSUPPORTED -4 /* valid request this build does not implement           */

#define B3R_F32 0
#define B3R_F64 1

/* Message of the last failed call on the calling thread ("" if none). */
const char* b3r_last_error(void);
/* Library version string. */
const char* b3r_version(void);

/* ===================================================================================
 * Part 1 -- reference op mirrors
 * =================================================================================== */

/* Residuals, Huber error and IRLS weights per observation.
 * Replaces residuals_with_rigs (sfm_jacobian_rigs.cu:1048-1101, kernel :129-259).
 * infos: int32 [3, n_imgs] = (cumulative obs count per image, node id, cam id);
 * K [n_cams,3,3]; P_rig2c [n_cams,4,4] with `P_rig2c_stride` floats between cameras;
 * P_w2rig [n_nodes,4,4]; z_coefs [n_imgs,C]; pts3d [n_tracks,3]; pids int32 [n_obs];
 * pix2d, pix2d_std [n_obs,2]; pix2d_dep [n_obs,C].
 * out: float [n_out, n_obs] with n_out = 9 if pnorm > 0 else 3 (rows: residual x,y,z,
 * err x,y,z, weight x,y,z); the reference returns it transposed as (n_obs, n_out).
 * Rows of observations whose camera depth is <= 1e-3 are zero.  pnorm must be -1 or in
 * (0, 2] (sfm_jacobian_rigs.cu:1067). */
int b3r_residuals_with_rigs(const int32_t* infos, int n_imgs, const float* K, int n_cams,
                            const float* P_rig2c, int64_t P_rig2c_stride, const float* P_w2rig,
                            int n_nodes, const float* z_coefs, int C, const float* pts3d,
                            int n_tracks, const int32_t* pids, int64_t n_obs, const float* pix2d,
                            const float* pix2d_std, const float* pix2d_dep, int is_depth_log,
                            float weight_z, float pnorm, float max_pix_err, float huber_delta,
                            float w_pts_nul, float* out, void* stream);

/* The objective of lm_step (inference/engine.py:263-281: the residual op's Huber errors,
 * summed) in one pass, without the [9, n_obs] buffer: loss_sum (device double [1]) = the sum
 * over observations and components of the Huber error (the reference's loss is
 * loss_sum / (3 n_obs)); residuals (device float [3, n_obs], or NULL) receives rows 0..2 of
 * b3r_residuals_with_rigs (the residuals the line search scores).  Same inputs and numerics as
 * b3r_residuals_with_rigs; pnorm in (0, 2]; the zero-weight value of clipped residuals does not
 * enter the loss.  No counterpart among the reference's native ops: it fuses its residual op
 * with the torch reduction that follows it. */
int b3r_residual_loss(const int32_t* infos, int n_imgs, const float* K, int n_cams, const float* P_rig2c,
                      int64_t P_rig2c_stride, const float* P_w2rig, int n_nodes, const float* z_coefs, int C,
                      const float* pts3d, int n_tracks, const int32_t* pids, int64_t n_obs, const float* pix2d,
                      const float* pix2d_std, const float* pix2d_dep, int is_depth_log, float weight_z,
                      float pnorm, float max_pix_err, float huber_delta, double* loss_sum, float* residuals,
                      void* stream);

/* Explicit Jacobians per observation.
 * Replaces jacobians_with_rigs (sfm_jacobian_rigs.cu:1105-1148, kernel :323-509).
 * J_cam [n_obs,3,8] (d/dfx, d/dfy, d/dtau x6), J_zcf [n_obs,1,C] (depth row only),
 * J_pts [n_obs,3,3]; element type float (output_float64 = 0) or double (= 1), computed
 * in that precision from the float inputs as the reference does.  The three outputs are
 * fully written (zero rows for invalid depth). */
int b3r_jacobians_with_rigs(const int32_t* infos, int n_imgs, const float* K, int n_cams,
                            const float* P_rig2c, int64_t P_rig2c_stride, const float* P_w2rig,
                            int n_nodes, const float* z_coefs, int C, const float* pts3d,
                            int n_tracks, const int32_t* pids, int64_t n_obs,
                            const float* pix2d_std, const float* pix2d_dep, int is_depth_log,
                            int output_float64, void* J_cam, void* J_zcf, void* J_pts,
                            void* stream);

/* Batched 3x3 SPD solve by guarded Cholesky with diagonal jitter.
 * Replaces chol3x3_solve (sfm_jacobian_rigs.cu:1151-1169, kernel :560-634).
 * blocks [N,3,3], rhs [N,3], out [N,3], dtype B3R_F32 or B3R_F64. */
int b3r_chol3x3_solve(const void* blocks, const void* rhs, void* out, int64_t N, double jitter,
                      int dtype, void* stream);

/* Block-COO matrix-vector product y = A x (transpose = 0) or y = A^T x (transpose = 1).
 * Replaces blockcoo_matvec (sfm_jacobian_rigs.cu:1171-1219, kernel :760-803).
 * blocks [N,bh,bw]; row/col indices int32 (index_is_64 = 0) or int64 (= 1), in blocks;
 * the matrix has HB1 x WB1 blocks; x has WB1*bw (HB1*bh if transposed) entries; y has
 * HB1*bh (WB1*bw) entries and is overwritten.  Any bh, bw in 1..32 is accepted (the
 * reference instantiates 31 fixed shapes). */
int b3r_blockcoo_matvec(const void* blocks, int bh, int bw, const void* row_idx,
                        const void* col_idx, int index_is_64, int64_t N, const void* x, void* y,
                        int64_t HB1, int64_t WB1, int transpose, int dtype, void* stream);

/* out[b] = left[b]^T right[b] for left [B,K,I] (strides l_bs, l_ks, unit inner stride) and
 * right [B,K,J] (strides r_bs, r_ks); out [B,I,J] contiguous.
 * Replaces fused_einsum_bki_bkj (sfm_jacobian_rigs.cu:1222-1250, kernel :880-941).
 * Any K, I, J with I*J <= 1024 is accepted. */
int b3r_fused_einsum_bki_bkj(const void* left, int64_t l_bs, int64_t l_ks, const void* right,
                             int64_t r_bs, int64_t r_ks, void* out, int64_t B, int K, int I, int J,
                             int dtype, void* stream);

/* ===================================================================================
 * Part 2 -- fused linearization + Schur assembly
 * =================================================================================== */

/* How one parameter type takes part, mirroring GaussNewtonSolver.enable
 * (inference/ba_solver.py:72-108): */
#define B3R_ENABLE_ALL 0   /* status True: every block is a variable                    */
#define B3R_ENABLE_ZERO 1  /* status False: columns kept, J zero, damped to 1e-12 * I    */
#define B3R_ENABLE_MASK 2  /* bool tensor: disabled blocks' columns are removed          */

typedef struct b3r_plan b3r_plan;

/* Problem structure, fixed for one BA phase.  `infos` and `pids` are HOST pointers
 * (the image-sorted observation layout of ObservedTracks / RigsData.infos,
 * inference/tracks.py:20-31, inference/rigs.py:50-51). */
typedef struct {
    int32_t n_imgs, n_cams, n_nodes, n_tracks;
    int64_t n_obs;
    int32_t C;                        /* number of depth coefficients per image            */
    const int32_t* infos;             /* host, int32 [3, n_imgs]                           */
    const int32_t* pids;              /* host, int32 [n_obs]                               */
    int32_t mode_K, mode_P, mode_Z, mode_X;          /* B3R_ENABLE_*                       */
    const uint8_t *mask_K, *mask_P, *mask_Z, *mask_X; /* host bool masks for MODE_MASK    */
    int32_t track_begin, track_end;   /* tracks owned by this rank (all: 0, n_tracks), used
                                         when track_owner is NULL                          */
    int32_t device;                   /* CUDA device ordinal the plan lives on; < 0 builds
                                         a host-only plan (info and pattern queries only) */
    int32_t obs_local;                /* 0: the per-observation arrays handed to the
                                         linearization (pix2d, pix2d_std, pix2d_dep, and
                                         residuals / w_pts) are the global image-sorted ones
                                         (n_obs rows); 1: they hold only the observations of
                                         this rank's tracks, in
                                         image-sorted order (n_obs_input rows, the order
                                         b3r_plan_get_input_obs lists), so a sharded caller
                                         keeps and copies only its own shard */
    const int32_t* track_owner;       /* host, int32 [n_tracks] or NULL: when given, this
                                         rank owns the tracks t with track_owner[t] == rank
                                         (any partition, e.g. by first image, so that a
                                         rank's tracks share images) instead of the range */
    int32_t rank;
    int32_t retain;                   /* 1: the plan keeps its host-side track, segment and
                                         pair lists so that b3r_plan_append can extend it
                                         (single-rank plans: every track owned, obs_local 0);
                                         costs host memory of about 40 B per observation
                                         plus 8 B per observation pair */
} b3r_plan_desc;

typedef struct {
    int64_t n_obs, n_obs_local, n_tracks_local;   /* observations / eliminated tracks here */
    int32_t n_blocks;                 /* typed parameter blocks (foc | tau | zcf)          */
    int32_t n_cam_params;             /* size of the reduced camera/depth vector           */
    int32_t n_points;                 /* point-block count of the full delta (3 each)      */
    int64_t nnzb;                     /* stored blocks of S (upper block triangle)         */
    int64_t nnz;                      /* floats in the S value array                       */
    int64_t n_pairs, n_segments, n_pair_tasks, n_point_tasks, n_diag_chunks;
    int64_t workspace_bytes;          /* scratch bytes b3r_linearize_* needs               */
    int32_t nb_K, nb_P, nb_Z;         /* blocks per type                                   */
    int32_t off_P, off_Z;             /* scalar offsets of the tau and zcf ranges          */
    int32_t record_floats;            /* floats per per-observation elimination record     */
    int64_t n_obs_input;              /* rows of the per-observation input arrays          */
    int32_t depth_stitch;             /* 1: only depth-coefficient blocks are active (focal
                                         and pose types off, C <= 8) and the linearization
                                         runs its depth-stitch passes                       */
    int32_t pcg_row_groups;           /* row groups of the PCG (one per block)             */
    int32_t pcg_resident;             /* 1: the PCG runs its resident kernel (one block per
                                         SM holding its rows of S in shared memory), 0: the
                                         streaming kernel (rows of S read from L2)          */
} b3r_plan_info;

/* Build the plan: image -> block maps, the track-sorted observation order, per-warp
 * point tasks, the image-pair segments with their observation-pair lists, and the
 * block-sparse pattern of S (upper block triangle, diagonal blocks stored in full).
 * The pattern is the same on every rank of a sharded problem (it is built from all
 * tracks); pair lists and tasks only cover tracks [track_begin, track_end).
 * Replaces the structure discovery the reference redoes every iteration inside
 * HStackMat.gram_matrix / OneBlockPerRow.__matmul__obpc_obpr (ba_solver.py:854-924). */
int b3r_plan_create(b3r_plan** plan, const b3r_plan_desc* desc);

/* Incremental planning for the online track merge.  `desc` describes the merged problem
 * `old | new` the way ObservedTracks.__or__ (inference/tracks.py:96-117) builds it for the
 * online loop (inference/pipeline.py:196-224): every image of `old` keeps its node, camera
 * and observations, which come first in its range; observations after them, and all
 * observations of images added at the end, belong to new tracks (ids >= old n_tracks);
 * nodes, cameras, images and tracks are only added.  Builds the merged plan from the
 * host state `old` retained (b3r_plan_desc.retain): old tracks keep their local order,
 * point tasks and pair lists (observation and image-major indices shifted), only the new
 * tracks are sorted, paired and bucketed, and the S pattern and solver tables are rebuilt.
 * The result is a plan for `desc` like b3r_plan_create's (same S pattern, same systems up
 * to summation order); it retains its own state when desc->retain is set.  `old` is not
 * changed.  A merge that adds more than a quarter of the observations (many frames at once)
 * is planned in full inside the call.  Returns B3R_E_INVALID, naming the first difference, when `desc` does not
 * extend `old` (track removal, reordering, other rules), in which case the caller plans
 * from scratch.  No counterpart in the reference, which rediscovers the structure every
 * iteration (ba_solver.py:854-924). */
int b3r_plan_append(b3r_plan** plan, const b3r_plan* old, const b3r_plan_desc* desc);
int b3r_plan_destroy(b3r_plan* plan);
int b3r_plan_get_info(const b3r_plan* plan, b3r_plan_info* info);

/* Host copies of the S pattern: row_ptr [n_blocks+1], col_idx [nnzb] (block columns,
 * ascending, >= row), val_off [nnzb] (offset of each dense row-major block in the value
 * array), block_size [n_blocks], block_off [n_blocks] (scalar offset in the reduced
 * camera/depth vector).  Any pointer may be NULL. */
int b3r_plan_get_pattern(const b3r_plan* plan, int32_t* row_ptr, int32_t* col_idx,
                         int64_t* val_off, int32_t* block_size, int32_t* block_off);

/* Global image-sorted index of every row of the per-observation input arrays
 * (b3r_plan_info.n_obs_input entries): 0, 1, ... n_obs-1 for a plan with obs_local = 0,
 * else the observations of this rank's tracks in image order.  Host pointer. */
int b3r_plan_get_input_obs(const b3r_plan* plan, int32_t* obs);

/* Gather the static observation data (device pointers, image-sorted reference layout:
 * pix2d [n_obs,2], pix2d_std [n_obs,2], pix2d_dep [n_obs,C]) into the plan's
 * track-sorted structure-of-arrays copy.  Call once per phase, or whenever those arrays
 * change; pix2d may be NULL when residuals and weights are passed to the linearization
 * instead of being recomputed. */
int b3r_plan_stage_obs(b3r_plan* plan, const float* pix2d, const float* pix2d_std,
                       const float* pix2d_dep, void* stream);

/* Per-iteration parameters (device pointers, reference layouts and dtypes). */
typedef struct {
    const float* K;            /* [n_cams,3,3]                                        */
    const float* P_rig2c;      /* [n_cams,4,4], P_rig2c_stride floats apart            */
    int64_t P_rig2c_stride;
    const float* P_w2rig;      /* [n_nodes,4,4]                                       */
    const float* z_coefs;      /* [n_imgs,C]                                          */
    const float* pts3d;        /* [n_tracks,3]                                        */
    const float* pix2d;        /* [n_obs,2] image-sorted; NULL: use residuals/w below */
    const float* pix2d_std;    /* [n_obs,2] image-sorted                              */
    const float* pix2d_dep;    /* [n_obs,C] image-sorted                              */
    /* residuals (n_obs,3) and IRLS weights (n_obs, w_cols in {1,3}) as the solver receives
     * them (ba_solver.py:110); strides in floats.  Used only when pix2d == NULL. */
    const float* residuals;
    int64_t res_stride_n, res_stride_c;
    const float* w_pts;
    int64_t w_stride_n, w_stride_c;
    int32_t w_cols;
} b3r_params;

/* Solver options (lm_step / GaussNewtonSolver arguments, engine.py:206-219, ba_solver.py:22,
 * residual op arguments sfm_jacobian_rigs.cu:1255-1258). */
typedef struct {
    int32_t is_depth_log;
    float weight_z, pnorm, max_pix_err, huber_delta, w_pts_nul;
    float clamp_w_lo, clamp_w_hi;     /* W clamp of solve_delta (1e-6, 1e6)              */
    double dampen;                    /* 1e-12                                           */
    int32_t adaptive_dampen;          /* damping x max |diag| per block type             */
    int32_t no_grad_f_from_rz, optim_Z0, optim_Z_1st_cam;
} b3r_lin_opts;

/* Device outputs of one linearization (caller-owned, overwritten). */
typedef struct {
    float* S_vals;     /* [nnz]           block values of S (upper block triangle)          */
    float* b;          /* [n_cam_params]  reduced gradient g_c - Hcp Hpp^-1 g_p            */
    float* diagA;      /* [n_cam_params]  undamped diag(Hcc) (needed across ranks)         */
    float* precond;    /* [n_cam_params]  max(diag(A) + damping, 1e-12), or NULL           */
    float* hpp_max;    /* [1]             max |diag(Hpp)| over this rank's tracks (NULL:
                          kept in the workspace; sharded callers pass it to all-reduce it) */
    float* residuals;  /* [3, n_obs_input] or NULL: the residuals of this plan's observations
                          (rows x, y, depth, at each observation's input row; others untouched),
                          as b3r_residuals_with_rigs computes them                            */
    double* loss;      /* [1] or NULL: the sum of their Huber errors (the objective's numerator;
                          a partial sum on each rank of a sharded problem).  Both need
                          params->pix2d (in-kernel residuals) and are written by
                          b3r_lin_assemble                                                    */
} b3r_outputs;

/* One full linearization on one GPU: b3r_lin_points, b3r_lin_assemble and
 * b3r_lin_finalize in sequence.  `workspace`: b3r_plan_info.workspace_bytes of device
 * memory, 256-byte aligned; it keeps the per-track Cholesky factors and per-observation
 * elimination records needed by b3r_backsub. */
int b3r_linearize_schur(b3r_plan* plan, const b3r_params* params, const b3r_lin_opts* opts,
                        void* workspace, const b3r_outputs* out, void* stream);

/* Same as b3r_linearize_schur, but allocates nothing and needs no caller workspace.
 * No counterpart in the reference.  For hosts that use this library only through its C
 * ABI and have no way to allocate device memory themselves (a Go, Java or plain C
 * program without a CUDA allocator, or an engine whose memory pool forbids allocations
 * inside its iteration loop).  The workspace is a fixed 32 MiB device array inside the
 * library, held by every GPU that loads it until the process exits; plans whose
 * b3r_plan_info.workspace_bytes exceed it are rejected with B3R_E_INVALID (enough for
 * an online window of ~150k observations).  The caller still passes the plan, the
 * parameters and the outputs.  The first call on a device looks up the array's device
 * address (make that first call before any stream capture); the address is kept for the
 * life of the process, so do not use this entry point after a cudaDeviceReset of that
 * device (the library's module, and the array's address, may change).  All calls on a device share
 * the one array, so calls that overlap on the GPU (other streams, other threads) race:
 * serialise them.  Back-substitution after this call is not available (it needs the
 * caller's workspace). */
int b3r_linearize_schur_noalloc(b3r_plan* plan, const b3r_params* params, const b3r_lin_opts* opts,
                                const b3r_outputs* out, void* stream);

/* Stage 1: per-track Hpp and g_p, and out->hpp_max (the adaptive damping of the point
 * blocks needs the max over ALL tracks: sharded callers all-reduce it before stage 2). */
int b3r_lin_points(b3r_plan* plan, const b3r_params* params, const b3r_lin_opts* opts,
                   void* workspace, const b3r_outputs* out, void* stream);
/* Stage 2: per-track factors, elimination records with the per-image diagonal blocks,
 * pair products, b and diag(A).
 * Zeroes and accumulates out->S_vals, out->b, out->diagA (partial sums on each rank). */
int b3r_lin_assemble(b3r_plan* plan, const b3r_params* params, const b3r_lin_opts* opts,
                     void* workspace, const b3r_outputs* out, void* stream);
/* Stage 3: per-type adaptive damping of S's diagonal from the (reduced) diag(A)
 * (ba_solver.py:510-517, 572-582) and the Jacobi preconditioner. */
int b3r_lin_finalize(b3r_plan* plan, const b3r_lin_opts* opts, void* workspace,
                     const b3r_outputs* out, void* stream);

/* Preconditioned conjugate gradient on the assembled S (the reference's _pcg,
 * inference/ba_solver.py:1197-1238, as solve_delta calls it at :202): solves S x = b from
 * x0 = 0 with the Jacobi preconditioner precond (out->precond of the linearization),
 * stopping at the first iterate with ||r|| <= tol ||b|| (converged, returned), breaking on a
 * non-finite r.z, else returning the best-so-far iterate after maxiter iterations.  One
 * cooperative kernel runs the whole loop on `stream`, in the pipelined form of the
 * iteration (one grid-wide barrier per iteration; every wait is bounded).  Where the plan's
 * row groups fit (b3r_plan_info.pcg_resident) each SM's block keeps its rows of S in shared
 * memory and its elements of the vectors in registers for the whole solve; else the rows of
 * S are streamed from L2 every iteration.  A stop is taken
 * only when the true residual b - S x meets the tolerance (if the recurrences' residual
 * has drifted, the iteration continues from true values).  `work` is a 256-byte aligned device
 * buffer of b3r_pcg_work_bytes(plan) bytes; `result` is a device int[4] receiving
 * (iterations, converged, device error, residual replacements) -- read it after
 * synchronising the stream.
 * b3r_pcg uses float vectors, b3r_pcg_f64 double vectors; S stays float either way.
 * Replaces the reference's per-iteration Python loop; no counterpart in its native ops. */
int64_t b3r_pcg_work_bytes(const b3r_plan* plan);
int b3r_pcg(const b3r_plan* plan, const float* S_vals, const float* precond, const float* b, float* x,
            double tol, int maxiter, void* work, int* result, void* stream);
int b3r_pcg_f64(const b3r_plan* plan, const float* S_vals, const float* precond, const double* b, double* x,
                double tol, int maxiter, void* work, int* result, void* stream);

/* The same solve with the vector type given by dtype (B3R_F32 or B3R_F64; b and x of that
 * type), and the limit of every grid-barrier wait inside the kernel: `barrier_spin_limit`
 * polls of about 32 ns each (<= 0: the default of b3r_pcg, about half a second).  A wait
 * that runs out makes every block leave the kernel at that barrier or the next, x is zeroed
 * and result[2] = 1; the context stays usable.  flags: 0, or
 * B3R_PCG_TEST_UNREACHABLE_BARRIER, a test of that failure path in which the first barrier
 * waits for an arrival that no block makes, B3R_PCG_STREAMING, which runs the streaming
 * kernel also where the resident one fits (both compute the same iteration), and
 * B3R_PCG_TEST_GLOBAL_TILES, a test of the resident kernel's path for rows of S beyond its
 * shared memory, taken here for every row. */
#define B3R_PCG_TEST_UNREACHABLE_BARRIER 1
#define B3R_PCG_STREAMING 2
#define B3R_PCG_TEST_GLOBAL_TILES 4
int b3r_pcg_ex(const b3r_plan* plan, const float* S_vals, const float* precond, const void* b, void* x, int dtype,
               double tol, int maxiter, int64_t barrier_spin_limit, int flags, void* work, int* result,
               void* stream);

/* The line search's reprojection score (the reference's reproj_score, inference/engine.py
 * :357-361, used by its step reject at :308-333): the mean of the floor(0.8 n) smallest
 * per-observation errors sqrt(x_i^2 + y_i^2), x_i = residuals[i * stride_obs],
 * y_i = residuals[i * stride_obs + stride_comp] (b3r_residuals_with_rigs writes component-
 * major rows: stride_obs 1, stride_comp n_obs).  Found by an exact radix select instead of
 * a sort.  `work`: 256-byte aligned device buffer of
 * b3r_reproj_score_work_bytes(n_obs) bytes; `score`: one device float (NaN when
 * floor(0.8 n) == 0, like the reference's empty mean). */
int64_t b3r_reproj_score_work_bytes(int64_t n_obs);
int b3r_reproj_score(const float* residuals, int64_t n_obs, int64_t stride_obs, int64_t stride_comp, void* work,
                     float* score, void* stream);

/* ===================================================================================
 * Part 4 -- dense tangent prior on the depth coefficients
 * =================================================================================== */

/* One image's dense maps (device pointers): the log-depth channels (H, W, channels with
 * `channel_stride` floats between pixels; the first C are used) and the reference pointmap
 * in camera coordinates (H, W, 3), both row-major. */
typedef struct {
    const float* log_depth;
    const float* pts3d_ref;
    int32_t H, W, channel_stride, reserved;
} b3r_dense_map;

/* The reference's _dense_tangent_prior_terms (inference/engine.py:15-158) with
 * confident_in_planar_regions (:161-179), for all images in one launch: per image, the
 * tangents of the points of the combined log-depth exp(min(sum_c z_coefs[i,c] L_c, 80)) on the
 * grid subsampled by `stride` (first sample at stride / 2) against those of the reference
 * pointmap, weighted by the planarity confidence of the reference depth.  maps: DEVICE
 * array [n_imgs]; cam_ids: device int32 [n_imgs] (infos[2]); K [n_cams,3,3]; z_coefs
 * [n_imgs, C] (device).  x0_scale: device [n_imgs] factor applied to each reference
 * pointmap (the median depth ratio the reference uses when normalize == 0), or NULL (1).
 * cells_hint: about the largest subsampled grid (H' W'), a launch-size hint only.
 * Outputs (device, double, overwritten): loss [1] = the prior's term of the objective;
 * unless g_z == H_z == NULL, g_z [n_imgs, C] and H_z [n_imgs, C, C], with channel 0 zeroed
 * when optim_Z0 == 0.  weight_tan <= 0 gives zeros, like the reference. */
int b3r_tangent_prior(const b3r_dense_map* maps, int32_t n_imgs, int32_t cells_hint, const float* K,
                      const int32_t* cam_ids, const float* z_coefs, int32_t C, const double* x0_scale,
                      int32_t stride, double weight_tan, double eps, int32_t optim_Z0, int32_t normalize,
                      double* loss, double* g_z, double* H_z, void* stream);

/* Adds the prior's Gauss-Newton terms to an assembled system between b3r_lin_assemble and
 * b3r_lin_finalize, as solve_delta adds z_prior (inference/ba_solver.py:141-173): H_z [n_imgs,
 * C, C] to each image's depth-coefficient diagonal block of S and its diagonal to diag(A),
 * g_z [n_imgs, C] to b (device, double).  An image whose depth coefficients are switched off
 * (optim_Z = False) then carries the prior alone, adaptively damped like the reference's
 * BlockDiagMat(H_z).  On a sharded problem call it on the solving rank only, after the
 * reduce. */
int b3r_lin_add_zprior(b3r_plan* plan, const double* H_z, const double* g_z, void* workspace,
                       const b3r_outputs* out, void* stream);

/* One pass of b3r_lin_points/b3r_lin_assemble on its own (profiling and custom
 * pipelines): B3R_PASS_PREP (per-image records), _POINTS (per-track Hpp, g_p), _FACTOR
 * (damped per-track Cholesky factors), _DIAG (elimination records and per-image diagonal
 * blocks, b, diag(A)), _PAIRS (off-diagonal pair products, which read the records _DIAG
 * writes).  Outputs are NOT zeroed here; the caller keeps the order prep, points, factor,
 * diag, pairs on zeroed S_vals / b / diagA.  B3R_PASS_ELIMINATE is the former name of
 * B3R_PASS_FACTOR (same value). */
#define B3R_PASS_PREP 0
#define B3R_PASS_POINTS 1
#define B3R_PASS_FACTOR 2
#define B3R_PASS_ELIMINATE B3R_PASS_FACTOR
#define B3R_PASS_DIAG 3
#define B3R_PASS_PAIRS 4
int b3r_lin_pass(b3r_plan* plan, const b3r_params* params, const b3r_lin_opts* opts, void* workspace,
                 const b3r_outputs* out, int pass, void* stream);

/* y = S x with S given by its upper block triangle (symmetric). x, y: [n_cam_params]. */
int b3r_schur_spmv(const b3r_plan* plan, const float* S_vals, const float* x, float* y,
                   void* stream);
/* Same in double precision (S values promoted on load). */
int b3r_schur_spmv_f64(const b3r_plan* plan, const float* S_vals, const double* x, double* y,
                       void* stream);

/* Point back-substitution delta_p = Hpp^-1 (g_p - Hpc delta_c) for this rank's tracks
 * (ba_solver.py:203).  Must follow a linearization of the same plan with the same
 * params/opts/workspace (it reuses the per-image records and the point damping kept in
 * the workspace); each track's point block is re-accumulated and solved in double.
 * delta_c: [n_cam_params]; delta_p: [n_points*3], only this rank's tracks written. */
int b3r_backsub(b3r_plan* plan, const b3r_params* params, const b3r_lin_opts* opts, void* workspace,
                const float* delta_c, float* delta_p, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* B3R_H */
