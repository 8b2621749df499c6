/*
 * warpgbm_b200.h -- C ABI of the B200-native WarpGBM tree-growing hot path.
 *
 * Library: warpgbm_b200/libwgb_b200.so (sm_100a).  All entry points are
 * asynchronous on the CUDA stream they are given (cudaStream_t passed as
 * void*; NULL = legacy default stream), take plain device pointers and
 * sizes, and return 0 on success or a non-zero wgb status; wgb_last_error()
 * returns the message of the last failure on the calling thread.
 *
 * Two groups of entry points:
 *
 * 1. Drop-in replacements for the reference's PyTorch extension
 *    warpgbm.cuda.node_kernel (warpgbm/cuda/node_kernel.cpp:41-46).  Same
 *    argument meaning and in-place semantics; they raise (return non-zero)
 *    on bad sizes where the reference only printf's a launch error.
 *
 * 2. The level-wise tree engine that warpgbm_b200.core.WarpGBM drives: one
 *    fused histogram build per tree level over all of that level's nodes,
 *    one split search per level, an on-device partition, and no host
 *    synchronisation inside a tree.  It replaces the depth-first recursion
 *    of warpgbm/core.py:543-658 and 692-744.
 */
#ifndef WARPGBM_B200_H
#define WARPGBM_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------------- */
/* status                                                                  */
/* ---------------------------------------------------------------------- */
#define WGB_OK 0
#define WGB_ERR_ARG 1      /* invalid argument (size, pointer, range) */
#define WGB_ERR_CUDA 2     /* a CUDA runtime call or kernel launch failed */
#define WGB_ERR_ALLOC 3    /* device scratch allocation failed */

const char *wgb_last_error(void);
int wgb_version(void);
/* sizeof(wgb_node), sizeof(wgb_ws): lets bindings check their struct layout */
int32_t wgb_sizeof_node(void);
int32_t wgb_sizeof_ws(void);

/* ---------------------------------------------------------------------- */
/* 1. reference-compatible operations                                       */
/* ---------------------------------------------------------------------- */

/* Replaces node_kernel.compute_histogram3 = launch_histogram_kernel_cuda_
 * configurable (warpgbm/cuda/histogram_kernel.cu:63-104,
 * node_kernel.cpp:16-26,42).  For every sample s in sample_indices[0..n) and
 * feature position j < k with b = bin_indices[s*F_master +
 * feature_indices[j]] in [0, num_bins):
 *     grad_hist[era[s]][j][b] += residuals[s];  hess_hist[...] += 1.
 * Accumulates into the caller's [num_eras][k][num_bins] fp32 buffers like
 * the reference.  The sums are formed exactly (int64 fixed point on a
 * power-of-two grid chosen from max|residual|), so the result is
 * deterministic.  threads_per_block / rows_per_thread are validated
 * (multiple of 32; 1..16) and otherwise ignored.  feature_indices must not
 * repeat a feature.  Allocates its int64 scratch from the stream-ordered
 * pool of the current device. */
int wgb_compute_histogram3(const int8_t *bin_indices, int64_t num_rows,
                           int64_t F_master, const float *residuals,
                           const int32_t *sample_indices, int64_t n,
                           const int32_t *feature_indices, int32_t k,
                           const int32_t *era_indices, float *grad_hist,
                           float *hess_hist, int32_t num_eras,
                           int32_t num_bins, int32_t threads_per_block,
                           int32_t rows_per_thread, void *stream);

/* wgb_compute_histogram3 for callers that may not allocate device memory.
 * No counterpart in the reference: it exists for hosts that give this
 * library a fixed memory budget, or run it where an allocation must not
 * happen (an allocator call can stall or fail there), and so cannot let
 * wgb_compute_histogram3 take its scratch from the stream-ordered pool.
 * Same arguments and result as wgb_compute_histogram3; its scratch is a
 * fixed 64 MiB block inside the library (reserved on every GPU where the
 * library's kernels are loaded, until the process exits).  A call needs
 * num_eras*k*(num_bins+1)*16 + F_master*4 + ceil(n/2048)*16 + 96 bytes (each
 * part rounded up to 256); larger calls return WGB_ERR_ARG.  Calls share the
 * block, so calls that may overlap on the GPU race; calls on one stream are
 * safe.  The first call on a device looks up the block's address and should
 * come before any stream capture. */
int wgb_compute_histogram3_noalloc(const int8_t *bin_indices, int64_t num_rows,
                                   int64_t F_master, const float *residuals,
                                   const int32_t *sample_indices, int64_t n,
                                   const int32_t *feature_indices, int32_t k,
                                   const int32_t *era_indices,
                                   float *grad_hist, float *hess_hist,
                                   int32_t num_eras, int32_t num_bins,
                                   int32_t threads_per_block,
                                   int32_t rows_per_thread, void *stream);

/* Replaces node_kernel.compute_split = launch_directional_split_kernel
 * (warpgbm/cuda/best_split_kernel.cu:57-88, node_kernel.cpp:6-14,43).
 * Per (era, feature): totals over all B bins, prefix over b < B-1;
 * gain = GL^2/(HL+eps) + GR^2/(HR+eps) - GT^2/(HT+eps) and
 * dir = (GL/(HL+eps) > GR/(HR+eps)) ? 1 : -1 where HL, HR >= min_child_samples,
 * else 0 / 0 -- with one IEEE rounding per operation, bit-identical to the
 * reference kernel.  Outputs [E][k][B-1].  min_split_gain is unused, as in the
 * reference. */
int wgb_compute_split(const float *G, const float *H, int32_t num_eras,
                      int32_t k, int32_t num_bins, float min_split_gain,
                      float min_child_samples, float eps, float *per_era_gain,
                      float *per_era_direction, int32_t threads, void *stream);

/* Replaces node_kernel.custom_cuda_binner = launch_bin_column_kernel
 * (warpgbm/cuda/binner.cu:29-52, node_kernel.cpp:28-31,44):
 * out[i] = number of leading edges with X[i] >= edge (NaN -> 0). */
int wgb_custom_cuda_binner(const float *X, int64_t n, const float *bin_edges,
                           int32_t num_edges, int8_t *bin_indices,
                           void *stream);

/* Replaces node_kernel.predict_forest = predict_with_forest
 * (warpgbm/cuda/predict.cu:48-76, node_kernel.cpp:33-38,45).  tree_tensor is
 * the flattened forest of warpgbm/core.py:1215-1252, [T][max_nodes][6] =
 * (feature, split_bin, left_id, right_id, is_leaf, leaf_value).
 * out[i] += learning_rate * leaf_t(i) for every tree t, summed in tree order
 * (deterministic; the reference's atomics use any order). */
int wgb_predict_forest(const int8_t *bin_indices, int64_t n, int64_t F,
                       const float *tree_tensor, int32_t T, int32_t max_nodes,
                       float learning_rate, float *out, void *stream);

/* ---------------------------------------------------------------------- */
/* 2. level-wise engine                                                    */
/* ---------------------------------------------------------------------- */

/* Pre-binned int8 input in one pass (replaces the per-column copy of
 * warpgbm/core.py:499-517): out [n][out_stride] = X (padding bytes 0),
 * colmax[f] = max over rows of X[:, f] (the reference's pre-binned test is
 * all(colmax < num_bins)), minmax[0] / minmax[1] = global min / max (bins
 * outside [0, num_bins) take the checked histogram path).  With n == 0,
 * colmax and minmax hold sentinels below / above every int8. */
int wgb_prebinned_ingest(const int8_t *X, int64_t n, int32_t F, int64_t x_stride,
                         int8_t *out, int64_t out_stride, int32_t *colmax,
                         int32_t *minmax, void *stream);

/* Binning of a row-major float32 matrix in one pass (replaces the per-column
 * loop of warpgbm/core.py:527-538 and core.py:902-915).  X is [n][F] with
 * row stride x_stride (elements); edges [F][num_bins-1]; out is int8
 * [n][out_stride] (out_stride >= F; padding bytes are written as 0).
 * Semantics of binner.cu:16-25 per element. */
int wgb_bin_matrix(const float *X, int64_t n, int32_t F, int64_t x_stride,
                   const float *edges, int32_t num_bins, int8_t *out,
                   int64_t out_stride, void *stream);

/* Quantile edges of every column of a row-major float32 matrix X [n][F]
 * (row stride x_stride elements): edges[f][j] = torch.quantile(X[:, f],
 * q[j]) with linear interpolation, bit for bit (q = linspace(0, 1, B+1)[1:-1]
 * as the reference builds it, warpgbm/core.py:529-534; any NaN in a column
 * makes its edges NaN).  Radix selection of the 2*nq order statistics, no
 * sort.  XT is caller scratch of F*ld floats, ld = n rounded up to a
 * multiple of 4 (the column-major copy), 16-byte aligned.
 * n <= 2^24 (torch's limit). */
int wgb_quantile_edges(const float *X, int64_t n, int32_t F, int64_t x_stride,
                       const float *q, int32_t nq, float *XT, float *edges,
                       void *stream);

/* The same edges for a column whose rows are spread over several ranks
 * (row-sharded fits; replaces the per-column torch.quantile of
 * warpgbm/core.py:529-534 over the full column): the radix selection one
 * digit pass at a time, pass = 0..3, nq <= 32.  wgb_quantile_pass
 * histograms the digit of this rank's n rows of the F columns of X (pass 0
 * first copies them column-major into XT, which later passes read: keep it)
 * into hist -- pass 0: [F][4096] words and nan_flags[F]; passes 1-3:
 * [F][16384] words -- from the digits resolved so far in state
 * ([F][129] words).  The caller sums hist (and, pass 0, nan_flags) over
 * the ranks as int32, then wgb_quantile_pick resolves the digit of every
 * target from the sums with the ranks' total row count n_total (<= 2^24,
 * torch's limit) into state; after pass 3 it writes edges[F][nq], bit for
 * bit torch.quantile over the concatenated column (NaN edges for a column
 * with any NaN, written at pass 0).  No row moves between ranks. */
int wgb_quantile_pass(int32_t pass, const float *X, int64_t n, int32_t F,
                      int64_t x_stride, int32_t nq, float *XT,
                      const uint32_t *state, uint32_t *hist, int32_t *nan_flags,
                      void *stream);
int wgb_quantile_pick(int32_t pass, const uint32_t *hist,
                      const int32_t *nan_flags, int64_t n_total, const float *q,
                      int32_t nq, int32_t F, uint32_t *state, float *edges,
                      void *stream);

/* One node of one tree level (64 bytes).  Global quantities (summed over all
 * ranks of a row-sharded job) and local ones (this rank's rows). */
typedef struct wgb_node {
    int64_t sumq;    /* global sum of quantised residuals of the node       */
    int64_t count;   /* global row count                                    */
    int64_t lsumq;   /* left-child sum (valid when fpos >= 0)               */
    int64_t lcount;  /* left-child count                                    */
    int32_t lstart;  /* local rows: positions [lstart, lstart+lcnt) of the  */
    int32_t lcnt;    /*   level's row order                                 */
    int32_t slot;    /* histogram slot                                      */
    int32_t built;   /* bit 0: histogram built from rows (else parent -     */
                     /*   sibling); bits 8..: the node's tree in the batch  */
    int32_t fpos;    /* chosen split: position in the tree's feature subset,
                        -1 = leaf                                           */
    int32_t bin;     /* chosen threshold bin (go left iff bin <= this)      */
    int32_t child;   /* index of the left child at the next level (-1)      */
    float leaf;      /* leaf value (mean residual) of the node              */
} wgb_node;

/* Device workspace of one fit on one rank.  The host allocates every buffer
 * and fills the pointers; sizes in comments.  N = local rows, S = bins row
 * stride, F = features, k = features per tree, E = eras, B = num_bins,
 * D = max_depth, K = output columns (1, or classes), T = ntree = trees grown
 * together (1; or K for a multiclass round: tree t updates output column
 * cls + t).  Per-level node arrays are packed: level d occupies
 * nodes[T((1<<d)-1) .. T((1<<(d+1))-1) - 1]; tree t's root is node t of
 * level 0, and its rows are the level-0 positions [tN, (t+1)N). */
typedef struct wgb_ws {
    /* data (fixed for the fit) */
    const int8_t *bins;      /* [N][S]                                       */
    const int8_t *bins_fm;   /* [F][NT] feature-major copy, NT = N rounded up */
                             /*   to 16 (wgb_bins_feature_major), or NULL     */
    const int32_t *era;      /* [N] dense era id per row, or NULL if E == 1   */
    const int32_t *root_order; /* [T][N] row ids sorted by era (stable), the  */
                             /*   same order repeated for every tree         */
    const float *y;          /* [N] regression target (NULL: g given)        */
    float *pred;             /* [N][K] running prediction                    */
    float *g;                /* [T][N] residual of the current trees         */
    int32_t *qg;             /* [T][N] quantised residual                     */
    /* per tree */
    const int32_t *feats;    /* [k] physical feature of each position         */
    int32_t *kpos;           /* [F] position of each physical feature or -1   */
    int8_t *bins_sub;        /* [N][S_sub] the tree's k features in position  */
                             /*   order (wgb_tree_subset), or NULL: the       */
                             /*   histograms then read `bins` through kpos    */
    int32_t *kpos_sub;       /* [S_sub] j for j < k, -1 past k                 */
    int64_t S_sub;           /* row stride of bins_sub (k rounded up to 32)   */
    /* row order per level (ping-pong) */
    int32_t *order[2];       /* [T*N]                                         */
    int32_t *posnode[2];     /* [T*N] node index (within level) per position  */
    uint8_t *flags;          /* [T*N + 16]                                    */
    int32_t *tile_cnt;       /* [ntiles]                                      */
    int32_t *tile_off;       /* [ntiles]                                      */
    int32_t *part;           /* [T 2^D][4] per-node partition scratch         */
    /* histograms */
    int64_t *hg;             /* histogram pool, T 2^(D-1) slots of         */
                             /*   2*E*k*(B+1) + 2 int64: [E][k][B+1] sums of */
                             /*   q, [E][k][B+1] counts, root sum, spare     */
    /* chunk work list of the histogram build */
    int32_t *chunks;         /* [chunk_cap][4] = node, p0, p1, -              */
    int32_t *nchunks;        /* [1]                                           */
    /* split search */
    int32_t *cand;           /* [T 2^(D-1)][ncand_blk][4] partial arg-max:   */
                             /*   ncand_blk >= ceil(k/8) with one era;       */
                             /*   with eras >= ceil(k/32) (num_bins <= 33)   */
                             /*   or ceil(k/8) (num_bins > 33)               */
    float *era_gain;         /* [T (2^D - 1)][E] per-era gain of chosen split */
    /* nodes and level sizes */
    wgb_node *nodes;         /* [T (2^(D+1) - 1)]                             */
    int32_t *nn;             /* [D+1] nodes per level (all trees)             */
    int32_t *nact;           /* [D+1] local positions per level (all trees)   */
    /* scalars of the current trees */
    float *maxabs;           /* [T] max |g| (bit pattern compared as int)     */
    int32_t *shift;          /* [T] s                                         */
    int64_t *rootsum;        /* [T] sum of q over local rows                  */
    int32_t *sync;           /* [4] zero-initialised counters of the fused    */
                             /*   per-level kernels (left at zero by them)    */
    void *part_hist;         /* per-chunk histogram words (8 bytes each), or  */
    int64_t part_hist_elems; /*   NULL: wgb_hist_part_elems(S, F, B, chunk_cap) */
                             /*   lets single-era levels skip global atomics  */
    /* era criterion (E > 1): the plan of wgb_era_mean_plan(E, k*(B-1), ...) */
    const int32_t *era_sched; /* [E] eras in the order the criterion adds them */
    const uint8_t *era_ops;  /* [era_nops] accumulator program                */
    float *crit_out;         /* optional [k][B-1]: criterion of node 0 of each */
                             /*   level (inspection), or NULL                  */
    /* feature-sliced multi-rank fits (nslice > 1): rank `slice` keeps the
     * histograms of positions [slice*ks, slice*ks + ks) only -- hg is then a
     * pool of slots laid out as above with ks in place of k -- and searches
     * splits among them; see wgb_level_hist / wgb_level_split / wgb_level_pick */
    int64_t *hstage;         /* [nslice][built slots of a level][slot_elems]: */
                             /*   the level's local histograms, slice-major,  */
                             /*   reduce-scattered over the ranks into hg     */
    int64_t hstage_elems;    /* capacity of hstage                            */
    int32_t *win;            /* [nslice][T 2^(D-1)][win_words]: every rank's  */
                             /*   best split per node of the level (all-gathered) */
    /* sizes */
    int64_t N, S;
    int64_t N_global;
    int32_t F, k, E, B, D, K;
    int32_t cls;             /* output column updated by tree 0 of the batch  */
    int32_t chunk_cap, ntiles, ncand_blk;
    int32_t hist_ew;         /* max eras per shared-memory window (0 = auto)  */
    int32_t regular;         /* 1 if every bin is known to lie in [0, B)      */
    int32_t era_nops, era_depth; /* program length and stack depth of the plan */
    int32_t ntree;           /* T, trees grown together (0 is taken as 1)     */
    int32_t nslice, slice;   /* ranks sharing the features (0 or 1: none), this rank */
    int32_t ks;              /* positions per slice (ceil(k / nslice))         */
    int32_t win_words;       /* 32-bit words per node record in win: 8 + E    */
                             /*   rounded up to even (int64 fields aligned)   */
    /* hyper-parameters (fp32 as the reference passes them) */
    float mcw, eps, msg, lr, mean_factor;
} wgb_ws;

/* Tree start: g = y - pred[:, cls] (if y != NULL), max|g| into *maxabs
 * (*maxabs must be 0 on entry; see wgb_tree_reset). */
int wgb_tree_residual(const wgb_ws *ws, void *stream);
/* Zero the per-tree scalars (maxabs, rootsum). */
int wgb_tree_reset(const wgb_ws *ws, void *stream);
/* Per tree, when ws->bins_sub != NULL: bins_sub[r][j] = bins[r][feats[j]]
 * for the tree's k feature positions (padding 0) and kpos_sub, so that the
 * level histograms read k bytes per row and update k features instead of
 * all F (colsample_bytree < 1, warpgbm/core.py:721-722). */
int wgb_tree_subset(const wgb_ws *ws, void *stream);
/* Quantise g (shift from *maxabs, which must already be the global max),
 * sum q over local rows into *rootsum. */
int wgb_tree_quantize(const wgb_ws *ws, void *stream);
/* Root record (its sum and leaf are set at level 0's split) and level
 * counters. */
int wgb_tree_root(const wgb_ws *ws, void *stream);
/* Level d: zero of the built slots, histogram build of the built nodes
 * from local rows (level 0 plans its chunk list here; level d > 0 uses the
 * list that wgb_level_partition(d - 1) planned).  Built slots of level d are
 * the contiguous range returned by wgb_level_slots; one int64 SUM all-reduce
 * over ranks of hg[first*P, (first+count)*P), P = 2*E*k*(B+1) + 2, covers
 * sums, counts and (level 0) the roots' sums of q, which wgb_level_hist
 * copies from rootsum[t] into the first spare cell of slot t. */
int wgb_level_hist(const wgb_ws *ws, int32_t d, void *stream);
/* Built slots of level d for one tree at a time (ntree = 1). */
void wgb_built_slots(int32_t d, int32_t *first, int32_t *count);
/* Built slots of level d of the workspace's batch of ntree trees. */
void wgb_level_slots(const wgb_ws *ws, int32_t d, int32_t *first, int32_t *count);
/* Elements (8 bytes each) of the per-chunk histogram buffer for `chunks`
 * chunks of a matrix with row stride S, F features and B bins. */
int64_t wgb_hist_part_elems(int64_t S, int32_t F, int32_t B, int64_t chunks);
/* Level d: sibling = parent - built (in place, fused into the split
 * search), split search, per-era gains, child totals, next level's node
 * records.  With eras the criterion is
 * torch's CUDA per_era_gain.mean(dim=0) (warpgbm/core.py:581-582) bit for
 * bit: the eras are added in the order of ws->era_sched / ws->era_ops. */
int wgb_level_split(const wgb_ws *ws, int32_t d, void *stream);
/* Level d of a feature-sliced fit (ws->nslice > 1), after wgb_level_split
 * wrote this rank's best split per node into its region of ws->win and the
 * regions were all-gathered: the best record per node by the split key
 * (directional agreement, criterion, position index -- the choice one rank
 * searching every position makes), its child totals and per-era gains into
 * the node, and the next level's node records.  No-op otherwise. */
int wgb_level_pick(const wgb_ws *ws, int32_t d, void *stream);

/* Plan of the order in which torch's CUDA mean(dim=0) of a contiguous fp32
 * [E][M] tensor adds its E rows (ATen's reduce kernel: rows spread over the
 * block's rows and over blocks, four accumulators per thread, fixed
 * combining trees; the launch shape depends on E, M, the SM count and the
 * threads per SM -- num_sms / max_threads_per_sm <= 0 take the current
 * device's).  Replaces the ordering of warpgbm/core.py:581-582's
 * per_era_gain.mean(dim=0) and per_era_direction.mean(dim=0) with M =
 * k*(num_bins-1).  Writes sched[E] (eras in the order they are first added)
 * and ops[] (0: push the accumulator and restart it at 0; 1: accumulator +=
 * popped value; 2: accumulator += next scheduled era); *depth = stack depth.
 * Returns the program length (write nothing with ops == NULL to size it;
 * ops_cap must hold it), or a negative status.  M == 1 (a single candidate)
 * is reduced by torch along another path; the plan is then a sequential
 * sum. */
int64_t wgb_era_mean_plan(int32_t E, int64_t M, int32_t num_sms,
                          int32_t max_threads_per_sm, int32_t *sched,
                          uint8_t *ops, int64_t ops_cap, int32_t *depth);
/* Feature-major copy of ws->bins into out ([F][NT], NT = N rounded up to a
 * multiple of 16, 16-byte aligned): the partition reads one feature of many
 * rows, which this layout makes contiguous.  Set ws->bins_fm = out after. */
int wgb_bins_feature_major(const wgb_ws *ws, int8_t *out, void *stream);
/* Level d: partition of local rows into the next level's order; rows of
 * nodes that became leaves get pred[:, cls] += lr * leaf; then the next
 * level's histogram chunk list.  At d = D - 1 every row gets its leaf
 * update (the children are the last level).  Stable (three launches) for
 * era fits; a one-era fit takes one launch that does not keep the rows'
 * relative order inside a child (nothing reads it: the histogram sums are
 * exact integers), with the layout wgb_level_split planned on one rank and
 * finished by the launch's last CTA on several. */
int wgb_level_partition(const wgb_ws *ws, int32_t d, void *stream);
/* Tree end: nothing left to launch (the last level's leaf updates happen in
 * wgb_level_partition(D - 1)); validates the workspace. */
int wgb_tree_finish(const wgb_ws *ws, void *stream);

/* The whole per-tree sequence as stream work issued from C++: reset,
 * residual (+ max |g| over ranks), quantise, root, and per level d < D the
 * histogram build, its int64 SUM over ranks (when comm != NULL), the split
 * search and the partition; then wgb_tree_finish.  A feature-sliced fit
 * (ws->nslice > 1, comm of those ranks) reduce-scatters the level's
 * histograms from ws->hstage instead of summing them everywhere, and
 * all-gathers ws->win before wgb_level_pick.  Replaces the reference's
 * per-node Python recursion (warpgbm/core.py:597-658, 692-744) and the
 * per-level Python loop of a host driving the entry points above.  comm ==
 * NULL: one rank. */
typedef struct wgb_comm wgb_comm;
int wgb_grow_tree(const wgb_ws *ws, wgb_comm *comm, void *stream);

/* Host-side decode of tree `root` of a batch of `ntree` trees in the
 * engine's level-packed node records (a copy of ws->nodes, depth D) into
 * pre-order arrays: packed[2i], packed[2i+1] = {feature, bin | right << 8}
 * for a split, {-1, float bits of the leaf} for a leaf (the
 * wgb_predict_packed format), leaf[i], samples[i] (row count of a leaf);
 * feats maps feature positions to features.  When imp != NULL the tree's
 * per-era split gains (era_gain, [ntree(2^D - 1)][E]) are added to imp
 * [E][F] in pre-order, the order of the reference's depth-first growth
 * (warpgbm/core.py:624-627); the nested-dict trees of core.py:597-658 are
 * built from these arrays.  Returns the node count (<= cap) or a negative
 * status.  Runs on the host; no device memory. */
int64_t wgb_decode_tree(const wgb_node *nodes, int32_t D, int32_t ntree,
                        int32_t root, const int32_t *feats,
                        const float *era_gain, int32_t E, float *imp,
                        int32_t F, int32_t *packed, float *leaf,
                        int64_t *samples, int64_t cap);

/* NCCL communicator of a row-sharded fit, owned by this library (NCCL's
 * entry points are resolved from the libnccl.so.2 already loaded in the
 * process).  Rank 0 makes the 128-byte id, the host distributes it, every
 * rank calls wgb_comm_init (collective).  wgb_comm_allreduce sums int64
 * (kind 0) or takes the max of float32 (kind 1) in place on `stream`. */
int wgb_comm_unique_id(uint8_t *id128);
int wgb_comm_init(int32_t rank, int32_t world, const uint8_t *id128,
                  wgb_comm **out);
int wgb_comm_destroy(wgb_comm *comm);
int wgb_comm_allreduce(wgb_comm *comm, void *buf, int64_t count, int32_t kind,
                       void *stream);
/* int64 SUM of every rank's send[world][recvcount]; rank r receives the sum
 * of block r (ncclReduceScatter) on `stream`. */
int wgb_comm_reduce_scatter(wgb_comm *comm, const int64_t *send, int64_t *recv,
                            int64_t recvcount, void *stream);
/* In place: every rank's buf[rank*count .. +count) to all ranks
 * (ncclAllGather of int32) on `stream`. */
int wgb_comm_allgather_i32(wgb_comm *comm, int32_t *buf, int64_t count,
                           void *stream);

/* Host -> device copy of `bytes` from pageable host memory, pipelined
 * through pinned staging buffers (parallel host copies overlapped with the
 * DMA, one cudaMemcpyAsync per 64 MiB chunk).  Returns once the source has
 * been read; the device copies complete in stream order.  Ingest path of
 * warpgbm/core.py:487-538 (the reference copies column by column). */
int wgb_h2d(void *dst, const void *src, int64_t bytes, void *stream);

/* Forest prediction with trees packed by warpgbm_b200 (pre-order, 8 bytes per
 * node: internal = {feature, bin | right_id << 8}, leaf = {-1, value bits}).
 * out[i*K + class_of_tree(t)] += lr * leaf_t(i), trees in order t = 0..T-1,
 * class_of_tree(t) = t % K.  tree_off[t] = first node of tree t. */
int wgb_predict_packed(const int8_t *bins, int64_t n, int64_t S,
                       const int32_t *nodes, const int32_t *tree_off,
                       int32_t T, int32_t K, float lr, float *out,
                       void *stream);

/* Forest prediction with trees of depth D <= 12 laid out as complete binary
 * trees (the fast path of warpgbm/cuda/predict.cu:5-45's traversal).  Tree t
 * is 2^(D+1) uint32 words at heap + t*2^(D+1) (heap 16-byte aligned): word i
 * < 2^D - 1 is heap slot i (children 2i+1, 2i+2) = (feature & 0xFFFF) |
 * (uint8 split bin << 16), a row going left iff its int8 bin <= the split
 * bin; the value of the leaf reached at depth-D slot h is word h + 1.  A
 * leaf at depth d < D is a chain of pass-through slots (feature 0, bin 127)
 * to its leftmost depth-D descendant, which holds its value.
 * out[i*K + t%K] += lr * leaf_t(i), trees in order t = 0..T-1 (fp32, the
 * same sums as wgb_predict_packed).  Rows are staged in shared memory when
 * at least 64 of them fit, else read from global memory (any width). */
int wgb_predict_heap(const int8_t *bins, int64_t n, int64_t S,
                     const uint32_t *heap, int32_t T, int32_t K, int32_t D,
                     float lr, float *out, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* WARPGBM_B200_H */
