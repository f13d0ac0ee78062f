// plan.h — device view of the symbolic structure and the host schedule built from it.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

namespace pp {

// largest residual of a front in the register-resident warp sweep of the bottom of the tree
constexpr int SWEEP_NNW = 16;
// and its largest nn + na: the fronts of the bottom of the tree's factorization for every element type (whose
// frontal matrix fits 32 KB of shared memory: 64 x 64 Float64), so that a solve sweeps all of the bottom of
// the tree while the top is still being factored
constexpr int SWEEP_NJW = 64;
// rows (residual range + root separator) of a subtree solved in shared memory, and the factor values (its
// fronts' D and O blocks) and separator slots its CTA stages there; the fronts of a subtree are at most its rows
constexpr int SUBTREE_ROWS = 64;
constexpr int SUBTREE_FAC = 640;
constexpr int SUBTREE_SLOTS = 640;
// solves with at least this many right-hand sides take two columns per lane in the subtree and bottom sweeps
constexpr int SWEEP_WIDE_K = 1024;
// threads of a CTA of the bottom factorization (a CTA per front)
constexpr int FB_THREADS = 256;
// tile edge of the persistent factorization of the top of the tree
constexpr int TOP_TILE = 64;
// rows of a block task of the top sweeps
constexpr int TOP_SWEEP_ROWS = 64;

// ints of the sweeps' scratch for k right-hand sides (tiles of 32 columns): the task counter (16 ints), then per
// (tile, front) a counter or flag, the top sweep's residual blocks done and its separator blocks done
inline int64_t sync_ints(int64_t nf, int64_t k) { return 3 * ((k + 31) / 32) * nf + 16; }

// Device arrays of a structure (0-based, positions = permuted labels).  Per front f: the residual is
// rlo[f] .. rlo[f]+nn[f]-1, the separator stgt[sptr[f] .. sptr[f+1]-1] with rel[] its positions in the
// parent's bag, the blocks of the factor arrays start at dptr[f] (nn x nn) and lptr[f] (nn x na / na x nn),
// and the front's update matrix lives in the workspace at mptr[f] with leading dimension mld[f].
struct DevPlan {
    int n, nf, nB;
    const int *rlo, *nn, *na;
    const int64_t *sptr;
    const int *stgt, *rel;
    const int64_t *dptr, *lptr;
    const int *chdptr, *chdtgt;
    const int64_t *mptr;
    const int *mld;
    const int64_t *fws;  // frontal matrix of a top front (elements), -1 for the bottom fronts
    const int64_t *nptr;
    const int *ntgt;
    const int *perm, *invp, *idx, *bptr, *fcc;
    const int *pnt;  // parent front, -1 for a root
};

// subtree tasks of one stage: roots[off .. off+count)
struct SubtreeList {
    int64_t off = 0;
    int count = 0;
};

// Algorithmic traffic (element count) and (x)(+) pairs of a set of fronts' factorization (profiler).
struct Cost {
    double bytes = 0, pairs = 0;
};

// One tree level of a solve stage: fronts d_sfronts[off .. off+count), with the per-right-hand-side sums the
// profiler needs (residual rows, separator rows, factor-block elements, (x)(+) pairs).
struct SLevel {
    int64_t off = 0;
    int count = 0;
    double res_rows = 0, sep_rows = 0, blk_elems = 0, pairs_col = 0;
};

// Solve schedule of one stage: components whose coupling predecessors (rmul) or successors (lmul) are all
// in earlier stages.
struct Stage {
    int64_t voff = 0;                             // offset into the device vertex list of the stage
    int nverts = 0;
    bool coupled = false;                          // any coupling entries touch the stage
};

}  // namespace pp
