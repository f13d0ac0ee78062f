// ops.h — the per-(semiring, element type) operation table the C ABI dispatches to.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "plan.h"

namespace pp {

// Kernel classes the profiler separates.
enum KClass { K_FACTOR_TOP = 0, K_SWEEP_FWD, K_SWEEP_BWD, K_COUPLING, K_PERMUTE, K_ASSEMBLE, K_FRONT_BOTTOM,
              K_SWEEP_FWD_BOTTOM, K_SWEEP_BWD_BOTTOM, K_SWEEP_FWD_SUBTREE, K_SWEEP_BWD_SUBTREE, K_NCLASS };
extern const char *const KCLASS_NAMES[K_NCLASS];

// Optional per-launch timing with CUDA events on the launching stream; off unless pp_set_profile enabled it.
struct Profiler {
    bool on = false;
    size_t esize = 0;
    struct Rec {
        int cls;
        cudaEvent_t a, b;
        double bytes, pairs;
    };
    std::vector<Rec> recs;
    std::vector<cudaEvent_t> pool;
    int64_t launches[K_NCLASS] = {};
    double ms[K_NCLASS] = {}, bytes[K_NCLASS] = {}, pairs[K_NCLASS] = {};
    int begin(int cls, cudaStream_t st) {
        if (!on) return -1;
        Rec r{cls, take(), take(), 0, 0};
        cudaEventRecord(r.a, st);
        recs.push_back(r);
        return (int)recs.size() - 1;
    }
    void end(int i, cudaStream_t st, double elems, double prs) {
        if (i < 0) return;
        recs[i].bytes = elems * (double)esize;
        recs[i].pairs = prs;
        cudaEventRecord(recs[i].b, st);
    }
    cudaEvent_t take() {
        if (pool.empty()) {
            cudaEvent_t e;
            cudaEventCreate(&e);
            return e;
        }
        cudaEvent_t e = pool.back();
        pool.pop_back();
        return e;
    }
    // after the stream is synchronised: add the recorded launches to the per-class totals
    void collect() {
        for (Rec &r : recs) {
            float t = 0;
            cudaEventElapsedTime(&t, r.a, r.b);
            launches[r.cls]++;
            ms[r.cls] += t;
            bytes[r.cls] += r.bytes;
            pairs[r.cls] += r.pairs;
            pool.push_back(r.a);
            pool.push_back(r.b);
        }
        recs.clear();
    }
    void reset() {
        collect();
        for (int c = 0; c < K_NCLASS; c++) {
            launches[c] = 0;
            ms[c] = bytes[c] = pairs[c] = 0;
        }
    }
    ~Profiler() {
        for (Rec &r : recs) {
            cudaEventDestroy(r.a);
            cudaEventDestroy(r.b);
        }
        for (cudaEvent_t e : pool) cudaEventDestroy(e);
    }
};

// Host copy of the schedule and of the per-front sizes the drivers need, plus the device lists.
struct HostPlan {
    int n = 0, nf = 0, nB = 0;
    std::vector<int> nn, na, chdptr, chdtgt;
    std::vector<int64_t> sptr, dptr, lptr;
    // workspace layout for the current element size
    size_t esize = 0;
    std::vector<int64_t> mptr, fws;
    std::vector<int> mld;
    int64_t ws_elems = 0;
    // top of the tree: the tile tasks of the persistent factorization (top.cuh), fronts by height; the first
    // top_ntasks_a tasks are every front but the roots of the tree, the rest the roots' (two launches, so that a
    // solve can sweep the lower fronts forward while the roots are factored)
    int top_ntasks = 0, top_ntasks_a = 0;
    const int4 *d_ttasks = nullptr;   // (front, I, J, 0): tile (I, J) of the front
    const int64_t *d_tfoff = nullptr;  // per front: first of its flags in d_tflags
    const int64_t *d_croff = nullptr;  // per child edge (index into chdtgt): first of its ranges in d_crng
    const int *d_crng = nullptr;       // per child edge: the parent's tile-block boundaries in the child's rel[]
    int *d_tflags = nullptr;           // [0] task counter, [1] error word, then the fronts' flags
    int64_t tflags_n = 0;
    // per-task timeline of the top factorization (pp_options.trace): TRACE_WORDS per task, or null
    unsigned long long *d_trace = nullptr;
    Cost top_cost;
    int64_t nN = 0;
    // solve schedules (lmul: components after their coupling successors; rmul: after their predecessors)
    std::vector<Stage> lstages, rstages;
    const int *d_sfronts = nullptr;   // fronts of every stage's levels (both schedules)
    const int2 *d_tentries = nullptr;  // (front, block) entries of the top sweeps' work lists
    const int *d_sverts = nullptr;    // vertices of every stage (both schedules)
    const int *d_rel = nullptr;
    DevPlan dev{};
    Profiler *prof = nullptr;
    // bottom of the tree for the persistent kernels: factorization (fronts with nn + na <= the bottom limit
    // whose whole subtree is such) and solves (nn <= SWEEP_NNW, nn + na <= SWEEP_NJW, whole subtree)
    int fb_count = 0, fb_maxnj = 0;
    double fb_bytes = 0, fb_pairs = 0;
    const int *d_fbottom = nullptr;    // work list, height ascending
    const int *d_fpending0 = nullptr;  // children per front (counter template)
    // per stage: bottom work lists of the solves in d_sfronts (forward ascending, backward descending)
    std::vector<std::pair<int64_t, int>> sb_fwd, sb_bwd;  // indexed like lstages / rstages: [stage] -> (off, count)
    std::vector<std::pair<int64_t, int>> sb_fwd_r, sb_bwd_r;
    std::vector<SLevel> sb_cost_l, sb_cost_r;  // per stage: sums over the bottom fronts (profiler)
    const int *d_spending0 = nullptr;  // bottom children per front (forward counters)
    // subtrees solved in shared memory (per stage), their roots, first descendants and separator slots
    std::vector<SubtreeList> sub_l, sub_r;
    // profiler sums of a subtree, by root front: (x)(+) pairs per column, rows per column (residual range and
    // root separator), factor elements; sroot_cost holds them in the order of the device root list
    std::vector<double> stree_pairs, stree_res, stree_sep, stree_fac;
    std::vector<double> sroot_pairs, sroot_res, sroot_sep, sroot_fac;
    const int *d_sroots = nullptr, *d_fdsc = nullptr, *d_slot = nullptr;
    int bot_fmax = 0, bot_namax = 0;   // largest nn * nn + nn * na and na of the other bottom fronts
    const int *d_sdone0 = nullptr;     // 1 for fronts outside the bottom, 0 inside (backward flags)
    // continuation of the bottom sweeps: per direction (lmul!, rmul!) each bottom front's segment and children
    // parts (sweep_bottom_kernel's sinfo), and the heavy child of each bottom front
    const int *d_sinfo[2] = {nullptr, nullptr};
    const int *d_sheavy = nullptr;
    // the top fronts of each stage for the persistent top sweep (forward ascending, backward descending heights)
    std::vector<std::pair<int64_t, int>> st_fwd, st_bwd, st_fwd_r, st_bwd_r;
    // per stage: the forward lists' entries of fronts other than roots (listed first; the roots' entries follow)
    std::vector<int> st_fwd_a, st_fwd_r_a;
    std::vector<SLevel> st_cost_l, st_cost_r;
    const int *d_tpending0 = nullptr;  // top children per front (forward counters of the top sweep)
    int *d_sync = nullptr;             // scratch: [0] task counter, [16, 16 + nf * tiles) counters
    int *d_err = nullptr;              // set by a persistent kernel whose bounded wait expired
    // The top of the tree is factored on top_stream, after ev_bottom (recorded on the calling stream behind the
    // bottom kernel); ev_factored marks its end.  A solve enqueued behind the factorization runs the first
    // early_sub[d] subtrees and early_bot[d] forward bottom fronts of its stage 0 (d = 0 lmul!, 1 rmul!; all of
    // them factored by the bottom kernel, listed first) before it waits for ev_factored.
    // ev_top_a marks the end of the first launch of the top factorization (every front but the roots).
    cudaStream_t top_stream = nullptr;
    cudaEvent_t ev_bottom = nullptr, ev_factored = nullptr, ev_top_a = nullptr;
    int early_sub[2] = {0, 0}, early_bot[2] = {0, 0};
    int64_t sync_cap = 0;              // ints allocated at d_sync
    int sm_count = 148;
    // algorithmic cost per front of the caller's (unpadded) structure, summed over the members of a merged
    // front (empty: the plan's fronts are the caller's): factorization (x)(+) pairs and elements moved, and the
    // (x)(+) pairs of one right-hand side through L* (or U*)
    std::vector<double> ufac_pairs, ufac_elems, usolve_pairs;
    // several GPUs (pp_comm_init): each rank's bottom kernel factors its own part of the bottom of the tree
    // (d_fbottom holds that part), then `exchange` runs on the calling stream and gives every rank the other
    // parts, before the top of the tree is factored on every rank
    cudaError_t (*exchange)(void *ctx, cudaStream_t st) = nullptr;
    void *exchange_ctx = nullptr;
};

struct Values {
    void *LD = nullptr, *LL = nullptr, *UD = nullptr, *UL = nullptr, *Nval = nullptr, *W = nullptr;
};

struct Ops {
    int sr, dt;
    size_t esize;
    int small_limit;  // largest block of pp_getrf_batched (shared memory)
    cudaError_t (*fill_zero)(void *p, int64_t n, cudaStream_t st);
    cudaError_t (*assemble)(const HostPlan &hp, const int *colptr, const int *rowval, const void *nzval,
                            const Values &v, cudaStream_t st);
    cudaError_t (*factor)(const HostPlan &hp, const Values &v, cudaStream_t st, int64_t *launches);
    cudaError_t (*solve)(const HostPlan &hp, const Values &v, int left, void *X, int64_t ldx, int k, cudaStream_t st,
                         int64_t *launches);
    cudaError_t (*unit_sources)(void *X, int64_t ldx, const int *invp, int64_t col0, int k, cudaStream_t st);
    cudaError_t (*rows_in)(const void *B, int64_t ldb, void *X, int64_t ldx, const int *invp, int n, int k,
                           cudaStream_t st);
    cudaError_t (*rows_out)(void *B, int64_t ldb, const void *X, int64_t ldx, const int *invp, int n, int k,
                            cudaStream_t st);
    cudaError_t (*unit_positions)(void *X, int64_t ldx, const int *pos, int k, cudaStream_t st);
    cudaError_t (*rows_out_mapped)(void *B, int64_t ldb, const void *X, int64_t ldx, const int *invp, const int *cmap,
                                   int n, int k, cudaStream_t st);
    cudaError_t (*cols_in)(const void *B, int64_t ldb, void *X, int64_t ldx, const int *invp, int n, int k,
                           cudaStream_t st);
    cudaError_t (*cols_out)(void *B, int64_t ldb, const void *X, int64_t ldx, const int *invp, int n, int k,
                            cudaStream_t st);
    cudaError_t (*gemm)(int64_t m, int64_t n, int64_t k, void *C, int64_t ldc, const void *A, int64_t lda,
                        const void *B, int64_t ldb, cudaStream_t st);
    cudaError_t (*getrf_batched)(int n, int64_t count, void *A, cudaStream_t st);
};

const Ops *get_ops(int sr, int dt);

// shared-memory budget of the one-CTA dense LU of pp_getrf_batched
constexpr size_t SMALL_FRONT_SMEM = 160 * 1024;

}  // namespace pp
