// engine_host.cuh — host drivers of the device kernels, templated on the semiring; instantiated once per
// (semiring, element type) in ops_*.cu.
//
// Factorization: one persistent launch for the bottom of the tree (factor_bottom_kernel), then one for the
// rest (factor_top_kernel, tile tasks) on a second stream, so that a solve enqueued behind it runs its bottom
// sweeps while the top of the tree is being factored.  Solves: per coupling stage and direction, one persistent
// launch each for the subtrees that fit shared memory, the other bottom fronts and the top fronts
// (sweep_top_kernel).
#pragma once

#include <algorithm>

#include "getrf.cuh"
#include "ops.h"
#include "persist.cuh"
#include "sweep_top.cuh"
#include "sweep_wide.cuh"
#include "top.cuh"

namespace pp {

#define PP_TRY(x)                              \
    do {                                       \
        cudaError_t e__ = (x);                 \
        if (e__ != cudaSuccess) return e__;    \
    } while (0)

inline int grid_for(int64_t n, int threads, int cap = 148 * 16) {
    int64_t g = (n + threads - 1) / threads;
    if (g < 1) g = 1;
    if (g > cap) g = cap;
    return (int)g;
}

template <int SR, typename T>
struct Engine {
    using S = Sem<SR, T>;

    static cudaError_t fill_zero(void *p, int64_t n, cudaStream_t st) {
        if (n <= 0) return cudaSuccess;
        fill_zero_kernel<SR, T><<<grid_for(n, 256, 148 * 32), 256, 0, st>>>(static_cast<T *>(p), n);
        return cudaGetLastError();
    }

    static cudaError_t assemble(const HostPlan &hp, const int *colptr, const int *rowval, const void *nzval,
                                const Values &v, cudaStream_t st) {
        const int64_t nD = hp.dptr[hp.nf], nL = hp.lptr[hp.nf];
        PP_TRY(fill_zero(v.LD, nD, st));
        PP_TRY(fill_zero(v.UD, nD, st));
        PP_TRY(fill_zero(v.LL, nL, st));
        PP_TRY(fill_zero(v.UL, nL, st));
        PP_TRY(fill_zero(v.Nval, hp.nN, st));
        if (hp.n == 0) return cudaSuccess;
        const int threads = 256;
        const int64_t blocks = ((int64_t)hp.n * 32 + threads - 1) / threads;
        assemble_kernel<T><<<(unsigned)blocks, threads, 0, st>>>(
            hp.dev, colptr, rowval, static_cast<const T *>(nzval), static_cast<T *>(v.LD), static_cast<T *>(v.LL),
            static_cast<T *>(v.UD), static_cast<T *>(v.UL), static_cast<T *>(v.Nval));
        return cudaGetLastError();
    }

    static cudaError_t set_attrs() {
        int dev = 0;
        cudaGetDevice(&dev);
        static bool attr[64] = {};
        if (dev < 64 && !attr[dev]) {
            PP_TRY(cudaFuncSetAttribute(factor_top_kernel<SR, T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)factor_top_smem<T>()));
            PP_TRY(cudaFuncSetAttribute(factor_bottom_kernel<SR, T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)SMALL_FRONT_SMEM));
            attr[dev] = true;
        }
        return cudaSuccess;
    }

    // scratch layout: d_sync[0] task counter of the current launch, d_sync + 16 the per-(tile, front) counters.
    // A bounded wait that expires sets hp.d_err; the C ABI reads it at the next synchronisation.
    static cudaError_t reset_sync(const HostPlan &hp, const int *init, int ntiles, cudaStream_t st) {
        PP_TRY(cudaMemsetAsync(hp.d_sync, 0, sizeof(int), st));
        if (ntiles == 1) return cudaMemcpyAsync(hp.d_sync + 16, init, sizeof(int) * hp.nf, cudaMemcpyDeviceToDevice, st);
        init_flags_kernel<<<grid_for((int64_t)hp.nf * ntiles, 256), 256, 0, st>>>(hp.d_sync + 16, init, hp.nf, ntiles);
        return cudaGetLastError();
    }

    static cudaError_t factor(const HostPlan &hp, const Values &v, cudaStream_t st, int64_t *launches) {
        T *LD = static_cast<T *>(v.LD), *LL = static_cast<T *>(v.LL), *UD = static_cast<T *>(v.UD),
          *UL = static_cast<T *>(v.UL), *W = static_cast<T *>(v.W);
        int64_t nl = 0;
        PP_TRY(set_attrs());
        if (hp.fb_count > 0) {
            PP_TRY(reset_sync(hp, hp.d_fpending0, 1, st));
            const size_t smem = (size_t)hp.fb_maxnj * hp.fb_maxnj * sizeof(T);
            int per_sm = 1;
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, factor_bottom_kernel<SR, T>, FB_THREADS, smem);
            const int grid = std::max(1, std::min(hp.fb_count, std::max(per_sm, 1) * hp.sm_count));
            const int pi = hp.prof ? hp.prof->begin(K_FRONT_BOTTOM, st) : -1;
            factor_bottom_kernel<SR, T><<<grid, FB_THREADS, smem, st>>>(hp.d_fbottom, hp.fb_count, hp.dev, LD, LL, UD, UL, W,
                                                                 hp.d_sync + 16, hp.d_sync, hp.d_err);
            PP_TRY(cudaGetLastError());
            if (pi >= 0) hp.prof->end(pi, st, hp.fb_bytes, hp.fb_pairs);
            nl++;
        }
        if (hp.exchange) PP_TRY(hp.exchange(hp.exchange_ctx, st));  // the other ranks' parts of the bottom
        cudaStream_t ts = st;
        if (hp.top_stream && hp.ev_bottom && hp.ev_factored) {
            ts = hp.top_stream;
            PP_TRY(cudaEventRecord(hp.ev_bottom, st));
            PP_TRY(cudaStreamWaitEvent(ts, hp.ev_bottom, 0));
        }
        if (hp.top_ntasks > 0) {
            constexpr size_t smem = factor_top_smem<T>();
            PP_TRY(cudaMemsetAsync(hp.d_tflags, 0, sizeof(int) * (size_t)hp.tflags_n, ts));
            int per_sm = 1;
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, factor_top_kernel<SR, T>, 256, smem);
            // two launches when the top runs on its own stream: every front but the roots, then the roots (the
            // tile flags persist, the task counter restarts); a solve sweeps the lower fronts in between
            const bool split = ts != st && hp.ev_top_a && hp.top_ntasks_a > 0 && hp.top_ntasks_a < hp.top_ntasks;
            const int parts[2][2] = {{0, split ? hp.top_ntasks_a : hp.top_ntasks},
                                     {split ? hp.top_ntasks_a : hp.top_ntasks, hp.top_ntasks}};
            for (int q = 0; q < 2; q++) {
                const int t0 = parts[q][0], cnt = parts[q][1] - parts[q][0];
                if (cnt <= 0) continue;
                if (q == 1) PP_TRY(cudaMemsetAsync(hp.d_tflags, 0, sizeof(int), ts));  // the task counter
                const int grid = std::max(1, std::min(cnt, std::max(per_sm, 1) * hp.sm_count));
                const int pi = hp.prof ? hp.prof->begin(K_FACTOR_TOP, ts) : -1;
                factor_top_kernel<SR, T><<<grid, 256, smem, ts>>>(
                    hp.d_ttasks + t0, cnt, hp.dev, hp.d_tfoff, hp.d_croff, hp.d_crng, LD, LL, UD, UL, W, hp.d_tflags,
                    hp.d_err, hp.d_trace ? hp.d_trace + (size_t)PP_TRACE_WORDS * t0 : nullptr);
                PP_TRY(cudaGetLastError());
                if (pi >= 0) hp.prof->end(pi, ts, q == 0 ? hp.top_cost.bytes : 0, q == 0 ? hp.top_cost.pairs : 0);
                nl++;
                if (q == 0 && ts != st && hp.ev_top_a) PP_TRY(cudaEventRecord(hp.ev_top_a, ts));
            }
        } else if (ts != st && hp.ev_top_a) {
            PP_TRY(cudaEventRecord(hp.ev_top_a, ts));
        }
        if (ts != st) PP_TRY(cudaEventRecord(hp.ev_factored, ts));
        if (launches) *launches += nl;
        return cudaSuccess;
    }

    template <bool FWD, bool TRANS>
    static cudaError_t sweep_wide(const HostPlan &hp, const std::pair<int64_t, int> &wl, const SLevel &cost,
                                  const T *Dv, const T *Ov, T *X, int64_t ldx, int k, int unit, cudaStream_t st,
                                  int64_t *nl, bool reset = true) {
        constexpr size_t smem = sweep_wide_smem<T>();
        int dev = 0;
        cudaGetDevice(&dev);
        static bool attr[64] = {};
        if (dev < 64 && !attr[dev]) {
            PP_TRY(cudaFuncSetAttribute(sweep_wide_kernel<SR, T, FWD, TRANS>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            attr[dev] = true;
        }
        const int ntiles = (k + SWW_CT - 1) / SWW_CT;
        const size_t cells = (size_t)ntiles * hp.nf;  // per (tile, front)
        if (FWD && !reset) {
            PP_TRY(cudaMemsetAsync(hp.d_sync, 0, sizeof(int), st));  // the task counter only
        } else if (FWD) {
            PP_TRY(reset_sync(hp, hp.d_tpending0, ntiles, st));
            PP_TRY(cudaMemsetAsync(hp.d_sync + 16 + cells, 0, sizeof(int) * 2 * cells, st));  // blocks done
        } else {
            PP_TRY(cudaMemsetAsync(hp.d_sync, 0, sizeof(int), st));
            PP_TRY(cudaMemsetAsync(hp.d_sync + 16, 0, sizeof(int) * 2 * cells, st));  // done flags, blocks done
        }
        int per_sm = 1;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, sweep_wide_kernel<SR, T, FWD, TRANS>, 256, smem);
        const int64_t tasks = (int64_t)wl.second * ntiles;
        const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(tasks, std::max(per_sm, 1) * hp.sm_count));
        const int pi = hp.prof ? hp.prof->begin(FWD ? K_SWEEP_FWD : K_SWEEP_BWD, st) : -1;
        sweep_wide_kernel<SR, T, FWD, TRANS><<<grid, 256, smem, st>>>(hp.d_tentries + wl.first, wl.second, hp.dev, Dv,
                                                                      Ov, X, ldx, k, unit, hp.d_sync + 16, hp.d_sync,
                                                                      hp.d_err);
        PP_TRY(cudaGetLastError());
        if (pi >= 0)
            hp.prof->end(pi, st, (double)k * (2.0 * cost.res_rows + (FWD ? 2.0 : 1.0) * cost.sep_rows) + cost.blk_elems,
                         (double)k * cost.pairs_col);
        (*nl)++;
        return cudaSuccess;
    }

    // the top fronts of a stage: one persistent launch (sweep_top_kernel), counters reset from a template
    template <bool FWD, bool TRANS>
    // reset = false (forward only) continues the counters of the previous launch (the first part of the list)
    static cudaError_t sweep_top(const HostPlan &hp, const std::pair<int64_t, int> &wl, const SLevel &cost,
                                 const T *Dv, const T *Ov, T *X, int64_t ldx, int k, int unit, cudaStream_t st,
                                 int64_t *nl, bool reset = true) {
        if (wl.second == 0) return cudaSuccess;
        // many right-hand sides (the star's panels, wide solves): 128-column tasks, when the rows of X allow
        // 16-byte vector loads
        if (k > 256 && ldx % 4 == 0 && reinterpret_cast<uintptr_t>(X) % 16 == 0)
            return sweep_wide<FWD, TRANS>(hp, wl, cost, Dv, Ov, X, ldx, k, unit, st, nl, reset);
        constexpr size_t smem = sweep_top_smem<T>();
        int dev = 0;
        cudaGetDevice(&dev);
        static bool attr[64] = {};
        if (dev < 64 && !attr[dev]) {
            PP_TRY(cudaFuncSetAttribute(sweep_top_kernel<SR, T, FWD, TRANS>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            attr[dev] = true;
        }
        const int ntiles = (k + SW_CT - 1) / SW_CT;
        const size_t cells = (size_t)ntiles * hp.nf;  // per (tile, front)
        if (FWD && !reset) {
            PP_TRY(cudaMemsetAsync(hp.d_sync, 0, sizeof(int), st));  // the task counter only
        } else if (FWD) {
            PP_TRY(reset_sync(hp, hp.d_tpending0, ntiles, st));
            PP_TRY(cudaMemsetAsync(hp.d_sync + 16 + cells, 0, sizeof(int) * 2 * cells, st));  // blocks done
        } else {
            PP_TRY(cudaMemsetAsync(hp.d_sync, 0, sizeof(int), st));
            PP_TRY(cudaMemsetAsync(hp.d_sync + 16, 0, sizeof(int) * 2 * cells, st));  // done flags, blocks done
        }
        int per_sm = 1;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, sweep_top_kernel<SR, T, FWD, TRANS>, 256, smem);
        const int64_t tasks = (int64_t)wl.second * ntiles;
        const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(tasks, std::max(per_sm, 1) * hp.sm_count));
        const int pi = hp.prof ? hp.prof->begin(FWD ? K_SWEEP_FWD : K_SWEEP_BWD, st) : -1;
        sweep_top_kernel<SR, T, FWD, TRANS><<<grid, 256, smem, st>>>(hp.d_tentries + wl.first, wl.second, hp.dev, Dv,
                                                                     Ov, X, ldx, k, unit, hp.d_sync + 16, hp.d_sync,
                                                                     hp.d_err);
        PP_TRY(cudaGetLastError());
        if (pi >= 0)
            hp.prof->end(pi, st, (double)k * (2.0 * cost.res_rows + (FWD ? 2.0 : 1.0) * cost.sep_rows) + cost.blk_elems,
                         (double)k * cost.pairs_col);
        (*nl)++;
        return cudaSuccess;
    }

    // reset = false continues the counters of the previous launch over the same list (its second part)
    // d: 0 lmul!, 1 rmul!; the launch sweeps the bottom fronts of segments seg_lo .. seg_hi (sweep_bottom_kernel)
    template <bool FWD, bool TRANS, int C>
    static cudaError_t sweep_bottom_c(const HostPlan &hp, int d, int seg_lo, int seg_hi,
                                      const std::pair<int64_t, int> &wl, const T *Dv, const T *Ov, T *X, int64_t ldx,
                                      int k, int unit, cudaStream_t st, bool reset) {
        const int ntiles = (k + 32 * C - 1) / (32 * C);
        if (reset) {
            PP_TRY(reset_sync(hp, FWD ? hp.d_spending0 : hp.d_sdone0, ntiles, st));
        } else {
            PP_TRY(cudaMemsetAsync(hp.d_sync, 0, sizeof(int), st));
        }
        const int fmax = std::max(hp.bot_fmax, 1), namax = std::max(hp.bot_namax, 1);
        const size_t smem = 8 * bottom_warp_bytes<T>(fmax, namax);
        int dev = 0;
        cudaGetDevice(&dev);
        static size_t attr[64] = {};
        if (dev < 64 && attr[dev] < smem) {
            PP_TRY(cudaFuncSetAttribute(sweep_bottom_kernel<SR, T, FWD, TRANS, C>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            attr[dev] = smem;
        }
        int per_sm = 1;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, sweep_bottom_kernel<SR, T, FWD, TRANS, C>, 256, smem);
        const int64_t tasks = (int64_t)wl.second * ntiles;
        const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((tasks + 7) / 8, std::max(per_sm, 1) * hp.sm_count));
        sweep_bottom_kernel<SR, T, FWD, TRANS, C><<<grid, 256, smem, st>>>(hp.d_sfronts + wl.first, wl.second, hp.dev,
                                                                           Dv, Ov, X, ldx, k, unit, hp.d_sync + 16,
                                                                           hp.d_sync, hp.d_err, fmax, namax,
                                                                           hp.d_sinfo[d], hp.d_sheavy, seg_lo, seg_hi);
        return cudaGetLastError();
    }

    template <bool FWD, bool TRANS>
    static cudaError_t sweep_bottom(const HostPlan &hp, int d, int seg_lo, int seg_hi,
                                    const std::pair<int64_t, int> &wl, const SLevel &cost,
                                    const T *Dv, const T *Ov, T *X, int64_t ldx, int k, int unit, cudaStream_t st,
                                    int64_t *nl, bool reset = true) {
        if (wl.second == 0) return cudaSuccess;
        const int pi = hp.prof ? hp.prof->begin(FWD ? K_SWEEP_FWD_BOTTOM : K_SWEEP_BWD_BOTTOM, st) : -1;
        // wide solves: two columns per lane (four in the forward sweep of 4-byte types), so each staged factor
        // value serves several (x)(+) pairs and each task's wait and staging serve more columns
        if (FWD && sizeof(T) == 4 && k >= 4 * SWEEP_WIDE_K)  // (backward measured slower at four)
            PP_TRY((sweep_bottom_c<FWD, TRANS, 4>(hp, d, seg_lo, seg_hi, wl, Dv, Ov, X, ldx, k, unit, st, reset)));
        else if (k >= SWEEP_WIDE_K)
            PP_TRY((sweep_bottom_c<FWD, TRANS, 2>(hp, d, seg_lo, seg_hi, wl, Dv, Ov, X, ldx, k, unit, st, reset)));
        else
            PP_TRY((sweep_bottom_c<FWD, TRANS, 1>(hp, d, seg_lo, seg_hi, wl, Dv, Ov, X, ldx, k, unit, st, reset)));
        if (pi >= 0)
            hp.prof->end(pi, st, (double)k * (2.0 * cost.res_rows + (FWD ? 2.0 : 1.0) * cost.sep_rows) + cost.blk_elems,
                         (double)k * cost.pairs_col);
        (*nl)++;
        return cudaSuccess;
    }

    template <bool FWD, bool TRANS, int C>
    static cudaError_t sweep_subtrees_c(const HostPlan &hp, const SubtreeList &sl, const T *Dv, const T *Ov, T *X,
                                        int64_t ldx, int k, int unit, cudaStream_t st) {
        const size_t smem = subtree_cta_bytes<T, C>();
        int dev = 0;
        cudaGetDevice(&dev);
        static size_t attr[64] = {};
        if (dev < 64 && attr[dev] < smem) {
            PP_TRY(cudaFuncSetAttribute(sweep_subtree_kernel<SR, T, FWD, TRANS, C>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            attr[dev] = smem;
        }
        constexpr int cw = 32 * SUBTREE_WARPS * C;
        const int64_t tasks = (int64_t)sl.count * ((k + cw - 1) / cw);  // (subtree, column group)
        sweep_subtree_kernel<SR, T, FWD, TRANS, C><<<(unsigned)tasks, 32 * SUBTREE_WARPS, smem, st>>>(
            hp.d_sroots + sl.off, sl.count, hp.dev, hp.d_fdsc, hp.d_slot, Dv, Ov, X, ldx, k, unit, hp.d_err);
        return cudaGetLastError();
    }

    template <bool FWD, bool TRANS>
    static cudaError_t sweep_subtrees(const HostPlan &hp, const SubtreeList &sl, const T *Dv, const T *Ov, T *X,
                                      int64_t ldx, int k, int unit, cudaStream_t st, int64_t *nl) {
        if (sl.count == 0) return cudaSuccess;
        const int pi = hp.prof ? hp.prof->begin(FWD ? K_SWEEP_FWD_SUBTREE : K_SWEEP_BWD_SUBTREE, st) : -1;
        // wide solves (the star's panels): two columns per lane, so each factor value read from shared memory
        // serves two (x)(+) pairs
        if (k >= SWEEP_WIDE_K)
            PP_TRY((sweep_subtrees_c<FWD, TRANS, 2>(hp, sl, Dv, Ov, X, ldx, k, unit, st)));
        else
            PP_TRY((sweep_subtrees_c<FWD, TRANS, 1>(hp, sl, Dv, Ov, X, ldx, k, unit, st)));
        if (pi >= 0) {
            double pairs = 0, elems = 0;
            for (int64_t i = sl.off; i < sl.off + sl.count && i < (int64_t)hp.sroot_pairs.size(); i++) {
                pairs += hp.sroot_pairs[i];
                elems += hp.sroot_fac[i] / k + 2.0 * hp.sroot_res[i] + (FWD ? 2.0 : 1.0) * hp.sroot_sep[i];
            }
            hp.prof->end(pi, st, elems * k, pairs * k);
        }
        (*nl)++;
        return cudaSuccess;
    }

    // The forward sweep of the bottom of stage s (subtrees, then the other bottom fronts).  In stage 0 the
    // fronts factored by the bottom kernel come first; the stream then waits for the end of the factorization
    // (a no-op once it has ended) and sweeps the rest.
    template <bool TRANS>
    static cudaError_t forward_bottom(const HostPlan &hp, int d, size_t s, const T *Dv, const T *Ov, T *X,
                                      int64_t ldx, int k, int unit, cudaStream_t st, int64_t *nl) {
        const SubtreeList &sub = (d ? hp.sub_r : hp.sub_l)[s];
        const std::pair<int64_t, int> &bot = (d ? hp.sb_fwd_r : hp.sb_fwd)[s];
        const SLevel &cost = (d ? hp.sb_cost_r : hp.sb_cost_l)[s];
        if (s > 0 || !hp.ev_factored) {
            PP_TRY((sweep_subtrees<true, TRANS>(hp, sub, Dv, Ov, X, ldx, k, unit, st, nl)));
            return sweep_bottom<true, TRANS>(hp, d, 2 * (int)s, 2 * (int)s + 1, bot, cost, Dv, Ov, X, ldx, k, unit, st,
                                             nl);
        }
        SubtreeList sa = sub, sb = sub;
        sa.count = std::min(hp.early_sub[d], sub.count);
        sb.off = sub.off + sa.count;
        sb.count = sub.count - sa.count;
        std::pair<int64_t, int> ba = bot, bb = bot;
        ba.second = std::min(hp.early_bot[d], bot.second);
        bb.first = bot.first + ba.second;
        bb.second = bot.second - ba.second;
        const SLevel none{};  // the profile counts the list's bytes and pairs once, with its first launch
        PP_TRY((sweep_subtrees<true, TRANS>(hp, sa, Dv, Ov, X, ldx, k, unit, st, nl)));
        PP_TRY((sweep_bottom<true, TRANS>(hp, d, 0, 0, ba, cost, Dv, Ov, X, ldx, k, unit, st, nl)));
        // the rest of the bottom needs the lower top fronts only (factored by the first top launch)
        PP_TRY(cudaStreamWaitEvent(st, hp.ev_top_a ? hp.ev_top_a : hp.ev_factored, 0));
        PP_TRY((sweep_subtrees<true, TRANS>(hp, sb, Dv, Ov, X, ldx, k, unit, st, nl)));
        return sweep_bottom<true, TRANS>(hp, d, 1, 1, bb, ba.second ? none : cost, Dv, Ov, X, ldx, k, unit, st, nl,
                                         ba.second == 0);
    }

    // The forward top sweep of stage s.  In stage 0, behind a factorization whose top ran in two launches, the
    // fronts other than the roots (listed first) are swept as soon as the first launch has ended, while the
    // roots are still being factored; the roots' entries follow once the factorization has ended, with the
    // counters of the first part.
    template <bool TRANS>
    static cudaError_t forward_top(const HostPlan &hp, size_t s, const std::pair<int64_t, int> &wl,
                                   const std::vector<int> &na, const SLevel &cost, const T *Dv, const T *Ov, T *X,
                                   int64_t ldx, int k, int unit, cudaStream_t st, int64_t *nl) {
        const int a = s < na.size() ? std::min(na[s], wl.second) : wl.second;
        if (s == 0 && hp.ev_factored && hp.ev_top_a && a < wl.second) {
            if (a > 0) PP_TRY((sweep_top<true, TRANS>(hp, {wl.first, a}, cost, Dv, Ov, X, ldx, k, unit, st, nl)));
            PP_TRY(cudaStreamWaitEvent(st, hp.ev_factored, 0));
            const SLevel none{};
            return sweep_top<true, TRANS>(hp, {wl.first + a, wl.second - a}, a > 0 ? none : cost, Dv, Ov, X, ldx, k,
                                          unit, st, nl, a == 0);
        }
        if (s == 0 && hp.ev_factored) PP_TRY(cudaStreamWaitEvent(st, hp.ev_factored, 0));
        return sweep_top<true, TRANS>(hp, wl, cost, Dv, Ov, X, ldx, k, unit, st, nl);
    }

    // the coupling kernels: a CTA row per coupled vertex, 256 columns per CTA
    static dim3 coupling_grid(int nverts, int k) {
        return dim3((unsigned)nverts, (unsigned)std::min(65535, (k + 255) / 256));
    }

    // left: lmul! (X <- A* X: per stage L* forward, U* backward, then the coupling scatter);
    // otherwise rmul! on the transposed layout (per stage the coupling gather, then U* forward, L* backward).
    // src/CPU/blocked/sgetrs.jl:203-255 and src/CPU/chordal/sgetrs.jl:29-51.
    static cudaError_t solve(const HostPlan &hp, const Values &v, int left, void *Xv, int64_t ldx, int k,
                             cudaStream_t st, int64_t *launches) {
        const T *LD = static_cast<const T *>(v.LD), *LL = static_cast<const T *>(v.LL),
                *UD = static_cast<const T *>(v.UD), *UL = static_cast<const T *>(v.UL),
                *Nv = static_cast<const T *>(v.Nval);
        T *X = static_cast<T *>(Xv);
        int64_t nl = 0;
        if (left) {
            for (size_t s = 0; s < hp.lstages.size(); s++) {
                const Stage &sg = hp.lstages[s];
                PP_TRY((forward_bottom<false>(hp, 0, s, LD, LL, X, ldx, k, 1, st, &nl)));
                PP_TRY((forward_top<false>(hp, s, hp.st_fwd[s], hp.st_fwd_a, hp.st_cost_l[s], LD, LL, X, ldx, k, 1, st, &nl)));
                PP_TRY((sweep_top<false, false>(hp, hp.st_bwd[s], hp.st_cost_l[s], UD, UL, X, ldx, k, 0, st, &nl)));
                PP_TRY((sweep_bottom<false, false>(hp, 0, 2 * (int)s, 2 * (int)s + 1, hp.sb_bwd[s], hp.sb_cost_l[s], UD,
                                                   UL, X, ldx, k, 0, st, &nl)));
                PP_TRY((sweep_subtrees<false, false>(hp, hp.sub_l[s], UD, UL, X, ldx, k, 0, st, &nl)));
                if (sg.coupled && sg.nverts > 0) {
                    const int pi = hp.prof ? hp.prof->begin(K_COUPLING, st) : -1;
                    coupling_scatter_kernel<SR, T><<<coupling_grid(sg.nverts, k), 256, 0, st>>>(
                        hp.d_sverts + sg.voff, hp.dev, Nv, X, ldx, k);
                    PP_TRY(cudaGetLastError());
                    if (pi >= 0) hp.prof->end(pi, st, 0, 0);
                    nl++;
                }
            }
        } else {
            for (size_t s = 0; s < hp.rstages.size(); s++) {
                const Stage &sg = hp.rstages[s];
                if (sg.coupled && sg.nverts > 0) {
                    const int pi = hp.prof ? hp.prof->begin(K_COUPLING, st) : -1;
                    coupling_gather_kernel<SR, T><<<coupling_grid(sg.nverts, k), 256, 0, st>>>(
                        hp.d_sverts + sg.voff, hp.dev, Nv, X, ldx, k);
                    PP_TRY(cudaGetLastError());
                    if (pi >= 0) hp.prof->end(pi, st, 0, 0);
                    nl++;
                }
                PP_TRY((forward_bottom<true>(hp, 1, s, UD, UL, X, ldx, k, 0, st, &nl)));
                PP_TRY((forward_top<true>(hp, s, hp.st_fwd_r[s], hp.st_fwd_r_a, hp.st_cost_r[s], UD, UL, X, ldx, k, 0, st, &nl)));
                PP_TRY((sweep_top<false, true>(hp, hp.st_bwd_r[s], hp.st_cost_r[s], LD, LL, X, ldx, k, 1, st, &nl)));
                PP_TRY((sweep_bottom<false, true>(hp, 1, 2 * (int)s, 2 * (int)s + 1, hp.sb_bwd_r[s], hp.sb_cost_r[s], LD,
                                                  LL, X, ldx, k, 1, st, &nl)));
                PP_TRY((sweep_subtrees<false, true>(hp, hp.sub_r[s], LD, LL, X, ldx, k, 1, st, &nl)));
            }
        }
        if (launches) *launches += nl;
        return cudaSuccess;
    }

    static cudaError_t unit_sources(void *X, int64_t ldx, const int *invp, int64_t col0, int k, cudaStream_t st) {
        unit_sources_kernel<SR, T><<<(k + 255) / 256, 256, 0, st>>>(static_cast<T *>(X), ldx, invp, col0, k);
        return cudaGetLastError();
    }

    static cudaError_t unit_positions(void *X, int64_t ldx, const int *pos, int k, cudaStream_t st) {
        unit_positions_kernel<SR, T><<<(k + 255) / 256, 256, 0, st>>>(static_cast<T *>(X), ldx, pos, k);
        return cudaGetLastError();
    }

    // 16-byte vectors on the caller's side when its base and column stride are 16-byte aligned
    static bool vec_ok(const void *B, int64_t ldb) {
        return ((uintptr_t)B % 16 == 0) && ((ldb * (int64_t)sizeof(T)) % 16 == 0);
    }
    static dim3 perm_grid(int n, int k) {
        constexpr int tc = PermTile<T>::TC;
        return dim3((n + PERM_TL - 1) / PERM_TL, (k + tc - 1) / tc);
    }
    static cudaError_t rows_out_mapped(void *B, int64_t ldb, const void *X, int64_t ldx, const int *invp,
                                       const int *cmap, int n, int k, cudaStream_t st) {
        rows_out_kernel<T><<<perm_grid(n, k), 256, 0, st>>>(static_cast<T *>(B), ldb, static_cast<const T *>(X), ldx,
                                                            invp, n, k, cmap, vec_ok(B, ldb));
        return cudaGetLastError();
    }

    static cudaError_t rows_in(const void *B, int64_t ldb, void *X, int64_t ldx, const int *invp, int n, int k,
                               cudaStream_t st) {
        rows_in_kernel<T><<<perm_grid(n, k), 256, 0, st>>>(static_cast<const T *>(B), ldb, static_cast<T *>(X), ldx,
                                                           invp, n, k, vec_ok(B, ldb));
        return cudaGetLastError();
    }
    static cudaError_t rows_out(void *B, int64_t ldb, const void *X, int64_t ldx, const int *invp, int n, int k,
                                cudaStream_t st) {
        return rows_out_mapped(B, ldb, X, ldx, invp, nullptr, n, k, st);
    }
    static cudaError_t cols_in(const void *B, int64_t ldb, void *X, int64_t ldx, const int *invp, int n, int k,
                               cudaStream_t st) {
        cols_in_kernel<T><<<n, 128, 0, st>>>(static_cast<const T *>(B), ldb, static_cast<T *>(X), ldx, invp, n, k);
        return cudaGetLastError();
    }
    static cudaError_t cols_out(void *B, int64_t ldb, const void *X, int64_t ldx, const int *invp, int n, int k,
                                cudaStream_t st) {
        cols_out_kernel<T><<<n, 128, 0, st>>>(static_cast<T *>(B), ldb, static_cast<const T *>(X), ldx, invp, n, k);
        return cudaGetLastError();
    }

    static cudaError_t gemm(int64_t m, int64_t n, int64_t k, void *C, int64_t ldc, const void *A, int64_t lda,
                            const void *B, int64_t ldb, cudaStream_t st) {
        return launch_gemm<SR, T>(m, n, k, static_cast<T *>(C), ldc, static_cast<const T *>(A), lda,
                                  static_cast<const T *>(B), ldb, st);
    }

    static cudaError_t getrf_batched(int n, int64_t count, void *A, cudaStream_t st) {
        if (n <= 128) {  // register-resident, one CTA per block
            T *a = static_cast<T *>(A);
            for (int64_t b0 = 0; b0 < count; b0 += (int64_t)1 << 30) {
                const unsigned cnt = (unsigned)std::min<int64_t>(count - b0, (int64_t)1 << 30);
                T *ab = a + b0 * n * n;
                if (n <= 16)
                    getrf_reg_kernel<SR, T, 1><<<cnt, 256, 0, st>>>(n, ab);
                else if (n <= 32)
                    getrf_reg_kernel<SR, T, 2><<<cnt, 256, 0, st>>>(n, ab);
                else if (n <= 64)
                    getrf_reg_kernel<SR, T, 4><<<cnt, 256, 0, st>>>(n, ab);
                else
                    getrf_reg_kernel<SR, T, 8><<<cnt, 256, 0, st>>>(n, ab);
                PP_TRY(cudaGetLastError());
            }
            return cudaSuccess;
        }
        const size_t smem = (size_t)n * n * sizeof(T);
        if (smem > SMALL_FRONT_SMEM) return cudaErrorInvalidValue;
        int dev = 0;
        cudaGetDevice(&dev);
        static bool attr[64] = {};
        if (dev < 64 && !attr[dev]) {
            PP_TRY(cudaFuncSetAttribute(getrf_batched_kernel<SR, T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)SMALL_FRONT_SMEM));
            attr[dev] = true;
        }
        for (int64_t b0 = 0; b0 < count; b0 += 65535 * 16) {
            const int64_t cnt = std::min<int64_t>(count - b0, 65535 * 16);
            getrf_batched_kernel<SR, T><<<(unsigned)cnt, 256, smem, st>>>(n, static_cast<T *>(A) + b0 * n * n);
            PP_TRY(cudaGetLastError());
        }
        return cudaSuccess;
    }

    static Ops make(int sr, int dt) {
        Ops o;
        o.sr = sr;
        o.dt = dt;
        o.esize = sizeof(T);
        o.small_limit = 1;
        while ((size_t)(o.small_limit + 1) * (o.small_limit + 1) * sizeof(T) <= SMALL_FRONT_SMEM) o.small_limit++;
        o.fill_zero = &fill_zero;
        o.assemble = &assemble;
        o.factor = &factor;
        o.solve = &solve;
        o.unit_sources = &unit_sources;
        o.rows_in = &rows_in;
        o.rows_out = &rows_out;
        o.unit_positions = &unit_positions;
        o.rows_out_mapped = &rows_out_mapped;
        o.cols_in = &cols_in;
        o.cols_out = &cols_out;
        o.gemm = &gemm;
        o.getrf_batched = &getrf_batched;
        return o;
    }
};

}  // namespace pp
