// engine_host.cuh — host drivers of the device kernels, templated on the semiring; instantiated once per
// (semiring, element type) in ops_*.cu.
#pragma once

#include <algorithm>

#include "engine.cuh"
#include "ops.h"

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

    static int threads_for(int nj) { return nj <= 16 ? 64 : (nj <= 32 ? 128 : 256); }

    static cudaError_t factor(const HostPlan &hp, const Values &v, cudaStream_t st, int64_t *launches) {
        T *LD = static_cast<T *>(v.LD), *LL = static_cast<T *>(v.LL), *UD = static_cast<T *>(v.UD),
          *UL = static_cast<T *>(v.UL), *W = static_cast<T *>(v.W);
        int64_t nl = 0;
        int dev = 0;
        cudaGetDevice(&dev);
        static bool attr[64] = {};
        if (dev < 64 && !attr[dev]) {
            PP_TRY(cudaFuncSetAttribute(front_small_kernel<SR, T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)SMALL_FRONT_SMEM));
            attr[dev] = true;
        }
        for (const Level &L : hp.flevels) {
            for (const FrontGroup &g : L.groups) {
                if (!g.large) {
                    const size_t smem = (size_t)g.max_nj * g.max_nj * sizeof(T);
                    const int pi = hp.prof ? hp.prof->begin(K_FRONT, st) : -1;
                    front_small_kernel<SR, T><<<g.count, threads_for(g.max_nj), smem, st>>>(
                        hp.d_ffronts + g.off, hp.dev, LD, LL, UD, UL, W);
                    PP_TRY(cudaGetLastError());
                    if (pi >= 0) hp.prof->end(pi, st, g.bytes, g.pairs);
                    nl++;
                    continue;
                }
                // large fronts one at a time (their ids are on the host in the same order)
                for (int t = 0; t < g.count; t++) {
                    PP_TRY(factor_large(hp, hp.h_ffronts[g.off + t], LD, LL, UD, UL, W, st, &nl));
                }
            }
        }
        if (launches) *launches += nl;
        return cudaSuccess;
    }

    static cudaError_t factor_large(const HostPlan &hp, int f, T *LD, T *LL, T *UD, T *UL, T *W, cudaStream_t st,
                                    int64_t *nl) {
        const int nn = hp.nn[f], na = hp.na[f], nj = nn + na;
        T *F = W + hp.fws[f];
        const int64_t nj2 = (int64_t)nj * nj;
        Profiler *pr = hp.prof;
        int pi = pr ? pr->begin(K_LARGE_AUX, st) : -1;
        PP_TRY(fill_zero(F, nj2, st));
        (*nl)++;
        double aux = (double)nj2;
        for (int c = hp.chdptr[f + 1] - 1; c >= hp.chdptr[f]; c--) {
            const int ch = hp.chdtgt[c];
            const int nac = hp.na[ch];
            extend_add_kernel<SR, T><<<grid_for((int64_t)nac * nac, 256), 256, 0, st>>>(
                F, nj, W + hp.mptr[ch], hp.mld[ch], hp.d_rel + hp.sptr[ch], nac);
            PP_TRY(cudaGetLastError());
            (*nl)++;
            aux += 3.0 * nac * nac;
        }
        combine_kernel<SR, T><<<grid_for(nj2, 256), 256, 0, st>>>(F, nn, na, hp.dptr[f], hp.lptr[f], LD, LL, UD, UL);
        PP_TRY(cudaGetLastError());
        (*nl)++;
        aux += 2.0 * nj2 + 2.0 * nn * nn + 2.0 * nn * na;
        if (pi >= 0) pr->end(pi, st, aux, 0);
        for (int k = 0; k < nn; k += PANEL_NB) {
            const int b = std::min(PANEL_NB, nn - k);
            const int rem = nj - k - b;
            const int nca = (rem + PANEL_THREADS - 1) / PANEL_THREADS;
            pi = pr ? pr->begin(K_PANEL, st) : -1;
            panel_kernel<SR, T><<<1 + 2 * nca, PANEL_THREADS, 0, st>>>(F, nj, nj, k, b, nca);
            PP_TRY(cudaGetLastError());
            if (pi >= 0)
                pr->end(pi, st, 2.0 * b * b + 4.0 * rem * b,
                        (double)(b - 1) * b * (2.0 * b - 1) / 6 + (double)rem * b * (b - 1));
            (*nl)++;
            if (rem > 0) {
                T *C = F + (k + b) + (int64_t)(k + b) * nj;
                const T *A = F + (k + b) + (int64_t)k * nj;
                const T *B = F + k + (int64_t)(k + b) * nj;
                pi = pr ? pr->begin(K_GEMM, st) : -1;
                PP_TRY((launch_gemm<SR, T>(rem, rem, b, C, nj, A, nj, B, nj, st)));
                if (pi >= 0) pr->end(pi, st, 2.0 * rem * b + 2.0 * rem * (double)rem, (double)rem * rem * b);
                (*nl)++;
            }
        }
        pi = pr ? pr->begin(K_LARGE_AUX, st) : -1;
        extract_kernel<T><<<grid_for((int64_t)nj * nn + (int64_t)nn * na, 256), 256, 0, st>>>(
            F, nn, na, hp.dptr[f], hp.lptr[f], LD, LL, UD, UL);
        PP_TRY(cudaGetLastError());
        if (pi >= 0) pr->end(pi, st, 2.0 * ((double)nj * nn + (double)nn * na), 0);
        (*nl)++;
        return cudaSuccess;
    }

    template <bool FWD, bool TRANS>
    static cudaError_t sweep_levels(const HostPlan &hp, const Stage &sg, bool ascending, const T *Dv, const T *Ov,
                                    T *X, int64_t ldx, int k, int unit, cudaStream_t st, int64_t *nl) {
        const int ny = (k + 31) / 32;
        const int nlev = (int)sg.levels.size();
        for (int t = 0; t < nlev; t++) {
            const SLevel &lv = sg.levels[ascending ? t : nlev - 1 - t];
            if (lv.count == 0) continue;
            dim3 grid((unsigned)lv.count, (unsigned)ny);
            const int pi = hp.prof ? hp.prof->begin(FWD ? K_SWEEP_FWD : K_SWEEP_BWD, st) : -1;
            sweep_kernel<SR, T, FWD, TRANS><<<grid, 256, 0, st>>>(hp.d_sfronts + lv.off, hp.dev, Dv, Ov, X, ldx, k,
                                                                 unit);
            PP_TRY(cudaGetLastError());
            if (pi >= 0)
                hp.prof->end(pi, st, (double)k * (2.0 * lv.res_rows + (FWD ? 2.0 : 1.0) * lv.sep_rows) + lv.blk_elems,
                             (double)k * lv.pairs_col);
            (*nl)++;
        }
        return cudaSuccess;
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
            for (const Stage &sg : hp.lstages) {
                PP_TRY((sweep_levels<true, false>(hp, sg, true, LD, LL, X, ldx, k, 1, st, &nl)));
                PP_TRY((sweep_levels<false, false>(hp, sg, false, UD, UL, X, ldx, k, 0, st, &nl)));
                if (sg.coupled && sg.nverts > 0) {
                    const int pi = hp.prof ? hp.prof->begin(K_COUPLING, st) : -1;
                    coupling_scatter_kernel<SR, T><<<(sg.nverts + 7) / 8, 256, 0, st>>>(
                        hp.d_sverts + sg.voff, sg.nverts, hp.dev, Nv, X, ldx, k);
                    PP_TRY(cudaGetLastError());
                    if (pi >= 0) hp.prof->end(pi, st, 0, 0);
                    nl++;
                }
            }
        } else {
            for (const Stage &sg : hp.rstages) {
                if (sg.coupled && sg.nverts > 0) {
                    const int pi = hp.prof ? hp.prof->begin(K_COUPLING, st) : -1;
                    coupling_gather_kernel<SR, T><<<(sg.nverts + 7) / 8, 256, 0, st>>>(
                        hp.d_sverts + sg.voff, sg.nverts, hp.dev, Nv, X, ldx, k);
                    PP_TRY(cudaGetLastError());
                    if (pi >= 0) hp.prof->end(pi, st, 0, 0);
                    nl++;
                }
                PP_TRY((sweep_levels<true, true>(hp, sg, true, UD, UL, X, ldx, k, 0, st, &nl)));
                PP_TRY((sweep_levels<false, true>(hp, sg, false, LD, LL, X, ldx, k, 1, st, &nl)));
            }
        }
        if (launches) *launches += nl;
        return cudaSuccess;
    }

    static cudaError_t unit_sources(void *X, int64_t ldx, const int *invp, int64_t col0, int k, cudaStream_t st) {
        unit_sources_kernel<SR, T><<<(k + 255) / 256, 256, 0, st>>>(static_cast<T *>(X), ldx, invp, col0, k);
        return cudaGetLastError();
    }

    static cudaError_t rows_in(const void *B, int64_t ldb, void *X, int64_t ldx, const int *invp, int n, int k,
                               cudaStream_t st) {
        dim3 grid((n + 31) / 32, (k + 31) / 32), block(32, 8);
        rows_in_kernel<T><<<grid, block, 0, st>>>(static_cast<const T *>(B), ldb, static_cast<T *>(X), ldx, invp, n, k);
        return cudaGetLastError();
    }
    static cudaError_t rows_out(void *B, int64_t ldb, const void *X, int64_t ldx, const int *invp, int n, int k,
                                cudaStream_t st) {
        dim3 grid((n + 31) / 32, (k + 31) / 32), block(32, 8);
        rows_out_kernel<T><<<grid, block, 0, st>>>(static_cast<T *>(B), ldb, static_cast<const T *>(X), ldx, invp, n, k);
        return cudaGetLastError();
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
        o.cols_in = &cols_in;
        o.cols_out = &cols_out;
        o.gemm = &gemm;
        o.getrf_batched = &getrf_batched;
        return o;
    }
};

}  // namespace pp
