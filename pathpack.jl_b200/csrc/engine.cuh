// engine.cuh — the device kernels of the factorization and the solves, templated on the semiring.
//
//   front_small_kernel   one CTA per front, the whole frontal matrix in shared memory: extend-add of the
//                        children's update matrices, combination with the assembled entries, partial LU over
//                        the front's pivots, write-back of the factor blocks and the update matrix.  Replaces
//                        sgetrf_loop!/sgetrf_loop_1!/sgetrf_send! (src/CPU/chordal/sgetrf.jl:35-290) and the
//                        reference GPU's front_diag_kernel!/extend-add kernels (batched/sgetrf.jl:11-286).
//   large-front path     frontal matrix in global memory: extend_add / combine kernels, then a blocked
//                        right-looking partial LU (panel_kernel: 64-pivot diagonal block in shared memory plus
//                        the column and row panels; the semiring GEMM for the trailing update, which includes
//                        the Schur complement), then extract_kernel.  Replaces factor_front_gpu!
//                        (ext/PATHPACKCUDAExt/chordal/sgetrf.jl:915-992) and dense/sgetrf.jl:31-176.
//   sweep_kernel         one CTA per (front, 32 right-hand sides): a blocked triangular solve on the front's
//                        residual rows and the (+)-scatter to (forward) or gather from (backward) its separator
//                        rows.  Replaces the per-front chordal solves (src/CPU/chordal/strsx.jl:130-1188) and
//                        the reference GPU sweeps (batched/sweep.jl:9-265, chordal/sgetrs.jl:536-1004).
//   coupling kernels     the products with the coupling N between components (src/CPU/sparse/sgemx.jl:101-213).
//   permutation kernels  permuterows!/permutecols! (src/CPU/utils.jl:207-257) fused with the transpose into
//                        the internal layout X[position][rhs] (right-hand sides contiguous).
//
// Every (x)(+) operation follows the per-element dataflow of the reference's CPU path (same operands, same
// stored intermediates), so idempotent semirings give the reference's bits.
#pragma once

#include "gemm.cuh"
#include "plan.h"

namespace pp {

constexpr int SWEEP_CH = 64;     // residual rows per chunk of the sweep
constexpr int PANEL_NB = 64;     // pivots per block of the large-front LU
constexpr int PANEL_THREADS = 128;

template <typename T>
__global__ void fill_kernel(T *__restrict__ p, int64_t n, T v) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        p[i] = v;
}

template <int SR, typename T>
__global__ void fill_zero_kernel(T *__restrict__ p, int64_t n) {
    const T z = Sem<SR, T>::zero();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        p[i] = z;
}

// Partial LU of the star over the first nn pivots of an nj x nj block in shared memory
// (scalar sgetrf2!, src/CPU/dense/sgetrf.jl:151-175, extended to the whole front: the column and row panels
// and the Schur complement take the same per-element steps as strsx2! and sgemx2! in sgetrf_loop!).
template <int SR, typename T>
__device__ __forceinline__ void lu_smem(T *F, int ld, int nj, int nn) {
    using S = Sem<SR, T>;
    const int tid = threadIdx.x, bd = blockDim.x, tx = tid & 31, ty = tid >> 5, nw = bd >> 5;
    for (int p = 0; p < nn; p++) {
        if (!S::integral) {
            const T s = S::star(F[p + p * ld]);
            for (int i = p + 1 + tid; i < nj; i += bd) F[i + p * ld] = S::mul(F[i + p * ld], s);
            __syncthreads();
        }
        for (int j = p + 1 + ty; j < nj; j += nw) {
            const T fpj = F[p + j * ld];
            for (int i = p + 1 + tx; i < nj; i += 32) F[i + j * ld] = S::muladd(F[i + p * ld], fpj, F[i + j * ld]);
        }
        __syncthreads();
    }
}

// combine the extend-added matrix F with the assembled entries (sgetrf_loop!, :101-112, :121-131;
// sgetrf_loop_1!, :217-231)
template <int SR, typename T>
__device__ __forceinline__ T combine_entry(T v, int i, int j, int nn, int na, int64_t Dp, int64_t Lp,
                                           const T *__restrict__ LD, const T *__restrict__ LL,
                                           const T *__restrict__ UD, const T *__restrict__ UL) {
    using S = Sem<SR, T>;
    if (j < nn) {
        if (i < nn) {
            const int64_t o = Dp + i + (int64_t)j * nn;
            return (nn == 1) ? S::add(UD[o], v) : (i > j ? S::add(v, LD[o]) : S::add(v, UD[o]));
        }
        return S::add(LL[Lp + (i - nn) + (int64_t)j * na], v);
    }
    if (i < nn) return S::add(UL[Lp + i + (int64_t)(j - nn) * nn], v);
    return v;
}

// write one entry of a factored front back into the factor arrays
template <typename T>
__device__ __forceinline__ void store_entry(T v, int i, int j, int nn, int na, int64_t Dp, int64_t Lp, T *LD,
                                            T *LL, T *UD, T *UL) {
    if (j < nn) {
        if (i < nn) {
            const int64_t o = Dp + i + (int64_t)j * nn;
            LD[o] = v;
            if (i <= j) UD[o] = v;
        } else {
            LL[Lp + (i - nn) + (int64_t)j * na] = v;
        }
    } else if (i < nn) {
        UL[Lp + i + (int64_t)(j - nn) * nn] = v;
    }
}

// Load through L2 only (ld.global.cg): data another CTA wrote during the same kernel must not come from a
// stale L1 line.
template <typename T>
__device__ __forceinline__ T ld_cg(const T *p) {
    return __ldcg(p);
}

// One front in shared memory (F: nj x nj, leading dimension nj), executed by the whole CTA.  COHERENT reads
// the children's update matrices through L2 (they may have been written by other CTAs of the same kernel).
template <int SR, typename T, bool COHERENT>
__device__ __forceinline__ void front_body(int f, const DevPlan &P, T *F, T *LD, T *LL, T *UD, T *UL, T *W) {
    using S = Sem<SR, T>;
    const int nn = P.nn[f], na = P.na[f], nj = nn + na, ld = nj;
    const int tid = threadIdx.x, bd = blockDim.x;
    const int nj2 = nj * nj;
    for (int e = tid; e < nj2; e += bd) F[e] = S::zero();
    __syncthreads();
    // extend-add of the children's update matrices, last child first (sgetrf_send!, :257-290)
    for (int c = P.chdptr[f + 1] - 1; c >= P.chdptr[f]; c--) {
        const int ch = P.chdtgt[c];
        const int nac = P.na[ch];
        const int *rel = P.rel + P.sptr[ch];
        const T *M = W + P.mptr[ch];
        const int mld = P.mld[ch];
        for (int e = tid; e < nac * nac; e += bd) {
            const int v = e % nac, w = e / nac;
            const int o = rel[v] + rel[w] * ld;
            const T m = COHERENT ? ld_cg(M + v + (int64_t)w * mld) : M[v + (int64_t)w * mld];
            F[o] = S::add(F[o], m);
        }
        __syncthreads();
    }
    const int64_t Dp = P.dptr[f], Lp = P.lptr[f];
    for (int e = tid; e < nj2; e += bd) {
        const int i = e % nj, j = e / nj;
        F[e] = combine_entry<SR, T>(F[e], i, j, nn, na, Dp, Lp, LD, LL, UD, UL);
    }
    __syncthreads();
    lu_smem<SR, T>(F, ld, nj, nn);
    T *Mf = W + P.mptr[f];
    for (int e = tid; e < nj2; e += bd) {
        const int i = e % nj, j = e / nj;
        const T v = F[e];
        if (i < nn || j < nn)
            store_entry<T>(v, i, j, nn, na, Dp, Lp, LD, LL, UD, UL);
        else
            Mf[(i - nn) + (int64_t)(j - nn) * na] = v;
    }
}

template <int SR, typename T>
__global__ void front_small_kernel(const int *__restrict__ fronts, DevPlan P, T *LD, T *LL, T *UD, T *UL, T *W) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    front_body<SR, T, false>(fronts[blockIdx.x], P, reinterpret_cast<T *>(smem_raw), LD, LL, UD, UL, W);
}

// dense blocks: in-place LU of the star of count independent n x n blocks (sgetrf! per block)
template <int SR, typename T>
__global__ void getrf_batched_kernel(int n, T *A) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T *F = reinterpret_cast<T *>(smem_raw);
    T *Ab = A + (int64_t)blockIdx.x * n * n;
    const int n2 = n * n;
    for (int e = threadIdx.x; e < n2; e += blockDim.x) F[e] = Ab[e];
    __syncthreads();
    lu_smem<SR, T>(F, n, n, n);
    for (int e = threadIdx.x; e < n2; e += blockDim.x) Ab[e] = F[e];
}

// ---------------------------------------------------------------- large fronts

template <int SR, typename T>
__global__ void extend_add_kernel(T *__restrict__ F, int ld, const T *__restrict__ M, int mld,
                                  const int *__restrict__ rel, int nac) {
    using S = Sem<SR, T>;
    const int64_t tot = (int64_t)nac * nac;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < tot; e += (int64_t)gridDim.x * blockDim.x) {
        const int v = (int)(e % nac), w = (int)(e / nac);
        const int64_t o = rel[v] + (int64_t)rel[w] * ld;
        F[o] = S::add(F[o], M[v + (int64_t)w * mld]);
    }
}

template <int SR, typename T>
__global__ void combine_kernel(T *__restrict__ F, int nn, int na, int64_t Dp, int64_t Lp, const T *LD,
                               const T *LL, const T *UD, const T *UL) {
    const int nj = nn + na;
    const int64_t tot = (int64_t)nj * nj;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < tot; e += (int64_t)gridDim.x * blockDim.x) {
        const int i = (int)(e % nj), j = (int)(e / nj);
        F[e] = combine_entry<SR, T>(F[e], i, j, nn, na, Dp, Lp, LD, LL, UD, UL);
    }
}

template <typename T>
__global__ void extract_kernel(const T *__restrict__ F, int nn, int na, int64_t Dp, int64_t Lp, T *LD, T *LL,
                               T *UD, T *UL) {
    const int nj = nn + na;
    const int64_t tot = (int64_t)nj * nn + (int64_t)nn * na;  // the first nn columns, then the first nn rows
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < tot; e += (int64_t)gridDim.x * blockDim.x) {
        int i, j;
        if (e < (int64_t)nj * nn) {
            i = (int)(e % nj);
            j = (int)(e / nj);
        } else {
            const int64_t r = e - (int64_t)nj * nn;
            i = (int)(r % nn);
            j = nn + (int)(r / nn);
        }
        store_entry<T>(F[i + (int64_t)j * nj], i, j, nn, na, Dp, Lp, LD, LL, UD, UL);
    }
}

// One block step of the right-looking partial LU of a frontal matrix F (nj x nj, leading dimension ld):
// every CTA factors the b x b diagonal block at (k, k) in shared memory (the same deterministic result);
// CTA 0 writes it back, CTAs 1..nca solve row chunks of the column panel (x <- x U*, strsx2! :R :U :N) and the
// rest column chunks of the row panel (x <- L* x, strsx2! :L :L :U).
template <int SR, typename T>
__global__ void __launch_bounds__(PANEL_THREADS) panel_kernel(T *__restrict__ F, int64_t ld, int nj, int k, int b,
                                                                int nca) {
    using S = Sem<SR, T>;
    constexpr int NB = PANEL_NB;
    __shared__ T D[NB * NB];
    for (int e = threadIdx.x; e < b * b; e += blockDim.x) {
        const int i = e % b, j = e / b;
        D[i + j * NB] = F[(k + i) + (int64_t)(k + j) * ld];
    }
    __syncthreads();
    lu_smem<SR, T>(D, NB, b, b);
    const int g = blockIdx.x;
    if (g == 0) {
        for (int e = threadIdx.x; e < b * b; e += blockDim.x) {
            const int i = e % b, j = e / b;
            F[(k + i) + (int64_t)(k + j) * ld] = D[i + j * NB];
        }
        return;
    }
    T x[NB];
    if (g <= nca) {
        const int r = k + b + (g - 1) * PANEL_THREADS + threadIdx.x;
        if (r >= nj) return;
#pragma unroll
        for (int p = 0; p < NB; p++)
            if (p < b) x[p] = F[r + (int64_t)(k + p) * ld];
#pragma unroll
        for (int p = 0; p < NB; p++) {
            if (p < b) {
                if (!S::integral) x[p] = S::mul(x[p], S::star(D[p + p * NB]));
#pragma unroll
                for (int q = p + 1; q < NB; q++)
                    if (q < b) x[q] = S::muladd(x[p], D[p + q * NB], x[q]);
            }
        }
#pragma unroll
        for (int p = 0; p < NB; p++)
            if (p < b) F[r + (int64_t)(k + p) * ld] = x[p];
    } else {
        const int c = k + b + (g - 1 - nca) * PANEL_THREADS + threadIdx.x;
        if (c >= nj) return;
        T *col = F + (int64_t)c * ld + k;
#pragma unroll
        for (int p = 0; p < NB; p++)
            if (p < b) x[p] = col[p];
#pragma unroll
        for (int p = 0; p < NB; p++) {
            if (p < b) {
#pragma unroll
                for (int q = p + 1; q < NB; q++)
                    if (q < b) x[q] = S::muladd(D[q + p * NB], x[p], x[q]);
            }
        }
#pragma unroll
        for (int p = 0; p < NB; p++)
            if (p < b) col[p] = x[p];
    }
}

// ---------------------------------------------------------------- solves
//
// X[position][rhs] with leading dimension ldx (right-hand sides contiguous).  TRANS selects how the stored
// blocks are read: false for lmul! (X <- L* X, X <- U* X: the blocks as stored), true for rmul! (the
// transposed solves, B <- B U* and B <- B L* on the rows of B).  FWD is the forward sweep with the (+)-scatter
// to the separator; otherwise the backward sweep gathering from it.  unit = diag :U (no star on the diagonal).

template <int SR, typename T, bool FWD, bool TRANS>
__global__ void __launch_bounds__(256) sweep_kernel(const int *__restrict__ fronts, DevPlan P,
                                                    const T *__restrict__ Dv, const T *__restrict__ Ov,
                                                    T *__restrict__ X, int64_t ldx, int k, int unit) {
    using S = Sem<SR, T>;
    constexpr int CH = SWEEP_CH, RPW = CH / 8;
    __shared__ T xs[CH][33];
    const int f = fronts[blockIdx.x];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int col = blockIdx.y * 32 + lane;
    const bool ok = col < k;
    const int rlo = P.rlo[f], nn = P.nn[f], na = P.na[f];
    const T *D = Dv + P.dptr[f];
    const T *O = Ov + P.lptr[f];
    const int *sep = P.stgt + P.sptr[f];
    T *Xc = X + (ok ? col : 0);
    const T z = S::zero();
    const bool scale = !unit && !S::integral;
    auto Te = [&](int r, int c) -> T { return TRANS ? D[c + (int64_t)r * nn] : D[r + (int64_t)c * nn]; };
    auto xg = [&](int row) -> T { return ok ? Xc[(int64_t)row * ldx] : z; };

    if (FWD) {
        for (int c0 = 0; c0 < nn; c0 += CH) {
            const int c1 = min(c0 + CH, nn);
            T acc[RPW];
#pragma unroll
            for (int t = 0; t < RPW; t++) {
                const int r = c0 + w + 8 * t;
                acc[t] = (r < c1) ? xg(rlo + r) : z;
            }
            for (int p = 0; p < c0; p++) {
                const T xp = xg(rlo + p);
#pragma unroll
                for (int t = 0; t < RPW; t++) {
                    const int r = c0 + w + 8 * t;
                    if (r < c1) acc[t] = S::muladd(Te(r, p), xp, acc[t]);
                }
            }
#pragma unroll
            for (int t = 0; t < RPW; t++) {
                const int r = c0 + w + 8 * t;
                if (r < c1) xs[r - c0][lane] = acc[t];
            }
            __syncthreads();
            for (int p = c0; p < c1; p++) {
                if (scale) {
                    if (w == 0) xs[p - c0][lane] = S::mul(xs[p - c0][lane], S::star(Te(p, p)));
                    __syncthreads();
                }
                const T xp = xs[p - c0][lane];
                for (int q = p + 1 + w; q < c1; q += 8) xs[q - c0][lane] = S::muladd(Te(q, p), xp, xs[q - c0][lane]);
                __syncthreads();
            }
            for (int r = c0 + w; r < c1; r += 8)
                if (ok) Xc[(int64_t)(rlo + r) * ldx] = xs[r - c0][lane];
            __syncthreads();
        }
        // separator: X[sep_i] <- X[sep_i] (+) (L21 x)_i
        for (int i0 = w * 4; i0 < na; i0 += 32) {
            T a4[4] = {z, z, z, z};
            for (int p = 0; p < nn; p++) {
                const T xp = (nn <= CH) ? xs[p][lane] : xg(rlo + p);
#pragma unroll
                for (int t = 0; t < 4; t++) {
                    const int i = i0 + t;
                    if (i < na) {
                        const T o = TRANS ? O[p + (int64_t)i * nn] : O[i + (int64_t)p * na];
                        a4[t] = S::muladd(o, xp, a4[t]);
                    }
                }
            }
#pragma unroll
            for (int t = 0; t < 4; t++) {
                const int i = i0 + t;
                if (i < na && ok) S::atomic_add(Xc + (int64_t)sep[i] * ldx, a4[t]);
            }
        }
    } else {
        for (int c1 = nn; c1 > 0; c1 -= CH) {
            const int c0 = max(0, c1 - CH);
            T acc[RPW];
#pragma unroll
            for (int t = 0; t < RPW; t++) {
                const int r = c0 + w + 8 * t;
                acc[t] = (r < c1) ? xg(rlo + r) : z;
            }
            for (int i = 0; i < na; i++) {
                const T xi = xg(sep[i]);
#pragma unroll
                for (int t = 0; t < RPW; t++) {
                    const int r = c0 + w + 8 * t;
                    if (r < c1) {
                        const T o = TRANS ? O[i + (int64_t)r * na] : O[r + (int64_t)i * nn];
                        acc[t] = S::muladd(o, xi, acc[t]);
                    }
                }
            }
            for (int p = nn - 1; p >= c1; p--) {
                const T xp = xg(rlo + p);
#pragma unroll
                for (int t = 0; t < RPW; t++) {
                    const int r = c0 + w + 8 * t;
                    if (r < c1) acc[t] = S::muladd(Te(r, p), xp, acc[t]);
                }
            }
#pragma unroll
            for (int t = 0; t < RPW; t++) {
                const int r = c0 + w + 8 * t;
                if (r < c1) xs[r - c0][lane] = acc[t];
            }
            __syncthreads();
            for (int p = c1 - 1; p >= c0; p--) {
                if (scale) {
                    if (w == 0) xs[p - c0][lane] = S::mul(S::star(Te(p, p)), xs[p - c0][lane]);
                    __syncthreads();
                }
                const T xp = xs[p - c0][lane];
                for (int q = c0 + w; q < p; q += 8) xs[q - c0][lane] = S::muladd(Te(q, p), xp, xs[q - c0][lane]);
                __syncthreads();
            }
            for (int r = c0 + w; r < c1; r += 8)
                if (ok) Xc[(int64_t)(rlo + r) * ldx] = xs[r - c0][lane];
            __syncthreads();
        }
    }
}

// lmul!: after the solve of a component, X[i] <- X[i] (+) N[i, j] (x) X[j] for its positions j
// (sgemx_sparse_st!, src/CPU/sparse/sgemx.jl:193-213); a warp per position, atomics as several j share rows i
template <int SR, typename T>
__global__ void coupling_scatter_kernel(const int *__restrict__ js, int cnt, DevPlan P, const T *__restrict__ Nval,
                                        T *X, int64_t ldx, int k) {
    using S = Sem<SR, T>;
    const int wid = (int)((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (wid >= cnt) return;
    const int j = js[wid];
    for (int64_t p = P.nptr[j]; p < P.nptr[j + 1]; p++) {
        const int i = P.ntgt[p];
        const T v = Nval[p];
        for (int c = lane; c < k; c += 32) S::atomic_add(X + (int64_t)i * ldx + c, S::mul(v, X[(int64_t)j * ldx + c]));
    }
}

// rmul!: before the solve of a component, X[j] <- X[j] (+) X[i] (x) N[i, j] (sgemx_sparse_st!, :101-113)
template <int SR, typename T>
__global__ void coupling_gather_kernel(const int *__restrict__ js, int cnt, DevPlan P, const T *__restrict__ Nval,
                                       T *X, int64_t ldx, int k) {
    using S = Sem<SR, T>;
    const int wid = (int)((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (wid >= cnt) return;
    const int j = js[wid];
    for (int c = lane; c < k; c += 32) {
        T acc = X[(int64_t)j * ldx + c];
        for (int64_t p = P.nptr[j]; p < P.nptr[j + 1]; p++)
            acc = S::muladd(X[(int64_t)P.ntgt[p] * ldx + c], Nval[p], acc);
        X[(int64_t)j * ldx + c] = acc;
    }
}

// X[invp[i]][c] = B[i + c * ldb] (lmul!: permuterows!(B, rinvp) into the internal layout)
template <typename T>
__global__ void rows_in_kernel(const T *__restrict__ B, int64_t ldb, T *__restrict__ X, int64_t ldx,
                               const int *__restrict__ invp, int n, int k) {
    __shared__ T t[32][33];
    const int i0 = blockIdx.x * 32, c0 = blockIdx.y * 32, tx = threadIdx.x, ty = threadIdx.y;
    for (int cc = ty; cc < 32; cc += 8) {
        const int i = i0 + tx, c = c0 + cc;
        if (i < n && c < k) t[cc][tx] = B[i + (int64_t)c * ldb];
    }
    __syncthreads();
    for (int ii = ty; ii < 32; ii += 8) {
        const int i = i0 + ii, c = c0 + tx;
        if (i < n && c < k) X[(int64_t)invp[i] * ldx + c] = t[tx][ii];
    }
}

// B[i + c * ldb] = X[invp[i]][c] (lmul!: permuterows!(B, cperm) out of the internal layout; also the star's
// column panels)
template <typename T>
__global__ void rows_out_kernel(T *__restrict__ B, int64_t ldb, const T *__restrict__ X, int64_t ldx,
                                const int *__restrict__ invp, int n, int k) {
    __shared__ T t[32][33];
    const int i0 = blockIdx.x * 32, c0 = blockIdx.y * 32, tx = threadIdx.x, ty = threadIdx.y;
    for (int ii = ty; ii < 32; ii += 8) {
        const int i = i0 + ii, c = c0 + tx;
        if (i < n && c < k) t[ii][tx] = X[(int64_t)invp[i] * ldx + c];
    }
    __syncthreads();
    for (int cc = ty; cc < 32; cc += 8) {
        const int i = i0 + tx, c = c0 + cc;
        if (i < n && c < k) B[i + (int64_t)c * ldb] = t[tx][cc];
    }
}

// rmul!: X[invp[j]][c] = B[c + j * ldb] and back (permutecols!, src/CPU/utils.jl:233-257)
template <typename T>
__global__ void cols_in_kernel(const T *__restrict__ B, int64_t ldb, T *__restrict__ X, int64_t ldx,
                               const int *__restrict__ invp, int n, int k) {
    const int j = blockIdx.x;
    if (j >= n) return;
    T *dst = X + (int64_t)invp[j] * ldx;
    const T *src = B + (int64_t)j * ldb;
    for (int c = threadIdx.x; c < k; c += blockDim.x) dst[c] = src[c];
}
template <typename T>
__global__ void cols_out_kernel(T *__restrict__ B, int64_t ldb, const T *__restrict__ X, int64_t ldx,
                                const int *__restrict__ invp, int n, int k) {
    const int j = blockIdx.x;
    if (j >= n) return;
    const T *src = X + (int64_t)invp[j] * ldx;
    T *dst = B + (int64_t)j * ldb;
    for (int c = threadIdx.x; c < k; c += blockDim.x) dst[c] = src[c];
}

// the star's unit sources: X = szero, X[invp[col0 + c]][c] = sone
template <int SR, typename T>
__global__ void unit_sources_kernel(T *__restrict__ X, int64_t ldx, const int *__restrict__ invp, int64_t col0,
                                    int k) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c < k) X[(int64_t)invp[col0 + c] * ldx + c] = Sem<SR, T>::one();
}

// copyto!(F, A) on the device (scopyto_loop!, src/CPU/chordal_slu.jl:221-321): a warp per column of A
__device__ __forceinline__ int64_t find_sorted(const int *a, int64_t lo, int64_t hi, int v) {
    while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if (a[mid] < v)
            lo = mid + 1;
        else
            hi = mid;
    }
    return lo;
}

template <typename T>
__global__ void assemble_kernel(DevPlan P, const int *__restrict__ colptr, const int *__restrict__ rowval,
                                const T *__restrict__ nzval, T *LD, T *LL, T *UD, T *UL, T *Nval) {
    const int co = (int)((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (co >= P.n) return;
    const int j = P.invp[co];
    const int f = P.idx[j];
    const int rlo = P.rlo[f], nn = P.nn[f], na = P.na[f];
    const int jstrt = P.bptr[P.fcc[f]];
    for (int p = colptr[co] + lane; p < colptr[co + 1]; p += 32) {
        const int i = P.invp[rowval[p]];
        const T v = nzval[p];
        if (i < jstrt) {
            const int64_t r = find_sorted(P.ntgt, P.nptr[j], P.nptr[j + 1], i);
            if (r < P.nptr[j + 1] && P.ntgt[r] == i) Nval[r] = v;
        } else if (i >= rlo && i < rlo + nn) {
            const int64_t o = P.dptr[f] + (i - rlo) + (int64_t)(j - rlo) * nn;
            LD[o] = v;
            UD[o] = v;
        } else if (i > j) {
            const int64_t q = find_sorted(P.stgt, P.sptr[f], P.sptr[f + 1], i);
            if (q < P.sptr[f + 1] && P.stgt[q] == i) LL[P.lptr[f] + (q - P.sptr[f]) + (int64_t)(j - rlo) * na] = v;
        } else {
            const int g = P.idx[i];
            const int64_t q = find_sorted(P.stgt, P.sptr[g], P.sptr[g + 1], j);
            if (q < P.sptr[g + 1] && P.stgt[q] == j)
                UL[P.lptr[g] + (i - P.rlo[g]) + (q - P.sptr[g]) * P.nn[g]] = v;
        }
    }
}

}  // namespace pp
