// engine.cuh — device building blocks of the factorization and the solves, templated on the semiring.
//
//   front_body           one front in shared memory, executed by one CTA: extend-add of the children's update
//                        matrices, combination with the assembled entries, partial LU over the front's pivots,
//                        write-back of the factor blocks and the update matrix (sgetrf_loop!/sgetrf_loop_1!/
//                        sgetrf_send!, src/CPU/chordal/sgetrf.jl:35-290); the bottom of the tree uses it.
//   lu_smem              right-looking partial LU of the star of a block in shared memory (sgetrf2!'s scalar
//                        path, src/CPU/dense/sgetrf.jl:151-175); also pp_getrf_batched.
//   coupling kernels     the products with the coupling N between components (src/CPU/sparse/sgemx.jl:101-213).
//   permutation kernels  permuterows!/permutecols! (src/CPU/utils.jl:207-257) fused with the transpose into
//                        the internal layout X[position][rhs] (right-hand sides contiguous).
//   assemble_kernel      copyto!(F, A) on the device (src/CPU/chordal_slu.jl:221-321).
//
// Every (x)(+) operation follows the per-element dataflow of the reference's CPU path (same operands, same
// stored intermediates), so idempotent semirings give the reference's bits.
#pragma once

#include "gemm.cuh"
#include "plan.h"

namespace pp {

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

// ---------------------------------------------------------------- solves
//
// X[position][rhs] with leading dimension ldx (right-hand sides contiguous).  TRANS selects how the stored
// blocks are read: false for lmul! (X <- L* X, X <- U* X: the blocks as stored), true for rmul! (the
// transposed solves, B <- B U* and B <- B L* on the rows of B).  FWD is the forward sweep with the (+)-scatter
// to the separator; otherwise the backward sweep gathering from it.  unit = diag :U (no star on the diagonal).

// The coupling products run a thread per (coupled vertex j, right-hand side c): blockIdx.x picks j, the
// threads of blockIdx.y cover the columns (coalesced rows of X), so that a stage with few coupled vertices
// still fills the GPU.
// lmul!: after the solve of a component, X[i] <- X[i] (+) N[i, j] (x) X[j] for its coupling entries
// (sgemx_sparse!, src/CPU/sparse/sgemx.jl:101-213); a zero product changes nothing and is not scattered.
template <int SR, typename T>
__global__ void coupling_scatter_kernel(const int *__restrict__ js, DevPlan P, const T *__restrict__ Nval, T *X,
                                        int64_t ldx, int k) {
    using S = Sem<SR, T>;
    const int j = js[blockIdx.x];
    const int64_t p0 = P.nptr[j], p1 = P.nptr[j + 1];
    for (int c = blockIdx.y * blockDim.x + threadIdx.x; c < k; c += gridDim.y * blockDim.x) {
        const T xj = X[(int64_t)j * ldx + c];
        for (int64_t p = p0; p < p1; p++) {
            const T m = S::mul(Nval[p], xj);
            if (!(m == S::zero())) S::atomic_add(X + (int64_t)P.ntgt[p] * ldx + c, m);
        }
    }
}

// rmul!: before the solve of a component, X[j] <- X[j] (+) X[i] (x) N[i, j] (sgemx_sparse_st!, :101-113)
template <int SR, typename T>
__global__ void coupling_gather_kernel(const int *__restrict__ js, DevPlan P, const T *__restrict__ Nval, T *X,
                                       int64_t ldx, int k) {
    using S = Sem<SR, T>;
    const int j = js[blockIdx.x];
    const int64_t p0 = P.nptr[j], p1 = P.nptr[j + 1];
    for (int c = blockIdx.y * blockDim.x + threadIdx.x; c < k; c += gridDim.y * blockDim.x) {
        T acc = X[(int64_t)j * ldx + c];
        for (int64_t p = p0; p < p1; p++) acc = S::muladd(X[(int64_t)P.ntgt[p] * ldx + c], Nval[p], acc);
        X[(int64_t)j * ldx + c] = acc;
    }
}

// The row permutations of lmul! fused with the transpose between the caller's column-major B (n x k) and the
// internal layout X[position][rhs].  A CTA moves a tile of 64 labels x 256 bytes of right-hand sides through
// shared memory: on the X side each label's row segment (256 contiguous bytes at position invp[label]) is moved
// as 16-byte vectors, on the B side each column's 64 consecutive labels, as 16-byte vectors when B's base and
// column stride allow it (vec_b).  Both sides are coalesced in runs of 256 bytes.
constexpr int PERM_TL = 64;  // labels per tile

template <typename T>
struct PermTile {
    static constexpr int NV = 16 / (int)sizeof(T);     // elements per 16-byte vector
    static constexpr int TC = 256 / (int)sizeof(T);    // right-hand sides per tile
    static constexpr int LD = TC + 1;                  // padded row of the shared tile
};

template <typename T>
union Vec16u {
    uint4 v;
    T e[16 / sizeof(T)];
};

// X[invp[i]][c] = B[i + c * ldb] (lmul!: permuterows!(B, rinvp) into the internal layout)
template <typename T>
__global__ void __launch_bounds__(256) rows_in_kernel(const T *__restrict__ B, int64_t ldb, T *__restrict__ X,
                                                      int64_t ldx, const int *__restrict__ invp, int n, int k,
                                                      bool vec_b) {
    using PT = PermTile<T>;
    constexpr int NV = PT::NV, TC = PT::TC, LD = PT::LD, GL = PERM_TL / NV, GC = TC / NV;
    __shared__ T t[PERM_TL * LD];
    const int l0 = blockIdx.x * PERM_TL, c0 = blockIdx.y * TC;
    // B: column c0 + cc, labels l0 + g NV .. (PERM_TL / NV groups per column)
#pragma unroll
    for (int q = 0; q < TC * GL / 256; q++) {
        const int v = threadIdx.x + 256 * q, cc = v / GL, g = v % GL, c = c0 + cc, l = l0 + g * NV;
        if (c >= k) continue;
        const T *src = B + (int64_t)c * ldb + l;
        Vec16u<T> u;
        if (vec_b && l + NV <= n) {
            u.v = __ldg(reinterpret_cast<const uint4 *>(src));
        } else {
#pragma unroll
            for (int e = 0; e < NV; e++) u.e[e] = l + e < n ? src[e] : T();
        }
#pragma unroll
        for (int e = 0; e < NV; e++) t[(g * NV + e) * LD + cc] = u.e[e];
    }
    __syncthreads();
    // X: the row of label l0 + r, right-hand sides c0 + cv NV ..
#pragma unroll
    for (int q = 0; q < PERM_TL * GC / 256; q++) {
        const int v = threadIdx.x + 256 * q, r = v / GC, cv = v % GC, l = l0 + r, c = c0 + cv * NV;
        if (l >= n || c >= k) continue;
        T *dst = X + (int64_t)invp[l] * ldx + c;
        Vec16u<T> u;
#pragma unroll
        for (int e = 0; e < NV; e++) u.e[e] = t[r * LD + cv * NV + e];
        if (c + NV <= k) {
            *reinterpret_cast<uint4 *>(dst) = u.v;  // ldx is a multiple of 4 elements: 16-byte aligned
        } else {
            for (int e = 0; c + e < k; e++) dst[e] = u.e[e];
        }
    }
}

// B[i + c * ldb] = X[invp[i]][c] (lmul!: permuterows!(B, cperm) out of the internal layout; also the star's
// column panels); with a column map, column c of the panel goes to column cmap[c] of B
template <typename T>
__global__ void __launch_bounds__(256) rows_out_kernel(T *__restrict__ B, int64_t ldb, const T *__restrict__ X,
                                                       int64_t ldx, const int *__restrict__ invp, int n, int k,
                                                       const int *__restrict__ cmap, bool vec_b) {
    using PT = PermTile<T>;
    constexpr int NV = PT::NV, TC = PT::TC, LD = PT::LD, GL = PERM_TL / NV, GC = TC / NV;
    __shared__ T t[PERM_TL * LD];
    const int l0 = blockIdx.x * PERM_TL, c0 = blockIdx.y * TC;
#pragma unroll
    for (int q = 0; q < PERM_TL * GC / 256; q++) {
        const int v = threadIdx.x + 256 * q, r = v / GC, cv = v % GC, l = l0 + r, c = c0 + cv * NV;
        if (l >= n || c >= k) continue;
        const T *src = X + (int64_t)invp[l] * ldx + c;
        Vec16u<T> u;
        if (c + NV <= k) {
            u.v = __ldcs(reinterpret_cast<const uint4 *>(src));  // read once: streaming
        } else {
#pragma unroll
            for (int e = 0; e < NV; e++) u.e[e] = c + e < k ? src[e] : T();
        }
#pragma unroll
        for (int e = 0; e < NV; e++) t[r * LD + cv * NV + e] = u.e[e];
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < TC * GL / 256; q++) {
        const int v = threadIdx.x + 256 * q, cc = v / GL, g = v % GL, c = c0 + cc, l = l0 + g * NV;
        if (c >= k || l >= n) continue;
        T *dst = B + (int64_t)(cmap ? cmap[c] : c) * ldb + l;
        Vec16u<T> u;
#pragma unroll
        for (int e = 0; e < NV; e++) u.e[e] = t[(g * NV + e) * LD + cc];
        if (vec_b && l + NV <= n) {
            __stcs(reinterpret_cast<uint4 *>(dst), u.v);
        } else {
            for (int e = 0; e < NV && l + e < n; e++) dst[e] = u.e[e];
        }
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

// X[pos[c]][c] = one: unit sources at given positions (the star's panels in elimination order)
template <int SR, typename T>
__global__ void unit_positions_kernel(T *__restrict__ X, int64_t ldx, const int *__restrict__ pos, int k) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c < k) X[(int64_t)pos[c] * ldx + c] = Sem<SR, T>::one();
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
