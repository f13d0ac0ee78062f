// top.cuh — the factorization of the fronts above the bottom of the tree: ONE persistent launch over tile tasks.
//
// Each top front keeps its whole frontal matrix F (nj x nj, column-major, leading dimension nj) in the
// workspace, tiled in 64 x 64 blocks: pivot blocks 0 .. kb-1 cover the residual (the last may be short) and
// separator blocks kb .. nbt-1 cover the separator, so the update matrix (the trailing na x na block) is a
// whole number of tiles that the parent reads in place.  The partial LU of the front is a left-looking tile
// algorithm; every task owns one tile:
//
//   EA(J)    assemble column block J: zero, extend-add of the children's update matrices (last child first),
//            then the entries of A (sgetrf_loop!, src/CPU/chordal/sgetrf.jl:101-131; sgetrf_send! :257-290)
//   T(I, J)  F[I, J] (+)= F[I, k] (x) F[k, J] for the pivot blocks k < min(I, J, kb), in increasing k, then
//              I == J < kb : partial LU of the diagonal tile                        (sgetrf2!, dense/sgetrf.jl)
//              J < kb < I or J < I < kb : x <- x U_JJ*   (strsx2! :R :U :N, dense/strsx.jl:596-672)
//              I < kb, I < J : x <- L_II* x             (strsx2! :L :L :U)
//              I, J >= kb : nothing more: the tile is final in the update matrix
//
// For every element this applies the pivots in increasing order with the same operands as the right-looking
// scalar LU, so the factor is bit-identical to the reference's.  Tasks come from one list in an order where
// every dependency is earlier (fronts by height, EA tasks first, tiles by (min(I, J), max(I, J))); CTAs take
// them from an atomic counter and wait (bounded) on per-tile flags, so the lowest unfinished task can always
// run and the launch cannot deadlock.  A front's finished separator tiles are counted, and its parent's EA
// tasks wait for the count.  The reference factors the top of the tree level by level with several launches
// per front (ext/PATHPACKCUDAExt/chordal/sgetrf_top.jl:1-254); here the whole top is one launch and
// independent tiles of different fronts and levels overlap.
//
// Flags of front f start at foff[f]: [J] EA done, [nbt + I * nbt + J] tile final, [nbt + nbt^2] separator
// tiles done.  flags[0] is the task counter, flags[1] the error word.
#pragma once

#include "persist.cuh"

namespace pp {

constexpr int TB = TOP_TILE;  // tile edge
constexpr int TLD = TB + 1;  // padded row of a shared tile

template <typename T>
constexpr size_t factor_top_smem() {
    return sizeof(T) * (2 * (size_t)TB * TLD + 2 * (2 * (size_t)TB + 2));
}

// first row/column and size of tile block b of a front (pivot blocks from 0, separator blocks from nn)
__device__ __forceinline__ void tile_range(int b, int nn, int na, int kb, int &start, int &size) {
    if (b < kb) {
        start = b * TB;
        size = min(TB, nn - start);
    } else {
        const int s = (b - kb) * TB;
        start = nn + s;
        size = min(TB, na - s);
    }
}

// thread 0 polls until *p >= target (bounded; gives up at once when another CTA reported an error)
__device__ __forceinline__ bool cta_wait_geq(const int *p, int target, int *err) {
    __shared__ int s_ok;
    if (threadIdx.x == 0) {
        long long it = 0;
        int ok = 1;
        while (true) {
            const int v = *(volatile const int *)p;
            if (v >= target) break;
            if (*(volatile const int *)err) {
                ok = 0;
                break;
            }
            if (++it > WAIT_LIMIT) {
                atomicExch(err, 1);
                ok = 0;
                break;
            }
            __nanosleep(64);
        }
        __threadfence();
        s_ok = ok;
    }
    __syncthreads();
    const bool ok = s_ok != 0;
    __syncthreads();  // s_ok is reused by the next wait
    return ok;
}

// first index in the ascending a[0 .. n) that is >= v
__device__ __forceinline__ int lower_bound_dev(const int *a, int n, int v) {
    int lo = 0, hi = n;
    while (lo < hi) {
        const int m = (lo + hi) >> 1;
        if (a[m] < v)
            lo = m + 1;
        else
            hi = m;
    }
    return lo;
}

template <int SR, typename T>
__global__ void __launch_bounds__(256) factor_top_kernel(const int4 *__restrict__ tasks, int ntasks, DevPlan P,
                                                         const int64_t *__restrict__ foff, T *LD, T *LL, T *UD,
                                                         T *UL, T *W, int *flags) {
    using S = Sem<SR, T>;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T *As = reinterpret_cast<T *>(smem_raw);  // [TB][TLD]: A operand (rows x k), or the diagonal tile
    T *Bs = As + TB * TLD;                     // [TB][TLD]: B operand (k x columns)
    T *sv = Bs + TB * TLD;                     // 2 x [column TB | row TB | 2]: pivot broadcasts, double-buffered
    int *next = flags, *err = flags + 1;
    const int tid = threadIdx.x, tc = tid & 15, tr = tid >> 4;
    const T z = S::zero();

    while (true) {
        const int t = cta_take(next);
        if (t >= ntasks) return;
        const int4 task = tasks[t];
        const int f = task.x, I = task.y, J = task.z;
        const int nn = P.nn[f], na = P.na[f], nj = nn + na;
        const int kb = (nn + TB - 1) / TB, nbt = kb + (na + TB - 1) / TB;
        int *fl = flags + foff[f];
        T *F = W + P.fws[f];
        const int64_t Dp = P.dptr[f], Lp = P.lptr[f];

        if (task.w == 0) {
            // ---- EA(J): assemble column block J of the frontal matrix
            for (int c = P.chdptr[f]; c < P.chdptr[f + 1]; c++) {
                const int ch = P.chdtgt[c];
                if (P.fws[ch] < 0) continue;  // a bottom child: finished by the earlier launch
                const int sbc = (P.na[ch] + TB - 1) / TB, nbc = (P.nn[ch] + TB - 1) / TB + sbc;
                if (!cta_wait_geq(flags + foff[ch] + nbc + nbc * nbc, sbc * sbc, err)) return;
            }
            int j0, mj;
            tile_range(J, nn, na, kb, j0, mj);
            for (int e = tid; e < nj * mj; e += blockDim.x) F[(e % nj) + (int64_t)(j0 + e / nj) * nj] = z;
            __syncthreads();
            for (int c = P.chdptr[f + 1] - 1; c >= P.chdptr[f]; c--) {
                const int ch = P.chdtgt[c];
                const int nac = P.na[ch];
                const int *rel = P.rel + P.sptr[ch];
                const T *M = W + P.mptr[ch];
                const int mld = P.mld[ch];
                const int wlo = lower_bound_dev(rel, nac, j0), whi = lower_bound_dev(rel, nac, j0 + mj);
                const int cnt = (whi - wlo) * nac;
                for (int e = tid; e < cnt; e += blockDim.x) {
                    const int v = e % nac, w = wlo + e / nac;
                    const int64_t o = rel[v] + (int64_t)rel[w] * nj;
                    F[o] = S::add(F[o], ld_cg(M + v + (int64_t)w * mld));
                }
                __syncthreads();
            }
            for (int e = tid; e < nj * mj; e += blockDim.x) {
                const int i = e % nj, j = j0 + e / nj;
                const int64_t o = i + (int64_t)j * nj;
                F[o] = combine_entry<SR, T>(F[o], i, j, nn, na, Dp, Lp, LD, LL, UD, UL);
            }
            __syncthreads();
            if (tid == 0) {
                __threadfence();
                atomicExch(fl + J, 1);
            }
            continue;
        }

        // ---- T(I, J)
        int i0, mi, j0, mj;
        tile_range(I, nn, na, kb, i0, mi);
        tile_range(J, nn, na, kb, j0, mj);
        if (!cta_wait_geq(fl + J, 1, err)) return;
        T acc[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int r = tr + 16 * i, c = tc + 16 * j;
                acc[i][j] = (r < mi && c < mj) ? ld_cg(F + (i0 + r) + (int64_t)(j0 + c) * nj) : z;
            }
        const int K = min(min(I, J), kb);
        for (int k = 0; k < K; k++) {
            if (!cta_wait_geq(fl + nbt + I * nbt + k, 1, err)) return;
            if (!cta_wait_geq(fl + nbt + k * nbt + J, 1, err)) return;
            const int k0 = k * TB, bk = min(TB, nn - k0);
            for (int e = tid; e < TB * TB; e += blockDim.x) {
                const int r = e % TB, kk = e / TB;
                As[r * TLD + kk] = (r < mi && kk < bk) ? ld_cg(F + (i0 + r) + (int64_t)(k0 + kk) * nj) : z;
                const int kr = e % TB, c = e / TB;
                Bs[kr * TLD + c] = (kr < bk && c < mj) ? ld_cg(F + (k0 + kr) + (int64_t)(j0 + c) * nj) : z;
            }
            __syncthreads();
            for (int kk = 0; kk < bk; kk++) {
                T a[4], b[4];
#pragma unroll
                for (int i = 0; i < 4; i++) a[i] = As[(tr + 16 * i) * TLD + kk];
#pragma unroll
                for (int j = 0; j < 4; j++) b[j] = Bs[kk * TLD + tc + 16 * j];
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int j = 0; j < 4; j++) acc[i][j] = S::muladd(a[i], b[j], acc[i][j]);
            }
            __syncthreads();
        }

        const bool pivot_region = I < kb || J < kb;
        if (pivot_region && I == J) {
            // partial LU of the diagonal tile (mi == mj == b): one barrier per pivot, broadcasts double-buffered
            const int b = mi;
            for (int p = 0; p < b; p++) {
                T *buf = sv + (p & 1) * (2 * TB + 2);
#pragma unroll
                for (int i = 0; i < 4; i++)
                    if (tr + 16 * i == p) {
#pragma unroll
                        for (int j = 0; j < 4; j++) buf[TB + tc + 16 * j] = acc[i][j];
                    }
#pragma unroll
                for (int j = 0; j < 4; j++)
                    if (tc + 16 * j == p) {
#pragma unroll
                        for (int i = 0; i < 4; i++) buf[tr + 16 * i] = acc[i][j];
                    }
                __syncthreads();
                const T s = S::integral ? S::one() : S::star(buf[TB + p]);
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int r = tr + 16 * i;
                    if (r <= p || r >= b) continue;
                    const T l = S::integral ? buf[r] : S::mul(buf[r], s);
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const int c = tc + 16 * j;
                        if (c == p) acc[i][j] = l;
                        else if (c > p && c < b) acc[i][j] = S::muladd(l, buf[TB + c], acc[i][j]);
                    }
                }
            }
            __syncthreads();
        } else if (pivot_region) {
            // a panel tile: stage the factored diagonal tile of its pivot block
            const int d = I > J ? J : I;
            if (!cta_wait_geq(fl + nbt + d * nbt + d, 1, err)) return;
            const int d0 = d * TB, b = min(TB, nn - d0);
            for (int e = tid; e < TB * TB; e += blockDim.x) {
                const int r = e % TB, c = e / TB;
                As[r * TLD + c] = (r < b && c < b) ? ld_cg(F + (d0 + r) + (int64_t)(d0 + c) * nj) : z;
            }
            __syncthreads();
            if (I > J) {
                // x <- x U*: row-wise over the pivot columns p; the pivot column is broadcast
                for (int p = 0; p < b; p++) {
                    T *buf = sv + (p & 1) * (2 * TB + 2);
#pragma unroll
                    for (int j = 0; j < 4; j++)
                        if (tc + 16 * j == p) {
#pragma unroll
                            for (int i = 0; i < 4; i++) buf[tr + 16 * i] = acc[i][j];
                        }
                    __syncthreads();
                    const T s = S::integral ? S::one() : S::star(As[p * TLD + p]);
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const int r = tr + 16 * i;
                        if (r >= mi) continue;
                        const T x = S::integral ? buf[r] : S::mul(buf[r], s);
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            const int c = tc + 16 * j;
                            if (c == p) acc[i][j] = x;
                            else if (c > p && c < b) acc[i][j] = S::muladd(x, As[p * TLD + c], acc[i][j]);
                        }
                    }
                }
            } else {
                // x <- L* x (unit diagonal): column-wise over the pivot rows p; the pivot row is broadcast
                for (int p = 0; p < b; p++) {
                    T *buf = sv + (p & 1) * (2 * TB + 2);
#pragma unroll
                    for (int i = 0; i < 4; i++)
                        if (tr + 16 * i == p) {
#pragma unroll
                            for (int j = 0; j < 4; j++) buf[TB + tc + 16 * j] = acc[i][j];
                        }
                    __syncthreads();
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const int r = tr + 16 * i;
                        if (r <= p || r >= b) continue;
                        const T l = As[r * TLD + p];
#pragma unroll
                        for (int j = 0; j < 4; j++)
                            if (tc + 16 * j < mj) acc[i][j] = S::muladd(l, buf[TB + tc + 16 * j], acc[i][j]);
                    }
                }
            }
            __syncthreads();
        }

        // store the tile (and its factor entries)
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int r = tr + 16 * i, c = tc + 16 * j;
                if (r < mi && c < mj) {
                    F[(i0 + r) + (int64_t)(j0 + c) * nj] = acc[i][j];
                    if (pivot_region) store_entry<T>(acc[i][j], i0 + r, j0 + c, nn, na, Dp, Lp, LD, LL, UD, UL);
                }
            }
        __syncthreads();
        if (tid == 0) {
            __threadfence();
            atomicExch(fl + nbt + I * nbt + J, 1);
            if (!pivot_region) atomicAdd(fl + nbt + nbt * nbt, 1);
        }
    }
}

}  // namespace pp
