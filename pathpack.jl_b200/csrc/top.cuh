// top.cuh — the factorization of the fronts above the bottom of the tree: ONE persistent launch over tile tasks.
//
// Each top front keeps its whole frontal matrix F (nj x nj, column-major, leading dimension nj) in the
// workspace, tiled in 64 x 64 blocks: pivot blocks 0 .. kb-1 cover the residual (the last may be short) and
// separator blocks kb .. nbt-1 cover the separator, so the update matrix (the trailing na x na block) is a
// whole number of tiles that the parent reads in place.  The partial LU of the front is a left-looking tile
// algorithm; every task owns one tile:
//
//   T(I, J)  assemble the tile in shared memory: zero, extend-add of the children's update matrices (last
//            child first), then the entries of A (sgetrf_loop!, src/CPU/chordal/sgetrf.jl:101-131; sgetrf_send!
//            :257-290); F[I, J] (+)= F[I, k] (x) F[k, J] for the pivot blocks k < min(I, J, kb), increasing k;
//              I == J < kb : partial LU of the diagonal tile                        (sgetrf2!, dense/sgetrf.jl)
//              J < kb < I or J < I < kb : x <- x U_JJ*   (strsx2! :R :U :N, dense/strsx.jl:596-672)
//              I < kb, I < J : x <- L_II* x             (strsx2! :L :L :U)
//              I, J >= kb : nothing more: the tile is final in the update matrix
//
// For every element this applies the pivots in increasing order with the same operands as the right-looking
// scalar LU, so the factor is bit-identical to the reference's.  Tasks come from one list in an order where
// every dependency is earlier (fronts by height, tiles by (min(I, J), max(I, J))); CTAs take them from an
// atomic counter and wait (bounded) on per-tile flags, so the lowest unfinished task can always run and the
// launch cannot deadlock.  A front's finished separator tiles are counted, and its parent's tiles wait for
// the count.  The children's rows and columns that land in each tile block of the parent are contiguous
// ranges of the sorted rel[] (crng, computed on the host), so a tile gathers exactly its own entries.  The reference factors the top of the tree level by level with several launches
// per front (ext/PATHPACKCUDAExt/chordal/sgetrf_top.jl:1-254); here the whole top is one launch and
// independent tiles of different fronts and levels overlap.
//
// Flags of front f start at foff[f]: [I * nbt + J] tile final, [nbt^2] separator tiles done.  flags[0] is the
// task counter; err is the error word of the factorization.
#pragma once

#include "pathpack_b200.h"
#include "persist.cuh"

namespace pp {

constexpr int TB = TOP_TILE;  // tile edge
constexpr int TLD = TB + 1;  // padded row of a shared tile
constexpr int CHILD_CHUNK = 32;  // children whose ranges are staged in shared memory at a time

template <typename T>
constexpr size_t factor_top_smem() {
    return sizeof(T) * 2 * (size_t)TB * TLD;
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

// acquire load of a flag another CTA publishes (__threadfence, then an atomic store): the data the producer
// wrote before the flag is visible to this thread, and to the rest of the CTA after the barrier that follows
__device__ __forceinline__ int ld_acquire(const int *p) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// thread 0 polls until *p >= target (bounded; gives up at once when another CTA reported an error)
__device__ __forceinline__ bool cta_wait_geq(const int *p, int target, int *err) {
    __shared__ int s_ok;
    if (threadIdx.x == 0) {
        WaitBound wb(err);
        int ok = 1;
        while (ld_acquire(p) < target) {
            if (*(volatile const int *)err) {
                ok = 0;
                break;
            }
            if (wb.expired()) {
                atomicExch(err, 1);
                ok = 0;
                break;
            }
            __nanosleep(64);
        }
        s_ok = ok;
    }
    __syncthreads();
    const bool ok = s_ok != 0;
    __syncthreads();  // s_ok is reused by the next wait
    return ok;
}

// the entry of A that combine_entry adds to the assembled value of element (i, j) of the front (z if none)
template <typename T>
__device__ __forceinline__ T a_entry(int i, int j, int nn, int na, int64_t Dp, int64_t Lp, const T *LD, const T *LL,
                                     const T *UD, const T *UL, T z) {
    if (j < nn) {
        if (i < nn) {
            const int64_t o = Dp + i + (int64_t)j * nn;
            return (nn == 1 || i <= j) ? UD[o] : LD[o];
        }
        return LL[Lp + (i - nn) + (int64_t)j * na];
    }
    if (i < nn) return UL[Lp + i + (int64_t)(j - nn) * nn];
    return z;
}

// combine_entry with the entry of A already loaded (a_entry): the same operations in the same order
template <int SR, typename T>
__device__ __forceinline__ T combine_with(T v, T a, int i, int j, int nn) {
    using S = Sem<SR, T>;
    if (j < nn) {
        if (i < nn) return nn == 1 ? S::add(a, v) : S::add(v, a);
        return S::add(a, v);
    }
    if (i < nn) return S::add(a, v);
    return v;
}

template <bool B>
struct Half {
    static constexpr bool hi = B;  // pivots 32 .. 63 (held in the second register set)
};

// x <- x U* for the 64 rows of the tile (strsx2! :R :U :N): U is the upper triangle of the b x b diagonal tile D
template <int SR, typename T>
__device__ __forceinline__ void tile_solve_right(T *X, const T *D, int b) {
    using S = Sem<SR, T>;
    const int l = threadIdx.x & 31, w = threadIdx.x >> 5;
    T x0[8], x1[8];
#pragma unroll
    for (int q = 0; q < 8; q++) {
        x0[q] = X[(8 * w + q) * TLD + l];
        x1[q] = X[(8 * w + q) * TLD + l + 32];
    }
    auto step = [&](int p, auto half) {
        constexpr bool hi = decltype(half)::hi;
        const T s = S::integral ? S::one() : S::star(D[p * TLD + p]);
        const T u0 = hi ? S::zero() : D[p * TLD + l], u1 = D[p * TLD + l + 32];
        const bool g0 = !hi && l > p && l < b, g1 = l + 32 > p && l + 32 < b;  // rows < 32 are done when hi
#pragma unroll
        for (int q = 0; q < 8; q++) {
            T xp = __shfl_sync(0xffffffffu, hi ? x1[q] : x0[q], p & 31);
            if (!S::integral) xp = S::mul(xp, s);
            if (!hi && l == p) x0[q] = xp;
            if (hi && l + 32 == p) x1[q] = xp;
            if (!hi) x0[q] = muladd_if<SR, T>(g0, xp, u0, x0[q]);
            x1[q] = muladd_if<SR, T>(g1, xp, u1, x1[q]);
        }
    };
    for (int p = 0; p < min(b, 32); p++) step(p, Half<false>());
    for (int p = 32; p < b; p++) step(p, Half<true>());
#pragma unroll
    for (int q = 0; q < 8; q++) {
        X[(8 * w + q) * TLD + l] = x0[q];
        X[(8 * w + q) * TLD + l + 32] = x1[q];
    }
}

// x <- L* x for the 64 columns of the tile (strsx2! :L :L :U): L is the strict lower triangle of D
template <int SR, typename T>
__device__ __forceinline__ void tile_solve_left(T *X, const T *D, int b) {
    using S = Sem<SR, T>;
    const int l = threadIdx.x & 31, w = threadIdx.x >> 5;
    T x0[8], x1[8];
#pragma unroll
    for (int q = 0; q < 8; q++) {
        x0[q] = X[l * TLD + 8 * w + q];
        x1[q] = X[(l + 32) * TLD + 8 * w + q];
    }
    auto step = [&](int p, auto half) {
        constexpr bool hi = decltype(half)::hi;
        const T l0 = hi ? S::zero() : D[l * TLD + p], l1 = D[(l + 32) * TLD + p];
        const bool g0 = !hi && l > p && l < b, g1 = l + 32 > p && l + 32 < b;  // rows < 32 are done when hi
#pragma unroll
        for (int q = 0; q < 8; q++) {
            const T xp = __shfl_sync(0xffffffffu, hi ? x1[q] : x0[q], p & 31);
            if (!hi) x0[q] = muladd_if<SR, T>(g0, l0, xp, x0[q]);
            x1[q] = muladd_if<SR, T>(g1, l1, xp, x1[q]);
        }
    };
    for (int p = 0; p < min(b, 32); p++) step(p, Half<false>());
    for (int p = 32; p < b; p++) step(p, Half<true>());
#pragma unroll
    for (int q = 0; q < 8; q++) {
        X[l * TLD + 8 * w + q] = x0[q];
        X[(l + 32) * TLD + 8 * w + q] = x1[q];
    }
}

// Per-task timeline (pp_options.trace): for task t, trace[TRACE_WORDS * t + ...] = global timer (ns) when the
// task was taken, when its tile was assembled (children's update matrices and A), when the products with the
// pivot blocks were done, when its flag was set, then (SM << 32) | front and (I << 32) | J.
constexpr int TRACE_WORDS = PP_TRACE_WORDS;  // include/pathpack_b200.h

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned smid() {
    unsigned s;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(s));
    return s;
}

// The partial LU of the b x b diagonal tile in X, held in registers: the scheme of getrf_reg_kernel (getrf.cuh)
// on a 64 x 64 tile (per element the scalar LU's operations in its order, sgetrf2!, src/CPU/dense/sgetrf.jl:
// 151-175, as lu_smem).  Thread (tr, tc) = (tid % 16, tid / 16) holds f[a][c] = X[tr + 16a][tc + 16c]; per pivot the
// half-warp holding column p scales it (the diagonal by a shuffle) and publishes it, the threads holding row p
// publish it, one barrier (column and row double-buffered in cb / rb, 2 x 16 x 4 elements each), then every
// thread updates its trailing entries.  Every thread of the CTA calls it.
template <int SR, typename T>
__device__ __forceinline__ void tile_lu_reg(T *X, int b, T *cb, T *rb) {
    using S = Sem<SR, T>;
    constexpr int R = 4;
    const int tid = threadIdx.x, tr = tid & 15, tc = tid >> 4, lane = tid & 31;
    const T z = S::zero();
    T f[R][R];
#pragma unroll
    for (int a = 0; a < R; a++)
#pragma unroll
        for (int c = 0; c < R; c++) {
            const int i = tr + 16 * a, j = tc + 16 * c;
            f[a][c] = (i < b && j < b) ? X[i * TLD + j] : z;
        }
#pragma unroll
    for (int q = 0; q < R; q++) {
        const int pend = min(16, b - 16 * q);  // pivots of this phase (uniform over the CTA)
        for (int pp = 0; pp < pend; pp++) {
            const int p = 16 * q + pp, buf = p & 1;
            T *colb = cb + buf * 16 * R, *rowb = rb + buf * 16 * R;
            if (tc == pp) {  // one half-warp holds column p
                if (!S::integral) {
                    const unsigned half = (lane & 16) ? 0xffff0000u : 0x0000ffffu;
                    const T s = S::star(__shfl_sync(half, f[q][q], (lane & 16) | pp));
#pragma unroll
                    for (int a = q; a < R; a++)
                        if (a > q || tr > pp) f[a][q] = S::mul(f[a][q], s);
                }
#pragma unroll
                for (int a = q; a < R; a++) colb[tr * R + a] = f[a][q];
            }
            if (tr == pp) {
#pragma unroll
                for (int c = q; c < R; c++) rowb[tc * R + c] = f[q][c];
            }
            __syncthreads();
            T cv[R], rv[R];
#pragma unroll
            for (int a = q; a < R; a++) cv[a] = colb[tr * R + a];
#pragma unroll
            for (int c = q; c < R; c++) rv[c] = rowb[tc * R + c];
            const bool r0 = tr > pp, c0 = tc > pp;  // row 16q + tr and column 16q + tc still trail pivot p
#pragma unroll
            for (int a = q; a < R; a++)
#pragma unroll
                for (int c = q; c < R; c++)
                    if ((a > q || r0) && (c > q || c0)) f[a][c] = S::muladd(cv[a], rv[c], f[a][c]);
        }
    }
#pragma unroll
    for (int a = 0; a < R; a++)
#pragma unroll
        for (int c = 0; c < R; c++) {
            const int i = tr + 16 * a, j = tc + 16 * c;
            if (i < b && j < b) X[i * TLD + j] = f[a][c];
        }
    __syncthreads();
}

template <int SR, typename T>
__global__ void __launch_bounds__(256) factor_top_kernel(const int4 *__restrict__ tasks, int ntasks, DevPlan P,
                                                         const int64_t *__restrict__ foff,
                                                         const int64_t *__restrict__ croff,
                                                         const int *__restrict__ crng, T *LD, T *LL, T *UD, T *UL,
                                                         T *W, int *flags, int *err, unsigned long long *trace) {
    using S = Sem<SR, T>;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T *As = reinterpret_cast<T *>(smem_raw);  // [TB][TLD]: A operand (rows x k), or the diagonal tile
    T *Bs = As + TB * TLD;                     // [TB][TLD]: B operand (k x columns)
    int *next = flags;
    __shared__ int4 s_child[CHILD_CHUNK];  // per child: first row, rows, first column, columns in this tile
    __shared__ int64_t s_cmat[CHILD_CHUNK];
    __shared__ int2 s_cmeta[CHILD_CHUNK];  // leading dimension of the update matrix, offset of rel
    __shared__ int s_ctop[CHILD_CHUNK];    // the child if it is a top front, else -1
    __shared__ int s_bad;
    __shared__ __align__(16) T s_luc[2 * 16 * 4], s_lur[2 * 16 * 4];  // tile_lu_reg's published column and row
    const int tid = threadIdx.x, tc = tid & 15, tr = tid >> 4;
    const T z = S::zero();

    while (true) {
        const int t = cta_take(next);
        if (t >= ntasks) return;
        unsigned long long *trc = trace && threadIdx.x == 0 ? trace + (size_t)TRACE_WORDS * t : nullptr;
        if (trc) trc[0] = global_ns();
        const int4 task = tasks[t];
        const int f = task.x, I = task.y, J = task.z;
        const int nn = P.nn[f], na = P.na[f], nj = nn + na;
        const int kb = (nn + TB - 1) / TB, nbt = kb + (na + TB - 1) / TB;
        int *fl = flags + foff[f];
        T *F = W + P.fws[f];
        const int64_t Dp = P.dptr[f], Lp = P.lptr[f];

        // ---- T(I, J): assemble the tile in shared memory once the children's update matrices are final
        int i0, mi, j0, mj;
        tile_range(I, nn, na, kb, i0, mi);
        tile_range(J, nn, na, kb, j0, mj);
        // issue the loads that do not depend on the children first: this thread's entries of A (element
        // e = tid + 256 k of the tile, column-major), and per child its ranges and update-matrix location
        const int c_lo = P.chdptr[f], c_hi = P.chdptr[f + 1];
        T aval[TB * TB / 256];
#pragma unroll
        for (int k = 0; k < TB * TB / 256; k++) {
            const int e = tid + 256 * k, r = e % TB, c = e / TB;
            aval[k] = (r < mi && c < mj) ? a_entry<T>(i0 + r, j0 + c, nn, na, Dp, Lp, LD, LL, UD, UL, z) : z;
        }
        for (int e = tid; e < TB * TB; e += blockDim.x) As[(e % TB) * TLD + e / TB] = z;
        for (int cb = c_hi; cb > c_lo; cb -= CHILD_CHUNK) {
            // children cb - CHILD_CHUNK .. cb - 1 (clamped), applied last first
            const int c0 = max(c_lo, cb - CHILD_CHUNK), nch = cb - c0;
            if (tid < nch) {
                const int c = c0 + tid, ch = P.chdtgt[c];
                const int *rng = crng + croff[c];
                const int vlo = rng[I], wlo = rng[J];
                s_child[tid] = make_int4(vlo, rng[I + 1] - vlo, wlo, rng[J + 1] - wlo);
                s_cmat[tid] = P.mptr[ch];
                s_cmeta[tid] = make_int2(P.mld[ch], (int)P.sptr[ch]);
                s_ctop[tid] = P.fws[ch] >= 0 ? ch : -1;
            }
            __syncthreads();
            if (tid == 0) {
                // the top children must have finished their update matrices (bottom ones did, earlier launch)
                int bad = 0;
                for (int q = 0; q < nch && !bad; q++) {
                    const int ch = s_ctop[q];
                    if (ch < 0) continue;
                    const int sbc = (P.na[ch] + TB - 1) / TB, nbc = (P.nn[ch] + TB - 1) / TB + sbc;
                    WaitBound wb(err);
                    while (ld_acquire(flags + foff[ch] + nbc * nbc) < sbc * sbc) {
                        if (*(volatile const int *)err || wb.expired()) {
                            atomicExch(err, 1);
                            bad = 1;
                            break;
                        }
                        __nanosleep(64);
                    }
                }
                s_bad = bad;
            }
            __syncthreads();
            if (s_bad) return;  // uniform: every thread reads the value thread 0 wrote before the barrier
            for (int q = nch - 1; q >= 0; q--) {
                const int4 cr = s_child[q];
                const int dv = cr.y, cnt = cr.y * cr.w;
                const T *M = W + s_cmat[q];
                const int mld = s_cmeta[q].x;
                const int *rel = P.rel + s_cmeta[q].y;
                for (int base = 0; base < cnt; base += 8 * 256) {
                    T m[8];
                    int o[8];
#pragma unroll
                    for (int k = 0; k < 8; k++) {
                        const int e = base + tid + 256 * k;
                        o[k] = -1;
                        if (e < cnt) {
                            const int v = cr.x + e % dv, w = cr.z + e / dv;
                            o[k] = (rel[v] - i0) * TLD + (rel[w] - j0);
                            m[k] = ld_cg(M + v + (int64_t)w * mld);
                        }
                    }
#pragma unroll
                    for (int k = 0; k < 8; k++)
                        if (o[k] >= 0) As[o[k]] = S::add(As[o[k]], m[k]);
                }
                __syncthreads();
            }
        }
#pragma unroll
        for (int k = 0; k < TB * TB / 256; k++) {
            const int e = tid + 256 * k, r = e % TB, c = e / TB;
            if (r < mi && c < mj) As[r * TLD + c] = combine_with<SR, T>(As[r * TLD + c], aval[k], i0 + r, j0 + c, nn);
        }
        __syncthreads();
        if (trc) trc[1] = global_ns();
        T acc[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) acc[i][j] = As[(tr + 16 * i) * TLD + tc + 16 * j];
        __syncthreads();
        const int K = min(min(I, J), kb);
        for (int k = 0; k < K; k++) {
            if (!cta_wait_geq(fl + I * nbt + k, 1, err)) return;
            if (!cta_wait_geq(fl + k * nbt + J, 1, err)) return;
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

        if (trc) trc[2] = global_ns();
        // the tile to shared memory (As: rows x columns); the triangular work runs on it warp by warp
        const bool pivot_region = I < kb || J < kb;
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) As[(tr + 16 * i) * TLD + tc + 16 * j] = acc[i][j];
        if (pivot_region && I != J) {
            // a panel tile: stage the factored diagonal tile of its pivot block in Bs
            const int d = I > J ? J : I;
            if (!cta_wait_geq(fl + d * nbt + d, 1, err)) return;
            const int d0 = d * TB, b = min(TB, nn - d0);
            for (int e = tid; e < TB * TB; e += blockDim.x) {
                const int r = e % TB, c = e / TB;
                Bs[r * TLD + c] = (r < b && c < b) ? ld_cg(F + (d0 + r) + (int64_t)(d0 + c) * nj) : z;
            }
        }
        __syncthreads();
        if (pivot_region) {
            if (I == J)
                tile_lu_reg<SR, T>(As, mi, s_luc, s_lur);
            else if (I > J)
                tile_solve_right<SR, T>(As, Bs, mj);
            else
                tile_solve_left<SR, T>(As, Bs, mi);
            __syncthreads();
        }

        // store the tile (and its factor entries) column by column
        for (int e = tid; e < TB * TB; e += blockDim.x) {
            const int r = e % TB, c = e / TB;
            if (r < mi && c < mj) {
                const T v = As[r * TLD + c];
                F[(i0 + r) + (int64_t)(j0 + c) * nj] = v;
                if (pivot_region) store_entry<T>(v, i0 + r, j0 + c, nn, na, Dp, Lp, LD, LL, UD, UL);
            }
        }
        __syncthreads();
        if (tid == 0) {
            __threadfence();
            atomicExch(fl + I * nbt + J, 1);
            if (!pivot_region) atomicAdd(fl + nbt * nbt, 1);
            if (trc) {
                trc[3] = global_ns();
                trc[4] = ((unsigned long long)smid() << 32) | (unsigned)f;
                trc[5] = ((unsigned long long)(unsigned)I << 32) | (unsigned)J;
            }
        }
    }
}

}  // namespace pp
