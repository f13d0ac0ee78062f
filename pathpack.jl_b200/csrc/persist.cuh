// persist.cuh — dependency-driven kernels for the bottom of the elimination tree.
//
// The bottom of the tree (the fronts whose whole subtree is small) is processed by ONE persistent launch per
// sweep instead of one launch per tree level: CTAs take fronts from a work list ordered by height (children
// before parents, so every front a CTA waits for was taken earlier by a running CTA and the lowest unfinished
// front can always proceed), wait for a per-front counter, process the front and signal its parent.  The
// reference level-schedules the same work (ext/PATHPACKCUDAExt/chordal/sgetrf.jl:324-343, batched/sweep.jl:9-21)
// with a launch per level.
//
// Every wait is bounded: after the handle's wait timeout the kernel records the failure in *err and returns,
// and the host reports PP_ETIMEOUT.  Data written by other CTAs during the same launch is read through L2
// (ld.global.cg) and published with __threadfence() before the counter update.
#pragma once

#include "engine.cuh"

namespace pp {

// polls of a wait on another warp of the same CTA (shared memory; that warp always progresses)
constexpr long long WAIT_LIMIT = 20000000;
// default bound of a wait on another CTA's progress, in nanoseconds (pp_options.wait_timeout_us overrides it)
constexpr unsigned long long WAIT_NS_DEFAULT = 2000000000ull;

// The error area of a handle: err[0] the error word, err[2..3] the bound of the waits on other CTAs in
// nanoseconds (0: WAIT_NS_DEFAULT).  A wait reads the bound once, then checks the global timer every 16 polls.
struct WaitBound {
    unsigned long long t0, lim;
    unsigned it = 0;
    __device__ __forceinline__ explicit WaitBound(const int *err) {
        const unsigned long long l = *(volatile const unsigned long long *)(err + 2);
        lim = l ? l : WAIT_NS_DEFAULT;
        t0 = now();
    }
    static __device__ __forceinline__ unsigned long long now() {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        return t;
    }
    __device__ __forceinline__ bool expired() { return (++it & 15) == 0 && now() - t0 > lim; }
};

// thread 0 of the CTA polls *p until it satisfies the predicate (or the limit expires); broadcast result
__device__ __forceinline__ bool cta_wait(const int *p, bool for_zero, int *err) {
    __shared__ int s_ok;
    if (threadIdx.x == 0) {
        WaitBound wb(err);
        int ok = 1;
        while (true) {
            const int v = *(volatile const int *)p;
            if (for_zero ? (v == 0) : (v != 0)) break;
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
        __threadfence();
        s_ok = ok;
    }
    __syncthreads();
    const bool res = s_ok != 0;
    __syncthreads();  // s_ok is reused by the next wait
    return res;
}

__device__ __forceinline__ int cta_take(int *next) {
    __shared__ int s_task;
    if (threadIdx.x == 0) s_task = atomicAdd(next, 1);
    __syncthreads();
    const int t = s_task;
    __syncthreads();
    return t;
}

// ---------------------------------------------------------------- factorization of the bottom fronts

// thread 0 polls the front's counter of unfinished children until it is 0, then claims the front (0 -> -1);
// -1 means another CTA claimed it.  Returns 1 (claimed here), 0 (claimed elsewhere) or -1 (a bounded wait
// expired, or another CTA reported an error).
__device__ __forceinline__ int cta_claim(int *p, int *err) {
    __shared__ int s_r;
    if (threadIdx.x == 0) {
        WaitBound wb(err);
        int r;
        while (true) {
            const int v = *(volatile const int *)p;
            if (v == -1) {
                r = 0;
                break;
            }
            if (v == 0) {
                r = atomicCAS(p, 0, -1) == 0 ? 1 : 0;
                break;
            }
            if (*(volatile const int *)err) {
                r = -1;
                break;
            }
            if (wb.expired()) {
                atomicExch(err, 1);
                r = -1;
                break;
            }
            __nanosleep(64);
        }
        __threadfence();
        s_r = r;
    }
    __syncthreads();
    const int r = s_r;
    __syncthreads();  // s_r is reused by the next claim
    return r;
}

// The bottom fronts in work-list order, a CTA each.  The CTA that finishes the last child of a bottom front
// claims that parent and factors it at once (no queue, no wait); a CTA that takes a front from the list waits
// for its children and factors it unless such a CTA claimed it first.  Every front is claimed exactly once
// (the counter goes 0 -> -1 by compare-and-swap).
template <int SR, typename T>
__global__ void __launch_bounds__(FB_THREADS) factor_bottom_kernel(const int *__restrict__ wl, int count, DevPlan P, T *LD,
                                                            T *LL, T *UD, T *UL, T *W, int *pending, int *next,
                                                            int *err) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T *F = reinterpret_cast<T *>(smem_raw);
    __shared__ int s_next;
    int f = -1;
    while (true) {
        if (f < 0) {
            const int t = cta_take(next);
            if (t >= count) return;
            const int g = wl[t];
            const int r = cta_claim(pending + g, err);
            if (r < 0) return;
            if (r == 0) continue;
            f = g;
        }
        front_body<SR, T, true>(f, P, F, LD, LL, UD, UL, W);
        __syncthreads();
        if (threadIdx.x == 0) {
            __threadfence();
            const int p = P.pnt[f];
            int nx = -1;
            // a bottom parent (fws < 0) whose last child this was: claim it
            if (p >= 0 && atomicSub(pending + p, 1) == 1 && P.fws[p] < 0 && atomicCAS(pending + p, 0, -1) == 0) {
                __threadfence();
                nx = p;
            }
            s_next = nx;
        }
        __syncthreads();
        f = s_next;
        __syncthreads();  // s_next is rewritten after the next front
    }
}

// ---------------------------------------------------------------- sweeps of the bottom fronts
//
// A CTA per front, warp w handles the 32-column tiles w, w + 8, ...; lane = right-hand side.  The front's
// residual (nn <= SWEEP_NNW) lives in registers, so the triangular solve needs no barrier.  Element reads of
// the factor blocks are warp-uniform (broadcast).  FWD: wait for the children (counter), solve, (+)-scatter
// to the separator with atomics, signal the parent.  Backward: wait for the parent's flag, gather from the
// separator, solve, set the front's flag.  Same per-element dataflow as sweep_top_kernel.

// one element (4 or 8 bytes) copied into shared memory asynchronously (cp.async); cp_async_wait_all waits for
// this thread's copies
template <typename T>
__device__ __forceinline__ void cp_async_elem(T *dst, const T *src) {
    static_assert(sizeof(T) == 4 || sizeof(T) == 8, "element copies of 4 or 8 bytes");
    const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
    if constexpr (sizeof(T) == 8)
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(d), "l"(src) : "memory");
    else
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// 16 bytes (both addresses 16-byte aligned), bypassing L1
__device__ __forceinline__ void cp_async_16(void *dst, const void *src) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}

// A warp copies `rows` rows of RS elements (columns cw0 .. cw0 + RS - 1 of X, rows row(s)) into shared memory at
// xw + s * RS, as 16-byte chunks (or zero-fills them when zero): the columns of a chunk are contiguous in both.
// Columns at or past k are zero-filled.  The data are visible to the warp after cp_async_wait_all + __syncwarp.
template <typename T, int RS, typename RowOf>
__device__ __forceinline__ void warp_stage_rows(T *xw, const T *X, int64_t ldx, int cw0, int k, int rows, RowOf row,
                                                bool zero, T z) {
    constexpr int NV = 16 / (int)sizeof(T), NCH = RS / NV;
    const int lane = threadIdx.x & 31;
    for (int e = lane; e < rows * NCH; e += 32) {
        const int s = e / NCH, ch = e - s * NCH, col = cw0 + ch * NV;
        T *dst = xw + s * RS + ch * NV;
        if (!zero && col + NV <= k) {
            cp_async_16(dst, X + (int64_t)row(s) * ldx + col);
        } else {
            const T *src = X + (int64_t)row(s) * ldx + col;
#pragma unroll
            for (int u = 0; u < NV; u++) {
                if (!zero && col + u < k)
                    cp_async_elem(dst + u, src + u);
                else
                    dst[u] = z;
            }
        }
    }
}

// shared memory of one warp of sweep_bottom_kernel: a front's factor blocks (D, then the off-diagonal block)
// and its separator positions
template <typename T>
__host__ __device__ constexpr size_t bottom_warp_bytes(int fmax, int namax) {
    return (sizeof(T) * (size_t)fmax + sizeof(int) * (size_t)namax + 15) & ~(size_t)15;
}

// One (front, tile of 32 C columns) task of the bottom sweeps, a lane holding the C columns lane + 32 j: the
// residual values (nn <= NMAX) in registers, the factor blocks and separator positions copied into the warp's
// shared memory (cp.async, all in flight at once), the separator values of the backward sweep loaded eight at
// a time ahead of their use.  Each factor value read from shared memory serves C (x)(+) pairs.
template <int SR, typename T, bool FWD, bool TRANS, int NMAX, int C>
__device__ __forceinline__ void warp_front_tile(int f, int tile, const DevPlan &P, const T *__restrict__ Dv,
                                                const T *__restrict__ Ov, T *X, int64_t ldx, int k, int unit,
                                                T *fb, int *sb) {
    using S = Sem<SR, T>;
    const int lane = threadIdx.x & 31;
    const int col0 = tile * 32 * C + lane;
    bool ok[C];
#pragma unroll
    for (int j = 0; j < C; j++) ok[j] = col0 + 32 * j < k;
    const int rlo = P.rlo[f], nn = P.nn[f], na = P.na[f];
    const T *D = Dv + P.dptr[f];
    const T *O = Ov + P.lptr[f];
    const int *sep = P.stgt + P.sptr[f];
    T *Xc = X + (ok[0] ? col0 : 0);  // column j of the lane at Xc + 32 j (read and written only when ok[j])
    const T z = S::zero();
    const bool scale = !unit && !S::integral;
    const int drs = TRANS ? nn : 1, dcs = TRANS ? 1 : nn;  // Te(r, c) = D[r * drs + c * dcs]
    T x[NMAX][C];
#pragma unroll
    for (int p = 0; p < NMAX; p++)
#pragma unroll
        for (int j = 0; j < C; j++) x[p][j] = (p < nn && ok[j]) ? ld_cg(Xc + (int64_t)(rlo + p) * ldx + 32 * j) : z;
    if (FWD && zero_absorbs<SR>) {
        // the right-hand sides are zero on the whole residual: the step changes nothing
        bool nz = false;
#pragma unroll
        for (int p = 0; p < NMAX; p++)
#pragma unroll
            for (int j = 0; j < C; j++) nz |= !(x[p][j] == z);
        if (!__any_sync(0xffffffffu, nz)) return;
    }
    for (int e = lane; e < nn * nn; e += 32) cp_async_elem(fb + e, D + e);
    for (int e = lane; e < nn * na; e += 32) cp_async_elem(fb + nn * nn + e, O + e);
    for (int e = lane; e < na; e += 32) cp_async_elem(sb + e, sep + e);
    cp_async_wait_all();
    __syncwarp();
    const T *Ds = fb, *Os = fb + nn * nn;
    if (FWD) {
        const int ors = TRANS ? nn : 1, ocs = TRANS ? 1 : na;  // O(i, p) = O[i * ors + p * ocs]
#pragma unroll
        for (int p = 0; p < NMAX; p++) {
            if (p < nn) {
                if (scale) {
                    const T s = S::star(Ds[p * (drs + dcs)]);
#pragma unroll
                    for (int j = 0; j < C; j++) x[p][j] = S::mul(x[p][j], s);
                }
#pragma unroll
                for (int q = p + 1; q < NMAX; q++)
                    if (q < nn) {
                        const T d = Ds[q * drs + p * dcs];
#pragma unroll
                        for (int j = 0; j < C; j++) x[q][j] = S::muladd(d, x[p][j], x[q][j]);
                    }
            }
        }
#pragma unroll
        for (int p = 0; p < NMAX; p++)
            if (p < nn)
#pragma unroll
                for (int j = 0; j < C; j++)
                    if (ok[j]) __stcg(Xc + (int64_t)(rlo + p) * ldx + 32 * j, x[p][j]);
        for (int i = 0; i < na; i++) {
            T a[C];
#pragma unroll
            for (int j = 0; j < C; j++) a[j] = z;
#pragma unroll
            for (int p = 0; p < NMAX; p++)
                if (p < nn) {
                    const T o = Os[i * ors + p * ocs];
#pragma unroll
                    for (int j = 0; j < C; j++) a[j] = S::muladd(o, x[p][j], a[j]);
                }
            T *xr = Xc + (int64_t)sb[i] * ldx;
#pragma unroll
            for (int j = 0; j < C; j++)
                if (ok[j] && !(a[j] == z)) S::atomic_add(xr + 32 * j, a[j]);  // (+) zero changes nothing
        }
    } else {
        const int ors = TRANS ? na : 1, ocs = TRANS ? 1 : nn;  // O(p, i) = O[p * ors + i * ocs]
        for (int i0 = 0; i0 < na; i0 += 8) {
            T xv[8][C];
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const T *xr = Xc + (int64_t)sb[min(i0 + u, na - 1)] * ldx;
#pragma unroll
                for (int j = 0; j < C; j++) xv[u][j] = (i0 + u < na && ok[j]) ? ld_cg(xr + 32 * j) : z;
            }
#pragma unroll
            for (int u = 0; u < 8; u++) {
                if (i0 + u < na) {
#pragma unroll
                    for (int p = 0; p < NMAX; p++)
                        if (p < nn) {
                            const T o = Os[p * ors + (i0 + u) * ocs];
#pragma unroll
                            for (int j = 0; j < C; j++) x[p][j] = S::muladd(o, xv[u][j], x[p][j]);
                        }
                }
            }
        }
#pragma unroll
        for (int p = NMAX - 1; p >= 0; p--) {
            if (p >= nn) continue;
            if (scale) {
                const T s = S::star(Ds[p * (drs + dcs)]);
#pragma unroll
                for (int j = 0; j < C; j++) x[p][j] = S::mul(s, x[p][j]);
            }
#pragma unroll
            for (int q = 0; q < p; q++) {
                const T d = Ds[q * drs + p * dcs];
#pragma unroll
                for (int j = 0; j < C; j++) x[q][j] = S::muladd(d, x[p][j], x[q][j]);
            }
        }
#pragma unroll
        for (int p = 0; p < NMAX; p++)
            if (p < nn)
#pragma unroll
                for (int j = 0; j < C; j++)
                    if (ok[j]) __stcg(Xc + (int64_t)(rlo + p) * ldx + 32 * j, x[p][j]);
    }
    __syncwarp();  // the buffers are reused by the warp's next task
}

// lane 0 of the warp polls *p until it satisfies the predicate (or the limit expires); broadcast result
__device__ __forceinline__ bool warp_wait(const int *p, bool for_zero, int *err) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0) {
        WaitBound wb(err);
        while (true) {
            const int v = *(volatile const int *)p;
            if (for_zero ? (v == 0) : (v != 0)) break;
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
        __threadfence();
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    __syncwarp();
    return ok != 0;
}

// Warp tasks (front, tile of 32 C columns), in work-list order with the tiles innermost; flags holds one counter
// (forward: children not yet done) or flag (backward: done) per (tile, front): flags[tile * nf + f].  A warp
// that finishes a front continues along the tree without a wait: forward with the parent, when its decrement
// of the parent's counter was the last one and the parent is swept by this launch; backward with the front's
// heavy child (the child with the costliest chain of bottom fronts below it).  The list's entries that a
// continuation reaches are skipped.  sinfo[f] of a bottom front: (segment << 3) | (heavy child of a bottom front
// << 2) | (has a bottom child of the late part of its stage << 1) | (has one of the early part); the segment is
// 2 * stage + part, part 0 for the fronts the bottom factorization kernel holds in stage 0 (swept while the
// top is factored), else 1.  The launch sweeps the segments seg_lo .. seg_hi.
__device__ __forceinline__ bool in_segs(int seg, int lo, int hi) { return seg >= lo && seg <= hi; }

template <int SR, typename T, bool FWD, bool TRANS, int C>
__global__ void __launch_bounds__(256) sweep_bottom_kernel(const int *__restrict__ wl, int count, DevPlan P,
                                                           const T *__restrict__ Dv, const T *__restrict__ Ov,
                                                           T *X, int64_t ldx, int k, int unit, int *flags,
                                                           int *next, int *err, int fmax, int namax,
                                                           const int *__restrict__ sinfo,
                                                           const int *__restrict__ heavy, int seg_lo, int seg_hi) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    unsigned char *mine = smem_raw + (size_t)(threadIdx.x >> 5) * bottom_warp_bytes<T>(fmax, namax);
    T *fb = reinterpret_cast<T *>(mine);
    int *sb = reinterpret_cast<int *>(fb + fmax);
    const int ntiles = (k + 32 * C - 1) / (32 * C);
    const int lane = threadIdx.x & 31;
    const int nf = P.nf;
    const int64_t ntask = (int64_t)count * ntiles;
    while (true) {
        int t = 0;
        if (lane == 0) t = atomicAdd(next, 1);
        t = __shfl_sync(0xffffffffu, t, 0);
        if (t >= ntask) return;
        const int idx = t / ntiles, tile = t - idx * ntiles;
        int f = wl[idx];
        int *fl = flags + (int64_t)tile * nf;
        {
            const int si = sinfo[f], seg = si >> 3;
            if (FWD) {
                // reached by the last of its children in this launch
                const bool early = (si & 1) && in_segs(seg & ~1, seg_lo, seg_hi);
                const bool late = (si & 2) && in_segs(seg | 1, seg_lo, seg_hi);
                if (early || late) continue;
                if (!warp_wait(fl + f, true, err)) return;  // its children ran in earlier launches
            } else {
                if (si & 4) continue;  // reached from its parent
                const int p = P.pnt[f];
                if (p >= 0 && !warp_wait(fl + p, false, err)) return;
            }
        }
        while (true) {
            const int nn = P.nn[f];
            if (nn <= 2)
                warp_front_tile<SR, T, FWD, TRANS, 2, C>(f, tile, P, Dv, Ov, X, ldx, k, unit, fb, sb);
            else if (nn <= 4)
                warp_front_tile<SR, T, FWD, TRANS, 4, C>(f, tile, P, Dv, Ov, X, ldx, k, unit, fb, sb);
            else if (nn <= 8)
                warp_front_tile<SR, T, FWD, TRANS, 8, C>(f, tile, P, Dv, Ov, X, ldx, k, unit, fb, sb);
            else
                warp_front_tile<SR, T, FWD, TRANS, SWEEP_NNW, C>(f, tile, P, Dv, Ov, X, ldx, k, unit, fb, sb);
            __syncwarp();
            int nxt = -1;
            if (lane == 0) {
                __threadfence();
                if (FWD) {
                    const int p = P.pnt[f];
                    if (p >= 0 && atomicSub(fl + p, 1) == 1) {
                        const int sp = sinfo[p];
                        if (sp >= 0 && in_segs(sp >> 3, seg_lo, seg_hi)) nxt = p;
                    }
                    if (nxt >= 0) __threadfence();  // the other children's updates of the parent's rows
                } else {
                    atomicExch(fl + f, 1);
                    nxt = heavy[f];
                }
            }
            nxt = __shfl_sync(0xffffffffu, nxt, 0);
            __syncwarp();
            if (nxt < 0) break;
            f = nxt;
        }
    }
}

// ---------------------------------------------------------------- subtrees of the bottom in shared memory
//
// A subtree rooted at r touches only its residual rows, the contiguous positions rlo(fd(r)) .. rhi(r), and the
// separator of r (the running-intersection property of the clique tree: a separator vertex of a front in the
// subtree is either in the subtree or in sep(r)).  A CTA task (subtree, 128-column group) stages everything the
// subtree's fronts read in shared memory once: their descriptors (sizes, first row, offsets of their blocks),
// the separator slots (slot[Sptr[g] + i] is the subtree row of the i-th separator vertex of front g) and the
// factor blocks D (nn x nn) and O (nn x na), which are contiguous ranges of the factor arrays because the
// subtree's fronts are contiguous in postorder.  Each warp then loads its columns' rows of the subtree, runs
// every front in postorder (forward) or reverse postorder (backward) from shared memory, and writes back
// once; the forward sweep (+)-scatters the accumulated separator rows with atomics.  A lane holds C columns,
// and touches only its own columns' rows, so the front loop needs no barrier.  The host admits a subtree only
// when its rows, slots and factor blocks fit the staging areas (SUBTREE_ROWS, SUBTREE_SLOTS, SUBTREE_FAC).

// warps per CTA of the subtree sweep; a lane holds C columns (1, or 2 for wide solves), so a CTA covers 128 C
constexpr int SUBTREE_WARPS = 4;

// shared memory of sweep_subtree_kernel: per warp the subtree's rows for its 32 * C columns, then the staged
// factor blocks, slots and front descriptors (int4 {nn, na, first row - subtree's first row, slot offset},
// int2 {offset of D, offset of O} in the staged factor area)
template <typename T, int C>
__host__ __device__ constexpr size_t subtree_cta_bytes() {
    return sizeof(T) * ((size_t)SUBTREE_WARPS * SUBTREE_ROWS * 32 * C + SUBTREE_FAC) +
           sizeof(int) * SUBTREE_SLOTS + (sizeof(int4) + sizeof(int2)) * SUBTREE_ROWS;
}

// One front of a subtree for this lane's C right-hand sides: its nn <= NMAX residual values in registers (the
// loops are unrolled to NMAX and guarded by nn), the factor blocks D and O and the slots sl in shared memory,
// the subtree's rows in xs (row s, column j of the lane at xs[s * 32C + 32j]).  Per element the same
// operations in the same order as warp_front_tile.
template <int SR, typename T, bool FWD, bool TRANS, int NMAX, int C>
__device__ __forceinline__ void subtree_front(int nn, int na, T *xg, T *xs, const T *D, const T *O, const int *sl,
                                              bool scale) {
    using S = Sem<SR, T>;
    constexpr int RS = 32 * C;  // row stride of xs
    const T z = S::zero();
    const int drs = TRANS ? nn : 1, dcs = TRANS ? 1 : nn;  // Te(r, c) = D[r * drs + c * dcs]
    T x[NMAX][C];
#pragma unroll
    for (int p = 0; p < NMAX; p++)
#pragma unroll
        for (int j = 0; j < C; j++) x[p][j] = p < nn ? xg[p * RS + 32 * j] : z;
    if (FWD) {
        const int ors = TRANS ? nn : 1, ocs = TRANS ? 1 : na;  // O(i, p) = O[i * ors + p * ocs]
#pragma unroll
        for (int p = 0; p < NMAX; p++) {
            if (p >= nn) break;
            if (scale) {
                const T s = S::star(D[p * (drs + dcs)]);
#pragma unroll
                for (int j = 0; j < C; j++) x[p][j] = S::mul(x[p][j], s);
            }
#pragma unroll
            for (int q = p + 1; q < NMAX; q++)
                if (q < nn) {
                    const T d = D[q * drs + p * dcs];
#pragma unroll
                    for (int j = 0; j < C; j++) x[q][j] = S::muladd(d, x[p][j], x[q][j]);
                }
        }
        for (int i = 0; i < na; i++) {
            T a[C];
#pragma unroll
            for (int j = 0; j < C; j++) a[j] = z;
#pragma unroll
            for (int p = 0; p < NMAX; p++)
                if (p < nn) {
                    const T o = O[i * ors + p * ocs];
#pragma unroll
                    for (int j = 0; j < C; j++) a[j] = S::muladd(o, x[p][j], a[j]);
                }
            T *c = xs + sl[i] * RS;
#pragma unroll
            for (int j = 0; j < C; j++) c[32 * j] = S::add(c[32 * j], a[j]);
        }
    } else {
        const int ors = TRANS ? na : 1, ocs = TRANS ? 1 : nn;  // O(p, i) = O[p * ors + i * ocs]
        // four separator rows per step, their slots and values loaded together; per element the terms in
        // increasing i
        int i = 0;
        for (; i + 4 <= na; i += 4) {
            T xi[4][C];
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const T *c = xs + sl[i + q] * RS;
#pragma unroll
                for (int j = 0; j < C; j++) xi[q][j] = c[32 * j];
            }
#pragma unroll
            for (int p = 0; p < NMAX; p++)
                if (p < nn) {
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        const T o = O[p * ors + (i + q) * ocs];
#pragma unroll
                        for (int j = 0; j < C; j++) x[p][j] = S::muladd(o, xi[q][j], x[p][j]);
                    }
                }
        }
        for (; i < na; i++) {
            const T *c = xs + sl[i] * RS;
            T xi[C];
#pragma unroll
            for (int j = 0; j < C; j++) xi[j] = c[32 * j];
#pragma unroll
            for (int p = 0; p < NMAX; p++)
                if (p < nn) {
                    const T o = O[p * ors + i * ocs];
#pragma unroll
                    for (int j = 0; j < C; j++) x[p][j] = S::muladd(o, xi[j], x[p][j]);
                }
        }
#pragma unroll
        for (int p = NMAX - 1; p >= 0; p--) {
            if (p >= nn) continue;
            if (scale) {
                const T s = S::star(D[p * (drs + dcs)]);
#pragma unroll
                for (int j = 0; j < C; j++) x[p][j] = S::mul(s, x[p][j]);
            }
#pragma unroll
            for (int q = 0; q < p; q++) {
                const T d = D[q * drs + p * dcs];
#pragma unroll
                for (int j = 0; j < C; j++) x[q][j] = S::muladd(d, x[p][j], x[q][j]);
            }
        }
    }
#pragma unroll
    for (int p = 0; p < NMAX; p++)
        if (p < nn)
#pragma unroll
            for (int j = 0; j < C; j++) xg[p * RS + 32 * j] = x[p][j];
}

template <int SR, typename T, bool FWD, bool TRANS, int C>
__global__ void __launch_bounds__(128) sweep_subtree_kernel(const int *__restrict__ roots, int nroots, DevPlan P,
                                                            const int *__restrict__ fdsc, const int *__restrict__ slot,
                                                            const T *__restrict__ Dv, const T *__restrict__ Ov, T *X,
                                                            int64_t ldx, int k, int unit, int *err) {
    using S = Sem<SR, T>;
    constexpr int RS = 32 * C, CW = SUBTREE_WARPS * RS;  // columns per CTA
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T *xs_all = reinterpret_cast<T *>(smem_raw);
    T *fac = xs_all + (size_t)SUBTREE_WARPS * SUBTREE_ROWS * RS;
    int *sls = reinterpret_cast<int *>(fac + SUBTREE_FAC);
    int4 *desc = reinterpret_cast<int4 *>(sls + SUBTREE_SLOTS);
    int2 *desc2 = reinterpret_cast<int2 *>(desc + SUBTREE_ROWS);
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int ngrp = (k + CW - 1) / CW;
    const int sidx = blockIdx.x / ngrp, grp = blockIdx.x % ngrp;
    if (sidx >= nroots) return;
    const int r = roots[sidx];
    const int f0 = fdsc[r], ng = r - f0 + 1;
    const int rlo0 = P.rlo[f0];
    const int nres = P.rlo[r] + P.nn[r] - rlo0;
    const int nsep = P.na[r];
    const int64_t dbase = P.dptr[f0], lbase = P.lptr[f0], sbase = P.sptr[f0];
    const int dlen = (int)(P.dptr[r + 1] - dbase), llen = (int)(P.lptr[r + 1] - lbase);
    const int slen = (int)(P.sptr[r + 1] - sbase);
    if (ng > SUBTREE_ROWS || nres + nsep > SUBTREE_ROWS || dlen + llen > SUBTREE_FAC || slen > SUBTREE_SLOTS) {
        if (tid == 0) atomicExch(err, 1);  // the host admitted a subtree that does not fit (uniform)
        return;
    }
    // this warp's columns c0 + 32j of the subtree's rows, copied asynchronously (all in flight at once);
    // forward, the separator rows start at zero
    const int cw0 = grp * CW + w * RS, c0 = cw0 + lane;
    T *const xw = xs_all + (size_t)w * SUBTREE_ROWS * RS;  // this warp's rows
    T *xs = xw + lane;                                     // this lane's column 0 of them
    const T z = S::zero();
    bool ok[C];
#pragma unroll
    for (int j = 0; j < C; j++) ok[j] = c0 + 32 * j < k;
    const int *sepr = P.stgt + P.sptr[r];
    // the subtree's rows as 16-byte chunks; forward, the separator rows start at zero
    warp_stage_rows<T, RS>(xw, X, ldx, cw0, k, nres, [&](int s) { return rlo0 + s; }, false, z);
    warp_stage_rows<T, RS>(xw + nres * RS, X, ldx, cw0, k, nsep, [&](int i) { return sepr[i]; }, FWD, z);
    bool nz = false;
    if (FWD && zero_absorbs<SR>) {
        // forward: the right-hand sides that are zero on the subtree's rows change nothing (the sources of
        // these columns lie outside the subtree); a CTA whose columns all are leaves before staging anything
        cp_async_wait_all();
        __syncwarp();
        for (int s = 0; s < nres; s++)
#pragma unroll
            for (int j = 0; j < C; j++) nz |= !(xs[s * RS + 32 * j] == z);
        if (!__syncthreads_or(nz)) return;
    }
    // stage the subtree's factor blocks, slots and front descriptors
    for (int e = tid; e < dlen; e += blockDim.x) cp_async_elem(fac + e, Dv + dbase + e);
    for (int e = tid; e < llen; e += blockDim.x) cp_async_elem(fac + dlen + e, Ov + lbase + e);
    for (int e = tid; e < slen; e += blockDim.x) cp_async_elem(sls + e, slot + sbase + e);
    for (int g = tid; g < ng; g += blockDim.x) {
        const int f = f0 + g;
        desc[g] = make_int4(P.nn[f], P.na[f], P.rlo[f] - rlo0, (int)(P.sptr[f] - sbase));
        desc2[g] = make_int2((int)(P.dptr[f] - dbase), dlen + (int)(P.lptr[f] - lbase));
    }
    cp_async_wait_all();
    __syncthreads();  // the staged blocks (the last barrier: warps leave independently from here)
    if (!__any_sync(0xffffffffu, ok[0])) return;
    if (FWD && zero_absorbs<SR> && !__any_sync(0xffffffffu, nz)) return;
    const bool scale = !unit && !S::integral;
    for (int gi = 0; gi < ng; gi++) {
        const int g = FWD ? gi : ng - 1 - gi;
        const int4 d = desc[g];
        const int2 o = desc2[g];
        const int nn = d.x, na = d.y;
        T *xg = xs + d.z * RS;
        const T *D = fac + o.x, *O = fac + o.y;
        const int *sl = sls + d.w;
        if (nn == 1)
            subtree_front<SR, T, FWD, TRANS, 1, C>(nn, na, xg, xs, D, O, sl, scale);
        else if (nn == 2)
            subtree_front<SR, T, FWD, TRANS, 2, C>(nn, na, xg, xs, D, O, sl, scale);
        else if (nn <= 4)
            subtree_front<SR, T, FWD, TRANS, 4, C>(nn, na, xg, xs, D, O, sl, scale);
        else if (nn <= 8)
            subtree_front<SR, T, FWD, TRANS, 8, C>(nn, na, xg, xs, D, O, sl, scale);
        else
            subtree_front<SR, T, FWD, TRANS, SWEEP_NNW, C>(nn, na, xg, xs, D, O, sl, scale);
    }
    // the residual rows back, as 16-byte chunks (a lane writes columns other lanes computed)
    __syncwarp();
    {
        constexpr int NV = 16 / (int)sizeof(T), NCH = RS / NV;
        for (int e = lane; e < nres * NCH; e += 32) {
            const int s = e / NCH, ch = e - s * NCH, col = cw0 + ch * NV;
            T *dst = X + (int64_t)(rlo0 + s) * ldx + col;
            const T *src = xw + s * RS + ch * NV;
            if (col + NV <= k) {
                *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(src);
            } else {
                for (int u = 0; u < NV && col + u < k; u++) dst[u] = src[u];
            }
        }
    }
    if (FWD)
        for (int i = 0; i < nsep; i++) {
            T *xr = X + (int64_t)sepr[i] * ldx + c0;
#pragma unroll
            for (int j = 0; j < C; j++) {
                const T v = xs[(nres + i) * RS + 32 * j];
                if (ok[j] && !(v == z)) S::atomic_add(xr + 32 * j, v);  // (+) zero changes nothing
            }
        }
}

// flags[t * nf + f] = init[f] for every tile t
static __global__ void init_flags_kernel(int *flags, const int *init, int nf, int ntiles) {
    const int64_t tot = (int64_t)nf * ntiles;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < tot; i += (int64_t)gridDim.x * blockDim.x)
        flags[i] = init[i % nf];
}

}  // namespace pp
