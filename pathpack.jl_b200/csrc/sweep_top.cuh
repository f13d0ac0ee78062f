// sweep_top.cuh — the triangular solves of the fronts above the bottom of the tree: ONE persistent launch per
// sweep direction and coupling stage.
//
// Tasks are (front, block of 64 rows, 32 right-hand sides), the fronts schedule-ordered (children first for the
// forward sweep, parents first for the backward one) and a front's blocks in solve order, so every task waits
// only for tasks taken earlier: forward for a counter of its top children (the last separator task of a child
// decrements it) and for the residual blocks before it, backward for its parent's flag and for the residual
// blocks after it.  A residual-block task solves its 64 rows, applying the blocks it depends on one at a time
// as they are published (so a large front's blocks proceed on several SMs at once); forward, separator-block
// tasks then (+)-scatter their 64 rows of L21 x with atomics; backward, each block starts with the gather from
// the separator rows.  The off-diagonal products
// are register-tiled (2 rows x 4 right-hand sides per thread) over operand chunks staged in shared memory,
// double-buffered; the 64 x 64 diagonal block is solved warp by warp (a warp holds 4 right-hand sides, a lane
// 8 rows of one of them) with the pivot values broadcast by shuffles, so the solve needs no CTA barrier.  Per
// element the operands and their order are those of the reference's strsx2! / sgemx2!
// (src/CPU/dense/strsx.jl:596-672, src/CPU/chordal/strsx.jl:187-265, 783-830): forward, contributions in
// increasing pivot order; backward, the separator first, then decreasing pivot order.  The reference sweeps
// the same fronts level by level, a launch per level (ext/PATHPACKCUDAExt/batched/sweep.jl:9-265).
#pragma once

#include "persist.cuh"

namespace pp {

constexpr int SW_RB = TOP_SWEEP_ROWS;   // rows per block task
constexpr int SW_CT = 32;   // right-hand sides per task
constexpr int SW_KC = 16;   // operand chunk
constexpr int SW_AL = SW_KC + 1;  // padded row of the staged matrix chunk
constexpr int SW_XL = SW_CT + 1;  // padded row of the staged right-hand-side chunk
constexpr int SW_DL = SW_RB + 1;  // padded row of the diagonal block

template <typename T>
constexpr size_t sweep_top_smem() {
    return sizeof(T) * (2 * (size_t)SW_RB * SW_AL + 2 * (size_t)SW_KC * SW_XL + (size_t)SW_RB * SW_DL +
                        (size_t)SW_RB * SW_XL);
}

// thread 0 polls until the low 16 bits of a front's block counter reach target (bounded); every thread gets
// the counter's value, or -1 when the wait failed.  Bit 16 and up: the forward sweep found the front's
// right-hand sides all zero.
__device__ __forceinline__ int cta_wait_blocks(const int *p, int target, int *err) {
    __shared__ int s_v;
    if (threadIdx.x == 0) {
        WaitBound wb(err);
        int v;
        while (true) {
            v = *(volatile const int *)p;
            if ((v & 0xffff) >= target) break;
            if (*(volatile const int *)err) {
                v = -1;
                break;
            }
            if (wb.expired()) {
                atomicExch(err, 1);
                v = -1;
                break;
            }
            __nanosleep(64);
        }
        __threadfence();
        s_v = v;
    }
    __syncthreads();
    const int v = s_v;
    __syncthreads();  // s_v is reused by the next wait
    return v;
}

// flags: [tile * nf + f] the forward counters of top children / backward done flags, then per (tile, front) the
// residual blocks done and (forward) the separator tasks done.  wl[i] = (front, block).
template <int SR, typename T, bool FWD, bool TRANS>
__global__ void __launch_bounds__(256) sweep_top_kernel(const int2 *__restrict__ wl, int count, DevPlan P,
                                                        const T *__restrict__ Dv, const T *__restrict__ Ov, T *X,
                                                        int64_t ldx, int k, int unit, int *flags, int *next,
                                                        int *err) {
    using S = Sem<SR, T>;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T *As = reinterpret_cast<T *>(smem_raw);  // 2 x [SW_RB][SW_AL]: matrix chunks
    T *Xs = As + 2 * SW_RB * SW_AL;            // 2 x [SW_KC][SW_XL]: right-hand-side chunks
    T *Dd = Xs + 2 * SW_KC * SW_XL;            // [SW_RB][SW_DL]: diagonal block
    T *Ys = Dd + SW_RB * SW_DL;                // [SW_RB][SW_XL]: the residual block being solved
    const int tid = threadIdx.x, tc = tid & 7, tr = tid >> 3;
    const int lane = tid & 31, w = tid >> 5, dc = 4 * w + (lane >> 3), dg = lane & 7;
    const int ntiles = (k + SW_CT - 1) / SW_CT, nf = P.nf;
    const int64_t ntask = (int64_t)count * ntiles;
    const T z = S::zero();
    const bool scale = !unit && !S::integral;
    int *const bdone = flags + (int64_t)ntiles * nf, *const sdone = bdone + (int64_t)ntiles * nf;

    while (true) {
        const int t = cta_take(next);
        if (t >= ntask) return;
        const int idx = t / ntiles, tile = t - idx * ntiles;
        const int2 task = wl[idx];
        const int f = task.x, b = task.y;
        int *fl = flags + (int64_t)tile * nf;
        int *bd = bdone + (int64_t)tile * nf + f;
        const int p = P.pnt[f];
        if (FWD) {
            if (!cta_wait(fl + f, true, err)) return;
        } else if (p >= 0) {
            if (!cta_wait(fl + p, false, err)) return;
        }
        const int c0 = tile * SW_CT;
        const int rlo = P.rlo[f], nn = P.nn[f], na = P.na[f];
        const T *D = Dv + P.dptr[f];
        const T *O = Ov + P.lptr[f];
        const int *sep = P.stgt + P.sptr[f];
        auto Te = [&](int r, int c) -> T { return TRANS ? D[c + (int64_t)r * nn] : D[r + (int64_t)c * nn]; };
        auto xres = [&](int q) { return rlo + q; };
        auto xsep = [&](int i) { return sep[i]; };

        T acc[2][4];
        auto load_acc = [&](int rowbase, int nrows, bool from_x) {
#pragma unroll
            for (int i = 0; i < 2; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int r = tr + 32 * i, c = c0 + tc + 8 * j;
                    acc[i][j] = (from_x && r < nrows && c < k) ? ld_cg(X + (int64_t)(rowbase + r) * ldx + c) : z;
                }
        };
        // acc[i][j] (+)= M(rb + row_i, kidx) (x) X[xrow(kidx)][col_j] for kidx in [kb, ke), ascending or
        // descending; chunk ch + 1 is loaded into registers while chunk ch is used
        auto accum = [&](int rb, int nrows, int kb, int ke, bool desc, auto M, auto xrow) {
            const int kn = ke - kb;
            if (kn <= 0) return;
            const int nch = (kn + SW_KC - 1) / SW_KC;
            T ra[4], rx[2];
            auto fetch = [&](int ch) {
                const int kc = min(SW_KC, kn - ch * SW_KC);
                const int cb = desc ? ke - ch * SW_KC - kc : kb + ch * SW_KC;
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    // consecutive threads read consecutive addresses: rows of the stored blocks, or (TRANS) columns
                    const int e = tid + 256 * q;
                    const int r = TRANS ? e / SW_KC : e % SW_RB, kk = TRANS ? e % SW_KC : e / SW_RB;
                    ra[q] = (r < nrows && kk < kc) ? M(rb + r, cb + kk) : z;
                }
#pragma unroll
                for (int q = 0; q < 2; q++) {
                    const int e = tid + 256 * q, kk = e / SW_CT, c = e % SW_CT;
                    rx[q] = (kk < kc && c0 + c < k) ? ld_cg(X + (int64_t)xrow(cb + kk) * ldx + c0 + c) : z;
                }
            };
            auto store = [&](int buf) {
                T *a = As + buf * SW_RB * SW_AL;
                T *x = Xs + buf * SW_KC * SW_XL;
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const int e = tid + 256 * q;
                    const int r = TRANS ? e / SW_KC : e % SW_RB, kk = TRANS ? e % SW_KC : e / SW_RB;
                    a[r * SW_AL + kk] = ra[q];
                }
#pragma unroll
                for (int q = 0; q < 2; q++) {
                    const int e = tid + 256 * q;
                    x[(e / SW_CT) * SW_XL + e % SW_CT] = rx[q];
                }
            };
            fetch(0);
            store(0);
            __syncthreads();
            for (int ch = 0; ch < nch; ch++) {
                if (ch + 1 < nch) fetch(ch + 1);
                const int kc = min(SW_KC, kn - ch * SW_KC);
                const T *a = As + (ch & 1) * SW_RB * SW_AL;
                const T *x = Xs + (ch & 1) * SW_KC * SW_XL;
                for (int u = 0; u < kc; u++) {
                    const int kk = desc ? kc - 1 - u : u;
                    const T a0 = a[tr * SW_AL + kk], a1 = a[(tr + 32) * SW_AL + kk];
                    T b[4];
#pragma unroll
                    for (int j = 0; j < 4; j++) b[j] = x[kk * SW_XL + tc + 8 * j];
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        acc[0][j] = S::muladd(a0, b[j], acc[0][j]);
                        acc[1][j] = S::muladd(a1, b[j], acc[1][j]);
                    }
                }
                if (ch + 1 < nch) store((ch + 1) & 1);
                __syncthreads();
            }
        };

        // the diagonal block of rows r0 .. r0 + nv - 1: acc -> Ys, solved warp by warp, written to X
        auto diag_solve = [&](int r0, int nv) {
#pragma unroll
            for (int i = 0; i < 2; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) Ys[(tr + 32 * i) * SW_XL + tc + 8 * j] = acc[i][j];
            for (int e = tid; e < SW_RB * SW_RB; e += 256) {
                const int q = TRANS ? e / SW_RB : e % SW_RB, c = TRANS ? e % SW_RB : e / SW_RB;
                Dd[q * SW_DL + c] = (q < nv && c < nv) ? Te(r0 + q, r0 + c) : z;
            }
            __syncthreads();
            // lane (dc, dg) holds rows dg + 8 u of right-hand side dc; pivot 8 u + g lives in lane (dc, g), slot u
            T y[8];
#pragma unroll
            for (int u = 0; u < 8; u++) y[u] = Ys[(dg + 8 * u) * SW_XL + dc];
            const int src = lane & ~7;
            if (FWD) {
#pragma unroll
                for (int u = 0; u < 8; u++)
                    for (int g = 0; g < 8; g++) {
                        const int q = 8 * u + g;
                        if (q >= nv) break;
                        T yq = __shfl_sync(0xffffffffu, y[u], src | g);
                        if (scale) yq = S::mul(yq, S::star(Dd[q * SW_DL + q]));
                        if (dg == g) y[u] = yq;
                        // rows dg + 8 v below pivot 8 u + g: v > u, or v == u and dg > g (u is unrolled, so only
                        // slot u is tested); rows at or past nv hold values that are never pivots or stored
#pragma unroll
                        for (int v = u; v < 8; v++)
                            if (v > u || dg > g) y[v] = S::muladd(Dd[(dg + 8 * v) * SW_DL + q], yq, y[v]);
                    }
            } else {
#pragma unroll
                for (int u = 7; u >= 0; u--)
                    for (int g = 7; g >= 0; g--) {
                        const int q = 8 * u + g;
                        if (q >= nv) continue;
                        T yq = __shfl_sync(0xffffffffu, y[u], src | g);
                        if (scale) yq = S::mul(S::star(Dd[q * SW_DL + q]), yq);
                        if (dg == g) y[u] = yq;
                        // rows dg + 8 v above pivot 8 u + g: v < u, or v == u and dg < g
#pragma unroll
                        for (int v = 0; v <= u; v++)
                            if (v < u || dg < g) y[v] = S::muladd(Dd[(dg + 8 * v) * SW_DL + q], yq, y[v]);
                    }
            }
#pragma unroll
            for (int u = 0; u < 8; u++) Ys[(dg + 8 * u) * SW_XL + dc] = y[u];
            __syncthreads();
            for (int e = tid; e < SW_RB * SW_CT; e += 256) {
                const int r = e / SW_CT, c = e % SW_CT;
                if (r < nv && c0 + c < k) X[(int64_t)(rlo + r0 + r) * ldx + c0 + c] = Ys[r * SW_XL + c];
            }
            __syncthreads();
        };

        const int kb = (nn + SW_RB - 1) / SW_RB, sbk = (na + SW_RB - 1) / SW_RB;
        if (FWD && b < kb) {
            // residual block b: its rows (+)= the solved blocks before it, then the diagonal solve
            const int r0 = b * SW_RB, nv = min(SW_RB, nn - r0);
            bool live = true;
            if (b == 0) {
                if (zero_absorbs<SR>) {
                    // the 32 right-hand sides are zero on the whole residual: the front changes nothing
                    bool nz = false;
                    for (int e = tid; e < nn * SW_CT; e += 256) {
                        const int c = c0 + e % SW_CT;
                        if (c < k) nz |= !(ld_cg(X + (int64_t)(rlo + e / SW_CT) * ldx + c) == z);
                    }
                    live = __syncthreads_or(nz) != 0;
                }
            } else {
                const int v = cta_wait_blocks(bd, 1, err);
                if (v < 0) return;
                live = (v >> 16) == 0;
            }
            if (live) {
                load_acc(rlo + r0, nv, true);
                for (int j = 0; j < b; j++) {
                    if (j > 0 && cta_wait_blocks(bd, j + 1, err) < 0) return;
                    accum(r0, nv, j * SW_RB, (j + 1) * SW_RB, false, Te, xres);
                }
                diag_solve(r0, nv);
            }
            __syncthreads();
            if (tid == 0) {
                __threadfence();
                atomicAdd(bd, (b == 0 && !live) ? 0x10001 : 1);
                if (b == kb - 1 && sbk == 0 && p >= 0) atomicSub(fl + p, 1);
            }
        } else if (FWD) {
            // separator block b - kb: X[sep_i] (+)= (L21 x)_i for its 64 rows, once every residual block is solved
            const int v = cta_wait_blocks(bd, kb, err);
            if (v < 0) return;
            if ((v >> 16) == 0) {
                auto Of = [&](int i, int q) -> T { return TRANS ? O[q + (int64_t)i * nn] : O[i + (int64_t)q * na]; };
                const int i0 = (b - kb) * SW_RB, nv = min(SW_RB, na - i0);
                load_acc(0, 0, false);
                accum(i0, nv, 0, nn, false, Of, xres);
#pragma unroll
                for (int i = 0; i < 2; i++)
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const int r = tr + 32 * i, c = c0 + tc + 8 * j;
                        // (+) with zero changes nothing: zero sums (columns whose sources lie outside the front's
                        // subtree) are not scattered
                        if (r < nv && c < k && !(acc[i][j] == z))
                            S::atomic_add(X + (int64_t)sep[i0 + r] * ldx + c, acc[i][j]);
                    }
            }
            __syncthreads();
            if (tid == 0) {
                __threadfence();
                if (atomicAdd(sdone + (int64_t)tile * nf + f, 1) == sbk - 1 && p >= 0) atomicSub(fl + p, 1);
            }
        } else {
            // residual block b, backward: the gather from the separator, the solved blocks after it (descending),
            // then the diagonal solve
            auto Ob = [&](int r, int i) -> T { return TRANS ? O[i + (int64_t)r * na] : O[r + (int64_t)i * nn]; };
            const int r0 = b * SW_RB, r1 = min(nn, r0 + SW_RB), nv = r1 - r0;
            load_acc(rlo + r0, nv, true);
            accum(r0, nv, 0, na, false, Ob, xsep);
            for (int j = kb - 1; j > b; j--) {
                if (cta_wait_blocks(bd, kb - j, err) < 0) return;
                accum(r0, nv, j * SW_RB, min(nn, (j + 1) * SW_RB), true, Te, xres);
            }
            diag_solve(r0, nv);
            __syncthreads();
            if (tid == 0) {
                __threadfence();
                atomicAdd(bd, 1);
                if (b == 0) atomicExch(fl + f, 1);
            }
        }
    }
}

}  // namespace pp
