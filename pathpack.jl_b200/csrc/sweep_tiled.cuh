// sweep_tiled.cuh — the triangular solves of the fronts above the bottom of the tree, tiled.
//
// A CTA per (front, 64 right-hand sides).  The front's residual rows are processed in blocks of 64 (forward:
// top-down; backward: bottom-up).  Each block first takes its contributions from the rows already final (the
// earlier residual blocks, or the separator and the later blocks) as a register-tiled product: operand chunks
// of 64 x 16 matrix elements and 16 x 64 right-hand-side elements are staged in shared memory and every thread
// accumulates a 4 x 4 tile.  Then the 64 x 64 diagonal block is solved in shared memory and written back.  The
// forward sweep ends with the (+)-scatter of L21 x to the separator rows (atomics), the backward sweep starts
// each block with the gather from them.  Per element the operands and their order are those of the reference's
// strsx2! / sgemx2! (src/CPU/dense/strsx.jl:596-672, src/CPU/chordal/strsx.jl:187-265, 783-830): contributions
// in increasing pivot order forward, separator first then decreasing pivot order backward.
#pragma once

#include "engine.cuh"

namespace pp {

constexpr int ST_RB = 64;  // residual rows per block
constexpr int ST_CT = 64;  // right-hand sides per CTA
constexpr int ST_KC = 16;  // operand chunk
constexpr int ST_LD = 65;  // padded row of the shared 64 x 64 tiles

template <typename T>
constexpr size_t sweep_tiled_smem() {
    return sizeof(T) * ((size_t)ST_RB * (ST_KC + 1) + (size_t)ST_KC * ST_LD + 2 * (size_t)ST_RB * ST_LD);
}

template <int SR, typename T, bool FWD, bool TRANS>
__global__ void __launch_bounds__(256) sweep_tiled_kernel(const int *__restrict__ fronts, DevPlan P,
                                                          const T *__restrict__ Dv, const T *__restrict__ Ov,
                                                          T *__restrict__ X, int64_t ldx, int k, int unit) {
    using S = Sem<SR, T>;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T *As = reinterpret_cast<T *>(smem_raw);  // [ST_RB][ST_KC + 1]
    T *Xs = As + ST_RB * (ST_KC + 1);          // [ST_KC][ST_LD]
    T *Dd = Xs + ST_KC * ST_LD;                // [ST_RB][ST_LD]: Dd[r * ST_LD + c] = Te(r0 + r, r0 + c)
    T *Ys = Dd + ST_RB * ST_LD;                // [ST_RB][ST_LD]

    const int f = fronts[blockIdx.x];
    const int c0 = blockIdx.y * ST_CT;
    const int tid = threadIdx.x, tc = tid & 15, tr = tid >> 4;
    const int rlo = P.rlo[f], nn = P.nn[f], na = P.na[f];
    const T *D = Dv + P.dptr[f];
    const T *O = Ov + P.lptr[f];
    const int *sep = P.stgt + P.sptr[f];
    const T z = S::zero();
    const bool scale = !unit && !S::integral;
    auto Te = [&](int r, int c) -> T { return TRANS ? D[c + (int64_t)r * nn] : D[r + (int64_t)c * nn]; };

    T acc[4][4];

    // acc[i][j] (+)= M(rb + row_i, kidx) (x) X[xrow(kidx)][col_j] for kidx in [kb, ke), ascending or descending
    auto accum = [&](int rb, int nrows, int kb, int ke, bool desc, auto M, auto xrow) {
        const int kn = ke - kb;
        for (int ch = 0; ch < kn; ch += ST_KC) {
            // chunk [cb, cb + kc) in index order, visited in the requested direction
            const int kc = min(ST_KC, kn - ch);
            const int cb = desc ? ke - ch - kc : kb + ch;
            for (int e = tid; e < ST_RB * ST_KC; e += 256) {
                const int r = e / ST_KC, kk = e % ST_KC;
                As[r * (ST_KC + 1) + kk] = (r < nrows && kk < kc) ? M(rb + r, cb + kk) : z;
            }
            for (int e = tid; e < ST_KC * ST_CT; e += 256) {
                const int kk = e / ST_CT, c = e % ST_CT;
                Xs[kk * ST_LD + c] = (kk < kc && c0 + c < k) ? X[(int64_t)xrow(cb + kk) * ldx + c0 + c] : z;
            }
            __syncthreads();
            for (int t = 0; t < kc; t++) {
                const int kk = desc ? kc - 1 - t : t;
                T a[4], x[4];
#pragma unroll
                for (int i = 0; i < 4; i++) a[i] = As[(tr + 16 * i) * (ST_KC + 1) + kk];
#pragma unroll
                for (int j = 0; j < 4; j++) x[j] = Xs[kk * ST_LD + tc + 16 * j];
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int j = 0; j < 4; j++) acc[i][j] = S::muladd(a[i], x[j], acc[i][j]);
            }
            __syncthreads();
        }
    };
    auto load_acc = [&](int rowbase, int nrows, bool from_x) {
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int r = tr + 16 * i, c = c0 + tc + 16 * j;
                acc[i][j] = (from_x && r < nrows && c < k) ? X[(int64_t)(rowbase + r) * ldx + c] : z;
            }
    };
    auto xres = [&](int p) { return rlo + p; };

    // diagonal block solve in shared memory: thread (c = tid % 64, g = tid / 64) owns rows g, g + 4, ...
    const int dc = tid & 63, dg = tid >> 6;
    auto diag_solve = [&](int r0, int nv) {
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) Ys[(tr + 16 * i) * ST_LD + tc + 16 * j] = acc[i][j];
        for (int e = tid; e < ST_RB * ST_RB; e += 256) {
            const int r = e / ST_RB, c = e % ST_RB;
            Dd[r * ST_LD + c] = (r < nv && c < nv) ? Te(r0 + r, r0 + c) : z;
        }
        __syncthreads();
        if (FWD) {
            for (int p = 0; p < nv; p++) {
                if (scale) {
                    if (dg == (p & 3)) Ys[p * ST_LD + dc] = S::mul(Ys[p * ST_LD + dc], S::star(Dd[p * ST_LD + p]));
                    __syncthreads();
                }
                const T yp = Ys[p * ST_LD + dc];
                for (int q = p + 1 + ((dg - p - 1) & 3); q < nv; q += 4)
                    Ys[q * ST_LD + dc] = S::muladd(Dd[q * ST_LD + p], yp, Ys[q * ST_LD + dc]);
                __syncthreads();
            }
        } else {
            for (int p = nv - 1; p >= 0; p--) {
                if (scale) {
                    if (dg == (p & 3)) Ys[p * ST_LD + dc] = S::mul(S::star(Dd[p * ST_LD + p]), Ys[p * ST_LD + dc]);
                    __syncthreads();
                }
                const T yp = Ys[p * ST_LD + dc];
                for (int q = dg; q < p; q += 4) Ys[q * ST_LD + dc] = S::muladd(Dd[q * ST_LD + p], yp, Ys[q * ST_LD + dc]);
                __syncthreads();
            }
        }
        for (int e = tid; e < ST_RB * ST_CT; e += 256) {
            const int r = e / ST_CT, c = e % ST_CT;
            if (r < nv && c0 + c < k) X[(int64_t)(rlo + r0 + r) * ldx + c0 + c] = Ys[r * ST_LD + c];
        }
        __syncthreads();
    };

    if (FWD) {
        for (int r0 = 0; r0 < nn; r0 += ST_RB) {
            const int nv = min(ST_RB, nn - r0);
            load_acc(rlo + r0, nv, true);
            accum(r0, nv, 0, r0, false, Te, xres);
            diag_solve(r0, nv);
        }
        // separator: X[sep_i] (+)= (L21 x)_i
        auto Of = [&](int i, int p) -> T { return TRANS ? O[p + (int64_t)i * nn] : O[i + (int64_t)p * na]; };
        for (int i0 = 0; i0 < na; i0 += ST_RB) {
            const int nv = min(ST_RB, na - i0);
            load_acc(0, 0, false);
            accum(i0, nv, 0, nn, false, Of, xres);
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int r = tr + 16 * i, c = c0 + tc + 16 * j;
                    if (r < nv && c < k) S::atomic_add(X + (int64_t)sep[i0 + r] * ldx + c, acc[i][j]);
                }
        }
    } else {
        auto Ob = [&](int r, int i) -> T { return TRANS ? O[i + (int64_t)r * na] : O[r + (int64_t)i * nn]; };
        auto xsep = [&](int i) { return sep[i]; };
        for (int r1 = nn; r1 > 0; r1 -= ST_RB) {
            const int r0 = max(0, r1 - ST_RB), nv = r1 - r0;
            load_acc(rlo + r0, nv, true);
            accum(r0, nv, 0, na, false, Ob, xsep);
            accum(r0, nv, r1, nn, true, Te, xres);
            diag_solve(r0, nv);
        }
    }
}

}  // namespace pp
