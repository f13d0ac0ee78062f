// sweep_wide.cuh — the triangular solves of the top fronts for many right-hand sides (the star's column panels,
// wide lmul! / rmul!): sweep_top_kernel's schedule, dependencies and per-element operation order, with tasks of
// (front, block of 64 rows, 128 right-hand sides).
//
// The products are a 64 x 128 tile per CTA, each thread a 4 x 8 block of accumulators fed by 128-bit shared-
// memory loads (one vector of 4 matrix rows, two vectors of 8 right-hand sides per k), over 16-deep operand
// chunks staged in shared memory, double-buffered, with the right-hand-side rows fetched as 16-byte vectors.
// Compared with the 64 x 32 tasks of sweep_top_kernel (2 x 4 accumulators, six scalar shared loads per k), a
// (x)(+) pair costs about an eighth of the shared-memory instructions, and the per-task work that does not scale
// with the columns (the diagonal block staged, the waits, the barriers) is shared by four times as many columns.
// The 64 x 64 diagonal solve is sweep_top_kernel's (a warp solves 4 right-hand sides with shuffles; here each
// warp does 4 such passes for its 16 columns); the forward separator scatter goes through shared memory so that
// consecutive threads (+)-scatter consecutive columns of a row.
//
// Per element the operands and their order are those of sweep_top_kernel, i.e. of the reference's strsx2! /
// sgemx2! (src/CPU/dense/strsx.jl:596-672, src/CPU/chordal/strsx.jl:187-265, 783-830).
#pragma once

#include <type_traits>

#include "sweep_top.cuh"

namespace pp {

constexpr int SWW_CT = 128;                 // right-hand sides per task
constexpr int SWW_AL = SW_RB + 4;           // padded row of the staged matrix chunk As[k][row] (16-byte rows)
constexpr int SWW_YL = SWW_CT + 1;          // padded row of the solved block Ys[row][rhs]

template <typename T>
constexpr size_t sweep_wide_stage_bytes() {
    return sizeof(T) * (2 * (size_t)SW_KC * SWW_AL + 2 * (size_t)SW_KC * SWW_CT);
}
template <typename T>
constexpr size_t sweep_wide_smem() {
    // the operand chunks and the block being solved are never live at once: Ys aliases them; Dd follows
    return (sweep_wide_stage_bytes<T>() > sizeof(T) * (size_t)SW_RB * SWW_YL ? sweep_wide_stage_bytes<T>()
                                                                              : sizeof(T) * (size_t)SW_RB * SWW_YL) +
           sizeof(T) * (size_t)SW_RB * SW_DL;
}

template <typename T>
struct Vec16;
template <>
struct Vec16<float> {
    using V = float4;
    static constexpr int n = 4;
};
template <>
struct Vec16<int32_t> {
    using V = int4;
    static constexpr int n = 4;
};
template <>
struct Vec16<double> {
    using V = double2;
    static constexpr int n = 2;
};

template <int SR, typename T, bool FWD, bool TRANS>
__global__ void __launch_bounds__(256, sizeof(T) == 8 ? 2 : (FWD ? 4 : 3)) sweep_wide_kernel(const int2 *__restrict__ wl, int count, DevPlan P,
                                                         const T *__restrict__ Dv, const T *__restrict__ Ov, T *X,
                                                         int64_t ldx, int k, int unit, int *flags, int *next,
                                                         int *err) {
    using S = Sem<SR, T>;
    using VT = typename Vec16<T>::V;
    constexpr int NV = Vec16<T>::n;                      // elements per 16-byte vector
    constexpr int XV = SW_KC * SWW_CT / NV / 256;        // right-hand-side vectors per thread per chunk
        extern __shared__ __align__(16) unsigned char smem_raw[];
    T *As = reinterpret_cast<T *>(smem_raw);              // 2 x [SW_KC][SWW_AL]
    T *Xs = As + 2 * SW_KC * SWW_AL;                      // 2 x [SW_KC][SWW_CT]
    T *Ys = As;                                           // [SW_RB][SWW_YL], aliases the chunks
    T *Dd = reinterpret_cast<T *>(smem_raw + (sweep_wide_smem<T>() - sizeof(T) * SW_RB * SW_DL));  // [SW_RB][SW_DL]
    const int tid = threadIdx.x, tr = tid & 15, tc = tid >> 4;  // products: rows 4tr .. 4tr+3, columns 8tc .. 8tc+7
    const int lane = tid & 31, w = tid >> 5, dg = lane & 7;
    const int ntiles = (k + SWW_CT - 1) / SWW_CT, nf = P.nf;
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
        const int c0 = tile * SWW_CT;
        const int rlo = P.rlo[f], nn = P.nn[f], na = P.na[f];
        const T *D = Dv + P.dptr[f];
        const T *O = Ov + P.lptr[f];
        const int *sep = P.stgt + P.sptr[f];
        auto Te = [&](int r, int c) -> T { return TRANS ? D[c + (int64_t)r * nn] : D[r + (int64_t)c * nn]; };
        auto xres = [&](int q) { return rlo + q; };
        auto xsep = [&](int i) { return sep[i]; };

        // tile rows per task: 64 (4 per thread), or 16 (1 per thread) when the task has at most 16 rows (most top
        // fronts have a few pivots; their 64-row tiles were mostly padding).  R is std::integral_constant<int, 4 or 1>.
        T acc[4][8];
        auto row_of = [&](auto R, int i) { return decltype(R)::value == 4 ? 4 * tr + i : tr; };
        auto load_acc = [&](auto R, int rowbase, int nrows, bool from_x) {
            constexpr int RPT = decltype(R)::value;
#pragma unroll
            for (int i = 0; i < RPT; i++)
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const int r = row_of(R, i), c = c0 + 8 * tc + j;
                    acc[i][j] = (from_x && r < nrows && c < k) ? ld_cg(X + (int64_t)(rowbase + r) * ldx + c) : z;
                }
        };
        // acc[i][j] (+)= M(rb + row_i, kidx) (x) X[xrow(kidx)][col_j] for kidx in [kb, ke), ascending or
        // descending; chunk ch + 1 is fetched into registers while chunk ch is used
        auto accum = [&](auto R, int rb, int nrows, int kb, int ke, bool desc, auto M, auto xrow) {
            constexpr int RPT = decltype(R)::value, TR = 16 * RPT, AER = SW_KC * TR / 256;
            const int kn = ke - kb;
            if (kn <= 0) return;
            const int nch = (kn + SW_KC - 1) / SW_KC;
            T ra[AER];
            VT rx[XV];
            auto fetch = [&](int ch) {
                const int kc = min(SW_KC, kn - ch * SW_KC);
                const int cb = desc ? ke - ch * SW_KC - kc : kb + ch * SW_KC;
#pragma unroll
                for (int q = 0; q < AER; q++) {
                    // consecutive threads read consecutive addresses: rows of the stored blocks, or (TRANS) columns
                    const int e = tid + 256 * q;
                    const int r = TRANS ? e / SW_KC : e % TR, kk = TRANS ? e % SW_KC : e / TR;
                    ra[q] = (r < nrows && kk < kc) ? M(rb + r, cb + kk) : z;
                }
#pragma unroll
                for (int q = 0; q < XV; q++) {
                    const int v = tid + 256 * q, kk = v / (SWW_CT / NV), c = (v % (SWW_CT / NV)) * NV;
                    if (kk < kc && c0 + c < k) {
                        rx[q] = __ldcg(reinterpret_cast<const VT *>(X + (int64_t)xrow(cb + kk) * ldx + c0 + c));
                    } else {
                        T *e = reinterpret_cast<T *>(&rx[q]);
#pragma unroll
                        for (int u = 0; u < NV; u++) e[u] = z;
                    }
                }
            };
            auto store = [&](int buf) {
                T *a = As + buf * SW_KC * SWW_AL;
                T *x = Xs + buf * SW_KC * SWW_CT;
#pragma unroll
                for (int q = 0; q < AER; q++) {
                    const int e = tid + 256 * q;
                    const int r = TRANS ? e / SW_KC : e % TR, kk = TRANS ? e % SW_KC : e / TR;
                    a[kk * SWW_AL + r] = ra[q];
                }
#pragma unroll
                for (int q = 0; q < XV; q++) {
                    const int v = tid + 256 * q, kk = v / (SWW_CT / NV), c = (v % (SWW_CT / NV)) * NV;
                    *reinterpret_cast<VT *>(x + kk * SWW_CT + c) = rx[q];
                }
            };
            fetch(0);
            store(0);
            __syncthreads();
            for (int ch = 0; ch < nch; ch++) {
                if (ch + 1 < nch) fetch(ch + 1);
                const int kc = min(SW_KC, kn - ch * SW_KC);
                const T *a = As + (ch & 1) * SW_KC * SWW_AL + (RPT == 4 ? 4 * tr : tr);
                const T *x = Xs + (ch & 1) * SW_KC * SWW_CT + 8 * tc;
                auto ldrow = [&](int kk, T *av, T *xv) {
                    if (RPT == 4) {
#pragma unroll
                        for (int q = 0; q < 4 / NV; q++)
                            *reinterpret_cast<VT *>(av + q * NV) =
                                *reinterpret_cast<const VT *>(a + kk * SWW_AL + q * NV);
                    } else {
                        av[0] = a[kk * SWW_AL];
                    }
#pragma unroll
                    for (int q = 0; q < 8 / NV; q++)
                        *reinterpret_cast<VT *>(xv + q * NV) = *reinterpret_cast<const VT *>(x + kk * SWW_CT + q * NV);
                };
                // MaxMin / MinMax in 4-byte types: two k per step (muladd2: min, min and one 3-input max, 3 ALU
                // instructions for 2 pairs instead of 4), the two terms in the sweep's order.  Elsewhere one k
                // (measured: the packed-add form of MinPlus Float32 ran slower here; 8-byte types run out of
                // registers)
                constexpr bool kpair = sizeof(T) == 4 && (SR == MAXMIN || SR == MINMAX);
                int u = 0;
                for (; kpair && u + 1 < kc; u += 2) {
                    const int k0 = desc ? kc - 1 - u : u, k1 = desc ? k0 - 1 : k0 + 1;
                    T av0[4], xv0[8], av1[4], xv1[8];
                    ldrow(k0, av0, xv0);
                    ldrow(k1, av1, xv1);
#pragma unroll
                    for (int i = 0; i < RPT; i++)
#pragma unroll
                        for (int j = 0; j < 8; j++) acc[i][j] = S::muladd2(acc[i][j], av0[i], av1[i], xv0[j], xv1[j]);
                }
                for (; u < kc; u++) {
                    T av[4], xv[8];
                    ldrow(desc ? kc - 1 - u : u, av, xv);
#pragma unroll
                    for (int i = 0; i < RPT; i++)
#pragma unroll
                        for (int j = 0; j < 8; j++) acc[i][j] = S::muladd(av[i], xv[j], acc[i][j]);
                }
                // buffer (ch + 1) & 1 was last read in chunk ch - 1, before the barrier that ended it; the barrier
                // here ends chunk ch (after the last chunk: every thread is done with both buffers)
                if (ch + 1 < nch) store((ch + 1) & 1);
                __syncthreads();
            }
        };
        auto acc_to_ys = [&](auto R) {
            constexpr int RPT = decltype(R)::value;
#pragma unroll
            for (int i = 0; i < RPT; i++)
#pragma unroll
                for (int j = 0; j < 8; j++) Ys[row_of(R, i) * SWW_YL + 8 * tc + j] = acc[i][j];
        };
        using R4 = std::integral_constant<int, 4>;
        using R1 = std::integral_constant<int, 1>;

        // the diagonal block of rows r0 .. r0 + nv - 1: acc -> Ys, solved warp by warp, written to X
        auto diag_solve = [&](auto R, int r0, int nv) {
            acc_to_ys(R);
            for (int e = tid; e < SW_RB * SW_RB; e += 256) {
                const int q = TRANS ? e / SW_RB : e % SW_RB, c = TRANS ? e % SW_RB : e / SW_RB;
                Dd[q * SW_DL + c] = (q < nv && c < nv) ? Te(r0 + q, r0 + c) : z;
            }
            __syncthreads();
            // blocked by 8 rows: per sub-block (in pivot order: ascending forward, descending backward) a thread per
            // right-hand side solves the sub-block's 8 x 8 triangle in registers, then the CTA applies the
            // sub-block's pivots to the block's remaining rows as a register-tiled product (4 right-hand sides x
            // the 8 pivots per thread, k in pivot order), so most of the block's pairs run at the product's rate
            const int nb8 = (nv + 7) >> 3;
            for (int jj = 0; jj < nb8; jj++) {
                const int J = FWD ? jj : nb8 - 1 - jj;
                const int j0 = 8 * J, jn = min(8, nv - j0);
                if (tid < SWW_CT) {
                    T y[8];
#pragma unroll
                    for (int r = 0; r < 8; r++) y[r] = r < jn ? Ys[(j0 + r) * SWW_YL + tid] : z;
                    if (FWD) {
#pragma unroll
                        for (int g = 0; g < 8; g++) {
                            if (g >= jn) break;
                            T yq = y[g];
                            if (scale) yq = S::mul(yq, S::star(Dd[(j0 + g) * SW_DL + j0 + g]));
                            y[g] = yq;
#pragma unroll
                            for (int v = g + 1; v < 8; v++)
                                if (v < jn) y[v] = S::muladd(Dd[(j0 + v) * SW_DL + j0 + g], yq, y[v]);
                        }
                    } else {
#pragma unroll
                        for (int g = 7; g >= 0; g--) {
                            if (g >= jn) continue;
                            T yq = y[g];
                            if (scale) yq = S::mul(S::star(Dd[(j0 + g) * SW_DL + j0 + g]), yq);
                            y[g] = yq;
#pragma unroll
                            for (int v = 0; v < g; v++) y[v] = S::muladd(Dd[(j0 + v) * SW_DL + j0 + g], yq, y[v]);
                        }
                    }
#pragma unroll
                    for (int r = 0; r < 8; r++)
                        if (r < jn) Ys[(j0 + r) * SWW_YL + tid] = y[r];
                }
                __syncthreads();
                // the rows the sub-block's pivots act on: below it (forward) or above it (backward)
                const int ra = FWD ? j0 + 8 : 0, rz = FWD ? nv : j0;
                if (rz > ra) {
                    const int cg = 4 * (tid & 31);  // right-hand sides cg .. cg + 3
                    T yv[8][4];
#pragma unroll
                    for (int kk = 0; kk < 8; kk++)
#pragma unroll
                        for (int c = 0; c < 4; c++) yv[kk][c] = kk < jn ? Ys[(j0 + kk) * SWW_YL + cg + c] : z;
                    for (int i = ra + (tid >> 5); i < rz; i += 8) {
                        T d[8];
#pragma unroll
                        for (int kk = 0; kk < 8; kk++) d[kk] = kk < jn ? Dd[i * SW_DL + j0 + kk] : z;
#pragma unroll
                        for (int c = 0; c < 4; c++) {
                            T a = Ys[i * SWW_YL + cg + c];
#pragma unroll
                            for (int u = 0; u < 8; u++) {
                                const int kk = FWD ? u : 7 - u;
                                a = S::muladd(d[kk], yv[kk][c], a);
                            }
                            Ys[i * SWW_YL + cg + c] = a;
                        }
                    }
                }
                __syncthreads();
            }
            for (int e = tid; e < SW_RB * SWW_CT; e += 256) {
                const int r = e / SWW_CT, c = e % SWW_CT;
                if (r < nv && c0 + c < k) X[(int64_t)(rlo + r0 + r) * ldx + c0 + c] = Ys[r * SWW_YL + c];
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
                    // the right-hand sides are zero on the whole residual: the front changes nothing
                    bool nz = false;
                    for (int e = tid; e < nn * SWW_CT; e += 256) {
                        const int c = c0 + e % SWW_CT;
                        if (c < k) nz |= !(ld_cg(X + (int64_t)(rlo + e / SWW_CT) * ldx + c) == z);
                    }
                    live = __syncthreads_or(nz) != 0;
                }
            } else {
                const int v = cta_wait_blocks(bd, 1, err);
                if (v < 0) return;
                live = (v >> 16) == 0;
            }
            if (live) {
                auto body = [&](auto R) -> bool {
                    load_acc(R, rlo + r0, nv, true);
                    for (int j = 0; j < b; j++) {
                        if (j > 0 && cta_wait_blocks(bd, j + 1, err) < 0) return false;
                        accum(R, r0, nv, j * SW_RB, (j + 1) * SW_RB, false, Te, xres);
                    }
                    diag_solve(R, r0, nv);
                    return true;
                };
                if (!(nv <= 16 ? body(R1{}) : body(R4{}))) return;
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
                auto body = [&](auto R) {
                    load_acc(R, 0, 0, false);
                    accum(R, i0, nv, 0, nn, false, Of, xres);
                    acc_to_ys(R);
                };
                if (nv <= 16)
                    body(R1{});
                else
                    body(R4{});
                __syncthreads();
                for (int e = tid; e < SW_RB * SWW_CT; e += 256) {
                    const int r = e / SWW_CT, c = e % SWW_CT;
                    const T v = Ys[r * SWW_YL + c];
                    // (+) with zero changes nothing: zero sums are not scattered
                    if (r < nv && c0 + c < k && !(v == z)) S::atomic_add(X + (int64_t)sep[i0 + r] * ldx + c0 + c, v);
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
            auto body = [&](auto R) -> bool {
                load_acc(R, rlo + r0, nv, true);
                accum(R, r0, nv, 0, na, false, Ob, xsep);
                for (int j = kb - 1; j > b; j--) {
                    if (cta_wait_blocks(bd, kb - j, err) < 0) return false;
                    accum(R, r0, nv, j * SW_RB, min(nn, (j + 1) * SW_RB), true, Te, xres);
                }
                diag_solve(R, r0, nv);
                return true;
            };
            if (!(nv <= 16 ? body(R1{}) : body(R4{}))) return;
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
