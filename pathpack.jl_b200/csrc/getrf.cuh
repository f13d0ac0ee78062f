// getrf.cuh — pp_getrf_batched for blocks of up to 128 x 128: the in-place LU of the star of each block
// (sgetrf! per block, src/CPU/dense/sgetrf.jl:151-175 scalar path; the reference GPU's sgetrf_gpu!,
// ext/PATHPACKCUDAExt/dense/sgetrf.jl:31-125), one 256-thread CTA per block with the block held in registers.
//
// Layout: the block is padded to NB = 16 R rows and columns and dealt 2D-cyclically over a 16 x 16 thread grid:
// thread (tr, tc) = (tid % 16, tid / 16) holds f[a][b] = F[tr + 16 a][tc + 16 b].  Cyclic ownership keeps the
// shrinking trailing matrix spread over all threads.  Pivots run in phases of 16 (phase q: pivots 16q .. 16q+15);
// in phase q the register rows a < q and columns b < q are finished for every thread, so the unrolled update
// touches (R - q)^2 registers, with only row a == q and column b == q under a per-thread predicate.
//
// Pivot p: the half-warp holding column p (tc == p % 16) scales its entries below the diagonal by star(F[p,p])
// (the diagonal comes from a shuffle within that half-warp) and publishes the column; the threads holding row p
// publish it; one barrier; every thread updates its trailing entries F[i,j] = F[i,p] (x) F[p,j] (+) F[i,j].
// The published column and row are double-buffered, so one barrier per pivot suffices: a buffer is rewritten
// two pivots later, after every thread has passed the barrier in between, i.e. after its reads.
//
// Per element the operations and their order are those of the scalar LU (scale once, then one multiply-add per
// earlier pivot in increasing order), so every semiring gives the bits of lu_smem and of the reference.
#pragma once

#include "semiring.cuh"

namespace pp {

template <int SR, typename T, int R>
__global__ void __launch_bounds__(256, sizeof(T) == 8 ? 1 : 2) getrf_reg_kernel(int n, T *A) {
    using S = Sem<SR, T>;
    __shared__ __align__(16) T colb[2][16][R];  // colb[buf][tr][a] = F[tr + 16a][p] (scaled below the diagonal)
    __shared__ __align__(16) T rowb[2][16][R];  // rowb[buf][tc][b] = F[p][tc + 16b]
    const int tid = threadIdx.x, tr = tid & 15, tc = tid >> 4, lane = tid & 31;
    T *Ab = A + (int64_t)blockIdx.x * n * n;
    const T z = S::zero();
    T f[R][R];
#pragma unroll
    for (int b = 0; b < R; b++) {
        const int j = tc + 16 * b;
#pragma unroll
        for (int a = 0; a < R; a++) {
            const int i = tr + 16 * a;
            f[a][b] = (i < n && j < n) ? Ab[i + (int64_t)j * n] : z;
        }
    }
#pragma unroll
    for (int q = 0; q < R; q++) {
        const int pend = min(16, n - 16 * q);  // pivots of this phase (uniform over the CTA)
        for (int pp = 0; pp < pend; pp++) {
            const int p = 16 * q + pp, buf = p & 1;
            if (tc == pp) {  // one half-warp holds column p
                if (!S::integral) {
                    const unsigned half = (lane & 16) ? 0xffff0000u : 0x0000ffffu;
                    const T s = S::star(__shfl_sync(half, f[q][q], (lane & 16) | pp));
#pragma unroll
                    for (int a = q; a < R; a++)
                        if (a > q || tr > pp) f[a][q] = S::mul(f[a][q], s);
                }
#pragma unroll
                for (int a = q; a < R; a++) colb[buf][tr][a] = f[a][q];
            }
            if (tr == pp) {
#pragma unroll
                for (int b = q; b < R; b++) rowb[buf][tc][b] = f[q][b];
            }
            __syncthreads();
            T cv[R], rv[R];
#pragma unroll
            for (int a = q; a < R; a++) cv[a] = colb[buf][tr][a];
#pragma unroll
            for (int b = q; b < R; b++) rv[b] = rowb[buf][tc][b];
            const bool r0 = tr > pp, c0 = tc > pp;  // row 16q + tr and column 16q + tc still trail pivot p
#pragma unroll
            for (int a = q; a < R; a++) {
#pragma unroll
                for (int b = q; b < R; b++) {
                    if ((a > q || r0) && (b > q || c0)) f[a][b] = S::muladd(cv[a], rv[b], f[a][b]);
                }
            }
        }
    }
#pragma unroll
    for (int b = 0; b < R; b++) {
        const int j = tc + 16 * b;
#pragma unroll
        for (int a = 0; a < R; a++) {
            const int i = tr + 16 * a;
            if (i < n && j < n) Ab[i + (int64_t)j * n] = f[a][b];
        }
    }
}

}  // namespace pp
