// gemm.cuh — the semiring GEMM C <- C (+) A (x) B on the ALUs (column-major operands).
//
// Replaces sgemx_gpu! and its kernels v2/v4/v6/v7/v8 (ext/PATHPACKCUDAExt/dense/sgemx.jl:27-737,
// dense/sgemx_simt.jl:1-502).  The non-field semirings have no tensor-core form, so this is a register-tiled
// SIMT kernel: a 256-thread CTA computes a BM x BN tile of C, each thread a TM x TN sub-tile held in registers,
// with A and B staged through double-buffered shared memory.
//
// Shared memory holds k-pairs: As[kp][m] = (A[m][2kp], A[m][2kp+1]) and Bs[kp][n] likewise, so one step of
// the inner loop combines two k's into each accumulator.  For Float32 MinPlus/MaxPlus that step is one
// packed add (add.f32x2, FADD2) and one 3-input min/max (FMNMX3): one instruction per (x)(+) pair, the same
// count as the reference's sm_100 kernel v8 (dense/sgemx_simt.jl:185-253).
//
// Thread (tr, tc) = (tid % 16, tid / 16) owns rows {q*16V + tr*V + e} and columns {q*16V + tc*V + e}, V pairs
// per 16-byte vector, so the shared-memory reads of a warp are contiguous 256-byte runs (no bank conflicts).
//
// Out-of-range operands read as szero, which leaves an accumulator unchanged in every semiring (szero is
// absorbing for (x) and the unit of (+); szero (x) szero = szero also for PlusProd).  Accumulators start from C
// and take k in increasing order, which for PlusProd is the order of the reference's sgemx2!.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include <type_traits>

#include "semiring.cuh"

namespace pp {

template <typename T>
struct alignas(2 * sizeof(T)) Pair {
    T x, y;
};

template <typename T>
struct GemmCfg;
template <>
struct GemmCfg<float> {
    static constexpr int TM = 8, TN = 4, BK = 16;  // 128 registers: two CTAs (16 warps) per SM
};
template <>
struct GemmCfg<int32_t> {
    static constexpr int TM = 8, TN = 8, BK = 16;
};
template <>
struct GemmCfg<double> {
    static constexpr int TM = 8, TN = 4, BK = 8;
};

template <int SR, typename T>
struct GemmKernel {
    using S = Sem<SR, T>;
    using P = Pair<T>;
    static constexpr int TM = GemmCfg<T>::TM, TN = GemmCfg<T>::TN, BK = GemmCfg<T>::BK;
    static constexpr int V = 16 / (int)sizeof(P);  // pairs per 16-byte vector
    static constexpr int BM = 16 * TM, BN = 16 * TN, KP = BK / 2;
    static constexpr int RA = 16 / (int)sizeof(T);  // rows of A per thread-chunk (one 16-byte load per column)
    static constexpr int RB = 16 / (int)sizeof(T);  // k's of B per thread-chunk
    static constexpr int ACH = (BM / RA) * KP;       // A chunks per tile
    static constexpr int BCH = BN * (BK / RB);       // B chunks per tile
    static constexpr int ANT = (ACH + 255) / 256, BNT = (BCH + 255) / 256;
    static_assert(TM % V == 0 && TN % V == 0, "tile");
    static constexpr size_t smem_bytes = 2 * (size_t)KP * (BM + BN) * sizeof(P);
};

template <typename T, int R>
struct Vec;
template <>
struct Vec<float, 4> {
    using type = float4;
};
template <>
struct Vec<int32_t, 4> {
    using type = int4;
};
template <>
struct Vec<double, 2> {
    using type = double2;
};

template <int SR, typename T>
__global__ void __launch_bounds__(256, sizeof(T) == 4 && GemmCfg<T>::TN == 4 ? 2 : 1)
    gemm_kernel(int M, int N, int K, T *__restrict__ C, int64_t ldc, const T *__restrict__ A, int64_t lda,
                const T *__restrict__ B, int64_t ldb) {
    using G = GemmKernel<SR, T>;
    using S = typename G::S;
    using P = typename G::P;
    constexpr int TM = G::TM, TN = G::TN, BK = G::BK, V = G::V, BM = G::BM, BN = G::BN, KP = G::KP;
    constexpr int RA = G::RA, RB = G::RB;
    using VecT = typename Vec<T, RA>::type;

    extern __shared__ __align__(16) unsigned char smem_raw[];
    P *As = reinterpret_cast<P *>(smem_raw);  // [2][KP][BM]
    P *Bs = As + 2 * KP * BM;                 // [2][KP][BN]

    const int tid = threadIdx.x;
    const int tr = tid & 15, tc = tid >> 4;
    const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
    const T z = S::zero();

    // accumulators start from C
    T acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; i++) {
        const int m = m0 + (i / V) * 16 * V + tr * V + (i % V);
#pragma unroll
        for (int j = 0; j < TN; j++) {
            const int n = n0 + (j / V) * 16 * V + tc * V + (j % V);
            acc[i][j] = (m < M && n < N) ? C[(int64_t)m + (int64_t)n * ldc] : z;
        }
    }

    const bool avec = ((reinterpret_cast<uintptr_t>(A) | (uintptr_t)(lda * sizeof(T))) & 15) == 0;
    const bool bvec = ((reinterpret_cast<uintptr_t>(B) | (uintptr_t)(ldb * sizeof(T))) & 15) == 0;

    T ra[G::ANT][2][RA];
    T rb[G::BNT][RB];

    auto load_tile = [&](int k0) {
#pragma unroll
        for (int t = 0; t < G::ANT; t++) {
            const int c = tid + t * 256;
            if (c < G::ACH) {
                const int kp = c / (BM / RA), mr = (c % (BM / RA)) * RA;
                const int m = m0 + mr;
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const int k = k0 + 2 * kp + h;
                    if (avec && k < K && m + RA <= M) {
                        const VecT v = *reinterpret_cast<const VecT *>(A + (int64_t)m + (int64_t)k * lda);
                        const T *pv = reinterpret_cast<const T *>(&v);
#pragma unroll
                        for (int e = 0; e < RA; e++) ra[t][h][e] = pv[e];
                    } else {
#pragma unroll
                        for (int e = 0; e < RA; e++)
                            ra[t][h][e] = (k < K && m + e < M) ? A[(int64_t)(m + e) + (int64_t)k * lda] : z;
                    }
                }
            }
        }
#pragma unroll
        for (int t = 0; t < G::BNT; t++) {
            const int c = tid + t * 256;
            if (c < G::BCH) {
                const int kc = c % (BK / RB), nn = c / (BK / RB);
                const int n = n0 + nn, k = k0 + kc * RB;
                if (bvec && n < N && k + RB <= K) {
                    const VecT v = *reinterpret_cast<const VecT *>(B + (int64_t)k + (int64_t)n * ldb);
                    const T *pv = reinterpret_cast<const T *>(&v);
#pragma unroll
                    for (int e = 0; e < RB; e++) rb[t][e] = pv[e];
                } else {
#pragma unroll
                    for (int e = 0; e < RB; e++)
                        rb[t][e] = (n < N && k + e < K) ? B[(int64_t)(k + e) + (int64_t)n * ldb] : z;
                }
            }
        }
    };
    auto store_tile = [&](int buf) {
        P *as = As + buf * KP * BM;
        P *bs = Bs + buf * KP * BN;
#pragma unroll
        for (int t = 0; t < G::ANT; t++) {
            const int c = tid + t * 256;
            if (c < G::ACH) {
                const int kp = c / (BM / RA), mr = (c % (BM / RA)) * RA;
#pragma unroll
                for (int e = 0; e < RA; e++) {
                    P p;
                    p.x = ra[t][0][e];
                    p.y = ra[t][1][e];
                    as[kp * BM + mr + e] = p;
                }
            }
        }
#pragma unroll
        for (int t = 0; t < G::BNT; t++) {
            const int c = tid + t * 256;
            if (c < G::BCH) {
                const int kc = c % (BK / RB), nn = c / (BK / RB);
#pragma unroll
                for (int e = 0; e < RB; e += 2) {
                    P p;
                    p.x = rb[t][e];
                    p.y = rb[t][e + 1];
                    bs[((kc * RB + e) / 2) * BN + nn] = p;
                }
            }
        }
    };

    const int nk = (K + BK - 1) / BK;
    if (nk > 0) {
        load_tile(0);
        store_tile(0);
    }
    __syncthreads();
    for (int kt = 0; kt < nk; kt++) {
        const int buf = kt & 1;
        if (kt + 1 < nk) load_tile((kt + 1) * BK);
        const P *as = As + buf * KP * BM;
        const P *bs = Bs + buf * KP * BN;
#pragma unroll
        for (int kp = 0; kp < KP; kp++) {
            P a[TM], b[TN];
#pragma unroll
            for (int q = 0; q < TM / V; q++) {
                const float4 v = *reinterpret_cast<const float4 *>(as + kp * BM + q * 16 * V + tr * V);
                const P *pv = reinterpret_cast<const P *>(&v);
#pragma unroll
                for (int e = 0; e < V; e++) a[q * V + e] = pv[e];
            }
#pragma unroll
            for (int q = 0; q < TN / V; q++) {
                const float4 v = *reinterpret_cast<const float4 *>(bs + kp * BN + q * 16 * V + tc * V);
                const P *pv = reinterpret_cast<const P *>(&v);
#pragma unroll
                for (int e = 0; e < V; e++) b[q * V + e] = pv[e];
            }
#pragma unroll
            for (int i = 0; i < TM; i++)
#pragma unroll
                for (int j = 0; j < TN; j++) acc[i][j] = S::muladd2(acc[i][j], a[i].x, a[i].y, b[j].x, b[j].y);
        }
        if (kt + 1 < nk) store_tile(buf ^ 1);
        __syncthreads();
    }

#pragma unroll
    for (int i = 0; i < TM; i++) {
        const int m = m0 + (i / V) * 16 * V + tr * V + (i % V);
#pragma unroll
        for (int j = 0; j < TN; j++) {
            const int n = n0 + (j / V) * 16 * V + tc * V + (j % V);
            if (m < M && n < N) C[(int64_t)m + (int64_t)n * ldc] = acc[i][j];
        }
    }
}

// PlusProd Float64: C <- C + A B on the FP64 tensor cores (DMMA, mma.sync m8n8k4 f64; tcgen05 has no f64 kind).
// A CTA of 4 warps computes a 64 x 64 tile of C, each warp 32 x 32 as 4 x 4 fragments of 8 x 8, over 16-deep
// k-chunks of A (As[k][m]) and B (Bs[k][n]) staged in shared memory, double-buffered.  Fragments (PTX m8n8k4
// .row.col): lane l holds A(l / 4, l % 4), B(l % 4, l / 4) and C(l / 4, 2 (l % 4) + {0, 1}).  Out-of-range
// operands read as 0.  The products of one instruction are summed in the tensor core's order, so results agree
// with the sequential sgemx2! within rounding (the PlusProd tolerance), not bit for bit.
constexpr int DM_BM = 64, DM_BN = 64, DM_BK = 16, DM_LD = 64 + 2;  // padded rows of the staged chunks

__device__ __forceinline__ void dmma_8x8x4(double &d0, double &d1, double a, double b) {
    asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};\n"
                 : "+d"(d0), "+d"(d1)
                 : "d"(a), "d"(b));
}

template <typename T>  // T = double (a template, so that only the translation unit that launches it defines it)
__global__ void __launch_bounds__(128) gemm_dmma_kernel(int M, int N, int K, T *__restrict__ C, int64_t ldc,
                                                        const T *__restrict__ A, int64_t lda,
                                                        const T *__restrict__ B, int64_t ldb) {
    static_assert(std::is_same<T, double>::value, "DMMA f64");
    __shared__ __align__(16) double As[2][DM_BK][DM_LD];
    __shared__ __align__(16) double Bs[2][DM_BK][DM_LD];
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int wm = (w & 1) * 32, wn = (w >> 1) * 32;  // the warp's 32 x 32 block of the tile
    const int g = lane >> 2, q = lane & 3;
    const int m0 = blockIdx.x * DM_BM, n0 = blockIdx.y * DM_BN;
    double acc[4][4][2];
#pragma unroll
    for (int mt = 0; mt < 4; mt++)
#pragma unroll
        for (int nt = 0; nt < 4; nt++)
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int m = m0 + wm + mt * 8 + g, n = n0 + wn + nt * 8 + 2 * q + h;
                acc[mt][nt][h] = (m < M && n < N) ? C[(int64_t)m + (int64_t)n * ldc] : 0.0;
            }
    // staging: A chunk 64 x 16 (rows m contiguous in memory), B chunk 16 x 64 (k contiguous); 8 each per thread
    double ra[8], rb[8];
    auto load = [&](int k0) {
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const int idx = tid + 128 * e;          // A: m = idx % 64, k = idx / 64
            const int m = m0 + (idx & 63), k = k0 + (idx >> 6);
            ra[e] = (m < M && k < K) ? A[(int64_t)m + (int64_t)k * lda] : 0.0;
            const int kb = k0 + (idx & 15), n = n0 + (idx >> 4);  // B: k = idx % 16, n = idx / 16
            rb[e] = (kb < K && n < N) ? B[(int64_t)kb + (int64_t)n * ldb] : 0.0;
        }
    };
    auto store = [&](int buf) {
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const int idx = tid + 128 * e;
            As[buf][idx >> 6][idx & 63] = ra[e];
            Bs[buf][idx & 15][idx >> 4] = rb[e];
        }
    };
    const int nk = (K + DM_BK - 1) / DM_BK;
    if (nk > 0) {
        load(0);
        store(0);
    }
    __syncthreads();
    for (int kt = 0; kt < nk; kt++) {
        const int buf = kt & 1;
        if (kt + 1 < nk) load((kt + 1) * DM_BK);
#pragma unroll
        for (int ks = 0; ks < DM_BK; ks += 4) {
            double af[4], bf[4];
#pragma unroll
            for (int mt = 0; mt < 4; mt++) af[mt] = As[buf][ks + q][wm + mt * 8 + g];
#pragma unroll
            for (int nt = 0; nt < 4; nt++) bf[nt] = Bs[buf][ks + q][wn + nt * 8 + g];
#pragma unroll
            for (int mt = 0; mt < 4; mt++)
#pragma unroll
                for (int nt = 0; nt < 4; nt++) dmma_8x8x4(acc[mt][nt][0], acc[mt][nt][1], af[mt], bf[nt]);
        }
        if (kt + 1 < nk) store(buf ^ 1);
        __syncthreads();
    }
#pragma unroll
    for (int mt = 0; mt < 4; mt++)
#pragma unroll
        for (int nt = 0; nt < 4; nt++)
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int m = m0 + wm + mt * 8 + g, n = n0 + wn + nt * 8 + 2 * q + h;
                if (m < M && n < N) C[(int64_t)m + (int64_t)n * ldc] = acc[mt][nt][h];
            }
}

// ---- PlusProd Float64 with TMA-staged tiles
//
// gemm_dmma_kernel's warp tiling and DMMA fragments, with the k-chunks of A and B fetched by the tensor memory
// accelerator (cp.async.bulk.tensor.2d) into a 4-stage shared-memory ring: one thread issues a stage's copies
// and arms its "full" barrier with the byte count; the four warps wait on it (mbarrier try_wait), compute, and
// arrive on the stage's "empty" barrier, after which the stage is refilled with chunk kt + 4.  No register
// staging and no CTA barrier in the main loop.  The boxes are shaped so that the fragment loads are free of
// bank conflicts without swizzling: A in boxes of 8 (m) x 16 (k) (a warp's A fragment, 8 m x 4 k, is 256
// contiguous bytes), B in boxes of 4 (k) x 64 (n) (a B fragment, 4 k x 8 n, likewise).  Out-of-range elements
// are filled with zeros by the copy (the PlusProd zero).  The tensor maps cover this GPU's memory only and
// no copy uses cluster multicast.  Every mbarrier wait is bounded (2 s of global time): one that runs out sets
// g_gemm_err, fills the CTA's tile of C with NaN, waits (bounded) for the copies it issued, and returns.
constexpr int DT_STAGES = 4, DT_BK = 16;
constexpr int DT_A_ELEMS = 64 * DT_BK, DT_B_ELEMS = DT_BK * 64;  // doubles per stage
constexpr unsigned DT_STAGE_BYTES = 8u * (DT_A_ELEMS + DT_B_ELEMS);
constexpr size_t dmma_tma_smem = 128 + (size_t)DT_STAGES * DT_STAGE_BYTES + 2 * DT_STAGES * sizeof(unsigned long long);

__device__ int g_gemm_err;

__device__ __forceinline__ unsigned smem_u32(const void *p) { return (unsigned)__cvta_generic_to_shared(p); }

__device__ __forceinline__ bool mbar_wait_bounded(unsigned long long *bar, unsigned phase) {
    unsigned long long t0 = 0;
    for (unsigned it = 0;; it++) {
        unsigned ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(phase)
            : "memory");
        if (ok) return true;
        if ((it & 63) == 0) {
            unsigned long long t;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
            if (it == 0)
                t0 = t;
            else if (t - t0 > 2000000000ull)
                return false;
        }
    }
}

template <typename T>  // T = double
__global__ void __launch_bounds__(128) gemm_dmma_tma_kernel(int M, int N, int K, T *__restrict__ C, int64_t ldc,
                                                            const __grid_constant__ CUtensorMap mapA,
                                                            const __grid_constant__ CUtensorMap mapB) {
    static_assert(std::is_same<T, double>::value, "DMMA f64");
    extern __shared__ __align__(128) unsigned char dt_smem[];
    unsigned char *base = dt_smem + ((128 - (smem_u32(dt_smem) & 127)) & 127);
    double *sA = reinterpret_cast<double *>(base);             // [stage][8 boxes][16 k][8 m]
    double *sB = sA + DT_STAGES * DT_A_ELEMS;                  // [stage][4 boxes][64 n][4 k]
    unsigned long long *full = reinterpret_cast<unsigned long long *>(sB + DT_STAGES * DT_B_ELEMS);
    unsigned long long *empty = full + DT_STAGES;
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int wm = (w & 1) * 32, wn = (w >> 1) * 32;
    const int g = lane >> 2, q = lane & 3;
    const int m0 = blockIdx.x * DM_BM, n0 = blockIdx.y * DM_BN;
    const int nk = (K + DT_BK - 1) / DT_BK;
    double acc[4][4][2];
#pragma unroll
    for (int mt = 0; mt < 4; mt++)
#pragma unroll
        for (int nt = 0; nt < 4; nt++)
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int m = m0 + wm + mt * 8 + g, n = n0 + wn + nt * 8 + 2 * q + h;
                acc[mt][nt][h] = (m < M && n < N) ? C[(int64_t)m + (int64_t)n * ldc] : 0.0;
            }
    if (tid == 0) {
        for (int st = 0; st < DT_STAGES; st++) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(full + st)) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 4;" ::"r"(smem_u32(empty + st)) : "memory");
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    auto issue = [&](int kt) {  // thread 0: chunk kt into stage kt % DT_STAGES
        const int st = kt % DT_STAGES;
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(full + st)),
                     "r"(DT_STAGE_BYTES)
                     : "memory");
        const int k0 = kt * DT_BK;
#pragma unroll
        for (int i = 0; i < 8; i++)  // A: box (m0 + 8 i .. + 8, k0 .. k0 + 16)
            asm volatile(
                "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                ::"r"(smem_u32(sA + st * DT_A_ELEMS + i * 128)), "l"(&mapA), "r"(m0 + 8 * i), "r"(k0),
                "r"(smem_u32(full + st))
                : "memory");
#pragma unroll
        for (int j = 0; j < 4; j++)  // B: box (k0 + 4 j .. + 4, n0 .. n0 + 64)
            asm volatile(
                "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                ::"r"(smem_u32(sB + st * DT_B_ELEMS + j * 256)), "l"(&mapB), "r"(k0 + 4 * j), "r"(n0),
                "r"(smem_u32(full + st))
                : "memory");
    };
    int issued = 0, consumed = 0;
    if (tid == 0)
        for (; issued < DT_STAGES && issued < nk; issued++) issue(issued);
    bool bad = false;
    for (int kt = 0; kt < nk; kt++) {
        const int st = kt % DT_STAGES;
        const unsigned ph = (unsigned)(kt / DT_STAGES) & 1u;
        if (!mbar_wait_bounded(full + st, ph)) {
            bad = true;
            break;
        }
        consumed = kt + 1;
        const double *a = sA + st * DT_A_ELEMS, *b = sB + st * DT_B_ELEMS;
#pragma unroll
        for (int ks = 0; ks < DT_BK; ks += 4) {
            double af[4], bf[4];
#pragma unroll
            for (int mt = 0; mt < 4; mt++) af[mt] = a[((wm >> 3) + mt) * 128 + (ks + q) * 8 + g];
#pragma unroll
            for (int nt = 0; nt < 4; nt++) bf[nt] = b[(ks >> 2) * 256 + (wn + nt * 8 + g) * 4 + q];
#pragma unroll
            for (int mt = 0; mt < 4; mt++)
#pragma unroll
                for (int nt = 0; nt < 4; nt++) dmma_8x8x4(acc[mt][nt][0], acc[mt][nt][1], af[mt], bf[nt]);
        }
        __syncwarp();
        if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(empty + st)) : "memory");
        if (tid == 0 && issued < nk) {  // refill this stage once every warp is done with it
            if (!mbar_wait_bounded(empty + st, ph)) {
                bad = true;
                break;
            }
            issue(issued++);
        }
    }
    if (bad) {
        atomicExch(&g_gemm_err, 1);
        if (tid == 0)  // the copies still in flight land in this CTA's shared memory: wait for them (bounded)
            for (int kt = consumed; kt < issued; kt++)
                if (!mbar_wait_bounded(full + kt % DT_STAGES, (unsigned)(kt / DT_STAGES) & 1u)) break;
    }
#pragma unroll
    for (int mt = 0; mt < 4; mt++)
#pragma unroll
        for (int nt = 0; nt < 4; nt++)
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int m = m0 + wm + mt * 8 + g, n = n0 + wn + nt * 8 + 2 * q + h;
                if (m < M && n < N) C[(int64_t)m + (int64_t)n * ldc] = bad ? CUDART_NAN : acc[mt][nt][h];
            }
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (the library links no libcuda)
static inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult qr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) != cudaSuccess ||
            qr != cudaDriverEntryPointSuccess)
            p = nullptr;
        cudaGetLastError();
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }();
    return fn;
}

// a 2D tensor map of a column-major double matrix (inner x outer, leading dimension ld) with the given box
static inline bool make_map(CUtensorMap *map, const double *ptr, int64_t inner, int64_t outer, int64_t ld,
                            unsigned box_inner, unsigned box_outer) {
    const auto enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * sizeof(double)};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT64, 2, const_cast<double *>(ptr), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// host launcher
template <int SR, typename T>
cudaError_t launch_gemm(int64_t M, int64_t N, int64_t K, T *C, int64_t ldc, const T *A, int64_t lda, const T *B,
                        int64_t ldb, cudaStream_t st) {
    using G = GemmKernel<SR, T>;
    if (M <= 0 || N <= 0 || K <= 0) return cudaSuccess;
    if constexpr (SR == PLUSPROD && std::is_same<T, double>::value) {
        dim3 grid((unsigned)((M + DM_BM - 1) / DM_BM), (unsigned)((N + DM_BN - 1) / DM_BN));
        // TMA-staged when the operands allow tensor maps: 16-byte aligned bases, leading dimensions of whole
        // 16-byte units; otherwise the register-staged kernel
        CUtensorMap ma, mb;
        const bool tma = ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B)) & 15) == 0 &&
                         (lda & 1) == 0 && (ldb & 1) == 0 && make_map(&ma, A, M, K, lda, 8, DT_BK) &&
                         make_map(&mb, B, K, N, ldb, 4, DM_BN);
        if (tma) {
            int dev = 0;
            cudaGetDevice(&dev);
            static bool attr[64] = {};
            if (dev < 64 && !attr[dev]) {
                cudaError_t e = cudaFuncSetAttribute(gemm_dmma_tma_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     (int)dmma_tma_smem);
                if (e != cudaSuccess) return e;
                attr[dev] = true;
            }
            gemm_dmma_tma_kernel<T><<<grid, 128, dmma_tma_smem, st>>>((int)M, (int)N, (int)K, C, ldc, ma, mb);
        } else {
            gemm_dmma_kernel<T><<<grid, 128, 0, st>>>((int)M, (int)N, (int)K, C, ldc, A, lda, B, ldb);
        }
        return cudaGetLastError();
    }
    int dev = 0;
    cudaGetDevice(&dev);
    static bool attr[64] = {};
    if (dev < 64 && !attr[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemm_kernel<SR, T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)G::smem_bytes);
        if (e != cudaSuccess) return e;
        attr[dev] = true;
    }
    dim3 grid((unsigned)((M + G::BM - 1) / G::BM), (unsigned)((N + G::BN - 1) / G::BN));
    gemm_kernel<SR, T><<<grid, 256, G::smem_bytes, st>>>((int)M, (int)N, (int)K, C, ldc, A, lda, B, ldb);
    return cudaGetLastError();
}

}  // namespace pp
