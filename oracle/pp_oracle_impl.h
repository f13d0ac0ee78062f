/*
 * pp_oracle_impl.h — the numeric body of the oracle, included once per (semiring, element type).
 *
 * TEST INFRASTRUCTURE ONLY (see pp_oracle.h).  Before each inclusion pp_oracle.c defines
 *   SRN                 name suffix, e.g. minplus_f32
 *   T                   element type
 *   SZERO, SONE         szero(s, T, Val(:N)), sone(s, T, Val(:N))
 *   SPLUS(a, b)         splus(s, a, b, Val(:N))      (x86 select semantics: vmin(x, y) = ifelse(x < y, x, y))
 *   SPROD(a, b)         sprod(s, a, b, Val(:N), Val(:N))
 *   SMULADD(a, b, c)    smuladd(s, a, b, c, Val(:N), Val(:N))
 *   SSTAR(a)            sstar(s, a)
 *   INTEGRAL            isintegral(s)
 * Matrices are column-major; element (i, j) of a matrix with leading dimension ld is at [i + j * ld].
 */
#define PPO_CAT2(a, b) a##_##b
#define PPO_CAT(a, b) PPO_CAT2(a, b)
#define FN(name) PPO_CAT(name, SRN)

/* ===== dense kernels ===== */

/* C (m x n) <- C (+) A (m x k) (x) B (k x n): generic sgemx2!, src/CPU/dense/sgemx.jl:606-635
   (loop order: column of C, then k, then row) */
static void FN(gemm)(int64_t m, int64_t n, int64_t k, T *C, int64_t ldc, const T *A, int64_t lda, const T *B,
                     int64_t ldb, int nt) {
    int64_t c;
#pragma omp parallel for schedule(static) num_threads(nt) if (nt > 1 && m * n * k > (int64_t)1 << 18)
    for (c = 0; c < n; c++) {
        T *Cc = C + c * ldc;
        for (int64_t j = 0; j < k; j++) {
            const T b = B[j + c * ldb];
            const T *Aj = A + j * lda;
            for (int64_t i = 0; i < m; i++) Cc[i] = SMULADD(Aj[i], b, Cc[i]);
        }
    }
}

/* B (n x m) <- A* B with A n x n triangular: generic strsx2! side :L, src/CPU/dense/strsx.jl:596-631.
   lower = uplo :L (forward), unit = diag :U */
static void FN(tri_left)(const T *A, int64_t lda, int64_t n, int lower, int unit, T *B, int64_t ldb, int64_t m) {
    for (int64_t j = 0; j < m; j++) {
        T *Bj = B + j * ldb;
        for (int64_t pp = 0; pp < n; pp++) {
            const int64_t p = lower ? pp : n - 1 - pp;
            if (!unit && !INTEGRAL) Bj[p] = SPROD(SSTAR(A[p + p * lda]), Bj[p]);
            const T bpj = Bj[p];
            if (lower) {
                for (int64_t q = p + 1; q < n; q++) Bj[q] = SMULADD(A[q + p * lda], bpj, Bj[q]);
            } else {
                for (int64_t q = 0; q < p; q++) Bj[q] = SMULADD(A[q + p * lda], bpj, Bj[q]);
            }
        }
    }
}

/* B (m x n) <- B A* with A n x n triangular: generic strsx2! side :R, src/CPU/dense/strsx.jl:633-672.
   upper = uplo :U (forward), unit = diag :U */
static void FN(tri_right)(const T *A, int64_t lda, int64_t n, int upper, int unit, T *B, int64_t ldb, int64_t m) {
    for (int64_t pp = 0; pp < n; pp++) {
        const int64_t p = upper ? pp : n - 1 - pp;
        T *Bp = B + p * ldb;
        if (!unit && !INTEGRAL) {
            const T s = SSTAR(A[p + p * lda]);
            for (int64_t i = 0; i < m; i++) Bp[i] = SPROD(Bp[i], s);
        }
        const int64_t q0 = upper ? p + 1 : 0, q1 = upper ? n : p;
        for (int64_t q = q0; q < q1; q++) {
            const T apq = A[p + q * lda];
            T *Bq = B + q * ldb;
            for (int64_t i = 0; i < m; i++) Bq[i] = SMULADD(Bp[i], apq, Bq[i]);
        }
    }
}

/* scalar sgetrf2!, src/CPU/dense/sgetrf.jl:151-175 */
static void FN(getrf2)(T *A, int64_t lda, int64_t n) {
    for (int64_t i = 0; i < n; i++) {
        if (!INTEGRAL) {
            const T s = SSTAR(A[i + i * lda]);
            for (int64_t k = i + 1; k < n; k++) A[k + i * lda] = SPROD(A[k + i * lda], s);
        }
        for (int64_t j = i + 1; j < n; j++) {
            const T aij = A[i + j * lda];
            T *Aj = A + j * lda;
            const T *Ai = A + i * lda;
            for (int64_t q = i + 1; q < n; q++) Aj[q] = SMULADD(Ai[q], aij, Aj[q]);
        }
    }
}

/* sgetrf! / blocked sgetrf_mt!, src/CPU/dense/sgetrf.jl:5-68 (SLU_NB = 128) */
static void FN(getrf)(T *A, int64_t lda, int64_t n, int nt) {
    const int64_t NB = 128;
    if (n <= NB) {
        FN(getrf2)(A, lda, n);
        return;
    }
    for (int64_t k = 0; k < n; k += NB) {
        const int64_t b = (n - k < NB) ? n - k : NB;
        T *Akk = A + k + k * lda;
        FN(getrf2)(Akk, lda, b);
        if (k + b < n) {
            T *Akn = A + k + (k + b) * lda;
            T *Ank = A + (k + b) + k * lda;
            T *Ann = A + (k + b) + (k + b) * lda;
            FN(tri_left)(Akk, lda, b, 1, 1, Akn, lda, n - k - b);  /* Akn <- Lkk* Akn */
            FN(tri_right)(Akk, lda, b, 1, 0, Ank, lda, n - k - b); /* Ank <- Ank Ukk* */
            FN(gemm)(n - k - b, n - k - b, b, Ann, lda, Ank, lda, Akn, lda, nt);
        }
    }
}

/* strsx_st! (side :L, uplo :U, diag :N) and (side :R, uplo :U, diag :N) as strtri_st! uses them;
   the blocking of the reference only reorders the same products, so the unblocked strsx2! is used. */

/* recursive dense star of an upper triangular block: strtri_st!, src/CPU/dense/strtri.jl:21-54,
   leaf strtri2!(::Val{:U}, ::Val{:N}), :237-269 (STRTRI_LEAF = 128) */
static void FN(strtri_upper)(T *A, int64_t lda, int64_t n) {
    if (n <= 128) {
        for (int64_t k = 0; k < n; k++) A[k + k * lda] = SSTAR(A[k + k * lda]);
        for (int64_t j = n - 1; j >= 0; j--) {
            T *Aj = A + j * lda;
            if (!INTEGRAL)
                for (int64_t i = 0; i < j; i++) Aj[i] = SPROD(Aj[i], Aj[j]);
            for (int64_t k = j - 1; k >= 0; k--) {
                if (!INTEGRAL) Aj[k] = SPROD(A[k + k * lda], Aj[k]);
                const T akj = Aj[k];
                const T *Ak = A + k * lda;
                for (int64_t q = 0; q < k; q++) Aj[q] = SMULADD(Ak[q], akj, Aj[q]);
            }
        }
        return;
    }
    const int64_t m = n >> 1;
    T *A11 = A, *A22 = A + m + m * lda, *A12 = A + m * lda;
    FN(tri_left)(A11, lda, m, 0, 0, A12, lda, n - m);  /* A12 <- A11* A12 */
    FN(tri_right)(A22, lda, n - m, 1, 0, A12, lda, m); /* A12 <- A12 A22* */
    FN(strtri_upper)(A11, lda, m);
    FN(strtri_upper)(A22, lda, n - m);
}

/* ===== assembly: scopyto_st! / scopyto_loop!, src/CPU/chordal_slu.jl:120-141, 221-321 ===== */

static int FN(assemble)(const ppo_struct *S, const int64_t *colptr, const int64_t *rowval, const T *nzval, T *LD,
                        T *LL, T *UD, T *UL, T *Nval) {
    const int64_t n = S->n, nf = S->nf;
    const int64_t nD = S->Dptr[nf], nL = S->Lptr[nf];
    for (int64_t i = 0; i < nD; i++) LD[i] = UD[i] = SZERO;
    for (int64_t i = 0; i < nL; i++) LL[i] = UL[i] = SZERO;
    for (int64_t i = 0; i < S->nN; i++) Nval[i] = SZERO;
    int64_t *ind = (int64_t *)malloc(sizeof(int64_t) * (n > 0 ? n : 1));
    int64_t *cur = (int64_t *)malloc(sizeof(int64_t) * (nf > 0 ? nf : 1));
    if (!ind || !cur) {
        free(ind);
        free(cur);
        return -2;
    }
    for (int64_t i = 0; i < n; i++) ind[i] = -1;
    for (int64_t f = 0; f < nf; f++) cur[f] = S->Sptr[f];
    for (int64_t f = 0; f < nf; f++) {
        const int64_t rlo = S->Rptr[f], rhi = S->Rptr[f + 1] - 1, nn = rhi - rlo + 1;
        const int64_t sstrt = S->Sptr[f], sstop = S->Sptr[f + 1] - 1, na = sstop - sstrt + 1;
        const int64_t Dp = S->Dptr[f], Lp = S->Lptr[f];
        const int64_t jstrt = S->Bptr[S->fcc[f]];
        for (int64_t q = sstrt; q <= sstop; q++) ind[S->Stgt[q]] = q - sstrt;
        for (int64_t j = rlo; j <= rhi; j++) {
            const int64_t c = S->perm[j];
            for (int64_t r = S->Nptr[j]; r < S->Nptr[j + 1]; r++) ind[S->Ntgt[r]] = r;
            for (int64_t p = colptr[c]; p < colptr[c + 1]; p++) {
                const int64_t i = S->invp[rowval[p]];
                if (i < jstrt) {
                    const int64_t r = ind[i];
                    if (r >= 0) Nval[r] = nzval[p];
                } else if (rlo <= i && i <= rhi) {
                    const int64_t o = Dp + (i - rlo) + (j - rlo) * nn;
                    LD[o] = nzval[p];
                    UD[o] = nzval[p];
                } else if (i > j) {
                    const int64_t k = ind[i];
                    if (k >= 0) LL[Lp + k + (j - rlo) * na] = nzval[p];
                } else {
                    const int64_t g = S->idx[i];
                    const int64_t qstrt = S->Sptr[g], qstop = S->Sptr[g + 1];
                    int64_t q = cur[g];
                    while (q < qstop && S->Stgt[q] < j) q++;
                    cur[g] = q;
                    if (q < qstop && S->Stgt[q] == j) {
                        const int64_t mlo = S->Rptr[g], mm = S->Rptr[g + 1] - mlo;
                        UL[S->Lptr[g] + (i - mlo) + (q - qstrt) * mm] = nzval[p];
                    }
                }
            }
            for (int64_t r = S->Nptr[j]; r < S->Nptr[j + 1]; r++) ind[S->Ntgt[r]] = -1;
        }
        for (int64_t q = sstrt; q <= sstop; q++) ind[S->Stgt[q]] = -1;
    }
    free(ind);
    free(cur);
    return 0;
}

/* ===== factorization: sgetrf_mt!, src/CPU/chordal/sgetrf.jl:9-290 ===== */

static int FN(factor)(const ppo_struct *S, T *LD, T *LL, T *UD, T *UL, int nt) {
    const int64_t nf = S->nf;
    /* workspace sizes: the largest front and the deepest update-matrix stack */
    int64_t maxnj = 1, depth = 0, maxdepth = 1;
    int64_t *Mptr = (int64_t *)malloc(sizeof(int64_t) * (nf + 2));
    if (!Mptr) return -2;
    {
        int64_t ns = 0;
        Mptr[0] = 0;
        for (int64_t j = 0; j < nf; j++) {
            const int64_t nn = S->Rptr[j + 1] - S->Rptr[j], na = S->Sptr[j + 1] - S->Sptr[j];
            if (nn + na > maxnj) maxnj = nn + na;
            for (int64_t c = S->chdptr[j]; c < S->chdptr[j + 1]; c++) {
                ns--;
                depth = Mptr[ns];
            }
            if (na > 0) {
                Mptr[ns + 1] = Mptr[ns] + na * na;
                ns++;
                depth = Mptr[ns];
                if (depth > maxdepth) maxdepth = depth;
            }
        }
    }
    T *Fval = (T *)malloc(sizeof(T) * maxnj * maxnj);
    T *Mval = (T *)malloc(sizeof(T) * maxdepth);
    if (!Fval || !Mval) {
        free(Fval);
        free(Mval);
        free(Mptr);
        return -2;
    }
    int64_t ns = 0;
    Mptr[0] = 0;
    for (int64_t j = 0; j < nf; j++) {
        const int64_t nn = S->Rptr[j + 1] - S->Rptr[j], na = S->Sptr[j + 1] - S->Sptr[j], nj = nn + na;
        const int64_t Dp = S->Dptr[j], Lp = S->Lptr[j];
        T *F = Fval;
        for (int64_t i = 0; i < nj * nj; i++) F[i] = SZERO;
        /* sgetrf_send! for the children, last first (the update matrices form a stack) */
        for (int64_t c = S->chdptr[j + 1] - 1; c >= S->chdptr[j]; c--) {
            const int64_t i = S->chdtgt[c];
            const int64_t nai = S->Sptr[i + 1] - S->Sptr[i];
            const int64_t *inj = S->rel + S->Sptr[i];
            const T *M = Mval + Mptr[ns - 1];
            for (int64_t w = 0; w < nai; w++) {
                const int64_t iw = inj[w];
                for (int64_t v = 0; v < nai; v++) {
                    const int64_t iv = inj[v];
                    F[iv + iw * nj] = SPLUS(F[iv + iw * nj], M[v + w * nai]);
                }
            }
            ns--;
        }
        if (nn == 1) {
            /* sgetrf_loop_1!, :153-255 */
            const T d11 = SPLUS(UD[Dp], F[0]);
            LD[Dp] = d11;
            UD[Dp] = d11;
            if (na > 0) {
                T *l21 = LL + Lp, *u12 = UL + Lp;
                for (int64_t i = 0; i < na; i++) {
                    l21[i] = SPLUS(l21[i], F[1 + i]);
                    u12[i] = SPLUS(u12[i], F[(1 + i) * nj]);
                }
                if (!INTEGRAL) {
                    const T ds = SSTAR(d11);
                    for (int64_t i = 0; i < na; i++) l21[i] = SPROD(l21[i], ds);
                }
                T *M = Mval + Mptr[ns];
                Mptr[ns + 1] = Mptr[ns] + na * na;
                ns++;
                for (int64_t cc = 0; cc < na; cc++)
                    for (int64_t r = 0; r < na; r++) M[r + cc * na] = F[(1 + r) + (1 + cc) * nj];
                /* sger_st!(s, N, N, :R, l21, u12, M): M[r, c] = smuladd(l21[r], u12[c], M[r, c]) */
                for (int64_t cc = 0; cc < na; cc++)
                    for (int64_t r = 0; r < na; r++) M[r + cc * na] = SMULADD(l21[r], u12[cc], M[r + cc * na]);
            }
        } else {
            /* sgetrf_loop!, :35-151 */
            T *L11 = LD + Dp, *U11 = UD + Dp, *L21 = LL + Lp, *U12 = UL + Lp;
            for (int64_t jj = 0; jj < nn; jj++)
                for (int64_t ii = 0; ii < nn; ii++) {
                    const int64_t o = ii + jj * nn;
                    L11[o] = (ii > jj) ? SPLUS(F[ii + jj * nj], L11[o]) : SPLUS(F[ii + jj * nj], U11[o]);
                }
            FN(getrf)(L11, nn, nn, nt);
            for (int64_t jj = 0; jj < nn; jj++)
                for (int64_t ii = 0; ii <= jj; ii++) U11[ii + jj * nn] = L11[ii + jj * nn];
            if (na > 0) {
                for (int64_t cc = 0; cc < nn; cc++)
                    for (int64_t r = 0; r < na; r++) L21[r + cc * na] = SPLUS(L21[r + cc * na], F[(nn + r) + cc * nj]);
                for (int64_t cc = 0; cc < na; cc++)
                    for (int64_t r = 0; r < nn; r++) U12[r + cc * nn] = SPLUS(U12[r + cc * nn], F[r + (nn + cc) * nj]);
                FN(tri_right)(L11, nn, nn, 1, 0, L21, na, na); /* L21 <- L21 U11* */
                FN(tri_left)(L11, nn, nn, 1, 1, U12, nn, na);  /* U12 <- L11* U12 */
                T *M = Mval + Mptr[ns];
                Mptr[ns + 1] = Mptr[ns] + na * na;
                ns++;
                for (int64_t cc = 0; cc < na; cc++)
                    for (int64_t r = 0; r < na; r++) M[r + cc * na] = F[(nn + r) + (nn + cc) * nj];
                FN(gemm)(na, na, nn, M, na, L21, na, U12, nn, nt);
            }
        }
    }
    free(Fval);
    free(Mval);
    free(Mptr);
    return 0;
}

/* ===== chordal solves: strsx_mt!, src/CPU/chordal/strsx.jl:79-126 ===== */

/* One front forward (strsx_fwd_upd!, :187-265): C1 <- D11* C1, C2 <- C2 (+) L21 C1.
   side_left: C is n x nrhs (rows are vertices); else C is nrhs x n (columns are vertices).
   uplo_lower: the triangle is L (Dval/Lval = LD/LL, L21 na x nn); else U (UD/UL, U12 nn x na). */
static void FN(front_fwd)(const ppo_struct *S, int64_t f, int side_left, int uplo_lower, int unit, const T *Dval,
                          const T *Lval, T *C, int64_t ldc, int64_t nrhs, T *M) {
    const int64_t rlo = S->Rptr[f], nn = S->Rptr[f + 1] - rlo;
    const int64_t *fsep = S->Stgt + S->Sptr[f];
    const int64_t na = S->Sptr[f + 1] - S->Sptr[f];
    const T *D11 = Dval + S->Dptr[f], *L21 = Lval + S->Lptr[f];
    if (side_left) {
        T *C1 = C + rlo;
        FN(tri_left)(D11, nn, nn, uplo_lower, unit, C1, ldc, nrhs);
        if (na > 0) {
            /* M2 (na x nrhs) <- L21 (na x nn) C1 */
            for (int64_t i = 0; i < na * nrhs; i++) M[i] = SZERO;
            for (int64_t k = 0; k < nrhs; k++)
                for (int64_t j = 0; j < nn; j++) {
                    const T b = C1[j + k * ldc];
                    for (int64_t i = 0; i < na; i++) M[i + k * na] = SMULADD(L21[i + j * na], b, M[i + k * na]);
                }
            for (int64_t k = 0; k < nrhs; k++)
                for (int64_t i = 0; i < na; i++) C[fsep[i] + k * ldc] = SPLUS(C[fsep[i] + k * ldc], M[i + k * na]);
        }
    } else {
        T *C1 = C + rlo * ldc;
        FN(tri_right)(D11, nn, nn, !uplo_lower, unit, C1, ldc, nrhs);
        if (na > 0) {
            /* M2 (nrhs x na) <- C1 (nrhs x nn) U12 (nn x na) */
            for (int64_t i = 0; i < na * nrhs; i++) M[i] = SZERO;
            for (int64_t c = 0; c < na; c++)
                for (int64_t j = 0; j < nn; j++) {
                    const T b = L21[j + c * nn];
                    const T *C1j = C1 + j * ldc;
                    for (int64_t k = 0; k < nrhs; k++) M[k + c * nrhs] = SMULADD(C1j[k], b, M[k + c * nrhs]);
                }
            for (int64_t c = 0; c < na; c++) {
                T *Cc = C + fsep[c] * ldc;
                for (int64_t k = 0; k < nrhs; k++) Cc[k] = SPLUS(Cc[k], M[k + c * nrhs]);
            }
        }
    }
}

/* One front backward (strsx_bwd_upd!, :783-830): C1 <- C1 (+) U12 C2, C1 <- D11* C1. */
static void FN(front_bwd)(const ppo_struct *S, int64_t f, int side_left, int uplo_lower, int unit, const T *Dval,
                          const T *Lval, T *C, int64_t ldc, int64_t nrhs, T *M) {
    const int64_t rlo = S->Rptr[f], nn = S->Rptr[f + 1] - rlo;
    const int64_t *fsep = S->Stgt + S->Sptr[f];
    const int64_t na = S->Sptr[f + 1] - S->Sptr[f];
    const T *D11 = Dval + S->Dptr[f], *U12 = Lval + S->Lptr[f];
    if (side_left) {
        T *C1 = C + rlo;
        if (na > 0) {
            /* M2 <- C2 (gather); C1 (nn x nrhs) <- U12 (nn x na) M2 (+) C1 */
            for (int64_t k = 0; k < nrhs; k++)
                for (int64_t i = 0; i < na; i++) M[i + k * na] = C[fsep[i] + k * ldc];
            for (int64_t k = 0; k < nrhs; k++)
                for (int64_t j = 0; j < na; j++) {
                    const T b = M[j + k * na];
                    for (int64_t i = 0; i < nn; i++) C1[i + k * ldc] = SMULADD(U12[i + j * nn], b, C1[i + k * ldc]);
                }
        }
        FN(tri_left)(D11, nn, nn, uplo_lower, unit, C1, ldc, nrhs);
    } else {
        T *C1 = C + rlo * ldc;
        if (na > 0) {
            /* M2 <- C2 (gather); C1 (nrhs x nn) <- M2 (nrhs x na) U12 (na x nn) (+) C1 */
            for (int64_t c = 0; c < na; c++)
                for (int64_t k = 0; k < nrhs; k++) M[k + c * nrhs] = C[k + fsep[c] * ldc];
            for (int64_t j = 0; j < nn; j++) {
                T *C1j = C1 + j * ldc;
                for (int64_t c = 0; c < na; c++) {
                    const T b = U12[c + j * na];
                    for (int64_t k = 0; k < nrhs; k++) C1j[k] = SMULADD(M[k + c * nrhs], b, C1j[k]);
                }
            }
        }
        FN(tri_right)(D11, nn, nn, !uplo_lower, unit, C1, ldc, nrhs);
    }
}

/* strsx_mt! over fronts fstrt..fstop: forward when isforward(uplo, :N, side) */
static void FN(chordal_strsx)(const ppo_struct *S, int side_left, int uplo_lower, int unit, const T *Dval,
                              const T *Lval, T *C, int64_t ldc, int64_t nrhs, int64_t fstrt, int64_t fstop, T *M) {
    const int forward = (side_left == uplo_lower);
    if (forward) {
        for (int64_t f = fstrt; f <= fstop; f++) FN(front_fwd)(S, f, side_left, uplo_lower, unit, Dval, Lval, C, ldc, nrhs, M);
    } else {
        for (int64_t f = fstop; f >= fstrt; f--) FN(front_bwd)(S, f, side_left, uplo_lower, unit, Dval, Lval, C, ldc, nrhs, M);
    }
}

/* chordal sgetrs_mt!, src/CPU/chordal/sgetrs.jl:29-51: lmul! applies L* then U*; rmul! U* then L* */
static void FN(chordal_sgetrs)(const ppo_struct *S, int side_left, const T *LD, const T *LL, const T *UD,
                               const T *UL, T *C, int64_t ldc, int64_t nrhs, int64_t fstrt, int64_t fstop, T *M) {
    if (side_left) {
        FN(chordal_strsx)(S, 1, 1, 1, LD, LL, C, ldc, nrhs, fstrt, fstop, M);
        FN(chordal_strsx)(S, 1, 0, 0, UD, UL, C, ldc, nrhs, fstrt, fstop, M);
    } else {
        FN(chordal_strsx)(S, 0, 0, 0, UD, UL, C, ldc, nrhs, fstrt, fstop, M);
        FN(chordal_strsx)(S, 0, 1, 1, LD, LL, C, ldc, nrhs, fstrt, fstop, M);
    }
}

/* coupling products sgemx_sparse_st!, src/CPU/sparse/sgemx.jl:101-113 (side :R) and :193-213 (side :L) */
static void FN(coupling)(const ppo_struct *S, int side_left, const T *Nval, T *C, int64_t ldc, int64_t nrhs,
                         int64_t jstrt, int64_t jstop) {
    if (side_left) {
        for (int64_t k = 0; k < nrhs; k++)
            for (int64_t j = jstrt; j <= jstop; j++) {
                const T u = C[j + k * ldc];
                for (int64_t p = S->Nptr[j]; p < S->Nptr[j + 1]; p++) {
                    const int64_t i = S->Ntgt[p];
                    C[i + k * ldc] = SMULADD(Nval[p], u, C[i + k * ldc]);
                }
            }
    } else {
        for (int64_t j = jstrt; j <= jstop; j++)
            for (int64_t p = S->Nptr[j]; p < S->Nptr[j + 1]; p++) {
                const int64_t kk = S->Ntgt[p];
                const T v = Nval[p];
                for (int64_t i = 0; i < nrhs; i++) C[i + j * ldc] = SMULADD(C[i + kk * ldc], v, C[i + j * ldc]);
            }
    }
}

/* blocked sgetrs_mt!, src/CPU/blocked/sgetrs.jl:203-255: components in order (rmul!) or reversed (lmul!) */
static void FN(blocked_sgetrs)(const ppo_struct *S, int side_left, const T *LD, const T *LL, const T *UD,
                               const T *UL, const T *Nval, T *C, int64_t ldc, int64_t nrhs, T *M) {
    if (!side_left) {
        for (int64_t c = 0; c < S->nB; c++) {
            FN(coupling)(S, 0, Nval, C, ldc, nrhs, S->Bptr[c], S->Bptr[c + 1] - 1);
            FN(chordal_sgetrs)(S, 0, LD, LL, UD, UL, C, ldc, nrhs, S->Fptr[c], S->Fptr[c + 1] - 1, M);
        }
    } else {
        for (int64_t c = S->nB - 1; c >= 0; c--) {
            FN(chordal_sgetrs)(S, 1, LD, LL, UD, UL, C, ldc, nrhs, S->Fptr[c], S->Fptr[c + 1] - 1, M);
            FN(coupling)(S, 1, Nval, C, ldc, nrhs, S->Bptr[c], S->Bptr[c + 1] - 1);
        }
    }
}

static int64_t FN(max_na)(const ppo_struct *S) {
    int64_t m = 1;
    for (int64_t f = 0; f < S->nf; f++) {
        const int64_t na = S->Sptr[f + 1] - S->Sptr[f];
        if (na > m) m = na;
    }
    return m;
}

/* sgetrs! on a ChordalSLU, src/CPU/chordal_slu.jl:337-377, with the right-hand sides split over
   threads as in src/CPU/blocked/sgetrs.jl:171-194 */
static int FN(sgetrs)(const ppo_struct *S, int side_left, const T *LD, const T *LL, const T *UD, const T *UL,
                      const T *Nval, T *B, int64_t ldb, int64_t k, int nt) {
    const int64_t n = S->n;
    /* permute into factor order: lmul! permuterows!(B, rinvp), rmul! permutecols!(B, cinvp) */
    T *W = (T *)malloc(sizeof(T) * (n > 0 ? n : 1) * (k > 0 ? k : 1));
    if (!W) return -2;
    if (side_left) {
        for (int64_t c = 0; c < k; c++)
            for (int64_t i = 0; i < n; i++) W[S->invp[i] + c * n] = B[i + c * ldb];
    } else {
        for (int64_t j = 0; j < n; j++)
            for (int64_t c = 0; c < k; c++) W[c + S->invp[j] * k] = B[c + j * ldb];
    }
    const int64_t maxna = FN(max_na)(S);
    int tasks = (nt > 1 && k >= 4 * nt) ? nt : 1;
    int fail = 0;
    int t;
#pragma omp parallel for schedule(static, 1) num_threads(tasks) if (tasks > 1)
    for (t = 0; t < tasks; t++) {
        const int64_t tsize = k / tasks;
        const int64_t c0 = t * tsize, c1 = (t < tasks - 1) ? (t + 1) * tsize : k;
        const int64_t nr = c1 - c0;
        T *M = (T *)malloc(sizeof(T) * maxna * (nr > 0 ? nr : 1));
        if (!M) {
#pragma omp atomic write
            fail = 1;
        } else {
            if (side_left)
                FN(blocked_sgetrs)(S, 1, LD, LL, UD, UL, Nval, W + c0 * n, n, nr, M);
            else {
                /* the k x n block rows c0..c1-1: copy to a compact nr x n buffer */
                T *Wt = (T *)malloc(sizeof(T) * nr * (n > 0 ? n : 1));
                if (!Wt) {
#pragma omp atomic write
                    fail = 1;
                } else {
                    for (int64_t j = 0; j < n; j++)
                        for (int64_t c = 0; c < nr; c++) Wt[c + j * nr] = W[(c0 + c) + j * k];
                    FN(blocked_sgetrs)(S, 0, LD, LL, UD, UL, Nval, Wt, nr, nr, M);
                    for (int64_t j = 0; j < n; j++)
                        for (int64_t c = 0; c < nr; c++) W[(c0 + c) + j * k] = Wt[c + j * nr];
                    free(Wt);
                }
            }
            free(M);
        }
    }
    if (!fail) {
        /* permute back: lmul! permuterows!(B, cperm), rmul! permutecols!(B, rperm) */
        if (side_left) {
            for (int64_t c = 0; c < k; c++)
                for (int64_t i = 0; i < n; i++) B[S->perm[i] + c * ldb] = W[i + c * n];
        } else {
            for (int64_t j = 0; j < n; j++)
                for (int64_t c = 0; c < k; c++) B[c + S->perm[j] * ldb] = W[c + j * k];
        }
    }
    free(W);
    return fail ? -2 : 0;
}

/* ===== star: sgetri!, src/CPU/chordal_slu.jl:501-513 ===== */

/* strtri_fwd! for the upper factor (UPLO :U, DIAG :N), src/CPU/chordal/strtri.jl:171-319.
   X is n x n column-major (ldx = n); rows rstrt..rstop are the descendants of f in the band. */
static void FN(strtri_front)(const ppo_struct *S, const T *UD, const T *UL, T *X, int64_t ldx, int64_t f,
                             int64_t rstrt, int64_t rstop, T *M) {
    const int64_t Rp = S->Rptr[f], nn = S->Rptr[f + 1] - Rp;
    const int64_t *fsep = S->Stgt + S->Sptr[f];
    const int64_t na = S->Sptr[f + 1] - S->Sptr[f];
    const T *D11 = UD + S->Dptr[f], *U12 = UL + S->Lptr[f];
    const int64_t nr = rstop - rstrt + 1;
    if (Rp <= rstop) {
        /* X11 <- D11 (upper triangle), X11 <- X11* */
        T *X11 = X + Rp + Rp * ldx;
        for (int64_t j = 0; j < nn; j++)
            for (int64_t i = 0; i <= j; i++) X11[i + j * ldx] = D11[i + j * nn];
        FN(strtri_upper)(X11, ldx, nn);
    }
    const int64_t qstop = (Rp - 1 < rstop) ? Rp - 1 : rstop;
    if (rstrt <= qstop) {
        /* X01 <- X01 D11* */
        FN(tri_right)(D11, nn, nn, 1, 0, X + rstrt + Rp * ldx, ldx, qstop - rstrt + 1);
    }
    if (na > 0) {
        /* M2 (nr x na) <- X1 (nr x nn) U12 (nn x na); X[fdsc, fsep] <- X[fdsc, fsep] (+) M2 */
        for (int64_t i = 0; i < nr * na; i++) M[i] = SZERO;
        FN(gemm)(nr, na, nn, M, nr, X + rstrt + Rp * ldx, ldx, U12, nn, 1);
        for (int64_t c = 0; c < na; c++) {
            T *Xc = X + rstrt + fsep[c] * ldx;
            for (int64_t i = 0; i < nr; i++) Xc[i] = SPLUS(Xc[i], M[i + c * nr]);
        }
    }
}

/* strtri_band!, src/CPU/chordal/strtri.jl:118-167 */
static void FN(strtri_band)(const ppo_struct *S, const T *UD, const T *UL, T *X, int64_t ldx, int64_t fstrt,
                            int64_t fstop, T *M) {
    const int64_t bstrt = S->Rptr[fstrt], bstop = S->Rptr[fstop + 1] - 1;
    for (int64_t j = 0; j < S->n; j++)
        for (int64_t i = bstrt; i <= bstop; i++) X[i + j * ldx] = SZERO;
    for (int64_t f = fstrt; f < S->nf; f++) {
        int64_t rstrt = S->Rptr[S->fdsc[f]], rstop = S->Rptr[f + 1] - 1;
        if (rstrt < bstrt) rstrt = bstrt;
        if (rstop > bstop) rstop = bstop;
        if (rstrt <= rstop) FN(strtri_front)(S, UD, UL, X, ldx, f, rstrt, rstop, M);
    }
}

/* sgetri_reach!, src/CPU/blocked/sgetri.jl:366-417 */
static int64_t FN(reach)(const ppo_struct *S, int64_t *anc, int64_t *mark, int64_t *stack, int64_t tag, int64_t d) {
    int64_t top = S->nB, head = 0;
    anc[head] = d;
    mark[d] = tag;
    stack[head] = S->Nptr[S->Bptr[d]];
    while (head >= 0) {
        const int64_t c = anc[head];
        int64_t p = stack[head];
        const int64_t pstop = S->Nptr[S->Bptr[c + 1]];
        int64_t b = -1;
        while (p < pstop) {
            const int64_t a = S->fcc[S->idx[S->Ntgt[p]]];
            p++;
            if (mark[a] != tag) {
                b = a;
                break;
            }
        }
        stack[head] = p;
        if (b >= 0) {
            mark[b] = tag;
            head++;
            anc[head] = b;
            stack[head] = S->Nptr[S->Bptr[b]];
        } else {
            head--;
            top--;
            anc[top] = c;
        }
    }
    return top;
}

static int FN(star)(const ppo_struct *S, const T *LD, const T *LL, const T *UD, const T *UL, const T *Nval, T *C,
                    int nt) {
    const int64_t n = S->n, nf = S->nf;
    if (n == 0) return 0;
    T *X = (T *)malloc(sizeof(T) * n * n);
    if (!X) return -2;
    const int64_t maxna = FN(max_na)(S);
    int fail = 0;
    /* X <- U*: bands of whole fronts (strtri_mt!, :18-89); each row is computed independently */
    {
        int64_t nb = nt > 1 ? 4 * nt : 1;
        int64_t bs = (n + nb - 1) / nb;
        int64_t *bptr = (int64_t *)malloc(sizeof(int64_t) * (nf + 2));
        int64_t nbands = 0, strt = 0;
        bptr[0] = 0;
        for (int64_t f = 0; f < nf; f++) {
            const int64_t stop = S->Rptr[f + 1];
            if (stop - strt >= bs) {
                bptr[++nbands] = f + 1;
                strt = stop;
            }
        }
        if (strt < n) bptr[++nbands] = nf;
        int64_t b;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nt) if (nt > 1)
        for (b = 0; b < nbands; b++) {
            const int64_t fs = bptr[b], fe = bptr[b + 1] - 1;
            int64_t rows = S->Rptr[fe + 1] - S->Rptr[fs];
            T *M = (T *)malloc(sizeof(T) * (rows > 0 ? rows : 1) * maxna);
            if (!M) {
#pragma omp atomic write
                fail = 1;
            } else {
                FN(strtri_band)(S, UD, UL, X, n, fs, fe, M);
                free(M);
            }
        }
        free(bptr);
    }
    /* X <- X L*: strsx_mt!(R, N, U(nit), L) over all rows, rows split over threads */
    if (!fail) {
        int tasks = nt > 1 ? nt : 1;
        int t;
#pragma omp parallel for schedule(static, 1) num_threads(tasks) if (tasks > 1)
        for (t = 0; t < tasks; t++) {
            const int64_t r0 = n * t / tasks, r1 = n * (t + 1) / tasks;
            if (r1 > r0) {
                T *M = (T *)malloc(sizeof(T) * (r1 - r0) * maxna);
                if (!M) {
#pragma omp atomic write
                    fail = 1;
                } else {
                    FN(chordal_strsx)(S, 0, 1, 1, LD, LL, X + r0, n, r1 - r0, 0, nf - 1, M);
                    free(M);
                }
            }
        }
    }
    /* off-diagonal component blocks: sgetri_offd!, src/CPU/blocked/sgetri.jl:300-362 */
    if (!fail && S->Nptr[n] > 0) {
        int64_t *anc = (int64_t *)malloc(sizeof(int64_t) * S->nB);
        int64_t *mark = (int64_t *)malloc(sizeof(int64_t) * S->nB);
        int64_t *stack = (int64_t *)malloc(sizeof(int64_t) * S->nB);
        T *M = (T *)malloc(sizeof(T) * maxna * n);
        if (!anc || !mark || !stack || !M) fail = 1;
        if (!fail) {
            for (int64_t c = 0; c < S->nB; c++) mark[c] = -1;
            for (int64_t d = 0; d < S->nB; d++) {
                const int64_t dstrt = S->Bptr[d], dstop = S->Bptr[d + 1] - 1;
                if (S->Nptr[dstrt] < S->Nptr[dstop + 1]) {
                    T *Cd = X + dstrt * n;
                    const int64_t nd = dstop - dstrt + 1;
                    const int64_t tstrt = FN(reach)(S, anc, mark, stack, d, d);
                    for (int64_t tt = tstrt; tt < S->nB; tt++) {
                        const int64_t c = anc[tt];
                        const int64_t jstrt = S->Bptr[c], jstop = S->Bptr[c + 1] - 1;
                        if (c != d)
                            FN(chordal_sgetrs)(S, 1, LD, LL, UD, UL, Cd, n, nd, S->Fptr[c], S->Fptr[c + 1] - 1, M);
                        if (S->Nptr[jstrt] < S->Nptr[jstop + 1]) FN(coupling)(S, 1, Nval, Cd, n, nd, jstrt, jstop);
                    }
                }
            }
        }
        free(anc);
        free(mark);
        free(stack);
        free(M);
    }
    /* C <- P^-1 X Q^-1: C[rperm[i], cperm[j]] = X[i, j] (permuterowscols!, src/CPU/utils.jl:261-319) */
    if (!fail) {
        int64_t j;
#pragma omp parallel for schedule(static) num_threads(nt) if (nt > 1)
        for (j = 0; j < n; j++) {
            T *Cj = C + S->perm[j] * n;
            const T *Xj = X + j * n;
            for (int64_t i = 0; i < n; i++) Cj[S->perm[i]] = Xj[i];
        }
    }
    free(X);
    return fail ? -2 : 0;
}

#undef FN
