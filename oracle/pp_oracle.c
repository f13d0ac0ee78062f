/*
 * pp_oracle.c — the oracle's semirings, structure derivation and dispatch.
 *
 * TEST INFRASTRUCTURE ONLY (see pp_oracle.h): the checker for the B200 library and the timed CPU
 * baseline.  Nothing in the product links this file.
 *
 * Semirings (the files in src/CPU/semiring/, with Julia's x86 select semantics vmin(x, y) = ifelse(x < y, x, y)
 * and vmax(x, y) = ifelse(x > y, x, y), src/CPU/semiring/semiring.jl:124-138):
 *   MinPlus  (min, +)   zero +Inf, one 0,    star a >= 0 ? 0 : -Inf     tropical.jl:84-218
 *   MaxPlus  (max, +)   zero -Inf, one 0,    star 0 >= a ? 0 : +Inf     (DualQuantale{MinPlus})
 *   MaxMin   (max, min) zero -Inf, one +Inf, star one, integral         bottleneck.jl, semiring.jl:409-424
 *   MinMax   (min, max) zero +Inf, one -Inf, star one, integral
 *   MaxProd  (max, *)   zero 0,    one 1,    star 1 >= a ? 1 : +Inf     (DualQuantale{MinProd})
 *   PlusProd (+, *)     zero 0,    one 1,    star a < 1 ? 1/(1-a) : Inf real.jl:17-66 (smuladd = muladd -> fma)
 *   OrAnd    (|, &)     zero 0,    one typemax(Int32), integral         boolean.jl:31-79, semiring.jl:293-299
 * A floating product that is NaN (Inf + -Inf, Inf * 0) is szero (tropical.jl:164-182); smuladd on x86
 * is splus(a + b, c) (tropical.jl:188-195), which keeps c when a + b is NaN.
 *
 * MinPlus over Int32: the reference's sprod is a wrapping a + b (tropical.jl:148-150), under which the
 * typemax(Int32) "no path" sentinel overflows.  This build defines Int32 MinPlus on [0, typemax(Int32)]
 * with a saturating product (the exact sum clamped to typemax, so the sentinel absorbs); the device
 * library uses the same definition.
 */
#include "pp_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

static inline float vminf_(float x, float y) { return x < y ? x : y; }
static inline float vmaxf_(float x, float y) { return x > y ? x : y; }
static inline double vmind_(double x, double y) { return x < y ? x : y; }
static inline double vmaxd_(double x, double y) { return x > y ? x : y; }
static inline float nanto_f(float c, float z) { return c != c ? z : c; }
static inline double nanto_d(double c, double z) { return c != c ? z : c; }
static inline int32_t satadd_i32(int32_t a, int32_t b) {
    int64_t s = (int64_t)a + (int64_t)b;
    if (s > INT32_MAX) s = INT32_MAX;
    if (s < INT32_MIN) s = INT32_MIN;
    return (int32_t)s;
}
static inline int32_t mini_(int32_t x, int32_t y) { return x < y ? x : y; }

/* ---------------- MinPlus ---------------- */
#define SRN minplus_f32
#define T float
#define SZERO ((float)INFINITY)
#define SONE 0.0f
#define SPLUS(a, b) vminf_((a), (b))
#define SPROD(a, b) nanto_f((a) + (b), (float)INFINITY)
#define SMULADD(a, b, c) vminf_((a) + (b), (c))
#define SSTAR(a) ((a) >= 0.0f ? 0.0f : -(float)INFINITY)
#define INTEGRAL 0
#include "pp_oracle_impl.h"
#undef SRN
#undef T
#undef SZERO
#undef SONE
#undef SPLUS
#undef SPROD
#undef SMULADD
#undef SSTAR
#undef INTEGRAL

#define SRN minplus_f64
#define T double
#define SZERO ((double)INFINITY)
#define SONE 0.0
#define SPLUS(a, b) vmind_((a), (b))
#define SPROD(a, b) nanto_d((a) + (b), (double)INFINITY)
#define SMULADD(a, b, c) vmind_((a) + (b), (c))
#define SSTAR(a) ((a) >= 0.0 ? 0.0 : -(double)INFINITY)
#define INTEGRAL 0
#include "pp_oracle_impl.h"
#undef SRN
#undef T
#undef SZERO
#undef SONE
#undef SPLUS
#undef SPROD
#undef SMULADD
#undef SSTAR
#undef INTEGRAL

#define SRN minplus_i32
#define T int32_t
#define SZERO ((int32_t)INT32_MAX)
#define SONE 0
#define SPLUS(a, b) mini_((a), (b))
#define SPROD(a, b) satadd_i32((a), (b))
#define SMULADD(a, b, c) mini_(satadd_i32((a), (b)), (c))
#define SSTAR(a) ((a) >= 0 ? 0 : (int32_t)INT32_MIN)
#define INTEGRAL 0
#include "pp_oracle_impl.h"
#undef SRN
#undef T
#undef SZERO
#undef SONE
#undef SPLUS
#undef SPROD
#undef SMULADD
#undef SSTAR
#undef INTEGRAL

/* ---------------- MaxPlus ---------------- */
#define SRN maxplus_f32
#define T float
#define SZERO (-(float)INFINITY)
#define SONE 0.0f
#define SPLUS(a, b) vmaxf_((a), (b))
#define SPROD(a, b) nanto_f((a) + (b), -(float)INFINITY)
#define SMULADD(a, b, c) vmaxf_((a) + (b), (c))
#define SSTAR(a) (0.0f >= (a) ? 0.0f : (float)INFINITY)
#define INTEGRAL 0
#include "pp_oracle_impl.h"
#undef SRN
#undef T
#undef SZERO
#undef SONE
#undef SPLUS
#undef SPROD
#undef SMULADD
#undef SSTAR
#undef INTEGRAL

#define SRN maxplus_f64
#define T double
#define SZERO (-(double)INFINITY)
#define SONE 0.0
#define SPLUS(a, b) vmaxd_((a), (b))
#define SPROD(a, b) nanto_d((a) + (b), -(double)INFINITY)
#define SMULADD(a, b, c) vmaxd_((a) + (b), (c))
#define SSTAR(a) (0.0 >= (a) ? 0.0 : (double)INFINITY)
#define INTEGRAL 0
#include "pp_oracle_impl.h"
#undef SRN
#undef T
#undef SZERO
#undef SONE
#undef SPLUS
#undef SPROD
#undef SMULADD
#undef SSTAR
#undef INTEGRAL

/* ---------------- MaxMin ---------------- */
#define SRN maxmin_f32
#define T float
#define SZERO (-(float)INFINITY)
#define SONE ((float)INFINITY)
#define SPLUS(a, b) vmaxf_((a), (b))
#define SPROD(a, b) vminf_((a), (b))
#define SMULADD(a, b, c) vmaxf_(vminf_((a), (b)), (c))
#define SSTAR(a) ((float)INFINITY)
#define INTEGRAL 1
#include "pp_oracle_impl.h"
#undef SRN
#undef T
#undef SZERO
#undef SONE
#undef SPLUS
#undef SPROD
#undef SMULADD
#undef SSTAR
#undef INTEGRAL

#define SRN maxmin_f64
#define T double
#define SZERO (-(double)INFINITY)
#define SONE ((double)INFINITY)
#define SPLUS(a, b) vmaxd_((a), (b))
#define SPROD(a, b) vmind_((a), (b))
#define SMULADD(a, b, c) vmaxd_(vmind_((a), (b)), (c))
#define SSTAR(a) ((double)INFINITY)
#define INTEGRAL 1
#include "pp_oracle_impl.h"
#undef SRN
#undef T
#undef SZERO
#undef SONE
#undef SPLUS
#undef SPROD
#undef SMULADD
#undef SSTAR
#undef INTEGRAL

/* ---------------- MinMax ---------------- */
#define SRN minmax_f32
#define T float
#define SZERO ((float)INFINITY)
#define SONE (-(float)INFINITY)
#define SPLUS(a, b) vminf_((a), (b))
#define SPROD(a, b) vmaxf_((a), (b))
#define SMULADD(a, b, c) vminf_(vmaxf_((a), (b)), (c))
#define SSTAR(a) (-(float)INFINITY)
#define INTEGRAL 1
#include "pp_oracle_impl.h"
#undef SRN
#undef T
#undef SZERO
#undef SONE
#undef SPLUS
#undef SPROD
#undef SMULADD
#undef SSTAR
#undef INTEGRAL

#define SRN minmax_f64
#define T double
#define SZERO ((double)INFINITY)
#define SONE (-(double)INFINITY)
#define SPLUS(a, b) vmind_((a), (b))
#define SPROD(a, b) vmaxd_((a), (b))
#define SMULADD(a, b, c) vmind_(vmaxd_((a), (b)), (c))
#define SSTAR(a) (-(double)INFINITY)
#define INTEGRAL 1
#include "pp_oracle_impl.h"
#undef SRN
#undef T
#undef SZERO
#undef SONE
#undef SPLUS
#undef SPROD
#undef SMULADD
#undef SSTAR
#undef INTEGRAL

/* ---------------- MaxProd ---------------- */
#define SRN maxprod_f32
#define T float
#define SZERO 0.0f
#define SONE 1.0f
#define SPLUS(a, b) vmaxf_((a), (b))
#define SPROD(a, b) nanto_f((a) * (b), 0.0f)
#define SMULADD(a, b, c) vmaxf_((a) * (b), (c))
#define SSTAR(a) (1.0f >= (a) ? 1.0f : (float)INFINITY)
#define INTEGRAL 0
#include "pp_oracle_impl.h"
#undef SRN
#undef T
#undef SZERO
#undef SONE
#undef SPLUS
#undef SPROD
#undef SMULADD
#undef SSTAR
#undef INTEGRAL

#define SRN maxprod_f64
#define T double
#define SZERO 0.0
#define SONE 1.0
#define SPLUS(a, b) vmaxd_((a), (b))
#define SPROD(a, b) nanto_d((a) * (b), 0.0)
#define SMULADD(a, b, c) vmaxd_((a) * (b), (c))
#define SSTAR(a) (1.0 >= (a) ? 1.0 : (double)INFINITY)
#define INTEGRAL 0
#include "pp_oracle_impl.h"
#undef SRN
#undef T
#undef SZERO
#undef SONE
#undef SPLUS
#undef SPROD
#undef SMULADD
#undef SSTAR
#undef INTEGRAL

/* ---------------- PlusProd ---------------- */
#define SRN plusprod_f32
#define T float
#define SZERO 0.0f
#define SONE 1.0f
#define SPLUS(a, b) ((a) + (b))
#define SPROD(a, b) ((a) * (b))
#define SMULADD(a, b, c) fmaf((a), (b), (c))
#define SSTAR(a) ((a) < 1.0f ? 1.0f / (1.0f - (a)) : (float)INFINITY)
#define INTEGRAL 0
#include "pp_oracle_impl.h"
#undef SRN
#undef T
#undef SZERO
#undef SONE
#undef SPLUS
#undef SPROD
#undef SMULADD
#undef SSTAR
#undef INTEGRAL

#define SRN plusprod_f64
#define T double
#define SZERO 0.0
#define SONE 1.0
#define SPLUS(a, b) ((a) + (b))
#define SPROD(a, b) ((a) * (b))
#define SMULADD(a, b, c) fma((a), (b), (c))
#define SSTAR(a) ((a) < 1.0 ? 1.0 / (1.0 - (a)) : (double)INFINITY)
#define INTEGRAL 0
#include "pp_oracle_impl.h"
#undef SRN
#undef T
#undef SZERO
#undef SONE
#undef SPLUS
#undef SPROD
#undef SMULADD
#undef SSTAR
#undef INTEGRAL

/* ---------------- OrAnd ---------------- */
#define SRN orand_i32
#define T int32_t
#define SZERO 0
#define SONE ((int32_t)INT32_MAX)
#define SPLUS(a, b) ((a) | (b))
#define SPROD(a, b) ((a) & (b))
#define SMULADD(a, b, c) (((a) & (b)) | (c))
#define SSTAR(a) ((int32_t)INT32_MAX)
#define INTEGRAL 1
#include "pp_oracle_impl.h"
#undef SRN
#undef T
#undef SZERO
#undef SONE
#undef SPLUS
#undef SPROD
#undef SMULADD
#undef SSTAR
#undef INTEGRAL

/* ===== structure ===== */

static int64_t *dup64(const int64_t *a, int64_t n) {
    int64_t *b = (int64_t *)malloc(sizeof(int64_t) * (n > 0 ? n : 1));
    if (b && n > 0) memcpy(b, a, sizeof(int64_t) * n);
    return b;
}

void ppo_struct_free(ppo_struct *S) {
    if (!S) return;
    free(S->Rptr);
    free(S->Sptr);
    free(S->Stgt);
    free(S->Bptr);
    free(S->Fptr);
    free(S->Nptr);
    free(S->Ntgt);
    free(S->perm);
    free(S->invp);
    free(S->Dptr);
    free(S->Lptr);
    free(S->pnt);
    free(S->chdptr);
    free(S->chdtgt);
    free(S->rel);
    free(S->idx);
    free(S->fcc);
    free(S->fdsc);
    free(S);
}

/* Derives what CliqueTrees' ChordalSymbolic holds besides res/sep: the parent of a front is the front
   of its first separator vertex, rel maps each separator vertex to its position in the parent's bag
   (residual first, then separator), chd lists the children in increasing order, Dptr/Lptr are the
   running sums of nn^2 and nn*na (docs/site_factors.jl:147-156), fcc maps fronts to components
   (src/CPU/chordal_ssymbolic.jl:197-210) and fdsc is each front's first descendant
   (src/CPU/chordal/strtri.jl:37-50). */
ppo_struct *ppo_struct_new(int64_t n, int64_t nf, int64_t nB, const int64_t *Rptr, const int64_t *Sptr,
                           const int64_t *Stgt, const int64_t *Bptr, const int64_t *Fptr, const int64_t *Nptr,
                           const int64_t *Ntgt, const int64_t *perm) {
    ppo_struct *S = (ppo_struct *)calloc(1, sizeof(ppo_struct));
    if (!S) return NULL;
    S->n = n;
    S->nf = nf;
    S->nB = nB;
    S->nS = Sptr[nf];
    S->nN = Nptr[n];
    S->Rptr = dup64(Rptr, nf + 1);
    S->Sptr = dup64(Sptr, nf + 1);
    S->Stgt = dup64(Stgt, S->nS);
    S->Bptr = dup64(Bptr, nB + 1);
    S->Fptr = dup64(Fptr, nB + 1);
    S->Nptr = dup64(Nptr, n + 1);
    S->Ntgt = dup64(Ntgt, S->nN);
    S->perm = dup64(perm, n);
    S->invp = (int64_t *)malloc(sizeof(int64_t) * (n > 0 ? n : 1));
    S->Dptr = (int64_t *)malloc(sizeof(int64_t) * (nf + 1));
    S->Lptr = (int64_t *)malloc(sizeof(int64_t) * (nf + 1));
    S->pnt = (int64_t *)malloc(sizeof(int64_t) * (nf > 0 ? nf : 1));
    S->chdptr = (int64_t *)calloc(nf + 2, sizeof(int64_t));
    S->chdtgt = (int64_t *)malloc(sizeof(int64_t) * (nf > 0 ? nf : 1));
    S->rel = (int64_t *)malloc(sizeof(int64_t) * (S->nS > 0 ? S->nS : 1));
    S->idx = (int64_t *)malloc(sizeof(int64_t) * (n > 0 ? n : 1));
    S->fcc = (int64_t *)malloc(sizeof(int64_t) * (nf > 0 ? nf : 1));
    S->fdsc = (int64_t *)malloc(sizeof(int64_t) * (nf > 0 ? nf : 1));
    if (!S->Rptr || !S->Sptr || !S->Stgt || !S->Bptr || !S->Fptr || !S->Nptr || !S->Ntgt || !S->perm || !S->invp ||
        !S->Dptr || !S->Lptr || !S->pnt || !S->chdptr || !S->chdtgt || !S->rel || !S->idx || !S->fcc || !S->fdsc) {
        ppo_struct_free(S);
        return NULL;
    }
    for (int64_t i = 0; i < n; i++) S->invp[i] = -1;
    for (int64_t i = 0; i < n; i++) {
        if (perm[i] < 0 || perm[i] >= n || S->invp[perm[i]] >= 0) goto bad;
        S->invp[perm[i]] = i;
    }
    if (Rptr[0] != 0 || Rptr[nf] != n || Sptr[0] != 0) goto bad;
    S->Dptr[0] = S->Lptr[0] = 0;
    for (int64_t f = 0; f < nf; f++) {
        const int64_t nn = Rptr[f + 1] - Rptr[f], na = Sptr[f + 1] - Sptr[f];
        if (nn <= 0 || na < 0) goto bad;
        S->Dptr[f + 1] = S->Dptr[f] + nn * nn;
        S->Lptr[f + 1] = S->Lptr[f] + nn * na;
        for (int64_t v = Rptr[f]; v < Rptr[f + 1]; v++) S->idx[v] = f;
    }
    for (int64_t f = 0; f < nf; f++) {
        const int64_t na = Sptr[f + 1] - Sptr[f];
        if (na == 0) {
            S->pnt[f] = -1;
            continue;
        }
        const int64_t v0 = Stgt[Sptr[f]];
        if (v0 < Rptr[f + 1] || v0 >= n) goto bad;
        const int64_t p = S->idx[v0];
        S->pnt[f] = p;
        S->chdptr[p + 1]++;
        const int64_t pr = Rptr[p], pnn = Rptr[p + 1] - pr;
        int64_t q = Sptr[p];
        for (int64_t k = Sptr[f]; k < Sptr[f + 1]; k++) {
            const int64_t v = Stgt[k];
            if (k > Sptr[f] && v <= Stgt[k - 1]) goto bad;
            if (v < pr + pnn) {
                if (v < pr) goto bad;
                S->rel[k] = v - pr;
            } else {
                while (q < Sptr[p + 1] && Stgt[q] < v) q++;
                if (q >= Sptr[p + 1] || Stgt[q] != v) goto bad;
                S->rel[k] = pnn + (q - Sptr[p]);
            }
        }
    }
    for (int64_t f = 0; f < nf; f++) S->chdptr[f + 1] += S->chdptr[f];
    {
        int64_t *fill = (int64_t *)malloc(sizeof(int64_t) * (nf > 0 ? nf : 1));
        if (!fill) goto bad;
        for (int64_t f = 0; f < nf; f++) fill[f] = S->chdptr[f];
        for (int64_t f = 0; f < nf; f++)
            if (S->pnt[f] >= 0) S->chdtgt[fill[S->pnt[f]]++] = f;
        free(fill);
    }
    for (int64_t f = 0; f < nf; f++) S->fdsc[f] = f;
    for (int64_t f = 0; f < nf; f++)
        if (S->pnt[f] >= 0 && S->fdsc[f] < S->fdsc[S->pnt[f]]) S->fdsc[S->pnt[f]] = S->fdsc[f];
    if (Bptr[0] != 0 || Bptr[nB] != n || Fptr[0] != 0 || Fptr[nB] != nf) goto bad;
    for (int64_t c = 0; c < nB; c++)
        for (int64_t f = Fptr[c]; f < Fptr[c + 1]; f++) S->fcc[f] = c;
    return S;
bad:
    ppo_struct_free(S);
    return NULL;
}

void ppo_struct_sizes(const ppo_struct *S, int64_t *out) {
    int64_t mx = 0;
    for (int64_t f = 0; f < S->nf; f++) {
        const int64_t nj = S->Rptr[f + 1] - S->Rptr[f] + S->Sptr[f + 1] - S->Sptr[f];
        if (nj > mx) mx = nj;
    }
    out[0] = S->Dptr[S->nf];
    out[1] = S->Lptr[S->nf];
    out[2] = S->nN;
    out[3] = mx;
}

void ppo_struct_derived(const ppo_struct *S, int64_t *pnt, int64_t *rel, int64_t *Dptr, int64_t *Lptr) {
    if (pnt) memcpy(pnt, S->pnt, sizeof(int64_t) * S->nf);
    if (rel) memcpy(rel, S->rel, sizeof(int64_t) * S->nS);
    if (Dptr) memcpy(Dptr, S->Dptr, sizeof(int64_t) * (S->nf + 1));
    if (Lptr) memcpy(Lptr, S->Lptr, sizeof(int64_t) * (S->nf + 1));
}

/* ===== dispatch ===== */

#define PPO_DISPATCH(sr, dt, CALL)                                                   \
    switch ((sr) * 3 + (dt)) {                                                       \
        case PPO_MINPLUS * 3 + PPO_F32: CALL(minplus_f32, float);                    \
        case PPO_MINPLUS * 3 + PPO_F64: CALL(minplus_f64, double);                   \
        case PPO_MINPLUS * 3 + PPO_I32: CALL(minplus_i32, int32_t);                  \
        case PPO_MAXPLUS * 3 + PPO_F32: CALL(maxplus_f32, float);                    \
        case PPO_MAXPLUS * 3 + PPO_F64: CALL(maxplus_f64, double);                   \
        case PPO_MAXMIN * 3 + PPO_F32: CALL(maxmin_f32, float);                      \
        case PPO_MAXMIN * 3 + PPO_F64: CALL(maxmin_f64, double);                     \
        case PPO_MINMAX * 3 + PPO_F32: CALL(minmax_f32, float);                      \
        case PPO_MINMAX * 3 + PPO_F64: CALL(minmax_f64, double);                     \
        case PPO_MAXPROD * 3 + PPO_F32: CALL(maxprod_f32, float);                    \
        case PPO_MAXPROD * 3 + PPO_F64: CALL(maxprod_f64, double);                   \
        case PPO_PLUSPROD * 3 + PPO_F32: CALL(plusprod_f32, float);                  \
        case PPO_PLUSPROD * 3 + PPO_F64: CALL(plusprod_f64, double);                 \
        case PPO_ORAND * 3 + PPO_I32: CALL(orand_i32, int32_t);                      \
        default: return -1;                                                          \
    }

int ppo_assemble(int sr, int dt, const ppo_struct *S, const int64_t *colptr, const int64_t *rowval, const void *nzval,
                 void *LD, void *LL, void *UD, void *UL, void *Nval) {
#define CALL(N, TT) \
    return assemble_##N(S, colptr, rowval, (const TT *)nzval, (TT *)LD, (TT *)LL, (TT *)UD, (TT *)UL, (TT *)Nval)
    PPO_DISPATCH(sr, dt, CALL)
#undef CALL
}

int ppo_factor(int sr, int dt, const ppo_struct *S, void *LD, void *LL, void *UD, void *UL, int nthreads) {
#define CALL(N, TT) return factor_##N(S, (TT *)LD, (TT *)LL, (TT *)UD, (TT *)UL, nthreads)
    PPO_DISPATCH(sr, dt, CALL)
#undef CALL
}

int ppo_lmul(int sr, int dt, const ppo_struct *S, const void *LD, const void *LL, const void *UD, const void *UL,
             const void *Nval, void *B, int64_t ldb, int64_t k, int nthreads) {
#define CALL(N, TT)                                                                                           \
    return sgetrs_##N(S, 1, (const TT *)LD, (const TT *)LL, (const TT *)UD, (const TT *)UL, (const TT *)Nval, \
                      (TT *)B, ldb, k, nthreads)
    PPO_DISPATCH(sr, dt, CALL)
#undef CALL
}

int ppo_rmul(int sr, int dt, const ppo_struct *S, const void *LD, const void *LL, const void *UD, const void *UL,
             const void *Nval, void *B, int64_t ldb, int64_t k, int nthreads) {
#define CALL(N, TT)                                                                                           \
    return sgetrs_##N(S, 0, (const TT *)LD, (const TT *)LL, (const TT *)UD, (const TT *)UL, (const TT *)Nval, \
                      (TT *)B, ldb, k, nthreads)
    PPO_DISPATCH(sr, dt, CALL)
#undef CALL
}

int ppo_star(int sr, int dt, const ppo_struct *S, const void *LD, const void *LL, const void *UD, const void *UL,
             const void *Nval, void *C, int nthreads) {
#define CALL(N, TT)                                                                                         \
    return star_##N(S, (const TT *)LD, (const TT *)LL, (const TT *)UD, (const TT *)UL, (const TT *)Nval, \
                    (TT *)C, nthreads)
    PPO_DISPATCH(sr, dt, CALL)
#undef CALL
}

int ppo_gemm(int sr, int dt, int64_t m, int64_t n, int64_t k, void *C, int64_t ldc, const void *A, int64_t lda,
             const void *B, int64_t ldb, int nthreads) {
#define CALL(N, TT)                                                                                     \
    gemm_##N(m, n, k, (TT *)C, ldc, (const TT *)A, lda, (const TT *)B, ldb, nthreads > 0 ? nthreads : 1); \
    return 0
    PPO_DISPATCH(sr, dt, CALL)
#undef CALL
}

int ppo_getrf(int sr, int dt, int64_t n, void *A, int64_t lda) {
#define CALL(N, TT)                   \
    getrf_##N((TT *)A, lda, n, 1);    \
    return 0
    PPO_DISPATCH(sr, dt, CALL)
#undef CALL
}

int ppo_getrf_batched(int sr, int dt, int64_t n, int64_t count, void *A, int nthreads) {
#define CALL(N, TT)                                                                          \
    {                                                                                        \
        int64_t b;                                                                           \
        TT *base = (TT *)A;                                                                  \
        _Pragma("omp parallel for schedule(dynamic, 4) num_threads(nthreads) if (nthreads > 1)") \
        for (b = 0; b < count; b++) getrf_##N(base + b * n * n, n, n, 1);                    \
        return 0;                                                                            \
    }
    PPO_DISPATCH(sr, dt, CALL)
#undef CALL
}
