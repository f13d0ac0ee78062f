/*
 * pp_oracle.h — CPU restatement of PATHPACK.jl's semiring multifrontal solver (the oracle).
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the B200 library and the timed CPU
 * baseline; only tests/, __graft_entry__.smoke() and bench.py (its cpu_baseline leg and its
 * `--impl reference` arm) may load it.  The product path never links or calls it.
 *
 * Every numeric routine restates a function of the reference (file:line relative to the reference
 * project root) with 0-based indices in place of Julia's 1-based ones:
 *   semirings      src/CPU/semiring/{semiring,tropical,bottleneck,real,boolean}.jl
 *   assembly       src/CPU/chordal_slu.jl:120-141, 221-321        (scopyto_st!, scopyto_loop!)
 *   factorization  src/CPU/chordal/sgetrf.jl:9-290                (sgetrf_mt!, sgetrf_loop!, sgetrf_loop_1!, sgetrf_send!)
 *                  src/CPU/dense/sgetrf.jl:21-68, 151-175         (blocked sgetrf_mt!, scalar sgetrf2!)
 *                  src/CPU/dense/strsx.jl:596-672                 (generic strsx2!)
 *                  src/CPU/dense/sgemx.jl:606-635                 (generic sgemx2!)
 *   solves         src/CPU/chordal_slu.jl:337-377                 (sgetrs! with permutations)
 *                  src/CPU/blocked/sgetrs.jl:145-255              (components in order, coupling N)
 *                  src/CPU/sparse/sgemx.jl:101-113, 193-213       (coupling products)
 *                  src/CPU/chordal/sgetrs.jl:29-51                (L then U, or U then L)
 *                  src/CPU/chordal/strsx.jl:79-126, 130-230, 729-830 (per-front forward/backward)
 *   star           src/CPU/chordal_slu.jl:501-513                 (sgetri! then permuterowscols!)
 *                  src/CPU/chordal/sgetri.jl:13-31                (X <- U*, X <- X L*)
 *                  src/CPU/chordal/strtri.jl:18-319               (banded star of the chordal U)
 *                  src/CPU/dense/strtri.jl:19-54, 237-269         (recursive dense star, leaf 128)
 *                  src/CPU/blocked/sgetri.jl:3-162                (off-diagonal component blocks)
 *                  src/CPU/utils.jl:261-319                       (permuterowscols!)
 *
 * Structure arrays follow CliqueTrees' ChordalSymbolic layout (0-based here): the residual of front
 * f is the vertex range Rptr[f] .. Rptr[f+1]-1 (permuted labels), its separator the sorted vertices
 * Stgt[Sptr[f] .. Sptr[f+1]-1]; Dptr/Lptr are the running sums of nn^2 and nn*na.  Components
 * (strongly connected) own vertex ranges Bptr[c] .. Bptr[c+1]-1 and front ranges Fptr[c] ..
 * Fptr[c+1]-1; the coupling N lists, for each vertex j, the earlier-component rows Ntgt[Nptr[j] ..
 * Nptr[j+1]-1].  perm[p] is the original vertex at permuted position p and invp its inverse
 * (rperm = cperm and rinvp = cinvp, src/CPU/chordal_slu.jl:58-61).
 */
#ifndef PP_ORACLE_H
#define PP_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { PPO_MINPLUS = 0, PPO_MAXPLUS = 1, PPO_MAXMIN = 2, PPO_MINMAX = 3, PPO_MAXPROD = 4, PPO_PLUSPROD = 5, PPO_ORAND = 6 };
enum { PPO_F32 = 0, PPO_F64 = 1, PPO_I32 = 2 };

typedef struct ppo_struct {
    int64_t n, nf, nB;
    int64_t *Rptr, *Sptr, *Stgt, *Bptr, *Fptr, *Nptr, *Ntgt, *perm, *invp;
    /* derived */
    int64_t *Dptr, *Lptr, *pnt, *chdptr, *chdtgt, *rel, *idx, *fcc, *fdsc;
    int64_t nS, nN;
} ppo_struct;

/* returns NULL on a malformed structure; the arrays are copied */
ppo_struct *ppo_struct_new(int64_t n, int64_t nf, int64_t nB, const int64_t *Rptr, const int64_t *Sptr,
                           const int64_t *Stgt, const int64_t *Bptr, const int64_t *Fptr, const int64_t *Nptr,
                           const int64_t *Ntgt, const int64_t *perm);
void ppo_struct_free(ppo_struct *S);
/* out[0] = |LD| = |UD|, out[1] = |LL| = |UL|, out[2] = |Nval|, out[3] = max front size nn + na */
void ppo_struct_sizes(const ppo_struct *S, int64_t *out);
/* copies pnt (nf), rel (nS), Dptr (nf+1), Lptr (nf+1) into the caller's arrays (any may be NULL) */
void ppo_struct_derived(const ppo_struct *S, int64_t *pnt, int64_t *rel, int64_t *Dptr, int64_t *Lptr);

/* all return 0 on success, -1 on an unsupported (semiring, dtype) pair, -2 on allocation failure */
int ppo_assemble(int sr, int dt, const ppo_struct *S, const int64_t *colptr, const int64_t *rowval, const void *nzval,
                 void *LD, void *LL, void *UD, void *UL, void *Nval);
int ppo_factor(int sr, int dt, const ppo_struct *S, void *LD, void *LL, void *UD, void *UL, int nthreads);
/* B <- A* B, B is n x k column-major with leading dimension ldb (lmul!) */
int ppo_lmul(int sr, int dt, const ppo_struct *S, const void *LD, const void *LL, const void *UD, const void *UL,
             const void *Nval, void *B, int64_t ldb, int64_t k, int nthreads);
/* B <- B A*, B is k x n column-major with leading dimension ldb (rmul!) */
int ppo_rmul(int sr, int dt, const ppo_struct *S, const void *LD, const void *LL, const void *UD, const void *UL,
             const void *Nval, void *B, int64_t ldb, int64_t k, int nthreads);
/* C <- A*, n x n column-major in original labels (Matrix(F)) */
int ppo_star(int sr, int dt, const ppo_struct *S, const void *LD, const void *LL, const void *UD, const void *UL,
             const void *Nval, void *C, int nthreads);
/* C <- C (+) A (x) B, column-major (sgemx!) */
int ppo_gemm(int sr, int dt, int64_t m, int64_t n, int64_t k, void *C, int64_t ldc, const void *A, int64_t lda,
             const void *B, int64_t ldb, int nthreads);
/* dense in-place LU of the star of an n x n block (sgetrf!) */
int ppo_getrf(int sr, int dt, int64_t n, void *A, int64_t lda);
/* `count` independent n x n blocks stored back to back (column-major, stride n*n) */
int ppo_getrf_batched(int sr, int dt, int64_t n, int64_t count, void *A, int nthreads);

#ifdef __cplusplus
}
#endif
#endif
