/*
 * pathpack_b200.h — C ABI of the B200 (sm_100a) backend for the numeric hot path of PATHPACK.jl's semiring
 * multifrontal solver: mlu / mstar / lmul! / rmul! / Matrix(F) over MinPlus, MaxPlus, MaxMin, MinMax, MaxProd,
 * PlusProd and OrAnd.
 *
 * The symbolic phase stays on the host (in PATHPACK.jl: `ssymbolic`, src/CPU/chordal_ssymbolic.jl:26-57, with
 * CliqueTrees.jl).  Its output crosses this ABI once (pp_set_structure); the numeric work runs on one GPU per
 * handle.  Plain C types only: no C++ or torch types cross the boundary.
 *
 * Conventions
 *   - Every function returns an int32 status: PP_OK (0) or a negative PP_E* code; pp_last_error() gives the
 *     message.  Nothing throws across the ABI.
 *   - Host arrays passed in are only read during the call (copied or staged); no pointer is retained.
 *   - Device memory is owned by the handle and released by pp_destroy, also after an error.
 *   - A handle is bound to one device and one stream; calls on one handle must be serialised by the caller.
 *     Different handles may be used from different threads.  Calls with host outputs return after the data
 *     is in host memory.  Calls whose outputs stay on the device (pp_factor, pp_lmul / pp_rmul / pp_star with
 *     PP_DEVICE, pp_update_values from device memory) only enqueue their work on the handle's stream
 *     (pp_stream) and return; a device error of such a call (PP_ETIMEOUT: a bounded wait of a persistent
 *     kernel expired) is returned by the next call that waits for the stream: pp_sync, a call with host
 *     inputs or outputs, pp_get_factor, pp_get_stats, pp_get_profile, pp_lmul_static.
 *   - Matrices are column-major (Julia's layout), with a leading dimension.
 *   - Index arrays are int64 and may be 1-based (as Julia and CliqueTrees hold them, `base` = 1) or 0-based.
 */
#ifndef PATHPACK_B200_H
#define PATHPACK_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PP_OK 0
#define PP_EINVAL (-1)       /* bad argument, shape or structure */
#define PP_EUNSUPPORTED (-2) /* semiring / element type pair the backend does not take */
#define PP_ENOMEM (-3)       /* device or host memory exhausted (checked before work starts) */
#define PP_EDEVICE (-4)      /* CUDA error */
#define PP_ETIMEOUT (-5)     /* a bounded device wait expired */
#define PP_ESTATE (-6)       /* call out of order (e.g. a solve before pp_factor) */

/* semirings: the reference's MinPlus, MaxPlus, MaxMin, MinMax, MaxProd, PlusProd, OrAnd
   (src/CPU/semiring/tropical.jl, bottleneck.jl, real.jl, boolean.jl) */
enum { PP_MINPLUS = 0, PP_MAXPLUS = 1, PP_MAXMIN = 2, PP_MINMAX = 3, PP_MAXPROD = 4, PP_PLUSPROD = 5, PP_ORAND = 6 };
/* element types */
enum { PP_F32 = 0, PP_F64 = 1, PP_I32 = 2 };
/* where a caller buffer lives */
enum { PP_HOST = 0, PP_DEVICE = 1 };

typedef struct pp_handle pp_handle;

typedef struct pp_stats {
    int64_t n, nf, nB;          /* vertices, fronts, strongly connected components */
    int64_t nlevels;            /* tree levels of the factorization schedule */
    int64_t nD, nL, nN;         /* lengths of LD/UD, LL/UL and Nval */
    int64_t max_front;          /* largest nn + na */
    double pairs_factor;        /* (x)(+) pairs of one factorization, unpadded structure */
    double ms_factor;           /* device time of the last pp_factor */
    double ms_solve;            /* device time of the last pp_lmul / pp_rmul / pp_star */
    double pairs_solve;         /* (x)(+) pairs of the last solve */
    int64_t device_bytes;       /* device memory held by the handle */
    int64_t kernel_launches;    /* kernels launched by the last call */
    int64_t plan_fronts;        /* fronts of the device plan: fewer than nf where chains of top fronts are merged */
} pp_stats;

/* The library's version, major * 10000 + minor * 100 + patch. */
int32_t pp_version(void);

/* Whether the backend takes the (semiring, element type) pair: PP_OK or PP_EUNSUPPORTED.
   Replaces check_semiring, ext/PATHPACKCUDAExt/runtime/config.jl:359-377.  Supported: every semiring over
   PP_F32 and PP_F64 except OrAnd; MinPlus and OrAnd over PP_I32.  Int32 MinPlus is defined on [0, INT32_MAX]
   with a saturating product (INT32_MAX is "no path" and absorbs). */
int32_t pp_check_semiring(int32_t semiring, int32_t dtype);

/* The message of the last failed call on this thread (h may be NULL), or "" after success. */
const char *pp_last_error(const pp_handle *h);

/* Create a handle on a CUDA device (stream, device structures created lazily). */
int32_t pp_create(int32_t device, pp_handle **h);

/* Handle options (the pp_options of the reference-facing plan: pp_create(device, const pp_options*, ...)).
   Start from pp_default_options and change fields.
     wait_timeout_us   bound of every device-side wait of the persistent kernels on another block's progress,
                       in microseconds; 0 = the default, 2 s.  A wait that runs out makes the kernels of the
                       call return early and the call report PP_ETIMEOUT at its next wait for the stream (the
                       results of that call are then undefined; the handle stays usable).  Raise it when the
                       GPU is time-sliced with other work.
     fail_alloc_after  testing: when >= 0, that many device allocations of the handle succeed and the next
                       one fails as if the device were out of memory (the call returns PP_ENOMEM, having freed
                       nothing it still needs and leaked nothing); -1 (default) = off.
     profile           1: per-launch timing (pp_set_profile).
     merge_width       amalgamation: the largest residual of a front merged from a chain of top fronts (the
                       reference's GPU amalgamation, ext/PATHPACKCUDAExt/chordal/amalgamate.jl); 0 = the
                       default, 64; 1 = no merging.  Read by pp_set_structure.  The factor arrays a caller
                       exchanges (pp_set_values, pp_get_factor) keep the caller's structure either way.
     trace             1: record the timeline of the top of the tree's factorization, task by task
                       (pp_get_trace). */
typedef struct pp_options {
    int64_t wait_timeout_us;
    int64_t fail_alloc_after;
    int32_t profile;
    int32_t merge_width;
    int32_t trace;
    int32_t reserved;
} pp_options;
void pp_default_options(pp_options *opt);
/* pp_create with options (opt may be NULL: the defaults). */
int32_t pp_create_with(int32_t device, const pp_options *opt, pp_handle **h);
/* Change the options of a handle (waits for the handle's work first). */
int32_t pp_set_options(pp_handle *h, const pp_options *opt);
int32_t pp_get_options(const pp_handle *h, pp_options *opt);
/* Release everything the handle holds.  Safe on NULL. */
int32_t pp_destroy(pp_handle *h);

/* Upload the symbolic structure (replaces the ChordalSSymbolic that `ChordalSLU` holds,
   src/CPU/chordal_slu.jl:1-26 and src/CPU/chordal_ssymbolic.jl:1-8):
     n, nf, nB          vertices, fronts, components
     Rptr[nf+1]         residual of front f = positions Rptr[f] .. Rptr[f+1]-1   (pointers(S.res))
     Sptr[nf+1], Stgt   separator of front f, sorted positions                   (pointers/targets(S.sep))
     Bptr[nB+1]         vertex range of each component                           (F.S.Bptr)
     Fptr[nB+1]         front range of each component                            (F.S.Fptr)
     Nptr[n+1], Ntgt    coupling: rows of earlier components of each position    (pointers/targets(F.S.N))
     perm[n]            original vertex at each position                         (F.rperm = F.cperm)
   Fronts must be in postorder and the parent of a front is the front of its first separator vertex.
   base = 1 for 1-based arrays (Julia), 0 for 0-based. */
int32_t pp_set_structure(pp_handle *h, int64_t n, int64_t nf, int64_t nB, const int64_t *Rptr, const int64_t *Sptr,
                         const int64_t *Stgt, const int64_t *Bptr, const int64_t *Fptr, const int64_t *Nptr,
                         const int64_t *Ntgt, const int64_t *perm, int32_t base);

/* Assemble A (n x n CSC on the host: colptr[n+1], rowval[nnz], nzval[nnz] of the element type; A[i, j] is the
   weight of the arc i -> j; no duplicate entries) into the factor arrays on the device.  Replaces
   copyto!(F::ChordalSLU, A), src/CPU/chordal_slu.jl:116-321. */
int32_t pp_assemble(pp_handle *h, int32_t semiring, int32_t dtype, const int64_t *colptr, const int64_t *rowval,
                    const void *nzval, int32_t base);

/* New weights for the pattern of the last pp_assemble (nzval in the same order, on the host or on this
   handle's device), re-assembled on the device: refactorization with the same structure, the use of the
   reference's plans (APSPPlan, ext/PATHPACKCUDAExt/api.jl:547-668; FactorPlan, chordal/sgetrf.jl:710-740).
   Int32 MinPlus weights from device memory are not checked for the [0, INT32_MAX] domain. */
int32_t pp_update_values(pp_handle *h, const void *nzval, int32_t where);

/* Upload already assembled factor arrays (host): LD, UD (|LD| values), LL, UL (|LL|), Nval (|Nval|). */
int32_t pp_set_values(pp_handle *h, int32_t semiring, int32_t dtype, const void *LD, const void *LL, const void *UD,
                      const void *UL, const void *Nval);

/* Factorize the star, A* = U* L*, in place on the device (enqueued; see the conventions above).  The top of
   the elimination tree is factored on a second, higher-priority stream of the handle, so that a solve enqueued
   next sweeps the bottom of the tree meanwhile; every call of the handle orders itself after it, and pp_sync
   waits for it.  Replaces lu!(F) -> sgetrf!(F), src/CPU/abstract_slu.jl:119-121 and
   src/CPU/chordal/sgetrf.jl:3-290. */
int32_t pp_factor(pp_handle *h);

/* Download the factor arrays to the host (any pointer may be NULL). */
int32_t pp_get_factor(pp_handle *h, void *LD, void *LL, void *UD, void *UL);

/* B <- A* B: lmul!(F, B), src/CPU/abstract_slu.jl:131-134.  B is n x k, column-major, leading dimension ldb,
   on the host (where = PP_HOST) or on this handle's device (PP_DEVICE). */
int32_t pp_lmul(pp_handle *h, void *B, int64_t ldb, int64_t k, int32_t where);

/* B <- B A*: rmul!(B, F), src/CPU/abstract_slu.jl:142-145.  B is k x n, column-major, leading dimension ldb. */
int32_t pp_rmul(pp_handle *h, void *B, int64_t ldb, int64_t k, int32_t where);

/* The transposed factor: B <- (A*)^T B = (A^T)* B, lmul!(transpose(F), B), and B <- B (A*)^T,
   rmul!(B, transpose(F)); src/CPU/abstract_slu.jl:131-145 with unwrap(F) giving trans = Val(:T), which
   sgetrs! (src/CPU/chordal/sgetrs.jl:88-110) runs as U* first, then L*.  Layouts as pp_lmul / pp_rmul. */
int32_t pp_lmul_t(pp_handle *h, void *B, int64_t ldb, int64_t k, int32_t where);
int32_t pp_rmul_t(pp_handle *h, void *B, int64_t ldb, int64_t k, int32_t where);

/* Columns col0 .. col0+ncols-1 of the star A* (original labels) into C (n x ncols, column-major, leading
   dimension ldc).  ncols = n and col0 = 0 is Matrix(F), src/CPU/abstract_slu.jl:10-14; column panels let
   several GPUs share one star. */
int32_t pp_star(pp_handle *h, void *C, int64_t ldc, int64_t col0, int64_t ncols, int32_t where);

/* Columns cols[0 .. ncols-1] of the star A* (original labels; any order, repeats allowed) into C (n x ncols,
   column-major, leading dimension ldc): the closure's entries towards a set of targets. */
int32_t pp_star_cols(pp_handle *h, void *C, int64_t ldc, const int64_t *cols, int64_t ncols, int32_t where);

/* Rows sources[0 .. k-1] of the star A* (original labels) into C (k x n, column-major, leading dimension ldc >= k):
   the closure from a set of sources, apsp_gpu(A, sources) of the reference (ext/PATHPACKCUDAExt/api.jl:103-154),
   computed as rmul! of unit rows. */
int32_t pp_star_rows(pp_handle *h, void *C, int64_t ldc, const int64_t *sources, int64_t k, int32_t where);

/* Wait for the handle's stream; reports a device error of the calls enqueued since the last wait. */
int32_t pp_sync(pp_handle *h);

/* ---- several GPUs: one handle per GPU (a process or thread each), joined into a group over NCCL ----
   The multi-GPU factorization of the reference (ext/PATHPACKCUDAExt/multigpu.jl:372-470 replicates the
   factor by peer copies; here the factorization itself is split).  Every rank sets the same structure and
   assembles the same matrix; then pp_factor on a joined handle factors only this rank's part of the bottom of
   the tree (maximal subtrees of small fronts, dealt to the ranks in runs of about equal estimated time), gives
   every rank the other parts with NCCL broadcasts on the handle's stream (the factor blocks and the children's
   update matrices, over NVLink), and factors the top of the tree on every rank, so that each rank ends with the
   whole factor and solves or computes star columns on its own (split the right-hand sides or the star's
   columns across the ranks).  Every rank must call pp_factor the same number of times (a collective).  NCCL
   (libnccl.so.2) is loaded when first needed.  A host wait on a joined handle's streams gives up after 60 s
   (30 x wait_timeout_us when that is set), aborts the communicator and reports PP_EDEVICE; the handle has
   then left the group (PP_ESTATE from the next pp_factor).  Plans (pp_plan_lmul) stay single-GPU. */
#define PP_COMM_ID_BYTES 128
/* A new group id (PP_COMM_ID_BYTES bytes): made on one rank and sent to the others. */
int32_t pp_comm_id(void *id);
/* Join the handle as `rank` of `nranks` (nranks = 1 leaves any group); blocks until every rank has joined. */
int32_t pp_comm_init(pp_handle *h, const void *id, int32_t nranks, int32_t rank);

/* ---- several GPUs driven by one process: a multi-device handle ----
   A pp_multi holds a handle per device of `devices`, joined into one group as above; each call runs the
   corresponding call on every device at once (one host thread per device, as the reference's multi-GPU driver
   runs one task per device, ext/PATHPACKCUDAExt/multigpu.jl:432-450) and returns the first failure (message:
   pp_last_error(NULL) on the calling thread).  pp_multi_lmul / pp_multi_rmul split the k right-hand sides of a
   host B into one contiguous panel per device (trans = 1: the transposed factor, as pp_lmul_t / pp_rmul_t);
   pp_multi_star splits the columns col0 .. col0+ncols-1 of A* into one contiguous panel per device, written into
   the host array C (n x ncols).  pp_multi_handle gives a device's handle for the one-device calls (device
   outputs: pp_star into each device's own memory). */
typedef struct pp_multi pp_multi;
int32_t pp_multi_create(const int32_t *devices, int32_t ndev, const pp_options *opt, pp_multi **m);
int32_t pp_multi_destroy(pp_multi *m);
int32_t pp_multi_handle(pp_multi *m, int32_t i, pp_handle **h);
int32_t pp_multi_set_structure(pp_multi *m, int64_t n, int64_t nf, int64_t nB, const int64_t *Rptr,
                               const int64_t *Sptr, const int64_t *Stgt, const int64_t *Bptr, const int64_t *Fptr,
                               const int64_t *Nptr, const int64_t *Ntgt, const int64_t *perm, int32_t base);
int32_t pp_multi_assemble(pp_multi *m, int32_t semiring, int32_t dtype, const int64_t *colptr, const int64_t *rowval,
                          const void *nzval, int32_t base);
/* the split factorization on every device; returns when it is complete everywhere */
int32_t pp_multi_factor(pp_multi *m);
int32_t pp_multi_lmul(pp_multi *m, void *B, int64_t ldb, int64_t k, int32_t trans);
int32_t pp_multi_rmul(pp_multi *m, void *B, int64_t ldb, int64_t k, int32_t trans);
int32_t pp_multi_star(pp_multi *m, void *C, int64_t ldc, int64_t col0, int64_t ncols);

/* ---- lmul! allocating nothing (no counterpart in the reference) ----
   pp_lmul_static is pp_lmul for device-resident B (n x k, leading dimension ldb, on the handle's device) that
   allocates nothing: no device memory, no host staging, no profiler events.  It is for callers that must not
   allocate while solving, such as a serving process that reserves all device memory at startup (its pool
   leaves cudaMalloc nothing to give, and a cudaMalloc may synchronise the device and stall the other streams'
   work).  Its scratch, the right-hand sides in the device layout and the sweep counters, is one static device
   array of PP_STATIC_SCRATCH_BYTES per device inside the library's device image:
       n * (k rounded up to 4) * element size, rounded up to 256 bytes, plus 4 * (3 * ceil(k / 32) * nfronts + 16)
   bytes must fit, else the call returns PP_EINVAL and touches nothing.  Nothing in the array has to start at
   zero: the counters are reset by the solve itself.  Each call looks up the array's address on the handle's
   device.  The first call on a device is also where the CUDA runtime (lazy module loading, the CUDA 12
   default) loads the library's device code on that device and so reserves the array's 32 MiB: make that first
   call before the caller reserves its memory pool, and before any stream capture.  All calls on one device
   share the array, so two calls that overlap in time (from different host threads, on any handles) race on it
   and return wrong results.  The call is synchronous: it returns after its work on the device is complete. */
#define PP_STATIC_SCRATCH_BYTES (32u << 20)
int32_t pp_lmul_static(pp_handle *h, void *B, int64_t ldb, int64_t k);

/* ---- plans: refactorization with new weights and a solve, replayed as one CUDA graph ----
   The reference's plans for repeated solves on one pattern (FactorPlan with graph replay,
   ext/PATHPACKCUDAExt/chordal/sgetrf.jl:710-740; APSPPlan, ext/PATHPACKCUDAExt/api.jl:547-668).
   pp_plan_lmul captures one step on the handle: pp_update_values from nzval (device memory, the order of
   the last pp_assemble), pp_factor, and Bout <- A* Bin (lmul!, Bin and Bout n x k column-major device arrays
   with leading dimension ldb; Bin may equal Bout).  It runs the step once uncaptured first, so that
   everything the step needs is allocated and errors are reported, then records it into a CUDA graph.
   pp_plan_launch enqueues one step on the handle's stream (pp_stream) and returns: write new weights into
   nzval (or new right-hand sides into Bin) on that stream first and launch again.  A device error of a
   launch is reported by the next call that waits (pp_sync).  The graph works on the handle's factor arrays
   and workspace, on scratch of its own (the right-hand sides in the device layout and the kernels' counters,
   so that the handle's other calls stay free to grow their buffers) and on the three arrays, whose addresses
   it keeps: keep them alive and do not change the handle's structure or semiring while a plan exists;
   pp_plan_destroy releases the graph and its scratch (not the handle). */
typedef struct pp_plan pp_plan;
int32_t pp_plan_lmul(pp_handle *h, const void *nzval, const void *Bin, void *Bout, int64_t ldb, int64_t k,
                     pp_plan **plan);
int32_t pp_plan_launch(pp_plan *plan);
/* kernels one launch of the plan runs */
int32_t pp_plan_launches(const pp_plan *plan, int64_t *launches);
int32_t pp_plan_destroy(pp_plan *plan);

/* The timeline of the last factorization's top of the tree (pp_options.trace = 1): PP_TRACE_WORDS words per
   tile task, in the order the tasks were listed: global timer in ns when the task was taken, when its tile was
   assembled, when its products with the pivot blocks were done and when it was published; the SM and front,
   (sm << 32) | front of the device plan; the tile, (I << 32) | J.  Copies at most max_tasks tasks, sets
   *ntasks to the number of tasks. */
#define PP_TRACE_WORDS 6
int32_t pp_get_trace(pp_handle *h, uint64_t *out, int64_t max_tasks, int64_t *ntasks);

/* Counters of the handle (sizes, pair counts, device times of the last calls). */
int32_t pp_get_stats(pp_handle *h, pp_stats *s);

/* Per-kernel-class device times: with profiling on, every launch of the handle is bracketed by CUDA events
   on its stream and accumulated per class with its algorithmic bytes and (x)(+) pairs.  pp_set_profile
   resets the totals. */
typedef struct pp_kernel_class {
    char name[32];
    int64_t launches;
    double ms;     /* summed device time of the launches */
    double bytes;  /* algorithmic bytes moved by the launches */
    double pairs;  /* (x)(+) pairs computed by the launches */
} pp_kernel_class;
int32_t pp_set_profile(pp_handle *h, int32_t on);
int32_t pp_get_profile(pp_handle *h, pp_kernel_class *out, int32_t max, int32_t *count);

/* The handle's CUDA stream (a cudaStream_t), for callers that order their own work after the handle's: work
   ordered after it follows every call enqueued before (the solves included); only the top of a factorization
   that no solve has followed yet may still be running (pp_sync waits for it). */
void *pp_stream(pp_handle *h);

/* ---- dense kernels on caller device memory (ordered on `stream`, a cudaStream_t or NULL) ---- */

/* C <- C (+) A (x) B, A m x k, B k x n, C m x n, column-major device arrays.
   Replaces sgemx_gpu!(s, C, A, B), ext/PATHPACKCUDAExt/dense/sgemx.jl:27-45 (and CPU.sgemx!). */
int32_t pp_gemm(int32_t semiring, int32_t dtype, int64_t m, int64_t n, int64_t k, void *C, int64_t ldc, const void *A,
                int64_t lda, const void *B, int64_t ldb, void *stream);

/* In-place LU of the star of `count` dense n x n blocks stored back to back (block b at A + b*n*n, column-major).
   Replaces sgetrf_gpu!(s, A) on each block, ext/PATHPACKCUDAExt/dense/sgetrf.jl:31-125 (and CPU.sgetrf!). */
int32_t pp_getrf_batched(int32_t semiring, int32_t dtype, int64_t n, int64_t count, void *A, void *stream);

/* ---- host symbolic stand-in (for callers without Julia's symbolic phase) ---- */

typedef struct pp_symbolic_result pp_symbolic_result;

/* SCCs, ordering and clique tree of the n x n pattern colptr/rowval (0-based CSC).  method 0 = nested
   dissection (leaf = piece size ordered by minimum degree, 0 = default), 1 = natural order.  The result is
   0-based; read it with pp_symbolic_sizes / pp_symbolic_get and release it with pp_symbolic_free. */
int32_t pp_symbolic(int64_t n, const int64_t *colptr, const int64_t *rowval, int32_t method, int32_t leaf,
                    pp_symbolic_result **out);
/* sizes[5] = n, nf, nB, |Stgt|, |Ntgt| */
void pp_symbolic_sizes(const pp_symbolic_result *r, int64_t *sizes);
void pp_symbolic_get(const pp_symbolic_result *r, int64_t *Rptr, int64_t *Sptr, int64_t *Stgt, int64_t *Bptr,
                     int64_t *Fptr, int64_t *Nptr, int64_t *Ntgt, int64_t *perm);
void pp_symbolic_free(pp_symbolic_result *r);

#ifdef __cplusplus
}
#endif

#endif
