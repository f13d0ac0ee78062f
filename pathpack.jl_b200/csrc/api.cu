// api.cu — the C ABI (include/pathpack_b200.h): handles, structure upload and checks, schedules, workspace,
// and the drivers of mlu / lmul! / rmul! / Matrix(F) on one GPU.
//
// What each entry point replaces in the reference is stated in the header.  The structure checks are those
// the reference's solver relies on (postorder clique tree, separators inside the parent's bag); the error
// conventions follow the reference's typed errors (check_semiring, ext/PATHPACKCUDAExt/runtime/config.jl:359-377;
// the memory check before any work, api.jl:1031-1045; freeing everything on failure, api.jl:141-147).

#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <condition_variable>
#include <mutex>
#include <thread>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <memory>
#include <new>
#include <queue>
#include <string>
#include <vector>

#include "ops.h"
#include "pathpack_b200_internal.h"

namespace pp {
extern const Ops ops_minplus_f32, ops_minplus_f64, ops_minplus_i32, ops_maxplus_f32, ops_maxplus_f64,
    ops_maxmin_f32, ops_maxmin_f64, ops_minmax_f32, ops_minmax_f64, ops_maxprod_f32, ops_maxprod_f64,
    ops_plusprod_f32, ops_plusprod_f64, ops_orand_i32;

const Ops *get_ops(int sr, int dt) {
    switch (sr * 3 + dt) {
        case PP_MINPLUS * 3 + 0: return &ops_minplus_f32;
        case PP_MINPLUS * 3 + 1: return &ops_minplus_f64;
        case PP_MINPLUS * 3 + 2: return &ops_minplus_i32;
        case PP_MAXPLUS * 3 + 0: return &ops_maxplus_f32;
        case PP_MAXPLUS * 3 + 1: return &ops_maxplus_f64;
        case PP_MAXMIN * 3 + 0: return &ops_maxmin_f32;
        case PP_MAXMIN * 3 + 1: return &ops_maxmin_f64;
        case PP_MINMAX * 3 + 0: return &ops_minmax_f32;
        case PP_MINMAX * 3 + 1: return &ops_minmax_f64;
        case PP_MAXPROD * 3 + 0: return &ops_maxprod_f32;
        case PP_MAXPROD * 3 + 1: return &ops_maxprod_f64;
        case PP_PLUSPROD * 3 + 0: return &ops_plusprod_f32;
        case PP_PLUSPROD * 3 + 1: return &ops_plusprod_f64;
        case PP_ORAND * 3 + 2: return &ops_orand_i32;
        default: return nullptr;
    }
}
}  // namespace pp

namespace pp {
const char *const KCLASS_NAMES[K_NCLASS] = {"factor_top_kernel", "sweep_top_kernel(fwd)",
                                            "sweep_top_kernel(bwd)", "coupling", "permute", "assemble_kernel",
                                            "factor_bottom_kernel", "sweep_bottom_kernel(fwd)",
                                            "sweep_bottom_kernel(bwd)", "sweep_subtree_kernel(fwd)",
                                            "sweep_subtree_kernel(bwd)"};
}

using namespace pp;

static thread_local std::string g_err;

// NCCL, for handles joined into a group of GPUs (pp_comm_init): loaded on first use with dlopen, so that the
// library itself loads and runs without it (nccl.h gives the types only).  A process that already holds
// libnccl.so.2 (PyTorch's, for instance) shares that copy.
struct NcclApi {
    bool ok = false;
    std::string why;
    ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
    ncclResult_t (*Broadcast)(const void *, void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    const char *(*GetErrorString)(ncclResult_t) = nullptr;
};

static const NcclApi &nccl_api() {
    static const NcclApi api = [] {
        NcclApi a;
        void *lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!lib) lib = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!lib) {
            const char *e = dlerror();
            a.why = std::string("libnccl.so.2 could not be loaded: ") + (e ? e : "?");
            return a;
        }
        bool all = true;
        auto sym = [&](auto &fn, const char *name) {
            fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(lib, name));
            all = all && fn;
        };
        sym(a.GetUniqueId, "ncclGetUniqueId");
        sym(a.CommInitRank, "ncclCommInitRank");
        sym(a.CommDestroy, "ncclCommDestroy");
        sym(a.CommAbort, "ncclCommAbort");
        sym(a.CommGetAsyncError, "ncclCommGetAsyncError");
        sym(a.Broadcast, "ncclBroadcast");
        sym(a.GroupStart, "ncclGroupStart");
        sym(a.GroupEnd, "ncclGroupEnd");
        sym(a.GetErrorString, "ncclGetErrorString");
        a.ok = all;
        if (!all) a.why = "libnccl.so.2 lacks a function the library needs";
        return a;
    }();
    return api;
}

// The allocation budget of the handle whose call is running on this thread (pp_options.fail_alloc_after):
// when it is >= 0, the allocation that finds it at 0 fails as if the device were out of memory.
static thread_local int64_t *t_alloc_budget = nullptr;

struct DevBuf {
    void *p = nullptr;
    size_t bytes = 0;
    ~DevBuf() { release(); }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        bytes = 0;
    }
    cudaError_t ensure(size_t b) {
        if (b <= bytes && p) return cudaSuccess;
        release();
        if (b == 0) b = 16;
        if (t_alloc_budget && *t_alloc_budget >= 0 && (*t_alloc_budget)-- == 0) return cudaErrorMemoryAllocation;
        cudaError_t e = cudaMalloc(&p, b);
        if (e == cudaSuccess)
            bytes = b;
        else
            cudaGetLastError();  // a failed allocation must not surface as the error of a later launch
        return e;
    }
    template <typename U>
    U *as() const {
        return static_cast<U *>(p);
    }
};

// A rank's part of the bottom of the tree (several GPUs): fronts [f0, f1) and the element ranges of their
// diagonal blocks (LD, UD), off-diagonal blocks (LL, UL) and workspace.
struct Part {
    int f0 = 0, f1 = 0;
    int64_t d0 = 0, d1 = 0, l0 = 0, l1 = 0, w0 = 0, w1 = 0;
};

// Page-locked host memory (cudaHostAlloc), released with the handle.
struct PinnedBuf {
    void *p = nullptr;
    size_t bytes = 0;
    ~PinnedBuf() { release(); }
    void release() {
        if (p) cudaFreeHost(p);
        p = nullptr;
        bytes = 0;
    }
    cudaError_t ensure(size_t b) {
        if (b <= bytes && p) return cudaSuccess;
        release();
        if (t_alloc_budget && *t_alloc_budget >= 0 && (*t_alloc_budget)-- == 0) return cudaErrorMemoryAllocation;
        cudaError_t e = cudaHostAlloc(&p, b, cudaHostAllocDefault);
        if (e == cudaSuccess)
            bytes = b;
        else
            cudaGetLastError();
        return e;
    }
};

struct pp_handle {
    int device = 0;
    cudaStream_t stream = nullptr;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;    // around the last solve
    cudaEvent_t fev0 = nullptr, fev1 = nullptr;  // around the last factorization
    cudaStream_t copy_stream = nullptr;           // copies that may overlap the handle's work
    // the top of the tree is factored on its own stream: a solve enqueued next on the handle's stream runs its
    // bottom sweeps meanwhile and waits for ev_factored before its top sweeps; every other call that reads or
    // writes the factor makes the handle's stream wait for ev_factored first (after_factor)
    cudaStream_t factor_stream = nullptr;
    cudaEvent_t ev_bottom = nullptr, ev_factored = nullptr;
    cudaEvent_t ev_top_a = nullptr;  // the end of the top factorization's first launch (every front but the roots)
    cudaEvent_t copy_ev = nullptr;
    // lmul! on host memory in column panels: panel p's upload done (in_ev) and solve done (out_ev); the results
    // go back on out_stream while the next panel is solved
    static constexpr int kSolvePanels = 4;
    cudaStream_t out_stream = nullptr;
    cudaEvent_t in_ev[kSolvePanels] = {}, out_ev[kSolvePanels] = {};
    cudaEvent_t panel_ready[2] = {}, panel_copied[2] = {};  // double-buffered star panels to host memory
    cudaEvent_t ring_ev[3] = {};  // star panels into pageable host memory: the pinned ring's slots filled
    PinnedBuf ring;               // three panels of page-locked host memory (allocated on first use)
    bool factor_pending = false, solve_pending = false;  // enqueued, times not yet read
    // set while a plan (pp_plan_lmul) captures the handle's calls into a CUDA graph: no timing events, no
    // profiler, and no wait for the previous factorization (a graph launch is ordered as a whole)
    bool capturing = false;
    std::string err;
    bool have_structure = false, have_values = false, factored = false;
    int sr = -1, dt = -1;
    const Ops *ops = nullptr;
    HostPlan hp;
    // host copies used by the drivers
    std::vector<int> invp;
    std::vector<int> star_host;  // pp_star's panel order: positions, then output columns
    // device structure
    DevBuf d_rlo, d_nn, d_na, d_sptr, d_stgt, d_rel, d_dptr, d_lptr, d_chdptr, d_chdtgt, d_mptr, d_mld, d_fws,
        d_nptr, d_ntgt, d_perm, d_invp, d_idx, d_bptr, d_fcc, d_sfronts, d_sverts, d_pnt, d_fbottom,
        d_fpending0, d_spending0, d_sdone0, d_tpending0, d_sync, d_tentries, d_sroots, d_fdsc, d_slot, d_ttasks, d_tfoff, d_tflags, d_croff,
        d_crng, d_err, d_sinfo_l, d_sinfo_r, d_sheavy;
    // the amalgamation map on the device: the caller's structure (R, Sp, St), each caller front's merged front
    // and the offsets of its blocks in the caller's arrays (merged plans only)
    DevBuf d_oR, d_oSp, d_oSt, d_ogroup, d_oDf, d_oLf, d_ostage;  // d_ostage: the caller's four arrays
    std::vector<int> pnt, height, rel;
    std::vector<int> sinfo_l, sinfo_r, sheavy;  // continuation of the bottom sweeps (host copies)
    std::vector<int> sfronts, sroots;  // host copies of the solve work lists (reordered by prepare_workspace)
    int maxh = 0;
    // values and work
    DevBuf LD, LL, UD, UL, Nval, W, X, stage_in, stage_out, csc_ptr, csc_row, csc_val, star_map;
    int64_t nD = 0, nL = 0;
    int64_t nnz_assembled = -1;
    size_t ws_esize = 0;
    pp_stats st{};
    Profiler prof;
    int sm_count = 148;
    // options (pp_options): the bound of the device waits on other CTAs (nanoseconds, kept on the device in
    // d_err[2..3]) and the allocation test hook
    uint64_t wait_ns = 0;
    int64_t fail_alloc_after = -1;
    // amalgamation: the caller's structure (0-based) and, when it has chains of top fronts to merge, the merged
    // one the device plan is built from (every semiring but PlusProd); group maps a caller's front to its
    // merged front.  The factor arrays on the device are in the plan's layout; pp_get_factor / pp_set_values
    // convert at the boundary.
    struct Structure {
        int64_t n = 0, nf = 0, nB = 0;
        std::vector<int64_t> R, Sp, St, Bp, Fp, Np, Nt, perm;
    } orig, mrg;
    std::vector<int> group;
    std::vector<double> ufac_pairs, ufac_elems, usolve_pairs;
    bool mergeable = false, merged = false;
    int merge_width = 64;
    bool trace_on = false;  // pp_options.trace
    DevBuf d_trace;
    // several GPUs (pp_comm_init): the NCCL communicator, this handle's rank, and every rank's part of the
    // bottom of the tree (element ranges of LD/UD, LL/UL and the workspace)
    void *comm = nullptr;
    int nranks = 1, rank = 0;
    bool comm_failed = false;
    double comm_wait_s = 60.0;  // bound of a host wait on the handle's streams while joined (seconds)
    std::string comm_msg;       // an NCCL failure met while enqueueing
    std::vector<Part> parts;
};

// Makes the handle's allocation budget the one DevBuf::ensure consults for the rest of the enclosing call.
struct AllocScope {
    int64_t *prev;
    explicit AllocScope(pp_handle *h) : prev(t_alloc_budget) { t_alloc_budget = h ? &h->fail_alloc_after : nullptr; }
    ~AllocScope() { t_alloc_budget = prev; }
};

static int32_t fail(pp_handle *h, int32_t code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    if (h) h->err = buf;
    return code;
}

static int32_t cuda_fail(pp_handle *h, cudaError_t e, const char *what) {
    if (e == cudaErrorMemoryAllocation) return fail(h, PP_ENOMEM, "%s: out of device memory", what);
    return fail(h, PP_EDEVICE, "%s: %s", what, cudaGetErrorString(e));
}

#define CK(h, x, what)                                         \
    do {                                                       \
        cudaError_t e_ = (x);                                  \
        if (e_ != cudaSuccess) return cuda_fail((h), e_, what); \
    } while (0)

static void ok(pp_handle *h) {
    g_err.clear();
    if (h) h->err.clear();
}

// Wait for a stream of the handle.  Joined into a group of GPUs, a collective whose peers never arrive would
// block for good: then the stream is polled, and after the group's bound (comm_wait_s) the communicator is
// aborted, which ends its collectives; the call reports cudaErrorLaunchTimeout and the handle leaves the group.
static cudaError_t stream_wait(pp_handle *h, cudaStream_t s) {
    if (!h->comm) return cudaStreamSynchronize(s);
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
        const cudaError_t e = cudaStreamQuery(s);
        if (e != cudaErrorNotReady) return e;
        ncclResult_t ae = ncclSuccess;
        const NcclApi &N = nccl_api();
        if (N.CommGetAsyncError(static_cast<ncclComm_t>(h->comm), &ae) != ncclSuccess || ae != ncclSuccess ||
            std::chrono::steady_clock::now() - t0 > std::chrono::duration<double>(h->comm_wait_s)) {
            N.CommAbort(static_cast<ncclComm_t>(h->comm));
            h->comm = nullptr;
            h->comm_failed = true;
            cudaStreamSynchronize(s);
            return cudaErrorLaunchTimeout;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

template <typename U>
static cudaError_t upload(DevBuf &b, const std::vector<U> &v, cudaStream_t st) {
    cudaError_t e = b.ensure(sizeof(U) * std::max<size_t>(v.size(), 1));
    if (e != cudaSuccess) return e;
    if (!v.empty()) e = cudaMemcpyAsync(b.p, v.data(), sizeof(U) * v.size(), cudaMemcpyHostToDevice, st);
    return e;
}

static int32_t check_pair(int32_t sr, int32_t dt) { return get_ops(sr, dt) ? PP_OK : PP_EUNSUPPORTED; }

extern "C" int32_t pp_version(void) { return 100; }

extern "C" int32_t pp_check_semiring(int32_t semiring, int32_t dtype) {
    if (check_pair(semiring, dtype) != PP_OK)
        return fail(nullptr, PP_EUNSUPPORTED, "semiring %d with element type %d is not supported", semiring, dtype);
    ok(nullptr);
    return PP_OK;
}

extern "C" const char *pp_last_error(const pp_handle *h) { return h ? h->err.c_str() : g_err.c_str(); }

extern "C" int32_t pp_create(int32_t device, pp_handle **out) {
    if (!out) return fail(nullptr, PP_EINVAL, "pp_create: null output pointer");
    *out = nullptr;
    int ndev = 0;
    cudaError_t e = cudaGetDeviceCount(&ndev);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "pp_create: no CUDA device");
    if (device < 0 || device >= ndev) return fail(nullptr, PP_EINVAL, "pp_create: device %d of %d", device, ndev);
    auto *h = new (std::nothrow) pp_handle();
    if (!h) return fail(nullptr, PP_ENOMEM, "pp_create: out of host memory");
    h->device = device;
    e = cudaSetDevice(device);
    int prio_low = 0, prio_high = 0;
    if (e == cudaSuccess) e = cudaDeviceGetStreamPriorityRange(&prio_low, &prio_high);
    if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&h->stream, cudaStreamNonBlocking, prio_low);
    if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&h->factor_stream, cudaStreamNonBlocking, prio_high);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&h->ev_bottom, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&h->ev_factored, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&h->ev_top_a, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreate(&h->ev0);
    if (e == cudaSuccess) e = cudaEventCreate(&h->ev1);
    if (e == cudaSuccess) e = cudaEventCreate(&h->fev0);
    if (e == cudaSuccess) e = cudaEventCreate(&h->fev1);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&h->copy_stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&h->copy_ev, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&h->out_stream, cudaStreamNonBlocking);
    for (int i = 0; i < pp_handle::kSolvePanels && e == cudaSuccess; i++) {
        e = cudaEventCreateWithFlags(&h->in_ev[i], cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&h->out_ev[i], cudaEventDisableTiming);
    }
    for (int i = 0; i < 2 && e == cudaSuccess; i++) {
        e = cudaEventCreateWithFlags(&h->panel_ready[i], cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&h->panel_copied[i], cudaEventDisableTiming);
    }
    for (int i = 0; i < 3 && e == cudaSuccess; i++) e = cudaEventCreateWithFlags(&h->ring_ev[i], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&h->sm_count, cudaDevAttrMultiProcessorCount, device);
    if (e != cudaSuccess) {
        pp_destroy(h);
        return cuda_fail(nullptr, e, "pp_create");
    }
    *out = h;
    ok(nullptr);
    return PP_OK;
}

extern "C" int32_t pp_destroy(pp_handle *h) {
    if (!h) return PP_OK;
    // best effort: the handle is released whatever the device's state
    if (cudaSetDevice(h->device) != cudaSuccess) cudaGetLastError();
    if (h->stream) stream_wait(h, h->stream);
    if (h->factor_stream) stream_wait(h, h->factor_stream);
    if (h->comm) {
        nccl_api().CommDestroy(static_cast<ncclComm_t>(h->comm));
        h->comm = nullptr;
    }
    if (h->ev0) cudaEventDestroy(h->ev0);
    if (h->ev1) cudaEventDestroy(h->ev1);
    if (h->fev0) cudaEventDestroy(h->fev0);
    if (h->fev1) cudaEventDestroy(h->fev1);
    if (h->copy_ev) cudaEventDestroy(h->copy_ev);
    if (h->factor_stream) {
        cudaStreamSynchronize(h->factor_stream);
        cudaStreamDestroy(h->factor_stream);
    }
    for (cudaEvent_t ev : {h->ev_bottom, h->ev_factored, h->ev_top_a})
        if (ev) cudaEventDestroy(ev);
    for (int i = 0; i < 2; i++) {
        if (h->panel_ready[i]) cudaEventDestroy(h->panel_ready[i]);
        if (h->panel_copied[i]) cudaEventDestroy(h->panel_copied[i]);
    }
    for (int i = 0; i < 3; i++)
        if (h->ring_ev[i]) cudaEventDestroy(h->ring_ev[i]);
    if (h->out_stream) {
        cudaStreamSynchronize(h->out_stream);
        cudaStreamDestroy(h->out_stream);
    }
    for (int i = 0; i < pp_handle::kSolvePanels; i++) {
        if (h->in_ev[i]) cudaEventDestroy(h->in_ev[i]);
        if (h->out_ev[i]) cudaEventDestroy(h->out_ev[i]);
    }
    if (h->copy_stream) {
        cudaStreamSynchronize(h->copy_stream);
        cudaStreamDestroy(h->copy_stream);
    }
    if (h->stream) cudaStreamDestroy(h->stream);
    delete h;  // DevBuf destructors free the device memory
    return PP_OK;
}

extern "C" void *pp_stream(pp_handle *h) { return h ? (void *)h->stream : nullptr; }

// ---------------------------------------------------------------- options

extern "C" void pp_default_options(pp_options *o) {
    if (!o) return;
    memset(o, 0, sizeof *o);
    o->wait_timeout_us = 0;
    o->fail_alloc_after = -1;
    o->profile = 0;
}

static int32_t apply_options(pp_handle *h, const pp_options *o, const char *who) {
    if (o->wait_timeout_us < 0) return fail(h, PP_EINVAL, "%s: wait_timeout_us = %lld", who, (long long)o->wait_timeout_us);
    if (o->merge_width < 0) return fail(h, PP_EINVAL, "%s: merge_width = %d", who, o->merge_width);
    if (o->wait_timeout_us > (int64_t)1 << 40) return fail(h, PP_EINVAL, "%s: wait_timeout_us too large", who);
    h->wait_ns = (uint64_t)o->wait_timeout_us * 1000u;
    h->fail_alloc_after = o->fail_alloc_after < 0 ? -1 : o->fail_alloc_after;
    if (h->d_err.p) {
        // nothing of the handle may be running while the bound changes; the copy is synchronous
        CK(h, stream_wait(h, h->factor_stream), who);
        CK(h, stream_wait(h, h->stream), who);
        CK(h, cudaMemcpy(h->d_err.as<int>() + 2, &h->wait_ns, sizeof(uint64_t), cudaMemcpyHostToDevice), who);
    }
    h->prof.on = o->profile != 0;
    h->merge_width = o->merge_width == 0 ? 64 : o->merge_width;
    h->trace_on = o->trace != 0;
    return PP_OK;
}

extern "C" int32_t pp_create_with(int32_t device, const pp_options *opt, pp_handle **out) {
    const int32_t r = pp_create(device, out);
    if (r != PP_OK || !opt) return r;
    const int32_t r2 = apply_options(*out, opt, "pp_create_with");
    if (r2 != PP_OK) {
        const std::string msg = (*out)->err;
        pp_destroy(*out);
        *out = nullptr;
        return fail(nullptr, r2, "%s", msg.c_str());
    }
    return PP_OK;
}

extern "C" int32_t pp_set_options(pp_handle *h, const pp_options *opt) {
    if (!h || !opt) return fail(h, PP_EINVAL, "pp_set_options: null argument");
    CK(h, cudaSetDevice(h->device), "pp_set_options");
    const int32_t r = apply_options(h, opt, "pp_set_options");
    if (r == PP_OK) ok(h);
    return r;
}

extern "C" int32_t pp_get_options(const pp_handle *h, pp_options *opt) {
    if (!h || !opt) return fail(nullptr, PP_EINVAL, "pp_get_options: null argument");
    pp_default_options(opt);
    opt->wait_timeout_us = (int64_t)(h->wait_ns / 1000u);
    opt->fail_alloc_after = h->fail_alloc_after;
    opt->profile = h->prof.on ? 1 : 0;
    opt->merge_width = h->merge_width;
    opt->trace = h->trace_on ? 1 : 0;
    return PP_OK;
}

// ---------------------------------------------------------------- structure

// Order of the fronts of one persistent launch (a bottom sweep, or the factorization of the bottom).  The
// launch hands its tasks to warps or CTAs in list order and one whose task is not ready waits, so the list
// follows a schedule simulated on the host: `slots` fronts at a time, front f costing fcost[f] (estimated
// microseconds), ready once its dependencies are done (up: its children in the list, as in a forward sweep or
// the factorization; down: its parent, as in a backward sweep), the ready front with the longest path of
// remaining work first.  Every front comes after the fronts it depends on.
static std::vector<int> schedule_order(const std::vector<int> &fronts, const std::vector<double> &fcost,
                                       const std::vector<int> &pnt, bool up, int slots) {
    const int m = (int)fronts.size();
    std::vector<int> pos(pnt.size(), -1);
    for (int i = 0; i < m; i++) pos[fronts[i]] = i;
    std::vector<double> cost(m), path(m, 0.0);
    std::vector<int> deps(m, 0), par(m, -1);
    for (int i = 0; i < m; i++) {
        const int f = fronts[i];
        cost[i] = fcost[f];
        par[i] = pnt[f] >= 0 ? pos[pnt[f]] : -1;
    }
    // the fronts arrive in height order (ascending for the forward list, descending for the backward one), so
    // a parent's position is after (forward) or before (backward) its children's
    std::vector<std::vector<int>> kids(m);
    for (int i = 0; i < m; i++)
        if (par[i] >= 0) kids[par[i]].push_back(i);
    if (up) {
        for (int i = m - 1; i >= 0; i--) path[i] = cost[i] + (par[i] >= 0 ? path[par[i]] : 0.0);
        for (int i = 0; i < m; i++) deps[i] = (int)kids[i].size();
    } else {
        for (int i = m - 1; i >= 0; i--) {
            double mx = 0;
            for (int c : kids[i]) mx = std::max(mx, path[c]);
            path[i] = cost[i] + mx;
        }
        for (int i = 0; i < m; i++) deps[i] = par[i] >= 0 ? 1 : 0;
    }
    using Ready = std::pair<double, int>;  // (remaining path, front)
    std::priority_queue<Ready> ready;
    using Run = std::pair<double, int>;  // (finish time, front), earliest first
    std::priority_queue<Run, std::vector<Run>, std::greater<Run>> running;
    for (int i = 0; i < m; i++)
        if (deps[i] == 0) ready.push({path[i], i});
    std::vector<int> order;
    order.reserve(m);
    double now = 0;
    while ((int)order.size() < m) {
        while (!ready.empty() && (int)running.size() < std::max(slots, 1)) {
            const int i = ready.top().second;
            ready.pop();
            order.push_back(fronts[i]);
            running.push({now + cost[i], i});
        }
        if (running.empty()) break;  // unreachable: the dependencies form a forest
        const Run r = running.top();
        running.pop();
        now = r.first;
        const int i = r.second;
        if (up) {
            if (par[i] >= 0 && --deps[par[i]] == 0) ready.push({path[par[i]], par[i]});
        } else {
            for (int c : kids[i])
                if (--deps[c] == 0) ready.push({path[c], c});
        }
    }
    return order;
}

static cudaError_t exchange_parts(void *ctx, cudaStream_t st);  // the split factorization's exchange (below)
static cudaError_t upload_merge_map(pp_handle *h, cudaStream_t st);  // the amalgamation map's inputs (below)

// Unpadded algorithmic costs per front of a merged plan (see HostPlan::ufac_pairs).
struct UCost {
    std::vector<double> fpairs, felems, spairs;
};

// Check the structure and build the device plan from it (pp_set_structure's work).  uc: the unpadded costs
// when the structure is a merged one.
static int32_t build_structure(pp_handle *h, int64_t n, int64_t nf, int64_t nB, const int64_t *Rptr,
                               const int64_t *Sptr, const int64_t *Stgt, const int64_t *Bptr, const int64_t *Fptr,
                               const int64_t *Nptr, const int64_t *Ntgt, const int64_t *perm, int32_t base,
                               const UCost *uc) {
    if (!h) return fail(nullptr, PP_EINVAL, "pp_set_structure: null handle");
    if (n < 0 || nf < 0 || nB < 0 || (n > 0 && (nf < 1 || nB < 1)) || n >= INT32_MAX)
        return fail(h, PP_EINVAL, "pp_set_structure: sizes n=%lld nf=%lld nB=%lld", (long long)n, (long long)nf,
                    (long long)nB);
    if (n > 0 && (!Rptr || !Sptr || !Bptr || !Fptr || !Nptr || !perm))
        return fail(h, PP_EINVAL, "pp_set_structure: null array");
    if (base != 0 && base != 1) return fail(h, PP_EINVAL, "pp_set_structure: base must be 0 or 1");
    CK(h, cudaSetDevice(h->device), "pp_set_structure");
    if (h->factor_stream) stream_wait(h, h->factor_stream);  // nothing in flight reads the old plan
    h->have_structure = h->have_values = h->factored = false;
    h->nnz_assembled = -1;
    HostPlan hp;
    hp.n = (int)n;
    hp.nf = (int)nf;
    hp.nB = (int)nB;
    const int64_t b = base;
    try {
        std::vector<int64_t> R(nf + 1), Sp(nf + 1), Bp(nB + 1), Fp(nB + 1), Np(n + 1);
        for (int64_t i = 0; i <= nf; i++) {
            R[i] = Rptr[i] - b;
            Sp[i] = Sptr[i] - b;
        }
        for (int64_t i = 0; i <= nB; i++) {
            Bp[i] = Bptr[i] - b;
            Fp[i] = Fptr[i] - b;
        }
        for (int64_t i = 0; i <= n; i++) Np[i] = Nptr[i] - b;
        if (R[0] != 0 || R[nf] != n || Sp[0] != 0 || Bp[0] != 0 || Bp[nB] != n || Fp[0] != 0 || Fp[nB] != nf ||
            Np[0] != 0)
            return fail(h, PP_EINVAL, "pp_set_structure: pointer arrays must start at the base and end at n/nf");
        const int64_t nS = Sp[nf], nN = Np[n];
        if (nS < 0 || nN < 0 || (nS > 0 && !Stgt) || (nN > 0 && !Ntgt))
            return fail(h, PP_EINVAL, "pp_set_structure: separator/coupling arrays");
        if (nS >= INT32_MAX || nN >= ((int64_t)1 << 40)) return fail(h, PP_EINVAL, "pp_set_structure: too large");
        hp.nn.resize(nf);
        hp.na.resize(nf);
        hp.sptr.resize(nf + 1);
        hp.dptr.assign(nf + 1, 0);
        hp.lptr.assign(nf + 1, 0);
        std::vector<int> rlo(nf), idx(n), stgt(nS), rel(nS), pnt(nf, -1), fcc(nf), permv(n), invp(n, -1), bptr(nB + 1);
        for (int64_t f = 0; f < nf; f++) {
            const int64_t nn = R[f + 1] - R[f], na = Sp[f + 1] - Sp[f];
            if (nn <= 0 || na < 0) return fail(h, PP_EINVAL, "pp_set_structure: front %lld is empty", (long long)f);
            rlo[f] = (int)R[f];
            hp.nn[f] = (int)nn;
            hp.na[f] = (int)na;
            hp.sptr[f] = Sp[f];
            hp.dptr[f + 1] = hp.dptr[f] + nn * nn;
            hp.lptr[f + 1] = hp.lptr[f] + nn * na;
            for (int64_t v = R[f]; v < R[f + 1]; v++) idx[v] = (int)f;
        }
        hp.sptr[nf] = nS;
        for (int64_t q = 0; q < nS; q++) {
            const int64_t v = Stgt[q] - b;
            if (v < 0 || v >= n) return fail(h, PP_EINVAL, "pp_set_structure: separator vertex out of range");
            stgt[q] = (int)v;
        }
        for (int64_t i = 0; i < n; i++) {
            const int64_t v = perm[i] - b;
            if (v < 0 || v >= n || invp[v] >= 0) return fail(h, PP_EINVAL, "pp_set_structure: perm is not a permutation");
            permv[i] = (int)v;
            invp[v] = (int)i;
        }
        // parents, relative indices, children (fronts in postorder: every parent after its children)
        std::vector<int> nchd(nf + 1, 0);
        for (int64_t f = 0; f < nf; f++) {
            const int na = hp.na[f];
            if (na == 0) continue;
            const int v0 = stgt[Sp[f]];
            if (v0 < R[f + 1]) return fail(h, PP_EINVAL, "pp_set_structure: separator of front %lld overlaps it", (long long)f);
            const int p = idx[v0];
            pnt[f] = p;
            nchd[p + 1]++;
            const int pr = rlo[p], pnn = hp.nn[p];
            int64_t q = Sp[p];
            for (int64_t k = Sp[f]; k < Sp[f + 1]; k++) {
                const int v = stgt[k];
                if (k > Sp[f] && v <= stgt[k - 1]) return fail(h, PP_EINVAL, "pp_set_structure: separator not sorted");
                if (v < pr) return fail(h, PP_EINVAL, "pp_set_structure: separator vertex before the parent");
                if (v < pr + pnn) {
                    rel[k] = v - pr;
                } else {
                    while (q < Sp[p + 1] && stgt[q] < v) q++;
                    if (q >= Sp[p + 1] || stgt[q] != v)
                        return fail(h, PP_EINVAL, "pp_set_structure: separator of front %lld not in its parent's bag",
                                    (long long)f);
                    rel[k] = pnn + (int)(q - Sp[p]);
                }
            }
        }
        hp.chdptr.assign(nf + 1, 0);
        for (int64_t f = 0; f < nf; f++) hp.chdptr[f + 1] = hp.chdptr[f] + nchd[f + 1];
        hp.chdtgt.assign(std::max<int64_t>(hp.chdptr[nf], 1), 0);
        {
            std::vector<int> fill(hp.chdptr.begin(), hp.chdptr.end() - 1);
            for (int64_t f = 0; f < nf; f++)
                if (pnt[f] >= 0) hp.chdtgt[fill[pnt[f]]++] = (int)f;
        }
        for (int64_t c = 0; c < nB; c++) {
            if (Bp[c + 1] < Bp[c] || Fp[c + 1] < Fp[c]) return fail(h, PP_EINVAL, "pp_set_structure: component pointers");
            bptr[c] = (int)Bp[c];
            for (int64_t f = Fp[c]; f < Fp[c + 1]; f++) fcc[f] = (int)c;
            if (Fp[c + 1] > Fp[c] && (R[Fp[c]] != Bp[c] || R[Fp[c + 1]] != Bp[c + 1]))
                return fail(h, PP_EINVAL, "pp_set_structure: component %lld fronts do not cover its vertices", (long long)c);
        }
        bptr[nB] = (int)n;
        std::vector<int> ntgt(std::max<int64_t>(nN, 1), 0);
        for (int64_t j = 0; j < n; j++) {
            if (Np[j + 1] < Np[j]) return fail(h, PP_EINVAL, "pp_set_structure: coupling pointers");
            const int jstrt = bptr[fcc[idx[j]]];
            for (int64_t p = Np[j]; p < Np[j + 1]; p++) {
                const int64_t i = Ntgt[p] - b;
                if (i < 0 || i >= jstrt) return fail(h, PP_EINVAL, "pp_set_structure: coupling row not in an earlier component");
                if (p > Np[j] && i <= ntgt[p - 1]) return fail(h, PP_EINVAL, "pp_set_structure: coupling rows not sorted");
                ntgt[p] = (int)i;
            }
        }
        hp.nN = nN;
        // heights: leaves 0, a parent one above its highest child
        std::vector<int> height(nf, 0);
        int maxh = 0;
        for (int64_t f = 0; f < nf; f++) {
            if (pnt[f] >= 0) {
                if (pnt[f] <= f) return fail(h, PP_EINVAL, "pp_set_structure: fronts are not in postorder");
                height[pnt[f]] = std::max(height[pnt[f]], height[f] + 1);
            }
            maxh = std::max(maxh, height[f]);
        }
        // coupling stages
        std::vector<int> comp_of_vertex(n);
        for (int64_t c = 0; c < nB; c++)
            for (int64_t v = Bp[c]; v < Bp[c + 1]; v++) comp_of_vertex[v] = (int)c;
        std::vector<int> lstage(nB, 0), rstage(nB, 0);
        std::vector<char> ccoupled(nB, 0);
        for (int64_t c = 0; c < nB; c++)  // rmul: after every predecessor
            for (int64_t j = Bp[c]; j < Bp[c + 1]; j++)
                for (int64_t p = Np[j]; p < Np[j + 1]; p++) {
                    const int a = comp_of_vertex[ntgt[p]];
                    rstage[c] = std::max(rstage[c], rstage[a] + 1);
                    ccoupled[c] = 1;
                }
        // lmul: after every successor (successors have larger indices)
        for (int64_t c = nB - 1; c >= 0; c--)
            for (int64_t j = Bp[c]; j < Bp[c + 1]; j++)
                for (int64_t p = Np[j]; p < Np[j + 1]; p++) {
                    const int a = comp_of_vertex[ntgt[p]];
                    lstage[a] = std::max(lstage[a], lstage[c] + 1);
                }
        // bottom of the tree for the persistent sweeps: nn <= SWEEP_NNW and nn + na <= SWEEP_NJW in the whole
        // subtree
        std::vector<char> sbot(nf, 0), allbot(nf, 1);
        for (int64_t f = 0; f < nf; f++) {
            sbot[f] = (hp.nn[f] <= SWEEP_NNW) && (hp.nn[f] + hp.na[f] <= SWEEP_NJW) && allbot[f];
            if (!sbot[f] && pnt[f] >= 0) allbot[pnt[f]] = 0;
        }
        // subtrees solved in shared memory: the whole subtree is in the bottom, its residual range plus the
        // root's separator fit SUBTREE_ROWS rows, and its fronts' factor blocks and separator slots fit the
        // staging areas (contiguous ranges, the subtree's fronts being contiguous); maximal such subtrees are
        // disjoint
        std::vector<int> fdsc(nf);
        for (int64_t f = 0; f < nf; f++) fdsc[f] = (int)f;
        for (int64_t f = 0; f < nf; f++)
            if (pnt[f] >= 0) fdsc[pnt[f]] = std::min(fdsc[pnt[f]], fdsc[f]);
        std::vector<char> qual(nf, 0), covered(nf, 0);
        for (int64_t f = 0; f < nf; f++)
            qual[f] = sbot[f] && (R[f + 1] - R[fdsc[f]] + hp.na[f] <= SUBTREE_ROWS) &&
                      (hp.dptr[f + 1] - hp.dptr[fdsc[f]] + hp.lptr[f + 1] - hp.lptr[fdsc[f]] <= SUBTREE_FAC) &&
                      (Sp[f + 1] - Sp[fdsc[f]] <= SUBTREE_SLOTS);
        std::vector<int> sroot_of(nf, -1);
        for (int64_t f = nf - 1; f >= 0; f--) {
            if (!qual[f]) continue;
            if (pnt[f] >= 0 && qual[pnt[f]]) {
                sroot_of[f] = sroot_of[pnt[f]];
            } else {
                sroot_of[f] = (int)f;
            }
            covered[f] = 1;
        }
        std::vector<int> slot(std::max<int64_t>(nS, 1), 0);
        for (int64_t f = 0; f < nf; f++) {
            if (!covered[f]) continue;
            const int r = sroot_of[f];
            const int64_t rlo0 = R[fdsc[r]], rhi = R[r + 1] - 1, nres = rhi - rlo0 + 1;
            for (int64_t q = Sp[f]; q < Sp[f + 1]; q++) {
                const int v = stgt[q];
                if (v <= rhi) {
                    slot[q] = (int)(v - rlo0);
                } else {
                    const int *b0 = stgt.data() + Sp[r], *b1 = stgt.data() + Sp[r + 1];
                    const int *it = std::lower_bound(b0, b1, v);
                    if (it == b1 || *it != v)
                        return fail(h, PP_EINVAL, "pp_set_structure: separator of front %lld leaves its subtree",
                                    (long long)f);
                    slot[q] = (int)(nres + (it - b0));
                }
            }
        }
        std::vector<int> spending0(nf, 0), sdone0(nf, 1), tpending0(nf, 0);
        for (int64_t f = 0; f < nf; f++) {
            const bool mid = sbot[f] && !covered[f];
            if (mid) sdone0[f] = 0;
            if (mid && pnt[f] >= 0) spending0[pnt[f]]++;
            if (mid) {
                hp.bot_fmax = std::max(hp.bot_fmax, hp.nn[f] * hp.nn[f] + hp.nn[f] * hp.na[f]);
                hp.bot_namax = std::max(hp.bot_namax, hp.na[f]);
            }
            if (!sbot[f] && pnt[f] >= 0) tpending0[pnt[f]]++;  // top children (the top sweep's counters)
        }
        // estimated time of a (front, 32-column tile) task of the bottom sweeps, fitted to measured task times
        std::vector<double> scost(nf);
        for (int64_t f = 0; f < nf; f++) scost[f] = 4.0 + hp.nn[f] * (double)hp.na[f] / 36.0;
        // and of a (front, 32-column tile) task of the top sweeps: the diagonal solve, the off-diagonal block
        std::vector<double> tscost(nf);
        for (int64_t f = 0; f < nf; f++) tscost[f] = 5.0 + hp.nn[f] / 8.0 + hp.nn[f] * (double)hp.na[f] / 1024.0;
        std::vector<double> subtree_cost(nf, 0.0);  // of a subtree root: its fronts' estimated task times
        for (int64_t f = 0; f < nf; f++)
            if (covered[f]) subtree_cost[sroot_of[f]] += scost[f];
        hp.stree_pairs.assign(nf, 0.0);
        hp.stree_res.assign(nf, 0.0);
        hp.stree_sep.assign(nf, 0.0);
        hp.stree_fac.assign(nf, 0.0);
        for (int64_t f = 0; f < nf; f++) {
            if (!covered[f]) continue;
            const int r = sroot_of[f];
            const double nn = hp.nn[f], na = hp.na[f];
            hp.stree_pairs[r] += nn * (nn - 1) / 2 + nn * na;
            hp.stree_fac[r] += nn * nn + nn * na;
            if (r == f) {
                hp.stree_res[r] = (double)(R[f + 1] - R[fdsc[f]]);
                hp.stree_sep[r] = na;
            }
        }
        if (uc) {
            hp.ufac_pairs = uc->fpairs;
            hp.ufac_elems = uc->felems;
            hp.usolve_pairs = uc->spairs;
        }
        // (x)(+) pairs of one right-hand side through the L* (or U*) part of front f, unpadded
        auto col_pairs = [&](int64_t f) {
            if (!hp.usolve_pairs.empty()) return hp.usolve_pairs[f];
            const double nn = hp.nn[f], na = hp.na[f];
            return nn * (nn - 1) / 2 + nn * na;
        };
        auto build_stages = [&](const std::vector<int> &stage_of, std::vector<Stage> &out, std::vector<int> &sfronts,
                                std::vector<int> &sverts, std::vector<std::pair<int64_t, int>> &bfwd,
                                std::vector<std::pair<int64_t, int>> &bbwd, std::vector<SLevel> &bcost,
                                std::vector<SubtreeList> &subs, std::vector<int> &sroots,
                                std::vector<std::pair<int64_t, int>> &tfwd, std::vector<std::pair<int64_t, int>> &tbwd,
                                std::vector<SLevel> &tcost, std::vector<int> &tentries, std::vector<int> &tfa) {
            int ns = 0;
            for (int64_t c = 0; c < nB; c++) ns = std::max(ns, stage_of[c] + 1);
            if (nB == 0) ns = 0;
            std::vector<std::vector<int>> comps(ns);
            for (int64_t c = 0; c < nB; c++) comps[stage_of[c]].push_back((int)c);
            out.clear();
            bfwd.clear();
            bbwd.clear();
            bcost.clear();
            subs.clear();
            tfwd.clear();
            tbwd.clear();
            tcost.clear();
            tfa.clear();
            for (int s = 0; s < ns; s++) {
                Stage sg;
                std::vector<std::vector<int>> byh(maxh + 1), bot(maxh + 1);
                SubtreeList sl;
                sl.off = (int64_t)sroots.size();
                for (int c : comps[s])
                    for (int64_t f = Fp[c]; f < Fp[c + 1]; f++) {
                        if (covered[f]) {
                            if (sroot_of[f] == f) sroots.push_back((int)f);
                            continue;
                        }
                        (sbot[f] ? bot : byh)[height[f]].push_back((int)f);
                    }
                sl.count = (int)(sroots.size() - sl.off);
                // the launch runs its subtrees in list order: the longest first
                std::stable_sort(sroots.begin() + sl.off, sroots.end(),
                                 [&](int a, int b) { return subtree_cost[a] > subtree_cost[b]; });
                subs.push_back(sl);
                SLevel bc;
                std::vector<int> up;  // the stage's other bottom fronts, children first
                for (int hh = 0; hh <= maxh; hh++) up.insert(up.end(), bot[hh].begin(), bot[hh].end());
                std::vector<int> down(up.rbegin(), up.rend());
                // fronts in flight: the launch's warps (8 per SM) over the tiles of a front (8 for 256 columns)
                const int fslots = h->sm_count;
                std::pair<int64_t, int> fw{(int64_t)sfronts.size(), 0};
                for (int f : schedule_order(up, scost, pnt, true, fslots)) {
                    sfronts.push_back(f);
                    const double nn = hp.nn[f], na = hp.na[f];
                    bc.count++;
                    bc.res_rows += nn;
                    bc.sep_rows += na;
                    bc.blk_elems += nn * nn + nn * na;
                    bc.pairs_col += col_pairs(f);
                }
                fw.second = (int)(sfronts.size() - fw.first);
                std::pair<int64_t, int> bw{(int64_t)sfronts.size(), 0};
                for (int f : schedule_order(down, scost, pnt, false, fslots)) sfronts.push_back(f);
                bw.second = (int)(sfronts.size() - bw.first);
                bfwd.push_back(fw);
                bbwd.push_back(bw);
                bcost.push_back(bc);
                // the top fronts: one work list per direction, schedule-ordered like the bottom ones (a CTA per
                // (front, tile) task, about two CTAs per SM over the eight tiles of a front); entries (front,
                // block of 64 rows): forward the residual blocks ascending, then the separator blocks, backward the
                // residual blocks descending
                SLevel tc;
                std::vector<int> tup;
                for (int hh = 0; hh <= maxh; hh++) tup.insert(tup.end(), byh[hh].begin(), byh[hh].end());
                std::vector<int> tdown(tup.rbegin(), tup.rend());
                const int tslots = std::max(1, h->sm_count / 4);
                auto blocks = [](int m) { return (m + TOP_SWEEP_ROWS - 1) / TOP_SWEEP_ROWS; };
                std::pair<int64_t, int> tf{(int64_t)tentries.size() / 2, 0};
                for (int f : schedule_order(tup, tscost, pnt, true, tslots)) {
                    for (int b = 0; b < blocks(hp.nn[f]) + blocks(hp.na[f]); b++) tentries.insert(tentries.end(), {f, b});
                    const double nn = hp.nn[f], na = hp.na[f];
                    tc.count++;
                    tc.res_rows += nn;
                    tc.sep_rows += na;
                    tc.blk_elems += nn * nn + nn * na;
                    tc.pairs_col += col_pairs(f);
                }
                tf.second = (int)(tentries.size() / 2 - tf.first);
                {
                    // the roots' entries last (a root is forward-swept once the whole factorization has ended)
                    std::vector<std::pair<int, int>> ent(tf.second);
                    for (int i = 0; i < tf.second; i++)
                        ent[i] = {tentries[2 * (tf.first + i)], tentries[2 * (tf.first + i) + 1]};
                    std::stable_partition(ent.begin(), ent.end(),
                                          [&](const std::pair<int, int> &e) { return pnt[e.first] >= 0; });
                    int na = 0;
                    for (int i = 0; i < tf.second; i++) {
                        tentries[2 * (tf.first + i)] = ent[i].first;
                        tentries[2 * (tf.first + i) + 1] = ent[i].second;
                        if (pnt[ent[i].first] >= 0) na++;
                    }
                    tfa.push_back(na);
                }
                std::pair<int64_t, int> tb{(int64_t)tentries.size() / 2, 0};
                for (int f : schedule_order(tdown, tscost, pnt, false, tslots))
                    for (int b = blocks(hp.nn[f]) - 1; b >= 0; b--) tentries.insert(tentries.end(), {f, b});
                tb.second = (int)(tentries.size() / 2 - tb.first);
                tfwd.push_back(tf);
                tbwd.push_back(tb);
                tcost.push_back(tc);
                sg.voff = (int64_t)sverts.size();
                for (int c : comps[s])
                    for (int64_t j = Bp[c]; j < Bp[c + 1]; j++)
                        if (Np[j + 1] > Np[j]) sverts.push_back((int)j);
                sg.nverts = (int)(sverts.size() - sg.voff);
                sg.coupled = sg.nverts > 0;
                out.push_back(std::move(sg));
            }
        };
        std::vector<int> sfronts, sverts, sroots, tentries;
        build_stages(lstage, hp.lstages, sfronts, sverts, hp.sb_fwd, hp.sb_bwd, hp.sb_cost_l, hp.sub_l, sroots,
                     hp.st_fwd, hp.st_bwd, hp.st_cost_l, tentries, hp.st_fwd_a);
        // rmul stages: the gather concerns the stage's own columns j (rows of earlier components feed them)
        build_stages(rstage, hp.rstages, sfronts, sverts, hp.sb_fwd_r, hp.sb_bwd_r, hp.sb_cost_r, hp.sub_r, sroots,
                     hp.st_fwd_r, hp.st_bwd_r, hp.st_cost_r, tentries, hp.st_fwd_r_a);
        (void)ccoupled;
        std::vector<int64_t> Np64(Np.begin(), Np.end());
        // device uploads
        cudaStream_t st = h->stream;
        CK(h, upload(h->d_rlo, rlo, st), "upload");
        CK(h, upload(h->d_nn, hp.nn, st), "upload");
        CK(h, upload(h->d_na, hp.na, st), "upload");
        CK(h, upload(h->d_sptr, hp.sptr, st), "upload");
        CK(h, upload(h->d_stgt, stgt, st), "upload");
        CK(h, upload(h->d_rel, rel, st), "upload");
        CK(h, upload(h->d_dptr, hp.dptr, st), "upload");
        CK(h, upload(h->d_lptr, hp.lptr, st), "upload");
        CK(h, upload(h->d_chdptr, hp.chdptr, st), "upload");
        CK(h, upload(h->d_chdtgt, hp.chdtgt, st), "upload");
        CK(h, upload(h->d_nptr, Np64, st), "upload");
        CK(h, upload(h->d_ntgt, ntgt, st), "upload");
        CK(h, upload(h->d_perm, permv, st), "upload");
        CK(h, upload(h->d_invp, invp, st), "upload");
        CK(h, upload(h->d_idx, idx, st), "upload");
        CK(h, upload(h->d_bptr, bptr, st), "upload");
        CK(h, upload(h->d_fcc, fcc, st), "upload");
        CK(h, upload(h->d_sfronts, sfronts, st), "upload");
        CK(h, upload(h->d_tentries, tentries, st), "upload");
        CK(h, upload(h->d_sverts, sverts, st), "upload");
        CK(h, upload(h->d_pnt, pnt, st), "upload");
        CK(h, upload(h->d_sroots, sroots, st), "upload");
        CK(h, upload(h->d_fdsc, fdsc, st), "upload");
        CK(h, upload(h->d_slot, slot, st), "upload");
        CK(h, upload(h->d_spending0, spending0, st), "upload");
        CK(h, upload(h->d_sdone0, sdone0, st), "upload");
        CK(h, upload(h->d_tpending0, tpending0, st), "upload");
        CK(h, h->d_sync.ensure(sizeof(int) * sync_ints(nf, 256)), "upload");
        CK(h, h->d_err.ensure(sizeof(int) * 4), "upload");
        CK(h, cudaMemsetAsync(h->d_err.p, 0, sizeof(int) * 4, st), "upload");
        CK(h, cudaMemcpyAsync(h->d_err.as<int>() + 2, &h->wait_ns, sizeof(uint64_t), cudaMemcpyHostToDevice, st),
           "upload");
        CK(h, stream_wait(h, st), "upload");
        DevPlan &d = hp.dev;
        d.n = (int)n;
        d.nf = (int)nf;
        d.nB = (int)nB;
        d.rlo = h->d_rlo.as<int>();
        d.nn = h->d_nn.as<int>();
        d.na = h->d_na.as<int>();
        d.sptr = h->d_sptr.as<int64_t>();
        d.stgt = h->d_stgt.as<int>();
        d.rel = h->d_rel.as<int>();
        d.dptr = h->d_dptr.as<int64_t>();
        d.lptr = h->d_lptr.as<int64_t>();
        d.chdptr = h->d_chdptr.as<int>();
        d.chdtgt = h->d_chdtgt.as<int>();
        d.nptr = h->d_nptr.as<int64_t>();
        d.ntgt = h->d_ntgt.as<int>();
        d.perm = h->d_perm.as<int>();
        d.invp = h->d_invp.as<int>();
        d.idx = h->d_idx.as<int>();
        d.bptr = h->d_bptr.as<int>();
        d.fcc = h->d_fcc.as<int>();
        d.pnt = h->d_pnt.as<int>();
        d.mptr = nullptr;
        d.mld = nullptr;
        d.fws = nullptr;
        hp.d_sfronts = h->d_sfronts.as<int>();
        hp.d_tentries = reinterpret_cast<const int2 *>(h->d_tentries.p);
        hp.d_sverts = h->d_sverts.as<int>();
        hp.d_rel = h->d_rel.as<int>();
        hp.d_spending0 = h->d_spending0.as<int>();
        hp.d_sroots = h->d_sroots.as<int>();
        hp.d_fdsc = h->d_fdsc.as<int>();
        hp.d_slot = h->d_slot.as<int>();
        hp.d_sdone0 = h->d_sdone0.as<int>();
        hp.d_tpending0 = h->d_tpending0.as<int>();
        hp.d_sync = h->d_sync.as<int>();
        hp.d_err = h->d_err.as<int>();
        hp.sync_cap = sync_ints(nf, 256);
        hp.sm_count = h->sm_count;
        hp.ev_bottom = h->ev_bottom;
        hp.ev_factored = h->ev_factored;
        hp.ev_top_a = h->ev_top_a;
        hp.top_stream = h->factor_stream;
        // a handle joined to a group of GPUs (pp_comm_init) before its structure was set keeps the exchange of
        // the ranks' parts
        hp.exchange = h->nranks > 1 ? exchange_parts : nullptr;
        hp.exchange_ctx = h->nranks > 1 ? h : nullptr;
        h->invp = invp;
        h->pnt = pnt;
        h->sfronts = sfronts;
        h->sroots = sroots;
        h->height = height;  // factorization heights and rel, kept for prepare_workspace
        h->rel = rel;
        h->maxh = maxh;
        h->hp = std::move(hp);
        h->hp.mld.clear();
        h->hp.esize = 0;
        h->nD = h->hp.dptr[nf];
        h->nL = h->hp.lptr[nf];
        h->ws_esize = 0;
        // counters
        pp_stats &s = h->st;
        s = pp_stats{};
        s.n = n;
        s.nf = nf;
        s.nB = nB;
        s.nlevels = maxh + 1;
        s.nD = h->nD;
        s.nL = h->nL;
        s.nN = nN;
        double pairs = 0;
        int64_t mx = 0;
        for (int64_t f = 0; f < nf; f++) {
            const double nn = h->hp.nn[f], na = h->hp.na[f], nj = nn + na;
            auto S2 = [](double m) { return (m - 1) * m * (2 * m - 1) / 6; };
            pairs += uc ? uc->fpairs[f] : S2(nj) - S2(na);
            mx = std::max<int64_t>(mx, (int64_t)nj);
        }
        s.pairs_factor = pairs;
        s.max_front = mx;
        s.plan_fronts = nf;
    } catch (const std::bad_alloc &) {
        return fail(h, PP_ENOMEM, "pp_set_structure: out of host memory");
    }
    h->have_structure = true;
    ok(h);
    return PP_OK;
}

// ---------------------------------------------------------------- several GPUs

// Every rank's part of the bottom of the tree to every rank: per part and factor array (and the workspace,
// which holds the update matrices the top of the tree reads) one NCCL broadcast from the part's rank, in place,
// all in one group on the calling stream.
static cudaError_t exchange_parts(void *ctx, cudaStream_t st) {
    pp_handle *h = static_cast<pp_handle *>(ctx);
    const NcclApi &N = nccl_api();
    const size_t es = h->ops->esize;
    ncclComm_t comm = static_cast<ncclComm_t>(h->comm);
    if (!comm) {
        h->comm_msg = "the handle left its group of GPUs after an earlier failure";
        return cudaErrorInvalidValue;
    }
    ncclResult_t r = N.GroupStart();
    for (int q = 0; q < h->nranks && r == ncclSuccess; q++) {
        const Part &pt = h->parts[q];
        const struct {
            void *p;
            int64_t a, b;
        } seg[5] = {{h->LD.p, pt.d0, pt.d1}, {h->UD.p, pt.d0, pt.d1}, {h->LL.p, pt.l0, pt.l1},
                    {h->UL.p, pt.l0, pt.l1}, {h->W.p, pt.w0, pt.w1}};
        for (const auto &g : seg)
            if (g.b > g.a && r == ncclSuccess) {
                char *p = static_cast<char *>(g.p) + es * (size_t)g.a;
                r = N.Broadcast(p, p, es * (size_t)(g.b - g.a), ncclUint8, q, comm, st);
            }
    }
    const ncclResult_t r2 = N.GroupEnd();
    if (r != ncclSuccess || r2 != ncclSuccess) {
        h->comm_msg = std::string("NCCL: ") + N.GetErrorString(r != ncclSuccess ? r : r2);
        return cudaErrorInvalidValue;
    }
    return cudaSuccess;
}

extern "C" int32_t pp_comm_id(void *id) {
    if (!id) return fail(nullptr, PP_EINVAL, "pp_comm_id: null id");
    const NcclApi &N = nccl_api();
    if (!N.ok) return fail(nullptr, PP_EUNSUPPORTED, "pp_comm_id: %s", N.why.c_str());
    ncclUniqueId u;
    const ncclResult_t r = N.GetUniqueId(&u);
    if (r != ncclSuccess) return fail(nullptr, PP_EDEVICE, "pp_comm_id: NCCL: %s", N.GetErrorString(r));
    static_assert(sizeof(ncclUniqueId) == PP_COMM_ID_BYTES, "NCCL unique id size");
    memcpy(id, &u, sizeof u);
    ok(nullptr);
    return PP_OK;
}

extern "C" int32_t pp_comm_init(pp_handle *h, const void *id, int32_t nranks, int32_t rank) {
    const char *who = "pp_comm_init";
    if (!h) return fail(nullptr, PP_EINVAL, "%s: null handle", who);
    if (nranks < 1 || rank < 0 || rank >= nranks || (nranks > 1 && !id))
        return fail(h, PP_EINVAL, "%s: rank %d of %d", who, rank, nranks);
    CK(h, cudaSetDevice(h->device), who);
    CK(h, stream_wait(h, h->factor_stream), who);
    CK(h, stream_wait(h, h->stream), who);
    if (h->comm) {
        nccl_api().CommDestroy(static_cast<ncclComm_t>(h->comm));
        h->comm = nullptr;
    }
    h->comm_failed = false;
    h->nranks = 1;
    h->rank = 0;
    h->hp.exchange = nullptr;
    h->hp.exchange_ctx = nullptr;
    h->ws_esize = 0;  // the bottom work list changes: prepared again before the next factorization
    if (nranks > 1) {
        const NcclApi &N = nccl_api();
        if (!N.ok) return fail(h, PP_EUNSUPPORTED, "%s: %s", who, N.why.c_str());
        ncclUniqueId u;
        memcpy(&u, id, sizeof u);
        ncclComm_t comm = nullptr;
        const ncclResult_t r = N.CommInitRank(&comm, nranks, u, rank);
        if (r != ncclSuccess) return fail(h, PP_EDEVICE, "%s: NCCL: %s", who, N.GetErrorString(r));
        h->comm = comm;
        h->nranks = nranks;
        h->rank = rank;
        h->hp.exchange = exchange_parts;
        h->hp.exchange_ctx = h;
        h->comm_wait_s = h->wait_ns ? std::max(1.0, 30e-9 * (double)h->wait_ns) : 60.0;
    }
    ok(h);
    return PP_OK;
}

// ---------------------------------------------------------------- amalgamation

// Chains of top fronts merged into one front (a relaxed supernode partition of the same elimination order):
// front c joins its parent f = c + 1 when c is f's last child (so the chain's residual vertices are
// contiguous), both fronts are too large for the bottom kernels (nn + na > 64), the merged residual stays
// within `nmax` vertices, and the zero padding the merge adds to the chain's columns, width x (na(f) -
// |sep(c) & sep(f)|), stays within max(8, alpha x width x na(c)).  This is the join rule of the reference's
// GPU amalgamation (ext/PATHPACKCUDAExt/chordal/amalgamate.jl:48-121), restricted to the top of the tree.
// The merged front has the union of the residuals and the last member's separator; by the clique-tree
// property every separator vertex of a member is in the merged residual or in that separator, so the
// member's blocks are sub-blocks of the merged ones and the rest is the semiring's zero, which the (x)
// absorbs: the partial LU of the merged front performs the members' operations on the same operands (plus
// products with zero), and the factor entries are the members' (up to the order in which equal values meet
// in (+), which can decide the sign of a zero).  Returns whether any front joined.
static bool merge_chains(const pp_handle::Structure &o, int nmax, double alpha, pp_handle::Structure &m,
                         std::vector<int> &group, UCost &uc) {
    const int64_t n = o.n, nf = o.nf;
    if (nf < 2) return false;
    std::vector<int> idx(n), pnt(nf, -1);
    for (int64_t f = 0; f < nf; f++)
        for (int64_t v = o.R[f]; v < o.R[f + 1]; v++) idx[v] = (int)f;
    auto nn = [&](int64_t f) { return o.R[f + 1] - o.R[f]; };
    auto na = [&](int64_t f) { return o.Sp[f + 1] - o.Sp[f]; };
    for (int64_t f = 0; f < nf; f++)
        if (na(f) > 0) pnt[f] = idx[o.St[o.Sp[f]]];
    std::vector<int64_t> width(nf);
    std::vector<char> joins(nf, 0);
    for (int64_t f = 0; f < nf; f++) width[f] = nn(f);
    bool any = false;
    for (int64_t f = 1; f < nf; f++) {
        const int64_t c = f - 1;
        if (pnt[c] != f || nn(c) + na(c) <= 64 || nn(f) + na(f) <= 64) continue;
        const int64_t w = width[c] + nn(f);
        if (w > nmax) continue;
        int64_t common = 0;  // |sep(c) & sep(f)|, both sorted
        for (int64_t a = o.Sp[c], b = o.Sp[f]; a < o.Sp[c + 1] && b < o.Sp[f + 1];) {
            const int64_t x = o.St[a], y = o.St[b];
            common += x == y;
            a += x <= y;
            b += y <= x;
        }
        const double zeros = (double)width[c] * (double)(na(f) - common);
        if (zeros > std::max(8.0, alpha * (double)width[c] * (double)std::max<int64_t>(na(c), 1))) continue;
        joins[c] = 1;
        width[f] = w;
        any = true;
    }
    if (!any) return false;
    group.assign(nf, 0);
    m.n = n;
    m.nB = o.nB;
    m.R.clear();
    m.Sp.assign(1, 0);
    m.St.clear();
    int ng = 0;
    for (int64_t f = 0, h0 = 0; f < nf; f++) {
        group[f] = ng;
        if (joins[f]) continue;
        m.R.push_back(o.R[h0]);
        m.St.insert(m.St.end(), o.St.begin() + o.Sp[f], o.St.begin() + o.Sp[f + 1]);
        m.Sp.push_back((int64_t)m.St.size());
        ng++;
        h0 = f + 1;
    }
    m.R.push_back(n);
    m.nf = ng;
    m.Bp = o.Bp;
    m.Fp.assign(o.nB + 1, ng);
    for (int64_t c = 0; c < o.nB; c++) m.Fp[c] = o.Fp[c] < nf ? group[o.Fp[c]] : ng;
    m.Np = o.Np;
    m.Nt = o.Nt;
    m.perm = o.perm;
    auto S2 = [](double x) { return (x - 1) * x * (2 * x - 1) / 6; };
    uc.fpairs.assign(ng, 0.0);
    uc.felems.assign(ng, 0.0);
    uc.spairs.assign(ng, 0.0);
    for (int64_t f = 0; f < nf; f++) {
        const double a = (double)nn(f), b = (double)na(f);
        const int q = group[f];
        uc.fpairs[q] += S2(a + b) - S2(b);
        uc.felems[q] += 4.0 * (a * a + a * b) + b * b;
        uc.spairs[q] += a * (a - 1) / 2 + a * b;
        if (pnt[f] >= 0) uc.felems[group[pnt[f]]] += b * b;  // the parent reads this update matrix
    }
    return true;
}

// Build the device plan from the caller's structure (merged = false) or from its merged one; the counters
// describe the caller's structure either way.
static int32_t use_plan(pp_handle *h, bool merged) {
    const pp_handle::Structure &s = merged ? h->mrg : h->orig;
    UCost uc;
    if (merged) {
        uc.fpairs = h->ufac_pairs;
        uc.felems = h->ufac_elems;
        uc.spairs = h->usolve_pairs;
    }
    const int32_t r = build_structure(h, s.n, s.nf, s.nB, s.R.data(), s.Sp.data(), s.St.data(), s.Bp.data(),
                                      s.Fp.data(), s.Np.data(), s.Nt.data(), s.perm.data(), 0, merged ? &uc : nullptr);
    if (r != PP_OK) return r;
    h->merged = merged;
    h->st.plan_fronts = h->hp.nf;
    h->st.nf = h->orig.nf;
    h->st.nD = h->st.nL = 0;
    for (int64_t f = 0; f < h->orig.nf; f++) {
        const int64_t a = h->orig.R[f + 1] - h->orig.R[f], b = h->orig.Sp[f + 1] - h->orig.Sp[f];
        h->st.nD += a * a;
        h->st.nL += a * b;
    }
    return PP_OK;
}

extern "C" int32_t pp_set_structure(pp_handle *h, int64_t n, int64_t nf, int64_t nB, const int64_t *Rptr,
                                    const int64_t *Sptr, const int64_t *Stgt, const int64_t *Bptr, const int64_t *Fptr,
                                    const int64_t *Nptr, const int64_t *Ntgt, const int64_t *perm, int32_t base) {
    AllocScope alloc_scope(h);
    int32_t r = build_structure(h, n, nf, nB, Rptr, Sptr, Stgt, Bptr, Fptr, Nptr, Ntgt, perm, base, nullptr);
    if (r != PP_OK) return r;
    try {
        // checked by build_structure: keep a 0-based copy
        pp_handle::Structure &o = h->orig;
        const int64_t b = base;
        auto copy = [&](std::vector<int64_t> &dst, const int64_t *src, int64_t len) {
            dst.resize(len);
            for (int64_t i = 0; i < len; i++) dst[i] = src[i] - b;
        };
        o.n = n;
        o.nf = nf;
        o.nB = nB;
        copy(o.R, Rptr, nf + 1);
        copy(o.Sp, Sptr, nf + 1);
        copy(o.St, Stgt, o.Sp[nf]);
        copy(o.Bp, Bptr, nB + 1);
        copy(o.Fp, Fptr, nB + 1);
        copy(o.Np, Nptr, n + 1);
        copy(o.Nt, Ntgt, o.Np[n]);
        copy(o.perm, perm, n);
        h->merged = false;
        UCost uc;
        h->mergeable = h->merge_width > 1 && merge_chains(o, h->merge_width, 0.5, h->mrg, h->group, uc);
        if (h->mergeable) {
            h->ufac_pairs = std::move(uc.fpairs);
            h->ufac_elems = std::move(uc.felems);
            h->usolve_pairs = std::move(uc.spairs);
            r = use_plan(h, true);
            if (r == PP_OK) CK(h, upload_merge_map(h, h->stream), "pp_set_structure");
        } else {
            h->group.clear();
            h->mrg = pp_handle::Structure();
        }
    } catch (const std::bad_alloc &) {
        h->have_structure = false;
        return fail(h, PP_ENOMEM, "pp_set_structure: out of host memory");
    }
    if (r == PP_OK) ok(h);
    return r;
}


// The amalgamation map, evaluated per entry on the device: each entry of the caller's factor arrays (LD, UD,
// LL, UL of the caller's structure) has one place in the blocks of its front's merged front; the other entries of
// the merged blocks are the semiring's zero.  A CTA per caller front f moves each of its entries between the
// caller's layout (c*) and the merged blocks (m*): TO_CALLER gathers
// (pp_get_factor), otherwise it scatters (pp_set_values; the merged arrays were filled with the semiring's
// zero first).  The row of a separator vertex in the merged front is its residual offset, or its place in
// the merged separator (binary search: separators are sorted).  U is an unsigned type of the element size.
template <typename U, bool TO_CALLER>
__global__ void merged_layout_kernel(const int64_t *__restrict__ oR, const int64_t *__restrict__ oSp,
                                     const int64_t *__restrict__ oSt, const int *__restrict__ group,
                                     const int64_t *__restrict__ oDf, const int64_t *__restrict__ oLf, DevPlan P,
                                     U *cLD, U *cUD, U *cLL, U *cUL, U *mLD, U *mUD, U *mLL, U *mUL) {
    const int64_t f = blockIdx.x;
    const int q = group[f];
    const int64_t nn = oR[f + 1] - oR[f], na = oSp[f + 1] - oSp[f];
    const int64_t rq = P.rlo[q], nnq = P.nn[q], naq = P.na[q], off = oR[f] - rq, Dq = P.dptr[q], Lq = P.lptr[q];
    const int64_t Df = oDf[f], Lf = oLf[f];
    const int *sq = P.stgt + P.sptr[q];
    auto move = [&](U *c, int64_t a, U *m, int64_t b) {
        if (TO_CALLER)
            c[a] = m[b];
        else
            m[b] = c[a];
    };
    for (int64_t e = threadIdx.x; e < nn * nn; e += blockDim.x) {
        const int64_t i = e % nn, j = e / nn, b = Dq + (off + i) + (off + j) * nnq;
        move(cLD, Df + e, mLD, b);
        move(cUD, Df + e, mUD, b);
    }
    // the merged row of the caller's separator vertex r
    auto mrow = [&](int64_t r, bool &inres) -> int64_t {
        const int64_t v = oSt[oSp[f] + r];
        inres = v < rq + nnq;
        if (inres) return v - rq;
        int64_t lo = 0, hi = naq;  // first separator entry >= v
        while (lo < hi) {
            const int64_t mid = (lo + hi) >> 1;
            if (sq[mid] < v)
                lo = mid + 1;
            else
                hi = mid;
        }
        return lo;
    };
    for (int64_t e = threadIdx.x; e < na * nn; e += blockDim.x) {
        const int64_t r = e % na, j = e / na;  // LL: na x nn
        bool inres;
        const int64_t row = mrow(r, inres);
        if (inres)
            move(cLL, Lf + e, mLD, Dq + row + (off + j) * nnq);
        else
            move(cLL, Lf + e, mLL, Lq + row + (off + j) * naq);
    }
    for (int64_t e = threadIdx.x; e < nn * na; e += blockDim.x) {
        const int64_t i = e % nn, r = e / nn;  // UL: nn x na
        bool inres;
        const int64_t row = mrow(r, inres);
        if (inres)
            move(cUL, Lf + e, mUD, Dq + (off + i) + row * nnq);
        else
            move(cUL, Lf + e, mUL, Lq + (off + i) + row * nnq);
    }
}

// the device copy of the amalgamation map's inputs (the caller's structure, groups, block offsets)
static cudaError_t upload_merge_map(pp_handle *h, cudaStream_t st) {
    const pp_handle::Structure &o = h->orig;
    std::vector<int64_t> Df(o.nf), Lf(o.nf);
    int64_t d = 0, l = 0;
    for (int64_t f = 0; f < o.nf; f++) {
        const int64_t nn = o.R[f + 1] - o.R[f], na = o.Sp[f + 1] - o.Sp[f];
        Df[f] = d;
        Lf[f] = l;
        d += nn * nn;
        l += nn * na;
    }
    cudaError_t e = upload(h->d_oR, o.R, st);
    if (e == cudaSuccess) e = upload(h->d_oSp, o.Sp, st);
    if (e == cudaSuccess) e = upload(h->d_oSt, o.St, st);
    if (e == cudaSuccess) e = upload(h->d_ogroup, h->group, st);
    if (e == cudaSuccess) e = upload(h->d_oDf, Df, st);
    if (e == cudaSuccess) e = upload(h->d_oLf, Lf, st);
    if (e == cudaSuccess) e = stream_wait(h, st);  // the host vectors are freed on return
    return e;
}

// caller layout <-> merged blocks on the device; c[4] = caller LD, UD, LL, UL in device memory
static cudaError_t merged_layout(pp_handle *h, void *const c[4], bool to_caller, cudaStream_t st) {
    const int64_t nf = h->orig.nf;
    if (nf == 0) return cudaSuccess;
    const int64_t *oR = h->d_oR.as<int64_t>(), *oSp = h->d_oSp.as<int64_t>(), *oSt = h->d_oSt.as<int64_t>();
    const int *grp = h->d_ogroup.as<int>();
    const int64_t *oDf = h->d_oDf.as<int64_t>(), *oLf = h->d_oLf.as<int64_t>();
    void *m[4] = {h->LD.p, h->UD.p, h->LL.p, h->UL.p};
    auto go = [&](auto tag) {
        using U = decltype(tag);
        U *cc[4], *mm[4];
        for (int a = 0; a < 4; a++) {
            cc[a] = static_cast<U *>(c[a]);
            mm[a] = static_cast<U *>(m[a]);
        }
        if (to_caller)
            merged_layout_kernel<U, true><<<(unsigned)nf, 128, 0, st>>>(oR, oSp, oSt, grp, oDf, oLf, h->hp.dev, cc[0],
                                                                         cc[1], cc[2], cc[3], mm[0], mm[1], mm[2],
                                                                         mm[3]);
        else
            merged_layout_kernel<U, false><<<(unsigned)nf, 128, 0, st>>>(oR, oSp, oSt, grp, oDf, oLf, h->hp.dev, cc[0],
                                                                          cc[1], cc[2], cc[3], mm[0], mm[1], mm[2],
                                                                          mm[3]);
    };
    if (h->ops->esize == 8)
        go((unsigned long long)0);
    else
        go((unsigned)0);
    return cudaGetLastError();
}

// Algorithmic traffic (elements) and (x)(+) pairs of one front's factorization: read the assembled blocks
// and the children's update matrices, write the factor blocks and the update matrix; the partial LU's pairs.
static void front_cost(const HostPlan &hp, int f, Cost &g) {
    if (!hp.ufac_pairs.empty()) {
        g.bytes += hp.ufac_elems[f];
        g.pairs += hp.ufac_pairs[f];
        return;
    }
    const double nn = hp.nn[f], na = hp.na[f], nj = nn + na;
    double e = 4.0 * (nn * nn + nn * na) + na * na;
    for (int c = hp.chdptr[f]; c < hp.chdptr[f + 1]; c++) {
        const double nac = hp.na[hp.chdtgt[c]];
        e += nac * nac;
    }
    auto S2 = [](double m) { return (m - 1) * m * (2 * m - 1) / 6; };
    g.bytes += e;
    g.pairs += S2(nj) - S2(na);
}

// Workspace layout and the factorization schedule.  The bottom of the tree (fronts with nn + na within 32 KB
// of shared memory whose whole subtree is such) is one persistent launch, front by front; each bottom front
// keeps a compact na x na update matrix.  Every other front keeps its whole nj x nj frontal matrix (its update
// matrix is the trailing block, read in place by the parent) and is factored by the tile tasks of top.cuh:
// per front, by height, its tiles in (min(I, J), max(I, J)) order.
static int32_t prepare_workspace(pp_handle *h) {
    HostPlan &hp = h->hp;
    if (h->ws_esize == h->ops->esize && !hp.mld.empty()) return PP_OK;
    const int nf = hp.nf;
    int fb_limit = 1;
    while ((size_t)(fb_limit + 1) * (fb_limit + 1) * h->ops->esize <= 32 * 1024) fb_limit++;
    std::vector<char> fbot(nf, 0), allbot(nf, 1);
    for (int f = 0; f < nf; f++) {
        fbot[f] = (hp.nn[f] + hp.na[f] <= fb_limit) && allbot[f];
        if (!fbot[f] && h->pnt[f] >= 0) allbot[h->pnt[f]] = 0;
    }
    hp.mptr.assign(nf, 0);
    hp.fws.assign(nf, -1);
    hp.mld.assign(nf, 1);
    // the bottom fronts' update matrices first, in front order (so that the fronts of a range of the tree have
    // one contiguous range of the workspace: a rank's part of the bottom, several GPUs), then the top fronts'
    // frontal matrices
    std::vector<int64_t> wend(nf, 0);
    int64_t off = 0;
    for (int pass = 0; pass < 2; pass++)
        for (int f = 0; f < nf; f++) {
            if ((fbot[f] != 0) != (pass == 0)) continue;
            const int nn = hp.nn[f], na = hp.na[f], nj = nn + na;
            if (fbot[f]) {
                hp.mptr[f] = off;
                hp.mld[f] = std::max(na, 1);
                off += (int64_t)na * na;
            } else {
                hp.fws[f] = off;
                hp.mptr[f] = off + nn + (int64_t)nn * nj;
                hp.mld[f] = nj;
                off += (int64_t)nj * nj;
            }
            off = (off + 3) & ~(int64_t)3;  // 16-byte alignment of every block
            wend[f] = off;
        }
    hp.ws_elems = off;
    // several GPUs: the maximal bottom subtrees (contiguous ranges of fronts in postorder) dealt to the ranks in
    // front order, each rank a contiguous run of about equal estimated time; a rank's part is then one range of
    // each factor array and of the workspace
    h->parts.clear();
    if (h->nranks > 1) {
        std::vector<int> fdsc(nf);
        for (int f = 0; f < nf; f++) fdsc[f] = f;
        for (int f = 0; f < nf; f++)
            if (h->pnt[f] >= 0) fdsc[h->pnt[f]] = std::min(fdsc[h->pnt[f]], fdsc[f]);
        std::vector<double> est(nf + 1, 0.0);  // prefix sums of the bottom fronts' estimated times
        for (int f = 0; f < nf; f++) {
            const double nj = hp.nn[f] + hp.na[f];
            est[f + 1] = est[f] + (fbot[f] ? 6.0 + nj * nj / 64.0 + hp.nn[f] * nj * nj / 512.0 : 0.0);
        }
        std::vector<std::pair<int, int>> roots;  // (first front, root) of each maximal bottom subtree
        for (int f = 0; f < nf; f++)
            if (fbot[f] && (h->pnt[f] < 0 || !fbot[h->pnt[f]])) roots.push_back({fdsc[f], f});
        // subtree q goes to the rank whose share of the total holds the middle of its estimated time: the ranks
        // of consecutive subtrees never decrease, so every part is one run
        h->parts.assign(h->nranks, Part{});
        std::vector<char> used(h->nranks, 0);
        for (const auto &rt : roots) {
            const double mid = 0.5 * (est[rt.first] + est[rt.second + 1]);
            const int r = est[nf] > 0 ? std::min(h->nranks - 1, (int)(mid * h->nranks / est[nf])) : 0;
            Part &pt = h->parts[r];
            if (!used[r]) {
                pt.f0 = rt.first;
                pt.w0 = hp.mptr[rt.first];
                used[r] = 1;
            }
            pt.f1 = rt.second + 1;
            pt.w1 = wend[rt.second];
        }
        for (int r = 0; r < h->nranks; r++) {
            Part &pt = h->parts[r];
            if (!used[r]) continue;  // an empty part: f0 = f1 = 0
            pt.d0 = hp.dptr[pt.f0];
            pt.d1 = hp.dptr[pt.f1];
            pt.l0 = hp.lptr[pt.f0];
            pt.l1 = hp.lptr[pt.f1];
        }
    }
    const int maxh = h->maxh;
    cudaStream_t st = h->stream;
    CK(h, stream_wait(h, h->factor_stream), "prepare_workspace");
    CK(h, stream_wait(h, st), "prepare_workspace");
    // stage 0 of each solve direction lists the subtrees and forward bottom fronts that the bottom kernel
    // factors first: a solve sweeps them while the top of the tree is factored.  fbot holds every child of a
    // front it holds, so the stable partition keeps each child before its parent.
    for (int d = 0; d < 2; d++) {
        const std::vector<SubtreeList> &subs = d ? hp.sub_r : hp.sub_l;
        const std::vector<std::pair<int64_t, int>> &fw = d ? hp.sb_fwd_r : hp.sb_fwd;
        hp.early_sub[d] = hp.early_bot[d] = 0;
        auto in_bottom = [&](int f) { return fbot[f] != 0; };
        if (!subs.empty() && subs[0].count > 0) {
            int *r = h->sroots.data() + subs[0].off;
            hp.early_sub[d] = (int)(std::stable_partition(r, r + subs[0].count, in_bottom) - r);
        }
        if (!fw.empty() && fw[0].second > 0) {
            int *b = h->sfronts.data() + fw[0].first;
            hp.early_bot[d] = (int)(std::stable_partition(b, b + fw[0].second, in_bottom) - b);
        }
    }
    // continuation of the bottom sweeps (sweep_bottom_kernel): per direction the segment of each bottom front
    // (2 * stage + part, part 0 for stage 0's early fronts) and which parts its bottom children lie in; the
    // heavy child of each bottom front, the one with the costliest chain of bottom fronts below it
    {
        std::vector<int> heavy(nf, -1), seg(nf, -1);
        std::vector<double> chain(nf, 0.0);
        for (int d = 0; d < 2; d++) {
            const std::vector<std::pair<int64_t, int>> &fw = d ? hp.sb_fwd_r : hp.sb_fwd;
            std::fill(seg.begin(), seg.end(), -1);
            for (size_t sidx = 0; sidx < fw.size(); sidx++)
                for (int i = 0; i < fw[sidx].second; i++) {
                    const int f = h->sfronts[fw[sidx].first + i];
                    seg[f] = 2 * (int)sidx + ((sidx == 0 && i < hp.early_bot[d]) ? 0 : 1);
                }
            std::vector<int> &info = d ? h->sinfo_r : h->sinfo_l;
            info.assign(nf, -1);
            for (int f = 0; f < nf; f++)
                if (seg[f] >= 0) info[f] = seg[f] << 3;
            if (d == 0) {
                for (int f = 0; f < nf; f++) {  // children before parents
                    if (seg[f] < 0) continue;
                    chain[f] += 4.0 + hp.nn[f] * (double)hp.na[f] / 36.0;
                    const int p = h->pnt[f];
                    if (p >= 0 && seg[p] >= 0 && (heavy[p] < 0 || chain[f] > chain[heavy[p]])) heavy[p] = f;
                    if (p >= 0 && seg[p] >= 0) chain[p] = std::max(chain[p], chain[f]);
                }
            }
            for (int f = 0; f < nf; f++) {
                const int p = h->pnt[f];
                if (seg[f] < 0 || p < 0 || seg[p] < 0) continue;
                info[p] |= (seg[f] & 1) ? 2 : 1;
                if (heavy[p] == f) info[f] |= 4;
            }
        }
        h->sheavy = heavy;
    }
    CK(h, upload(h->d_sinfo_l, h->sinfo_l, st), "upload");
    CK(h, upload(h->d_sinfo_r, h->sinfo_r, st), "upload");
    CK(h, upload(h->d_sheavy, h->sheavy, st), "upload");
    hp.d_sinfo[0] = h->d_sinfo_l.as<int>();
    hp.d_sinfo[1] = h->d_sinfo_r.as<int>();
    hp.d_sheavy = h->d_sheavy.as<int>();
    hp.sroot_pairs.resize(h->sroots.size());
    hp.sroot_res.resize(h->sroots.size());
    hp.sroot_sep.resize(h->sroots.size());
    hp.sroot_fac.resize(h->sroots.size());
    for (size_t i = 0; i < h->sroots.size(); i++) {
        const int r = h->sroots[i];
        hp.sroot_pairs[i] = hp.stree_pairs[r];
        hp.sroot_res[i] = hp.stree_res[r];
        hp.sroot_sep[i] = hp.stree_sep[r];
        hp.sroot_fac[i] = hp.stree_fac[r];
    }
    CK(h, upload(h->d_sroots, h->sroots, st), "upload");
    CK(h, upload(h->d_sfronts, h->sfronts, st), "upload");
    hp.d_sroots = h->d_sroots.as<int>();
    hp.d_sfronts = h->d_sfronts.as<int>();
    {
        std::vector<std::vector<int>> byh(maxh + 1);
        std::vector<int> pending0(nf, 0);
        Cost acc;
        hp.fb_maxnj = 0;
        for (int f = 0; f < nf; f++)
            if (fbot[f]) {
                byh[h->height[f]].push_back(f);
                if (h->pnt[f] >= 0) pending0[h->pnt[f]]++;
                hp.fb_maxnj = std::max(hp.fb_maxnj, hp.nn[f] + hp.na[f]);
                front_cost(hp, f, acc);
            }
        std::vector<int> hl;
        for (int hh = 0; hh <= maxh; hh++) hl.insert(hl.end(), byh[hh].begin(), byh[hh].end());
        // estimated time of a bottom front (a CTA): a fixed part, the assembly and the partial LU
        std::vector<double> fcost(nf, 0.0);
        for (int f : hl) {
            const double nj = hp.nn[f] + hp.na[f];
            fcost[f] = 6.0 + nj * nj / 64.0 + hp.nn[f] * nj * nj / 512.0;
        }
        std::vector<int> wl = schedule_order(hl, fcost, h->pnt, true, h->sm_count * 6);
        if (h->nranks > 1) {  // this rank's part only (the list order keeps children first)
            const Part &pt = h->parts[h->rank];
            std::vector<int> mine;
            Cost part;
            for (int f : wl)
                if (f >= pt.f0 && f < pt.f1) {
                    mine.push_back(f);
                    front_cost(hp, f, part);
                }
            wl.swap(mine);
            acc = part;
        }
        hp.fb_count = (int)wl.size();
        hp.fb_bytes = acc.bytes;
        hp.fb_pairs = acc.pairs;
        CK(h, upload(h->d_fbottom, wl, st), "upload");
        CK(h, upload(h->d_fpending0, pending0, st), "upload");
        hp.d_fbottom = h->d_fbottom.as<int>();
        hp.d_fpending0 = h->d_fpending0.as<int>();
    }
    {
        std::vector<int> tl;  // the top fronts, children first
        {
            std::vector<std::vector<int>> byh(maxh + 1);
            for (int f = 0; f < nf; f++)
                if (!fbot[f]) byh[h->height[f]].push_back(f);
            for (int hh = 0; hh <= maxh; hh++) tl.insert(tl.end(), byh[hh].begin(), byh[hh].end());
        }
        // schedule order of the fronts (their tile tasks stay together): a front's critical path is about 50 us
        // per 64-column pivot block; some sixteen tile tasks of a front are in flight on two CTAs per SM
        std::vector<double> tcost(nf, 0.0);
        for (int f : tl) tcost[f] = 20.0 + 50.0 * ((hp.nn[f] + TOP_TILE - 1) / TOP_TILE);
        tl = schedule_order(tl, tcost, h->pnt, true, std::max(1, h->sm_count * 2 / 16));
        // the roots of the tree last: the factorization's second launch (every dependency of a root is earlier)
        std::stable_partition(tl.begin(), tl.end(), [&](int f) { return h->pnt[f] >= 0; });
        int ntasks_a = -1;
        std::vector<int> tasks, crng;
        std::vector<int64_t> foff(nf, 0), croff(std::max<size_t>(hp.chdtgt.size(), 1), 0);
        int64_t nflags = 16;
        Cost acc;
        std::vector<std::pair<int, int>> tiles;
        std::vector<int> bounds;
        for (int f : tl) {
            if (ntasks_a < 0 && h->pnt[f] < 0) ntasks_a = (int)(tasks.size() / 4);
            const int nn = hp.nn[f], na = hp.na[f];
            const int kb = (nn + TOP_TILE - 1) / TOP_TILE, nbt = kb + (na + TOP_TILE - 1) / TOP_TILE;
            foff[f] = nflags;
            nflags += (int64_t)nbt * nbt + 1;
            // tile block boundaries of the front, and where each child's separator crosses them
            bounds.clear();
            for (int b = 0; b < kb; b++) bounds.push_back(b * TOP_TILE);
            for (int b = kb; b < nbt; b++) bounds.push_back(nn + (b - kb) * TOP_TILE);
            bounds.push_back(nn + na);
            for (int c = hp.chdptr[f]; c < hp.chdptr[f + 1]; c++) {
                const int ch = hp.chdtgt[c];
                const int *r0 = h->rel.data() + hp.sptr[ch], *r1 = r0 + hp.na[ch];
                croff[c] = (int64_t)crng.size();
                for (int b : bounds) crng.push_back((int)(std::lower_bound(r0, r1, b) - r0));
            }
            tiles.clear();
            for (int I = 0; I < nbt; I++)
                for (int J = 0; J < nbt; J++) tiles.push_back({I, J});
            std::stable_sort(tiles.begin(), tiles.end(), [](const std::pair<int, int> &a,
                                                             const std::pair<int, int> &b) {
                const int a0 = std::min(a.first, a.second), b0 = std::min(b.first, b.second);
                if (a0 != b0) return a0 < b0;
                return std::max(a.first, a.second) < std::max(b.first, b.second);
            });
            for (const auto &t : tiles) tasks.insert(tasks.end(), {f, t.first, t.second, 0});
            front_cost(hp, f, acc);
        }
        hp.top_ntasks = (int)(tasks.size() / 4);
        hp.top_ntasks_a = ntasks_a < 0 ? hp.top_ntasks : ntasks_a;
        hp.top_cost = acc;
        hp.tflags_n = nflags;
        if (tasks.empty()) tasks.assign(4, 0);
        CK(h, upload(h->d_ttasks, tasks, st), "upload");
        CK(h, upload(h->d_tfoff, foff, st), "upload");
        CK(h, upload(h->d_croff, croff, st), "upload");
        CK(h, upload(h->d_crng, crng, st), "upload");
        CK(h, h->d_tflags.ensure(sizeof(int) * (size_t)nflags), "upload");
        hp.d_ttasks = reinterpret_cast<const int4 *>(h->d_ttasks.p);
        hp.d_tfoff = h->d_tfoff.as<int64_t>();
        hp.d_croff = h->d_croff.as<int64_t>();
        hp.d_crng = h->d_crng.as<int>();
        hp.d_tflags = h->d_tflags.as<int>();
    }
    CK(h, upload(h->d_mptr, hp.mptr, st), "upload");
    CK(h, upload(h->d_mld, hp.mld, st), "upload");
    CK(h, upload(h->d_fws, hp.fws, st), "upload");
    CK(h, stream_wait(h, st), "upload");
    hp.dev.mptr = h->d_mptr.as<int64_t>();
    hp.dev.mld = h->d_mld.as<int>();
    hp.dev.fws = h->d_fws.as<int64_t>();
    h->ws_esize = h->ops->esize;
    return PP_OK;
}

static int32_t need_memory(pp_handle *h, size_t bytes, const char *what) {
    if (bytes == 0) return PP_OK;  // nothing to allocate: no driver query on the solve path
    size_t fr = 0, tot = 0;
    if (cudaMemGetInfo(&fr, &tot) == cudaSuccess && bytes > fr)
        return fail(h, PP_ENOMEM, "%s: needs %.3f GB of device memory, %.3f GB free", what, bytes / 1e9, fr / 1e9);
    return PP_OK;
}

static int32_t ensure_sync(pp_handle *h, int64_t k);

static int32_t set_semiring(pp_handle *h, int32_t sr, int32_t dt, const char *who) {
    // the values are being replaced: until this call and its caller succeed there are none to factor or solve
    // with (a failed allocation below may have released buffers the device plan points into)
    h->have_values = h->factored = false;
    h->nnz_assembled = -1;  // pp_update_values needs the pattern of a completed pp_assemble
    const Ops *o = get_ops(sr, dt);
    if (!o) return fail(h, PP_EUNSUPPORTED, "%s: semiring %d with element type %d is not supported", who, sr, dt);
    // merged fronts for every semiring whose zero absorbs in (x): not PlusProd, where 0 * Inf is NaN and a
    // padded zero times a divergent star would reach entries of the caller's structure
    const bool want_merged = h->mergeable && sr != PP_PLUSPROD;
    if (want_merged != h->merged) {
        h->ops = nullptr;
        const int32_t r = use_plan(h, want_merged);
        if (r != PP_OK) return r;
    }
    if (h->ops != o) {
        h->ops = o;
        h->ws_esize = 0;
    }
    h->sr = sr;
    h->dt = dt;
    h->prof.esize = o->esize;
    h->hp.prof = &h->prof;
    int32_t r = prepare_workspace(h);
    if (r != PP_OK) return r;
    const size_t es = o->esize;
    const size_t need = es * (2 * (size_t)h->nD + 2 * (size_t)h->nL + (size_t)h->hp.nN);
    if (need_memory(h, need, who) != PP_OK) return PP_ENOMEM;
    CK(h, h->LD.ensure(es * std::max<int64_t>(h->nD, 1)), who);
    CK(h, h->UD.ensure(es * std::max<int64_t>(h->nD, 1)), who);
    CK(h, h->LL.ensure(es * std::max<int64_t>(h->nL, 1)), who);
    CK(h, h->UL.ensure(es * std::max<int64_t>(h->nL, 1)), who);
    CK(h, h->Nval.ensure(es * std::max<int64_t>(h->hp.nN, 1)), who);
    return PP_OK;
}

static Values values_of(pp_handle *h) {
    Values v;
    v.LD = h->LD.p;
    v.LL = h->LL.p;
    v.UD = h->UD.p;
    v.UL = h->UL.p;
    v.Nval = h->Nval.p;
    v.W = h->W.p;
    return v;
}

// The handle's stream waits for the top of the last factorization (a no-op if there was none): every call that
// writes the factor's values or workspace orders itself after it this way.
static cudaError_t after_factor(pp_handle *h) {
    return h->capturing ? cudaSuccess : cudaStreamWaitEvent(h->stream, h->ev_factored, 0);
}

// timing events of the last factorization / solve (not while a plan is captured)
static cudaError_t record_timing(pp_handle *h, cudaEvent_t ev, cudaStream_t st) {
    return h->capturing ? cudaSuccess : cudaEventRecord(ev, st);
}

extern "C" int32_t pp_assemble(pp_handle *h, int32_t semiring, int32_t dtype, const int64_t *colptr,
                               const int64_t *rowval, const void *nzval, int32_t base) {
    AllocScope alloc_scope(h);
    if (!h) return fail(nullptr, PP_EINVAL, "pp_assemble: null handle");
    if (!h->have_structure) return fail(h, PP_ESTATE, "pp_assemble: no structure (call pp_set_structure first)");
    if (base != 0 && base != 1) return fail(h, PP_EINVAL, "pp_assemble: base must be 0 or 1");
    CK(h, cudaSetDevice(h->device), "pp_assemble");
    CK(h, stream_wait(h, h->factor_stream), "pp_assemble");  // buffers may be reallocated below
    int32_t r = set_semiring(h, semiring, dtype, "pp_assemble");
    if (r != PP_OK) return r;
    const int n = h->hp.n;
    if (n > 0 && (!colptr || (colptr[n] - base > 0 && (!rowval || !nzval))))
        return fail(h, PP_EINVAL, "pp_assemble: null array");
    std::vector<int> cp(n + 1), rv;
    try {
        for (int j = 0; j <= n; j++) {
            const int64_t v = colptr[j] - base;
            if (v < 0 || (j > 0 && v < cp[j - 1]) || v >= INT32_MAX) return fail(h, PP_EINVAL, "pp_assemble: colptr");
            cp[j] = (int)v;
        }
        if (cp[0] != 0) return fail(h, PP_EINVAL, "pp_assemble: colptr must start at the base");
        rv.resize(std::max(cp[n], 1));
        for (int p = 0; p < cp[n]; p++) {
            const int64_t v = rowval[p] - base;
            if (v < 0 || v >= n) return fail(h, PP_EINVAL, "pp_assemble: row index out of range");
            rv[p] = (int)v;
        }
        // no duplicate entries within a column (sparse() combines them before copyto!)
        std::vector<int> mark(n, -1);
        for (int j = 0; j < n; j++)
            for (int p = cp[j]; p < cp[j + 1]; p++) {
                if (mark[rv[p]] == j) return fail(h, PP_EINVAL, "pp_assemble: duplicate entry in column %d", j);
                mark[rv[p]] = j;
            }
        if (semiring == PP_MINPLUS && dtype == PP_I32) {
            const int32_t *a = static_cast<const int32_t *>(nzval);
            for (int p = 0; p < cp[n]; p++)
                if (a[p] < 0) return fail(h, PP_EUNSUPPORTED, "pp_assemble: Int32 MinPlus takes weights in [0, INT32_MAX]");
        }
    } catch (const std::bad_alloc &) {
        return fail(h, PP_ENOMEM, "pp_assemble: out of host memory");
    }
    cudaStream_t st = h->stream;
    const size_t es = h->ops->esize;
    CK(h, upload(h->csc_ptr, cp, st), "pp_assemble");
    CK(h, upload(h->csc_row, rv, st), "pp_assemble");
    CK(h, h->csc_val.ensure(es * std::max(cp[n], 1)), "pp_assemble");
    if (cp[n] > 0) CK(h, cudaMemcpyAsync(h->csc_val.p, nzval, es * cp[n], cudaMemcpyHostToDevice, st), "pp_assemble");
    int pi = h->prof.begin(K_ASSEMBLE, st);
    CK(h, h->ops->assemble(h->hp, h->csc_ptr.as<int>(), h->csc_row.as<int>(), h->csc_val.p, values_of(h), st),
       "pp_assemble");
    h->prof.end(pi, st, 2.0 * (h->nD + h->nL) + h->hp.nN + (double)cp[n] * (1.0 + 8.0 / es), 0);
    CK(h, stream_wait(h, st), "pp_assemble");
    h->prof.collect();
    h->nnz_assembled = cp[n];
    h->have_values = true;
    h->factored = false;
    ok(h);
    return PP_OK;
}

extern "C" int32_t pp_update_values(pp_handle *h, const void *nzval, int32_t where) {
    AllocScope alloc_scope(h);
    if (!h) return fail(nullptr, PP_EINVAL, "pp_update_values: null handle");
    if (!h->have_structure || h->nnz_assembled < 0)
        return fail(h, PP_ESTATE, "pp_update_values: no pattern (call pp_assemble first)");
    if (where != PP_HOST && where != PP_DEVICE) return fail(h, PP_EINVAL, "pp_update_values: where");
    const int64_t nnz = h->nnz_assembled;
    if (nnz > 0 && !nzval) return fail(h, PP_EINVAL, "pp_update_values: null nzval");
    CK(h, cudaSetDevice(h->device), "pp_update_values");
    const size_t es = h->ops->esize;
    if (where == PP_HOST && h->sr == PP_MINPLUS && h->dt == PP_I32) {
        const int32_t *a = static_cast<const int32_t *>(nzval);
        for (int64_t p = 0; p < nnz; p++)
            if (a[p] < 0) return fail(h, PP_EUNSUPPORTED, "pp_update_values: Int32 MinPlus takes weights in [0, INT32_MAX]");
    }
    cudaStream_t st = h->stream;
    CK(h, after_factor(h), "pp_update_values");
    if (nnz > 0)
        CK(h, cudaMemcpyAsync(h->csc_val.p, nzval, es * nnz, where == PP_HOST ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice,
                              st), "pp_update_values");
    int pi = h->prof.begin(K_ASSEMBLE, st);
    CK(h, h->ops->assemble(h->hp, h->csc_ptr.as<int>(), h->csc_row.as<int>(), h->csc_val.p, values_of(h), st),
       "pp_update_values");
    h->prof.end(pi, st, 2.0 * (h->nD + h->nL) + h->hp.nN + (double)nnz * (1.0 + 8.0 / es), 0);
    if (where == PP_HOST) CK(h, stream_wait(h, st), "pp_update_values");  // the caller's array is free
    h->have_values = true;
    h->factored = false;
    ok(h);
    return PP_OK;
}

extern "C" int32_t pp_set_values(pp_handle *h, int32_t semiring, int32_t dtype, const void *LD, const void *LL,
                                 const void *UD, const void *UL, const void *Nval) {
    AllocScope alloc_scope(h);
    if (!h) return fail(nullptr, PP_EINVAL, "pp_set_values: null handle");
    if (!h->have_structure) return fail(h, PP_ESTATE, "pp_set_values: no structure");
    CK(h, cudaSetDevice(h->device), "pp_set_values");
    CK(h, stream_wait(h, h->factor_stream), "pp_set_values");
    int32_t r = set_semiring(h, semiring, dtype, "pp_set_values");
    if (r != PP_OK) return r;
    const size_t es = h->ops->esize;
    cudaStream_t st = h->stream;
    if ((h->st.nD > 0 && (!LD || !UD)) || (h->st.nL > 0 && (!LL || !UL)) || (h->hp.nN > 0 && !Nval))
        return fail(h, PP_EINVAL, "pp_set_values: null array");
    if (h->merged) {
        // the caller's blocks uploaded as they are, then placed into the zero-filled merged blocks on the device
        // (the amalgamation map, merged_layout_kernel)
        const int64_t cD = h->st.nD, cL = h->st.nL;
        const size_t sb = es * (size_t)std::max<int64_t>(2 * cD + 2 * cL, 1);
        if (sb > h->d_ostage.bytes && need_memory(h, sb, "pp_set_values") != PP_OK) return PP_ENOMEM;
        CK(h, h->d_ostage.ensure(sb), "pp_set_values");
        char *stg = static_cast<char *>(h->d_ostage.p);
        void *c[4] = {stg, stg + es * cD, stg + es * 2 * cD, stg + es * (2 * cD + cL)};
        const void *srcs[4] = {LD, UD, LL, UL};
        for (int a = 0; a < 4; a++)
            if (a < 2 ? cD : cL)
                CK(h, cudaMemcpyAsync(c[a], srcs[a], es * (a < 2 ? cD : cL), cudaMemcpyHostToDevice, st), "pp_set_values");
        if (h->nD) CK(h, h->ops->fill_zero(h->LD.p, h->nD, st), "pp_set_values");
        if (h->nD) CK(h, h->ops->fill_zero(h->UD.p, h->nD, st), "pp_set_values");
        if (h->nL) CK(h, h->ops->fill_zero(h->LL.p, h->nL, st), "pp_set_values");
        if (h->nL) CK(h, h->ops->fill_zero(h->UL.p, h->nL, st), "pp_set_values");
        CK(h, merged_layout(h, c, false, st), "pp_set_values");
        if (h->hp.nN) CK(h, cudaMemcpyAsync(h->Nval.p, Nval, es * h->hp.nN, cudaMemcpyHostToDevice, st), "pp_set_values");
        CK(h, stream_wait(h, st), "pp_set_values");
        h->have_values = true;
        h->factored = false;
        ok(h);
        return PP_OK;
    }
    if (h->nD) CK(h, cudaMemcpyAsync(h->LD.p, LD, es * h->nD, cudaMemcpyHostToDevice, st), "pp_set_values");
    if (h->nD) CK(h, cudaMemcpyAsync(h->UD.p, UD, es * h->nD, cudaMemcpyHostToDevice, st), "pp_set_values");
    if (h->nL) CK(h, cudaMemcpyAsync(h->LL.p, LL, es * h->nL, cudaMemcpyHostToDevice, st), "pp_set_values");
    if (h->nL) CK(h, cudaMemcpyAsync(h->UL.p, UL, es * h->nL, cudaMemcpyHostToDevice, st), "pp_set_values");
    if (h->hp.nN) CK(h, cudaMemcpyAsync(h->Nval.p, Nval, es * h->hp.nN, cudaMemcpyHostToDevice, st), "pp_set_values");
    CK(h, stream_wait(h, st), "pp_set_values");
    h->have_values = true;
    h->factored = false;
    ok(h);
    return PP_OK;
}

// Wait for the handle's stream, then take the times of the calls enqueued since the last wait and the error
// word of the persistent kernels (set when a bounded wait expired; cleared once reported).
static int32_t settle(pp_handle *h, const char *who) {
    CK(h, stream_wait(h, h->factor_stream), who);
    CK(h, stream_wait(h, h->stream), who);
    if (h->factor_pending) {
        float ms = 0;
        if (cudaEventElapsedTime(&ms, h->fev0, h->fev1) == cudaSuccess) h->st.ms_factor = ms;
        h->factor_pending = false;
    }
    if (h->solve_pending) {
        float ms = 0;
        if (cudaEventElapsedTime(&ms, h->ev0, h->ev1) == cudaSuccess) h->st.ms_solve = ms;
        h->solve_pending = false;
    }
    h->prof.collect();
    if (h->hp.d_err) {
        int err = 0;
        CK(h, cudaMemcpy(&err, h->hp.d_err, sizeof(int), cudaMemcpyDeviceToHost), who);
        if (err) {
            CK(h, cudaMemset(h->hp.d_err, 0, sizeof(int)), who);
            return fail(h, PP_ETIMEOUT, "%s: a bounded device wait expired (a dependency of the persistent kernels "
                        "never completed)", who);
        }
    }
    return PP_OK;
}

extern "C" int32_t pp_factor(pp_handle *h) {
    AllocScope alloc_scope(h);
    if (!h) return fail(nullptr, PP_EINVAL, "pp_factor: null handle");
    if (!h->have_values) return fail(h, PP_ESTATE, "pp_factor: no values (call pp_assemble or pp_set_values)");
    CK(h, cudaSetDevice(h->device), "pp_factor");
    if (h->ws_esize != h->ops->esize || h->hp.mld.empty()) {  // joined or left a group since the last one
        const int32_t r = prepare_workspace(h);
        if (r != PP_OK) {
            h->factored = false;
            return r;
        }
    }
    const size_t wbytes = h->ops->esize * std::max<int64_t>(h->hp.ws_elems, 1);
    if (wbytes > h->W.bytes) {
        CK(h, stream_wait(h, h->factor_stream), "pp_factor");
        CK(h, stream_wait(h, h->stream), "pp_factor");
        h->W.release();
        h->factored = false;
        if (need_memory(h, wbytes, "pp_factor") != PP_OK) return PP_ENOMEM;
        CK(h, h->W.ensure(wbytes), "pp_factor");
    }
    if (ensure_sync(h, 1) != PP_OK) return PP_ENOMEM;  // the bottom kernel's counters
    h->hp.d_trace = nullptr;
    if (h->trace_on && h->hp.top_ntasks > 0) {
        CK(h, h->d_trace.ensure(sizeof(unsigned long long) * PP_TRACE_WORDS * (size_t)h->hp.top_ntasks), "pp_factor");
        CK(h, cudaMemsetAsync(h->d_trace.p, 0, sizeof(unsigned long long) * PP_TRACE_WORDS * (size_t)h->hp.top_ntasks,
                              h->stream),
           "pp_factor");
        h->hp.d_trace = h->d_trace.as<unsigned long long>();
    }
    if (h->comm_failed) return fail(h, PP_ESTATE, "pp_factor: the handle left its group of GPUs after a failure");
    cudaStream_t st = h->stream;
    int64_t nl = 0;
    CK(h, after_factor(h), "pp_factor");  // the previous top factorization reads the bottom's update matrices
    CK(h, record_timing(h, h->fev0, st), "pp_factor");
    h->comm_msg.clear();
    const cudaError_t fe = h->ops->factor(h->hp, values_of(h), st, &nl);
    if (fe != cudaSuccess && !h->comm_msg.empty()) {
        h->factored = false;
        return fail(h, PP_EDEVICE, "pp_factor: %s", h->comm_msg.c_str());
    }
    CK(h, fe, "pp_factor");
    CK(h, record_timing(h, h->fev1, h->factor_stream), "pp_factor");  // the top of the tree ends there
    h->factor_pending = !h->capturing;
    h->st.kernel_launches = nl;
    h->factored = true;
    ok(h);
    return PP_OK;
}

extern "C" int32_t pp_get_factor(pp_handle *h, void *LD, void *LL, void *UD, void *UL) {
    if (!h) return fail(nullptr, PP_EINVAL, "pp_get_factor: null handle");
    if (!h->have_values) return fail(h, PP_ESTATE, "pp_get_factor: no values");
    CK(h, cudaSetDevice(h->device), "pp_get_factor");
    const size_t es = h->ops->esize;
    cudaStream_t st = h->stream;
    if (h->merged) {
        // the caller's layout gathered from the merged blocks on the device (the amalgamation map,
        // merged_layout_kernel), then downloaded
        const int64_t cD = h->st.nD, cL = h->st.nL;
        const size_t sb = es * (size_t)std::max<int64_t>(2 * cD + 2 * cL, 1);
        if (sb > h->d_ostage.bytes && need_memory(h, sb, "pp_get_factor") != PP_OK) return PP_ENOMEM;
        CK(h, h->d_ostage.ensure(sb), "pp_get_factor");
        char *stg = static_cast<char *>(h->d_ostage.p);
        void *c[4] = {stg, stg + es * cD, stg + es * 2 * cD, stg + es * (2 * cD + cL)};
        void *dst[4] = {LD, UD, LL, UL};
        CK(h, after_factor(h), "pp_get_factor");
        CK(h, merged_layout(h, c, true, st), "pp_get_factor");
        for (int a = 0; a < 4; a++)
            if (dst[a] && (a < 2 ? cD : cL))
                CK(h, cudaMemcpyAsync(dst[a], c[a], es * (a < 2 ? cD : cL), cudaMemcpyDeviceToHost, st), "pp_get_factor");
        const int32_t r = settle(h, "pp_get_factor");
        if (r != PP_OK) return r;
        ok(h);
        return PP_OK;
    }
    CK(h, after_factor(h), "pp_get_factor");  // the top of the tree is factored on its own stream
    if (LD && h->nD) CK(h, cudaMemcpyAsync(LD, h->LD.p, es * h->nD, cudaMemcpyDeviceToHost, st), "pp_get_factor");
    if (UD && h->nD) CK(h, cudaMemcpyAsync(UD, h->UD.p, es * h->nD, cudaMemcpyDeviceToHost, st), "pp_get_factor");
    if (LL && h->nL) CK(h, cudaMemcpyAsync(LL, h->LL.p, es * h->nL, cudaMemcpyDeviceToHost, st), "pp_get_factor");
    if (UL && h->nL) CK(h, cudaMemcpyAsync(UL, h->UL.p, es * h->nL, cudaMemcpyDeviceToHost, st), "pp_get_factor");
    const int32_t r = settle(h, "pp_get_factor");
    if (r != PP_OK) return r;
    ok(h);
    return PP_OK;
}

static double solve_pairs_per_rhs(const HostPlan &hp) {
    double s = 0;
    if (!hp.usolve_pairs.empty()) {
        for (double x : hp.usolve_pairs) s += 2 * x;
        return s + (double)hp.nN;
    }
    for (int f = 0; f < hp.nf; f++) {
        const double nn = hp.nn[f], na = hp.na[f];
        s += nn * (nn - 1) + 2 * nn * na;
    }
    return s + (double)hp.nN;
}

// the per-(tile, front) counters of the persistent sweeps for k right-hand sides
static int32_t ensure_sync(pp_handle *h, int64_t k) {
    const int64_t need = sync_ints(h->hp.nf, k);
    if (need <= h->hp.sync_cap) return PP_OK;
    if (need_memory(h, sizeof(int) * need, "sweep counters") != PP_OK) return PP_ENOMEM;
    h->d_sync.release();
    h->hp.d_sync = nullptr;  // no call may use the released counters
    h->hp.sync_cap = 0;
    cudaError_t e = h->d_sync.ensure(sizeof(int) * need);
    if (e != cudaSuccess) return cuda_fail(h, e, "sweep counters");
    h->hp.d_sync = h->d_sync.as<int>();
    h->hp.sync_cap = need;
    return PP_OK;
}

// The device part of a solve on caller-layout device buffers: Bin permuted into X, the sweeps, X permuted
// out into Bout (Bin == Bout in place; both leading dimension ldb).  X and the counters must be allocated.
static int32_t enqueue_solve(pp_handle *h, const void *Bin, void *Bout, int64_t ldb, int64_t k, int left, int trans,
                             const char *who, bool first = true, bool last = true) {
    const int n = h->hp.n;
    const int64_t ldx = (k + 3) & ~(int64_t)3;
    cudaStream_t st = h->stream;
    int64_t nl = 0;
    if (first) {
        h->st.pairs_solve = 0;
        h->st.kernel_launches = 0;
        CK(h, record_timing(h, h->ev0, st), who);
    }
    int pi = h->prof.begin(K_PERMUTE, st);
    if (left)
        CK(h, h->ops->rows_in(Bin, ldb, h->X.p, ldx, h->hp.dev.invp, n, (int)k, st), who);
    else
        CK(h, h->ops->cols_in(Bin, ldb, h->X.p, ldx, h->hp.dev.invp, n, (int)k, st), who);
    h->prof.end(pi, st, 2.0 * n * k, 0);
    CK(h, h->ops->solve(h->hp, values_of(h), trans ? !left : left, h->X.p, ldx, (int)k, st, &nl), who);
    pi = h->prof.begin(K_PERMUTE, st);
    if (left)
        CK(h, h->ops->rows_out(Bout, ldb, h->X.p, ldx, h->hp.dev.invp, n, (int)k, st), who);
    else
        CK(h, h->ops->cols_out(Bout, ldb, h->X.p, ldx, h->hp.dev.invp, n, (int)k, st), who);
    h->prof.end(pi, st, 2.0 * n * k, 0);
    if (last) {
        CK(h, record_timing(h, h->ev1, st), who);
        h->solve_pending = !h->capturing;
    }
    h->st.pairs_solve += solve_pairs_per_rhs(h->hp) * (double)k;
    h->st.kernel_launches += nl + 2;
    return PP_OK;
}

// lmul! / rmul! on the device layout X[position][rhs].  `left` selects the caller's layout (B n x k for
// lmul!, k x n for rmul!), `trans` the transposed factor: lmul!(transpose(F), B) = (rmul!(B^T, F))^T and
// rmul!(B, transpose(F)) = (lmul!(F, B^T))^T for the commutative (x) of every semiring here, so a transposed
// solve runs the other direction's sweeps (U* forward then L* backward for lmul!, src/CPU/chordal/sgetrs.jl:
// 88-110 with trans = :T) on this layout.
static int32_t run_solve(pp_handle *h, void *B, int64_t ldb, int64_t k, int32_t where, int left, int trans,
                         const char *who) {
    AllocScope alloc_scope(h);
    if (!h) return fail(nullptr, PP_EINVAL, "%s: null handle", who);
    if (!h->factored) return fail(h, PP_ESTATE, "%s: no factorization (call pp_factor)", who);
    const int n = h->hp.n;
    if (k < 0 || k >= INT32_MAX / 2) return fail(h, PP_EINVAL, "%s: k = %lld", who, (long long)k);
    if (where != PP_HOST && where != PP_DEVICE) return fail(h, PP_EINVAL, "%s: where", who);
    if (k == 0 || n == 0) {
        ok(h);
        return PP_OK;
    }
    if (!B) return fail(h, PP_EINVAL, "%s: null B", who);
    if (left ? ldb < n : ldb < k) return fail(h, PP_EINVAL, "%s: leading dimension %lld", who, (long long)ldb);
    CK(h, cudaSetDevice(h->device), who);
    const size_t es = h->ops->esize;
    const int64_t ldx = (k + 3) & ~(int64_t)3;
    const size_t xbytes = es * (size_t)n * ldx;
    const size_t bbytes = es * (size_t)n * k;
    size_t need = (xbytes > h->X.bytes ? xbytes : 0) + (where == PP_HOST && bbytes > h->stage_in.bytes ? bbytes : 0);
    if (need_memory(h, need, who) != PP_OK) return PP_ENOMEM;
    CK(h, h->X.ensure(xbytes), who);
    if (ensure_sync(h, k) != PP_OK) return PP_ENOMEM;
    cudaStream_t st = h->stream;
    void *Bd = B;
    int64_t ldbd = ldb;
    if (where == PP_HOST && left && bbytes >= ((size_t)32 << 20) && k >= 128) {
        // B in host memory, in up to four column panels of at least 128 right-hand sides: the uploads run on the
        // copy stream (overlapping a factorization still queued on the handle's stream), panel p is solved on the
        // handle's stream once its upload is done, and its result goes back on the output stream while panel
        // p + 1 is solved, so that most of the PCIe traffic overlaps the solves
        CK(h, h->stage_in.ensure(bbytes), who);
        char *Bdev = static_cast<char *>(h->stage_in.p);
        char *Bh = static_cast<char *>(B);
        const int np = (int)std::min<int64_t>(pp_handle::kSolvePanels, k / 128);
        // uploads, solves and downloads are enqueued in that order, so that a copy that blocks the host (pageable
        // memory) finds the GPU work behind it already queued
        for (int p = 0; p < np; p++) {
            const int64_t c0 = k * p / np, c1 = k * (p + 1) / np;
            CK(h, cudaMemcpy2DAsync(Bdev + es * n * c0, es * n, Bh + es * ldb * c0, es * ldb, es * n, c1 - c0,
                                    cudaMemcpyHostToDevice, h->copy_stream), who);
            CK(h, cudaEventRecord(h->in_ev[p], h->copy_stream), who);
        }
        for (int p = 0; p < np; p++) {
            const int64_t c0 = k * p / np, c1 = k * (p + 1) / np;
            CK(h, cudaStreamWaitEvent(st, h->in_ev[p], 0), who);
            void *Bp = Bdev + es * n * c0;
            const int32_t r = enqueue_solve(h, Bp, Bp, n, c1 - c0, left, trans, who, p == 0, p == np - 1);
            if (r != PP_OK) return r;
            CK(h, cudaEventRecord(h->out_ev[p], st), who);
        }
        for (int p = 0; p < np; p++) {
            const int64_t c0 = k * p / np, c1 = k * (p + 1) / np;
            CK(h, cudaStreamWaitEvent(h->out_stream, h->out_ev[p], 0), who);
            CK(h, cudaMemcpy2DAsync(Bh + es * ldb * c0, es * ldb, Bdev + es * n * c0, es * n, es * n, c1 - c0,
                                    cudaMemcpyDeviceToHost, h->out_stream), who);
        }
        // the handle's stream ends after the last download, and the call returns with the result in host memory
        CK(h, cudaEventRecord(h->copy_ev, h->out_stream), who);
        CK(h, cudaStreamWaitEvent(st, h->copy_ev, 0), who);
        const int32_t r2 = settle(h, who);
        if (r2 != PP_OK) return r2;
        ok(h);
        return PP_OK;
    }
    if (where == PP_HOST) {
        // the copy runs on the copy stream, so it overlaps work still queued on the handle's stream (a
        // factorization enqueued just before); the stream waits for it before the solve reads B
        CK(h, h->stage_in.ensure(bbytes), who);
        Bd = h->stage_in.p;
        if (left) {
            ldbd = n;
            CK(h, cudaMemcpy2DAsync(Bd, es * n, B, es * ldb, es * n, k, cudaMemcpyHostToDevice, h->copy_stream), who);
        } else {
            ldbd = k;
            CK(h, cudaMemcpy2DAsync(Bd, es * k, B, es * ldb, es * k, n, cudaMemcpyHostToDevice, h->copy_stream), who);
        }
        CK(h, cudaEventRecord(h->copy_ev, h->copy_stream), who);
        CK(h, cudaStreamWaitEvent(st, h->copy_ev, 0), who);
    }
    const int32_t r = enqueue_solve(h, Bd, Bd, ldbd, k, left, trans, who);
    if (r != PP_OK) return r;
    if (where == PP_HOST) {
        if (left)
            CK(h, cudaMemcpy2DAsync(B, es * ldb, Bd, es * n, es * n, k, cudaMemcpyDeviceToHost, st), who);
        else
            CK(h, cudaMemcpy2DAsync(B, es * ldb, Bd, es * k, es * k, n, cudaMemcpyDeviceToHost, st), who);
        const int32_t r2 = settle(h, who);  // the result is in host memory when the call returns
        if (r2 != PP_OK) return r2;
    }
    ok(h);
    return PP_OK;
}

extern "C" int32_t pp_lmul(pp_handle *h, void *B, int64_t ldb, int64_t k, int32_t where) {
    return run_solve(h, B, ldb, k, where, 1, 0, "pp_lmul");
}

extern "C" int32_t pp_lmul_t(pp_handle *h, void *B, int64_t ldb, int64_t k, int32_t where) {
    return run_solve(h, B, ldb, k, where, 1, 1, "pp_lmul_t");
}

// lmul! on device-resident B with the caller's scratch instead of the handle's: the right-hand-side
// workspace first, the sweep counters after it.  Allocates nothing (no device memory, no profiler events);
// the counters are reset by the sweeps themselves before each persistent launch, so the scratch may hold
// anything on entry.
int32_t pp_internal_lmul_scratch(pp_handle *h, void *B, int64_t ldb, int64_t k, void *scratch, size_t cap,
                                 const char *who) {
    if (!h) return fail(nullptr, PP_EINVAL, "%s: null handle", who);
    if (!h->factored) return fail(h, PP_ESTATE, "%s: no factorization (call pp_factor)", who);
    const int n = h->hp.n;
    if (k < 0 || k >= INT32_MAX / 2) return fail(h, PP_EINVAL, "%s: k = %lld", who, (long long)k);
    if (k == 0 || n == 0) {
        ok(h);
        return PP_OK;
    }
    if (!B) return fail(h, PP_EINVAL, "%s: null B", who);
    if (ldb < n) return fail(h, PP_EINVAL, "%s: leading dimension %lld < n = %d", who, (long long)ldb, n);
    const size_t need = pp_internal_lmul_scratch_bytes(h, k);
    if (need > cap)
        return fail(h, PP_EINVAL,
                    "%s: n = %d and k = %lld need %zu bytes of scratch, the static scratch holds %zu; "
                    "use pp_lmul or fewer right-hand sides per call",
                    who, n, (long long)k, need, cap);
    CK(h, cudaSetDevice(h->device), who);
    cudaPointerAttributes pa{};
    CK(h, cudaPointerGetAttributes(&pa, B), who);
    if (pa.type != cudaMemoryTypeDevice && pa.type != cudaMemoryTypeManaged)
        return fail(h, PP_EINVAL, "%s: B must be device memory", who);
    if (pa.type == cudaMemoryTypeDevice && pa.device != h->device)
        return fail(h, PP_EINVAL, "%s: B is on device %d, the handle on device %d", who, pa.device, h->device);
    const size_t es = h->ops->esize;
    const int64_t ldx = (k + 3) & ~(int64_t)3;
    const size_t xbytes = ((es * (size_t)n * ldx) + 255) & ~(size_t)255;
    void *X = scratch;
    int *sync = reinterpret_cast<int *>(static_cast<unsigned char *>(scratch) + xbytes);
    // borrow the counters and switch the profiler off for this call; both are put back before returning
    int *const save_sync = h->hp.d_sync;
    const int64_t save_cap = h->hp.sync_cap;
    Profiler *const save_prof = h->hp.prof;
    h->hp.d_sync = sync;
    h->hp.sync_cap = (int64_t)((cap - xbytes) / sizeof(int));
    h->hp.prof = nullptr;
    cudaStream_t st = h->stream;
    int64_t nl = 0;
    cudaError_t e = cudaEventRecord(h->ev0, st);
    if (e == cudaSuccess) e = h->ops->rows_in(B, ldb, X, ldx, h->hp.dev.invp, n, (int)k, st);
    if (e == cudaSuccess) e = h->ops->solve(h->hp, values_of(h), 1, X, ldx, (int)k, st, &nl);
    if (e == cudaSuccess) e = h->ops->rows_out(B, ldb, X, ldx, h->hp.dev.invp, n, (int)k, st);
    if (e == cudaSuccess) e = cudaEventRecord(h->ev1, st);
    h->hp.d_sync = save_sync;
    h->hp.sync_cap = save_cap;
    h->hp.prof = save_prof;
    if (e != cudaSuccess) return cuda_fail(h, e, who);
    h->solve_pending = true;
    h->st.pairs_solve = solve_pairs_per_rhs(h->hp) * (double)k;
    h->st.kernel_launches = nl + 2;
    const int32_t r = settle(h, who);  // the scratch is free again when the call returns
    if (r != PP_OK) return r;
    ok(h);
    return PP_OK;
}

int32_t pp_internal_device(const pp_handle *h, int *device) {
    if (!h || !device) return PP_EINVAL;
    *device = h->device;
    return PP_OK;
}

int32_t pp_internal_fail(pp_handle *h, int32_t code, const char *msg) { return fail(h, code, "%s", msg); }

size_t pp_internal_esize(const pp_handle *h) { return h && h->ops ? h->ops->esize : 0; }

// scratch bytes of pp_internal_lmul_scratch for k right-hand sides: the workspace (rounded to 256 bytes)
// and the counters of ensure_sync
size_t pp_internal_lmul_scratch_bytes(const pp_handle *h, int64_t k) {
    if (!h || !h->ops || k <= 0) return 0;
    const int64_t ldx = (k + 3) & ~(int64_t)3;
    const size_t xbytes = ((h->ops->esize * (size_t)h->hp.n * ldx) + 255) & ~(size_t)255;
    const int64_t counters = sync_ints(h->hp.nf, k);
    return xbytes + sizeof(int) * (size_t)counters;
}

extern "C" int32_t pp_rmul(pp_handle *h, void *B, int64_t ldb, int64_t k, int32_t where) {
    return run_solve(h, B, ldb, k, where, 0, 0, "pp_rmul");
}

extern "C" int32_t pp_rmul_t(pp_handle *h, void *B, int64_t ldb, int64_t k, int32_t where) {
    return run_solve(h, B, ldb, k, where, 0, 1, "pp_rmul_t");
}

// Host threads that copy star panels out of the pinned ring into the caller's pageable array: every thread
// copies its share of the columns of every panel, in panel order, while the GPU computes the next panels.
struct RingCopier {
    struct Job {  // w runs of col_bytes: run c from src + c * col_bytes to dst + c * ldc_bytes
        const unsigned char *src = nullptr;
        unsigned char *dst = nullptr;
        size_t col_bytes = 0, ldc_bytes = 0;
        int w = 0;
    };
    int T;
    std::vector<Job> jobs;
    std::vector<int> done;  // threads finished, per panel
    int posted = 0;
    bool stop = false;
    std::mutex mu;
    std::condition_variable cv_post, cv_done;
    std::vector<std::thread> th;

    RingCopier(int nthreads, int64_t npanels) : T(nthreads), jobs(npanels), done(npanels, 0) {
        for (int t = 0; t < T; t++) th.emplace_back([this, t] { run(t); });
    }
    ~RingCopier() {
        {
            std::lock_guard<std::mutex> lk(mu);
            stop = true;
        }
        cv_post.notify_all();
        for (auto &x : th) x.join();
    }
    void run(int t) {
        for (int p = 0;; p++) {
            Job j;
            {
                std::unique_lock<std::mutex> lk(mu);
                cv_post.wait(lk, [&] { return stop || posted > p; });
                if (posted <= p) return;
                j = jobs[p];
            }
            const int a = (int)((int64_t)j.w * t / T), b = (int)((int64_t)j.w * (t + 1) / T);
            for (int c = a; c < b; c++) memcpy(j.dst + c * j.ldc_bytes, j.src + c * j.col_bytes, j.col_bytes);
            {
                std::lock_guard<std::mutex> lk(mu);
                done[p]++;
            }
            cv_done.notify_all();
        }
    }
    void post(int p, const Job &j) {
        {
            std::lock_guard<std::mutex> lk(mu);
            jobs[p] = j;
            posted = p + 1;
        }
        cv_post.notify_all();
    }
    void wait(int p) {
        std::unique_lock<std::mutex> lk(mu);
        cv_done.wait(lk, [&] { return done[p] == T; });
    }
};

// Columns of A* into C (n x ncols): col0 .. col0 + ncols - 1, or cols[0 .. ncols - 1] (original labels) when cols is
// given.  rows: the rows cols[0 .. ncols - 1] of A* into C (ncols x n), rmul! of unit rows.
static int32_t star_impl(pp_handle *h, void *C, int64_t ldc, int64_t col0, int64_t ncols, const int64_t *cols,
                         int32_t where, const char *who, bool rows = false) {
    AllocScope alloc_scope(h);
    if (!h) return fail(nullptr, PP_EINVAL, "%s: null handle", who);
    if (!h->factored) return fail(h, PP_ESTATE, "%s: no factorization (call pp_factor)", who);
    const int n = h->hp.n;
    if (cols) col0 = 0;
    if (col0 < 0 || ncols < 0 || (cols ? ncols > INT32_MAX : col0 + ncols > n))
        return fail(h, PP_EINVAL, "%s: columns out of range", who);
    if (where != PP_HOST && where != PP_DEVICE) return fail(h, PP_EINVAL, "%s: where", who);
    if (ncols == 0) {
        ok(h);
        return PP_OK;
    }
    if (!C || ldc < (rows ? ncols : n)) return fail(h, PP_EINVAL, "%s: C / ldc", who);
    if (cols)
        for (int64_t c = 0; c < ncols; c++)
            if (cols[c] < 0 || cols[c] >= n) return fail(h, PP_EINVAL, "%s: column %lld out of range", who, (long long)cols[c]);
    CK(h, cudaSetDevice(h->device), who);
    const size_t es = h->ops->esize;
    // panel width, a multiple of 32 columns: wide panels give the sweeps of the top fronts, whose 64-row blocks
    // form dependency chains, many independent column tiles to run beside each chain, and each panel pays the
    // launches' tails once (about 8 GB of right-hand sides per panel, at most 32,768 columns: config 3's star
    // 255.7 -> 228.7 ms against 2 GB panels of at most 16,384); host output uses panels of about 256 MB so that
    // the copy of one panel to the host overlaps the computation of the next
    const int64_t budget = where == PP_DEVICE ? ((int64_t)1 << 33) : ((int64_t)1 << 28);
    int64_t pw = budget / std::max<int64_t>((int64_t)es * n, 1);
    pw = std::max<int64_t>(32, std::min<int64_t>(pw & ~(int64_t)31, where == PP_DEVICE ? 32768 : 4096));
    pw = std::min<int64_t>(pw, (ncols + 31) & ~(int64_t)31);
    const int64_t ldx = pw;
    const size_t xbytes = es * (size_t)n * ldx;
    const size_t sbytes = where == PP_HOST ? 2 * es * (size_t)n * pw : 0;  // two staging panels
    if (need_memory(h, (xbytes > h->X.bytes ? xbytes : 0) + (sbytes > h->stage_out.bytes ? sbytes : 0), who) != PP_OK)
        return PP_ENOMEM;
    CK(h, h->X.ensure(xbytes), who);
    if (sbytes) CK(h, h->stage_out.ensure(sbytes), who);
    if (ensure_sync(h, pw) != PP_OK) return PP_ENOMEM;
    cudaStream_t st = h->stream;
    int64_t nl = 0;
    // device output: the requested columns are taken in elimination order (sorted positions) and each panel
    // column is written to its own column of C, so the 32 sources of a tile lie in a few neighbouring subtrees
    // and the forward sweep skips every front outside their root paths (its zero test is per tile)
    const bool mapped = !rows && where == PP_DEVICE && ncols > 32;
    const int *d_pos = nullptr, *d_cmap = nullptr;
    std::vector<int> &hm = h->star_host;
    if (mapped) {
        // hm[0 .. ncols): the positions of the sources in elimination order; hm[ncols + j]: the output column
        hm.resize(2 * (size_t)ncols);
        std::vector<int> order(ncols);
        for (int64_t c = 0; c < ncols; c++) order[c] = (int)c;
        auto src = [&](int c) { return (int)(cols ? cols[c] : col0 + c); };
        std::sort(order.begin(), order.end(), [&](int a, int b) { return h->invp[src(a)] < h->invp[src(b)]; });
        for (int64_t c = 0; c < ncols; c++) {
            hm[c] = h->invp[src(order[c])];
            hm[ncols + c] = order[c];
        }
    } else if (cols) {
        // caller order: hm[j] the position of source j
        hm.resize((size_t)ncols);
        for (int64_t c = 0; c < ncols; c++) hm[c] = h->invp[cols[c]];
    }
    if (mapped || cols) {
        CK(h, h->star_map.ensure(sizeof(int) * hm.size()), who);
        CK(h, cudaMemcpyAsync(h->star_map.p, hm.data(), sizeof(int) * hm.size(), cudaMemcpyHostToDevice, st), who);
        d_pos = h->star_map.as<int>();
        if (mapped) d_cmap = d_pos + ncols;
    }
    // host output into pageable memory (not page-locked, not registered): the copy engine cannot write it at full
    // speed, so each panel goes to a slot of a page-locked ring first and host threads copy it into C from there
    // while the GPU computes the next panels; page-locked C takes the copies directly
    bool use_ring = false;
    if (where == PP_HOST) {
        cudaPointerAttributes pa{};
        if (cudaPointerGetAttributes(&pa, C) != cudaSuccess) cudaGetLastError();
        use_ring = pa.type == cudaMemoryTypeUnregistered;
    }
    const size_t slot_bytes = es * (size_t)n * pw;
    std::unique_ptr<RingCopier> copier;
    if (use_ring) {
        CK(h, h->ring.ensure(3 * slot_bytes), who);
        const unsigned hw = std::thread::hardware_concurrency();
        const int T = (int)std::max(1u, std::min(16u, hw ? hw : 4u));
        try {
            copier.reset(new RingCopier(T, (ncols + pw - 1) / pw));
        } catch (const std::exception &) {
            return fail(h, PP_ENOMEM, "%s: could not start the host copy threads", who);
        }
    }
    auto ring_job = [&](int64_t p) {
        RingCopier::Job j;
        const int w = (int)std::min<int64_t>(pw, ncols - p * pw);
        j.src = static_cast<const unsigned char *>(h->ring.p) + (size_t)(p % 3) * slot_bytes;
        j.ldc_bytes = es * (size_t)ldc;
        if (rows) {  // n runs of w elements: row block p * pw .. of every column of C
            j.dst = static_cast<unsigned char *>(C) + es * (size_t)(p * pw);
            j.col_bytes = es * (size_t)w;
            j.w = n;
        } else {  // w columns of n elements
            j.dst = static_cast<unsigned char *>(C) + es * (size_t)(p * pw) * (size_t)ldc;
            j.col_bytes = es * (size_t)n;
            j.w = w;
        }
        return j;
    };
    CK(h, cudaEventRecord(h->ev0, st), who);
    // host output: panel i is written to staging buffer i % 2 and copied to C on the copy stream while panel
    // i + 1 is computed; panel i + 2 waits for that copy before it reuses the buffer
    int64_t panel = 0;
    for (int64_t c0 = 0; c0 < ncols; c0 += pw, panel++) {
        const int w = (int)std::min<int64_t>(pw, ncols - c0);
        const int buf = (int)(panel & 1);
        CK(h, h->ops->fill_zero(h->X.p, (int64_t)n * ldx, st), who);
        if (d_pos)
            CK(h, h->ops->unit_positions(h->X.p, ldx, d_pos + c0, w, st), who);
        else
            CK(h, h->ops->unit_sources(h->X.p, ldx, h->hp.dev.invp, col0 + c0, w, st), who);
        CK(h, h->ops->solve(h->hp, values_of(h), rows ? 0 : 1, h->X.p, ldx, w, st, &nl), who);
        void *stage = static_cast<char *>(h->stage_out.p) + (size_t)buf * es * (size_t)n * pw;
        // the panel's first element in C: column c0 (n x ncols), or row c0 (ncols x n)
        char *cpan = static_cast<char *>(C) + es * (size_t)c0 * (rows ? 1 : (size_t)ldc);
        void *dst = where == PP_HOST ? stage : (void *)cpan;
        const int64_t lddst = where == PP_HOST ? (rows ? w : n) : ldc;
        if (where == PP_HOST && panel >= 2) CK(h, cudaStreamWaitEvent(st, h->panel_copied[buf], 0), who);
        const int pi = h->prof.begin(K_PERMUTE, st);
        if (mapped)
            CK(h, h->ops->rows_out_mapped(C, ldc, h->X.p, ldx, h->hp.dev.invp, d_cmap + c0, n, w, st), who);
        else if (rows)
            CK(h, h->ops->cols_out(dst, lddst, h->X.p, ldx, h->hp.dev.invp, n, w, st), who);
        else
            CK(h, h->ops->rows_out(dst, lddst, h->X.p, ldx, h->hp.dev.invp, n, w, st), who);
        h->prof.end(pi, st, 2.0 * n * w, 0);
        nl += 3;
        if (where == PP_HOST && use_ring) {
            // slot panel % 3 of the ring: free once the host threads copied panel - 3 out of it
            const int slot = (int)(panel % 3);
            if (panel >= 3) copier->wait((int)(panel - 3));
            CK(h, cudaEventRecord(h->panel_ready[buf], st), who);
            CK(h, cudaStreamWaitEvent(h->copy_stream, h->panel_ready[buf], 0), who);
            CK(h, cudaMemcpyAsync(static_cast<char *>(h->ring.p) + (size_t)slot * slot_bytes, stage, es * (size_t)n * w,
                                  cudaMemcpyDeviceToHost, h->copy_stream),
               who);
            CK(h, cudaEventRecord(h->panel_copied[buf], h->copy_stream), who);
            CK(h, cudaEventRecord(h->ring_ev[slot], h->copy_stream), who);
            if (panel >= 1) {  // the previous panel has reached the ring (or will soon): hand it to the threads
                CK(h, cudaEventSynchronize(h->ring_ev[(panel - 1) % 3]), who);
                copier->post((int)(panel - 1), ring_job(panel - 1));
            }
        } else if (where == PP_HOST) {
            CK(h, cudaEventRecord(h->panel_ready[buf], st), who);
            CK(h, cudaStreamWaitEvent(h->copy_stream, h->panel_ready[buf], 0), who);
            if (rows)  // n columns of w elements
                CK(h, cudaMemcpy2DAsync(cpan, es * ldc, stage, es * w, es * w, n, cudaMemcpyDeviceToHost, h->copy_stream),
                   who);
            else
                CK(h, cudaMemcpy2DAsync(cpan, es * ldc, stage, es * n, es * n, w, cudaMemcpyDeviceToHost, h->copy_stream),
                   who);
            CK(h, cudaEventRecord(h->panel_copied[buf], h->copy_stream), who);
        }
    }
    if (use_ring && panel >= 1) {
        CK(h, cudaEventSynchronize(h->ring_ev[(panel - 1) % 3]), who);
        copier->post((int)(panel - 1), ring_job(panel - 1));
        for (int64_t p = std::max<int64_t>(0, panel - 3); p < panel; p++) copier->wait((int)p);
    }
    if (where == PP_HOST) {
        CK(h, cudaEventRecord(h->copy_ev, h->copy_stream), who);
        CK(h, cudaStreamWaitEvent(st, h->copy_ev, 0), who);  // the last copies are part of the call
    }
    CK(h, cudaEventRecord(h->ev1, st), who);
    h->solve_pending = true;
    h->st.pairs_solve = solve_pairs_per_rhs(h->hp) * (double)ncols;
    h->st.kernel_launches = nl;
    if (where == PP_HOST) {
        const int32_t r = settle(h, who);
        if (r != PP_OK) return r;
    }
    ok(h);
    return PP_OK;
}

extern "C" int32_t pp_star(pp_handle *h, void *C, int64_t ldc, int64_t col0, int64_t ncols, int32_t where) {
    return star_impl(h, C, ldc, col0, ncols, nullptr, where, "pp_star");
}

extern "C" int32_t pp_star_cols(pp_handle *h, void *C, int64_t ldc, const int64_t *cols, int64_t ncols, int32_t where) {
    if (ncols > 0 && !cols) return fail(h, PP_EINVAL, "pp_star_cols: null cols");
    return star_impl(h, C, ldc, 0, ncols, cols, where, "pp_star_cols");
}

extern "C" int32_t pp_star_rows(pp_handle *h, void *C, int64_t ldc, const int64_t *sources, int64_t k, int32_t where) {
    if (k > 0 && !sources) return fail(h, PP_EINVAL, "pp_star_rows: null sources");
    return star_impl(h, C, ldc, 0, k, sources, where, "pp_star_rows", true);
}

extern "C" int32_t pp_sync(pp_handle *h) {
    if (!h) return fail(nullptr, PP_EINVAL, "pp_sync: null handle");
    CK(h, cudaSetDevice(h->device), "pp_sync");
    const int32_t r = settle(h, "pp_sync");
    if (r != PP_OK) return r;
    ok(h);
    return PP_OK;
}

extern "C" int32_t pp_get_trace(pp_handle *h, uint64_t *out, int64_t max_tasks, int64_t *ntasks) {
    if (!h || !ntasks || (max_tasks > 0 && !out)) return fail(h, PP_EINVAL, "pp_get_trace: null argument");
    CK(h, cudaSetDevice(h->device), "pp_get_trace");
    const int32_t r = settle(h, "pp_get_trace");
    if (r != PP_OK) return r;
    const int64_t have = h->d_trace.p && h->trace_on ? (int64_t)h->hp.top_ntasks : 0;
    *ntasks = have;
    const int64_t m = std::min<int64_t>(have, std::max<int64_t>(max_tasks, 0));
    if (m > 0)
        CK(h, cudaMemcpy(out, h->d_trace.p, sizeof(uint64_t) * PP_TRACE_WORDS * (size_t)m, cudaMemcpyDeviceToHost),
           "pp_get_trace");
    ok(h);
    return PP_OK;
}

extern "C" int32_t pp_get_stats(pp_handle *h, pp_stats *s) {
    if (!h || !s) return fail(h, PP_EINVAL, "pp_get_stats: null argument");
    CK(h, cudaSetDevice(h->device), "pp_get_stats");
    const int32_t r = settle(h, "pp_get_stats");
    if (r != PP_OK) return r;
    int64_t bytes = 0;
    for (DevBuf *b : {&h->d_rlo, &h->d_nn, &h->d_na, &h->d_sptr, &h->d_stgt, &h->d_rel, &h->d_dptr, &h->d_lptr,
                      &h->d_chdptr, &h->d_chdtgt, &h->d_mptr, &h->d_mld, &h->d_fws, &h->d_nptr, &h->d_ntgt,
                      &h->d_perm, &h->d_invp, &h->d_idx, &h->d_bptr, &h->d_fcc, &h->d_sfronts,
                      &h->d_sverts, &h->LD, &h->LL, &h->UD, &h->UL, &h->Nval, &h->W, &h->X, &h->stage_in,
                      &h->stage_out, &h->csc_ptr, &h->csc_row, &h->csc_val})
        bytes += (int64_t)b->bytes;
    h->st.device_bytes = bytes;
    *s = h->st;
    ok(h);
    return PP_OK;
}

extern "C" int32_t pp_set_profile(pp_handle *h, int32_t on) {
    if (!h) return fail(nullptr, PP_EINVAL, "pp_set_profile: null handle");
    CK(h, cudaSetDevice(h->device), "pp_set_profile");
    const int32_t r = settle(h, "pp_set_profile");
    if (r != PP_OK) return r;
    h->prof.reset();
    h->prof.on = on != 0;
    ok(h);
    return PP_OK;
}

extern "C" int32_t pp_get_profile(pp_handle *h, pp_kernel_class *out, int32_t max, int32_t *count) {
    if (!h || (!out && max > 0)) return fail(h, PP_EINVAL, "pp_get_profile: null argument");
    CK(h, cudaSetDevice(h->device), "pp_get_profile");
    const int32_t r = settle(h, "pp_get_profile");
    if (r != PP_OK) return r;
    int c = 0;
    for (int k = 0; k < K_NCLASS && c < max; k++) {
        if (h->prof.launches[k] == 0) continue;
        pp_kernel_class &o = out[c++];
        std::memset(&o, 0, sizeof o);
        std::strncpy(o.name, KCLASS_NAMES[k], sizeof o.name - 1);
        o.launches = h->prof.launches[k];
        o.ms = h->prof.ms[k];
        o.bytes = h->prof.bytes[k];
        o.pairs = h->prof.pairs[k];
    }
    if (count) *count = c;
    ok(h);
    return PP_OK;
}

// ---------------------------------------------------------------- plans: refactor + solve as one CUDA graph

// Record the events that order the handle's calls after a factorization (ev_bottom, ev_factored) on the
// handle's stream, outside any capture, so that they mark everything enqueued on it so far.
static cudaError_t uncapture_events(pp_handle *h) {
    cudaError_t e = cudaEventRecord(h->ev_bottom, h->stream);
    if (e == cudaSuccess) e = cudaEventRecord(h->ev_factored, h->stream);
    if (e == cudaSuccess) e = cudaEventRecord(h->ev_top_a, h->stream);
    return e;
}

// A plan owns the scratch its graph uses (the right-hand sides in the device layout and the counters of the
// persistent kernels), so that later calls of the handle, which may grow and so reallocate the handle's own
// buffers, never free memory the graph points into.
struct pp_plan {
    pp_handle *h = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    int64_t launches = 0;
    DevBuf X, sync;
};

// The calls of one plan step, enqueued on the handle's stream: new weights from device memory re-assembled,
// the factorization, and lmul! of Bin into Bout.
static int32_t plan_step(pp_handle *h, const void *nzval, const void *Bin, void *Bout, int64_t ldb, int64_t k,
                         int64_t *launches) {
    int32_t r = pp_update_values(h, nzval, PP_DEVICE);
    if (r != PP_OK) return r;
    r = pp_factor(h);
    if (r != PP_OK) return r;
    int64_t nl = 6 + h->st.kernel_launches;  // the re-assembly's fills and kernel, then the factorization's
    r = enqueue_solve(h, Bin, Bout, ldb, k, 1, 0, "pp_plan_lmul");
    if (r != PP_OK) return r;
    if (launches) *launches = nl + h->st.kernel_launches;
    return PP_OK;
}

// plan_step on the plan's own scratch: the handle's right-hand-side buffer and counters are swapped for the
// plan's for the duration of the step (the captured graph then points into the plan's buffers only)
static int32_t plan_step_own(pp_plan *p, const void *nzval, const void *Bin, void *Bout, int64_t ldb, int64_t k) {
    pp_handle *h = p->h;
    std::swap(h->X.p, p->X.p);
    std::swap(h->X.bytes, p->X.bytes);
    int *const save_sync = h->hp.d_sync;
    const int64_t save_cap = h->hp.sync_cap;
    h->hp.d_sync = p->sync.as<int>();
    h->hp.sync_cap = (int64_t)(p->sync.bytes / sizeof(int));
    const int32_t r = plan_step(h, nzval, Bin, Bout, ldb, k, &p->launches);
    h->hp.d_sync = save_sync;
    h->hp.sync_cap = save_cap;
    std::swap(h->X.p, p->X.p);
    std::swap(h->X.bytes, p->X.bytes);
    return r;
}

extern "C" int32_t pp_plan_lmul(pp_handle *h, const void *nzval, const void *Bin, void *Bout, int64_t ldb, int64_t k,
                                pp_plan **out) {
    AllocScope alloc_scope(h);
    const char *who = "pp_plan_lmul";
    if (!out) return fail(h, PP_EINVAL, "%s: null output pointer", who);
    *out = nullptr;
    if (!h) return fail(nullptr, PP_EINVAL, "%s: null handle", who);
    if (!h->have_structure || h->nnz_assembled < 0)
        return fail(h, PP_ESTATE, "%s: no pattern (call pp_assemble first)", who);
    if (h->nranks > 1) return fail(h, PP_ESTATE, "%s: plans are for a handle on one GPU (not joined by pp_comm_init)", who);
    const int n = h->hp.n;
    if (n == 0 || k <= 0 || k >= INT32_MAX / 2) return fail(h, PP_EINVAL, "%s: n = %d, k = %lld", who, n, (long long)k);
    if ((h->nnz_assembled > 0 && !nzval) || !Bin || !Bout || ldb < n) return fail(h, PP_EINVAL, "%s: arrays", who);
    CK(h, cudaSetDevice(h->device), who);
    for (const void *p : {nzval, Bin, (const void *)Bout}) {
        if (!p) continue;
        cudaPointerAttributes pa{};
        CK(h, cudaPointerGetAttributes(&pa, p), who);
        if ((pa.type != cudaMemoryTypeDevice && pa.type != cudaMemoryTypeManaged) ||
            (pa.type == cudaMemoryTypeDevice && pa.device != h->device))
            return fail(h, PP_EINVAL, "%s: nzval, Bin and Bout must be memory of the handle's device", who);
    }
    // one uncaptured step allocates everything the step uses (workspace, right-hand sides, counters) and
    // reports any error; the captured step then allocates nothing
    const size_t es = h->ops ? h->ops->esize : 8;
    const int64_t ldx = (k + 3) & ~(int64_t)3;
    const size_t xbytes = es * (size_t)n * ldx;
    if (need_memory(h, xbytes > h->X.bytes ? xbytes : 0, who) != PP_OK) return PP_ENOMEM;
    CK(h, h->X.ensure(xbytes), who);
    if (ensure_sync(h, k) != PP_OK) return PP_ENOMEM;
    int32_t r = plan_step(h, nzval, Bin, Bout, ldb, k, nullptr);
    if (r != PP_OK) return r;
    r = settle(h, who);
    if (r != PP_OK) return r;
    auto *p = new (std::nothrow) pp_plan();
    if (!p) return fail(h, PP_ENOMEM, "%s: out of host memory", who);
    p->h = h;
    {
        const size_t sbytes = sizeof(int) * (size_t)sync_ints(h->hp.nf, k);
        cudaError_t ea = p->X.ensure(xbytes);
        if (ea == cudaSuccess) ea = p->sync.ensure(sbytes);
        if (ea != cudaSuccess) {
            delete p;
            return cuda_fail(h, ea, who);
        }
    }
    Profiler *const save_prof = h->hp.prof;
    h->hp.prof = nullptr;
    h->capturing = true;
    cudaError_t e = cudaStreamBeginCapture(h->stream, cudaStreamCaptureModeRelaxed);
    if (e == cudaSuccess) {
        r = plan_step_own(p, nzval, Bin, Bout, ldb, k);
        e = cudaStreamEndCapture(h->stream, &p->graph);  // also ends a capture that a failed call left open
    }
    h->capturing = false;
    h->hp.prof = save_prof;
    // the captured step recorded the handle's factorization events inside the graph, where later calls may not
    // wait on them: record them again on the stream, after everything enqueued so far
    uncapture_events(h);
    if (e == cudaSuccess && r == PP_OK) e = cudaGraphInstantiate(&p->exec, p->graph, 0);
    if (e != cudaSuccess || r != PP_OK) {
        if (p->graph) cudaGraphDestroy(p->graph);
        delete p;
        cudaGetLastError();
        return r != PP_OK ? r : cuda_fail(h, e, who);
    }
    *out = p;
    ok(h);
    return PP_OK;
}

extern "C" int32_t pp_plan_launch(pp_plan *p) {
    if (!p || !p->exec) return fail(nullptr, PP_EINVAL, "pp_plan_launch: null plan");
    pp_handle *h = p->h;
    CK(h, cudaSetDevice(h->device), "pp_plan_launch");
    CK(h, cudaGraphLaunch(p->exec, h->stream), "pp_plan_launch");
    // the graph's factorization ends inside the launch: later calls order themselves after the launch
    CK(h, uncapture_events(h), "pp_plan_launch");
    h->factored = true;
    h->have_values = true;
    h->st.kernel_launches = p->launches;
    ok(h);
    return PP_OK;
}

extern "C" int32_t pp_plan_launches(const pp_plan *p, int64_t *launches) {
    if (!p || !launches) return fail(nullptr, PP_EINVAL, "pp_plan_launches: null argument");
    *launches = p->launches;
    return PP_OK;
}

extern "C" int32_t pp_plan_destroy(pp_plan *p) {
    if (!p) return PP_OK;
    if (p->h && cudaSetDevice(p->h->device) == cudaSuccess) cudaStreamSynchronize(p->h->stream);
    if (p->exec) cudaGraphExecDestroy(p->exec);
    if (p->graph) cudaGraphDestroy(p->graph);
    delete p;
    return PP_OK;
}

// ---------------------------------------------------------------- dense kernels on caller memory

extern "C" int32_t pp_gemm(int32_t semiring, int32_t dtype, int64_t m, int64_t n, int64_t k, void *C, int64_t ldc,
                           const void *A, int64_t lda, const void *B, int64_t ldb, void *stream) {
    const Ops *o = get_ops(semiring, dtype);
    if (!o) return fail(nullptr, PP_EUNSUPPORTED, "pp_gemm: semiring %d with element type %d", semiring, dtype);
    if (m < 0 || n < 0 || k < 0 || m >= INT32_MAX || n >= INT32_MAX || k >= INT32_MAX)
        return fail(nullptr, PP_EINVAL, "pp_gemm: sizes");
    if (m == 0 || n == 0 || k == 0) {
        ok(nullptr);
        return PP_OK;
    }
    if (!C || !A || !B || ldc < m || lda < m || ldb < k) return fail(nullptr, PP_EINVAL, "pp_gemm: arrays / leading dimensions");
    cudaError_t e = o->gemm(m, n, k, C, ldc, A, lda, B, ldb, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "pp_gemm");
    ok(nullptr);
    return PP_OK;
}

extern "C" int32_t pp_getrf_batched(int32_t semiring, int32_t dtype, int64_t n, int64_t count, void *A, void *stream) {
    const Ops *o = get_ops(semiring, dtype);
    if (!o) return fail(nullptr, PP_EUNSUPPORTED, "pp_getrf_batched: semiring %d with element type %d", semiring, dtype);
    if (n < 0 || count < 0) return fail(nullptr, PP_EINVAL, "pp_getrf_batched: sizes");
    if (n == 0 || count == 0) {
        ok(nullptr);
        return PP_OK;
    }
    if (n > o->small_limit)
        return fail(nullptr, PP_EUNSUPPORTED, "pp_getrf_batched: blocks larger than %d x %d", o->small_limit, o->small_limit);
    if (!A) return fail(nullptr, PP_EINVAL, "pp_getrf_batched: null A");
    cudaError_t e = o->getrf_batched((int)n, count, A, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "pp_getrf_batched");
    ok(nullptr);
    return PP_OK;
}
