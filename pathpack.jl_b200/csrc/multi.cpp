// multi.cpp — pp_multi: one process driving several GPUs (the reference's multi-GPU driver runs one task per
// device, ext/PATHPACKCUDAExt/multigpu.jl:432-450).  A pp_multi is a handle per device, joined into one NCCL group
// (pp_comm_init) so that pp_multi_factor splits the factorization; every call fans out over one host thread per
// device and returns the first failure (its message through pp_last_error(NULL) on the calling thread).
// Solves and stars split their right-hand sides or columns into one contiguous panel per device; host arrays
// are written by the devices' calls into disjoint panels.
#include <algorithm>
#include <new>
#include <string>
#include <thread>
#include <vector>

#include "pathpack_b200_internal.h"

struct pp_multi {
    std::vector<pp_handle *> h;
};

namespace {

// fn(i) on device i's handle, one host thread per device; the first failure, recorded on the calling thread
template <typename Fn>
int32_t fan_out(pp_multi *m, const char *who, Fn fn) {
    const size_t nd = m->h.size();
    std::vector<int32_t> rc(nd, PP_OK);
    std::vector<std::thread> th;
    try {
        for (size_t i = 0; i < nd; i++) th.emplace_back([&, i] { rc[i] = fn(i); });
    } catch (const std::exception &) {
        for (auto &t : th) t.join();
        return pp_internal_fail(nullptr, PP_ENOMEM, "pp_multi: could not start the device threads");
    }
    for (auto &t : th) t.join();
    for (size_t i = 0; i < nd; i++)
        if (rc[i] != PP_OK) {
            const std::string msg = std::string(who) + " (device " + std::to_string(i) + "): " + pp_last_error(m->h[i]);
            return pp_internal_fail(nullptr, rc[i], msg.c_str());
        }
    return PP_OK;
}

// [c0, c0 + w) of n items for part i of nd, sizes differing by at most one
void panel(int64_t n, size_t nd, size_t i, int64_t &c0, int64_t &w) {
    const int64_t base = n / (int64_t)nd, extra = n % (int64_t)nd;
    c0 = (int64_t)i * base + std::min<int64_t>((int64_t)i, extra);
    w = base + ((int64_t)i < extra ? 1 : 0);
}

}  // namespace

extern "C" int32_t pp_multi_create(const int32_t *devices, int32_t ndev, const pp_options *opt, pp_multi **out) {
    if (!out || !devices || ndev < 1) return pp_internal_fail(nullptr, PP_EINVAL, "pp_multi_create: arguments");
    *out = nullptr;
    auto *m = new (std::nothrow) pp_multi();
    if (!m) return pp_internal_fail(nullptr, PP_ENOMEM, "pp_multi_create: out of host memory");
    for (int32_t i = 0; i < ndev; i++) {
        pp_handle *h = nullptr;
        const int32_t r = pp_create_with(devices[i], opt, &h);
        if (r != PP_OK) {
            const std::string msg = std::string("pp_multi_create: device ") + std::to_string(devices[i]) + ": " +
                                    pp_last_error(nullptr);
            pp_multi_destroy(m);
            return pp_internal_fail(nullptr, r, msg.c_str());
        }
        m->h.push_back(h);
    }
    if (ndev > 1) {
        unsigned char id[PP_COMM_ID_BYTES];
        int32_t r = pp_comm_id(id);
        if (r == PP_OK)  // every rank joins at once (NCCL's initialisation waits for all of them)
            r = fan_out(m, "pp_multi_create", [&](size_t i) { return pp_comm_init(m->h[i], id, ndev, (int32_t)i); });
        if (r != PP_OK) {
            const std::string msg = pp_last_error(nullptr);
            pp_multi_destroy(m);
            return pp_internal_fail(nullptr, r, msg.c_str());
        }
    }
    *out = m;
    return PP_OK;
}

extern "C" int32_t pp_multi_destroy(pp_multi *m) {
    if (!m) return PP_OK;
    for (pp_handle *h : m->h) pp_destroy(h);
    delete m;
    return PP_OK;
}

extern "C" int32_t pp_multi_handle(pp_multi *m, int32_t i, pp_handle **h) {
    if (!m || !h || i < 0 || (size_t)i >= m->h.size()) return pp_internal_fail(nullptr, PP_EINVAL, "pp_multi_handle: arguments");
    *h = m->h[i];
    return PP_OK;
}

extern "C" int32_t pp_multi_set_structure(pp_multi *m, int64_t n, int64_t nf, int64_t nB, const int64_t *Rptr,
                                          const int64_t *Sptr, const int64_t *Stgt, const int64_t *Bptr,
                                          const int64_t *Fptr, const int64_t *Nptr, const int64_t *Ntgt,
                                          const int64_t *perm, int32_t base) {
    if (!m) return pp_internal_fail(nullptr, PP_EINVAL, "pp_multi_set_structure: null group");
    return fan_out(m, "pp_multi_set_structure", [&](size_t i) {
        return pp_set_structure(m->h[i], n, nf, nB, Rptr, Sptr, Stgt, Bptr, Fptr, Nptr, Ntgt, perm, base);
    });
}

extern "C" int32_t pp_multi_assemble(pp_multi *m, int32_t semiring, int32_t dtype, const int64_t *colptr,
                                     const int64_t *rowval, const void *nzval, int32_t base) {
    if (!m) return pp_internal_fail(nullptr, PP_EINVAL, "pp_multi_assemble: null group");
    return fan_out(m, "pp_multi_assemble",
                   [&](size_t i) { return pp_assemble(m->h[i], semiring, dtype, colptr, rowval, nzval, base); });
}

extern "C" int32_t pp_multi_factor(pp_multi *m) {
    if (!m) return pp_internal_fail(nullptr, PP_EINVAL, "pp_multi_factor: null group");
    return fan_out(m, "pp_multi_factor", [&](size_t i) {
        const int32_t r = pp_factor(m->h[i]);
        return r != PP_OK ? r : pp_sync(m->h[i]);
    });
}

extern "C" int32_t pp_multi_lmul(pp_multi *m, void *B, int64_t ldb, int64_t k, int32_t trans) {
    if (!m || (k > 0 && !B) || k < 0) return pp_internal_fail(nullptr, PP_EINVAL, "pp_multi_lmul: arguments");
    return fan_out(m, "pp_multi_lmul", [&](size_t i) {
        int64_t c0, w;
        panel(k, m->h.size(), i, c0, w);
        if (w == 0) return (int32_t)PP_OK;
        void *Bi = static_cast<char *>(B) + (size_t)c0 * (size_t)ldb * pp_internal_esize(m->h[i]);
        return trans ? pp_lmul_t(m->h[i], Bi, ldb, w, PP_HOST) : pp_lmul(m->h[i], Bi, ldb, w, PP_HOST);
    });
}

extern "C" int32_t pp_multi_rmul(pp_multi *m, void *B, int64_t ldb, int64_t k, int32_t trans) {
    if (!m || (k > 0 && !B) || k < 0) return pp_internal_fail(nullptr, PP_EINVAL, "pp_multi_rmul: arguments");
    return fan_out(m, "pp_multi_rmul", [&](size_t i) {
        int64_t r0, w;
        panel(k, m->h.size(), i, r0, w);
        if (w == 0) return (int32_t)PP_OK;
        void *Bi = static_cast<char *>(B) + (size_t)r0 * pp_internal_esize(m->h[i]);
        return trans ? pp_rmul_t(m->h[i], Bi, ldb, w, PP_HOST) : pp_rmul(m->h[i], Bi, ldb, w, PP_HOST);
    });
}

extern "C" int32_t pp_multi_star(pp_multi *m, void *C, int64_t ldc, int64_t col0, int64_t ncols) {
    if (!m || (ncols > 0 && !C) || ncols < 0) return pp_internal_fail(nullptr, PP_EINVAL, "pp_multi_star: arguments");
    return fan_out(m, "pp_multi_star", [&](size_t i) {
        int64_t c0, w;
        panel(ncols, m->h.size(), i, c0, w);
        if (w == 0) return (int32_t)PP_OK;
        void *Ci = static_cast<char *>(C) + (size_t)c0 * (size_t)ldc * pp_internal_esize(m->h[i]);
        return pp_star(m->h[i], Ci, ldc, col0 + c0, w, PP_HOST);
    });
}
