// ops.h — the per-(semiring, element type) operation table the C ABI dispatches to.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "plan.h"

namespace pp {

// Host copy of the schedule and of the per-front sizes the drivers need, plus the device lists.
struct HostPlan {
    int n = 0, nf = 0, nB = 0;
    std::vector<int> nn, na, chdptr, chdtgt;
    std::vector<int64_t> sptr, dptr, lptr;
    // workspace layout for the current element size
    size_t esize = 0;
    std::vector<int64_t> mptr, fws;
    std::vector<int> mld;
    int64_t ws_elems = 0;
    // factorization schedule: tree levels by height, each split into size classes
    std::vector<Level> flevels;
    std::vector<int> h_ffronts;
    const int *d_ffronts = nullptr;
    int64_t nN = 0;
    // solve schedules (lmul: components after their coupling successors; rmul: after their predecessors)
    std::vector<Stage> lstages, rstages;
    const int *d_sfronts = nullptr;   // fronts of every stage's levels (both schedules)
    const int *d_sverts = nullptr;    // vertices of every stage (both schedules)
    const int *d_rel = nullptr;
    DevPlan dev{};
};

struct Values {
    void *LD = nullptr, *LL = nullptr, *UD = nullptr, *UL = nullptr, *Nval = nullptr, *W = nullptr;
};

struct Ops {
    int sr, dt;
    size_t esize;
    int small_limit;  // largest nn + na of a front factored in shared memory
    cudaError_t (*fill_zero)(void *p, int64_t n, cudaStream_t st);
    cudaError_t (*assemble)(const HostPlan &hp, const int *colptr, const int *rowval, const void *nzval,
                            const Values &v, cudaStream_t st);
    cudaError_t (*factor)(const HostPlan &hp, const Values &v, cudaStream_t st, int64_t *launches);
    cudaError_t (*solve)(const HostPlan &hp, const Values &v, int left, void *X, int64_t ldx, int k, cudaStream_t st,
                         int64_t *launches);
    cudaError_t (*unit_sources)(void *X, int64_t ldx, const int *invp, int64_t col0, int k, cudaStream_t st);
    cudaError_t (*rows_in)(const void *B, int64_t ldb, void *X, int64_t ldx, const int *invp, int n, int k,
                           cudaStream_t st);
    cudaError_t (*rows_out)(void *B, int64_t ldb, const void *X, int64_t ldx, const int *invp, int n, int k,
                            cudaStream_t st);
    cudaError_t (*cols_in)(const void *B, int64_t ldb, void *X, int64_t ldx, const int *invp, int n, int k,
                           cudaStream_t st);
    cudaError_t (*cols_out)(void *B, int64_t ldb, const void *X, int64_t ldx, const int *invp, int n, int k,
                            cudaStream_t st);
    cudaError_t (*gemm)(int64_t m, int64_t n, int64_t k, void *C, int64_t ldc, const void *A, int64_t lda,
                        const void *B, int64_t ldb, cudaStream_t st);
    cudaError_t (*getrf_batched)(int n, int64_t count, void *A, cudaStream_t st);
};

const Ops *get_ops(int sr, int dt);

// shared-memory budget of the one-CTA front kernel
constexpr size_t SMALL_FRONT_SMEM = 160 * 1024;

}  // namespace pp
