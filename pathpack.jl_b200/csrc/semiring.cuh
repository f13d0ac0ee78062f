// semiring.cuh — the semirings of PATHPACK.jl as device functors.
//
// Each Sem<SR, T> provides the scalar interface the solver reaches (src/CPU/semiring/semiring.jl:50-101):
// zero (szero), one (sone), add (splus), mul (sprod), muladd (smuladd), star (sstar), the integral flag
// (isintegral, semiring.jl:478-519), an atomic (+) for scatters (the reference's atomic_splus!,
// ext/PATHPACKCUDAExt/batched/sweep.jl:267-356), and muladd2, two multiply-adds into one accumulator for the
// GEMM inner loop.
//
//   MinPlus  (min, +)   zero +Inf  one 0     star a >= 0 ? 0 : -Inf      tropical.jl:84-218
//   MaxPlus  (max, +)   zero -Inf  one 0     star 0 >= a ? 0 : +Inf      (DualQuantale{MinPlus})
//   MaxMin   (max, min) zero -Inf  one +Inf  integral                    bottleneck.jl:15-65
//   MinMax   (min, max) zero +Inf  one -Inf  integral
//   MaxProd  (max, *)   zero 0     one 1     star 1 >= a ? 1 : +Inf      (DualQuantale{MinProd})
//   PlusProd (+, *)     zero 0     one 1     star a < 1 ? 1/(1-a) : +Inf real.jl:17-66, smuladd = fma
//   OrAnd    (|, &)     zero 0     one INT32_MAX  integral               boolean.jl:31-79
//
// A floating product that is NaN (Inf + -Inf, Inf * 0) is szero (tropical.jl:164-182).  Float64 min/max are
// the CPU's select (x < y ? x : y, vmin_d / vmax_d below); Float32 min/max are fminf/fmaxf, which also drop a
// NaN sum, as the reference's GPU kernels do (llvm.minnum, ext/PATHPACKCUDAExt.jl:46-49).  Those differ from
// the select only on +0/-0 ties and NaN accumulators, neither of which the solver produces from NaN-free
// inputs without -0.0 weights.
//
// Int32 MinPlus is defined on [0, INT32_MAX] with a saturating product: operands are non-negative, so the
// 32-bit unsigned sum cannot wrap and min(a + b, c) over unsigned values with c <= INT32_MAX is the
// saturated result.  The reference's wrapping a + b (tropical.jl:148-150) overflows on the typemax sentinel.
#pragma once

#include <cuda_runtime.h>
#include <math_constants.h>
#include <stdint.h>

namespace pp {

enum { MINPLUS = 0, MAXPLUS = 1, MAXMIN = 2, MINMAX = 3, MAXPROD = 4, PLUSPROD = 5, ORAND = 6 };

// 3-input min/max.f32 (sm_100a): one instruction for two reductions
__device__ __forceinline__ float min3f(float a, float b, float c) {
    float d;
    asm("min.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// Float64 min / max with the reference's x86 select semantics, vmin(x, y) = ifelse(x < y, x, y) and
// vmax(x, y) = ifelse(x > y, x, y) (src/CPU/semiring/semiring.jl:124-138): a NaN x gives y.  A compare and a
// select is also faster on sm_100a than fmin/fmax.
__device__ __forceinline__ double vmin_d(double x, double y) { return x < y ? x : y; }
__device__ __forceinline__ double vmax_d(double x, double y) { return x > y ? x : y; }

// atomic (+) for float min/max by the integer order of IEEE bit patterns: a non-negative value orders
// like a signed integer, a negative one like the reverse of an unsigned integer
// (the same idea as the reference's atomic_splus!, ext/PATHPACKCUDAExt/batched/sweep.jl:320-333)
__device__ __forceinline__ void atomic_min_f32(float *p, float v) {
    if (!signbit(v))
        atomicMin(reinterpret_cast<int *>(p), __float_as_int(v));
    else
        atomicMax(reinterpret_cast<unsigned int *>(p), __float_as_uint(v));
}
__device__ __forceinline__ void atomic_max_f32(float *p, float v) {
    if (!signbit(v))
        atomicMax(reinterpret_cast<int *>(p), __float_as_int(v));
    else
        atomicMin(reinterpret_cast<unsigned int *>(p), __float_as_uint(v));
}
__device__ __forceinline__ void atomic_min_f64(double *p, double v) {
    if (!signbit(v))
        atomicMin(reinterpret_cast<long long *>(p), __double_as_longlong(v));
    else
        atomicMax(reinterpret_cast<unsigned long long *>(p), (unsigned long long)__double_as_longlong(v));
}
__device__ __forceinline__ void atomic_max_f64(double *p, double v) {
    if (!signbit(v))
        atomicMax(reinterpret_cast<long long *>(p), __double_as_longlong(v));
    else
        atomicMin(reinterpret_cast<unsigned long long *>(p), (unsigned long long)__double_as_longlong(v));
}

// Whether the semiring's zero absorbs in the solves: muladd(zero, b, c) = c and mul(zero, b) = zero for every
// b a factor can hold (a NaN product is zero; the x86 select keeps c).  Then a forward-sweep step whose
// right-hand-side rows are all zero changes nothing and may be skipped.  Not PlusProd: 0 * Inf is NaN there.
template <int SR>
constexpr bool zero_absorbs = SR != PLUSPROD;

template <int SR, typename T>
struct Sem;

// ---------------------------------------------------------------- MinPlus
template <>
struct Sem<MINPLUS, float> {
    using T = float;
    static constexpr bool integral = false;
    static __device__ __forceinline__ T zero() { return CUDART_INF_F; }
    static __device__ __forceinline__ T one() { return 0.f; }
    static __device__ __forceinline__ T add(T a, T b) { return fminf(a, b); }
    static __device__ __forceinline__ T mul(T a, T b) {
        const T c = a + b;
        return c != c ? zero() : c;
    }
    static __device__ __forceinline__ T muladd(T a, T b, T c) { return fminf(a + b, c); }
    static __device__ __forceinline__ T muladd2(T acc, T a0, T a1, T b0, T b1) {
        const float2 s = __fadd2_rn(make_float2(a0, a1), make_float2(b0, b1));
        return min3f(acc, s.x, s.y);
    }
    static __device__ __forceinline__ T star(T a) { return a >= 0.f ? 0.f : -CUDART_INF_F; }
    static __device__ __forceinline__ void atomic_add(T *p, T v) { atomic_min_f32(p, v); }
};
template <>
struct Sem<MINPLUS, double> {
    using T = double;
    static constexpr bool integral = false;
    static __device__ __forceinline__ T zero() { return CUDART_INF; }
    static __device__ __forceinline__ T one() { return 0.; }
    static __device__ __forceinline__ T add(T a, T b) { return vmin_d(a, b); }
    static __device__ __forceinline__ T mul(T a, T b) {
        const T c = a + b;
        return c != c ? zero() : c;
    }
    static __device__ __forceinline__ T muladd(T a, T b, T c) { return vmin_d(a + b, c); }
    static __device__ __forceinline__ T muladd2(T acc, T a0, T a1, T b0, T b1) {
        return vmin_d(a1 + b1, vmin_d(a0 + b0, acc));
    }
    static __device__ __forceinline__ T star(T a) { return a >= 0. ? 0. : -CUDART_INF; }
    static __device__ __forceinline__ void atomic_add(T *p, T v) { atomic_min_f64(p, v); }
};
template <>
struct Sem<MINPLUS, int32_t> {
    using T = int32_t;
    static constexpr bool integral = false;
    static __device__ __forceinline__ T zero() { return INT32_MAX; }
    static __device__ __forceinline__ T one() { return 0; }
    static __device__ __forceinline__ T add(T a, T b) { return min(a, b); }
    static __device__ __forceinline__ T mul(T a, T b) {
        return (T)min((unsigned)a + (unsigned)b, (unsigned)INT32_MAX);
    }
    static __device__ __forceinline__ T muladd(T a, T b, T c) {
        return (T)__viaddmin_u32((unsigned)a, (unsigned)b, (unsigned)c);
    }
    static __device__ __forceinline__ T muladd2(T acc, T a0, T a1, T b0, T b1) {
        return muladd(a1, b1, muladd(a0, b0, acc));
    }
    static __device__ __forceinline__ T star(T a) { return a >= 0 ? 0 : INT32_MIN; }
    static __device__ __forceinline__ void atomic_add(T *p, T v) { atomicMin(p, v); }
};

// ---------------------------------------------------------------- MaxPlus
template <>
struct Sem<MAXPLUS, float> {
    using T = float;
    static constexpr bool integral = false;
    static __device__ __forceinline__ T zero() { return -CUDART_INF_F; }
    static __device__ __forceinline__ T one() { return 0.f; }
    static __device__ __forceinline__ T add(T a, T b) { return fmaxf(a, b); }
    static __device__ __forceinline__ T mul(T a, T b) {
        const T c = a + b;
        return c != c ? zero() : c;
    }
    static __device__ __forceinline__ T muladd(T a, T b, T c) { return fmaxf(a + b, c); }
    static __device__ __forceinline__ T muladd2(T acc, T a0, T a1, T b0, T b1) {
        const float2 s = __fadd2_rn(make_float2(a0, a1), make_float2(b0, b1));
        return max3f(acc, s.x, s.y);
    }
    static __device__ __forceinline__ T star(T a) { return 0.f >= a ? 0.f : CUDART_INF_F; }
    static __device__ __forceinline__ void atomic_add(T *p, T v) { atomic_max_f32(p, v); }
};
template <>
struct Sem<MAXPLUS, double> {
    using T = double;
    static constexpr bool integral = false;
    static __device__ __forceinline__ T zero() { return -CUDART_INF; }
    static __device__ __forceinline__ T one() { return 0.; }
    static __device__ __forceinline__ T add(T a, T b) { return vmax_d(a, b); }
    static __device__ __forceinline__ T mul(T a, T b) {
        const T c = a + b;
        return c != c ? zero() : c;
    }
    static __device__ __forceinline__ T muladd(T a, T b, T c) { return vmax_d(a + b, c); }
    static __device__ __forceinline__ T muladd2(T acc, T a0, T a1, T b0, T b1) {
        return vmax_d(a1 + b1, vmax_d(a0 + b0, acc));
    }
    static __device__ __forceinline__ T star(T a) { return 0. >= a ? 0. : CUDART_INF; }
    static __device__ __forceinline__ void atomic_add(T *p, T v) { atomic_max_f64(p, v); }
};

// ---------------------------------------------------------------- MaxMin (widest paths)
template <>
struct Sem<MAXMIN, float> {
    using T = float;
    static constexpr bool integral = true;
    static __device__ __forceinline__ T zero() { return -CUDART_INF_F; }
    static __device__ __forceinline__ T one() { return CUDART_INF_F; }
    static __device__ __forceinline__ T add(T a, T b) { return fmaxf(a, b); }
    static __device__ __forceinline__ T mul(T a, T b) { return fminf(a, b); }
    static __device__ __forceinline__ T muladd(T a, T b, T c) { return fmaxf(fminf(a, b), c); }
    static __device__ __forceinline__ T muladd2(T acc, T a0, T a1, T b0, T b1) {
        return max3f(acc, fminf(a0, b0), fminf(a1, b1));
    }
    static __device__ __forceinline__ T star(T) { return one(); }
    static __device__ __forceinline__ void atomic_add(T *p, T v) { atomic_max_f32(p, v); }
};
template <>
struct Sem<MAXMIN, double> {
    using T = double;
    static constexpr bool integral = true;
    static __device__ __forceinline__ T zero() { return -CUDART_INF; }
    static __device__ __forceinline__ T one() { return CUDART_INF; }
    static __device__ __forceinline__ T add(T a, T b) { return vmax_d(a, b); }
    static __device__ __forceinline__ T mul(T a, T b) { return vmin_d(a, b); }
    static __device__ __forceinline__ T muladd(T a, T b, T c) { return vmax_d(vmin_d(a, b), c); }
    static __device__ __forceinline__ T muladd2(T acc, T a0, T a1, T b0, T b1) {
        return vmax_d(vmin_d(a1, b1), vmax_d(vmin_d(a0, b0), acc));
    }
    static __device__ __forceinline__ T star(T) { return one(); }
    static __device__ __forceinline__ void atomic_add(T *p, T v) { atomic_max_f64(p, v); }
};

// ---------------------------------------------------------------- MinMax (bottleneck)
template <>
struct Sem<MINMAX, float> {
    using T = float;
    static constexpr bool integral = true;
    static __device__ __forceinline__ T zero() { return CUDART_INF_F; }
    static __device__ __forceinline__ T one() { return -CUDART_INF_F; }
    static __device__ __forceinline__ T add(T a, T b) { return fminf(a, b); }
    static __device__ __forceinline__ T mul(T a, T b) { return fmaxf(a, b); }
    static __device__ __forceinline__ T muladd(T a, T b, T c) { return fminf(fmaxf(a, b), c); }
    static __device__ __forceinline__ T muladd2(T acc, T a0, T a1, T b0, T b1) {
        return min3f(acc, fmaxf(a0, b0), fmaxf(a1, b1));
    }
    static __device__ __forceinline__ T star(T) { return one(); }
    static __device__ __forceinline__ void atomic_add(T *p, T v) { atomic_min_f32(p, v); }
};
template <>
struct Sem<MINMAX, double> {
    using T = double;
    static constexpr bool integral = true;
    static __device__ __forceinline__ T zero() { return CUDART_INF; }
    static __device__ __forceinline__ T one() { return -CUDART_INF; }
    static __device__ __forceinline__ T add(T a, T b) { return vmin_d(a, b); }
    static __device__ __forceinline__ T mul(T a, T b) { return vmax_d(a, b); }
    static __device__ __forceinline__ T muladd(T a, T b, T c) { return vmin_d(vmax_d(a, b), c); }
    static __device__ __forceinline__ T muladd2(T acc, T a0, T a1, T b0, T b1) {
        return vmin_d(vmax_d(a1, b1), vmin_d(vmax_d(a0, b0), acc));
    }
    static __device__ __forceinline__ T star(T) { return one(); }
    static __device__ __forceinline__ void atomic_add(T *p, T v) { atomic_min_f64(p, v); }
};

// ---------------------------------------------------------------- MaxProd (most reliable paths)
template <>
struct Sem<MAXPROD, float> {
    using T = float;
    static constexpr bool integral = false;
    static __device__ __forceinline__ T zero() { return 0.f; }
    static __device__ __forceinline__ T one() { return 1.f; }
    static __device__ __forceinline__ T add(T a, T b) { return fmaxf(a, b); }
    static __device__ __forceinline__ T mul(T a, T b) {
        const T c = a * b;
        return c != c ? zero() : c;
    }
    static __device__ __forceinline__ T muladd(T a, T b, T c) { return fmaxf(a * b, c); }
    static __device__ __forceinline__ T muladd2(T acc, T a0, T a1, T b0, T b1) {
        const float2 s = __fmul2_rn(make_float2(a0, a1), make_float2(b0, b1));
        return max3f(acc, s.x, s.y);
    }
    static __device__ __forceinline__ T star(T a) { return 1.f >= a ? 1.f : CUDART_INF_F; }
    static __device__ __forceinline__ void atomic_add(T *p, T v) { atomic_max_f32(p, v); }
};
template <>
struct Sem<MAXPROD, double> {
    using T = double;
    static constexpr bool integral = false;
    static __device__ __forceinline__ T zero() { return 0.; }
    static __device__ __forceinline__ T one() { return 1.; }
    static __device__ __forceinline__ T add(T a, T b) { return vmax_d(a, b); }
    static __device__ __forceinline__ T mul(T a, T b) {
        const T c = a * b;
        return c != c ? zero() : c;
    }
    static __device__ __forceinline__ T muladd(T a, T b, T c) { return vmax_d(a * b, c); }
    static __device__ __forceinline__ T muladd2(T acc, T a0, T a1, T b0, T b1) {
        return vmax_d(a1 * b1, vmax_d(a0 * b0, acc));
    }
    static __device__ __forceinline__ T star(T a) { return 1. >= a ? 1. : CUDART_INF; }
    static __device__ __forceinline__ void atomic_add(T *p, T v) { atomic_max_f64(p, v); }
};

// ---------------------------------------------------------------- PlusProd (walk sums)
template <>
struct Sem<PLUSPROD, float> {
    using T = float;
    static constexpr bool integral = false;
    static __device__ __forceinline__ T zero() { return 0.f; }
    static __device__ __forceinline__ T one() { return 1.f; }
    static __device__ __forceinline__ T add(T a, T b) { return a + b; }
    static __device__ __forceinline__ T mul(T a, T b) { return a * b; }
    static __device__ __forceinline__ T muladd(T a, T b, T c) { return __fmaf_rn(a, b, c); }
    static __device__ __forceinline__ T muladd2(T acc, T a0, T a1, T b0, T b1) {
        return __fmaf_rn(a1, b1, __fmaf_rn(a0, b0, acc));
    }
    static __device__ __forceinline__ T star(T a) { return a < 1.f ? 1.f / (1.f - a) : CUDART_INF_F; }
    static __device__ __forceinline__ void atomic_add(T *p, T v) { atomicAdd(p, v); }
};
template <>
struct Sem<PLUSPROD, double> {
    using T = double;
    static constexpr bool integral = false;
    static __device__ __forceinline__ T zero() { return 0.; }
    static __device__ __forceinline__ T one() { return 1.; }
    static __device__ __forceinline__ T add(T a, T b) { return a + b; }
    static __device__ __forceinline__ T mul(T a, T b) { return a * b; }
    static __device__ __forceinline__ T muladd(T a, T b, T c) { return __fma_rn(a, b, c); }
    static __device__ __forceinline__ T muladd2(T acc, T a0, T a1, T b0, T b1) {
        return __fma_rn(a1, b1, __fma_rn(a0, b0, acc));
    }
    static __device__ __forceinline__ T star(T a) { return a < 1. ? 1. / (1. - a) : CUDART_INF; }
    static __device__ __forceinline__ void atomic_add(T *p, T v) { atomicAdd(p, v); }
};

// ---------------------------------------------------------------- OrAnd (label sets, reachability)
template <>
struct Sem<ORAND, int32_t> {
    using T = int32_t;
    static constexpr bool integral = true;
    static __device__ __forceinline__ T zero() { return 0; }
    static __device__ __forceinline__ T one() { return INT32_MAX; }
    static __device__ __forceinline__ T add(T a, T b) { return a | b; }
    static __device__ __forceinline__ T mul(T a, T b) { return a & b; }
    static __device__ __forceinline__ T muladd(T a, T b, T c) { return (a & b) | c; }
    static __device__ __forceinline__ T muladd2(T acc, T a0, T a1, T b0, T b1) {
        return (a0 & b0) | (a1 & b1) | acc;
    }
    static __device__ __forceinline__ T star(T) { return one(); }
    static __device__ __forceinline__ void atomic_add(T *p, T v) { atomicOr(p, v); }
};

// pred ? muladd(a, b, c) : c.  For Float64 (min, +) and (max, +) the predicate folds into the select of the
// (+): x = pred && a * b < c ? a * b : c is vmin_d(a * b, c) with the same operands.
template <int SR, typename T>
__device__ __forceinline__ T muladd_if(bool pred, T a, T b, T c) {
    if constexpr ((SR == MINPLUS || SR == MAXPLUS) && sizeof(T) == 8 && !Sem<SR, T>::integral) {
        const T t = a + b;
        if constexpr (SR == MINPLUS)
            return (pred && t < c) ? t : c;
        else
            return (pred && t > c) ? t : c;
    } else {
        return pred ? Sem<SR, T>::muladd(a, b, c) : c;
    }
}

}  // namespace pp
