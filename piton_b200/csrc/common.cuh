// Shared helpers of libpiton_b200: error reporting, argument checks, per-device
// caches and the QPU float model used by the PITON_B200_QPU_ROUNDING mode.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "piton_b200.h"

namespace piton {

// Records the calling thread's error message and returns `code`.
int set_error(int code, const char *fmt, ...);
void clear_error();

// Maps the last CUDA error (launch configuration or a sticky fault) to a status.
int check_launch(const char *what, int launches = 1);

// SM count of the current device (cached per device).
int num_sms();

// Counts this library's kernel launches (all threads); read with
// piton_b200_launch_count().  check_launch() adds `n` per operator call.
void count_launches(int n);

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

#define PITON_REQUIRE(cond, ...)                                   \
    do {                                                           \
        if (!(cond)) return ::piton::set_error(PITON_B200_EINVAL, __VA_ARGS__); \
    } while (0)

#define PITON_CUDA(call)                                                                          \
    do {                                                                                          \
        cudaError_t err_ = (call);                                                                \
        if (err_ != cudaSuccess)                                                                  \
            return ::piton::set_error(PITON_B200_ECUDA, "%s: %s", #call, cudaGetErrorString(err_)); \
    } while (0)

inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
__host__ __device__ inline int64_t cdiv_dev(int64_t a, int64_t b) { return (a + b - 1) / b; }

// ---------------------------------------------------------------------------
// QPU float model (device side).  The VideoCore IV float ALUs truncate the
// exact result toward zero, read denormal operands as +0 and NaN operands as
// infinities of their sign, write every result below 2^-126 in magnitude
// (zeros included) as +0, give inf for results of 2^128 or more, 0*inf = +0
// and, for inf + -inf, the second operand (piton/qpu/emulator.py:137-212).
// The CUDA round-toward-zero intrinsics give the truncated exact result; the
// helpers below add the operand and result rules around them.
// ---------------------------------------------------------------------------

__device__ __forceinline__ float qpu_in(float x) {
    uint32_t u = __float_as_uint(x);
    uint32_t e = (u >> 23) & 0xFFu;
    if (e == 0) return 0.0f;                                   // +-0 and denormals read as +0
    if (e == 255) return (u >> 31) ? -__int_as_float(0x7F800000) : __int_as_float(0x7F800000);
    return x;
}

__device__ __forceinline__ float qpu_out(float r, double exact_abs_hint) {
    // r is the IEEE round-toward-zero result; IEEE RZ saturates at FLT_MAX where
    // the QPU writes inf once the exact value reaches 2^128.
    float a = fabsf(r);
    if (a < 1.17549435e-38f) return 0.0f;
    if (a == 3.40282347e38f && exact_abs_hint >= 3.4028236692093846e38) return copysignf(__int_as_float(0x7F800000), r);
    return r;
}

__device__ __forceinline__ float qpu_fadd(float a, float b) {
    a = qpu_in(a);
    b = qpu_in(b);
    if (isinf(b)) return b;
    if (isinf(a)) return a;
    float r = __fadd_rz(a, b);
    // an exact sum of two floats reaches 2^128 only when the exponents differ by
    // less than 30, and then the double sum is exact
    double hint = (fabsf(r) == 3.40282347e38f) ? fabs((double)a + (double)b) : 0.0;
    return qpu_out(r, hint);
}

__device__ __forceinline__ float qpu_fmul(float a, float b) {
    a = qpu_in(a);
    b = qpu_in(b);
    if ((a == 0.0f && isinf(b)) || (isinf(a) && b == 0.0f)) return 0.0f;
    if (isinf(a) || isinf(b)) return __fmul_rn(a, b);          // inf * finite nonzero: signed inf
    float r = __fmul_rz(a, b);
    double hint = (fabsf(r) == 3.40282347e38f) ? fabs((double)a * (double)b) : 0.0;   // exact in double
    return qpu_out(r, hint);
}

}  // namespace piton
