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

__device__ __forceinline__ float qpu_fsub(float a, float b) {
    return qpu_fadd(a, __uint_as_float(__float_as_uint(b) ^ 0x80000000u));
}

// fmin / fmax order the raw words as sign-magnitude keys, a negative key only for a negative
// sign with a non-zero exponent (emulator.py:201-206); max keeps the first operand only when
// its key is strictly larger, min when its key is not larger
__device__ __forceinline__ long long qpu_fkey(float x) {
    const uint32_t u = __float_as_uint(x);
    const long long m = u & 0x7FFFFFFFu;
    return ((u >> 31) && ((u >> 23) & 0xFFu)) ? -m : m;
}
__device__ __forceinline__ float qpu_fmax(float a, float b) { return qpu_fkey(a) > qpu_fkey(b) ? a : b; }
__device__ __forceinline__ float qpu_fmin(float a, float b) { return qpu_fkey(a) <= qpu_fkey(b) ? a : b; }

__device__ __forceinline__ bool qpu_is_nan(float x) { return (__float_as_uint(x) & 0x7FFFFFFFu) > 0x7F800000u; }

// ftoi: truncation to the low 32 bits; a zero / denormal exponent or |x| >= 2^55 gives 0
// (emulator.py:208-212).  itof: int32 -> float rounded toward zero.
__device__ __forceinline__ int32_t qpu_ftoi(float a) {
    const uint32_t e = (__float_as_uint(a) >> 23) & 0xFFu;
    if (e == 0 || e >= 127 + 55) return 0;
    return (int32_t)(uint32_t)(unsigned long long)__float2ll_rz(a);
}
__device__ __forceinline__ float qpu_itof(int32_t n) { return __int2float_rz(n); }

// The compiler's ALU-only exp / exp2 (piton/backend/lower.py:2716-2797): clamp, y = x log2(e)
// (exp), n = ftoi(y +- 0.5), reduction r = (x - n ln2_hi) - n ln2_lo (exp) or (x - n) ln2
// (exp2), a degree-6 polynomial in Horner form, then 2^n put in through the exponent field
// in two steps so that n beyond the normal range still lands; every step a QPU add or
// multiply.  The float32 constants are the nearest floats to the reference's decimal
// literals, written as bits.
__device__ __forceinline__ float qpu_exp(float x, bool base2) {
    float xc = qpu_fmin(x, base2 ? 128.0f : 89.0f);
    xc = qpu_fmax(xc, base2 ? -150.0f : -104.0f);
    const float LOG2E = __uint_as_float(0x3fb8aa3bu), LN2 = __uint_as_float(0x3f317218u),
                LN2_HI = __uint_as_float(0x3f317200u), LN2_LO = __uint_as_float(0x35bfbe8eu);
    const float y = base2 ? xc : qpu_fmul(xc, LOG2E);
    const float half = __uint_as_float((__float_as_uint(y) & 0x80000000u) | 0x3F000000u);
    const int32_t n = qpu_ftoi(qpu_fadd(y, half));
    const float nf = qpu_itof(n);
    float r;
    if (base2) {
        r = qpu_fmul(qpu_fsub(xc, nf), LN2);
    } else {
        const float t2 = qpu_fsub(xc, qpu_fmul(nf, LN2_HI));
        r = qpu_fsub(t2, qpu_fmul(nf, LN2_LO));
    }
    const uint32_t cs[5] = {0x3c088889u, 0x3d2aaaabu, 0x3e2aaaabu, 0x3f000000u, 0x3f800000u};
    float p = qpu_fmul(r, __uint_as_float(0x3ab60b61u));
#pragma unroll
    for (int i = 0; i < 5; ++i) p = qpu_fmul(qpu_fadd(p, __uint_as_float(cs[i])), r);
    const float q = qpu_fadd(p, 1.0f);
    const int32_t nc = n < -127 ? -127 : (n > 127 ? 127 : n);
    const float q2 = __uint_as_float(__float_as_uint(q) + ((uint32_t)(n - nc) << 23));
    float d = qpu_fmul(q2, __uint_as_float((uint32_t)(nc + 127) << 23));
    if (base2) {
        if (!(__float_as_uint(qpu_fsub(x, 128.0f)) >> 31)) d = __uint_as_float(0x7F800000u);
    } else {
        if (__float_as_uint(qpu_fsub(__uint_as_float(0x42B17217u), x)) >> 31) d = __uint_as_float(0x7F800000u);
    }
    if (qpu_is_nan(x)) d = x;
    return d;
}

// Newton reciprocal from the seed 0x7EF311C3 - bits(b), three steps r = r (2 - b r), then the
// large / zero / nan cases (lower.py:633-667); a / b = a * recip(b) with the nan cases of
// lower.py:669-694.
__device__ __forceinline__ float qpu_recip(float b) {
    float r = __uint_as_float(0x7EF311C3u - __float_as_uint(b));
#pragma unroll
    for (int k = 0; k < 3; ++k) r = qpu_fmul(r, qpu_fsub(2.0f, qpu_fmul(b, r)));
    const uint32_t eb = __float_as_uint(b) & 0x7F800000u, sg = __float_as_uint(b) & 0x80000000u;
    if ((int32_t)(eb - 0x7E800000u) >= 0) r = __uint_as_float(sg);
    if (eb == 0) r = __uint_as_float(sg | 0x7F800000u);
    if (qpu_is_nan(b)) r = b;
    return r;
}
__device__ __forceinline__ float qpu_fdiv(float a, float b) {
    float d = qpu_fmul(a, qpu_recip(b));
    const uint32_t ma = __float_as_uint(a) & 0x7FFFFFFFu, mb = __float_as_uint(b) & 0x7FFFFFFFu;
    const uint32_t mx = ma > mb ? ma : mb;
    if ((int32_t)(mx - 0x7F800001u) >= 0) d = __uint_as_float(0x7FC00000u);
    if ((int32_t)((ma | mb) - 0x00800000u) < 0) d = __uint_as_float(0x7FC00000u);
    if ((int32_t)((ma & mb) - 0x7F800000u) >= 0) d = __uint_as_float(0x7FC00000u);
    return d;
}

}  // namespace piton
