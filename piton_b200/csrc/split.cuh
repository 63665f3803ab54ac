// Transposing split of an fp32 matrix into tensor-core operands for the attention
// (V -> V^T tf32 high / low halves + bf16 copy).
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>

namespace piton {

__device__ __forceinline__ float split_tf32_trunc(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }

// bf16 of a value (round to nearest): non-finite values as 0, finite ones clamped to the bf16 range
__device__ __forceinline__ __nv_bfloat16 split_bf16_of(float v) {
    constexpr float BF16_MAX = 3.3895313892515355e38f;
    return __float2bfloat16_rn(isfinite(v) ? fminf(fmaxf(v, -BF16_MAX), BF16_MAX) : 0.0f);
}

// two bf16 (split_bf16_of) in one word, `a` in the low half
__device__ __forceinline__ uint32_t split_bf16_pair(float a, float b) {
    return (uint32_t)__bfloat16_as_ushort(split_bf16_of(a)) | ((uint32_t)__bfloat16_as_ushort(split_bf16_of(b)) << 16);
}

enum : int { SPLIT_T_ATTN_V = 1 };

// Destination row r (r < rows) of head h holds the source elements src[h * s_h + c * s_col + r],
// c < cols: the transpose of a source whose elements along r are contiguous (rows % 4 == 0,
// 16-byte aligned base, s_col and s_h multiples of 4).  64 x 64 tiles through shared memory:
// 16-byte loads along r, and per thread 8 consecutive c of one destination row out, in 16-byte
// stores (eight neighbouring threads cover 64 consecutive c of a row, so a warp writes 4 runs of
// 256 contiguous bytes).  Grid (cdiv(cols, 64), cdiv(rows, 64), heads), 256 threads.
//  SPLIT_T_ATTN_V: hi, lo[r * ld + c] = tf32 high half and tf32 of the rest, x[r * ldx + c] = bf16(v).
// Per head the destinations advance by rows * ld (hi, lo) and rows * ldx (x).
template <int MODE>
__global__ void __launch_bounds__(256) split_transpose_kernel(const float *__restrict__ src, int64_t rows,
                                                              int64_t cols, int64_t s_col, int64_t s_h,
                                                              float *__restrict__ hi, float *__restrict__ lo,
                                                              __nv_bfloat16 *__restrict__ x, int64_t ld, int64_t ldx) {
    __shared__ float tile[64][65];   // [c][r]
    const int64_t h = blockIdx.z;
    const int64_t c0 = (int64_t)blockIdx.x * 64, r0 = (int64_t)blockIdx.y * 64;
    const float *s = src + h * s_h;
    const int t = threadIdx.x;
#pragma unroll
    for (int i = t; i < 64 * 16; i += 256) {
        const int cc = i >> 4, q = i & 15;
        const int64_t c = c0 + cc, r = r0 + 4 * q;
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (c < cols && r < rows) v = __ldcs(reinterpret_cast<const float4 *>(s + c * s_col + r));
        tile[cc][4 * q] = v.x;
        tile[cc][4 * q + 1] = v.y;
        tile[cc][4 * q + 2] = v.z;
        tile[cc][4 * q + 3] = v.w;
    }
    __syncthreads();
    static_assert(MODE == SPLIT_T_ATTN_V, "the attention's V is the only transposing split");
    const int64_t c_end = cols;
    float *hh = hi + h * rows * ld;
    float *ll = lo + h * rows * ld;
    __nv_bfloat16 *xx = x + h * rows * ldx;
#pragma unroll
    for (int i = t; i < 64 * 8; i += 256) {
        const int g = i & 7, rr = i >> 3;   // 8 consecutive threads: 64 consecutive c of one row
        const int64_t r = r0 + rr, c = c0 + 8 * g;
        if (r >= rows || c >= c_end) continue;
        float v[8], vh[8], vl[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            v[e] = tile[8 * g + e][rr];   // 0 past cols (the load's fill)
            vh[e] = split_tf32_trunc(v[e]);
            vl[e] = isfinite(v[e]) ? v[e] - vh[e] : 0.0f;
        }
        const bool whole = c + 8 <= cols;
        float *hrow = hh + r * ld + c;
        if (whole) {
            reinterpret_cast<float4 *>(hrow)[0] = make_float4(vh[0], vh[1], vh[2], vh[3]);
            reinterpret_cast<float4 *>(hrow)[1] = make_float4(vh[4], vh[5], vh[6], vh[7]);
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e)
                if (c + e < cols) hrow[e] = vh[e];
        }
        {
            float *lrow = ll + r * ld + c;
#pragma unroll
            for (int e = 0; e < 8; ++e) vl[e] = split_tf32_trunc(vl[e]);
            if (whole) {
                reinterpret_cast<float4 *>(lrow)[0] = make_float4(vl[0], vl[1], vl[2], vl[3]);
                reinterpret_cast<float4 *>(lrow)[1] = make_float4(vl[4], vl[5], vl[6], vl[7]);
                *reinterpret_cast<uint4 *>(xx + r * ldx + c) =
                    make_uint4(split_bf16_pair(v[0], v[1]), split_bf16_pair(v[2], v[3]), split_bf16_pair(v[4], v[5]),
                               split_bf16_pair(v[6], v[7]));
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e)
                    if (c + e < cols) {
                        lrow[e] = vl[e];
                        xx[r * ldx + c + e] = split_bf16_of(v[e]);
                    }
            }
        }
    }
}

}  // namespace piton
