// Row LayerNorm without affine parameters (tests/test_reroll_reduce.py:199-208
// layernorm_kernel): y = (x - mean) / sqrt(var + eps) over the first n_cols
// columns, var the biased (1/n) variance.  One warp per row for rows of up
// to 1024 columns (row kept in registers), one CTA per row above that.
#include "common.cuh"

namespace piton {

template <int ITEMS>
__global__ void __launch_bounds__(256) layernorm_warp_kernel(const float *__restrict__ x, float *__restrict__ y,
                                                             int64_t rows, int64_t n, int64_t sx, int64_t sy,
                                                             float eps) {
    int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float *src = x + row * sx;
    float v[ITEMS];
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
        int64_t c = lane + 32 * i;
        v[i] = c < n ? src[c] : 0.0f;
        s += v[i];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    float mean = s / (float)n;
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
        int64_t c = lane + 32 * i;
        v[i] = c < n ? v[i] - mean : 0.0f;
        q += v[i] * v[i];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    float r = rsqrtf(q / (float)n + eps);
    float *dst = y + row * sy;
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
        int64_t c = lane + 32 * i;
        if (c < n) dst[c] = v[i] * r;
    }
}

__global__ void __launch_bounds__(512) layernorm_cta_kernel(const float *__restrict__ x, float *__restrict__ y,
                                                            int64_t n, int64_t sx, int64_t sy, float eps) {
    __shared__ float red[32];
    const float *src = x + (int64_t)blockIdx.x * sx;
    float *dst = y + (int64_t)blockIdx.x * sy;
    auto block_sum = [&](float v) {
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        __syncthreads();
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
        __syncthreads();
        v = (threadIdx.x & 31) < (blockDim.x >> 5) ? red[threadIdx.x & 31] : 0.0f;
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        return v;
    };
    float s = 0.0f;
    for (int64_t c = threadIdx.x; c < n; c += blockDim.x) s += src[c];
    float mean = block_sum(s) / (float)n;
    float q = 0.0f;
    for (int64_t c = threadIdx.x; c < n; c += blockDim.x) {
        float d = src[c] - mean;
        q += d * d;
    }
    float r = rsqrtf(block_sum(q) / (float)n + eps);
    for (int64_t c = threadIdx.x; c < n; c += blockDim.x) dst[c] = (src[c] - mean) * r;
}

}  // namespace piton

using namespace piton;

extern "C" int piton_b200_layernorm_f32(const piton_layernorm_args *a, void *stream) {
    PITON_REQUIRE(a != nullptr, "args is NULL");
    PITON_REQUIRE(a->rows >= 0 && a->n_cols >= 0, "bad shape");
    PITON_REQUIRE(a->flags == 0, "unknown flags 0x%x", a->flags);
    if (a->rows == 0 || a->n_cols == 0) return PITON_B200_OK;
    PITON_REQUIRE(a->x && a->y, "NULL pointer");
    const float *x = reinterpret_cast<const float *>(a->x);
    float *y = reinterpret_cast<float *>(a->y);
    cudaStream_t s = as_stream(stream);
    float eps = (float)a->eps;
    unsigned wblocks = (unsigned)cdiv(a->rows, 8);
    int64_t n = a->n_cols;
    if (n <= 32) layernorm_warp_kernel<1><<<wblocks, 256, 0, s>>>(x, y, a->rows, n, a->x_row_stride, a->y_row_stride, eps);
    else if (n <= 128) layernorm_warp_kernel<4><<<wblocks, 256, 0, s>>>(x, y, a->rows, n, a->x_row_stride, a->y_row_stride, eps);
    else if (n <= 512) layernorm_warp_kernel<16><<<wblocks, 256, 0, s>>>(x, y, a->rows, n, a->x_row_stride, a->y_row_stride, eps);
    else if (n <= 1024) layernorm_warp_kernel<32><<<wblocks, 256, 0, s>>>(x, y, a->rows, n, a->x_row_stride, a->y_row_stride, eps);
    else layernorm_cta_kernel<<<(unsigned)a->rows, 512, 0, s>>>(x, y, n, a->x_row_stride, a->y_row_stride, eps);
    return check_launch("layernorm");
}
