// The remaining example operators: element-wise float ops, exact 32-bit
// integer division, row reductions, tile transpose and Conway's Life.
//
//  * elementwise (examples/primitive_kernels.py copy_kernel / fma_kernel /
//    log_kernel, examples/elementwise.py mul_kernel, examples/kernels.py
//    scaled_relu_kernel, examples/sfu_tests.py sfu_kernel): out[i] = f(x[i] (,
//    y[i])) for i < min(n, grid_x * BLOCK).  fma is x*alpha + y with two
//    roundings, as the reference's separate multiply and add; the QPU rounding
//    mode makes mul / fma / scaled_relu bit-exact with the emulator.
//  * idiv (primitive_kernels.py idiv_kernel): C-semantics truncating // and %
//    on int32 (INT_MIN / -1 wraps to INT_MIN, remainder 0) or uint32; exact.
//  * row_reduce (kernels.py row_sum_kernel, primitive_kernels.py
//    row_max_kernel): rows [0, grid_x * BLOCK_M) reduced over the columns the
//    reference program loads, ceil(n_cols / BLOCK_N) * BLOCK_N of them
//    (its loads are unmasked); max starts from -FLT_MAX.
//  * transpose (primitive_kernels.py transpose_kernel): out[c, r] = x[r, c]
//    for the tiles of programs below grid_x.
//  * life (examples/life.py life_kernel / life_rows_kernel / life_bits_kernel):
//    one generation on a torus, alive next iff the 3x3 block holds 3 live
//    cells, or 4 and the cell is alive; int32 0/1 cells or 32 cells per
//    uint32 word; only cells of the programs the launch grid covers are written.
// All HBM-bound; grid-stride loops with 4-wide vector access where the
// layout allows.
#include "common.cuh"

namespace piton {

enum ElemOp : int {
    OP_COPY = 0, OP_MUL = 1, OP_FMA = 2, OP_SCALED_RELU = 3, OP_EXP2 = 4, OP_LOG2 = 5, OP_RECIP = 6,
    OP_RSQRT = 7, OP_EXP = 8, OP_SQRT = 9, OP_LOG = 10, OP_SIGMOID = 11,
};

template <int OP, bool QPU>
__device__ __forceinline__ float elem(float x, float y, float alpha) {
    if constexpr (OP == OP_COPY) return x;
    else if constexpr (OP == OP_MUL) return QPU ? qpu_fmul(x, y) : __fmul_rn(x, y);
    else if constexpr (OP == OP_FMA) return QPU ? qpu_fadd(qpu_fmul(x, alpha), y) : __fadd_rn(__fmul_rn(x, alpha), y);
    else if constexpr (OP == OP_SCALED_RELU) return x > 0.0f ? (QPU ? qpu_fmul(x, alpha) : __fmul_rn(x, alpha)) : 0.0f;
    else if constexpr (OP == OP_EXP2) return exp2f(x);
    else if constexpr (OP == OP_LOG2) return log2f(x);
    else if constexpr (OP == OP_RECIP) return __fdiv_rn(1.0f, x);
    else if constexpr (OP == OP_RSQRT) return rsqrtf(x);
    else if constexpr (OP == OP_EXP) return expf(x);
    else if constexpr (OP == OP_SQRT) return __fsqrt_rn(x);
    else if constexpr (OP == OP_SIGMOID) return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x)));   // tl.sigmoid
    else return logf(x);
}

template <int OP, bool QPU>
__global__ void __launch_bounds__(256) elementwise_kernel(const float *__restrict__ x, const float *__restrict__ y,
                                                          float *__restrict__ out, int64_t n, float alpha, int vec) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (vec) {
        const int64_t n4 = n / 4;
        for (int64_t i = t0; i < n4; i += stride) {
            float4 a = __ldcs(reinterpret_cast<const float4 *>(x) + i);
            float4 b = y ? __ldcs(reinterpret_cast<const float4 *>(y) + i) : make_float4(0, 0, 0, 0);
            float4 r = make_float4(elem<OP, QPU>(a.x, b.x, alpha), elem<OP, QPU>(a.y, b.y, alpha),
                                   elem<OP, QPU>(a.z, b.z, alpha), elem<OP, QPU>(a.w, b.w, alpha));
            __stcs(reinterpret_cast<float4 *>(out) + i, r);
        }
        for (int64_t i = 4 * n4 + t0; i < n; i += stride) out[i] = elem<OP, QPU>(x[i], y ? y[i] : 0.0f, alpha);
    } else {
        for (int64_t i = t0; i < n; i += stride) out[i] = elem<OP, QPU>(x[i], y ? y[i] : 0.0f, alpha);
    }
}

template <int OP>
static void launch_elem(const piton_elementwise_args *a, int64_t n, cudaStream_t s) {
    const float *x = reinterpret_cast<const float *>(a->x);
    const float *y = reinterpret_cast<const float *>(a->y);
    float *out = reinterpret_cast<float *>(a->out);
    int vec = ((a->x | a->y | a->out) & 15u) == 0;
    int64_t blocks = cdiv(vec ? n / 4 + 1 : n, 256);
    int64_t cap = (int64_t)num_sms() * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    if (a->flags & PITON_B200_QPU_ROUNDING)
        elementwise_kernel<OP, true><<<(unsigned)blocks, 256, 0, s>>>(x, y, out, n, (float)a->alpha, vec);
    else
        elementwise_kernel<OP, false><<<(unsigned)blocks, 256, 0, s>>>(x, y, out, n, (float)a->alpha, vec);
}

// ---- exact 32-bit division ----

template <bool SIGNED>
__global__ void __launch_bounds__(256) idiv_kernel(const uint32_t *__restrict__ x, const uint32_t *__restrict__ y,
                                                   uint32_t *__restrict__ q, uint32_t *__restrict__ r, int64_t n) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        uint32_t a = x[i], b = y[i], qq, rr;
        if (b == 0) {                       // undefined in the reference; defined here as q = all ones, r = a
            qq = 0xFFFFFFFFu;
            rr = a;
        } else if (SIGNED) {
            int32_t sa = (int32_t)a, sb = (int32_t)b;
            if (sb == -1) {                 // INT_MIN / -1 wraps (C semantics on 32 bits)
                qq = 0u - a;
                rr = 0u;
            } else {
                qq = (uint32_t)(sa / sb);
                rr = (uint32_t)(sa % sb);
            }
        } else {
            qq = a / b;
            rr = a % b;
        }
        q[i] = qq;
        r[i] = rr;
    }
}

// ---- row reductions ----

template <bool MAX>
__global__ void __launch_bounds__(256) row_reduce_kernel(const float *__restrict__ x, float *__restrict__ out,
                                                         int64_t rows, int64_t cols, int64_t stride) {
    const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float *src = x + row * stride;
    float acc = MAX ? -3.4028234663852886e38f : 0.0f;
    for (int64_t c = lane; c < cols; c += 32) acc = MAX ? fmaxf(acc, src[c]) : acc + src[c];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        float v = __shfl_xor_sync(0xffffffffu, acc, o);
        acc = MAX ? fmaxf(acc, v) : acc + v;
    }
    if (lane == 0) out[row] = acc;
}

// ---- transpose ----

__global__ void __launch_bounds__(256) transpose_kernel(const float *__restrict__ x, float *__restrict__ out,
                                                        int64_t n_rows, int64_t n_cols, int64_t sx, int64_t so,
                                                        int64_t bm, int64_t bn, int64_t grid_x) {
    __shared__ float tile[32][33];
    const int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    const int64_t tiles_n = cdiv_dev(n_cols, bn);
    for (int j = ty; j < 32; j += 8) {
        int64_t r = r0 + j, c = c0 + tx;
        tile[j][tx] = (r < n_rows && c < n_cols) ? x[r * sx + c] : 0.0f;
    }
    __syncthreads();
    for (int j = ty; j < 32; j += 8) {
        int64_t c = c0 + j, r = r0 + tx;   // out[c][r]
        if (r < n_rows && c < n_cols && (r / bm) * tiles_n + c / bn < grid_x) out[c * so + r] = tile[tx][j];
    }
}

// ---- Life ----

__device__ __forceinline__ int64_t wrap_prev(int64_t i, int64_t n) { return i == 0 ? n - 1 : i - 1; }
__device__ __forceinline__ int64_t wrap_next(int64_t i, int64_t n) { return i == n - 1 ? 0 : i + 1; }

// mode 0: life_kernel tiles (BLOCK_R x BLOCK_C, row-major tile ids < grid_x);
// mode 1: life_rows_kernel strips (columns BLOCK wide on grid axis 0, ROWS rows on axis 1)
__global__ void __launch_bounds__(256) life_cells_kernel(const int32_t *__restrict__ src, int32_t *__restrict__ dst,
                                                         int64_t n_rows, int64_t n_cols, int64_t stride, int mode,
                                                         int64_t br, int64_t bc, int64_t gx, int64_t gy) {
    const int64_t total = n_rows * n_cols;
    const int64_t col_blocks = cdiv_dev(n_cols, bc);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / n_cols, c = i % n_cols;
        bool covered = mode == 0 ? (r / br) * col_blocks + c / bc < gx : (c / bc < gx && r / br < gy);
        if (!covered) continue;
        const int64_t ru = wrap_prev(r, n_rows), rd = wrap_next(r, n_rows);
        const int64_t cl = wrap_prev(c, n_cols), cr = wrap_next(c, n_cols);
        const int32_t *up = src + ru * stride, *mid = src + r * stride, *dn = src + rd * stride;
        int32_t alive = mid[c];
        int32_t t = up[cl] + up[c] + up[cr] + mid[cl] + alive + mid[cr] + dn[cl] + dn[c] + dn[cr];
        dst[r * stride + c] = (t == 3 || (t == 4 && alive != 0)) ? 1 : 0;
    }
}

// 32 cells per word (bit j of word k = column 32k + j); strips of BLOCK words x ROWS rows
__global__ void __launch_bounds__(256) life_bits_kernel(const uint32_t *__restrict__ src, uint32_t *__restrict__ dst,
                                                        int64_t n_rows, int64_t n_words, int64_t stride, int64_t rows_per,
                                                        int64_t words_per, int64_t gx, int64_t gy) {
    const int64_t total = n_rows * n_words;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / n_words, w = i % n_words;
        if (!(w / words_per < gx && r / rows_per < gy)) continue;
        const int64_t ru = wrap_prev(r, n_rows), rd = wrap_next(r, n_rows);
        const int64_t wl = wrap_prev(w, n_words), wr = wrap_next(w, n_words);
        uint32_t cnt[3][3];
        const int64_t rr[3] = {ru, r, rd};
        // per row: the words holding each cell's left neighbour, itself and right neighbour
        uint32_t sum0 = 0, sum1 = 0, sum2 = 0, sum3 = 0;   // bit-sliced 4-bit counter
        for (int k = 0; k < 3; ++k) {
            const uint32_t *row = src + rr[k] * stride;
            uint32_t mid = row[w], left = row[wl], right = row[wr];
            cnt[k][0] = (mid << 1) | (left >> 31);    // bit j: the cell left of column j
            cnt[k][1] = mid;
            cnt[k][2] = (mid >> 1) | (right << 31);   // bit j: the cell right of column j
            for (int m = 0; m < 3; ++m) {
                uint32_t v = cnt[k][m];
                uint32_t c0 = sum0 & v;
                sum0 ^= v;
                uint32_t c1 = sum1 & c0;
                sum1 ^= c0;
                uint32_t c2 = sum2 & c1;
                sum2 ^= c1;
                sum3 |= c2;
            }
        }
        const uint32_t alive = cnt[1][1];
        // total == 3: 0011; total == 4: 0100
        const uint32_t three = sum0 & sum1 & ~sum2 & ~sum3;
        const uint32_t four = ~sum0 & ~sum1 & sum2 & ~sum3;
        dst[r * stride + w] = three | (four & alive);
    }
}

static unsigned grid_for(int64_t n) {
    int64_t b = cdiv(n, 256);
    int64_t cap = (int64_t)num_sms() * 8;
    if (b > cap) b = cap;
    return (unsigned)(b < 1 ? 1 : b);
}

}  // namespace piton

using namespace piton;

extern "C" int piton_b200_elementwise_f32(const piton_elementwise_args *a, void *stream) {
    PITON_REQUIRE(a != nullptr, "args is NULL");
    PITON_REQUIRE(a->n_elements >= 0 && a->block_size > 0 && a->grid_x >= 0, "bad shape");
    PITON_REQUIRE(a->op >= OP_COPY && a->op <= OP_SIGMOID, "unknown op %d", a->op);
    PITON_REQUIRE((a->flags & ~PITON_B200_QPU_ROUNDING) == 0, "unknown flags 0x%x", a->flags);
    PITON_REQUIRE(!(a->flags & PITON_B200_QPU_ROUNDING) || a->op <= OP_SCALED_RELU,
                  "QPU rounding applies to copy, mul, fma and scaled_relu");
    int64_t covered = a->grid_x * a->block_size;
    int64_t n = a->n_elements < covered ? a->n_elements : covered;
    if (n == 0) return PITON_B200_OK;
    bool binary = a->op == OP_MUL || a->op == OP_FMA;
    PITON_REQUIRE(a->x && a->out && (!binary || a->y), "NULL pointer");
    piton_elementwise_args b = *a;
    if (!binary) b.y = 0;
    cudaStream_t s = as_stream(stream);
    switch (a->op) {
        case OP_COPY: launch_elem<OP_COPY>(&b, n, s); break;
        case OP_MUL: launch_elem<OP_MUL>(&b, n, s); break;
        case OP_FMA: launch_elem<OP_FMA>(&b, n, s); break;
        case OP_SCALED_RELU: launch_elem<OP_SCALED_RELU>(&b, n, s); break;
        case OP_EXP2: launch_elem<OP_EXP2>(&b, n, s); break;
        case OP_LOG2: launch_elem<OP_LOG2>(&b, n, s); break;
        case OP_RECIP: launch_elem<OP_RECIP>(&b, n, s); break;
        case OP_RSQRT: launch_elem<OP_RSQRT>(&b, n, s); break;
        case OP_EXP: launch_elem<OP_EXP>(&b, n, s); break;
        case OP_SQRT: launch_elem<OP_SQRT>(&b, n, s); break;
        case OP_SIGMOID: launch_elem<OP_SIGMOID>(&b, n, s); break;
        default: launch_elem<OP_LOG>(&b, n, s); break;
    }
    return check_launch("elementwise");
}

extern "C" int piton_b200_idiv_i32(const piton_idiv_args *a, void *stream) {
    PITON_REQUIRE(a != nullptr, "args is NULL");
    PITON_REQUIRE(a->n_elements >= 0 && a->block_size > 0 && a->grid_x >= 0 && a->flags == 0, "bad arguments");
    int64_t covered = a->grid_x * a->block_size;
    int64_t n = a->n_elements < covered ? a->n_elements : covered;
    if (n == 0) return PITON_B200_OK;
    PITON_REQUIRE(a->x && a->y && a->q && a->r, "NULL pointer");
    const uint32_t *x = reinterpret_cast<const uint32_t *>(a->x), *y = reinterpret_cast<const uint32_t *>(a->y);
    uint32_t *q = reinterpret_cast<uint32_t *>(a->q), *r = reinterpret_cast<uint32_t *>(a->r);
    if (a->is_signed) idiv_kernel<true><<<grid_for(n), 256, 0, as_stream(stream)>>>(x, y, q, r, n);
    else idiv_kernel<false><<<grid_for(n), 256, 0, as_stream(stream)>>>(x, y, q, r, n);
    return check_launch("idiv");
}

extern "C" int piton_b200_row_reduce_f32(const piton_row_reduce_args *a, void *stream) {
    PITON_REQUIRE(a != nullptr, "args is NULL");
    PITON_REQUIRE(a->n_cols >= 0 && a->block_m > 0 && a->block_n > 0 && a->grid_x >= 0 && a->flags == 0 &&
                      (a->reduce == 0 || a->reduce == 1),
                  "bad arguments");
    int64_t rows = a->grid_x * a->block_m;
    int64_t cols = cdiv(a->n_cols, a->block_n) * a->block_n;
    if (rows == 0) return PITON_B200_OK;
    PITON_REQUIRE(a->x && a->out, "NULL pointer");
    unsigned blocks = (unsigned)cdiv(rows, 8);
    const float *x = reinterpret_cast<const float *>(a->x);
    float *out = reinterpret_cast<float *>(a->out);
    if (a->reduce) row_reduce_kernel<true><<<blocks, 256, 0, as_stream(stream)>>>(x, out, rows, cols, a->stride);
    else row_reduce_kernel<false><<<blocks, 256, 0, as_stream(stream)>>>(x, out, rows, cols, a->stride);
    return check_launch("row_reduce");
}

extern "C" int piton_b200_transpose_f32(const piton_transpose_args *a, void *stream) {
    PITON_REQUIRE(a != nullptr, "args is NULL");
    PITON_REQUIRE(a->n_rows >= 0 && a->n_cols >= 0 && a->block_m > 0 && a->block_n > 0 && a->grid_x >= 0 &&
                      a->flags == 0,
                  "bad arguments");
    if (a->n_rows == 0 || a->n_cols == 0 || a->grid_x == 0) return PITON_B200_OK;
    PITON_REQUIRE(a->x && a->out, "NULL pointer");
    PITON_REQUIRE(cdiv(a->n_rows, 32) < 65536, "too many rows");
    dim3 g((unsigned)cdiv(a->n_cols, 32), (unsigned)cdiv(a->n_rows, 32));
    transpose_kernel<<<g, 256, 0, as_stream(stream)>>>(reinterpret_cast<const float *>(a->x),
                                                       reinterpret_cast<float *>(a->out), a->n_rows, a->n_cols,
                                                       a->stride_x, a->stride_out, a->block_m, a->block_n, a->grid_x);
    return check_launch("transpose");
}

extern "C" int piton_b200_life_step(const piton_life_args *a, void *stream) {
    PITON_REQUIRE(a != nullptr, "args is NULL");
    PITON_REQUIRE(a->n_rows >= 0 && a->n_cols >= 0 && a->block_r > 0 && a->block_c > 0 && a->grid_x >= 0 &&
                      a->grid_y >= 0 && a->mode >= 0 && a->mode <= 2 && a->flags == 0,
                  "bad arguments");
    if (a->n_rows == 0 || a->n_cols == 0) return PITON_B200_OK;
    PITON_REQUIRE(a->src && a->dst, "NULL pointer");
    PITON_REQUIRE(a->src != a->dst, "src and dst must differ (ping-pong buffers)");
    cudaStream_t s = as_stream(stream);
    if (a->mode == 2)
        life_bits_kernel<<<grid_for(a->n_rows * a->n_cols), 256, 0, s>>>(
            reinterpret_cast<const uint32_t *>(a->src), reinterpret_cast<uint32_t *>(a->dst), a->n_rows, a->n_cols,
            a->stride, a->block_r, a->block_c, a->grid_x, a->grid_y);
    else
        life_cells_kernel<<<grid_for(a->n_rows * a->n_cols), 256, 0, s>>>(
            reinterpret_cast<const int32_t *>(a->src), reinterpret_cast<int32_t *>(a->dst), a->n_rows, a->n_cols,
            a->stride, a->mode, a->block_r, a->block_c, a->grid_x, a->grid_y);
    return check_launch("life");
}
