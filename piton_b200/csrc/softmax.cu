// Fused row softmax (examples/kernels.py:60-76 softmax_kernel): for each of
// grid_x rows, out = exp(x - max(x)) / sum(exp(x - max(x))) over the first
// min(n_cols, BLOCK_SIZE) columns; the reference reads masked columns as -inf,
// which adds nothing to the sum, so they are simply not touched.
//
// HBM-bound (8 bytes per element: one read, one write).  A row is held in
// registers between the max, sum and scale passes, so HBM sees each element
// once in each direction:
//   * rows up to 1024 (vectorised) / 256 (scalar) columns: one warp per row,
//     warp-shuffle reductions;
//   * up to 32768 / 8192 columns: one CTA per row, shuffles then a shared
//     memory exchange between warps;
//   * longer rows: a CTA per row with an online max/sum pass and a second
//     read for the scaled write (12 bytes per element).
#include "common.cuh"
#include "gemm_tc.cuh"

namespace piton {

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Reduction over the TPR threads of one row group.  TPR == 32: a warp; TPR > 32:
// the whole CTA (one row per CTA), through `red` in shared memory.
template <int TPR, bool IS_MAX>
__device__ __forceinline__ float group_reduce(float v, float *red) {
    v = IS_MAX ? warp_max(v) : warp_sum(v);
    if constexpr (TPR > 32) {
        constexpr int NW = TPR / 32;
        int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
        __syncthreads();                     // red may still be read from the previous reduction
        if (lane == 0) red[w] = v;
        __syncthreads();
        v = lane < NW ? red[lane] : (IS_MAX ? -INFINITY : 0.0f);
        v = IS_MAX ? warp_max(v) : warp_sum(v);
    }
    return v;
}

template <int VEC>
struct VecT;
template <>
struct VecT<1> {
    using T = float;
};
template <>
struct VecT<4> {
    using T = float4;
};

__device__ __forceinline__ float &el(float &v, int) { return v; }
__device__ __forceinline__ float &el(float4 &v, int i) { return (&v.x)[i]; }

// Destinations of the fused all-gather: row `row` of this rank's shard goes to row row0 + row
// (row stride ld) of every rank's full output p[0 .. world), starting with the next rank's, so
// that the ranks' NVLink stores spread over the peers.
struct GatherOut {
    float *p[MAX_PEERS];
    int world, rank;
    int64_t row0, ld;
};

// Each row group of TPR threads owns a row; thread t holds, for item i, the VEC
// columns starting at VEC * (t + i * TPR).  With GATHER the row is stored into every
// rank's full output instead of `out` (VEC == 4 only).
template <int TPR, int ITEMS, int VEC, bool GATHER = false>
__global__ void __launch_bounds__(TPR > 32 ? TPR : 256) softmax_reg_kernel(float *__restrict__ out,
                                                                           const float *__restrict__ in,
                                                                           int64_t in_stride, int64_t out_stride,
                                                                           int64_t n, int64_t rows,
                                                                           GatherOut g = GatherOut{}) {
    using V = typename VecT<VEC>::T;
    __shared__ float red[32];
    int64_t row;
    int t;
    if constexpr (TPR == 32) {
        row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
        t = threadIdx.x & 31;
    } else {
        row = blockIdx.x;
        t = threadIdx.x;
    }
    if (row >= rows) return;          // whole warps (TPR == 32) or whole CTAs leave together
    const V *src = reinterpret_cast<const V *>(in + row * in_stride);
    V *dst = reinterpret_cast<V *>(out + row * out_stride);
    const int64_t nv = n / VEC;        // vectors in the row (n % VEC == 0 when VEC > 1)
    V x[ITEMS];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
        int64_t c = t + (int64_t)i * TPR;
        if (c < nv) {
            x[i] = __ldcs(src + c);
#pragma unroll
            for (int j = 0; j < VEC; ++j) m = fmaxf(m, el(x[i], j));
        }
    }
    m = group_reduce<TPR, true>(m, red);
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
        int64_t c = t + (int64_t)i * TPR;
        if (c < nv) {
#pragma unroll
            for (int j = 0; j < VEC; ++j) {
                float e = expf(el(x[i], j) - m);
                el(x[i], j) = e;
                s += e;
            }
        }
    }
    s = group_reduce<TPR, false>(s, red);
    float r = 1.0f / s;
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
        int64_t c = t + (int64_t)i * TPR;
        if (c < nv) {
#pragma unroll
            for (int j = 0; j < VEC; ++j) el(x[i], j) *= r;
            if constexpr (!GATHER) __stcs(dst + c, x[i]);
        }
    }
    if constexpr (GATHER) {
        for (int d = 0; d < g.world; ++d) {
            int dr = g.rank + 1 + d;
            dr = dr >= g.world ? dr - g.world : dr;
            V *gd = reinterpret_cast<V *>(g.p[dr] + (g.row0 + row) * g.ld);
#pragma unroll
            for (int i = 0; i < ITEMS; ++i) {
                int64_t c = t + (int64_t)i * TPR;
                if (c < nv) __stcs(gd + c, x[i]);
            }
        }
    }
}

// Rows too long for registers: pass 1 keeps a running (max, sum) per thread,
// rescaling the sum when the max grows; pass 2 re-reads and writes.
__global__ void __launch_bounds__(1024) softmax_long_kernel(float *__restrict__ out, const float *__restrict__ in,
                                                            int64_t in_stride, int64_t out_stride, int64_t n) {
    __shared__ float red[32];
    const float *src = in + (int64_t)blockIdx.x * in_stride;
    float *dst = out + (int64_t)blockIdx.x * out_stride;
    float m = -INFINITY, s = 0.0f;
    for (int64_t c = threadIdx.x; c < n; c += blockDim.x) {
        float v = src[c];
        if (v == -INFINITY) continue;          // masked entries add nothing
        if (v > m) {
            s = s * expf(m - v) + 1.0f;
            m = v;
        } else {
            s += expf(v - m);
        }
    }
    float gm = group_reduce<1024, true>(m, red);
    float contrib = (m == -INFINITY) ? 0.0f : s * expf(m - gm);
    float gs = group_reduce<1024, false>(contrib, red);
    float r = 1.0f / gs;
    for (int64_t c = threadIdx.x; c < n; c += blockDim.x) dst[c] = expf(src[c] - gm) * r;
}

template <int TPR, int ITEMS, int VEC, bool GATHER>
static void launch_reg(const piton_softmax_args *a, int64_t n, cudaStream_t s, const GatherOut &g) {
    float *out = reinterpret_cast<float *>(a->out);
    const float *in = reinterpret_cast<const float *>(a->in);
    if constexpr (TPR == 32) {
        int64_t blocks = cdiv(a->grid_x, 8);
        softmax_reg_kernel<32, ITEMS, VEC, GATHER><<<(unsigned)blocks, 256, 0, s>>>(out, in, a->in_row_stride,
                                                                                    a->out_row_stride, n, a->grid_x, g);
    } else {
        softmax_reg_kernel<TPR, ITEMS, VEC, GATHER><<<(unsigned)a->grid_x, TPR, 0, s>>>(
            out, in, a->in_row_stride, a->out_row_stride, n, a->grid_x, g);
    }
}

template <int VEC, bool GATHER = false>
static bool dispatch_reg(const piton_softmax_args *a, int64_t n, cudaStream_t s, const GatherOut &g = GatherOut{}) {
    int64_t per = cdiv(n, VEC);   // vectors per row
    if (per <= 32) launch_reg<32, 1, VEC, GATHER>(a, n, s, g);
    else if (per <= 64) launch_reg<32, 2, VEC, GATHER>(a, n, s, g);
    else if (per <= 128) launch_reg<32, 4, VEC, GATHER>(a, n, s, g);
    else if (per <= 256) launch_reg<32, 8, VEC, GATHER>(a, n, s, g);
    else if (per <= 512) launch_reg<256, 2, VEC, GATHER>(a, n, s, g);
    else if (per <= 1024) launch_reg<256, 4, VEC, GATHER>(a, n, s, g);
    else if (per <= 2048) launch_reg<256, 8, VEC, GATHER>(a, n, s, g);
    else if (per <= 4096) launch_reg<512, 8, VEC, GATHER>(a, n, s, g);
    else if (per <= 8192) launch_reg<1024, 8, VEC, GATHER>(a, n, s, g);
    else return false;
    return true;
}

}  // namespace piton

using namespace piton;

// QPU rounding mode: the reference's softmax_kernel program on the QPU float model, bit for bit
// (examples/kernels.py:60-76 as lowered by piton/backend/lower.py).  A row's BLOCK columns sit
// 16 to a vector register: the maximum is an fmax fold over the columns in order (-inf for the
// masked ones), then exp(x - max) with the ALU exp, the sum accumulates the registers lane by
// lane in order and finishes with the rotate-and-add butterfly of lower.py:4043-4064
// (lane i += lane i - s, s = 8, 4, 2, 1; lane 0 holds the sum), and each output is e / sum with
// the Newton reciprocal.  16 threads per row stand for the 16 lanes; 16 rows per CTA.
__global__ void __launch_bounds__(256) softmax_qpu_kernel(float *__restrict__ out, const float *__restrict__ in,
                                                          int64_t sin, int64_t sout, int64_t n_cols, int64_t block,
                                                          int64_t rows) {
    const int l = threadIdx.x & 15;
    const int64_t row = (int64_t)blockIdx.x * 16 + (threadIdx.x >> 4);
    const bool live = row < rows;
    const int64_t n = n_cols < block ? n_cols : block;
    const float *x = in + (live ? row : 0) * sin;
    // the fold's result: the column of the largest key, the last one among equal keys
    long long key = qpu_fkey(-INFINITY);
    int64_t idx = -1;
    for (int64_t j = l; j < block; j += 16) {
        const long long kj = qpu_fkey(live && j < n ? x[j] : -INFINITY);
        if (kj >= key) {
            key = kj;
            idx = j;
        }
    }
#pragma unroll
    for (int o = 8; o >= 1; o >>= 1) {
        const long long ok = __shfl_xor_sync(0xffffffffu, key, o, 16);
        const int64_t oi = __shfl_xor_sync(0xffffffffu, idx, o, 16);
        if (ok > key || (ok == key && oi > idx)) {
            key = ok;
            idx = oi;
        }
    }
    const float m = (live && idx >= 0 && idx < n) ? x[idx] : -INFINITY;
    float acc = 0.0f;   // lanes past BLOCK hold +0
    for (int64_t j = l; j < block; j += 16) {
        const float e = qpu_exp(qpu_fsub(live && j < n ? x[j] : -INFINITY, m), false);
        acc = j == l ? e : qpu_fadd(acc, e);
    }
#pragma unroll
    for (int sft = 8; sft >= 1; sft >>= 1) acc = qpu_fadd(acc, __shfl_sync(0xffffffffu, acc, (l - sft) & 15, 16));
    const float sum = __shfl_sync(0xffffffffu, acc, 0, 16);
    if (live)
        for (int64_t j = l; j < n; j += 16) out[row * sout + j] = qpu_fdiv(qpu_exp(qpu_fsub(x[j], m), false), sum);
}

extern "C" int piton_b200_softmax_f32(const piton_softmax_args *a, void *stream) {
    PITON_REQUIRE(a != nullptr, "args is NULL");
    PITON_REQUIRE(a->grid_x >= 0 && a->n_cols >= 0 && a->block_size > 0, "bad shape: rows %lld cols %lld BLOCK %lld",
                  (long long)a->grid_x, (long long)a->n_cols, (long long)a->block_size);
    PITON_REQUIRE((a->flags & ~PITON_B200_QPU_ROUNDING) == 0, "unknown flags 0x%x", a->flags);
    PITON_REQUIRE(a->grid_x < (1ll << 31), "too many rows");
    int64_t n = a->n_cols < a->block_size ? a->n_cols : a->block_size;
    if (n == 0 || a->grid_x == 0) return PITON_B200_OK;
    PITON_REQUIRE(a->in && a->out, "NULL pointer");
    cudaStream_t s = as_stream(stream);
    if (a->flags & PITON_B200_QPU_ROUNDING) {
        softmax_qpu_kernel<<<(unsigned)cdiv(a->grid_x, (int64_t)16), 256, 0, s>>>(
            reinterpret_cast<float *>(a->out), reinterpret_cast<const float *>(a->in), a->in_row_stride,
            a->out_row_stride, a->n_cols, a->block_size, a->grid_x);
        return check_launch("softmax_qpu");
    }
    bool vec = ((a->in | a->out) & 15u) == 0 && a->in_row_stride % 4 == 0 && a->out_row_stride % 4 == 0 && n % 4 == 0;
    bool done = vec ? dispatch_reg<4>(a, n, s) : dispatch_reg<1>(a, n, s);
    if (!done)
        softmax_long_kernel<<<(unsigned)a->grid_x, 1024, 0, s>>>(reinterpret_cast<float *>(a->out),
                                                                 reinterpret_cast<const float *>(a->in),
                                                                 a->in_row_stride, a->out_row_stride, n);
    return check_launch("softmax");
}

// Softmax over this rank's rows with the output all-gather fused into the kernel: row r of the
// shard (rows [row_offset, row_offset + grid_x) of the full output) is stored into row
// row_offset + r of every rank's full output through NVLink peer stores, so no separate
// all-gather runs.  The caller orders completion across ranks (a barrier on every rank after
// the call) before reading the output.
extern "C" int piton_b200_softmax_allgather_f32(const piton_softmax_args *a, const piton_allgather_args *g,
                                                void *stream) {
    PITON_REQUIRE(a != nullptr && g != nullptr, "args is NULL");
    PITON_REQUIRE(a->grid_x >= 0 && a->n_cols >= 0 && a->block_size > 0, "bad shape: rows %lld cols %lld BLOCK %lld",
                  (long long)a->grid_x, (long long)a->n_cols, (long long)a->block_size);
    PITON_REQUIRE(a->flags == 0, "unknown flags 0x%x", a->flags);
    PITON_REQUIRE(a->grid_x < (1ll << 31), "too many rows");
    PITON_REQUIRE(g->world >= 1 && g->world <= MAX_PEERS && g->rank >= 0 && g->rank < g->world,
                  "world %d / rank %d outside 1..%d", g->world, g->rank, MAX_PEERS);
    int64_t n = a->n_cols < a->block_size ? a->n_cols : a->block_size;
    PITON_REQUIRE(g->row_offset >= 0 && g->ldc >= n && g->ldc % 4 == 0, "bad row_offset / ldc");
    for (int i = 0; i < g->world; ++i)
        PITON_REQUIRE(g->peer_c[i] != 0 && (g->peer_c[i] & 15) == 0, "peer output %d is NULL or misaligned", i);
    if (n == 0 || a->grid_x == 0) return PITON_B200_OK;
    PITON_REQUIRE(a->in, "NULL pointer");
    PITON_REQUIRE((a->in & 15u) == 0 && a->in_row_stride % 4 == 0 && n % 4 == 0 && n <= 4 * 8192,
                  "the all-gather softmax needs 16-byte aligned rows, n_cols %% 4 == 0 and n_cols <= 32768");
    GatherOut go{};
    for (int i = 0; i < g->world; ++i) go.p[i] = reinterpret_cast<float *>(g->peer_c[i]);
    go.world = g->world;
    go.rank = g->rank;
    go.row0 = g->row_offset;
    go.ld = g->ldc;
    dispatch_reg<4, true>(a, n, as_stream(stream), go);
    return check_launch("softmax_allgather");
}
