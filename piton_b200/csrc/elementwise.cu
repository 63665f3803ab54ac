// Vector add (examples/kernels.py:6-15 add_kernel): out[i] = x[i] + y[i] for
// i < min(n_elements, grid_x * BLOCK_SIZE).
//
// HBM-bound: 12 bytes of traffic per element.  Each thread moves UNROLL
// 16-byte vectors per array with streaming (evict-first) loads and stores, all
// loads issued before the adds so that 3 * UNROLL * 16 bytes are in flight per
// thread; a scalar kernel covers the tail and misaligned pointers.
#include "common.cuh"
#include "gemm_tc.cuh"

namespace piton {

template <bool QPU>
__device__ __forceinline__ float add1(float a, float b) {
    if constexpr (QPU) return qpu_fadd(a, b);
    else return a + b;
}

constexpr int ADD_THREADS = 256;
constexpr int ADD_UNROLL = 4;

template <bool QPU>
__global__ void __launch_bounds__(ADD_THREADS) add_vec4_kernel(const float4 *__restrict__ x, const float4 *__restrict__ y,
                                                               float4 *__restrict__ out, int64_t n4) {
    int64_t base = (int64_t)blockIdx.x * (ADD_THREADS * ADD_UNROLL) + threadIdx.x;
    float4 a[ADD_UNROLL], b[ADD_UNROLL];
#pragma unroll
    for (int u = 0; u < ADD_UNROLL; ++u) {
        int64_t i = base + (int64_t)u * ADD_THREADS;
        if (i < n4) {
            a[u] = __ldcs(x + i);
            b[u] = __ldcs(y + i);
        }
    }
#pragma unroll
    for (int u = 0; u < ADD_UNROLL; ++u) {
        int64_t i = base + (int64_t)u * ADD_THREADS;
        if (i < n4) {
            float4 r;
            r.x = add1<QPU>(a[u].x, b[u].x);
            r.y = add1<QPU>(a[u].y, b[u].y);
            r.z = add1<QPU>(a[u].z, b[u].z);
            r.w = add1<QPU>(a[u].w, b[u].w);
            __stcs(out + i, r);
        }
    }
}

// The all-gather variant: element i of this rank's range goes to element e0 + i of every rank's
// full output p[0 .. world), starting with the next rank's, so that the ranks' NVLink stores
// spread over the peers.  All loads are issued before the adds, as above; the sums are kept in
// registers and stored to each destination in turn.
struct AddGather {
    float4 *p[MAX_PEERS];
    int world, rank;
};

__global__ void __launch_bounds__(ADD_THREADS) add_vec4_gather_kernel(const float4 *__restrict__ x,
                                                                      const float4 *__restrict__ y, int64_t n4,
                                                                      int64_t e0_4, AddGather g) {
    int64_t base = (int64_t)blockIdx.x * (ADD_THREADS * ADD_UNROLL) + threadIdx.x;
    float4 a[ADD_UNROLL], b[ADD_UNROLL];
#pragma unroll
    for (int u = 0; u < ADD_UNROLL; ++u) {
        int64_t i = base + (int64_t)u * ADD_THREADS;
        if (i < n4) {
            a[u] = __ldcs(x + i);
            b[u] = __ldcs(y + i);
        }
    }
#pragma unroll
    for (int u = 0; u < ADD_UNROLL; ++u) {
        a[u].x += b[u].x;
        a[u].y += b[u].y;
        a[u].z += b[u].z;
        a[u].w += b[u].w;
    }
    for (int d = 0; d < g.world; ++d) {
        int dr = g.rank + 1 + d;
        dr = dr >= g.world ? dr - g.world : dr;
        float4 *dst = g.p[dr] + e0_4;
#pragma unroll
        for (int u = 0; u < ADD_UNROLL; ++u) {
            int64_t i = base + (int64_t)u * ADD_THREADS;
            if (i < n4) __stcs(dst + i, a[u]);
        }
    }
}

template <bool QPU>
__global__ void add_scalar_kernel(const float *__restrict__ x, const float *__restrict__ y, float *__restrict__ out,
                                  int64_t begin, int64_t end) {
    int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = begin + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < end; i += stride)
        out[i] = add1<QPU>(x[i], y[i]);
}

template <bool QPU>
static int launch_add(const piton_add_args *a, cudaStream_t s, int64_t n) {
    const float *x = reinterpret_cast<const float *>(a->x);
    const float *y = reinterpret_cast<const float *>(a->y);
    float *out = reinterpret_cast<float *>(a->out);
    bool aligned = ((a->x | a->y | a->out) & 15u) == 0;
    int64_t n4 = aligned ? n / 4 : 0;
    if (n4 > 0) {
        int64_t blocks = cdiv(n4, ADD_THREADS * ADD_UNROLL);
        add_vec4_kernel<QPU><<<(unsigned)blocks, ADD_THREADS, 0, s>>>(
            reinterpret_cast<const float4 *>(x), reinterpret_cast<const float4 *>(y), reinterpret_cast<float4 *>(out), n4);
    }
    int64_t rest = n - 4 * n4;
    if (rest > 0) {
        int64_t blocks = cdiv(rest, 256);
        if (blocks > 4 * num_sms()) blocks = 4 * num_sms();
        add_scalar_kernel<QPU><<<(unsigned)blocks, 256, 0, s>>>(x, y, out, 4 * n4, n);
    }
    return check_launch("add", (n4 > 0) + (rest > 0));
}

}  // namespace piton

using namespace piton;

extern "C" int piton_b200_add_f32(const piton_add_args *a, void *stream) {
    PITON_REQUIRE(a != nullptr, "args is NULL");
    PITON_REQUIRE(a->n_elements >= 0, "n_elements %lld < 0", (long long)a->n_elements);
    PITON_REQUIRE(a->block_size > 0 && a->grid_x >= 0, "bad BLOCK_SIZE %lld / grid %lld", (long long)a->block_size,
                  (long long)a->grid_x);
    PITON_REQUIRE((a->flags & ~PITON_B200_QPU_ROUNDING) == 0, "unknown flags 0x%x", a->flags);
    int64_t covered = a->grid_x * a->block_size;
    int64_t n = a->n_elements < covered ? a->n_elements : covered;
    if (n == 0) return PITON_B200_OK;
    PITON_REQUIRE(a->x && a->y && a->out, "NULL pointer");
    cudaStream_t s = as_stream(stream);
    return (a->flags & PITON_B200_QPU_ROUNDING) ? launch_add<true>(a, s, n) : launch_add<false>(a, s, n);
}

// Vector add over this rank's element range with the output all-gather fused into the kernel:
// element i of the range (elements [row_offset, row_offset + n) of the full output) is stored
// into element row_offset + i of every rank's full output through NVLink peer stores.  IEEE
// rounding; n, row_offset and the pointers 16-byte multiples.  The caller orders completion
// across ranks (a barrier on every rank after the call) before reading the output.
extern "C" int piton_b200_add_allgather_f32(const piton_add_args *a, const piton_allgather_args *g, void *stream) {
    PITON_REQUIRE(a != nullptr && g != nullptr, "args is NULL");
    PITON_REQUIRE(a->n_elements >= 0, "n_elements %lld < 0", (long long)a->n_elements);
    PITON_REQUIRE(a->block_size > 0 && a->grid_x >= 0, "bad BLOCK_SIZE %lld / grid %lld", (long long)a->block_size,
                  (long long)a->grid_x);
    PITON_REQUIRE(a->flags == 0, "the all-gather add takes no flags (IEEE rounding only), got 0x%x", a->flags);
    PITON_REQUIRE(g->world >= 1 && g->world <= MAX_PEERS && g->rank >= 0 && g->rank < g->world,
                  "world %d / rank %d outside 1..%d", g->world, g->rank, MAX_PEERS);
    for (int i = 0; i < g->world; ++i)
        PITON_REQUIRE(g->peer_c[i] != 0 && (g->peer_c[i] & 15) == 0, "peer output %d is NULL or misaligned", i);
    int64_t covered = a->grid_x * a->block_size;
    int64_t n = a->n_elements < covered ? a->n_elements : covered;
    if (n == 0) return PITON_B200_OK;
    PITON_REQUIRE(a->x && a->y, "NULL pointer");
    PITON_REQUIRE(((a->x | a->y) & 15u) == 0 && n % 4 == 0 && g->row_offset >= 0 && g->row_offset % 4 == 0,
                  "the all-gather add needs 16-byte aligned inputs and n, row_offset multiples of 4");
    AddGather ag{};
    for (int i = 0; i < g->world; ++i) ag.p[i] = reinterpret_cast<float4 *>(g->peer_c[i]);
    ag.world = g->world;
    ag.rank = g->rank;
    const int64_t n4 = n / 4;
    const int64_t blocks = cdiv(n4, ADD_THREADS * ADD_UNROLL);
    add_vec4_gather_kernel<<<(unsigned)blocks, ADD_THREADS, 0, as_stream(stream)>>>(
        reinterpret_cast<const float4 *>(a->x), reinterpret_cast<const float4 *>(a->y), n4, g->row_offset / 4, ag);
    return check_launch("add_allgather");
}
