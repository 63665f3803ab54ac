// The digits classifier 64 -> 128 -> 64 -> 16 (examples/digits_model.py:120-139)
// in one launch: normalise (u8 / 16), three dense layers with bias, ReLU on
// the first two, then argmax over the first n_classes logits.
//
// Latency-bound (62.6 MFLOP for 1797 images): one CTA of 256 threads per 32
// images keeps the activations in shared memory, reads the 70 KB of weights
// through L1/L2, and register-blocks each thread over several images so that
// every weight load feeds several multiply-adds.  The QPU rounding mode
// accumulates in k order with round-toward-zero products and adds, as the
// emulator's dense layers do (piton/backend/lower.py:3761-3878), so the
// logits then match three emulated dense_layer_kernel launches bit for bit.
#include "common.cuh"

namespace piton {

constexpr int MLP_ROWS = 16, MLP_THREADS = 256;   // 16 images per CTA: 113 CTAs for 1797 images

template <bool QPU>
__device__ __forceinline__ float mac(float acc, float a, float b) {
    if constexpr (QPU) return qpu_fadd(acc, qpu_fmul(a, b));
    else return fmaf(a, b, acc);
}

// out[r][n] = act(sum_k in[r][k] * W[k][n] + b[n]) for the CTA's rows; thread t
// owns column t % N and rows (t / N) * RPT ... + RPT.
template <bool QPU, int K, int N, bool RELU>
__device__ __forceinline__ void layer(const float *in, float *out, const float *__restrict__ W,
                                      const float *__restrict__ b) {
    constexpr int RPT = MLP_ROWS * N / MLP_THREADS;   // rows per thread
    const int n = threadIdx.x % N, r0 = (threadIdx.x / N) * RPT;
    float acc[RPT];
#pragma unroll
    for (int i = 0; i < RPT; ++i) acc[i] = 0.0f;
#pragma unroll 32
    for (int k = 0; k < K; ++k) {
        float w = __ldg(W + k * N + n);   // 32 weight loads in flight per thread: L2 latency, not FMA, bounds this
#pragma unroll
        for (int i = 0; i < RPT; ++i) acc[i] = mac<QPU>(acc[i], in[(r0 + i) * K + k], w);
    }
    float bias = __ldg(b + n);
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
        float v = QPU ? qpu_fadd(acc[i], bias) : acc[i] + bias;
        if (RELU) v = fmaxf(v, 0.0f);
        out[(r0 + i) * N + n] = v;
    }
}

template <bool QPU, bool U8>
__global__ void __launch_bounds__(MLP_THREADS, 1) mlp_kernel(piton_mlp_args a) {
    __shared__ float x[MLP_ROWS * 64];
    __shared__ float h1[MLP_ROWS * 128];
    __shared__ float h2[MLP_ROWS * 64];
    __shared__ float lg[MLP_ROWS * 16];
    const int64_t row0 = (int64_t)blockIdx.x * MLP_ROWS;
    const int rows = (int)((a.M - row0) < MLP_ROWS ? (a.M - row0) : MLP_ROWS);
    for (int i = threadIdx.x; i < MLP_ROWS * 64; i += MLP_THREADS) {
        int r = i / 64;
        float v = 0.0f;
        if (r < rows) {
            if constexpr (U8) v = (float)reinterpret_cast<const uint8_t *>(a.images)[(row0 + r) * 64 + i % 64] * 0.0625f;
            else v = reinterpret_cast<const float *>(a.images)[(row0 + r) * 64 + i % 64];
        }
        x[i] = v;
    }
    __syncthreads();
    layer<QPU, 64, 128, true>(x, h1, reinterpret_cast<const float *>(a.w1), reinterpret_cast<const float *>(a.b1));
    __syncthreads();
    layer<QPU, 128, 64, true>(h1, h2, reinterpret_cast<const float *>(a.w2), reinterpret_cast<const float *>(a.b2));
    __syncthreads();
    layer<QPU, 64, 16, false>(h2, lg, reinterpret_cast<const float *>(a.w3), reinterpret_cast<const float *>(a.b3));
    __syncthreads();
    float *logits = reinterpret_cast<float *>(a.logits);
    for (int i = threadIdx.x; i < rows * 16; i += MLP_THREADS) logits[row0 * 16 + i] = lg[i];
    if (a.pred && threadIdx.x < rows) {
        const float *l = lg + threadIdx.x * 16;
        int best = 0;
        for (int c = 1; c < a.n_classes; ++c)
            if (l[c] > l[best]) best = c;       // first maximum, as numpy.argmax
        reinterpret_cast<int32_t *>(a.pred)[row0 + threadIdx.x] = best;
    }
}

}  // namespace piton

using namespace piton;

extern "C" int piton_b200_mlp_f32(const piton_mlp_args *a, void *stream) {
    PITON_REQUIRE(a != nullptr, "args is NULL");
    PITON_REQUIRE(a->M >= 0, "M %lld < 0", (long long)a->M);
    PITON_REQUIRE(a->n_classes >= 1 && a->n_classes <= 16, "n_classes %d outside 1..16", a->n_classes);
    PITON_REQUIRE((a->flags & ~PITON_B200_QPU_ROUNDING) == 0, "unknown flags 0x%x", a->flags);
    if (a->M == 0) return PITON_B200_OK;
    PITON_REQUIRE(a->images && a->w1 && a->b1 && a->w2 && a->b2 && a->w3 && a->b3 && a->logits, "NULL pointer");
    unsigned blocks = (unsigned)cdiv(a->M, MLP_ROWS);
    cudaStream_t s = as_stream(stream);
    bool qpu = (a->flags & PITON_B200_QPU_ROUNDING) != 0;
    if (qpu) {
        if (a->images_u8) mlp_kernel<true, true><<<blocks, MLP_THREADS, 0, s>>>(*a);
        else mlp_kernel<true, false><<<blocks, MLP_THREADS, 0, s>>>(*a);
    } else {
        if (a->images_u8) mlp_kernel<false, true><<<blocks, MLP_THREADS, 0, s>>>(*a);
        else mlp_kernel<false, false><<<blocks, MLP_THREADS, 0, s>>>(*a);
    }
    return check_launch("mlp");
}
