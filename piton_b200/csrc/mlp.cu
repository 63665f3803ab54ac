// The digits classifier 64 -> 128 -> 64 -> 16 (examples/digits_model.py:120-139)
// in one launch: normalise (u8 / 16), three dense layers with bias, ReLU on
// the first two, then argmax over the first n_classes logits.
//
// Latency-bound (62.6 MFLOP for 1797 images): one CTA of 256 threads per 16
// images.  Thread 0 starts six bulk copies (cp.async.bulk) of the 70 KB of
// weights and biases into shared memory as soon as the CTA begins, while all
// threads load the images, so the whole weight fetch costs one L2 round trip
// instead of one per weight-load batch inside the k-loops; the layers then read
// weights and activations from shared memory (activations four k-values per
// 16-byte load), each thread register-blocked over several images.  Weights
// that are not 16-byte aligned are read from global memory instead.  The QPU
// rounding mode accumulates in k order with round-toward-zero products and
// adds, as the emulator's dense layers do (piton/backend/lower.py:3761-3878), so
// the logits then match three emulated dense_layer_kernel launches bit for bit.
#include "common.cuh"
#include "sm100.cuh"

namespace piton {

using namespace sm100;

constexpr int MLP_ROWS = 16, MLP_THREADS = 256;   // 16 images per CTA: 113 CTAs for 1797 images
// shared memory, in floats: weights and biases, then the activations of the CTA's rows
constexpr int OFF_W1 = 0, OFF_W2 = OFF_W1 + 64 * 128, OFF_W3 = OFF_W2 + 128 * 64, OFF_B1 = OFF_W3 + 64 * 16,
              OFF_B2 = OFF_B1 + 128, OFF_B3 = OFF_B2 + 64, W_FLOATS = OFF_B3 + 16;
constexpr int OFF_X = W_FLOATS, OFF_H1 = OFF_X + MLP_ROWS * 64, OFF_H2 = OFF_H1 + MLP_ROWS * 128,
              OFF_LG = OFF_H2 + MLP_ROWS * 64, MLP_FLOATS = OFF_LG + MLP_ROWS * 16;
constexpr uint32_t MLP_SMEM = MLP_FLOATS * 4 + 16;   // + the mbarrier
static_assert(OFF_X % 4 == 0 && OFF_H1 % 4 == 0 && OFF_H2 % 4 == 0, "16-byte aligned activation rows");

template <bool QPU>
__device__ __forceinline__ float mac(float acc, float a, float b) {
    if constexpr (QPU) return qpu_fadd(acc, qpu_fmul(a, b));
    else return fmaf(a, b, acc);
}

// out[r][n] = act(sum_k in[r][k] * W[k][n] + b[n]) for the CTA's rows; thread t
// owns column t % N and rows (t / N) * RPT ... + RPT; k in order (the QPU mode's
// sequential accumulation), four k-values of a row per 16-byte shared-memory load.
template <bool QPU, int K, int N, bool RELU>
__device__ __forceinline__ void layer(const float *in, float *out, const float *W, const float *b) {
    constexpr int RPT = MLP_ROWS * N / MLP_THREADS;   // rows per thread
    const int n = threadIdx.x % N, r0 = (threadIdx.x / N) * RPT;
    float acc[RPT];
#pragma unroll
    for (int i = 0; i < RPT; ++i) acc[i] = 0.0f;
#pragma unroll 4
    for (int k = 0; k < K; k += 4) {
        const float w0 = W[k * N + n], w1 = W[(k + 1) * N + n], w2 = W[(k + 2) * N + n], w3 = W[(k + 3) * N + n];
#pragma unroll
        for (int i = 0; i < RPT; ++i) {
            const float4 x = *reinterpret_cast<const float4 *>(in + (r0 + i) * K + k);
            acc[i] = mac<QPU>(acc[i], x.x, w0);
            acc[i] = mac<QPU>(acc[i], x.y, w1);
            acc[i] = mac<QPU>(acc[i], x.z, w2);
            acc[i] = mac<QPU>(acc[i], x.w, w3);
        }
    }
    const float bias = b[n];
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
        float v = QPU ? qpu_fadd(acc[i], bias) : acc[i] + bias;
        if (RELU) v = fmaxf(v, 0.0f);
        out[(r0 + i) * N + n] = v;
    }
}

template <bool QPU, bool U8>
__global__ void __launch_bounds__(MLP_THREADS, 1) mlp_kernel(piton_mlp_args a, int staged) {
    extern __shared__ __align__(16) float sm[];
    uint64_t *bar = reinterpret_cast<uint64_t *>(sm + MLP_FLOATS);
    const float *w1 = reinterpret_cast<const float *>(a.w1), *w2 = reinterpret_cast<const float *>(a.w2),
                *w3 = reinterpret_cast<const float *>(a.w3), *b1 = reinterpret_cast<const float *>(a.b1),
                *b2 = reinterpret_cast<const float *>(a.b2), *b3 = reinterpret_cast<const float *>(a.b3);
    if (staged) {
        if (threadIdx.x == 0) {
            mbar_init(bar, 1);
            fence_mbarrier_init();
            mbar_arrive_expect_tx(bar, W_FLOATS * 4);
            bulk_load(sm + OFF_W1, w1, 64 * 128 * 4, bar);
            bulk_load(sm + OFF_W2, w2, 128 * 64 * 4, bar);
            bulk_load(sm + OFF_W3, w3, 64 * 16 * 4, bar);
            bulk_load(sm + OFF_B1, b1, 128 * 4, bar);
            bulk_load(sm + OFF_B2, b2, 64 * 4, bar);
            bulk_load(sm + OFF_B3, b3, 16 * 4, bar);
        }
    }
    float *x = sm + OFF_X, *h1 = sm + OFF_H1, *h2 = sm + OFF_H2, *lg = sm + OFF_LG;
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
    __syncthreads();   // the barrier is initialised before anyone waits on it
    bool landed = false;
    if (staged) {
        // bounded: should the copies not land, the layers read the weights from global memory
        // (the same values), and the CTA waits for the copies once more before it exits
        landed = __syncthreads_and(mbar_wait(bar, 0)) != 0;
        if (landed) {
            w1 = sm + OFF_W1; w2 = sm + OFF_W2; w3 = sm + OFF_W3;
            b1 = sm + OFF_B1; b2 = sm + OFF_B2; b3 = sm + OFF_B3;
        }
    }
    layer<QPU, 64, 128, true>(x, h1, w1, b1);
    __syncthreads();
    layer<QPU, 128, 64, true>(h1, h2, w2, b2);
    __syncthreads();
    layer<QPU, 64, 16, false>(h2, lg, w3, b3);
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
    if (staged && !landed && threadIdx.x == 0) mbar_wait(bar, 0);
}

template <bool QPU, bool U8>
int launch_mlp(const piton_mlp_args &a, unsigned blocks, int staged, cudaStream_t s) {
    static bool attr[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr[dev]) {
        PITON_CUDA(cudaFuncSetAttribute(mlp_kernel<QPU, U8>, cudaFuncAttributeMaxDynamicSharedMemorySize, MLP_SMEM));
        attr[dev] = true;
    }
    mlp_kernel<QPU, U8><<<blocks, MLP_THREADS, MLP_SMEM, s>>>(a, staged);
    return PITON_B200_OK;
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
    // bulk copies need 16-byte aligned sources (the sizes are multiples of 16)
    const int staged = ((a->w1 | a->w2 | a->w3 | a->b1 | a->b2 | a->b3) & 15) == 0;
    const bool qpu = (a->flags & PITON_B200_QPU_ROUNDING) != 0;
    int rc;
    if (qpu) rc = a->images_u8 ? launch_mlp<true, true>(*a, blocks, staged, s) : launch_mlp<true, false>(*a, blocks, staged, s);
    else rc = a->images_u8 ? launch_mlp<false, true>(*a, blocks, staged, s) : launch_mlp<false, false>(*a, blocks, staged, s);
    if (rc) return rc;
    return check_launch("mlp");
}
