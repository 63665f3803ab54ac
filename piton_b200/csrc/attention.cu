// Flash-attention forward (examples/attention.py:33-113 attn_fwd_kernel):
// Out = softmax(Q K^T * sm_scale) V per head, optionally causal, with the
// online softmax in base 2 (qk_scale = sm_scale * log2(e), attention.py:95).
//
// Semantics kept from the reference program:
//  * keys >= N_CTX never contribute; with EVEN_N set on a non-causal launch the
//    reference promises N_CTX % BLOCK_N == 0 and skips the ragged tail
//    (attention.py:104-111), so keys >= (N_CTX / BLOCK_N) * BLOCK_N are then
//    skipped here too;
//  * causal: key j contributes to query i only when j <= i;
//  * query rows >= min(N_CTX, grid_x * BLOCK_M) and heads >= grid_y are not
//    written (attention.py:112-113).
//
// CUDA-core version: a CTA of 128 threads owns 64 query rows, walks the keys
// in blocks of 64 staged in shared memory; each thread holds a 4 x 8 block of
// scores and a 4 x D/8 block of the output accumulator.
#include "attention.cuh"
#include "common.cuh"

namespace piton {

constexpr int AT_BM = 64, AT_BN = 64, AT_THREADS = 128;

template <int D>
__global__ void __launch_bounds__(AT_THREADS) attn_simt_kernel(AttnParams p) {
    extern __shared__ float4 smem4[];
    float *Qt = reinterpret_cast<float *>(smem4);   // [D][BM]
    float *Kt = Qt + D * AT_BM;                     // [D][BN]
    float *Vs = Kt + D * AT_BN;                     // [BN][D]
    float *Pt = Vs + AT_BN * D;                     // [BN][BM]
    constexpr int DC = D / 8;                       // output columns per thread

    const int tid = threadIdx.x, ty = tid >> 3, tx = tid & 7;
    const int64_t head = blockIdx.y;
    const int64_t q0 = (int64_t)blockIdx.x * AT_BM;
    const float *Q = p.q + head * p.sqh;
    const float *K = p.k + head * p.skh;
    const float *V = p.v + head * p.svh;
    float *O = p.o + head * p.soh;

    for (int i = tid; i < AT_BM * D; i += AT_THREADS) {
        int r = i / D, d = i % D;
        int64_t m = q0 + r;
        Qt[d * AT_BM + r] = m < p.n_ctx ? Q[m * p.sqm + d] : 0.0f;
    }

    float m_i[4], l_i[4], acc[4][DC];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m_i[i] = -INFINITY;
        l_i[i] = 0.0f;
#pragma unroll
        for (int c = 0; c < DC; ++c) acc[i][c] = 0.0f;
    }
    const float qk_scale = p.qk_scale;
    int64_t kend = p.key_end;
    if (p.causal) {
        int64_t last = q0 + AT_BM;
        if (last < kend) kend = last;
    }
    for (int64_t k0 = 0; k0 < kend; k0 += AT_BN) {
        __syncthreads();      // previous block's Kt/Vs/Pt fully used
        for (int i = tid; i < AT_BN * D; i += AT_THREADS) {
            int c = i / D, d = i % D;
            int64_t n = k0 + c;
            bool ok = n < p.key_end;
            Kt[d * AT_BN + c] = ok ? K[n * p.skn + (int64_t)d * p.skk] : 0.0f;
            Vs[c * D + d] = ok ? V[n * p.svn + d] : 0.0f;
        }
        __syncthreads();
        float s[4][8];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 8; ++j) s[i][j] = 0.0f;
#pragma unroll 4
        for (int d = 0; d < D; ++d) {
            float4 qa = *reinterpret_cast<const float4 *>(Qt + d * AT_BM + ty * 4);
            float4 ka = *reinterpret_cast<const float4 *>(Kt + d * AT_BN + tx * 8);
            float4 kb = *reinterpret_cast<const float4 *>(Kt + d * AT_BN + tx * 8 + 4);
            float qv[4] = {qa.x, qa.y, qa.z, qa.w};
            float kv[8] = {ka.x, ka.y, ka.z, ka.w, kb.x, kb.y, kb.z, kb.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) s[i][j] = fmaf(qv[i], kv[j], s[i][j]);
        }
        // scale, mask, online softmax (row groups of 8 lanes)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            int64_t row = q0 + ty * 4 + i;
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                int64_t col = k0 + tx * 8 + j;
                float v = s[i][j] * qk_scale;
                if (col >= p.key_end || (p.causal && col > row)) v = -INFINITY;
                s[i][j] = v;
                mx = fmaxf(mx, v);
            }
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            float m_new = fmaxf(m_i[i], mx);
            float m_use = m_new == -INFINITY ? 0.0f : m_new;
            float alpha = exp2f(m_i[i] - m_use);
            float sum = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                float e = exp2f(s[i][j] - m_use);
                s[i][j] = e;
                sum += e;
            }
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            sum += __shfl_xor_sync(0xffffffffu, sum, 4);
            l_i[i] = l_i[i] * alpha + sum;
            m_i[i] = m_new;
#pragma unroll
            for (int c = 0; c < DC; ++c) acc[i][c] *= alpha;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j)
            *reinterpret_cast<float4 *>(Pt + (tx * 8 + j) * AT_BM + ty * 4) = make_float4(s[0][j], s[1][j], s[2][j], s[3][j]);
        __syncthreads();
        int cmax = (int)((kend - k0) < AT_BN ? (kend - k0) : AT_BN);
        for (int c = 0; c < cmax; ++c) {
            float4 pa = *reinterpret_cast<const float4 *>(Pt + c * AT_BM + ty * 4);
            float pv[4] = {pa.x, pa.y, pa.z, pa.w};
            float vv[DC];
            if constexpr (DC % 4 == 0) {
#pragma unroll
                for (int q = 0; q < DC; q += 4) {
                    float4 t = *reinterpret_cast<const float4 *>(Vs + c * D + tx * DC + q);
                    vv[q] = t.x; vv[q + 1] = t.y; vv[q + 2] = t.z; vv[q + 3] = t.w;
                }
            } else {
#pragma unroll
                for (int q = 0; q < DC; ++q) vv[q] = Vs[c * D + tx * DC + q];
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int q = 0; q < DC; ++q) acc[i][q] = fmaf(pv[i], vv[q], acc[i][q]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        int64_t row = q0 + ty * 4 + i;
        if (row >= p.row_end) continue;
        float inv = 1.0f / l_i[i];
#pragma unroll
        for (int q = 0; q < DC; ++q) O[row * p.som + tx * DC + q] = acc[i][q] * inv;
    }
}

template <int D>
static int launch_attn_simt(const AttnParams &p, cudaStream_t s) {
    size_t smem = sizeof(float) * (size_t)(D * AT_BM + D * AT_BN + AT_BN * D + AT_BN * AT_BM);
    static bool attr_done[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr_done[dev]) {
        PITON_CUDA(cudaFuncSetAttribute(attn_simt_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        attr_done[dev] = true;
    }
    dim3 grid((unsigned)cdiv(p.row_end, AT_BM), (unsigned)p.heads);
    attn_simt_kernel<D><<<grid, AT_THREADS, smem, s>>>(p);
    return check_launch("attention");
}

int attention_simt(const AttnParams &p, cudaStream_t s) {
    switch (p.head_dim) {
        case 16: return launch_attn_simt<16>(p, s);
        case 32: return launch_attn_simt<32>(p, s);
        case 64: return launch_attn_simt<64>(p, s);
        case 128: return launch_attn_simt<128>(p, s);
        default: return set_error(PITON_B200_ENOTSUP, "HEAD_DIM %lld: supported 16, 32, 64, 128", (long long)p.head_dim);
    }
}

}  // namespace piton

using namespace piton;

static int attn_params(const piton_attention_args *a, AttnParams &p) {
    PITON_REQUIRE(a != nullptr, "args is NULL");
    PITON_REQUIRE(a->n_ctx >= 0 && a->head_dim > 0 && a->block_m > 0 && a->block_n > 0 && a->grid_x >= 0 &&
                      a->grid_y >= 0,
                  "bad shape");
    PITON_REQUIRE((a->flags & ~PITON_B200_FORCE_SIMT) == 0, "unknown flags 0x%x", a->flags);
    p = AttnParams{};
    p.q = reinterpret_cast<const float *>(a->q);
    p.k = reinterpret_cast<const float *>(a->k);
    p.v = reinterpret_cast<const float *>(a->v);
    p.o = reinterpret_cast<float *>(a->out);
    p.sqh = a->stride_qh; p.sqm = a->stride_qm;
    p.skh = a->stride_kh; p.skn = a->stride_kn; p.skk = a->stride_kk;
    p.svh = a->stride_vh; p.svn = a->stride_vn;
    p.soh = a->stride_oh; p.som = a->stride_om;
    p.n_ctx = a->n_ctx;
    p.head_dim = a->head_dim;
    p.heads = a->grid_y;
    p.causal = a->causal != 0;
    p.qk_scale = (float)a->sm_scale * 1.44269504f;
    p.key_end = (!a->causal && a->even_n) ? (a->n_ctx / a->block_n) * a->block_n : a->n_ctx;
    int64_t rows = a->grid_x * a->block_m;
    p.row_end = rows < a->n_ctx ? rows : a->n_ctx;
    return PITON_B200_OK;
}

static bool use_tc(const piton_attention_args *a, const AttnParams &p) {
    return !(a->flags & PITON_B200_FORCE_SIMT) && p.row_end > 0 && p.heads > 0 && attention_tc_supported(p);
}

extern "C" size_t piton_b200_attention_workspace_size(const piton_attention_args *a) {
    AttnParams p;
    if (attn_params(a, p) != PITON_B200_OK || !use_tc(a, p)) return 0;
    return attention_tc_workspace_bytes(p);
}

extern "C" int piton_b200_attention_f32(const piton_attention_args *a, void *stream) {
    AttnParams p;
    int rc = attn_params(a, p);
    if (rc) return rc;
    if (p.row_end <= 0 || p.heads == 0) return PITON_B200_OK;
    PITON_REQUIRE(p.heads < 65536, "too many heads for one launch");
    PITON_REQUIRE(a->q && a->k && a->v && a->out, "NULL pointer");
    if (use_tc(a, p)) {
        size_t need = attention_tc_workspace_bytes(p);
        if (a->workspace_bytes < need || !a->workspace)
            return set_error(PITON_B200_EWORKSPACE, "attention needs %zu bytes of workspace, got %llu", need,
                             (unsigned long long)a->workspace_bytes);
        return attention_tc(p, reinterpret_cast<void *>(a->workspace), as_stream(stream));
    }
    return attention_simt(p, as_stream(stream));
}

extern "C" int piton_b200_attention_allgather_f32(const piton_attention_args *a, const piton_allgather_args *g,
                                                  void *stream) {
    AttnParams p;
    int rc = attn_params(a, p);
    if (rc) return rc;
    PITON_REQUIRE(g != nullptr, "allgather args is NULL");
    PITON_REQUIRE(g->world >= 1 && g->world <= MAX_PEERS && g->rank >= 0 && g->rank < g->world,
                  "world %d / rank %d outside 1..%d", g->world, g->rank, MAX_PEERS);
    PITON_REQUIRE(g->row_offset >= 0, "bad first head %lld", (long long)g->row_offset);
    if (g->multicast_c)
        return set_error(PITON_B200_ENOTSUP, "the all-gather attention stores to peers only (no multicast output)");
    PITON_REQUIRE(a->stride_oh % 4 == 0 && a->stride_om % 4 == 0, "output strides must be multiples of 4 elements");
    for (int i = 0; i < g->world; ++i)
        PITON_REQUIRE(g->peer_c[i] != 0 && (g->peer_c[i] & 15) == 0, "peer output %d is NULL or misaligned", i);
    if (p.row_end <= 0 || p.heads == 0) return PITON_B200_OK;
    PITON_REQUIRE(p.heads < 65536, "too many heads for one launch");
    PITON_REQUIRE(a->q && a->k && a->v, "NULL pointer");
    if (!use_tc(a, p))
        return set_error(PITON_B200_ENOTSUP, "the all-gather attention runs on the tensor-core path only "
                                             "(HEAD_DIM 64, n_ctx >= 64)");
    size_t need = attention_tc_workspace_bytes(p);
    if (a->workspace_bytes < need || !a->workspace)
        return set_error(PITON_B200_EWORKSPACE, "attention needs %zu bytes of workspace, got %llu", need,
                         (unsigned long long)a->workspace_bytes);
    p.world = g->world;
    p.rank = g->rank;
    for (int i = 0; i < g->world; ++i) p.peer_o[i] = reinterpret_cast<float *>(g->peer_c[i]) + g->row_offset * a->stride_oh;
    p.o = p.peer_o[g->rank];
    return attention_tc(p, reinterpret_cast<void *>(a->workspace), as_stream(stream));
}
