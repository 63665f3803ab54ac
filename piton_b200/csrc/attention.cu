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
#include <climits>

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

// ---- QPU rounding mode: attn_fwd_kernel on the QPU float model, bit for bit -----------------
//
// The reference program per query row (examples/attention.py:37-113 as lowered by
// piton/backend/lower.py): qk_scale = sm_scale * 1.44269504 (a QPU multiply); per key block of
// BLOCK_N keys: each score a sequential-d dot (QPU multiply, then add), times qk_scale, -inf
// where masked; the block maximum an fmax fold over the keys in order; m_ij = fmax(m_i, max);
// p = exp2(s - m_ij), alpha = exp2(m_i - m_ij) with the ALU exp; l_i = l_i alpha + the 16-lane
// sum of p (lanes accumulate in order, then the rotate-and-add butterfly); acc[t] = acc[t]
// alpha, then + p_j v[j][t] over the keys in order; the row's output acc / l_i with the Newton
// reciprocal.  Causal launches walk keys [0, lo) unmasked and [lo, hi) with the causal mask
// (lo = the query block's first row rounded down to BLOCK_N, hi = its end); non-causal ones
// [0, N_CTX rounded down to BLOCK_N) unmasked, then the ragged tail with the key mask unless
// EVEN_N.  A warp per query row: lane j holds key j (+ 32 c) of a block, lane t dimension t
// (+ 32 u) of the accumulator.
struct QpuAttnArgs {
    const float *q, *k, *v;
    float *o;
    int64_t sqh, sqm, skh, skn, skk, svh, svn, soh, som;
    int64_t n_ctx, bm, bn, row_end;
    float sm_scale;
    int causal, even_n;
};

constexpr int QA_WARPS = 8, QA_MAXC = 4;   // rows per CTA; BLOCK_N up to 128 (4 keys per lane)

template <int D>
__global__ void __launch_bounds__(QA_WARPS * 32) attn_qpu_kernel(QpuAttnArgs a) {
    __shared__ float qs[QA_WARPS][D];
    constexpr int DU = (D + 31) / 32;   // accumulator dimensions per lane
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * QA_WARPS + warp, h = blockIdx.y;
    if (row >= a.row_end) return;   // whole warps only: no block barrier below
    const float *q = a.q + h * a.sqh + row * a.sqm, *kh = a.k + h * a.skh, *vh = a.v + h * a.svh;
    for (int t = lane; t < D; t += 32) qs[warp][t] = q[t];
    __syncwarp();
    const float qk_scale = qpu_fmul(a.sm_scale, __uint_as_float(0x3fb8aa3bu));
    float m_i = -INFINITY, l_i = 0.0f, acc[DU];
#pragma unroll
    for (int u = 0; u < DU; ++u) acc[u] = 0.0f;
    const int bn = (int)a.bn;
    const int nc = (bn + 31) / 32;   // keys per lane
    auto run = [&](int64_t lo, int64_t hi, bool mask_keys, bool causal_mask) {
        for (int64_t start = lo; start < hi; start += bn) {
            float s[QA_MAXC];
#pragma unroll
            for (int c = 0; c < QA_MAXC; ++c) {
                const int j = lane + 32 * c;
                float v = -INFINITY;
                if (c < nc && j < bn) {
                    const int64_t col = start + j;
                    const bool in = col < a.n_ctx;
                    float dot = 0.0f;
                    for (int t = 0; t < D; ++t)
                        dot = qpu_fadd(dot, qpu_fmul(qs[warp][t], in ? kh[col * a.skn + t * a.skk] : 0.0f));
                    v = qpu_fmul(dot, qk_scale);
                    if (mask_keys && !in) v = -INFINITY;
                    if (causal_mask && !(row >= col)) v = -INFINITY;
                }
                s[c] = v;
            }
            // block maximum: the fold keeps the last of the keys with the largest key word
            long long key = LLONG_MIN;
            int idx = -1;
#pragma unroll
            for (int c = 0; c < QA_MAXC; ++c) {
                const int j = lane + 32 * c;
                if (c < nc && j < bn) {
                    const long long kj = qpu_fkey(s[c]);
                    if (kj >= key) {
                        key = kj;
                        idx = j;
                    }
                }
            }
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) {
                const long long ok = __shfl_xor_sync(0xffffffffu, key, o);
                const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
                if (ok > key || (ok == key && oi > idx)) {
                    key = ok;
                    idx = oi;
                }
            }
            float mx = -INFINITY;
#pragma unroll
            for (int c = 0; c < QA_MAXC; ++c) {
                const float sv = __shfl_sync(0xffffffffu, s[c], idx & 31);
                if (idx >> 5 == c) mx = sv;
            }
            const float m_ij = qpu_fmax(m_i, mx);
#pragma unroll
            for (int c = 0; c < QA_MAXC; ++c) s[c] = qpu_exp(qpu_fsub(s[c], m_ij), true);   // p
            const float alpha = qpu_exp(qpu_fsub(m_i, m_ij), true);
            // 16-lane sum of p: lane l (< 16) adds p[l + 16 r] for r = 0, 1, ... in order
            float ls = 0.0f;
            for (int r = 0; 16 * r < bn; ++r) {
                const int j = (lane & 15) + 16 * r;   // p[j] sits in lane j % 32, slot j / 32
                float pj = 0.0f;
#pragma unroll
                for (int c = 0; c < QA_MAXC; ++c) {
                    const float x = __shfl_sync(0xffffffffu, s[c], j & 31);
                    if (j >> 5 == c) pj = x;
                }
                if (j < bn) ls = r == 0 ? pj : qpu_fadd(ls, pj);
            }
#pragma unroll
            for (int sft = 8; sft >= 1; sft >>= 1) ls = qpu_fadd(ls, __shfl_sync(0xffffffffu, ls, ((lane & 15) - sft) & 15, 16));
            const float psum = __shfl_sync(0xffffffffu, ls, 0);
            l_i = qpu_fadd(qpu_fmul(l_i, alpha), psum);
#pragma unroll
            for (int u = 0; u < DU; ++u) acc[u] = qpu_fmul(acc[u], alpha);
            for (int j = 0; j < bn; ++j) {
                float pj = 0.0f;
#pragma unroll
                for (int c = 0; c < QA_MAXC; ++c) {
                    const float x = __shfl_sync(0xffffffffu, s[c], j & 31);
                    if (j >> 5 == c) pj = x;
                }
                const int64_t col = start + j;
                const bool in = col < a.n_ctx;
#pragma unroll
                for (int u = 0; u < DU; ++u) {
                    const int t = lane + 32 * u;
                    if (t < D) acc[u] = qpu_fadd(acc[u], qpu_fmul(pj, in ? vh[col * a.svn + t] : 0.0f));
                }
            }
            m_i = m_ij;
        }
    };
    if (a.causal) {
        const int64_t sm = row / a.bm;
        const int64_t lo = (sm * a.bm) / bn * bn;
        const int64_t hi = (sm + 1) * a.bm < a.n_ctx ? (sm + 1) * a.bm : a.n_ctx;
        run(0, lo, false, false);
        run(lo, hi, !a.even_n, true);
    } else {
        const int64_t n_full = a.n_ctx / bn * bn;
        run(0, n_full, false, false);
        if (!a.even_n) run(n_full, a.n_ctx, true, false);
    }
    float *o = a.o + h * a.soh + row * a.som;
#pragma unroll
    for (int u = 0; u < DU; ++u) {
        const int t = lane + 32 * u;
        if (t < D) o[t] = qpu_fdiv(acc[u], l_i);
    }
}

template <int D>
static int launch_attn_qpu(const QpuAttnArgs &a, int64_t heads, cudaStream_t s) {
    dim3 grid((unsigned)cdiv(a.row_end, (int64_t)QA_WARPS), (unsigned)heads);
    attn_qpu_kernel<D><<<grid, QA_WARPS * 32, 0, s>>>(a);
    return check_launch("attention_qpu");
}

int attention_qpu(const QpuAttnArgs &a, int64_t head_dim, int64_t heads, cudaStream_t s) {
    switch (head_dim) {
        case 16: return launch_attn_qpu<16>(a, heads, s);
        case 32: return launch_attn_qpu<32>(a, heads, s);
        case 64: return launch_attn_qpu<64>(a, heads, s);
        case 128: return launch_attn_qpu<128>(a, heads, s);
        default: return set_error(PITON_B200_ENOTSUP, "HEAD_DIM %lld: supported 16, 32, 64, 128", (long long)head_dim);
    }
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
    PITON_REQUIRE((a->flags & ~(PITON_B200_FORCE_SIMT | PITON_B200_QPU_ROUNDING)) == 0, "unknown flags 0x%x",
                  a->flags);
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
    return !(a->flags & (PITON_B200_FORCE_SIMT | PITON_B200_QPU_ROUNDING)) && p.row_end > 0 && p.heads > 0 &&
           attention_tc_supported(p);
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
    if (a->flags & PITON_B200_QPU_ROUNDING) {
        QpuAttnArgs q;
        q.q = p.q; q.k = p.k; q.v = p.v; q.o = p.o;
        q.sqh = p.sqh; q.sqm = p.sqm; q.skh = p.skh; q.skn = p.skn; q.skk = p.skk;
        q.svh = p.svh; q.svn = p.svn; q.soh = p.soh; q.som = p.som;
        q.n_ctx = p.n_ctx; q.bm = a->block_m; q.bn = a->block_n; q.row_end = p.row_end;
        q.sm_scale = (float)a->sm_scale;
        q.causal = a->causal != 0;
        q.even_n = a->even_n != 0;
        PITON_REQUIRE(a->block_n <= 32 * QA_MAXC, "QPU rounding: BLOCK_N up to %d", 32 * QA_MAXC);
        return attention_qpu(q, p.head_dim, p.heads, as_stream(stream));
    }
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
    if (a->flags & PITON_B200_QPU_ROUNDING)
        return set_error(PITON_B200_ENOTSUP, "the all-gather attention has no QPU rounding mode");
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
