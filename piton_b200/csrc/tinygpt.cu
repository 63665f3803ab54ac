// TinyGPT greedy decoding (no counterpart in the reference, which has the pieces
// but not the model): character-level decoder, vocab 65, d_model 128, 4
// pre-LayerNorm blocks of 4-head causal attention (head dim 32) and a 4x GELU
// MLP, learned positions, tied input/output embeddings, context 128.
//
// Step kernel (batches above the cluster kernel's): one launch per decode.  A CTA owns SEQ
// sequences and feeds their positions one after another; for each it runs every
// layer with the activations in shared memory, appends the token's keys and
// values to the caller's KV cache, attends over the cached positions (one warp
// per sequence x head), and writes the greedy next token (argmax of the 65
// tied-embedding logits, first maximum) into the token buffer, which its next
// position reads: no CTA waits on another and the generation needs no host
// round trips.  Weights (3.2 MB) stay L2-resident and are read through L1.
//
// Packed weight layout (fp32, row-major, input-by-output matrices):
//   wte[V,D] wpe[CTX,D]
//   per layer: ln1_g[D] ln1_b[D] w_qkv[D,3D] b_qkv[3D] w_o[D,D] b_o[D]
//              ln2_g[D] ln2_b[D] w_fc[D,4D] b_fc[4D] w_pr[4D,D] b_pr[D]
//   lnf_g[D] lnf_b[D]
// KV cache: fp32 [L][2][B][CTX][D] (keys, then values).
#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "common.cuh"

namespace piton {
namespace tg {

constexpr int V = 65, D = 128, L = 4, H = 4, HD = 32, F = 4 * D, CTX = 128;
constexpr int SEQ = 2, THREADS = 256;
constexpr int PRE_W = 2;   // weight quads per thread requested ahead of a linear layer (step kernel; 2 measured best of 1-16)
constexpr int LAYER_FLOATS = 2 * D + D * 3 * D + 3 * D + D * D + D + 2 * D + D * F + F + F * D + D;
// offsets of a layer's tensors in its packed block
constexpr int O_LN1 = 0, O_WQKV = 2 * D, O_BQKV = O_WQKV + D * 3 * D, O_WO = O_BQKV + 3 * D, O_BO = O_WO + D * D,
              O_LN2 = O_BO + D, O_WFC = O_LN2 + 2 * D, O_BFC = O_WFC + D * F, O_WPR = O_BFC + F,
              O_BPR = O_WPR + F * D;
static_assert(O_BPR + D == LAYER_FLOATS, "layer layout");
// a layer's gains and biases as the step kernel keeps them in shared memory
constexpr int P_LN1 = 0, P_BQKV = 2 * D, P_BO = P_BQKV + 3 * D, P_LN2 = P_BO + D, P_BFC = P_LN2 + 2 * D,
              P_BPR = P_BFC + F, P_LAYER = P_BPR + D;
constexpr int64_t TOTAL_FLOATS = (int64_t)V * D + (int64_t)CTX * D + (int64_t)L * LAYER_FLOATS + 2 * D;

struct StepArgs {
    const float *w;
    float *kv;
    int32_t *tokens;
    float *logits;
    int64_t batch;
    int steps;        // positions fed, 0 .. steps - 1, all in one launch
    int prompt_len;   // the next token is written when prompt_len - 1 <= pos and pos + 1 < end
    int end;          // prompt_len + new_tokens
};

// out[s][n] = act(sum_k in[s][k] W[k][n] + b[n]) for the CTA's SEQ rows.  A
// thread owns 4 adjacent columns (16-byte weight loads) of one k-group; the
// k range is split into G groups so that every thread has work, and the
// partial sums meet in `scratch` (SEQ * THREADS * 4 floats).  The k-loop is
// unrolled so that many 16-byte weight loads are in flight per thread: the
// weights come from L2 and this loop is latency-bound otherwise.  b is in
// shared memory.
//
// PRE > 0: the first PRE weight quads of the thread's k-range were requested earlier by
// linear_prefetch (before the phase that precedes this layer) and arrive in `pre`.
template <int K, int N> struct LinearTiling {
    static constexpr int NQ = N / 4;                              // column quads
    static constexpr int G = THREADS / NQ > 0 ? THREADS / NQ : 1;  // k-groups
    static constexpr int KG = K / G;
    static_assert(N % 4 == 0 && K % G == 0 && NQ * G <= THREADS && G >= 2, "linear tiling");
};

// The first PRE weight quads of this thread's k-range of linear<K, N>: the weights do not depend
// on the activations, so they are requested before the phase that precedes the layer (a
// LayerNorm, the attention) and their L2 latency runs under it instead of opening the layer.
template <int K, int N, int PRE>
__device__ __forceinline__ void linear_prefetch(const float *__restrict__ W, float4 (&pre)[PRE]) {
    using T = LinearTiling<K, N>;
    static_assert(PRE <= T::KG, "prefetch within the k-range");
    const int q = threadIdx.x % T::NQ, g = threadIdx.x / T::NQ;
    if (g < T::G) {
        const float4 *w4 = reinterpret_cast<const float4 *>(W) + q;
#pragma unroll
        for (int i = 0; i < PRE; ++i) pre[i] = __ldg(w4 + (int64_t)(g * T::KG + i) * T::NQ);
    }
}

template <int K, int N, bool GELU, int PRE = 0>
__device__ __forceinline__ void linear(const float *in, float *out, const float *__restrict__ W, const float *b,
                                       float *scratch, bool residual, const float4 (&pre)[PRE > 0 ? PRE : 1]) {
    constexpr int NQ = LinearTiling<K, N>::NQ, G = LinearTiling<K, N>::G, KG = LinearTiling<K, N>::KG;
    const int tid = threadIdx.x;
    const int q = tid % NQ, g = tid / NQ;
    float4 acc[SEQ];
#pragma unroll
    for (int s = 0; s < SEQ; ++s) acc[s] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (g < G) {
        const float4 *w4 = reinterpret_cast<const float4 *>(W) + q;
#pragma unroll
        for (int i = 0; i < PRE; ++i) {
            const float4 w = pre[i];
            const int k = g * KG + i;
#pragma unroll
            for (int s = 0; s < SEQ; ++s) {
                float xv = in[s * K + k];
                acc[s].x = fmaf(xv, w.x, acc[s].x);
                acc[s].y = fmaf(xv, w.y, acc[s].y);
                acc[s].z = fmaf(xv, w.z, acc[s].z);
                acc[s].w = fmaf(xv, w.w, acc[s].w);
            }
        }
#pragma unroll 32
        for (int k = g * KG + PRE; k < (g + 1) * KG; ++k) {
            float4 w = __ldg(w4 + (int64_t)k * NQ);
#pragma unroll
            for (int s = 0; s < SEQ; ++s) {
                float xv = in[s * K + k];
                acc[s].x = fmaf(xv, w.x, acc[s].x);
                acc[s].y = fmaf(xv, w.y, acc[s].y);
                acc[s].z = fmaf(xv, w.z, acc[s].z);
                acc[s].w = fmaf(xv, w.w, acc[s].w);
            }
        }
    }
    {
        float4 *sc4 = reinterpret_cast<float4 *>(scratch);
        if (g < G) {
#pragma unroll
            for (int s = 0; s < SEQ; ++s) sc4[s * THREADS + g * NQ + q] = acc[s];
        }
        __syncthreads();
    }
    for (int i = tid; i < SEQ * NQ; i += THREADS) {
        const int s = i / NQ, qq = i % NQ;
        const float4 *sc4 = reinterpret_cast<const float4 *>(scratch);
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int gg = 0; gg < G; ++gg) {
            float4 p = sc4[s * THREADS + gg * NQ + qq];
            v.x += p.x; v.y += p.y; v.z += p.z; v.w += p.w;
        }
        float4 bb = reinterpret_cast<const float4 *>(b)[qq];   // shared memory
        float r[4] = {v.x + bb.x, v.y + bb.y, v.z + bb.z, v.w + bb.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (GELU) r[j] = 0.5f * r[j] * (1.0f + erff(r[j] * 0.70710678118654752f));
            const int n = 4 * qq + j;
            out[s * N + n] = residual ? out[s * N + n] + r[j] : r[j];
        }
    }
    __syncthreads();
}

// y[s] = LayerNorm(x[s]) * g + b, one warp per sequence (biased variance, eps 1e-5); g and b in
// shared memory.
__device__ __forceinline__ void layernorm(const float *x, float *y, const float *g, const float *b) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp < SEQ) {
        const float *xs = x + warp * D;
        float v[D / 32], sum = 0.0f;
#pragma unroll
        for (int i = 0; i < D / 32; ++i) {
            v[i] = xs[lane + 32 * i];
            sum += v[i];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        float mean = sum * (1.0f / D), q = 0.0f;
#pragma unroll
        for (int i = 0; i < D / 32; ++i) {
            v[i] -= mean;
            q += v[i] * v[i];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
        float r = rsqrtf(q * (1.0f / D) + 1e-5f);
#pragma unroll
        for (int i = 0; i < D / 32; ++i) {
            int c = lane + 32 * i;
            y[warp * D + c] = v[i] * r * g[c] + b[c];
        }
    }
    __syncthreads();
}

__global__ void __launch_bounds__(THREADS, 1) tinygpt_step_kernel(StepArgs a) {
    __shared__ __align__(16) float x[SEQ * D], h[SEQ * D], qkv[SEQ * 3 * D], att[SEQ * D], f[SEQ * F];
    __shared__ __align__(16) float scratch[SEQ * THREADS * 4];
    // the attention's probabilities share the linear layers' split-k scratch (never live together)
    static_assert(SEQ * H * CTX <= SEQ * THREADS * 4, "probabilities fit the scratch");
    float (*probs)[CTX] = reinterpret_cast<float (*)[CTX]>(scratch);
    __shared__ float lg[SEQ][V + 3];
    __shared__ __align__(16) float prm[L * P_LAYER + 2 * D];   // every layer's gains and biases, lnf
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t b0 = (int64_t)blockIdx.x * SEQ;
    const float *wte = a.w, *wpe = a.w + V * D;

    // the gains and biases of all layers into shared memory, requested together with the
    // embeddings below (one L2 round trip instead of one per LayerNorm and linear layer)
    {
        const float *lw0 = a.w + V * D + CTX * D;
        for (int i = tid; i < (L * P_LAYER + 2 * D) / 4; i += THREADS) {
            const int l = (4 * i) / P_LAYER, q = 4 * i - l * P_LAYER;
            const float *lw = lw0 + (int64_t)l * LAYER_FLOATS;
            const float *src = l == L                ? lw + q                      // lnf_g, lnf_b
                               : q < P_BQKV          ? lw + O_LN1 + q
                               : q < P_BO            ? lw + O_BQKV + (q - P_BQKV)
                               : q < P_BFC           ? lw + O_BO + (q - P_BO)      // b_o, ln2_g, ln2_b
                               : q < P_BPR           ? lw + O_BFC + (q - P_BFC)
                                                     : lw + O_BPR + (q - P_BPR);
            *reinterpret_cast<float4 *>(prm + 4 * i) = __ldg(reinterpret_cast<const float4 *>(src));
        }
    }

    // one position after another; the CTA's sequences depend on no other CTA, so the whole
    // decode is one launch (the gains and biases above are loaded once)
    for (int pos = 0; pos < a.steps; ++pos) {
        // token + position embedding
        for (int i = tid; i < SEQ * D; i += THREADS) {
            int s = i / D, c = i % D;
            int64_t b = b0 + s;
            float v = 0.0f;
            if (b < a.batch) {
                int tok = a.tokens[b * CTX + pos];
                tok = tok < 0 ? 0 : (tok >= V ? V - 1 : tok);
                v = __ldg(wte + tok * D + c) + __ldg(wpe + pos * D + c);
            }
            x[i] = v;
        }
        __syncthreads();

        const float *lw = a.w + V * D + CTX * D;
        for (int l = 0; l < L; ++l, lw += LAYER_FLOATS) {
            const float *pl = prm + l * P_LAYER;
            const float *ln1_g = pl + P_LN1, *ln1_b = ln1_g + D, *b_qkv = pl + P_BQKV, *b_o = pl + P_BO;
            const float *ln2_g = pl + P_LN2, *ln2_b = ln2_g + D, *b_fc = pl + P_BFC, *b_pr = pl + P_BPR;
            const float *w_qkv = lw + O_WQKV, *w_o = lw + O_WO, *w_fc = lw + O_WFC, *w_pr = lw + O_WPR;
            float *kc = a.kv + ((int64_t)l * 2 + 0) * a.batch * CTX * D;
            float *vc = a.kv + ((int64_t)l * 2 + 1) * a.batch * CTX * D;

            float4 pre_qkv[PRE_W], pre_o[PRE_W], pre_fc[PRE_W], no_pre[1];
            linear_prefetch<D, 3 * D>(w_qkv, pre_qkv);
            layernorm(x, h, ln1_g, ln1_b);
            linear<D, 3 * D, false, PRE_W>(h, qkv, w_qkv, b_qkv, scratch, false, pre_qkv);
            linear_prefetch<D, D>(w_o, pre_o);   // under the key / value append and the attention
            // append this position's keys and values
            for (int i = tid; i < SEQ * D; i += THREADS) {
                int s = i / D, c = i % D;
                int64_t b = b0 + s;
                if (b < a.batch) {
                    kc[(b * CTX + pos) * D + c] = qkv[s * 3 * D + D + c];
                    vc[(b * CTX + pos) * D + c] = qkv[s * 3 * D + 2 * D + c];
                }
            }
            __syncthreads();
            // causal attention over positions 0..pos: warp = (sequence, head)
            {
                const int s = warp / H, hh = warp % H;
                const int64_t b = b0 + s;
                if (b < a.batch) {
                    const float *q = qkv + s * 3 * D + hh * HD;
                    const float scale = 0.17677669529663688f;   // 1 / sqrt(32)
                    float sc[CTX / 32];
                    float mx = -INFINITY;
    #pragma unroll
                    for (int j = 0; j < CTX / 32; ++j) {
                        int t = lane + 32 * j;
                        float dot = -INFINITY;
                        if (t <= pos) {
                            const float *kr = kc + (b * CTX + t) * D + hh * HD;
                            float acc = 0.0f;
    #pragma unroll
                            for (int d = 0; d < HD; d += 4) {
                                float4 k4 = *reinterpret_cast<const float4 *>(kr + d);
                                acc = fmaf(q[d], k4.x, acc);
                                acc = fmaf(q[d + 1], k4.y, acc);
                                acc = fmaf(q[d + 2], k4.z, acc);
                                acc = fmaf(q[d + 3], k4.w, acc);
                            }
                            dot = acc * scale;
                        }
                        sc[j] = dot;
                        mx = fmaxf(mx, dot);
                    }
    #pragma unroll
                    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                    float sum = 0.0f;
    #pragma unroll
                    for (int j = 0; j < CTX / 32; ++j) {
                        int t = lane + 32 * j;
                        float p = t <= pos ? expf(sc[j] - mx) : 0.0f;
                        probs[warp][t] = p;
                        sum += p;
                    }
    #pragma unroll
                    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
                    __syncwarp();
                    float o_acc = 0.0f;
                    for (int t = 0; t <= pos; ++t) o_acc = fmaf(probs[warp][t], vc[(b * CTX + t) * D + hh * HD + lane], o_acc);
                    att[s * D + hh * HD + lane] = o_acc / sum;
                } else {
                    att[s * D + hh * HD + lane] = 0.0f;
                }
            }
            __syncthreads();
            linear<D, D, false, PRE_W>(att, x, w_o, b_o, scratch, true, pre_o);          // x += attn @ Wo + bo
            linear_prefetch<D, F>(w_fc, pre_fc);
            layernorm(x, h, ln2_g, ln2_b);
            linear<D, F, true, PRE_W>(h, f, w_fc, b_fc, scratch, false, pre_fc);         // f = gelu(h @ Wfc + bfc)
            linear<F, D, false>(f, x, w_pr, b_pr, scratch, true, no_pre);   // x += f @ Wpr + bpr
        }
        const float *lnf_g = prm + L * P_LAYER, *lnf_b = lnf_g + D;
        layernorm(x, h, lnf_g, lnf_b);
        // tied head: logits[s][v] = h[s] . wte[v]; a warp per (s, v) pair, lanes over D, the
        // pairs' embedding rows requested together (one L2 round trip for all of a warp's pairs)
        {
            constexpr int PV = (SEQ * V + THREADS / 32 - 1) / (THREADS / 32);   // pairs per warp
            float ew[PV][D / 32];
    #pragma unroll
            for (int i = 0; i < PV; ++i) {
                const int pv = warp + i * (THREADS / 32);
                const int vv = pv < SEQ * V ? pv % V : 0;
    #pragma unroll
                for (int c = 0; c < D / 32; ++c) ew[i][c] = __ldg(wte + vv * D + lane + 32 * c);
            }
    #pragma unroll
            for (int i = 0; i < PV; ++i) {
                const int pv = warp + i * (THREADS / 32);
                if (pv < SEQ * V) {
                    const int s = pv / V, vv = pv % V;
                    float acc = 0.0f;
    #pragma unroll
                    for (int c = 0; c < D / 32; ++c) acc = fmaf(h[s * D + lane + 32 * c], ew[i][c], acc);
    #pragma unroll
                    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
                    if (lane == 0) lg[s][vv] = acc;
                }
            }
        }
        __syncthreads();
        // greedy token: warp s takes sequence s's argmax, lanes over the vocabulary, first maximum
        // on ties (as numpy.argmax)
        if (warp < SEQ && pos + 1 >= a.prompt_len && pos + 1 < a.end) {
            const int64_t b = b0 + warp;
            if (b < a.batch) {
                float bv = -INFINITY;
                int bi = V;
                for (int vv = lane; vv < V; vv += 32)   // each lane's entries in increasing order
                    if (bi == V || lg[warp][vv] > bv) {
                        bv = lg[warp][vv];
                        bi = vv;
                    }
    #pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                    if (ov > bv || (ov == bv && oi < bi)) {
                        bv = ov;
                        bi = oi;
                    }
                }
                if (lane == 0) a.tokens[b * CTX + pos + 1] = bi;
            }
        }
        if (a.logits && pos == a.steps - 1) {
            for (int i = tid; i < SEQ * V; i += THREADS) {
                int s = i / V, vv = i % V;
                int64_t b = b0 + s;
                if (b < a.batch) a.logits[b * V + vv] = lg[s][vv];
            }
        }
        __syncthreads();   // the next token and the KV-cache rows written, shared buffers free
    }
}

// ---------------------------------------------------------------------------
// Small batches: one thread-block cluster of CS = 16 CTAs per sequence, one
// launch per decode.  The weights (3.2 MB) are split by output column across
// the 16 CTAs and held in their shared memory for the whole decode (each CTA
// keeps its 1/16 of every matrix, ~195 KB); every CTA keeps a full copy of the
// residual stream.  Per linear layer each CTA computes its slice of the outputs
// (a warp per output column, lanes over k) and stores it into all 16 CTAs'
// shared memory (st.shared::cluster), then the cluster barrier makes the whole
// vector visible everywhere: five exchanges per layer plus one for the logits.
// Attention head h runs in CTA h.  Every CTA computes the same greedy argmax,
// so all of them feed the same next token.
// ---------------------------------------------------------------------------

constexpr int CS = 16;                           // CTAs per cluster (non-portable size)
constexpr int QKV_C = 3 * D / CS;                // q/k/v columns per CTA (24)
constexpr int V_C = (V + CS - 1) / CS;           // vocabulary rows per CTA (5)
// The MLP's hidden units are split unevenly: CTAs 0..H-1 also run an attention head and
// hold that head's 32 rows of W_o, so they take FC_SMALL hidden units, the others FC_BIG.
constexpr int FC_SMALL = 8, FC_BIG = (F - H * FC_SMALL) / (CS - H);   // 8 and 40
static_assert(H * FC_SMALL + (CS - H) * FC_BIG == F, "hidden-unit split");
__host__ __device__ constexpr int fc_count(int r) { return r < H ? FC_SMALL : FC_BIG; }
__host__ __device__ constexpr int fc_first(int r) { return r < H ? r * FC_SMALL : H * FC_SMALL + (r - H) * FC_BIG; }
// per-layer weight floats of one CTA: W_qkv columns (column-major), then for head CTAs the
// head's W_o rows, then W_fc columns (column-major) and the matching W_pr rows
constexpr int W_QKV = QKV_C * D, W_OH = HD * D, W_TE = V_C * D;
__host__ __device__ constexpr int layer_floats(int r) { return W_QKV + (r < H ? W_OH : 0) + 2 * fc_count(r) * D; }
constexpr int W_LAYER_MAX = W_QKV + 2 * FC_BIG * D;                  // the larger of the two kinds
static_assert(W_LAYER_MAX >= W_QKV + W_OH + 2 * FC_SMALL * D, "layer slice bound");
constexpr int ACT = D /*x*/ + D /*h*/ + 3 * D /*qkv*/ + FC_BIG /*f*/ + H * D /*o partials*/ + CS * D /*pr partials*/ +
                    CS * V_C /*logits*/ + 2 * 256 + 16 /*reductions*/;
constexpr size_t CLUSTER_SMEM = (size_t)(L * W_LAYER_MAX + W_TE + ACT) * 4;

struct ClusterArgs {
    const float *w;
    float *kv;
    int32_t *tokens;
    float *logits;
    int64_t batch;
    int prompt_len, end, steps;
};

__device__ __forceinline__ uint32_t cl_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cl_id() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cl_count() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cl_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// v into the same shared-memory slot in CTA `rank` of the cluster
__device__ __forceinline__ void st_cluster(float *local, uint32_t rank, float v) {
    uint32_t a = (uint32_t)__cvta_generic_to_shared(local), r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(r), "f"(v) : "memory");
}

// This CTA's nc output columns [c0, c0 + nc) of in . W + b, W held column-major as ws[j][k];
// a warp per column, lanes over k.  Each value goes to out[c0 + j] in all CS CTAs.
template <int K>
__device__ __forceinline__ void slice_linear_bcast(const float *in, const float *ws, const float *__restrict__ b, int c0,
                                                   int nc, float *out) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int j = warp; j < nc; j += THREADS / 32) {
        const float *wc = ws + j * K;
        float acc = 0.0f;
#pragma unroll 4
        for (int k = lane; k < K; k += 32) acc = fmaf(in[k], wc[k], acc);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        const float v = acc + __ldg(b + c0 + j);
        if (lane < CS) st_cluster(out + c0 + j, lane, v);
    }
}

// out[n] = sum_i in[i] * wr[i][n] for n < D (wr: `rows` rows of D), sent to slot[n] of all CS CTAs
__device__ __forceinline__ void rows_partial_bcast(const float *in, const float *wr, int rows, float *slot) {
    for (int n = threadIdx.x; n < D; n += THREADS) {
        float acc = 0.0f;
        for (int i = 0; i < rows; ++i) acc = fmaf(in[i], wr[i * D + n], acc);
        for (uint32_t r = 0; r < CS; ++r) st_cluster(slot + n, r, acc);
    }
}

// LayerNorm of x (D) into y by warp 0, then the CTA syncs
__device__ __forceinline__ void ln_cta(const float *x, float *y, const float *__restrict__ g,
                                       const float *__restrict__ b) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp == 0) {
        float v[D / 32], sum = 0.0f;
#pragma unroll
        for (int i = 0; i < D / 32; ++i) {
            v[i] = x[lane + 32 * i];
            sum += v[i];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        const float mean = sum * (1.0f / D);
        float q = 0.0f;
#pragma unroll
        for (int i = 0; i < D / 32; ++i) {
            v[i] -= mean;
            q += v[i] * v[i];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
        const float r = rsqrtf(q * (1.0f / D) + 1e-5f);
#pragma unroll
        for (int i = 0; i < D / 32; ++i) {
            const int c = lane + 32 * i;
            y[c] = v[i] * r * __ldg(g + c) + __ldg(b + c);
        }
    }
    __syncthreads();
}

// Per layer, three cluster exchanges:
//  1. q/k/v: each CTA's 24 columns to every CTA;
//  2. attention head h in CTA h, which also multiplies its 32 outputs by the head's rows of
//     W_o: the four 128-wide partial products go to every CTA, which adds them to x;
//  3. each CTA's hidden units of the MLP (GELU) times the matching rows of W_pr: sixteen
//     128-wide partial products, added to x everywhere.
__global__ void __launch_bounds__(THREADS, 1) tinygpt_cluster_kernel(ClusterArgs a) {
    extern __shared__ __align__(16) float sm[];
    const uint32_t rank = cl_rank();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nfc = fc_count((int)rank), fc0 = fc_first((int)rank);
    const int lfl = layer_floats((int)rank);
    float *wl = sm;                                  // [L][lfl]
    float *wte_s = wl + L * W_LAYER_MAX;             // [V_C][D]
    float *x = wte_s + W_TE, *h = x + D, *qkv = h + D, *fl = qkv + 3 * D, *opart = fl + FC_BIG;
    float *prpart = opart + H * D, *lg = prpart + CS * D, *red = lg + CS * V_C;   // red: 2 x 256 + 16
    const float *wte = a.w, *wpe = a.w + V * D;
    const float *lw0 = a.w + V * D + CTX * D;

    // this CTA's weight slices, once per decode
    for (int l = 0; l < L; ++l) {
        const float *lw = lw0 + (int64_t)l * LAYER_FLOATS;
        const float *w_qkv = lw + 2 * D, *w_o = w_qkv + D * 3 * D + 3 * D, *w_fc = w_o + D * D + D + 2 * D;
        const float *w_pr = w_fc + D * F + F;
        float *s_qkv = wl + l * lfl, *s_oh = s_qkv + W_QKV, *s_fc = s_oh + (rank < H ? W_OH : 0);
        float *s_pr = s_fc + nfc * D;
        for (int i = tid; i < W_QKV; i += THREADS) s_qkv[i] = __ldg(w_qkv + (i % D) * 3 * D + rank * QKV_C + i / D);
        if (rank < H)
            for (int i = tid; i < W_OH; i += THREADS) s_oh[i] = __ldg(w_o + (rank * HD + i / D) * D + i % D);
        for (int i = tid; i < nfc * D; i += THREADS) {
            s_fc[i] = __ldg(w_fc + (i % D) * F + fc0 + i / D);     // column-major [j][k]
            s_pr[i] = __ldg(w_pr + (fc0 + i / D) * D + i % D);      // rows [j][n]
        }
    }
    for (int i = tid; i < W_TE; i += THREADS) {
        const int v = (int)rank * V_C + i / D;
        wte_s[i] = v < V ? __ldg(wte + v * D + i % D) : 0.0f;
    }
    __syncthreads();
    cl_sync();   // every CTA of the cluster is running before any stores into its shared memory

    for (int64_t b = cl_id(); b < a.batch; b += cl_count()) {
        int tok = a.tokens[b * CTX];
        for (int pos = 0; pos < a.steps; ++pos) {
            if (pos < a.prompt_len) tok = a.tokens[b * CTX + pos];
            tok = tok < 0 ? 0 : (tok >= V ? V - 1 : tok);
            for (int c = tid; c < D; c += THREADS) x[c] = __ldg(wte + tok * D + c) + __ldg(wpe + pos * D + c);
            __syncthreads();
            for (int l = 0; l < L; ++l) {
                const float *lw = lw0 + (int64_t)l * LAYER_FLOATS;
                const float *ln1_g = lw, *ln1_b = ln1_g + D, *b_qkv = ln1_b + D + D * 3 * D;
                const float *b_o = b_qkv + 3 * D + D * D, *ln2_g = b_o + D, *ln2_b = ln2_g + D;
                const float *b_fc = ln2_b + D + D * F, *b_pr = b_fc + F + F * D;
                const float *s_qkv = wl + l * lfl, *s_oh = s_qkv + W_QKV, *s_fc = s_oh + (rank < H ? W_OH : 0);
                const float *s_pr = s_fc + nfc * D;
                float *kc = a.kv + ((int64_t)l * 2 + 0) * a.batch * CTX * D;
                float *vc = a.kv + ((int64_t)l * 2 + 1) * a.batch * CTX * D;

                // 1. q, k, v
                ln_cta(x, h, ln1_g, ln1_b);
                slice_linear_bcast<D>(h, s_qkv, b_qkv, rank * QKV_C, QKV_C, qkv);
                cl_sync();
                // 2. attention head `rank` over positions 0..pos, then its share of the output projection
                if (rank < H) {
                    const int hh = rank;
                    float *kr_base = kc + (b * CTX) * D + hh * HD, *vr_base = vc + (b * CTX) * D + hh * HD;
                    if (tid < HD) {
                        kr_base[pos * D + tid] = qkv[D + hh * HD + tid];
                        vr_base[pos * D + tid] = qkv[2 * D + hh * HD + tid];
                    }
                    __syncthreads();
                    const float scale = 0.17677669529663688f;   // 1 / sqrt(32)
                    float sc = -INFINITY;
                    if (tid <= pos) {
                        const float *kr = kr_base + tid * D;
                        float acc = 0.0f;
#pragma unroll
                        for (int d = 0; d < HD; d += 4) {
                            const float4 k4 = *reinterpret_cast<const float4 *>(kr + d);
                            acc = fmaf(qkv[hh * HD + d], k4.x, acc);
                            acc = fmaf(qkv[hh * HD + d + 1], k4.y, acc);
                            acc = fmaf(qkv[hh * HD + d + 2], k4.z, acc);
                            acc = fmaf(qkv[hh * HD + d + 3], k4.w, acc);
                        }
                        sc = acc * scale;
                    }
                    float m = sc;
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
                    if (lane == 0) red[512 + warp] = m;
                    __syncthreads();
                    m = red[512];
                    for (int w2 = 1; w2 < THREADS / 32; ++w2) m = fmaxf(m, red[512 + w2]);
                    const float p = tid <= pos ? expf(sc - m) : 0.0f;
                    float ssum = p;
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) ssum += __shfl_xor_sync(0xffffffffu, ssum, o);
                    red[tid] = p;
                    __syncthreads();
                    if (lane == 0) red[512 + 8 + warp] = ssum;
                    // output dimension d = tid % 32 over positions t = tid / 32, tid / 32 + 8, ...
                    // (unrolled over the whole context so the value loads are issued together)
                    const int d = tid & 31, tg0 = tid >> 5;
                    float o_acc = 0.0f;
#pragma unroll
                    for (int i = 0; i < CTX / (THREADS / 32); ++i) {
                        const int t = tg0 + i * (THREADS / 32);
                        if (t <= pos) o_acc = fmaf(red[t], vr_base[t * D + d], o_acc);
                    }
                    red[256 + tid] = o_acc;
                    __syncthreads();
                    if (tid < HD) {
                        float tot = 0.0f;
                        for (int w2 = 0; w2 < THREADS / 32; ++w2) tot += red[512 + 8 + w2];
                        float v = 0.0f;
                        for (int g2 = 0; g2 < THREADS / 32; ++g2) v += red[256 + g2 * 32 + tid];
                        red[tid] = v / tot;   // this head's 32 attention outputs
                    }
                    __syncthreads();
                    rows_partial_bcast(red, s_oh, HD, opart + hh * D);
                }
                cl_sync();
                for (int c = tid; c < D; c += THREADS) {
                    float v = __ldg(b_o + c);
#pragma unroll
                    for (int hh = 0; hh < H; ++hh) v += opart[hh * D + c];
                    x[c] += v;
                }
                __syncthreads();
                // 3. this CTA's hidden units, then their share of the projection back to D
                ln_cta(x, h, ln2_g, ln2_b);
                for (int j = warp; j < nfc; j += THREADS / 32) {
                    const float *wc = s_fc + j * D;
                    float acc = 0.0f;
#pragma unroll 4
                    for (int k = lane; k < D; k += 32) acc = fmaf(h[k], wc[k], acc);
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
                    if (lane == 0) {
                        const float v = acc + __ldg(b_fc + fc0 + j);
                        fl[j] = 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
                    }
                }
                __syncthreads();
                rows_partial_bcast(fl, s_pr, nfc, prpart + rank * D);
                cl_sync();
                for (int c = tid; c < D; c += THREADS) {
                    float v = __ldg(b_pr + c);
#pragma unroll
                    for (int r = 0; r < CS; ++r) v += prpart[r * D + c];
                    x[c] += v;
                }
                __syncthreads();
            }
            const float *lnf = lw0 + (int64_t)L * LAYER_FLOATS;
            ln_cta(x, h, lnf, lnf + D);
            // tied head: this CTA's vocabulary rows, a warp per row
            for (int j = warp; j < V_C; j += THREADS / 32) {
                float acc = 0.0f;
#pragma unroll
                for (int k = lane; k < D; k += 32) acc = fmaf(h[k], wte_s[j * D + k], acc);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
                if (lane < CS) st_cluster(lg + rank * V_C + j, lane, acc);
            }
            cl_sync();
            int best = 0;
            for (int v = 1; v < V; ++v)
                if (lg[v] > lg[best]) best = v;     // first maximum, as numpy.argmax
            if (pos + 1 >= a.prompt_len && pos + 1 < a.end) {
                tok = best;
                if (rank == 0 && tid == 0) a.tokens[b * CTX + pos + 1] = best;
            }
            if (a.logits && pos == a.steps - 1 && rank == 0)
                for (int v = tid; v < V; v += THREADS) a.logits[b * V + v] = lg[v];
            __syncthreads();
        }
    }
    cl_sync();   // no CTA leaves while another may still store into its shared memory
}

// ---------------------------------------------------------------------------
// Larger batches: one cluster of H = 4 CTAs per group of up to GS sequences, one launch per
// decode.  CTA r of a cluster owns attention head r and hidden units [128 r, 128 r + 128) of
// the MLP.  Per layer it computes, for every sequence of its group, the head's 96 q, k and v
// columns of W_qkv (appending k and v to the KV cache), the head's causal attention, the
// head's share of the output projection (its 32 outputs times the head's 32 rows of W_o), its
// 128 GELU hidden units (W_fc columns) and their share of the MLP projection (the matching 128
// rows of W_pr).  The two 128-wide partial products per layer go to all four CTAs' shared
// memory (st.shared::cluster) and one cluster barrier each publishes them; every CTA adds the
// four partials in rank order, so all four keep the same residual stream without further
// exchange.  Each CTA reads a quarter of the weights per position (the step kernel's CTAs read
// all of them), and the whole decode is one launch with 9 cluster barriers per position.
//
// The decode is a chain of short dependent phases, so every global read is taken off it:
// each phase's weight slice (and its biases / LayerNorm parameters) is copied into one of two
// shared-memory buffers with cp.async while the previous phase computes; the CTA's vocabulary
// rows stay in shared memory for the whole decode; the attention issues all of a sequence's
// key and value loads at once (lanes over positions) and sums P.V with a reduce-scatter.
// ---------------------------------------------------------------------------

constexpr int HC = H;                 // CTAs per cluster, one per head (portable cluster size)
constexpr int GS = 8;                 // sequences per group at most
constexpr int HT = 512;               // threads per CTA (16 warps: latency hidden by more warps)
constexpr int SH = 2;                 // sequence halves of a group in the split-k linears
constexpr int KGRP = 8;               // k-groups of the split-k linears
constexpr int FH = F / HC;            // hidden units per CTA (128)
constexpr int V_R = (V + HC - 1) / HC;   // vocabulary rows per CTA (17)
constexpr int LG_LD = V + 3;
// weight-slice buffer: up to 128 x 128 floats plus the phase's small parameters
constexpr int WB_MAT = D * FH, WB_PAR = 2 * D + FH;   // 16384 + 384 floats
constexpr int WB = WB_MAT + WB_PAR;
// the four phases of a layer, in order
enum Phase { PH_QKV = 0, PH_O = 1, PH_FC = 2, PH_PR = 3 };

struct HeadsSmem {
    float wbuf[2][WB];                // weight slices, double-buffered
    float x[GS][D];                   // residual stream (the same in all four CTAs)
    float h[GS][D];                   // LayerNorm output
    float q[GS][HD];                  // this head's queries
    float att[GS][HD];                // this head's attention outputs
    float f[GS][FH];                  // this CTA's GELU hidden units
    float part[2][HC][GS][D];         // partial products from every CTA, two slots used in turn
    float red[KGRP][GS][D];           // split-k partial sums
    float lg[GS][LG_LD];              // logits, every CTA's vocabulary rows
    float wte_s[V_R][D];              // this CTA's vocabulary rows of the tied embedding
    float lnf[2 * D];                 // final LayerNorm gain and bias
    int tok[GS];
};

struct HeadsArgs {
    const float *w;
    float *kv;
    int32_t *tokens;
    float *logits;
    int64_t batch;
    int prompt_len, end, steps;
    int group;                        // sequences per group (1..GS)
};

__device__ __forceinline__ void st_cluster4(float *local, uint32_t rank, float4 v) {
    uint32_t a = (uint32_t)__cvta_generic_to_shared(local), r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(r), "f"(v.x), "f"(v.y), "f"(v.z),
                 "f"(v.w)
                 : "memory");
}

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
                 "l"(gmem)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Starts the copies of phase `ph` of layer `l` into buffer `buf` (one commit group per call):
//   QKV: the head's 96 columns of W_qkv [128 x 96], then ln1 gain, bias, the 96 q/k/v biases;
//   O:   the head's 32 rows of W_o [32 x 128], then b_o;
//   FC:  the CTA's 128 columns of W_fc [128 x 128], then ln2 gain, bias, the 128 biases;
//   PR:  the CTA's 128 rows of W_pr [128 x 128], then b_pr.
__device__ __forceinline__ void prefetch_phase(float *buf, const float *__restrict__ w, int l, int ph, int rank) {
    const float *lw = w + V * D + CTX * D + (int64_t)l * LAYER_FLOATS;
    const float *ln1_g = lw, *ln1_b = ln1_g + D, *w_qkv = ln1_b + D, *b_qkv = w_qkv + D * 3 * D;
    const float *w_o = b_qkv + 3 * D, *b_o = w_o + D * D, *ln2_g = b_o + D, *ln2_b = ln2_g + D;
    const float *w_fc = ln2_b + D, *b_fc = w_fc + D * F, *w_pr = b_fc + F, *b_pr = w_pr + F * D;
    float *par = buf + WB_MAT;
    const int tid = threadIdx.x;
    if (ph == PH_QKV) {
        for (int i = tid; i < D * 24; i += HT) {       // 24 quads per row: q, k, v sections of 8 quads
            const int k = i / 24, j = i % 24;
            cp_async16(buf + k * 96 + 4 * j, w_qkv + (int64_t)k * 3 * D + (j >> 3) * D + rank * HD + 4 * (j & 7));
        }
        for (int i = tid; i < 2 * D / 4 + 24; i += HT) {
            if (i < D / 4) cp_async16(par + 4 * i, ln1_g + 4 * i);
            else if (i < D / 2) cp_async16(par + 4 * i, ln1_b + 4 * (i - D / 4));
            else {
                const int j = i - D / 2;
                cp_async16(par + 2 * D + 4 * j, b_qkv + (j >> 3) * D + rank * HD + 4 * (j & 7));
            }
        }
    } else if (ph == PH_O) {
        for (int i = tid; i < HD * D / 4; i += HT) cp_async16(buf + 4 * i, w_o + (int64_t)rank * HD * D + 4 * i);
        for (int i = tid; i < D / 4; i += HT) cp_async16(par + 4 * i, b_o + 4 * i);
    } else if (ph == PH_FC) {
        for (int i = tid; i < D * FH / 4; i += HT) {
            const int k = i / (FH / 4), j = i % (FH / 4);
            cp_async16(buf + k * FH + 4 * j, w_fc + (int64_t)k * F + rank * FH + 4 * j);
        }
        for (int i = tid; i < (2 * D + FH) / 4; i += HT) {
            if (i < D / 4) cp_async16(par + 4 * i, ln2_g + 4 * i);
            else if (i < D / 2) cp_async16(par + 4 * i, ln2_b + 4 * (i - D / 4));
            else cp_async16(par + 4 * i, b_fc + rank * FH + 4 * (i - D / 2));
        }
    } else {
        for (int i = tid; i < FH * D / 4; i += HT) cp_async16(buf + 4 * i, w_pr + (int64_t)rank * FH * D + 4 * i);
        for (int i = tid; i < D / 4; i += HT) cp_async16(par + 4 * i, b_pr + 4 * i);
    }
    cp_async_commit();
}

// Split-k product of the group's rows in[s][0..K) (shared memory, row stride K) with the NQ quads
// of columns of a weight slice in shared memory (row-major, row stride 4 NQ).  Thread (j, g) sums
// k-group g for all GS rows; the KGRP partial sums meet in red, and epi(s, j, float4) receives each
// finished quad once.
template <int K, int NQ, typename Epi>
__device__ __forceinline__ void group_linear(const float *in, const float *ws, float (*red)[GS][D], Epi epi) {
    constexpr int KG = K / KGRP, GH = GS / SH;
    static_assert(K % KGRP == 0 && NQ * KGRP * SH <= HT && NQ * 4 <= D && GS % SH == 0, "group_linear tiling");
    const int tid = threadIdx.x;
    const int j = tid % NQ, g = (tid / NQ) % KGRP, sh = tid / (NQ * KGRP);
    static_assert(KG % 4 == 0, "k-groups of whole float4s");
    if (sh < SH) {
        // thread (j, g, sh): column quad j, k-group g, rows [GH sh, GH sh + GH)
        float4 acc[GH];
#pragma unroll
        for (int s = 0; s < GH; ++s) acc[s] = make_float4(0.f, 0.f, 0.f, 0.f);
        const float *wp = ws + (g * KG) * (4 * NQ) + 4 * j;
        const float *inh = in + (GH * sh) * K;
        // four k-values at a time: per row one 16-byte load of the inputs, per k one of the weights
#pragma unroll
        for (int k4 = 0; k4 < KG; k4 += 4) {
            float4 w[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) w[u] = *reinterpret_cast<const float4 *>(wp + (k4 + u) * (4 * NQ));
#pragma unroll
            for (int s = 0; s < GH; ++s) {
                const float4 x4 = *reinterpret_cast<const float4 *>(inh + s * K + g * KG + k4);
                const float xv[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    acc[s].x = fmaf(xv[u], w[u].x, acc[s].x);
                    acc[s].y = fmaf(xv[u], w[u].y, acc[s].y);
                    acc[s].z = fmaf(xv[u], w[u].z, acc[s].z);
                    acc[s].w = fmaf(xv[u], w[u].w, acc[s].w);
                }
            }
        }
#pragma unroll
        for (int s = 0; s < GH; ++s) *reinterpret_cast<float4 *>(&red[g][GH * sh + s][4 * j]) = acc[s];
    }
    __syncthreads();
    for (int i = tid; i < GS * NQ; i += HT) {
        const int s = i / NQ, jj = i % NQ;
        float4 v = *reinterpret_cast<const float4 *>(&red[0][s][4 * jj]);
#pragma unroll
        for (int gg = 1; gg < KGRP; ++gg) {
            const float4 p = *reinterpret_cast<const float4 *>(&red[gg][s][4 * jj]);
            v.x += p.x; v.y += p.y; v.z += p.z; v.w += p.w;
        }
        epi(s, jj, v);
    }
    __syncthreads();
}

// LayerNorm of the group's rows of x into h, a warp per sequence (biased variance, eps 1e-5);
// gain and bias in shared memory.
__device__ __forceinline__ void group_ln(const float (*x)[D], float (*h)[D], const float *g, const float *b) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int s = warp; s < GS; s += HT / 32) {
        float v[D / 32], sum = 0.0f;
#pragma unroll
        for (int i = 0; i < D / 32; ++i) {
            v[i] = x[s][lane + 32 * i];
            sum += v[i];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        const float mean = sum * (1.0f / D);
        float q = 0.0f;
#pragma unroll
        for (int i = 0; i < D / 32; ++i) {
            v[i] -= mean;
            q += v[i] * v[i];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
        const float r = rsqrtf(q * (1.0f / D) + 1e-5f);
#pragma unroll
        for (int i = 0; i < D / 32; ++i) {
            const int c = lane + 32 * i;
            h[s][c] = v[i] * r * g[c] + b[c];
        }
    }
    __syncthreads();
}

// this CTA's partial product part[s][4 j ..] to slot `slot` of every CTA of the cluster
__device__ __forceinline__ void send_part(HeadsSmem &S, int slot, uint32_t rank, int s, int j, float4 v) {
#pragma unroll
    for (uint32_t r = 0; r < HC; ++r) st_cluster4(&S.part[slot][rank][s][4 * j], r, v);
}

// x[s][c] += bias[c] + the four CTAs' partials of `slot`, added in rank order
__device__ __forceinline__ void add_parts(HeadsSmem &S, int slot, const float *bias) {
    for (int i = threadIdx.x; i < GS * D; i += HT) {
        const int s = i / D, c = i % D;
        float v = bias[c];
#pragma unroll
        for (int r = 0; r < HC; ++r) v += S.part[slot][r][s][c];
        S.x[s][c] += v;
    }
    __syncthreads();
}

// Causal attention of one sequence's head over positions 0..pos, by one warp: lanes over
// positions t = lane + 32 j; every key and value row the warp needs is requested at once.
// q: the head's 32 queries (shared memory); kr / vr: the head's cached rows (row stride D).
// Returns this lane's output dimension (lane) of softmax(q.K^T / sqrt(32)) V.
__device__ __forceinline__ float head_attention(const float *q, const float *kr, const float *vr, int pos,
                                                int lane) {
    constexpr int NJ = CTX / 32;
    const float scale = 0.17677669529663688f;   // 1 / sqrt(32)
    float sc[NJ];
    float mx = -INFINITY;
    // positions past pos read row pos instead (written, finite) and are masked afterwards, so
    // that the loads carry no branch and all of them are in flight together
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
        const int t = lane + 32 * j;
        const float4 *k4 = reinterpret_cast<const float4 *>(kr + (int64_t)min(t, pos) * D);
        float acc = 0.0f;
#pragma unroll
        for (int d = 0; d < HD / 4; ++d) {
            const float4 kv = k4[d];
            const float4 qv = reinterpret_cast<const float4 *>(q)[d];
            acc = fmaf(qv.x, kv.x, acc);
            acc = fmaf(qv.y, kv.y, acc);
            acc = fmaf(qv.z, kv.z, acc);
            acc = fmaf(qv.w, kv.w, acc);
        }
        sc[j] = t <= pos ? acc * scale : -INFINITY;
        mx = fmaxf(mx, sc[j]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.0f;
    float acc[HD];
#pragma unroll
    for (int d = 0; d < HD; ++d) acc[d] = 0.0f;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
        const int t = lane + 32 * j;
        const float p = t <= pos ? expf(sc[j] - mx) : 0.0f;
        sum += p;
        const float4 *v4 = reinterpret_cast<const float4 *>(vr + (int64_t)min(t, pos) * D);
#pragma unroll
        for (int d = 0; d < HD / 4; ++d) {
            const float4 vv = v4[d];
            acc[4 * d] = fmaf(p, vv.x, acc[4 * d]);
            acc[4 * d + 1] = fmaf(p, vv.y, acc[4 * d + 1]);
            acc[4 * d + 2] = fmaf(p, vv.z, acc[4 * d + 2]);
            acc[4 * d + 3] = fmaf(p, vv.w, acc[4 * d + 3]);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    // reduce-scatter: after the stage of width w, lane L holds the partial sums of the w dims whose
    // index agrees with L in the bits above w; at the end lane L holds dimension L
#pragma unroll
    for (int w = HD / 2; w >= 1; w >>= 1) {
        const bool upper = (lane & w) != 0;
#pragma unroll
        for (int i = 0; i < w; ++i) {
            const float give = upper ? acc[i] : acc[i + w];
            const float keep = upper ? acc[i + w] : acc[i];
            acc[i] = keep + __shfl_xor_sync(0xffffffffu, give, w);
        }
    }
    return acc[0] / sum;
}

__global__ void __launch_bounds__(HT, 1) tinygpt_heads_kernel(HeadsArgs a) {
    extern __shared__ __align__(16) unsigned char heads_smem[];
    HeadsSmem &S = *reinterpret_cast<HeadsSmem *>(heads_smem);
    const uint32_t rank = cl_rank();
    const int hh = (int)rank;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const float *wte = a.w, *wpe = a.w + V * D;
    const float *lw0 = a.w + V * D + CTX * D;
    const int64_t groups = cdiv_dev(a.batch, a.group);
    const int v0 = (int)rank * V_R, nv = min(V_R, V - v0);
    // the CTA's vocabulary rows and the final LayerNorm, for the whole decode
    for (int i = tid; i < V_R * D; i += HT) S.wte_s[i / D][i % D] = i / D < nv ? __ldg(wte + (v0 + i / D) * D + i % D) : 0.f;
    for (int i = tid; i < 2 * D; i += HT) S.lnf[i] = __ldg(lw0 + (int64_t)L * LAYER_FLOATS + i);
    int slot = 0, buf = 0;
    prefetch_phase(S.wbuf[0], a.w, 0, PH_QKV, (int)rank);   // the first phase's slice
    cl_sync();   // every CTA of the cluster is running before any stores into its shared memory

    for (int64_t grp = cl_id(); grp < groups; grp += cl_count()) {
        const int64_t b0 = grp * a.group;
        const int gs = (int)min((int64_t)a.group, a.batch - b0);
        if (tid < GS) S.tok[tid] = tid < gs ? a.tokens[(b0 + tid) * CTX] : 0;
        __syncthreads();
        for (int pos = 0; pos < a.steps; ++pos) {
            if (tid < gs && pos < a.prompt_len) S.tok[tid] = a.tokens[(b0 + tid) * CTX + pos];
            __syncthreads();
            for (int i = tid; i < GS * D; i += HT) {
                const int s = i / D, c = i % D;
                int t = S.tok[s];
                t = t < 0 ? 0 : (t >= V ? V - 1 : t);
                S.x[s][c] = s < gs ? __ldg(wte + t * D + c) + __ldg(wpe + pos * D + c) : 0.0f;
            }
            __syncthreads();
            for (int l = 0; l < L; ++l) {
                float *kc = a.kv + ((int64_t)l * 2 + 0) * a.batch * CTX * D;
                float *vc = a.kv + ((int64_t)l * 2 + 1) * a.batch * CTX * D;
                // each phase: start the next phase's copies, wait for this phase's, compute
                // 1. LayerNorm and this head's q, k, v: quads 0-7 q, 8-15 k, 16-23 v
                prefetch_phase(S.wbuf[buf ^ 1], a.w, l, PH_O, (int)rank);
                cp_async_wait<1>();
                __syncthreads();
                {
                    const float *wq = S.wbuf[buf], *par = wq + WB_MAT;
                    group_ln(S.x, S.h, par, par + D);
                    group_linear<D, 24>(&S.h[0][0], wq, S.red, [&](int s, int j, float4 v) {
                        const float4 bb = *reinterpret_cast<const float4 *>(par + 2 * D + 4 * j);
                        v.x += bb.x; v.y += bb.y; v.z += bb.z; v.w += bb.w;
                        if (j < 8) {
                            *reinterpret_cast<float4 *>(&S.q[s][4 * j]) = v;
                        } else if (s < gs) {
                            float *cache = j < 16 ? kc : vc;
                            *reinterpret_cast<float4 *>(cache + ((b0 + s) * CTX + pos) * D + hh * HD +
                                                        4 * (j & 7)) = v;
                        }
                    });
                }
                buf ^= 1;
                // 2. causal attention of head hh, a warp per sequence
                prefetch_phase(S.wbuf[buf ^ 1], a.w, l, PH_FC, (int)rank);
                for (int s = warp; s < GS; s += HT / 32) {
                    if (s < gs) {
                        const float o = head_attention(S.q[s], kc + ((b0 + s) * CTX) * D + hh * HD,
                                                       vc + ((b0 + s) * CTX) * D + hh * HD, pos, lane);
                        S.att[s][lane] = o;
                    } else {
                        S.att[s][lane] = 0.0f;
                    }
                }
                cp_async_wait<1>();
                __syncthreads();
                // 3. the head's share of the output projection, to every CTA; x += b_o + the four shares
                {
                    const float *wo = S.wbuf[buf];
                    group_linear<HD, D / 4>(&S.att[0][0], wo, S.red,
                                            [&](int s, int j, float4 v) { send_part(S, slot, rank, s, j, v); });
                    cl_sync();
                    add_parts(S, slot, wo + WB_MAT);
                    slot ^= 1;
                }
                buf ^= 1;
                // 4. LayerNorm and this CTA's 128 GELU hidden units
                prefetch_phase(S.wbuf[buf ^ 1], a.w, l, PH_PR, (int)rank);
                cp_async_wait<1>();
                __syncthreads();
                {
                    const float *wf = S.wbuf[buf], *par = wf + WB_MAT;
                    group_ln(S.x, S.h, par, par + D);
                    group_linear<D, FH / 4>(&S.h[0][0], wf, S.red, [&](int s, int j, float4 v) {
                        const float4 bb = *reinterpret_cast<const float4 *>(par + 2 * D + 4 * j);
                        float r4[4] = {v.x + bb.x, v.y + bb.y, v.z + bb.z, v.w + bb.w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) r4[e] = 0.5f * r4[e] * (1.0f + erff(r4[e] * 0.70710678118654752f));
                        *reinterpret_cast<float4 *>(&S.f[s][4 * j]) = make_float4(r4[0], r4[1], r4[2], r4[3]);
                    });
                }
                buf ^= 1;
                // 5. their share of the MLP projection, to every CTA; x += b_pr + the four shares
                {
                    const int nl = l + 1 < L ? l + 1 : 0;   // the next phase: the next layer's (or position's) QKV
                    prefetch_phase(S.wbuf[buf ^ 1], a.w, nl, PH_QKV, (int)rank);
                }
                cp_async_wait<1>();
                __syncthreads();
                {
                    const float *wp = S.wbuf[buf];
                    group_linear<FH, D / 4>(&S.f[0][0], wp, S.red,
                                            [&](int s, int j, float4 v) { send_part(S, slot, rank, s, j, v); });
                    cl_sync();
                    add_parts(S, slot, wp + WB_MAT);
                    slot ^= 1;
                }
                buf ^= 1;
            }
            const bool next_from_model = pos + 1 >= a.prompt_len && pos + 1 < a.end;
            const bool want_logits = a.logits && pos == a.steps - 1;
            if (!next_from_model && !want_logits) continue;
            // final LayerNorm and the tied head: this CTA's vocabulary rows, a warp per (sequence, row)
            group_ln(S.x, S.h, S.lnf, S.lnf + D);
            for (int pv = warp; pv < gs * nv; pv += HT / 32) {
                const int s = pv / nv, v = pv % nv;
                float acc = 0.0f;
#pragma unroll
                for (int i = 0; i < D / 32; ++i) acc = fmaf(S.h[s][lane + 32 * i], S.wte_s[v][lane + 32 * i], acc);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
                if (lane < HC) st_cluster(&S.lg[s][v0 + v], lane, acc);
            }
            cl_sync();
            if (tid < gs) {
                int best = 0;
                for (int v = 1; v < V; ++v)
                    if (S.lg[tid][v] > S.lg[tid][best]) best = v;     // first maximum, as numpy.argmax
                if (next_from_model) {
                    S.tok[tid] = best;
                    if (rank == 0) a.tokens[(b0 + tid) * CTX + pos + 1] = best;
                }
            }
            if (want_logits && rank == 0)
                for (int i = tid; i < gs * V; i += HT) a.logits[(b0 + i / V) * V + i % V] = S.lg[i / V][i % V];
            __syncthreads();
        }
    }
    cp_async_wait<0>();   // the last, unused prefetch lands before the CTA's shared memory goes
    cl_sync();            // no CTA leaves while another may still store into its shared memory
}

}  // namespace tg
}  // namespace piton

using namespace piton;

extern "C" int64_t piton_b200_tinygpt_weight_floats(void) { return tg::TOTAL_FLOATS; }

namespace {

// Clusters of 16 CTAs with the cluster kernel's shared memory that fit on the current
// device at once (0: the cluster path is unavailable), looked up once per device.
int cluster_capacity() {
    static int cache[64];
    static bool known[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    if (known[dev]) return cache[dev];
    int n = 0;
    bool failed = true;
    if (cudaFuncSetAttribute(tg::tinygpt_cluster_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
            cudaSuccess &&
        cudaFuncSetAttribute(tg::tinygpt_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)tg::CLUSTER_SMEM) == cudaSuccess) {
        failed = false;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(tg::CS);
        cfg.blockDim = dim3(tg::THREADS);
        cfg.dynamicSmemBytes = tg::CLUSTER_SMEM;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = tg::CS;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n, tg::tinygpt_cluster_kernel, &cfg) != cudaSuccess) {
            n = 0;
            failed = true;
        }
    }
    if (failed) cudaGetLastError();   // a refused attribute or query only disables this path
    cache[dev] = n;
    known[dev] = true;
    return n;
}

void launch_cluster(const tg::ClusterArgs &c, int clusters, cudaStream_t q) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(clusters * tg::CS));
    cfg.blockDim = dim3(tg::THREADS);
    cfg.dynamicSmemBytes = tg::CLUSTER_SMEM;
    cfg.stream = q;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = tg::CS;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, tg::tinygpt_cluster_kernel, c);
}

// Clusters of 4 CTAs with the heads kernel's shared memory that fit on the current device at
// once (0: that path is unavailable), looked up once per device.
int heads_capacity() {
    static int cache[64];
    static bool known[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    if (known[dev]) return cache[dev];
    int n = 0;
    if (cudaFuncSetAttribute(tg::tinygpt_heads_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)sizeof(tg::HeadsSmem)) == cudaSuccess) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(tg::HC);
        cfg.blockDim = dim3(tg::HT);
        cfg.dynamicSmemBytes = sizeof(tg::HeadsSmem);
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = tg::HC;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n, tg::tinygpt_heads_kernel, &cfg) != cudaSuccess) n = 0;
    }
    cudaGetLastError();   // a refused attribute or query only disables this path
    cache[dev] = n;
    known[dev] = true;
    return n;
}

void launch_heads(const tg::HeadsArgs &h, int clusters, cudaStream_t q) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(clusters * tg::HC));
    cfg.blockDim = dim3(tg::HT);
    cfg.dynamicSmemBytes = sizeof(tg::HeadsSmem);
    cfg.stream = q;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = tg::HC;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, tg::tinygpt_heads_kernel, h);
}

// PITON_B200_TINYGPT_KERNEL=cluster|heads|step picks a decode kernel for comparisons; by default
// batches up to the number of 16-CTA clusters that fit use the cluster kernel and larger ones (or
// every batch when no cluster launch is possible) the step kernel.
int forced_kernel() {
    const char *e = getenv("PITON_B200_TINYGPT_KERNEL");
    if (!e || !*e) return 0;
    if (!strcmp(e, "cluster")) return 1;
    if (!strcmp(e, "heads")) return 2;
    if (!strcmp(e, "step")) return 3;
    return -1;
}

}  // namespace

// ---------------------------------------------------------------------------
// CUDA-graph cache: with PITON_B200_CUDA_GRAPH a decode's launch is captured
// once per argument set (stream capture on an internal stream, thread-local
// mode), instantiated, and replayed with one cudaGraphLaunch on the caller's
// stream, so a repeated decode skips the host launch path and its argument set-up.
// ---------------------------------------------------------------------------
#include <mutex>

namespace {

constexpr int GRAPH_CACHE = 16;

struct GraphEntry {
    piton_tinygpt_args key{};
    cudaGraphExec_t exec = nullptr;
    uint64_t used = 0;
    int launches = 0;
};

struct DeviceGraphs {
    cudaStream_t capture = nullptr;
    GraphEntry entries[GRAPH_CACHE];
    uint64_t clock = 0;
};

std::mutex g_graph_mu;
DeviceGraphs g_graphs[64];

bool same_args(const piton_tinygpt_args &a, const piton_tinygpt_args &b) {
    return a.weights == b.weights && a.kv_cache == b.kv_cache && a.tokens == b.tokens && a.logits == b.logits &&
           a.batch == b.batch && a.prompt_len == b.prompt_len && a.new_tokens == b.new_tokens && a.flags == b.flags;
}

}  // namespace

extern "C" int piton_b200_graph_cache_entries(int *entries) {
    PITON_REQUIRE(entries != nullptr, "entries is NULL");
    int dev = 0;
    PITON_CUDA(cudaGetDevice(&dev));
    PITON_REQUIRE(dev >= 0 && dev < 64, "device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_graph_mu);
    int n = 0;
    for (auto &e : g_graphs[dev].entries) n += e.exec != nullptr;
    *entries = n;
    return PITON_B200_OK;
}

extern "C" int piton_b200_graph_cache_clear(void) {
    int dev = 0;
    PITON_CUDA(cudaGetDevice(&dev));
    PITON_REQUIRE(dev >= 0 && dev < 64, "device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_graph_mu);
    for (auto &e : g_graphs[dev].entries) {
        if (e.exec) cudaGraphExecDestroy(e.exec);
        e = GraphEntry{};
    }
    return PITON_B200_OK;
}

extern "C" int piton_b200_tinygpt_generate(const piton_tinygpt_args *a, void *stream) {
    using namespace tg;
    PITON_REQUIRE(a != nullptr, "args is NULL");
    PITON_REQUIRE(a->vocab == V && a->d_model == D && a->n_layer == L && a->n_head == H && a->ctx == CTX,
                  "only the configuration vocab %d, d_model %d, %d layers, %d heads, context %d is built", V, D, L, H,
                  CTX);
    PITON_REQUIRE(a->batch >= 0 && a->prompt_len >= 1 && a->new_tokens >= 0, "bad batch/prompt/new_tokens");
    PITON_REQUIRE(a->prompt_len + a->new_tokens <= CTX, "prompt_len + new_tokens = %lld exceeds the context %d",
                  (long long)(a->prompt_len + a->new_tokens), CTX);
    PITON_REQUIRE((a->flags & ~PITON_B200_CUDA_GRAPH) == 0, "unknown flags 0x%x", a->flags);
    if (a->batch == 0) return PITON_B200_OK;
    PITON_REQUIRE(a->weights && a->kv_cache && a->tokens, "NULL pointer");
    PITON_REQUIRE(a->batch <= (int64_t)SEQ * 65535 * 1024, "batch too large");
    StepArgs s;
    s.w = reinterpret_cast<const float *>(a->weights);
    s.kv = reinterpret_cast<float *>(a->kv_cache);
    s.tokens = reinterpret_cast<int32_t *>(a->tokens);
    s.batch = a->batch;
    s.prompt_len = (int)a->prompt_len;
    s.end = (int)(a->prompt_len + a->new_tokens);
    // one launch per fed position; with no new tokens, logits (if asked for) come from the last prompt token
    int steps = s.end - 1;
    if (a->new_tokens == 0 && a->logits) steps = (int)a->prompt_len;
    const unsigned grid = (unsigned)cdiv(a->batch, SEQ);
    cudaStream_t st = as_stream(stream);
    // small batches: one 16-CTA cluster per sequence, weights resident in shared memory; larger
    // ones: the step kernel (2 sequences per CTA); each is one launch per decode.  The 4-CTA-cluster
    // heads kernel runs only when asked for (PITON_B200_TINYGPT_KERNEL=heads): measured against the
    // step kernel at batches 16-256 it is as fast at 16 and slower above (2.22 against 2.45 M
    // tokens/s at 128, 3.01 against 3.67 M at 192), with the same tokens
    const int forced = forced_kernel();
    PITON_REQUIRE(forced >= 0, "PITON_B200_TINYGPT_KERNEL must be cluster, heads or step");
    const int clusters = cluster_capacity();
    const int hcap = heads_capacity();
    bool use_cluster = clusters > 0 && a->batch <= clusters;
    bool use_heads = false;
    if (forced == 1) {
        PITON_REQUIRE(clusters > 0 && a->batch <= clusters, "the cluster kernel takes at most %d sequences", clusters);
        use_cluster = true, use_heads = false;
    } else if (forced == 2) {
        PITON_REQUIRE(hcap > 0, "the heads kernel cannot be launched on this device");
        use_cluster = false, use_heads = true;
    } else if (forced == 3) {
        use_cluster = use_heads = false;
    }
    int group = 0, hclusters = 0;
    if (use_heads) {
        group = (int)std::min<int64_t>(GS, std::max<int64_t>(1, cdiv(a->batch, hcap)));
        hclusters = (int)std::min<int64_t>(hcap, cdiv(a->batch, group));
    }
    const int launches = 1;
    auto enqueue = [&](cudaStream_t q) {
        if (use_heads) {
            HeadsArgs h;
            h.w = s.w;
            h.kv = s.kv;
            h.tokens = s.tokens;
            h.logits = reinterpret_cast<float *>(a->logits);
            h.batch = a->batch;
            h.prompt_len = s.prompt_len;
            h.end = s.end;
            h.steps = steps;
            h.group = group;
            launch_heads(h, hclusters, q);
            return;
        }
        if (use_cluster) {
            ClusterArgs c;
            c.w = s.w;
            c.kv = s.kv;
            c.tokens = s.tokens;
            c.logits = reinterpret_cast<float *>(a->logits);
            c.batch = a->batch;
            c.prompt_len = s.prompt_len;
            c.end = s.end;
            c.steps = steps;
            launch_cluster(c, (int)a->batch, q);
            return;
        }
        s.steps = steps;
        s.logits = reinterpret_cast<float *>(a->logits);
        tinygpt_step_kernel<<<grid, THREADS, 0, q>>>(s);
    };
    if (!(a->flags & PITON_B200_CUDA_GRAPH)) {
        enqueue(st);
        return check_launch("tinygpt", launches);
    }
    int dev = 0;
    PITON_CUDA(cudaGetDevice(&dev));
    PITON_REQUIRE(dev >= 0 && dev < 64, "device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_graph_mu);
    DeviceGraphs &G = g_graphs[dev];
    GraphEntry *hit = nullptr;
    for (auto &e : G.entries)
        if (e.exec && same_args(e.key, *a)) {
            hit = &e;
            break;
        }
    if (!hit) {
        // a free entry, else the least recently used one
        GraphEntry *victim = nullptr;
        for (auto &e : G.entries)
            if (!e.exec) {
                victim = &e;
                break;
            }
        if (!victim) {
            victim = &G.entries[0];
            for (auto &e : G.entries)
                if (e.used < victim->used) victim = &e;
        }
        if (!G.capture) PITON_CUDA(cudaStreamCreateWithFlags(&G.capture, cudaStreamNonBlocking));
        if (victim->exec) cudaGraphExecDestroy(victim->exec);
        *victim = GraphEntry{};
        cudaGraph_t graph = nullptr;
        PITON_CUDA(cudaStreamBeginCapture(G.capture, cudaStreamCaptureModeThreadLocal));
        enqueue(G.capture);
        cudaError_t launch_err = cudaGetLastError();
        cudaError_t end_err = cudaStreamEndCapture(G.capture, &graph);
        if (launch_err != cudaSuccess || end_err != cudaSuccess) {
            if (graph) cudaGraphDestroy(graph);
            return set_error(PITON_B200_ECUDA, "tinygpt graph capture: %s",
                             cudaGetErrorString(launch_err != cudaSuccess ? launch_err : end_err));
        }
        cudaError_t inst = cudaGraphInstantiate(&victim->exec, graph, 0);
        cudaGraphDestroy(graph);
        if (inst != cudaSuccess) {
            victim->exec = nullptr;
            return set_error(PITON_B200_ECUDA, "tinygpt graph instantiate: %s", cudaGetErrorString(inst));
        }
        victim->key = *a;
        victim->launches = launches;
        hit = victim;
    }
    hit->used = ++G.clock;
    PITON_CUDA(cudaGraphLaunch(hit->exec, st));
    return check_launch("tinygpt graph", hit->launches);
}
