// TinyGPT greedy decoding (no counterpart in the reference, which has the pieces
// but not the model): character-level decoder, vocab 65, d_model 128, 4
// pre-LayerNorm blocks of 4-head causal attention (head dim 32) and a 4x GELU
// MLP, learned positions, tied input/output embeddings, context 128.
//
// One launch per token position.  A CTA owns SEQ sequences; for its new token
// it runs every layer with the activations in shared memory, appends the
// token's keys and values to the caller's KV cache, attends over the cached
// positions (one warp per sequence x head), and at the end writes the greedy
// next token (argmax of the 65 tied-embedding logits, first maximum) into
// the token buffer, which the next launch reads: the whole generation runs
// on the stream without host round trips.  Weights (3.2 MB) stay L2-resident
// and are read through L1.
//
// Packed weight layout (fp32, row-major, input-by-output matrices):
//   wte[V,D] wpe[CTX,D]
//   per layer: ln1_g[D] ln1_b[D] w_qkv[D,3D] b_qkv[3D] w_o[D,D] b_o[D]
//              ln2_g[D] ln2_b[D] w_fc[D,4D] b_fc[4D] w_pr[4D,D] b_pr[D]
//   lnf_g[D] lnf_b[D]
// KV cache: fp32 [L][2][B][CTX][D] (keys, then values).
#include "common.cuh"

namespace piton {
namespace tg {

constexpr int V = 65, D = 128, L = 4, H = 4, HD = 32, F = 4 * D, CTX = 128;
constexpr int SEQ = 2, THREADS = 256;
constexpr int LAYER_FLOATS = 2 * D + D * 3 * D + 3 * D + D * D + D + 2 * D + D * F + F + F * D + D;
constexpr int64_t TOTAL_FLOATS = (int64_t)V * D + (int64_t)CTX * D + (int64_t)L * LAYER_FLOATS + 2 * D;

struct StepArgs {
    const float *w;
    float *kv;
    int32_t *tokens;
    float *logits;
    int64_t batch;
    int pos;          // position of the token fed at this step
    int prompt_len;   // the next token is written when prompt_len - 1 <= pos and pos + 1 < end
    int end;          // prompt_len + new_tokens
};

// out[s][n] = act(sum_k in[s][k] W[k][n] + b[n]) for the CTA's SEQ rows.  A
// thread owns 4 adjacent columns (16-byte weight loads) of one k-group; the
// k range is split into G groups so that every thread has work, and the
// partial sums meet in `scratch` (SEQ * THREADS * 4 floats).  Eight k-steps
// are unrolled so 8 x 16 bytes of weights are in flight per thread: the
// weights come from L2 and this loop is latency-bound otherwise.
template <int K, int N, bool GELU>
__device__ __forceinline__ void linear(const float *in, float *out, const float *__restrict__ W,
                                       const float *__restrict__ b, float *scratch, bool residual) {
    constexpr int NQ = N / 4;                             // column quads
    constexpr int G = THREADS / NQ > 0 ? THREADS / NQ : 1;  // k-groups
    constexpr int KG = K / G;
    static_assert(N % 4 == 0 && K % G == 0 && NQ * G <= THREADS && G >= 2, "linear tiling");
    const int tid = threadIdx.x;
    const int q = tid % NQ, g = tid / NQ;
    float4 acc[SEQ];
#pragma unroll
    for (int s = 0; s < SEQ; ++s) acc[s] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (g < G) {
        const float4 *w4 = reinterpret_cast<const float4 *>(W) + q;
#pragma unroll 8
        for (int k = g * KG; k < (g + 1) * KG; ++k) {
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
        float4 bb = __ldg(reinterpret_cast<const float4 *>(b) + qq);
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

// y[s] = LayerNorm(x[s]) * g + b, one warp per sequence (biased variance, eps 1e-5).
__device__ __forceinline__ void layernorm(const float *x, float *y, const float *__restrict__ g,
                                          const float *__restrict__ b) {
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
            y[warp * D + c] = v[i] * r * __ldg(g + c) + __ldg(b + c);
        }
    }
    __syncthreads();
}

__global__ void __launch_bounds__(THREADS) tinygpt_step_kernel(StepArgs a) {
    __shared__ __align__(16) float x[SEQ * D], h[SEQ * D], qkv[SEQ * 3 * D], att[SEQ * D], f[SEQ * F];
    __shared__ float probs[SEQ * H][CTX];
    __shared__ __align__(16) float scratch[SEQ * THREADS * 4];
    __shared__ float lg[SEQ][V + 3];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t b0 = (int64_t)blockIdx.x * SEQ;
    const int pos = a.pos;
    const float *wte = a.w, *wpe = a.w + V * D;

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
        const float *ln1_g = lw, *ln1_b = ln1_g + D, *w_qkv = ln1_b + D, *b_qkv = w_qkv + D * 3 * D;
        const float *w_o = b_qkv + 3 * D, *b_o = w_o + D * D, *ln2_g = b_o + D, *ln2_b = ln2_g + D;
        const float *w_fc = ln2_b + D, *b_fc = w_fc + D * F, *w_pr = b_fc + F, *b_pr = w_pr + F * D;
        float *kc = a.kv + ((int64_t)l * 2 + 0) * a.batch * CTX * D;
        float *vc = a.kv + ((int64_t)l * 2 + 1) * a.batch * CTX * D;

        layernorm(x, h, ln1_g, ln1_b);
        linear<D, 3 * D, false>(h, qkv, w_qkv, b_qkv, scratch, false);
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
        linear<D, D, false>(att, x, w_o, b_o, scratch, true);          // x += attn @ Wo + bo
        layernorm(x, h, ln2_g, ln2_b);
        linear<D, F, true>(h, f, w_fc, b_fc, scratch, false);         // f = gelu(h @ Wfc + bfc)
        linear<F, D, false>(f, x, w_pr, b_pr, scratch, true);          // x += f @ Wpr + bpr
    }
    const float *lnf_g = lw, *lnf_b = lnf_g + D;
    layernorm(x, h, lnf_g, lnf_b);
    // tied head: logits[s][v] = h[s] . wte[v]; warp per (s, v) pair, lanes over D
    for (int pv = warp; pv < SEQ * V; pv += THREADS / 32) {
        int s = pv / V, vv = pv % V;
        float acc = 0.0f;
#pragma unroll
        for (int i = 0; i < D / 32; ++i) acc = fmaf(h[s * D + lane + 32 * i], __ldg(wte + vv * D + lane + 32 * i), acc);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) lg[s][vv] = acc;
    }
    __syncthreads();
    if (tid < SEQ && pos + 1 >= a.prompt_len && pos + 1 < a.end) {
        int64_t b = b0 + tid;
        if (b < a.batch) {
            int best = 0;
            for (int vv = 1; vv < V; ++vv)
                if (lg[tid][vv] > lg[tid][best]) best = vv;     // first maximum, as numpy.argmax
            a.tokens[b * CTX + pos + 1] = best;
        }
    }
    if (a.logits) {
        for (int i = tid; i < SEQ * V; i += THREADS) {
            int s = i / V, vv = i % V;
            int64_t b = b0 + s;
            if (b < a.batch) a.logits[b * V + vv] = lg[s][vv];
        }
    }
}

}  // namespace tg
}  // namespace piton

using namespace piton;

extern "C" int64_t piton_b200_tinygpt_weight_floats(void) { return tg::TOTAL_FLOATS; }

// ---------------------------------------------------------------------------
// CUDA-graph cache: a decode is ~80 launches of one small kernel, so the host
// launch path costs a few microseconds a token.  With PITON_B200_CUDA_GRAPH the
// sequence is captured once per argument set (stream capture on an internal
// stream, thread-local mode), instantiated, and replayed with one
// cudaGraphLaunch on the caller's stream.
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
    auto enqueue = [&](cudaStream_t q) {
        for (int p = 0; p < steps; ++p) {
            s.pos = p;
            s.logits = p == steps - 1 ? reinterpret_cast<float *>(a->logits) : nullptr;
            tinygpt_step_kernel<<<grid, THREADS, 0, q>>>(s);
        }
    };
    if (!(a->flags & PITON_B200_CUDA_GRAPH)) {
        enqueue(st);
        return check_launch("tinygpt", steps);
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
        victim->launches = steps;
        hit = victim;
    }
    hit->used = ++G.clock;
    PITON_CUDA(cudaGraphLaunch(hit->exec, st));
    return check_launch("tinygpt graph", hit->launches);
}
