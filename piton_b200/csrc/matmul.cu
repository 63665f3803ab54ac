// Entry points of the tutorial matmul (examples/kernels.py:18-57) and the dense
// layer (examples/nn_kernels.py:23-74): argument checks and the choice between
// the tcgen05 split-operand path (gemm_tc.cu: tf32 high halves + bf16 cross terms) and the
// CUDA-core path (gemm_simt.cu).
#include "common.cuh"
#include "gemm_simt.cuh"
#include "gemm_tc.cuh"

using namespace piton;

static int check_matmul(const piton_matmul_args *a) {
    PITON_REQUIRE(a != nullptr, "args is NULL");
    PITON_REQUIRE(a->M >= 0 && a->N >= 0 && a->K >= 0, "negative shape %lld x %lld x %lld", (long long)a->M,
                  (long long)a->N, (long long)a->K);
    PITON_REQUIRE(a->block_m > 0 && a->block_n > 0 && a->block_k > 0 && a->group_m > 0 && a->grid_x >= 0,
                  "bad tile/group/grid");
    PITON_REQUIRE((a->flags & ~(PITON_B200_QPU_ROUNDING | PITON_B200_FORCE_SIMT)) == 0, "unknown flags 0x%x",
                  a->flags);
    return PITON_B200_OK;
}

static TcGemmShape tc_shape(const piton_matmul_args *a) {
    TcGemmShape t;
    t.a = reinterpret_cast<const float *>(a->a);
    t.b = reinterpret_cast<const float *>(a->b);
    t.c = reinterpret_cast<float *>(a->c);
    t.M = a->M; t.N = a->N; t.K = a->K;
    t.sam = a->stride_am; t.sak = a->stride_ak; t.sbk = a->stride_bk; t.sbn = a->stride_bn;
    t.scm = a->stride_cm; t.scn = a->stride_cn;
    return t;
}

// The tensor-core path computes every element of C, so it needs a grid that
// covers every reference tile and a non-degenerate problem.
static bool use_tc(const piton_matmul_args *a) {
    if (a->flags & (PITON_B200_QPU_ROUNDING | PITON_B200_FORCE_SIMT)) return false;
    if (a->grid_x < grouped_tiles(a->M, a->N, a->block_m, a->block_n)) return false;
    return tc_gemm_supported(tc_shape(a));
}

extern "C" size_t piton_b200_matmul_workspace_size(const piton_matmul_args *a) {
    if (check_matmul(a) != PITON_B200_OK || !use_tc(a)) return 0;
    return tc_gemm_workspace_bytes(tc_shape(a));
}

extern "C" int piton_b200_matmul_f32(const piton_matmul_args *a, void *stream) {
    int rc = check_matmul(a);
    if (rc) return rc;
    if (a->M == 0 || a->N == 0 || a->grid_x == 0) return PITON_B200_OK;
    PITON_REQUIRE(a->a && a->b && a->c, "NULL pointer");
    cudaStream_t s = as_stream(stream);
    if (use_tc(a)) {
        size_t need = tc_gemm_workspace_bytes(tc_shape(a));
        if (a->workspace_bytes < need || (need && !a->workspace))
            return set_error(PITON_B200_EWORKSPACE, "matmul needs %zu bytes of workspace, got %llu", need,
                             (unsigned long long)a->workspace_bytes);
        return tc_gemm(tc_shape(a), reinterpret_cast<void *>(a->workspace), s);
    }
    GemmSimtParams p{};
    p.a = reinterpret_cast<const float *>(a->a);
    p.b = reinterpret_cast<const float *>(a->b);
    p.c = reinterpret_cast<float *>(a->c);
    p.M = a->M; p.N = a->N; p.K = a->K;
    p.sam = a->stride_am; p.sak = a->stride_ak; p.sbk = a->stride_bk; p.sbn = a->stride_bn;
    p.scm = a->stride_cm; p.scn = a->stride_cn;
    p.ref_bm = a->block_m; p.ref_bn = a->block_n; p.ref_group = a->group_m; p.grid_x = a->grid_x;
    p.check_grid = a->grid_x < grouped_tiles(a->M, a->N, a->block_m, a->block_n);
    return gemm_simt(p, (a->flags & PITON_B200_QPU_ROUNDING) != 0, s);
}

extern "C" int piton_b200_dense_f32(const piton_dense_args *a, void *stream) {
    PITON_REQUIRE(a != nullptr, "args is NULL");
    PITON_REQUIRE(a->M >= 0 && a->N > 0 && a->K > 0, "bad shape %lld x %lld x %lld", (long long)a->M,
                  (long long)a->N, (long long)a->K);
    PITON_REQUIRE(a->block_m > 0 && a->block_n > 0 && a->block_k > 0 && a->group_m > 0 && a->grid_x >= 0,
                  "bad tile/group/grid");
    PITON_REQUIRE((a->flags & ~(PITON_B200_QPU_ROUNDING | PITON_B200_FORCE_SIMT)) == 0, "unknown flags 0x%x",
                  a->flags);
    if (a->M == 0 || a->grid_x == 0) return PITON_B200_OK;
    PITON_REQUIRE(a->x && a->w && a->y && (!a->add_bias || a->bias), "NULL pointer");
    GemmSimtParams p{};
    p.a = reinterpret_cast<const float *>(a->x);
    p.b = reinterpret_cast<const float *>(a->w);
    p.c = reinterpret_cast<float *>(a->y);
    p.bias = a->add_bias ? reinterpret_cast<const float *>(a->bias) : nullptr;
    p.relu = a->relu != 0;
    p.M = a->M; p.N = a->N; p.K = a->K;
    p.sam = a->K; p.sak = 1; p.sbk = a->N; p.sbn = 1; p.scm = a->N; p.scn = 1;
    p.ref_bm = a->block_m; p.ref_bn = a->block_n; p.ref_group = a->group_m; p.grid_x = a->grid_x;
    p.check_grid = a->grid_x < grouped_tiles(a->M, a->N, a->block_m, a->block_n);
    return gemm_simt(p, (a->flags & PITON_B200_QPU_ROUNDING) != 0, as_stream(stream));
}

// ---------------------------------------------------------------------------
// Matmul without any allocation by the caller or the library.
//
// Some callers cannot call cudaMalloc at all: real-time or embedded hosts
// whose device memory is fixed at start-up, plugin hosts that hand out device
// pointers but own every allocation themselves, and processes whose device
// memory is all held by another allocator's pool.  For them this entry point
// takes the tensor-core path's scratch
// (the tf32 hi/lo operand split) from one file-scope device array instead of
// the caller's workspace.  The array holds PITON_B200_NOALLOC_SCRATCH_BYTES;
// every GPU that loads this library keeps it until the process exits.
//
// In host code `g_matmul_scratch` names a host-side stand-in, not a device
// address, so the device address is looked up with cudaGetSymbolAddress (with
// the device current) the first time a call runs in a CUDA context, and cached
// under that context's process-unique id (cuCtxGetId).  A later call in a new
// context on the same device (after cudaDeviceReset, or with another context
// made current) sees a different id and looks the address up again, so no
// stale address is ever used.  A call that does the look-up should come before
// any stream capture.  Every call shares the array and it keeps the last
// call's contents; nothing in it needs to start at zero (the split kernel
// writes every element the GEMM reads).  Calls that overlap on the GPU (other
// streams, other host threads on the same device) race on it and must be
// serialised by the caller.
// ---------------------------------------------------------------------------

#include <cuda.h>
#include <mutex>

static __device__ __align__(256) uint8_t g_matmul_scratch[PITON_B200_NOALLOC_SCRATCH_BYTES];

// The driver functions are reached through cudaGetDriverEntryPoint, so the library keeps no
// link-time dependency on libcuda (it must load on machines without a driver, for its CPU tests).
static bool current_context_id(unsigned long long *id) {
    typedef CUresult (*get_current_t)(CUcontext *);
    typedef CUresult (*get_id_t)(CUcontext, unsigned long long *);
    static get_current_t get_current = nullptr;
    static get_id_t get_id = nullptr;
    if (!get_current || !get_id) {
        void *p1 = nullptr, *p2 = nullptr;
        cudaDriverEntryPointQueryResult q1, q2;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p1, cudaEnableDefault, &q1) != cudaSuccess ||
            q1 != cudaDriverEntryPointSuccess ||
            cudaGetDriverEntryPoint("cuCtxGetId", &p2, cudaEnableDefault, &q2) != cudaSuccess ||
            q2 != cudaDriverEntryPointSuccess)
            return false;
        get_current = reinterpret_cast<get_current_t>(p1);
        get_id = reinterpret_cast<get_id_t>(p2);
    }
    CUcontext ctx = nullptr;
    if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return false;
    return get_id(ctx, id) == CUDA_SUCCESS;
}

static void *noalloc_scratch(int *rc) {
    static std::mutex mu;
    static void *ptrs[64] = {nullptr};
    static unsigned long long ctx_ids[64] = {0};
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) {
        *rc = set_error(PITON_B200_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(err));
        return nullptr;
    }
    if (dev < 0 || dev >= 64) {
        *rc = set_error(PITON_B200_EINVAL, "device %d out of range", dev);
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(mu);
    unsigned long long id = 0;
    bool have_id = current_context_id(&id);   // false before the runtime has made a context current
    if (!have_id || !ptrs[dev] || ctx_ids[dev] != id) {
        void *p = nullptr;
        err = cudaGetSymbolAddress(&p, g_matmul_scratch);   // also makes the primary context current
        if (err != cudaSuccess) {
            *rc = set_error(PITON_B200_ECUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(err));
            return nullptr;
        }
        if (!current_context_id(&id)) {
            *rc = set_error(PITON_B200_ECUDA, "no current CUDA context after cudaGetSymbolAddress");
            return nullptr;
        }
        ptrs[dev] = p;
        ctx_ids[dev] = id;
    }
    *rc = PITON_B200_OK;
    return ptrs[dev];
}

extern "C" int piton_b200_matmul_f32_noalloc(const piton_matmul_args *a, void *stream) {
    int rc = check_matmul(a);
    if (rc) return rc;
    if (a->M == 0 || a->N == 0 || a->grid_x == 0) return PITON_B200_OK;
    PITON_REQUIRE(a->a && a->b && a->c, "NULL pointer");
    if (!use_tc(a)) {
        // the CUDA-core path uses no scratch at all
        piton_matmul_args b = *a;
        b.workspace = 0;
        b.workspace_bytes = 0;
        return piton_b200_matmul_f32(&b, stream);
    }
    size_t need = tc_gemm_workspace_bytes(tc_shape(a));
    if (need > (size_t)PITON_B200_NOALLOC_SCRATCH_BYTES)
        return set_error(PITON_B200_EINVAL,
                         "matmul %lld x %lld x %lld needs %zu bytes of scratch; the no-alloc entry point holds %zu "
                         "(use piton_b200_matmul_f32 with a workspace)",
                         (long long)a->M, (long long)a->N, (long long)a->K, need,
                         (size_t)PITON_B200_NOALLOC_SCRATCH_BYTES);
    void *scratch = noalloc_scratch(&rc);
    if (!scratch) return rc;
    return tc_gemm(tc_shape(a), scratch, as_stream(stream));
}

// ---------------------------------------------------------------------------
// Matmul sharded by M rows with the output all-gather fused into the GEMM:
// this rank computes rows [row_offset, row_offset + M) of the full C and the
// epilogue stores every finished tile into each rank's full C through peer
// pointers (NVLink stores, overlapped with the next tiles' MMAs), so no
// separate all-gather runs.  The caller orders completion across ranks (a
// barrier after the call on every rank) before reading C.
// ---------------------------------------------------------------------------
extern "C" int piton_b200_matmul_allgather_f32(const piton_matmul_args *a, const piton_allgather_args *g,
                                               void *stream) {
    int rc = check_matmul(a);
    if (rc) return rc;
    PITON_REQUIRE(g != nullptr, "allgather args is NULL");
    PITON_REQUIRE(g->world >= 1 && g->world <= MAX_PEERS && g->rank >= 0 && g->rank < g->world,
                  "world %d / rank %d outside 1..%d", g->world, g->rank, MAX_PEERS);
    PITON_REQUIRE(g->row_offset >= 0 && g->ldc >= a->N && g->ldc % 4 == 0, "bad row_offset / ldc");
    if (g->multicast_c)
        PITON_REQUIRE((g->multicast_c & 15) == 0, "multicast output is misaligned");
    else
        for (int i = 0; i < g->world; ++i)
            PITON_REQUIRE(g->peer_c[i] != 0 && (g->peer_c[i] & 15) == 0, "peer output %d is NULL or misaligned", i);
    if (a->M == 0 || a->N == 0 || a->grid_x == 0) return PITON_B200_OK;
    PITON_REQUIRE(a->a && a->b, "NULL pointer");
    if (!use_tc(a))
        return set_error(PITON_B200_ENOTSUP, "the all-gather matmul runs on the tensor-core path only "
                                             "(full grid, no QPU rounding, M, N >= 128)");
    size_t need = tc_gemm_workspace_bytes(tc_shape(a));
    if (a->workspace_bytes < need || !a->workspace)
        return set_error(PITON_B200_EWORKSPACE, "matmul needs %zu bytes of workspace, got %llu", need,
                         (unsigned long long)a->workspace_bytes);
    TcGemmShape t = tc_shape(a);
    t.world = g->world;
    t.rank = g->rank;
    t.row_offset = g->row_offset;
    t.ldc_peer = g->ldc;
    for (int i = 0; i < g->world; ++i) t.peer_c[i] = reinterpret_cast<float *>(g->peer_c[i]);
    t.multicast_c = reinterpret_cast<float *>(g->multicast_c);
    return tc_gemm(t, reinterpret_cast<void *>(a->workspace), as_stream(stream));
}

// ---------------------------------------------------------------------------
// Matmul on host buffers with the copies pipelined against the GEMM.
//
// The reference's launch copies every array to the device, runs the kernel
// and copies every array back, one after the other (run_emulator,
// piton/runtime/launcher.py:168-214).  Here A is cut into row blocks: B goes
// over PCIe first, then A's blocks, each on a copy stream; the GEMM of block i
// starts as soon as its rows have landed (B split once, by the first block's
// call) and C's block i goes back on a second copy stream while block i + 1
// computes.  The call's stream waits for the last D2H, so it completes like
// any other entry point.  The result is bit-identical to
// piton_b200_matmul_f32: each element of C is the same dot product whatever
// block its row falls in.
// ---------------------------------------------------------------------------

namespace {

constexpr int HOST_MAX_BLOCKS = 16;
constexpr int64_t HOST_MIN_BLOCK_ROWS = 1024;

struct HostPipe {
    cudaStream_t h2d = nullptr, d2h = nullptr;
    cudaEvent_t start = nullptr, b_in = nullptr, done = nullptr;
    cudaEvent_t a_in[HOST_MAX_BLOCKS] = {}, c_out[HOST_MAX_BLOCKS] = {};
};

// Row blocks of A / C: multiples of 128 rows, at least HOST_MIN_BLOCK_ROWS, at
// most HOST_MAX_BLOCKS of them; a tail under 128 rows joins the block before it.
// Every block has at least 128 rows (the tensor-core path's minimum).
int host_blocks(int64_t M, int64_t *start, int64_t *rows) {
    int64_t per = cdiv(cdiv(M, (int64_t)HOST_MAX_BLOCKS), (int64_t)128) * 128;
    if (per < HOST_MIN_BLOCK_ROWS) per = HOST_MIN_BLOCK_ROWS;
    int n = (int)cdiv(M, per);
    if (n > 1 && M - (int64_t)(n - 1) * per < 128) --n;
    for (int i = 0; i < n; ++i) {
        start[i] = (int64_t)i * per;
        rows[i] = (i == n - 1) ? M - start[i] : per;
    }
    // Nothing overlaps the last block's GEMM and D2H, so cut it in halves down to
    // ~256 rows (1024 -> 512, 256, 256): the pipeline's tail shrinks to a small block.
    if (n >= 2) {
        int64_t s0 = start[n - 1], rem = rows[n - 1];
        --n;
        while (rem > 256 && n < HOST_MAX_BLOCKS - 1) {
            const int64_t piece = cdiv(cdiv(rem, (int64_t)2), (int64_t)128) * 128;
            if (rem - piece < 128) break;
            start[n] = s0;
            rows[n] = piece;
            ++n;
            s0 += piece;
            rem -= piece;
        }
        start[n] = s0;
        rows[n] = rem;
        ++n;
    }
    return n;
}

size_t align1k(size_t b) { return (b + 1023) / 1024 * 1024; }

// Byte offsets of the device copies of B, A, C and the split scratch in the workspace.
// An operand already in the current device's memory is used in place (no copy, no room).
struct HostLayout {
    size_t b, a, c, split, total;
    bool dev_a, dev_b, dev_c;
};

bool on_this_device(uint64_t p) {
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, reinterpret_cast<const void *>(p)) != cudaSuccess) {
        cudaGetLastError();   // an unknown host pointer: not device memory
        return false;
    }
    int dev = -1;
    cudaGetDevice(&dev);
    return at.type == cudaMemoryTypeDevice && at.device == dev;
}

bool host_layout(const piton_matmul_args *a, HostLayout *L, int *n_blocks, int64_t *start, int64_t *rows) {
    if (a->flags != 0) return false;
    if (a->grid_x < grouped_tiles(a->M, a->N, a->block_m, a->block_n)) return false;
    if (a->stride_am != a->K || a->stride_ak != 1 || a->stride_bk != a->N || a->stride_bn != 1 ||
        a->stride_cm != a->N || a->stride_cn != 1)
        return false;
    int n = host_blocks(a->M, start, rows);
    size_t split = 0;
    for (int i = 0; i < n; ++i) {
        TcGemmShape t = tc_shape(a);
        t.M = rows[i];
        if (!tc_gemm_supported(t)) return false;
        size_t need = tc_gemm_workspace_bytes(t);
        if (need > split) split = need;
    }
    L->dev_a = on_this_device(a->a);
    L->dev_b = on_this_device(a->b);
    L->dev_c = on_this_device(a->c);
    L->b = 0;
    L->a = L->b + (L->dev_b ? 0 : align1k((size_t)a->K * a->N * 4));
    L->c = L->a + (L->dev_a ? 0 : align1k((size_t)a->M * a->K * 4));
    L->split = L->c + (L->dev_c ? 0 : align1k((size_t)a->M * a->N * 4));
    L->total = L->split + split;
    *n_blocks = n;
    return true;
}

HostPipe *host_pipe(int *rc) {
    static std::mutex mu;
    static HostPipe pipes[64];
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess || dev < 0 || dev >= 64) {
        *rc = set_error(PITON_B200_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(err));
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(mu);
    HostPipe &p = pipes[dev];
    if (!p.h2d) {
        HostPipe q;
        bool ok = cudaStreamCreateWithFlags(&q.h2d, cudaStreamNonBlocking) == cudaSuccess &&
                  cudaStreamCreateWithFlags(&q.d2h, cudaStreamNonBlocking) == cudaSuccess &&
                  cudaEventCreateWithFlags(&q.start, cudaEventDisableTiming) == cudaSuccess &&
                  cudaEventCreateWithFlags(&q.b_in, cudaEventDisableTiming) == cudaSuccess &&
                  cudaEventCreateWithFlags(&q.done, cudaEventDisableTiming) == cudaSuccess;
        for (int i = 0; ok && i < HOST_MAX_BLOCKS; ++i)
            ok = cudaEventCreateWithFlags(&q.a_in[i], cudaEventDisableTiming) == cudaSuccess &&
                 cudaEventCreateWithFlags(&q.c_out[i], cudaEventDisableTiming) == cudaSuccess;
        if (!ok) {
            *rc = set_error(PITON_B200_ECUDA, "creating the copy streams: %s", cudaGetErrorString(cudaGetLastError()));
            return nullptr;
        }
        p = q;
    }
    *rc = PITON_B200_OK;
    return &p;
}

}  // namespace

extern "C" size_t piton_b200_matmul_host_workspace_size(const piton_matmul_args *a) {
    if (check_matmul(a) != PITON_B200_OK) return 0;
    HostLayout L;
    int n = 0;
    int64_t start[HOST_MAX_BLOCKS], rows[HOST_MAX_BLOCKS];
    if (a->M == 0 || a->N == 0 || !host_layout(a, &L, &n, start, rows)) return 0;
    return L.total;
}

extern "C" int piton_b200_matmul_f32_host(const piton_matmul_args *a, void *stream) {
    int rc = check_matmul(a);
    if (rc) return rc;
    if (a->M == 0 || a->N == 0 || a->grid_x == 0) return PITON_B200_OK;
    PITON_REQUIRE(a->a && a->b && a->c, "NULL pointer");
    HostLayout L;
    int n = 0;
    int64_t start[HOST_MAX_BLOCKS], rows[HOST_MAX_BLOCKS];
    if (!host_layout(a, &L, &n, start, rows))
        return set_error(PITON_B200_ENOTSUP, "the host-buffer matmul needs dense row-major A, B, C, a grid that "
                                             "covers C, no flags, and blocks the tensor-core path takes");
    if (!a->workspace || a->workspace_bytes < L.total)
        return set_error(PITON_B200_EWORKSPACE, "host matmul needs %zu bytes of workspace, got %llu", L.total,
                         (unsigned long long)a->workspace_bytes);
    // C must not share memory with A or B: its blocks go back while later A blocks are still copied in
    const uintptr_t c0 = a->c, c1 = a->c + (uintptr_t)a->M * a->N * 4;
    const uintptr_t a0 = a->a, a1 = a->a + (uintptr_t)a->M * a->K * 4;
    const uintptr_t b0 = a->b, b1 = a->b + (uintptr_t)a->K * a->N * 4;
    PITON_REQUIRE((c1 <= a0 || a1 <= c0) && (c1 <= b0 || b1 <= c0), "C overlaps A or B");
    HostPipe *p = host_pipe(&rc);
    if (!p) return rc;
    cudaStream_t s = as_stream(stream);
    uint8_t *ws = reinterpret_cast<uint8_t *>(a->workspace);
    float *dB = L.dev_b ? reinterpret_cast<float *>(a->b) : reinterpret_cast<float *>(ws + L.b);
    float *dA = L.dev_a ? reinterpret_cast<float *>(a->a) : reinterpret_cast<float *>(ws + L.a);
    float *dC = L.dev_c ? reinterpret_cast<float *>(a->c) : reinterpret_cast<float *>(ws + L.c);
    const float *hA = reinterpret_cast<const float *>(a->a), *hB = reinterpret_cast<const float *>(a->b);
    float *hC = reinterpret_cast<float *>(a->c);

    // the copy streams start after everything already queued on the call's stream
    PITON_CUDA(cudaEventRecord(p->start, s));
    PITON_CUDA(cudaStreamWaitEvent(p->h2d, p->start, 0));
    PITON_CUDA(cudaStreamWaitEvent(p->d2h, p->start, 0));
    if (!L.dev_b) PITON_CUDA(cudaMemcpyAsync(dB, hB, (size_t)a->K * a->N * 4, cudaMemcpyDefault, p->h2d));
    PITON_CUDA(cudaEventRecord(p->b_in, p->h2d));
    for (int i = 0; i < n; ++i) {
        if (!L.dev_a)
            PITON_CUDA(cudaMemcpyAsync(dA + start[i] * a->K, hA + start[i] * a->K, (size_t)rows[i] * a->K * 4,
                                       cudaMemcpyDefault, p->h2d));
        PITON_CUDA(cudaEventRecord(p->a_in[i], p->h2d));
    }
    PITON_CUDA(cudaStreamWaitEvent(s, p->b_in, 0));
    for (int i = 0; i < n; ++i) {
        PITON_CUDA(cudaStreamWaitEvent(s, p->a_in[i], 0));
        TcGemmShape t = tc_shape(a);
        t.a = dA + start[i] * a->K;
        t.b = dB;
        t.c = dC + start[i] * a->N;
        t.M = rows[i];
        t.split_b = (i == 0);
        if ((rc = tc_gemm(t, ws + L.split, s)) != PITON_B200_OK) return rc;
        PITON_CUDA(cudaEventRecord(p->c_out[i], s));
        PITON_CUDA(cudaStreamWaitEvent(p->d2h, p->c_out[i], 0));
        if (!L.dev_c)
            PITON_CUDA(cudaMemcpyAsync(hC + start[i] * a->N, dC + start[i] * a->N, (size_t)rows[i] * a->N * 4,
                                       cudaMemcpyDefault, p->d2h));
    }
    PITON_CUDA(cudaEventRecord(p->done, p->d2h));
    PITON_CUDA(cudaStreamWaitEvent(s, p->done, 0));
    return PITON_B200_OK;
}
