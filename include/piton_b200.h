/*
 * piton_b200.h - C ABI of libpiton_b200.so, the B200 (sm_100a) backend of the
 * PIton `kernel[grid](..., device="b200")` launch.
 *
 * Every operator entry point takes one argument struct (device pointers as
 * uint64_t, sizes and strides in ELEMENTS as int64_t, the launch's grid and
 * constexprs) and a CUDA stream (`void*`, NULL = the legacy default stream),
 * enqueues its kernels and returns without synchronising.  The shape follows
 * the reference's AOT launcher `<sym>_launch(const <sym>_args_t*, gx, gy, gz)`
 * (piton/tools/compile.py:71-90, pi/runtime/piton_rt.h:37) except that the
 * grid travels inside the struct and the return value is a status code
 * instead of elapsed microseconds (time with CUDA events around the call).
 *
 * Status codes are 0 (ok) or one of the negative PITON_B200_E* values; the
 * calling thread's last error message is available from
 * piton_b200_last_error().  Pointer arguments follow the reference's launch
 * semantics (piton/runtime/launcher.py:66-95): a pointer is the address the
 * kernel indexes from, so a negative row stride addresses memory below it.
 *
 * Threading: the library keeps no per-call global state except the calling
 * thread's error message and per-device caches (SM count, kernel attributes),
 * so one host thread per device may call it concurrently.
 */
#ifndef PITON_B200_H
#define PITON_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PITON_B200_ABI_VERSION 1

#if defined(__GNUC__)
#define PITON_B200_API __attribute__((visibility("default")))
#else
#define PITON_B200_API
#endif

/* status codes */
#define PITON_B200_OK 0
#define PITON_B200_EINVAL (-1)     /* bad argument: shape, stride, pointer, flag */
#define PITON_B200_ECUDA (-2)      /* a CUDA runtime call failed */
#define PITON_B200_ETIMEOUT (-3)   /* a bounded wait ran out */
#define PITON_B200_ENOTSUP (-4)    /* no B200 implementation for this constexpr combination */
#define PITON_B200_ENOMEM (-5)     /* allocation failed */
#define PITON_B200_EWORKSPACE (-6) /* workspace missing or smaller than *_workspace_size() */

/* flags (bitwise or) */
#define PITON_B200_QPU_ROUNDING 0x1u /* reproduce the QPU's float semantics bit for bit: round-toward-zero
                                        adds and multiplies, no FMA, sequential-k dots, denormals read and
                                        written as +0 (piton/qpu/emulator.py:137-212). add, matmul, dense. */
#define PITON_B200_FORCE_SIMT 0x2u   /* matmul/dense/attention: take the CUDA-core path even where tensor cores apply */
#define PITON_B200_CUDA_GRAPH 0x4u   /* tinygpt_generate: capture the per-position launches into a CUDA graph once
                                        per distinct argument set and replay it with one graph launch afterwards */

/* ---- runtime (replaces pi/runtime/piton_rt.h:37-107: allocation, launch, sync, timers) ---- */

PITON_B200_API int piton_b200_abi_version(void);
PITON_B200_API const char *piton_b200_last_error(void);
/* Kernels this library has launched since it was loaded (all threads). */
PITON_B200_API uint64_t piton_b200_launch_count(void);
/* Make `device` current for the calling thread and create its context. */
PITON_B200_API int piton_b200_init(int device);
PITON_B200_API int piton_b200_device_count(int *count);
/* The calling thread's current device (cudaGetDevice). */
PITON_B200_API int piton_b200_get_device(int *device);
PITON_B200_API int piton_b200_malloc(uint64_t *ptr, size_t bytes);
PITON_B200_API int piton_b200_free(uint64_t ptr);
PITON_B200_API int piton_b200_memcpy_h2d(uint64_t dst, const void *src, size_t bytes, void *stream);
PITON_B200_API int piton_b200_memcpy_d2h(void *dst, uint64_t src, size_t bytes, void *stream);
PITON_B200_API int piton_b200_memset(uint64_t dst, int value, size_t bytes, void *stream);
/* Wait for `stream` with a deadline: polls cudaStreamQuery, returns PITON_B200_ETIMEOUT
   after `timeout_s` seconds instead of blocking for ever
   (the counterpart of piton_rt.c:150-189's 20 s launch timeout). */
PITON_B200_API int piton_b200_stream_wait(void *stream, double timeout_s);
/* Device-side status of the current device's tensor-core kernels, then reset to 0:
   0 = ok, else the bounded wait that ran out (1 producer, 2 MMA, 3 epilogue, 4 drain).
   Those kernels never trap or spin for ever: they record this, drain and return. */
PITON_B200_API int piton_b200_device_status(int *status);

/* ---- vector add: examples/kernels.py:6-15 add_kernel ---- */
typedef struct {
    uint64_t x, y, out;   /* float* */
    int64_t n_elements;
    int64_t block_size;   /* BLOCK_SIZE constexpr */
    int64_t grid_x;       /* programs launched: elements [0, min(n, grid_x*BLOCK_SIZE)) are written */
    uint32_t flags;       /* PITON_B200_QPU_ROUNDING */
    uint32_t _pad;
} piton_add_args;
PITON_B200_API int piton_b200_add_f32(const piton_add_args *args, void *stream);

/* ---- fused row softmax: examples/kernels.py:60-76 softmax_kernel ---- */
typedef struct {
    uint64_t out, in;     /* float* */
    int64_t in_row_stride, out_row_stride, n_cols;
    int64_t block_size;   /* BLOCK_SIZE constexpr: columns >= BLOCK_SIZE are neither read nor written */
    int64_t grid_x;       /* rows = programs launched */
    uint32_t flags;       /* PITON_B200_QPU_ROUNDING: the QPU float model, bit for bit (ALU exp, Newton
                             reciprocal, 16-lane sum); otherwise IEEE expf and division */
    uint32_t _pad;
} piton_softmax_args;
PITON_B200_API int piton_b200_softmax_f32(const piton_softmax_args *args, void *stream);

/* ---- grouped tutorial matmul: examples/kernels.py:18-57 matmul_kernel ---- */
typedef struct {
    uint64_t a, b, c;     /* float* */
    int64_t M, N, K;
    int64_t stride_am, stride_ak, stride_bk, stride_bn, stride_cm, stride_cn;
    int64_t block_m, block_n, block_k, group_m;   /* constexprs */
    int64_t grid_x;       /* programs launched (grouped pid order decides which C tiles exist) */
    uint64_t workspace;   /* device scratch for the tensor-core path, >= piton_b200_matmul_workspace_size() */
    uint64_t workspace_bytes;
    uint32_t flags;       /* PITON_B200_QPU_ROUNDING, PITON_B200_FORCE_SIMT */
    uint32_t _pad;
} piton_matmul_args;
/* Bytes of workspace the call needs (0 when it takes the CUDA-core path). */
PITON_B200_API size_t piton_b200_matmul_workspace_size(const piton_matmul_args *args);
PITON_B200_API int piton_b200_matmul_f32(const piton_matmul_args *args, void *stream);

/* The same matmul for callers that cannot allocate device memory (hosts whose device memory is
   fixed at start-up, plugin hosts that own every allocation, processes whose memory is all held
   by another allocator's pool).  It has no counterpart in the reference.  The tensor-core path's scratch comes from one static device
   array of PITON_B200_NOALLOC_SCRATCH_BYTES inside this library (held by every GPU that loads
   it, until exit) instead of args->workspace, which is ignored; the call allocates nothing.
   Only tensor-core-path problems whose scratch would exceed that size are rejected, with
   PITON_B200_EINVAL; problems that take the CUDA-core path (QPU rounding, FORCE_SIMT, a partial
   grid, M or N below 128) need no scratch and run at any size.  The first call in a CUDA context
   on a device looks the array's address up (cudaGetSymbolAddress; again after cudaDeviceReset),
   so make it before any stream capture.  All calls share the array: calls that overlap on the
   GPU race. */
#define PITON_B200_NOALLOC_SCRATCH_BYTES (32u << 20)
PITON_B200_API int piton_b200_matmul_f32_noalloc(const piton_matmul_args *args, void *stream);

/* The same matmul on HOST buffers, replacing the copy-in / launch / copy-back sequence of the
   reference's launch (run_emulator, piton/runtime/launcher.py:168-214) for this operator: args->a, b, c are
   host addresses (pinned memory makes the copies asynchronous; pageable memory works, each copy then waits
   for the host), A [M,K], B [K,N], C [M,N] dense row-major (stride_am == K, stride_ak == 1, stride_bk == N,
   stride_bn == 1, stride_cm == N, stride_cn == 1), a grid that covers every tile and no flags, so that every
   element of C is written.  B is copied first, then A in row blocks on a copy stream; each block's GEMM
   starts when its rows have landed and its C rows go back on a second copy stream while the next block
   computes.  An operand already in the current device's memory is used in place (no copy), so host
   and device operands mix (e.g. host A and C with a device-resident B).  Bit-identical to
   piton_b200_matmul_f32.  args->workspace: device scratch of
   piton_b200_matmul_host_workspace_size() bytes (device copies of A, B, C and the split operands; 0 when the
   problem does not qualify, and the call then returns PITON_B200_ENOTSUP).  C must not overlap A or B.
   Enqueues on `stream` like every entry point: the host buffers must stay valid until it has finished.
   One host thread per device (the copy streams are per device). */
PITON_B200_API size_t piton_b200_matmul_host_workspace_size(const piton_matmul_args *args);
PITON_B200_API int piton_b200_matmul_f32_host(const piton_matmul_args *args, void *stream);

/* ---- matmul sharded by M rows with the output all-gather fused into the GEMM epilogue ----
   No counterpart in the reference (it runs on one device); this is the north star's
   "matmul by M-tiles + all-gather" as one kernel: this rank computes rows
   [row_offset, row_offset + args->M) of the full C (args->c and stride_cm/cn are ignored), and
   every finished tile is stored into each rank's full row-major C (peer_c[r], row stride ldc)
   through NVLink peer stores.  peer_c holds device pointers valid in this process: the own
   buffer and the others opened with piton_b200_ipc_open (or symmetric-memory peer mappings).  Tensor-core path only (ENOTSUP
   otherwise).  Every rank must pass a barrier after its call before C is read anywhere. */
typedef struct {
    uint64_t peer_c[8];
    int32_t world, rank;
    int64_t row_offset;
    int64_t ldc;
    uint64_t multicast_c; /* 0, or an NVSwitch multicast address bound to every rank's full C (16-byte
                             aligned): each tile is then stored once with multimem.st, which the switch
                             writes into all ranks' C; peer_c is not used */
} piton_allgather_args;
PITON_B200_API int piton_b200_matmul_allgather_f32(const piton_matmul_args *args, const piton_allgather_args *g,
                                                   void *stream);
/* All-gather of equal pieces without NCCL, for the other operators' shards (softmax rows, attention
   heads, add ranges, MLP / TinyGPT batch rows): this rank's `bytes` at `src` are stored into
   peer_c[r] + rank * bytes for every r < world (the own buffer included) with 16-byte peer stores
   (byte stores when a pointer or `bytes` is not 16-byte aligned).  row_offset, ldc and multicast_c
   are not used.  No counterpart in the reference (it runs on one device); it stands beside the
   NCCL all-gather the Python path uses.  Every rank must pass a barrier after its call before the
   output is read anywhere. */
PITON_B200_API int piton_b200_allgather(const piton_allgather_args *g, uint64_t src, size_t bytes, void *stream);

/* Softmax sharded by rows and vector add sharded by element ranges, each with the output all-gather
   fused into the kernel (the north star's "softmax by rows / add by elements + all-gather" as one
   kernel per rank).  No counterpart in the reference (it runs on one device).  Softmax: this rank
   computes rows [row_offset, row_offset + args->grid_x) of the full output and stores each finished
   row into row row_offset + r (row stride ldc) of every rank's full output peer_c[*]; rows
   16-byte aligned, n_cols a multiple of 4 up to 32768.  Add: this rank computes elements
   [row_offset, row_offset + n) (n = min(n_elements, grid_x * BLOCK_SIZE)) and stores them at the
   same offsets of every rank's full output; IEEE rounding, 16-byte aligned inputs, n and row_offset
   multiples of 4.  args->out is not used; multicast_c is not used.  Every rank must pass a barrier
   after its call before the output is read anywhere. */
PITON_B200_API int piton_b200_softmax_allgather_f32(const piton_softmax_args *args, const piton_allgather_args *g,
                                                    void *stream);
PITON_B200_API int piton_b200_add_allgather_f32(const piton_add_args *args, const piton_allgather_args *g,
                                                void *stream);

/* CUDA IPC of a cudaMalloc'd buffer (64-byte handle) for the peer pointers above. */
PITON_B200_API int piton_b200_ipc_handle(uint64_t ptr, void *handle);
PITON_B200_API int piton_b200_ipc_open(const void *handle, uint64_t *ptr);
PITON_B200_API int piton_b200_ipc_close(uint64_t ptr);

/* ---- dense layer Y = X W (+b) (ReLU): examples/nn_kernels.py:23-74 dense_layer_kernel ---- */
typedef struct {
    uint64_t x, w, bias, y;  /* float*: X[M,K], W[K,N], bias[N], Y[M,N], contiguous row-major */
    int64_t M, N, K;
    int64_t block_m, block_n, block_k, group_m;
    int64_t grid_x;
    int32_t add_bias, relu;
    uint32_t flags;
    uint32_t _pad;
} piton_dense_args;
PITON_B200_API int piton_b200_dense_f32(const piton_dense_args *args, void *stream);

/* ---- digits MLP 64->128->64->16 in one launch: examples/digits_model.py:120-139 ----
   images: uint8 intensities 0..16 (x = v/16) when `images_u8` is set, else float 0..1.
   logits[M,16] always written; argmax of the first `n_classes` logits into pred[M] when pred != 0. */
typedef struct {
    uint64_t images;      /* uint8_t* or float* [M,64] */
    uint64_t w1, b1, w2, b2, w3, b3;   /* float*: [64,128],[128],[128,64],[64],[64,16],[16] */
    uint64_t logits;      /* float* [M,16] */
    uint64_t pred;        /* int32_t* [M] or 0 */
    int64_t M;
    int32_t images_u8, n_classes;
    uint32_t flags;
    uint32_t _pad;
} piton_mlp_args;
PITON_B200_API int piton_b200_mlp_f32(const piton_mlp_args *args, void *stream);

/* ---- causal / full attention: examples/attention.py:75-113 attn_fwd_kernel ----
   Q, V, Out rows [n_ctx, head_dim] with row strides; K through stride_kn (key) and
   stride_kk (dim), so K may be [n_ctx, D] or pre-transposed [D, n_ctx].  Heads advance by
   stride_*h.  Rows >= min(n_ctx, grid_x*block_m) and heads >= grid_y are not written. */
typedef struct {
    uint64_t q, k, v, out;  /* float* */
    double sm_scale;
    int64_t stride_qh, stride_qm, stride_kh, stride_kn, stride_kk, stride_vh, stride_vn, stride_oh, stride_om;
    int64_t n_ctx, head_dim, block_m, block_n;
    int64_t grid_x, grid_y;
    int32_t causal, even_n;
    uint64_t workspace;   /* device scratch for the tensor-core path, >= piton_b200_attention_workspace_size() */
    uint64_t workspace_bytes;
    uint32_t flags;       /* PITON_B200_FORCE_SIMT; PITON_B200_QPU_ROUNDING: the reference program on the QPU
                             float model, bit for bit (BLOCK_N <= 128, a warp per query row) */
    uint32_t _pad;
} piton_attention_args;
/* Bytes of workspace the call needs (0 when it takes the CUDA-core path: HEAD_DIM != 64, n_ctx < 64). */
PITON_B200_API size_t piton_b200_attention_workspace_size(const piton_attention_args *args);
PITON_B200_API int piton_b200_attention_f32(const piton_attention_args *args, void *stream);

/* ---- attention sharded by heads with the output all-gather fused into the kernel ----
   No counterpart in the reference (it runs on one device); the north star's "attention by
   batch x head + all-gather of Out" as one kernel: this rank computes heads
   [row_offset, row_offset + args->grid_y) of the full output (args->out is ignored; q, k, v
   hold this rank's heads), and every finished 128-row block of a head is stored into each
   rank's full output peer_c[r] (head h at peer_c[r] + h * stride_oh, rows stride_om apart,
   the same strides on every rank, multiples of 4 elements): into the own one by the fold
   warps, into the others by a gather warp that trails them (NVLink peer stores, overlapped
   with the next blocks' math).  Tensor-core path only (ENOTSUP otherwise); ldc is not used and
   a nonzero multicast_c is rejected with ENOTSUP.  Every rank must pass a barrier after its
   call before the output is read anywhere. */
PITON_B200_API int piton_b200_attention_allgather_f32(const piton_attention_args *args,
                                                      const piton_allgather_args *g, void *stream);

/* ---- row LayerNorm without affine: tests/test_reroll_reduce.py:199-208 layernorm_kernel ---- */
typedef struct {
    uint64_t x, y;        /* float* */
    int64_t rows, n_cols, x_row_stride, y_row_stride;
    double eps;
    uint32_t flags;
    uint32_t _pad;
} piton_layernorm_args;
PITON_B200_API int piton_b200_layernorm_f32(const piton_layernorm_args *args, void *stream);

/* ---- element-wise float operators: out[i] = f(x[i] (, y[i])) for i < min(n, grid_x * BLOCK) ----
   op: 0 copy (examples/primitive_kernels.py:12-17 copy_kernel), 1 mul (examples/elementwise.py:5-9 mul_kernel),
   2 fma x*alpha + y with two roundings (primitive_kernels.py:20-27 fma_kernel), 3 scaled ReLU x > 0 ? x*alpha : 0
   (examples/kernels.py:79-85), 4 exp2, 5 log2, 6 1/x, 7 rsqrt, 8 exp, 9 sqrt (examples/sfu_tests.py sfu_kernel
   OP 0-5), 10 natural log (primitive_kernels.py log_kernel), 11 sigmoid 1 / (1 + exp(-x)), each step
   rounded as tl.sigmoid composes it (piton/language/core.py:787-790).  QPU rounding: ops 0-3. */
typedef struct {
    uint64_t x, y, out;   /* float*; y only for mul and fma */
    int64_t n_elements, block_size, grid_x;
    double alpha;
    int32_t op;
    uint32_t flags;
} piton_elementwise_args;
PITON_B200_API int piton_b200_elementwise_f32(const piton_elementwise_args *args, void *stream);

/* ---- exact 32-bit // and % (examples/primitive_kernels.py:30-38 idiv_kernel): C truncation semantics,
   int32 (is_signed; INT_MIN / -1 = INT_MIN rem 0) or uint32; a zero divisor gives q = all ones, r = x. ---- */
typedef struct {
    uint64_t x, y, q, r;  /* int32_t* or uint32_t* */
    int64_t n_elements, block_size, grid_x;
    int32_t is_signed;
    uint32_t flags;
} piton_idiv_args;
PITON_B200_API int piton_b200_idiv_i32(const piton_idiv_args *args, void *stream);

/* ---- row sum / row max (examples/kernels.py:88-96 row_sum_kernel, primitive_kernels.py:41-50 row_max_kernel):
   out[r] for r < grid_x*BLOCK_M over the ceil(n_cols/BLOCK_N)*BLOCK_N columns the reference loads. ---- */
typedef struct {
    uint64_t x, out;
    int64_t n_cols, stride, block_m, block_n, grid_x;
    int32_t reduce;       /* 0 sum, 1 max (from -FLT_MAX) */
    uint32_t flags;
} piton_row_reduce_args;
PITON_B200_API int piton_b200_row_reduce_f32(const piton_row_reduce_args *args, void *stream);

/* ---- tile transpose (examples/primitive_kernels.py:53-66 transpose_kernel): out[c*stride_out + r] =
   x[r*stride_x + c] for the tiles of programs below grid_x. ---- */
typedef struct {
    uint64_t x, out;
    int64_t n_rows, n_cols, stride_x, stride_out, block_m, block_n, grid_x;
    uint32_t flags;
    uint32_t _pad;
} piton_transpose_args;
PITON_B200_API int piton_b200_transpose_f32(const piton_transpose_args *args, void *stream);

/* ---- one Game of Life generation on a torus (examples/life.py:39-147): mode 0 life_kernel (int32 cells,
   BLOCK_R x BLOCK_C tiles in row-major order, tile ids < grid_x), 1 life_rows_kernel (int32 cells, BLOCK-column
   strips on grid axis 0 by ROWS rows on axis 1), 2 life_bits_kernel (32 cells per uint32 word, n_cols = words).
   block_r / block_c: BLOCK_R / BLOCK_C, or ROWS / BLOCK. ---- */
typedef struct {
    uint64_t src, dst;
    int64_t n_rows, n_cols, stride, block_r, block_c, grid_x, grid_y;
    int32_t mode;
    uint32_t flags;
} piton_life_args;
PITON_B200_API int piton_b200_life_step(const piton_life_args *args, void *stream);

/* ---- TinyGPT greedy decoding (a model the reference does not have; built from its pieces:
   dense layers examples/nn_kernels.py:23-74, attention examples/attention.py:75-113, layer norm
   tests/test_reroll_reduce.py:199-208).  Only vocab 65, d_model 128, 4 layers, 4 heads, context
   128 is built.  tokens: int32 [batch, 128]; positions [0, prompt_len) hold the prompt, and
   positions [prompt_len, prompt_len + new_tokens) receive the greedy tokens.  weights: packed fp32,
   piton_b200_tinygpt_weight_floats() floats (layout in csrc/tinygpt.cu).  kv_cache: caller scratch,
   fp32 [4][2][batch][128][128].  logits (optional): fp32 [batch, 65] of the last fed position. ---- */
typedef struct {
    uint64_t weights, kv_cache, tokens, logits;
    int64_t batch, prompt_len, new_tokens;
    int32_t vocab, d_model, n_layer, n_head, ctx;
    uint32_t flags;
} piton_tinygpt_args;
PITON_B200_API int64_t piton_b200_tinygpt_weight_floats(void);
/* flags: 0 or PITON_B200_CUDA_GRAPH.  With the graph flag the launches are captured on an internal stream
   the first time an argument set (every field, pointers included) is seen on a device, instantiated, and
   cached (16 per device, least recently used evicted); every call, the first included, then enqueues one
   cudaGraphLaunch on `stream`.  A replay does exactly what the launches with those arguments would do, so
   the caller's buffers need only be valid at each call, as without the flag. */
PITON_B200_API int piton_b200_tinygpt_generate(const piton_tinygpt_args *args, void *stream);
/* Instantiated graphs cached on the current device; piton_b200_graph_cache_clear() destroys them. */
PITON_B200_API int piton_b200_graph_cache_entries(int *entries);
PITON_B200_API int piton_b200_graph_cache_clear(void);

#ifdef __cplusplus
}
#endif
#endif /* PITON_B200_H */
