// fp32 GEMM on the 5th-generation tensor cores from a split of each operand
// (tutorial matmul, examples/kernels.py:18-57, default rounding mode).
//
// fp32 accuracy from TF32 / BF16 tensor cores: each operand x is split into
// x_hi = x with the low 13 mantissa bits cleared (exactly representable in
// TF32) and x_lo = x - x_hi (exact in fp32, at most 2^-10 |x|), and
//   C = A_hi B_hi + (A_lo B + A B_lo)
// where A_hi B_hi is a kind::tf32 product (exact products) and the bracket is
// one kind::f16 product of bf16 operands, concatenated along k: per group of 8
// k-values the A operand holds [bf16(A_lo), bf16(A)] and the B operand
// [bf16(B), bf16(B_lo)], so one 16-deep bf16 MMA adds A_lo B + A B_lo over the
// same 8 k-values a tf32 MMA covers.  A B_lo + A_lo B = A_hi B_lo + A_lo B_hi +
// 2 A_lo B_lo; with A_lo B_lo below 2^-20 of the product, the bracket carries
// the two cross terms of the classic 3xTF32 split (and the lo x lo term once
// more, at most 2^-20 of the product).  Rounding both operands of a cross term
// to bf16 (8-bit mantissas) costs at most 2^-8 of a term that is itself at most
// 2^-10 of the product: at most 2^-17 + 2^-20 per product, ~2^-19.6 rms, with
// unbiased (round-to-nearest) signs.  A bf16 MMA of depth 16 issues as
// fast as a tf32 MMA of depth 8, so each 8-deep k-step takes two MMAs instead
// of 3xTF32's three, from the same shared-memory bytes.
//
// Two kernels per call:
//  1. split: reads A and B with their (arbitrary) element strides and writes
//     A_hi as [M, ld] fp32 (ld = K rounded up to 4) and the cross operand A_x
//     as [M, ldx] bf16 (ldx = 2 x K rounded up to 16), and B_hi, B_x
//     transposed as [N, ld] / [N, ldx] (K-major), into the caller's workspace.
//     HBM-bound.  A row-major A is its own A_hi (see below).
//  2. gemm: persistent, one CTA per SM (320 threads): warp 0 issues TMA tile
//     loads (128x16 A tiles, 256x16 B tiles (fp32) and the bf16 tiles of the
//     same 16 k-values, 64-byte swizzle, 4-stage mbarrier ring), warp 1 owns
//     512 TMEM columns (two 128x256 fp32 accumulators) and issues, from one
//     thread, tcgen05.mma kind::tf32 128x256x8 and kind::f16 128x256x16,
//     warps 2-9 drain finished accumulators with tcgen05.ld.
//
// The tensor cores add into the TMEM accumulator with truncation, and that
// bias grows with the number of accumulation steps (at K = 8192 it is ~30x
// the error of an fp32 FFMA loop).  So an accumulator only ever holds a chunk
// of KC = 256 k-values: the MMA warp alternates between the two TMEM
// buffers per chunk, and the epilogue warps add every finished chunk into an
// fp32 register sum (round to nearest), then store the tile with C's element
// strides.  The error is then at the level of an fp32 FFMA loop.
// Every mbarrier wait is bounded (2 s of global time): on expiry the kernel
// records a status word, drains its own TMA copies and MMAs, frees TMEM and
// returns.
#include <algorithm>
#include <vector>

#include <cuda_bf16.h>

#include "attention.cuh"
#include "common.cuh"
#include "gemm_tc.cuh"
#include "sm100.cuh"
#include "split.cuh"

namespace piton {

using namespace sm100;

__device__ int g_tc_status = 0;

namespace {

constexpr int BM = 128, BK = 16, STAGES = 4;
constexpr int THREADS = 320;
constexpr int EPI_WARPS = 8;
constexpr int KC_BLOCKS = 16;   // k-blocks of BK per accumulation chunk (KC = 256)
constexpr uint32_t A_TILE_BYTES = BM * BK * 4;   // 8 KB: 128 rows x 16 fp32, or x 32 bf16 (cross operand)
// BN (tile width along N) is 256, or 224 where that packs the tiles into fewer
// rounds over the SMs (tile_width()); a B tile is BN x 16 fp32 (14 or 16 KB), and
// its cross tile BN x 32 bf16 as many bytes
__host__ __device__ constexpr uint32_t b_tile_bytes(int bn) { return (uint32_t)bn * BK * 4; }
__host__ __device__ constexpr uint32_t stage_bytes(int bn) { return 2 * A_TILE_BYTES + 2 * b_tile_bytes(bn); }
__host__ __device__ constexpr uint32_t smem_bytes(int bn) { return STAGES * stage_bytes(bn) + 1024 /*barriers*/ + 1024 /*alignment*/; }
constexpr int TMEM_COLS = 512;
constexpr int GROUP_M = 16;

__device__ __forceinline__ float tf32_trunc(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }

// Cross operand of value v (at k) in a row of the bf16 array x: per group of 8
// k-values, positions [16 g, 16 g + 8) hold the first part and [16 g + 8, 16 g + 16)
// the second.  A side: (bf16(lo), bf16(v)); B side: (bf16(v), bf16(lo)), so that one
// 16-deep product of the two adds A_lo B + A B_lo.  Non-finite values contribute 0
// (their high half carries them), finite ones are clamped to the bf16 range.
__device__ __forceinline__ void put_cross(__nv_bfloat16 *xrow, int64_t c, float v, float lo, bool a_side) {
    const int64_t p = 16 * (c >> 3) + (c & 7);
    xrow[p] = a_side ? split_bf16_of(lo) : split_bf16_of(v);
    xrow[p + 8] = a_side ? split_bf16_of(v) : split_bf16_of(lo);
}

// hi[r * ld + c] (if hi) and the cross operand x[r * ldx + ...] from src[r * s_row + c * s_col],
// r < rows, c < cols, through 32 x 32 shared-memory tiles so that both the strided read and the
// write coalesce; k-values from cols up to the next multiple of 8 are written as zeros.
__global__ void __launch_bounds__(256) split_kernel(const float *__restrict__ src, int64_t rows, int64_t cols,
                                                    int64_t s_row, int64_t s_col, float *__restrict__ hi,
                                                    __nv_bfloat16 *__restrict__ x, int64_t ld, int64_t ldx,
                                                    int lanes_along_rows, int a_side) {
    __shared__ float tile[32][33];
    const int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;    // 32 x 8
    for (int j = ty; j < 32; j += 8) {
        int64_t r = lanes_along_rows ? r0 + tx : r0 + j;
        int64_t c = lanes_along_rows ? c0 + j : c0 + tx;
        float v = (r < rows && c < cols) ? src[r * s_row + c * s_col] : 0.0f;
        if (lanes_along_rows) tile[tx][j] = v;
        else tile[j][tx] = v;
    }
    __syncthreads();
    const int64_t cols8 = (cols + 7) / 8 * 8;
    for (int j = ty; j < 32; j += 8) {
        int64_t r = r0 + j, c = c0 + tx;
        if (r < rows && c < cols8) {
            const float v = c < cols ? tile[j][tx] : 0.0f;
            const float h = tf32_trunc(v);
            if (hi && c < cols) hi[r * ld + c] = h;
            put_cross(x + r * ldx, c, v, isfinite(v) ? v - h : 0.0f, a_side != 0);
        }
    }
}

// Row-major A with unit column stride and 16-byte aligned rows: kind::tf32 MMAs ignore
// the low 13 bits of an fp32 operand (the raw value multiplies exactly as its truncated
// high half), so the GEMM reads A_hi straight from the source and only the cross operand
// is written: per thread 4 k-values in (one float4), 4 + 4 bf16 out (two 8-byte stores).
__global__ void __launch_bounds__(256) split_rows_vec4_kernel(const float *__restrict__ src, int64_t rows,
                                                              int64_t cols, int64_t s_row,
                                                              __nv_bfloat16 *__restrict__ x, int64_t ldx) {
    const int64_t q_per_row = (cols + 7) / 8 * 2;   // cols % 4 == 0: whole float4s, up to the 8-group
    const int64_t total = rows * q_per_row;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / q_per_row, c = 4 * (i % q_per_row);
        const float4 v = c < cols ? __ldcs(reinterpret_cast<const float4 *>(src + r * s_row + c))
                                  : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        const float vv[4] = {v.x, v.y, v.z, v.w};
        __align__(8) __nv_bfloat16 lo[4], full[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float h = tf32_trunc(vv[e]);
            lo[e] = split_bf16_of(isfinite(vv[e]) ? vv[e] - h : 0.0f);
            full[e] = split_bf16_of(vv[e]);
        }
        __nv_bfloat16 *p = x + r * ldx + 16 * (c >> 3) + (c & 7);
        *reinterpret_cast<uint2 *>(p) = *reinterpret_cast<const uint2 *>(lo);
        *reinterpret_cast<uint2 *>(p + 8) = *reinterpret_cast<const uint2 *>(full);
    }
}

struct GemmArgs {
    float *c;
    int64_t M, N, K, scm, scn;
    int tiles_m, tiles_n, num_tiles, k_blocks;
    int group;                       // tile rows per group of the tile order (L2 reuse of B)
    int world, rank;                 // world > 0: all-gather epilogue into peer_c
    int64_t row_offset, ldc_peer;
    float *peer_c[MAX_PEERS];
    float *mc_c;                     // multicast all-gather: one multimem store reaches every rank
};

// multimem stores: the NVSwitch writes the value into the memory of every GPU bound
// to the multicast address (relaxed, system scope; the kernel ends with a system fence)
__device__ __forceinline__ void multimem_st_v4(float *addr, float a, float b, float c, float d) {
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b),
                 "f"(c), "f"(d)
                 : "memory");
}
__device__ __forceinline__ void multimem_st(float *addr, float a) {
    asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;" ::"l"(addr), "f"(a) : "memory");
}

__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int group_m, int &tm, int &tn) {
    int per_group = group_m * tiles_n;
    int group = t / per_group;
    int first = group * group_m;
    int gsize = min(tiles_m - first, group_m);
    int in = t % per_group;
    tm = first + in % gsize;
    tn = in / gsize;
}

__device__ __forceinline__ void record_status(int code) { atomicCAS(&g_tc_status, 0, code); }

// All-gather epilogue: rows [row_base + r0, row_base + r1) of finished tile column
// tn, already stored in this rank's own output, are copied to every other rank's
// output (float4 peer stores).  Called by the 256 epilogue threads (`et` = 0..255), a few rows per
// accumulation chunk of the next tile, so the NVLink traffic is spread evenly
// over the MMAs instead of bursting at the end of each tile.
template <int BN>
__device__ __forceinline__ void copy_rows_to_peers(const GemmArgs &args, int64_t row_base, int tn, int r0, int r1,
                                                   int et) {
    const float *src_base = args.peer_c[args.rank];
    const int64_t col_base = (int64_t)tn * BN;
    const int per_row = BN / 4;
    for (int i = et; i < (r1 - r0) * per_row; i += 256) {
        const int r = r0 + i / per_row, q = i % per_row;
        const int64_t row = row_base + r;
        const int64_t col = col_base + 4 * q;
        if (row >= args.M || col >= args.N) continue;
        const int64_t off = (args.row_offset + row) * args.ldc_peer + col;
        if (col + 4 <= args.N) {
            float4 v = *reinterpret_cast<const float4 *>(src_base + off);
            for (int p = 1; p < args.world; ++p)
                *reinterpret_cast<float4 *>(args.peer_c[(args.rank + p) % args.world] + off) = v;
        } else {
            for (int j = 0; col + j < args.N; ++j) {
                float v = src_base[off + j];
                for (int p = 1; p < args.world; ++p) args.peer_c[(args.rank + p) % args.world][off + j] = v;
            }
        }
    }
}

template <int BN>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_3xtf32_kernel(const __grid_constant__ CUtensorMap tm_ahi, const __grid_constant__ CUtensorMap tm_ax,
                       const __grid_constant__ CUtensorMap tm_bhi, const __grid_constant__ CUtensorMap tm_bx,
                       GemmArgs args) {
    constexpr uint32_t B_TILE_BYTES = b_tile_bytes(BN);
    constexpr uint32_t STAGE_BYTES = stage_bytes(BN);
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE_BYTES);
    uint64_t *empty = full + STAGES;
    uint64_t *tfull = empty + STAGES;
    uint64_t *tempty = tfull + 2;
    uint64_t *drain = tempty + 2;
    uint64_t *epi_bar = drain + 1;   // the 8 epilogue warps: a finished tile is in the own output
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(epi_bar + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], EPI_WARPS);
        }
        mbar_init(drain, 1);
        mbar_init(epi_bar, EPI_WARPS);
        *abort_flag = 0;
        fence_mbarrier_init();
        prefetch_tmap(&tm_ahi);
        prefetch_tmap(&tm_ax);
        prefetch_tmap(&tm_bhi);
        prefetch_tmap(&tm_bx);
    }
    if (warp == 1) tmem_alloc<TMEM_COLS>(tmem_holder);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    const int kb_total = args.k_blocks;
    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            uint32_t it = 0;
            for (int t = blockIdx.x; t < args.num_tiles && !*abort_flag; t += gridDim.x) {
                int tm, tn;
                tile_coords(t, args.tiles_m, args.tiles_n, args.group, tm, tn);
                for (int kb = 0; kb < kb_total; ++kb, ++it) {
                    uint32_t s = it % STAGES, round = it / STAGES;
                    if (!mbar_wait(&empty[s], (round & 1) ^ 1)) {
                        record_status(STATUS_TIMEOUT_PRODUCER);
                        *abort_flag = 1;
                        break;
                    }
                    uint8_t *st = smem + s * STAGE_BYTES;
                    mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
                    const int kx = kb * BK, kxx = 2 * kb * BK;   // fp32 and bf16 (cross) columns
                    tma_load_2d(st, &tm_ahi, &full[s], kx, tm * BM);
                    tma_load_2d(st + A_TILE_BYTES, &tm_ax, &full[s], kxx, tm * BM);
                    tma_load_2d(st + 2 * A_TILE_BYTES, &tm_bhi, &full[s], kx, tn * BN);
                    tma_load_2d(st + 2 * A_TILE_BYTES + B_TILE_BYTES, &tm_bx, &full[s], kxx, tn * BN);
                }
            }
            // drain: every copy this thread issued has landed before the CTA may exit
            uint32_t first = it > STAGES ? it - STAGES : 0;
            for (uint32_t j = first; j < it; ++j)
                if (!mbar_wait(&full[j % STAGES], (j / STAGES) & 1)) record_status(STATUS_TIMEOUT_DRAIN);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t IDESC = idesc_tf32(BM, BN), IDESC_X = idesc_bf16(BM, BN);
            uint32_t it = 0, chunk = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < args.num_tiles && !*abort_flag; t += gridDim.x) {
                for (int kb0 = 0; ok && kb0 < kb_total; kb0 += KC_BLOCKS, ++chunk) {
                    const int acc = chunk & 1;
                    const uint32_t use = chunk >> 1;
                    if (!mbar_wait(&tempty[acc], (use & 1) ^ 1)) {
                        record_status(STATUS_TIMEOUT_MMA);
                        *abort_flag = 1;
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + acc * BN;
                    const int kb1 = min(kb0 + KC_BLOCKS, kb_total);
                    for (int kb = kb0; kb < kb1; ++kb, ++it) {
                        uint32_t s = it % STAGES, round = it / STAGES;
                        if (!mbar_wait(&full[s], round & 1)) {
                            record_status(STATUS_TIMEOUT_MMA);
                            *abort_flag = 1;
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        uint32_t base = smem_u32(smem + s * STAGE_BYTES);
                        uint32_t a_hi = base, a_x = base + A_TILE_BYTES;
                        uint32_t b_hi = base + 2 * A_TILE_BYTES, b_x = b_hi + B_TILE_BYTES;
#pragma unroll
                        for (int ks = 0; ks < BK / 8; ++ks) {
                            // 8 tf32, or the 16 bf16 of the same 8 k-values: 32 bytes along K in the row
                            uint32_t off = ks * 32;
                            uint64_t dah = smem_desc_kmajor(a_hi + off, 64, LAYOUT_SWIZZLE_64B);
                            uint64_t dax = smem_desc_kmajor(a_x + off, 64, LAYOUT_SWIZZLE_64B);
                            uint64_t dbh = smem_desc_kmajor(b_hi + off, 64, LAYOUT_SWIZZLE_64B);
                            uint64_t dbx = smem_desc_kmajor(b_x + off, 64, LAYOUT_SWIZZLE_64B);
                            uint32_t first = (kb == kb0 && ks == 0) ? 0u : 1u;
                            mma_bf16(d_tmem, dax, dbx, IDESC_X, first);   // A_lo B + A B_lo
                            mma_tf32(d_tmem, dah, dbh, IDESC, 1u);        // A_hi B_hi
                        }
                        mma_commit(&empty[s]);   // stage s free once these MMAs have read it
                    }
                    if (!ok) break;
                    mma_commit(&tfull[acc]);     // chunk ready for the epilogue
                }
            }
            // drain: all MMAs issued by this thread complete before TMEM is freed
            mma_commit(drain);
            if (!mbar_wait(drain, 0)) record_status(STATUS_TIMEOUT_DRAIN);
        }
    } else {
        // ---------------- epilogue (warps 2-9) ----------------
        const int quarter = warp & 3;                 // TMEM lanes [32*quarter, 32*quarter + 32)
        const int half = (warp - 2) >> 2;             // columns [128*half, 128*half + 128)
        float sum[BN / 2];
        uint32_t chunk = 0;
        bool ok = true;
        const int et = threadIdx.x - 64;                      // epilogue thread index 0..255
        const int n_chunks = (kb_total + KC_BLOCKS - 1) / KC_BLOCKS;
        const int rows_per_chunk = (BM + n_chunks - 1) / n_chunks;
        int pend_tm = -1, pend_tn = -1;                       // finished tile still to be sent to peers
        uint32_t tiles_done = 0;
        for (int t = blockIdx.x; ok && t < args.num_tiles; t += gridDim.x) {
            for (int kb0 = 0, ci = 0; kb0 < kb_total; kb0 += KC_BLOCKS, ++chunk, ++ci) {
                const int acc = chunk & 1;
                const uint32_t use = chunk >> 1;
                bool got = !*abort_flag && mbar_wait(&tfull[acc], use & 1);
                if (!__all_sync(0xffffffffu, got)) {   // one decision per warp: tcgen05.ld is warp-wide
                    if (lane == 0) record_status(STATUS_TIMEOUT_EPILOGUE);
                    *abort_flag = 1;
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN + half * (BN / 2);
                if (kb0 == 0) {
#pragma unroll
                    for (int j = 0; j < BN / 2; ++j) sum[j] = 0.0f;
                }
#pragma unroll
                for (int part = 0; part < BN / 2 / 16; ++part) {
                    uint32_t r[16];
                    tmem_ld_32x32b_x16(taddr + part * 16, r);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 16; ++j) sum[part * 16 + j] += __uint_as_float(r[j]);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[acc]);   // TMEM buffer free for the next chunk
                if (args.world > 1 && pend_tm >= 0)
                    copy_rows_to_peers<BN>(args, (int64_t)pend_tm * BM, pend_tn, min(ci * rows_per_chunk, BM),
                                       min((ci + 1) * rows_per_chunk, BM), et);
            }
            if (!ok) break;
            int tm, tn;
            tile_coords(t, args.tiles_m, args.tiles_n, args.group, tm, tn);
            const int64_t row = (int64_t)tm * BM + quarter * 32 + lane;
            if (row < args.M) {
                const int64_t col0 = (int64_t)tn * BN + half * (BN / 2);
                if (args.mc_c) {
                    // multicast all-gather: one store per element, replicated to every rank by the switch
                    float *mrow = args.mc_c + (args.row_offset + row) * args.ldc_peer;
#pragma unroll
                    for (int j = 0; j < BN / 2; j += 4) {
                        if (col0 + j + 4 <= args.N) {
                            multimem_st_v4(mrow + col0 + j, sum[j], sum[j + 1], sum[j + 2], sum[j + 3]);
                        } else {
#pragma unroll
                            for (int q = 0; q < 4; ++q)
                                if (col0 + j + q < args.N) multimem_st(mrow + col0 + j + q, sum[j + q]);
                        }
                    }
                } else if (args.world > 0) {
                    // all-gather epilogue: the tile goes into this rank's own full output now,
                    // and to the other ranks' outputs during the next tile's chunks
                    float *crow = args.peer_c[args.rank] + (args.row_offset + row) * args.ldc_peer;
#pragma unroll
                    for (int j = 0; j < BN / 2; j += 4) {
                        if (col0 + j + 4 <= args.N) {
                            *reinterpret_cast<float4 *>(crow + col0 + j) =
                                make_float4(sum[j], sum[j + 1], sum[j + 2], sum[j + 3]);
                        } else {
#pragma unroll
                            for (int q = 0; q < 4; ++q)
                                if (col0 + j + q < args.N) crow[col0 + j + q] = sum[j + q];
                        }
                    }
                } else {
                    float *crow = args.c + row * args.scm;
                    const bool vec = args.scn == 1 &&
                                     ((reinterpret_cast<uintptr_t>(args.c) | (uintptr_t)(args.scm * 4)) & 15) == 0;
                    if (vec) {
#pragma unroll
                        for (int j = 0; j < BN / 2; j += 4) {
                            if (col0 + j + 4 <= args.N) {
                                *reinterpret_cast<float4 *>(crow + col0 + j) =
                                    make_float4(sum[j], sum[j + 1], sum[j + 2], sum[j + 3]);
                            } else {
#pragma unroll
                                for (int q = 0; q < 4; ++q)
                                    if (col0 + j + q < args.N) crow[col0 + j + q] = sum[j + q];
                            }
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < BN / 2; ++j)
                            if (col0 + j < args.N) crow[(col0 + j) * args.scn] = sum[j];
                    }
                }
            }
            if (args.world > 1 && !args.mc_c) {
                // every epilogue warp has stored its part of the tile (bounded wait, not bar.sync:
                // a warp that gave up must not leave the others waiting for ever)
                __threadfence_block();
                __syncwarp();
                if (lane == 0) mbar_arrive(epi_bar);
                bool got = mbar_wait(epi_bar, tiles_done & 1);
                if (!__all_sync(0xffffffffu, got)) {
                    if (lane == 0) record_status(STATUS_TIMEOUT_EPILOGUE);
                    *abort_flag = 1;
                    ok = false;
                    break;
                }
                pend_tm = tm;
                pend_tn = tn;
            }
            ++tiles_done;
        }
        if (ok && args.world > 1 && pend_tm >= 0)
            copy_rows_to_peers<BN>(args, (int64_t)pend_tm * BM, pend_tn, 0, BM, et);
        if (args.mc_c) __threadfence_system();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc<TMEM_COLS>(tmem_base);
    }
}

// ---- the same GEMM on CTA pairs: tcgen05.mma.cta_group::2 --------------------------------
//
// A cluster of two CTAs on neighbouring SMs computes a 256 x BNP tile: each CTA loads
// its 128 rows of A and its BNP / 2 rows of B^T (hi and lo), the even CTA issues
// tcgen05.mma.cta_group::2 (M = 256, N = BNP), which reads both CTAs' shared memory
// and writes each CTA's 128 rows of the accumulator into its own TMEM.  Per SM a
// 128 x BNP x 8 product then reads 4 KB of A and only BNP / 2 rows of B from shared
// memory (the shared-memory path feeding the tensor core is what bounds the one-CTA
// kernel).  The TMA loads of both CTAs complete on the even CTA's stage barrier; its
// MMA commits (multicast) free the stage in both CTAs and hand finished accumulator
// chunks to both CTAs' epilogue warps, which release the accumulator by arriving on
// the even CTA's barrier.  Waits are bounded as in the one-CTA kernel; the two
// cluster barriers (after set-up, before TMEM is freed) are reached unconditionally.

constexpr int STAGES2 = 6;
constexpr uint32_t A2_TILE_BYTES = BM * BK * 4;   // 8 KB: this CTA's 128 rows
__host__ __device__ constexpr uint32_t b2_tile_bytes(int bnp) { return (uint32_t)(bnp / 2) * BK * 4; }
__host__ __device__ constexpr uint32_t stage2_bytes(int bnp) { return 2 * A2_TILE_BYTES + 2 * b2_tile_bytes(bnp); }
__host__ __device__ constexpr uint32_t smem2_bytes(int bnp) { return STAGES2 * stage2_bytes(bnp) + 1024 + 1024; }

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// shared::cluster address of the same variable in CTA rank 0 of the cluster
__device__ __forceinline__ uint32_t cluster_addr_rank0(const void *p) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(r) : "r"(smem_u32(p)));
    return r;
}
__device__ __forceinline__ void cluster_barrier() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// TMA tile load into this CTA's shared memory, completing on a barrier of the pair (cta_group::2, no multicast)
__device__ __forceinline__ void tma_load_2d_pair(void *dst, const CUtensorMap *map, uint32_t bar_cluster, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
        "[%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void mma_tf32_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0u)
        : "memory");
}
__device__ __forceinline__ void mma_bf16_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0u)
        : "memory");
}
// arrives on `bar` in both CTAs of the pair once this thread's MMAs have completed
__device__ __forceinline__ void mma_commit_pair(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"((uint16_t)3)
        : "memory");
}

template <int BNP>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_3xtf32_2sm_kernel(const __grid_constant__ CUtensorMap tm_ahi, const __grid_constant__ CUtensorMap tm_ax,
                           const __grid_constant__ CUtensorMap tm_bhi, const __grid_constant__ CUtensorMap tm_bx,
                           GemmArgs args) {
    constexpr uint32_t B_TILE = b2_tile_bytes(BNP), STAGE = stage2_bytes(BNP);
    constexpr int HALF = BNP / 2;   // accumulator columns per epilogue warpgroup, and B rows per CTA
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + STAGES2 * STAGE);
    uint64_t *empty = full + STAGES2;
    uint64_t *tfull = empty + STAGES2;
    uint64_t *tempty = tfull + 2;
    uint64_t *drain = tempty + 2;
    uint64_t *epi_bar = drain + 1;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(epi_bar + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES2; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 2 * EPI_WARPS);   // the epilogue warps of both CTAs
        }
        mbar_init(drain, 1);
        mbar_init(epi_bar, EPI_WARPS);
        *abort_flag = 0;
        fence_mbarrier_init();
        prefetch_tmap(&tm_ahi);
        prefetch_tmap(&tm_ax);
        prefetch_tmap(&tm_bhi);
        prefetch_tmap(&tm_bx);
    }
    if (warp == 1) {   // the same warp of both CTAs allocates the pair's TMEM
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    cluster_barrier();   // both CTAs' barriers initialised and TMEM allocated
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;
    const int kb_total = args.k_blocks;

    if (warp == 0) {
        // ---------------- TMA producer (both CTAs) ----------------
        if (lane == 0) {
            uint32_t it = 0;
            for (int t = pair; t < args.num_tiles && !*abort_flag; t += npairs) {
                int tm, tn;
                tile_coords(t, args.tiles_m, args.tiles_n, args.group, tm, tn);
                const int arow = tm * 2 * BM + (int)rank * BM, brow = tn * BNP + (int)rank * HALF;
                for (int kb = 0; kb < kb_total; ++kb, ++it) {
                    const uint32_t s = it % STAGES2, round = it / STAGES2;
                    if (!mbar_wait(&empty[s], (round & 1) ^ 1)) {
                        record_status(STATUS_TIMEOUT_PRODUCER);
                        *abort_flag = 1;
                        break;
                    }
                    uint8_t *st = smem + s * STAGE;
                    const uint32_t bar = cluster_addr_rank0(&full[s]);
                    if (leader) mbar_arrive_expect_tx(&full[s], 2 * STAGE);   // both CTAs' bytes
                    const int kx = kb * BK, kxx = 2 * kb * BK;   // fp32 and bf16 (cross) columns
                    tma_load_2d_pair(st, &tm_ahi, bar, kx, arow);
                    tma_load_2d_pair(st + A2_TILE_BYTES, &tm_ax, bar, kxx, arow);
                    tma_load_2d_pair(st + 2 * A2_TILE_BYTES, &tm_bhi, bar, kx, brow);
                    tma_load_2d_pair(st + 2 * A2_TILE_BYTES + B_TILE, &tm_bx, bar, kxx, brow);
                }
            }
            // drain: every copy of both CTAs completes on the even CTA's stage barriers
            if (leader) {
                const uint32_t first = it > STAGES2 ? it - STAGES2 : 0;
                for (uint32_t j = first; j < it; ++j)
                    if (!mbar_wait(&full[j % STAGES2], (j / STAGES2) & 1)) record_status(STATUS_TIMEOUT_DRAIN);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (even CTA) ----------------
        if (lane == 0 && leader) {
            constexpr uint32_t IDESC = idesc_tf32(2 * BM, BNP), IDESC_X = idesc_bf16(2 * BM, BNP);
            uint32_t it = 0, chunk = 0;
            bool ok = true;
            for (int t = pair; ok && t < args.num_tiles && !*abort_flag; t += npairs) {
                for (int kb0 = 0; ok && kb0 < kb_total; kb0 += KC_BLOCKS, ++chunk) {
                    const int acc = chunk & 1;
                    const uint32_t use = chunk >> 1;
                    if (!mbar_wait(&tempty[acc], (use & 1) ^ 1)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + acc * BNP;
                    const int kb1 = min(kb0 + KC_BLOCKS, kb_total);
                    for (int kb = kb0; kb < kb1; ++kb, ++it) {
                        const uint32_t s = it % STAGES2, round = it / STAGES2;
                        if (!mbar_wait(&full[s], round & 1)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t base = smem_u32(smem + s * STAGE);
                        const uint32_t a_hi = base, a_x = base + A2_TILE_BYTES;
                        const uint32_t b_hi = base + 2 * A2_TILE_BYTES, b_x = b_hi + B_TILE;
#pragma unroll
                        for (int ks = 0; ks < BK / 8; ++ks) {
                            const uint32_t off = ks * 32;
                            const uint64_t dah = smem_desc_kmajor(a_hi + off, 64, LAYOUT_SWIZZLE_64B);
                            const uint64_t dax = smem_desc_kmajor(a_x + off, 64, LAYOUT_SWIZZLE_64B);
                            const uint64_t dbh = smem_desc_kmajor(b_hi + off, 64, LAYOUT_SWIZZLE_64B);
                            const uint64_t dbx = smem_desc_kmajor(b_x + off, 64, LAYOUT_SWIZZLE_64B);
                            const uint32_t first = (kb == kb0 && ks == 0) ? 0u : 1u;
                            mma_bf16_pair(d_tmem, dax, dbx, IDESC_X, first);   // A_lo B + A B_lo
                            mma_tf32_pair(d_tmem, dah, dbh, IDESC, 1u);        // A_hi B_hi
                        }
                        mma_commit_pair(&empty[s]);   // stage s free in both CTAs
                    }
                    if (!ok) break;
                    mma_commit_pair(&tfull[acc]);     // chunk ready for both CTAs' epilogues
                }
            }
            if (!ok) {
                record_status(STATUS_TIMEOUT_MMA);
                *abort_flag = 1;
            }
            asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             smem_u32(drain))
                         : "memory");
            if (!mbar_wait(drain, 0)) record_status(STATUS_TIMEOUT_DRAIN);
        }
    } else {
        // ---------------- epilogue (warps 2-9 of both CTAs): this CTA's 128 rows ----------------
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2;
        float sum[HALF];
        uint32_t chunk = 0;
        bool ok = true;
        const int et = threadIdx.x - 64;
        const int n_chunks = (kb_total + KC_BLOCKS - 1) / KC_BLOCKS;
        const int rows_per_chunk = (BM + n_chunks - 1) / n_chunks;
        const uint32_t tempty_pair[2] = {cluster_addr_rank0(&tempty[0]), cluster_addr_rank0(&tempty[1])};
        int pend_tn = -1;
        int64_t pend_row = -1;
        uint32_t tiles_done = 0;
        for (int t = pair; ok && t < args.num_tiles; t += npairs) {
            for (int kb0 = 0, ci = 0; kb0 < kb_total; kb0 += KC_BLOCKS, ++chunk, ++ci) {
                const int acc = chunk & 1;
                const uint32_t use = chunk >> 1;
                bool got = !*abort_flag && mbar_wait(&tfull[acc], use & 1);
                if (!__all_sync(0xffffffffu, got)) {
                    if (lane == 0) record_status(STATUS_TIMEOUT_EPILOGUE);
                    *abort_flag = 1;
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BNP + half * HALF;
                if (kb0 == 0) {
#pragma unroll
                    for (int j = 0; j < HALF; ++j) sum[j] = 0.0f;
                }
#pragma unroll
                for (int part = 0; part < HALF / 16; ++part) {
                    uint32_t r[16];
                    tmem_ld_32x32b_x16(taddr + part * 16, r);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 16; ++j) sum[part * 16 + j] += __uint_as_float(r[j]);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(tempty_pair[acc]);   // accumulator free (even CTA's barrier)
                if (args.world > 1 && pend_row >= 0)
                    copy_rows_to_peers<BNP>(args, pend_row, pend_tn, min(ci * rows_per_chunk, BM),
                                            min((ci + 1) * rows_per_chunk, BM), et);
            }
            if (!ok) break;
            int tm, tn;
            tile_coords(t, args.tiles_m, args.tiles_n, args.group, tm, tn);
            const int64_t row_base = (int64_t)tm * 2 * BM + (int64_t)rank * BM;
            const int64_t row = row_base + quarter * 32 + lane;
            if (row < args.M && args.mc_c) {
                // multicast all-gather: one store per element, replicated to every rank by the switch
                const int64_t col0 = (int64_t)tn * BNP + half * HALF;
                float *mrow = args.mc_c + (args.row_offset + row) * args.ldc_peer;
#pragma unroll
                for (int j = 0; j < HALF; j += 4) {
                    if (col0 + j + 4 <= args.N) {
                        multimem_st_v4(mrow + col0 + j, sum[j], sum[j + 1], sum[j + 2], sum[j + 3]);
                    } else {
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            if (col0 + j + q < args.N) multimem_st(mrow + col0 + j + q, sum[j + q]);
                    }
                }
            } else if (row < args.M) {
                const int64_t col0 = (int64_t)tn * BNP + half * HALF;
                float *crow;
                bool vec;
                int64_t scn;
                if (args.world > 0) {
                    crow = args.peer_c[args.rank] + (args.row_offset + row) * args.ldc_peer;
                    vec = true;
                    scn = 1;
                } else {
                    crow = args.c + row * args.scm;
                    scn = args.scn;
                    vec = scn == 1 && ((reinterpret_cast<uintptr_t>(args.c) | (uintptr_t)(args.scm * 4)) & 15) == 0;
                }
                if (vec) {
#pragma unroll
                    for (int j = 0; j < HALF; j += 4) {
                        if (col0 + j + 4 <= args.N) {
                            *reinterpret_cast<float4 *>(crow + col0 + j) =
                                make_float4(sum[j], sum[j + 1], sum[j + 2], sum[j + 3]);
                        } else {
#pragma unroll
                            for (int q = 0; q < 4; ++q)
                                if (col0 + j + q < args.N) crow[col0 + j + q] = sum[j + q];
                        }
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < HALF; ++j)
                        if (col0 + j < args.N) crow[(col0 + j) * scn] = sum[j];
                }
            }
            if (args.world > 1 && !args.mc_c) {
                __threadfence_block();
                __syncwarp();
                if (lane == 0) mbar_arrive(epi_bar);
                bool got = mbar_wait(epi_bar, tiles_done & 1);
                if (!__all_sync(0xffffffffu, got)) {
                    if (lane == 0) record_status(STATUS_TIMEOUT_EPILOGUE);
                    *abort_flag = 1;
                    ok = false;
                    break;
                }
                pend_row = row_base;
                pend_tn = tn;
            }
            ++tiles_done;
        }
        if (ok && args.world > 1 && pend_row >= 0) copy_rows_to_peers<BNP>(args, pend_row, pend_tn, 0, BM, et);
        if (args.mc_c) __threadfence_system();
    }
    tc_fence_before();
    __syncthreads();
    cluster_barrier();   // the even CTA's MMAs are done with both CTAs' shared memory and TMEM
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS) : "memory");
    }
}

// ---- host side -------------------------------------------------------------------

using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
    static EncodeTiled fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    }
    return fn;
}

// Row-major [rows, ld] fp32 (inner extent `cols`), box [box_rows, BK], 64-byte swizzle.
int make_map(CUtensorMap *map, const float *base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
    EncodeTiled enc = encode_fn();
    if (!enc) return set_error(PITON_B200_ECUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * 4)};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(PITON_B200_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return PITON_B200_OK;
}

// bf16 cross operand [rows, ldx]: 16 bf16 (32 bytes) per group of 8 k-values; box [box_rows, 2 * BK]
// (the same 64 bytes per row as an fp32 box of BK), 64-byte swizzle.
int make_map_x(CUtensorMap *map, const __nv_bfloat16 *base, int64_t rows, int64_t ldx, int box_rows) {
    EncodeTiled enc = encode_fn();
    if (!enc) return set_error(PITON_B200_ECUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {(cuuint64_t)ldx, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(ldx * 2)};
    cuuint32_t box[2] = {(cuuint32_t)(2 * BK), (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<__nv_bfloat16 *>(base), dims, strides, box,
                     estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(PITON_B200_ECUDA, "cuTensorMapEncodeTiled (bf16) failed (%d)", (int)r);
    return PITON_B200_OK;
}

int64_t ld_of(int64_t K) { return (K + 3) / 4 * 4; }
int64_t ldx_of(int64_t K) { return (K + 7) / 8 * 16; }

// CTA pairs (2-SM MMAs) for problems with at least two 256-row tiles; tile width along N
// chosen as for one CTA, over the pairs.
bool use_pairs(int64_t M, int64_t N) { return M >= 512 && N >= 256 && num_sms() >= 2; }
int pair_tile_width(int64_t M, int64_t N) {
    const int64_t pairs = num_sms() / 2, tm = cdiv(M, (int64_t)(2 * BM));
    const int64_t cost256 = cdiv(tm * cdiv(N, (int64_t)256), pairs) * 256;
    const int64_t cost224 = cdiv(tm * cdiv(N, (int64_t)224), pairs) * 224;
    return cost224 < cost256 ? 224 : 256;
}

template <int BNP>
int launch_pairs(const CUtensorMap &a_hi, const CUtensorMap &a_x, const CUtensorMap &b_hi, const CUtensorMap &b_x,
                 GemmArgs g, cudaStream_t stream) {
    static bool attr[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr[dev]) {
        PITON_CUDA(cudaFuncSetAttribute(gemm_3xtf32_2sm_kernel<BNP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        smem2_bytes(BNP)));
        attr[dev] = true;
    }
    const int pairs = std::min<int>(g.num_tiles, num_sms() / 2);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(2 * pairs));
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = smem2_bytes(BNP);
    cfg.stream = stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    PITON_CUDA(cudaLaunchKernelEx(&cfg, gemm_3xtf32_2sm_kernel<BNP>, a_hi, a_x, b_hi, b_x, g));
    return PITON_B200_OK;
}

// Tile width along N: the persistent grid runs ceil(tiles / SMs) rounds, each as long as
// one tile (proportional to its width), so take the width with the fewer column-rounds;
// 256 on a tie (fewer, larger tiles).  E.g. M = 1024, N = 8192 on 148 SMs: 256 wide is
// 256 tiles in 2 rounds, 224 wide is 296 tiles in 2 rounds of 7/8 the length.
int tile_width(int64_t M, int64_t N) {
    const int64_t sms = num_sms(), tm = cdiv(M, (int64_t)BM);
    const int64_t cost256 = cdiv(tm * cdiv(N, (int64_t)256), sms) * 256;
    const int64_t cost224 = cdiv(tm * cdiv(N, (int64_t)224), sms) * 224;
    return cost224 < cost256 ? 224 : 256;
}
size_t region(int64_t rows, int64_t K) { return ((size_t)rows * ld_of(K) * 4 + 1023) / 1024 * 1024; }
size_t xregion(int64_t rows, int64_t K) { return ((size_t)rows * ldx_of(K) * 2 + 1023) / 1024 * 1024; }

}  // namespace

bool tc_gemm_supported(const TcGemmShape &s) {
    // tiny problems are cheaper on the CUDA cores; the tensor-core path needs a
    // device new enough for cudaGetDriverEntryPoint to find the TMA encoder
    if (s.M < 128 || s.N < 128 || s.K < 16) return false;
    if ((double)s.M * s.N * s.K < 4.0e6) return false;
    if (s.M > (1ll << 31) || s.N > (1ll << 31) || s.K > (1ll << 31)) return false;
    if (cdiv(s.M, 32) > 65535 || cdiv(s.N, 32) > 65535) return false;   // split-kernel grid.y
    return encode_fn() != nullptr;
}

size_t tc_gemm_workspace_bytes(const TcGemmShape &s) {
    return region(s.M, s.K) + xregion(s.M, s.K) + region(s.N, s.K) + xregion(s.N, s.K);
}

int tc_gemm(const TcGemmShape &s, void *workspace, cudaStream_t stream) {
    const int64_t ld = ld_of(s.K), ldx = ldx_of(s.K);
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    const size_t nb = region(s.N, s.K) + xregion(s.N, s.K);   // B's operands first: their place does not depend on M
    float *b_hi = reinterpret_cast<float *>(ws);
    __nv_bfloat16 *b_x = reinterpret_cast<__nv_bfloat16 *>(ws + region(s.N, s.K));
    float *a_hi = reinterpret_cast<float *>(ws + nb);
    __nv_bfloat16 *a_x = reinterpret_cast<__nv_bfloat16 *>(ws + nb + region(s.M, s.K));

    // 1. split A [M, K] and B^T [N, K] into the tf32 high halves and the bf16 cross operands.
    //    A row-major A with 16-byte aligned rows is its own high half (the tensor core ignores the
    //    low 13 bits): only A_x is written and the A_hi tensor map reads A in place.
    const bool vec_a = s.sak == 1 && s.K % 4 == 0 && s.sam % 4 == 0 && s.sam >= s.K && s.sam < (1ll << 37) &&
                       (reinterpret_cast<uintptr_t>(s.a) & 15) == 0;
    {
        dim3 ga((unsigned)cdiv(s.K, 32), (unsigned)cdiv(s.M, 32));
        if (vec_a) {
            int64_t blocks = cdiv(s.M * (ldx / 8), 256);
            if (blocks > (int64_t)num_sms() * 16) blocks = (int64_t)num_sms() * 16;
            split_rows_vec4_kernel<<<(unsigned)blocks, 256, 0, stream>>>(s.a, s.M, s.K, s.sam, a_x, ldx);
        } else {
            int along_rows_a = llabs(s.sam) < llabs(s.sak);
            split_kernel<<<ga, 256, 0, stream>>>(s.a, s.M, s.K, s.sam, s.sak, a_hi, a_x, ld, ldx, along_rows_a, 1);
        }
        if (s.split_b) {
            // row-major B (unit n stride, 16-byte aligned rows): 64 x 64-tile transpose with 16-byte stores
            const bool vec_b = s.sbn == 1 && s.N % 4 == 0 && s.sbk % 4 == 0 && (reinterpret_cast<uintptr_t>(s.b) & 15) == 0;
            if (vec_b) {
                dim3 gb((unsigned)cdiv(s.K, 64), (unsigned)cdiv(s.N, 64));
                split_transpose_kernel<SPLIT_T_GEMM_B><<<gb, 256, 0, stream>>>(s.b, s.N, s.K, s.sbk, 0, b_hi, nullptr,
                                                                                b_x, ld, ldx);
            } else {
                dim3 gb((unsigned)cdiv(s.K, 32), (unsigned)cdiv(s.N, 32));
                int along_rows_b = llabs(s.sbn) < llabs(s.sbk);
                split_kernel<<<gb, 256, 0, stream>>>(s.b, s.N, s.K, s.sbn, s.sbk, b_hi, b_x, ld, ldx, along_rows_b, 0);
            }
        }
    }
    // 2. persistent tcgen05 GEMM
    const bool pairs = use_pairs(s.M, s.N);
    const int bn = pairs ? pair_tile_width(s.M, s.N) : tile_width(s.M, s.N);
    const int b_box = pairs ? bn / 2 : bn;   // rows of B^T one CTA loads
    CUtensorMap m_ahi, m_ax, m_bhi, m_bx;
    int rc;
    if ((rc = vec_a ? make_map(&m_ahi, s.a, s.M, s.K, s.sam, BM) : make_map(&m_ahi, a_hi, s.M, s.K, ld, BM)) ||
        (rc = make_map_x(&m_ax, a_x, s.M, ldx, BM)) || (rc = make_map(&m_bhi, b_hi, s.N, s.K, ld, b_box)) ||
        (rc = make_map_x(&m_bx, b_x, s.N, ldx, b_box)))
        return rc;
    GemmArgs g;
    g.c = s.c;
    g.M = s.M; g.N = s.N; g.K = s.K; g.scm = s.scm; g.scn = s.scn;
    g.k_blocks = (int)cdiv(s.K, BK);
    g.world = s.world;
    g.rank = s.rank;
    g.row_offset = s.row_offset;
    g.ldc_peer = s.ldc_peer;
    for (int i = 0; i < MAX_PEERS; ++i) g.peer_c[i] = s.peer_c[i];
    g.mc_c = s.multicast_c;
    if (pairs) {
        g.tiles_m = (int)cdiv(s.M, (int64_t)(2 * BM));
        g.group = GROUP_M / 2;   // 8 tile rows of 256 = 2048 rows of A per group
        g.tiles_n = (int)cdiv(s.N, (int64_t)bn);
        g.num_tiles = g.tiles_m * g.tiles_n;
        rc = bn == 224 ? launch_pairs<224>(m_ahi, m_ax, m_bhi, m_bx, g, stream)
                       : launch_pairs<256>(m_ahi, m_ax, m_bhi, m_bx, g, stream);
        if (rc) return rc;
        return check_launch("gemm_3xtf32_2sm", s.split_b ? 3 : 2);
    }
    static bool attr[64][2] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr[dev][bn == 224]) {
        if (bn == 224)
            PITON_CUDA(cudaFuncSetAttribute(gemm_3xtf32_kernel<224>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            smem_bytes(224)));
        else
            PITON_CUDA(cudaFuncSetAttribute(gemm_3xtf32_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            smem_bytes(256)));
        attr[dev][bn == 224] = true;
    }
    g.tiles_m = (int)cdiv(s.M, BM);
    g.group = GROUP_M;
    g.tiles_n = (int)cdiv(s.N, (int64_t)bn);
    g.num_tiles = g.tiles_m * g.tiles_n;
    int grid = g.num_tiles < num_sms() ? g.num_tiles : num_sms();
    if (bn == 224)
        gemm_3xtf32_kernel<224><<<grid, THREADS, smem_bytes(224), stream>>>(m_ahi, m_ax, m_bhi, m_bx, g);
    else
        gemm_3xtf32_kernel<256><<<grid, THREADS, smem_bytes(256), stream>>>(m_ahi, m_ax, m_bhi, m_bx, g);
    return check_launch("gemm_3xtf32", s.split_b ? 3 : 2);
}

int tc_status_read_and_clear(int *status) {
    int zero = 0;
    PITON_CUDA(cudaMemcpyFromSymbol(status, g_tc_status, sizeof(int)));
    PITON_CUDA(cudaMemcpyToSymbol(g_tc_status, &zero, sizeof(int)));
    return PITON_B200_OK;
}

}  // namespace piton

extern "C" int piton_b200_device_status(int *status) {
    PITON_REQUIRE(status != nullptr, "status is NULL");
    int gemm = 0, attn = 0, rc;
    if ((rc = piton::tc_status_read_and_clear(&gemm)) != PITON_B200_OK) return rc;
    if ((rc = piton::attention_tc_status_read_and_clear(&attn)) != PITON_B200_OK) return rc;
    *status = gemm ? gemm : attn;
    return PITON_B200_OK;
}
