// fp32 GEMM on the 5th-generation tensor cores from an fp16 split of each operand
// (tutorial matmul, examples/kernels.py:18-57, default rounding mode).
//
// fp32 accuracy from FP16 tensor cores: every 256-deep chunk of a row of A (and of a
// column of B) is scaled by a power of two 2^e that brings its largest finite magnitude
// into [2^14, 2^15), and each scaled value s is split into s_hi = fp16(s) and
// s_lo = fp16(s - s_hi) (s - s_hi is exact in fp32), 22 significant bits in all.  Then
//   C = sum over chunks of 2^-(e_A + e_B) (A_hi B_hi + A_hi B_lo + A_lo B_hi)
// with three kind::f16 MMAs per 16 k-values (fp16 products are exact in the fp32
// accumulator); the dropped A_lo B_lo and the rounding of the low halves cost about
// 2^-21 of a product, against ~2^-17 for a tf32 high half with bf16 cross terms, and the
// operands take 4 bytes per element (hi + lo) instead of 8.  A value too small for fp16's
// subnormals after scaling (below 2^-25 of its chunk's largest) contributes ~nothing.  A
// chunk holding an inf or nan is marked (exponent NONFINITE): split products cannot keep
// IEEE semantics there (inf x a zero low half is nan), so a small kernel after the GEMM
// recomputes that row (or column) of C with fp32 FMAs from A and B.
//
// Two kernels per call:
//  1. split: reads A and B with their (arbitrary) element strides and writes A_hi, A_lo
//     as [M, ldh] fp16 and B_hi, B_lo transposed as [N, ldh] (K-major, ldh = K rounded up
//     to 8) and the chunk exponents e as int8 [chunks, M] / [chunks, N], into the
//     caller's workspace.  HBM-bound.
//  2. gemm: persistent, one CTA per SM (320 threads): warp 0 issues TMA tile loads
//     (128x32 A_hi / A_lo tiles and BNx32 B_hi / B_lo tiles, 64-byte swizzle, 4-stage
//     mbarrier ring), warp 1 owns 512 TMEM columns (two 128xBN fp32 accumulators) and
//     issues, from one thread, three tcgen05.mma kind::f16 128xBNx16 per 16 k-values,
//     warps 2-9 drain finished accumulators with tcgen05.ld and apply the chunk scales.
//
// The tensor cores add into the TMEM accumulator with truncation, and that bias grows
// with the number of accumulation steps (at K = 8192 it is ~30x the error of an fp32
// FFMA loop).  So an accumulator only ever holds a chunk of KC = 256 k-values (one
// scaling chunk): the MMA warp alternates between the two TMEM buffers per chunk, and
// the epilogue warps multiply every finished chunk by its 2^-(e_A + e_B) and add it into
// an fp32 register sum (round to nearest), then store the tile with C's element strides.
// Every mbarrier wait is bounded (2 s of global time): on expiry the kernel records a
// status word, drains its own TMA copies and MMAs, frees TMEM and returns.
#include <algorithm>
#include <vector>

#include <cuda_fp16.h>

#include "attention.cuh"
#include "common.cuh"
#include "gemm_tc.cuh"
#include "sm100.cuh"

namespace piton {

using namespace sm100;

__device__ int g_tc_status = 0;

namespace {

constexpr int BM = 128, BK = 32, STAGES = 4;   // BK: fp16 k-values per stage (64-byte rows)
constexpr int THREADS = 320;
constexpr int EPI_WARPS = 8;
constexpr int KC = 256;                         // k-values per accumulation and scaling chunk
constexpr int KC_BLOCKS = KC / BK;              // k-blocks per chunk
constexpr uint32_t A_TILE_BYTES = BM * BK * 2;   // 8 KB: 128 rows x 32 fp16 (A_hi, or A_lo)
// BN (tile width along N) is 256, or 224 where that packs the tiles into fewer
// rounds over the SMs (tile_width()); a B tile is BN x 32 fp16 (14 or 16 KB), hi and lo
__host__ __device__ constexpr uint32_t b_tile_bytes(int bn) { return (uint32_t)bn * BK * 2; }
__host__ __device__ constexpr uint32_t stage_bytes(int bn) { return 2 * A_TILE_BYTES + 2 * b_tile_bytes(bn); }
__host__ __device__ constexpr uint32_t smem_bytes(int bn) { return STAGES * stage_bytes(bn) + 1024 /*barriers*/ + 1024 /*alignment*/; }
constexpr int TMEM_COLS = 512;
constexpr int GROUP_M = 16;

// Marker exponent of a chunk that holds an inf or a nan (outside the clamp range below).
constexpr int NONFINITE = -128;

// Exponent e of a chunk's scale 2^e: its largest finite magnitude m goes into [2^14, 2^15);
// 0 for a chunk without a finite non-zero value; clamped to [-112, 112] (2^e and 2^-e normal).
__device__ __forceinline__ int chunk_exponent(float m) {
    if (!(m > 0.0f)) return 0;
    int E;
    frexpf(m, &E);   // m = f 2^E, f in [0.5, 1)
    return max(-112, min(112, 15 - E));
}

// s = v 2^e split into fp16 halves: hi = fp16(s), lo = fp16(s - hi); non-finite s keeps its
// high half and a zero low half.
__device__ __forceinline__ void split_half(float v, float sc, __half &hi, __half &lo) {
    const float s = v * sc;
    hi = __float2half_rn(s);
    lo = __float2half_rn(isfinite(s) ? s - __half2float(hi) : 0.0f);
}

__device__ __forceinline__ float finite_abs(float v) { return isfinite(v) ? fabsf(v) : 0.0f; }

// Rows with unit stride along k (row-major A, or B stored column-major): one warp per
// (row, 256-deep chunk), 8 consecutive k-values per lane (two 16-byte loads when `vec`),
// the chunk's maximum by shuffles, 16-byte stores of both halves.  k-values from K up to
// ldh (K rounded up to 8) are written as zeros; the exponent goes to ex[chunk * ld_ex + row].
__global__ void __launch_bounds__(256) split16_rows_kernel(const float *__restrict__ src, int64_t rows, int64_t K,
                                                           int64_t s_row, __half *__restrict__ hi,
                                                           __half *__restrict__ lo, int8_t *__restrict__ ex,
                                                           int64_t ldh, int64_t ld_ex, int chunks, int vec) {
    const int lane = threadIdx.x & 31;
    const int64_t w = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (w >= rows * chunks) return;
    const int64_t r = w / chunks;
    const int c = (int)(w % chunks);
    const int64_t k0 = (int64_t)c * KC + 8 * lane;
    const float *row = src + r * s_row;
    float v[8];
    if (vec && k0 + 8 <= K) {
        const float4 p = __ldcs(reinterpret_cast<const float4 *>(row + k0));
        const float4 q = __ldcs(reinterpret_cast<const float4 *>(row + k0 + 4));
        v[0] = p.x; v[1] = p.y; v[2] = p.z; v[3] = p.w; v[4] = q.x; v[5] = q.y; v[6] = q.z; v[7] = q.w;
    } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = k0 + e < K ? row[k0 + e] : 0.0f;
    }
    float m = 0.0f;
    bool bad = false;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        m = fmaxf(m, finite_abs(v[e]));
        bad |= !isfinite(v[e]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    bad = __any_sync(0xffffffffu, bad);
    const int ee = chunk_exponent(m);
    const float sc = ldexpf(1.0f, ee);
    __align__(16) __half h[8], l[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) split_half(v[e], sc, h[e], l[e]);
    if (k0 < ldh) {
        *reinterpret_cast<uint4 *>(hi + r * ldh + k0) = *reinterpret_cast<const uint4 *>(h);
        *reinterpret_cast<uint4 *>(lo + r * ldh + k0) = *reinterpret_cast<const uint4 *>(l);
    }
    if (lane == 0) ex[(int64_t)c * ld_ex + r] = (int8_t)(bad ? NONFINITE : ee);
}

// Any strides (row-major B transposed into K-major rows, transposed or strided A): a CTA
// stages a 32-row x 256-k tile in shared memory, reading with the lanes along whichever of
// rows and k has the unit (smaller) stride so that the loads coalesce (lanes_along_rows 1 or
// 0; 2: unit row stride and 16-byte aligned columns, float4 loads), then each warp splits
// four rows: a half2 of consecutive k-values per lane, 128-byte stores per warp.
__global__ void __launch_bounds__(256) split16_tile_kernel(const float *__restrict__ src, int64_t rows, int64_t K,
                                                           int64_t s_row, int64_t s_col, __half *__restrict__ hi,
                                                           __half *__restrict__ lo, int8_t *__restrict__ ex,
                                                           int64_t ldh, int64_t ld_ex, int lanes_along_rows) {
    __shared__ float tile[32][KC + 1];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int c = blockIdx.x;
    const int64_t r0 = (int64_t)blockIdx.y * 32, k0 = (int64_t)c * KC;
    if (lanes_along_rows == 2) {
        // unit stride along rows, 16-byte aligned columns (row-major B): float4 of 4 rows,
        // 8 per thread in flight; lanes cover 4 k x 8 row quads, conflict-free into the padded tile
        const int n0 = 4 * (threadIdx.x & 7), kr = threadIdx.x >> 3;
        const int64_t r = r0 + n0;
        float4 f[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int64_t k = k0 + kr + 32 * i;
            if (k < K && r + 3 < rows) {
                f[i] = __ldcs(reinterpret_cast<const float4 *>(src + r + k * s_col));
            } else {
                float e[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) e[j] = (k < K && r + j < rows) ? src[r + j + k * s_col] : 0.0f;
                f[i] = make_float4(e[0], e[1], e[2], e[3]);
            }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int kk = kr + 32 * i;
            tile[n0][kk] = f[i].x;
            tile[n0 + 1][kk] = f[i].y;
            tile[n0 + 2][kk] = f[i].z;
            tile[n0 + 3][kk] = f[i].w;
        }
    } else if (lanes_along_rows) {
        // 16 loads in flight per thread before they go to shared memory
        const int64_t r = r0 + lane;
        const bool rin = r < rows;
#pragma unroll
        for (int i0 = 0; i0 < KC / 8; i0 += 16) {
            float v[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int64_t k = k0 + warp + 8 * (i0 + i);
                v[i] = (rin && k < K) ? __ldcs(src + r * s_row + k * s_col) : 0.0f;
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) tile[lane][warp + 8 * (i0 + i)] = v[i];
        }
    } else {
        for (int rr = warp; rr < 32; rr += 8) {
            const int64_t r = r0 + rr;
            for (int kk = lane; kk < KC; kk += 32) {
                const int64_t k = k0 + kk;
                tile[rr][kk] = (r < rows && k < K) ? src[r * s_row + k * s_col] : 0.0f;
            }
        }
    }
    __syncthreads();
    for (int rr = warp; rr < 32; rr += 8) {
        const int64_t r = r0 + rr;
        if (r >= rows) break;
        float m = 0.0f;
        bool bad = false;
#pragma unroll
        for (int e = 0; e < KC / 64; ++e) {
            const float v0 = tile[rr][2 * lane + 64 * e], v1 = tile[rr][2 * lane + 64 * e + 1];
            m = fmaxf(m, fmaxf(finite_abs(v0), finite_abs(v1)));
            bad |= !isfinite(v0) || !isfinite(v1);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        bad = __any_sync(0xffffffffu, bad);
        const int ee = chunk_exponent(m);
        const float sc = ldexpf(1.0f, ee);
#pragma unroll
        for (int e = 0; e < KC / 64; ++e) {
            const int64_t k = k0 + 2 * lane + 64 * e;
            if (k < ldh) {
                __half h0, l0, h1, l1;
                split_half(tile[rr][2 * lane + 64 * e], sc, h0, l0);
                split_half(tile[rr][2 * lane + 64 * e + 1], sc, h1, l1);
                *reinterpret_cast<__half2 *>(hi + r * ldh + k) = __halves2half2(h0, h1);
                *reinterpret_cast<__half2 *>(lo + r * ldh + k) = __halves2half2(l0, l1);
            }
        }
        if (lane == 0) ex[(int64_t)c * ld_ex + r] = (int8_t)(bad ? NONFINITE : ee);
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
    const int8_t *ea, *eb;           // chunk exponents of A [chunks, ld_ea] and of B [chunks, ld_eb]
    int64_t ld_ea, ld_eb;
    const float *a, *b;              // the fp32 operands (chunks marked NONFINITE are recomputed from them)
    int64_t sam, sak, sbk, sbn;
};

// The contribution of a finished chunk product `acc` to C: acc 2^-(ea + eb), applied as two
// factors 2^-t1 and 2^-t2 with t1 + t2 = ea + eb, each built from its exponent bits and always
// a normal float (|t1|, |t2| <= 112), so the result is exact wherever it is a normal float (an
// intermediate over- or underflows only when the result does too).  Rows and columns with a
// chunk marked NONFINITE get garbage here and are rewritten by nonfinite_fixup_kernel after
// the GEMM.
__device__ __forceinline__ float chunk_value(float acc, int ea, int eb) {
    const int t = ea + eb, t1 = t >> 1, t2 = t - t1;
    return acc * __int_as_float((127 - t1) << 23) * __int_as_float((127 - t2) << 23);
}

// After the GEMM: every row of A and every column of B with a chunk marked NONFINITE (an inf or
// a nan, which split products cannot carry with IEEE semantics: inf times a zero low half is nan)
// has its row / column of C recomputed with fp32 FMAs over the whole K, a warp per row or column.
// Without such values each warp only reads its row's or column's chunk exponents.
__global__ void __launch_bounds__(256) nonfinite_fixup_kernel(GemmArgs g, int chunks) {
    const int lane = threadIdx.x & 31;
    const int64_t idx = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    const bool is_row = idx < g.M;
    if (idx >= g.M + g.N) return;
    const int64_t i = is_row ? idx : idx - g.M;
    bool bad = false;
    for (int c = lane; c < chunks; c += 32)
        bad |= (is_row ? g.ea[(int64_t)c * g.ld_ea + i] : g.eb[(int64_t)c * g.ld_eb + i]) == NONFINITE;
    if (!__any_sync(0xffffffffu, bad)) return;
    const int64_t n_out = is_row ? g.N : g.M;
    for (int64_t o = lane; o < n_out; o += 32) {
        const int64_t row = is_row ? i : o, col = is_row ? o : i;
        float s = 0.0f;
        for (int64_t k = 0; k < g.K; ++k) s = fmaf(g.a[row * g.sam + k * g.sak], g.b[k * g.sbk + col * g.sbn], s);
        if (g.world > 0) {
            for (int r = 0; r < g.world; ++r) g.peer_c[r][(g.row_offset + row) * g.ldc_peer + col] = s;
        } else {
            g.c[row * g.scm + col * g.scn] = s;
        }
    }
}

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
    gemm_f16x3_kernel(const __grid_constant__ CUtensorMap tm_ah, const __grid_constant__ CUtensorMap tm_al,
                      const __grid_constant__ CUtensorMap tm_bh, const __grid_constant__ CUtensorMap tm_bl,
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
        prefetch_tmap(&tm_ah);
        prefetch_tmap(&tm_al);
        prefetch_tmap(&tm_bh);
        prefetch_tmap(&tm_bl);
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
                    const int kx = kb * BK;
                    tma_load_2d(st, &tm_ah, &full[s], kx, tm * BM);
                    tma_load_2d(st + A_TILE_BYTES, &tm_al, &full[s], kx, tm * BM);
                    tma_load_2d(st + 2 * A_TILE_BYTES, &tm_bh, &full[s], kx, tn * BN);
                    tma_load_2d(st + 2 * A_TILE_BYTES + B_TILE_BYTES, &tm_bl, &full[s], kx, tn * BN);
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
            constexpr uint32_t IDESC = idesc_f16(BM, BN);
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
                        uint32_t a_hi = base, a_lo = base + A_TILE_BYTES;
                        uint32_t b_hi = base + 2 * A_TILE_BYTES, b_lo = b_hi + B_TILE_BYTES;
#pragma unroll
                        for (int ks = 0; ks < BK / 16; ++ks) {
                            // 16 fp16 k-values: 32 bytes along K in the row
                            uint32_t off = ks * 32;
                            uint64_t dah = smem_desc_kmajor(a_hi + off, 64, LAYOUT_SWIZZLE_64B);
                            uint64_t dal = smem_desc_kmajor(a_lo + off, 64, LAYOUT_SWIZZLE_64B);
                            uint64_t dbh = smem_desc_kmajor(b_hi + off, 64, LAYOUT_SWIZZLE_64B);
                            uint64_t dbl = smem_desc_kmajor(b_lo + off, 64, LAYOUT_SWIZZLE_64B);
                            uint32_t first = (kb == kb0 && ks == 0) ? 0u : 1u;
                            mma_f16(d_tmem, dah, dbh, IDESC, first);   // A_hi B_hi
                            mma_f16(d_tmem, dah, dbl, IDESC, 1u);      // A_hi B_lo
                            mma_f16(d_tmem, dal, dbh, IDESC, 1u);      // A_lo B_hi
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
            int tm, tn;
            tile_coords(t, args.tiles_m, args.tiles_n, args.group, tm, tn);
            const int64_t row = (int64_t)tm * BM + quarter * 32 + lane;
            const int64_t col0 = (int64_t)tn * BN + half * (BN / 2);
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
                const int ea = row < args.M ? (int)args.ea[(int64_t)ci * args.ld_ea + row] : 0;
                const int8_t *ebc = args.eb + (int64_t)ci * args.ld_eb;
#pragma unroll
                for (int part = 0; part < BN / 2 / 16; ++part) {
                    uint32_t r[16];
                    tmem_ld_32x32b_x16(taddr + part * 16, r);
                    // the 16 columns' exponents in one load (rows of ld_eb, a multiple of 16, zero padded)
                    const int64_t c16 = col0 + part * 16;
                    uint4 e16 = make_uint4(0u, 0u, 0u, 0u);
                    if (c16 < args.ld_eb) e16 = __ldg(reinterpret_cast<const uint4 *>(ebc + c16));
                    const uint32_t ew[4] = {e16.x, e16.y, e16.z, e16.w};
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int eb = (int)(int8_t)(ew[j >> 2] >> (8 * (j & 3)));
                        sum[part * 16 + j] += chunk_value(__uint_as_float(r[j]), ea, eb);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[acc]);   // TMEM buffer free for the next chunk
                if (args.world > 1 && pend_tm >= 0)
                    copy_rows_to_peers<BN>(args, (int64_t)pend_tm * BM, pend_tn, min(ci * rows_per_chunk, BM),
                                       min((ci + 1) * rows_per_chunk, BM), et);
            }
            if (!ok) break;
            if (row < args.M) {
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

// BK2: fp16 k-values per stage of the pair kernel (64: 128-byte rows, 128-byte swizzle; 32:
// 64-byte rows, 64-byte swizzle); STAGES2 stages fill the shared memory.  At 8192^3 64 x 3
// stages measured 411.5 TFLOP/s per step against 395.6 for 32 x 6 and 392 for 32 x 7.
#ifndef PITON_GEMM2_BK
#define PITON_GEMM2_BK 64
#endif
#ifndef PITON_GEMM2_STAGES
#define PITON_GEMM2_STAGES 3
#endif
constexpr int BK2 = PITON_GEMM2_BK, STAGES2 = PITON_GEMM2_STAGES;
static_assert(BK2 == 32 || BK2 == 64, "pair k-block: 32 or 64 fp16");
constexpr int KC_BLOCKS2 = KC / BK2;
constexpr uint64_t LAYOUT2 = BK2 == 64 ? LAYOUT_SWIZZLE_128B : LAYOUT_SWIZZLE_64B;
constexpr uint32_t A2_TILE_BYTES = BM * BK2 * 2;   // this CTA's 128 rows x BK2 fp16
__host__ __device__ constexpr uint32_t b2_tile_bytes(int bnp) { return (uint32_t)(bnp / 2) * BK2 * 2; }
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
__device__ __forceinline__ void mma_f16_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
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

// GATHER: the output goes to the ranks' buffers (peer stores or a multicast address); the
// single-GPU instantiation carries none of that code.
template <int BNP, bool GATHER>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_f16x3_2sm_kernel(const __grid_constant__ CUtensorMap tm_ah, const __grid_constant__ CUtensorMap tm_al,
                          const __grid_constant__ CUtensorMap tm_bh, const __grid_constant__ CUtensorMap tm_bl,
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
        prefetch_tmap(&tm_ah);
        prefetch_tmap(&tm_al);
        prefetch_tmap(&tm_bh);
        prefetch_tmap(&tm_bl);
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
                    const int kx = kb * BK2;
                    tma_load_2d_pair(st, &tm_ah, bar, kx, arow);
                    tma_load_2d_pair(st + A2_TILE_BYTES, &tm_al, bar, kx, arow);
                    tma_load_2d_pair(st + 2 * A2_TILE_BYTES, &tm_bh, bar, kx, brow);
                    tma_load_2d_pair(st + 2 * A2_TILE_BYTES + B_TILE, &tm_bl, bar, kx, brow);
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
            constexpr uint32_t IDESC = idesc_f16(2 * BM, BNP);
            uint32_t it = 0, chunk = 0;
            bool ok = true;
            for (int t = pair; ok && t < args.num_tiles && !*abort_flag; t += npairs) {
                for (int kb0 = 0; ok && kb0 < kb_total; kb0 += KC_BLOCKS2, ++chunk) {
                    const int acc = chunk & 1;
                    const uint32_t use = chunk >> 1;
                    if (!mbar_wait(&tempty[acc], (use & 1) ^ 1)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + acc * BNP;
                    const int kb1 = min(kb0 + KC_BLOCKS2, kb_total);
                    for (int kb = kb0; kb < kb1; ++kb, ++it) {
                        const uint32_t s = it % STAGES2, round = it / STAGES2;
                        if (!mbar_wait(&full[s], round & 1)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t base = smem_u32(smem + s * STAGE);
                        const uint32_t a_hi = base, a_lo = base + A2_TILE_BYTES;
                        const uint32_t b_hi = base + 2 * A2_TILE_BYTES, b_lo = b_hi + B_TILE;
#pragma unroll
                        for (int ks = 0; ks < BK2 / 16; ++ks) {
                            const uint32_t off = ks * 32;   // 16 fp16 k-values
                            const uint64_t dah = smem_desc_kmajor(a_hi + off, BK2 * 2, LAYOUT2);
                            const uint64_t dal = smem_desc_kmajor(a_lo + off, BK2 * 2, LAYOUT2);
                            const uint64_t dbh = smem_desc_kmajor(b_hi + off, BK2 * 2, LAYOUT2);
                            const uint64_t dbl = smem_desc_kmajor(b_lo + off, BK2 * 2, LAYOUT2);
                            const uint32_t first = (kb == kb0 && ks == 0) ? 0u : 1u;
                            mma_f16_pair(d_tmem, dah, dbh, IDESC, first);   // A_hi B_hi
                            mma_f16_pair(d_tmem, dah, dbl, IDESC, 1u);      // A_hi B_lo
                            mma_f16_pair(d_tmem, dal, dbh, IDESC, 1u);      // A_lo B_hi
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
        const int n_chunks = (kb_total + KC_BLOCKS2 - 1) / KC_BLOCKS2;
        const int rows_per_chunk = (BM + n_chunks - 1) / n_chunks;
        const uint32_t tempty_pair[2] = {cluster_addr_rank0(&tempty[0]), cluster_addr_rank0(&tempty[1])};
        int pend_tn = -1;
        int64_t pend_row = -1;
        uint32_t tiles_done = 0;
        for (int t = pair; ok && t < args.num_tiles; t += npairs) {
            int tm, tn;
            tile_coords(t, args.tiles_m, args.tiles_n, args.group, tm, tn);
            const int64_t row_base = (int64_t)tm * 2 * BM + (int64_t)rank * BM;
            const int64_t row = row_base + quarter * 32 + lane;
            const int64_t col0 = (int64_t)tn * BNP + half * HALF;
            for (int kb0 = 0, ci = 0; kb0 < kb_total; kb0 += KC_BLOCKS2, ++chunk, ++ci) {
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
                const int ea = row < args.M ? (int)args.ea[(int64_t)ci * args.ld_ea + row] : 0;
                const int8_t *ebc = args.eb + (int64_t)ci * args.ld_eb;
#pragma unroll
                for (int part = 0; part < HALF / 16; ++part) {
                    uint32_t r[16];
                    tmem_ld_32x32b_x16(taddr + part * 16, r);
                    // the 16 columns' exponents in one load (rows of ld_eb, a multiple of 16, zero padded)
                    const int64_t c16 = col0 + part * 16;
                    uint4 e16 = make_uint4(0u, 0u, 0u, 0u);
                    if (c16 < args.ld_eb) e16 = __ldg(reinterpret_cast<const uint4 *>(ebc + c16));
                    const uint32_t ew[4] = {e16.x, e16.y, e16.z, e16.w};
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int eb = (int)(int8_t)(ew[j >> 2] >> (8 * (j & 3)));
                        sum[part * 16 + j] += chunk_value(__uint_as_float(r[j]), ea, eb);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(tempty_pair[acc]);   // accumulator free (even CTA's barrier)
                if (GATHER && args.world > 1 && pend_row >= 0)
                    copy_rows_to_peers<BNP>(args, pend_row, pend_tn, min(ci * rows_per_chunk, BM),
                                            min((ci + 1) * rows_per_chunk, BM), et);
            }
            if (!ok) break;
            if (GATHER && row < args.M && args.mc_c) {
                // multicast all-gather: one store per element, replicated to every rank by the switch
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
                float *crow;
                bool vec;
                int64_t scn;
                if (GATHER && args.world > 0) {
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
            if (GATHER && args.world > 1 && !args.mc_c) {
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
        if (GATHER && ok && args.world > 1 && pend_row >= 0) copy_rows_to_peers<BNP>(args, pend_row, pend_tn, 0, BM, et);
        if (GATHER && args.mc_c) __threadfence_system();
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

// Row-major [rows, ldh] fp16, box [box_rows, box_k]: box_k 32 (64-byte rows, 64-byte swizzle)
// or 64 (128-byte rows, 128-byte swizzle).
int make_map16(CUtensorMap *map, const __half *base, int64_t rows, int64_t ldh, int box_rows, int box_k = BK) {
    EncodeTiled enc = encode_fn();
    if (!enc) return set_error(PITON_B200_ECUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {(cuuint64_t)ldh, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(ldh * 2)};
    cuuint32_t box[2] = {(cuuint32_t)box_k, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE,
                     box_k == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(PITON_B200_ECUDA, "cuTensorMapEncodeTiled (fp16) failed (%d)", (int)r);
    return PITON_B200_OK;
}

int64_t ldh_of(int64_t K) { return (K + 7) / 8 * 8; }        // fp16 row: 16-byte multiple
int64_t chunks_of(int64_t K) { return (K + KC - 1) / KC; }
int64_t lde_of(int64_t rows) { return (rows + 15) / 16 * 16; }   // exponent row per chunk

// CTA pairs (2-SM MMAs) for problems with at least two 256-row tiles; tile width along N
// chosen as for one CTA, over the pairs.
bool use_pairs(int64_t M, int64_t N) { return M >= 512 && N >= 256 && num_sms() >= 2; }
int pair_tile_width(int64_t M, int64_t N) {
    const int64_t pairs = num_sms() / 2, tm = cdiv(M, (int64_t)(2 * BM));
    const int64_t cost256 = cdiv(tm * cdiv(N, (int64_t)256), pairs) * 256;
    const int64_t cost224 = cdiv(tm * cdiv(N, (int64_t)224), pairs) * 224;
    return cost224 < cost256 ? 224 : 256;
}

template <int BNP, bool GATHER>
int launch_pairs(const CUtensorMap &a_hi, const CUtensorMap &a_lo, const CUtensorMap &b_hi, const CUtensorMap &b_lo,
                 GemmArgs g, cudaStream_t stream) {
    static bool attr[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr[dev]) {
        PITON_CUDA(cudaFuncSetAttribute(gemm_f16x3_2sm_kernel<BNP, GATHER>, cudaFuncAttributeMaxDynamicSharedMemorySize,
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
    PITON_CUDA(cudaLaunchKernelEx(&cfg, gemm_f16x3_2sm_kernel<BNP, GATHER>, a_hi, a_lo, b_hi, b_lo, g));
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
size_t hregion(int64_t rows, int64_t K) { return ((size_t)rows * ldh_of(K) * 2 + 1023) / 1024 * 1024; }
size_t eregion(int64_t rows, int64_t K) { return ((size_t)chunks_of(K) * lde_of(rows) + 1023) / 1024 * 1024; }
// one operand's split: hi and lo [rows, ldh] fp16, then the chunk exponents [chunks, lde] int8
size_t oregion(int64_t rows, int64_t K) { return 2 * hregion(rows, K) + eregion(rows, K); }

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

size_t tc_gemm_workspace_bytes(const TcGemmShape &s) { return oregion(s.N, s.K) + oregion(s.M, s.K); }

namespace {

// hi, lo and exponents of one operand from its workspace region
struct Split16 {
    __half *hi, *lo;
    int8_t *ex;
};
Split16 split_at(uint8_t *base, int64_t rows, int64_t K) {
    Split16 p;
    p.hi = reinterpret_cast<__half *>(base);
    p.lo = reinterpret_cast<__half *>(base + hregion(rows, K));
    p.ex = reinterpret_cast<int8_t *>(base + 2 * hregion(rows, K));
    return p;
}

// src[r * s_row + k * s_col] (r < rows, k < K) into the fp16 halves and chunk exponents
void split16(const float *src, int64_t rows, int64_t K, int64_t s_row, int64_t s_col, const Split16 &d,
             cudaStream_t stream) {
    const int64_t ldh = ldh_of(K), chunks = chunks_of(K), lde = lde_of(rows);
    if (s_col == 1) {
        const int vec = s_row % 4 == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0;
        const int64_t warps = rows * chunks;
        split16_rows_kernel<<<(unsigned)cdiv(warps, 8), 256, 0, stream>>>(src, rows, K, s_row, d.hi, d.lo, d.ex, ldh,
                                                                            lde, (int)chunks, vec);
    } else {
        dim3 g((unsigned)chunks, (unsigned)cdiv(rows, 32));
        const bool vec_rows = s_row == 1 && s_col % 4 == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0;
        split16_tile_kernel<<<g, 256, 0, stream>>>(src, rows, K, s_row, s_col, d.hi, d.lo, d.ex, ldh, lde,
                                                   vec_rows ? 2 : (int)(llabs(s_row) < llabs(s_col)));
    }
}

}  // namespace

int tc_gemm(const TcGemmShape &s, void *workspace, cudaStream_t stream) {
    const int64_t ldh = ldh_of(s.K);
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    // B's operands first: their place does not depend on M
    const Split16 B = split_at(ws, s.N, s.K);
    const Split16 A = split_at(ws + oregion(s.N, s.K), s.M, s.K);

    // 1. split A [M, K] and B^T [N, K] (row n of B^T is column n of B) into scaled fp16 halves
    split16(s.a, s.M, s.K, s.sam, s.sak, A, stream);
    if (s.split_b) split16(s.b, s.N, s.K, s.sbn, s.sbk, B, stream);
    // 2. persistent tcgen05 GEMM
    const bool pairs = use_pairs(s.M, s.N);
    const int bn = pairs ? pair_tile_width(s.M, s.N) : tile_width(s.M, s.N);
    const int b_box = pairs ? bn / 2 : bn;   // rows of B^T one CTA loads
    const int bk = pairs ? BK2 : BK;         // k-values per stage
    CUtensorMap m_ah, m_al, m_bh, m_bl;
    int rc;
    if ((rc = make_map16(&m_ah, A.hi, s.M, ldh, BM, bk)) || (rc = make_map16(&m_al, A.lo, s.M, ldh, BM, bk)) ||
        (rc = make_map16(&m_bh, B.hi, s.N, ldh, b_box, bk)) || (rc = make_map16(&m_bl, B.lo, s.N, ldh, b_box, bk)))
        return rc;
    GemmArgs g;
    g.c = s.c;
    g.M = s.M; g.N = s.N; g.K = s.K; g.scm = s.scm; g.scn = s.scn;
    g.k_blocks = (int)cdiv(s.K, (int64_t)bk);
    g.world = s.world;
    g.rank = s.rank;
    g.row_offset = s.row_offset;
    g.ldc_peer = s.ldc_peer;
    for (int i = 0; i < MAX_PEERS; ++i) g.peer_c[i] = s.peer_c[i];
    g.mc_c = s.multicast_c;
    g.ea = A.ex;
    g.eb = B.ex;
    g.ld_ea = lde_of(s.M);
    g.ld_eb = lde_of(s.N);
    g.a = s.a;
    g.b = s.b;
    g.sam = s.sam; g.sak = s.sak; g.sbk = s.sbk; g.sbn = s.sbn;
    if (pairs) {
        g.tiles_m = (int)cdiv(s.M, (int64_t)(2 * BM));
        // 8 tile rows of 256 = 2048 rows of A per group: at 8192^3 the fewest DRAM bytes (2.33 GB
        // read, against 3.11 / 2.58 / 2.50 GB for groups of 4 / 6 / 12) at the same speed
        g.group = GROUP_M / 2;
        g.tiles_n = (int)cdiv(s.N, (int64_t)bn);
        g.num_tiles = g.tiles_m * g.tiles_n;
        const bool gather = g.world > 0 || g.mc_c != nullptr;
        if (gather)
            rc = bn == 224 ? launch_pairs<224, true>(m_ah, m_al, m_bh, m_bl, g, stream)
                           : launch_pairs<256, true>(m_ah, m_al, m_bh, m_bl, g, stream);
        else
            rc = bn == 224 ? launch_pairs<224, false>(m_ah, m_al, m_bh, m_bl, g, stream)
                           : launch_pairs<256, false>(m_ah, m_al, m_bh, m_bl, g, stream);
        if (rc) return rc;
        nonfinite_fixup_kernel<<<(unsigned)cdiv(s.M + s.N, 8), 256, 0, stream>>>(g, (int)chunks_of(s.K));
        return check_launch("gemm_f16x3_2sm", s.split_b ? 4 : 3);
    }
    static bool attr[64][2] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr[dev][bn == 224]) {
        if (bn == 224)
            PITON_CUDA(cudaFuncSetAttribute(gemm_f16x3_kernel<224>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            smem_bytes(224)));
        else
            PITON_CUDA(cudaFuncSetAttribute(gemm_f16x3_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            smem_bytes(256)));
        attr[dev][bn == 224] = true;
    }
    g.tiles_m = (int)cdiv(s.M, BM);
    g.group = GROUP_M;
    g.tiles_n = (int)cdiv(s.N, (int64_t)bn);
    g.num_tiles = g.tiles_m * g.tiles_n;
    int grid = g.num_tiles < num_sms() ? g.num_tiles : num_sms();
    if (bn == 224)
        gemm_f16x3_kernel<224><<<grid, THREADS, smem_bytes(224), stream>>>(m_ah, m_al, m_bh, m_bl, g);
    else
        gemm_f16x3_kernel<256><<<grid, THREADS, smem_bytes(256), stream>>>(m_ah, m_al, m_bh, m_bl, g);
    nonfinite_fixup_kernel<<<(unsigned)cdiv(s.M + s.N, 8), 256, 0, stream>>>(g, (int)chunks_of(s.K));
    return check_launch("gemm_f16x3", s.split_b ? 4 : 3);
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
