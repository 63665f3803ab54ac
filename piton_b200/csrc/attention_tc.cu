// Flash-attention forward on the 5th-generation tensor cores with a 3xTF32-class
// split: tf32 products of the high halves (and hi x lo stacked beside them), bf16
// products for the lo x hi cross terms (examples/attention.py:33-113; the
// semantics are those of attention.cu's header: key_end, causal mask, row_end,
// base-2 online softmax).
//
// Per call:
//  1. split (HBM-bound): K -> K_lo (tf32 of the rest) and K_bf (bf16) as
//     [heads * n_ctx, D], and K_hi unless K itself can serve (the tensor core
//     ignores the low 13 bits of an fp32 operand: K is read in place when its
//     rows are one 16-byte-multiple stride apart across heads); V -> V^T_hi,
//     V^T_lo as [heads * D, ld] (ld = n_ctx rounded up to 4) and V^T_bf as
//     [heads * D, ldb] (ldb = n_ctx rounded up to 8), through 64 x 64 tiles
//     with 16-byte stores (split.cuh) when V's rows are 16-byte aligned.
//  2. persistent CTAs walk (head, 128-query block) items, 352 threads:
//     * warps 2-9, two per TMEM lane quarter (one thread per query row =
//       TMEM lane in each), each warp of a pair on half of the columns: they
//       load their half of the row of Q, split it and store Q_hi (tf32) and
//       Q_lo (bf16, two per column) into TMEM; per 64-key block each reads
//       its 32 keys' scores S from TMEM, applies scale and masks, exchanges
//       its row maximum with the other warp through shared memory (an
//       mbarrier per pair and block parity), updates the running max and its
//       partial sum in registers, writes P_hi over S and P_lo (bf16) next to
//       it in TMEM, then folds its 32 output dimensions of the block's P.V
//       into an fp32 register accumulator (round to nearest); at the end of
//       an item the pair adds its partial sums and each stores its half of
//       O / l.  (One warp per row ran latency-bound at ~5 cycles per
//       instruction, slower than the tensor core.)
//     * warp 0 streams Q and the K tiles, warp 10 the V^T tiles, with TMA
//       (128-byte swizzle; separate two-stage rings, since a K tile is free
//       after S and a V tile only after P.V);
//     * warp 11, only in the all-gather launch (384 threads), copies each item's
//       stored rows from this rank's output to every other rank's (NVLink peer
//       stores), one item behind the softmax warps;
//     * warp 1 issues, from one thread, per 8-wide k-step one tf32 MMA of Q_hi
//       against the stacked [K_hi; K_lo] tile (N = 128: Q_hi K_hi in columns
//       0-63, Q_hi K_lo in 64-127), and per 16-wide k-step one bf16 MMA of
//       Q_lo against K_bf (N = 64, added to columns 0-63); likewise P_hi
//       [V_hi; V_lo] and P_lo V_bf for P.V.  The softmax warps add the two
//       halves in fp32 registers (round to nearest), so the hi/lo sums are not
//       truncated by the tensor core.  The lo x hi cross term is at most
//       2^-10 of the product, so rounding both of its operands to bf16 (8-bit
//       mantissas) leaves it correct to at most 2^-18 of the product, while a
//       bf16 MMA covers twice the k range of a tf32 one in the same issue
//       time: 12 MMAs per 64-key block for S and 12 for P.V instead of 16 each.
//     A block's P.V lands in its own TMEM accumulator that the softmax warps
//     add into registers, so the tensor core's truncating accumulation never
//     spans more than one 64-key block.
// The scores of block j+1 are computed while the softmax warps work on block
// j (two S/P buffers), and a block's P.V accumulator is folded into the
// registers after the next block's P is written, so the tensor core and the
// softmax warps overlap.  TMEM columns: Q_hi [0,64) Q_lo [64,96), S/P x2
// [128,384) (128 each), O_blk [384,512) (512 allocated).  All waits are
// bounded (2 s): on expiry the kernel records a status, drains its copies and
// MMAs, frees TMEM and returns.
#include <algorithm>

#include <cuda_bf16.h>

#include "attention.cuh"
#include "common.cuh"
#include "sm100.cuh"
#include "split.cuh"

namespace piton {

// Status word of this file's kernels (a device variable is private to its translation
// unit without relocatable device code; piton_b200_device_status reads it through
// attention_tc_status_read_and_clear).
__device__ int g_attn_status = 0;

namespace {

using namespace sm100;

constexpr int BM = 128, BN = 64, HD = 64, KSTAGES = 2, VSTAGES = 2, THREADS = 352;
constexpr int SOFTMAX_WARPS = 8;                          // warps 2-9: two per TMEM lane quarter
constexpr int GATHER_WARP = 11;                           // copies finished rows to the peers (world > 1)
constexpr int GATHER_THREADS = THREADS + 32;              // launch with the gather warp
constexpr uint32_t BOX_BYTES = 64 * 32 * 4;               // 64 rows x 128 bytes (32 fp32 or 64 bf16)
// K stage: for each 32-wide box b of d the hi box and the lo box are adjacent,
// [K_hi b0][K_lo b0][K_hi b1][K_lo b1][K_bf], so one 128-row B operand covers hi rows
// 0-63 and lo rows 64-127; then the bf16 tile (64 keys x 64 d).  V stage: the same over
// 32-wide boxes of keys of V^T, then V^T_bf (64 d x 64 keys).
constexpr uint32_t PAIR_BYTES = 2 * BOX_BYTES;
constexpr uint32_t BF_OFF = 2 * PAIR_BYTES;
constexpr uint32_t STAGE_BYTES = 2 * PAIR_BYTES + BOX_BYTES;
constexpr uint32_t Q_BYTES = BM * HD * 4;                // raw Q rows of one item: two 128 x 32 boxes
// row maxima exchanged between the two warps of a lane quarter ([block parity][half][row]) and
// the row sums at the end of an item ([half][row])
constexpr uint32_t XCHG_BYTES = (2 * 2 * BM + 2 * BM) * 4;
constexpr uint32_t SMEM_BYTES = (KSTAGES + VSTAGES) * STAGE_BYTES + Q_BYTES + XCHG_BYTES + 1024 + 1024;
constexpr int TMEM_COLS = 512;
// TMEM: Q_hi, Q_lo (bf16 pairs), two 128-column S/P buffers (S: Q_hi.K_hi (+ Q_lo.K_bf) in
// 0-63 and Q_hi.K_lo in 64-127; P: P_hi in 0-63, P_lo (bf16 pairs) in 64-95) and a
// 128-column O_blk (P_hi.V_hi (+ P_lo.V_bf) in 0-63, P_hi.V_lo in 64-127)
constexpr uint32_t COL_QHI = 0, COL_QLO = 64, COL_S0 = 128, COL_O = 384;
static_assert(KSTAGES == VSTAGES, "the producers share one ring depth");

// two floats -> bf16 pair (round to nearest), `lo_k` in the low half
__device__ __forceinline__ uint32_t pack_bf16(float lo_k, float hi_k) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo_k, hi_k);
    return *reinterpret_cast<uint32_t *>(&v);
}

__device__ __forceinline__ float tf32_trunc(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }
__device__ __forceinline__ void record_status(int code) { atomicCAS(&g_attn_status, 0, code); }

// hi/lo[h][r][c] (row stride ld) and bf[h][r][c] (row stride ldb; bf16 of the value, round
// to nearest, non-finite values as 0 and finite ones clamped to the bf16 range) from
// src + h*s_h + r*s_r + c*s_c, r < rows, c < cols, through 32 x 32 shared-memory tiles
// (grid.z = heads)
__global__ void __launch_bounds__(256) attn_split_kernel(const float *__restrict__ src, int64_t rows, int64_t cols,
                                                         int64_t s_h, int64_t s_r, int64_t s_c,
                                                         float *__restrict__ hi, float *__restrict__ lo, int64_t ld,
                                                         __nv_bfloat16 *__restrict__ bf, int64_t ldb,
                                                         int lanes_along_rows) {
    __shared__ float tile[32][33];
    const int64_t h = blockIdx.z;
    const int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    const float *base = src + h * s_h;
    for (int j = ty; j < 32; j += 8) {
        int64_t r = lanes_along_rows ? r0 + tx : r0 + j;
        int64_t c = lanes_along_rows ? c0 + j : c0 + tx;
        float v = (r < rows && c < cols) ? base[r * s_r + c * s_c] : 0.0f;
        if (lanes_along_rows) tile[tx][j] = v;
        else tile[j][tx] = v;
    }
    __syncthreads();
    float *hh = hi + h * rows * ld, *ll = lo + h * rows * ld;
    __nv_bfloat16 *bb = bf + h * rows * ldb;
    for (int j = ty; j < 32; j += 8) {
        int64_t r = r0 + j, c = c0 + tx;
        if (r < rows && c < cols) {
            float v = tile[j][tx];
            float x = tf32_trunc(v);
            const bool fin = isfinite(v);
            hh[r * ld + c] = x;
            ll[r * ld + c] = fin ? tf32_trunc(v - x) : 0.0f;
            bb[r * ldb + c] = split_bf16_of(v);
        }
    }
}

// K rows with unit d stride and 16-byte aligned rows: no transpose, float4 in; lo (tf32 of the
// rest) and bf (bf16 of the value) out, and hi (the tf32 high half) unless the kernel reads K in
// place (hi == nullptr).  One thread per 4 d-values; grid-stride over heads x n_ctx x 16.
__global__ void __launch_bounds__(256) attn_split_rows_kernel(const float *__restrict__ src, int64_t n_ctx,
                                                              int64_t heads, int64_t s_h, int64_t s_r,
                                                              float *__restrict__ hi, float *__restrict__ lo,
                                                              __nv_bfloat16 *__restrict__ bf) {
    const int64_t total = heads * n_ctx * (HD / 4);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t q = i % (HD / 4), row = i / (HD / 4), h = row / n_ctx, r = row % n_ctx;
        const float4 v = __ldcs(reinterpret_cast<const float4 *>(src + h * s_h + r * s_r + 4 * q));
        const float vv[4] = {v.x, v.y, v.z, v.w};
        float vh[4], vl[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            vh[e] = tf32_trunc(vv[e]);
            vl[e] = isfinite(vv[e]) ? tf32_trunc(vv[e] - vh[e]) : 0.0f;
        }
        const int64_t o = row * HD + 4 * q;
        if (hi) *reinterpret_cast<float4 *>(hi + o) = make_float4(vh[0], vh[1], vh[2], vh[3]);
        *reinterpret_cast<float4 *>(lo + o) = make_float4(vl[0], vl[1], vl[2], vl[3]);
        *reinterpret_cast<uint2 *>(bf + o) = make_uint2(split_bf16_pair(vv[0], vv[1]), split_bf16_pair(vv[2], vv[3]));
    }
}

struct TcAttnArgs {
    float *o;
    int64_t soh, som;
    int64_t n_ctx, key_end, row_end, heads, q_blocks, items;
    float qk_scale;
    int causal;
};

// The all-gather launch: o is this rank's part of its own full output, and every finished row
// is also stored at the same offset from peer_o[r] (rank r's full output, offset to this rank's
// first head) for every other rank r.  (A separate type keeps the plain kernel's parameters,
// and with them its register allocation, as they are.)
struct TcAttnGatherArgs : TcAttnArgs {
    int world, rank;
    float *peer_o[MAX_PEERS];
};
template <int NTHREADS> struct AttnArgsOf { using type = TcAttnArgs; };
template <> struct AttnArgsOf<GATHER_THREADS> { using type = TcAttnGatherArgs; };

__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity) {
    bool ok = mbar_wait(bar, parity);
    return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Work item -> (head, query block): items of one head are consecutive (its K / V stay in
// L2 while they run), the heavy late query blocks of a head first.  Every item has at
// least one key block (attention_tc_supported requires key_end >= 1).
struct Item {
    int64_t head, q0;
    int nblocks;
};

__device__ __forceinline__ Item item_of(const TcAttnArgs &a, int64_t it) {
    Item r;
    r.head = it / a.q_blocks;
    const int64_t qb = a.q_blocks - 1 - it % a.q_blocks;
    r.q0 = qb * BM;
    int64_t kend = a.key_end;
    if (a.causal && r.q0 + BM < kend) kend = r.q0 + BM;
    r.nblocks = kend > 0 ? (int)((kend + BN - 1) / BN) : 0;
    return r;
}

template <int NTHREADS>   // THREADS, or GATHER_THREADS for the all-gather
__global__ void __launch_bounds__(NTHREADS, 1)
    attn_3xtf32_kernel(const __grid_constant__ CUtensorMap m_q, const __grid_constant__ CUtensorMap m_khi,
                       const __grid_constant__ CUtensorMap m_klo, const __grid_constant__ CUtensorMap m_kbf,
                       const __grid_constant__ CUtensorMap m_vhi, const __grid_constant__ CUtensorMap m_vlo,
                       const __grid_constant__ CUtensorMap m_vbf, const typename AttnArgsOf<NTHREADS>::type a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *kst = smem;                                          // K stages
    uint8_t *vst = smem + KSTAGES * STAGE_BYTES;                  // V^T stages
    uint8_t *qbuf = vst + VSTAGES * STAGE_BYTES;                  // raw Q rows of the next item
    float *xmax = reinterpret_cast<float *>(qbuf + Q_BYTES);       // [2][2][BM]
    float *xsum = xmax + 2 * 2 * BM;                               // [2][BM]
    uint64_t *k_full = reinterpret_cast<uint64_t *>(qbuf + Q_BYTES + XCHG_BYTES);
    uint64_t *k_empty = k_full + KSTAGES;
    uint64_t *v_full = k_empty + KSTAGES;
    uint64_t *v_empty = v_full + VSTAGES;
    uint64_t *s_full = v_empty + VSTAGES;     // [2]
    uint64_t *p_full = s_full + 2;            // [2]
    uint64_t *q_full = p_full + 2;            // Q rows landed in qbuf
    uint64_t *q_empty = q_full + 1;           // qbuf consumed (moved to TMEM)
    uint64_t *q_ready = q_empty + 1;          // Q_hi / Q_lo in TMEM
    uint64_t *o_full = q_ready + 1;
    uint64_t *o_empty = o_full + 1;
    uint64_t *drain = o_empty + 1;
    uint64_t *max_bar = drain + 1;            // [4 quarters][2 block parities], 64 arrivals
    uint64_t *sum_bar = max_bar + 8;          // [4 quarters], 64 arrivals
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(sum_bar + 4);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);
    volatile int *rows_stored = abort_flag + 1;   // softmax-warp item stores done (8 per item)

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < KSTAGES; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
        }
        for (int s = 0; s < VSTAGES; ++s) {
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&s_full[b], 1);
            mbar_init(&p_full[b], SOFTMAX_WARPS);
        }
        mbar_init(q_full, 1);
        mbar_init(q_empty, SOFTMAX_WARPS);
        mbar_init(q_ready, SOFTMAX_WARPS);
        mbar_init(o_full, 1);
        mbar_init(o_empty, SOFTMAX_WARPS);
        mbar_init(drain, 1);
        for (int b = 0; b < 8; ++b) mbar_init(&max_bar[b], 64);
        for (int b = 0; b < 4; ++b) mbar_init(&sum_bar[b], 64);
        *abort_flag = 0;
        if constexpr (NTHREADS > THREADS) *rows_stored = 0;
        fence_mbarrier_init();
        prefetch_tmap(&m_q);
        prefetch_tmap(&m_khi);
        prefetch_tmap(&m_klo);
        prefetch_tmap(&m_kbf);
        prefetch_tmap(&m_vhi);
        prefetch_tmap(&m_vlo);
        prefetch_tmap(&m_vbf);
    }
    if (warp == 1) tmem_alloc<TMEM_COLS>(tmem_holder);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp == 0 || warp == 10) {
        // ---------------- TMA producers: warp 0 Q rows (one item ahead) and K tiles, warp 10 V^T tiles ----------------
        if (lane == 0) {
            const bool is_k = warp == 0;
            uint64_t *full = is_k ? k_full : v_full, *empty = is_k ? k_empty : v_empty;
            uint8_t *stages = is_k ? kst : vst;
            const CUtensorMap *m_hi = is_k ? &m_khi : &m_vhi, *m_lo = is_k ? &m_klo : &m_vlo,
                              *m_bf = is_k ? &m_kbf : &m_vbf;
            constexpr int NST = KSTAGES;   // == VSTAGES
            uint32_t g = 0, nq = 0;        // blocks and Q tiles issued
            bool ok = true;
            auto load_q = [&](int64_t it) -> bool {
                // qbuf is free once the previous Q tile has been moved into TMEM
                if (nq > 0 && !mbar_wait(q_empty, (nq - 1) & 1)) return false;
                const Item n = item_of(a, it);
                mbar_arrive_expect_tx(q_full, Q_BYTES);
                tma_load_3d(qbuf, &m_q, q_full, 0, (int)n.q0, (int)n.head);
                tma_load_3d(qbuf + Q_BYTES / 2, &m_q, q_full, 32, (int)n.q0, (int)n.head);
                ++nq;
                return true;
            };
            if (is_k && (int64_t)blockIdx.x < a.items) ok = load_q(blockIdx.x);
            for (int64_t it = blockIdx.x; ok && it < a.items && !*abort_flag; it += gridDim.x) {
                const Item w = item_of(a, it);
                const bool next = it + gridDim.x < a.items;
                for (int j = 0; j < w.nblocks && !*abort_flag; ++j, ++g) {
                    const int s = g % NST;
                    if (!mbar_wait(&empty[s], ((g / NST) & 1) ^ 1)) {
                        ok = false;
                        break;
                    }
                    uint8_t *st = stages + s * STAGE_BYTES;
                    mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
                    // K: rows = keys of this head, x = d; V^T: rows = d of this head, x = keys
                    const int row = is_k ? (int)(w.head * a.n_ctx + (int64_t)j * BN) : (int)(w.head * HD);
                    const int x0 = is_k ? 0 : j * BN;
                    for (int box = 0; box < 2; ++box) {
                        tma_load_2d(st + box * PAIR_BYTES, m_hi, &full[s], x0 + box * 32, row);
                        tma_load_2d(st + box * PAIR_BYTES + BOX_BYTES, m_lo, &full[s], x0 + box * 32, row);
                    }
                    tma_load_2d(st + BF_OFF, m_bf, &full[s], x0, row);
                    // the next item's Q, once this item's Q has left qbuf (early in this item)
                    if (is_k && next && j == (w.nblocks > 1 ? 1 : 0) && !(ok = load_q(it + gridDim.x))) break;
                }
            }
            if (!ok) {
                record_status(STATUS_TIMEOUT_PRODUCER);
                *abort_flag = 1;
            }
            for (uint32_t j = g > NST ? g - NST : 0; j < g; ++j)
                if (!mbar_wait(&full[j % NST], (j / NST) & 1)) record_status(STATUS_TIMEOUT_DRAIN);
            if (is_k && nq > 0 && !mbar_wait(q_full, (nq - 1) & 1)) record_status(STATUS_TIMEOUT_DRAIN);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer: S of block j+1 is issued before P_j V so it overlaps softmax j ----------------
        if (lane == 0) {
            constexpr uint32_t IDESC_N128 = idesc_tf32(BM, 2 * BN), IDESC_BF = idesc_bf16(BM, BN);
            uint32_t g = 0, k = 0;   // global block counter, items done
            bool ok = true;
            auto issue_s = [&](uint32_t gg) -> bool {
                const int s = gg % KSTAGES;
                if (!mbar_wait(&k_full[s], (gg / KSTAGES) & 1)) return false;
                tc_fence_after();
                const uint32_t base = smem_u32(kst + s * STAGE_BYTES);
                const uint32_t d = tmem + COL_S0 + (gg & 1) * 2 * BN;
#pragma unroll
                for (int ks = 0; ks < HD / 8; ++ks) {
                    const uint32_t pair = base + (ks >> 2) * PAIR_BYTES + (ks & 3) * 32;
                    const uint64_t b_pair = smem_desc_kmajor(pair, 128, LAYOUT_SWIZZLE_128B);   // K_hi; K_lo rows
                    mma_tf32_ts(d, tmem + COL_QHI + 8 * ks, b_pair, IDESC_N128, ks > 0 ? 1u : 0u);
                }
#pragma unroll
                for (int kb = 0; kb < HD / 16; ++kb)   // Q_lo . K_bf, 16 d per MMA
                    mma_bf16_ts(d, tmem + COL_QLO + 8 * kb,
                                smem_desc_kmajor(base + BF_OFF + kb * 32, 128, LAYOUT_SWIZZLE_128B), IDESC_BF);
                mma_commit(&s_full[gg & 1]);
                mma_commit(&k_empty[s]);
                return true;
            };
            for (int64_t it = blockIdx.x; ok && it < a.items && !*abort_flag; it += gridDim.x, ++k) {
                const Item w = item_of(a, it);
                if (!mbar_wait(q_ready, k & 1)) {   // this item's Q in TMEM
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (!(ok = issue_s(g))) break;
                for (int j = 0; j < w.nblocks && !*abort_flag; ++j, ++g) {
                    if (j + 1 < w.nblocks && !(ok = issue_s(g + 1))) break;
                    const int s = g % VSTAGES;
                    if (!mbar_wait(&p_full[g & 1], (g >> 1) & 1) || (g > 0 && !mbar_wait(o_empty, (g - 1) & 1)) ||
                        !mbar_wait(&v_full[s], (g / VSTAGES) & 1)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t base = smem_u32(vst + s * STAGE_BYTES);
                    const uint32_t pcol = tmem + COL_S0 + (g & 1) * 2 * BN;
#pragma unroll
                    for (int ks = 0; ks < BN / 8; ++ks) {
                        const uint32_t pair = base + (ks >> 2) * PAIR_BYTES + (ks & 3) * 32;
                        const uint64_t b_pair = smem_desc_kmajor(pair, 128, LAYOUT_SWIZZLE_128B);   // V^T_hi; V^T_lo
                        mma_tf32_ts(tmem + COL_O, pcol + 8 * ks, b_pair, IDESC_N128, ks > 0 ? 1u : 0u);   // P_hi
                    }
#pragma unroll
                    for (int kb = 0; kb < BN / 16; ++kb)   // P_lo . V_bf, 16 keys per MMA
                        mma_bf16_ts(tmem + COL_O, pcol + BN + 8 * kb,
                                    smem_desc_kmajor(base + BF_OFF + kb * 32, 128, LAYOUT_SWIZZLE_128B), IDESC_BF);
                    mma_commit(o_full);
                    mma_commit(&v_empty[s]);
                }
            }
            if (!ok) {
                record_status(STATUS_TIMEOUT_MMA);
                *abort_flag = 1;
            }
            mma_commit(drain);
            if (!mbar_wait(drain, 0)) record_status(STATUS_TIMEOUT_DRAIN);
        }
    } else if (NTHREADS > THREADS && warp == GATHER_WARP) {
        // ---------------- all-gather (world > 1): each item's stored rows to every other rank ----------------
        // The rows are read back from this rank's own output (L2) once all eight softmax warps
        // have stored them, so the NVLink stores never hold up the softmax warps; this warp
        // trails them by up to the items still in flight and finishes the kernel's last ones.
        if constexpr (NTHREADS > THREADS) {
            int need = 0;
            for (int64_t it = blockIdx.x; it < a.items; it += gridDim.x) {
                need += SOFTMAX_WARPS;
                int go = 1;
                if (lane == 0 && *rows_stored < need) {
                    const uint64_t t0 = globaltimer();
                    while (*rows_stored < need) {
                        if (*abort_flag || globaltimer() - t0 > 2000000000ull) {
                            go = 0;
                            break;
                        }
                        __nanosleep(200);
                    }
                }
                if (!__shfl_sync(0xffffffffu, go, 0)) {
                    if (lane == 0 && !*abort_flag) record_status(STATUS_TIMEOUT_EPILOGUE);
                    break;
                }
                __threadfence();   // pairs with the softmax warps' fence before their count
                const Item w = item_of(a, it);
                const int64_t r_end = w.q0 + BM < a.row_end ? w.q0 + BM : a.row_end;
                const int n4 = (int)(r_end - w.q0) * (HD / 4);
                const int64_t base = w.head * a.soh + w.q0 * a.som;
                constexpr int U = 8;   // float4 loads in flight per lane
                for (int i0 = 0; i0 < n4; i0 += 32 * U) {
                    float4 v[U];
                    int64_t off[U];
#pragma unroll
                    for (int u = 0; u < U; ++u) {
                        const int i = i0 + u * 32 + lane;
                        off[u] = base + (int64_t)(i >> 4) * a.som + 4 * (i & 15);
                        if (i < n4) v[u] = __ldcg(reinterpret_cast<const float4 *>(a.o + off[u]));
                    }
                    for (int p = 1; p < a.world; ++p) {
                        float *dst = a.peer_o[(a.rank + p) % a.world];
#pragma unroll
                        for (int u = 0; u < U; ++u)
                            if (i0 + u * 32 + lane < n4) *reinterpret_cast<float4 *>(dst + off[u]) = v[u];
                    }
                }
            }
        }
    } else {
        // ---------------- softmax / accumulate / store (warps 2-9) ----------------
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2;    // this warp's 32 keys of a block and 32 dimensions of O
        const int rloc = quarter * 32 + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
        uint32_t g = 0, nq = 0, k = 0;
        bool ok = true;
        // qbuf (raw Q rows, 128-byte swizzle, two 32-column boxes) -> tf32 hi / bf16 lo -> TMEM;
        // this warp converts columns [32 * half, 32 * half + 32) = box `half`
        auto q_to_tmem = [&]() -> bool {
            if (*abort_flag || !warp_wait(q_full, nq & 1)) return false;
            uint32_t hi[2][16], lo[16];
#pragma unroll
            for (int v4 = 0; v4 < 8; ++v4) {
                const float4 x = *reinterpret_cast<const float4 *>(qbuf + half * (Q_BYTES / 2) + rloc * 128 +
                                                                   ((v4 ^ (rloc & 7)) << 4));
                const float xv[4] = {x.x, x.y, x.z, x.w};
                float l[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float h = tf32_trunc(xv[e]);
                    hi[v4 >> 2][4 * (v4 & 3) + e] = __float_as_uint(h);
                    l[e] = isfinite(xv[e]) ? xv[e] - h : 0.0f;
                }
                lo[2 * v4] = pack_bf16(l[0], l[1]);
                lo[2 * v4 + 1] = pack_bf16(l[2], l[3]);
            }
            tmem_st_32x32b_x16(lane_base + COL_QHI + 32 * half, hi[0]);
            tmem_st_32x32b_x16(lane_base + COL_QHI + 32 * half + 16, hi[1]);
            tmem_st_32x32b_x16(lane_base + COL_QLO + 16 * half, lo);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(q_empty);
                mbar_arrive(q_ready);
            }
            ++nq;
            return true;
        };
        constexpr int HH = HD / 2;
        float acc[HH];
        // acc = acc * alpha + this warp's 32 dimensions of O_blk of global block gg
        auto fold = [&](uint32_t gg, float alpha) -> bool {
            if (*abort_flag || !warp_wait(o_full, gg & 1)) return false;
            tc_fence_after();
            uint32_t r[2 * HH];
#pragma unroll
            for (int c = 0; c < HH; c += 16) {
                tmem_ld_32x32b_x16(lane_base + COL_O + HH * half + c, *reinterpret_cast<uint32_t(*)[16]>(r + c));
                tmem_ld_32x32b_x16(lane_base + COL_O + HD + HH * half + c, *reinterpret_cast<uint32_t(*)[16]>(r + HH + c));
            }
            tmem_ld_wait();
#pragma unroll
            for (int c = 0; c < HH; ++c)
                acc[c] = fmaf(acc[c], alpha, __uint_as_float(r[c]) + __uint_as_float(r[HH + c]));
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(o_empty);
            return true;
        };
        const bool o_vec = ((reinterpret_cast<uintptr_t>(a.o) | (uintptr_t)(a.soh * 4) | (uintptr_t)(a.som * 4)) & 15) == 0;
        if ((int64_t)blockIdx.x < a.items) ok = q_to_tmem();
        for (int64_t it = blockIdx.x; ok && it < a.items; it += gridDim.x, ++k) {
            const Item w = item_of(a, it);
            const int64_t row = w.q0 + rloc;
            const bool next = it + gridDim.x < a.items;   // its Q follows this item's last P
            float m_i = -INFINITY, l_i = 0.0f, alpha_prev = 1.0f;
#pragma unroll
            for (int d = 0; d < HH; ++d) acc[d] = 0.0f;
            for (int j = 0; j < w.nblocks; ++j, ++g) {
                if (*abort_flag || !warp_wait(&s_full[g & 1], (g >> 1) & 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                constexpr int KH = BN / 2;
                const int64_t k0 = (int64_t)j * BN + KH * half;   // this warp's first key
                const uint32_t scol = COL_S0 + (g & 1) * 2 * BN, pcol = scol + BN;
                float sc[KH];
                {
                    uint32_t r[2 * KH];
#pragma unroll
                    for (int c = 0; c < KH; c += 16) {
                        tmem_ld_32x32b_x16(lane_base + scol + KH * half + c, *reinterpret_cast<uint32_t(*)[16]>(r + c));
                        tmem_ld_32x32b_x16(lane_base + scol + BN + KH * half + c,
                                           *reinterpret_cast<uint32_t(*)[16]>(r + KH + c));
                    }
                    tmem_ld_wait();
#pragma unroll
                    for (int c = 0; c < KH; ++c) sc[c] = __uint_as_float(r[c]) + __uint_as_float(r[KH + c]);
                }
                // masks only on the blocks that reach past key_end or the causal diagonal
                const bool masked = k0 + KH > a.key_end || (a.causal && k0 + KH - 1 > w.q0);
                if (masked) {
#pragma unroll
                    for (int c = 0; c < KH; ++c) {
                        const int64_t col = k0 + c;
                        if (col >= a.key_end || (a.causal && col > row)) sc[c] = -INFINITY;
                    }
                }
                float m0 = sc[0], m1 = sc[1], m2 = sc[2], m3 = sc[3];
#pragma unroll
                for (int c = 4; c < KH; c += 4) {
                    m0 = fmaxf(m0, sc[c]);
                    m1 = fmaxf(m1, sc[c + 1]);
                    m2 = fmaxf(m2, sc[c + 2]);
                    m3 = fmaxf(m3, sc[c + 3]);
                }
                // the row maximum over both halves (scale > 0, so max(s) * scale = max(s * scale))
                const float m_mine = fmaxf(fmaxf(m0, m1), fmaxf(m2, m3));
                float *xm = xmax + (g & 1) * 2 * BM;
                xm[half * BM + rloc] = m_mine;
                mbar_arrive(&max_bar[quarter * 2 + (g & 1)]);
                if (!warp_wait(&max_bar[quarter * 2 + (g & 1)], (g >> 1) & 1)) {
                    ok = false;
                    break;
                }
                const float m_new = fmaxf(m_i, fmaxf(m_mine, xm[(half ^ 1) * BM + rloc]) * a.qk_scale);
                const float m_use = m_new == -INFINITY ? 0.0f : m_new;
                const float alpha = fast_exp2(m_i - m_use);
                float ps0 = 0.0f, ps1 = 0.0f;
                uint32_t hi[2][16], lo[16];
#pragma unroll
                for (int e = 0; e < KH; e += 2) {
                    const float p0 = fast_exp2(fmaf(sc[e], a.qk_scale, -m_use));
                    const float p1 = fast_exp2(fmaf(sc[e + 1], a.qk_scale, -m_use));
                    ps0 += p0;
                    ps1 += p1;
                    const float h0 = tf32_trunc(p0), h1 = tf32_trunc(p1);
                    hi[e >> 4][e & 15] = __float_as_uint(h0);
                    hi[e >> 4][(e & 15) + 1] = __float_as_uint(h1);
                    lo[e >> 1] = pack_bf16(p0 - h0, p1 - h1);   // the differences are exact
                }
                tmem_st_32x32b_x16(lane_base + scol + KH * half, hi[0]);
                tmem_st_32x32b_x16(lane_base + scol + KH * half + 16, hi[1]);
                tmem_st_32x32b_x16(lane_base + pcol + 16 * half, lo);
                l_i = l_i * alpha + (ps0 + ps1);
                m_i = m_new;
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[g & 1]);
                // after the item's last scores: the next item's Q (this item's S MMAs are all done)
                if (j == w.nblocks - 1 && next && !(ok = q_to_tmem())) break;
                // fold the previous block's P.V while this block's runs on the tensor core
                if (j > 0 && !fold(g - 1, alpha_prev)) {
                    ok = false;
                    break;
                }
                alpha_prev = alpha;
            }
            if (ok && !fold(g - 1, alpha_prev)) ok = false;
            if (!ok) break;
            // the row sum: this warp's keys plus the other warp's
            xsum[half * BM + rloc] = l_i;
            mbar_arrive(&sum_bar[quarter]);
            if (!warp_wait(&sum_bar[quarter], k & 1)) {
                ok = false;
                break;
            }
            l_i += xsum[(half ^ 1) * BM + rloc];
            if (row < a.row_end) {
                const float inv = 1.0f / l_i;
                float *orow = a.o + w.head * a.soh + row * a.som + HH * half;
                if (o_vec) {   // 16-byte stores: a warp's store covers 32 rows x 16 bytes instead of 32 x 4
#pragma unroll
                    for (int d = 0; d < HH; d += 4)
                        *reinterpret_cast<float4 *>(orow + d) =
                            make_float4(acc[d] * inv, acc[d + 1] * inv, acc[d + 2] * inv, acc[d + 3] * inv);
                } else {
#pragma unroll
                    for (int d = 0; d < HH; ++d) orow[d] = acc[d] * inv;
                }
            }
            if constexpr (NTHREADS > THREADS) {   // the item's rows are in this rank's output: hand them to the gather warp
                __threadfence();
                __syncwarp();
                if (lane == 0) atomicAdd(const_cast<int *>(rows_stored), 1);
            }
        }
        if (!ok) {
            if (lane == 0) record_status(STATUS_TIMEOUT_EPILOGUE);
            *abort_flag = 1;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc<TMEM_COLS>(tmem);
    }
}

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

// row-major fp32 [rows, ld] with inner extent `cols`; boxes of 64 rows x 32 columns, 128-byte swizzle
int make_map(CUtensorMap *map, const float *base, int64_t rows, int64_t cols, int64_t ld) {
    EncodeTiled enc = encode_fn();
    if (!enc) return set_error(PITON_B200_ECUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * 4)};
    cuuint32_t box[2] = {32, 64};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(PITON_B200_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return PITON_B200_OK;
}

// row-major bf16 [rows, ld] with inner extent `cols`; boxes of 64 rows x 64 columns, 128-byte swizzle
int make_map_bf16(CUtensorMap *map, const __nv_bfloat16 *base, int64_t rows, int64_t cols, int64_t ld) {
    EncodeTiled enc = encode_fn();
    if (!enc) return set_error(PITON_B200_ECUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
    cuuint32_t box[2] = {64, 64};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<__nv_bfloat16 *>(base), dims, strides, box,
                     estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(PITON_B200_ECUDA, "cuTensorMapEncodeTiled (bf16) failed (%d)", (int)r);
    return PITON_B200_OK;
}

// Q rows [heads][n_ctx][64] as a 3-D tensor map (row stride sqm, head stride sqh, in floats);
// boxes of 128 rows x 32 columns, 128-byte swizzle.
int make_map_q(CUtensorMap *map, const float *base, int64_t n_ctx, int64_t heads, int64_t sqm, int64_t sqh) {
    EncodeTiled enc = encode_fn();
    if (!enc) return set_error(PITON_B200_ECUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[3] = {(cuuint64_t)HD, (cuuint64_t)n_ctx, (cuuint64_t)heads};
    cuuint64_t strides[2] = {(cuuint64_t)(sqm * 4), (cuuint64_t)(sqh * 4)};
    cuuint32_t box[3] = {32, (cuuint32_t)BM, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(PITON_B200_ECUDA, "cuTensorMapEncodeTiled (Q) failed (%d)", (int)r);
    return PITON_B200_OK;
}

// Q is read by TMA in place when its rows and heads are 16-byte aligned; otherwise it is
// first copied into the workspace as [heads][n_ctx][64].
bool q_in_place(const AttnParams &p) {
    return (reinterpret_cast<uintptr_t>(p.q) & 15) == 0 && p.sqm > 0 && p.sqh > 0 && p.sqm % 4 == 0 &&
           p.sqh % 4 == 0 && p.sqm < (1ll << 37) && p.sqh < (1ll << 37);
}

__global__ void __launch_bounds__(256) attn_q_copy_kernel(const float *__restrict__ src, int64_t n_ctx, int64_t s_h,
                                                          int64_t s_r, float *__restrict__ dst) {
    const int64_t h = blockIdx.y;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_ctx * HD; i += (int64_t)gridDim.x * blockDim.x)
        dst[h * n_ctx * HD + i] = src[h * s_h + (i / HD) * s_r + i % HD];
}

// K split without a transpose: unit d stride, 16-byte aligned rows and heads
bool k_rows_vec(const AttnParams &p) {
    return p.skk == 1 && p.skn % 4 == 0 && p.skh % 4 == 0 && (reinterpret_cast<uintptr_t>(p.k) & 15) == 0;
}
// K read in place as its own tf32 high half (the tensor core ignores the low 13 bits): the rows
// of all heads one stride apart, as the 2-D tensor map [heads * n_ctx, HD] needs
bool k_in_place(const AttnParams &p) {
    return k_rows_vec(p) && p.skn >= HD && p.skh == p.n_ctx * p.skn && p.skn < (1ll << 37);
}
// V^T by the 64 x 64-tile transposing split: d contiguous (always), keys and heads 16-byte aligned
bool v_vec(const AttnParams &p) {
    return p.svn % 4 == 0 && p.svh % 4 == 0 && (reinterpret_cast<uintptr_t>(p.v) & 15) == 0;
}

int64_t v_ld(int64_t n_ctx) { return (n_ctx + 3) / 4 * 4; }
int64_t v_ldb(int64_t n_ctx) { return (n_ctx + 7) / 8 * 8; }   // bf16 rows: 16-byte multiple
size_t k_region(const AttnParams &p) { return ((size_t)p.heads * p.n_ctx * HD * 4 + 1023) / 1024 * 1024; }
size_t v_region(const AttnParams &p) { return ((size_t)p.heads * HD * v_ld(p.n_ctx) * 4 + 1023) / 1024 * 1024; }
size_t kb_region(const AttnParams &p) { return ((size_t)p.heads * p.n_ctx * HD * 2 + 1023) / 1024 * 1024; }
size_t vb_region(const AttnParams &p) { return ((size_t)p.heads * HD * v_ldb(p.n_ctx) * 2 + 1023) / 1024 * 1024; }
size_t q_region(const AttnParams &p) {
    return q_in_place(p) ? 0 : ((size_t)p.heads * p.n_ctx * HD * 4 + 1023) / 1024 * 1024;
}

}  // namespace

bool attention_tc_supported(const AttnParams &p) {
    if (p.head_dim != HD || p.n_ctx < 64 || p.heads < 1 || p.key_end < 1) return false;
    if (p.heads * p.n_ctx >= (1ll << 31) || p.heads * HD >= (1ll << 31)) return false;
    if ((p.n_ctx + 31) / 32 > 65535 || p.heads > 65535) return false;
    int64_t q_blocks = (p.row_end + BM - 1) / BM;
    if (q_blocks * p.heads >= (1ll << 31)) return false;
    return encode_fn() != nullptr;
}

size_t attention_tc_workspace_bytes(const AttnParams &p) {
    return 2 * k_region(p) + 2 * v_region(p) + kb_region(p) + vb_region(p) + q_region(p);
}

int attention_tc(const AttnParams &p, void *workspace, cudaStream_t stream) {
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    float *k_hi = reinterpret_cast<float *>(ws);
    float *k_lo = reinterpret_cast<float *>(ws + k_region(p));
    float *v_hi = reinterpret_cast<float *>(ws + 2 * k_region(p));
    float *v_lo = reinterpret_cast<float *>(ws + 2 * k_region(p) + v_region(p));
    __nv_bfloat16 *k_bf = reinterpret_cast<__nv_bfloat16 *>(ws + 2 * k_region(p) + 2 * v_region(p));
    __nv_bfloat16 *v_bf = reinterpret_cast<__nv_bfloat16 *>(ws + 2 * k_region(p) + 2 * v_region(p) + kb_region(p));
    const int64_t ldv = v_ld(p.n_ctx), ldvb = v_ldb(p.n_ctx);
    // K [n_ctx, D] per head (strides skn, skk) -> [heads * n_ctx, D]
    const bool k_direct = k_in_place(p);
    if (k_rows_vec(p)) {
        const int64_t total = p.heads * p.n_ctx * (HD / 4);
        const int64_t blocks = std::min<int64_t>(cdiv(total, (int64_t)256), (int64_t)num_sms() * 16);
        attn_split_rows_kernel<<<(unsigned)blocks, 256, 0, stream>>>(p.k, p.n_ctx, p.heads, p.skh, p.skn,
                                                                     k_direct ? nullptr : k_hi, k_lo, k_bf);
    } else {
        dim3 g((unsigned)cdiv(HD, 32), (unsigned)cdiv(p.n_ctx, 32), (unsigned)p.heads);
        int along_rows = llabs(p.skn) < llabs(p.skk);
        attn_split_kernel<<<g, 256, 0, stream>>>(p.k, p.n_ctx, HD, p.skh, p.skn, p.skk, k_hi, k_lo, HD, k_bf, HD,
                                                 along_rows);
    }
    // V [n_ctx, D] per head (strides svn, 1) -> V^T [heads * D, ldv]
    if (v_vec(p)) {
        dim3 g((unsigned)cdiv(p.n_ctx, 64), 1, (unsigned)p.heads);
        split_transpose_kernel<SPLIT_T_ATTN_V><<<g, 256, 0, stream>>>(p.v, HD, p.n_ctx, p.svn, p.svh, v_hi, v_lo, v_bf,
                                                                       ldv, ldvb);
    } else {
        dim3 g((unsigned)cdiv(p.n_ctx, 32), (unsigned)cdiv(HD, 32), (unsigned)p.heads);
        attn_split_kernel<<<g, 256, 0, stream>>>(p.v, HD, p.n_ctx, p.svh, 1, p.svn, v_hi, v_lo, ldv, v_bf, ldvb, 1);
    }
    int launches = 3;
    const float *q = p.q;
    int64_t sqm = p.sqm, sqh = p.sqh;
    if (!q_in_place(p)) {
        float *qc = reinterpret_cast<float *>(ws + 2 * k_region(p) + 2 * v_region(p) + kb_region(p) + vb_region(p));
        dim3 g((unsigned)std::min<int64_t>(cdiv(p.n_ctx * HD, (int64_t)256), 4096), (unsigned)p.heads);
        attn_q_copy_kernel<<<g, 256, 0, stream>>>(p.q, p.n_ctx, p.sqh, p.sqm, qc);
        q = qc;
        sqm = HD;
        sqh = p.n_ctx * HD;
        ++launches;
    }
    CUtensorMap mq, mkh, mkl, mkb, mvh, mvl, mvb;
    int rc;
    if ((rc = make_map_q(&mq, q, p.n_ctx, p.heads, sqm, sqh)) ||
        (rc = k_direct ? make_map(&mkh, p.k, p.heads * p.n_ctx, HD, p.skn) : make_map(&mkh, k_hi, p.heads * p.n_ctx, HD, HD)) ||
        (rc = make_map(&mkl, k_lo, p.heads * p.n_ctx, HD, HD)) ||
        (rc = make_map_bf16(&mkb, k_bf, p.heads * p.n_ctx, HD, HD)) ||
        (rc = make_map(&mvh, v_hi, p.heads * HD, p.n_ctx, ldv)) || (rc = make_map(&mvl, v_lo, p.heads * HD, p.n_ctx, ldv)) ||
        (rc = make_map_bf16(&mvb, v_bf, p.heads * HD, p.n_ctx, ldvb)))
        return rc;
    static bool attr[64][2] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const bool gather = p.world > 1;
    if (dev < 64 && !attr[dev][gather]) {
        if (gather)
            PITON_CUDA(cudaFuncSetAttribute(attn_3xtf32_kernel<GATHER_THREADS>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
        else
            PITON_CUDA(cudaFuncSetAttribute(attn_3xtf32_kernel<THREADS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            SMEM_BYTES));
        attr[dev][gather] = true;
    }
    TcAttnArgs a;
    a.o = p.o;
    a.soh = p.soh; a.som = p.som;
    a.n_ctx = p.n_ctx; a.key_end = p.key_end; a.row_end = p.row_end; a.heads = p.heads;
    a.q_blocks = (p.row_end + BM - 1) / BM;
    a.items = a.q_blocks * p.heads;
    a.qk_scale = p.qk_scale;
    a.causal = p.causal;
    // persistent: one CTA per SM walks the items (head-major, heavy query blocks first)
    const int64_t grid = std::min<int64_t>(a.items, (int64_t)num_sms());
    if (grid > 0 && gather) {
        TcAttnGatherArgs ga;
        static_cast<TcAttnArgs &>(ga) = a;
        ga.world = p.world;
        ga.rank = p.rank;
        for (int i = 0; i < MAX_PEERS; ++i) ga.peer_o[i] = p.peer_o[i];
        attn_3xtf32_kernel<GATHER_THREADS>
            <<<(unsigned)grid, GATHER_THREADS, SMEM_BYTES, stream>>>(mq, mkh, mkl, mkb, mvh, mvl, mvb, ga);
    } else if (grid > 0)
        attn_3xtf32_kernel<THREADS><<<(unsigned)grid, THREADS, SMEM_BYTES, stream>>>(mq, mkh, mkl, mkb, mvh, mvl, mvb, a);
    return check_launch("attention_3xtf32", launches);
}

int attention_tc_status_read_and_clear(int *status) {
    int zero = 0;
    PITON_CUDA(cudaMemcpyFromSymbol(status, g_attn_status, sizeof(int)));
    PITON_CUDA(cudaMemcpyToSymbol(g_attn_status, &zero, sizeof(int)));
    return PITON_B200_OK;
}

}  // namespace piton
