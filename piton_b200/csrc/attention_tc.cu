// Flash-attention forward on the 5th-generation tensor cores with the 3xTF32
// split (examples/attention.py:33-113; the semantics are those of
// attention.cu's header: key_end, causal mask, row_end, base-2 online softmax).
//
// Per call:
//  1. split: K -> K_hi, K_lo as [heads * n_ctx, D] and V -> V^T_hi, V^T_lo as
//     [heads * D, ld] (ld = n_ctx rounded up to 4), tf32 hi/lo halves, into the
//     workspace.
//  2. one CTA per (head, 128-query block), 192 threads:
//     * warps 2-5 (one thread per query row = TMEM lane) load the row of Q,
//       split it and store Q_hi, Q_lo into TMEM; per 64-key block they read
//       the scores S from TMEM, apply scale and masks, update the running max
//       and sum in registers (no shuffles: a row lives in one thread), write
//       P_hi over S and P_lo next to it in TMEM, then fold the block's P.V
//       into an fp32 register accumulator (round to nearest) and finally
//       store O / l;
//     * warp 0 streams K and V^T tiles with TMA (128-byte swizzle);
//     * warp 1 issues, from one thread, per 8-wide k-step two MMAs: Q_hi
//       against the stacked [K_hi; K_lo] tile (N = 128: Q_hi K_hi in columns
//       0-63, Q_hi K_lo in 64-127) and Q_lo against K_hi (N = 64, added to
//       columns 0-63); likewise P_hi [V_hi; V_lo] and P_lo V_hi for P.V.  The
//       softmax warps add the two halves in fp32 registers (round to
//       nearest), so each MMA instruction carries more work and the hi/lo sums
//       are not truncated by the tensor core.
//     A block's P.V lands in its own TMEM accumulator that the softmax warps
//     add into registers, so the tensor core's truncating accumulation never
//     spans more than one 64-key block.
// The scores of block j+1 are computed while the softmax warps work on block
// j (two S/P buffers), and a block's P.V accumulator is folded into the
// registers after the next block's P is written, so the tensor core and the
// softmax warps overlap.  TMEM columns: Q_hi [0,64) Q_lo [64,128)
// S/P x2 [128,384) (128 each) O_blk [384,512) (512 allocated).
// K / V^T tiles: 3-stage TMA ring.  All waits are bounded (2 s): on expiry
// the kernel records a status, drains its copies and MMAs, frees TMEM, returns.
#include <algorithm>

#include "attention.cuh"
#include "common.cuh"
#include "sm100.cuh"

namespace piton {

// Status word of this file's kernels (a device variable is private to its translation
// unit without relocatable device code; piton_b200_device_status reads it through
// attention_tc_status_read_and_clear).
__device__ int g_attn_status = 0;

namespace {

using namespace sm100;

constexpr int BM = 128, BN = 64, HD = 64, STAGES = 3, THREADS = 192;
constexpr uint32_t BOX_BYTES = 64 * 32 * 4;               // 64 rows x 128 bytes
constexpr uint32_t TILE_BYTES = 2 * BOX_BYTES;            // one 64 x 64 fp32 operand tile
constexpr uint32_t STAGE_BYTES = 4 * TILE_BYTES;          // K_hi, K_lo, V^T_hi, V^T_lo
// Stage layout: for each 32-wide box b (d for K, keys for V^T) the hi box and the lo
// box are adjacent, [K_hi b0][K_lo b0][K_hi b1][K_lo b1][V_hi b0][V_lo b0][V_hi b1][V_lo b1],
// so one 128-row B operand covers hi rows 0-63 and lo rows 64-127.
constexpr uint32_t PAIR_BYTES = 2 * BOX_BYTES;
constexpr uint32_t V_BASE = 2 * PAIR_BYTES;
constexpr uint32_t Q_BYTES = BM * HD * 4;                // raw Q rows of one item: two 128 x 32 boxes
constexpr uint32_t SMEM_BYTES = STAGES * STAGE_BYTES + Q_BYTES + 1024 + 1024;
constexpr int TMEM_COLS = 512;
// TMEM: Q_hi, Q_lo, two 128-column S/P buffers (S: Q_hi.K_hi (+ Q_lo.K_hi) in 0-63 and
// Q_hi.K_lo in 64-127; P: P_hi in 0-63, P_lo in 64-127) and a 128-column O_blk
// (P_hi.V_hi (+ P_lo.V_hi) in 0-63, P_hi.V_lo in 64-127)
constexpr uint32_t COL_QHI = 0, COL_QLO = 64, COL_S0 = 128, COL_O = 384;

__device__ __forceinline__ float tf32_trunc(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }
__device__ __forceinline__ void record_status(int code) { atomicCAS(&g_attn_status, 0, code); }

// hi/lo[h][r][c] (row stride ld) from src + h*s_h + r*s_r + c*s_c, r < rows, c < cols,
// through 32 x 32 shared-memory tiles (grid.z = heads)
__global__ void __launch_bounds__(256) attn_split_kernel(const float *__restrict__ src, int64_t rows, int64_t cols,
                                                         int64_t s_h, int64_t s_r, int64_t s_c,
                                                         float *__restrict__ hi, float *__restrict__ lo, int64_t ld,
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
    for (int j = ty; j < 32; j += 8) {
        int64_t r = r0 + j, c = c0 + tx;
        if (r < rows && c < cols) {
            float v = tile[j][tx];
            float x = tf32_trunc(v);
            hh[r * ld + c] = x;
            ll[r * ld + c] = isfinite(v) ? tf32_trunc(v - x) : 0.0f;
        }
    }
}

struct TcAttnArgs {
    float *o;
    int64_t soh, som;
    int64_t n_ctx, key_end, row_end, heads, q_blocks, items;
    float qk_scale;
    int causal;
};

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

__global__ void __launch_bounds__(THREADS, 1)
    attn_3xtf32_kernel(const __grid_constant__ CUtensorMap m_q, const __grid_constant__ CUtensorMap m_khi,
                       const __grid_constant__ CUtensorMap m_klo, const __grid_constant__ CUtensorMap m_vhi,
                       const __grid_constant__ CUtensorMap m_vlo, TcAttnArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *qbuf = smem + STAGES * STAGE_BYTES;                 // raw Q rows of the next item
    uint64_t *kv_full = reinterpret_cast<uint64_t *>(qbuf + Q_BYTES);
    uint64_t *kv_empty = kv_full + STAGES;
    uint64_t *s_full = kv_empty + STAGES;     // [2]
    uint64_t *p_full = s_full + 2;            // [2]
    uint64_t *q_full = p_full + 2;            // Q rows landed in qbuf
    uint64_t *q_empty = q_full + 1;           // qbuf consumed (moved to TMEM)
    uint64_t *q_ready = q_empty + 1;          // Q_hi / Q_lo in TMEM
    uint64_t *o_full = q_ready + 1;
    uint64_t *o_empty = o_full + 1;
    uint64_t *drain = o_empty + 1;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&s_full[b], 1);
            mbar_init(&p_full[b], 4);
        }
        mbar_init(q_full, 1);
        mbar_init(q_empty, 4);
        mbar_init(q_ready, 4);
        mbar_init(o_full, 1);
        mbar_init(o_empty, 4);
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbarrier_init();
        prefetch_tmap(&m_q);
        prefetch_tmap(&m_khi);
        prefetch_tmap(&m_klo);
        prefetch_tmap(&m_vhi);
        prefetch_tmap(&m_vlo);
    }
    if (warp == 1) tmem_alloc<TMEM_COLS>(tmem_holder);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp == 0) {
        // ---------------- TMA producer: Q rows one item ahead, K and V^T tiles ----------------
        if (lane == 0) {
            uint32_t g = 0, nq = 0;   // K/V blocks and Q tiles issued
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
            if ((int64_t)blockIdx.x < a.items) ok = load_q(blockIdx.x);
            for (int64_t it = blockIdx.x; ok && it < a.items && !*abort_flag; it += gridDim.x) {
                const Item w = item_of(a, it);
                const bool next = it + gridDim.x < a.items;
                for (int j = 0; j < w.nblocks && !*abort_flag; ++j, ++g) {
                    const int s = g % STAGES;
                    if (!mbar_wait(&kv_empty[s], ((g / STAGES) & 1) ^ 1)) {
                        ok = false;
                        break;
                    }
                    uint8_t *st = smem + s * STAGE_BYTES;
                    mbar_arrive_expect_tx(&kv_full[s], STAGE_BYTES);
                    const int krow = (int)(w.head * a.n_ctx + (int64_t)j * BN);
                    const int vrow = (int)(w.head * HD);
                    const int kx = j * BN;
                    for (int box = 0; box < 2; ++box) {
                        tma_load_2d(st + box * PAIR_BYTES, &m_khi, &kv_full[s], box * 32, krow);
                        tma_load_2d(st + box * PAIR_BYTES + BOX_BYTES, &m_klo, &kv_full[s], box * 32, krow);
                        tma_load_2d(st + V_BASE + box * PAIR_BYTES, &m_vhi, &kv_full[s], kx + box * 32, vrow);
                        tma_load_2d(st + V_BASE + box * PAIR_BYTES + BOX_BYTES, &m_vlo, &kv_full[s], kx + box * 32,
                                    vrow);
                    }
                    // the next item's Q, once this item's Q has left qbuf (early in this item)
                    if (next && j == (w.nblocks > 1 ? 1 : 0) && !(ok = load_q(it + gridDim.x))) break;
                }
            }
            if (!ok) {
                record_status(STATUS_TIMEOUT_PRODUCER);
                *abort_flag = 1;
            }
            for (uint32_t j = g > STAGES ? g - STAGES : 0; j < g; ++j)
                if (!mbar_wait(&kv_full[j % STAGES], (j / STAGES) & 1)) record_status(STATUS_TIMEOUT_DRAIN);
            if (nq > 0 && !mbar_wait(q_full, (nq - 1) & 1)) record_status(STATUS_TIMEOUT_DRAIN);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer: S of block j+1 is issued before P_j V so it overlaps softmax j ----------------
        if (lane == 0) {
            constexpr uint32_t IDESC_N128 = idesc_tf32(BM, 2 * BN), IDESC_N64 = idesc_tf32(BM, BN);
            uint32_t g = 0, k = 0;   // global block counter, items done
            bool ok = true;
            auto issue_s = [&](uint32_t gg) -> bool {
                const int s = gg % STAGES;
                if (!mbar_wait(&kv_full[s], (gg / STAGES) & 1)) return false;
                tc_fence_after();
                const uint32_t base = smem_u32(smem + s * STAGE_BYTES);
                const uint32_t d = tmem + COL_S0 + (gg & 1) * 2 * BN;
#pragma unroll
                for (int ks = 0; ks < HD / 8; ++ks) {
                    const uint32_t pair = base + (ks >> 2) * PAIR_BYTES + (ks & 3) * 32;
                    const uint64_t b_pair = smem_desc_kmajor(pair, 128, LAYOUT_SWIZZLE_128B);   // K_hi; K_lo rows
                    mma_tf32_ts(d, tmem + COL_QHI + 8 * ks, b_pair, IDESC_N128, ks > 0 ? 1u : 0u);
                    mma_tf32_ts(d, tmem + COL_QLO + 8 * ks, b_pair, IDESC_N64, 1u);              // K_hi rows only
                }
                mma_commit(&s_full[gg & 1]);
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
                    if (!mbar_wait(&p_full[g & 1], (g >> 1) & 1) || (g > 0 && !mbar_wait(o_empty, (g - 1) & 1))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const int s = g % STAGES;
                    const uint32_t base = smem_u32(smem + s * STAGE_BYTES) + V_BASE;
                    const uint32_t pcol = tmem + COL_S0 + (g & 1) * 2 * BN;
#pragma unroll
                    for (int ks = 0; ks < BN / 8; ++ks) {
                        const uint32_t pair = base + (ks >> 2) * PAIR_BYTES + (ks & 3) * 32;
                        const uint64_t b_pair = smem_desc_kmajor(pair, 128, LAYOUT_SWIZZLE_128B);   // V^T_hi; V^T_lo
                        mma_tf32_ts(tmem + COL_O, pcol + 8 * ks, b_pair, IDESC_N128, ks > 0 ? 1u : 0u);   // P_hi
                        mma_tf32_ts(tmem + COL_O, pcol + BN + 8 * ks, b_pair, IDESC_N64, 1u);           // P_lo . V_hi
                    }
                    mma_commit(o_full);
                    mma_commit(&kv_empty[s]);
                }
            }
            if (!ok) {
                record_status(STATUS_TIMEOUT_MMA);
                *abort_flag = 1;
            }
            mma_commit(drain);
            if (!mbar_wait(drain, 0)) record_status(STATUS_TIMEOUT_DRAIN);
        }
    } else {
        // ---------------- softmax / accumulate / store (warps 2-5) ----------------
        const int quarter = warp & 3;
        const int rloc = quarter * 32 + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
        uint32_t g = 0, nq = 0;
        bool ok = true;
        // qbuf (raw Q rows, 128-byte swizzle, two 32-column boxes) -> tf32 hi / lo -> TMEM
        auto q_to_tmem = [&]() -> bool {
            if (*abort_flag || !warp_wait(q_full, nq & 1)) return false;
#pragma unroll
            for (int c = 0; c < HD; c += 16) {
                uint32_t hi[16], lo[16];
#pragma unroll
                for (int v4 = 0; v4 < 4; ++v4) {
                    const int col = c + 4 * v4, box = col >> 5, chunk = (col & 31) >> 2;
                    const float4 x = *reinterpret_cast<const float4 *>(qbuf + box * (Q_BYTES / 2) + rloc * 128 +
                                                                       ((chunk ^ (rloc & 7)) << 4));
                    const float xv[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float h = tf32_trunc(xv[e]);
                        hi[4 * v4 + e] = __float_as_uint(h);
                        lo[4 * v4 + e] = __float_as_uint(isfinite(xv[e]) ? tf32_trunc(xv[e] - h) : 0.0f);
                    }
                }
                tmem_st_32x32b_x16(lane_base + COL_QHI + c, hi);
                tmem_st_32x32b_x16(lane_base + COL_QLO + c, lo);
            }
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
        float acc[HD];
        // acc = acc * alpha + O_blk of global block gg (its P.V accumulator in TMEM)
        auto fold = [&](uint32_t gg, float alpha) -> bool {
            if (*abort_flag || !warp_wait(o_full, gg & 1)) return false;
            tc_fence_after();
            uint32_t r[2 * HD];
#pragma unroll
            for (int c = 0; c < 2 * HD; c += 16)
                tmem_ld_32x32b_x16(lane_base + COL_O + c, *reinterpret_cast<uint32_t(*)[16]>(r + c));
            tmem_ld_wait();
#pragma unroll
            for (int c = 0; c < HD; ++c)
                acc[c] = fmaf(acc[c], alpha, __uint_as_float(r[c]) + __uint_as_float(r[HD + c]));
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(o_empty);
            return true;
        };
        const bool o_vec = ((reinterpret_cast<uintptr_t>(a.o) | (uintptr_t)(a.soh * 4) | (uintptr_t)(a.som * 4)) & 15) == 0;
        if ((int64_t)blockIdx.x < a.items) ok = q_to_tmem();
        for (int64_t it = blockIdx.x; ok && it < a.items; it += gridDim.x) {
            const Item w = item_of(a, it);
            const int64_t row = w.q0 + rloc;
            const bool next = it + gridDim.x < a.items;   // its Q follows this item's last P
            float m_i = -INFINITY, l_i = 0.0f, alpha_prev = 1.0f;
#pragma unroll
            for (int d = 0; d < HD; ++d) acc[d] = 0.0f;
            for (int j = 0; j < w.nblocks; ++j, ++g) {
                if (*abort_flag || !warp_wait(&s_full[g & 1], (g >> 1) & 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const int64_t k0 = (int64_t)j * BN;
                const uint32_t scol = COL_S0 + (g & 1) * 2 * BN, pcol = scol + BN;
                float sc[BN];
                {
                    uint32_t r[2 * BN];
#pragma unroll
                    for (int c = 0; c < 2 * BN; c += 16)
                        tmem_ld_32x32b_x16(lane_base + scol + c, *reinterpret_cast<uint32_t(*)[16]>(r + c));
                    tmem_ld_wait();   // one wait for all eight loads
#pragma unroll
                    for (int c = 0; c < BN; ++c) sc[c] = __uint_as_float(r[c]) + __uint_as_float(r[BN + c]);
                }
                // masks only on the blocks that reach past key_end or the causal diagonal
                const bool masked = k0 + BN > a.key_end || (a.causal && k0 + BN - 1 > w.q0);
                if (masked) {
#pragma unroll
                    for (int c = 0; c < BN; ++c) {
                        const int64_t col = k0 + c;
                        if (col >= a.key_end || (a.causal && col > row)) sc[c] = -INFINITY;
                    }
                }
                float m0 = sc[0], m1 = sc[1], m2 = sc[2], m3 = sc[3];
#pragma unroll
                for (int c = 4; c < BN; c += 4) {
                    m0 = fmaxf(m0, sc[c]);
                    m1 = fmaxf(m1, sc[c + 1]);
                    m2 = fmaxf(m2, sc[c + 2]);
                    m3 = fmaxf(m3, sc[c + 3]);
                }
                // scale > 0, so max(s) * scale = max(s * scale)
                const float m_new = fmaxf(m_i, fmaxf(fmaxf(m0, m1), fmaxf(m2, m3)) * a.qk_scale);
                const float m_use = m_new == -INFINITY ? 0.0f : m_new;
                const float alpha = fast_exp2(m_i - m_use);
                float ps0 = 0.0f, ps1 = 0.0f;
#pragma unroll
                for (int c = 0; c < BN; c += 16) {
                    uint32_t hi[16], lo[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        float p = fast_exp2(fmaf(sc[c + e], a.qk_scale, -m_use));
                        if (e & 1) ps1 += p;
                        else ps0 += p;
                        float h = tf32_trunc(p);
                        hi[e] = __float_as_uint(h);
                        lo[e] = __float_as_uint(p - h);   // exact; the tensor core reads its tf32 part
                    }
                    tmem_st_32x32b_x16(lane_base + scol + c, hi);
                    tmem_st_32x32b_x16(lane_base + pcol + c, lo);
                }
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
            if (row < a.row_end) {
                const float inv = 1.0f / l_i;
                float *orow = a.o + w.head * a.soh + row * a.som;
                if (o_vec) {   // 16-byte stores: a warp's store covers 32 rows x 16 bytes instead of 32 x 4
#pragma unroll
                    for (int d = 0; d < HD; d += 4)
                        *reinterpret_cast<float4 *>(orow + d) =
                            make_float4(acc[d] * inv, acc[d + 1] * inv, acc[d + 2] * inv, acc[d + 3] * inv);
                } else {
#pragma unroll
                    for (int d = 0; d < HD; ++d) orow[d] = acc[d] * inv;
                }
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

int64_t v_ld(int64_t n_ctx) { return (n_ctx + 3) / 4 * 4; }
size_t k_region(const AttnParams &p) { return ((size_t)p.heads * p.n_ctx * HD * 4 + 1023) / 1024 * 1024; }
size_t v_region(const AttnParams &p) { return ((size_t)p.heads * HD * v_ld(p.n_ctx) * 4 + 1023) / 1024 * 1024; }
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

size_t attention_tc_workspace_bytes(const AttnParams &p) { return 2 * k_region(p) + 2 * v_region(p) + q_region(p); }

int attention_tc(const AttnParams &p, void *workspace, cudaStream_t stream) {
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    float *k_hi = reinterpret_cast<float *>(ws);
    float *k_lo = reinterpret_cast<float *>(ws + k_region(p));
    float *v_hi = reinterpret_cast<float *>(ws + 2 * k_region(p));
    float *v_lo = reinterpret_cast<float *>(ws + 2 * k_region(p) + v_region(p));
    const int64_t ldv = v_ld(p.n_ctx);
    // K [n_ctx, D] per head (strides skn, skk) -> [heads * n_ctx, D]
    {
        dim3 g((unsigned)cdiv(HD, 32), (unsigned)cdiv(p.n_ctx, 32), (unsigned)p.heads);
        int along_rows = llabs(p.skn) < llabs(p.skk);
        attn_split_kernel<<<g, 256, 0, stream>>>(p.k, p.n_ctx, HD, p.skh, p.skn, p.skk, k_hi, k_lo, HD, along_rows);
    }
    // V [n_ctx, D] per head (strides svn, 1) -> V^T [heads * D, ldv]
    {
        dim3 g((unsigned)cdiv(p.n_ctx, 32), (unsigned)cdiv(HD, 32), (unsigned)p.heads);
        attn_split_kernel<<<g, 256, 0, stream>>>(p.v, HD, p.n_ctx, p.svh, 1, p.svn, v_hi, v_lo, ldv, 1);
    }
    int launches = 3;
    const float *q = p.q;
    int64_t sqm = p.sqm, sqh = p.sqh;
    if (!q_in_place(p)) {
        float *qc = reinterpret_cast<float *>(ws + 2 * k_region(p) + 2 * v_region(p));
        dim3 g((unsigned)std::min<int64_t>(cdiv(p.n_ctx * HD, (int64_t)256), 4096), (unsigned)p.heads);
        attn_q_copy_kernel<<<g, 256, 0, stream>>>(p.q, p.n_ctx, p.sqh, p.sqm, qc);
        q = qc;
        sqm = HD;
        sqh = p.n_ctx * HD;
        ++launches;
    }
    CUtensorMap mq, mkh, mkl, mvh, mvl;
    int rc;
    if ((rc = make_map_q(&mq, q, p.n_ctx, p.heads, sqm, sqh)) ||
        (rc = make_map(&mkh, k_hi, p.heads * p.n_ctx, HD, HD)) || (rc = make_map(&mkl, k_lo, p.heads * p.n_ctx, HD, HD)) ||
        (rc = make_map(&mvh, v_hi, p.heads * HD, p.n_ctx, ldv)) || (rc = make_map(&mvl, v_lo, p.heads * HD, p.n_ctx, ldv)))
        return rc;
    static bool attr[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr[dev]) {
        PITON_CUDA(cudaFuncSetAttribute(attn_3xtf32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
        attr[dev] = true;
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
    if (grid > 0) attn_3xtf32_kernel<<<(unsigned)grid, THREADS, SMEM_BYTES, stream>>>(mq, mkh, mkl, mvh, mvl, a);
    return check_launch("attention_3xtf32", launches);
}

int attention_tc_status_read_and_clear(int *status) {
    int zero = 0;
    PITON_CUDA(cudaMemcpyFromSymbol(status, g_attn_status, sizeof(int)));
    PITON_CUDA(cudaMemcpyToSymbol(g_attn_status, &zero, sizeof(int)));
    return PITON_B200_OK;
}

}  // namespace piton
