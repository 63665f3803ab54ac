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
constexpr uint32_t SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 1024;
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
    const float *q;
    float *o;
    int64_t sqh, sqm, soh, som;
    int64_t n_ctx, key_end, row_end, heads, q_blocks;
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

__global__ void __launch_bounds__(THREADS, 1)
    attn_3xtf32_kernel(const __grid_constant__ CUtensorMap m_khi, const __grid_constant__ CUtensorMap m_klo,
                       const __grid_constant__ CUtensorMap m_vhi, const __grid_constant__ CUtensorMap m_vlo,
                       TcAttnArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *kv_full = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE_BYTES);
    uint64_t *kv_empty = kv_full + STAGES;
    uint64_t *s_full = kv_empty + STAGES;     // [2]
    uint64_t *p_full = s_full + 2;            // [2]
    uint64_t *q_ready = p_full + 2;
    uint64_t *o_full = q_ready + 1;
    uint64_t *o_empty = o_full + 1;
    uint64_t *drain = o_empty + 1;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // all query blocks of a head run close together (its K / V stay in L2), heavy (late) blocks first
    const int64_t head = (int64_t)blockIdx.x / a.q_blocks;
    const int64_t qb = a.q_blocks - 1 - (int64_t)blockIdx.x % a.q_blocks;
    const int64_t q0 = qb * BM;
    int64_t kend = a.key_end;
    if (a.causal && q0 + BM < kend) kend = q0 + BM;
    const int nblocks = kend > 0 ? (int)((kend + BN - 1) / BN) : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&s_full[b], 1);
            mbar_init(&p_full[b], 4);
        }
        mbar_init(q_ready, 4);
        mbar_init(o_full, 1);
        mbar_init(o_empty, 4);
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbarrier_init();
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
        // ---------------- TMA producer: K and V^T tiles ----------------
        if (lane == 0) {
            int issued = 0;
            for (int j = 0; j < nblocks && !*abort_flag; ++j, ++issued) {
                const int s = j % STAGES;
                if (!mbar_wait(&kv_empty[s], ((j / STAGES) & 1) ^ 1)) {
                    record_status(STATUS_TIMEOUT_PRODUCER);
                    *abort_flag = 1;
                    break;
                }
                uint8_t *st = smem + s * STAGE_BYTES;
                mbar_arrive_expect_tx(&kv_full[s], STAGE_BYTES);
                const int krow = (int)(head * a.n_ctx + (int64_t)j * BN);
                const int vrow = (int)(head * HD);
                const int kx = j * BN;
                for (int box = 0; box < 2; ++box) {
                    tma_load_2d(st + box * PAIR_BYTES, &m_khi, &kv_full[s], box * 32, krow);
                    tma_load_2d(st + box * PAIR_BYTES + BOX_BYTES, &m_klo, &kv_full[s], box * 32, krow);
                    tma_load_2d(st + V_BASE + box * PAIR_BYTES, &m_vhi, &kv_full[s], kx + box * 32, vrow);
                    tma_load_2d(st + V_BASE + box * PAIR_BYTES + BOX_BYTES, &m_vlo, &kv_full[s], kx + box * 32, vrow);
                }
            }
            for (int j = issued > STAGES ? issued - STAGES : 0; j < issued; ++j)
                if (!mbar_wait(&kv_full[j % STAGES], (j / STAGES) & 1)) record_status(STATUS_TIMEOUT_DRAIN);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer: S_{j+1} is issued before P_j V so it overlaps softmax j ----------------
        if (lane == 0) {
            constexpr uint32_t IDESC_N128 = idesc_tf32(BM, 2 * BN), IDESC_N64 = idesc_tf32(BM, BN);
            bool ok = mbar_wait(q_ready, 0);
            tc_fence_after();
            auto issue_s = [&](int j) -> bool {
                const int s = j % STAGES;
                if (!mbar_wait(&kv_full[s], (j / STAGES) & 1)) return false;
                tc_fence_after();
                const uint32_t base = smem_u32(smem + s * STAGE_BYTES);
                const uint32_t d = tmem + COL_S0 + (j & 1) * 2 * BN;
#pragma unroll
                for (int ks = 0; ks < HD / 8; ++ks) {
                    const uint32_t pair = base + (ks >> 2) * PAIR_BYTES + (ks & 3) * 32;
                    const uint64_t b_pair = smem_desc_kmajor(pair, 128, LAYOUT_SWIZZLE_128B);   // K_hi; K_lo rows
                    mma_tf32_ts(d, tmem + COL_QHI + 8 * ks, b_pair, IDESC_N128, ks > 0 ? 1u : 0u);
                    mma_tf32_ts(d, tmem + COL_QLO + 8 * ks, b_pair, IDESC_N64, 1u);              // K_hi rows only
                }
                mma_commit(&s_full[j & 1]);
                return true;
            };
            if (ok && nblocks > 0) ok = issue_s(0);
            for (int j = 0; ok && j < nblocks && !*abort_flag; ++j) {
                if (j + 1 < nblocks && !issue_s(j + 1)) {
                    ok = false;
                    break;
                }
                if (!mbar_wait(&p_full[j & 1], (j >> 1) & 1) || (j > 0 && !mbar_wait(o_empty, (j - 1) & 1))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const int s = j % STAGES;
                const uint32_t base = smem_u32(smem + s * STAGE_BYTES) + V_BASE;
                const uint32_t p = tmem + COL_S0 + (j & 1) * 2 * BN;
#pragma unroll
                for (int ks = 0; ks < BN / 8; ++ks) {
                    const uint32_t pair = base + (ks >> 2) * PAIR_BYTES + (ks & 3) * 32;
                    const uint64_t b_pair = smem_desc_kmajor(pair, 128, LAYOUT_SWIZZLE_128B);   // V^T_hi; V^T_lo rows
                    mma_tf32_ts(tmem + COL_O, p + 8 * ks, b_pair, IDESC_N128, ks > 0 ? 1u : 0u);        // P_hi
                    mma_tf32_ts(tmem + COL_O, p + BN + 8 * ks, b_pair, IDESC_N64, 1u);                // P_lo . V_hi
                }
                mma_commit(o_full);
                mma_commit(&kv_empty[s]);
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
        const int64_t row = q0 + quarter * 32 + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
        bool ok = true;
        {
            // Q row -> tf32 hi / lo -> TMEM
            const float *qr = a.q + head * a.sqh + row * a.sqm;
            const bool live = row < a.n_ctx;
#pragma unroll
            for (int c = 0; c < HD; c += 16) {
                uint32_t hi[16], lo[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    float v = live ? qr[c + j] : 0.0f;
                    float h = tf32_trunc(v);
                    hi[j] = __float_as_uint(h);
                    lo[j] = __float_as_uint(isfinite(v) ? tf32_trunc(v - h) : 0.0f);
                }
                tmem_st_32x32b_x16(lane_base + COL_QHI + c, hi);
                tmem_st_32x32b_x16(lane_base + COL_QLO + c, lo);
            }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(q_ready);
        }
        float m_i = -INFINITY, l_i = 0.0f, alpha_prev = 1.0f;
        float acc[HD];
#pragma unroll
        for (int d = 0; d < HD; ++d) acc[d] = 0.0f;
        // acc = acc * alpha + O_blk of block jj (its P.V accumulator in TMEM)
        auto fold = [&](int jj, float alpha) -> bool {
            if (*abort_flag || !warp_wait(o_full, jj & 1)) return false;
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
        for (int j = 0; j < nblocks; ++j) {
            if (*abort_flag || !warp_wait(&s_full[j & 1], (j >> 1) & 1)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int64_t k0 = (int64_t)j * BN;
            const uint32_t scol = COL_S0 + (j & 1) * 2 * BN, pcol = scol + BN;
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
            const bool masked = k0 + BN > a.key_end || (a.causal && k0 + BN - 1 > q0);
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
            if (lane == 0) mbar_arrive(&p_full[j & 1]);
            // fold the previous block's P.V while this block's runs on the tensor core
            if (j > 0 && !fold(j - 1, alpha_prev)) {
                ok = false;
                break;
            }
            alpha_prev = alpha;
        }
        if (ok && nblocks > 0 && !fold(nblocks - 1, alpha_prev)) ok = false;
        if (!ok) {
            if (lane == 0) record_status(STATUS_TIMEOUT_EPILOGUE);
            *abort_flag = 1;
        } else if (row < a.row_end) {
            const float inv = 1.0f / l_i;
            float *orow = a.o + head * a.soh + row * a.som;
#pragma unroll
            for (int d = 0; d < HD; ++d) orow[d] = acc[d] * inv;
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

int64_t v_ld(int64_t n_ctx) { return (n_ctx + 3) / 4 * 4; }
size_t k_region(const AttnParams &p) { return ((size_t)p.heads * p.n_ctx * HD * 4 + 1023) / 1024 * 1024; }
size_t v_region(const AttnParams &p) { return ((size_t)p.heads * HD * v_ld(p.n_ctx) * 4 + 1023) / 1024 * 1024; }

}  // namespace

bool attention_tc_supported(const AttnParams &p) {
    if (p.head_dim != HD || p.n_ctx < 64 || p.heads < 1) return false;
    if (p.heads * p.n_ctx >= (1ll << 31) || p.heads * HD >= (1ll << 31)) return false;
    if ((p.n_ctx + 31) / 32 > 65535 || p.heads > 65535) return false;
    int64_t q_blocks = (p.row_end + BM - 1) / BM;
    if (q_blocks * p.heads >= (1ll << 31)) return false;
    return encode_fn() != nullptr;
}

size_t attention_tc_workspace_bytes(const AttnParams &p) { return 2 * k_region(p) + 2 * v_region(p); }

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
    CUtensorMap mkh, mkl, mvh, mvl;
    int rc;
    if ((rc = make_map(&mkh, k_hi, p.heads * p.n_ctx, HD, HD)) || (rc = make_map(&mkl, k_lo, p.heads * p.n_ctx, HD, HD)) ||
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
    a.q = p.q;
    a.o = p.o;
    a.sqh = p.sqh; a.sqm = p.sqm; a.soh = p.soh; a.som = p.som;
    a.n_ctx = p.n_ctx; a.key_end = p.key_end; a.row_end = p.row_end; a.heads = p.heads;
    a.q_blocks = (p.row_end + BM - 1) / BM;
    a.qk_scale = p.qk_scale;
    a.causal = p.causal;
    attn_3xtf32_kernel<<<(unsigned)(a.q_blocks * p.heads), THREADS, SMEM_BYTES, stream>>>(mkh, mkl, mvh, mvl, a);
    return check_launch("attention_3xtf32", 3);
}

int attention_tc_status_read_and_clear(int *status) {
    int zero = 0;
    PITON_CUDA(cudaMemcpyFromSymbol(status, g_attn_status, sizeof(int)));
    PITON_CUDA(cudaMemcpyToSymbol(g_attn_status, &zero, sizeof(int)));
    return PITON_B200_OK;
}

}  // namespace piton
