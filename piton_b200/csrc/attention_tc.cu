// Flash-attention forward on the 5th-generation tensor cores with an fp16 split of
// every operand (examples/attention.py:33-113; the semantics are those of attention.cu's
// header: key_end, causal mask, row_end, base-2 online softmax).
//
// Each operand is scaled by a power of two and split into fp16 halves x_hi = fp16(x 2^e),
// x_lo = fp16(x 2^e - x_hi) (22 significant bits): a Q row by its own scale (largest
// magnitude into [2^14, 2^15)), K and V by one scale per 64-key block of a head, P (in
// [0, 1]) by 2^14.  A product x y is then x_hi y_hi + x_hi y_lo + x_lo y_hi (the dropped
// lo x lo term and the rounding of the low halves cost ~2^-21 of it), and the scales come
// back out in the softmax warps' score multiplier and fold, where they cost nothing.
//
// Per call:
//  1. split (HBM-bound): K -> K_hi, K_lo as [heads * n_ctx, 64] fp16 and V -> V^T_hi,
//     V^T_lo as [heads * 64, ldv] fp16 (ldv = n_ctx rounded up to 64), each 64-key block
//     with its exponent in an int8 [heads, blocks] array; a CTA per (head, block).
//  2. persistent CTAs walk (head, 128-query block) items, 480 threads:
//     * warps 2-9, two per TMEM lane quarter (one thread per query row = TMEM lane in
//       each), each warp of a pair on half of the keys: they read the raw row of Q, take
//       its scale and store their half of Q_hi, Q_lo (fp16 pairs) into TMEM; per 64-key
//       block each reads its 32 keys' scores S from TMEM, applies the scale and the masks,
//       exchanges its row maximum with the other warp through shared memory (an mbarrier
//       per pair and block parity), updates the running max and its partial sum in
//       registers, writes P_hi and P_lo (fp16 pairs) over S in TMEM and hands the block's
//       rescale factor (alpha per row) to the fold warp through shared memory;
//     * warps 11-14, one per lane quarter (the FlashAttention-4 division of labour): per
//       block they take alpha, read the block's P.V accumulator from TMEM and fold it,
//       unscaled, into an fp32 register accumulator (round to nearest); at the end of an
//       item they take the row sums and store O / l;
//     * warp 0 streams Q and the K tiles, warp 10 the V^T tiles, with TMA (128-byte
//       swizzle; separate rings, since a K tile is free after S and a V tile only after P.V);
//     * warp 15, only in the all-gather launch (512 threads), copies each item's stored
//       rows from this rank's output to every other rank's (NVLink peer stores), one item
//       behind the fold warps;
//     * warp 1 issues, from one thread, per 16-wide k-step one kind::f16 MMA of Q_hi
//       against the stacked [K_hi; K_lo] tile (N = 128: Q_hi K_hi in columns 0-63, Q_hi K_lo
//       in 64-127) and one of Q_lo against K_hi (N = 64, added to columns 0-63); likewise
//       P_hi [V_hi; V_lo] and P_lo V_hi for P.V: 8 MMAs per 64-key block for S and 8 for
//       P.V.  The softmax and fold warps add the two halves in fp32 registers (round to
//       nearest), so the hi/lo sums are not truncated by the tensor core.
//     A block's P.V lands in its own TMEM accumulator that the fold warps add into
//     registers, so the tensor core's truncating accumulation never spans more than one
//     64-key block.
// The scores of block j+1 are computed while the softmax warps work on block j (two S/P
// buffers), and the fold warps take a block's P.V while the softmax warps turn the next
// block's S into P, so the tensor core, the softmax and the fold overlap.  TMEM columns:
// Q_hi [0,32) Q_lo [32,64), S/P x2 [128,384) (128 each; P_hi in the first 32, P_lo in
// 64-95), O_blk [384,512) (512 allocated).  All waits are bounded (2 s): on expiry the
// kernel records a status, drains its copies and MMAs, frees TMEM and returns.
#include <algorithm>

#include <cuda_fp16.h>

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

constexpr int BM = 128, BN = 64, HD = 64, KSTAGES = 3, VSTAGES = 3, THREADS = 480;
constexpr int SOFTMAX_WARPS = 8;                          // warps 2-9: two per TMEM lane quarter
constexpr int FOLD_WARP0 = 11, FOLD_WARPS = 4;            // warps 11-14: one per lane quarter, all of O's columns
constexpr int GATHER_WARP = 15;                           // copies finished rows to the peers (world > 1)
constexpr int GATHER_THREADS = THREADS + 32;              // launch with the gather warp
constexpr uint32_t BOX_BYTES = 64 * 64 * 2;               // 64 rows x 128 bytes (64 fp16)
// K stage: [K_hi][K_lo], so one 128-row B operand covers hi rows 0-63 and lo rows 64-127;
// V stage: [V^T_hi][V^T_lo] (64 d x 64 keys each), the same way
constexpr uint32_t STAGE_BYTES = 2 * BOX_BYTES;
constexpr uint32_t Q_BYTES = BM * HD * 4;                // raw Q rows of one item: two 128 x 32 boxes
// row maxima exchanged between the two softmax warps of a lane quarter ([block parity][half][row]),
// their row sums at the end of an item ([half][row]), and what they hand to the fold warps: the
// rescale factor of every block ([block parity][row]) and the row sum of every item ([item parity][row])
constexpr uint32_t XCHG_BYTES = (2 * 2 * BM + 2 * BM + 2 * BM + 2 * BM) * 4;
constexpr uint32_t SMEM_BYTES = (KSTAGES + VSTAGES) * STAGE_BYTES + Q_BYTES + XCHG_BYTES + 1024 + 1024;
constexpr int TMEM_COLS = 512;
// TMEM: Q_hi, Q_lo (fp16 pairs), two 128-column S/P buffers (S: Q_hi.K_hi (+ Q_lo.K_hi) in
// 0-63 and Q_hi.K_lo in 64-127; P: P_hi (fp16 pairs) in 0-31, P_lo in 64-95) and a 128-column
// O_blk (P_hi.V_hi (+ P_lo.V_hi) in 0-63, P_hi.V_lo in 64-127)
constexpr uint32_t COL_QHI = 0, COL_QLO = 32, COL_S0 = 128, COL_O = 384;
constexpr float P_SCALE = 16384.0f;                       // P in [0, 1] -> [0, 2^14]
static_assert(KSTAGES == VSTAGES, "the producers share one ring depth");

// two floats -> fp16 pair (round to nearest), `lo_k` in the low half
__device__ __forceinline__ uint32_t pack_f16(float lo_k, float hi_k) {
    __half2 v = __floats2half2_rn(lo_k, hi_k);
    return *reinterpret_cast<uint32_t *>(&v);
}
// x (already scaled) -> fp16 hi and the fp16 of the rest; non-finite x keeps hi and a zero lo
__device__ __forceinline__ void split_f16(float x, float &hi, float &lo) {
    hi = __half2float(__float2half_rn(x));
    lo = isfinite(x) ? x - hi : 0.0f;
}
// 2^e for e in [-126, 127] from its exponent bits
__device__ __forceinline__ float pow2i(int e) { return __int_as_float((127 + e) << 23); }
// exponent e of a block's scale 2^e: its largest finite magnitude m goes into [2^14, 2^15);
// 0 for a block without a finite non-zero value; clamped to [-112, 112]
__device__ __forceinline__ int block_exponent(float m) {
    if (!(m > 0.0f)) return 0;
    int E;
    frexpf(m, &E);
    return max(-112, min(112, 15 - E));
}
__device__ __forceinline__ float finite_abs(float v) { return isfinite(v) ? fabsf(v) : 0.0f; }

__device__ __forceinline__ void record_status(int code) { atomicCAS(&g_attn_status, 0, code); }

// One 64-key block of one head, [keys, 64] from src + h*s_h + key*s_r + d*s_c (keys past
// n_ctx read as zeros), scaled by the block's power of two and split into fp16 halves:
//  TRANSPOSE == false (K): rows h * n_ctx + key of hi / lo, 64 fp16 each;
//  TRANSPOSE == true  (V): rows h * 64 + d of hi / lo (row length ld = n_ctx rounded up to 64),
//  keys key0 .. key0 + 63.
// The block's exponent goes to ex[h * blocks + block].  A CTA of 256 threads per (block, head),
// the block staged in shared memory (loads along whichever of keys and d has the smaller stride).
template <bool TRANSPOSE>
__global__ void __launch_bounds__(256) attn_split16_kernel(const float *__restrict__ src, int64_t n_ctx, int64_t s_h,
                                                           int64_t s_r, int64_t s_c, __half *__restrict__ hi,
                                                           __half *__restrict__ lo, int64_t ld,
                                                           int8_t *__restrict__ ex, int64_t blocks) {
    __shared__ float tile[64][65];   // [key][d]
    __shared__ float wmax[8];
    const int64_t blk = blockIdx.x, h = blockIdx.y, key0 = blk * 64;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const float *base = src + h * s_h;
    const bool keys_fast = llabs(s_r) < llabs(s_c);
    float m = 0.0f;
    for (int i = t; i < 64 * 64; i += 256) {
        const int key = keys_fast ? (i & 63) : (i >> 6), d = keys_fast ? (i >> 6) : (i & 63);
        const float v = key0 + key < n_ctx ? base[(key0 + key) * s_r + (int64_t)d * s_c] : 0.0f;
        tile[key][d] = v;
        m = fmaxf(m, finite_abs(v));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) wmax[warp] = m;
    __syncthreads();
    m = wmax[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) m = fmaxf(m, wmax[w]);
    const int e = block_exponent(m);
    const float sc = pow2i(e);
    // 512 runs of 8 consecutive outputs (16-byte stores), two per thread
    for (int c = t; c < 512; c += 256) {
        const int a8 = c >> 3, b8 = (c & 7) * 8;   // K: key a8, d b8..; V: d a8, keys b8..
        if (!TRANSPOSE && key0 + a8 >= n_ctx) continue;
        __align__(16) __half hh[8], ll[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float v = (TRANSPOSE ? tile[b8 + q][a8] : tile[a8][b8 + q]) * sc;
            float vh, vl;
            split_f16(v, vh, vl);
            hh[q] = __float2half_rn(vh);
            ll[q] = __float2half_rn(vl);
        }
        const int64_t off = TRANSPOSE ? (h * HD + a8) * ld + key0 + b8 : (h * n_ctx + key0 + a8) * HD + b8;
        *reinterpret_cast<uint4 *>(hi + off) = *reinterpret_cast<const uint4 *>(hh);
        *reinterpret_cast<uint4 *>(lo + off) = *reinterpret_cast<const uint4 *>(ll);
    }
    if (t == 0) ex[h * blocks + blk] = (int8_t)e;
}

// The same split for rows with unit stride along d and 16-byte aligned rows (the common
// contiguous layout): thread t holds key t / 4, dimensions 16 (t % 4) .. + 15, loaded as four
// float4 before any is used, so a CTA has its whole 16 KB block in flight at once.  K is
// written straight from registers (32-byte runs per half); V goes through shared memory
// for the transpose.
template <bool TRANSPOSE>
__global__ void __launch_bounds__(256) attn_split16_vec_kernel(const float *__restrict__ src, int64_t n_ctx,
                                                               int64_t s_h, int64_t s_r, __half *__restrict__ hi,
                                                               __half *__restrict__ lo, int64_t ld,
                                                               int8_t *__restrict__ ex, int64_t blocks) {
    __shared__ float tile[TRANSPOSE ? 64 : 1][65];   // [key][d]
    __shared__ float wmax[8];
    const int64_t blk = blockIdx.x, h = blockIdx.y, key0 = blk * 64;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int key = t >> 2, d0 = (t & 3) * 16;
    const bool live = key0 + key < n_ctx;
    float v[16];
    if (live) {
        const float4 *p = reinterpret_cast<const float4 *>(src + h * s_h + (key0 + key) * s_r + d0);
        float4 f[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) f[j] = __ldcs(p + j);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            v[4 * j] = f[j].x; v[4 * j + 1] = f[j].y; v[4 * j + 2] = f[j].z; v[4 * j + 3] = f[j].w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = 0.0f;
    }
    float m = 0.0f;
#pragma unroll
    for (int j = 0; j < 16; ++j) m = fmaxf(m, finite_abs(v[j]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) wmax[warp] = m;
    if (TRANSPOSE) {
#pragma unroll
        for (int j = 0; j < 16; ++j) tile[key][d0 + j] = v[j];
    }
    __syncthreads();
    m = wmax[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) m = fmaxf(m, wmax[w]);
    const int e = block_exponent(m);
    const float sc = pow2i(e);
    if (!TRANSPOSE) {
        if (live) {
            __align__(16) __half hh[16], ll[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                float vh, vl;
                split_f16(v[j] * sc, vh, vl);
                hh[j] = __float2half_rn(vh);
                ll[j] = __float2half_rn(vl);
            }
            const int64_t off = (h * n_ctx + key0 + key) * HD + d0;
            uint4 *ph = reinterpret_cast<uint4 *>(hi + off), *pl = reinterpret_cast<uint4 *>(lo + off);
            ph[0] = reinterpret_cast<const uint4 *>(hh)[0];
            ph[1] = reinterpret_cast<const uint4 *>(hh)[1];
            pl[0] = reinterpret_cast<const uint4 *>(ll)[0];
            pl[1] = reinterpret_cast<const uint4 *>(ll)[1];
        }
    } else {
        // 512 runs of 8 consecutive keys of one dimension (16-byte stores), two per thread
        for (int c = t; c < 512; c += 256) {
            const int a8 = c >> 3, b8 = (c & 7) * 8;   // d a8, keys b8 ..
            __align__(16) __half hh[8], ll[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                float vh, vl;
                split_f16(tile[b8 + q][a8] * sc, vh, vl);
                hh[q] = __float2half_rn(vh);
                ll[q] = __float2half_rn(vl);
            }
            const int64_t off = (h * HD + a8) * ld + key0 + b8;
            *reinterpret_cast<uint4 *>(hi + off) = *reinterpret_cast<const uint4 *>(hh);
            *reinterpret_cast<uint4 *>(lo + off) = *reinterpret_cast<const uint4 *>(ll);
        }
    }
    if (t == 0) ex[h * blocks + blk] = (int8_t)e;
}

struct TcAttnArgs {
    float *o;
    int64_t soh, som;
    int64_t n_ctx, key_end, row_end, heads, q_blocks, items;
    float qk_scale;
    int causal;
    const int8_t *ek, *ev;   // exponents of the K and V blocks [heads, kv_blocks]
    int64_t kv_blocks;
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
    attn_f16x3_kernel(const __grid_constant__ CUtensorMap m_q, const __grid_constant__ CUtensorMap m_khi,
                      const __grid_constant__ CUtensorMap m_klo, const __grid_constant__ CUtensorMap m_vhi,
                      const __grid_constant__ CUtensorMap m_vlo, const typename AttnArgsOf<NTHREADS>::type a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *kst = smem;                                          // K stages
    uint8_t *vst = smem + KSTAGES * STAGE_BYTES;                  // V^T stages
    uint8_t *qbuf = vst + VSTAGES * STAGE_BYTES;                  // raw Q rows of the next item
    float *xmax = reinterpret_cast<float *>(qbuf + Q_BYTES);       // [2][2][BM]
    float *xsum = xmax + 2 * 2 * BM;                               // [2][BM]
    float *xalpha = xsum + 2 * BM;                                 // [2][BM]
    float *xl = xalpha + 2 * BM;                                   // [2][BM]
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
    uint64_t *a_full = sum_bar + 4;           // [4 quarters][2 block parities]: alpha of a block written
    uint64_t *a_empty = a_full + 8;           // ... and read by the quarter's fold warp
    uint64_t *l_full = a_empty + 8;           // [4 quarters][2 item parities]: an item's row sums written
    uint64_t *l_empty = l_full + 8;           // ... and read
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(l_empty + 8);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);
    volatile int *rows_stored = abort_flag + 1;   // fold-warp item stores done (4 per item)

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
        mbar_init(o_empty, FOLD_WARPS);
        mbar_init(drain, 1);
        for (int b = 0; b < 8; ++b) mbar_init(&max_bar[b], 64);
        for (int b = 0; b < 4; ++b) mbar_init(&sum_bar[b], 64);
        for (int b = 0; b < 8; ++b) {
            mbar_init(&a_full[b], 1);
            mbar_init(&a_empty[b], 1);
            mbar_init(&l_full[b], 1);
            mbar_init(&l_empty[b], 1);
        }
        *abort_flag = 0;
        if constexpr (NTHREADS > THREADS) *rows_stored = 0;
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

    if (warp == 0 || warp == 10) {
        // ---------------- TMA producers: warp 0 Q rows (one item ahead) and K tiles, warp 10 V^T tiles ----------------
        if (lane == 0) {
            const bool is_k = warp == 0;
            uint64_t *full = is_k ? k_full : v_full, *empty = is_k ? k_empty : v_empty;
            uint8_t *stages = is_k ? kst : vst;
            const CUtensorMap *m_hi = is_k ? &m_khi : &m_vhi, *m_lo = is_k ? &m_klo : &m_vlo;
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
                    tma_load_2d(st, m_hi, &full[s], x0, row);
                    tma_load_2d(st + BOX_BYTES, m_lo, &full[s], x0, row);
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
            constexpr uint32_t IDESC_N128 = idesc_f16(BM, 2 * BN), IDESC_N64 = idesc_f16(BM, BN);
            uint32_t g = 0, k = 0;   // global block counter, items done
            bool ok = true;
            auto issue_s = [&](uint32_t gg) -> bool {
                const int s = gg % KSTAGES;
                if (!mbar_wait(&k_full[s], (gg / KSTAGES) & 1)) return false;
                tc_fence_after();
                const uint32_t base = smem_u32(kst + s * STAGE_BYTES);
                const uint32_t d = tmem + COL_S0 + (gg & 1) * 2 * BN;
#pragma unroll
                for (int kb = 0; kb < HD / 16; ++kb)   // Q_hi . [K_hi; K_lo], 16 d per MMA
                    mma_f16_ts(d, tmem + COL_QHI + 8 * kb, smem_desc_kmajor(base + kb * 32, 128, LAYOUT_SWIZZLE_128B),
                               IDESC_N128, kb > 0 ? 1u : 0u);
#pragma unroll
                for (int kb = 0; kb < HD / 16; ++kb)   // Q_lo . K_hi
                    mma_f16_ts(d, tmem + COL_QLO + 8 * kb, smem_desc_kmajor(base + kb * 32, 128, LAYOUT_SWIZZLE_128B),
                               IDESC_N64, 1u);
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
                    for (int kb = 0; kb < BN / 16; ++kb)   // P_hi . [V^T_hi; V^T_lo], 16 keys per MMA
                        mma_f16_ts(tmem + COL_O, pcol + 8 * kb,
                                   smem_desc_kmajor(base + kb * 32, 128, LAYOUT_SWIZZLE_128B), IDESC_N128,
                                   kb > 0 ? 1u : 0u);
#pragma unroll
                    for (int kb = 0; kb < BN / 16; ++kb)   // P_lo . V^T_hi
                        mma_f16_ts(tmem + COL_O, pcol + BN + 8 * kb,
                                   smem_desc_kmajor(base + kb * 32, 128, LAYOUT_SWIZZLE_128B), IDESC_N64, 1u);
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
                need += FOLD_WARPS;
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
    } else if (warp >= FOLD_WARP0 && warp < FOLD_WARP0 + FOLD_WARPS) {
        // ---------------- fold / store (warps 11-14, one per TMEM lane quarter) ----------------
        // acc = acc * alpha + O_blk * vs for every block, alpha handed over by the quarter's softmax
        // warps through shared memory; at the end of an item O = acc / l.
        const int quarter = warp & 3;
        const int rloc = quarter * 32 + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
        uint32_t g = 0, k = 0;
        bool ok = true;
        float acc[HD];
        const bool o_vec = ((reinterpret_cast<uintptr_t>(a.o) | (uintptr_t)(a.soh * 4) | (uintptr_t)(a.som * 4)) & 15) == 0;
        for (int64_t it = blockIdx.x; ok && it < a.items; it += gridDim.x, ++k) {
            const Item w = item_of(a, it);
            const int64_t row = w.q0 + rloc;
            const int8_t *evh = a.ev + w.head * a.kv_blocks;
            int ev_n = __ldg(evh);
#pragma unroll
            for (int d = 0; d < HD; ++d) acc[d] = 0.0f;
            for (int j = 0; j < w.nblocks; ++j, ++g) {
                const int ev = ev_n;
                if (j + 1 < w.nblocks) ev_n = __ldg(evh + j + 1);
                const float vs = pow2i(-(ev + 14));   // P (2^14) and V block scales out
                if (*abort_flag || !warp_wait(&a_full[quarter * 2 + (g & 1)], (g >> 1) & 1)) {
                    ok = false;
                    break;
                }
                const float alpha = xalpha[(g & 1) * BM + rloc];
                __syncwarp();
                if (lane == 0) mbar_arrive(&a_empty[quarter * 2 + (g & 1)]);
                if (*abort_flag || !warp_wait(o_full, g & 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                // once the rows' maxima have settled (alpha exactly 1 in all 32 rows) the rescale
                // drops out and the block's scale goes into one fused multiply-add
                const bool settled = __all_sync(0xffffffffu, alpha == 1.0f);
#pragma unroll
                for (int c = 0; c < HD; c += 16) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x16(lane_base + COL_O + c, *reinterpret_cast<uint32_t(*)[16]>(r));
                    tmem_ld_32x32b_x16(lane_base + COL_O + HD + c, *reinterpret_cast<uint32_t(*)[16]>(r + 16));
                    tmem_ld_wait();
                    if (settled) {
#pragma unroll
                        for (int e = 0; e < 16; ++e)
                            acc[c + e] = fmaf(__uint_as_float(r[e]) + __uint_as_float(r[16 + e]), vs, acc[c + e]);
                    } else {
#pragma unroll
                        for (int e = 0; e < 16; ++e)
                            acc[c + e] =
                                fmaf(acc[c + e], alpha, (__uint_as_float(r[e]) + __uint_as_float(r[16 + e])) * vs);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(o_empty);
            }
            if (!ok) break;
            // the item's row sums from the softmax warps
            if (*abort_flag || !warp_wait(&l_full[quarter * 2 + (k & 1)], (k >> 1) & 1)) {
                ok = false;
                break;
            }
            const float l_i = xl[(k & 1) * BM + rloc];
            __syncwarp();
            if (lane == 0) mbar_arrive(&l_empty[quarter * 2 + (k & 1)]);
            if (row < a.row_end) {
                const float inv = 1.0f / l_i;
                float *orow = a.o + w.head * a.soh + row * a.som;
                if (o_vec) {   // 16-byte stores
#pragma unroll
                    for (int d = 0; d < HD; d += 4)
                        *reinterpret_cast<float4 *>(orow + d) =
                            make_float4(acc[d] * inv, acc[d + 1] * inv, acc[d + 2] * inv, acc[d + 3] * inv);
                } else {
#pragma unroll
                    for (int d = 0; d < HD; ++d) orow[d] = acc[d] * inv;
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
    } else {
        // ---------------- softmax (warps 2-9): S -> P, row maxima and sums ----------------
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2;    // this warp's 32 keys of a block and 32 columns of Q
        const int rloc = quarter * 32 + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
        uint32_t g = 0, nq = 0, k = 0;
        bool ok = true;
        // qbuf (raw Q rows, 128-byte swizzle, two 32-column boxes) -> the row's scale 2^eq (from
        // the whole row, so both warps of the pair agree) -> fp16 hi / lo pairs of this warp's
        // columns [32 * half, 32 * half + 32) (box `half`) -> TMEM
        int eq_next = 0;   // the scale exponent of the Q rows last moved into TMEM
        auto q_to_tmem = [&]() -> bool {
            if (*abort_flag || !warp_wait(q_full, nq & 1)) return false;
            float xv[32];
            float m = 0.0f;
#pragma unroll
            for (int bx = 0; bx < 2; ++bx)
#pragma unroll
                for (int v4 = 0; v4 < 8; ++v4) {
                    const float4 x = *reinterpret_cast<const float4 *>(qbuf + bx * (Q_BYTES / 2) + rloc * 128 +
                                                                       ((v4 ^ (rloc & 7)) << 4));
                    m = fmaxf(fmaxf(m, fmaxf(finite_abs(x.x), finite_abs(x.y))),
                              fmaxf(finite_abs(x.z), finite_abs(x.w)));
                    if (bx == half) {
                        xv[4 * v4] = x.x;
                        xv[4 * v4 + 1] = x.y;
                        xv[4 * v4 + 2] = x.z;
                        xv[4 * v4 + 3] = x.w;
                    }
                }
            eq_next = block_exponent(m);
            const float sc = pow2i(eq_next);
            uint32_t hi[16], lo[16];
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                float h0, l0, h1, l1;
                split_f16(xv[2 * c] * sc, h0, l0);
                split_f16(xv[2 * c + 1] * sc, h1, l1);
                hi[c] = pack_f16(h0, h1);
                lo[c] = pack_f16(l0, l1);
            }
            tmem_st_32x32b_x16(lane_base + COL_QHI + 16 * half, hi);
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
        if ((int64_t)blockIdx.x < a.items) ok = q_to_tmem();
        for (int64_t it = blockIdx.x; ok && it < a.items; it += gridDim.x, ++k) {
            const Item w = item_of(a, it);
            const int64_t row = w.q0 + rloc;
            const bool next = it + gridDim.x < a.items;   // its Q follows this item's last P
            float m_i = -INFINITY, l_i = 0.0f;
            // the score multiplier without the block's K scale, and the blocks' exponents, each
            // loaded one block ahead of its use
            const float fq = a.qk_scale * pow2i(-eq_next);
            const int8_t *ekh = a.ek + w.head * a.kv_blocks;
            int ek_n = __ldg(ekh);
            for (int j = 0; j < w.nblocks; ++j, ++g) {
                if (*abort_flag || !warp_wait(&s_full[g & 1], (g >> 1) & 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const int ek = ek_n;
                if (j + 1 < w.nblocks) ek_n = __ldg(ekh + j + 1);
                const float f = fq * pow2i(-ek);                  // score scale of this block
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
                // the row maximum over both halves (f > 0, so max(s) * f = max(s * f))
                const float m_mine = fmaxf(fmaxf(m0, m1), fmaxf(m2, m3));
                float *xm = xmax + (g & 1) * 2 * BM;
                xm[half * BM + rloc] = m_mine;
                mbar_arrive(&max_bar[quarter * 2 + (g & 1)]);
                if (!warp_wait(&max_bar[quarter * 2 + (g & 1)], (g >> 1) & 1)) {
                    ok = false;
                    break;
                }
                const float m_new = fmaxf(m_i, fmaxf(m_mine, xm[(half ^ 1) * BM + rloc]) * f);
                const float m_use = m_new == -INFINITY ? 0.0f : m_new;
                const float alpha = fast_exp2(m_i - m_use);
                float ps0 = 0.0f, ps1 = 0.0f;
                uint32_t hi[16], lo[16];
#pragma unroll
                for (int e = 0; e < KH; e += 2) {
                    const float p0 = fast_exp2(fmaf(sc[e], f, -m_use));
                    const float p1 = fast_exp2(fmaf(sc[e + 1], f, -m_use));
                    ps0 += p0;
                    ps1 += p1;
                    // p is finite (exp2 of a finite value or of -inf): the pair's halves directly
                    const float s0 = p0 * P_SCALE, s1 = p1 * P_SCALE;
                    const __half2 h2 = __floats2half2_rn(s0, s1);
                    const float2 hf = __half22float2(h2);
                    const __half2 l2 = __floats2half2_rn(s0 - hf.x, s1 - hf.y);
                    hi[e >> 1] = *reinterpret_cast<const uint32_t *>(&h2);
                    lo[e >> 1] = *reinterpret_cast<const uint32_t *>(&l2);
                }
                tmem_st_32x32b_x16(lane_base + scol + 16 * half, hi);
                tmem_st_32x32b_x16(lane_base + pcol + 16 * half, lo);
                l_i = l_i * alpha + (ps0 + ps1);
                m_i = m_new;
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[g & 1]);
                // the block's rescale factor to the quarter's fold warp (both halves hold the same)
                if (half == 0) {
                    if (!warp_wait(&a_empty[quarter * 2 + (g & 1)], ((g >> 1) & 1) ^ 1)) {
                        ok = false;
                        break;
                    }
                    xalpha[(g & 1) * BM + rloc] = alpha;
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&a_full[quarter * 2 + (g & 1)]);
                }
                // after the item's last scores: the next item's Q (this item's S MMAs are all done)
                if (j == w.nblocks - 1 && next && !(ok = q_to_tmem())) break;
            }
            if (!ok) break;
            // the row sum: this warp's keys plus the other warp's, to the fold warp
            xsum[half * BM + rloc] = l_i;
            mbar_arrive(&sum_bar[quarter]);
            if (!warp_wait(&sum_bar[quarter], k & 1)) {
                ok = false;
                break;
            }
            if (half == 0) {
                const float l_all = l_i + xsum[BM + rloc];
                if (!warp_wait(&l_empty[quarter * 2 + (k & 1)], ((k >> 1) & 1) ^ 1)) {
                    ok = false;
                    break;
                }
                xl[(k & 1) * BM + rloc] = l_all;
                __syncwarp();
                if (lane == 0) mbar_arrive(&l_full[quarter * 2 + (k & 1)]);
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

// row-major fp16 [rows, ld] with inner extent `cols`; boxes of 64 rows x 64 columns (128 bytes),
// 128-byte swizzle
int make_map16(CUtensorMap *map, const __half *base, int64_t rows, int64_t cols, int64_t ld) {
    EncodeTiled enc = encode_fn();
    if (!enc) return set_error(PITON_B200_ECUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
    cuuint32_t box[2] = {64, 64};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(PITON_B200_ECUDA, "cuTensorMapEncodeTiled (fp16) failed (%d)", (int)r);
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

int64_t kv_blocks_of(int64_t n_ctx) { return (n_ctx + BN - 1) / BN; }
int64_t v_ld(int64_t n_ctx) { return kv_blocks_of(n_ctx) * BN; }   // V^T row: whole 64-key blocks
size_t align1k(size_t b) { return (b + 1023) / 1024 * 1024; }
size_t k_region(const AttnParams &p) { return align1k((size_t)p.heads * p.n_ctx * HD * 2); }
size_t v_region(const AttnParams &p) { return align1k((size_t)p.heads * HD * v_ld(p.n_ctx) * 2); }
size_t e_region(const AttnParams &p) { return align1k((size_t)p.heads * kv_blocks_of(p.n_ctx)); }
size_t q_region(const AttnParams &p) { return q_in_place(p) ? 0 : align1k((size_t)p.heads * p.n_ctx * HD * 4); }

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
    return 2 * k_region(p) + 2 * v_region(p) + 2 * e_region(p) + q_region(p);
}

int attention_tc(const AttnParams &p, void *workspace, cudaStream_t stream) {
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    __half *k_hi = reinterpret_cast<__half *>(ws);
    __half *k_lo = reinterpret_cast<__half *>(ws + k_region(p));
    __half *v_hi = reinterpret_cast<__half *>(ws + 2 * k_region(p));
    __half *v_lo = reinterpret_cast<__half *>(ws + 2 * k_region(p) + v_region(p));
    int8_t *ek = reinterpret_cast<int8_t *>(ws + 2 * k_region(p) + 2 * v_region(p));
    int8_t *ev = ek + e_region(p);
    const int64_t blocks = kv_blocks_of(p.n_ctx), ldv = v_ld(p.n_ctx);
    // K [n_ctx, D] per head (strides skn, skk) -> [heads * n_ctx, D]; V [n_ctx, D] (svn, 1) -> V^T
    dim3 g((unsigned)blocks, (unsigned)p.heads);
    auto rows16 = [](const float *base, int64_t s_h, int64_t s_r) {   // 16-byte aligned unit-stride rows
        return (reinterpret_cast<uintptr_t>(base) & 15) == 0 && s_h % 4 == 0 && s_r % 4 == 0;
    };
    if (p.skk == 1 && rows16(p.k, p.skh, p.skn))
        attn_split16_vec_kernel<false><<<g, 256, 0, stream>>>(p.k, p.n_ctx, p.skh, p.skn, k_hi, k_lo, HD, ek, blocks);
    else
        attn_split16_kernel<false><<<g, 256, 0, stream>>>(p.k, p.n_ctx, p.skh, p.skn, p.skk, k_hi, k_lo, HD, ek,
                                                          blocks);
    if (rows16(p.v, p.svh, p.svn))
        attn_split16_vec_kernel<true><<<g, 256, 0, stream>>>(p.v, p.n_ctx, p.svh, p.svn, v_hi, v_lo, ldv, ev, blocks);
    else
        attn_split16_kernel<true><<<g, 256, 0, stream>>>(p.v, p.n_ctx, p.svh, p.svn, 1, v_hi, v_lo, ldv, ev, blocks);
    int launches = 3;
    const float *q = p.q;
    int64_t sqm = p.sqm, sqh = p.sqh;
    if (!q_in_place(p)) {
        float *qc = reinterpret_cast<float *>(ws + 2 * k_region(p) + 2 * v_region(p) + 2 * e_region(p));
        dim3 gq((unsigned)std::min<int64_t>(cdiv(p.n_ctx * HD, (int64_t)256), 4096), (unsigned)p.heads);
        attn_q_copy_kernel<<<gq, 256, 0, stream>>>(p.q, p.n_ctx, p.sqh, p.sqm, qc);
        q = qc;
        sqm = HD;
        sqh = p.n_ctx * HD;
        ++launches;
    }
    CUtensorMap mq, mkh, mkl, mvh, mvl;
    int rc;
    if ((rc = make_map_q(&mq, q, p.n_ctx, p.heads, sqm, sqh)) ||
        (rc = make_map16(&mkh, k_hi, p.heads * p.n_ctx, HD, HD)) || (rc = make_map16(&mkl, k_lo, p.heads * p.n_ctx, HD, HD)) ||
        (rc = make_map16(&mvh, v_hi, p.heads * HD, ldv, ldv)) || (rc = make_map16(&mvl, v_lo, p.heads * HD, ldv, ldv)))
        return rc;
    static bool attr[64][2] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const bool gather = p.world > 1;
    if (dev < 64 && !attr[dev][gather]) {
        if (gather)
            PITON_CUDA(cudaFuncSetAttribute(attn_f16x3_kernel<GATHER_THREADS>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
        else
            PITON_CUDA(cudaFuncSetAttribute(attn_f16x3_kernel<THREADS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
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
    a.ek = ek;
    a.ev = ev;
    a.kv_blocks = blocks;
    // persistent: one CTA per SM walks the items (head-major, heavy query blocks first)
    const int64_t grid = std::min<int64_t>(a.items, (int64_t)num_sms());
    if (grid > 0 && gather) {
        TcAttnGatherArgs ga;
        static_cast<TcAttnArgs &>(ga) = a;
        ga.world = p.world;
        ga.rank = p.rank;
        for (int i = 0; i < MAX_PEERS; ++i) ga.peer_o[i] = p.peer_o[i];
        attn_f16x3_kernel<GATHER_THREADS>
            <<<(unsigned)grid, GATHER_THREADS, SMEM_BYTES, stream>>>(mq, mkh, mkl, mvh, mvl, ga);
    } else if (grid > 0)
        attn_f16x3_kernel<THREADS><<<(unsigned)grid, THREADS, SMEM_BYTES, stream>>>(mq, mkh, mkl, mvh, mvl, a);
    return check_launch("attention_f16x3", launches);
}

int attention_tc_status_read_and_clear(int *status) {
    int zero = 0;
    PITON_CUDA(cudaMemcpyFromSymbol(status, g_attn_status, sizeof(int)));
    PITON_CUDA(cudaMemcpyToSymbol(g_attn_status, &zero, sizeof(int)));
    return PITON_B200_OK;
}

}  // namespace piton
