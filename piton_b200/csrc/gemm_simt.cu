// CUDA-core fp32 GEMM for the tutorial matmul (examples/kernels.py:18-57) and
// the dense layer (examples/nn_kernels.py:23-74) wherever the tensor-core path
// does not apply: arbitrary (also negative) element strides, unaligned
// pointers, partial launch grids, small problems, and the QPU rounding mode.
//
// Semantics kept from the reference programs:
//  * C[m, n] = sum_k A[m, k] B[k, n] over the whole K (the K-tail mask of the
//    reference loads zeros, which add nothing);
//  * only elements of C tiles whose grouped program id (GROUP_SIZE_M order,
//    examples/kernels.py:26-35) is below grid_x are written; with a full grid
//    every element of C is;
//  * dense: bias added after the dot, then ReLU (nn_kernels.py:66-69).
//  * QPU rounding: each output accumulates round-toward-zero products in k
//    order with round-toward-zero adds (piton/backend/lower.py:3761-3878), so
//    results match the QPU emulator bit for bit.
//
// Tile 64x64x16, 256 threads, 4x4 outputs per thread, both operand tiles
// staged through shared memory with generic strided loads.
#include "common.cuh"
#include "gemm_simt.cuh"

namespace piton {

constexpr int GS_BM = 64, GS_BN = 64, GS_BK = 16;

template <bool QPU>
__global__ void __launch_bounds__(256) gemm_simt_kernel(GemmSimtParams p) {
    __shared__ float As[GS_BK][GS_BM + 1];
    __shared__ float Bs[GS_BK][GS_BN + 1];
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int64_t m0 = (int64_t)blockIdx.y * GS_BM, n0 = (int64_t)blockIdx.x * GS_BN;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;

    for (int64_t k0 = 0; k0 < p.K; k0 += GS_BK) {
#pragma unroll
        for (int e = 0; e < (GS_BM * GS_BK) / 256; ++e) {
            int idx = tid + e * 256;
            int r = idx / GS_BK, kk = idx % GS_BK;      // A tile: consecutive threads walk k
            int64_t m = m0 + r, k = k0 + kk;
            As[kk][r] = (m < p.M && k < p.K) ? p.a[m * p.sam + k * p.sak] : 0.0f;
        }
#pragma unroll
        for (int e = 0; e < (GS_BN * GS_BK) / 256; ++e) {
            int idx = tid + e * 256;
            int kk = idx / GS_BN, c = idx % GS_BN;      // B tile: consecutive threads walk n
            int64_t n = n0 + c, k = k0 + kk;
            Bs[kk][c] = (n < p.N && k < p.K) ? p.b[k * p.sbk + n * p.sbn] : 0.0f;
        }
        __syncthreads();
        int kmax = (int)((p.K - k0) < GS_BK ? (p.K - k0) : GS_BK);
        for (int kk = 0; kk < kmax; ++kk) {
            float av[4], bv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) av[i] = As[kk][ty + 16 * i];
#pragma unroll
            for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx + 16 * j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if constexpr (QPU) acc[i][j] = qpu_fadd(acc[i][j], qpu_fmul(av[i], bv[j]));
                    else acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
                }
        }
        __syncthreads();
    }

    // grouped program order: which reference program owns tile (pid_m, pid_n)
    const int64_t num_pid_m = cdiv_d(p.M, p.ref_bm), num_pid_n = cdiv_d(p.N, p.ref_bn);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        int64_t m = m0 + ty + 16 * i;
        if (m >= p.M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            int64_t n = n0 + tx + 16 * j;
            if (n >= p.N) continue;
            if (p.check_grid) {
                int64_t pid_m = m / p.ref_bm, pid_n = n / p.ref_bn;
                int64_t group_id = pid_m / p.ref_group;
                int64_t first = group_id * p.ref_group;
                int64_t gsize = num_pid_m - first < p.ref_group ? num_pid_m - first : p.ref_group;
                int64_t pid = group_id * p.ref_group * num_pid_n + pid_n * gsize + (pid_m - first);
                if (pid >= p.grid_x) continue;
            }
            float v = acc[i][j];
            if (p.bias) {
                if constexpr (QPU) v = qpu_fadd(v, p.bias[n]);
                else v += p.bias[n];
            }
            if (p.relu) v = fmaxf(v, 0.0f);
            p.c[m * p.scm + n * p.scn] = v;
        }
    }
}

int gemm_simt(const GemmSimtParams &p, bool qpu, cudaStream_t s) {
    if (p.M <= 0 || p.N <= 0) return PITON_B200_OK;
    dim3 grid((unsigned)cdiv(p.N, GS_BN), (unsigned)cdiv(p.M, GS_BM));
    PITON_REQUIRE(grid.y < 65536u, "M too large for the CUDA-core path");
    if (qpu) gemm_simt_kernel<true><<<grid, 256, 0, s>>>(p);
    else gemm_simt_kernel<false><<<grid, 256, 0, s>>>(p);
    return check_launch("gemm_simt");
}

}  // namespace piton
