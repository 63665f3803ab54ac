// Parameters of the CUDA-core GEMM shared by matmul and the dense layer.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace piton {

struct GemmSimtParams {
    const float *a, *b;
    float *c;
    const float *bias;      // nullptr: no bias
    int64_t M, N, K;
    int64_t sam, sak, sbk, sbn, scm, scn;
    int64_t ref_bm, ref_bn, ref_group, grid_x;   // the reference launch's tiles, group and grid
    int check_grid;         // 0: every element of C is written
    int relu;
};

__host__ __device__ inline int64_t cdiv_d(int64_t a, int64_t b) { return (a + b - 1) / b; }

int gemm_simt(const GemmSimtParams &p, bool qpu, cudaStream_t s);

// Number of reference programs (tiles) of a grouped launch.
inline int64_t grouped_tiles(int64_t M, int64_t N, int64_t bm, int64_t bn) { return cdiv_d(M, bm) * cdiv_d(N, bn); }

}  // namespace piton
