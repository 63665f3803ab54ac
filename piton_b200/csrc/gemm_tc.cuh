// Interface of the tcgen05 3xTF32 GEMM (gemm_tc.cu).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace piton {

constexpr int MAX_PEERS = 8;

struct TcGemmShape {
    const float *a, *b;
    float *c;
    int64_t M, N, K;
    int64_t sam, sak, sbk, sbn, scm, scn;
    // all-gather epilogue (world > 0): every C tile is stored into each peer's
    // row-major [*, ldc_peer] output at rows row_offset + m, instead of into c
    int world = 0, rank = 0;
    int64_t row_offset = 0, ldc_peer = 0;
    float *peer_c[MAX_PEERS] = {};
    float *multicast_c = nullptr;   // non-null: multimem stores through the NVSwitch instead of peer copies
    // false: B's split operands (high half and bf16 cross operand) are already in
    // the workspace from an earlier call with the same B, N and K (the workspace
    // holds B's operands first, so their place does not depend on M)
    bool split_b = true;
};

// True when the tensor-core path can run this problem (layout and alignment).
bool tc_gemm_supported(const TcGemmShape &s);
// Scratch bytes the path needs for the split operands.
size_t tc_gemm_workspace_bytes(const TcGemmShape &s);
int tc_gemm(const TcGemmShape &s, void *workspace, cudaStream_t stream);

}  // namespace piton
