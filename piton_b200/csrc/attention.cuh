// Parameters shared by the attention kernels.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "gemm_tc.cuh"   // MAX_PEERS

namespace piton {

struct AttnParams {
    const float *q, *k, *v;
    float *o;
    int64_t sqh, sqm, skh, skn, skk, svh, svn, soh, som;
    int64_t n_ctx, head_dim, heads;
    int64_t key_end;   // keys >= key_end never contribute
    int64_t row_end;   // query rows >= row_end are not written
    float qk_scale;    // sm_scale * log2(e)
    int causal;
    // all-gather (world > 1, tensor-core path): o = peer_o[rank]; every row is also stored at the
    // same offset from each other rank's peer_o (full outputs, offset to this rank's first head)
    int world = 0, rank = 0;
    float *peer_o[MAX_PEERS] = {};
};

int attention_simt(const AttnParams &p, cudaStream_t s);
// tcgen05 3xTF32 kernel (attention_tc.cu): HEAD_DIM 64, n_ctx >= 64.
bool attention_tc_supported(const AttnParams &p);
size_t attention_tc_workspace_bytes(const AttnParams &p);
int attention_tc(const AttnParams &p, void *workspace, cudaStream_t s);
// The tensor-core attention kernel's status word (0, or the bounded wait that ran out), then reset.
int attention_tc_status_read_and_clear(int *status);

}  // namespace piton
