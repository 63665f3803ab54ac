// Parameters shared by the attention kernels.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

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
};

int attention_simt(const AttnParams &p, cudaStream_t s);
// Picks the tensor-core kernel where it applies, else the CUDA-core one.
int attention_dispatch(const AttnParams &p, cudaStream_t s);

}  // namespace piton
