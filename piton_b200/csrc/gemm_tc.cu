// tcgen05 3xTF32 GEMM: placeholder until the tensor-core path lands.
#include "common.cuh"
#include "gemm_tc.cuh"

namespace piton {
bool tc_gemm_supported(const TcGemmShape &) { return false; }
size_t tc_gemm_workspace_bytes(const TcGemmShape &) { return 0; }
int tc_gemm(const TcGemmShape &, void *, cudaStream_t) { return set_error(PITON_B200_ENOTSUP, "tensor-core GEMM not built"); }
}  // namespace piton
