// All-gather of equal output pieces without NCCL: the other operators' shards (softmax
// rows, attention heads, add ranges, MLP / TinyGPT batch rows) stored by this rank into
// every rank's full output through NVLink peer stores.  Each 16-byte chunk of the local
// piece is loaded once and stored to every destination (the own buffer included), so the
// traffic leaving a GPU is (world - 1) pieces and the HBM read is one piece.
#include "common.cuh"
#include "gemm_tc.cuh"

namespace {

struct Dests {
    char *p[piton::MAX_PEERS];
};

__global__ void __launch_bounds__(256) allgather_vec16_kernel(const uint4 *__restrict__ src, int64_t n16, Dests d,
                                                              int world, int64_t dst_off16) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x) {
        const uint4 v = src[i];
        for (int r = 0; r < world; ++r) reinterpret_cast<uint4 *>(d.p[r])[dst_off16 + i] = v;
    }
}

__global__ void __launch_bounds__(256) allgather_bytes_kernel(const unsigned char *__restrict__ src, int64_t n, Dests d,
                                                              int world, int64_t dst_off) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const unsigned char v = src[i];
        for (int r = 0; r < world; ++r) d.p[r][dst_off + i] = v;
    }
}

}  // namespace

extern "C" int piton_b200_allgather(const piton_allgather_args *g, uint64_t src, size_t bytes, void *stream) {
    using namespace piton;
    PITON_REQUIRE(g != nullptr, "allgather args is NULL");
    PITON_REQUIRE(g->world >= 1 && g->world <= MAX_PEERS && g->rank >= 0 && g->rank < g->world,
                  "world %d / rank %d outside 1..%d", g->world, g->rank, MAX_PEERS);
    for (int i = 0; i < g->world; ++i) PITON_REQUIRE(g->peer_c[i] != 0, "peer output %d is NULL", i);
    if (bytes == 0) return PITON_B200_OK;
    PITON_REQUIRE(src != 0, "NULL source");
    Dests d;
    uintptr_t align = src | (uintptr_t)bytes;
    for (int i = 0; i < MAX_PEERS; ++i) {
        d.p[i] = i < g->world ? reinterpret_cast<char *>(g->peer_c[i]) : nullptr;
        if (i < g->world) align |= g->peer_c[i];
    }
    const int64_t off = (int64_t)g->rank * (int64_t)bytes;
    cudaStream_t s = as_stream(stream);
    const int64_t units = (align & 15) == 0 ? (int64_t)bytes / 16 : (int64_t)bytes;
    int64_t blocks = cdiv(units, (int64_t)256);
    if (blocks > (int64_t)num_sms() * 8) blocks = (int64_t)num_sms() * 8;
    if ((align & 15) == 0)
        allgather_vec16_kernel<<<(unsigned)blocks, 256, 0, s>>>(reinterpret_cast<const uint4 *>(src), units, d, g->world,
                                                                off / 16);
    else
        allgather_bytes_kernel<<<(unsigned)blocks, 256, 0, s>>>(reinterpret_cast<const unsigned char *>(src), units, d,
                                                                g->world, off);
    return check_launch("allgather", 1);
}
