"""CUDA graphs on the device-resident path.

* TinyGPT: the library captures a decode's launch once per argument set and
  replays it with one graph launch (PITON_B200_CUDA_GRAPH);
  the tokens are the ones the plain launches produce.
* The launch surface under torch.cuda.graph capture: ``kernel[grid](...)`` with
  CUDA tensors is recorded into the graph (no host copies, timing events or
  synchronisation), so a loop of launches -- here the reference's digits MLP as
  three dense_layer_kernel launches, and a tensor-core matmul whose workspace
  comes from the graph's pool -- replays with new inputs and gives the bits of
  the eager launches.  numpy arguments are refused under capture.
"""

import ctypes as C

import numpy as np
import pytest

import piton_b200 as triton
from piton_b200 import kernels as K
from piton_b200 import tinygpt
from piton_b200.runtime.cuda import _lib, lib

pytestmark = pytest.mark.gpu


def entries():
    n = C.c_int(-1)
    _lib.check(lib().piton_b200_graph_cache_entries(C.byref(n)), "graph entries")
    return n.value


def test_tinygpt_graph_replay_same_tokens(cuda):
    torch = cuda
    model = tinygpt.TinyGPT(tinygpt.init_weights(0))
    prompts = tinygpt.random_prompts(5, seed=3)
    buf = np.zeros((5, tinygpt.CTX), np.int32)
    buf[:, :16] = prompts
    eager = torch.from_numpy(buf).cuda()
    model.generate_device(eager, 16, 64)
    _lib.check(lib().piton_b200_graph_cache_clear(), "clear")
    assert entries() == 0
    graphed = torch.from_numpy(buf).cuda()
    n0 = lib().piton_b200_launch_count()
    model.generate_device(graphed, 16, 64, graph=True)
    torch.cuda.synchronize()
    assert entries() == 1
    # every decode kernel (cluster, heads, step) runs the whole decode in one launch
    assert lib().piton_b200_launch_count() - n0 == 1
    np.testing.assert_array_equal(graphed.cpu().numpy(), eager.cpu().numpy())
    # replay: same buffers and sizes, the prompt region rewritten, no new capture
    graphed[:, 16:] = 0
    model.generate_device(graphed, 16, 64, graph=True)
    torch.cuda.synchronize()
    assert entries() == 1
    np.testing.assert_array_equal(graphed.cpu().numpy(), eager.cpu().numpy())
    # other sizes: a second entry
    short = torch.from_numpy(buf).cuda()
    model.generate_device(short, 16, 8, graph=True)
    torch.cuda.synchronize()
    assert entries() == 2
    np.testing.assert_array_equal(short.cpu().numpy()[:, :24], eager.cpu().numpy()[:, :24])
    _lib.check(lib().piton_b200_graph_cache_clear(), "clear")
    assert entries() == 0


def test_tinygpt_graph_cache_evicts_least_recently_used(cuda):
    torch = cuda
    model = tinygpt.TinyGPT(tinygpt.init_weights(1))
    _lib.check(lib().piton_b200_graph_cache_clear(), "clear")
    buf = np.zeros((2, tinygpt.CTX), np.int32)
    buf[:, :4] = tinygpt.random_prompts(2, seed=1, length=4)
    outs = []
    for new in range(1, 20):           # 19 argument sets > 16 entries
        t = torch.from_numpy(buf).cuda()
        model.generate_device(t, 4, new, graph=True)
        outs.append(t)
    torch.cuda.synchronize()
    assert entries() == 16
    ref = torch.from_numpy(buf).cuda()
    model.generate_device(ref, 4, 19)
    torch.cuda.synchronize()
    for new, t in zip(range(1, 20), outs):
        np.testing.assert_array_equal(t.cpu().numpy()[:, :4 + new], ref.cpu().numpy()[:, :4 + new])
    _lib.check(lib().piton_b200_graph_cache_clear(), "clear")


def _mlp_three_launches(x, w1, b1, w2, b2, w3, b3, h1, h2, out):
    M = x.shape[0]
    for (xi, w, b, y, n, k, relu) in ((x, w1, b1, h1, 128, 64, True), (h1, w2, b2, h2, 64, 128, True),
                                      (h2, w3, b3, out, 16, 64, False)):
        bm, bn, bk = K.dense_tiles(n)
        K.dense_layer_kernel[(triton.cdiv(M, bm) * triton.cdiv(n, bn),)](
            xi, w, b, y, M, n, k, BLOCK_SIZE_M=bm, BLOCK_SIZE_N=bn, BLOCK_SIZE_K=bk, GROUP_SIZE_M=8, ADD_BIAS=True,
            RELU=relu, device="b200")


def test_launcher_captured_into_torch_graph(cuda):
    torch = cuda
    rng = np.random.default_rng(0)
    M = 1797
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()
    w1, b1 = dev(rng.normal(0, 0.1, (64, 128))), dev(rng.normal(0, 0.1, 128))
    w2, b2 = dev(rng.normal(0, 0.1, (128, 64))), dev(rng.normal(0, 0.1, 64))
    w3, b3 = dev(rng.normal(0, 0.1, (64, 16))), dev(rng.normal(0, 0.1, 16))
    x = dev(rng.integers(0, 17, (M, 64)) / 16.0)
    h1, h2, out = (torch.empty(M, n, device="cuda") for n in (128, 64, 16))
    # matmul on the tensor-core path, workspace from the graph's pool
    A, B = dev(rng.uniform(-1, 1, (512, 384))), dev(rng.uniform(-1, 1, (384, 640)))
    Cg = torch.empty(512, 640, device="cuda")

    def step():
        _mlp_three_launches(x, w1, b1, w2, b2, w3, b3, h1, h2, out)
        K.matmul_kernel[(triton.cdiv(512, 8) * triton.cdiv(640, 64),)](
            A, B, Cg, 512, 640, 384, 384, 1, 640, 1, 640, 1, BLOCK_SIZE_M=8, BLOCK_SIZE_N=64, BLOCK_SIZE_K=8,
            GROUP_SIZE_M=8, device="b200")

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()                              # warm-up outside the capture (first-use attributes)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    n0 = lib().piton_b200_launch_count()
    with torch.cuda.graph(g):
        step()
    captured = lib().piton_b200_launch_count() - n0
    assert captured >= 4
    for trial in range(3):
        x.copy_(dev(rng.integers(0, 17, (M, 64)) / 16.0))
        A.copy_(dev(rng.uniform(-1, 1, (512, 384))))
        g.replay()
        torch.cuda.synchronize()
        got_out, got_c = out.clone(), Cg.clone()
        step()                              # eager launches on the same inputs
        torch.cuda.synchronize()
        np.testing.assert_array_equal(got_out.cpu().numpy().view(np.uint32), out.cpu().numpy().view(np.uint32))
        np.testing.assert_array_equal(got_c.cpu().numpy().view(np.uint32), Cg.cpu().numpy().view(np.uint32))
    ref = A.double() @ B.double()
    assert float((Cg.double() - ref).abs().max() / ref.abs().max()) <= 4e-6
    del g


def test_numpy_arguments_refused_under_capture(cuda):
    torch = cuda
    xs = np.ones(1024, np.float32)
    y = torch.ones(1024, device="cuda")
    o = torch.empty(1024, device="cuda")
    K.add_kernel[(4,)](y, y, o, 1024, BLOCK_SIZE=256, device="b200")   # warm-up
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with pytest.raises(TypeError, match="CUDA-graph capture"):
        with torch.cuda.graph(g):
            K.add_kernel[(4,)](xs, y, o, 1024, BLOCK_SIZE=256, device="b200")
