"""ctypes binding of libpiton_b200.so (include/piton_b200.h).

The library is loaded from the package directory, where ``python -m
piton_b200.build`` puts it.  There is no fallback: a missing or unloadable
library raises ``ImportError`` naming the file, so nothing silently runs
elsewhere.
"""

from __future__ import annotations

import ctypes as C
import os

PKG = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
LIB_PATH = os.environ.get("PITON_B200_LIB", os.path.join(PKG, "libpiton_b200.so"))

OK, EINVAL, ECUDA, ETIMEOUT, ENOTSUP, ENOMEM, EWORKSPACE = 0, -1, -2, -3, -4, -5, -6
QPU_ROUNDING, FORCE_SIMT, CUDA_GRAPH = 0x1, 0x2, 0x4
NOALLOC_SCRATCH_BYTES = 32 << 20   # PITON_B200_NOALLOC_SCRATCH_BYTES

u64, i64, i32, u32, f64 = C.c_uint64, C.c_int64, C.c_int32, C.c_uint32, C.c_double


class AddArgs(C.Structure):
    _fields_ = [("x", u64), ("y", u64), ("out", u64), ("n_elements", i64), ("block_size", i64), ("grid_x", i64),
                ("flags", u32), ("_pad", u32)]


class SoftmaxArgs(C.Structure):
    _fields_ = [("out", u64), ("in_", u64), ("in_row_stride", i64), ("out_row_stride", i64), ("n_cols", i64),
                ("block_size", i64), ("grid_x", i64), ("flags", u32), ("_pad", u32)]


class MatmulArgs(C.Structure):
    _fields_ = [("a", u64), ("b", u64), ("c", u64), ("M", i64), ("N", i64), ("K", i64),
                ("stride_am", i64), ("stride_ak", i64), ("stride_bk", i64), ("stride_bn", i64),
                ("stride_cm", i64), ("stride_cn", i64), ("block_m", i64), ("block_n", i64), ("block_k", i64),
                ("group_m", i64), ("grid_x", i64), ("workspace", u64), ("workspace_bytes", u64),
                ("flags", u32), ("_pad", u32)]


class AllgatherArgs(C.Structure):
    _fields_ = [("peer_c", u64 * 8), ("world", i32), ("rank", i32), ("row_offset", i64), ("ldc", i64),
                ("multicast_c", u64)]


class DenseArgs(C.Structure):
    _fields_ = [("x", u64), ("w", u64), ("bias", u64), ("y", u64), ("M", i64), ("N", i64), ("K", i64),
                ("block_m", i64), ("block_n", i64), ("block_k", i64), ("group_m", i64), ("grid_x", i64),
                ("add_bias", i32), ("relu", i32), ("flags", u32), ("_pad", u32)]


class MlpArgs(C.Structure):
    _fields_ = [("images", u64), ("w1", u64), ("b1", u64), ("w2", u64), ("b2", u64), ("w3", u64), ("b3", u64),
                ("logits", u64), ("pred", u64), ("M", i64), ("images_u8", i32), ("n_classes", i32),
                ("flags", u32), ("_pad", u32)]


class AttentionArgs(C.Structure):
    _fields_ = [("q", u64), ("k", u64), ("v", u64), ("out", u64), ("sm_scale", f64),
                ("stride_qh", i64), ("stride_qm", i64), ("stride_kh", i64), ("stride_kn", i64), ("stride_kk", i64),
                ("stride_vh", i64), ("stride_vn", i64), ("stride_oh", i64), ("stride_om", i64),
                ("n_ctx", i64), ("head_dim", i64), ("block_m", i64), ("block_n", i64), ("grid_x", i64),
                ("grid_y", i64), ("causal", i32), ("even_n", i32), ("workspace", u64), ("workspace_bytes", u64),
                ("flags", u32), ("_pad", u32)]


class LayernormArgs(C.Structure):
    _fields_ = [("x", u64), ("y", u64), ("rows", i64), ("n_cols", i64), ("x_row_stride", i64),
                ("y_row_stride", i64), ("eps", f64), ("flags", u32), ("_pad", u32)]


class ElementwiseArgs(C.Structure):
    _fields_ = [("x", u64), ("y", u64), ("out", u64), ("n_elements", i64), ("block_size", i64), ("grid_x", i64),
                ("alpha", f64), ("op", i32), ("flags", u32)]


class IdivArgs(C.Structure):
    _fields_ = [("x", u64), ("y", u64), ("q", u64), ("r", u64), ("n_elements", i64), ("block_size", i64),
                ("grid_x", i64), ("is_signed", i32), ("flags", u32)]


class RowReduceArgs(C.Structure):
    _fields_ = [("x", u64), ("out", u64), ("n_cols", i64), ("stride", i64), ("block_m", i64), ("block_n", i64),
                ("grid_x", i64), ("reduce", i32), ("flags", u32)]


class TransposeArgs(C.Structure):
    _fields_ = [("x", u64), ("out", u64), ("n_rows", i64), ("n_cols", i64), ("stride_x", i64), ("stride_out", i64),
                ("block_m", i64), ("block_n", i64), ("grid_x", i64), ("flags", u32), ("_pad", u32)]


class LifeArgs(C.Structure):
    _fields_ = [("src", u64), ("dst", u64), ("n_rows", i64), ("n_cols", i64), ("stride", i64), ("block_r", i64),
                ("block_c", i64), ("grid_x", i64), ("grid_y", i64), ("mode", i32), ("flags", u32)]


class TinyGPTArgs(C.Structure):
    _fields_ = [("weights", u64), ("kv_cache", u64), ("tokens", u64), ("logits", u64), ("batch", i64),
                ("prompt_len", i64), ("new_tokens", i64), ("vocab", i32), ("d_model", i32), ("n_layer", i32),
                ("n_head", i32), ("ctx", i32), ("flags", u32)]


# name -> (restype, argtypes); every function include/piton_b200.h declares
PROTOTYPES = {
    "piton_b200_abi_version": (C.c_int, []),
    "piton_b200_last_error": (C.c_char_p, []),
    "piton_b200_launch_count": (C.c_uint64, []),
    "piton_b200_init": (C.c_int, [C.c_int]),
    "piton_b200_device_count": (C.c_int, [C.POINTER(C.c_int)]),
    "piton_b200_get_device": (C.c_int, [C.POINTER(C.c_int)]),
    "piton_b200_malloc": (C.c_int, [C.POINTER(u64), C.c_size_t]),
    "piton_b200_free": (C.c_int, [u64]),
    "piton_b200_memcpy_h2d": (C.c_int, [u64, C.c_void_p, C.c_size_t, C.c_void_p]),
    "piton_b200_memcpy_d2h": (C.c_int, [C.c_void_p, u64, C.c_size_t, C.c_void_p]),
    "piton_b200_memset": (C.c_int, [u64, C.c_int, C.c_size_t, C.c_void_p]),
    "piton_b200_stream_wait": (C.c_int, [C.c_void_p, C.c_double]),
    "piton_b200_device_status": (C.c_int, [C.POINTER(C.c_int)]),
    "piton_b200_add_f32": (C.c_int, [C.POINTER(AddArgs), C.c_void_p]),
    "piton_b200_softmax_f32": (C.c_int, [C.POINTER(SoftmaxArgs), C.c_void_p]),
    "piton_b200_matmul_workspace_size": (C.c_size_t, [C.POINTER(MatmulArgs)]),
    "piton_b200_matmul_f32": (C.c_int, [C.POINTER(MatmulArgs), C.c_void_p]),
    "piton_b200_matmul_f32_noalloc": (C.c_int, [C.POINTER(MatmulArgs), C.c_void_p]),
    "piton_b200_matmul_host_workspace_size": (C.c_size_t, [C.POINTER(MatmulArgs)]),
    "piton_b200_matmul_f32_host": (C.c_int, [C.POINTER(MatmulArgs), C.c_void_p]),
    "piton_b200_matmul_allgather_f32": (C.c_int, [C.POINTER(MatmulArgs), C.POINTER(AllgatherArgs), C.c_void_p]),
    "piton_b200_allgather": (C.c_int, [C.POINTER(AllgatherArgs), u64, C.c_size_t, C.c_void_p]),
    "piton_b200_ipc_handle": (C.c_int, [u64, C.c_void_p]),
    "piton_b200_ipc_open": (C.c_int, [C.c_void_p, C.POINTER(u64)]),
    "piton_b200_ipc_close": (C.c_int, [u64]),
    "piton_b200_dense_f32": (C.c_int, [C.POINTER(DenseArgs), C.c_void_p]),
    "piton_b200_mlp_f32": (C.c_int, [C.POINTER(MlpArgs), C.c_void_p]),
    "piton_b200_attention_workspace_size": (C.c_size_t, [C.POINTER(AttentionArgs)]),
    "piton_b200_attention_f32": (C.c_int, [C.POINTER(AttentionArgs), C.c_void_p]),
    "piton_b200_softmax_allgather_f32": (C.c_int, [C.POINTER(SoftmaxArgs), C.POINTER(AllgatherArgs), C.c_void_p]),
    "piton_b200_add_allgather_f32": (C.c_int, [C.POINTER(AddArgs), C.POINTER(AllgatherArgs), C.c_void_p]),
    "piton_b200_attention_allgather_f32": (C.c_int, [C.POINTER(AttentionArgs), C.POINTER(AllgatherArgs),
                                                     C.c_void_p]),
    "piton_b200_layernorm_f32": (C.c_int, [C.POINTER(LayernormArgs), C.c_void_p]),
    "piton_b200_elementwise_f32": (C.c_int, [C.POINTER(ElementwiseArgs), C.c_void_p]),
    "piton_b200_idiv_i32": (C.c_int, [C.POINTER(IdivArgs), C.c_void_p]),
    "piton_b200_row_reduce_f32": (C.c_int, [C.POINTER(RowReduceArgs), C.c_void_p]),
    "piton_b200_transpose_f32": (C.c_int, [C.POINTER(TransposeArgs), C.c_void_p]),
    "piton_b200_life_step": (C.c_int, [C.POINTER(LifeArgs), C.c_void_p]),
    "piton_b200_tinygpt_weight_floats": (C.c_int64, []),
    "piton_b200_tinygpt_generate": (C.c_int, [C.POINTER(TinyGPTArgs), C.c_void_p]),
    "piton_b200_graph_cache_entries": (C.c_int, [C.POINTER(C.c_int)]),
    "piton_b200_graph_cache_clear": (C.c_int, []),
}

STRUCTS = {"piton_allgather_args": AllgatherArgs, "piton_add_args": AddArgs, "piton_softmax_args": SoftmaxArgs, "piton_matmul_args": MatmulArgs,
           "piton_dense_args": DenseArgs, "piton_mlp_args": MlpArgs, "piton_attention_args": AttentionArgs,
           "piton_layernorm_args": LayernormArgs, "piton_tinygpt_args": TinyGPTArgs,
           "piton_elementwise_args": ElementwiseArgs, "piton_idiv_args": IdivArgs,
           "piton_row_reduce_args": RowReduceArgs, "piton_transpose_args": TransposeArgs, "piton_life_args": LifeArgs}

_lib = None


def lib():
    """The loaded library (loaded once)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m piton_b200.build` "
                              f"(the B200 backend has no CPU fallback)")
        try:
            handle = C.CDLL(LIB_PATH)
        except OSError as e:
            raise ImportError(f"cannot load {LIB_PATH}: {e}") from e
        for name, (res, argtypes) in PROTOTYPES.items():
            f = getattr(handle, name)
            f.restype = res
            f.argtypes = argtypes
        _lib = handle
    return _lib


class B200Error(RuntimeError):
    pass


def check(rc: int, what: str = "") -> None:
    if rc == OK:
        return
    msg = lib().piton_b200_last_error().decode(errors="replace")
    text = f"{what}: {msg}" if what else msg
    if rc == EINVAL:
        raise ValueError(text)
    if rc == ENOTSUP:
        raise NotImplementedError(text)
    if rc == ETIMEOUT:
        raise TimeoutError(text)
    if rc == ENOMEM:
        raise MemoryError(text)
    raise B200Error(f"[{rc}] {text}")
