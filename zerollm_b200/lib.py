"""ctypes binding of libzerollm_b200.so (the C ABI in include/zerollm_b200.h).

The shared library is the product: there is no Python or CPU fallback.  If the
library is missing, loading fails with an error that says how to build it.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libzerollm_b200.so")

ZL_OK, ZL_EINVAL, ZL_ECUDA, ZL_ETIMEOUT, ZL_ENCCL, ZL_ENOMEM, ZL_EUNSUPPORTED, ZL_ESTATE, ZL_EIO = range(9)
EPI_BIAS, EPI_RELU, EPI_RESIDUAL, EPI_RELU_MASK, EPI_ROPE = 1, 2, 4, 8, 16
EPI_ACCUM, EPI_OUT_F32 = 64, 128
A_KMAJOR, B_KMAJOR = 1, 2

vp = C.c_void_p
i32, i64, f32, u64 = C.c_int, C.c_int64, C.c_float, C.c_uint64


class ZLError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"zerollm_b200 error {code}: {msg}")
        self.code = code


class Epilogue(C.Structure):
    _fields_ = [("bias", vp), ("residual", vp), ("aux", vp), ("rope_cos", vp), ("rope_sin", vp),
                ("rope_cols", i32), ("rope_seq", i32), ("head_dim", i32), ("rope_pair_major", i32)]


class ModelConfig(C.Structure):
    _fields_ = [("vocab_size", i32), ("embed_dim", i32), ("num_layers", i32), ("num_heads", i32),
                ("ff_hidden_dim", i32), ("max_seq_len", i32), ("norm", i32), ("pos", i32), ("tied", i32),
                ("bias", i32), ("eps", f32), ("rope_base", f32)]


class AdamWConfig(C.Structure):
    _fields_ = [("beta1", f32), ("beta2", f32), ("eps", f32), ("weight_decay", f32)]


# name -> (restype, argtypes); every zl_* returning zl_status uses i32
SIGNATURES = {
    "zl_last_error": (C.c_char_p, []),
    "zl_version": (C.c_char_p, []),
    "zl_device_error": (i32, [C.POINTER(i32)]),
    "zl_matmul_f32": (i32, [vp, vp, vp, i32, i32, i32, vp]),
    "zl_matmul_at_b_f32": (i32, [vp, vp, vp, i32, i32, i32, vp]),
    "zl_matmul_a_bt_f32": (i32, [vp, vp, vp, i32, i32, i32, vp]),
    "zl_linear_forward_f32": (i32, [vp, vp, vp, vp, i64, i64, i64, i32, vp]),
    "zl_linear_backward_f32": (i32, [vp, vp, vp, vp, vp, vp, i64, i64, i64, i32, vp]),
    "zl_mha_forward_f32": (i32, [vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, i32, vp]),
    "zl_mha_backward_f32": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, i32, i32, vp]),
    "zl_layernorm_forward_f32": (i32, [vp, vp, vp, vp, vp, vp, i64, i64, f32, vp]),
    "zl_layernorm_backward_f32": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, vp]),
    "zl_rmsnorm_forward_f32": (i32, [vp, vp, vp, vp, i64, i64, f32, vp]),
    "zl_rmsnorm_backward_f32": (i32, [vp, vp, vp, vp, vp, vp, i64, i64, vp]),
    "zl_softmax_f32": (i32, [vp, vp, i32, i32, vp]),
    "zl_cross_entropy_backward_f32": (i32, [vp, vp, vp, i32, i32, vp]),
    "zl_cross_entropy_forward_f32": (i32, [vp, vp, i32, i32, f32, vp, vp]),
    "zl_embedding_forward_f32": (i32, [vp, vp, vp, vp, i32, i32, i32, i32, i32, vp]),
    "zl_embedding_backward_f32": (i32, [vp, vp, vp, i32, i32, i32, i32, vp]),
    "zl_add_f32": (i32, [vp, vp, vp, i32, vp]),
    "zl_add_inplace_f32": (i32, [vp, vp, i32, vp]),
    "zl_relu_forward_f32": (i32, [vp, vp, i32, vp]),
    "zl_relu_backward_f32": (i32, [vp, vp, vp, i32, vp]),
    "zl_transpose_f32": (i32, [vp, vp, i32, i32, vp]),
    "zl_adamw_step_f32": (i32, [vp, vp, vp, vp, i64] + [f32] * 7 + [vp]),
    "zl_adam_step_f32": (i32, [vp, vp, vp, vp, i64] + [f32] * 6 + [vp]),
    "zl_sgd_step_f32": (i32, [vp, vp, vp, i64, f32, f32, f32, vp]),
    "zl_gemm_bf16": (i32, [vp, vp, vp, i32, i32, i32, i32, i32, C.POINTER(Epilogue), vp, vp]),
    "zl_gemm_bf16_colsum": (i32, [vp, vp, vp, i32, i32, i32, i32, i32, C.POINTER(Epilogue), vp, vp, vp]),
    "zl_gemm_bf16_relu_bits": (i32, [vp, vp, vp, i32, i32, i32, i32, i32, C.POINTER(Epilogue), vp, vp, vp, vp]),
    "zl_gemm_bf16_sched": (i32, [vp, vp, vp, i32, i32, i32, i32, i32, C.POINTER(Epilogue), vp, vp, vp]),
    "zl_gemm_workspace_floats": (i64, [i32, i32, i32, i32, i32]),
    "zl_attention_forward_bf16": (i32, [vp, vp, vp, i32, i32, i32, i32, vp]),
    "zl_attention_backward_bf16": (i32, [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, vp, vp, vp]),
    "zl_attention_workspace_floats": (i64, [i32, i32, i32, i32]),
    "zl_norm_forward_bf16": (i32, [i32, vp, vp, vp, vp, vp, vp, i64, i32, f32, vp]),
    "zl_norm_backward_bf16": (i32, [i32, vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i32, vp]),
    "zl_norm_bwd_blocks": (i32, [i64]),
    "zl_embedding_forward_bf16": (i32, [vp, vp, vp, vp, i64, i32, i32, i32, vp]),
    "zl_embedding_backward_bf16": (i32, [vp, vp, vp, i64, i32, i32, vp]),
    "zl_cross_entropy_fused_bf16": (i32, [vp, vp, i32, i32, f32, f32, vp, vp, vp]),
    "zl_colsum_bf16": (i32, [vp, vp, vp, i64, i32, vp]),
    "zl_linear_forward_bf16": (i32, [vp, vp, vp, vp, i64, i64, i64, i32, vp]),
    "zl_linear_backward_bf16": (i32, [vp, vp, vp, vp, vp, vp, i64, i64, i64, i32, vp]),
    "zl_mha_forward_bf16": (i32, [vp, vp, vp, vp, vp, C.c_size_t, vp, i64, i64, i64, i64, i32, vp]),
    "zl_mha_backward_bf16": (i32, [vp, vp, vp, vp, vp, C.c_size_t, vp, vp, vp, vp, i64, i64, i64, i64, i32, i32,
                                   vp]),
    "zl_mha_state_bytes_bf16": (C.c_size_t, [i64, i64, i64, i64]),
    "zl_layernorm_forward_bf16": (i32, [vp, vp, vp, vp, vp, vp, i64, i64, f32, vp]),
    "zl_layernorm_backward_bf16": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, vp]),
    "zl_softmax_bf16": (i32, [vp, vp, i32, i32, vp]),
    "zl_add_bf16": (i32, [vp, vp, vp, i32, vp]),
    "zl_add_inplace_bf16": (i32, [vp, vp, i32, vp]),
    "zl_relu_forward_bf16": (i32, [vp, vp, i32, vp]),
    "zl_relu_backward_bf16": (i32, [vp, vp, vp, i32, vp]),
    "zl_adamw_step_bf16": (i32, [vp, vp, vp, vp, i64] + [f32] * 7 + [vp]),
    "zl_colsum_workspace_floats": (i64, [i64, i32]),
    "zl_colsum_bf16_noalloc": (i32, [vp, vp, i64, i32, vp]),
    "zl_colsum_noalloc_max_floats": (i64, []),
    "zl_adamw_flat": (i32, [vp, vp, vp, vp, vp, i64] + [f32] * 8 + [vp]),
    "zl_f32_to_bf16": (i32, [vp, vp, i64, vp]),
    "zl_model_create": (i32, [C.POINTER(ModelConfig), i64, u64, f32, C.POINTER(vp)]),
    "zl_model_destroy": (i32, [vp]),
    "zl_model_param_layout": (i32, [C.POINTER(ModelConfig), vp, vp, vp, i32, C.POINTER(i32), C.POINTER(i64)]),
    "zl_model_num_params": (i32, [vp, C.POINTER(i64)]),
    "zl_model_buffers": (i32, [vp, C.POINTER(vp), C.POINTER(vp), C.POINTER(vp), C.POINTER(vp)]),
    "zl_model_params_updated": (i32, [vp, vp]),
    "zl_model_set_optimizer": (i32, [vp, C.POINTER(AdamWConfig)]),
    "zl_model_train_step": (i32, [vp, vp, vp, i32, i32, f32, i32, vp, vp]),
    "zl_model_forward": (i32, [vp, vp, i32, i32, vp, vp]),
    "zl_model_backward": (i32, [vp, vp, vp, i32, i32, vp]),
    "zl_model_zero_grad": (i32, [vp, vp]),
    "zl_model_step": (i32, [vp, f32, vp]),
    "zl_model_last_launches": (i32, [vp, C.POINTER(i32)]),
    "zl_model_set_graph": (i32, [vp, i32]),
    "zl_model_set_kernel_timing": (i32, [vp, i32]),
    "zl_model_kernel_times": (i32, [vp, C.POINTER(f32), C.POINTER(f32)]),
    "zl_model_step_times": (i32, [vp, C.POINTER(f32), C.POINTER(f32)]),
    "zl_nccl_unique_id": (i32, [vp, C.c_size_t]),
    "zl_model_attach_nccl": (i32, [vp, vp, i32, i32, i64]),
    "zl_bucket_plan": (i32, [vp, vp, i32, i64, vp, vp, i32, C.POINTER(i32)]),
    "zl_model_param_checksum": (i32, [vp, C.POINTER(u64), vp]),
    "zl_model_save": (i32, [vp, C.c_char_p, i32]),
    "zl_model_load": (i32, [vp, C.c_char_p, i32]),
    "zl_checkpoint_manifest": (i32, [C.POINTER(ModelConfig), C.c_char_p, i64, C.POINTER(i64)]),
    "zl_loader_create": (i32, [vp, vp, i64, i32, i32, i32, i32, i32, u64, C.POINTER(vp)]),
    "zl_loader_destroy": (i32, [vp]),
    "zl_loader_reset": (i32, [vp]),
    "zl_loader_info": (i32, [vp, C.POINTER(i64), C.POINTER(i64)]),
    "zl_loader_next": (i32, [vp, vp, vp, C.POINTER(i32)]),
    "zl_loader_start": (i32, [vp, i32]),
    "zl_loader_next_device": (i32, [vp, vp, vp, C.POINTER(i32), vp]),
    "zl_comm_create": (i32, [vp, i32, i32, C.c_double, C.POINTER(vp)]),
    "zl_comm_create_from_file": (i32, [C.c_char_p, i32, i32, C.c_double, C.POINTER(vp)]),
    "zl_comm_destroy": (i32, [vp]),
    "zl_comm_all_reduce": (i32, [vp, vp, C.c_size_t, i32, i32, vp]),
    "zl_comm_broadcast": (i32, [vp, vp, C.c_size_t, i32, i32, vp]),
    "zl_comm_all_gather": (i32, [vp, vp, vp, C.c_size_t, i32, vp]),
    "zl_comm_check": (i32, [vp, vp, C.c_double]),
    "zl_comm_rank": (i32, [vp, C.POINTER(i32), C.POINTER(i32)]),
}

_LIB = None


def load():
    """Loads the library (once).  Raises if it has not been built."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} not found: build it with `python -m zerollm_b200.build` "
                               "(the CUDA library is required; there is no fallback)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def check(status: int):
    if status != ZL_OK:
        msg = load().zl_last_error()
        raise ZLError(status, msg.decode() if msg else "")


def call(name: str, *args):
    """Calls a zl_* entry point returning zl_status and raises on failure."""
    check(getattr(load(), name)(*args))
