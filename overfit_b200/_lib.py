"""ctypes binding of libovf_cuda.so (the C ABI in include/ovf.h).

The library is loaded from this package directory only; there is no CPU
fallback.  Every call checks the returned ovf_status and raises the
exception type the reference throws for the same condition.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libovf_cuda.so")

OVF_OK = 0
OVF_EINVAL = -1
OVF_ENOMEM = -2
OVF_ECUDA = -3
OVF_ENCCL = -4
OVF_ETIMEDOUT = -5
OVF_ESTATE = -6
OVF_EUNSUPPORTED = -7
OVF_EBUSY = -8
OPT_PREFILL_SINGLE = 1
TP_HANDLE_BYTES = 64

TYPE_F32, TYPE_F16, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q6_K = 0, 1, 8, 12, 14
TENSORS_PER_LAYER = 14


class OverfitRuntimeError(RuntimeError):
    """Counterpart of the reference's OverfitRuntimeException."""


class OverfitCudaError(RuntimeError):
    """A CUDA/NCCL failure or a device-side bounded wait that gave up."""


class Tensor(C.Structure):
    _fields_ = [("type", C.c_int32), ("data", C.c_void_p), ("rows", C.c_int64), ("cols", C.c_int64)]


class ModelConfig(C.Structure):
    _fields_ = [("n_layers", C.c_int32), ("d_model", C.c_int32), ("n_heads", C.c_int32), ("n_kv_heads", C.c_int32),
                ("head_dim", C.c_int32), ("d_ff", C.c_int32), ("vocab", C.c_int32), ("rope_split_half", C.c_int32),
                ("n_experts", C.c_int32), ("n_experts_used", C.c_int32), ("normalize_experts", C.c_int32),
                ("eps", C.c_float), ("rope_theta", C.c_float)]


P, I32, I64, F = C.c_void_p, C.c_int32, C.c_int64, C.c_float

# name -> (restype, argtypes); the list is the contract of include/ovf.h and
# tests/test_abi.py checks that every declared symbol is exported.
SIGNATURES = {
    "ovf_last_error": (C.c_char_p, []),
    "ovf_version": (I32, []),
    "ovf_device_error": (I32, [I32, P]),
    "ovf_quantize_q8k": (I32, [P, I64, P, P, P, P]),
    "ovf_quantize_q8_0": (I32, [P, I64, P, P, P]),
    "ovf_kq_project": (I32, [I32, P, P, I64, I64, P, P, P, P, P, P]),
    "ovf_kq_project_prequantized": (I32, [I32, P, I64, I64, P, P, P, P, P, P]),
    "ovf_q4k_project_gate_up": (I32, [P, P, P, I64, I64, P, P, P, P, P, P]),
    "ovf_kq_project_batched": (I32, [I32, P, I64, P, I64, I64, P, P, P, P, P, P]),
    "ovf_tc_scratch_bytes": (I64, [I64, I64]),
    "ovf_kq_project_batched_tc": (I32, [I32, P, I64, P, I64, I64, P, P, P, P, P, P, P]),
    "ovf_q8_0_project": (I32, [P, P, P, I64, I64, P, P, P, P, P]),
    "ovf_q8_0_project_batched": (I32, [P, I64, P, P, I64, I64, P, P, P, P, P]),
    "ovf_q8_0_project_batched_tc": (I32, [P, I64, P, P, I64, I64, P, P, P, P, P, P]),
    "ovf_quantize_q4k": (I32, [P, I64, I64, P, P]),
    "ovf_quantize_q6k": (I32, [P, I64, I64, P, P]),
    "ovf_quantize_q8_0_gguf": (I32, [P, I64, P, P]),
    "ovf_q8_0_deinterleave": (I32, [P, I64, P, P, P]),
    "ovf_dequant_rows": (I32, [I32, P, P, I64, I64, I64, P, P]),
    "ovf_requant_q8_0": (I32, [I32, P, I64, I64, P, P, P]),
    "ovf_rmsnorm": (I32, [P, P, P, I64, F, P]),
    "ovf_rope_apply": (I32, [P, I32, I32, P, P, I32, P]),
    "ovf_exp_f32": (I32, [P, P, I64, P]),
    "ovf_swiglu": (I32, [P, P, P, I64, P]),
    "ovf_attention_scratch_bytes": (I64, [I32, I32, I32]),
    "ovf_attention_decode": (I32, [P, P, P, P, I32, I32, I32, I32, I32, F, P, P, P]),
    "ovf_attention_decode_noalloc": (I32, [P, P, P, P, I32, I32, I32, I32, I32, F, P]),
    "ovf_attention_single_head": (I32, [P, P, P, P, I32, I32, I32, I32, I32, F, P]),
    "ovf_attention_single_head_f16": (I32, [P, P, P, P, I32, I32, I32, I32, I32, F, P]),
    "ovf_attention_single_head_q8": (I32, [P, P, P, P, P, P, I32, I32, I32, I32, I32, F, P]),
    "ovf_model_create": (I32, [I32, P, P, I32, P]),
    "ovf_model_destroy": (I32, [P]),
    "ovf_model_weight_bytes": (I64, [P]),
    "ovf_session_create": (I32, [P, I32, P]),
    "ovf_session_create_kv": (I32, [P, I32, I32, P]),
    "ovf_session_destroy": (I32, [P]),
    "ovf_session_reset": (I32, [P]),
    "ovf_session_position": (I32, [P]),
    "ovf_session_decode": (I32, [P, I32, P, P]),
    "ovf_session_prefill": (I32, [P, P, I32, P, P]),
    "ovf_session_generate_greedy": (I32, [P, I32, P]),
    "ovf_session_stream": (P, [P]),
    "ovf_session_decode_batch": (I32, [P, I32, P, P, P]),
    "ovf_session_set_option": (I32, [P, I32, I32]),
    "ovf_model_create_tp": (I32, [I32, P, P, I32, I32, I32, P]),
    "ovf_model_tp_export": (I32, [P, P]),
    "ovf_model_tp_connect": (I32, [P, P]),
    "ovf_session_verify": (I32, [P, P, I32, P, P]),
    "ovf_session_truncate": (I32, [P, I32]),
    "ovf_session_prefix_bytes": (I64, [P]),
    "ovf_session_save_prefix": (I32, [P, P, P, P]),
    "ovf_session_restore_prefix": (I32, [P, P, P, I32]),
}

_lib = None


def load() -> C.CDLL:
    """Loads the in-tree library; raises if it was not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} is missing: build it with `python -m overfit_b200.build` "
                          "(there is no CPU fallback)")
        lib = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def last_error() -> str:
    msg = load().ovf_last_error()
    return msg.decode() if msg else ""


def check(status: int, what: str = "") -> None:
    if status == OVF_OK:
        return
    msg = f"{what}: {last_error()}" if what else last_error()
    if status == OVF_EINVAL:
        raise ValueError(msg)  # the reference's ArgumentException
    if status in (OVF_ESTATE, OVF_EBUSY):
        raise OverfitRuntimeError(msg)
    if status == OVF_ENOMEM:
        raise MemoryError(msg)
    if status == OVF_EUNSUPPORTED:
        raise NotImplementedError(msg)
    raise OverfitCudaError(f"status {status}: {msg}")
