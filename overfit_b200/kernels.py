"""Host mirror of the reference's quantized kernel classes over device tensors.

Names, argument meaning and error behaviour follow the reference's static
kernel classes (paths relative to ``Sources/Main/LanguageModels/``):

* ``Q4KDotKernel``  — Runtime/Q4KDotKernel.cs
* ``Q6KDotKernel``  — Runtime/Q6KDotKernel.cs
* ``Q8DotKernel``   — Runtime/Q8DotKernel.cs
* ``GgmlQuant`` / ``GgmlDequant`` — Loading/GgmlQuant.cs, Loading/GgmlDequant.cs
* ``CachedAttentionKernel`` — Runtime/CachedAttentionKernel.cs

Buffers are torch CUDA tensors (torch is used for device memory and
streams only); every call goes through libovf_cuda.so and runs on the
current torch CUDA stream.  As in the reference the caller owns the
activation-quantization scratch; shape errors raise ``ValueError`` (the
reference's ArgumentException) before anything is launched.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from ._lib import TYPE_F32, TYPE_Q4_K, TYPE_Q6_K, TYPE_Q8_0, check

SUPER_BLOCK_ELEMENTS = 256
GROUP_SIZE = 16
Q8_BLOCK = 32
BLOCK_BYTES = {TYPE_Q4_K: 144, TYPE_Q6_K: 210}


def _ptr(t):
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _need(t, dtype, n, name):
    if t is None:
        raise ValueError(f"{name} is required")
    if not t.is_cuda or t.dtype != dtype or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous CUDA {dtype} tensor")
    if t.numel() < n:
        raise ValueError(f"{name} span is smaller than {n}")


@dataclass
class KQuantWeight:
    """Q4KWeight / Q6KWeight (Runtime/Q4KWeight.cs:23, Q6KWeight.cs:28):
    verbatim GGUF super-blocks, output-major, on the device."""

    blocks: torch.Tensor
    input_size: int
    output_size: int
    type: int = TYPE_Q4_K

    def __post_init__(self):
        if self.input_size % SUPER_BLOCK_ELEMENTS:
            raise ValueError(f"inputSize ({self.input_size}) must be a multiple of {SUPER_BLOCK_ELEMENTS}")
        need = self.output_size * (self.input_size // SUPER_BLOCK_ELEMENTS) * BLOCK_BYTES[self.type]
        _need(self.blocks, torch.uint8, need, "blocks")

    @property
    def super_blocks_per_row(self) -> int:
        return self.input_size // SUPER_BLOCK_ELEMENTS

    def decode_row(self, row: int, dst: torch.Tensor) -> None:
        """Q4KWeight.DecodeRow (Runtime/Q4KWeight.cs:122-140)."""
        if not 0 <= row < self.output_size:
            raise ValueError("row out of range")
        _need(dst, torch.float32, self.input_size, "dst")
        check(_lib.load().ovf_dequant_rows(self.type, _ptr(self.blocks), None, row, 1, self.input_size,
                                           _ptr(dst), _stream()), "DecodeRow")


def Q4KWeight(blocks, input_size, output_size) -> KQuantWeight:
    return KQuantWeight(blocks, input_size, output_size, TYPE_Q4_K)


def Q6KWeight(blocks, input_size, output_size) -> KQuantWeight:
    return KQuantWeight(blocks, input_size, output_size, TYPE_Q6_K)


@dataclass
class Q8Weight:
    """Runtime/Q8Weight.cs:21-60: int8 quants [out x in] + fp32 scales [out x in/32]."""

    quants: torch.Tensor
    scales: torch.Tensor
    input_size: int
    output_size: int

    def __post_init__(self):
        if self.input_size % Q8_BLOCK:
            raise ValueError(f"inputSize ({self.input_size}) must be a multiple of {Q8_BLOCK}")
        _need(self.quants, torch.int8, self.output_size * self.input_size, "quants")
        _need(self.scales, torch.float32, self.output_size * self.input_size // Q8_BLOCK, "scales")

    @staticmethod
    def from_gguf(gguf: torch.Tensor, input_size: int, output_size: int) -> "Q8Weight":
        """GgufReader.LoadTensorQ8_0Raw (Loading/GgufReader.cs:198-266)."""
        n = input_size * output_size
        _need(gguf, torch.uint8, n // 32 * 34, "gguf")
        q = torch.empty(n, dtype=torch.int8, device=gguf.device)
        s = torch.empty(n // 32, dtype=torch.float32, device=gguf.device)
        check(_lib.load().ovf_q8_0_deinterleave(_ptr(gguf), n, _ptr(q), _ptr(s), _stream()), "LoadTensorQ8_0Raw")
        return Q8Weight(q, s, input_size, output_size)

    @staticmethod
    def quantize_rows(w: torch.Tensor) -> "Q8Weight":
        """Q8Weight.QuantizeRows (Runtime/Q8Weight.cs:115-158), fp32 [rows x len]."""
        rows, length = w.shape
        w = w.contiguous()
        q = torch.empty(rows * length, dtype=torch.int8, device=w.device)
        s = torch.empty(rows * length // 32, dtype=torch.float32, device=w.device)
        check(_lib.load().ovf_requant_q8_0(TYPE_F32, _ptr(w), rows, length, _ptr(q), _ptr(s), _stream()),
              "QuantizeRows")
        return Q8Weight(q, s, length, rows)


class _KQuantKernel:
    TYPE = TYPE_Q4_K

    @staticmethod
    def quantize_activation_q8k(source, quants, block_scales, bsums) -> None:
        """QuantizeActivationQ8K (Runtime/Q4KDotKernel.cs:71-136)."""
        n = source.numel()
        if n % SUPER_BLOCK_ELEMENTS:
            raise ValueError(f"Source length ({n}) must be a multiple of {SUPER_BLOCK_ELEMENTS}.")
        _need(source, torch.float32, n, "source")
        _need(quants, torch.int8, n, "quants")
        _need(block_scales, torch.float32, n // 256, "blockScales")
        _need(bsums, torch.int16, n // 16, "bsums")
        check(_lib.load().ovf_quantize_q8k(_ptr(source), n, _ptr(quants), _ptr(block_scales), _ptr(bsums),
                                           _stream()), "QuantizeActivationQ8K")

    @classmethod
    def _check_weight(cls, weight):
        if not isinstance(weight, KQuantWeight) or weight.type != cls.TYPE:
            raise ValueError(f"weight must be a {'Q4_K' if cls.TYPE == TYPE_Q4_K else 'Q6_K'} weight")

    @classmethod
    def project_parallel(cls, input, weight, bias, output, activation_quants, activation_scales,
                         activation_bsums) -> None:
        """ProjectParallel (Runtime/Q4KDotKernel.cs:485-523; Q6KDotKernel.cs:314-352)."""
        cls._check_weight(weight)
        k, n = weight.input_size, weight.output_size
        _need(input, torch.float32, k, "input")
        _need(output, torch.float32, n, "output")
        if bias is not None:
            _need(bias, torch.float32, n, "bias")
        _need(activation_quants, torch.int8, k, "activationQuants")
        _need(activation_scales, torch.float32, k // 256, "activationScales")
        _need(activation_bsums, torch.int16, k // 16, "activationBsums")
        check(_lib.load().ovf_kq_project(cls.TYPE, _ptr(input), _ptr(weight.blocks), n, k, _ptr(bias), _ptr(output),
                                         _ptr(activation_quants), _ptr(activation_scales), _ptr(activation_bsums),
                                         _stream()), "ProjectParallel")

    project = project_parallel  # Project is the sequential twin; bit-identical

    @classmethod
    def project_pre_quantized(cls, weight, bias, output, activation_quants, activation_scales,
                              activation_bsums) -> None:
        """ProjectPreQuantized (Runtime/Q4KDotKernel.cs:445-476)."""
        cls._check_weight(weight)
        k, n = weight.input_size, weight.output_size
        _need(output, torch.float32, n, "output")
        if bias is not None:
            _need(bias, torch.float32, n, "bias")
        _need(activation_quants, torch.int8, k, "activationQuants")
        _need(activation_scales, torch.float32, k // 256, "activationScales")
        _need(activation_bsums, torch.int16, k // 16, "activationBsums")
        check(_lib.load().ovf_kq_project_prequantized(cls.TYPE, _ptr(weight.blocks), n, k, _ptr(bias), _ptr(output),
                                                      _ptr(activation_quants), _ptr(activation_scales),
                                                      _ptr(activation_bsums), _stream()), "ProjectPreQuantized")

    @classmethod
    def project_batched(cls, input, rows, weight, bias, output, activation_quants, activation_scales,
                        activation_bsums) -> None:
        """ProjectBatched / ProjectBatchedWeightStationary (Runtime/Q4KDotKernel.cs:663,819)."""
        cls._check_weight(weight)
        if rows <= 0:
            raise ValueError("rows must be positive")
        k, n = weight.input_size, weight.output_size
        _need(input, torch.float32, rows * k, "input")
        _need(output, torch.float32, rows * n, "output")
        _need(activation_quants, torch.int8, rows * k, "activationQuants")
        _need(activation_scales, torch.float32, rows * k // 256, "activationScales")
        _need(activation_bsums, torch.int16, rows * k // 16, "activationBsums")
        check(_lib.load().ovf_kq_project_batched(cls.TYPE, _ptr(input), rows, _ptr(weight.blocks), n, k, _ptr(bias),
                                                 _ptr(output), _ptr(activation_quants), _ptr(activation_scales),
                                                 _ptr(activation_bsums), _stream()), "ProjectBatched")

    project_batched_weight_stationary = project_batched


class Q4KDotKernel(_KQuantKernel):
    TYPE = TYPE_Q4_K

    @staticmethod
    def project_gate_up_parallel(input, gate, up, gate_output, up_output, activation_quants, activation_scales,
                                 activation_bsums) -> None:
        """ProjectGateUpParallel (Runtime/Q4KDotKernel.cs:563-645)."""
        for w in (gate, up):
            Q4KDotKernel._check_weight(w)
        if gate.input_size != up.input_size or gate.output_size != up.output_size:
            raise ValueError("gate and up must share input/output sizes")
        k, n = gate.input_size, gate.output_size
        _need(input, torch.float32, k, "input")
        _need(gate_output, torch.float32, n, "gateOutput")
        _need(up_output, torch.float32, n, "upOutput")
        check(_lib.load().ovf_q4k_project_gate_up(_ptr(input), _ptr(gate.blocks), _ptr(up.blocks), n, k,
                                                  _ptr(gate_output), _ptr(up_output), _ptr(activation_quants),
                                                  _ptr(activation_scales), _ptr(activation_bsums), _stream()),
              "ProjectGateUpParallel")


def _kq_tc(type_, input, rows, weight, bias, output, activation_quants, activation_scales, activation_bsums, scratch):
    k, n = weight.input_size, weight.output_size
    _need(input, torch.float32, rows * k, "input")
    _need(output, torch.float32, rows * n, "output")
    _need(activation_quants, torch.int8, rows * k, "activationQuants")
    _need(activation_scales, torch.float32, rows * k // 256, "activationScales")
    _need(activation_bsums, torch.int16, rows * k // 16, "activationBsums")
    _need(scratch, torch.uint8, tc_scratch_bytes(rows, k), "scratch")
    check(_lib.load().ovf_kq_project_batched_tc(type_, _ptr(input), rows, _ptr(weight.blocks), n, k, _ptr(bias),
                                                _ptr(output), _ptr(activation_quants), _ptr(activation_scales),
                                                _ptr(activation_bsums), _ptr(scratch), _stream()),
          "ProjectBatched (tensor cores)")


def tc_scratch_bytes(rows: int, k: int) -> int:
    """Packed-operand scratch of Q4KDotKernel.project_batched_tensor_cores."""
    return int(_lib.load().ovf_tc_scratch_bytes(rows, k))


def _q4k_tc(*args):
    _kq_tc(TYPE_Q4_K, *args)


def _q6k_tc(*args):
    _kq_tc(TYPE_Q6_K, *args)


Q4KDotKernel.project_batched_tensor_cores = staticmethod(_q4k_tc)


class Q6KDotKernel(_KQuantKernel):
    TYPE = TYPE_Q6_K


# ProjectBatched on the tensor cores (K a multiple of 2048); bit-identical to project_batched
Q6KDotKernel.project_batched_tensor_cores = staticmethod(_q6k_tc)


class Q8DotKernel:
    BLOCK_SIZE = Q8_BLOCK

    @staticmethod
    def quantize(source, quants, scales) -> None:
        """Quantize (Runtime/Q8DotKernel.cs:42-91)."""
        n = source.numel()
        if n % Q8_BLOCK:
            raise ValueError(f"Source length ({n}) must be a multiple of {Q8_BLOCK}.")
        _need(source, torch.float32, n, "source")
        _need(quants, torch.int8, n, "quants")
        _need(scales, torch.float32, n // 32, "scales")
        check(_lib.load().ovf_quantize_q8_0(_ptr(source), n, _ptr(quants), _ptr(scales), _stream()), "Quantize")

    @staticmethod
    def project_parallel(input, weight: Q8Weight, bias, output, input_quants, input_scales) -> None:
        """ProjectParallel (Runtime/Q8DotKernel.cs:252-328)."""
        k, n = weight.input_size, weight.output_size
        _need(input, torch.float32, k, "input")
        _need(output, torch.float32, n, "output")
        if bias is not None:
            _need(bias, torch.float32, n, "bias")
        _need(input_quants, torch.int8, k, "inputQuants")
        _need(input_scales, torch.float32, k // 32, "inputScales")
        check(_lib.load().ovf_q8_0_project(_ptr(input), _ptr(weight.quants), _ptr(weight.scales), n, k, _ptr(bias),
                                           _ptr(output), _ptr(input_quants), _ptr(input_scales), _stream()),
              "Q8 ProjectParallel")

    project = project_parallel

    @staticmethod
    def project_batched(input, rows, weight: Q8Weight, bias, output, input_quants, input_scales) -> None:
        """ProjectBatched (Runtime/Q8DotKernel.cs:352-445)."""
        k, n = weight.input_size, weight.output_size
        if rows <= 0:
            raise ValueError("rows must be positive")
        _need(input, torch.float32, rows * k, "input")
        _need(output, torch.float32, rows * n, "output")
        _need(input_quants, torch.int8, rows * k, "inputQuants")
        _need(input_scales, torch.float32, rows * k // 32, "inputScales")
        check(_lib.load().ovf_q8_0_project_batched(_ptr(input), rows, _ptr(weight.quants), _ptr(weight.scales), n, k,
                                                   _ptr(bias), _ptr(output), _ptr(input_quants), _ptr(input_scales),
                                                   _stream()), "Q8 ProjectBatched")

    @staticmethod
    def project_batched_tensor_cores(input, rows, weight: Q8Weight, bias, output, input_quants, input_scales,
                                     scratch) -> None:
        """ProjectBatched (Runtime/Q8DotKernel.cs:352-445) on the tensor cores:
        the same outputs as project_batched, bit for bit; K a multiple of 64,
        `scratch` uint8 of tc_scratch_bytes(rows, K)."""
        k, n = weight.input_size, weight.output_size
        if rows <= 0:
            raise ValueError("rows must be positive")
        _need(input, torch.float32, rows * k, "input")
        _need(output, torch.float32, rows * n, "output")
        _need(input_quants, torch.int8, rows * k, "inputQuants")
        _need(input_scales, torch.float32, rows * k // 32, "inputScales")
        _need(scratch, torch.uint8, tc_scratch_bytes(rows, k), "scratch")
        check(_lib.load().ovf_q8_0_project_batched_tc(_ptr(input), rows, _ptr(weight.quants), _ptr(weight.scales), n,
                                                      k, _ptr(bias), _ptr(output), _ptr(input_quants),
                                                      _ptr(input_scales), _ptr(scratch), _stream()),
              "Q8 ProjectBatched (tensor cores)")


class GgmlQuant:
    """Loading/GgmlQuant.cs plus the Q6_K / Q8_0 encoders the reference lacks."""

    @staticmethod
    def quantize_q4_k(f32: torch.Tensor, input_size: int, output_size: int) -> torch.Tensor:
        """QuantizeQ4_K (Loading/GgmlQuant.cs:141-161)."""
        if input_size % SUPER_BLOCK_ELEMENTS:
            raise ValueError(f"inputSize ({input_size}) must be a multiple of {SUPER_BLOCK_ELEMENTS}.")
        _need(f32, torch.float32, input_size * output_size, "f32")
        out = torch.empty(output_size * input_size // 256 * 144, dtype=torch.uint8, device=f32.device)
        check(_lib.load().ovf_quantize_q4k(_ptr(f32), output_size, input_size, _ptr(out), _stream()), "QuantizeQ4_K")
        return out

    @staticmethod
    def quantize_q6_k(f32: torch.Tensor, input_size: int, output_size: int) -> torch.Tensor:
        if input_size % SUPER_BLOCK_ELEMENTS:
            raise ValueError(f"inputSize ({input_size}) must be a multiple of {SUPER_BLOCK_ELEMENTS}.")
        _need(f32, torch.float32, input_size * output_size, "f32")
        out = torch.empty(output_size * input_size // 256 * 210, dtype=torch.uint8, device=f32.device)
        check(_lib.load().ovf_quantize_q6k(_ptr(f32), output_size, input_size, _ptr(out), _stream()), "Q6_K encode")
        return out

    @staticmethod
    def quantize_q8_0(f32: torch.Tensor) -> torch.Tensor:
        n = f32.numel()
        _need(f32, torch.float32, n, "f32")
        out = torch.empty(n // 32 * 34, dtype=torch.uint8, device=f32.device)
        check(_lib.load().ovf_quantize_q8_0_gguf(_ptr(f32), n, _ptr(out), _stream()), "Q8_0 encode")
        return out

    @staticmethod
    def requantize_q8_0(type_: int, data: torch.Tensor, rows: int, k: int) -> Q8Weight:
        """K-quant attn_output -> per-head Q8_0 (Loading/GgufLlamaLoader.cs:977-995,1298-1336)."""
        q = torch.empty(rows * k, dtype=torch.int8, device=data.device)
        s = torch.empty(rows * k // 32, dtype=torch.float32, device=data.device)
        check(_lib.load().ovf_requant_q8_0(type_, _ptr(data), rows, k, _ptr(q), _ptr(s), _stream()), "requant")
        return Q8Weight(q, s, k, rows)


class GgmlDequant:
    @staticmethod
    def dequantize_rows(type_: int, data: torch.Tensor, rows: int, k: int, scales=None, row0: int = 0):
        out = torch.empty(rows, k, dtype=torch.float32, device=data.device)
        check(_lib.load().ovf_dequant_rows(type_, _ptr(data), _ptr(scales), row0, rows, k, _ptr(out), _stream()),
              "dequantize")
        return out


def rms_normalize(input, gamma, output, eps) -> None:
    """RmsNormalize (Runtime/CachedTransformerBlock.cs:525-552)."""
    check(_lib.load().ovf_rmsnorm(_ptr(input), _ptr(gamma), _ptr(output), input.numel(), float(eps), _stream()),
          "RmsNormalize")


def exp(input: torch.Tensor, output: torch.Tensor) -> None:
    """MathF.Exp elementwise, with the host C library's expf bits."""
    check(_lib.load().ovf_exp_f32(_ptr(input), _ptr(output), input.numel(), _stream()), "MathF.Exp")


def apply_swiglu(gate: torch.Tensor, up: torch.Tensor, output: torch.Tensor) -> None:
    """ApplySiLU then Multiply (Runtime/CachedFeedForwardBlock.cs:464-472, :309):
    output = gate * sigmoid(gate) * up."""
    check(_lib.load().ovf_swiglu(_ptr(gate), _ptr(up), _ptr(output), gate.numel(), _stream()), "ApplySiLU")


def rope_apply(vectors: torch.Tensor, cos_row: torch.Tensor, sin_row: torch.Tensor, split_half: bool) -> None:
    """RopeKernel.Apply (Rope/RopeKernel.cs:46-93) on [n_vec x head_dim], in place."""
    n_vec, hd = vectors.shape
    check(_lib.load().ovf_rope_apply(_ptr(vectors), n_vec, hd, _ptr(cos_row), _ptr(sin_row), int(split_half),
                                     _stream()), "RopeKernel.Apply")


class CachedAttentionKernel:
    @staticmethod
    def scratch_bytes(n_heads, n_kv_heads, head_dim) -> int:
        return int(_lib.load().ovf_attention_scratch_bytes(n_heads, n_kv_heads, head_dim))

    @staticmethod
    def compute_single_head_all(query, k_cache, v_cache, output, n_heads, n_kv_heads, head_dim, seq_len,
                                scale) -> None:
        """ComputeSingleHead (Runtime/CachedAttentionKernel.cs:36-128) for every
        query head, over F32 caches [n_kv_heads, max_ctx, hd], in the
        reference's operation order (bit-identical)."""
        max_ctx = k_cache.shape[1]
        check(_lib.load().ovf_attention_single_head(_ptr(query), _ptr(k_cache), _ptr(v_cache), _ptr(output),
                                                    n_heads, n_kv_heads, head_dim, max_ctx, seq_len, float(scale),
                                                    _stream()), "ComputeSingleHead")

    @staticmethod
    def compute_single_head_f16_all(query, k_cache, v_cache, output, n_heads, n_kv_heads, head_dim, seq_len,
                                    scale) -> None:
        """ComputeSingleHead for every query head over fp16 caches
        [n_kv_heads, max_ctx, hd] (float16 tensors): the reference's order on
        the widened values (bit-identical)."""
        max_ctx = k_cache.shape[1]
        check(_lib.load().ovf_attention_single_head_f16(_ptr(query), _ptr(k_cache), _ptr(v_cache), _ptr(output),
                                                        n_heads, n_kv_heads, head_dim, max_ctx, seq_len, float(scale),
                                                        _stream()), "ComputeSingleHead")

    @staticmethod
    def compute_single_head_q8_all(query, k_q, k_scales, v_q, v_scales, output, n_heads, n_kv_heads, head_dim,
                                   seq_len, scale) -> None:
        """ComputeSingleHeadQ8 (Runtime/CachedAttentionKernel.cs:139-200) for
        every query head over a Q8 cache: int8 [n_kv_heads, max_ctx, hd] and
        fp32 scales [n_kv_heads, max_ctx], in the reference's order."""
        max_ctx = k_q.shape[1]
        check(_lib.load().ovf_attention_single_head_q8(_ptr(query), _ptr(k_q), _ptr(k_scales), _ptr(v_q),
                                                       _ptr(v_scales), _ptr(output), n_heads, n_kv_heads, head_dim,
                                                       max_ctx, seq_len, float(scale), _stream()),
              "ComputeSingleHeadQ8")

    @staticmethod
    def compute_all_heads(query, k_cache, v_cache, output, n_heads, n_kv_heads, head_dim, seq_len, scale,
                          scratch, counters) -> None:
        """ComputeSingleHead (Runtime/CachedAttentionKernel.cs:36-128) for every
        query head of a GQA layer.  k_cache/v_cache: fp16 [n_kv_heads, max_ctx, hd]."""
        max_ctx = k_cache.shape[1]
        check(_lib.load().ovf_attention_decode(_ptr(query), _ptr(k_cache), _ptr(v_cache), _ptr(output), n_heads,
                                               n_kv_heads, head_dim, max_ctx, seq_len, float(scale), _ptr(scratch),
                                               _ptr(counters), _stream()), "ComputeSingleHead")
