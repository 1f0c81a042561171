"""The C-ABI library loads without a GPU, exports every entry point that
include/ovf.h declares, and rejects bad arguments on the host before any
CUDA call (the reference's ArgumentException cases)."""
import ctypes as C
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def lib():
    from overfit_b200 import build
    build.build()
    from overfit_b200 import _lib
    return _lib.load()


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "ovf.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ovf_[a-z0-9_]+)\s*\(", src)))


def test_every_declared_symbol_is_exported(lib):
    names = declared_symbols()
    assert len(names) >= 30
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/ovf.h but not exported"


def test_binding_covers_header():
    from overfit_b200 import _lib
    assert set(declared_symbols()) == set(_lib.SIGNATURES), "ctypes signature table out of sync with include/ovf.h"


def test_version(lib):
    assert lib.ovf_version() == 10000


def test_argument_errors_without_gpu(lib):
    from overfit_b200 import _lib
    # QuantizeActivationQ8K: length not a multiple of 256
    assert lib.ovf_quantize_q8k(None, 100, None, None, None, None) == _lib.OVF_EINVAL
    assert b"multiple of 256" in lib.ovf_last_error()
    # Q8 Quantize: length not a multiple of 32
    assert lib.ovf_quantize_q8_0(None, 33, None, None, None) == _lib.OVF_EINVAL
    # projection: not a K-quant type / bad K / unaligned weight
    assert lib.ovf_kq_project(8, None, None, 4, 256, None, None, None, None, None, None) == _lib.OVF_EINVAL
    assert lib.ovf_kq_project(12, None, None, 4, 300, None, None, None, None, None, None) == _lib.OVF_EINVAL
    assert lib.ovf_kq_project(12, None, C.c_void_p(17), 4, 256, None, None, None, None, None, None) == _lib.OVF_EINVAL
    assert lib.ovf_q8_0_project(None, None, None, 4, 48, None, None, None, None, None) == _lib.OVF_EINVAL
    assert lib.ovf_dequant_rows(3, None, None, 0, 1, 256, None, None) == _lib.OVF_EINVAL
    assert lib.ovf_rope_apply(None, 1, 63, None, None, 0, None) == _lib.OVF_EINVAL
    assert lib.ovf_model_create(0, None, None, 0, None) == _lib.OVF_EINVAL
    assert lib.ovf_session_decode(None, 0, None, None) == _lib.OVF_EINVAL
    assert lib.ovf_attention_scratch_bytes(32, 8, 128) > 0
    # ComputeSingleHead on F32 caches: null buffers, seq_len outside [1, max_ctx]
    assert lib.ovf_attention_single_head(None, None, None, None, 32, 8, 128, 64, 8, 1.0, None) == _lib.OVF_EINVAL
    p16 = C.c_void_p(16)
    assert lib.ovf_attention_single_head(p16, p16, p16, p16, 32, 8, 128, 64, 65, 1.0, None) == _lib.OVF_EINVAL
    assert lib.ovf_attention_single_head(p16, p16, p16, p16, 32, 8, 128, 64, 0, 1.0, None) == _lib.OVF_EINVAL
    # unsupported head_dim / heads not a multiple of the KV heads
    assert lib.ovf_attention_single_head(p16, p16, p16, p16, 32, 8, 96, 64, 8, 1.0, None) == _lib.OVF_EINVAL
    assert lib.ovf_attention_single_head(p16, p16, p16, p16, 30, 8, 128, 64, 8, 1.0, None) == _lib.OVF_EINVAL
    # sessions: null model / unknown KV dtype
    out = C.c_void_p()
    assert lib.ovf_session_create_kv(None, 64, 0, C.byref(out)) == _lib.OVF_EINVAL
    # RMSNorm and the projections reject null buffers on the host
    assert lib.ovf_q4k_project_gate_up(None, None, None, 4, 256, None, None, None, None, None, None) == _lib.OVF_EINVAL
    # ProjectBatched / ProjectBatchedWeightStationary: rows must be positive,
    # buffers non-null and 16-byte aligned (before any device work)
    p16 = C.c_void_p(16)
    assert lib.ovf_kq_project_batched(12, p16, 0, p16, 4, 256, None, p16, p16, p16, p16, None) == _lib.OVF_EINVAL
    assert lib.ovf_kq_project_batched(12, None, 2, p16, 4, 256, None, p16, p16, p16, p16, None) == _lib.OVF_EINVAL
    assert lib.ovf_kq_project_batched(12, C.c_void_p(20), 2, p16, 4, 256, None, p16, p16, p16, p16,
                                      None) == _lib.OVF_EINVAL
    assert b"aligned" in lib.ovf_last_error()
    assert lib.ovf_q8_0_project_batched(p16, 0, p16, p16, 4, 64, None, p16, p16, p16, None) == _lib.OVF_EINVAL
    assert lib.ovf_q8_0_project_batched(p16, 2, p16, p16, 4, 48, None, p16, p16, p16, None) == _lib.OVF_EINVAL
    assert lib.ovf_q8_0_project_batched(p16, 2, C.c_void_p(8), p16, 4, 64, None, p16, p16, p16,
                                        None) == _lib.OVF_EINVAL


def test_python_mirror_raises_value_error():
    from overfit_b200 import _lib
    with pytest.raises(ValueError):
        _lib.check(_lib.OVF_EINVAL, "x")
    with pytest.raises(_lib.OverfitRuntimeError):
        _lib.check(_lib.OVF_ESTATE, "x")


def test_tensor_core_projection_host_checks():
    """Scratch sizes and argument checks of the tensor-core projections run on
    the host (no device work): one scratch size covers Q4_K, Q6_K and Q8_0,
    unsupported shapes and types are rejected before any launch."""
    from overfit_b200 import _lib
    lib = _lib.load()
    for rows in (1, 63, 64, 65, 2048):
        for k in (4096, 14336):
            mt = -(-rows // 64)
            got = lib.ovf_tc_scratch_bytes(rows, k)
            assert got >= mt * 64 * k * 2 + mt * (k // 256) * (2048 + 256)  # fp16 tiles, bsum16 tiles, scales
            assert got >= mt * 64 * k + mt * (k // 32) * 64 * 4             # int8 tiles, block scales
    assert lib.ovf_tc_scratch_bytes(16, 896) > 0       # Q8_0 widths (multiples of 64)
    assert lib.ovf_tc_scratch_bytes(16, 100) == 0
    assert lib.ovf_tc_scratch_bytes(0, 4096) == 0
    p16 = C.c_void_p(16)
    # Q8_0 as a K-quant, Q6_K with k not a multiple of 2048, rows out of range, null scratch
    assert lib.ovf_kq_project_batched_tc(8, p16, 4, p16, 4, 4096, None, p16, p16, p16, p16, p16, None) == _lib.OVF_EINVAL
    assert lib.ovf_kq_project_batched_tc(14, p16, 4, p16, 4, 1024, None, p16, p16, p16, p16, p16, None) == _lib.OVF_EINVAL
    assert lib.ovf_kq_project_batched_tc(12, p16, 0, p16, 4, 4096, None, p16, p16, p16, p16, p16, None) == _lib.OVF_EINVAL
    assert lib.ovf_kq_project_batched_tc(12, p16, 4, p16, 4, 4096, None, p16, p16, p16, p16, None, None) == _lib.OVF_EINVAL
    assert lib.ovf_q8_0_project_batched_tc(p16, 4, p16, p16, 4, 96, None, p16, p16, p16, p16, None) == _lib.OVF_EINVAL
    assert lib.ovf_q8_0_project_batched_tc(p16, 4, C.c_void_p(8), p16, 4, 128, None, p16, p16, p16, p16,
                                           None) == _lib.OVF_EINVAL
