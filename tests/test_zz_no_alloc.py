"""The allocation-free attention entry point (ovf_attention_decode_noalloc).

Some callers of this library cannot call cudaMalloc — a host whose device
memory belongs to one sanctioned allocator, or an allocation-free hot path —
so they cannot hand ovf_attention_decode its scratch buffer.  The no-alloc
variant keeps that scratch in a device array inside the library.  This test
calls it through the C ABI twice in a row (the array keeps the previous
call's contents, so the second call checks that it is reset properly) and
compares each result with ovf_attention_decode on a caller-owned buffer,
within the attention tolerance of tests/test_gpu_kernels.py.

It lives in a file of its own that pytest collects last.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from overfit_b200 import build, _lib
    build.build()
    return _lib


def _run_pair(L, H, KVH, hd, seq, seed):
    rng = np.random.default_rng(seed)
    max_ctx = seq + 3
    kc = torch.from_numpy(rng.normal(0, 1, (KVH, max_ctx, hd)).astype(np.float16)).cuda()
    vc = torch.from_numpy(rng.normal(0, 1, (KVH, max_ctx, hd)).astype(np.float16)).cuda()
    q = torch.from_numpy(rng.normal(0, 1, (H, hd)).astype(np.float32)).cuda()
    scale = float(1.0 / np.sqrt(hd))
    lib = L.load()
    stream = torch.cuda.current_stream().cuda_stream
    ref = torch.empty(H * hd, device="cuda")
    scratch = torch.empty(lib.ovf_attention_scratch_bytes(H, KVH, hd) // 4 + 1, device="cuda")
    counters = torch.zeros(KVH, dtype=torch.int32, device="cuda")
    L.check(lib.ovf_attention_decode(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), ref.data_ptr(), H, KVH, hd,
                                     max_ctx, seq, scale, scratch.data_ptr(), counters.data_ptr(), stream))
    got = torch.full((H * hd,), float("nan"), device="cuda")
    L.check(lib.ovf_attention_decode_noalloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), got.data_ptr(), H, KVH,
                                             hd, max_ctx, seq, scale, stream))
    torch.cuda.synchronize()
    r, g = ref.cpu().numpy().reshape(H, hd), got.cpu().numpy().reshape(H, hd)
    for h in range(H):
        rel = np.linalg.norm(g[h] - r[h]) / max(np.linalg.norm(r[h]), 1e-30)
        assert rel < 1e-5, (h, rel)


def test_noalloc_matches_caller_scratch_two_calls(lib):
    # Llama-3-8B attention layout, then a different layout on the same array.
    _run_pair(lib, 32, 8, 128, 2049, seed=1)
    _run_pair(lib, 14, 2, 64, 300, seed=2)


def test_noalloc_rejects_oversized_layout(lib):
    lib_ = lib.load()
    # 64 query heads on one KV head at head_dim 256 needs more than 1 MiB.
    assert lib_.ovf_attention_scratch_bytes(64, 1, 256) > (1 << 20)
    rc = lib_.ovf_attention_decode_noalloc(C.c_void_p(16), C.c_void_p(16), C.c_void_p(16), C.c_void_p(16), 64, 1,
                                           256, 8, 4, 1.0, None)
    assert rc == lib.OVF_EINVAL
    assert b"1048576" in lib_.ovf_last_error() or b"built-in buffer" in lib_.ovf_last_error()
