"""Kernel-level parity on the GPU, through the C ABI, against the CPU
restatement of the reference (oracle/).

Integer/byte work and the GEMV tails are required to be BIT-EXACT (the
reference's fp32 operation order is reproduced); RMSNorm and attention use
tolerances (their sums are reordered / use the device exp), stated per test.
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def K():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from overfit_b200 import build, kernels
    build.build()
    return kernels


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


# ------------------------------------------------------------- quantizers
@pytest.mark.parametrize("k", [256, 4096, 14336])
def test_quantize_q8k_bit_exact(K, orc, k):
    rng = np.random.default_rng(k)
    x = rng.normal(0, 1, k).astype(np.float32)
    x[:256] = 0.0  # an all-zero block (Q4KDotKernelTests.cs:199-216)
    q, s, b = (torch.empty(k, dtype=torch.int8, device="cuda"), torch.empty(k // 256, device="cuda"),
               torch.empty(k // 16, dtype=torch.int16, device="cuda"))
    K.Q4KDotKernel.quantize_activation_q8k(dev(x), q, s, b)
    rq, rs, rb = orc.quantize_q8k(x)
    np.testing.assert_array_equal(host(q), rq)
    np.testing.assert_array_equal(host(s), rs)
    np.testing.assert_array_equal(host(b), rb)


def test_quantize_q8k_half_way_ties(K, orc):
    """Values that land exactly on .5 steps: round half to even like MathF.Round."""
    x = np.zeros(256, np.float32)
    x[0] = 127.0
    x[1:40] = np.arange(39, dtype=np.float32) + 0.5
    q, s, b = (torch.empty(256, dtype=torch.int8, device="cuda"), torch.empty(1, device="cuda"),
               torch.empty(16, dtype=torch.int16, device="cuda"))
    K.Q4KDotKernel.quantize_activation_q8k(dev(x), q, s, b)
    np.testing.assert_array_equal(host(q), orc.quantize_q8k(x)[0])


@pytest.mark.parametrize("k", [32, 896, 4864])
def test_quantize_q8_0_bit_exact(K, orc, k):
    x = np.random.default_rng(k).normal(0, 1, k).astype(np.float32)
    q, s = torch.empty(k, dtype=torch.int8, device="cuda"), torch.empty(k // 32, device="cuda")
    K.Q8DotKernel.quantize(dev(x), q, s)
    rq, rs = orc.quantize_q8_0(x)
    np.testing.assert_array_equal(host(q), rq)
    np.testing.assert_array_equal(host(s), rs)


# ------------------------------------------------------------------ codecs
@pytest.mark.parametrize("rows,k", [(8, 512), (64, 4096)])
def test_encoders_bit_exact(K, orc, rows, k):
    w = np.random.default_rng(rows).normal(0, 0.02, (rows, k)).astype(np.float32)
    w[0, :256] = 0.37  # constant super-block (GgmlQuantTests.cs:86-107)
    w[1, :32] = 0.0
    np.testing.assert_array_equal(host(K.GgmlQuant.quantize_q4_k(dev(w), k, rows)), orc.quantize_q4k(w))
    np.testing.assert_array_equal(host(K.GgmlQuant.quantize_q6_k(dev(w), k, rows)), orc.quantize_q6k(w))
    np.testing.assert_array_equal(host(K.GgmlQuant.quantize_q8_0(dev(w))), orc.quantize_q8_0_gguf(w))


def test_decoders_and_requant_bit_exact(K, orc):
    rng = np.random.default_rng(3)
    rows, k = 16, 768
    w = rng.normal(0, 0.02, (rows, k)).astype(np.float32)
    for t, enc in ((orc.Q4_K, orc.quantize_q4k), (orc.Q6_K, orc.quantize_q6k)):
        b = enc(w)
        got = host(K.GgmlDequant.dequantize_rows(t, dev(b), rows - 3, k, row0=3))
        np.testing.assert_array_equal(got, orc.dequant_rows(t, b, rows - 3, k, row0=3))
        qw = K.GgmlQuant.requantize_q8_0(t, dev(b), rows, k)
        rq, rs = orc.requant_q8_0(t, b, rows, k)
        np.testing.assert_array_equal(host(qw.quants), rq)
        np.testing.assert_array_equal(host(qw.scales), rs)
    g = orc.quantize_q8_0_gguf(w)
    w8 = K.Q8Weight.from_gguf(dev(g), k, rows)
    rq, rs = orc.q8_0_deinterleave(g, rows * k)
    np.testing.assert_array_equal(host(w8.quants), rq)
    np.testing.assert_array_equal(host(w8.scales), rs)


def test_known_answer_blocks_on_gpu(K):
    """The reference's hand-built decode cases (GgmlDequantTests.cs) through the device decoder."""
    import json
    cases = json.load(open(os.path.join(GOLDEN, "known_answers.json")))["cases"]
    for c in cases:
        if c["kind"] in ("decode_q4k", "decode_q6k"):
            t = 12 if c["kind"] == "decode_q4k" else 14
            got = host(K.GgmlDequant.dequantize_rows(t, dev(np.array(c["block"], np.uint8)), 1, 256))[0]
            np.testing.assert_allclose(got, c["expected"], atol=c["abs_tol"], err_msg=c["ref"])


# -------------------------------------------------------------- projections
def _act_scratch(k):
    return (torch.empty(k, dtype=torch.int8, device="cuda"), torch.empty(k // 256, device="cuda"),
            torch.empty(k // 16, dtype=torch.int16, device="cuda"))


@pytest.mark.parametrize("typ,n,k,with_bias", [
    ("q4k", 96, 512, True), ("q4k", 97, 768, False), ("q4k", 4096, 4096, False), ("q4k", 14336, 4096, False),
    ("q4k", 4096, 14336, True), ("q6k", 64, 768, True), ("q6k", 1024, 4096, False), ("q6k", 4096, 14336, False),
    ("q6k", 131, 2560, False), ("q6k", 3, 256, False)])
def test_kq_project_bit_exact(K, orc, typ, n, k, with_bias):
    rng = np.random.default_rng(n * 7 + k)
    w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    x = rng.normal(0, 1, k).astype(np.float32)
    bias = rng.normal(0, 0.1, n).astype(np.float32) if with_bias else None
    t = orc.Q4_K if typ == "q4k" else orc.Q6_K
    wb = orc.quantize_q4k(w) if typ == "q4k" else orc.quantize_q6k(w)
    ref = orc.kq_project(t, x, wb, n, k, bias)
    weight = K.KQuantWeight(dev(wb), k, n, t)
    y = torch.empty(n, device="cuda")
    q, s, b = _act_scratch(k)
    kern = K.Q4KDotKernel if typ == "q4k" else K.Q6KDotKernel
    kern.project_parallel(dev(x), weight, None if bias is None else dev(bias), y, q, s, b)
    np.testing.assert_array_equal(host(y), ref)
    # the caller's scratch holds the Q8_K activation, as in the reference
    rq, rs, rb = orc.quantize_q8k(x)
    np.testing.assert_array_equal(host(q), rq)
    np.testing.assert_array_equal(host(b), rb)
    # pre-quantized entry point on the same scratch
    y2 = torch.empty(n, device="cuda")
    kern.project_pre_quantized(weight, None if bias is None else dev(bias), y2, q, s, b)
    np.testing.assert_array_equal(host(y2), ref)


def test_golden_fixture_projections(K):
    """Committed expectations (tests/golden/parity_small.npz) — no oracle needed."""
    z = np.load(os.path.join(GOLDEN, "parity_small.npz"))
    y = torch.empty(96, device="cuda")
    q, s, b = _act_scratch(512)
    K.Q4KDotKernel.project_parallel(dev(z["q4k_x"]), K.Q4KWeight(dev(z["q4k_w"]), 512, 96), dev(z["q4k_bias"]), y,
                                    q, s, b)
    np.testing.assert_array_equal(host(y), z["q4k_y"])
    y = torch.empty(64, device="cuda")
    q, s, b = _act_scratch(768)
    K.Q6KDotKernel.project_parallel(dev(z["q6k_x"]), K.Q6KWeight(dev(z["q6k_w"]), 768, 64), None, y, q, s, b)
    np.testing.assert_array_equal(host(y), z["q6k_y"])
    w8 = K.Q8Weight.from_gguf(dev(z["q8_gguf"]), 352, 80)
    y = torch.empty(80, device="cuda")
    K.Q8DotKernel.project_parallel(dev(z["q8_x"]), w8, None, y, torch.empty(352, dtype=torch.int8, device="cuda"),
                                   torch.empty(11, device="cuda"))
    np.testing.assert_array_equal(host(y), z["q8_y"])


def test_gate_up_bit_exact(K, orc):
    rng = np.random.default_rng(5)
    n, k = 1000, 1024
    wg, wu = (rng.normal(0, 0.02, (n, k)).astype(np.float32) for _ in range(2))
    x = rng.normal(0, 1, k).astype(np.float32)
    bg, bu = orc.quantize_q4k(wg), orc.quantize_q4k(wu)
    g, u = torch.empty(n, device="cuda"), torch.empty(n, device="cuda")
    q, s, b = _act_scratch(k)
    K.Q4KDotKernel.project_gate_up_parallel(dev(x), K.Q4KWeight(dev(bg), k, n), K.Q4KWeight(dev(bu), k, n), g, u,
                                            q, s, b)
    np.testing.assert_array_equal(host(g), orc.kq_project(orc.Q4_K, x, bg, n, k))
    np.testing.assert_array_equal(host(u), orc.kq_project(orc.Q4_K, x, bu, n, k))


@pytest.mark.parametrize("rows", [1, 3, 16])
def test_batched_bit_exact(K, orc, rows):
    """ProjectBatched == per-row Project, bit for bit (Q4KDotKernelTests.cs:96-136)."""
    rng = np.random.default_rng(rows)
    n, k = 96, 512
    w = orc.quantize_q4k(rng.normal(0, 0.02, (n, k)).astype(np.float32))
    x = rng.uniform(-1, 1, (rows, k)).astype(np.float32)
    bias = rng.uniform(-1, 1, n).astype(np.float32)
    y = torch.empty(rows * n, device="cuda")
    q = torch.empty(rows * k, dtype=torch.int8, device="cuda")
    s = torch.empty(rows * k // 256, device="cuda")
    b = torch.empty(rows * k // 16, dtype=torch.int16, device="cuda")
    K.Q4KDotKernel.project_batched(dev(x), rows, K.Q4KWeight(dev(w), k, n), dev(bias), y, q, s, b)
    np.testing.assert_array_equal(host(y).reshape(rows, n), orc.kq_project_batched(orc.Q4_K, x, w, n, k, bias))


@pytest.mark.parametrize("type_name,rows,n,k,with_bias", [
    ("Q4_K", 5, 33, 1280, True),      # ragged: 5 activation rows, 33 weight rows, 5 super-blocks (partial chunk)
    ("Q6_K", 9, 70, 768, False),      # Q6_K rows start 2 bytes past a 16-byte boundary
    ("Q6_K", 17, 31, 4096, True),
    ("Q4_K", 64, 14336, 4096, False),  # prefill GEMM shape (gate/up, M = 64)
    ("Q6_K", 24, 4096, 14336, False),  # down projection shape
])
def test_weight_stationary_kq_bit_exact(K, orc, type_name, rows, n, k, with_bias):
    """ProjectBatchedWeightStationary over ragged tiles: every row equal to
    the restatement's per-row projection, and the scratch holds each row's
    own Q8_K activation (Q4KDotKernelTests.cs:96-136)."""
    t = getattr(orc, type_name)
    rng = np.random.default_rng(rows * 7 + n)
    wf = orc.fill_normal(n * k, rows + 3, 0.0, 0.02).reshape(n, k)
    w = orc.quantize_q4k(wf) if type_name == "Q4_K" else orc.quantize_q6k(wf)
    x = rng.normal(0, 1, (rows, k)).astype(np.float32)
    x[0, :256] = 0.0  # an all-zero activation block
    bias = rng.uniform(-1, 1, n).astype(np.float32) if with_bias else None
    y = torch.empty(rows * n, device="cuda")
    q = torch.empty(rows * k, dtype=torch.int8, device="cuda")
    s = torch.empty(rows * k // 256, device="cuda")
    b = torch.empty(rows * k // 16, dtype=torch.int16, device="cuda")
    cls = K.Q4KDotKernel if type_name == "Q4_K" else K.Q6KDotKernel
    cls.project_batched(dev(x), rows, K.KQuantWeight(dev(w), k, n, t), None if bias is None else dev(bias), y, q, s, b)
    np.testing.assert_array_equal(host(y).reshape(rows, n), orc.kq_project_batched(t, x, w, n, k, bias))
    rq, rs, rb = orc.quantize_q8k(x.reshape(-1))
    np.testing.assert_array_equal(host(q), rq)
    np.testing.assert_array_equal(host(s), rs)
    np.testing.assert_array_equal(host(b), rb)


@pytest.mark.parametrize("rows,n,k,with_bias", [(1, 80, 352, True), (11, 45, 1056, False), (16, 896, 4864, True),
                                                (40, 4864, 896, False)])
def test_q8_project_batched_bit_exact(K, orc, rows, n, k, with_bias):
    """Q8DotKernel.ProjectBatched: ragged row/activation tiles and a partial
    32-block chunk (k = 1056 = 33 blocks), bit-exact to the restatement."""
    rng = np.random.default_rng(rows + n + k)
    w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    x = rng.normal(0, 1, (rows, k)).astype(np.float32)
    bias = rng.normal(0, 0.1, n).astype(np.float32) if with_bias else None
    g = orc.quantize_q8_0_gguf(w)
    rq, rs = orc.q8_0_deinterleave(g, n * k)
    ref = orc.q8_0_project_batched(x, rq, rs, n, k, bias)
    w8 = K.Q8Weight.from_gguf(dev(g), k, n)
    y = torch.empty(rows * n, device="cuda")
    xq, xs = torch.empty(rows * k, dtype=torch.int8, device="cuda"), torch.empty(rows * k // 32, device="cuda")
    K.Q8DotKernel.project_batched(dev(x), rows, w8, None if bias is None else dev(bias), y, xq, xs)
    np.testing.assert_array_equal(host(y).reshape(rows, n), ref)


@pytest.mark.parametrize("n,k,with_bias", [(80, 352, True), (896, 896, False), (4864, 896, False),
                                           (896, 4864, True), (4096, 4096, False), (151936 // 64, 896, False)])
def test_q8_project_bit_exact(K, orc, n, k, with_bias):
    rng = np.random.default_rng(n + k)
    w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    x = rng.normal(0, 1, k).astype(np.float32)
    bias = rng.normal(0, 0.1, n).astype(np.float32) if with_bias else None
    g = orc.quantize_q8_0_gguf(w)
    rq, rs = orc.q8_0_deinterleave(g, n * k)
    ref = orc.q8_0_project(x, rq, rs, n, k, bias)
    w8 = K.Q8Weight.from_gguf(dev(g), k, n)
    y = torch.empty(n, device="cuda")
    xq, xs = torch.empty(k, dtype=torch.int8, device="cuda"), torch.empty(k // 32, device="cuda")
    K.Q8DotKernel.project_parallel(dev(x), w8, None if bias is None else dev(bias), y, xq, xs)
    np.testing.assert_array_equal(host(y), ref)


def test_argument_errors_raise(K):
    w = K.Q4KWeight(torch.zeros(144 * 4, dtype=torch.uint8, device="cuda"), 256, 4)
    y = torch.empty(4, device="cuda")
    q, s, b = _act_scratch(256)
    with pytest.raises(ValueError):
        K.Q4KDotKernel.project_parallel(torch.zeros(100, device="cuda"), w, None, y, q, s, b)
    with pytest.raises(ValueError):
        K.Q6KDotKernel.project_parallel(torch.zeros(256, device="cuda"), w, None, y, q, s, b)
    with pytest.raises(ValueError):
        K.KQuantWeight(torch.zeros(10, dtype=torch.uint8, device="cuda"), 300, 1)


# ------------------------------------------------------------------- small ops
@pytest.mark.parametrize("d", [896, 4096, 14336])
def test_rmsnorm_bit_exact(K, orc, d):
    """RmsNormalize with the reference's sequential sum of squares: bit-exact."""
    x = np.random.default_rng(9 + d).normal(0, 3, d).astype(np.float32)
    gmm = np.random.default_rng(10 + d).normal(1, 0.1, d).astype(np.float32)
    y = torch.empty(d, device="cuda")
    K.rms_normalize(dev(x), dev(gmm), y, 1e-6)
    np.testing.assert_array_equal(host(y), orc.rmsnorm(x, gmm, 1e-6))


def test_lm_head_full_size_bit_exact(K, orc):
    """The largest projection of the benchmark step at its full size: the
    Llama-3-8B Q6_K output head, 128256 x 4096, against the restatement."""
    n, k = 128256, 4096
    w = orc.fill_normal(n * k, 77, 0.0, 0.02).reshape(n, k)
    wb = orc.quantize_q6k(w)
    del w
    x = np.random.default_rng(78).normal(0, 1, k).astype(np.float32)
    ref = orc.kq_project(orc.Q6_K, x, wb, n, k)
    y = torch.empty(n, device="cuda")
    q, s, b = _act_scratch(k)
    K.Q6KDotKernel.project_parallel(dev(x), K.KQuantWeight(dev(wb), k, n, orc.Q6_K), None, y, q, s, b)
    np.testing.assert_array_equal(host(y), ref)


@pytest.mark.parametrize("split_half", [0, 1])
def test_rope_bit_exact(K, orc, split_half):
    c, s = orc.rope_table(64, 128, 500000.0)
    v = np.random.default_rng(2).normal(size=(6, 128)).astype(np.float32)
    t = dev(v)
    K.rope_apply(t, dev(c[37]), dev(s[37]), bool(split_half))
    ref = np.stack([orc.rope_apply(v[i], c[37], s[37], split_half) for i in range(6)])
    np.testing.assert_array_equal(host(t), ref)


@pytest.mark.parametrize("H,KVH,hd,seq", [(32, 8, 128, 1), (32, 8, 128, 2049), (14, 2, 64, 300), (4, 4, 32, 7),
                                          (8, 2, 256, 33)])
def test_attention_exact_f32(K, orc, H, KVH, hd, seq):
    """F32-cache attention in the reference's order vs the restated
    ComputeSingleHead: bit-identical (the device exp has the host expf's bits)."""
    rng = np.random.default_rng(seq + hd)
    max_ctx = seq + 5
    kc = rng.normal(0, 1, (KVH, max_ctx, hd)).astype(np.float32)
    vc = rng.normal(0, 1, (KVH, max_ctx, hd)).astype(np.float32)
    q = rng.normal(0, 1, (H, hd)).astype(np.float32)
    scale = np.float32(1.0 / np.sqrt(hd))
    out = torch.empty(H * hd, device="cuda")
    K.CachedAttentionKernel.compute_single_head_all(dev(q), dev(kc), dev(vc), out, H, KVH, hd, seq, scale)
    got = host(out).reshape(H, hd)
    ref = np.stack([orc.attention_single_head(q[h], kc[h // (H // KVH), :seq], vc[h // (H // KVH), :seq], scale)
                    for h in range(H)])
    np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("H,KVH,hd,seq", [(32, 8, 128, 1), (32, 8, 128, 2049), (14, 2, 64, 300), (4, 4, 32, 7),
                                          (8, 2, 256, 33)])
def test_attention_exact_f16_cache(K, orc, H, KVH, hd, seq):
    """fp16-cache attention: the reference's ComputeSingleHead order on the
    widened fp16 values, bit-identical to the restatement run on the same
    (rounded) values."""
    rng = np.random.default_rng(seq + 7 * hd)
    max_ctx = seq + 3
    kc = rng.normal(0, 1, (KVH, max_ctx, hd)).astype(np.float16)
    vc = rng.normal(0, 1, (KVH, max_ctx, hd)).astype(np.float16)
    q = rng.normal(0, 1, (H, hd)).astype(np.float32)
    scale = np.float32(1.0 / np.sqrt(hd))
    out = torch.empty(H * hd, device="cuda")
    K.CachedAttentionKernel.compute_single_head_f16_all(dev(q), dev(kc), dev(vc), out, H, KVH, hd, seq, scale)
    got = host(out).reshape(H, hd)
    kf, vf = kc.astype(np.float32), vc.astype(np.float32)
    ref = np.stack([orc.attention_single_head(q[h], kf[h // (H // KVH), :seq], vf[h // (H // KVH), :seq], scale)
                    for h in range(H)])
    np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("H,KVH,hd,seq", [(32, 8, 128, 1), (32, 8, 128, 2049), (14, 2, 64, 300), (7, 1, 32, 20),
                                          (8, 2, 256, 33)])
def test_attention_q8_cache_bit_exact(K, orc, H, KVH, hd, seq):
    """Q8 KV cache (Q8KvQuant vectors) attended in ComputeSingleHeadQ8's order
    vs the restatement: bit-identical."""
    rng = np.random.default_rng(seq * 3 + hd)
    max_ctx = seq + 5
    kf = rng.normal(0, 1, (KVH, max_ctx, hd)).astype(np.float32)
    vf = rng.normal(0, 1, (KVH, max_ctx, hd)).astype(np.float32)
    kq = np.zeros((KVH, max_ctx, hd), np.int8); vq = np.zeros((KVH, max_ctx, hd), np.int8)
    ks = np.zeros((KVH, max_ctx), np.float32); vs = np.zeros((KVH, max_ctx), np.float32)
    for g in range(KVH):
        for t in range(max_ctx):
            kq[g, t], ks[g, t] = orc.q8kv_quantize(kf[g, t])
            vq[g, t], vs[g, t] = orc.q8kv_quantize(vf[g, t])
    q = rng.normal(0, 1, (H, hd)).astype(np.float32)
    scale = np.float32(1.0 / np.sqrt(hd))
    out = torch.empty(H * hd, device="cuda")
    K.CachedAttentionKernel.compute_single_head_q8_all(dev(q), dev(kq), dev(ks), dev(vq), dev(vs), out, H, KVH, hd,
                                                       seq, scale)
    got = host(out).reshape(H, hd)
    G = H // KVH
    ref = np.stack([orc.attention_single_head_q8(q[h], kq[h // G, :seq], ks[h // G, :seq], vq[h // G, :seq],
                                                 vs[h // G, :seq], scale) for h in range(H)])
    np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("H,KVH,hd,seq", [(32, 8, 128, 1), (32, 8, 128, 2049), (14, 2, 64, 300), (4, 4, 32, 7)])
def test_attention_close(K, orc, H, KVH, hd, seq):
    """Split-K flash-decode vs the reference's single-head loop on the same
    fp16-representable cache: rel L2 < 1e-5 per head (fp32 everywhere, only
    the exp and the summation order differ)."""
    rng = np.random.default_rng(seq)
    max_ctx = seq + 5
    kc = rng.normal(0, 1, (KVH, max_ctx, hd)).astype(np.float16)
    vc = rng.normal(0, 1, (KVH, max_ctx, hd)).astype(np.float16)
    q = rng.normal(0, 1, (H, hd)).astype(np.float32)
    scale = 1.0 / np.sqrt(hd)
    out = torch.empty(H * hd, device="cuda")
    scratch = torch.empty(K.CachedAttentionKernel.scratch_bytes(H, KVH, hd) // 4 + 1, device="cuda")
    counters = torch.zeros(KVH, dtype=torch.int32, device="cuda")
    K.CachedAttentionKernel.compute_all_heads(dev(q), dev(kc), dev(vc), out, H, KVH, hd, seq, scale, scratch,
                                              counters)
    got = host(out).reshape(H, hd)
    for h in range(H):
        g = h // (H // KVH)
        ref = orc.attention_single_head(q[h], kc[g, :seq].astype(np.float32), vc[g, :seq].astype(np.float32), scale)
        rel = np.linalg.norm(got[h] - ref) / max(np.linalg.norm(ref), 1e-30)
        assert rel < 1e-5, (h, rel)
    assert not host(counters).any()  # counters are left zero for the next call


# ------------------------------------------------------------ exp and SiLU
def test_exp_matches_host_expf_exhaustively(K, orc):
    """The device exp against the host C library's expf (MathF.Exp) on every
    float32 bit pattern: identical bits, NaNs compared as NaN."""
    chunk = 1 << 28
    x = torch.empty(chunk, dtype=torch.float32, device="cuda")
    y = torch.empty_like(x)
    for c in range(1 << 32 >> 28):
        bits = torch.arange(c * chunk, (c + 1) * chunk, dtype=torch.int64, device="cuda")
        x.copy_((bits - (bits >= (1 << 31)).to(torch.int64) * (1 << 32)).to(torch.int32).view(torch.float32))
        del bits
        K.exp(x, y)
        xh = host(x)
        got = host(y).view(np.uint32)
        ref = orc.expf_array(xh).view(np.uint32)
        nan = np.isnan(xh)
        bad = np.flatnonzero((got != ref) & ~nan)
        assert bad.size == 0, (c, xh[bad[:8]], got[bad[:8]], ref[bad[:8]])
        assert np.isnan(host(y)[nan]).all()


def test_swiglu_bit_exact(K, orc):
    """ApplySiLU(g) * u against the restatement over a wide argument range."""
    rng = np.random.default_rng(5)
    g = np.concatenate([rng.normal(0, 3, 1 << 20), rng.uniform(-120, 120, 1 << 16),
                        [0.0, -0.0, 88.0, -88.0, 89.0, -104.0, 1e-30]]).astype(np.float32)
    u = rng.normal(0, 1, g.size).astype(np.float32)
    out = torch.empty(g.size, device="cuda")
    K.apply_swiglu(dev(g), dev(u), out)
    ref = orc.silu(g.copy()) * u
    np.testing.assert_array_equal(host(out), ref)


# ------------------------------------------------ tensor-core projection
@pytest.mark.parametrize("rows,n,k,with_bias", [(1, 128, 256, False), (130, 300, 512, True), (64, 256, 4096, False),
                                                (257, 14336, 4096, False)])
def test_tensor_core_projection_bit_exact(K, orc, rows, n, k, with_bias):
    """ProjectBatchedWeightStationary on tcgen05 tensor cores: every output
    equal to the restatement's per-row dot (ragged row and token tiles)."""
    rng = np.random.default_rng(rows + n)
    wf = orc.fill_normal(n * k, rows + 5, 0.0, 0.02).reshape(n, k)
    w = orc.quantize_q4k(wf)
    x = rng.normal(0, 1, (rows, k)).astype(np.float32)
    x[0, :256] = 0.0
    bias = rng.uniform(-1, 1, n).astype(np.float32) if with_bias else None
    y = torch.empty(rows * n, device="cuda")
    q = torch.empty(rows * k, dtype=torch.int8, device="cuda")
    s = torch.empty(rows * k // 256, device="cuda")
    b = torch.empty(rows * k // 16, dtype=torch.int16, device="cuda")
    scratch = torch.empty(K.tc_scratch_bytes(rows, k), dtype=torch.uint8, device="cuda")
    wt = K.Q4KWeight(dev(w), k, n)
    bd = None if bias is None else dev(bias)
    K.Q4KDotKernel.project_batched_tensor_cores(dev(x), rows, wt, bd, y, q, s, b, scratch)
    if rows * n * k <= 1 << 30:
        ref = orc.kq_project_batched(orc.Q4_K, x, w, n, k, bias)
    else:  # the 8B shape: against the dp4a kernel (itself bit-exact to the restatement above)
        y2 = torch.empty(rows * n, device="cuda")
        K.Q4KDotKernel.project_batched(dev(x), rows, wt, bd, y2, q, s, b)
        ref = host(y2).reshape(rows, n)
    np.testing.assert_array_equal(host(y).reshape(rows, n), ref)


def test_tensor_core_projection_extreme_magnitudes(K, orc):
    """The largest integer sums the format allows (6-bit scales of 63, nibbles
    0 and 15, activations of +-127) stay exact in the fp32 accumulators:
    identical to the dp4a weight-stationary kernel."""
    n, k, rows = 128, 512, 128
    blk = np.zeros((n, k // 256, 144), np.uint8)
    blk[:, :, 0:2] = np.frombuffer(np.float16(0.01).tobytes(), np.uint8)
    blk[:, :, 2:4] = np.frombuffer(np.float16(0.005).tobytes(), np.uint8)
    blk[:, :, 4:16] = 0xFF                       # every scale and min 63
    blk[: n // 2, :, 16:] = 0x00                 # nibbles 0 (centered -8)
    blk[n // 2:, :, 16:] = 0xFF                  # nibbles 15
    w = blk.reshape(-1)
    x = np.ones((rows, k), np.float32)
    x[rows // 2:] = -1.0
    outs = []
    for tc in (True, False):
        y = torch.empty(rows * n, device="cuda")
        q = torch.empty(rows * k, dtype=torch.int8, device="cuda")
        s = torch.empty(rows * k // 256, device="cuda")
        b = torch.empty(rows * k // 16, dtype=torch.int16, device="cuda")
        wt = K.Q4KWeight(dev(w), k, n)
        if tc:
            scratch = torch.empty(K.tc_scratch_bytes(rows, k), dtype=torch.uint8, device="cuda")
            K.Q4KDotKernel.project_batched_tensor_cores(dev(x), rows, wt, None, y, q, s, b, scratch)
        else:
            K.Q4KDotKernel.project_batched(dev(x), rows, wt, None, y, q, s, b)
        outs.append(host(y))
        assert int(np.abs(host(q)).min()) == 127
    np.testing.assert_array_equal(outs[0], outs[1])


@pytest.mark.parametrize("rows,n,k,with_bias", [(1, 80, 384, True), (40, 4864, 896, False), (130, 896, 4864, True),
                                                (257, 300, 1024, False)])
def test_q8_tensor_core_projection_bit_exact(K, orc, rows, n, k, with_bias):
    """Q8DotKernel.ProjectBatched on tcgen05 (kind::i8): ragged weight-row and
    token tiles, Qwen2-0.5B shapes, bit-exact to the restatement."""
    rng = np.random.default_rng(rows * 3 + n + k)
    w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    x = rng.normal(0, 1, (rows, k)).astype(np.float32)
    x[0, :64] = 0.0
    bias = rng.normal(0, 0.1, n).astype(np.float32) if with_bias else None
    g = orc.quantize_q8_0_gguf(w)
    rq, rs = orc.q8_0_deinterleave(g, n * k)
    ref = orc.q8_0_project_batched(x, rq, rs, n, k, bias)
    w8 = K.Q8Weight.from_gguf(dev(g), k, n)
    y = torch.empty(rows * n, device="cuda")
    xq, xs = torch.empty(rows * k, dtype=torch.int8, device="cuda"), torch.empty(rows * k // 32, device="cuda")
    scratch = torch.empty(K.tc_scratch_bytes(rows, k), dtype=torch.uint8, device="cuda")
    K.Q8DotKernel.project_batched_tensor_cores(dev(x), rows, w8, None if bias is None else dev(bias), y, xq, xs,
                                               scratch)
    np.testing.assert_array_equal(host(y).reshape(rows, n), ref)


def test_q8_tensor_core_projection_large_and_extreme(K):
    """The 8B gate shape against the dp4a kernel, and weights and activations
    at +-127 (the largest block dots) exact in the int32 accumulators."""
    n, k, rows = 14336, 4096, 200
    g = torch.Generator(device="cuda").manual_seed(7)
    w8 = K.Q8Weight.from_gguf(K.GgmlQuant.quantize_q8_0(torch.randn(n, k, device="cuda", generator=g) * 0.02), k, n)
    x = torch.randn(rows * k, device="cuda", generator=g)
    for extreme in (False, True):
        if extreme:
            w8.quants.copy_(torch.where(torch.arange(n * k, device="cuda").reshape(n, k) % 3 == 0, -127, 127)
                            .to(torch.int8).reshape(w8.quants.shape))
            x = torch.where(torch.arange(rows * k, device="cuda") % 5 == 0, -1.0, 1.0)
        outs = []
        for tc in (True, False):
            y = torch.empty(rows * n, device="cuda")
            xq, xs = torch.empty(rows * k, dtype=torch.int8, device="cuda"), torch.empty(rows * k // 32, device="cuda")
            if tc:
                scratch = torch.empty(K.tc_scratch_bytes(rows, k), dtype=torch.uint8, device="cuda")
                K.Q8DotKernel.project_batched_tensor_cores(x, rows, w8, None, y, xq, xs, scratch)
            else:
                K.Q8DotKernel.project_batched(x, rows, w8, None, y, xq, xs)
            outs.append(host(y))
        np.testing.assert_array_equal(outs[0], outs[1])


@pytest.mark.parametrize("rows,n,k,with_bias", [(1, 96, 2048, True), (130, 300, 4096, False), (33, 1024, 4096, True),
                                                (200, 4096, 14336, False)])
def test_q6k_tensor_core_projection_bit_exact(K, orc, rows, n, k, with_bias):
    """Q6KDotKernel.ProjectBatched on tcgen05 (split 8-bit scales): ragged
    weight-row and token tiles, the 8B attn_v / ffn_down shapes."""
    rng = np.random.default_rng(rows + 2 * n + k)
    wf = orc.fill_normal(n * k, rows + 11, 0.0, 0.02).reshape(n, k)
    w = orc.quantize_q6k(wf)
    x = rng.normal(0, 1, (rows, k)).astype(np.float32)
    x[0, :256] = 0.0
    bias = rng.uniform(-1, 1, n).astype(np.float32) if with_bias else None
    y = torch.empty(rows * n, device="cuda")
    q = torch.empty(rows * k, dtype=torch.int8, device="cuda")
    s = torch.empty(rows * k // 256, device="cuda")
    b = torch.empty(rows * k // 16, dtype=torch.int16, device="cuda")
    scratch = torch.empty(K.tc_scratch_bytes(rows, k), dtype=torch.uint8, device="cuda")
    wt = K.Q6KWeight(dev(w), k, n)
    bd = None if bias is None else dev(bias)
    K.Q6KDotKernel.project_batched_tensor_cores(dev(x), rows, wt, bd, y, q, s, b, scratch)
    if rows * n * k <= 1 << 30:
        ref = orc.kq_project_batched(orc.Q6_K, x, w, n, k, bias)
    else:  # against the dp4a kernel (itself bit-exact to the restatement)
        y2 = torch.empty(rows * n, device="cuda")
        K.Q6KDotKernel.project_batched(dev(x), rows, wt, bd, y2, q, s, b)
        ref = host(y2).reshape(rows, n)
    np.testing.assert_array_equal(host(y).reshape(rows, n), ref)


def test_q6k_tensor_core_projection_extreme_magnitudes(K):
    """6-bit values 0 and 63 under scales -128 and 127 against activations of
    +-127: the largest sub-block products stay exact in both accumulators."""
    n, k, rows = 256, 2048, 96
    blk = np.zeros((n, k // 256, 210), np.uint8)
    blk[: n // 2, :, :192] = 0x00            # q = 0
    blk[n // 2:, :, :192] = 0xFF             # q = 63
    blk[:, :, 192:208:2] = np.uint8(0x80)    # scale -128
    blk[:, :, 193:208:2] = np.uint8(0x7F)    # scale 127
    blk[:, :, 208:210] = np.frombuffer(np.float16(0.01).tobytes(), np.uint8)
    w = blk.reshape(-1)
    x = np.ones((rows, k), np.float32)
    x[rows // 3:] = -1.0
    outs = []
    for tc in (True, False):
        y = torch.empty(rows * n, device="cuda")
        q = torch.empty(rows * k, dtype=torch.int8, device="cuda")
        s = torch.empty(rows * k // 256, device="cuda")
        b = torch.empty(rows * k // 16, dtype=torch.int16, device="cuda")
        wt = K.Q6KWeight(dev(w), k, n)
        if tc:
            scratch = torch.empty(K.tc_scratch_bytes(rows, k), dtype=torch.uint8, device="cuda")
            K.Q6KDotKernel.project_batched_tensor_cores(dev(x), rows, wt, None, y, q, s, b, scratch)
        else:
            K.Q6KDotKernel.project_batched(dev(x), rows, wt, None, y, q, s, b)
        outs.append(host(y))
    np.testing.assert_array_equal(outs[0], outs[1])
