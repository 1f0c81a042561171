"""Pins the CPU restatement (oracle/) to the reference.

The reference commits no golden numeric vectors for this path; it pins it by
hand-built known answers and by properties.  Both are ported here: the known
answers come from tests/golden/known_answers.json (built as the reference's
tests build them), the properties follow the reference tests named in each
docstring, with their shapes and tolerances.
"""
import json
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _cases(kind):
    with open(os.path.join(GOLDEN, "known_answers.json")) as f:
        return [c for c in json.load(f)["cases"] if c["kind"] == kind]


def test_known_answer_unpack_q4k(orc):
    for c in _cases("unpack_q4k"):
        sc, m = orc.unpack_q4k_scales_mins(np.array(c["packed"], np.uint8))
        assert list(sc) == c["scales"], c["ref"]
        assert list(m) == c["mins"], c["ref"]


def test_known_answer_decode_q4k(orc):
    for c in _cases("decode_q4k"):
        out = orc.decode_q4k_block(np.array(c["block"], np.uint8))
        np.testing.assert_allclose(out, c["expected"], atol=c["abs_tol"], err_msg=c["ref"])


def test_known_answer_decode_q6k(orc):
    for c in _cases("decode_q6k"):
        out = orc.decode_q6k_block(np.array(c["block"], np.uint8))
        np.testing.assert_allclose(out, c["expected"], atol=c["abs_tol"], err_msg=c["ref"])
    for c in _cases("decode_q6k_points"):
        out = orc.decode_q6k_block(np.array(c["block"], np.uint8))
        for i, v in c["points"].items():
            assert abs(out[int(i)] - v) <= c["abs_tol"], c["ref"]


def test_known_answer_decode_q8_0(orc):
    for c in _cases("decode_q8_0"):
        q, s = orc.q8_0_deinterleave(np.array(c["blocks"], np.uint8), c["n"])
        out = orc.dequant_rows(orc.Q8_0, q, 1, c["n"], scales=s)[0]
        np.testing.assert_allclose(out, c["expected"], atol=c["abs_tol"], err_msg=c["ref"])


def test_known_answer_attention(orc):
    for c in _cases("attention"):
        hd, seq = c["hd"], c["seq"]
        keys = np.array(c["keys"], np.float32).reshape(seq, hd)
        vals = np.array(c["values"], np.float32).reshape(seq, hd)
        out = orc.attention_single_head(np.array(c["q"], np.float32), keys, vals, c["scale"])
        np.testing.assert_allclose(out, c["expected"], atol=max(c["tol"], 1e-6) * 10, err_msg=c["ref"])
        assert np.all(np.isfinite(out))


def test_q8k_all_zeros_block(orc):
    """Q4KDotKernelTests.cs:199-216."""
    q, s, b = orc.quantize_q8k(np.zeros(256, np.float32))
    assert s[0] == 0.0 and not q.any() and not b.any()


def test_q8k_reconstruction_and_bsums(orc):
    """Q4KDotKernelTests.cs:167-196: |s*q - x| <= s and exact group sums."""
    x = np.random.default_rng(7).uniform(-1, 1, 256).astype(np.float32)
    q, s, b = orc.quantize_q8k(x)
    assert np.all(np.abs(s[0] * q.astype(np.float32) - x) <= s[0])
    np.testing.assert_array_equal(q.reshape(16, 16).astype(np.int32).sum(1), b)


def _random_q4k_blocks(rng, n, k):
    """Q4KDotKernelTests.cs:225-247: random bytes with sane fp16 d/dmin."""
    nb = n * (k // 256)
    blocks = rng.integers(0, 256, size=(nb, 144), dtype=np.uint8)
    d = (rng.random(nb) * 0.05 + 0.001).astype(np.float16).view(np.uint8).reshape(nb, 2)
    dm = (rng.random(nb) * 0.03 + 0.001).astype(np.float16).view(np.uint8).reshape(nb, 2)
    blocks[:, 0:2] = d
    blocks[:, 2:4] = dm
    return blocks.reshape(-1)


def _random_q6k_blocks(rng, n, k):
    nb = n * (k // 256)
    blocks = rng.integers(0, 256, size=(nb, 210), dtype=np.uint8)
    blocks[:, 208:210] = (rng.random(nb) * 0.01 + 0.0005).astype(np.float16).view(np.uint8).reshape(nb, 2)
    return blocks.reshape(-1)


@pytest.mark.parametrize("kind", ["q4k", "q6k"])
def test_project_matches_f32_decode(orc, kind):
    """Q4KDotKernelTests.cs:32-65 / Q6KDotKernelTests.cs:31-64: L2-rel < 3%
    against the F32 decode at 96 x 512."""
    rng = np.random.default_rng(20260519)
    n, k = 96, 512
    t = orc.Q4_K if kind == "q4k" else orc.Q6_K
    w = _random_q4k_blocks(rng, n, k) if kind == "q4k" else _random_q6k_blocks(rng, n, k)
    x = rng.uniform(-1, 1, k).astype(np.float32)
    y = orc.kq_project(t, x, w, n, k)
    ref = orc.dequant_rows(t, w, n, k).astype(np.float64) @ x.astype(np.float64)
    l2 = np.sqrt(((y - ref) ** 2).sum() / (ref ** 2).sum())
    assert l2 < 0.03


@pytest.mark.parametrize("rows", [1, 3, 16])
def test_batched_bit_identical_to_per_row(orc, rows):
    """Q4KDotKernelTests.cs:96-136 and the weight-stationary parity test
    (Parity/Q4KWeightStationaryParityTests.cs:20): batched == per-row Project."""
    rng = np.random.default_rng(rows * 17 + 5)
    n, k = 96, 512
    w = _random_q4k_blocks(rng, n, k)
    bias = rng.uniform(-1, 1, n).astype(np.float32)
    x = rng.uniform(-1, 1, (rows, k)).astype(np.float32)
    per_row = np.stack([orc.kq_project(orc.Q4_K, x[r], w, n, k, bias) for r in range(rows)])
    batched = orc.kq_project_batched(orc.Q4_K, x, w, n, k, bias)
    np.testing.assert_array_equal(per_row, batched)


def test_bias_applied(orc):
    """Q4KDotKernelTests.cs:139-165."""
    rng = np.random.default_rng(99)
    n, k = 32, 256
    w = _random_q4k_blocks(rng, n, k)
    x = rng.uniform(-1, 1, k).astype(np.float32)
    b = rng.uniform(-1, 1, n).astype(np.float32)
    np.testing.assert_allclose(orc.kq_project(orc.Q4_K, x, w, n, k) + b, orc.kq_project(orc.Q4_K, x, w, n, k, b),
                               atol=1e-3)


@pytest.mark.parametrize("seed", [1, 2, 3])
def test_q4k_encoder_round_trip(orc, seed):
    """GgmlQuantTests.cs:27-84: cosine > 0.995 and RMSE < 2% of the mean row range."""
    rng = np.random.default_rng(seed)
    n, k = 8, 512
    i = np.arange(n * k)
    f = ((rng.random(n * k) * 2 - 1) * (0.2 + (i % 7) * 0.1)).astype(np.float32).reshape(n, k)
    back = orc.dequant_rows(orc.Q4_K, orc.quantize_q4k(f), n, k)
    cos = (f * back).sum() / np.sqrt((f.astype(np.float64) ** 2).sum() * (back.astype(np.float64) ** 2).sum())
    rmse = np.sqrt(((f - back).astype(np.float64) ** 2).mean())
    avg_range = (f.max(1) - f.min(1)).mean()
    assert cos > 0.995 and rmse < 0.02 * avg_range


def test_q4k_constant_row(orc):
    """GgmlQuantTests.cs:86-107."""
    f = np.full((1, 256), 0.37, np.float32)
    back = orc.dequant_rows(orc.Q4_K, orc.quantize_q4k(f), 1, 256)
    assert np.abs(back - 0.37).max() < 1e-3


def test_q6k_and_q8_encoders_round_trip(orc):
    """The Q6_K and Q8_0 encoders (ours; the reference only decodes these)
    round-trip within their precision."""
    rng = np.random.default_rng(5)
    f = rng.normal(0, 0.02, (16, 512)).astype(np.float32)
    b6 = orc.dequant_rows(orc.Q6_K, orc.quantize_q6k(f), 16, 512)
    q, s = orc.q8_0_deinterleave(orc.quantize_q8_0_gguf(f), f.size)
    b8 = orc.dequant_rows(orc.Q8_0, q, 16, 512, scales=s)
    for back, tol in ((b6, 0.03), (b8, 0.01)):
        rel = np.sqrt(((f - back) ** 2).sum() / (f ** 2).sum())
        assert rel < tol


def test_q8_dot_matches_f32(orc):
    """Q8DotKernelTests.cs: the Q8_0 projection tracks the F32 product within
    Q8 noise at the reference's 2048 x 512 shape."""
    rng = np.random.default_rng(11)
    n, k = 512, 2048
    w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    x = rng.normal(0, 1, k).astype(np.float32)
    wq, ws = orc.quantize_q8_0(w.reshape(-1))
    y = orc.q8_0_project(x, wq, ws, n, k)
    ref = w.astype(np.float64) @ x
    assert np.sqrt(((y - ref) ** 2).sum() / (ref ** 2).sum()) < 0.02


def test_moe_topk_ties_keep_lower_index(orc):
    """MoeRouter.cs:40-128 / MoeRouterTests.cs: descending order, ties keep the
    lower index, softmax over the selected."""
    idx, w = orc.moe_select_topk(np.array([0.5, 2.0, 2.0, -1.0], np.float32), 2)
    assert list(idx) == [1, 2]
    np.testing.assert_allclose(w, [0.5, 0.5], atol=1e-7)
    idx, w = orc.moe_select_topk(np.array([1.0, 3.0, 2.0], np.float32), 2)
    assert list(idx) == [1, 2]
    e = np.exp(-1.0)
    np.testing.assert_allclose(w, [1 / (1 + e), e / (1 + e)], rtol=1e-6)


@pytest.mark.parametrize("split_half", [0, 1])
def test_rope_relative_position_invariance(orc, split_half):
    """Runtime/Parity/RopeConventionTests.cs:23-100: position 0 is the
    identity and q.k depends only on the position difference."""
    c, s = orc.rope_table(64, 16, 10000.0)
    rng = np.random.default_rng(3)
    q = rng.normal(size=16).astype(np.float32)
    k = rng.normal(size=16).astype(np.float32)
    np.testing.assert_array_equal(orc.rope_apply(q, c[0], s[0], split_half), q)
    d1 = orc.rope_apply(q, c[10], s[10], split_half) @ orc.rope_apply(k, c[7], s[7], split_half)
    d2 = orc.rope_apply(q, c[33], s[33], split_half) @ orc.rope_apply(k, c[30], s[30], split_half)
    assert abs(d1 - d2) < 1e-4


def test_parity_fixtures_reproduce(orc):
    """The committed parity vectors still come out of the restatement bit for
    bit (guards the fixtures the GPU tests compare against)."""
    z = np.load(os.path.join(GOLDEN, "parity_small.npz"))
    np.testing.assert_array_equal(orc.kq_project(orc.Q4_K, z["q4k_x"], z["q4k_w"], 96, 512, z["q4k_bias"]),
                                  z["q4k_y"])
    np.testing.assert_array_equal(orc.kq_project(orc.Q6_K, z["q6k_x"], z["q6k_w"], 64, 768), z["q6k_y"])
    q, s = orc.q8_0_deinterleave(z["q8_gguf"], 80 * 352)
    np.testing.assert_array_equal(orc.q8_0_project(z["q8_x"], q, s, 80, 352), z["q8_y"])


def test_q8kv_quantize_properties(orc):
    """Q8KvQuant.Quantize (Runtime/Q8KvQuant.cs:25-77): |scale*q - x| <= scale/2
    (round to nearest), max |q| = 127 at the largest element, zero vector ->
    scale 0 and zero bytes."""
    rng = np.random.default_rng(31)
    for n in (32, 64, 128):
        x = rng.normal(0, 2, n).astype(np.float32)
        q, s = orc.q8kv_quantize(x)
        assert s == np.float32(np.abs(x).max() / np.float32(127))
        assert np.abs(q).max() == 127
        assert np.all(np.abs(s * q.astype(np.float32) - x) <= s * 0.5 + 1e-7)
    q, s = orc.q8kv_quantize(np.zeros(64, np.float32))
    assert s == 0.0 and not q.any()


def test_q8kv_attention_tracks_f32(orc):
    """ComputeSingleHeadQ8 vs ComputeSingleHead on the same keys/values:
    the int8 round trip is not bit-identical but cosine ~ 1 (the reference's
    own claim, Runtime/CachedAttentionKernel.cs:129-137)."""
    rng = np.random.default_rng(32)
    hd, seq = 128, 300
    K = rng.normal(size=(seq, hd)).astype(np.float32)
    V = rng.normal(size=(seq, hd)).astype(np.float32)
    kq = np.empty((seq, hd), np.int8); vq = np.empty((seq, hd), np.int8)
    ks = np.empty(seq, np.float32); vs = np.empty(seq, np.float32)
    for t in range(seq):
        kq[t], ks[t] = orc.q8kv_quantize(K[t])
        vq[t], vs[t] = orc.q8kv_quantize(V[t])
    q = rng.normal(size=hd).astype(np.float32)
    a = orc.attention_single_head_q8(q, kq, ks, vq, vs, 1 / np.sqrt(hd))
    b = orc.attention_single_head(q, K, V, np.float32(1 / np.sqrt(hd)))
    assert float(a @ b / np.linalg.norm(a) / np.linalg.norm(b)) > 0.999
