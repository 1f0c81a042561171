"""Generate the golden fixtures in this folder.

Two kinds of fixture:

1. ``known_answers.json`` — the reference's own hand-built known-answer tests,
   restated as data.  Each case names the reference test it comes from; the
   inputs are built exactly as that test builds them and the expected values
   are the ones that test asserts (Tests/LanguageModels/...).  These pin the
   CPU restatement (oracle/) to the reference without running .NET.

2. ``parity_*.npz`` — seeded inputs with the restatement's outputs, so the GPU
   parity tests also have a committed expectation that does not depend on
   rebuilding the oracle on the GPU box.  Regenerate after any change to the
   oracle; ``tests/test_oracle_golden.py`` checks the oracle still reproduces
   them bit for bit.

Run from the repository root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import math
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)


def fp16_bytes(v: float) -> list[int]:
    u = int(np.array([v], dtype=np.float16).view(np.uint16)[0])
    return [u & 0xFF, u >> 8]


def q4k_block(d, dmin, packed12, nibble_fill) -> list[int]:
    # GgmlDequantTests.cs:473-482 (BuildQ4_KBlock)
    return fp16_bytes(d) + fp16_bytes(dmin) + list(packed12) + [nibble_fill] * 128


def q6k_block(d, scales16, ql, qh_fill) -> list[int]:
    # GgmlDequantTests.cs:491-502 (BuildQ6_KBlock)
    b = list(ql) + [qh_fill] * 64 + [s & 0xFF for s in scales16] + fp16_bytes(d)
    assert len(b) == 210
    return b


def scales_all_ones_mins_all_zeros() -> list[int]:
    # GgmlDequantTests.cs:504-520
    p = [0] * 12
    for i in range(4):
        p[i] = 0x01
    for i in range(8, 12):
        p[i] = 0x01
    return p


def known_answers() -> dict:
    cases = []
    # GgmlDequantTests.cs:99-131 UnpackQ4_KScalesMins_LowerBranch_Jbelow4_Trivial
    p = [10, 20, 30, 40, 5, 15, 21, 27, 0, 0, 0, 0]
    cases.append({"kind": "unpack_q4k", "ref": "Tests/LanguageModels/Loading/GgmlDequantTests.cs:99-131",
                  "packed": p, "scales": [10, 20, 30, 40, 0, 0, 0, 0], "mins": [5, 15, 21, 27, 0, 0, 0, 0]})
    # GgmlDequantTests.cs:133-172 UnpackQ4_KScalesMins_UpperBranch_Jat4Plus_HighBitsContribute
    p = [0xC0] * 4 + [0x80] * 4 + [0x35] * 4
    cases.append({"kind": "unpack_q4k", "ref": "Tests/LanguageModels/Loading/GgmlDequantTests.cs:133-172",
                  "packed": p, "scales": [0] * 4 + [0x35] * 4, "mins": [0] * 4 + [0x23] * 4})
    # GgmlDequantTests.cs:189-210 DecodeQ4_KBlock_AllSubBlocksUseScale1Min0_NibbleEqualsValue
    blk = q4k_block(1.0, 0.0, scales_all_ones_mins_all_zeros(), 0x21)
    exp = []
    for p_ in range(4):
        exp += [1.0] * 32 + [2.0] * 32
    cases.append({"kind": "decode_q4k", "ref": "Tests/LanguageModels/Loading/GgmlDequantTests.cs:189-210",
                  "block": blk, "expected": exp, "abs_tol": 5e-7})
    # GgmlDequantTests.cs:212-249 DecodeQ4_KBlock_ScaleAndMinApplyPerSubBlock
    packed = [0] * 12
    for i in range(4):
        packed[i] = i + 1
        packed[i + 4] = i
    for j in range(4, 8):
        sc, mn = j + 1, j
        packed[j + 4] = ((mn << 4) | (sc & 0x0F)) & 0xFF
    blk = q4k_block(2.0, 1.0, packed, 0x53)
    exp = []
    for p_ in range(4):
        lo = 2.0 * (2 * p_ + 1) * 3 - 1.0 * (2 * p_)
        hi = 2.0 * (2 * p_ + 2) * 5 - 1.0 * (2 * p_ + 1)
        exp += [lo] * 32 + [hi] * 32
    cases.append({"kind": "decode_q4k", "ref": "Tests/LanguageModels/Loading/GgmlDequantTests.cs:212-249",
                  "block": blk, "expected": exp, "abs_tol": 5e-5})
    # GgmlDequantTests.cs:262-276 DecodeQ6_KBlock_AllZerosWithUnitScale_GivesBiasMinus32
    blk = q6k_block(1.0, [1] * 16, [0] * 128, 0)
    cases.append({"kind": "decode_q6k", "ref": "Tests/LanguageModels/Loading/GgmlDequantTests.cs:262-276",
                  "block": blk, "expected": [-32.0] * 256, "abs_tol": 5e-5})
    # GgmlDequantTests.cs:278-293 DecodeQ6_KBlock_HighBitsAndSignedScalesApply
    blk = q6k_block(0.5, [-1] * 16, [0xFF] * 128, 0xFF)
    cases.append({"kind": "decode_q6k", "ref": "Tests/LanguageModels/Loading/GgmlDequantTests.cs:278-293",
                  "block": blk, "expected": [-15.5] * 256, "abs_tol": 5e-5})
    # GgmlDequantTests.cs:295-319 DecodeQ6_KBlock_LowAndHighNibblesDecodeIndependently
    ql = [0] * 128
    ql[0] = 0x10
    blk = q6k_block(1.0, [1] * 16, ql, 0)
    cases.append({"kind": "decode_q6k_points", "ref": "Tests/LanguageModels/Loading/GgmlDequantTests.cs:295-319",
                  "block": blk, "points": {"64": -31.0, "0": -32.0, "32": -32.0, "96": -32.0,
                                           "128": -32.0, "255": -32.0}, "abs_tol": 5e-5})
    # GgmlDequantTests.cs:20-47 Q8_0_DequantizesSingleBlock_RoundTrip (scale 2.0, fp16-exact)
    qs = [-128, -1, 0, 1, 127] + [i - 16 for i in range(5, 32)]
    blk = fp16_bytes(2.0) + [q & 0xFF for q in qs]
    cases.append({"kind": "decode_q8_0", "ref": "Tests/LanguageModels/Loading/GgmlDequantTests.cs:20-47",
                  "blocks": blk, "n": 32, "expected": [2.0 * q for q in qs], "abs_tol": 5e-5})
    # GgmlDequantTests.cs:49-78 Q8_0_DequantizesMultipleBlocks_DifferentScales
    scales = [0.5, 1.0, 0.125]
    blk, exp = [], []
    for b in range(3):
        q = [b * 10 + i - 5 for i in range(32)]
        blk += fp16_bytes(scales[b]) + [v & 0xFF for v in q]
        exp += [scales[b] * v for v in q]
    cases.append({"kind": "decode_q8_0", "ref": "Tests/LanguageModels/Loading/GgmlDequantTests.cs:49-78",
                  "blocks": blk, "n": 96, "expected": exp, "abs_tol": 5e-5})
    # Runtime/Kernels/CachedAttentionKernelTests.cs: known-answer softmax cases
    e1, e0 = math.exp(1.0), 1.0
    cases += [
        {"kind": "attention", "ref": "Tests/LanguageModels/Runtime/Kernels/CachedAttentionKernelTests.cs:13-33",
         "q": [1, 2], "keys": [], "values": [], "seq": 0, "hd": 2, "scale": 1.0, "expected": [0, 0], "tol": 0},
        {"kind": "attention", "ref": "Tests/LanguageModels/Runtime/Kernels/CachedAttentionKernelTests.cs:35-57",
         "q": [1, 0, 0], "keys": [0.5, 0.25, -1], "values": [10, 20, 30], "seq": 1, "hd": 3, "scale": 1.0,
         "expected": [10, 20, 30], "tol": 1e-5},
        {"kind": "attention", "ref": "Tests/LanguageModels/Runtime/Kernels/CachedAttentionKernelTests.cs:59-93",
         "q": [1, 0], "keys": [1, 0, 0, 1], "values": [10, 0, 0, 20], "seq": 2, "hd": 2, "scale": 1.0,
         "expected": [10 * e1 / (e1 + e0), 20 * e0 / (e1 + e0)], "tol": 1e-5},
        {"kind": "attention", "ref": "Tests/LanguageModels/Runtime/Kernels/CachedAttentionKernelTests.cs:95-130",
         "q": [1000, 1000], "keys": [1000, 1000, 999, 999], "values": [1, 2, 3, 4], "seq": 2, "hd": 2,
         "scale": 1.0, "expected": [1, 2], "tol": 1e-5},
        {"kind": "attention", "ref": "Tests/LanguageModels/Runtime/Kernels/CachedAttentionKernelTests.cs:132-150",
         "q": [1], "keys": [1], "values": [7], "seq": 1, "hd": 1, "scale": 1.0, "expected": [7], "tol": 1e-5},
    ]
    # Runtime/Q4KDotKernelTests.cs:199-216 QuantizeActivationQ8K_AllZeros_ProducesZeroBlock
    cases.append({"kind": "q8k_zeros", "ref": "Tests/LanguageModels/Runtime/Q4KDotKernelTests.cs:199-216"})
    # Loading/GgmlQuantTests.cs:86-107 QuantizeQ4K_ConstantRow_IsExact (0.37 -> max abs err < 1e-3)
    cases.append({"kind": "q4k_constant_row", "ref": "Tests/LanguageModels/Loading/GgmlQuantTests.cs:86-107",
                  "value": 0.37, "max_abs": 1e-3})
    return {"cases": cases}


def parity_fixtures():
    """Seeded GEMV/attention parity vectors from the restatement."""
    from oracle import oracle as orc

    rng = np.random.default_rng(0)
    out = {}
    # Q4_K projection, 96 x 512 with bias (the reference's test shape,
    # Q4KDotKernelTests.cs:68-94), weights from the reference quantizer.
    w = rng.normal(0, 0.02, size=(96, 512)).astype(np.float32)
    x = rng.normal(0, 1, size=512).astype(np.float32)
    b = rng.normal(0, 0.1, size=96).astype(np.float32)
    wq = orc.quantize_q4k(w)
    out["q4k_w"], out["q4k_x"], out["q4k_bias"] = wq, x, b
    out["q4k_y"] = orc.kq_project(orc.Q4_K, x, wq, 96, 512, b)
    # Q6_K projection 64 x 768
    w6 = rng.normal(0, 0.02, size=(64, 768)).astype(np.float32)
    x6 = rng.normal(0, 1, size=768).astype(np.float32)
    w6q = orc.quantize_q6k(w6)
    out["q6k_w"], out["q6k_x"] = w6q, x6
    out["q6k_y"] = orc.kq_project(orc.Q6_K, x6, w6q, 64, 768)
    # Q8_0 projection 80 x 352 (GGUF bytes -> de-interleaved)
    w8 = rng.normal(0, 0.02, size=(80, 352)).astype(np.float32)
    x8 = rng.normal(0, 1, size=352).astype(np.float32)
    g8 = orc.quantize_q8_0_gguf(w8)
    q8, s8 = orc.q8_0_deinterleave(g8, w8.size)
    out["q8_gguf"], out["q8_x"] = g8, x8
    out["q8_y"] = orc.q8_0_project(x8, q8, s8, 80, 352)
    np.savez_compressed(os.path.join(HERE, "parity_small.npz"), **out)


def main():
    with open(os.path.join(HERE, "known_answers.json"), "w") as f:
        json.dump(known_answers(), f, indent=1)
    parity_fixtures()
    print("wrote", os.listdir(HERE))


if __name__ == "__main__":
    main()
