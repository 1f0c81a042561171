"""Shared helpers for the model-level parity tests: small random-init model
files (host numpy, on-disk formats, quantized by the CPU restatement) and
their conversion to the restatement's resident form, following the
reference loader's residency choices (Loading/GgufLlamaLoader.cs:941-1203)."""
from __future__ import annotations

import numpy as np

from oracle import oracle as orc

Q4KM = dict(wq=orc.Q4_K, wk=orc.Q4_K, wv=orc.Q6_K, wo=orc.Q4_K, gate=orc.Q4_K, up=orc.Q4_K, down=orc.Q6_K,
            embed=orc.Q4_K, lm_head=orc.Q6_K)

TINY_LLAMA = dict(n_layers=2, d_model=512, n_heads=8, n_kv_heads=2, head_dim=64, d_ff=1024, vocab=2000,
                  theta=500000.0, eps=1e-6, rope_split_half=0, tied=False, qkv_bias=False, scheme="q4_k_m")
TINY_MIXTRAL = dict(n_layers=2, d_model=512, n_heads=8, n_kv_heads=2, head_dim=64, d_ff=512, vocab=1000,
                    theta=1000000.0, eps=1e-6, rope_split_half=0, tied=False, qkv_bias=False, scheme="q4_k_m",
                    n_experts=4, n_experts_used=2, normalize_experts=1)
TINY_QWEN = dict(n_layers=2, d_model=224, n_heads=7, n_kv_heads=1, head_dim=32, d_ff=608, vocab=1500,
                 theta=1000000.0, eps=1e-6, rope_split_half=1, tied=True, qkv_bias=True, scheme="q8_0")


def make_model_file(cfg: dict, seed: int, std: float = 0.02) -> dict:
    rng = np.random.default_rng(seed)
    D, H, KVH, hd, FF, V = (cfg[k] for k in ("d_model", "n_heads", "n_kv_heads", "head_dim", "d_ff", "vocab"))
    q4km = cfg["scheme"] == "q4_k_m"

    def mat(rows, cols, key):
        w = rng.normal(0, std, size=(rows, cols)).astype(np.float32)
        t = Q4KM[key] if q4km else orc.Q8_0
        if t == orc.Q4_K:
            return (t, orc.quantize_q4k(w), rows, cols)
        if t == orc.Q6_K:
            return (t, orc.quantize_q6k(w), rows, cols)
        return (t, orc.quantize_q8_0_gguf(w), rows, cols)

    def vec(n):
        return rng.normal(0, std, size=n).astype(np.float32)

    layers = []
    E = cfg.get("n_experts", 0)
    for _ in range(cfg["n_layers"]):
        L = dict(attn_norm=(1 + rng.normal(0, 0.1, D)).astype(np.float32),
                 ffn_norm=(1 + rng.normal(0, 0.1, D)).astype(np.float32),
                 wq=mat(H * hd, D, "wq"), wk=mat(KVH * hd, D, "wk"), wv=mat(KVH * hd, D, "wv"),
                 wo=mat(D, H * hd, "wo"))
        if E:
            # Mixtral: ffn_gate_inp as the loader hands it to the engine,
            # input-major F32 [d_model x n_experts]; experts in file formats
            L["router"] = rng.normal(0, std * 5, size=(D, E)).astype(np.float32)
            L["experts"] = [dict(gate=mat(FF, D, "gate"), up=mat(FF, D, "up"), down=mat(D, FF, "down"))
                            for _ in range(E)]
        else:
            L.update(gate=mat(FF, D, "gate"), up=mat(FF, D, "up"), down=mat(D, FF, "down"))
        if cfg.get("qkv_bias"):
            L.update(bq=vec(H * hd), bk=vec(KVH * hd), bv=vec(KVH * hd))
        layers.append(L)
    m = dict(layers=layers, embed=mat(V, D, "embed"), final_norm=(1 + rng.normal(0, 0.1, D)).astype(np.float32))
    m["lm_head"] = None if cfg.get("tied") else mat(V, D, "lm_head")
    return m


def _resident(entry, force_q8=False):
    """(type, data, rows, cols) in file format -> oracle (type, data, scales, rows, cols)."""
    t, data, rows, cols = entry
    if t == orc.Q8_0:
        q, s = orc.q8_0_deinterleave(data, rows * cols)
        return (orc.Q8_0, q, s, rows, cols)
    if force_q8:
        q, s = orc.requant_q8_0(t, data, rows, cols)
        return (orc.Q8_0, q, s, rows, cols)
    return (t, data, None, rows, cols)


def oracle_weights(model_file: dict) -> dict:
    layers = []
    for L in model_file["layers"]:
        o = dict(attn_norm=L["attn_norm"], ffn_norm=L["ffn_norm"])
        for k in ("wq", "wk", "wv"):
            o[k] = _resident(L[k])
        if "experts" in L:
            o["router"] = np.ascontiguousarray(L["router"], dtype=np.float32).reshape(-1)
            o["experts"] = [{k: _resident(ex[k]) for k in ("gate", "up", "down")} for ex in L["experts"]]
        else:
            for k in ("gate", "up", "down"):
                o[k] = _resident(L[k])
        o["wo"] = _resident(L["wo"], force_q8=True)
        for b in ("bq", "bk", "bv", "bo"):
            o[b] = L.get(b)
        layers.append(o)
    t, data, rows, cols = model_file["embed"]
    if t == orc.Q8_0:  # the reference dequantizes a Q8_0 embedding to F32
        q, s = orc.q8_0_deinterleave(data, rows * cols)
        emb = (orc.F32, orc.dequant_rows(orc.Q8_0, q, rows, cols, scales=s).reshape(-1), None, rows, cols)
    else:
        emb = (t, data, None, rows, cols)
    lm = model_file["lm_head"] if model_file["lm_head"] is not None else model_file["embed"]
    return dict(layers=layers, embed=emb, final_norm=model_file["final_norm"], lm_head=_resident(lm))


def oracle_session(cfg: dict, model_file: dict, max_ctx: int) -> orc.OracleSession:
    return orc.OracleSession(cfg, oracle_weights(model_file), max_ctx)
