"""ctypes binding of the CPU restatement (``libovf_oracle.so``).

TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA product and the CPU
baseline that ``bench.py`` times.  Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU legs import this module; the product package
(``overfit_b200``) never does.

Each wrapper names the reference routine it restates (paths relative to
``Sources/Main/LanguageModels/`` of DevOnBike/Overfit); the C source carries
the line citations.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libovf_oracle.so")

F32, F16, Q8_0, Q4_K, Q6_K = 0, 1, 8, 12, 14
QK_K = 256
BLOCK_BYTES = {Q4_K: 144, Q6_K: 210, Q8_0: 34}


def build(force: bool = False) -> str:
    """Compile the restatement with its Makefile (gcc, no fast-math)."""
    src = os.path.join(HERE, "ovf_oracle.c")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


P = C.c_void_p
I64 = C.c_int64


def _declare(L):
    sig = {
        "orc_unpack_q4k_scales_mins": (None, [P, P, P]),
        "orc_decode_q4k_block": (None, [P, P]),
        "orc_decode_q6k_block": (None, [P, P]),
        "orc_encode_q4k_block": (None, [P, P]),
        "orc_quantize_q4k": (None, [P, I64, I64, P]),
        "orc_encode_q6k_block": (None, [P, P]),
        "orc_quantize_q6k": (None, [P, I64, I64, P]),
        "orc_quantize_q8_0_gguf": (None, [P, I64, P]),
        "orc_q8_0_deinterleave": (None, [P, I64, P, P]),
        "orc_dequant_rows": (None, [C.c_int, P, P, I64, I64, I64, P]),
        "orc_requant_q8_0": (None, [C.c_int, P, I64, I64, P, P]),
        "orc_quantize_q8k": (None, [P, I64, P, P, P]),
        "orc_quantize_q8_0": (None, [P, I64, P, P]),
        "orc_q4k_dot": (C.c_float, [P, P, C.c_float, P]),
        "orc_q6k_dot": (C.c_float, [P, P, C.c_float, P]),
        "orc_q8_0_dot": (C.c_float, [P, P, P, P, I64]),
        "orc_kq_project_prequantized": (None, [C.c_int, P, I64, I64, P, P, P, P, P]),
        "orc_kq_project": (None, [C.c_int, P, P, I64, I64, P, P, P, P, P]),
        "orc_kq_project_batched": (None, [C.c_int, P, I64, P, I64, I64, P, P]),
        "orc_q8_0_project": (None, [P, P, P, I64, I64, P, P, P, P]),
        "orc_q8_0_project_batched": (None, [P, I64, P, P, I64, I64, P, P]),
        "orc_f32_project_input_major": (None, [P, P, I64, I64, P]),
        "orc_rmsnorm": (None, [P, P, P, I64, C.c_float]),
        "orc_rope_table": (None, [C.c_int, C.c_int, C.c_float, P, P]),
        "orc_rope_apply": (None, [P, C.c_int, P, P, C.c_int]),
        "orc_attention_single_head": (None, [P, P, P, P, P, C.c_int, C.c_int, C.c_float]),
        "orc_silu_inplace": (None, [P, I64]),
        "orc_moe_select_topk": (C.c_int, [P, C.c_int, C.c_int, P, P, C.c_int]),
        "orc_argmax": (C.c_int, [P, I64]),
        "orc_session_create": (P, [P, C.c_int]),
        "orc_session_destroy": (None, [P]),
        "orc_session_reset": (None, [P]),
        "orc_session_set_kv_fp16": (None, [P, C.c_int]),
        "orc_session_set_kv_q8": (None, [P, C.c_int]),
        "orc_q8kv_quantize": (C.c_float, [P, C.c_int, P]),
        "orc_attention_single_head_q8": (None, [P, P, P, P, P, P, P, C.c_int, C.c_int, C.c_float]),
        "orc_expf_array": (None, [C.c_void_p, C.c_void_p, C.c_int64]),
        "orc_session_fill_context": (C.c_int, [P, C.c_int, C.c_uint64]),
        "orc_session_position": (C.c_int, [P]),
        "orc_session_decode": (C.c_int, [P, C.c_int, P]),
        "orc_session_decode_layers": (C.c_int, [P, C.c_int, C.c_int, C.c_int, P]),
        "orc_num_threads": (C.c_int, []),
        "orc_set_num_threads": (None, [C.c_int]),
        "orc_fill_normal": (None, [P, I64, C.c_uint64, C.c_float, C.c_float]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args


def _p(a):
    return None if a is None else a.ctypes.data


# ----------------------------------------------------------------- codecs
def unpack_q4k_scales_mins(packed12: np.ndarray):
    p = np.ascontiguousarray(packed12, dtype=np.uint8)
    sc = np.zeros(8, np.uint8)
    m = np.zeros(8, np.uint8)
    lib().orc_unpack_q4k_scales_mins(_p(p), _p(sc), _p(m))
    return sc, m


def decode_q4k_block(block: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(block, dtype=np.uint8)
    out = np.zeros(256, np.float32)
    lib().orc_decode_q4k_block(_p(b), _p(out))
    return out


def decode_q6k_block(block: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(block, dtype=np.uint8)
    out = np.zeros(256, np.float32)
    lib().orc_decode_q6k_block(_p(b), _p(out))
    return out


def quantize_q4k(w: np.ndarray) -> np.ndarray:
    """GgmlQuant.QuantizeQ4_K: fp32 [rows x k] -> Q4_K bytes (output-major)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, k = w.shape
    out = np.empty(rows * (k // QK_K) * 144, np.uint8)
    lib().orc_quantize_q4k(_p(w), rows, k, _p(out))
    return out


def quantize_q6k(w: np.ndarray) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, k = w.shape
    out = np.empty(rows * (k // QK_K) * 210, np.uint8)
    lib().orc_quantize_q6k(_p(w), rows, k, _p(out))
    return out


def quantize_q8_0_gguf(w: np.ndarray) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.float32).reshape(-1)
    out = np.empty(w.size // 32 * 34, np.uint8)
    lib().orc_quantize_q8_0_gguf(_p(w), w.size, _p(out))
    return out


def q8_0_deinterleave(g: np.ndarray, n: int):
    g = np.ascontiguousarray(g, dtype=np.uint8)
    q = np.empty(n, np.int8)
    s = np.empty(n // 32, np.float32)
    lib().orc_q8_0_deinterleave(_p(g), n, _p(q), _p(s))
    return q, s


def dequant_rows(type_: int, data: np.ndarray, rows: int, k: int, scales=None, row0: int = 0) -> np.ndarray:
    out = np.empty((rows, k), np.float32)
    lib().orc_dequant_rows(type_, _p(data), _p(scales), row0, rows, k, _p(out))
    return out


def requant_q8_0(type_: int, data: np.ndarray, rows: int, k: int):
    """attn_output residency: decode then per-32 Q8_0 with fp32 scales."""
    q = np.empty(rows * k, np.int8)
    s = np.empty(rows * k // 32, np.float32)
    lib().orc_requant_q8_0(type_, _p(data), rows, k, _p(q), _p(s))
    return q, s


# ----------------------------------------------------------- quantizers
def quantize_q8k(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32)
    k = x.size
    q = np.empty(k, np.int8)
    s = np.empty(k // QK_K, np.float32)
    b = np.empty(k // 16, np.int16)
    lib().orc_quantize_q8k(_p(x), k, _p(q), _p(s), _p(b))
    return q, s, b


def quantize_q8_0(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32)
    q = np.empty(x.size, np.int8)
    s = np.empty(x.size // 32, np.float32)
    lib().orc_quantize_q8_0(_p(x), x.size, _p(q), _p(s))
    return q, s


# ---------------------------------------------------------- projections
def kq_project(type_: int, x: np.ndarray, w: np.ndarray, n: int, k: int, bias=None) -> np.ndarray:
    """Q4KDotKernel.ProjectParallel / Q6KDotKernel.ProjectParallel."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(n, np.float32)
    q = np.empty(k, np.int8)
    s = np.empty(k // QK_K, np.float32)
    b = np.empty(k // 16, np.int16)
    bias = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    lib().orc_kq_project(type_, _p(x), _p(w), n, k, _p(bias), _p(y), _p(q), _p(s), _p(b))
    return y


def kq_project_prequantized(type_, w, n, k, q, s, b, bias=None) -> np.ndarray:
    y = np.empty(n, np.float32)
    bias = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    lib().orc_kq_project_prequantized(type_, _p(w), n, k, _p(bias), _p(y), _p(q), _p(s), _p(b))
    return y


def kq_project_batched(type_, x: np.ndarray, w, n, k, bias=None) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows = x.shape[0]
    y = np.empty((rows, n), np.float32)
    bias = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    lib().orc_kq_project_batched(type_, _p(x), rows, _p(w), n, k, _p(bias), _p(y))
    return y


def q8_0_project(x, wq, ws, n, k, bias=None) -> np.ndarray:
    """Q8DotKernel.ProjectParallel over the de-interleaved Q8Weight."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(n, np.float32)
    xq = np.empty(k, np.int8)
    xs = np.empty(k // 32, np.float32)
    bias = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    lib().orc_q8_0_project(_p(x), _p(wq), _p(ws), n, k, _p(bias), _p(y), _p(xq), _p(xs))
    return y


def q8_0_project_batched(x, wq, ws, n, k, bias=None) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows = x.shape[0]
    y = np.empty((rows, n), np.float32)
    bias = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    lib().orc_q8_0_project_batched(_p(x), rows, _p(wq), _p(ws), n, k, _p(bias), _p(y))
    return y


# ------------------------------------------------------------ small ops
def rmsnorm(x, gamma, eps):
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().orc_rmsnorm(_p(x), _p(gamma), _p(y), x.size, eps)
    return y


def rope_table(max_seq, head_dim, theta):
    c = np.empty((max_seq, head_dim // 2), np.float32)
    s = np.empty_like(c)
    lib().orc_rope_table(max_seq, head_dim, theta, _p(c), _p(s))
    return c, s


def rope_apply(v, cos_p, sin_p, split_half):
    v = np.array(v, dtype=np.float32, copy=True)
    lib().orc_rope_apply(_p(v), v.size, _p(np.ascontiguousarray(cos_p)), _p(np.ascontiguousarray(sin_p)),
                         int(split_half))
    return v


def attention_single_head(q, keys, values, scale):
    q = np.ascontiguousarray(q, dtype=np.float32)
    keys = np.ascontiguousarray(keys, dtype=np.float32)
    values = np.ascontiguousarray(values, dtype=np.float32)
    seq, hd = keys.shape
    out = np.empty(hd, np.float32)
    scr = np.empty(max(seq, 1), np.float32)
    lib().orc_attention_single_head(_p(q), _p(keys), _p(values), _p(out), _p(scr), seq, hd, scale)
    return out


def moe_select_topk(logits, top_k, normalize=True):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    idx = np.empty(top_k, np.int32)
    w = np.empty(top_k, np.float32)
    k = lib().orc_moe_select_topk(_p(logits), logits.size, top_k, _p(idx), _p(w), int(normalize))
    return idx[:k], w[:k]


def silu(v):
    v = np.array(v, dtype=np.float32, copy=True)
    lib().orc_silu_inplace(_p(v), v.size)
    return v


def fill_normal(n, seed, mean=0.0, std=1.0) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().orc_fill_normal(_p(out), n, seed, mean, std)
    return out


def set_threads(n: int):
    lib().orc_set_num_threads(n)


def num_threads() -> int:
    return lib().orc_num_threads()


# ------------------------------------------------------------- the model
class OrcWeight(C.Structure):
    _fields_ = [("type", C.c_int), ("data", P), ("scales", P), ("rows", I64), ("cols", I64)]


class OrcLayer(C.Structure):
    _fields_ = [("attn_norm", P), ("wq", OrcWeight), ("wk", OrcWeight), ("wv", OrcWeight), ("wo", OrcWeight),
                ("bq", P), ("bk", P), ("bv", P), ("bo", P), ("ffn_norm", P),
                ("w_gate", OrcWeight), ("w_up", OrcWeight), ("w_down", OrcWeight),
                ("router", P), ("e_gate", P), ("e_up", P), ("e_down", P)]


class OrcModel(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("d_model", C.c_int), ("n_heads", C.c_int), ("n_kv_heads", C.c_int),
                ("head_dim", C.c_int), ("d_ff", C.c_int), ("vocab", C.c_int), ("max_ctx", C.c_int),
                ("rope_split_half", C.c_int), ("n_experts", C.c_int), ("n_experts_used", C.c_int),
                ("normalize_experts", C.c_int), ("eps", C.c_float), ("theta", C.c_float),
                ("embed", OrcWeight), ("layers", P), ("final_norm", P), ("lm_head", OrcWeight)]


def _ow(t):
    """(type, data ndarray, scales ndarray|None, rows, cols) -> OrcWeight."""
    type_, data, scales, rows, cols = t
    return OrcWeight(type_, data.ctypes.data, None if scales is None else scales.ctypes.data, rows, cols)


class OracleSession:
    """CachedLlamaSession restated: greedy single-token decode over a model
    given as host arrays (see ``overfit_b200.model`` for the weight dict)."""

    def __init__(self, cfg: dict, weights: dict, max_ctx: int):
        self._keep = []  # keep every array alive while C holds pointers
        L = lib()
        nl = cfg["n_layers"]
        layers = (OrcLayer * nl)()
        for i in range(nl):
            lw = weights["layers"][i]
            lay = layers[i]
            lay.attn_norm = lw["attn_norm"].ctypes.data
            lay.ffn_norm = lw["ffn_norm"].ctypes.data
            for nm in ("wq", "wk", "wv", "wo"):
                setattr(lay, nm, _ow(lw[nm]))
            for nm in ("bq", "bk", "bv", "bo"):
                v = lw.get(nm)
                setattr(lay, nm, None if v is None else v.ctypes.data)
            if "router" in lw:
                lay.router = lw["router"].ctypes.data
                ne = len(lw["experts"])
                eg, eu, ed = (OrcWeight * ne)(), (OrcWeight * ne)(), (OrcWeight * ne)()
                for e, ex in enumerate(lw["experts"]):
                    eg[e], eu[e], ed[e] = _ow(ex["gate"]), _ow(ex["up"]), _ow(ex["down"])
                self._keep += [eg, eu, ed]
                lay.e_gate, lay.e_up, lay.e_down = (C.addressof(eg), C.addressof(eu), C.addressof(ed))
            else:
                lay.w_gate, lay.w_up, lay.w_down = _ow(lw["gate"]), _ow(lw["up"]), _ow(lw["down"])
        m = OrcModel()
        for f in ("n_layers", "d_model", "n_heads", "n_kv_heads", "head_dim", "d_ff", "vocab"):
            setattr(m, f, cfg[f])
        m.max_ctx = max_ctx
        m.rope_split_half = int(cfg.get("rope_split_half", 0))
        m.n_experts = cfg.get("n_experts", 0)
        m.n_experts_used = cfg.get("n_experts_used", 0)
        m.normalize_experts = int(cfg.get("normalize_experts", 1))
        m.eps = cfg["eps"]
        m.theta = cfg["theta"]
        m.embed = _ow(weights["embed"])
        m.layers = C.addressof(layers)
        m.final_norm = weights["final_norm"].ctypes.data
        m.lm_head = _ow(weights["lm_head"])
        self._keep += [layers, m, weights]
        self.cfg = cfg
        self._m = m
        self._s = L.orc_session_create(C.byref(m), max_ctx)

    def decode(self, token: int, want_logits: bool = True):
        logits = np.empty(self.cfg["vocab"], np.float32) if want_logits else None
        rc = lib().orc_session_decode(self._s, int(token), _p(logits))
        if rc != 0:
            raise RuntimeError("oracle decode failed (cache full or bad token)")
        return logits

    def decode_layers(self, token: int, n_layers: int, with_logits: bool):
        logits = np.empty(self.cfg["vocab"], np.float32) if with_logits else None
        lib().orc_session_decode_layers(self._s, int(token), n_layers, int(with_logits), _p(logits))
        return logits

    def reset(self):
        lib().orc_session_reset(self._s)

    def set_kv_q8(self, on: bool = True):
        """KvCacheDType.Q8: per-vector int8 K/V + one scale each (set before
        the first token)."""
        lib().orc_session_set_kv_q8(self._s, int(on))

    def fill_context(self, n: int, seed: int = 7):
        """Timing support: n cached positions of N(0, 0.5) rows, position n."""
        if lib().orc_session_fill_context(self._s, int(n), int(seed)) != 0:
            raise ValueError("fill_context: n out of range or Q8 cache")

    def set_kv_fp16(self, on: bool = True):
        """Round cached K/V to fp16 as the GPU cache does (test switch)."""
        lib().orc_session_set_kv_fp16(self._s, int(on))

    @property
    def position(self) -> int:
        return lib().orc_session_position(self._s)

    def close(self):
        if self._s:
            lib().orc_session_destroy(self._s)
            self._s = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def expf_array(x: np.ndarray) -> np.ndarray:
    """MathF.Exp elementwise: the host C library's expf."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().orc_expf_array(x.ctypes.data, y.ctypes.data, x.size)
    return y


def q8kv_quantize(v: np.ndarray):
    """Q8KvQuant.Quantize: one vector -> (int8 values, scale)."""
    v = np.ascontiguousarray(v, dtype=np.float32)
    q = np.empty(v.size, np.int8)
    sc = lib().orc_q8kv_quantize(_p(v), v.size, _p(q))
    return q, np.float32(sc)


def attention_single_head_q8(q, kq, ks, vq, vs, scale) -> np.ndarray:
    """CachedAttentionKernel.ComputeSingleHeadQ8 over seq = len(ks) positions."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    kq = np.ascontiguousarray(kq, dtype=np.int8)
    vq = np.ascontiguousarray(vq, dtype=np.int8)
    ks = np.ascontiguousarray(ks, dtype=np.float32)
    vs = np.ascontiguousarray(vs, dtype=np.float32)
    hd, seq = q.size, ks.size
    out = np.empty(hd, np.float32)
    scr = np.empty(max(seq, 1), np.float32)
    lib().orc_attention_single_head_q8(_p(q), _p(kq), _p(ks), _p(vq), _p(vs), _p(out), _p(scr), seq, hd,
                                       float(scale))
    return out

