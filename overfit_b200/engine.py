"""Engine / session mirror of the reference's LLM runtime interfaces.

``CudaLlamaInferenceEngine`` and ``CudaLlamaSession`` follow
``ISlmInferenceEngine`` / ``ISlmSession`` (Contracts/ISlmInferenceEngine.cs:9,
Contracts/ISlmSession.cs:8) as ``CachedLlamaInferenceEngine`` /
``CachedLlamaSession`` implement them (Runtime/CachedLlamaInferenceEngine.cs:33,
Runtime/CachedLlamaSession.cs:26): reset, prefill, greedy next token, last
logits, position.  All device work happens inside libovf_cuda.so
(ovf_model_* / ovf_session_*); this module only marshals the tensor table.

Weights come in as a *model file* dict holding what a GGUF loader hands over
(host numpy arrays in on-disk formats), see ``tensor_table``.
``synthetic_model`` builds such a dict with random-init weights quantized by
the library's own device codecs (the bench's Llama-3-8B / Qwen2-0.5B shapes).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from ._lib import (TENSORS_PER_LAYER, TYPE_F32, TYPE_Q4_K, TYPE_Q6_K, TYPE_Q8_0, ModelConfig, OverfitRuntimeError,
                   Tensor, check)

LAYER_KEYS = ("attn_norm", "wq", "wk", "wv", "wo", "bq", "bk", "bv", "bo", "ffn_norm", "gate", "up", "down", "router")

# Benchmark model shapes (random-init, synthetic).  eps follows the reference,
# which uses 1e-6 for every GGUF model (Runtime/CachedLlamaInferenceEngine.cs:139).
LLAMA3_8B = dict(n_layers=32, d_model=4096, n_heads=32, n_kv_heads=8, head_dim=128, d_ff=14336, vocab=128256,
                 theta=500000.0, eps=1e-6, rope_split_half=0, tied=False, qkv_bias=False, scheme="q4_k_m")
QWEN2_05B = dict(n_layers=24, d_model=896, n_heads=14, n_kv_heads=2, head_dim=64, d_ff=4864, vocab=151936,
                 theta=1000000.0, eps=1e-6, rope_split_half=1, tied=True, qkv_bias=True, scheme="q8_0")

# Q4_K_M tensor map used for synthetic files (our choice: Q4_K for q/k/o/gate/up/embedding, Q6_K for v/down/output):
# Q6_K for attn_v, ffn_down and the output head, Q4_K elsewhere.
_Q4KM = dict(wq=TYPE_Q4_K, wk=TYPE_Q4_K, wv=TYPE_Q6_K, wo=TYPE_Q4_K, gate=TYPE_Q4_K, up=TYPE_Q4_K,
             down=TYPE_Q6_K, embed=TYPE_Q4_K, lm_head=TYPE_Q6_K)


def tensor_of(entry) -> tuple:
    """Normalizes a weight entry to (type, ndarray, rows, cols)."""
    if entry is None:
        return (-1, None, 0, 0)
    if isinstance(entry, np.ndarray):  # f32 vector
        return (TYPE_F32, np.ascontiguousarray(entry, dtype=np.float32), 1, entry.size)
    t, data, rows, cols = entry
    return (t, np.ascontiguousarray(data), rows, cols)


def moe_layer_entries(layer: dict) -> dict:
    """A Mixtral layer (``router`` [d_model x n_experts] F32 input-major,
    ``experts`` = [{gate, up, down}] in file formats) as the tensor table
    wants it: the experts' matrices back to back in one entry per kind."""
    if "experts" not in layer:
        return layer
    out = dict(layer)
    r = np.ascontiguousarray(layer["router"], dtype=np.float32)
    out["router"] = (TYPE_F32, r.reshape(-1), r.shape[0], r.shape[1])
    for k in ("gate", "up", "down"):
        parts = [tensor_of(ex[k]) for ex in layer["experts"]]
        t = parts[0][0]
        if any(p[0] != t for p in parts):
            raise ValueError(f"experts' {k} matrices must share a type")
        out[k] = (t, np.concatenate([p[1].reshape(-1) for p in parts]), sum(p[2] for p in parts), parts[0][3])
    return out


def tensor_table(cfg: dict, model_file: dict):
    """Builds the ovf_tensor table (include/ovf.h) and the list of arrays it
    points into (keep it alive until ovf_model_create returns)."""
    nl = cfg["n_layers"]
    table = (Tensor * (nl * TENSORS_PER_LAYER + 3))()
    keep = []
    for l, layer in enumerate(model_file["layers"]):
        layer = moe_layer_entries(layer)
        for j, key in enumerate(LAYER_KEYS):
            t, data, rows, cols = tensor_of(layer.get(key))
            if data is not None:
                keep.append(data)
            table[l * TENSORS_PER_LAYER + j] = Tensor(t, None if data is None else data.ctypes.data, rows, cols)
    base = nl * TENSORS_PER_LAYER
    for j, key in enumerate(("embed", "final_norm", "lm_head")):
        t, data, rows, cols = tensor_of(model_file.get(key))
        if data is not None:
            keep.append(data)
        table[base + j] = Tensor(t, None if data is None else data.ctypes.data, rows, cols)
    return table, keep


def model_config(cfg: dict) -> ModelConfig:
    return ModelConfig(cfg["n_layers"], cfg["d_model"], cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"],
                       cfg["d_ff"], cfg["vocab"], int(cfg.get("rope_split_half", 0)), cfg.get("n_experts", 0),
                       cfg.get("n_experts_used", 0), int(cfg.get("normalize_experts", 1)), float(cfg["eps"]),
                       float(cfg["theta"]))


def tp_check(cfg: dict, world: int) -> None:
    """The shapes tensor parallelism over `world` ranks accepts (the checks
    ovf_model_create_tp makes): KV heads, FFN rows in 256-blocks and the
    vocabulary split evenly; MoE models split their experts whole (expert
    parallelism, attention still split by heads)."""
    if world < 1 or world > 8:
        raise ValueError("tensor parallelism: 1..8 ranks")
    if world == 1:
        return
    if cfg["n_kv_heads"] % world:
        raise ValueError(f"tensor parallelism: {cfg['n_kv_heads']} KV heads do not split over {world} ranks")
    if cfg.get("n_experts", 0):
        # expert parallel: rank r owns the experts e with e % world == r
        if cfg["n_experts"] % world:
            raise ValueError(f"expert parallelism: {cfg['n_experts']} experts do not split over {world} ranks")
    elif cfg["d_ff"] % world or (cfg["d_ff"] // world) % 256:
        raise ValueError(f"tensor parallelism: d_ff {cfg['d_ff']} must split into multiples of 256")
    if cfg["vocab"] % world:
        raise ValueError(f"tensor parallelism: vocab {cfg['vocab']} must split evenly")


def exchange_handles(handle: bytes, group=None) -> bytes:
    """All ranks' exchange-arena handles, concatenated in rank order, through
    the torch.distributed process group (host-side plumbing; the data path
    itself is peer memory)."""
    import torch.distributed as dist

    gathered = [None] * dist.get_world_size(group)
    dist.all_gather_object(gathered, bytes(handle), group=group)
    if any(len(h) != _lib.TP_HANDLE_BYTES for h in gathered):
        raise ValueError("tensor parallelism: malformed exchange handle")
    return b"".join(gathered)


class CudaLlamaInferenceEngine:
    """GPU engine behind ISlmInferenceEngine (weights resident on one device).

    ``tp_group``: a torch.distributed process group of one process per GPU;
    with more than one rank the model is split tensor-parallel (every rank
    passes the full model file, uploads its shard and connects to the other
    ranks' exchange buffers) and every rank must then make the same session
    calls in the same order."""

    def __init__(self, cfg: dict, model_file: dict, device: int = 0, tp_group=None):
        self.cfg = dict(cfg)
        self.device = device
        lib = _lib.load()
        table, keep = tensor_table(cfg, model_file)
        mc = model_config(cfg)
        handle = C.c_void_p()
        world, rank = 1, 0
        if tp_group is not None:
            import torch.distributed as dist
            world, rank = dist.get_world_size(tp_group), dist.get_rank(tp_group)
        self.tp_world, self.tp_rank = world, rank
        if world == 1:
            check(lib.ovf_model_create(device, C.byref(mc), table, len(table), C.byref(handle)), "ovf_model_create")
        else:
            tp_check(cfg, world)
            check(lib.ovf_model_create_tp(device, C.byref(mc), table, len(table), rank, world, C.byref(handle)),
                  "ovf_model_create_tp")
        del keep
        self._h = handle
        if world > 1:
            mine = (C.c_char * _lib.TP_HANDLE_BYTES)()
            check(lib.ovf_model_tp_export(self._h, mine), "tp_export")
            allh = exchange_handles(bytes(mine), tp_group)
            buf = (C.c_char * len(allh)).from_buffer_copy(allh)
            check(lib.ovf_model_tp_connect(self._h, buf), "tp_connect")

    @property
    def weight_bytes(self) -> int:
        """Bytes of weights one decode step streams from HBM."""
        return int(_lib.load().ovf_model_weight_bytes(self._h))

    @property
    def vocabulary_size(self) -> int:
        return self.cfg["vocab"]

    def create_session(self, max_context: int, kv_cache_dtype: str = "f32") -> "CudaLlamaSession":
        """CreateSession(maxContextLength, kvCacheDType): "f32" (the reference's
        default, bit-exact attention), "q8" (the reference's Q8 cache, its
        exact ComputeSingleHeadQ8 order) or "f16" (no reference counterpart)."""
        return CudaLlamaSession(self, max_context, kv_cache_dtype)

    def decode_batch(self, sessions, tokens, want_logits: bool = True) -> np.ndarray:
        """One DecodeToken in each session (distinct sessions of this engine),
        batched on the device; returns the argmax per session.  Each session
        ends exactly as its own decode() would leave it."""
        n = len(sessions)
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        if toks.size != n:
            raise ValueError("one token per session")
        handles = (C.c_void_p * n)(*[s._h for s in sessions])
        am = np.empty(n, np.int32)
        logits = np.empty((n, self.cfg["vocab"]), np.float32) if want_logits else None
        check(_lib.load().ovf_session_decode_batch(handles, n, toks.ctypes.data,
                                                   logits.ctypes.data if want_logits else None, am.ctypes.data),
              "DecodeBatch")
        for i, s in enumerate(sessions):
            if want_logits:
                s._logits[:] = logits[i]
            s._have_logits = want_logits
        return am

    def close(self):
        if self._h:
            _lib.load().ovf_model_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class CudaLlamaSession:
    """ISlmSession over the device-resident decode loop (greedy sampling on
    the device; logits are copied out only when asked for)."""

    KV_DTYPES = {"f32": 0, "q8": 1, "f16": 2}

    def __init__(self, engine: CudaLlamaInferenceEngine, max_context: int, kv_cache_dtype: str = "f32"):
        self.engine = engine
        self.max_context_length = max_context
        if kv_cache_dtype not in self.KV_DTYPES:
            raise ValueError(f"kv_cache_dtype must be one of {sorted(self.KV_DTYPES)}")
        self.kv_cache_dtype = kv_cache_dtype
        h = C.c_void_p()
        check(_lib.load().ovf_session_create_kv(engine._h, max_context, self.KV_DTYPES[kv_cache_dtype], C.byref(h)),
              "ovf_session_create")
        self._h = h
        self._logits = np.zeros(engine.cfg["vocab"], np.float32)
        self._have_logits = False
        self._last_argmax = -1
        self._spec_ema = 0.0      # committed tokens per verify (EMA); starts gated
        self._spec_countdown = 0  # the first gated step probes

    @property
    def vocabulary_size(self) -> int:
        return self.engine.cfg["vocab"]

    @property
    def current_position(self) -> int:
        return int(_lib.load().ovf_session_position(self._h))

    def reset(self, prompt_tokens=None) -> None:
        """ISlmSession.Reset / Reset(prompt)."""
        check(_lib.load().ovf_session_reset(self._h), "Reset")
        self._have_logits = False
        if prompt_tokens is not None:
            self.prefill(prompt_tokens)

    def prefill(self, prompt_tokens) -> int:
        """CachedLlamaSession.Prefill; returns the greedy next token and keeps
        the last logits.  Prompts of 16 tokens or more take the batched path
        (PrefillBatchedQuant, bit-identical to the single-token loop, which
        ``disable_batched_prefill_for_parity`` forces)."""
        toks = np.ascontiguousarray(np.asarray(prompt_tokens, dtype=np.int32))
        if toks.size == 0:
            return -1
        am = C.c_int32()
        check(_lib.load().ovf_session_prefill(self._h, toks.ctypes.data, toks.size, self._logits.ctypes.data,
                                              C.byref(am)), "Prefill")
        self._have_logits = True
        self._last_argmax = am.value
        return am.value

    def decode(self, token: int, want_logits: bool = True) -> int:
        """Feeds one token (CachedLlamaSession.DecodeToken); returns argmax."""
        am = C.c_int32()
        ptr = self._logits.ctypes.data if want_logits else None
        check(_lib.load().ovf_session_decode(self._h, int(token), ptr, C.byref(am)), "DecodeToken")
        self._have_logits = want_logits
        self._last_argmax = am.value
        return am.value

    def generate_greedy(self, n_steps: int) -> np.ndarray:
        """n x GenerateNextToken with greedy sampling; the argmax is fed back on
        the device.  Returns the sampled tokens (each one was decoded)."""
        if not self._have_logits and self.current_position == 0:
            raise OverfitRuntimeError("Session is empty. Call Reset with at least one prompt token first.")
        out = np.empty(n_steps, np.int32)
        check(_lib.load().ovf_session_generate_greedy(self._h, n_steps, out.ctypes.data), "GenerateNextToken")
        self._have_logits = False
        return out

    @property
    def disable_batched_prefill_for_parity(self) -> bool:
        """CachedLlamaSession.DisableBatchedPrefillForParity (:808)."""
        return getattr(self, "_prefill_single", False)

    @disable_batched_prefill_for_parity.setter
    def disable_batched_prefill_for_parity(self, on: bool) -> None:
        check(_lib.load().ovf_session_set_option(self._h, _lib.OPT_PREFILL_SINGLE, int(bool(on))), "set_option")
        self._prefill_single = bool(on)

    # ---------------------------------------------- speculative decoding
    def verify(self, tokens, want_logits: bool = False):
        """The speculative verify forward (GenerateSpeculativeCore :468-477):
        appends `tokens` in one batched forward and returns the argmax of
        every row (and the [n, vocab] logits when asked)."""
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        n = toks.size
        am = np.empty(n, np.int32)
        lg = np.empty((n, self.engine.cfg["vocab"]), np.float32) if want_logits else None
        check(_lib.load().ovf_session_verify(self._h, toks.ctypes.data, n, None if lg is None else lg.ctypes.data,
                                             am.ctypes.data), "Verify")
        self._have_logits = False
        return (am, lg) if want_logits else am

    def rollback_to(self, length: int) -> None:
        """CachedLlamaSession.RollbackTo (:318) -> KeyValueCache.TruncateTo."""
        check(_lib.load().ovf_session_truncate(self._h, int(length)), "TruncateTo")
        self._have_logits = False

    def generate_speculative(self, history, max_draft: int = 4, ngram_min: int = 1, ngram_max: int = 3) -> list:
        """Greedy GenerateSpeculative (Runtime/CachedLlamaSession.cs:335-530):
        t0 = argmax of the current logits; prompt-lookup drafts from
        history + [t0]; one batched verify of [t0, drafts...]; drafts are
        accepted while they equal the verify row's argmax; the rejected
        drafts' rows are rolled back and the correction (or bonus) token is
        decoded so the session holds its logits.  Returns the committed tokens
        (>= 1): greedy output identical to single-token steps.  The adaptive
        gate (EMA of committed tokens per verify, probe every 64 steps) follows
        the reference."""
        if self.current_position == 0:
            raise OverfitRuntimeError("Session is empty. Call Reset with a prompt first.")
        if max_draft <= 0:
            raise ValueError("maxDraft must be positive")
        t0 = int(np.argmax(self.get_last_logits())) if self._have_logits else self._last_argmax
        gated = self._spec_ema < 3.0
        probe = False
        if gated:
            if self._spec_countdown > 0:
                self._spec_countdown -= 1
            else:
                probe = True
                self._spec_countdown = 64
        draft = []
        if not gated or probe:
            draft = prompt_lookup_draft(list(history) + [t0], max_draft, ngram_min, ngram_max)
        base = self.current_position
        if not draft or base + 1 + len(draft) + 1 > self.max_context_length:
            self._last_argmax = self.decode(t0)
            return [t0]
        am = self.verify([t0] + draft)
        committed, accepted, correction = [t0], 0, -1
        for j, d in enumerate(draft):
            if int(am[j]) == d:
                committed.append(d)
                accepted += 1
            else:
                correction = int(am[j])
                break
        if correction < 0:
            correction = int(am[len(draft)])
        self.rollback_to(base + 1 + accepted)
        committed.append(correction)
        self._last_argmax = self.decode(correction)
        self._spec_ema = 0.5 * len(committed) + 0.5 * self._spec_ema
        return committed

    # ---------------------------------------------------- prefix KV reuse
    def save_prefix(self) -> dict:
        """CachedLlamaSession.SavePrefix (:231): the live KV rows packed
        [layer][kv_head][position][head_dim] (F32, or fp16 for an fp16 cache)."""
        nbytes = int(_lib.load().ovf_session_prefix_bytes(self._h))
        k = np.empty(max(nbytes, 1), np.uint8)
        v = np.empty(max(nbytes, 1), np.uint8)
        n = C.c_int32()
        check(_lib.load().ovf_session_save_prefix(self._h, k.ctypes.data, v.ctypes.data, C.byref(n)), "SavePrefix")
        return dict(keys=k[:nbytes], values=v[:nbytes], length=n.value, kv=self.kv_cache_dtype)

    def restore_prefix(self, prefix: dict) -> None:
        """CachedLlamaSession.RestorePrefix (:242): a copy, not a forward pass."""
        if prefix["kv"] != self.kv_cache_dtype:
            raise ValueError("Snapshot shape does not match this cache")
        check(_lib.load().ovf_session_restore_prefix(self._h, prefix["keys"].ctypes.data,
                                                     prefix["values"].ctypes.data, int(prefix["length"])),
              "RestorePrefix")
        self._have_logits = False

    @property
    def stream_handle(self) -> int:
        """cudaStream_t of the session (for event timing)."""
        return int(_lib.load().ovf_session_stream(self._h) or 0)

    def get_last_logits(self) -> np.ndarray:
        if not self._have_logits:
            raise OverfitRuntimeError("no logits: decode with want_logits=True first")
        return self._logits.copy()

    def close(self):
        if self._h:
            _lib.load().ovf_session_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def prompt_lookup_draft(history, max_draft: int, ngram_min: int = 1, ngram_max: int = 3) -> list:
    """PromptLookupDrafter.Draft (Runtime/PromptLookupDrafter.cs:24-74): the
    longest suffix n-gram (ngram_max down to ngram_min) matched against its
    most recent earlier occurrence; proposes the tokens that followed it."""
    if max_draft <= 0:
        return []
    if ngram_min <= 0:
        raise ValueError("ngramMin must be positive")
    ngram_max = max(ngram_max, ngram_min)
    n_hist = len(history)
    for n in range(min(ngram_max, n_hist - 1), ngram_min - 1, -1):
        suffix = history[n_hist - n:]
        for i in range(n_hist - n - 1, -1, -1):
            if history[i:i + n] == suffix:
                follow = i + n
                return list(history[follow:follow + min(max_draft, n_hist - follow)])
    return []


# ------------------------------------------------------------- synthetic
def synthetic_model(cfg: dict, seed: int = 1, device: int = 0, std: float = 0.02, n_layers: int | None = None):
    """Random-init model file with the given shape, N(0, std) weights drawn
    on the device (torch generator, `seed`) and quantized by the library's
    device encoders (Q4_K: the reference's GgmlQuant scheme; Q6_K / Q8_0:
    ours).  Norm weights are 1 (the usual RMSNorm init), biases N(0, std).
    Returns host numpy arrays in on-disk formats."""
    import torch

    from .kernels import GgmlQuant

    dev = torch.device("cuda", device)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    nl = cfg["n_layers"] if n_layers is None else n_layers
    D, H, KVH, hd, FF, V = (cfg[k] for k in ("d_model", "n_heads", "n_kv_heads", "head_dim", "d_ff", "vocab"))
    scheme = cfg.get("scheme", "q4_k_m")

    def qtype(key):
        return _Q4KM[key] if scheme == "q4_k_m" else TYPE_Q8_0

    def mat(rows, cols, t):
        chunks = []
        step = max(1, (1 << 27) // cols)
        for r0 in range(0, rows, step):
            r = min(step, rows - r0)
            w = torch.randn(r, cols, generator=g, device=dev, dtype=torch.float32) * std
            if t == TYPE_Q4_K:
                q = GgmlQuant.quantize_q4_k(w, cols, r)
            elif t == TYPE_Q6_K:
                q = GgmlQuant.quantize_q6_k(w, cols, r)
            elif t == TYPE_Q8_0:
                q = GgmlQuant.quantize_q8_0(w)
            else:
                q = w
            chunks.append(q.reshape(-1).cpu())
        data = torch.cat(chunks).numpy()
        return (t, data, rows, cols)

    def vec(n):
        return (torch.randn(n, generator=g, device=dev) * std).cpu().numpy().astype(np.float32)

    layers = []
    for _ in range(nl):
        L = dict(attn_norm=np.ones(D, np.float32), ffn_norm=np.ones(D, np.float32),
                 wq=mat(H * hd, D, qtype("wq")), wk=mat(KVH * hd, D, qtype("wk")), wv=mat(KVH * hd, D, qtype("wv")),
                 wo=mat(D, H * hd, qtype("wo")), gate=mat(FF, D, qtype("gate")), up=mat(FF, D, qtype("up")),
                 down=mat(D, FF, qtype("down")))
        if cfg.get("qkv_bias"):
            L.update(bq=vec(H * hd), bk=vec(KVH * hd), bv=vec(KVH * hd))
        layers.append(L)
    model = dict(layers=layers, embed=mat(V, D, qtype("embed")), final_norm=np.ones(D, np.float32))
    model["lm_head"] = None if cfg.get("tied") else mat(V, D, qtype("lm_head"))
    return model
