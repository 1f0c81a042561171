"""Model-level parity on the GPU: the whole decode step (engine/session over
the C ABI) against the CPU restatement of CachedLlamaSession on the same
seeded synthetic weights.

Bar: logits within 1e-2 relative L2 at every step and identical greedy
tokens for 32 decode steps; the GPU path keeps the reference's operation
order throughout, so the tests require bit-identical logits (the fp16 and Q8
caches against the restatement run with the same cache type).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from model_helpers import TINY_LLAMA, TINY_QWEN, make_model_file, oracle_session  # noqa: E402

REL_L2 = 1e-2


@pytest.fixture(scope="module")
def E():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from overfit_b200 import build, engine
    build.build()
    return engine


def rel_l2(a, b):
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


@pytest.mark.parametrize("cfg", [TINY_LLAMA, TINY_QWEN], ids=["llama_q4km", "qwen2_q8_0"])
def test_greedy_parity_32_steps(E, orc, cfg):
    mf = make_model_file(cfg, seed=1)
    eng = E.CudaLlamaInferenceEngine(cfg, mf)
    sess = eng.create_session(128)
    ref = oracle_session(cfg, mf, 128)
    prompt = np.random.default_rng(7).integers(0, cfg["vocab"], 20)
    # prefill: the reference's single-token path; logits of the last token
    tok = sess.prefill(prompt)
    for t in prompt:
        lg_ref = ref.decode(int(t))
    assert rel_l2(sess.get_last_logits(), lg_ref) < REL_L2
    assert tok == int(np.argmax(lg_ref))
    # 32 greedy steps, token by token with logits
    for step in range(32):
        nxt_ref = int(np.argmax(lg_ref))
        assert tok == nxt_ref, f"greedy token differs at step {step}"
        tok = sess.decode(tok)
        lg_ref = ref.decode(nxt_ref)
        r = rel_l2(sess.get_last_logits(), lg_ref)
        assert r < REL_L2, (step, r)
    assert sess.current_position == 20 + 32


def test_device_greedy_loop_matches_host_loop(E):
    """generate_greedy (argmax fed back on the device, graph replay) produces
    the same tokens as decoding them one by one from the host."""
    cfg = TINY_LLAMA
    mf = make_model_file(cfg, seed=2)
    eng = E.CudaLlamaInferenceEngine(cfg, mf)
    prompt = [5, 17, 99, 3]
    a = eng.create_session(64)
    first = a.prefill(prompt)
    dev_tokens = a.generate_greedy(24)
    b = eng.create_session(64)
    tok = b.prefill(prompt)
    assert tok == first
    host_tokens = []
    for _ in range(24):
        host_tokens.append(tok)
        tok = b.decode(tok)
    np.testing.assert_array_equal(dev_tokens, host_tokens)


def test_session_edge_cases(E):
    cfg = TINY_QWEN
    mf = make_model_file(cfg, seed=3)
    eng = E.CudaLlamaInferenceEngine(cfg, mf)
    s = eng.create_session(8)
    from overfit_b200._lib import OverfitRuntimeError
    with pytest.raises(OverfitRuntimeError):
        s.generate_greedy(1)  # empty session (CachedLlamaSession.cs:274-278)
    assert s.prefill([]) == -1
    with pytest.raises(ValueError):
        s.decode(cfg["vocab"])  # token out of range
    s.prefill([1, 2, 3, 4, 5, 6])
    s.generate_greedy(2)
    assert s.current_position == 8
    with pytest.raises(ValueError):
        s.decode(1)  # KV cache full (ContextLength reached)
    s.reset([1, 2])
    assert s.current_position == 2
    # reset then the same prompt reproduces the same logits
    l1 = s.get_last_logits()
    s.reset([1, 2])
    np.testing.assert_array_equal(s.get_last_logits(), l1)


@pytest.mark.parametrize("cfg", [TINY_LLAMA, TINY_QWEN], ids=["llama_q4km", "qwen2_q8_0"])
def test_fp16_kv_session_bit_exact(E, orc, cfg):
    """The fp16-KV session (the benchmark config's cache, no reference
    counterpart; attended in ComputeSingleHead's order on the widened values)
    against the restatement with its cache rounded to fp16 the same way:
    bit-identical logits at every step and identical greedy tokens for 32
    steps."""
    mf = make_model_file(cfg, seed=1)
    eng = E.CudaLlamaInferenceEngine(cfg, mf)
    sess = eng.create_session(128, "f16")
    ref = oracle_session(cfg, mf, 128)
    ref.set_kv_fp16(True)
    prompt = np.random.default_rng(7).integers(0, cfg["vocab"], 20)
    tok = sess.prefill(prompt)
    for t in prompt:
        lg_ref = ref.decode(int(t))
    np.testing.assert_array_equal(sess.get_last_logits(), lg_ref)
    for step in range(32):
        nxt_ref = int(np.argmax(lg_ref))
        assert tok == nxt_ref, f"greedy token differs at step {step}"
        tok = sess.decode(tok)
        lg_ref = ref.decode(nxt_ref)
        np.testing.assert_array_equal(sess.get_last_logits(), lg_ref, err_msg=f"step {step}")


@pytest.mark.parametrize("cfg", [TINY_LLAMA, TINY_QWEN], ids=["llama_q4km", "qwen2_q8_0"])
def test_q8_kv_session_bit_exact(E, orc, cfg):
    """KvCacheDType.Q8 session (Q8KvQuant on append, ComputeSingleHeadQ8 on
    attend) against the restatement's Q8 session: bit-identical logits at
    every step and identical greedy tokens."""
    mf = make_model_file(cfg, seed=1)
    eng = E.CudaLlamaInferenceEngine(cfg, mf)
    sess = eng.create_session(128, "q8")
    ref = oracle_session(cfg, mf, 128)
    ref.set_kv_q8(True)
    prompt = np.random.default_rng(7).integers(0, cfg["vocab"], 20)
    tok = sess.prefill(prompt)
    for t in prompt:
        lg_ref = ref.decode(int(t))
    np.testing.assert_array_equal(sess.get_last_logits(), lg_ref)
    for step in range(16):
        nxt_ref = int(np.argmax(lg_ref))
        assert tok == nxt_ref, f"greedy token differs at step {step}"
        tok = sess.decode(tok)
        lg_ref = ref.decode(nxt_ref)
        np.testing.assert_array_equal(sess.get_last_logits(), lg_ref, err_msg=f"step {step}")



def oracle_for(cfg, mf, max_ctx, kv):
    ref = oracle_session(cfg, mf, max_ctx)
    if kv == "f16":
        ref.set_kv_fp16(True)
    elif kv == "q8":
        ref.set_kv_q8(True)
    return ref


@pytest.mark.parametrize("kv", ["f32", "q8", "f16"])
@pytest.mark.parametrize("cfg", [TINY_LLAMA, TINY_QWEN], ids=["llama_q4km", "qwen2_q8_0"])
def test_batched_prefill_bit_exact_vs_restatement(E, orc, cfg, kv):
    """PrefillBatchedQuant (two 256-row chunks for 300 tokens, then a second
    prefill of 40 from a non-zero position) against the restatement decoding
    the same tokens one at a time: the same last logits bit for bit, and the
    same greedy continuation; the parity switch (single-token loop) agrees
    too."""
    mf = make_model_file(cfg, seed=3)
    eng = E.CudaLlamaInferenceEngine(cfg, mf)
    rng = np.random.default_rng(23)
    p1, p2 = rng.integers(0, cfg["vocab"], 300), rng.integers(0, cfg["vocab"], 40)
    ref = oracle_for(cfg, mf, 384, kv)
    for t in p1:
        r1 = ref.decode(int(t))
    for t in p2:
        r2 = ref.decode(int(t))
    for single in (False, True):
        s = eng.create_session(384, kv)
        s.disable_batched_prefill_for_parity = single
        s.prefill(p1)
        np.testing.assert_array_equal(s.get_last_logits(), r1, err_msg=f"single={single}")
        tok = s.prefill(p2)
        np.testing.assert_array_equal(s.get_last_logits(), r2, err_msg=f"single={single}")
        if not single:
            lg = r2
            for i in range(8):
                nxt = int(np.argmax(lg))
                assert tok == nxt, i
                tok = s.decode(tok)
                lg = ref.decode(nxt)
                np.testing.assert_array_equal(s.get_last_logits(), lg, err_msg=f"decode step {i}")
            assert s.current_position == 340 + 8
        s.close()
    eng.close()


@pytest.mark.parametrize("cfg", [TINY_LLAMA, TINY_QWEN], ids=["llama_q4km", "qwen2_q8_0"])
def test_decode_batch_bit_exact_vs_restatement(E, orc, cfg):
    """Concurrent sessions decoded as one batch (weights read once for all of
    them), at different positions with F32, Q8 and fp16 caches, against one
    restatement session each: the same logits bit for bit and the same greedy
    tokens; the device greedy loop then continues identically."""
    mf = make_model_file(cfg, seed=5)
    eng = E.CudaLlamaInferenceEngine(cfg, mf)
    rng = np.random.default_rng(31)
    prompts = [rng.integers(0, cfg["vocab"], n) for n in (3, 20, 7, 1)]
    kvs = ["f32", "q8", "f16", "f32"]
    batch = [eng.create_session(96, kv) for kv in kvs]
    refs = [oracle_for(cfg, mf, 96, kv) for kv in kvs]
    tb = [s.prefill(p) for s, p in zip(batch, prompts)]
    lr = []
    for r, p in zip(refs, prompts):
        for t in p:
            lg = r.decode(int(t))
        lr.append(lg)
    assert tb == [int(np.argmax(lg)) for lg in lr]
    for step in range(6):
        tb = list(eng.decode_batch(batch, tb))
        lr = [r.decode(int(np.argmax(lg))) for r, lg in zip(refs, lr)]
        assert tb == [int(np.argmax(lg)) for lg in lr], step
        for a, lg in zip(batch, lr):
            np.testing.assert_array_equal(a.get_last_logits(), lg, err_msg=f"step {step}")
    for a, r, lg in zip(batch, refs, lr):
        toks = a.generate_greedy(4)
        want = []
        for _ in range(4):
            want.append(int(np.argmax(lg)))
            lg = r.decode(want[-1])
        np.testing.assert_array_equal(toks, want)
    for s in batch:
        s.close()
    eng.close()


@pytest.mark.parametrize("kv", ["f32", "f16"])
def test_verify_rows_bit_exact(E, orc, kv):
    """The speculative verify forward: every row's logits equal the
    restatement's single-token decode of the same tokens, and the session
    then continues like one that decoded them one at a time."""
    cfg = TINY_LLAMA
    mf = make_model_file(cfg, seed=8)
    eng = E.CudaLlamaInferenceEngine(cfg, mf)
    s = eng.create_session(64, kv)
    ref = oracle_for(cfg, mf, 64, kv)
    prompt = [11, 22, 33, 44, 55]
    s.prefill(prompt)
    for t in prompt:
        ref.decode(t)
    rows = [7, 1999, 3, 3, 250]
    am, lg = s.verify(rows, want_logits=True)
    for j, t in enumerate(rows):
        r = ref.decode(t)
        np.testing.assert_array_equal(lg[j], r, err_msg=f"row {j}")
        assert am[j] == int(np.argmax(r))
    assert s.current_position == 10
    first = int(np.argmax(r))
    np.testing.assert_array_equal(s.generate_greedy(3), [first] + _greedy(ref, first, 2))
    s.close()
    eng.close()


def _greedy(ref, tok, n):
    out = []
    for _ in range(n):
        lg = ref.decode(tok)
        tok = int(np.argmax(lg))
        out.append(tok)
    return out


@pytest.mark.parametrize("kv", ["f32", "f16"])
def test_speculative_greedy_matches_single_token_greedy(E, orc, kv):
    """GenerateSpeculative (prompt-lookup drafts, one batched verify, rollback
    of rejected drafts, correction decoded) commits exactly the tokens plain
    greedy decoding produces, checked against the restatement; drafting is
    forced on (gate open) so both accepted and rejected drafts occur."""
    cfg = TINY_LLAMA
    mf = make_model_file(cfg, seed=9)
    eng = E.CudaLlamaInferenceEngine(cfg, mf)
    s = eng.create_session(160, kv)
    ref = oracle_for(cfg, mf, 160, kv)
    prompt = [5, 6, 7, 8] * 6
    s.prefill(prompt)
    for t in prompt:
        lg = ref.decode(t)
    want = []
    tok = int(np.argmax(lg))
    for _ in range(60):
        want.append(tok)
        lg = ref.decode(tok)
        tok = int(np.argmax(lg))
    history = list(prompt)
    got, verifies = [], 0
    while len(got) < 48:
        s._spec_ema = 10.0  # keep the adaptive gate open
        pos0 = s.current_position
        c = s.generate_speculative(history, max_draft=4)
        verifies += len(c) > 1 or s.current_position - pos0 > 1
        got += c
        history += c
    np.testing.assert_array_equal(got[:48], want[:48])
    assert verifies > 0
    s.close()
    eng.close()


@pytest.mark.parametrize("kv", ["f32", "f16"])
def test_prefix_save_restore_and_truncate(E, orc, kv):
    """SavePrefix / RestorePrefix into another session, and TruncateTo: the
    continuation's logits equal the restatement's that decoded prefix +
    continuation from scratch, bit for bit."""
    cfg = TINY_QWEN
    mf = make_model_file(cfg, seed=10)
    eng = E.CudaLlamaInferenceEngine(cfg, mf)
    rng = np.random.default_rng(3)
    pre, turn, junk = (rng.integers(0, cfg["vocab"], n) for n in (40, 12, 9))
    ref = oracle_for(cfg, mf, 96, kv)
    for t in list(pre) + list(turn):
        r = ref.decode(int(t))
    a = eng.create_session(96, kv)
    a.prefill(pre)
    snap = a.save_prefix()
    assert snap["length"] == 40
    b = eng.create_session(80, kv)
    b.prefill(junk)
    b.restore_prefix(snap)
    assert b.current_position == 40
    b.prefill(turn)
    np.testing.assert_array_equal(b.get_last_logits(), r)
    a.prefill(junk)
    a.rollback_to(40)
    a.prefill(turn)
    np.testing.assert_array_equal(a.get_last_logits(), r)
    with pytest.raises(ValueError):
        a.rollback_to(a.current_position + 1)
    q = eng.create_session(64, "q8")
    q.prefill(junk)
    with pytest.raises(NotImplementedError):
        q.save_prefix()
    for x in (a, b, q):
        x.close()
    eng.close()


@pytest.mark.parametrize("kv", ["f32", "f16"])
def test_moe_greedy_parity_bit_exact(E, orc, kv):
    """Mixtral-style MoE (router top-2 with softmax over the pair, experts'
    SwiGLU combined in top-k order) decoded on the device, the routed expert
    picked inside the CUDA graph, against the restatement: bit-identical
    logits after a 20-token prompt (batched prefill: rows grouped per expert)
    and for 32 greedy steps."""
    from model_helpers import TINY_MIXTRAL
    cfg = TINY_MIXTRAL
    mf = make_model_file(cfg, seed=12)
    eng = E.CudaLlamaInferenceEngine(cfg, mf)
    sess = eng.create_session(96, kv)
    ref = oracle_for(cfg, mf, 96, kv)
    prompt = np.random.default_rng(4).integers(0, cfg["vocab"], 20)
    tok = sess.prefill(prompt)
    for t in prompt:
        lg_ref = ref.decode(int(t))
    np.testing.assert_array_equal(sess.get_last_logits(), lg_ref)
    for step in range(32):
        nxt_ref = int(np.argmax(lg_ref))
        assert tok == nxt_ref, f"greedy token differs at step {step}"
        tok = sess.decode(tok)
        lg_ref = ref.decode(nxt_ref)
        np.testing.assert_array_equal(sess.get_last_logits(), lg_ref, err_msg=f"step {step}")
    # the device greedy loop (graph replay with the routing on the device)
    want = []
    t = int(np.argmax(lg_ref))
    for _ in range(8):
        want.append(t)
        t = int(np.argmax(ref.decode(t)))
    np.testing.assert_array_equal(sess.generate_greedy(8), want)
    sess.close()
    eng.close()


def test_moe_decode_batch_bit_exact(E, orc):
    """MoE sessions decoded as one batch (rows grouped per expert) against
    the restatement, bit for bit."""
    from model_helpers import TINY_MIXTRAL
    cfg = TINY_MIXTRAL
    mf = make_model_file(cfg, seed=13)
    eng = E.CudaLlamaInferenceEngine(cfg, mf)
    rng = np.random.default_rng(6)
    prompts = [rng.integers(0, cfg["vocab"], n) for n in (5, 17, 2)]
    batch = [eng.create_session(64, "f32") for _ in prompts]
    refs = [oracle_for(cfg, mf, 64, "f32") for _ in prompts]
    toks = [s.prefill(p) for s, p in zip(batch, prompts)]
    lr = []
    for r, p in zip(refs, prompts):
        for t in p:
            lg = r.decode(int(t))
        lr.append(lg)
    for step in range(5):
        toks = list(eng.decode_batch(batch, toks))
        lr = [r.decode(int(np.argmax(lg))) for r, lg in zip(refs, lr)]
        for a, lg in zip(batch, lr):
            np.testing.assert_array_equal(a.get_last_logits(), lg, err_msg=f"step {step}")
    for s in batch:
        s.close()
    eng.close()
