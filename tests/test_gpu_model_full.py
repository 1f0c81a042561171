"""Whole-model parity at the benchmark shapes, against the CPU restatement
with the reference's own exp (the host C library's expf, MathF.Exp).

* Qwen2-0.5B (24 layers, d 896, 14/2 heads, vocab 151936, tied Q8_0
  embeddings, q/k/v biases) — the Qwen2 config: 128-token prompt, 32 greedy
  steps, F32 KV cache (the reference's default).
* Llama-3-8B (32 layers, d 4096, 32/8 heads, vocab 128256, Q4_K_M) — the
  benchmark's decode config: fp16 KV cache (the timed session) against the
  restatement with an fp16-rounded cache, and the F32 cache; a 256-token
  prompt and 32 greedy steps by default (OVF_FULL_PROMPT=2048 runs the
  config's full prompt; the CPU restatement then needs minutes).

Bar (north star): logits within 1e-2 relative L2 at every step and identical
greedy tokens for 32 steps.  Every session is also required to be
bit-identical (the fp16 cache against the restatement with its cache rounded
to fp16), which is what the GPU path is built to be: random-init models of
this depth amplify a single differently rounded value into percent-level
logit differences within a few hundred tokens, so only the reference's exact
operation order holds the bar.

Weights are N(0, 0.02) drawn on the device and quantized by the library's
device encoders (bit-identical to the restatement's), then handed to both
sides as host arrays, as a GGUF loader would.
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from model_helpers import oracle_session  # noqa: E402

REL_L2 = 1e-2
PROMPT_8B = int(os.environ.get("OVF_FULL_PROMPT", "256"))


@pytest.fixture(scope="module")
def E():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from overfit_b200 import build, engine
    build.build()
    return engine


def rel_l2(a, b):
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def run_parity(sess, ref, prompt, steps, exact):
    """Prompt through both sides, then `steps` greedy tokens; returns the
    per-step relative L2 list."""
    tok = sess.prefill(prompt)
    for t in prompt:
        lg_ref = ref.decode(int(t))
    errs = [rel_l2(sess.get_last_logits(), lg_ref)]
    if exact:
        np.testing.assert_array_equal(sess.get_last_logits(), lg_ref, err_msg="after the prompt")
    assert errs[0] < REL_L2, errs
    for step in range(steps):
        nxt_ref = int(np.argmax(lg_ref))
        assert tok == nxt_ref, f"greedy token differs at step {step}"
        tok = sess.decode(tok)
        lg_ref = ref.decode(nxt_ref)
        errs.append(rel_l2(sess.get_last_logits(), lg_ref))
        if exact:
            np.testing.assert_array_equal(sess.get_last_logits(), lg_ref, err_msg=f"step {step}")
        assert errs[-1] < REL_L2, (step, errs[-1])
    assert tok == int(np.argmax(lg_ref))
    return errs


def test_qwen2_05b_config_bit_exact(E, orc):
    cfg = dict(E.QWEN2_05B)
    mf = E.synthetic_model(cfg, seed=1)
    eng = E.CudaLlamaInferenceEngine(cfg, mf)
    sess = eng.create_session(192)
    ref = oracle_session(cfg, mf, 192)
    prompt = np.random.default_rng(128).integers(0, cfg["vocab"], 128)
    run_parity(sess, ref, prompt, 32, exact=True)
    sess.close()
    eng.close()


@pytest.fixture(scope="module")
def llama8b(E):
    cfg = dict(E.LLAMA3_8B)
    mf = E.synthetic_model(cfg, seed=1)
    eng = E.CudaLlamaInferenceEngine(cfg, mf)
    yield cfg, mf, eng
    eng.close()


@pytest.mark.parametrize("kv", ["f16", "f32"])
def test_llama3_8b_shape_parity(E, orc, llama8b, kv):
    cfg, mf, eng = llama8b
    n = PROMPT_8B + 40
    sess = eng.create_session(n, kv)
    ref = oracle_session(cfg, mf, n)
    if kv == "f16":
        ref.set_kv_fp16(True)
    prompt = np.random.default_rng(2048).integers(0, cfg["vocab"], PROMPT_8B)
    errs = run_parity(sess, ref, prompt, 32, exact=True)
    print(f"llama3-8b {kv} KV: max rel L2 {max(errs):.3g} over {len(errs)} steps")
    sess.close()
