"""Tensor parallelism on 2 GPUs (one process per GPU, peer memory over
NVLink): the split model's decode is bit-identical to the restatement of the
unsplit reference, at every step, for the tiny Llama model (Q4_K_M, 8 query
/ 2 KV heads) with F32 and fp16 KV caches, and for the Llama-3-8B layer shape
over 2 layers.  Skipped on a machine with fewer than 2 GPUs."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import torch.multiprocessing as mp  # noqa: E402


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, cfg, seed, kv, prompt, steps, q):
    try:
        import sys
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, root)
        sys.path.insert(0, os.path.join(root, "tests"))
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        import torch.distributed as dist
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from model_helpers import make_model_file
        from overfit_b200 import engine
        mf = make_model_file(cfg, seed=seed) if cfg.get("tiny", True) else engine.synthetic_model(cfg, seed, rank)
        eng = engine.CudaLlamaInferenceEngine(cfg, mf, device=rank, tp_group=dist.group.WORLD)
        s = eng.create_session(len(prompt) + steps + 8, kv)
        tok = s.prefill(prompt)
        logits = [s.get_last_logits().copy()]
        toks = [tok]
        for _ in range(steps):
            tok = s.decode(tok)
            toks.append(tok)
            logits.append(s.get_last_logits().copy())
        dev = s.generate_greedy(4)
        s.close()
        eng.close()
        q.put((rank, toks, logits, list(dev), mf if rank == 0 else None))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as ex:  # report to the parent instead of hanging it
        q.put((rank, "error", repr(ex), None, None))


def _run(cfg, seed, kv, prompt, steps, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, cfg, seed, kv, prompt, steps, q))
             for r in range(world)]
    for p in procs:
        p.start()
    out = sorted((q.get(timeout=600) for _ in procs), key=lambda x: x[0])
    for p in procs:
        p.join(timeout=120)
    for r in out:
        assert r[1] != "error", r[2]
    return out


needs2 = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                            reason="needs 2 GPUs")


@needs2
@pytest.mark.parametrize("kv", ["f32", "f16"])
def test_tp2_tiny_llama_bit_exact(orc, kv):
    from model_helpers import TINY_LLAMA, oracle_session
    cfg = dict(TINY_LLAMA)
    prompt = [int(x) for x in np.random.default_rng(5).integers(0, cfg["vocab"], 12)]
    out = _run(cfg, 21, kv, prompt, 16)
    (_, t0, l0, d0, mf), (_, t1, l1, d1, _) = out
    assert t0 == t1 and d0 == d1
    for a, b in zip(l0, l1):
        np.testing.assert_array_equal(a, b)
    ref = oracle_session(cfg, mf, len(prompt) + 32)
    if kv == "f16":
        ref.set_kv_fp16(True)
    for t in prompt:
        lg = ref.decode(t)
    for i, (tok, got) in enumerate(zip(t0, l0)):
        np.testing.assert_array_equal(got, lg, err_msg=f"step {i}")
        assert tok == int(np.argmax(lg))
        if i < len(t0) - 1:
            lg = ref.decode(tok)


@needs2
def test_ep2_tiny_mixtral_bit_exact(orc):
    """Expert parallelism: Mixtral-style MoE with experts split whole over 2
    ranks (rank r owns experts e % 2 == r, attention split by heads); the
    owner of each selected expert sends its output to every rank, which sum
    them in top-k order: bit-identical to the unsplit restatement."""
    from model_helpers import TINY_MIXTRAL, oracle_session
    cfg = dict(TINY_MIXTRAL)
    prompt = [int(x) for x in np.random.default_rng(8).integers(0, cfg["vocab"], 10)]
    out = _run(cfg, 22, "f32", prompt, 16)
    (_, t0, l0, d0, mf), (_, t1, l1, d1, _) = out
    assert t0 == t1 and d0 == d1
    ref = oracle_session(cfg, mf, len(prompt) + 32)
    for t in prompt:
        lg = ref.decode(t)
    for i, (tok, got) in enumerate(zip(t0, l0)):
        np.testing.assert_array_equal(got, lg, err_msg=f"step {i}")
        assert tok == int(np.argmax(lg))
        if i < len(t0) - 1:
            lg = ref.decode(tok)
