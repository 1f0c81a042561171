"""The N > 1 path of bench.py on CPU: independent replicas (no data-path
collective), the job time is the max over ranks, the value counts every
rank's tokens.  Two gloo ranks on 127.0.0.1."""
import os
import socket

import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import bench
    # rank r pretends its timed region took 1 + r seconds
    t = bench.max_over_ranks(1.0 + rank)
    v = bench.replica_value(256, world, t)
    q.put((rank, t, v))
    dist.destroy_process_group()


def test_two_rank_replica_timing():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, t, v in out:
        assert t == 2.0                      # the slowest rank's time
        assert v == pytest.approx(2 * 256 / 2.0)


def test_single_process_is_identity():
    import bench
    assert bench.max_over_ranks(3.5) == 3.5
    assert bench.replica_value(10, 1, 2.0) == 5.0


def _exchange_main(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from overfit_b200 import engine
    got = engine.exchange_handles(bytes([rank + 1]) * 64)
    q.put((rank, got))
    dist.destroy_process_group()


def test_tp_handle_exchange_two_ranks():
    """Tensor parallelism's host-side set-up: every rank ends with all ranks'
    exchange handles in rank order (what ovf_model_tp_connect takes)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, got in out:
        assert got == bytes([1]) * 64 + bytes([2]) * 64


def test_tp_split_rules():
    """The shard plan of the north star's tensor parallelism: Llama-3-8B
    splits over 2, 4 and 8 ranks; shapes that do not divide are refused
    before anything is uploaded."""
    from overfit_b200 import engine
    cfg = dict(engine.LLAMA3_8B)
    for w in (1, 2, 4, 8):
        engine.tp_check(cfg, w)
    with pytest.raises(ValueError):
        engine.tp_check(cfg, 3)  # 8 KV heads over 3 ranks
    with pytest.raises(ValueError):
        engine.tp_check(dict(cfg, d_ff=14336 + 256), 8)
    engine.tp_check(dict(cfg, n_experts=8, n_experts_used=2, d_ff=14336 + 256), 8)  # experts stay whole
    with pytest.raises(ValueError):
        engine.tp_check(dict(cfg, n_experts=6, n_experts_used=2), 4)
    with pytest.raises(ValueError):
        engine.tp_check(cfg, 16)
