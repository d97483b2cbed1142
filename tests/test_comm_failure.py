"""Failure handling of the sharded (ZeRO-1) step: the exchanges between its
phases are all-reduces over the ranks; with ``exchange_timeout`` a rank that
left, or one that stops answering, ends ``step()`` with TurboAdamCommError
within the deadline instead of a hang, and the optimizer refuses to step
again until a checkpoint is loaded.

The failures are made on the host: a rank process that exits between phases
(or between steps), or one that sleeps instead of joining the next
exchange. CPU tests drive ``run_exchanges`` (the driver ``TurboAdam.step``
uses) with ``gloo`` ranks and a stand-in phase generator that yields regions
of the real kinds (fp64 alpha chunk sums, then three int32 histograms). The
GPU test runs the real phased step with two processes on cuda:0 over gloo;
its departing rank leaves between steps, with nothing of its own in flight.
No GPU wait is made to fail.
"""
import datetime
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

TIMEOUT_S = 1.5


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _fake_phases(rank, log):
    """Regions as TurboAdam._step_gen yields them, each filled with rank + 1."""
    regions = [torch.zeros(6, dtype=torch.float64)] + [torch.zeros(8, dtype=torch.int32)
                                                         for _ in range(3)]
    for k, r in enumerate(regions):
        r.fill_(rank + 1)
        yield r
        log.append((k, r.tolist()))
    return "loss"


def _put(q, item):
    q.put(item)
    q.close()
    q.join_thread()


def _rank(rank, world, port, q, scenario):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    from turboadam_b200.optimizer import TurboAdamCommError, run_exchanges

    log = []
    if rank == 1 and scenario != "ok":
        gen = _fake_phases(rank, log)
        region = next(gen)
        dist.all_reduce(region)  # exchange 0 with the others
        if scenario == "leave":
            _put(q, (rank, "left after exchange 0"))
            os._exit(0)  # the process is gone before exchange 1
        time.sleep(4 * TIMEOUT_S)  # "stall": alive, but never joins exchange 1
        _put(q, (rank, "stalled"))
        os._exit(0)
    t0 = time.monotonic()
    try:
        out = run_exchanges(_fake_phases(rank, log), None, timeout=TIMEOUT_S)
        res = ("ok", out, log)
    except TurboAdamCommError as e:
        res = ("error", str(e), time.monotonic() - t0)
    _put(q, (rank, res))
    os._exit(0)


def _run(scenario, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q, scenario))
             for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=90) for _ in range(world))
    for p in procs:
        p.join(timeout=30)
    return res


def test_exchanges_complete_and_sum():
    res = _run("ok")
    for r in (0, 1):
        kind, out, log = res[r]
        assert kind == "ok" and out == "loss"
        assert [k for k, _ in log] == [0, 1, 2, 3]
        assert all(all(x == 3 for x in vals) for _, vals in log)  # (0 + 1) + (1 + 1)


def test_rank_leaving_between_phases_raises_not_hangs():
    res = _run("leave")
    kind, msg, dt = res[0]
    assert kind == "error", res
    assert "exchange 1" in msg and "histogram, round 0" in msg
    assert dt < 30


def test_stalled_rank_hits_the_deadline():
    res = _run("stall")
    kind, msg, dt = res[0]
    assert kind == "error", res
    assert "exchange 1" in msg
    assert TIMEOUT_S * 0.9 <= dt < TIMEOUT_S + 20


def test_failed_step_blocks_further_steps_until_a_checkpoint_is_loaded(monkeypatch):
    """The optimizer-level contract, with the phase generator replaced by
    one whose exchange fails (a single-rank gloo group whose all-reduce is
    made to raise)."""
    from turboadam_b200 import TurboAdam, TurboAdamCommError

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(_free_port())
    dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        p = torch.nn.Parameter(torch.zeros(4096 * 2))
        opt = TurboAdam([p], spanning=[(0, 4096 * 4)], exchange_timeout=TIMEOUT_S)
        sd = opt.state_dict()
        monkeypatch.setattr(opt, "_step_gen", lambda closure=None: _fake_phases(0, []))

        def broken(*a, **k):
            raise RuntimeError("Connection closed by peer")

        monkeypatch.setattr(dist, "all_reduce", broken)
        with pytest.raises(TurboAdamCommError, match="exchange 0"):
            opt.step()
        with pytest.raises(TurboAdamCommError, match="previous step stopped part way"):
            opt.step()
        monkeypatch.undo()
        monkeypatch.setattr(opt, "_step_gen", lambda closure=None: _fake_phases(0, []))
        opt.load_state_dict(sd)
        assert opt.step() == "loss"
    finally:
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# the real phased step on one GPU, two processes over gloo
# ---------------------------------------------------------------------------

SHAPES = [(5000, 300), (777,), (4100, 256)]


def _gpu_rank(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(0)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    from turboadam_b200 import TurboAdam, TurboAdamCommError
    from turboadam_b200.sharding import zero1_partition, zero1_spanning

    numels = [int(torch.tensor(s).prod()) for s in SHAPES]
    parts = zero1_partition(numels, world)
    mine = parts[rank]
    ps = [torch.nn.Parameter(torch.randn(e1 - e0, device="cuda") * 0.02)
          for _, e0, e1, _, _ in mine]
    opt = TurboAdam(ps, tensor_ids=[t for t, *_ in mine],
                    shards=[(b, g) for _, _, _, b, g in mine], spanning=zero1_spanning(parts),
                    exchange_timeout=TIMEOUT_S, lr=6e-4, v_bits=4, seed=3)
    for p in ps:
        p.grad = torch.randn_like(p) * 1e-3
    opt.step()  # every rank completes step 1
    torch.cuda.synchronize()
    if rank == 1:  # leaves between steps, nothing of its own in flight
        _put(q, (rank, "left after step 1"))
        os._exit(0)
    t0 = time.monotonic()
    try:
        opt.step()
        res = ("ok", None)
    except TurboAdamCommError as e:
        res = ("error", str(e), time.monotonic() - t0)
    torch.cuda.synchronize()  # the GPU is still usable
    x = torch.ones(8, device="cuda").sum().item()
    _put(q, (rank, res + (x,)))
    os._exit(0)


@pytest.mark.gpu
def test_sharded_step_peer_gone_raises_on_gpu():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gpu_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=30)
    kind, msg, dt, x = res[0]
    assert kind == "error", res
    assert "exchange 0" in msg and dt < 30
    assert x == 8.0
