"""ZeRO-1 across processes: world-2 ranks step their shards with
TurboAdam(shards=..., spanning=...) (alpha chunk sums and threshold
histograms all-reduced between the phases) and compare every shard bit for
bit with an unsharded step computed on the same GPU; then, with full
parameter replicas, step the shard views and gather after every step
(Zero1ParamGather), and compare every full parameter.

Two transports: NCCL with one GPU per rank (skipped with fewer than two
GPUs), and gloo with both ranks on cuda:0 (gloo all-reduces and broadcasts
CUDA tensors through host memory), which runs the same host logic -- the
phase generator, the exchange layout, the all-reduces between phases, the
post-step gather -- as separate processes on a one-GPU machine. The ranks'
kernels never wait on one another (the exchanges are host-side collectives
between launches), so sharing a GPU is safe."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SHAPES = [(5000, 300), (777,), (4100, 256), (96, 70), (3000, 700)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out, backend="nccl"):
    import traceback

    try:
        _rank_body(rank, world, port, out, backend)
    except Exception:
        out.put((rank, ["exception: " + traceback.format_exc()]))
        raise


def _rank_body(rank, world, port, out, backend):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    gpu = rank if backend == "nccl" else 0
    torch.cuda.set_device(gpu)
    dev = torch.device("cuda", gpu)
    if backend == "nccl":
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
    else:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
    try:
        from turboadam_b200 import TurboAdam
        from turboadam_b200.sharding import zero1_partition, zero1_spanning

        numels = [int(np.prod(s)) for s in SHAPES]
        init = [torch.randn(n, generator=torch.Generator().manual_seed(40 + i)) * 0.02
                for i, n in enumerate(numels)]
        grads = [[torch.randn(n, generator=torch.Generator().manual_seed(1000 * s + i)) * 1e-3
                  for i, n in enumerate(numels)] for s in range(3)]
        kw = dict(lr=6e-4, weight_decay=0.01, v_bits=4, seed=9)
        full = [torch.nn.Parameter(x.clone().to(dev)) for x in init]
        ofull = TurboAdam(full, **kw)
        parts = zero1_partition(numels, world)
        mine = parts[rank]
        ps = [torch.nn.Parameter(init[t][e0:e1].clone().to(dev)) for t, e0, e1, _, _ in mine]
        opt = TurboAdam(ps, tensor_ids=[t for t, *_ in mine],
                        shards=[(b, g) for _, _, _, b, g in mine], spanning=zero1_spanning(parts),
                        **kw)
        for s in range(3):
            for p, g in zip(full, grads[s]):
                p.grad = g.to(dev)
            ofull.step()
            for (t, e0, e1, _, _), p in zip(mine, ps):
                p.grad = grads[s][t][e0:e1].to(dev)
            opt.step()
        torch.cuda.synchronize()
        bad = []
        for (t, e0, e1, boff, _), p in zip(mine, ps):
            ref = full[t]
            if not torch.equal(p.data.view(-1).view(torch.int32),
                               ref.data.view(-1)[e0:e1].view(torch.int32)):
                bad.append(f"rank {rank} tensor {t} params")
            a, b = opt.state[p], ofull.state[ref]
            B0, B1 = boff, boff + (e1 - e0 + 127) // 128
            if not torch.equal(a["compressed_v"]["indices"][:e1 - e0],
                               b["compressed_v"]["indices"][e0:e1]):
                bad.append(f"rank {rank} tensor {t} indices")
            if "m_mgr" in a:
                ea, eb = a["m_mgr"]._encoded, b["m_mgr"]._encoded
                if float(a["m_mgr"]._alpha) != float(b["m_mgr"]._alpha):
                    bad.append(f"rank {rank} tensor {t} alpha")
                if not torch.equal(ea["labels"], eb["labels"][B0:B1]):
                    bad.append(f"rank {rank} tensor {t} labels")
                if not torch.equal(ea["sign_packed"], eb["sign_packed"][e0 // 8:(e1 + 7) // 8]):
                    bad.append(f"rank {rank} tensor {t} signs")
        # ZeRO-1 with full replicas: step the shard views, gather after each step
        from turboadam_b200.sharding import Zero1ParamGather

        rep = [torch.nn.Parameter(x.clone().to(dev)) for x in init]
        zg = Zero1ParamGather(rep)
        sps, zkw = zg.optimizer_args()
        zopt = TurboAdam(sps, **zkw, **kw)
        for s in range(3):
            for (t, e0, e1, _, _), p in zip(zg.partition[rank], sps):
                p.grad = grads[s][t][e0:e1].to(dev)
            zopt.step()
            zg.gather()
        torch.cuda.synchronize()
        for t, (p, ref) in enumerate(zip(rep, full)):
            if not torch.equal(p.data.view(-1).view(torch.int32), ref.data.view(-1).view(torch.int32)):
                bad.append(f"rank {rank} tensor {t} gathered params")
        out.put((rank, bad))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _run_world(backend):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q, backend)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert results == {0: [], 1: []}, results


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_zero1_over_nccl_matches_unsharded():
    _run_world("nccl")


def test_zero1_two_processes_one_gpu_gloo_matches_unsharded():
    _run_world("gloo")
