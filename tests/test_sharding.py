"""By-tensor sharding over data-parallel ranks (the multi-GPU path of the step).

* the LPT owner assignment is a deterministic pure function of the sizes and
  balances the Llama-3-8B-shaped set;
* world_size-2 ``gloo`` ranks on CPU: each rank replays the step (checker)
  on its own shard with global tensor ids, and the gathered packed state is
  bit-identical to the unsharded replay; the max-over-ranks timing reduction
  behaves as the bench uses it;
* on a GPU: ``TurboAdam(shard, tensor_ids=global ids)`` reproduces the
  unsharded optimizer's state for those tensors bit for bit.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from turboadam_b200.sharding import lpt_owners, rank_loads, shard_by_tensor

SHAPES = [(768,), (768, 2304), (2304,), (768, 768), (3072, 768), (768, 3072), (3072,),
          (50, 768), (4096,), (1000, 129), (777,), (96, 70)]


def llama3_8b_numels():
    d, kv, ffn, vocab = 4096, 1024, 14336, 128256
    layer = [d * d, kv * d, kv * d, d * d, ffn * d, ffn * d, d * ffn, d, d]
    return [vocab * d] + layer * 32 + [d, vocab * d]


def test_lpt_owners_deterministic_and_balanced():
    n = llama3_8b_numels()
    for world in (1, 2, 4, 8):
        own = lpt_owners(n, world)
        assert own == lpt_owners(list(n), world)
        assert set(own) == set(range(world))
        loads = rank_loads(n, world)
        assert sum(loads) == sum(n)
        # LPT: no rank exceeds the mean by more than the largest tensor
        assert max(loads) - sum(n) / world <= max(n)
        assert max(loads) / (sum(n) / world) < 1.02
    with pytest.raises(ValueError):
        lpt_owners(n, 0)


def test_shard_by_tensor_partitions():
    ts = [torch.empty(s) for s in SHAPES]
    seen = []
    for r in range(3):
        local, ids = shard_by_tensor(ts, 3, r)
        assert [t.shape for t in local] == [ts[i].shape for i in ids]
        seen += ids
    assert sorted(seen) == list(range(len(ts)))
    with pytest.raises(ValueError):
        shard_by_tensor(ts, 2, 2)


def _replay(oracle, ids, nsteps, seed=77):
    """Checker replay of the step over the tensors ``ids`` (global indices),
    4-bit v + CoState, Philox draws keyed by the global index."""
    params = []
    for i in ids:
        rng = np.random.default_rng(1000 + i)
        params.append(oracle.OracleParam(
            (rng.standard_normal(int(np.prod(SHAPES[i]))) * 0.02).astype(np.float32)))
    opt = oracle.OracleTurboAdam([oracle.OracleTurboAdam.make_group(
        params, lr=6e-4, weight_decay=0.01, v_bits=4)])
    for s in range(nsteps):
        for i, p in zip(ids, params):
            rng = np.random.default_rng(10_000 * (s + 1) + i)
            p.grad = (rng.standard_normal(p.n) * 1e-3).astype(np.float32)
        opt.step(uniforms=lambda oi, st, npad: oracle.sr_uniforms(params[oi].n, ids[oi], st,
                                                                   seed))
    out = {}
    for i, p in zip(ids, params):
        st = opt.state[id(p)]
        rec = {"p": p.data.copy(), "idx": st.v_idx.copy(), "hdr": st.v_hdr.copy()}
        if st.compress_m:
            m = st.mgr
            rec.update(alpha=np.array([m.alpha], np.float32), labels=m.labels.copy(),
                       signs=m.signs.copy(), norms=m.norms.copy(), amp=m.amp.copy())
        else:
            rec["exp_avg"] = st.exp_avg.copy()
        out[i] = rec
    return out


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    import sys

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), ".."))
    from oracle import oracle as O

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        own = lpt_owners([int(np.prod(s)) for s in SHAPES], world)
        mine = [i for i, o in enumerate(own) if o == rank]
        # every rank computes the same owners without communication
        allown = [None] * world
        dist.all_gather_object(allown, own)
        assert all(a == own for a in allown)
        res = _replay(O, mine, nsteps=3)
        gathered = [None] * world
        dist.all_gather_object(gathered, res)
        # max-over-ranks timing as the bench reduces it
        t = torch.tensor([1.5 + rank])
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            merged = {}
            for g in gathered:
                merged.update(g)
            q.put((sorted(merged), merged, float(t[0])))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_match_unsharded(oracle):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    keys, merged, tmax = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert keys == list(range(len(SHAPES)))
    assert tmax == 2.5
    ref = _replay(oracle, list(range(len(SHAPES))), nsteps=3)
    for i in keys:
        for k, v in ref[i].items():
            np.testing.assert_array_equal(np.asarray(merged[i][k]).view(np.uint8),
                                          np.asarray(v).view(np.uint8), err_msg=f"{i} {k}")


@pytest.mark.gpu
def test_turboadam_shard_with_global_ids_matches_unsharded():
    from turboadam_b200 import TurboAdam

    def make(ids):
        ps = []
        for i in ids:
            g = torch.Generator().manual_seed(500 + i)
            ps.append(torch.nn.Parameter((torch.randn(SHAPES[i], generator=g) * 0.02).cuda()))
        return ps

    def run(opt, ps, ids):
        for s in range(3):
            for i, p in zip(ids, ps):
                g = torch.Generator().manual_seed(9000 * (s + 1) + i)
                p.grad = (torch.randn(SHAPES[i], generator=g) * 1e-3).cuda()
            opt.step()
        torch.cuda.synchronize()

    all_ids = list(range(len(SHAPES)))
    full = make(all_ids)
    ofull = TurboAdam(full, lr=6e-4, weight_decay=0.01, seed=5)
    run(ofull, full, all_ids)
    for rank in range(2):
        _, ids = shard_by_tensor(full, 2, rank)
        part = make(ids)
        opart = TurboAdam(part, lr=6e-4, weight_decay=0.01, seed=5, tensor_ids=ids)
        run(opart, part, ids)
        for p, i in zip(part, ids):
            q = full[i]
            assert torch.equal(p.data.view(torch.int32), q.data.view(torch.int32)), i
            a, b = opart.state[p], ofull.state[q]
            assert torch.equal(a["compressed_v"]["indices"], b["compressed_v"]["indices"]), i
            if "m_mgr" in a:
                ea, eb = a["m_mgr"]._encoded, b["m_mgr"]._encoded
                for k in ("labels", "sign_packed"):
                    assert torch.equal(ea[k], eb[k]), (i, k)
    with pytest.raises(ValueError):
        TurboAdam(full, tensor_ids=[0])


def test_zero1_partition_cuts_on_chunk_boundaries():
    from turboadam_b200.sharding import ALIGN_BLOCKS, zero1_partition

    n = llama3_8b_numels()
    for world in (1, 2, 4, 8):
        parts = zero1_partition(n, world)
        covered = {}
        for shards in parts:
            for t, e0, e1, boff, gn in shards:
                assert gn == n[t] and boff * 128 == e0
                assert e0 % (ALIGN_BLOCKS * 128) == 0 or e0 == 0
                assert e1 == n[t] or e1 % (ALIGN_BLOCKS * 128) == 0
                covered.setdefault(t, []).append((e0, e1))
        for t, spans in covered.items():  # every tensor exactly covered
            spans.sort()
            assert spans[0][0] == 0 and spans[-1][1] == n[t]
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        loads = [sum(e1 - e0 for _, e0, e1, _, _ in s) for s in parts]
        assert max(loads) - min(loads) <= 2 * ALIGN_BLOCKS * 128


ZSHAPES = [(5000, 300), (777,), (4100, 256), (96, 70), (3000, 700)]


@pytest.mark.gpu
@pytest.mark.parametrize("ef", [False, True])
@pytest.mark.parametrize("world", [2, 3, 5])
def test_zero1_phased_step_matches_unsharded(world, ef):
    """ZeRO-1 shards stepped through the phased C ABI, ranks emulated in one
    process (their exchange regions summed between phases, what the NCCL
    all-reduce does across GPUs): every parameter and packed-state bit --
    with error feedback, every residual bit -- equals the unsharded step's."""
    from turboadam_b200 import TurboAdam
    from turboadam_b200.sharding import zero1_partition, zero1_spanning

    numels = [int(np.prod(s)) for s in ZSHAPES]
    init = [(torch.randn(n, generator=torch.Generator().manual_seed(40 + i)) * 0.02)
            for i, n in enumerate(numels)]
    grads = [[torch.randn(n, generator=torch.Generator().manual_seed(1000 * s + i)) * 1e-3
              for i, n in enumerate(numels)] for s in range(3)]
    kw = dict(lr=6e-4, weight_decay=0.01, v_bits=4, seed=9, error_feedback=ef)

    full = [torch.nn.Parameter(x.clone().cuda()) for x in init]
    ofull = TurboAdam(full, **kw)
    for s in range(3):
        for p, g in zip(full, grads[s]):
            p.grad = g.cuda()
        ofull.step()

    parts = zero1_partition(numels, world)
    spanning = zero1_spanning(parts)
    assert spanning  # the case splits at least one CoState tensor
    ranks = []
    for shards in parts:
        ps = [torch.nn.Parameter(init[t][e0:e1].clone().cuda()) for t, e0, e1, _, _ in shards]
        opt = TurboAdam(ps, tensor_ids=[t for t, *_ in shards],
                        shards=[(boff, gn) for _, _, _, boff, gn in shards], spanning=spanning,
                        **kw)
        ranks.append((shards, ps, opt))
    for s in range(3):
        for shards, ps, _ in ranks:
            for (t, e0, e1, _, _), p in zip(shards, ps):
                p.grad = grads[s][t][e0:e1].cuda()
        gens = [opt._step_gen() for _, _, opt in ranks]
        regions = [next(g) for g in gens]
        while regions:
            total = torch.stack(regions).sum(0)
            for r in regions:
                r.copy_(total)
            nxt = []
            for g in gens:  # resume every rank, also past its last exchange
                try:
                    nxt.append(g.send(None))
                except StopIteration:
                    pass
            assert len(nxt) in (0, len(gens))
            regions = nxt
    torch.cuda.synchronize()
    for shards, ps, opt in ranks:
        for (t, e0, e1, boff, _), p in zip(shards, ps):
            q = full[t]
            tag = f"world {world} tensor {t} [{e0}, {e1})"
            assert torch.equal(p.data.view(-1).view(torch.int32),
                               q.data.view(-1)[e0:e1].view(torch.int32)), tag
            a, b = opt.state[p], ofull.state[q]
            B0, B1 = boff, boff + (e1 - e0 + 127) // 128
            assert torch.equal(a["compressed_v"]["indices"][:(e1 - e0)],
                               b["compressed_v"]["indices"][e0:e1]), tag
            assert torch.equal(a["compressed_v"]["scales"].view(torch.int16)[:B1 - B0],
                               b["compressed_v"]["scales"].view(torch.int16)[B0:B1]), tag
            if "m_mgr" in a:
                ea, eb = a["m_mgr"]._encoded, b["m_mgr"]._encoded
                assert float(a["m_mgr"]._alpha) == float(b["m_mgr"]._alpha), tag
                assert torch.equal(ea["labels"], eb["labels"][B0:B1]), tag
                assert torch.equal(ea["sign_packed"], eb["sign_packed"][e0 // 8:(e1 + 7) // 8]), tag
                assert torch.equal(ea["block_norms"].view(torch.int32),
                                   eb["block_norms"][B0:B1].view(torch.int32)), tag
                if ef:
                    ra, rb = a["m_mgr"]._ef_residual, b["m_mgr"]._ef_residual
                    assert torch.equal(ra.reshape(-1).view(torch.int32),
                                       rb.reshape(-1)[e0:e1].view(torch.int32)), tag


def _gather_rank(rank, world, port, flat, q):
    import sys

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), ".."))
    from turboadam_b200.sharding import Zero1ParamGather

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shapes = [(1000, 300), (777,), (4100, 256), (96, 70)]
        numels = [int(np.prod(s)) for s in shapes]
        if flat:
            buf = torch.zeros(sum(numels))
            params, off = [], 0
            for s, n in zip(shapes, numels):
                params.append(buf[off:off + n].view(s))
                off += n
        else:
            params = [torch.zeros(s) for s in shapes]
        zg = Zero1ParamGather(params, block_size=128)
        assert (zg._flat is not None) == flat
        shard_params, kw = zg.optimizer_args()
        # a stand-in for the step: each rank writes its own marks into its shards
        for sp, (t, e0, e1, _, _) in zip(shard_params, zg.partition[rank]):
            sp.data.copy_(torch.arange(e0, e1, dtype=torch.float32) + 1e6 * (t + 1))
        zg.gather()
        ok = all(torch.equal(p.view(-1), torch.arange(n, dtype=torch.float32) + 1e6 * (t + 1))
                 for t, (p, n) in enumerate(zip(params, numels)))
        q.put((rank, ok, len(kw["spanning"])))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("flat", [True, False])
@pytest.mark.parametrize("world", [2, 3])
def test_zero1_param_gather_gloo(world, flat):
    """Post-step all-gather of ZeRO-1 ranges (flat buffer: one broadcast per
    rank; separate tensors: one per shard) leaves every rank with every
    rank's updates."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_rank, args=(r, world, port, flat, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    assert all(ok for _, ok, _ in res), res
