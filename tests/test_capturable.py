"""capturable=True (device-resident step counts and bias corrections, CUDA
graph replay) and the GradScaler hand-off (grad_scale / found_inf) against
the default step, bit for bit."""
import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPES = [(300, 200), (3000,), (4096 + 77,)]


def _params(bf16=True):
    g = torch.Generator().manual_seed(3)
    ps = [torch.nn.Parameter((torch.randn(s, generator=g) * 0.02).cuda()) for s in SHAPES]
    if bf16:
        ps.append(torch.nn.Parameter((torch.randn(257, 64, generator=g) * 0.02)
                                     .to(torch.bfloat16).cuda()))
    return ps


def _grads(ps, step, scale=1.0):
    g = torch.Generator().manual_seed(100 + step)
    return [(torch.randn(p.shape, generator=g) * 1e-3 * scale).to(p.dtype).cuda() for p in ps]


def _same(oa, a, ob, b):
    for pa, pb in zip(a, b):
        assert torch.equal(pa.detach().view(-1).view(torch.uint8),
                           pb.detach().view(-1).view(torch.uint8))
        sa, sb = oa.state[pa], ob.state[pb]
        assert int(sa["step"]) == int(sb["step"])
        assert torch.equal(sa["compressed_v"]["indices"], sb["compressed_v"]["indices"])
        if "m_mgr" in sa:
            assert float(sa["m_mgr"]._alpha) == float(sb["m_mgr"]._alpha)
            for k in ("labels", "sign_packed", "block_norms"):
                assert torch.equal(sa["m_mgr"]._encoded[k].view(torch.uint8),
                                   sb["m_mgr"]._encoded[k].view(torch.uint8)), k
            ea, eb = sa["m_mgr"]._ef_residual, sb["m_mgr"]._ef_residual
            assert (ea is None) == (eb is None)
            if ea is not None:
                assert torch.equal(ea.view(torch.int32), eb.view(torch.int32))
        if "exp_avg" in sa:
            assert torch.equal(sa["exp_avg"], sb["exp_avg"])


KW = dict(lr=6e-4, weight_decay=0.01, v_bits=4, seed=11)


def test_capturable_eager_matches_default():
    from turboadam_b200 import TurboAdam

    a, b = _params(), _params()
    oa, ob = TurboAdam(a, **KW), TurboAdam(b, capturable=True, **KW)
    for s in range(4):
        for ps in (a, b):
            for p, g in zip(ps, _grads(ps, s)):
                p.grad = g
        oa.step()
        ob.step()
    torch.cuda.synchronize()
    _same(oa, a, ob, b)
    assert isinstance(ob.state[b[0]]["step"], torch.Tensor)


@pytest.mark.parametrize("error_feedback", [False, True])
def test_cuda_graph_replay_matches_default(error_feedback):
    from turboadam_b200 import TurboAdam

    a, b = _params(), _params()
    kw = dict(KW, error_feedback=error_feedback)
    oa, ob = TurboAdam(a, **kw), TurboAdam(b, capturable=True, **kw)
    for p, g in zip(b, _grads(b, 0)):
        p.grad = g  # static gradient storage for the graph
    for p, g in zip(a, _grads(a, 0)):
        p.grad = g
    oa.step()
    ob.step()  # first step eager: uploads the plan
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph):
            ob.step()
    torch.cuda.current_stream().wait_stream(side)
    for s in range(1, 5):
        for p, g in zip(b, _grads(b, s)):
            p.grad.copy_(g)
        graph.replay()
        for p, g in zip(a, _grads(a, s)):
            p.grad = g
        oa.step()
    torch.cuda.synchronize()
    _same(oa, a, ob, b)
    assert ob.read_status() == 0


@pytest.mark.parametrize("capturable", [False, True])
def test_grad_scale_and_found_inf_handoff(capturable):
    """grad_scale / found_inf as GradScaler hands them over == unscale_ then
    step; found_inf set == no step at all."""
    from turboadam_b200 import TurboAdam

    scale = torch.tensor(1024.0, device="cuda")
    a, b = _params(), _params()
    oa, ob = TurboAdam(a, **KW), TurboAdam(b, capturable=capturable, **KW)
    for s in range(3):
        for p, g in zip(a, _grads(a, s, 1024.0)):
            p.grad = g
        inv = scale.double().reciprocal().float()
        torch._amp_foreach_non_finite_check_and_unscale_(
            [p.grad for p in a if p.dtype == torch.float32], torch.zeros(1, device="cuda"), inv)
        for p in a:  # the unscale kernel takes fp32 only; bf16: fp32 product rounded back
            if p.dtype == torch.bfloat16:
                p.grad.mul_(inv)
        oa.step()
        for p, g in zip(b, _grads(b, s, 1024.0)):
            p.grad = g
        ob.grad_scale = scale
        ob.found_inf = torch.zeros((), device="cuda")
        ob.step()
    torch.cuda.synchronize()
    _same(oa, a, ob, b)
    before = [p.detach().clone() for p in b]
    steps = [int(ob.state[p]["step"]) for p in b]
    for p, g in zip(b, _grads(b, 9, 1024.0)):
        p.grad = g
    ob.found_inf = torch.ones((), device="cuda")
    ob.step()
    torch.cuda.synchronize()
    for p, q in zip(b, before):
        assert torch.equal(p.detach(), q)
    assert [int(ob.state[p]["step"]) for p in b] == steps


def test_torch_gradscaler_fused_path_matches_unscale_path():
    """torch.amp.GradScaler drives the fused hand-off; an optimizer without
    _step_supports_amp_scaling gets unscale_ + inf check + step instead."""
    from turboadam_b200 import TurboAdam

    class Unfused(TurboAdam):
        _step_supports_amp_scaling = False

    a, b = _params(bf16=False), _params(bf16=False)
    oa, ob = Unfused(a, **KW), TurboAdam(b, **KW)
    sa = torch.amp.GradScaler("cuda", init_scale=256.0)
    sb = torch.amp.GradScaler("cuda", init_scale=256.0)
    for s in range(3):
        for ps, opt, sc in ((a, oa, sa), (b, ob, sb)):
            loss = sum((p.float() * g.float()).sum() for p, g in zip(ps, _grads(ps, s)))
            opt.zero_grad()
            sc.scale(loss).backward()
            sc.step(opt)
            sc.update()
    torch.cuda.synchronize()
    _same(oa, a, ob, b)
