"""Reference behaviour of TurboAdam (reference tests/test_optimizer.py,
test_costate.py, test_oneq.py semantics) on the sm_100a path."""

import pytest
import torch
import torch.nn as nn

pytestmark = pytest.mark.gpu


def T():
    from turboadam_b200 import TurboAdam

    return TurboAdam


def make_params(seed=42):
    torch.manual_seed(seed)
    return [nn.Parameter(torch.randn(10, 10, device="cuda")),
            nn.Parameter(torch.randn(20, device="cuda"))]


def step_with_grad(opt, params):
    for p in params:
        p.grad = torch.randn_like(p)
    opt.step()


def quad_run(steps=200, **kw):
    torch.manual_seed(0)
    x = nn.Parameter(torch.randn(50, device="cuda"))
    opt = T()([x], lr=1e-2, **kw)
    init = (x ** 2).sum().item()
    for _ in range(steps):
        opt.zero_grad()
        (x ** 2).sum().backward()
        opt.step()
    return init, (x ** 2).sum().item()


@pytest.mark.parametrize("kw", [{}, dict(compress_m=False, compress_v=False),
                                dict(compress_m=True, compress_v=False),
                                dict(compress_m=False, compress_v=True)])
def test_converges_quadratic(kw):
    init, final = quad_run(**kw)
    assert final < 0.10 * init


@pytest.mark.parametrize("bits", [4, 6, 8])
def test_converges_at_bits(bits):
    init, final = quad_run(steps=500, v_bits=bits)
    assert final < 0.10 * init


def test_state_structure():
    params = make_params()
    opt = T()(params)
    step_with_grad(opt, params)
    for p in params:
        st = opt.state[p]
        assert st["step"] == 1
        cv = st["compressed_v"]
        assert set(cv) == {"indices", "scales", "n_bits", "original_shape", "original_length",
                           "block_size"}
        B = (p.numel() + 127) // 128
        assert cv["indices"].dtype == torch.uint8 and cv["indices"].numel() == B * 128
        assert cv["scales"].dtype == torch.float16 and tuple(cv["scales"].shape) == (B, 2)
        assert "exp_avg_sq" not in st
        assert "exp_avg" in st  # < 4096 elements: fp32 m
        assert st["exp_avg"].dtype == torch.float32


def test_costate_state_for_large_params():
    torch.manual_seed(0)
    p = nn.Parameter(torch.randn(64, 64, device="cuda"))
    opt = T()([p])
    step_with_grad(opt, [p])
    mgr = opt.state[p]["m_mgr"]
    assert mgr._has_state and mgr._original_numel == 4096
    enc = mgr._encoded
    assert enc["labels"].dtype == torch.uint8 and enc["labels"].numel() == 32
    assert enc["sign_packed"].numel() == 512
    assert enc["block_norms"].dtype == torch.float32 and enc["scales"].dtype == torch.float16
    assert "exp_avg" not in opt.state[p]
    labels = enc["labels"].cpu()
    assert int((labels == 0).sum()) >= 1 and int((labels == 2).sum()) >= 1


def test_step_counter_and_v_changes():
    from turboadam_b200.oneq import decompress_v

    params = make_params()
    opt = T()(params)
    step_with_grad(opt, params)
    v1 = decompress_v(opt.state[params[0]]["compressed_v"]).clone()
    for s in range(2, 6):
        step_with_grad(opt, params)
        for p in params:
            assert opt.state[p]["step"] == s
    v2 = decompress_v(opt.state[params[0]]["compressed_v"])
    assert v2.shape == params[0].shape
    assert not torch.allclose(v1, v2)
    assert (v2 >= 0).all()


def test_no_compression_matches_adam():
    torch.manual_seed(7)
    grads = [[torch.randn(10, 10), torch.randn(20)] for _ in range(10)]

    def run(cls, **kw):
        ps = [nn.Parameter(torch.ones(10, 10, device="cuda")),
              nn.Parameter(torch.ones(20, device="cuda"))]
        opt = cls(ps, lr=1e-3, betas=(0.9, 0.999), **kw)
        for gs in grads:
            for p, g in zip(ps, gs):
                p.grad = g.cuda().clone()
            opt.step()
        return [p.detach().cpu() for p in ps]

    a = run(torch.optim.Adam)
    t = run(T(), compress_m=False, compress_v=False)
    for x, y in zip(a, t):
        assert torch.allclose(x, y, atol=1e-6)


def test_close_to_adam_10_steps():
    torch.manual_seed(7)
    grads = [[torch.randn(10, 10), torch.randn(20)] for _ in range(10)]

    def run(cls, **kw):
        ps = [nn.Parameter(torch.ones(10, 10, device="cuda")),
              nn.Parameter(torch.ones(20, device="cuda"))]
        opt = cls(ps, lr=1e-3, **kw)
        for gs in grads:
            for p, g in zip(ps, gs):
                p.grad = g.cuda().clone()
            opt.step()
        return [p.detach().cpu() for p in ps]

    for x, y in zip(run(torch.optim.Adam), run(T())):
        assert (x - y).norm().item() / (x.norm().item() + 1e-8) < 0.15


def test_weight_decay_known_answer():
    x = nn.Parameter(torch.ones(10, 10, device="cuda"))
    opt = T()([x], lr=1e-2, weight_decay=0.1)
    x.grad = torch.zeros_like(x)
    opt.step()
    assert abs(x.mean().item() - (1.0 - 1e-2 * 0.1)) < 1e-4


def test_param_groups_and_add_group():
    torch.manual_seed(0)
    x = nn.Parameter(torch.randn(10, 10, device="cuda"))
    y = nn.Parameter(torch.randn(10, 10, device="cuda"))
    opt = T()([x], lr=1e-2)
    for _ in range(5):
        opt.zero_grad()
        (x ** 2).sum().backward()
        opt.step()
    opt.add_param_group({"params": [y], "lr": 1e-3})
    opt.zero_grad()
    (x ** 2 + y ** 2).sum().backward()
    opt.step()
    assert opt.state[x]["step"] == 6 and opt.state[y]["step"] == 1


def test_closure_returns_loss():
    x = nn.Parameter(torch.randn(10, device="cuda"))
    opt = T()([x], lr=1e-2)

    def closure():
        opt.zero_grad()
        loss = (x ** 2).sum()
        loss.backward()
        return loss

    assert opt.step(closure).item() > 0


def test_state_dict_roundtrip_bitexact(tmp_path):
    """Save -> load -> continue equals the uninterrupted run bit for bit
    (the Philox draws are keyed by (seed, tensor, step), so unlike the
    reference's rand_buf they survive a checkpoint)."""
    torch.manual_seed(0)
    x = nn.Parameter(torch.randn(100, 50, device="cuda"))
    y = nn.Parameter(torch.randn(30, device="cuda"))
    opt = T()([x, y], lr=1e-2, v_bits=4, seed=99)

    def loss_of(a, b):
        return (a ** 2).sum() + (b ** 2).sum()

    for _ in range(5):
        opt.zero_grad()
        loss_of(x, y).backward()
        opt.step()
    path = tmp_path / "opt.pt"
    torch.save(opt.state_dict(), path)
    x2 = nn.Parameter(x.detach().clone())
    y2 = nn.Parameter(y.detach().clone())
    opt2 = T()([x2, y2], lr=1e-2, v_bits=4, seed=99)
    opt2.load_state_dict(torch.load(path, weights_only=False))
    for _ in range(3):
        for o, a, b in ((opt, x, y), (opt2, x2, y2)):
            o.zero_grad()
            loss_of(a, b).backward()
            o.step()
    assert torch.equal(x, x2) and torch.equal(y, y2)
    for key in ("labels", "sign_packed", "block_norms", "scales"):
        assert torch.equal(opt.state[x]["m_mgr"]._encoded[key], opt2.state[x2]["m_mgr"]._encoded[key])


def test_min_m_compress_elements():
    x = nn.Parameter(torch.randn(100, device="cuda"))
    opt = T()([x], min_m_compress_elements=200)
    opt.zero_grad()
    (x ** 2).sum().backward()
    opt.step()
    assert "exp_avg" in opt.state[x] and "m_mgr" not in opt.state[x]
    z = nn.Parameter(torch.randn(5000, device="cuda"))
    opt = T()([z], min_m_compress_elements=100)
    (z ** 2).sum().backward()
    opt.step()
    assert "m_mgr" in opt.state[z] and "exp_avg" not in opt.state[z]


def test_costate_first_call_is_ema_from_zero():
    from turboadam_b200.costate import CoStateManager

    torch.manual_seed(3)
    mgr = CoStateManager(block_size=128)
    g = torch.randn(256, device="cuda")
    m = mgr.update(g, 0.9)
    assert torch.allclose(m, 0.1 * g, atol=1e-6)
    assert mgr._has_state


def test_nonfinite_grad_flag():
    x = nn.Parameter(torch.randn(64, 64, device="cuda"))
    opt = T()([x])
    x.grad = torch.randn_like(x)
    opt.step()
    assert opt.read_status() == 0
    g = torch.randn_like(x)
    g[3, 5] = float("inf")
    x.grad = g
    opt.step()
    from turboadam_b200._lib import TA_STATUS_NONFINITE_GRAD

    assert opt.read_status() & TA_STATUS_NONFINITE_GRAD


def test_thresholds_seam():
    """compute_thresholds seam vs torch.sort indexing (costate.py:94-118); the
    codec seams are checked bit for bit in test_gpu_seams.py."""
    from turboadam_b200.costate import compute_thresholds

    torch.manual_seed(1)
    r = torch.rand(10007, device="cuda")
    t0, t1 = compute_thresholds(r)
    s = torch.sort(r.cpu()).values
    n = r.numel()
    assert t0.item() == s[max(0, int(0.1 * n) - 1)].item()
    assert t1.item() == s[min(n - 1, int(0.9 * n))].item()
