"""The tape's generic ops (ttrl/engine/ops/*) on the B200 kernels: forward
values and gradients against a float64 PyTorch CPU reference of the same
composition. Tolerance 1e-5 relative (fp32 elementwise arithmetic)."""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from tests.helpers import rel  # noqa: E402

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _run(build_ours, build_ref, arrays):
    """build_*(*tensors) -> scalar loss. Returns (ours, ref) loss and grads."""
    from ttrl_b200.engine.autograd import Tensor
    ts = [Tensor.from_numpy(a, "cuda", requires_grad=True) for a in arrays]
    loss = build_ours(*ts)
    loss.backward()
    got = [t.grad.detach().cpu().numpy() if t.grad is not None else np.zeros_like(a)
           for t, a in zip(ts, arrays)]
    rs = [torch.tensor(a, dtype=torch.float64, requires_grad=True) for a in arrays]
    rl = build_ref(*rs)
    rl.backward()
    want = [r.grad.numpy() if r.grad is not None else np.zeros_like(a)
            for r, a in zip(rs, arrays)]
    return loss.numpy().reshape(-1)[0], rl.item(), got, want


CASES = {
    "add_broadcast": (lambda o, a, b: o.sum_all(o.mul(o.add(a, b), a)),
                      lambda a, b: ((a + b) * a).sum(), [(8, 6), (1, 6)]),
    "sub_div": (lambda o, a, b: o.sum_all(o.div(o.sub(a, b), o.add(o.square(b), 1.0))),
                lambda a, b: ((a - b) / (b * b + 1.0)).sum(), [(5, 7), (5, 7)]),
    "unary_chain": (lambda o, a: o.sum_all(o.mul(o.tanh(o.exp(o.mul(a, 0.3))), o.sigmoid(a))),
                    lambda a: (torch.tanh(torch.exp(a * 0.3)) * torch.sigmoid(a)).sum(),
                    [(16, 9)]),
    "log_sqrt_abs": (lambda o, a: o.sum_all(o.add(o.log(o.add(o.abs_(a), 1.0)),
                                                  o.sqrt(o.add(o.square(a), 2.0)))),
                     lambda a: (torch.log(a.abs() + 1.0) + torch.sqrt(a * a + 2.0)).sum(),
                     [(12, 4)]),
    "relu_mean_dim": (lambda o, a: o.mean_all(o.mean_dim(o.relu(a), dim=-1)),
                      lambda a: torch.relu(a).mean(dim=-1, keepdim=True).mean(), [(10, 5)]),
    "log_softmax_entropy": (
        lambda o, a: o.add(o.mean_all(o.entropy(a)), o.sum_all(o.mul(o.log_softmax(a), 0.1))),
        lambda a: (-(torch.softmax(a, -1) * torch.log_softmax(a, -1)).sum(-1)).mean()
        + 0.1 * torch.log_softmax(a, -1).sum(),
        [(32, 6)]),
    "huber": (lambda o, a, b: o.mean_all(o.huber(a, b, 1.0)),
              lambda a, b: torch.nn.functional.huber_loss(a, b, reduction="mean", delta=1.0),
              [(32, 1), (32, 1)]),
    "matmul": (lambda o, a, b: o.sum_all(o.mul(o.matmul(a, b), o.matmul(a, b))),
               lambda a, b: ((a @ b) ** 2).sum(), [(7, 33), (33, 5)]),
    "concat_split": (lambda o, a, b: o.sum_all(o.mul(o.split(o.concat([a, b], -1), (3, 4), -1)[1],
                                                     2.0)),
                     lambda a, b: (torch.cat([a, b], -1)[:, 3:] * 2.0).sum(),
                     [(4, 2), (4, 5)]),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_generic_op(name):
    _need_gpu()
    from ttrl_b200.engine import ops as o
    ours, refn, shapes = CASES[name]
    rng = np.random.default_rng(abs(hash(name)) % 2**32)
    arrays = [rng.standard_normal(s).astype(np.float32) for s in shapes]
    lo, lr, got, want = _run(lambda *t: ours(o, *t), refn, arrays)
    assert rel(lo, lr) <= TOL
    for g, w in zip(got, want):
        assert rel(g, w) <= TOL


def test_clamp_gradient_is_zero_at_and_beyond_bounds():
    """ops/select.py:54-63: the relu-identity clamp passes gradient strictly
    inside (lo, hi) and blocks it at the bounds themselves."""
    _need_gpu()
    from ttrl_b200.engine import ops as o
    from ttrl_b200.engine.autograd import Tensor
    x = Tensor.from_numpy(np.array([[-2.0, -1.0, 0.0, 1.0, 2.0]], np.float32), "cuda",
                          requires_grad=True)
    y = o.clamp(x, -1.0, 1.0)
    o.sum_all(y).backward()
    assert np.array_equal(y.numpy(), [[-1.0, -1.0, 0.0, 1.0, 1.0]])
    assert np.array_equal(x.grad.cpu().numpy(), [[0.0, 0.0, 1.0, 0.0, 0.0]])


def test_argmax_first_max_and_one_hot_gather():
    _need_gpu()
    from ttrl_b200.engine import ops as o
    from ttrl_b200.engine.autograd import Tensor
    q = Tensor.from_numpy(np.array([[1, 3, 3, 0], [5, 1, 5, 2]], np.float32), "cuda")
    idx = o.argmax_dim_detached(q, dim=-1)
    assert idx.numpy().reshape(-1).tolist() == [1.0, 0.0]
    picked = o.one_hot_gather(q, idx, 4)
    assert picked.numpy().reshape(-1).tolist() == [3.0, 5.0]


def test_gru_unroll_matches_torch_reference():
    _need_gpu()
    from ttrl_b200.engine import ops as o
    from ttrl_b200.engine.autograd import Tensor
    from ttrl_b200.engine.recurrent import GRU
    np.random.seed(0)
    T, B, F, H = 5, 3, 8, 6
    gru = GRU(F, H, "cuda")
    rng = np.random.default_rng(1)
    x = rng.standard_normal((T, B, F)).astype(np.float32)
    h0 = rng.standard_normal((B, H)).astype(np.float32)
    done = (rng.random((T, B, 1)) < 0.3).astype(np.float32)
    xs = Tensor.from_numpy(x, "cuda", requires_grad=True)
    hs = Tensor.from_numpy(h0, "cuda", requires_grad=True)
    out, hT = gru(xs, hs, Tensor.from_numpy(done, "cuda"))
    o.sum_all(o.add(o.sum_all(out), o.sum_all(o.mul(hT, hT)))).backward()

    cell = gru.cell
    W_ih = torch.tensor(cell.weight_ih.numpy(), dtype=torch.float64, requires_grad=True)
    W_hh = torch.tensor(cell.weight_hh.numpy(), dtype=torch.float64, requires_grad=True)
    b_ih = torch.tensor(cell.bias_ih.numpy(), dtype=torch.float64, requires_grad=True)
    b_hh = torch.tensor(cell.bias_hh.numpy(), dtype=torch.float64, requires_grad=True)
    tx = torch.tensor(x, dtype=torch.float64, requires_grad=True)
    th = torch.tensor(h0, dtype=torch.float64, requires_grad=True)
    h = th
    outs = []
    for t in range(T):
        h = h * (1 - torch.tensor(done[t], dtype=torch.float64))
        gi = tx[t] @ W_ih + b_ih
        gh = h @ W_hh + b_hh
        r = torch.sigmoid(gi[:, :H] + gh[:, :H])
        z = torch.sigmoid(gi[:, H:2 * H] + gh[:, H:2 * H])
        n = torch.tanh(gi[:, 2 * H:] + r * gh[:, 2 * H:])
        h = (1 - z) * n + z * h
        outs.append(h)
    loss = torch.stack(outs).sum() + (h * h).sum()
    loss.backward()
    assert rel(out.numpy(), torch.stack(outs).detach().numpy()) <= TOL
    for ours, ref in ((cell.weight_ih, W_ih), (cell.weight_hh, W_hh), (cell.bias_ih, b_ih),
                      (cell.bias_hh, b_hh)):
        assert rel(ours.grad.cpu().numpy(), ref.grad.numpy()) <= 1e-4
    assert rel(xs.grad.cpu().numpy(), tx.grad.numpy()) <= 1e-4
    assert rel(hs.grad.cpu().numpy(), th.grad.numpy()) <= 1e-4


@pytest.mark.parametrize("T,B,F,H,masked", [(5, 3, 8, 8, True), (32, 16, 64, 256, True),
                                             (1, 4, 10, 8, False), (7, 2, 5, 12, True),
                                             (6, 40, 16, 64, False)])
def test_gru_sequence_kernels_equal_step_by_step(T, B, F, H, masked):
    """The one-launch cluster unroll (forward and BPTT) against the per-step
    GEMM + gate-kernel path on the same inputs: outputs and every gradient to
    2e-5 relative (fp32 CUDA-core dots against split-TF32 GEMMs)."""
    _need_gpu()
    from ttrl_b200.device import context
    from ttrl_b200.engine import ops as o
    from ttrl_b200.engine.autograd import Tensor
    from ttrl_b200.engine.recurrent import GRU, gru_unroll
    from ttrl_b200.engine.ops import linear, reshape
    ctx = context("cuda")
    assert ctx.gru_sequence_supported(B, H)
    rng = np.random.default_rng(T * 100 + H)
    x = rng.standard_normal((T, B, F)).astype(np.float32)
    h0 = rng.standard_normal((B, H)).astype(np.float32)
    done = (rng.random((T, B, 1)) < 0.2).astype(np.float32) if masked else None
    up = rng.standard_normal((T, B, H)).astype(np.float32)
    results = []
    for persistent in (True, False):
        np.random.seed(4)
        gru = GRU(F, H, "cuda")
        c = gru.cell
        xs = Tensor.from_numpy(x, "cuda", requires_grad=True)
        hs = Tensor.from_numpy(h0, "cuda", requires_grad=True)
        gi = linear(reshape(xs, (T * B, F)), c.weight_ih, c.bias_ih)
        out = gru_unroll(gi, hs, None if done is None else Tensor.from_numpy(done, "cuda"),
                         c.weight_hh, c.bias_hh, steps=T, persistent=persistent)
        o.sum_all(o.mul(out, Tensor.from_numpy(up, "cuda"))).backward()
        results.append([out.numpy(), xs.grad.cpu().numpy(), hs.grad.cpu().numpy()]
                       + [p.grad.cpu().numpy() for p in (c.weight_ih, c.weight_hh, c.bias_ih,
                                                         c.bias_hh)])
    names = ("out", "dx", "dh0", "dW_ih", "dW_hh", "db_ih", "db_hh")
    for name, a, b in zip(names, *results):
        assert rel(a, b) <= 2e-5, name


def test_gru_sequence_refuses_shapes_without_a_plan():
    _need_gpu()
    from ttrl_b200.device import context
    from ttrl_b200._lib import lib
    ctx = context("cuda")
    assert not ctx.gru_sequence_supported(4, 6)   # hidden not a multiple of 4
    assert not ctx.gru_sequence_supported(0, 8)
    rc = lib().ttrl_gru_sequence_fwd(None, None, None, None, None, None, None, None, None,
                                     3, 4, 6, None)
    assert rc == 4  # TTRL_EUNSUPPORTED
    assert b"has no plan" in lib().ttrl_last_error()
