"""The CUDA path against golden vectors produced by the reference's own code
(tests/golden/make_golden.py): the fused DQN and PPO loss kernels, the fused
Adam kernel over several steps (weight decay, a parameter that misses a
step), the device grad norm and clip factor, the Linear tape (Flatten ->
Linear -> ReLU -> Linear, forward and backward), the GRU cell tape and the
conv tower forward.

Tolerances: fp32 elementwise 1e-6 (Adam, the DQN head); exp/log chains 1e-5
(PPO, GRU); GEMM paths 1e-4 (split-TF32 tensor cores, inside the spec's
1e-3 TF32 bar).
"""

import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from tests.helpers import rel  # noqa: E402

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return np.load(os.path.join(GOLDEN, f"{name}.npz"))


def dev(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda", dtype)


def host(t):
    return t.detach().cpu().numpy()


def _ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from ttrl_b200.device import context
    return context(0)


@pytest.mark.parametrize("name", ["vanilla", "double", "double_mask", "double_per"])
def test_dqn_loss_kernel(name):
    ctx = _ctx()
    d = load("dqn_loss")
    g = {k[len(name) + 1:]: d[k] for k in d.files if k.startswith(name + "_")}
    double, mask_n, per = (int(v) for v in g["flags"])
    B, A = g["q"].shape
    loss = torch.zeros(1, device="cuda")
    mean_q = torch.zeros(1, device="cuda")
    td_abs = torch.zeros(B, device="cuda")
    dq = torch.zeros((B, A), device="cuda")
    q_sel = g["q_next_online"] if double else g["q_next_target"]
    ctx.dqn_loss(dev(g["q"]), dev(q_sel), dev(g["q_next_target"]), dev(g["onehot"]),
                 dev(g["rewards"]), dev(g["dones"]), dev(g["discounts"]),
                 dev(g["next_mask"]) if mask_n else None,
                 dev(g["is_weights"]) if per else None, loss, mean_q, td_abs, dq, 1.0)
    assert rel(host(loss), g["loss"].reshape(-1)) <= 1e-6
    assert abs(host(mean_q)[0] - g["mean_q"].reshape(-1)[0]) <= 1e-6
    assert rel(host(dq), g["dq"]) <= 1e-6
    if per:
        assert rel(host(td_abs), g["td_abs"].reshape(-1)) <= 1e-6


@pytest.mark.parametrize("name", ["mean", "masked"])
def test_ppo_loss_kernel(name):
    ctx = _ctx()
    d = load("ppo_objective")
    g = {k[len(name) + 1:]: d[k] for k in d.files if k.startswith(name + "_")}
    B, A = g["logits"].shape
    metrics = torch.zeros(4, device="cuda")
    new_logp = torch.zeros(B, device="cuda")
    dlogits = torch.zeros((B, A), device="cuda")
    dvalue = torch.zeros(B, device="cuda")
    ctx.ppo_loss(dev(g["logits"]), dev(g["value"]), dev(g["actions"], torch.int32),
                 dev(g["old_logp"]), dev(g["adv"]), dev(g["returns"]), dev(g["old_values"]),
                 dev(g["valid"]) if name == "masked" else None, metrics, new_logp, dlogits,
                 dvalue, 0.1, 0.1, 0.5, 0.01)
    m = host(metrics)
    for i, k in enumerate(("loss", "policy_loss", "value_loss", "entropy")):
        assert rel(m[i], g[k].reshape(-1)) <= 1e-5, k
    assert rel(host(new_logp), g["new_logp"].reshape(-1)) <= 1e-5
    assert rel(host(dlogits), g["dlogits"]) <= 1e-5
    assert rel(host(dvalue), g["dvalue"].reshape(-1)) <= 1e-5


@pytest.mark.parametrize("case", [0, 1, 2])
def test_adam_kernel(case):
    ctx = _ctx()
    d = load("adam_steps")
    pre = f"c{case}_"
    lr, eps, wd = (float(v) for v in d[pre + "hyper"])
    n = 3
    ps = [dev(d[pre + f"p{i}_init"]) for i in range(n)]
    S = [torch.zeros_like(p) for p in ps]
    V = [torch.zeros_like(p) for p in ps]
    steps = torch.zeros(n, dtype=torch.int32, device="cuda")
    ticket = torch.zeros(1, dtype=torch.int32, device="cuda")
    grads = [d[pre + f"p{i}_grads"] for i in range(n)]
    for step in range(grads[0].shape[0]):
        live = [i for i in range(n) if not (i == 1 and step == 2)]
        gs = {i: dev(grads[i][step]) for i in live}
        ctx.adam_step([(ps[i], gs[i], S[i], V[i], i) for i in live], steps, ticket, None,
                      lr, 0.9, 0.999, eps, wd)
    assert host(steps).tolist() == d[pre + "steps"].tolist()
    for i in range(n):
        assert rel(host(ps[i]), d[pre + f"p{i}_final"]) <= 1e-6
        assert rel(host(S[i]), d[pre + f"p{i}_S"]) <= 1e-6
        assert rel(host(V[i]), d[pre + f"p{i}_V"]) <= 1e-6


@pytest.mark.parametrize("case", [0, 1])
def test_grad_norm_clip_kernel(case):
    ctx = _ctx()
    d = load("grad_clip")
    pre = f"c{case}_"
    gs = [d[pre + f"g{i}"] for i in range(3)]
    max_norm = float(d[pre + "max_norm"])
    out = torch.zeros(2, device="cuda")
    ws = torch.zeros(ctx.sqnorm_workspace_bytes([g.size for g in gs]), dtype=torch.uint8,
                     device="cuda")
    ctx.grad_sqnorm([dev(g) for g in gs], out, max_norm, ws)
    sq, factor = host(out)
    norm = float(d[pre + "norm"])
    assert abs(np.sqrt(sq) - norm) / norm <= 1e-6
    for i, g in enumerate(gs):
        want = d[pre + f"clipped{i}"]
        assert rel(g * np.float32(factor), want) <= 1e-6


def test_linear_tape():
    _ctx()
    from ttrl_b200.engine.autograd import Tensor
    from ttrl_b200.engine.layers import Flatten, Linear
    from ttrl_b200.engine.ops import mean_all, mul
    d = load("linear_mlp")
    B = d["x_nhwc"].shape[0]
    fc1 = Linear(144, 32, "cuda")
    fc2 = Linear(32, 6, "cuda")
    for layer, w, b in ((fc1, "w1", "b1"), (fc2, "w2", "b2")):
        layer.weight.data.copy_(dev(d[w]))
        layer.bias.data.copy_(dev(d[b]))
    x = Tensor.from_numpy(d["x_nhwc"].reshape(1, 1, B * 9, 16), "cuda", requires_grad=True)
    y = fc2(fc1.forward_relu(Flatten(3, 3, 16)(x)))
    loss = mul(mean_all(mul(y, Tensor.from_numpy(d["upstream"], "cuda"))), float(B * 6))
    loss.backward()
    assert rel(y.numpy(), d["y"]) <= 1e-4
    for t, k in ((fc1.weight, "dw1"), (fc1.bias, "db1"), (fc2.weight, "dw2"),
                 (fc2.bias, "db2")):
        assert rel(host(t.grad), d[k]) <= 1e-4, k
    assert rel(host(x.grad).reshape(d["dx"].shape), d["dx"]) <= 1e-4


def test_gru_cell_tape():
    _ctx()
    from ttrl_b200.engine.autograd import Tensor
    from ttrl_b200.engine.ops import mean_all, mul
    from ttrl_b200.engine.recurrent import GRUCell
    d = load("gru_cell")
    B, I = d["x"].shape
    H = d["h"].shape[1]
    cell = GRUCell(I, H, "cuda")
    for name, p in cell.named_parameters():
        p.data.copy_(dev(d["param." + name]))
    x = Tensor.from_numpy(d["x"], "cuda", requires_grad=True)
    h = Tensor.from_numpy(d["h"], "cuda", requires_grad=True)
    h1 = cell(x, h)
    loss = mul(mean_all(mul(h1, Tensor.from_numpy(d["upstream"], "cuda"))), float(B * H))
    loss.backward()
    assert rel(h1.numpy(), d["h1"]) <= 1e-4
    assert rel(host(x.grad), d["dx"]) <= 1e-4
    assert rel(host(h.grad), d["dh"]) <= 1e-4
    for name, p in cell.named_parameters():
        assert rel(host(p.grad), d["grad." + name]) <= 1e-4, name


def test_conv_tower_forward():
    ctx = _ctx()
    from ttrl_b200.device import conv_geom
    from oracle.layers import oihw_to_krsc
    d = load("conv_tower")
    frames = d["nature_frames"]  # [N, C, H, W] uint8
    n, c, h, w = frames.shape
    x = dev(frames.transpose(0, 2, 3, 1).reshape(-1, c).astype(np.float32))
    for i, (k, s) in enumerate(((8, 4), (4, 2), (3, 1))):
        wt = d[f"nature_w{i}"]
        cout = wt.shape[0]
        g = conv_geom(n, h, w, c, cout, k, k, s, 0)
        y = torch.empty((n * g.oh * g.ow, cout), device="cuda")
        ctx.conv_fprop(x, dev(oihw_to_krsc(wt)), dev(d[f"nature_b{i}"]), y, g, 1.0, True)
        x, h, w, c = y, g.oh, g.ow, cout
    got = host(x).reshape(n, -1)
    assert rel(got, d["nature_features"]) <= 1e-4
