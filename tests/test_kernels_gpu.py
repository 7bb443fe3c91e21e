"""Parity of the tcgen05 GEMM family, Adam and frame conversion against the
numpy oracle, called through the C ABI (ctypes) on a B200.

Tolerances (relative Frobenius error against a float64 oracle):
  split-TF32 contractions  <= 1e-4   (measured ~1e-6; budget in the spec 1e-3)
  single-pass TF32         <= 5e-3   (informational mode, not the default)
  fp32 elementwise (Adam)  <= 1e-6   relative per element, max over elements
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import layers as ol  # noqa: E402

pytestmark = pytest.mark.gpu

TOL_X3 = 1e-4
TOL_TF32 = 5e-3


def _ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from ttrl_b200.device import context
    return context(0)


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("m,k,n,relu,bias", [
    (32, 3136, 512, 1, 1), (32, 512, 6, 0, 1), (256, 512, 6, 0, 1), (256, 3136, 512, 1, 1),
    (7, 11, 5, 1, 1), (130, 64, 200, 0, 0), (256, 14, 256, 1, 1),
])
def test_linear_fwd(m, k, n, relu, bias):
    ctx = _ctx()
    rng = np.random.default_rng(m * 7 + k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = (rng.standard_normal((k, n)) / np.sqrt(k)).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    ref = ol.linear(x.astype(np.float64), w.astype(np.float64), b if bias else None)
    if relu:
        ref = np.maximum(ref, 0)
    y = torch.empty((m, n), device="cuda")
    ctx.linear_fwd(dev(x), dev(w), dev(b) if bias else None, y, relu=bool(relu))
    got = host(y)
    ctx.check_status()
    assert rel(got, ref) <= TOL_X3


@pytest.mark.parametrize("m,k,n", [(32, 3136, 512), (32, 512, 6), (256, 512, 6), (5, 13, 7),
                                   (256, 3136, 512)])
def test_linear_dgrad_masked(m, k, n):
    ctx = _ctx()
    rng = np.random.default_rng(m + k + n)
    g = rng.standard_normal((m, n)).astype(np.float32)
    w = rng.standard_normal((k, n)).astype(np.float32)
    mask = rng.standard_normal((m, k)).astype(np.float32)
    ref = (g.astype(np.float64) @ w.astype(np.float64).T) * (mask > 0)
    dx = torch.empty((m, k), device="cuda")
    ctx.linear_dgrad(dev(g), dev(w), dev(mask), dx, accumulate=False)
    assert rel(host(dx), ref) <= TOL_X3
    # accumulate into the previous result
    ctx.linear_dgrad(dev(g), dev(w), None, dx, accumulate=True)
    ref2 = ref + g.astype(np.float64) @ w.astype(np.float64).T
    assert rel(host(dx), ref2) <= TOL_X3


@pytest.mark.parametrize("m,k,n", [(32, 3136, 512), (32, 512, 6), (256, 14, 256), (5, 13, 7),
                                   (256, 3136, 512),
                                   # ones row inside a partly filled 32-row box, a
                                   # reduction that ends inside a k-block
                                   (64, 200, 128), (40, 1000, 256)])
def test_linear_wgrad_with_bias_grad(m, k, n):
    ctx = _ctx()
    rng = np.random.default_rng(3 * m + k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    g = rng.standard_normal((m, n)).astype(np.float32)
    dw = torch.empty((k, n), device="cuda")
    db = torch.empty((n,), device="cuda")
    ctx.linear_wgrad(dev(x), dev(g), dw, db, accumulate=False, accumulate_db=False)
    ref_w = x.astype(np.float64).T @ g.astype(np.float64)
    ref_b = g.astype(np.float64).sum(0)
    assert rel(host(dw), ref_w) <= TOL_X3
    assert rel(host(db), ref_b) <= TOL_X3
    ctx.linear_wgrad(dev(x), dev(g), dw, db, accumulate=True, accumulate_db=True)
    assert rel(host(dw), 2 * ref_w) <= TOL_X3
    assert rel(host(db), 2 * ref_b) <= TOL_X3


CONV_CASES = [
    # n, h, w, c, cout, k, stride, pad
    (2, 84, 84, 4, 32, 8, 4, 0),     # Nature conv1
    (2, 20, 20, 32, 64, 4, 2, 0),    # Nature conv2
    (2, 9, 9, 64, 64, 3, 1, 0),      # Nature conv3
    (2, 10, 10, 8, 16, 3, 1, 1),     # padded
    (3, 9, 9, 3, 5, 3, 2, 1),        # odd channels: scalar gather path
    # C a multiple of 32: windows by TMA im2col mode
    (2, 21, 21, 64, 32, 2, 1, 0),    # Nature conv1 in space-to-depth form
    (3, 11, 11, 32, 48, 3, 1, 1),    # padded; 363 pixels, 288 wgrad rows (partial tiles)
    (2, 13, 13, 64, 32, 5, 2, 2),    # 5x5 stride 2, padded
    # data gradient as one sub-pixel GEMM (no padding, stride | kernel)
    (3, 14, 14, 32, 64, 4, 2, 0),    # 147 window rows, 4 parity classes
    (2, 12, 12, 16, 24, 4, 2, 0),    # dY channels not a multiple of 32: gathered windows
]


def _conv_inputs(case, seed):
    n, h, w, c, cout, k, s, p = case
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((n, h, w, c)).astype(np.float32)
    wt = (rng.standard_normal((cout, c, k, k)) / np.sqrt(c * k * k)).astype(np.float32)
    b = rng.standard_normal(cout).astype(np.float32)
    return x, wt, b


@pytest.mark.parametrize("case", CONV_CASES)
def test_conv_fprop(case):
    from ttrl_b200.device import conv_geom
    ctx = _ctx()
    n, h, w, c, cout, k, s, p = case
    x, wt, b = _conv_inputs(case, 1)
    alpha = 0.5
    ref = ol.conv2d_nhwc(x.astype(np.float64), wt.astype(np.float64), b, stride=s, padding=p,
                         input_scale=alpha, apply_relu=True)
    geom = conv_geom(n, h, w, c, cout, k, k, s, p)
    y = torch.empty((n * geom.oh * geom.ow, cout), device="cuda")
    ctx.conv_fprop(dev(x.reshape(-1, c)), dev(ol.oihw_to_krsc(wt)), dev(b), y, geom, alpha, True)
    assert rel(host(y).reshape(ref.shape), ref) <= TOL_X3


@pytest.mark.parametrize("case", CONV_CASES)
def test_conv_dgrad_masked(case):
    from ttrl_b200.device import conv_geom
    ctx = _ctx()
    n, h, w, c, cout, k, s, p = case
    x, wt, _ = _conv_inputs(case, 2)
    geom = conv_geom(n, h, w, c, cout, k, k, s, p)
    rng = np.random.default_rng(5)
    dy = rng.standard_normal((n, geom.oh, geom.ow, cout)).astype(np.float32)
    mask = rng.standard_normal((n, h, w, c)).astype(np.float32)
    ref = ol.conv2d_dgrad(dy.astype(np.float64), wt.astype(np.float64), (n, h, w, c), stride=s,
                          padding=p) * (mask > 0)
    dx = torch.empty((n * h * w, c), device="cuda")
    ctx.conv_dgrad(dev(dy.reshape(-1, cout)), dev(ol.oihw_to_krsc(wt)),
                   dev(mask.reshape(-1, c)), dx, geom, accumulate=False)
    assert rel(host(dx).reshape(ref.shape), ref) <= TOL_X3


@pytest.mark.parametrize("case", [CONV_CASES[1], CONV_CASES[2]])
def test_conv_dgrad_accumulates_unmasked(case):
    """The sub-pixel data gradient adding into an existing dX (a tensor read
    by two consumers), without a mask."""
    from ttrl_b200.device import conv_geom
    ctx = _ctx()
    n, h, w, c, cout, k, s, p = case
    _, wt, _ = _conv_inputs(case, 4)
    geom = conv_geom(n, h, w, c, cout, k, k, s, p)
    rng = np.random.default_rng(6)
    dy = rng.standard_normal((n, geom.oh, geom.ow, cout)).astype(np.float32)
    prior = rng.standard_normal((n, h, w, c)).astype(np.float32)
    ref = ol.conv2d_dgrad(dy.astype(np.float64), wt.astype(np.float64), (n, h, w, c), stride=s,
                          padding=p) + prior
    dx = dev(prior.reshape(-1, c))
    ctx.conv_dgrad(dev(dy.reshape(-1, cout)), dev(ol.oihw_to_krsc(wt)), None, dx, geom,
                   accumulate=True)
    assert rel(host(dx).reshape(ref.shape), ref) <= TOL_X3


@pytest.mark.parametrize("case", CONV_CASES)
def test_conv_dgrad_two_step_equals_one_call(case):
    """ttrl_conv_dgrad_weights + ttrl_conv_dgrad_prepared reproduce
    ttrl_conv_dgrad bit for bit where the sub-pixel path applies, and refuse
    (0 bytes) where it does not."""
    from ttrl_b200.device import conv_geom
    ctx = _ctx()
    n, h, w, c, cout, k, s, p = case
    _, wt, _ = _conv_inputs(case, 7)
    geom = conv_geom(n, h, w, c, cout, k, k, s, p)
    nbytes = ctx.conv_dgrad_weights_bytes(geom)
    direct = p == 0 and k % s == 0 and h == (geom.oh - 1) * s + k and w == (geom.ow - 1) * s + k
    assert (nbytes > 0) == direct
    if not direct:
        return
    rng = np.random.default_rng(8)
    dy = dev(rng.standard_normal((n * geom.oh * geom.ow, cout)).astype(np.float32))
    mask = dev(rng.standard_normal((n * h * w, c)).astype(np.float32))
    krsc = dev(ol.oihw_to_krsc(wt))
    one = torch.empty((n * h * w, c), device="cuda")
    ctx.conv_dgrad(dy, krsc, mask, one, geom, accumulate=False)
    stacked = torch.empty(nbytes // 4, device="cuda")
    ctx.conv_dgrad_weights(krsc, stacked, geom)
    two = torch.empty_like(one)
    ctx.conv_dgrad_prepared(dy, stacked, mask, two, geom, accumulate=False)
    assert torch.equal(one, two)


@pytest.mark.parametrize("case", CONV_CASES)
def test_conv_wgrad_with_bias_grad(case):
    from ttrl_b200.device import conv_geom
    ctx = _ctx()
    n, h, w, c, cout, k, s, p = case
    x, _, _ = _conv_inputs(case, 3)
    geom = conv_geom(n, h, w, c, cout, k, k, s, p)
    rng = np.random.default_rng(6)
    dy = rng.standard_normal((n, geom.oh, geom.ow, cout)).astype(np.float32)
    alpha = 1.0 / 255.0
    ref_w = ol.conv2d_wgrad(x.astype(np.float64), dy.astype(np.float64), k, stride=s,
                            padding=p, input_scale=alpha)
    ref_b = dy.astype(np.float64).reshape(-1, cout).sum(0)
    dw = torch.empty((cout, k, k, c), device="cuda")
    db = torch.empty((cout,), device="cuda")
    ctx.conv_wgrad(dev(x.reshape(-1, c)), dev(dy.reshape(-1, cout)), dw, db, geom, alpha,
                   accumulate=False, accumulate_db=False)
    assert rel(ol.krsc_to_oihw(host(dw)), ref_w) <= TOL_X3
    assert rel(host(db), ref_b) <= TOL_X3


def test_conv_wgrad_split_k_is_deterministic():
    from ttrl_b200.device import conv_geom
    ctx = _ctx()
    geom = conv_geom(32, 84, 84, 4, 32, 8, 8, 4, 0)
    rng = np.random.default_rng(9)
    x = dev(rng.integers(0, 256, (32 * 84 * 84, 4)).astype(np.float32))
    dy = dev(rng.standard_normal((32 * 400, 32)).astype(np.float32))
    outs = []
    for _ in range(3):
        dw = torch.empty((32, 8, 8, 4), device="cuda")
        db = torch.empty((32,), device="cuda")
        ctx.conv_wgrad(x, dy, dw, db, geom, 1 / 255, False, False)
        outs.append((host(dw), host(db)))
    for dw, db in outs[1:]:
        assert np.array_equal(dw, outs[0][0]) and np.array_equal(db, outs[0][1])


def test_tf32_single_pass_rounds_to_nearest():
    """All-positive operands: a truncating tf32 conversion would bias every
    product low by about 2^-10 and the sums by ~1e-3 relative; rounding to
    nearest leaves an unbiased error orders of magnitude smaller."""
    from ttrl_b200 import _lib
    ctx = _ctx()
    rng = np.random.default_rng(12)
    x = rng.random((128, 2048)).astype(np.float32)
    w = rng.random((2048, 64)).astype(np.float32)
    ref = x.astype(np.float64) @ w.astype(np.float64)
    y = torch.empty((128, 64), device="cuda")
    ctx.linear_fwd(dev(x), dev(w), None, y, relu=False, precision=_lib.PREC_TF32)
    assert rel(host(y), ref) <= 2e-4


def test_tf32_single_pass_mode_is_looser_but_close():
    from ttrl_b200 import _lib
    ctx = _ctx()
    rng = np.random.default_rng(11)
    x = rng.standard_normal((64, 512)).astype(np.float32)
    w = rng.standard_normal((512, 128)).astype(np.float32)
    ref = x.astype(np.float64) @ w.astype(np.float64)
    y = torch.empty((64, 128), device="cuda")
    ctx.linear_fwd(dev(x), dev(w), None, y, relu=False, precision=_lib.PREC_TF32)
    e1 = rel(host(y), ref)
    ctx.linear_fwd(dev(x), dev(w), None, y, relu=False, precision=_lib.PREC_TF32X3)
    e3 = rel(host(y), ref)
    assert e1 <= TOL_TF32
    assert e3 <= TOL_X3
    assert e3 < e1


def test_u8_frames_to_nhwc_with_gather():
    ctx = _ctx()
    rng = np.random.default_rng(12)
    frames = rng.integers(0, 256, (6, 4, 84, 84), dtype=np.uint8)
    index = np.array([5, 0, 3], dtype=np.int32)
    out = torch.empty((3 * 84 * 84, 4), device="cuda")
    ctx.u8_to_f32(torch.from_numpy(frames).cuda(), torch.from_numpy(index).cuda(), out, 1.0)
    ref = frames[index].transpose(0, 2, 3, 1).reshape(-1, 4).astype(np.float32)
    assert np.array_equal(host(out), ref)


def test_adam_matches_reference_sv_form():
    ctx = _ctx()
    rng = np.random.default_rng(13)
    shapes = [(3136, 512), (512,), (32, 8, 8, 4), (6,), (1,)]
    ps = [rng.standard_normal(s).astype(np.float32) for s in shapes]
    Ss = [np.zeros(s, np.float32) for s in shapes]
    Vs = [np.zeros(s, np.float32) for s in shapes]
    dps = [dev(p) for p in ps]
    dS = [dev(s) for s in Ss]
    dV = [dev(v) for v in Vs]
    steps = torch.zeros(len(shapes), dtype=torch.int32, device="cuda")
    ticket = torch.zeros(1, dtype=torch.int32, device="cuda")
    hp = dict(lr=1e-4, b1=0.9, b2=0.999, eps=1.5e-4)
    for t in range(1, 4):
        gs = [rng.standard_normal(s).astype(np.float32) for s in shapes]
        dgs = [dev(g) for g in gs]
        ctx.adam_step([(dps[i], dgs[i], dS[i], dV[i], i) for i in range(len(shapes))], steps,
                      ticket, None, hp["lr"], hp["b1"], hp["b2"], hp["eps"], 0.0)
        for i in range(len(shapes)):
            ps[i], Ss[i], Vs[i] = ol.adam_step_sv(ps[i], gs[i], Ss[i], Vs[i], t, **hp)
    for i in range(len(shapes)):
        for got, want in ((host(dps[i]), ps[i]), (host(dS[i]), Ss[i]), (host(dV[i]), Vs[i])):
            # normwise (max-abs over max-abs) relative error; elementwise
            # relative error is ill-conditioned where S = g + b1*S cancels.
            err = np.max(np.abs(got.astype(np.float64) - want)) / np.max(np.abs(want))
            assert err <= 1e-6
    assert host(steps).tolist() == [3] * len(shapes)
    assert int(host(ticket)[0]) == 0


def test_adam_shared_launch_equals_separate_steps():
    """Two Adams joined by share_launch (different learning rates and
    parameter counts, as SAC's policy and temperature) stepped by
    step_together in one launch: bit for bit the two separate steps, with
    each optimizer's counters and rate its own; a later lr change of one of
    them is seen by the joint launch."""
    from ttrl_b200.engine.autograd import Tensor
    from ttrl_b200.engine.optim import Adam, share_launch, step_together
    rng = np.random.default_rng(15)
    shapes_a, shapes_b = [(256, 17), (256,), (3, 256)], [(1, 1)]

    def make():
        pa = [Tensor(dev(rng0.standard_normal(s).astype(np.float32)), True) for s in shapes_a]
        pb = [Tensor(dev(rng0.standard_normal(s).astype(np.float32)), True) for s in shapes_b]
        return pa, pb, Adam(pa, lr=3e-4), Adam(pb, lr=1e-3)

    rng0 = np.random.default_rng(1)
    pa1, pb1, oa1, ob1 = make()
    rng0 = np.random.default_rng(1)
    pa2, pb2, oa2, ob2 = make()
    share_launch([oa2, ob2])
    from ttrl_b200._lib import lib
    for t in range(3):
        if t == 2:
            ob1.lr = ob2.lr = 5e-4
        grads = [rng.standard_normal(p.shape).astype(np.float32) for p in pa1 + pb1]
        for params in ((pa1 + pb1), (pa2 + pb2)):
            for p, g in zip(params, grads):
                p.grad = dev(g)
        oa1.step()
        ob1.step()
        before = lib().ttrl_launch_count()
        step_together([oa2, ob2])
        assert lib().ttrl_launch_count() - before == 1
    for p1, p2 in zip(pa1 + pb1, pa2 + pb2):
        assert np.array_equal(host(p1.data), host(p2.data))
    for o1, o2 in ((oa1, oa2), (ob1, ob2)):
        assert o1.steps == o2.steps and o1.t == o2.t
        assert host(o2._dev_steps).tolist() == o2.steps
        for m1, m2 in zip(o1.m + o1.v, o2.m + o2.v):
            assert np.array_equal(host(m1), host(m2))


def test_grad_sqnorm_and_clip_factor():
    ctx = _ctx()
    rng = np.random.default_rng(14)
    gs = [rng.standard_normal(s).astype(np.float32) for s in [(100000,), (513,), (7, 3)]]
    ref = sum(float(np.sum(g.astype(np.float64) ** 2)) for g in gs)
    out = torch.zeros(2, device="cuda")
    ws = torch.zeros(ctx.sqnorm_workspace_bytes([g.size for g in gs]), dtype=torch.uint8,
                     device="cuda")
    ctx.grad_sqnorm([dev(g) for g in gs], out, 0.5, ws)
    got = host(out)
    assert abs(got[0] - ref) / ref <= 1e-6
    want_scale = 0.5 / (np.sqrt(ref) + 1e-6)
    assert abs(got[1] - want_scale) / want_scale <= 1e-6


@pytest.mark.parametrize("m,n,k,splits,transposed", [
    (300, 40, 2048, 2, False), (128, 32, 4096, 3, False), (257, 64, 1024, 5, True),
    (100, 128, 4096, 8, False), (128, 96, 8192, 16, True), (64, 32, 16384, 24, False),
    (130, 32, 32768, 32, True),
])
def test_gemm_split_k_cluster_and_global(m, n, k, splits, transposed):
    """Split-K with an explicit split count: up to 16 splits reduce across a
    thread-block cluster in distributed shared memory, more go through the
    global workspace. Ragged tiles, bias and ReLU in the epilogue; results
    match float64 and are bit-identical from run to run."""
    import ctypes
    from ttrl_b200 import _lib
    ctx = _ctx()
    rng = np.random.default_rng(m + n + k + splits)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((n, k)).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    da, db, dbias = dev(a), dev(b), dev(bias)
    ref = np.maximum(a.astype(np.float64) @ b.astype(np.float64).T + bias, 0.0)
    outs = []
    for _ in range(2):
        y = torch.full((n, m) if transposed else (m, n), float("nan"), device="cuda")
        d = _lib.GemmDesc()
        d.m, d.n, d.k, d.precision, d.splits = m, n, k, _lib.PREC_TF32X3, splits
        d.a.ptr, d.a.kind, d.a.rows, d.a.kdim, d.a.rs, d.a.ks = da.data_ptr(), 0, m, k, k, 1
        d.b.ptr, d.b.kind, d.b.rows, d.b.kdim, d.b.rs, d.b.ks = db.data_ptr(), 0, n, k, k, 1
        d.ep.out = y.data_ptr()
        d.ep.ors, d.ep.ocs = (1, m) if transposed else (n, 1)
        d.ep.alpha = 1.0
        d.ep.bias, d.ep.bias_mode = dbias.data_ptr(), _lib.BIAS_COL
        d.ep.relu = 1
        need = _lib.lib().ttrl_gemm_workspace_bytes(ctypes.byref(d))
        ws, wsb = ctx.workspace(need)
        _lib.check(_lib.lib().ttrl_gemm(ctypes.byref(d), ws, wsb, ctx.status_ptr(), ctx.stream),
                   "ttrl_gemm")
        got = host(y)
        outs.append(got.T if transposed else got)
    ctx.check_status()
    assert np.isfinite(outs[0]).all()
    assert rel(outs[0], ref) <= TOL_X3
    assert np.array_equal(outs[0], outs[1])


@pytest.mark.parametrize("n,k,prec,transposed", [
    (32, 256, 0, False), (64, 512, 0, True), (128, 64, 0, False), (96, 2048, 0, False),
    (32, 256, 1, True), (128, 320, 1, False),
])
def test_gemm_many_waves_half_footprint(n, k, prec, transposed):
    """Grids of several waves run the half-footprint GEMM (two CTAs per
    SM): every tile, split-TF32 and single-pass TF32, bias + ReLU epilogue,
    row-major and transposed outputs."""
    import ctypes
    from ttrl_b200 import _lib
    ctx = _ctx()
    m = 128 * 170 + 37  # > 148 tiles, ragged last tile
    rng = np.random.default_rng(n + k + prec)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((n, k)).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    da, db, dbias = dev(a), dev(b), dev(bias)
    y = torch.full((n, m) if transposed else (m, n), float("nan"), device="cuda")
    d = _lib.GemmDesc()
    d.m, d.n, d.k, d.precision, d.splits = m, n, k, prec, 1
    d.a.ptr, d.a.kind, d.a.rows, d.a.kdim, d.a.rs, d.a.ks = da.data_ptr(), 0, m, k, k, 1
    d.b.ptr, d.b.kind, d.b.rows, d.b.kdim, d.b.rs, d.b.ks = db.data_ptr(), 0, n, k, k, 1
    d.ep.out = y.data_ptr()
    d.ep.ors, d.ep.ocs = (1, m) if transposed else (n, 1)
    d.ep.alpha = 1.0
    d.ep.bias, d.ep.bias_mode = dbias.data_ptr(), _lib.BIAS_COL
    d.ep.relu = 1
    ws, wsb = ctx.workspace(_lib.lib().ttrl_gemm_workspace_bytes(ctypes.byref(d)))
    _lib.check(_lib.lib().ttrl_gemm(ctypes.byref(d), ws, wsb, ctx.status_ptr(), ctx.stream),
               "ttrl_gemm")
    got = host(y)
    got = got.T if transposed else got
    ctx.check_status()
    ref = np.maximum(a.astype(np.float64) @ b.astype(np.float64).T + bias, 0.0)
    assert np.isfinite(got).all()
    assert rel(got, ref) <= (TOL_X3 if prec == 0 else TOL_TF32)


@pytest.mark.parametrize("n,relu", [(32, 0), (128, 1)])
def test_gemm_half_footprint_epilogue_mask_row_bias_accumulate(n, relu):
    """The half-footprint GEMM's row-major epilogue with every global input
    it reads per group (the ReLU-backward mask, the old output when
    accumulating, a per-row bias), over a ragged many-wave grid:
    out = old + relu?((alpha * acc + bias[row]) * [mask > 0])."""
    import ctypes
    from ttrl_b200 import _lib
    ctx = _ctx()
    m, k, alpha = 128 * 170 + 37, 64, 0.5
    rng = np.random.default_rng(n + relu)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((n, k)).astype(np.float32)
    bias = rng.standard_normal(m).astype(np.float32)
    mask = rng.standard_normal((m, n)).astype(np.float32)
    old = rng.standard_normal((m, n)).astype(np.float32)
    da, db, dbias, dmask = dev(a), dev(b), dev(bias), dev(mask)
    y = dev(old)
    d = _lib.GemmDesc()
    d.m, d.n, d.k, d.precision, d.splits = m, n, k, _lib.PREC_TF32X3, 1
    d.a.ptr, d.a.kind, d.a.rows, d.a.kdim, d.a.rs, d.a.ks = da.data_ptr(), 0, m, k, k, 1
    d.b.ptr, d.b.kind, d.b.rows, d.b.kdim, d.b.rs, d.b.ks = db.data_ptr(), 0, n, k, k, 1
    d.ep.out, d.ep.ors, d.ep.ocs, d.ep.alpha = y.data_ptr(), n, 1, alpha
    d.ep.bias, d.ep.bias_mode = dbias.data_ptr(), _lib.BIAS_ROW
    d.ep.mask, d.ep.mrs, d.ep.mcs = dmask.data_ptr(), n, 1
    d.ep.relu, d.ep.accumulate = relu, 1
    ws, wsb = ctx.workspace(_lib.lib().ttrl_gemm_workspace_bytes(ctypes.byref(d)))
    _lib.check(_lib.lib().ttrl_gemm(ctypes.byref(d), ws, wsb, ctx.status_ptr(), ctx.stream),
               "ttrl_gemm")
    got = host(y)
    ctx.check_status()
    v = alpha * (a.astype(np.float64) @ b.astype(np.float64).T) + bias[:, None]
    v = np.where(mask > 0, v, 0.0)
    if relu:
        v = np.maximum(v, 0.0)
    assert rel(got, old + v) <= TOL_X3


def test_bounded_wait_gives_up_and_the_context_stays_usable():
    """A wait on a barrier that nothing completes (ttrl_wait_probe) gives up
    after the library's bound, records status 1001, and the next launches on
    the same context run normally."""
    import time
    from ttrl_b200._lib import lib
    ctx = _ctx()
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    assert lib().ttrl_wait_probe(status.data_ptr(), ctx.stream) == 0
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert int(status[0].item()) == 1001
    assert 1.0 < waited < 10.0  # the bound is two seconds of wall time
    x = torch.randn(64, 32, device="cuda")
    w = torch.randn(32, 16, device="cuda")
    y = torch.empty(64, 16, device="cuda")
    ctx.linear_fwd(x, w, None, y, relu=False)
    assert rel(host(y), host(x).astype(np.float64) @ host(w).astype(np.float64)) <= TOL_X3


_REF_CONV = (("conv1", 4), ("conv1s2d", 1), ("conv2", 2), ("conv3", 1))


@pytest.mark.parametrize("name,stride", _REF_CONV)
def test_conv_backward_matches_the_reference_composition(name, stride):
    """The tcgen05 weight and data gradients against the reference's own
    conv backward (tests/golden/conv_backward.npz: ttrl/engine/conv/
    backward.py weight_grad -- k*k strided slices, one matmul, x input_scale,
    dw_to_prepared -- and input_grad -- transpose_weight then
    conv_transpose2d), at the Nature geometries and conv1's space-to-depth
    form. Split-TF32 against the fixture's fp32: 1e-4 relative."""
    import os
    from ttrl_b200.device import conv_geom
    d = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden",
                             "conv_backward.npz"))
    x, wt, dy = d[name + ".x"], d[name + ".w"], d[name + ".dy"]
    scale = float(d[name + ".scale"])
    n, h, w, c = x.shape
    cout, k = wt.shape[0], wt.shape[2]
    ctx = _ctx()
    geom = conv_geom(n, h, w, c, cout, k, k, stride, 0)
    dw = torch.empty((cout, k, k, c), device="cuda")
    db = torch.empty((cout,), device="cuda")
    ctx.conv_wgrad(dev(x.reshape(-1, c)), dev(dy.reshape(-1, cout)), dw, db, geom, scale,
                   accumulate=False, accumulate_db=False)
    assert rel(ol.krsc_to_oihw(host(dw)), d[name + ".dw"]) <= TOL_X3
    # The reference scales the transposed weight by input_scale; the data
    # gradient is linear in it, so the same scale goes on the weight here.
    dx = torch.empty((n * h * w, c), device="cuda")
    ctx.conv_dgrad(dev(dy.reshape(-1, cout)), dev(ol.oihw_to_krsc(wt * np.float32(scale))),
                   None, dx, geom, accumulate=False)
    assert rel(host(dx).reshape(x.shape), d[name + ".dx"]) <= TOL_X3


# The stream-K weight gradient (csrc/wgrad_sk.cu) serves layers whose input
# is exact in tf32 (raw frames): conv1 in its space-to-depth form and any
# exact-input layer with C a multiple of 32, Cout 32 or 64, kh*kw*C <= 256.
SK_CASES = [
    # n, h, w, c, cout, k, stride: batch sizes that leave a partial last
    # 32-pixel block (n=1: 400 pixels), a few k-blocks per CTA (n=32) and the
    # PPO minibatch (n=256); a 128-row, 64-channel case
    (1, 21, 21, 64, 32, 2, 1),
    (3, 21, 21, 64, 32, 2, 1),
    (32, 21, 21, 64, 32, 2, 1),
    (256, 21, 21, 64, 32, 2, 1),
    (8, 9, 9, 32, 64, 2, 1),
]


@pytest.mark.parametrize("case", SK_CASES)
def test_stream_k_conv_wgrad(case):
    """dW (scaled by alpha) and db against the float64 oracle at 1e-4; then,
    on the same buffers, the accumulate flags add a second call's result; and
    two identical calls agree bit for bit (partials summed in a fixed order)."""
    from ttrl_b200.device import conv_geom
    ctx = _ctx()
    n, h, w, c, cout, k, s = case
    geom = conv_geom(n, h, w, c, cout, k, k, s, 0).with_exact_input(True)
    rng = np.random.default_rng(n * 31 + c)
    x = rng.integers(0, 256, (n, h, w, c)).astype(np.float32)  # exact in tf32
    dy = rng.standard_normal((n, geom.oh, geom.ow, cout)).astype(np.float32)
    alpha = 1.0 / 255.0
    ref_w = ol.conv2d_wgrad(x.astype(np.float64), dy.astype(np.float64), k, stride=s,
                            input_scale=alpha)
    ref_b = dy.astype(np.float64).reshape(-1, cout).sum(0)
    xd, dyd = dev(x.reshape(-1, c)), dev(dy.reshape(-1, cout))
    dw = torch.empty((cout, k, k, c), device="cuda")
    db = torch.empty((cout,), device="cuda")
    ctx.conv_wgrad(xd, dyd, dw, db, geom, alpha, accumulate=False, accumulate_db=False)
    first_w, first_b = host(dw).copy(), host(db).copy()
    assert rel(ol.krsc_to_oihw(first_w), ref_w) <= TOL_X3
    assert rel(first_b, ref_b) <= TOL_X3
    ctx.conv_wgrad(xd, dyd, dw, db, geom, alpha, accumulate=False, accumulate_db=False)
    assert np.array_equal(host(dw), first_w) and np.array_equal(host(db), first_b)
    ctx.conv_wgrad(xd, dyd, dw, db, geom, alpha, accumulate=True, accumulate_db=True)
    assert rel(ol.krsc_to_oihw(host(dw)), 2 * ref_w) <= TOL_X3
    assert rel(host(db), 2 * ref_b) <= TOL_X3
    ctx.check_status()


def test_stream_k_conv_wgrad_single_pass_tf32():
    """One TF32 pass over dY rounded to nearest (the windows are exact): the
    accuracy class of the reference's HiFi4 matmuls, 1e-3."""
    from ttrl_b200._lib import PREC_TF32
    from ttrl_b200.device import conv_geom
    ctx = _ctx()
    geom = conv_geom(32, 21, 21, 64, 32, 2, 2, 1, 0).with_exact_input(True)
    rng = np.random.default_rng(9)
    x = rng.integers(0, 256, (32, 21, 21, 64)).astype(np.float32)
    dy = rng.standard_normal((32, 20, 20, 32)).astype(np.float32)
    ref_w = ol.conv2d_wgrad(x.astype(np.float64), dy.astype(np.float64), 2, stride=1)
    dw = torch.empty((32, 2, 2, 64), device="cuda")
    db = torch.empty((32,), device="cuda")
    ctx.conv_wgrad(dev(x.reshape(-1, 64)), dev(dy.reshape(-1, 32)), dw, db, geom, 1.0,
                   accumulate=False, accumulate_db=False, precision=PREC_TF32)
    assert rel(ol.krsc_to_oihw(host(dw)), ref_w) <= 1e-3
    assert rel(host(db), dy.astype(np.float64).reshape(-1, 32).sum(0)) <= 1e-5


def test_gather_rows_multi_equals_one_gather_per_array():
    """The minibatch gather of ttrl/buffers/rollout.py:271-282 for several
    arrays sharing one index list (int32 actions, fp32 fields, rows of
    several words) in one launch: bit for bit one gather per array, with
    repeated and out-of-order indices."""
    ctx = _ctx()
    rng = np.random.default_rng(21)
    n_src, n = 300, 97
    idx = torch.from_numpy(rng.integers(0, n_src, n).astype(np.int32)).cuda()
    srcs = [torch.from_numpy(rng.integers(0, 6, n_src).astype(np.int32)).cuda(),
            dev(rng.standard_normal(n_src).astype(np.float32)),
            dev(rng.standard_normal((n_src, 7)).astype(np.float32)),
            dev(rng.standard_normal((n_src, 3, 4)).astype(np.float32))]
    one = [torch.empty((n,) + tuple(s.shape[1:]), dtype=s.dtype, device="cuda") for s in srcs]
    multi = [torch.empty_like(o) for o in one]
    for s, o in zip(srcs, one):
        ctx.gather_rows(s, idx, o)
    from ttrl_b200._lib import lib
    before = lib().ttrl_launch_count()
    ctx.gather_rows_multi(list(zip(srcs, multi)), idx)
    assert lib().ttrl_launch_count() - before == 1
    for s, o, m in zip(srcs, one, multi):
        want = s.cpu().numpy()[idx.cpu().numpy()]
        assert np.array_equal(host(o), want)
        assert np.array_equal(host(m), want)
