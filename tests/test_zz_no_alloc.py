"""ttrl_linear_fwd_noalloc, the workspace-free Linear forward, against
ttrl_linear_fwd with a caller workspace, both through the C ABI.

The no-alloc variant takes its split-K scratch from one fixed array per
device that every call shares, so the checks run two calls in a row on one
stream: the second must not see anything the first left behind. Outputs
must be bit-identical, since both calls run the same split-K schedule and
reduce in the same order. This file is collected last so it also runs after
every other GPU test has used the library in the same process.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

NOALLOC_SCRATCH_BYTES = 4 << 20  # TTRL_NOALLOC_SCRATCH_BYTES
EWORKSPACE = 3


def _setup():
    from ttrl_b200 import _lib
    lib = _lib.lib()
    _lib.check(lib.ttrl_init(0), "ttrl_init")
    return _lib, lib


def _inputs(rng, m, k, n, dev):
    x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).to(dev)
    w = torch.from_numpy((rng.standard_normal((k, n)) / np.sqrt(k)).astype(np.float32)).to(dev)
    b = torch.from_numpy(rng.standard_normal(n).astype(np.float32)).to(dev)
    return x, w, b


@pytest.mark.parametrize("m,k,n,relu,use_bias,prec", [
    (32, 32768, 128, 1, True, 0),  # long K: 32 splits summed through the fixed scratch
    (32, 3136, 512, 1, True, 0),   # Nature-CNN fc1 at batch 32: split-K inside a cluster
    (256, 512, 64, 0, True, 0),    # a few splits inside a cluster
    (128, 512, 512, 1, False, 1),  # single-pass TF32
    (8, 16, 6, 0, True, 0),        # one k-block, no split
])
def test_noalloc_matches_workspace_entry(m, k, n, relu, use_bias, prec):
    _lib, lib = _setup()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev).cuda_stream
    rng = np.random.default_rng(m * 7919 + k * 31 + n)
    status = torch.zeros(4, dtype=torch.int32, device=dev)
    ws_bytes = 64 << 20
    ws = torch.zeros(ws_bytes // 4, dtype=torch.float32, device=dev)

    sets = [_inputs(rng, m, k, n, dev) for _ in range(2)]
    want = [torch.empty((m, n), device=dev) for _ in range(2)]
    got = [torch.full((m, n), float("nan"), device=dev) for _ in range(2)]
    for (x, w, b), y in zip(sets, want):
        _lib.check(lib.ttrl_linear_fwd(
            x.data_ptr(), w.data_ptr(), b.data_ptr() if use_bias else None, y.data_ptr(),
            m, k, n, relu, prec, ws.data_ptr(), ws_bytes, status.data_ptr(), stream),
            "ttrl_linear_fwd")
    # Two no-alloc calls back to back on one stream, no host sync between.
    for (x, w, b), y in zip(sets, got):
        _lib.check(lib.ttrl_linear_fwd_noalloc(
            x.data_ptr(), w.data_ptr(), b.data_ptr() if use_bias else None, y.data_ptr(),
            m, k, n, relu, prec, status.data_ptr(), stream), "ttrl_linear_fwd_noalloc")
    torch.cuda.synchronize(dev)
    assert status.cpu().tolist() == [0, 0, 0, 0]
    for y_want, y_got in zip(want, got):
        assert torch.isfinite(y_got).all()
        assert torch.equal(y_want, y_got)
    # And the result is the linear layer (fp32 within the TF32 tolerance).
    x, w, b = sets[1]
    ref = x.double() @ w.double() + (b.double() if use_bias else 0.0)
    if relu:
        ref = ref.clamp_min(0.0)
    err = (got[1].double() - ref).abs().max().item() / max(ref.abs().max().item(), 1e-30)
    assert err <= 1e-3, err


def test_noalloc_refuses_oversized_scratch():
    _lib, lib = _setup()
    dev = torch.device("cuda", 0)
    m, k, n = 256, 32768, 256  # long K: 32 splits x 256 KB of partial sums
    x = torch.zeros((m, k), device=dev)
    w = torch.zeros((k, n), device=dev)
    y = torch.zeros((m, n), device=dev)
    status = torch.zeros(4, dtype=torch.int32, device=dev)
    torch.cuda.synchronize(dev)
    launched = lib.ttrl_launch_count()
    rc = lib.ttrl_linear_fwd_noalloc(x.data_ptr(), w.data_ptr(), None, y.data_ptr(), m, k, n,
                                     0, 0, status.data_ptr(),
                                     torch.cuda.current_stream(dev).cuda_stream)
    assert rc == EWORKSPACE
    # Refused before anything was enqueued: no kernel of the library ran.
    assert lib.ttrl_launch_count() == launched
    msg = lib.ttrl_last_error().decode()
    assert "ttrl_linear_fwd_noalloc" in msg and str(NOALLOC_SCRATCH_BYTES) in msg
    torch.cuda.synchronize(dev)
    assert status.cpu().tolist() == [0, 0, 0, 0]
