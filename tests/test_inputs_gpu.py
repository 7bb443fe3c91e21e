"""InputBinder's pinned ring and coalesced uploads (ttrl/engine/step/inputs.py
semantics: `load_input` writes a host array into the bound device buffer in
place, the address never changes).

Checks, on the DQN input arena: after each flush the device buffers hold
exactly the arrays loaded last, including when only some inputs are loaded
(the others keep their previous values) and when more loads than ring slots
are in flight before the host waits.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _batch(rng, B):
    return {"obs": rng.integers(0, 256, (B, 4, 84, 84), dtype=np.uint8),
            "next_obs": rng.integers(0, 256, (B, 4, 84, 84), dtype=np.uint8),
            "actions_onehot": np.eye(6, dtype=np.float32)[rng.integers(0, 6, B)],
            "rewards": rng.standard_normal((B, 1)).astype(np.float32),
            "dones": (rng.random((B, 1)) < 0.5).astype(np.float32),
            "discounts": np.full((B, 1), 0.99, np.float32)}


@pytest.mark.parametrize("deferred", [False, True])
def test_binder_uploads_every_batch_in_place(deferred):
    from ttrl_b200.algos.dqn import step_inputs
    from ttrl_b200.engine.step import InputBinder
    B = 32
    inputs = step_inputs((4, 84, 84), "cuda", batch=B, num_actions=6)
    ptrs = {k: v.data.data_ptr() for k, v in inputs.items()}
    binder = InputBinder("cuda", inputs, deferred=deferred)
    assert binder._arena is not None  # one allocation, coalesced copies
    rng = np.random.default_rng(0)
    current = {}
    history = []
    # Seven batches back to back (more than the ring's three slots), some
    # loading only a subset of the inputs.
    for step in range(7):
        batch = _batch(rng, B)
        names = list(batch) if step % 3 != 1 else ["obs", "rewards", "discounts"]
        for k in names:
            binder.load(k, batch[k])
            current[k] = batch[k]
        binder.flush()
        # A device-side snapshot of what a replay at this point would read.
        history.append(({k: v.data.clone() for k, v in inputs.items()}, dict(current)))
    torch.cuda.synchronize()
    for snap, want in history:
        for k, arr in want.items():
            got = snap[k].cpu().numpy().reshape(arr.shape)
            assert np.array_equal(got, arr.astype(got.dtype)), k
    assert {k: v.data.data_ptr() for k, v in inputs.items()} == ptrs
    binder.close()


def test_pinned_inputs_upload_without_a_host_copy():
    """TrainStep-style deferred binder fed from its pinned mirror: each flush
    is one transfer of the whole batch, and the device sees the mirror's
    contents at the time of the flush."""
    from ttrl_b200.algos.dqn import step_inputs
    from ttrl_b200.engine.step import InputBinder
    B = 16
    inputs = step_inputs((4, 84, 84), "cuda", batch=B, num_actions=6)
    binder = InputBinder("cuda", inputs, deferred=True)
    pinned = binder.pinned_inputs()
    rng = np.random.default_rng(3)
    for step in range(4):
        batch = _batch(rng, B)
        if binder.last_upload is not None:
            binder.last_upload.synchronize()  # the previous upload read the mirror
        for k, v in batch.items():
            pinned[k].copy_(torch.from_numpy(v).reshape(pinned[k].shape))
        for k in batch:
            binder.load(k, pinned[k])
        binder.flush()
        torch.cuda.synchronize()
        for k, v in batch.items():
            got = inputs[k].data.cpu().numpy().reshape(v.shape)
            assert np.array_equal(got, v.astype(got.dtype)), (step, k)
    binder.close()
