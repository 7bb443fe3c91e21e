"""Small, self-contained kernel cases for profiling (`ncu -k ... python -m
ttrl_b200.profile_case <case>`): each case builds seeded inputs of the
Nature-CNN shapes and launches one kernel family a few times.

    python -m ttrl_b200.profile_case conv1_fprop --batch 256 --reps 3
    python -m ttrl_b200.profile_case dqn_update --reps 3
    python -m ttrl_b200.profile_case ppo_update --reps 2
"""

from __future__ import annotations

import argparse

import numpy as np
import torch

from ttrl_b200.device import context, conv_geom

#: (input extent, in channels, out channels, kernel, stride). conv1s2d is
#: conv1 in the space-to-depth form the nets run it in (fold 4).
CONV = {"conv1": (84, 4, 32, 8, 4), "conv1s2d": (21, 64, 32, 2, 1),
        "conv2": (20, 32, 64, 4, 2), "conv3": (9, 64, 64, 3, 1)}


def _conv_case(layer: str, kind: str, batch: int, reps: int) -> None:
    hw, c, co, k, s = CONV[layer]
    g = conv_geom(batch, hw, hw, c, co, k, k, s, 0)
    rng = np.random.default_rng(0)
    dev = torch.device("cuda", 0)
    x = torch.from_numpy(rng.standard_normal((batch * hw * hw, c)).astype(np.float32)).to(dev)
    w = torch.from_numpy(rng.standard_normal((co, k, k, c)).astype(np.float32)).to(dev)
    b = torch.zeros(co, device=dev)
    y = torch.empty((batch * g.oh * g.ow, co), device=dev)
    ctx = context(dev)
    for _ in range(reps):
        if kind == "fprop":
            ctx.conv_fprop(x, w, b, y, g, 1.0, True)
        elif kind == "dgrad":
            ctx.conv_dgrad(y, w, x, torch.empty_like(x), g, False)
        else:
            ctx.conv_wgrad(x, y, torch.empty_like(w), b, g, 1.0, False, False)
    torch.cuda.synchronize()


def _linear_case(reps: int, batch: int) -> None:
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(0)
    x = torch.from_numpy(rng.standard_normal((batch, 3136)).astype(np.float32)).to(dev)
    w = torch.from_numpy(rng.standard_normal((3136, 512)).astype(np.float32)).to(dev)
    b = torch.zeros(512, device=dev)
    y = torch.empty((batch, 512), device=dev)
    ctx = context(dev)
    for _ in range(reps):
        ctx.linear_fwd(x, w, b, y, True)
    torch.cuda.synchronize()


def _dqn_case(reps: int) -> None:
    from ttrl_b200.algos import dqn
    from ttrl_b200.engine.optim import Adam
    from ttrl_b200.engine.step import TrainStep
    from ttrl_b200.nets import build_q_net
    np.random.seed(0)
    online = build_q_net((4, 84, 84), 6, "cuda", batch=32)
    target = build_q_net((4, 84, 84), 6, "cuda", batch=32)
    opt = Adam(list(online.parameters()), lr=1e-4, eps=1.5e-4)
    inputs = dqn.step_inputs((4, 84, 84), "cuda", batch=32, num_actions=6)
    step = TrainStep(lambda i: dqn.update_loss(online, target, i, num_actions=6), inputs,
                     "cuda", optimizer=opt, mode="traced_fwd_bwd")
    rng = np.random.default_rng(1)
    step.load_input("obs", rng.integers(0, 256, (32, 4, 84, 84), dtype=np.uint8))
    step.load_input("next_obs", rng.integers(0, 256, (32, 4, 84, 84), dtype=np.uint8))
    step.load_input("actions_onehot", np.eye(6, dtype=np.float32)[rng.integers(0, 6, 32)])
    for _ in range(reps):
        step.launch()
    torch.cuda.synchronize()
    step.close()


def _ppo_case(reps: int) -> None:
    """One PPO rollout update (8 x 128 frames, 4 epochs x 4 minibatches of
    256) replayed `reps` times from its CUDA graph."""
    from ttrl_b200.algos.ppo import PPOConfig, PPOLearner, initial_old_logp
    from ttrl_b200.nets import build_actor_critic
    np.random.seed(0)
    net = build_actor_critic((4, 84, 84), 6, "cuda", batch=256)
    learner = PPOLearner(net, 1024, (4, 84, 84), "cuda", cfg=PPOConfig(epochs=4, minibatch_size=256))
    rng = np.random.default_rng(0)
    obs = rng.integers(0, 256, (1024, 4, 84, 84), dtype=np.uint8)
    actions = rng.integers(0, 6, 1024)
    old_logp, values = initial_old_logp(net, obs, actions, "cuda")
    learner.load_rollout(obs, actions, old_logp, values, rng.standard_normal(1024),
                         rng.standard_normal(1024))
    learner.draw_permutations()
    learner.capture()
    for _ in range(reps):
        learner.replay()
    torch.cuda.synchronize()
    learner.close()


def _rppo_case(reps: int) -> None:
    """One recurrent PPO rollout update (16 x 128 frames, T=32, GRU 256,
    4 epochs x 4 minibatches of 16 sequences) replayed `reps` times."""
    from ttrl_b200.algos.ppo import PPOConfig
    from ttrl_b200.algos.recurrent_ppo import RecurrentPPOLearner
    from ttrl_b200.nets import build_recurrent_actor_critic
    np.random.seed(0)
    net = build_recurrent_actor_critic((4, 84, 84), 6, "cuda", batch=512, hidden_size=256)
    learner = RecurrentPPOLearner(net, 128, 16, (4, 84, 84), "cuda",
                                  cfg=PPOConfig(minibatch_size=512), seq_len=32)
    rng = np.random.default_rng(0)
    shape = (128, 16)
    learner.load_rollout(rng.integers(0, 256, shape + (4, 84, 84), dtype=np.uint8),
                         rng.integers(0, 6, shape), np.full(shape, np.log(1 / 6), np.float32),
                         rng.standard_normal(shape), rng.standard_normal(shape),
                         rng.standard_normal(shape),
                         starts=(rng.random(shape) < 0.01).astype(np.float32),
                         hidden=np.zeros((4, 16, 256), np.float32))
    learner.draw_permutations()
    learner.capture()
    for _ in range(reps):
        learner.replay()
    torch.cuda.synchronize()
    learner.close()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("case")
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--reps", type=int, default=3)
    a = ap.parse_args()
    if a.case == "dqn_update":
        _dqn_case(a.reps)
        return
    if a.case == "ppo_update":
        _ppo_case(a.reps)
        return
    if a.case == "rppo_update":
        _rppo_case(a.reps)
        return
    if a.case == "fc1_fwd":
        _linear_case(a.reps, a.batch)
        return
    layer, kind = a.case.split("_")
    _conv_case(layer, kind, a.batch, a.reps)


if __name__ == "__main__":
    main()
