"""Learner updates of the three algorithms (ttrl/algos): DQN's update body,
PPO's objective and minibatch update, SAC's losses and regions, and the
gradient-norm utilities, running on the fused B200 kernels."""
