"""The recurrent actor-critic (ttrl/nets/recurrent.py): trunk, then a GRU
memory, then the policy and value heads.

`forward` is the training path over a minibatch of whole sequences: rows
time-major (row t * n_seq + s), one h0 per memory, and the (seq_len, n_seq, 1)
episode-start mask the unroll applies to the state entering each timestep.
`step` is the acting path, one timestep from a caller-owned state, with the
same done mask in the same position (on the state entering the cell).

The observation here is one leaf, so the trunk and the memory are shared by
both heads (the reference's symmetric case, ttrl/nets/recurrent.py:164-196);
`hidden_sizes` then names one memory, "actor".
"""

from __future__ import annotations

from ttrl_b200.engine.nn import Module, ModuleDict
from ttrl_b200.engine.ops import apply_done_mask, reshape
from ttrl_b200.engine.recurrent import GRU
from ttrl_b200.nets.build import build_encoder
from ttrl_b200.nets.heads import CategoricalHead, ValueHead
from ttrl_b200.nets.models import _leaf

__all__ = ["ACTOR", "CRITIC", "RecurrentActorCritic", "build_recurrent_actor_critic"]

ACTOR = "actor"
CRITIC = "critic"


class RecurrentActorCritic(Module):
    """Trunk -> GRU -> policy and value heads, with the state supplied
    (ttrl/nets/recurrent.py:49-161)."""

    def __init__(self, actor, critic, memories: ModuleDict, policy, value, hidden_size: int):
        self.encoders = ModuleDict({ACTOR: actor, CRITIC: critic})
        self.memories = memories
        self.heads = ModuleDict({"policy": policy, "value": value})
        self.hidden_size = int(hidden_size)
        self._shared = memories[ACTOR] is memories[CRITIC]

    @property
    def shared(self) -> bool:
        return self._shared

    @property
    def hidden_sizes(self) -> dict:
        if self.shared:
            return {ACTOR: self.hidden_size}
        return {ACTOR: self.hidden_size, CRITIC: self.hidden_size}

    # -- training -----------------------------------------------------------

    def forward(self, obs, h0: dict, starts, *, seq_len: int):
        self._check_states(h0, "forward")
        actor_state = self._unroll(ACTOR, obs, h0[ACTOR], starts, seq_len)
        policy_out = self.heads["policy"](actor_state)
        if self.shared:
            return policy_out, self.heads["value"](actor_state)
        critic_state = self._unroll(CRITIC, obs, h0[CRITIC], starts, seq_len)
        return policy_out, self.heads["value"](critic_state)

    def _unroll(self, which: str, obs, h0, starts, seq_len: int):
        features = self.encoders[which](_leaf(obs))
        rows, width = (int(d) for d in features.shape)
        if rows % seq_len:
            raise ValueError(
                f"RecurrentActorCritic: {rows} rows is not a whole number of sequences of "
                f"seq_len={seq_len}. A recurrent minibatch is a set of whole sequences, so "
                f"choose a minibatch_size that is a multiple of recurrent.seq_len."
            )
        n_seq = rows // seq_len
        sequence = reshape(features, (seq_len, n_seq, width))
        outputs, _final = self.memories[which](sequence, h0, starts)
        return reshape(outputs, (rows, self.hidden_size))

    # -- acting -------------------------------------------------------------

    def step(self, obs, h_prev: dict, start: dict):
        """One timestep -> (policy_out, value, h_next by memory name)."""
        self._check_states(h_prev, "step")
        self._check_states(start, "step")
        actor_next = self._cell(ACTOR, obs, h_prev[ACTOR], start[ACTOR])
        policy_out = self.heads["policy"](actor_next)
        if self.shared:
            return policy_out, self.heads["value"](actor_next), {ACTOR: actor_next}
        critic_next = self._cell(CRITIC, obs, h_prev[CRITIC], start[CRITIC])
        return (policy_out, self.heads["value"](critic_next),
                {ACTOR: actor_next, CRITIC: critic_next})

    def _cell(self, which: str, obs, h_prev, start):
        features = self.encoders[which](_leaf(obs))
        return self.memories[which].cell(features, apply_done_mask(h_prev, start))

    def _check_states(self, states: dict, where: str) -> None:
        wanted = set(self.hidden_sizes)
        if set(states) != wanted:
            raise ValueError(
                f"RecurrentActorCritic.{where}: this network carries memories "
                f"{sorted(wanted)} and was given {sorted(states)}."
            )


def build_recurrent_actor_critic(obs_shape, n_actions: int, device=None, *, batch: int,
                                 hidden_size: int, **encoder_kwargs) -> RecurrentActorCritic:
    """`build_actor_critic`'s recurrent twin: a GRU between trunk and heads.
    Parameters are drawn in the reference's order (trunk, GRU, policy head,
    value head), so one numpy seed gives both sides the same weights."""
    if hidden_size < 1:
        raise ValueError(f"build_recurrent_actor_critic: hidden_size must be >= 1, got "
                         f"{hidden_size}")
    trunk = build_encoder(obs_shape, device, batch=batch, **encoder_kwargs)
    memory = GRU(trunk.out_features, hidden_size, device)
    return RecurrentActorCritic(trunk, trunk, ModuleDict({ACTOR: memory, CRITIC: memory}),
                                CategoricalHead(hidden_size, n_actions, device),
                                ValueHead(hidden_size, device), hidden_size)
