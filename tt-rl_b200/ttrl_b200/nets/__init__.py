"""Networks for the learner hot path (ttrl/nets): the Nature-CNN tower, the
MLP tower, Q / categorical / value / Gaussian heads, the composed models and
their builders, and the recurrent actor-critic. Module trees and parameter names follow the reference's, so
state_dicts are interchangeable."""

from ttrl_b200.nets.build import build_actor_critic, build_q_net, build_sac_nets
from ttrl_b200.nets.heads import CategoricalHead, GaussianHead, QHead, ValueHead
from ttrl_b200.nets.models import ActorCritic, ContinuousCritic, EncoderHead, SacNets
from ttrl_b200.nets.towers import NATURE_CNN, ConvStage
from ttrl_b200.nets.encoders import Encoder, image_encoder, vector_encoder
from ttrl_b200.nets.multi import MultiEncoder
from ttrl_b200.nets.recurrent import RecurrentActorCritic, build_recurrent_actor_critic

__all__ = ["build_actor_critic", "build_q_net", "build_sac_nets", "CategoricalHead",
           "GaussianHead", "QHead", "ValueHead", "ActorCritic", "ContinuousCritic",
           "EncoderHead", "SacNets", "NATURE_CNN", "ConvStage", "Encoder", "image_encoder",
           "vector_encoder", "MultiEncoder", "RecurrentActorCritic", "build_recurrent_actor_critic"]
