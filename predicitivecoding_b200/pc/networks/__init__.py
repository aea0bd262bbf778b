"""Advanced predictive-coding architectures built on :class:`~predicitivecoding_b200.pc.network.Network`.

Reference: PredicitiveCoding/Networks/*/ (17 wrappers).  Each module cites its reference file.
"""
from .temporal import TemporalNetwork
from .moe import (HierarchicalMixtureOfExperts, HierarchicalMoEConfig, MixtureOfExperts, MixtureOfExpertsConfig,
                  TemporalMixtureOfExperts, TemporalMoEConfig, compute_gates)
from .ensemble import EnsembleConfig, EnsembleNetwork
from .variants import AttentiveNetwork, AttentiveNetworkConfig, ResidualNetwork, ResidualNetworkConfig
from .compositions import (ActiveNetwork, ActiveNetworkConfig, DeepRecurrentNetwork, DeepRecurrentNetworkConfig,
                           GatedStateNetwork, GatedStateNetworkConfig, GenerativeNetwork, GenerativeNetworkConfig,
                           GraphPredictiveNetwork, GraphPredictiveNetworkConfig, HierarchicalNetwork,
                           HierarchicalNetworkConfig, HopfieldMemory, HopfieldNetwork, HopfieldNetworkConfig)
from .extras import (MemoryBank, MemoryNetwork, MemoryNetworkConfig, ModalityConfig, MultiModalNetwork,
                     MultiModalNetworkConfig, RoutedNetwork, RoutedNetworkConfig, RoutedPrediction, SpikingNetwork,
                     SpikingNetworkConfig)
