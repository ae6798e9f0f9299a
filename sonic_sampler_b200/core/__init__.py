from sonic_sampler_b200.core.flags import Indicator, indicator_tensor
from sonic_sampler_b200.core.buffers import (
    Flags,
    GumbelNoise,
    RepetitionPenalties,
    SamplingBuffers,
    StochasticWeights,
    TokenCounts,
)
