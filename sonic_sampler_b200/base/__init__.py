from sonic_sampler_b200.base.sampler import (
    DEFAULT_TOP_LOGPROBS,
    LogProbabilities,
    Selection,
    TopTargets,
    Verification,
)
