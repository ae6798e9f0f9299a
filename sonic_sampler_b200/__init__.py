"""B200 (sm_100a) fused LLM sampling and speculative verification, drop-in for the
`sonic_sampler.interface` API of tachyontrails/sonic-sampler.

All GPU work goes through the C ABI of `_lib/libsonic_b200.so` (include/sonic_b200.h)."""

__version__ = "0.1.0"
