"""acm_b200 -- B200-native engine for auto-commit-msg's token loop.

Load a GGUF model, prefill the prompt, decode with the top-k sampler, all on
hand-written sm_100a kernels behind the C ABI of libacmcuda.so
(include/acm.h).  The Python layer mirrors the reference's internal/infer API.
"""
from ._lib import AcmError, Config, lib  # noqa: F401
from .infer import (Engine, Load, LoadBytes, LoadConfig, LoadConfigBytes, LoadMulti, MaxLogit, Model,  # noqa: F401
                    Sampler, Stats)

__all__ = ["AcmError", "Config", "Engine", "Load", "LoadBytes", "LoadConfig", "LoadConfigBytes", "LoadMulti", "MaxLogit",
           "Model", "Sampler", "Stats", "lib"]
