"""redukt_b200: a B200-native (sm_100a) engine for redukt's backbone decode step.

The product is libredukt_gpu.so (C ABI in include/redukt_gpu.h), a drop-in for redukt's GPU
backbone plugin.  This package builds it and binds it for Python hosts and tests.
"""
from .plugin import (BackendInfo, BackendResult, PluginBackend, PluginError, PluginLibrary, PluginStreams,
                     validate_batch_args)
from .rbin import MAMBA_130M, REFERENCE_TEST_DIMS, MambaDims

__all__ = ["BackendInfo", "BackendResult", "PluginBackend", "PluginError", "PluginLibrary", "PluginStreams",
           "validate_batch_args", "MAMBA_130M", "REFERENCE_TEST_DIMS", "MambaDims"]
