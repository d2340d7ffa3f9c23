"""B200 batched token sampler: Python front end of libllamars_sampler.so.

The package directory llama.rs_b200/ is put on sys.path by callers
(tests/conftest.py, bench.py, __graft_entry__.py); this module is `lrs`.
"""
from .sampler import (  # noqa: F401
    EXPORTS, LRS_E_CUDA, LRS_E_INTERNAL, LRS_E_INVALID, LRS_E_NAN, LRS_E_NCCL, LRS_E_NOMEM, LRS_E_TIMEOUT,
    LRS_OK, ROW_INFO_DTYPE, TOKEN_NONE, BatchSampler, Sampler, SamplerError, SamplerPanic, SamplingParams, lib,
)
from .workloads import PARAMS_DTYPE  # noqa: F401
