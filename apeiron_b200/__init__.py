"""apeiron_b200 — B200-native (sm_100a) backend for apeiron's integer Q8-activation
projection: the Q8_0 / Q4_K / Q6_K decode GEMV (`matvec_q8act`) and the prefill GEMM
(`matmat_q8act`), exact in Q32.32 against the reference's CPU contract.

The compute lives in ``libapeiron_cuda.so`` (C ABI, include/apeiron_cuda.h); this package
is the host-side mirror of the reference interface (``chart``) plus benchmark inputs
(``synth``) and multi-GPU row sharding (``shard``).
"""
from ._abi import Q4_K, Q6_K, Q8_0  # noqa: F401
from .chart import (  # noqa: F401
    AccumulatorOverflow, Backend, BackendError, FixedOverflow, LengthOverflow, MatvecError,
    NonFiniteScale, OutputOverflow, QuantAct, QuantRefused, ShapeMismatch, ShortPayload,
    Tensor, UnsupportedQuant,
)

__version__ = "0.1.0"
