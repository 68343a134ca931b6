"""B200-native (sm_100a) implementation of TurboQwenFare's token-sampling path.

The product is libtqfsample.so (CUDA, C ABI in include/tqfs.h); this package
is the host-side mirror of the crate's API over that ABI.
"""
from .decode import DecodeLoop, MtpDecodeLoop
from .mtp import MtpController, MtpStatistics, VerifyOutcome, verify_pair
from .params import PARAMS_DTYPE, SamplingParams, pack
from .sampler import (LogitCandidate, Sampler, Xoshiro256PlusPlus, apply_penalties, params_tensor,
                      sample_batch, top_logit_candidates)

__all__ = [
    "SamplingParams", "PARAMS_DTYPE", "pack", "Sampler", "Xoshiro256PlusPlus", "LogitCandidate",
    "top_logit_candidates", "sample_batch", "apply_penalties", "params_tensor", "verify_pair", "VerifyOutcome",
    "MtpStatistics", "MtpController", "DecodeLoop", "MtpDecodeLoop",
]
