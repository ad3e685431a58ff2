"""nsrl_b200 -- B200-native (sm_100a) implementation of the NSRL integer
transformer hot path: the i16 x i8 linears, the causal base-2 integer softmax
attention block, the integer RMS norm, gated MLP and residuals, and the i16
KV-cache decode attention.

The compute lives in libnsrl_b200.so (hand-written CUDA behind a C ABI,
include/nsrl_b200.h).  `nsrl_b200.core` mirrors the reference's nsrl-core
function names over device tensors and returns None where the reference
returns `None`.  Importing this package does not load the library; the first
call does, and fails loudly if the library or a CUDA device is missing.
"""
