"""lollm_b200 — B200-native (sm_100a) qwen3_5 MTP speculative-decoding step.

The product is libqsp.so (CUDA kernels + C ABI, include/qsp.h) and the host mirror of the
reference family seams in `lollm_b200.qwen3_5` (config, paged cache, forward, MTP head,
speculative decoder) plus the shared loop in `lollm_b200.generate`.
"""

__version__ = "0.1.0"
