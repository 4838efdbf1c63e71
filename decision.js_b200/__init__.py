"""decision.js on B200: the q8/q4 dequantizing matmul, RMSNorm, RoPE, GLU and attention hot path of
Jacqkues/decision.js as sm_100a CUDA kernels behind a C ABI (include/decision_cuda.h), with the reference's
Decision API on top."""
from ._lib import Context, DecisionError, device_count, lib
from .decision import Decision, forest, passes, shard
from .questions import answer, check_question, softmax

D1 = Decision

__all__ = ["Context", "Decision", "D1", "DecisionError", "answer", "check_question", "device_count", "forest", "lib",
           "passes", "shard", "softmax"]
