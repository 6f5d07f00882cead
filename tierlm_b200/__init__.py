"""tierlm_b200 - the B200 (sm_100a) tier of tierlm's quantised MoE decoder step.

The product is libtlmg.so (CUDA kernels for sm_100a behind the C ABI in
include/tlmg.h). This package builds and loads it and offers a thin Python
mirror of the reference interfaces for tests and benchmarks:

- tierlm_b200.quant  - tlm_quantize_act / tlm_matvec_rows / tlm_vec_dot
- tierlm_b200.moe    - HBM expert slots, expert FFN, the moe() block
- tierlm_b200.attention - decode attention over a paged KV cache (attn_heads)
"""
from ._lib import TlmError, load  # noqa: F401

__all__ = ["TlmError", "load"]
