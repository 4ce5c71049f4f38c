"""theorem_b200 -- B200 (sm_100a) CUDA implementation of Theorem's forward hot path.

Ops (functional API in ``theorem_b200.ops``; drop-in ``custom_kernel``s in
``theorem_b200.kernels.<op>``):

* causal_conv1d   -- depthwise causal conv (HBM stencil)
* recompute_w_u   -- WY recompute w = A(k beta e^g), u = A(v beta), optional
                     in-kernel triangular solve for A (tcgen05 + TMEM)
* chunk_fwd_h     -- inter-chunk state recurrence, reference or gated delta
                     rule (tcgen05, state resident in TMEM)
* chunk_fwd_o     -- chunkwise output (tcgen05 + TMEM)
* chain           -- the gated-DeltaNet layer forward built from the above

All compute runs in ``libtheorem_b200.so`` (C ABI: include/theorem_b200.h);
the Python layer only validates, allocates and launches.
"""
from . import ops  # noqa: F401

__all__ = ["ops"]
__version__ = "0.1.0"
