"""B200-native (sm_100a) FlashMoE hot path: Q4 decode matvec, MoE FFN layer
(on-device routing, SwiGLU experts, combine), behind the C ABI in
include/pbmoe_cuda.h. `pb_b200.capi` binds the library; `pb_b200.build`
compiles it."""

from . import capi  # noqa: F401
