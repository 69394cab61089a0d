"""B200-native filtered-QKV hot path of nanochat-filter.

The fused, head-interleaved QKV + decay-logit projection (tcgen05 tensor cores) and the
time-variable low-pass scan h_t = (1 - alpha_t) h_{t-1} + alpha_t u_t, forward and backward,
plus the one-step decode update — behind the reference's own `torch.ops.nanochat_cuda` operator
schemas and module classes. Importing the package registers the operators; the CUDA library
(libltvqkv.so, C ABI in include/ltvqkv.h) is loaded on first use and must have been built.
"""

from . import ops  # noqa: F401  (registers torch.ops.nanochat_cuda.*)
from .filters import (  # noqa: F401
    LtvCombinedHeadMajorQkvFilter,
    LtvCombinedQkvFilterBase,
    LtvCudaFusedConcatHeadMajorRegisterCastBlellochScanQkvFilter,
)
from .kv_cache import KVCache  # noqa: F401
from .lookback import (  # noqa: F401
    UNBOUNDED_LAYER_SPEC,
    UNBOUNDED_P,
    ChunksAndHistory,
    LtvLookBackFusedConcatHeadMajorRegisterCastBlellochScanQkvFilter,
    LtvLookBackFusedConcatHeadMajorRegisterCastSequentialScanQkvFilter,
    LtvLookBackHeadMajorQkvFilter,
    LtvLookBackQkvComputerModule,
    advance_kv_cache,
)
from .module import LtvCombinedQkvComputerModule  # noqa: F401
from .ops import (  # noqa: F401
    fused_linear_transpose,
    ltv_cuda_fused_concat_head_major_register_cast_blelloch_scan,
    ltv_decode_step,
)
from .util import LtvInitValues  # noqa: F401
