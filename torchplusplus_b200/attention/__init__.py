"""torchpp.attention on B200: GQA / MQA / MHA / sliding-window / cross
attention over the sm_100a flash-attention kernels (no flash_attn package)."""
from .ca import CrossAttention  # noqa: F401
from .gqa import GroupedQueryAttention  # noqa: F401
from .mha import MultiHeadAttention  # noqa: F401
from .mqa import MultiQueryAttention  # noqa: F401
from .swa import SlidingWindowAttention  # noqa: F401
