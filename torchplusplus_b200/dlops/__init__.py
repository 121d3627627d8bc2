"""torchpp.dlops on B200: fused norms, RoPE and fused linear+activation."""
from .normalization import LayerNormFused, RmsNormFused, LayerNorm4D  # noqa: F401
from .rope import compute_rope_params, qkrope_apply, rope_apply  # noqa: F401
from .linear import Dense, LinearGELU, LinearNBBf16, LinearNBFp16, LinearSILU  # noqa: F401
