"""The op layer every model component calls.

Each op has a plain-PyTorch path (CPU; the numerical oracle the tests use)
and an sm_100a path (CUDA tensors): hand-written kernels compiled into the
in-tree extension ``vagus_b200_C`` (``ops/csrc``), wired into autograd here.
On a CUDA tensor the extension must load -- a missing build raises instead of
falling back to eager PyTorch.
"""

from ._core import BF16, check_error, kernels_active, native  # noqa: F401
from .attention import attention, attention_ref, attention_layer, attention_layer_ok  # noqa: F401
from .ce import fused_linear_ce  # noqa: F401
from .gdn import conv_silu, gdn_mixer, gdr_chunk, gdr_decode  # noqa: F401
from .kda import kda_mixer  # noqa: F401
from .kda import kda_chunk  # noqa: F401
from .linear import linear, linear_residual  # noqa: F401
from .mobius import mobius_scan  # noqa: F401
from .pointwise import (embedding, qk_norm_rope, rmsnorm, rmsnorm_gated, rmsnorm_pass, sigmoid_gate,  # noqa: F401
                        swiglu)
