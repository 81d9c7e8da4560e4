"""B200-native (sm_100a) q6 affine linear and image feed-forward MLP.

Drop-in for the q6 path of qwen-image-shardedit-mlx: MLX-layout 6-bit affine
weights (packed uint32 codes + bf16 per-group scale/bias), the reference's
`affine_q6_qmm_t` / `fused_q6_mlp` call surface, computed by hand-written
tcgen05 / CUDA-core kernels behind the C ABI in include/q6_b200.h.
"""

from qwen_image_shardedit_mlx_b200.ops import (  # noqa: F401
    clear_device_error,
    device_error,
    last_path,
    q6_dequantize,
    q6_linear,
    q6_mlp,
)
from qwen_image_shardedit_mlx_b200.q6_metal_mlp import (  # noqa: F401
    DenseLinearWeights,
    Q6LinearSpec,
    QuantizedLinear,
    QwenFeedForward,
    affine_q6_qmm_t,
    dense_mlp,
    dense_mlp_from_q6,
    dequantize_linear,
    eager_q6_mlp,
    fused_q6_mlp,
    make_feed_forward_callables,
    quantized_linear_spec,
)
from qwen_image_shardedit_mlx_b200.quantize import pack_codes, quantize_affine_q6, unpack_codes  # noqa: F401

__version__ = "0.1.0"
