"""B200-native (sm_100a) encoder self-attention for fast-gpu-asr.

Drop-in replacement for the reference's three attention TensorRT plugins
(``parakeet_relative_attention``, ``zipformer_relative_attention``,
``zipformer_attention_value``) and its two convolution-module plugins
(``parakeet_conformer_convolution``, ``zipformer_convolution``): hand-written CUDA
kernels behind the C ABI in ``include/fga_attention.h`` and ``include/fga_convolution.h``,
the same plugin identities for TensorRT, and a data-parallel batch-sharding launcher.
"""

from .attention import (  # noqa: F401
    parakeet_relative_attention,
    zipformer_attention_fused,
    zipformer_attention_value,
    zipformer_relative_attention,
)
from .convolution import (  # noqa: F401
    parakeet_conformer_convolution,
    zipformer_convolution,
)
from .constants import (  # noqa: F401
    PARAKEET_CONFORMER_CONVOLUTION_PLUGIN_NAME,
    PARAKEET_RELATIVE_ATTENTION_PLUGIN_NAME,
    PLUGIN_VERSION,
    TENSORRT_PLUGIN_NAMESPACE,
    ZIPFORMER_ATTENTION_VALUE_PLUGIN_NAME,
    ZIPFORMER_CONVOLUTION_PLUGIN_NAME,
    ZIPFORMER_RELATIVE_ATTENTION_PLUGIN_NAME,
)

__version__ = "0.1.0"
