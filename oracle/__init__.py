"""CPU oracle for the encoder self-attention hot path and the convolution-module plugins
(test infrastructure only).

Imported only by ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py``; the ``fast_gpu_asr_b200`` package never imports it.
"""

from .attention_oracle import (  # noqa: F401
    PADDED_QUERY_HALO,
    parakeet_attention_weights,
    parakeet_relative_attention,
    zipformer_attention_value,
    zipformer_relative_attention,
)
from .convolution_oracle import depthwise_convolution  # noqa: F401,E402
