"""Plugin identifiers and numeric constants shared with the reference.

Names, version and namespace must equal the reference's
(``src/fast_gpu_asr/constants.py:36-47``, ``tensorrt_plugins/plugin_namespace.h:12``):
TensorRT resolves ONNX custom nodes and serialized engines by exactly these strings.
"""

ONNX_OPSET_VERSION = 20
TENSORRT_PLUGIN_NAMESPACE = "fast_gpu_asr"
PLUGIN_VERSION = "1"
PARAKEET_RELATIVE_ATTENTION_PLUGIN_NAME = "parakeet_relative_attention"
ZIPFORMER_RELATIVE_ATTENTION_PLUGIN_NAME = "zipformer_relative_attention"
ZIPFORMER_ATTENTION_VALUE_PLUGIN_NAME = "zipformer_attention_value"
PARAKEET_CONFORMER_CONVOLUTION_PLUGIN_NAME = "parakeet_conformer_convolution"
ZIPFORMER_CONVOLUTION_PLUGIN_NAME = "zipformer_convolution"

# zipformer_relative_attention_plugin.cu:41-42
ZIPFORMER_POSITION_HEAD_DIM = 4
ZIPFORMER_PADDED_QUERY_HALO = 7

# Frame strides used to convert valid frames to audio seconds.
PARAKEET_FRAME_SECONDS = 0.08  # 8x subsampling of 10 ms features
ZIPFORMER_INPUT_FRAME_SECONDS = 0.02  # 50 Hz encoder input frames (2x conv-embed stride)
