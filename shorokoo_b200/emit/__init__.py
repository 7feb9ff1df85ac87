"""Stand-in for the reference's ONNX emission: wire writer and the five benchmark graphs."""
from .graphs import CONFIGS, ModelCase, build, mlp, resnet, retinanet, stacked_linear  # noqa: F401
