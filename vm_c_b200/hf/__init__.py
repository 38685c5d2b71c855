"""HuggingFace checkpoints: safetensors container and a tensor source under GGUF names."""
from .safetensors_io import SafetensorsFile, save_file  # noqa: F401
from .source import HfSource  # noqa: F401
