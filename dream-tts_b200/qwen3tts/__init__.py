"""qwen3tts's hot path on B200: the decoder stack and paged decode state (stack.py), the lane
scheduler (talker.py) and the codec's conv stack (codec.py), over the ttsnn operators."""
from .stack import Geometry, Graph, LayerTensors, PagedKv, Stack  # noqa: F401
