"""qwen3tts's hot path on B200: the decoder stack and paged decode state (stack.py), the depth
predictor (predictor.py), the lane scheduler (talker.py) and the codec's conv stack (codec.py),
over the ttsnn operators."""
from .stack import Geometry, Graph, LayerTensors, PagedKv, Stack  # noqa: F401
from .predictor import PREDICTOR_GEOMETRY, Predictor, resize_tables  # noqa: F401
