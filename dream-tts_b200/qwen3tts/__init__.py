"""qwen3tts's hot path on B200: the decoder stack and paged decode state (stack.py), the depth
predictor (predictor.py), the reference's talker loop body (frames.py), the lane scheduler
(talker.py) and the codec's conv stack (codec.py), over the ttsnn operators."""
from .stack import Geometry, Graph, LayerTensors, PagedKv, PickState, Stack  # noqa: F401
from .predictor import PREDICTOR_GEOMETRY, Predictor, TextFeed, resize_tables  # noqa: F401
from .frames import FrameLoop, reference_pick  # noqa: F401
