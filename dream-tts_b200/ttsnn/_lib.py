"""ctypes binding of libtts_cuda.so (the C ABI declared in include/tts_cuda.h).

Loading fails loudly when the library has not been built: there is no other implementation
behind these functions.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libtts_cuda.so")
# TTS_LIB selects another build of the same library (the timeline build, for tracing)
LIB_PATH = os.environ.get("TTS_LIB") or LIB_PATH

TTS_OK = 0
STATUS = {0: "OK", 1: "INVALID_ARG", 2: "UNSUPPORTED_SHAPE", 3: "CUDA", 4: "TIMEOUT", 5: "OOM"}

EPI_F32, EPI_F16, EPI_RESIDUAL_F32, EPI_SWIGLU_F16 = 0, 1, 2, 3


class TtsError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS.get(status, status)}: {msg}")
        self.status = status


class KvCache(C.Structure):
    _fields_ = [("k_pages", C.c_void_p), ("v_pages", C.c_void_p), ("block_table", C.c_void_p),
                ("max_blocks", C.c_int), ("block_size", C.c_int), ("num_blocks", C.c_int),
                ("n_kv", C.c_int), ("head_dim", C.c_int)]


class StackGeometry(C.Structure):
    _fields_ = [("dim", C.c_int), ("layers", C.c_int), ("heads", C.c_int), ("n_kv", C.c_int),
                ("head_dim", C.c_int), ("ffn", C.c_int), ("eps", C.c_float),
                ("rope_base", C.c_double), ("rope_len", C.c_int), ("codebooks", C.c_int),
                ("vocab", C.c_int)]


class LayerWeights(C.Structure):
    _fields_ = [("attn_norm", C.c_void_p), ("ffn_norm", C.c_void_p), ("wqkv", C.c_void_p),
                ("qk_norms", C.c_void_p), ("wo", C.c_void_p), ("w_gate_up", C.c_void_p),
                ("w_down", C.c_void_p)]


class DecodeState(C.Structure):
    _fields_ = [("lanes", C.c_int), ("positions", C.c_void_p), ("block_table", C.c_void_p),
                ("max_blocks", C.c_int), ("block_size", C.c_int), ("num_blocks", C.c_int),
                ("k_pages", C.c_void_p), ("v_pages", C.c_void_p), ("max_span", C.c_int)]


class PredictorWeights(C.Structure):
    _fields_ = [("resize", C.c_void_p), ("resize_bias", C.c_void_p), ("heads", C.c_void_p),
                ("resized", C.c_void_p), ("tables", C.c_void_p), ("steps", C.c_int),
                ("embed_dim", C.c_int)]


class KvPoolDesc(C.Structure):
    _fields_ = [("layers", C.c_int), ("n_kv", C.c_int), ("head_dim", C.c_int),
                ("block_size", C.c_int), ("num_blocks", C.c_int), ("max_lanes", C.c_int),
                ("max_blocks", C.c_int), ("k_pages", C.c_void_p), ("v_pages", C.c_void_p),
                ("block_table", C.c_void_p), ("positions", C.c_void_p)]


class PickRule(C.Structure):
    _fields_ = [("ban", C.c_void_p), ("counts", C.c_void_p), ("frames", C.c_void_p),
                ("penalty", C.c_float), ("eos", C.c_int), ("min_new", C.c_int)]


class TextFeed(C.Structure):
    _fields_ = [("rows", C.c_void_p), ("len", C.c_int), ("pad", C.c_void_p),
                ("frames", C.c_void_p)]


class TensorView(C.Structure):
    _fields_ = [("name", C.c_char_p), ("dtype", C.c_int), ("ndim", C.c_int),
                ("shape", C.c_longlong * 8), ("data", C.c_void_p), ("nbytes", C.c_size_t)]


P = C.c_void_p
I = C.c_int
L = C.c_long
F = C.c_float

# name -> argtypes; every function returns tts_status (int) unless listed in _RESTYPE.
SIGNATURES = {
    "tts_abi_version": [],
    "tts_last_error": [],
    "tts_launch_count": [I],
    "tts_ctx_create": [I, I, C.POINTER(P)],
    "tts_ctx_destroy": [P],
    "tts_ctx_check": [P, P],
    "tts_proj_forward": [P, P, I, I, P, I, I, P, I, P],
    "tts_interleave_gate_up": [P, P, P, I, I, P, P],
    "tts_weight_pack": [P, P, I, I, P, P],
    "tts_proj_forward_packed": [P, P, I, I, P, I, I, P, I, P],
    "tts_proj_forward_rows": [P, P, I, I, P, I, I, P, I, P],
    "tts_rms_norm": [P, P, P, I, I, F, P, P, P],
    "tts_swiglu_mul": [P, P, P, L, P, I, P],
    "tts_snake_beta_nlc": [P, P, I, P, P, L, I, P, I, P],
    "tts_qk_rope_append": [P, P, I, I, P, P, P, I, P, C.POINTER(KvCache), F, P, P],
    "tts_decode_attention": [P, P, I, I, C.POINTER(KvCache), P, I, I, P, I, P],
    "tts_decode_attention_static": [P, I, I, C.POINTER(KvCache), P, I, I, P, I, P],
    "tts_decode_attention_static_check": [P],
    "tts_argmax": [P, P, I, I, P, P, P],
    "tts_conv1d_nlc": [P, P, I, I, I, P, I, I, I, I, P, P, P, P, P, P],
    "tts_stack_create": [P, C.POINTER(StackGeometry), C.POINTER(P)],
    "tts_stack_set_layer": [P, I, C.POINTER(LayerWeights)],
    "tts_stack_set_head": [P, P, P, P],
    "tts_stack_set_feedback": [P, P],
    "tts_stack_destroy": [P],
    "tts_stack_decode_step": [P, C.POINTER(DecodeState), P, P, P, P, P],
    "tts_stack_graph_capture": [P, C.POINTER(DecodeState), P, P, P, P, P, C.POINTER(P)],
    "tts_graph_launch": [P, P],
    "tts_graph_destroy": [P],
    "tts_predictor_create": [P, C.POINTER(PredictorWeights), C.POINTER(P)],
    "tts_predictor_destroy": [P],
    "tts_predictor_frame": [P, C.POINTER(DecodeState), P, P, C.POINTER(TextFeed), P, P, P],
    "tts_predictor_graph_capture": [P, C.POINTER(DecodeState), P, P, C.POINTER(TextFeed), P, P,
                                    P, C.POINTER(P)],
    "tts_stack_set_pick": [P, C.POINTER(PickRule)],
    "tts_talker_pick": [P, P, I, I, C.POINTER(PickRule), I, P, P],
    "tts_topk_sample": [P, P, I, I, P, I, F, P, P],
    "tts_predictor_set_sampling": [P, P, I, I, F],
    "tts_stack_prefill": [P, C.POINTER(DecodeState), P, P, P, P],
    "tts_rvq_gather": [P, P, I, I, I, I, P, I, I, P, P],
    "tts_rope_rows": [P, P, I, I, I, I, I, P, P, I, P],
    "tts_window_attention": [P, P, I, I, I, I, F, P, I, P],
    "tts_layer_norm": [P, P, P, P, I, I, F, P, I, P],
    "tts_depthwise_conv": [P, P, I, I, I, P, I, P, P, P],
    "tts_bias_act": [P, P, I, I, P, I, P, P, P, I, P],
    "tts_safetensors_open": [C.c_char_p, C.POINTER(P)],
    "tts_safetensors_count": [P],
    "tts_safetensors_at": [P, I, C.POINTER(TensorView)],
    "tts_safetensors_find": [P, C.c_char_p, C.POINTER(TensorView)],
    "tts_safetensors_close": [P],
    "tts_talker_frame": [P, C.POINTER(DecodeState), P, C.POINTER(DecodeState),
                         C.POINTER(TextFeed), P, P, P, P],
    "tts_talker_frame_capture": [P, C.POINTER(DecodeState), P, C.POINTER(DecodeState),
                                 C.POINTER(TextFeed), P, P, P, P, C.POINTER(P)],
    "tts_timeline_read": [P, I, C.POINTER(I), I],
    "tts_kv_pool_create": [P, C.POINTER(KvPoolDesc), C.POINTER(P)],
    "tts_kv_pool_destroy": [P],
    "tts_kv_pool_admit": [P, I, I, I, P],
    "tts_kv_pool_admit_pages": [P, I, C.POINTER(I), I, I, P],
    "tts_kv_pool_share_prefix": [P, I, I, I, I, P],
    "tts_kv_pool_release": [P, I],
    "tts_kv_pool_free_pages": [P],
    "tts_kv_pool_page_refs": [P, I],
    "tts_kv_pool_lane_pages": [P, I, C.POINTER(I), I, C.POINTER(I)],
    "tts_kv_pool_state": [P, I, I, C.POINTER(DecodeState)],
}
_RESTYPE = {"tts_last_error": C.c_char_p, "tts_launch_count": C.c_longlong,
            "tts_safetensors_count": C.c_int, "tts_kv_pool_free_pages": C.c_int,
            "tts_kv_pool_page_refs": C.c_int}

_lib = None


def load() -> C.CDLL:
    """The loaded library; raises if it was never built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python dream-tts_b200/build.py` "
                "(there is no fallback implementation)")
        lib = C.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = _RESTYPE.get(name, C.c_int)
        _lib = lib
    return _lib


def call(name: str, *args) -> None:
    """Calls a tts_status-returning entry point and raises TtsError on failure."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != TTS_OK:
        msg = lib.tts_last_error()
        raise TtsError(rc, msg.decode() if msg else name)


def last_error() -> str:
    msg = load().tts_last_error()
    return msg.decode() if msg else ""
