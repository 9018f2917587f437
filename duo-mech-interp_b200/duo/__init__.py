"""duo: B200 (sm_100a) token-mixing engine for Qwen3.5-shaped decoders.

Host mirror of scasella/duo-mech-interp's engine/model.js `Model` over the C ABI of libduo_mixer.so
(include/duo_mixer.h).  PyTorch is used for device memory and streams only; every kernel is hand-written CUDA.
"""
from . import ops
from .config import Config, qwen35_0p8b
from .lib import DuoError
from .model import Model
from .weights import Weights, from_state_dict, random_weights

__all__ = ["Config", "qwen35_0p8b", "Model", "Weights", "from_state_dict", "random_weights", "ops", "DuoError"]
