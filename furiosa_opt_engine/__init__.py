"""Load Hugging Face checkpoints onto NVIDIA Blackwell GPUs and call their computations from
Python: the public surface of the engine (checkpoints, load options, devices, buffers, tensors,
decoders and their caches)."""

from ._api import *  # noqa: F401,F403
from ._api import __all__ as __all__
