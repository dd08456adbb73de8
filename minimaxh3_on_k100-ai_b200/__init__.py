"""B200-native (sm_100a) MiniMax-H3 DiT-block hot path.

Host side in Python/PyTorch over the C-ABI library ``libh3b200.so``
(include/h3_b200.h).  ``ops`` mirrors the reference operator API (h3_* fused
pointwise ops, mha, linear, and the fp32 linear / row gather / SiLU ops of the
model wrapper); ``block`` composes one DiT block, ``step`` the 40-block
denoising step, ``model`` the whole transformer forward around it (input
projections, token refiner, packing, output norm and projections);
``ulysses`` shards the block over GPUs with the head<->sequence all-to-all.
"""
from . import ops  # noqa: F401
from .ops import *  # noqa: F401,F403
from ._lib import library_path, load  # noqa: F401

__version__ = "0.1.0"
