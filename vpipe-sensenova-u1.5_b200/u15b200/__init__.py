"""u15b200: the SenseNova-U1.5 MoT backbone layer on B200 (sm_100a).

The product is libu15c.so (include/u15c.h); this package is its host-side
mirror of the reference's operator and backbone interfaces.
"""
from ._lib import U15Error, header_symbols, lib  # noqa: F401
from ._lib import (ATTN_BIDIRECTIONAL, ATTN_BLOCK_CAUSAL, ATTN_CAUSAL,  # noqa: F401
                   EPI_RESIDUAL, EPI_STORE, EPI_SWIGLU, EXPERT_GEN, EXPERT_UND)
from .image import FULL_IMAGE, ImagePath  # noqa: F401
from .model import FULL, KvCache, Model  # noqa: F401
from .ops import CudaOps  # noqa: F401
