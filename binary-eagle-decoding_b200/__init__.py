"""bitdraft-b200: B200 (sm_100a) kernels for the one-bit HE4 drafter hot path.

The model/config API mirrors ``w1a1_eagle.model`` of the reference
(philippesic/binary-eagle-decoding): ``Geometry``, ``Projection``, ``Layer``,
``HE4``, ``hard_sign``, ``bound_latents``, ``clamp_latents``, ``cache_storage``,
``rms``, ``rope``; ``export`` writes the FFN layers as the reference's GGUF
format.  All computation on the hot path runs in ``libbitdraft.so``
(C ABI in ``include/bitdraft.h``); there is no CPU fallback.
"""

from . import _lib, export, ops  # noqa: F401
from .model import (HE4, FrozenLinear, Geometry, LatentGradients, Layer, Projection, bound_latents,  # noqa: F401
                    cache_storage, clamp_latents, hard_sign, rms, rope)
