"""glypr_b200: a B200-native (sm_100a) backend for glypr's EmbeddingGemma text path.

The product is ``libglypr_cuda.so`` (C ABI declared in ``include/glypr_cuda.h``); this
package is a thin host-side mirror of the reference's embedder API over that library.
"""
from .api import (GlyprEmbedder, GlyprError, cosine_similarity, l2_normalize,  # noqa: F401
                  library_path, load_library, truncate_mrl)
