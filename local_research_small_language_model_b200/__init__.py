"""B200-native (sm_100a) forecast-guided block-sparse attention for SparDA.

Drop-in for the reference's attention-backend / forecast API
(model/attention/*, model/forecast.py of tyborra/local-research-Small-Language-Model):

* ``KVBlockCompressor``, ``ForecastBlockSelector``  (model/forecast.py)
* ``B200SparseAttention``, ``gather_kv_blocks``      (model/attention/sparse.py)
* ``B200KVCache``                                    (model/attention/base.py KVCache)
* ``B200OffloadKVCache``                             (model/attention/offload.py, async_offload.py)
* ``install(model)`` swaps the attention of every layer of a reference model.

All compute runs in libspardab200.so (hand-written CUDA for sm_100a, C ABI in
include/spardab200.h).  There is no CPU path.
"""

from .config import ModelConfig
from .cache import B200KVCache
from .offload import B200OffloadKVCache
from .forecast import ForecastBlockSelector, ForecastProjection, KVBlockCompressor
from .attention import B200SparseAttention, BaseAttention
from .ops import gather_kv_blocks
from .rope import RotaryEmbedding
from . import ops
from ._lib import SparDAError, load as load_library

__all__ = ["ModelConfig", "B200KVCache", "B200OffloadKVCache", "ForecastBlockSelector", "ForecastProjection", "KVBlockCompressor",
           "B200SparseAttention", "BaseAttention", "gather_kv_blocks", "RotaryEmbedding", "ops", "SparDAError",
           "load_library", "install"]


def install(model, rule: str = "reference"):
    """Replaces ``layer.attention`` of every layer of a reference-style model
    with B200SparseAttention, keeping wq/wk/wv/wo (the factory in
    model/transformer.py:34-51 has no registry, so the swap is by module)."""
    import torch
    for layer in model.layers:
        old = layer.attention
        new = B200SparseAttention(old.config, old.layer_idx, mode=getattr(old, "mode", None), rule=rule)
        with torch.no_grad():
            for name in ("wq", "wk", "wv", "wo"):
                getattr(new, name).weight.copy_(getattr(old, name).weight)
        new.to(device=old.wq.weight.device, dtype=old.wq.weight.dtype)
        layer.attention = new
    return model
