"""The LeanKV prototype's TurboQuant interface (prototype/turboquant) on B200.

Same import surface as the prototype package: rotation, lloyd_max and
qjl_residual helpers, TurboQuantizer / QuantizedKV (quantizer) and LeanKVCache
(kv_cache).  The per-vector encode and decode run in the fused CUDA kernels of
libleankv_tq.so (tq_proto_encode_cuda / tq_proto_decode_cuda); tensors live on
a CUDA device (device="cuda").  Rotation matrices and Lloyd-Max codebooks are
generated once on the host, as in the prototype.
"""
from .quantizer import QuantizedKV, TurboQuantizer
from .kv_cache import LeanKVCache

__all__ = ["QuantizedKV", "TurboQuantizer", "LeanKVCache"]
