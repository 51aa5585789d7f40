"""rus_b200 — B200-native (sm_100a) fused lm_head cross-entropy head.

Drop-in for the chunked vocabulary head of fokyso82002-rgb/rus
(``solution/ops.py:174-349``): ``chunked_lm_head`` returns the loss and the
per-token NLL, Shannon entropy and argmax without materialising [N, V] logits,
and its backward produces dX and dW from hand-written tcgen05/TMA kernels
(``liblmce.so``, C ABI in include/lmce.h).
"""
from .ops import V_CHUNK_DEFAULT, FusedChunkedLMHeadFn, chunked_lm_head
from .tied import TiedGradSlot, tied_embedding

__all__ = ["V_CHUNK_DEFAULT", "FusedChunkedLMHeadFn", "chunked_lm_head", "TiedGradSlot", "tied_embedding"]
