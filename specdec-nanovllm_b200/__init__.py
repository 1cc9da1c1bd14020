"""specdec_nanovllm_b200: the decode / speculative-verify hot path of
henry-tmp-de/specdec-nanovllm rebuilt for B200 (sm_100a).

Host code is Python/PyTorch over one C-ABI shared library
(``libspecdec_b200.so``, declared in ``include/specdec_b200.h``) of hand-written
CUDA kernels.  Public surface, mirroring the reference's call signatures:

* ``attention``: ``Attention``, ``paged_attention``, ``paged_decode_attention``,
  ``paged_decode_attention_cuda``, ``flash_attn_with_kvcache``,
  ``flash_attn_varlen_func``, ``store_kvcache``
* ``verify``: ``verify_batch`` -> ``VerifyResult``; ``verify_batch_vocab_parallel`` over
  vocabulary shards (three small all-gathers instead of gathering the logits)
* ``sampler``: ``Sampler``, ``sample``, ``draft_sample_step``
* ``prologue``: ``qk_norm_rope_store`` (split + q/k RMSNorm + rotary + KV store),
  ``rope_cos_sin_cache``
* ``quant``: ``int8_linear``, ``quantize_weight``, ``dequantize_weight``
* ``partition``: sequence sharding and tensor-parallel head sharding
* ``context``: ``Context`` / ``set_context`` / ``get_context`` / ``reset_context``
"""

from . import _lib  # noqa: F401
from .attention import (Attention, flash_attn_varlen_func, flash_attn_with_kvcache,  # noqa: F401
                        paged_attention, paged_attention_readonly, paged_decode_attention,
                        paged_decode_attention_cuda, store_kvcache)
from .context import Context, get_context, reset_context, set_context  # noqa: F401
from .quant import dequantize_weight, int8_linear, quantize_weight  # noqa: F401
from .prologue import qk_norm_rope_store, rope_cos_sin_cache  # noqa: F401
from .sampler import Sampler, draft_sample_step, sample  # noqa: F401
from .verify import VerifyResult, VocabParallelVerify, verify_batch, verify_batch_vocab_parallel  # noqa: F401

LIB_PATH = _lib.LIB_PATH


def load_library():
    """Load the compiled library (raises if it has not been built)."""
    return _lib.lib()
