"""B200 (sm_100a) paged-KV attention forward behind the reference's vLLM backend surface.

``toy_flash_attn.ToyFlashAttentionBackend`` is resolved lazily so the kernel entry points
(``toy_flash_attn.flash_attention_func``) import without vLLM.
"""

__all__ = ["ToyFlashAttentionBackend"]


def __getattr__(name):
    if name == "ToyFlashAttentionBackend":
        from .backend import ToyFlashAttentionBackend

        return ToyFlashAttentionBackend
    raise AttributeError(name)
