"""vLLM attention backend registration (``ToyFlashAttentionBackend``).

Same surface as ``flash_attention_backend/toy_flash_attn/backend.py:20-139`` of the
reference: backend name ``CUSTOM``, KV-cache shape ``(2, num_blocks, block_size,
num_kv_heads, head_size)`` in NHD order, block sizes ``MultipleOf(16)``, bf16 KV only,
decoder attention only. The compute-capability gate is the one real difference: the
kernels are built for sm_100a only, so only compute capability 10.x is accepted.

Register with::

    from vllm.v1.attention.backends.registry import AttentionBackendEnum, register_backend
    register_backend(AttentionBackendEnum.CUSTOM, "toy_flash_attn.ToyFlashAttentionBackend")
"""

from dataclasses import dataclass

import torch
from vllm.config.cache import CacheDType
from vllm.platforms.interface import DeviceCapability
from vllm.v1.attention.backend import (
    AttentionBackend,
    AttentionImplBase,
    AttentionMetadata,
    AttentionMetadataBuilder,
    AttentionType,
    CommonAttentionMetadata,
    MultipleOf,
)

from .impl import ToyFlashAttentionImpl


class ToyFlashAttentionBackend(AttentionBackend):
    forward_includes_kv_cache_update = False
    accept_output_buffer = True

    @staticmethod
    def get_supported_kernel_block_sizes() -> list[int | MultipleOf]:
        return [MultipleOf(16)]

    @staticmethod
    def get_name() -> str:
        return "CUSTOM"

    @staticmethod
    def get_impl_cls() -> type["AttentionImplBase"]:
        return ToyFlashAttentionImpl

    @staticmethod
    def get_builder_cls():
        return ToyFlashAttentionMetadataBuilder

    @staticmethod
    def get_kv_cache_shape(
        num_blocks: int,
        block_size: int,
        num_kv_heads: int,
        head_size: int,
        cache_dtype_str: str = "auto",
    ) -> tuple[int, ...]:
        return (2, num_blocks, block_size, num_kv_heads, head_size)

    @staticmethod
    def get_kv_cache_stride_order(include_num_layers_dimension: bool = False) -> tuple[int, ...]:
        if include_num_layers_dimension:
            raise NotImplementedError("include_num_layers_dimension is not supported")
        return (0, 1, 2, 3, 4)  # NHD

    @classmethod
    def supports_head_size(cls, head_size: int) -> bool:
        return head_size in (64, 128)

    @classmethod
    def supports_kv_cache_dtype(cls, kv_cache_dtype: "CacheDType | None") -> bool:
        if kv_cache_dtype is None:
            return True
        return kv_cache_dtype in ["bfloat16"]

    @classmethod
    def supports_alibi_sqrt(cls) -> bool:
        return False

    @classmethod
    def supports_mm_prefix(cls) -> bool:
        return False

    @classmethod
    def is_sparse(cls) -> bool:
        return False

    @classmethod
    def supports_attn_type(cls, attn_type: str) -> bool:
        return attn_type == AttentionType.DECODER

    @classmethod
    def supports_compute_capability(cls, capability: "DeviceCapability") -> bool:
        return capability.major == 10

    @classmethod
    def supports_combination(
        cls,
        head_size: int,
        dtype: torch.dtype,
        kv_cache_dtype: "CacheDType | None",
        block_size: int,
        use_mla: bool,
        has_sink: bool,
        use_sparse: bool,
        device_capability: "DeviceCapability",
    ) -> str | None:
        if has_sink or use_sparse or use_mla:
            return "not implement"
        return None


@dataclass
class ToyFlashAttentionMetadata(AttentionMetadata):
    num_actual_tokens: int
    max_query_len: int
    query_start_loc: torch.Tensor
    max_seq_len: int
    seq_lens: torch.Tensor
    block_table: torch.Tensor
    slot_mapping: torch.Tensor
    causal: bool = True


class ToyFlashAttentionMetadataBuilder(AttentionMetadataBuilder[ToyFlashAttentionMetadata]):
    def __init__(self, kv_cache_spec, layer_names, vllm_config, device: torch.device):
        super().__init__(kv_cache_spec, layer_names, vllm_config, device)

    def build(
        self,
        common_prefix_len: int,
        common_attn_metadata: CommonAttentionMetadata,
        fast_build: bool = False,
    ) -> ToyFlashAttentionMetadata:
        del common_prefix_len, fast_build
        return ToyFlashAttentionMetadata(
            num_actual_tokens=common_attn_metadata.num_actual_tokens,
            max_query_len=common_attn_metadata.max_query_len,
            query_start_loc=common_attn_metadata.query_start_loc,
            max_seq_len=common_attn_metadata.max_seq_len,
            seq_lens=common_attn_metadata.seq_lens,
            block_table=common_attn_metadata.block_table_tensor,
            slot_mapping=common_attn_metadata.slot_mapping,
            causal=common_attn_metadata.causal,
        )
