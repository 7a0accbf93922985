"""fna2_b200 -- B200-native (sm_100a) FNA2 fused relational-bias attention.

``from fna2_b200 import flash_naylis_attn, BLOCK_R`` is the drop-in for the
reference's ``from flash_naylis_attn import flash_naylis_attn, BLOCK_R``
(attention_fna2.py:51).
"""
from .flash_naylis_attn import (BLOCK_M, BLOCK_N, BLOCK_R, FlashNaylisAttnFunc,  # noqa: F401
                                flash_naylis_attn)

__all__ = ["flash_naylis_attn", "FlashNaylisAttnFunc", "BLOCK_M", "BLOCK_N", "BLOCK_R"]
