from flash_attention.interface import flash_attn_func
from flash_attention.streaming import flash_attn_func_host

__all__ = ["flash_attn_func", "flash_attn_func_host"]
