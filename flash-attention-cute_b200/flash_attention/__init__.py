from flash_attention.interface import flash_attn_func

__all__ = ["flash_attn_func"]
