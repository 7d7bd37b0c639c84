"""GPT model on the sm_100a kernels (mirrors cutile_gpt/models/__init__.py)."""
from .config import GPTConfig
from .gpt import CutileGPT

__all__ = ['GPTConfig', 'CutileGPT']
