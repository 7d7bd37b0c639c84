"""GPT configuration (same fields, presets and names as cutile_gpt/models/config.py:9-87)."""
from __future__ import annotations

from dataclasses import dataclass


@dataclass
class GPTConfig:
    """Hyper-parameters of a GPT-2-style decoder."""
    vocab_size: int = 50257
    block_size: int = 1024
    n_layer: int = 12
    n_head: int = 12
    n_embd: int = 768

    @property
    def head_dim(self) -> int:
        return self.n_embd // self.n_head

    @classmethod
    def gpt_nano(cls) -> 'GPTConfig':
        """3 layers, 48 dims, 3 heads (block_size 128 as in the reference preset)."""
        return cls(n_layer=3, n_head=3, n_embd=48, block_size=128)

    @classmethod
    def gpt_micro(cls) -> 'GPTConfig':
        return cls(n_layer=4, n_head=4, n_embd=128, block_size=256)

    @classmethod
    def gpt_mini(cls) -> 'GPTConfig':
        return cls(n_layer=6, n_head=6, n_embd=192, block_size=256)

    @classmethod
    def gpt2(cls) -> 'GPTConfig':
        """GPT-2 124M: 12 layers, 768 dims, 12 heads."""
        return cls(n_layer=12, n_head=12, n_embd=768, block_size=1024)

    @classmethod
    def gpt2_medium(cls) -> 'GPTConfig':
        return cls(n_layer=24, n_head=16, n_embd=1024, block_size=1024)

    @classmethod
    def gpt2_large(cls) -> 'GPTConfig':
        return cls(n_layer=36, n_head=20, n_embd=1280, block_size=1024)

    @classmethod
    def gpt2_xl(cls) -> 'GPTConfig':
        """GPT-2 XL 1.56B: 48 layers, 1600 dims, 25 heads."""
        return cls(n_layer=48, n_head=25, n_embd=1600, block_size=1024)

    @classmethod
    def gpt_tile_small(cls) -> 'GPTConfig':
        return cls(n_layer=4, n_head=4, n_embd=64, block_size=128)

    @classmethod
    def gpt_tile_medium(cls) -> 'GPTConfig':
        return cls(n_layer=6, n_head=4, n_embd=128, block_size=256)

    @classmethod
    def gpt_tile_large(cls) -> 'GPTConfig':
        return cls(n_layer=8, n_head=8, n_embd=256, block_size=512)

    @classmethod
    def from_name(cls, name: str) -> 'GPTConfig':
        configs = {
            'nano': cls.gpt_nano,
            'micro': cls.gpt_micro,
            'mini': cls.gpt_mini,
            'gpt2': cls.gpt2,
            'gpt2-medium': cls.gpt2_medium,
            'gpt2-large': cls.gpt2_large,
            'gpt2-xl': cls.gpt2_xl,
            'tile-small': cls.gpt_tile_small,
            'tile-medium': cls.gpt_tile_medium,
            'tile-large': cls.gpt_tile_large,
        }
        if name not in configs:
            raise ValueError(f"Unknown config: {name}. Available: {list(configs.keys())}")
        return configs[name]()
