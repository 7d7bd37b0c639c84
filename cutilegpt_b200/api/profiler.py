"""Data profiler of the Tile API (same classes as cutile_gpt/api/profiler.py:13-195).

Recommendations are advisory, as in the reference: the kernels choose their
own tiles. The recommendation rule (tile 32 / 64 / 128 by average sequence
length, batch sized against an 8 GB budget) is kept identical because
callers may display or log it.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Dict, List

import numpy as np


@dataclass
class DataProfile:
    name: str = ""
    source: str = ""
    sample_count: int = 0
    sequence_lengths: List[int] = field(default_factory=list)
    avg_sequence_length: float = 0.0
    max_sequence_length: int = 0
    min_sequence_length: int = 0
    vocab_size: int = 0
    unique_tokens: int = 0
    token_distribution: Dict[int, int] = field(default_factory=dict)
    recommended_tile_m: int = 64
    recommended_tile_n: int = 64
    recommended_batch_size: int = 1
    estimated_memory_mb: float = 0.0

    def __repr__(self) -> str:
        return (f"DataProfile(name={self.name!r}, source={self.source!r}, samples={self.sample_count}, "
                f"seq_len min/max/avg={self.min_sequence_length}/{self.max_sequence_length}/"
                f"{self.avg_sequence_length:.1f}, vocab={self.vocab_size}, unique={self.unique_tokens}, "
                f"tile_m={self.recommended_tile_m}, tile_n={self.recommended_tile_n}, "
                f"batch={self.recommended_batch_size}, est_mem={self.estimated_memory_mb:.1f} MB)")


class DataAnalyzer:
    """Profiles a dataset (HF dataset, list, array or iterable) and recommends tile sizes."""

    def __init__(self, tokenizer=None):
        self.tokenizer = tokenizer

    def analyze(self, data: Any, name: str = "dataset", max_samples: int = 1000) -> DataProfile:
        prof = DataProfile(name=name)
        if 'Dataset' in type(data).__name__:
            prof.source = "huggingface"
            samples = self._extract_hf_samples(data, max_samples)
        elif isinstance(data, list):
            prof.source = "list"
            samples = data[:max_samples]
        elif isinstance(data, np.ndarray):
            prof.source = "array"
            samples = [data] if data.ndim == 1 else list(data)
        else:
            prof.source = "custom"
            samples = list(data)[:max_samples]
        toks = self._ensure_tokenized(samples)
        prof.sample_count = len(toks)
        prof.sequence_lengths = [len(s) for s in toks if len(s) > 0]
        if prof.sequence_lengths:
            prof.avg_sequence_length = float(np.mean(prof.sequence_lengths))
            prof.max_sequence_length = max(prof.sequence_lengths)
            prof.min_sequence_length = min(prof.sequence_lengths)
        flat = [int(t) for s in toks for t in s]
        prof.unique_tokens = len(set(flat))
        if self.tokenizer:
            prof.vocab_size = getattr(self.tokenizer, 'vocab_size', None) or len(self.tokenizer)
        else:
            prof.vocab_size = max(flat) + 1 if flat else 50257
        return self._compute_recommendations(prof)

    def _extract_hf_samples(self, dataset, max_samples: int) -> List:
        out = []
        for i, item in enumerate(dataset):
            if i >= max_samples:
                break
            for key in ('text', 'content', 'input_ids'):
                if key in item:
                    out.append(item[key])
                    break
            else:
                strs = [v for v in item.values() if isinstance(v, str)]
                if strs:
                    out.append(strs[0])
        return out

    def _ensure_tokenized(self, samples: List) -> List:
        out = []
        for s in samples:
            if isinstance(s, str):
                out.append(self.tokenizer.encode(s) if self.tokenizer else [ord(c) % 50257 for c in s])
            elif isinstance(s, np.ndarray):
                out.append(list(s))
            elif isinstance(s, list):
                out.append(s)
            else:
                out.append([int(s)])
        return out

    def _compute_recommendations(self, prof: DataProfile) -> DataProfile:
        avg = prof.avg_sequence_length
        tile_ = 32 if avg <= 128 else 64 if avg <= 512 else 128
        prof.recommended_tile_m = prof.recommended_tile_n = tile_
        per_sample_mb = (prof.max_sequence_length * 768 * 4) / (1024 * 1024)
        budget_mb = 8000
        batch = int(budget_mb / (per_sample_mb * 50)) if per_sample_mb > 0 else 32
        prof.recommended_batch_size = min(max(1, batch), 32)
        prof.estimated_memory_mb = per_sample_mb * prof.recommended_batch_size * 10
        return prof
