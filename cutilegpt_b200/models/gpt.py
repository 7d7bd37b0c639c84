"""CutileGPT on the sm_100a kernels — the drop-in for cutile_gpt/models/gpt.py.

Same public surface as the reference class (cutile_gpt/models/gpt.py:24-343):
``CutileGPT(config)``, ``weights`` dict with the same keys, ``forward(idx) ->
(logits, None)``, ``generate(idx, max_new_tokens, temperature, top_k)``,
``load_from_huggingface`` and ``load_from_mingpt``. Tensors are torch CUDA
tensors (CuPy arrays are accepted through DLPack).

What runs differently (all on libgpt_b200 kernels, no torch compute ops on
the forward path):
  * one fused token+position embedding kernel (gpt.py:110-113);
  * QKV GEMM output [B, T, 3C] is read in place by the attention kernel,
    whose output [B, T, C] feeds c_proj directly (no split/transpose copies,
    gpt.py:133-146);
  * bias, tanh-GELU and the residual add are GEMM epilogues (gpt.py:125-174);
  * weights are stored once in the [out, in] layout the tensor-core GEMM
    reads (no cached transposes, gpt.py:83-90);
  * generate() keeps a KV cache: one prefill, then per token a decode step
    (M = batch GEMMs, split-KV attention, lm_head on the last position only)
    captured once in a CUDA graph and replayed. The reference re-runs the
    whole prefix each step (gpt.py:204-206). Past block_size the reference
    re-encodes the last block_size tokens at positions 0.. (gpt.py:205); that
    windowed re-prefill is reproduced exactly by the non-cached path.
"""
from __future__ import annotations

import math
from typing import Dict, Optional, Tuple

import torch

from .. import _lib as L
from ..kernels import ops
from ..kernels._common import as_cuda
from .config import GPTConfig
from .init import init_state, weight_names

# Greedy decode steps captured into one CUDA graph (the remainder of a
# generate call replays the one-step graph).
_GRAPH_STEPS = 8


class _Workspace:
    """Activation buffers for one (B, T) prefill shape."""

    def __init__(self, cfg: GPTConfig, B: int, T: int, dtype, device, fold: bool = False):
        M, C = B * T, cfg.n_embd
        self.B, self.T = B, T
        self.fold = fold
        if fold:   # row statistics of the residual stream, two ping-pong slots [2, ceil(C/128), M, 2]
            self.stats = torch.empty((2, (C + 127) // 128, M, 2), dtype=torch.float32, device=device)
        self.x = torch.empty((M, C), dtype=dtype, device=device)       # residual stream
        self.h = torch.empty((M, C), dtype=dtype, device=device)       # LayerNorm output
        self.qkv = torch.empty((M, 3 * C), dtype=dtype, device=device)
        self.att = torch.empty((M, C), dtype=dtype, device=device)
        self.f = torch.empty((M, 4 * C), dtype=dtype, device=device)   # MLP hidden


class _DecodeState:
    """Buffers of the KV-cache generation loop for one (B, Tmax)."""

    def __init__(self, cfg: GPTConfig, B: int, Tmax: int, dtype, device, fold: bool = True):
        C, H = cfg.n_embd, cfg.n_head
        D = C // H
        self.B, self.Tmax = B, Tmax
        self.cache = torch.empty((cfg.n_layer, 2, B, H, Tmax, D), dtype=dtype, device=device)
        self.x = torch.empty((B, C), dtype=dtype, device=device)
        self.h = torch.empty((B, C), dtype=dtype, device=device)
        self.qkv = torch.empty((B, 3 * C), dtype=dtype, device=device)
        self.att = torch.empty((B, C), dtype=dtype, device=device)
        self.f = torch.empty((B, 4 * C), dtype=dtype, device=device)
        self.logits = torch.empty((B, cfg.vocab_size), dtype=dtype, device=device)
        self.tok = torch.empty((B,), dtype=torch.int64, device=device)
        self.pos = torch.zeros((1,), dtype=torch.int64, device=device)
        self.seq = torch.empty((B, Tmax), dtype=torch.int64, device=device)
        nbytes = ops.decode_workspace_bytes(B, H, D, Tmax)
        self.dec_ws = torch.empty((max(nbytes, 16),), dtype=torch.uint8, device=device)
        self.graph: Optional[torch.cuda.CUDAGraph] = None          # greedy step
        self.graph_multi: Optional[torch.cuda.CUDAGraph] = None    # _GRAPH_STEPS greedy steps
        self.sample_graphs: Dict[Tuple[float, int], torch.cuda.CUDAGraph] = {}   # per (temperature, top_k)
        self.seed = torch.zeros((1,), dtype=torch.int64, device=device)   # RNG seed of the sampling kernel
        # folded decode step: bf16, up to 128 rows (the split-K receive buffers of the fused GEMMs
        # fit shared memory up to there), 16-byte row pitches for the TMA operands
        self.fold = (fold and dtype == torch.bfloat16 and 1 <= B <= 128 and C % 16 == 0 and D % 16 == 0
                     and cfg.n_layer >= 1)
        if self.fold:
            # exact fp64 row totals (sum, sum of squares) of the residual stream: slot 2i = rows entering
            # block i, 2i+1 = after its attention, 2L = entering ln_f; slots >= 1 are accumulated into
            self.sums = torch.zeros((2 * cfg.n_layer + 1, B, 2), dtype=torch.float64, device=device)


class CutileGPT:
    """GPT-2 inference model on hand-written sm_100a kernels."""

    def __init__(self, config: GPTConfig, dtype: torch.dtype = torch.float32,
                 device: Optional[torch.device | str] = None, seed: Optional[int] = None):
        self._setup(config, dtype, torch.device(device) if device is not None else torch.device('cuda'))
        self._init_weights(seed)

    def _setup(self, config: GPTConfig, dtype: torch.dtype, device: torch.device) -> None:
        self.config = config
        self.dtype = dtype
        self.device = device
        self.weights: Dict[str, torch.Tensor] = {}
        # The reference caches [in, out] copies of every weight (gpt.py:83-90);
        # the tensor-core GEMM reads [out, in] directly, so this stays empty.
        self.weight_transposes: Dict[str, torch.Tensor] = {}
        self._ws: Dict[Tuple[int, int], _Workspace] = {}
        self._dec: Dict[Tuple[int, int], _DecodeState] = {}
        # Optional object with start(flops) / stop() around every GEMM launch.
        self.kernel_timer = None
        # Folded decode step (default for bf16, up to 128 sequences; set False for the per-op step):
        # ln_1 / ln_2 / ln_f folded into the following GEMMs (row statistics produced by the residual
        # GEMMs' epilogues) and the KV append fused into the QKV GEMM: 5 launches per block instead
        # of 9. B200, GPT-2 124M, B=64: 0.49 ms per step vs 0.54 ms for the per-op step.
        self.fold_decode = True
        # The same fold in prefill (opt-in; bf16): 1 row-statistics launch instead
        # of 2L + 1 LayerNorm launches. Correct and tested, but the fold epilogue costs the large
        # prefill GEMMs more than the LayerNorm kernels it replaces (B200, M = 16384: QKV +7 us,
        # c_fc +17 us, residual + statistics +3-5 us, lm_head +300 us vs 10.3 us per LayerNorm).
        self.fold_prefill = False
        self._folded: Optional[Dict[str, Tuple[torch.Tensor, torch.Tensor, torch.Tensor]]] = None

    # ------------------------------------------------------------------ weights
    def _init_weights(self, seed: Optional[int] = None):
        """Random init with the reference's distributions (gpt.py:39-81)."""
        if seed is None:
            seed = int(torch.randint(0, 2**31 - 1, (1,)).item())
        self.load_state(init_state(self.config, seed))

    def load_state(self, state: Dict[str, torch.Tensor]) -> None:
        """Installs a weight dict in the reference key layout (Linear weights [out, in]).

        ``lm_head.weight`` stays tied to ``wte`` when both entries are the same
        tensor (or equal); otherwise it is stored separately, as minGPT's
        untied head is (gpt.py:340).
        """
        cfg = self.config
        missing = [k for k in weight_names(cfg) if k not in state]
        if missing:
            raise KeyError(f"missing weights: {missing[:5]}{'...' if len(missing) > 5 else ''}")
        self._check_shapes(state)
        conv = {}
        for k in weight_names(cfg):
            if k == 'lm_head.weight':
                continue
            conv[k] = state[k].detach().to(device=self.device, dtype=self.dtype).contiguous()
        lm = state['lm_head.weight']
        tied = lm is state['wte'] or (lm.shape == state['wte'].shape and
                                      lm.data_ptr() == state['wte'].data_ptr())
        conv['lm_head.weight'] = conv['wte'] if tied else lm.detach().to(
            device=self.device, dtype=self.dtype).contiguous()
        self.weights = conv
        self._dec.clear()
        self._folded = None

    def _check_shapes(self, state):
        cfg = self.config
        C, V = cfg.n_embd, cfg.vocab_size
        want = {'wte': (V, C), 'wpe': (cfg.block_size, C), 'lm_head.weight': (V, C),
                'ln_f.weight': (C,), 'ln_f.bias': (C,)}
        for i in range(cfg.n_layer):
            p = f'h.{i}.'
            want.update({p + 'attn.c_attn.weight': (3 * C, C), p + 'attn.c_attn.bias': (3 * C,),
                         p + 'attn.c_proj.weight': (C, C), p + 'attn.c_proj.bias': (C,),
                         p + 'mlp.c_fc.weight': (4 * C, C), p + 'mlp.c_fc.bias': (4 * C,),
                         p + 'mlp.c_proj.weight': (C, 4 * C), p + 'mlp.c_proj.bias': (C,),
                         p + 'ln_1.weight': (C,), p + 'ln_1.bias': (C,), p + 'ln_2.weight': (C,),
                         p + 'ln_2.bias': (C,)})
        for k, shp in want.items():
            if tuple(state[k].shape) != shp:
                raise ValueError(f"weight {k}: shape {tuple(state[k].shape)} != expected {shp}")

    def _w(self, key: str) -> torch.Tensor:
        return self.weights[key]

    def _gemm(self, a, w, out, **kw):
        """ops.gemm, bracketed by the optional kernel timer's CUDA events (used by bench.py)."""
        t = self.kernel_timer
        if t is None:
            return ops.gemm(a, w, out, **kw)
        t.start(2 * a.shape[0] * w.shape[0] * w.shape[1])
        ops.gemm(a, w, out, **kw)
        t.stop()
        return out

    def _gemm_fused(self, a, w, out, **kw):
        """ops.gemm_fused under the same optional kernel timer."""
        t = self.kernel_timer
        if t is None:
            return ops.gemm_fused(a, w, out, **kw)
        t.start(2 * a.shape[0] * w.shape[0] * w.shape[1])
        ops.gemm_fused(a, w, out, **kw)
        t.stop()
        return out

    def _prefill_fold_ok(self, M: int) -> bool:
        """LayerNorms folded into the prefill GEMMs: bf16, and row counts the fused GEMMs serve
        (few-row kernel up to 128 rows, CTA-pair tcgen05 kernel above 256)."""
        return (self.fold_prefill and self.dtype == torch.bfloat16 and self.config.n_embd % 8 == 0
                and (M <= 128 or M > 256))

    # ------------------------------------------------------------------ forward
    def __call__(self, idx) -> Tuple[torch.Tensor, None]:
        return self.forward(idx)

    def _workspace(self, B: int, T: int) -> _Workspace:
        key = (B, T)
        ws = self._ws.get(key)
        if ws is None:
            if len(self._ws) >= 4:  # bounded cache of activation buffers
                self._ws.pop(next(iter(self._ws)))
            ws = _Workspace(self.config, B, T, self.dtype, self.device, fold=self._prefill_fold_ok(B * T))
            self._ws[key] = ws
        if ws.fold:
            self._fold_weights()
        return ws

    def _blocks(self, idx: torch.Tensor, ws: _Workspace, cache: Optional[torch.Tensor] = None) -> None:
        """Embedding and all transformer blocks; appends K/V to `cache`. Result: ws.h = ln_f(x), or,
        with the LayerNorm fold (ws.fold), the residual stream ws.x and its row statistics ws.last_stats
        (ln_f is then applied by the lm_head GEMM, see _lm_head)."""
        cfg = self.config
        B, T = idx.shape
        C, H = cfg.n_embd, cfg.n_head
        D = C // H
        scale = 1.0 / math.sqrt(D)
        ops.embedding_pos(idx, self._w('wte'), self._w('wpe'), ws.x)
        qkv4 = ws.qkv.view(B, T, 3, H, D)
        q, k, v = (qkv4[:, :, j].transpose(1, 2) for j in range(3))    # [B, H, T, D] views
        att4 = ws.att.view(B, T, H, D).transpose(1, 2)
        if ws.fold:
            # ln_1 / ln_2 folded into the QKV / c_fc GEMMs; the residual GEMMs emit the row
            # statistics they need (slot 0: rows entering a block, slot 1: after its attention)
            F = self._fold_weights()
            eps = 1e-5
            ops.row_stats(ws.x, ws.stats[0, :1])
            cur = ws.stats[0, :1]
            for i in range(cfg.n_layer):
                p = f'h.{i}.'
                wf, u, v_ = F[p + 'attn']
                self._gemm_fused(ws.x, wf, ws.qkv, epilogue=L.EPI_BIAS, ln=(cur, eps, u, v_))
                if cache is not None:
                    ops.kv_append(ws.qkv.view(B, T, 3 * C), cache[i, 0], cache[i, 1], pos0=0)
                ops.attention_prefill(q, k, v, att4, scale)
                self._gemm_fused(ws.att, self._w(p + 'attn.c_proj.weight'), ws.x,
                                 bias=self._w(p + 'attn.c_proj.bias'), resid=ws.x, row_stats=ws.stats[1])
                wf, u, v_ = F[p + 'fc']
                self._gemm_fused(ws.x, wf, ws.f, epilogue=L.EPI_BIAS_GELU, ln=(ws.stats[1], eps, u, v_))
                self._gemm_fused(ws.f, self._w(p + 'mlp.c_proj.weight'), ws.x,
                                 bias=self._w(p + 'mlp.c_proj.bias'), resid=ws.x, row_stats=ws.stats[0])
                cur = ws.stats[0]
            ws.last_stats = cur
            return
        for i in range(cfg.n_layer):
            p = f'h.{i}.'
            ops.layernorm(ws.x, self._w(p + 'ln_1.weight'), self._w(p + 'ln_1.bias'), ws.h)
            self._gemm(ws.h, self._w(p + 'attn.c_attn.weight'), ws.qkv, bias=self._w(p + 'attn.c_attn.bias'))
            if cache is not None:
                ops.kv_append(ws.qkv.view(B, T, 3 * C), cache[i, 0], cache[i, 1], pos0=0)
            ops.attention_prefill(q, k, v, att4, scale)
            self._gemm(ws.att, self._w(p + 'attn.c_proj.weight'), ws.x, bias=self._w(p + 'attn.c_proj.bias'),
                     resid=ws.x)
            ops.layernorm(ws.x, self._w(p + 'ln_2.weight'), self._w(p + 'ln_2.bias'), ws.h)
            self._gemm(ws.h, self._w(p + 'mlp.c_fc.weight'), ws.f, bias=self._w(p + 'mlp.c_fc.bias'),
                     epilogue=L.EPI_BIAS_GELU)
            self._gemm(ws.f, self._w(p + 'mlp.c_proj.weight'), ws.x, bias=self._w(p + 'mlp.c_proj.bias'),
                     resid=ws.x)
        ops.layernorm(ws.x, self._w('ln_f.weight'), self._w('ln_f.bias'), ws.h)

    def _prep_idx(self, idx) -> torch.Tensor:
        idx = as_cuda(idx, "idx")
        if idx.dim() != 2:
            raise ValueError(f"idx must be (batch, seq_len), got shape {tuple(idx.shape)}")
        if idx.device != self.device and self.device.index is not None:
            idx = idx.to(self.device)
        return idx.to(torch.int64).contiguous()

    def forward(self, idx) -> Tuple[torch.Tensor, None]:
        """Logits (batch, seq_len, vocab) in the model dtype for every position."""
        idx = self._prep_idx(idx)
        B, T = idx.shape
        cfg = self.config
        assert T <= cfg.block_size, f"Sequence length {T} > block_size {cfg.block_size}"
        logits = torch.empty((B, T, cfg.vocab_size), dtype=self.dtype, device=self.device)
        if B * T == 0:
            return logits, None
        ws = self._workspace(B, T)
        self._blocks(idx, ws)
        self._lm_head(ws, logits.view(B * T, cfg.vocab_size))
        return logits, None

    def _lm_head(self, ws: _Workspace, out: torch.Tensor) -> None:
        """Logits of every row of the workspace: ln_f (folded into the GEMM when ws.fold) + lm_head."""
        if ws.fold:
            wf, u, v = self._fold_weights()['lm']
            self._gemm_fused(ws.x, wf, out, epilogue=L.EPI_NONE, ln=(ws.last_stats, 1e-5, u, v))
        else:
            self._gemm(ws.h, self._w('lm_head.weight'), out)

    def forward_last(self, idx, out: Optional[torch.Tensor] = None,
                     cache: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Logits of the last position only, (batch, vocab): the prefill step of generation."""
        idx = self._prep_idx(idx)
        B, T = idx.shape
        assert T <= self.config.block_size
        ws = self._workspace(B, T)
        self._blocks(idx, ws, cache)
        if out is None:
            out = torch.empty((B, self.config.vocab_size), dtype=self.dtype, device=self.device)
        if ws.fold:   # ln_f on the B last rows only (into the first rows of ws.h)
            last_x = ws.x.view(B, T, -1)[:, T - 1, :]
            last = ws.h[:B]
            ops.layernorm(last_x.contiguous(), self._w('ln_f.weight'), self._w('ln_f.bias'), last)
        else:
            last = ws.h.view(B, T, -1)[:, T - 1, :]          # row-strided [B, C] view
        self._gemm(last, self._w('lm_head.weight'), out)
        return out

    # ------------------------------------------------------------------ decode
    def _decode_state(self, B: int, Tmax: int) -> _DecodeState:
        key = (B, Tmax)
        st = self._dec.get(key)
        if st is None:
            if len(self._dec) >= 2:
                self._dec.pop(next(iter(self._dec)))
            st = _DecodeState(self.config, B, Tmax, self.dtype, self.device, fold=self.fold_decode)
            self._dec[key] = st
        if st.fold:
            self._fold_weights()   # eager, outside any graph capture
        return st

    def _fold_weights(self) -> Dict[str, Tuple[torch.Tensor, torch.Tensor, torch.Tensor]]:
        """(gamma-scaled weight, u, v) of every Linear that follows a LayerNorm (see ops.lnfold_weights)."""
        if self._folded is None:
            cfg = self.config
            f = {}
            for i in range(cfg.n_layer):
                p = f'h.{i}.'
                f[p + 'attn'] = ops.lnfold_weights(self._w(p + 'attn.c_attn.weight'), self._w(p + 'ln_1.weight'),
                                                   self._w(p + 'ln_1.bias'), self._w(p + 'attn.c_attn.bias'))
                f[p + 'fc'] = ops.lnfold_weights(self._w(p + 'mlp.c_fc.weight'), self._w(p + 'ln_2.weight'),
                                                 self._w(p + 'ln_2.bias'), self._w(p + 'mlp.c_fc.bias'))
            f['lm'] = ops.lnfold_weights(self._w('lm_head.weight'), self._w('ln_f.weight'), self._w('ln_f.bias'),
                                         None)
            self._folded = f
        return self._folded

    def _decode_step(self, st: _DecodeState) -> None:
        """One token per sequence at device position *st.pos: logits into st.logits."""
        cfg = self.config
        C, H = cfg.n_embd, cfg.n_head
        scale = 1.0 / math.sqrt(C // H)
        B = st.B
        ops.embedding_pos(st.tok.view(B, 1), self._w('wte'), self._w('wpe'), st.x, pos0=0, pos_dev=st.pos)
        q = st.qkv[:, :C]
        if st.fold:
            # LayerNorms folded into the GEMMs that follow them (exact fp64 row sums, see _DecodeState);
            # the first launch writes slot 0 and clears the accumulators of the others.
            F = self._fold_weights()
            eps = 1e-5
            ops.row_sums(st.x, st.sums[0], zero=st.sums[1:])
            for i in range(cfg.n_layer):
                p = f'h.{i}.'
                wf, u, v = F[p + 'attn']
                ops.gemm_fused(st.x, wf, st.qkv, epilogue=L.EPI_BIAS, ln=(st.sums[2 * i], eps, u, v),
                               kv=(st.cache[i, 0], st.cache[i, 1], st.pos, 0))
                ops.attention_decode(q, st.cache[i, 0], st.cache[i, 1], st.att, 1, st.dec_ws, scale,
                                     len_dev=st.pos)
                ops.gemm_fused(st.att, self._w(p + 'attn.c_proj.weight'), st.x, bias=self._w(p + 'attn.c_proj.bias'),
                               resid=st.x, row_stats=st.sums[2 * i + 1])
                wf, u, v = F[p + 'fc']
                ops.gemm_fused(st.x, wf, st.f, epilogue=L.EPI_BIAS_GELU, ln=(st.sums[2 * i + 1], eps, u, v))
                ops.gemm_fused(st.f, self._w(p + 'mlp.c_proj.weight'), st.x, bias=self._w(p + 'mlp.c_proj.bias'),
                               resid=st.x, row_stats=st.sums[2 * i + 2])
            wf, u, v = F['lm']
            ops.gemm_fused(st.x, wf, st.logits, epilogue=L.EPI_NONE, ln=(st.sums[2 * cfg.n_layer], eps, u, v))
            return
        for i in range(cfg.n_layer):
            p = f'h.{i}.'
            ops.layernorm(st.x, self._w(p + 'ln_1.weight'), self._w(p + 'ln_1.bias'), st.h)
            self._gemm(st.h, self._w(p + 'attn.c_attn.weight'), st.qkv, bias=self._w(p + 'attn.c_attn.bias'))
            ops.kv_append(st.qkv.view(B, 1, 3 * C), st.cache[i, 0], st.cache[i, 1], pos0=0, pos_dev=st.pos)
            ops.attention_decode(q, st.cache[i, 0], st.cache[i, 1], st.att, 1, st.dec_ws, scale,
                                 len_dev=st.pos)
            self._gemm(st.att, self._w(p + 'attn.c_proj.weight'), st.x, bias=self._w(p + 'attn.c_proj.bias'),
                     resid=st.x)
            ops.layernorm(st.x, self._w(p + 'ln_2.weight'), self._w(p + 'ln_2.bias'), st.h)
            self._gemm(st.h, self._w(p + 'mlp.c_fc.weight'), st.f, bias=self._w(p + 'mlp.c_fc.bias'),
                     epilogue=L.EPI_BIAS_GELU)
            self._gemm(st.f, self._w(p + 'mlp.c_proj.weight'), st.x, bias=self._w(p + 'mlp.c_proj.bias'),
                     resid=st.x)
        ops.layernorm(st.x, self._w('ln_f.weight'), self._w('ln_f.bias'), st.h)
        self._gemm(st.h, self._w('lm_head.weight'), st.logits)

    def _greedy_step(self, st: _DecodeState, seq: torch.Tensor) -> None:
        self._decode_step(st)
        ops.argmax(st.logits, st.tok)
        ops.decode_advance(st.tok, st.pos, seq)

    def _sample_step(self, st: _DecodeState, seq: torch.Tensor, temperature: float, top_k: Optional[int]) -> None:
        """Decode step + the sampling kernel; the draw is keyed by (seed, row, position of the token)."""
        self._decode_step(st)
        ops.sample(st.logits, st.tok, temperature, top_k, st.seed, st.pos)
        ops.decode_advance(st.tok, st.pos, seq)

    @staticmethod
    def _new_seed(generator: Optional[torch.Generator]) -> torch.Tensor:
        """A 62-bit seed drawn from `generator` (or torch's default RNG), so torch.manual_seed reproduces runs."""
        dev = generator.device if generator is not None else torch.device('cpu')
        return torch.randint(0, 2 ** 62, (1,), generator=generator, device=dev, dtype=torch.int64)

    def _sample(self, logits: torch.Tensor, temperature: float, top_k: Optional[int],
                generator: Optional[torch.Generator]) -> torch.Tensor:
        """Temperature / top-k / multinomial draw (gpt.py:207-225) for every row, one kernel launch."""
        out = torch.empty((logits.shape[0],), dtype=torch.int64, device=logits.device)
        seed = self._new_seed(generator).to(logits.device)
        return ops.sample(logits, out, temperature, top_k, seed)

    @torch.no_grad()
    def generate(self, idx, max_new_tokens: int, temperature: float = 1.0, top_k: Optional[int] = None,
                 use_kv_cache: bool = True, use_cuda_graph: bool = True,
                 generator: Optional[torch.Generator] = None) -> torch.Tensor:
        """Autoregressive generation; returns (batch, seq_len + max_new_tokens) int64.

        ``top_k=1`` is greedy decoding (deterministic argmax, ties to the
        lowest token id). Other settings sample with ``temperature`` / ``top_k``.
        """
        idx = self._prep_idx(idx)
        B, T0 = idx.shape
        cfg = self.config
        if max_new_tokens <= 0:
            return idx.clone()
        total = T0 + max_new_tokens
        greedy = top_k == 1
        if not use_kv_cache or total > cfg.block_size:
            return self._generate_reforward(idx, max_new_tokens, temperature, top_k, generator)
        st = self._decode_state(B, total)
        seq = st.seq
        seq[:, :T0] = idx
        # prefill: K/V of the prompt into the cache, logits of the last position
        self.forward_last(idx, out=st.logits, cache=st.cache)
        if greedy:
            ops.argmax(st.logits, st.tok)
        else:
            if temperature <= 0:
                raise ValueError("temperature must be > 0")
            st.seed.copy_(self._new_seed(generator))
            # the draw for the token after position T0 - 1; decode steps use the device position
            ops.sample(st.logits, st.tok, temperature, top_k, st.seed, None, step0=T0 - 1)
        seq[:, T0] = st.tok
        st.pos.fill_(T0)
        steps = max_new_tokens - 1
        if not greedy:
            key = (float(temperature), 0 if top_k is None else int(top_k))
            g = st.sample_graphs.get(key)
            if not use_cuda_graph or (g is None and steps < 2):
                for _ in range(steps):
                    self._sample_step(st, seq, temperature, top_k)
            else:
                if g is None:
                    self._sample_step(st, seq, temperature, top_k)
                    steps -= 1
                    g = self._capture_fn(lambda: self._sample_step(st, st.seq, temperature, top_k))
                    st.sample_graphs[key] = g
                for _ in range(steps):
                    g.replay()
        elif not use_cuda_graph or steps < 2:
            for _ in range(steps):
                self._greedy_step(st, seq)
        else:
            if st.graph is None:
                # one eager step warms every kernel, then the step is captured once per state
                self._greedy_step(st, seq)
                steps -= 1
                self._capture(st)
            # Several steps per graph launch: inside one graph each step's first
            # kernel overlaps the previous step's last (programmatic dependent
            # launch), which separate graph launches do not allow.
            if steps >= _GRAPH_STEPS and st.graph_multi is None:
                def multi():
                    for _ in range(_GRAPH_STEPS):
                        self._greedy_step(st, st.seq)
                st.graph_multi = self._capture_fn(multi)
            for _ in range(steps // _GRAPH_STEPS):
                st.graph_multi.replay()
            for _ in range(steps % _GRAPH_STEPS):
                st.graph.replay()
        return seq.clone()

    def _capture_fn(self, fn) -> torch.cuda.CUDAGraph:
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                fn()
        torch.cuda.current_stream(self.device).wait_stream(s)
        return g

    def _capture(self, st: _DecodeState) -> None:
        st.graph = self._capture_fn(lambda: self._greedy_step(st, st.seq))

    def _generate_reforward(self, idx, max_new_tokens, temperature, top_k, generator) -> torch.Tensor:
        """Reference semantics without a cache: re-run the (cropped) prefix each step."""
        cfg = self.config
        for _ in range(max_new_tokens):
            idx_cond = idx if idx.shape[1] <= cfg.block_size else idx[:, -cfg.block_size:].contiguous()
            logits = self.forward_last(idx_cond)
            if top_k == 1:
                nxt = torch.empty((idx.shape[0],), dtype=torch.int64, device=self.device)
                ops.argmax(logits, nxt)
            else:
                nxt = self._sample(logits, temperature, top_k, generator)
            idx = torch.cat([idx, nxt.view(-1, 1)], dim=1)
        return idx

    # ------------------------------------------------------------------ loaders
    def load_from_state_dict(self, sd: Dict[str, torch.Tensor], layout: str = 'hf') -> None:
        """Loads a GPT-2 state dict with HF (Conv1D [in, out]) or minGPT (Linear [out, in]) layout.

        Key mapping and transposes follow gpt.py:262-299 (HF) and gpt.py:316-340 (minGPT).
        """
        cfg = self.config
        conv1d = layout == 'hf'
        w: Dict[str, torch.Tensor] = {}

        def get(k):
            t = sd[k]
            return t.detach().float().cpu() if isinstance(t, torch.Tensor) else torch.as_tensor(t).float()

        w['wte'] = get('transformer.wte.weight')
        w['wpe'] = get('transformer.wpe.weight')
        for i in range(cfg.n_layer):
            p, s = f'h.{i}.', f'transformer.h.{i}.'
            for n in ('ln_1.weight', 'ln_1.bias', 'ln_2.weight', 'ln_2.bias', 'attn.c_attn.bias',
                      'attn.c_proj.bias', 'mlp.c_fc.bias', 'mlp.c_proj.bias'):
                w[p + n] = get(s + n)
            for n in ('attn.c_attn.weight', 'attn.c_proj.weight', 'mlp.c_fc.weight', 'mlp.c_proj.weight'):
                t = get(s + n)
                w[p + n] = t.t().contiguous() if conv1d else t
        w['ln_f.weight'] = get('transformer.ln_f.weight')
        w['ln_f.bias'] = get('transformer.ln_f.bias')
        if conv1d or 'lm_head.weight' not in sd:
            w['lm_head.weight'] = w['wte']           # tied (gpt.py:299)
        else:
            w['lm_head.weight'] = get('lm_head.weight')
        self.load_state(w)

    def load_from_huggingface(self, model_name: str = 'gpt2'):
        """Loads pretrained GPT-2 weights through transformers (gpt.py:231-304)."""
        try:
            from transformers import GPT2LMHeadModel
        except ImportError as e:  # pragma: no cover
            raise ImportError("load_from_huggingface requires the 'transformers' package") from e
        hf_model = GPT2LMHeadModel.from_pretrained(model_name)
        self.load_from_state_dict(hf_model.state_dict(), layout='hf')
        print(f"Loaded weights from HuggingFace: {model_name}")

    def save_packed(self, path: str) -> None:
        """Writes config + weights in the packed on-disk format (models/packed.py): the device layout and
        dtype as they are, the tied lm_head once, for fast replica start-up (from_packed)."""
        from . import packed
        tied = self.weights['lm_head.weight'] is self.weights['wte']
        packed.save(path, self.config, self.weights, tied)

    @classmethod
    def from_packed(cls, path: str, device: Optional[torch.device | str] = None) -> 'CutileGPT':
        """A model whose config, dtype and weights come from a packed file (no random init)."""
        from . import packed
        dev = torch.device(device) if device is not None else torch.device('cuda')
        cfg, dt, w = packed.load(path, dev)
        m = cls.__new__(cls)
        m._setup(cfg, dt, dev)
        m.load_state(w)
        return m

    def load_from_mingpt(self, mingpt_model):
        """Loads weights from a minGPT model instance (gpt.py:306-343)."""
        self.load_from_state_dict(mingpt_model.state_dict(), layout='mingpt')
        print("Loaded weights from minGPT")
