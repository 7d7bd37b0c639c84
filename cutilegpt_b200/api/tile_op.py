"""Fluent Tile API (same surface as cutile_gpt/api/tile_op.py:26-534), executed on libgpt_b200.

    y = tile(x, "hidden").linear(w_fc, b_fc).gelu().linear(w_proj, b_proj).execute()

Differences from the reference: inputs are torch CUDA tensors (CuPy through
DLPack); `_optimize_graph` is not a no-op — a LINEAR_BIAS followed by GELU
becomes one GEMM with the bias+GELU epilogue (the hidden activation is
written once instead of twice), and the ATTENTION node reads q/k/v in place
from the fused QKV tensor.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from enum import Enum, auto
from typing import Any, Dict, List, Optional

import torch

from .. import _lib as L
from ..kernels import ops
from ..kernels._common import as_cuda
from .config import DType, Layout, TensorSpec, TileConfig


class OpType(Enum):
    INPUT = auto()
    LINEAR = auto()
    LINEAR_BIAS = auto()
    GELU = auto()
    LAYERNORM = auto()
    ATTENTION = auto()
    FUSED_MLP = auto()
    RESHAPE = auto()
    TRANSPOSE = auto()
    LINEAR_BIAS_GELU = auto()   # produced by _optimize_graph


@dataclass
class OpNode:
    op_type: OpType
    inputs: List[Any] = field(default_factory=list)
    params: Dict[str, Any] = field(default_factory=dict)
    output_spec: Optional[TensorSpec] = None
    tile_config: Optional[TileConfig] = None

    def __repr__(self) -> str:
        return f"OpNode({self.op_type.name}, out={self.output_spec})"


class TileOp:
    """Builder: each method returns a new TileOp with one more node."""

    def __init__(self, data: Optional[torch.Tensor] = None, spec: Optional[TensorSpec] = None,
                 ops_: Optional[List[OpNode]] = None, tile_config: Optional[TileConfig] = None, **kw):
        self._data = data
        self._spec = spec
        self._ops: List[OpNode] = ops_ if ops_ is not None else list(kw.get('ops') or [])
        self._tile_config = tile_config or TileConfig()
        self._name = spec.name if spec else "tensor"

    # ---- construction
    @classmethod
    def from_tensor(cls, tensor, name: str = "input", layout: Layout = Layout.ROW_MAJOR) -> 'TileOp':
        t = as_cuda(tensor, name)
        spec = TensorSpec(shape=tuple(t.shape), dtype=DType.from_torch(t.dtype), layout=layout, name=name)
        return cls(data=t, spec=spec, ops_=[OpNode(OpType.INPUT, inputs=[t], output_spec=spec)])

    @classmethod
    def placeholder(cls, shape: tuple, dtype: DType = DType.FLOAT32, name: str = "placeholder") -> 'TileOp':
        spec = TensorSpec(shape=tuple(shape), dtype=dtype, name=name)
        return cls(spec=spec, ops_=[OpNode(OpType.INPUT, output_spec=spec)])

    def _then(self, op: OpNode) -> 'TileOp':
        return TileOp(data=self._data, spec=op.output_spec, ops_=self._ops + [op], tile_config=self._tile_config)

    def _spec_like(self, shape, suffix, dim_names=None) -> TensorSpec:
        return TensorSpec(shape=tuple(shape), dtype=self._spec.dtype, layout=self._spec.layout,
                          name=f"{self._name}_{suffix}",
                          dim_names=self._spec.dim_names if dim_names is None else dim_names)

    def declare_shape(self, **dims) -> 'TileOp':
        expected = tuple(dims.values())
        if self._spec and self._spec.shape != expected:
            raise ValueError(f"Declared shape {expected} doesn't match actual shape {self._spec.shape}")
        if self._spec:
            self._spec = TensorSpec(shape=self._spec.shape, dtype=self._spec.dtype, layout=self._spec.layout,
                                    name=self._spec.name, dim_names=tuple(dims.keys()))
        return self

    def with_tile_config(self, config: TileConfig) -> 'TileOp':
        self._tile_config = config
        return self

    # ---- operations
    def linear(self, weight, bias=None, out_features: Optional[int] = None,
               weight_transposed: bool = False) -> 'TileOp':
        in_f = self._spec.shape[-1]
        out_w, in_w = (weight.shape[1], weight.shape[0]) if weight_transposed else (weight.shape[0], weight.shape[1])
        if in_w != in_f:
            raise ValueError(f"Weight in_features ({in_w}) doesn't match input dim ({in_f})")
        if out_features and out_features != out_w:
            raise ValueError(f"Declared out_features ({out_features}) doesn't match weight shape ({out_w})")
        dims = self._spec.dim_names[:-1] + ("out_features",) if self._spec.dim_names else ()
        spec = self._spec_like(self._spec.shape[:-1] + (out_w,), "linear", dims)
        kind = OpType.LINEAR_BIAS if bias is not None else OpType.LINEAR
        return self._then(OpNode(kind, inputs=[weight, bias] if bias is not None else [weight],
                                 params={"in_features": in_f, "out_features": out_w,
                                         "weight_transposed": weight_transposed},
                                 output_spec=spec, tile_config=self._tile_config))

    def gelu(self, approximate: bool = True) -> 'TileOp':
        return self._then(OpNode(OpType.GELU, params={"approximate": approximate},
                                 output_spec=self._spec_like(self._spec.shape, "gelu"),
                                 tile_config=self._tile_config))

    def layernorm(self, weight, bias, eps: float = 1e-5, normalized_shape: Optional[tuple] = None) -> 'TileOp':
        norm_shape = normalized_shape or (self._spec.shape[-1],)
        if tuple(weight.shape) != tuple(norm_shape):
            raise ValueError(f"Weight shape {tuple(weight.shape)} doesn't match normalized_shape {norm_shape}")
        return self._then(OpNode(OpType.LAYERNORM, inputs=[weight, bias],
                                 params={"eps": eps, "normalized_shape": norm_shape},
                                 output_spec=self._spec_like(self._spec.shape, "ln"), tile_config=self._tile_config))

    def attention(self, n_head: int, head_dim: Optional[int] = None, causal: bool = True,
                  scale: Optional[float] = None) -> 'TileOp':
        n_embd = self._spec.shape[-1]
        fused = n_embd % 3 == 0
        out_embd = n_embd // 3 if fused else n_embd
        if head_dim is None:
            head_dim = out_embd // n_head
        if scale is None:
            scale = 1.0 / math.sqrt(head_dim)
        return self._then(OpNode(OpType.ATTENTION,
                                 params={"n_head": n_head, "head_dim": head_dim, "causal": causal, "scale": scale},
                                 output_spec=self._spec_like(self._spec.shape[:-1] + (out_embd,), "attn"),
                                 tile_config=self._tile_config))

    def fused_mlp(self, w_fc, b_fc, w_proj, b_proj, hidden_features: Optional[int] = None) -> 'TileOp':
        if hidden_features and hidden_features != w_fc.shape[0]:
            raise ValueError(f"Declared hidden_features ({hidden_features}) doesn't match w_fc shape "
                             f"({w_fc.shape[0]})")
        spec = self._spec_like(self._spec.shape[:-1] + (w_proj.shape[0],), "mlp")
        return self._then(OpNode(OpType.FUSED_MLP, inputs=[w_fc, b_fc, w_proj, b_proj],
                                 params={"in_features": self._spec.shape[-1], "hidden_features": w_fc.shape[0],
                                         "out_features": w_proj.shape[0]},
                                 output_spec=spec, tile_config=self._tile_config))

    def reshape(self, *shape) -> 'TileOp':
        shape = list(shape)
        if shape.count(-1) > 1:
            raise ValueError("Only one dimension can be -1")
        if -1 in shape:
            known = 1
            for s in shape:
                if s != -1:
                    known *= s
            shape[shape.index(-1)] = self._spec.numel // known
        spec = TensorSpec(shape=tuple(shape), dtype=self._spec.dtype, layout=self._spec.layout,
                          name=f"{self._name}_reshape")
        return self._then(OpNode(OpType.RESHAPE, params={"shape": tuple(shape)}, output_spec=spec))

    def transpose(self, *dims) -> 'TileOp':
        if not dims:
            dims = tuple(range(self._spec.ndim - 2)) + (self._spec.ndim - 1, self._spec.ndim - 2)
        names = tuple(self._spec.dim_names[d] for d in dims) if self._spec.dim_names else ()
        spec = TensorSpec(shape=tuple(self._spec.shape[d] for d in dims), dtype=self._spec.dtype,
                          layout=self._spec.layout, name=f"{self._name}_transpose", dim_names=names)
        return self._then(OpNode(OpType.TRANSPOSE, params={"dims": dims}, output_spec=spec))

    # ---- execution
    def execute(self, optimize: bool = True) -> torch.Tensor:
        if optimize:
            self._optimize_graph()
        return self._execute_ops()

    def _optimize_graph(self) -> None:
        """Fuses LINEAR_BIAS -> GELU into one GEMM with the bias+GELU epilogue."""
        fused: List[OpNode] = []
        i = 0
        while i < len(self._ops):
            op = self._ops[i]
            nxt = self._ops[i + 1] if i + 1 < len(self._ops) else None
            if (op.op_type == OpType.LINEAR_BIAS and nxt is not None and nxt.op_type == OpType.GELU
                    and nxt.params.get("approximate", True) and not op.params.get("weight_transposed")):
                fused.append(OpNode(OpType.LINEAR_BIAS_GELU, inputs=op.inputs, params=dict(op.params),
                                    output_spec=nxt.output_spec, tile_config=op.tile_config))
                i += 2
                continue
            fused.append(op)
            i += 1
        self._ops = fused

    @staticmethod
    def _weight(op: OpNode) -> torch.Tensor:
        w = as_cuda(op.inputs[0], "weight")
        return (w.t() if op.params.get("weight_transposed") else w).contiguous()

    def _execute_ops(self) -> torch.Tensor:
        from ..kernels import (cutile_causal_attention, cutile_fused_mlp, cutile_gelu, cutile_layer_norm,
                               cutile_linear, cutile_linear_bias)
        cur = self._data
        for op in self._ops:
            t = op.op_type
            if t == OpType.INPUT:
                if op.inputs:
                    cur = op.inputs[0]
            elif t == OpType.LINEAR:
                cur = cutile_linear(cur, self._weight(op))
            elif t == OpType.LINEAR_BIAS:
                cur = cutile_linear_bias(cur, self._weight(op), op.inputs[1])
            elif t == OpType.LINEAR_BIAS_GELU:
                w, b = self._weight(op), as_cuda(op.inputs[1], "bias").contiguous()
                x2 = as_cuda(cur, "x").reshape(-1, w.shape[1]).contiguous()
                y = torch.empty((x2.shape[0], w.shape[0]), dtype=x2.dtype, device=x2.device)
                ops.gemm(x2, w, y, bias=b, epilogue=L.EPI_BIAS_GELU)
                cur = y.reshape(*cur.shape[:-1], w.shape[0])
            elif t == OpType.GELU:
                cur = cutile_gelu(cur)
            elif t == OpType.LAYERNORM:
                cur = cutile_layer_norm(cur, op.inputs[0], op.inputs[1], op.params.get("eps", 1e-5))
            elif t == OpType.ATTENTION:
                H = op.params["n_head"]
                B, T, three = cur.shape
                C = three // 3
                D = C // H
                q4 = cur.contiguous().view(B, T, 3, H, D)
                y = torch.empty((B, T, C), dtype=cur.dtype, device=cur.device)
                ops.attention_prefill(q4[:, :, 0].transpose(1, 2), q4[:, :, 1].transpose(1, 2),
                                      q4[:, :, 2].transpose(1, 2), y.view(B, T, H, D).transpose(1, 2),
                                      op.params.get("scale"))
                cur = y
            elif t == OpType.FUSED_MLP:
                cur = cutile_fused_mlp(cur, *op.inputs)
            elif t == OpType.RESHAPE:
                cur = cur.reshape(op.params["shape"])
            elif t == OpType.TRANSPOSE:
                cur = cur.permute(*op.params["dims"])
        return cur

    # ---- inspection
    @property
    def spec(self) -> TensorSpec:
        return self._spec

    @property
    def shape(self) -> tuple:
        return self._spec.shape if self._spec else ()

    def describe(self) -> str:
        lines = ["TileOp Computation Graph:", "=" * 40]
        for i, op in enumerate(self._ops):
            lines.append(f"{'→' if i else ' '} [{i}] {op.op_type.name}")
            if op.output_spec:
                lines.append(f"      Output: {op.output_spec.shape}")
            for k, v in op.params.items():
                lines.append(f"      {k}: {v}")
        if self._spec:
            lines += ["=" * 40, f"Final: {self._spec}"]
        return "\n".join(lines)

    def __repr__(self) -> str:
        return f"TileOp({self._spec})"


def tile(tensor, name: str = "input") -> TileOp:
    """Shorthand for TileOp.from_tensor()."""
    return TileOp.from_tensor(tensor, name=name)
