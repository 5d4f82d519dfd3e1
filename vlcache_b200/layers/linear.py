"""Linear layers of the recomputed rows, drop-in for nanovllm/layers/linear.py:1-160.

Same classes, constructor arguments, parameter layout (``weight`` [out, in], optional
``bias``) and ``weight_loader`` shard semantics as the reference, so the model and its
loader are unchanged; ``forward`` runs this library's tcgen05 GEMM (``vlc_linear``)
instead of ``F.linear``.  Tensor parallelism is not part of this path (the north star
partitions work by request, one whole model per GPU), so the layers are built for a
tensor-parallel size of 1 and need no process group.

Two fused entry points replace a layer plus its neighbour:
  * ``MergedColumnParallelLinear.forward_silu_mul(x)`` — gate_up_proj then SiluAndMul
    (nanovllm/models/qwen3.py:112-114) in one kernel;
  * ``QKVParallelLinear.forward_rope_store(x, positions, rotary_emb, attn)`` — qkv_proj,
    the split, rotary_emb and the attention layer's store_kvcache
    (nanovllm/models/qwen3.py:75-84, nanovllm/layers/attention.py:59-62) in one kernel;
    returns the roped q for ``attn`` (whose cache then already holds this step's K/V).
"""
from __future__ import annotations

import torch
from torch import nn

from .. import ops
from ..utils.context import get_context


def divide(numerator: int, denominator: int) -> int:
    assert numerator % denominator == 0
    return numerator // denominator


class LinearBase(nn.Module):

    def __init__(self, input_size: int, output_size: int, bias: bool = False, tp_dim: int | None = None):
        super().__init__()
        self.tp_dim = tp_dim
        self.tp_rank = 0
        self.tp_size = 1
        self.weight = nn.Parameter(torch.empty(output_size, input_size), requires_grad=False)
        self.weight.weight_loader = self.weight_loader
        if bias:
            self.bias = nn.Parameter(torch.empty(output_size), requires_grad=False)
            self.bias.weight_loader = self.weight_loader
        else:
            self.register_parameter("bias", None)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        y = ops.linear(x.reshape(-1, x.shape[-1]), self.weight, self.bias)
        return y.view(*lead, y.shape[-1])


class ReplicatedLinear(LinearBase):

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor):
        param.data.copy_(loaded_weight)


class ColumnParallelLinear(LinearBase):

    def __init__(self, input_size: int, output_size: int, bias: bool = False):
        super().__init__(input_size, output_size, bias, 0)

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor):
        param.data.copy_(loaded_weight)


class MergedColumnParallelLinear(ColumnParallelLinear):

    def __init__(self, input_size: int, output_sizes: list[int], bias: bool = False):
        self.output_sizes = list(output_sizes)
        super().__init__(input_size, sum(output_sizes), bias)

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor, loaded_shard_id: int):
        shard_offset = sum(self.output_sizes[:loaded_shard_id])
        shard_size = self.output_sizes[loaded_shard_id]
        param.data.narrow(self.tp_dim, shard_offset, shard_size).copy_(loaded_weight)

    def forward_silu_mul(self, x: torch.Tensor) -> torch.Tensor:
        """``SiluAndMul()(self(x))`` for the [gate | up] layout of two equal halves."""
        assert len(self.output_sizes) == 2 and self.output_sizes[0] == self.output_sizes[1] and self.bias is None
        lead = x.shape[:-1]
        y = ops.linear_silu_mul(x.reshape(-1, x.shape[-1]), self.weight)
        return y.view(*lead, y.shape[-1])


class QKVParallelLinear(ColumnParallelLinear):

    def __init__(self, hidden_size: int, head_size: int, total_num_heads: int, total_num_kv_heads: int | None = None,
                 bias: bool = False):
        total_num_kv_heads = total_num_kv_heads or total_num_heads
        self.head_size = head_size
        self.num_heads = total_num_heads
        self.num_kv_heads = total_num_kv_heads
        super().__init__(hidden_size, (total_num_heads + 2 * total_num_kv_heads) * head_size, bias)

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor, loaded_shard_id: str):
        assert loaded_shard_id in ("q", "k", "v")
        q_size, kv_size = self.num_heads * self.head_size, self.num_kv_heads * self.head_size
        offset, size = {"q": (0, q_size), "k": (q_size, kv_size), "v": (q_size + kv_size, kv_size)}[loaded_shard_id]
        param.data.narrow(self.tp_dim, offset, size).copy_(loaded_weight)

    def forward_rope_store(self, x: torch.Tensor, positions: torch.Tensor, rotary_emb: nn.Module,
                           attn: nn.Module) -> torch.Tensor:
        """qkv_proj + rotary_emb + store_kvcache for this step's rows: returns the roped q
        ``[tokens, num_heads, head_size]``; the roped k and the v rows are in ``attn``'s
        cache at the context's ``slot_mapping``, so call ``attn`` without K/V to store."""
        context = get_context()
        return ops.qkv_rope_store_kvcache(x.reshape(-1, x.shape[-1]), self.weight, self.bias, positions,
                                          rotary_emb.cos_sin_cache, attn.k_cache, attn.v_cache,
                                          context.slot_mapping, self.num_heads, self.num_kv_heads)


class RowParallelLinear(LinearBase):

    def __init__(self, input_size: int, output_size: int, bias: bool = False):
        super().__init__(input_size, output_size, bias, 1)

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor):
        param.data.copy_(loaded_weight)
