"""Reference-compatible tensor-parallel MLP (reference model.py:8-57, main.py:25-39).

``Ultimate_TP_MLP(config, world_size)`` keeps the reference's constructor, submodule
names (``gate_proj``, ``up_proj``, ``down_proj`` holding this rank's shard), its mutable
knobs ``mode`` ("base" / "flash"), ``bits``, ``group_size``, ``quant_type`` and the
``last_comm_latency`` attribute (ms).  The forward runs on this package's kernels: one
tcgen05 GEMM with a fused SwiGLU epilogue for gate/up, one GEMM for down, then

* ``mode == "flash"``: the fused quantized all-reduce kernel (fp16 result, like the
  reference's flash_all_reduce);
* ``mode == "base"``: NCCL all-reduce in the activation dtype (the reference's baseline).

``last_comm_latency`` is measured with CUDA events around the all-reduce when
``time_comm`` is True (the reference brackets it with two host synchronisations), and is
left at 0.0 otherwise so that the forward stays free of host syncs.

``inject_ultimate_layers(model, rank, world_size)`` swaps the MLP of every decoder layer
of a Hugging Face Llama model for an ``Ultimate_TP_MLP`` holding the rank's shard.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn as nn

from .communication import get_quant_all_reduce
from .ops import gemm as G
from .parallel.staged import staged_all_reduce

__all__ = ["Ultimate_TP_MLP", "inject_ultimate_layers"]


class Ultimate_TP_MLP(nn.Module):
    def __init__(self, config, world_size: int, group=None):
        super().__init__()
        self.world_size = world_size
        self.group = group
        self.mode = "base"
        self.bits = 16
        self.group_size = 128
        self.quant_type = "asym"
        self.time_comm = False
        self.hidden_size = config.hidden_size
        self.shard_size = config.intermediate_size // world_size
        self.gate_proj = nn.Linear(self.hidden_size, self.shard_size, bias=False)
        self.up_proj = nn.Linear(self.hidden_size, self.shard_size, bias=False)
        self.down_proj = nn.Linear(self.shard_size, self.hidden_size, bias=False)
        self.act_fn = nn.SiLU()
        self.last_comm_latency = 0.0
        self._gate_up = None
        self._gate_up_src = None

    def _fused_gate_up(self) -> torch.Tensor:
        src = (self.gate_proj.weight.data_ptr(), self.up_proj.weight.data_ptr(), self.gate_proj.weight._version,
               self.up_proj.weight._version)
        if self._gate_up is None or self._gate_up_src != src:
            self._gate_up = torch.cat([self.gate_proj.weight.detach(), self.up_proj.weight.detach()], 0).contiguous()
            self._gate_up_src = src
        return self._gate_up

    def _all_reduce(self, partial: torch.Tensor) -> torch.Tensor:
        W = self.world_size
        if self.mode == "flash":
            if partial.is_cuda and 8 <= self.group_size <= 256:
                ar = get_quant_all_reduce(self.group, partial.device)
                return ar(partial, out_dtype=torch.float16, bits=self.bits, group_size=self.group_size,
                          quant_type=self.quant_type, algo="two_shot")
            return staged_all_reduce(partial, self.bits, self.group_size, self.quant_type, torch.float16, self.group,
                                     torch.float16)
        if W > 1:
            dist.all_reduce(partial, group=self.group)
        return partial

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        fast = (x.is_cuda and x.dtype == torch.bfloat16 and self.gate_proj.weight.dtype == torch.bfloat16)
        if fast:
            act = G.linear_swiglu(x.contiguous(), self._fused_gate_up())
            partial = G.linear(act, self.down_proj.weight)
        else:
            partial = self.down_proj(self.act_fn(self.gate_proj(x)) * self.up_proj(x))
        if self.time_comm and partial.is_cuda:
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record()
            out = self._all_reduce(partial)
            e.record()
            e.synchronize()
            self.last_comm_latency = s.elapsed_time(e)
        else:
            out = self._all_reduce(partial)
        return out


def inject_ultimate_layers(model, rank: int, world_size: int, group=None):
    """Replace every decoder layer's MLP of a Hugging Face Llama model by its TP shard."""
    config = model.config
    dtype = next(model.parameters()).dtype
    device = next(model.parameters()).device
    shard = config.intermediate_size // world_size
    lo, hi = rank * shard, (rank + 1) * shard
    for layer in model.model.layers:
        old = layer.mlp
        new = Ultimate_TP_MLP(config, world_size, group).to(device=device, dtype=dtype)
        with torch.no_grad():
            new.gate_proj.weight.copy_(old.gate_proj.weight[lo:hi, :])
            new.up_proj.weight.copy_(old.up_proj.weight[lo:hi, :])
            new.down_proj.weight.copy_(old.down_proj.weight[:, lo:hi])
        layer.mlp = new
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
    return model
