"""Quantized all-reduce over peer memory: the fused single-kernel path.

:class:`QuantAllReduce` owns a :class:`SymmetricWorkspace` for one process group and
launches the fused kernel of ``csrc/allreduce.cu`` (two-shot for large messages, one-shot
for small ones).  It never calls NCCL on the data path.

Reference capability: ``flash_all_reduce`` (communication.py:7-97); knobs ``bits``
(16 / 8 / 6 / 4), ``group_size`` and ``quant_type`` ("asym" / "sym") keep their meaning.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch
import torch.distributed as dist

from .._ext import ext
from .symm_mem import EmulatedWorkspaces, SymmetricWorkspace, default_timeout_ms

__all__ = ["QuantAllReduce", "EmulatedQuantAllReduce", "ONE_SHOT_MAX_BYTES", "set_norm_warps_per_row",
           "set_two_shot_stages"]

# Messages up to this many input bytes use the one-shot algorithm under algo="auto".
ONE_SHOT_MAX_BYTES = 512 * 1024

_OUT_PAIRS = {
    (torch.bfloat16, torch.bfloat16), (torch.bfloat16, torch.float16), (torch.float16, torch.float16),
    (torch.float32, torch.float32), (torch.float32, torch.float16),
}


def set_norm_warps_per_row(wpr: int) -> int:
    """Warps that share a row in the sequence-parallel all-reduce + norm kernel (1, 2, 4
    or 8; process-wide, initially QFC_NORM_WARPS_PER_ROW or 1).  Returns the previous
    value.  More than one warp per row multiplies the kernel's grid, for row counts per
    rank that leave SMs idle with one warp per row."""
    return int(ext().set_norm_warps_per_row(int(wpr)))


def set_two_shot_stages(stages: int) -> int:
    """Stages per CTA of the 16-per-lane two-shot all-reduce (1, or 2: each CTA's units in
    two halves with their own flags, so that one half's waits and NVLink traffic overlap
    the other half's work).  Process-wide, initially QFC_AR_STAGES or 1.  Returns the
    previous value."""
    return int(ext().set_two_shot_stages(int(stages)))


def _pick_one_shot(algo: str, nbytes: int, one_shot_max: int) -> bool:
    if algo == "one_shot":
        return True
    if algo == "two_shot":
        return False
    if algo != "auto":
        raise ValueError(f"algo must be 'auto', 'one_shot' or 'two_shot', got {algo!r}")
    return nbytes <= one_shot_max


def _aligned(t: torch.Tensor) -> torch.Tensor:
    t = t.contiguous()
    if t.data_ptr() % 16:
        t = t.clone()
    return t


class _Base:
    def __init__(self, bits: int, group_size: int, quant_type: str, scale_dtype: torch.dtype, algo: str,
                 one_shot_max_bytes: int, quantize_local: bool, timeout_ms: Optional[float]):
        if quant_type not in ("asym", "sym"):
            raise ValueError("quant_type must be 'asym' or 'sym'")
        if group_size < 8 or group_size > 256 or group_size & (group_size - 1):
            raise ValueError("the fused all-reduce takes power-of-two group sizes 8..256")
        self.bits = bits
        self.group_size = group_size
        self.quant_type = quant_type
        self.scale_dtype = scale_dtype
        self.algo = algo
        self.one_shot_max_bytes = one_shot_max_bytes
        self.quantize_local = quantize_local
        self.timeout_ms = default_timeout_ms() if timeout_ms is None else timeout_ms

    def _plan(self, n: int, W: int, elem: int, bits: int, gs: int, fp32: bool, one_shot: bool):
        _, need_rs, need_ag, need_os = ext().ar_plan(n, W, bits, gs, fp32, elem, one_shot)
        return need_rs, need_ag, need_os

    def _plan_rows(self, M: int, H: int, W: int, bits: int, fp32: bool):
        _, need_rs, need_ag, need_os = ext().ar_plan_rows(M, H, W, bits, fp32)
        return need_rs, need_ag, need_os


class QuantAllReduce(_Base):
    """Fused quantized all-reduce for one process group (one rank per GPU).

    ``ar(x)`` returns the all-reduced tensor (``out`` may alias ``x``).  Every rank must
    call it with the same shape, dtype and settings, in the same order.
    """

    def __init__(self, group: Optional[dist.ProcessGroup] = None, device=None, bits: int = 8,
                 group_size: int = 128, quant_type: str = "asym", scale_dtype: torch.dtype = torch.float16,
                 algo: str = "auto", one_shot_max_bytes: int = ONE_SHOT_MAX_BYTES,
                 quantize_local: bool = True, timeout_ms: Optional[float] = None,
                 reserve_elems: int = 0, reserve_dtype: torch.dtype = torch.bfloat16):
        super().__init__(bits, group_size, quant_type, scale_dtype, algo, one_shot_max_bytes, quantize_local,
                         timeout_ms)
        self.group = group
        self.ws = SymmetricWorkspace(group, device)
        self.world = self.ws.world
        self.rank = self.ws.rank
        if reserve_elems:
            self.reserve(reserve_elems, reserve_dtype)

    def reserve(self, max_elems: int, dtype: torch.dtype = torch.bfloat16, bits_options: Sequence[int] = (16, 8, 6, 4)):
        """Size the workspace for messages up to ``max_elems`` (call before graph capture)."""
        elem = torch.empty((), dtype=dtype).element_size()
        rs = ag = os_ = 0
        for b in bits_options:
            for one in (False, True):
                if one and max_elems * elem > self.one_shot_max_bytes and self.algo != "one_shot":
                    continue
                r, a, o = self._plan(max_elems, self.world, elem, b, self.group_size,
                                     self.scale_dtype == torch.float32, one)
                rs, ag, os_ = max(rs, r), max(ag, a), max(os_, o)
        self.ws.ensure(rs, ag, os_)

    def __call__(self, x: torch.Tensor, out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
                 bits: Optional[int] = None, group_size: Optional[int] = None, quant_type: Optional[str] = None,
                 algo: Optional[str] = None) -> torch.Tensor:
        bits = self.bits if bits is None else bits
        gs = self.group_size if group_size is None else group_size
        qt = self.quant_type if quant_type is None else quant_type
        algo = self.algo if algo is None else algo
        x = _aligned(x)
        if out is None:
            out = torch.empty(x.shape, dtype=out_dtype or x.dtype, device=x.device)
        if (x.dtype, out.dtype) not in _OUT_PAIRS:
            raise TypeError(f"unsupported (input, output) dtypes {x.dtype}, {out.dtype}")
        one = _pick_one_shot(algo, x.numel() * x.element_size(), self.one_shot_max_bytes)
        fp32 = self.scale_dtype == torch.float32
        self.ws.ensure(*self._plan(x.numel(), self.world, x.element_size(), bits, gs, fp32, one))
        ext().quant_all_reduce([self.ws.native], [x], [out], bits, gs, qt == "sym", fp32, one,
                               self.quantize_local, self.timeout_ms)
        return out

    def reserve_rows(self, max_rows: int, hidden: int, bits_options: Sequence[int] = (16, 8, 6, 4)):
        """Size the workspace for row-blocked all-reduce + norm calls of up to ``max_rows``
        rows of ``hidden`` (call before graph capture)."""
        fp32 = self.scale_dtype == torch.float32
        rs = ag = 0
        for b in bits_options:
            r, a, _ = self._plan_rows(max_rows, hidden, self.world, b, fp32)
            rs, ag = max(rs, r), max(ag, a)
        self.ws.ensure(rs, ag, 0)

    def all_reduce_norm(self, partial: torch.Tensor, residual_shard: torch.Tensor, weight: torch.Tensor, eps: float,
                        out: Optional[torch.Tensor] = None, bits: Optional[int] = None,
                        quant_type: Optional[str] = None) -> torch.Tensor:
        """Sequence-parallel all-reduce + residual + RMSNorm of a row-parallel layer.

        ``partial [M, H]`` is this rank's partial sum; this rank owns rows
        ``[r*R, (r+1)*R)`` (``R = ceil(M / world)``) of the residual stream, held in
        ``residual_shard [R, H]`` and updated in place (``h += sum``).  Returns
        ``x [M, H] = all_gather(rmsnorm(h) * weight)`` (quantized on the wire), identical
        on every rank.  Group size 128, bf16.
        """
        bits = self.bits if bits is None else bits
        qt = self.quant_type if quant_type is None else quant_type
        partial = _aligned(partial)
        M, H = partial.shape
        if out is None:
            out = torch.empty(M, H, dtype=torch.bfloat16, device=partial.device)
        fp32 = self.scale_dtype == torch.float32
        self.ws.ensure(*self._plan_rows(M, H, self.world, bits, fp32))
        ext().quant_all_reduce_norm([self.ws.native], [partial], [residual_shard], weight, [out], bits, qt == "sym",
                                    fp32, self.quantize_local, float(eps), self.timeout_ms)
        return out

    def gemm_all_reduce_norm(self, a: torch.Tensor, w: torch.Tensor, residual_shard: torch.Tensor,
                             weight: torch.Tensor, eps: float, out: Optional[torch.Tensor] = None,
                             bits: Optional[int] = None, quant_type: Optional[str] = None) -> torch.Tensor:
        """``all_reduce_norm(a @ w.T, ...)`` with the reduce-scatter fused into the GEMM
        epilogue (every 128-column group of a tile goes to its row owner's slot)."""
        bits = self.bits if bits is None else bits
        qt = self.quant_type if quant_type is None else quant_type
        a2 = a.reshape(-1, a.shape[-1])
        M, H = a2.shape[0], w.shape[0]
        if out is None:
            out = torch.empty(M, H, dtype=torch.bfloat16, device=a.device)
        fp32 = self.scale_dtype == torch.float32
        self.ws.ensure(*self._plan_rows(M, H, self.world, bits, fp32))
        ext().gemm_all_reduce_norm(self.ws.native, a2, w, residual_shard, weight, out, bits, qt == "sym", fp32,
                                   float(eps), self.timeout_ms)
        return out

    def gemm_all_reduce(self, a: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None,
                        bits: Optional[int] = None, quant_type: Optional[str] = None) -> torch.Tensor:
        """``all_reduce(a @ w.T)`` with the two-shot reduce-scatter fused into the GEMM.

        The tcgen05 GEMM's epilogue quantizes each 128-column group of its output tile and
        stores it straight into the owning rank's reduce-scatter slot over NVLink, so the
        transfer overlaps the remaining tiles; a second kernel then reduces, requantizes and
        all-gathers.  Bit-identical to ``self(linear(a, w))`` with two-shot and group size 128.
        """
        bits = self.bits if bits is None else bits
        qt = self.quant_type if quant_type is None else quant_type
        a2 = a.reshape(-1, a.shape[-1])
        M, N = a2.shape[0], w.shape[0]
        if out is None:
            out = torch.empty(*a.shape[:-1], N, dtype=torch.bfloat16, device=a.device)
        fp32 = self.scale_dtype == torch.float32
        self.ws.ensure(*self._plan(M * N, self.world, 2, bits, 128, fp32, False))
        ext().gemm_all_reduce(self.ws.native, a2, w, out, bits, 128, qt == "sym", fp32, self.timeout_ms)
        return out

    def argmax(self, val: torch.Tensor, idx: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Global argmax per row from every rank's (score fp32, global index int64) pair:
        the highest score wins, ties go to the lower rank (one kernel, at most 512 rows)."""
        out = torch.empty(val.numel(), dtype=torch.int64, device=val.device) if out is None else out
        ext().argmax_gather(self.ws.native, val.contiguous(), idx.contiguous(), out, self.timeout_ms)
        return out

    def check(self, synchronize: bool = True):
        self.ws.check(synchronize)


class EmulatedQuantAllReduce(_Base):
    """W ranks of the fused all-reduce inside single launches on one GPU (testing aid)."""

    def __init__(self, world: int, device=None, bits: int = 8, group_size: int = 128, quant_type: str = "asym",
                 scale_dtype: torch.dtype = torch.float16, algo: str = "auto",
                 one_shot_max_bytes: int = ONE_SHOT_MAX_BYTES, quantize_local: bool = True,
                 timeout_ms: Optional[float] = None):
        super().__init__(bits, group_size, quant_type, scale_dtype, algo, one_shot_max_bytes, quantize_local,
                         timeout_ms)
        self.ws = EmulatedWorkspaces(world, device)
        self.world = world

    def __call__(self, xs: List[torch.Tensor], outs: Optional[List[torch.Tensor]] = None,
                 out_dtype: Optional[torch.dtype] = None, bits: Optional[int] = None,
                 group_size: Optional[int] = None, quant_type: Optional[str] = None,
                 algo: Optional[str] = None) -> List[torch.Tensor]:
        assert len(xs) == self.world
        bits = self.bits if bits is None else bits
        gs = self.group_size if group_size is None else group_size
        qt = self.quant_type if quant_type is None else quant_type
        algo = self.algo if algo is None else algo
        xs = [_aligned(x) for x in xs]
        if outs is None:
            outs = [torch.empty(x.shape, dtype=out_dtype or x.dtype, device=x.device) for x in xs]
        one = _pick_one_shot(algo, xs[0].numel() * xs[0].element_size(), self.one_shot_max_bytes)
        fp32 = self.scale_dtype == torch.float32
        self.ws.ensure(*self._plan(xs[0].numel(), self.world, xs[0].element_size(), bits, gs, fp32, one))
        ext().quant_all_reduce(self.ws.all, xs, outs, bits, gs, qt == "sym", fp32, one, self.quantize_local,
                               self.timeout_ms)
        return outs

    def check(self, synchronize: bool = True):
        self.ws.check(synchronize)

    def all_reduce_norm(self, partials: List[torch.Tensor], residual_shards: List[torch.Tensor],
                        weight: torch.Tensor, eps: float, bits: Optional[int] = None,
                        quant_type: Optional[str] = None) -> List[torch.Tensor]:
        """All W ranks of :meth:`QuantAllReduce.all_reduce_norm` in one launch."""
        assert len(partials) == self.world == len(residual_shards)
        bits = self.bits if bits is None else bits
        qt = self.quant_type if quant_type is None else quant_type
        partials = [_aligned(x) for x in partials]
        M, H = partials[0].shape
        outs = [torch.empty(M, H, dtype=torch.bfloat16, device=x.device) for x in partials]
        fp32 = self.scale_dtype == torch.float32
        self.ws.ensure(*self._plan_rows(M, H, self.world, bits, fp32))
        ext().quant_all_reduce_norm(self.ws.all, partials, list(residual_shards), weight, outs, bits, qt == "sym",
                                    fp32, self.quantize_local, float(eps), self.timeout_ms)
        return outs
